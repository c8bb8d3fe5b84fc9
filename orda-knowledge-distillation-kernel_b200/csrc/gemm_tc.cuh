// Persistent warp-specialised tcgen05 GEMM for sm_100a:  D[m, n] = sum_k A[m, k] * B[n, k].
//
//   warp 0      : TMA producer (one thread) - 128B-swizzled tiles into a multi-stage smem ring
//   warp 1      : TMEM allocator + MMA issuer (one thread) - tcgen05.mma kind::f16, fp32 accumulators
//   warps 2..5  : epilogue - tcgen05.ld of the finished accumulator, one thread per tile row
//
// Two TMEM accumulator buffers let the epilogue of tile i overlap the mainloop of tile i+1.
// Operands are bf16 or fp16; each may be K-major (k contiguous) or MN-major (m / n contiguous),
// which covers the three GEMMs of the loss: logits = H W^T (K/K), dH = dZ W (K/MN),
// dW = dZ^T H (MN/MN). The loss itself runs on the CTA-pair kernels (gemm_tc2.cuh, gemm_tc2w.cuh);
// this single-CTA kernel is the reference GEMM of the layout tests (orda_debug_gemm). This header
// also holds the parameter block, the operand descriptors, the tile rasterisation and the store
// epilogue that the pair kernels share.
// No cluster launch and no multicast: every CTA loads its own tiles.
#pragma once

#include "distill_common.cuh"
#include "fwd_epilogue.cuh"
#include "sm100_ptx.cuh"

namespace orda {

enum EpiKind { EPI_FWD_STATS = 0, EPI_STORE = 1 };

constexpr int kBK = 64;                       // k elements per stage (128 B of 16-bit data)
constexpr uint32_t kATileBytes = kTileRows * kBK * 2;
constexpr int kGemmThreads = 192;
constexpr uint32_t kSmemBudget = 200 * 1024;

struct StoreEpiParams {
  void* out;         // D destination
  int64_t ldo;
  int64_t M, N;      // valid extent of D
  int32_t out_f32;   // 1: fp32 output, 0: compute dtype
  int32_t accumulate;// 1: D = out + acc
  // Row routing to the owning GPU (fused reduce-scatter of a data-parallel weight gradient, 16-bit
  // output only): with peers > 0, row v of D is stored to
  //   peer_base[v / slab_rows] + (slot * slab_rows + v % slab_rows) * ldo
  // (peer addresses mapped into this GPU's address space), and `accumulate` adds the local partial
  // at acc_src + v * ldo instead of the destination's previous value.
  int32_t peers;
  int32_t slot;
  int64_t slab_rows;
  const void* acc_src;
  void* peer_base[ORDA_MAX_PEERS];
};

struct TcGemmParams {
  CUtensorMap a0, b0, a1, b1;
  CUtensorMap ws_s_map, ws_t_map;  // wide kernel: TMA stores of the shifted logits [rows, ld_ws], 64 x 32 boxes
  // wide kernel, store epilogue with st_tma = 1: the 16-bit output [M, N] (64 x 32 boxes, 128-byte
  // swizzle); the epilogue stages each 32-row x 64-column piece in shared memory and stores it by TMA
  CUtensorMap out_map;
  int32_t st_tma;
  // with st_tma and rows routed to peers (st.peers > 0, slab_rows a multiple of 512): map k covers
  // this GPU's slot [slab_rows, N] in peer k's slot buffer
  CUtensorMap peer_maps[ORDA_MAX_PEERS];
  int32_t m_tiles, n_tiles;
  int32_t kb0, kb1;  // k blocks of segment 0 / 1
  int32_t group_m;
  // k split (wide kernel, single segment): unit t covers output tile t % (m_tiles*n_tiles) over k
  // blocks [ks*kb_split, (ks+1)*kb_split) with ks = t / (m_tiles*n_tiles), and stores its fp32
  // partial at st.out + ks * split_bytes. ksplit <= 1: no split.
  int32_t ksplit, kb_split;
  int64_t split_bytes;
  int32_t prof_slot;  // >= 0: accumulate pipeline wait counters into g_tc2_prof[prof_slot] (testing hook)
  int32_t* status;
  FwdEpiParams fwd;
  StoreEpiParams st;
};

template <int BN>
struct GemmShape {
  static constexpr uint32_t kBBytes = BN * kBK * 2;
  static constexpr uint32_t kStageBytes = kATileBytes + kBBytes;
  static constexpr int kStages = (kSmemBudget / kStageBytes) > 8 ? 8 : (kSmemBudget / kStageBytes);
  static constexpr uint32_t kAccCols = BN;  // one accumulator buffer
  static constexpr uint32_t kTmemCols = 2 * kAccCols;
  static constexpr uint32_t kBarBytes = (2 * kStages + 4) * 8 + 16;
  static constexpr uint32_t kSmemBytes = kStages * kStageBytes + kBarBytes + 1024;
  static_assert(kTmemCols <= 512, "accumulators exceed TMEM");
  static_assert(kTmemCols == 256 || kTmemCols == 512, "TMEM allocation must be a power of two");
  static_assert(kStages >= 2, "need at least two pipeline stages");
};

// Grouped rasterisation of the persistent tile index. group > 0: groups of `group` m-tiles, m fastest
// inside a group (consecutive tiles share the B tile). group < 0: groups of -group n-tiles, n fastest
// (consecutive tiles share the A tile).
__device__ __forceinline__ void tile_coords(int32_t t, int32_t m_tiles, int32_t n_tiles, int32_t group,
                                            int32_t& mt, int32_t& nt) {
  if (group > 0) {
    const int32_t per_group = group * n_tiles;
    const int32_t g = t / per_group;
    const int32_t first_m = g * group;
    const int32_t gm = min(group, m_tiles - first_m);
    const int32_t local = t - g * per_group;
    mt = first_m + local % gm;
    nt = local / gm;
  } else {
    const int32_t gsz = -group;
    const int32_t per_group = gsz * m_tiles;
    const int32_t g = t / per_group;
    const int32_t first_n = g * gsz;
    const int32_t gn = min(gsz, n_tiles - first_n);
    const int32_t local = t - g * per_group;
    nt = first_n + local % gn;
    mt = local / gn;
  }
}

template <bool MN>
__device__ __forceinline__ void load_operand(uint32_t dst, const CUtensorMap* map, uint32_t bar, int32_t mn0,
                                             int32_t k0, int rows) {
  if constexpr (MN) {
#pragma unroll 1
    for (int j = 0; j < rows / 64; ++j) tma_load_2d(dst + j * 8192u, map, bar, mn0 + 64 * j, k0);
  } else {
    tma_load_2d(dst, map, bar, k0, mn0);
  }
}

template <bool MN>
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int kk) {
  if constexpr (MN) return smem_desc_sw128(base + kk * 2048u, 8192u, 1024u);
  else return smem_desc_sw128(base + kk * 32u, 16u, 1024u);
}

template <typename T16>
__device__ __forceinline__ void store_epilogue(const StoreEpiParams& st, uint32_t tbase, int64_t row, int64_t n0,
                                               int bn) {
  const bool row_ok = row < st.M;
#pragma unroll 1
  for (int c = 0; c < bn / 32; ++c) {
    float v[32];
    tmem_ld32(tbase + c * 32, v);
    if (!row_ok) continue;
    const int64_t col0 = n0 + c * 32;
    if (col0 >= st.N) continue;
    const int cnt = static_cast<int>((st.N - col0 < 32 ? st.N - col0 : (int64_t)32));
    if (st.out_f32) {
      float* o = static_cast<float*>(st.out) + row * st.ldo + col0;
      if (cnt == 32 && (st.ldo % 4) == 0) {
        float4* o4 = reinterpret_cast<float4*>(o);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float4 a = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
          if (st.accumulate) {
            const float4 b = o4[j];
            a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
          }
          o4[j] = a;
        }
      } else {
        for (int j = 0; j < cnt; ++j) o[j] = st.accumulate ? o[j] + v[j] : v[j];
      }
    } else {
      T16* o;
      const T16* prev_src;
      if (st.peers > 0) {
        const int64_t owner = row / st.slab_rows;
        o = static_cast<T16*>(st.peer_base[owner]) + (st.slot * st.slab_rows + row - owner * st.slab_rows) * st.ldo +
            col0;
        prev_src = st.acc_src ? static_cast<const T16*>(st.acc_src) + row * st.ldo + col0 : nullptr;
      } else {
        o = static_cast<T16*>(st.out) + row * st.ldo + col0;
        prev_src = o;
      }
      if (cnt == 32 && (st.ldo % 8) == 0) {
        if (st.accumulate && prev_src) {
          const uint4* i4 = reinterpret_cast<const uint4*>(prev_src);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 b = i4[q];
            const T16* bh = reinterpret_cast<const T16*>(&b);
#pragma unroll
            for (int j = 0; j < 8; ++j) v[8 * q + j] += Conv<T16>::to_f(bh[j]);
          }
        }
        store_chunk32<T16>(o, v);
      } else {
        for (int j = 0; j < cnt; ++j) {
          const float prev = st.accumulate && prev_src ? Conv<T16>::to_f(prev_src[j]) : 0.f;
          o[j] = Conv<T16>::from_f(prev + v[j]);
        }
      }
    }
  }
}

template <int BN, bool A_MN, bool B_MN, typename T16>
__global__ void __launch_bounds__(kGemmThreads, 1) tc_gemm_kernel(const __grid_constant__ TcGemmParams p) {
  using S = GemmShape<BN>;
  constexpr uint32_t kIdesc =
      make_idesc_f16(sizeof(T16) == 2 && std::is_same<T16, __nv_bfloat16>::value ? 1u : 0u, kTileRows, BN,
                     A_MN ? 1u : 0u, B_MN ? 1u : 0u);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t tiles_addr = (raw_addr + 1023u) & ~1023u;
  const uint32_t bar_addr = tiles_addr + S::kStages * S::kStageBytes;
  auto full_bar = [&](int s) { return bar_addr + 8u * s; };
  auto empty_bar = [&](int s) { return bar_addr + 8u * (S::kStages + s); };
  auto tfull_bar = [&](int b) { return bar_addr + 8u * (2 * S::kStages + b); };
  auto tempty_bar = [&](int b) { return bar_addr + 8u * (2 * S::kStages + 2 + b); };
  const uint32_t tmem_slot = bar_addr + 8u * (2 * S::kStages + 4);
  uint32_t* tmem_slot_ptr = reinterpret_cast<uint32_t*>(smem_raw + (tmem_slot - raw_addr));

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const int32_t num_tiles = p.m_tiles * p.n_tiles;
  const int32_t kb_total = p.kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), 128);
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.a0);
    tma_prefetch_desc(&p.b0);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot_ptr;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int32_t t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int32_t mt, nt;
        tile_coords(t, p.m_tiles, p.n_tiles, p.group_m, mt, nt);
        const int32_t m0 = mt * kTileRows, n0 = nt * BN;
        for (int32_t kb = 0; kb < kb_total; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.status)) { ok = false; break; }
          const uint32_t sa = tiles_addr + stage * S::kStageBytes;
          const uint32_t sb = sa + kATileBytes;
          mbar_arrive_expect_tx(full_bar(stage), S::kStageBytes);
          load_operand<A_MN>(sa, &p.a0, full_bar(stage), m0, kb * kBK, kTileRows);
          load_operand<B_MN>(sb, &p.b0, full_bar(stage), n0, kb * kBK, BN);
          if (++stage == S::kStages) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int32_t t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
        const int buf = it & 1;
        const uint32_t bphase = (it >> 1) & 1;
        if (!mbar_wait(tempty_bar(buf), bphase ^ 1u, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t acc0 = tmem_base + buf * S::kAccCols;
        for (int32_t kb = 0; kb < kb_total; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, p.status)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = tiles_addr + stage * S::kStageBytes;
          const uint32_t sb = sa + kATileBytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            tc_mma_f16(acc0, operand_desc<A_MN>(sa, kk), operand_desc<B_MN>(sb, kk), kIdesc, (kb | kk) != 0);
          tc_commit(empty_bar(stage));
          if (++stage == S::kStages) { stage = 0; phase ^= 1u; }
        }
        if (ok) tc_commit(tfull_bar(buf));
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    int it = 0;
    for (int32_t t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
      const int buf = it & 1;
      const uint32_t bphase = (it >> 1) & 1;
      if (!mbar_wait(tfull_bar(buf), bphase, p.status)) break;
      tc_fence_after();
      int32_t mt, nt;
      tile_coords(t, p.m_tiles, p.n_tiles, p.group_m, mt, nt);
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * S::kAccCols;
      const int64_t row = static_cast<int64_t>(mt) * kTileRows + r;
      store_epilogue<T16>(p.st, tbase, row, static_cast<int64_t>(nt) * BN, BN);
      tc_fence_before();
      mbar_arrive(tempty_bar(buf));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (*reinterpret_cast<volatile int32_t*>(p.status) == ORDA_ERR_TIMEOUT) __nanosleep(1000000);  // let in-flight copies land
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

}  // namespace orda
