// Persistent warp-specialised tcgen05 GEMM on CTA pairs with 512 x 256 tiles ("wide" pair kernel).
//
// Each tile issues two M=256 pair MMAs per k step (tcgen05.mma.cta_group::2, N=256) into two
// accumulators that fill all 512 TMEM columns of each CTA. Per CTA and 64-deep k block the kernel
// loads 256 A rows and its 128-column half of B (48 KB) for 2 x 128 x 256 x 64 multiply-adds: two
// thirds of the operand bytes per MMA of the 256 x 256 pair kernel. That ratio is what keeps the
// tensor pipe fed from L2: the 256 x 256 kernel leaves the MMA issuer waiting for loaded stages
// about 16% of the time.
//
// The accumulators are single-buffered. Two groups of epilogue warps drain them in parallel,
// releasing each as soon as it is read, and the MMA issuer of the next tile waits for each one
// separately. The logits epilogue reads each 128-column vocab tile from TMEM with all its loads in
// flight at once, stages the shifted logits in shared memory (128-byte swizzle) and writes them with
// TMA stores, so the part of the epilogue that is not hidden stays short.
//
//   warp 0 (each CTA) : TMA producer; transaction bytes of both CTAs land on the leader's barrier
//   warp 1 (leader)   : MMA issuer
//   warps 2..9        : epilogue; warps 2..5 drain accumulator 0 and warps 6..9 accumulator 1
//                       (TMEM lanes 32 * (warp % 4) .. + 31 each)
//
// Row mapping of a tile (pair rows 0..511; CTA rank r, accumulator j, TMEM lane l):
//   A_PLAIN      : row j*256 + r*128 + l
//   A_INTERLEAVE : token j*128 + r*64 + (l & 63); lanes 0..63 student (A0), 64..127 teacher (A1)
#pragma once

#include "distill_common.cuh"
#include "fwd_epilogue.cuh"
#include "gemm_tc.cuh"
#include "gemm_tc2.cuh"
#include "sm100_ptx.cuh"

namespace orda {

constexpr uint32_t kWideAcc = 2;                              // accumulators per CTA (256 columns each)
constexpr uint32_t kWideStageBytes = 2 * kATileBytes + kATileBytes;  // A: 2 x 128 rows, B: 128-column half
constexpr uint32_t kWideStagingPerWarp = 4096;                // 32 rows x 64 columns, 16-bit

template <int EPI>
struct WideShape {
  static constexpr int kStages = 4;
  // Both epilogues run 8 warps, 4 per accumulator, so the two accumulators drain at once and the
  // part of the drain the next tile's MMAs wait for is halved.
  static constexpr int kEpiWarps = 8;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr uint32_t kStaging = kEpiWarps * kWideStagingPerWarp;  // both epilogues stage via TMA
  static constexpr uint32_t kBarBytes = (2 * kStages + 4) * 8 + 16;
  static constexpr uint32_t kSmemBytes = kStages * kWideStageBytes + kStaging + kBarBytes + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

// Logits epilogue of one 256-column accumulator for the warp's 32 rows (one row per lane): per
// 128-column vocab tile the tile maximum, the exact label logit and the logits shifted by the maximum
// as base-2 exponents (16-bit, staged in the warp's 4 KB shared-memory buffer 64 columns at a time and written with TMA
// stores).
template <typename WsT>
__device__ __forceinline__ void wide_fwd_acc(const FwdEpiParams& p, const CUtensorMap* ws_map, bool write_ws,
                                             uint32_t tbase, uint32_t staging, int64_t row, int64_t y0,
                                             int64_t n0, bool student, int lane, int64_t label_raw) {
  const bool row_ok = row < p.rows;
  int64_t label_local = -1;
  if (row_ok) {
    bool ignored;
    const int64_t y = safe_label(label_raw, p.ignore_index, p.vocab_total, &ignored);
    if (!ignored) label_local = y - p.vocab_offset;
  }
  const int tile0 = static_cast<int>(n0 / kVocabTile);
  const int ntiles = p.n_vtiles - tile0 < 2 ? p.n_vtiles - tile0 : 2;  // warp-uniform, >= 1
#pragma unroll 1
  for (int h = 0; h < ntiles; ++h) {
    const int64_t nh = n0 + h * kVocabTile;
    const int tile = tile0 + h;
    const int nvalid = static_cast<int>(p.vocab - nh < kVocabTile ? p.vocab - nh : kVocabTile);
    const int label_col = (label_local >= nh && label_local < nh + nvalid) ? static_cast<int>(label_local - nh) : -1;
    uint32_t r[4][32];
#pragma unroll
    for (int c = 0; c < 4; ++c) tmem_ld32_async(tbase + h * kVocabTile + c * 32, r[c]);
    tmem_wait_ld();
    float m = -CUDART_INF_F;
    if (nvalid == kVocabTile) {
      float pm[8];  // independent partial maxima: short dependency chains
#pragma unroll
      for (int q = 0; q < 8; ++q) pm[q] = -CUDART_INF_F;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int j = 0; j < 32; ++j) pm[j & 7] = fmaxf(pm[j & 7], __uint_as_float(r[c][j]));
#pragma unroll
      for (int q = 0; q < 8; ++q) m = fmaxf(m, pm[q]);
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c * 32 + j < nvalid) m = fmaxf(m, __uint_as_float(r[c][j]));
    }
    float zy = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (__any_sync(0xffffffffu, static_cast<unsigned>(label_col - c * 32) < 32u)) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c * 32 + j == label_col) zy = __uint_as_float(r[c][j]);
      }
    }
    if (write_ws) {
      const float mL = m * kLog2e;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        // the previous TMA store of this warp must have read the staging buffer
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
        // row `lane`, 64 columns: 16-byte chunk q of the 128-byte row lands at q ^ (lane & 7)
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int c = hf * 2 + (q >> 2), e0 = (q & 3) * 8;
          // base-2 exponents relative to the tile maximum: (z - m) * log2 e
          auto y = [&](int e) { return fmaf(__uint_as_float(r[c][e]), kLog2e, -mL); };
          const uint32_t w0 = pack2<WsT>(y(e0), y(e0 + 1));
          const uint32_t w1 = pack2<WsT>(y(e0 + 2), y(e0 + 3));
          const uint32_t w2 = pack2<WsT>(y(e0 + 4), y(e0 + 5));
          const uint32_t w3 = pack2<WsT>(y(e0 + 6), y(e0 + 7));
          const uint32_t addr = staging + static_cast<uint32_t>(lane) * 128u +
                                ((static_cast<uint32_t>(q) ^ static_cast<uint32_t>(lane & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w0), "r"(w1), "r"(w2), "r"(w3)
                       : "memory");
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(ws_map, staging, static_cast<int32_t>(nh + hf * 64), static_cast<int32_t>(y0));
          bulk_commit_group();
        }
      }
    }
    if (row_ok) {
      p.tile_stats[(row * p.n_vtiles + tile) * kTileStats + (student ? TS_MAX_S : TS_MAX_T)] = m;
      if (label_col >= 0) p.label_logits[row * 2 + (student ? 0 : 1)] = zy;
    }
  }
}

// Softmax sums of the vocab tiles [n0, n0 + 256) of one row, read back from the workspace after this
// warp's TMA stores of them have completed: per 128-column tile, sum 2^y over its valid columns (the
// stored base-2 exponents relative to the tile maximum) and, at a temperature T != 1, sum 2^(y / T). Runs after the accumulator has been released,
// so its ex2 work overlaps the next tile's MMAs instead of delaying them. Every lane reads its own
// row (16-byte vectors through L2, where the stores have just landed).
template <typename WsT>
__device__ __forceinline__ void wide_tile_sums(const FwdEpiParams& p, int64_t row, int64_t n0, bool student) {
  if (row >= p.rows) return;
  const WsT* src = static_cast<const WsT*>(student ? p.ws_s : p.ws_t) + row * p.ld_ws + n0;
  const int tile0 = static_cast<int>(n0 / kVocabTile);
  const int ntiles = p.n_vtiles - tile0 < 2 ? p.n_vtiles - tile0 : 2;
  const bool tempered = (p.flags & F_T_NOT_ONE) != 0;  // also sum 2^(y / T) for the tempered softmax
  const float it = p.inv_t;
  for (int h = 0; h < ntiles; ++h) {
    const int64_t nh = n0 + h * kVocabTile;
    const int nvalid = static_cast<int>(p.vocab - nh < kVocabTile ? p.vocab - nh : kVocabTile);
    uint4 v[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) v[k] = __ldcg(reinterpret_cast<const uint4*>(src + h * kVocabTile) + k);
    float acc[4] = {0.f, 0.f, 0.f, 0.f}, accT[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const uint32_t w[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float a, b;
        unpack2<WsT>(w[q], a, b);
        const int col = k * 8 + q * 2;
        const bool va = nvalid == kVocabTile || col < nvalid, vb = nvalid == kVocabTile || col + 1 < nvalid;
        acc[q] += (va ? ex2_approx(a) : 0.f) + (vb ? ex2_approx(b) : 0.f);
        if (tempered) accT[q] += (va ? ex2_approx(a * it) : 0.f) + (vb ? ex2_approx(b * it) : 0.f);
      }
    }
    const float s1 = (acc[0] + acc[1]) + (acc[2] + acc[3]);
    if (tempered) {
      float* rec = p.tile_sums + (row * p.n_vtiles + tile0 + h) * 4 + (student ? 0 : 2);
      rec[0] = s1;
      rec[1] = (accT[0] + accT[1]) + (accT[2] + accT[3]);
    } else {
      p.tile_sums[(row * p.n_vtiles + tile0 + h) * 2 + (student ? 0 : 1)] = s1;
    }
  }
}

// Store epilogue through shared memory and TMA (16-bit output, N a multiple of 64; rows routed to
// peers go to the owner's slot through that owner's map): the warp's 32 rows x 256 columns leave as
// four 32 x 64 TMA stores of full 128-byte lines, instead of 16-byte stores one row per lane. When accumulating, each lane's previous 64 values are
// loaded before the TMEM wait and added in fp32 before the one rounding.
template <typename T16>
__device__ __forceinline__ void wide_store_tma(const TcGemmParams& p, uint32_t tbase, uint32_t staging, int64_t y0,
                                               int64_t n0, int lane) {
  const StoreEpiParams& st = p.st;
  const int64_t row = y0 + lane;
  const bool row_ok = row < st.M;
#pragma unroll 1
  for (int g = 0; g < kPairBN / 64; ++g) {
    const int64_t c0 = n0 + g * 64;
    uint4 prev[8];
    const T16* prev_base = static_cast<const T16*>(st.peers > 0 ? st.acc_src : st.out);
    const bool acc = st.accumulate && prev_base && row_ok && c0 < st.N;
    if (acc) {
      const uint4* src = reinterpret_cast<const uint4*>(prev_base + row * st.ldo + c0);
#pragma unroll
      for (int q = 0; q < 8; ++q) prev[q] = src[q];
    }
    uint32_t r[2][32];
    tmem_ld32_async(tbase + g * 64, r[0]);
    tmem_ld32_async(tbase + g * 64 + 32, r[1]);
    tmem_wait_ld();
    if (c0 >= st.N) continue;  // warp-uniform
    // the previous TMA store of this warp must have read the staging buffer
    if (lane == 0) bulk_wait_read_all();
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(r[q >> 2][(q & 3) * 8 + e]);
      if (acc) {
        const T16* ph = reinterpret_cast<const T16*>(&prev[q]);
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] += Conv<T16>::to_f(ph[e]);
      }
      const uint32_t addr = staging + static_cast<uint32_t>(lane) * 128u +
                            ((static_cast<uint32_t>(q) ^ static_cast<uint32_t>(lane & 7)) << 4);
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(pack2<T16>(v[0], v[1])),
                   "r"(pack2<T16>(v[2], v[3])), "r"(pack2<T16>(v[4], v[5])), "r"(pack2<T16>(v[6], v[7]))
                   : "memory");
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (st.peers > 0) {  // the whole 512-row tile belongs to one owner (slab_rows % 512 == 0)
        const int64_t owner = y0 / st.slab_rows;
        tma_store_2d(&p.peer_maps[owner], staging, static_cast<int32_t>(c0),
                     static_cast<int32_t>(y0 - owner * st.slab_rows));
      } else {
        tma_store_2d(&p.out_map, staging, static_cast<int32_t>(c0), static_cast<int32_t>(y0));
      }
      bulk_commit_group();
    }
  }
}

template <bool A_MN, bool B_MN, int AMODE, bool TWO_SEG, int EPI, typename T16>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(WideShape<EPI>::kThreads, 1)
    tc2w_gemm_kernel(const __grid_constant__ TcGemmParams p) {
  using S = WideShape<EPI>;
  constexpr uint32_t kIdesc = make_idesc_f16(std::is_same<T16, __nv_bfloat16>::value ? 1u : 0u, 256, kPairBN,
                                             A_MN ? 1u : 0u, B_MN ? 1u : 0u);
  constexpr uint32_t kTmemCols = 512;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t tiles_addr = (raw_addr + 1023u) & ~1023u;
  const uint32_t staging_addr = tiles_addr + S::kStages * kWideStageBytes;
  const uint32_t bar_addr = staging_addr + S::kStaging;
  auto full_bar = [&](int s) { return bar_addr + 8u * s; };
  auto empty_bar = [&](int s) { return bar_addr + 8u * (S::kStages + s); };
  const uint32_t tfull = bar_addr + 8u * (2 * S::kStages);
  auto tempty_bar = [&](int j) { return bar_addr + 8u * (2 * S::kStages + 1 + j); };
  const uint32_t tmem_slot = bar_addr + 8u * (2 * S::kStages + 4);
  uint32_t* tmem_slot_ptr = reinterpret_cast<uint32_t*>(smem_raw + (tmem_slot - raw_addr));

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const int32_t pair = blockIdx.x / 2, npairs = gridDim.x / 2;
  const int32_t mn_tiles = p.m_tiles * p.n_tiles;
  const int32_t ks_n = p.ksplit > 1 ? p.ksplit : 1;
  const int32_t num_tiles = mn_tiles * ks_n;
  const int32_t kb_total = TWO_SEG ? p.kb0 + p.kb1 : p.kb0;
  // work unit t -> output tile (mt, nt), k split ks, k blocks [kb_begin, kb_begin + kb_count)
  auto decode = [&](int32_t t, int32_t& mt, int32_t& nt, int32_t& ks, int32_t& kb_begin, int32_t& kb_count) {
    ks = t / mn_tiles;
    tile_coords(t - ks * mn_tiles, p.m_tiles, p.n_tiles, p.group_m, mt, nt);
    kb_begin = ks_n > 1 ? ks * p.kb_split : 0;
    kb_count = ks_n > 1 ? (kb_total - kb_begin < p.kb_split ? kb_total - kb_begin : p.kb_split) : kb_total;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(tfull, 1);
    for (int j = 0; j < 2; ++j) mbar_init(tempty_bar(j), 8);  // one elected lane per epilogue warp of both CTAs
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&p.a0);
    tma_prefetch_desc(&p.b0);
    if (AMODE == A_INTERLEAVE || TWO_SEG) tma_prefetch_desc(&p.a1);
    if (TWO_SEG) tma_prefetch_desc(&p.b1);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot_ptr;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      const bool prof = p.prof_slot >= 0;
      long long w_empty = 0, t_start = prof ? clk() : 0;
      for (int32_t t = pair; t < num_tiles && ok; t += npairs) {
        int32_t mt, nt, ks, kb_begin, kb_count;
        decode(t, mt, nt, ks, kb_begin, kb_count);
        const int32_t n_cta = nt * kPairBN + static_cast<int32_t>(rank) * 128;
        for (int32_t kbl = 0; kbl < kb_count; ++kbl) {
          const int32_t kb = kb_begin + kbl;
          const long long c0 = prof ? clk() : 0;
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.status)) { ok = false; break; }
          if (prof) w_empty += clk() - c0;
          const uint32_t sa = tiles_addr + stage * kWideStageBytes;
          const uint32_t sb = sa + 2 * kATileBytes;
          const uint32_t lead_full = map_to_cta(full_bar(stage), 0);
          if (rank == 0) mbar_arrive_expect_tx(full_bar(stage), 2 * kWideStageBytes);
          const bool seg1 = TWO_SEG && kb >= p.kb0;
          const int32_t k0 = (seg1 ? kb - p.kb0 : kb) * kBK;
          const CUtensorMap* amap = seg1 ? &p.a1 : &p.a0;
          const CUtensorMap* bmap = seg1 ? &p.b1 : &p.b0;
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const uint32_t saj = sa + j * kATileBytes;
            if constexpr (AMODE == A_INTERLEAVE) {
              const int32_t r = mt * 256 + j * 128 + static_cast<int32_t>(rank) * 64;
              tma_load_2d_pair(saj, &p.a0, lead_full, k0, r);
              tma_load_2d_pair(saj + 8192u, &p.a1, lead_full, k0, r);
            } else {
              const int32_t m_cta = mt * 512 + j * 256 + static_cast<int32_t>(rank) * 128;
              if constexpr (A_MN) {
                tma_load_2d_pair(saj, amap, lead_full, m_cta, k0);
                tma_load_2d_pair(saj + 8192u, amap, lead_full, m_cta + 64, k0);
              } else {
                tma_load_2d_pair(saj, amap, lead_full, k0, m_cta);
              }
            }
          }
          if constexpr (B_MN) {
            tma_load_2d_pair(sb, bmap, lead_full, n_cta, k0);
            tma_load_2d_pair(sb + 8192u, bmap, lead_full, n_cta + 64, k0);
          } else {
            tma_load_2d_pair(sb, bmap, lead_full, k0, n_cta);
          }
          if (++stage == S::kStages) { stage = 0; phase ^= 1u; }
        }
      }
      if (prof) {
        atomicAdd(&g_tc2_prof[p.prof_slot][5], static_cast<unsigned long long>(w_empty));
        atomicAdd(&g_tc2_prof[p.prof_slot][6], static_cast<unsigned long long>(clk() - t_start));
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader CTA only)
    if (rank == 0 && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      const bool prof = p.prof_slot >= 0;
      long long w_acc = 0, w_full = 0, t_start = prof ? clk() : 0;
      for (int32_t t = pair; t < num_tiles && ok; t += npairs, ++it) {
        const uint32_t bphase = static_cast<uint32_t>(it & 1);
        int32_t mt_u, nt_u, ks_u, kb_begin_u, kb_count;
        decode(t, mt_u, nt_u, ks_u, kb_begin_u, kb_count);
        (void)mt_u; (void)nt_u; (void)ks_u; (void)kb_begin_u;
        // Head of the tile: the first `nhead` stages feed accumulator 0 as soon as the epilogue has
        // drained it, while the epilogue still drains accumulator 1; then the same stages feed
        // accumulator 1. After the head both accumulators advance together stage by stage.
        const int32_t nhead = kb_count < S::kStages ? kb_count : S::kStages;
        const int stage0 = stage;
        long long c0 = prof ? clk() : 0;
        if (!mbar_wait_cluster(tempty_bar(0), bphase ^ 1u, p.status)) { ok = false; break; }
        if (prof) w_acc += clk() - c0;
        tc_fence_after();
        for (int32_t kb = 0; kb < nhead; ++kb) {
          if (prof) c0 = clk();
          if (!mbar_wait(full_bar(stage), phase, p.status)) { ok = false; break; }
          if (prof) w_full += clk() - c0;
          tc_fence_after();
          const uint32_t sa = tiles_addr + stage * kWideStageBytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            tc_mma_f16_pair(tmem_base, operand_desc<A_MN>(sa, kk), operand_desc<B_MN>(sa + 2 * kATileBytes, kk),
                            kIdesc, (kb | kk) != 0);
          if (++stage == S::kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        if (prof) c0 = clk();
        if (!mbar_wait_cluster(tempty_bar(1), bphase ^ 1u, p.status)) { ok = false; break; }
        if (prof) w_acc += clk() - c0;
        tc_fence_after();
        for (int32_t kb = 0; kb < nhead; ++kb) {
          const int hs = (stage0 + kb) % S::kStages;
          const uint32_t sa = tiles_addr + hs * kWideStageBytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            tc_mma_f16_pair(tmem_base + kPairBN, operand_desc<A_MN>(sa + kATileBytes, kk),
                            operand_desc<B_MN>(sa + 2 * kATileBytes, kk), kIdesc, (kb | kk) != 0);
          tc_commit_pair_mc(empty_bar(hs), 3);
        }
        for (int32_t kb = nhead; kb < kb_count; ++kb) {
          if (prof) c0 = clk();
          // the stage's bytes of both CTAs complete on this CTA's barrier: a CTA-scope wait suffices
          if (!mbar_wait(full_bar(stage), phase, p.status)) { ok = false; break; }
          if (prof) w_full += clk() - c0;
          tc_fence_after();
          const uint32_t sa = tiles_addr + stage * kWideStageBytes;
          const uint32_t sb = sa + 2 * kATileBytes;
#pragma unroll
          for (int jj = 0; jj < 2; ++jj)
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              tc_mma_f16_pair(tmem_base + jj * kPairBN, operand_desc<A_MN>(sa + jj * kATileBytes, kk),
                              operand_desc<B_MN>(sb, kk), kIdesc, 1u);
          tc_commit_pair_mc(empty_bar(stage), 3);  // frees the stage in both CTAs with one commit
          if (++stage == S::kStages) { stage = 0; phase ^= 1u; }
        }
        if (ok) {
          tc_commit_pair(map_to_cta(tfull, 0));
          tc_commit_pair(map_to_cta(tfull, 1));
        }
      }
      if (prof) {
        atomicAdd(&g_tc2_prof[p.prof_slot][0], static_cast<unsigned long long>(w_acc));
        atomicAdd(&g_tc2_prof[p.prof_slot][1], static_cast<unsigned long long>(w_full));
        atomicAdd(&g_tc2_prof[p.prof_slot][2], static_cast<unsigned long long>(clk() - t_start));
        atomicAdd(&g_tc2_prof[p.prof_slot][7], static_cast<unsigned long long>(it));
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2.., both CTAs)
    // TMEM lanes 32*(warp % 4) .. +31 belong to this warp; with 8 epilogue warps, warps 2..5 drain
    // accumulator 0 and warps 6..9 accumulator 1
    const int quarter = warp & 3;
    const int ew = warp - 2;
    const int j_first = S::kEpiWarps == 8 ? (ew >> 2) : 0, j_last = S::kEpiWarps == 8 ? (ew >> 2) : 1;
    const uint32_t staging = staging_addr + static_cast<uint32_t>(ew) * kWideStagingPerWarp;
    int it = 0;
    const bool prof = p.prof_slot >= 0 && warp == 2 && lane == 0;
    long long w_tfull = 0, busy = 0;

    for (int32_t t = pair; t < num_tiles; t += npairs, ++it) {
      // labels of this lane's two rows, loaded before the wait so their latency is hidden
      int64_t lab[2] = {0, 0};
      if constexpr (EPI == EPI_FWD_STATS) {
        int32_t mt0, nt0, ks0, kbb0, kbc0;
        decode(t, mt0, nt0, ks0, kbb0, kbc0);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          if (j < j_first || j > j_last) continue;
          const int64_t row = AMODE == A_INTERLEAVE
                                  ? static_cast<int64_t>(mt0) * 256 + j * 128 + rank * 64 + (quarter & 1) * 32 + lane
                                  : static_cast<int64_t>(mt0) * 512 + j * 256 + rank * 128 + quarter * 32 + lane;
          if (row < p.fwd.rows) lab[j] = p.fwd.labels[row];
        }
      }
      if constexpr (EPI == EPI_STORE) {
        // accumulating store (a later row chunk of dW): pull this lane's previous values of the tile
        // into L2 while the MMAs still run, so the read-modify-write after the wait hits L2
        if (p.st.accumulate) {
          int32_t mt0, nt0, ks0, kbb0, kbc0;
          decode(t, mt0, nt0, ks0, kbb0, kbc0);
          const int64_t n0p = static_cast<int64_t>(nt0) * kPairBN;
          const void* prev = p.st.peers > 0 ? p.st.acc_src : p.st.out;
          const int64_t es = p.st.out_f32 ? 4 : 2;
          if (prev && n0p < p.st.N) {
            const int64_t bytes = (p.st.N - n0p < kPairBN ? p.st.N - n0p : kPairBN) * es;
            for (int j = j_first; j <= j_last; ++j) {
              const int64_t row = static_cast<int64_t>(mt0) * 512 + j * 256 + rank * 128 + quarter * 32 + lane;
              if (row >= p.st.M) continue;
              const char* base = static_cast<const char*>(prev) + (row * p.st.ldo + n0p) * es;
              for (int64_t off = 0; off < bytes; off += 128)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(base + off));
            }
          }
        }
      }
      const long long c0 = prof ? clk() : 0;
      if (!mbar_wait(tfull, static_cast<uint32_t>(it & 1), p.status)) break;
      const long long c1 = prof ? clk() : 0;
      if (prof) w_tfull += c1 - c0;
      tc_fence_after();
      int32_t mt, nt, ks, kbb, kbc;
      decode(t, mt, nt, ks, kbb, kbc);
      const int64_t n0 = static_cast<int64_t>(nt) * kPairBN;
#pragma unroll 1
      for (int j = j_first; j <= j_last; ++j) {
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + j * kPairBN;
        if constexpr (EPI == EPI_FWD_STATS) {
          if constexpr (AMODE == A_INTERLEAVE) {
            const bool student = quarter < 2;
            const int64_t y0 = static_cast<int64_t>(mt) * 256 + j * 128 + rank * 64 + (quarter & 1) * 32;
            const bool write_ws = (p.fwd.flags & (student ? F_WRITE_WS_S : F_WRITE_WS_T)) != 0;
            wide_fwd_acc<T16>(p.fwd, student ? &p.ws_s_map : &p.ws_t_map, write_ws, tbase, staging, y0 + lane, y0, n0,
                              student, lane, j ? lab[1] : lab[0]);
          } else {
            const int64_t y0 = static_cast<int64_t>(mt) * 512 + j * 256 + rank * 128 + quarter * 32;
            const bool tdist = p.fwd.plain_teacher != 0;  // separate teacher: a second launch over (ht, Wt)
            wide_fwd_acc<T16>(p.fwd, tdist ? &p.ws_t_map : &p.ws_s_map,
                              (p.fwd.flags & (tdist ? F_WRITE_WS_T : F_WRITE_WS_S)) != 0, tbase, staging, y0 + lane,
                              y0, n0, !tdist, lane, j ? lab[1] : lab[0]);
          }
        } else {
          const int64_t y0 = static_cast<int64_t>(mt) * 512 + j * 256 + rank * 128 + quarter * 32;
          if (p.st_tma) {
            wide_store_tma<T16>(p, tbase, staging, y0, n0, lane);
          } else {
            StoreEpiParams st = p.st;
            if (ks_n > 1) st.out = static_cast<uint8_t*>(st.out) + ks * p.split_bytes;
            store_epilogue<T16>(st, tbase, y0 + lane, n0, kPairBN);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (rank == 0) mbar_arrive(tempty_bar(j));
          else mbar_arrive_cluster(map_to_cta(tempty_bar(j), 0));
        }
        if constexpr (EPI == EPI_FWD_STATS) {
          if (p.fwd.tile_sums) {
            // the accumulator is free again; the softmax sums come from the tile just stored
            if (lane == 0) {
              bulk_wait_all();
              fence_proxy_async_global();
            }
            __syncwarp();
            int64_t row, y0;
            bool student;
            if constexpr (AMODE == A_INTERLEAVE) {
              student = quarter < 2;
              y0 = static_cast<int64_t>(mt) * 256 + j * 128 + rank * 64 + (quarter & 1) * 32;
            } else {
              student = p.fwd.plain_teacher == 0;
              y0 = static_cast<int64_t>(mt) * 512 + j * 256 + rank * 128 + quarter * 32;
            }
            row = y0 + lane;
            wide_tile_sums<T16>(p.fwd, row, n0, student);
          }
        }
      }
      if (prof) busy += clk() - c1;
    }
    if (EPI == EPI_FWD_STATS || p.st_tma) {
      if (lane == 0) bulk_wait_all();  // staged stores complete before the shared memory goes away
    }
    if constexpr (EPI != EPI_FWD_STATS) {
      // stores routed to other GPUs are visible system-wide once this kernel has finished
      if (p.st.peers > 0) __threadfence_system();
    }
    if (prof) {
      atomicAdd(&g_tc2_prof[p.prof_slot][3], static_cast<unsigned long long>(w_tfull));
      atomicAdd(&g_tc2_prof[p.prof_slot][4], static_cast<unsigned long long>(busy));
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer's epilogue and the leader's MMAs are all done before TMEM is freed
  if (warp == 1) {
    tc_fence_after();
    if (*reinterpret_cast<volatile int32_t*>(p.status) == ORDA_ERR_TIMEOUT) __nanosleep(1000000);
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

}  // namespace orda
