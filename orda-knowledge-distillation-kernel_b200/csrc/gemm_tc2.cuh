// Persistent warp-specialised tcgen05 GEMM on CTA pairs (cta_group::2), 256 x 256 tiles, storing D.
//
// A pair of CTAs (a 2-CTA cluster) computes one 256-row x 256-column tile: each CTA loads its own
// 128 A rows and its own half (128 rows or columns) of the B tile, the leader CTA issues
// tcgen05.mma.cta_group::2 (M=256, N=256) and both CTAs receive a 128 x 256 fp32 accumulator in
// their own TMEM. Two accumulator buffers (512 TMEM columns) let the epilogue of one tile overlap
// the mainloop of the next. Every CTA loads only the tiles it consumes (no multicast).
// Used for dHidden (few output tiles: 256 x 256 tiles fill more SMs than the 512 x 256 tiles of the
// wide kernel in gemm_tc2w.cuh) and for the testing GEMM.
//
//   warp 0 (each CTA) : TMA producer; transaction bytes of both CTAs land on the leader's barrier
//   warp 1 (leader)   : MMA issuer; one multicast commit releases the smem stage in both CTAs
//   warps 2..5        : epilogue of the CTA's own 128 accumulator rows
//
// A modes (the wide kernel uses the same names):
//   A_PLAIN      : 128 consecutive rows of A0 per CTA (a pair covers 256 rows)
//   A_INTERLEAVE : tied teacher - TMEM lanes 0..63 hold 64 student rows (A0) and lanes 64..127 the
//                  SAME 64 rows of the teacher (A1); one lm_head stream feeds both distributions.
// TWO_SEG: (A0, B0) over K0 then (A1, B1) over K1 into one accumulator (dW of the tied teacher).
#pragma once

#include "distill_common.cuh"
#include "fwd_epilogue.cuh"
#include "gemm_tc.cuh"
#include "sm100_ptx.cuh"

namespace orda {

enum AMode { A_PLAIN = 0, A_INTERLEAVE = 1 };

constexpr int kPairBN = 256;                           // tile columns of a pair
constexpr uint32_t kPairStageBytes = 2 * kATileBytes;  // per CTA: A 128x64 + B-half 128x64

// Pipeline counters of the pair kernel (testing hook, enabled per launch by prof_slot >= 0), in SM
// clock cycles summed over CTAs: [0] MMA issuer waiting for a free accumulator, [1] MMA issuer waiting
// for a loaded stage, [2] MMA issuer total, [3] epilogue waiting for a finished accumulator,
// [4] epilogue working, [5] producer waiting for a free stage, [6] producer total, [7] tiles.
constexpr int kProfSlots = 4;
__device__ unsigned long long g_tc2_prof[kProfSlots][8];

__device__ __forceinline__ long long clk() { return clock64(); }

template <int AMODE>
struct PairShape {
  static constexpr int kStages = 6;
  static constexpr uint32_t kBarBytes = (2 * kStages + 4) * 8 + 16;
  static constexpr uint32_t kSmemBytes = kStages * kPairStageBytes + kBarBytes + 1024;
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
};

template <bool A_MN, bool B_MN, int AMODE, bool TWO_SEG, int EPI, typename T16>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    tc2_gemm_kernel(const __grid_constant__ TcGemmParams p) {
  static_assert(EPI == EPI_STORE, "the 256 x 256 pair kernel stores D; the logits epilogue runs in the wide kernel");
  using S = PairShape<AMODE>;
  constexpr uint32_t kIdesc = make_idesc_f16(std::is_same<T16, __nv_bfloat16>::value ? 1u : 0u, 256, kPairBN,
                                             A_MN ? 1u : 0u, B_MN ? 1u : 0u);
  constexpr uint32_t kTmemCols = 512;  // two 256-column accumulator buffers

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t tiles_addr = (raw_addr + 1023u) & ~1023u;
  const uint32_t bar_addr = tiles_addr + S::kStages * kPairStageBytes;
  auto full_bar = [&](int s) { return bar_addr + 8u * s; };
  auto empty_bar = [&](int s) { return bar_addr + 8u * (S::kStages + s); };
  auto tfull_bar = [&](int b) { return bar_addr + 8u * (2 * S::kStages + b); };
  auto tempty_bar = [&](int b) { return bar_addr + 8u * (2 * S::kStages + 2 + b); };
  const uint32_t tmem_slot = bar_addr + 8u * (2 * S::kStages + 4);
  uint32_t* tmem_slot_ptr = reinterpret_cast<uint32_t*>(smem_raw + (tmem_slot - raw_addr));

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const int32_t pair = blockIdx.x / 2, npairs = gridDim.x / 2;
  const int32_t num_tiles = p.m_tiles * p.n_tiles;
  const int32_t kb_total = TWO_SEG ? p.kb0 + p.kb1 : p.kb0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull_bar(b), 1);
      mbar_init(tempty_bar(b), 8);  // one elected lane per epilogue warp of both CTAs
    }
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
        int32_t mt, nt;
        tile_coords(t, p.m_tiles, p.n_tiles, p.group_m, mt, nt);
        const int32_t n_cta = nt * kPairBN + static_cast<int32_t>(rank) * 128;
        for (int32_t kb = 0; kb < kb_total; ++kb) {
          const long long c0 = prof ? clk() : 0;
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.status)) { ok = false; break; }
          if (prof) w_empty += clk() - c0;
          const uint32_t sa = tiles_addr + stage * kPairStageBytes;
          const uint32_t sb = sa + kATileBytes;
          const uint32_t lead_full = map_to_cta(full_bar(stage), 0);
          if (rank == 0) mbar_arrive_expect_tx(full_bar(stage), 2 * kPairStageBytes);
          const bool seg1 = TWO_SEG && kb >= p.kb0;
          const int32_t k0 = (seg1 ? kb - p.kb0 : kb) * kBK;
          const CUtensorMap* amap = seg1 ? &p.a1 : &p.a0;
          const CUtensorMap* bmap = seg1 ? &p.b1 : &p.b0;
          if constexpr (AMODE == A_INTERLEAVE) {
            const int32_t r = mt * 128 + static_cast<int32_t>(rank) * 64;
            tma_load_2d_pair(sa, &p.a0, lead_full, k0, r);
            tma_load_2d_pair(sa + 8192u, &p.a1, lead_full, k0, r);
          } else {
            const int32_t m_cta = mt * 256 + static_cast<int32_t>(rank) * 128;
            if constexpr (A_MN) {
              tma_load_2d_pair(sa, amap, lead_full, m_cta, k0);
              tma_load_2d_pair(sa + 8192u, amap, lead_full, m_cta + 64, k0);
            } else {
              tma_load_2d_pair(sa, amap, lead_full, k0, m_cta);
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
        const int buf = it & 1;
        const uint32_t bphase = (it >> 1) & 1;
        long long c0 = prof ? clk() : 0;
        if (!mbar_wait_cluster(tempty_bar(buf), bphase ^ 1u, p.status)) { ok = false; break; }
        if (prof) w_acc += clk() - c0;
        tc_fence_after();
        const uint32_t acc = tmem_base + buf * kPairBN;
        for (int32_t kb = 0; kb < kb_total; ++kb) {
          if (prof) c0 = clk();
          // the stage's bytes of both CTAs complete on this CTA's barrier: a CTA-scope wait suffices
          if (!mbar_wait(full_bar(stage), phase, p.status)) { ok = false; break; }
          if (prof) w_full += clk() - c0;
          tc_fence_after();
          const uint32_t sa = tiles_addr + stage * kPairStageBytes;
          const uint32_t sb = sa + kATileBytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            tc_mma_f16_pair(acc, operand_desc<A_MN>(sa, kk), operand_desc<B_MN>(sb, kk), kIdesc, (kb | kk) != 0);
          tc_commit_pair_mc(empty_bar(stage), 3);  // frees the stage in both CTAs with one commit
          if (++stage == S::kStages) { stage = 0; phase ^= 1u; }
        }
        if (ok) {
          tc_commit_pair(map_to_cta(tfull_bar(buf), 0));
          tc_commit_pair(map_to_cta(tfull_bar(buf), 1));
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
    // ------------------------------------------------------------ epilogue (warps 2..5, both CTAs)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    int it = 0;
    const bool prof = p.prof_slot >= 0 && warp == 2 && lane == 0;
    long long w_tfull = 0, busy = 0;
    for (int32_t t = pair; t < num_tiles; t += npairs, ++it) {
      const int buf = it & 1;
      const uint32_t bphase = (it >> 1) & 1;
      const long long c0 = prof ? clk() : 0;
      if (!mbar_wait(tfull_bar(buf), bphase, p.status)) break;
      const long long c1 = prof ? clk() : 0;
      if (prof) w_tfull += c1 - c0;
      tc_fence_after();
      int32_t mt, nt;
      tile_coords(t, p.m_tiles, p.n_tiles, p.group_m, mt, nt);
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + buf * kPairBN;
      const int64_t n0 = static_cast<int64_t>(nt) * kPairBN;
      const int64_t row = static_cast<int64_t>(mt) * 256 + rank * 128 + r;
      store_epilogue<T16>(p.st, tbase, row, n0, kPairBN);
      tc_fence_before();
      __syncwarp();
      if (prof) busy += clk() - c1;
      if (lane == 0) {
        if (rank == 0) mbar_arrive(tempty_bar(buf));
        else mbar_arrive_cluster(map_to_cta(tempty_bar(buf), 0));
      }
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
