// Row-wise kernels between the logits GEMM and the gradient GEMMs.
//
//   row_merge_kernel   : merge the per-(row, vocab tile) records of one shard into a row record
//   merge_records_kernel: LSE-merge row records gathered from several vocab shards
//   row_loss_kernel    : per-row student CE, teacher CE and divergence from a (global) row record
//   jsd_sweep_kernel   : per-row JSD value and sum_j p_s g_j (needs the full row)
//   grad_sweep_kernel  : dlogits written in place over the shifted logits (workspace)
//   finalize_kernel    : deterministic reduction of the per-row losses to the reference's scalars
//
// Math follows the reference row kernels (ops/tied_teacher.py:116-189) and the torch formula
// (api.py:302-334); reverse KL and JSD follow the restatements documented in the C ABI header.
#pragma once

#include "distill_common.cuh"
#include "orda_b200.h"

namespace orda {

struct RowParams {
  int64_t rows;           // rows of this chunk
  int64_t vocab, vocab_offset, vocab_total;
  int64_t ignore_index;
  int32_t n_vtiles;
  uint32_t flags;
  float temperature, inv_t, jsd_beta;
  float w_s, w_t, w_kl;   // student CE, teacher CE, divergence weights
  const int64_t* labels;  // chunk labels
  const float* tile_stats;
  const float* label_logits;
  float* row_stats;       // [rows][kRowStats]
  const float* row_sums;  // [rows][2] JSD value / sum p_s g (JSD only)
  float* row_losses;      // [3][ld_row_losses] (student CE, teacher CE, divergence), chunk-offset
  int64_t ld_row_losses;
  void* ws_s; void* ws_t; int64_t ld_ws;
  const void* t_gmem; int64_t ld_tg; int32_t tg_dtype;
  int32_t tg_vec;         // teacher rows 16-byte aligned (vector loads)
  int32_t* status;
  const float* grad_scale;  // optional device scalar multiplying the dlogits (1/count for mean)
  // Column parts: each row is swept as `parts` column ranges of `part_cols` (a multiple of 256)
  // handled by different warps, so that the number of warp tasks balances over the SMs. With
  // parts > 1 row_stats writes one record per part into part_records[part][rows][kRowStats]; the
  // records are merged like vocab shards.
  int32_t parts;
  int64_t part_cols;
  float* part_records;
  // Epilogue-statistics path (16-bit, T = 1, teacher from an accumulator or none): the logits
  // epilogue wrote per-tile softmax sums (tile_sums, [rows][n_vtiles] float2), so the row records come
  // from tile_merge_kernel instead of a pass over the logits. The divergence's row sums go to
  // cross_parts ([parts][rows], JSD [2][parts][rows]): the forward-KL cross term
  // sum_j p_t,j (u_j - z_j) from the dlogits sweep, reverse KL's R and JSD's J and G from
  // div_sweep_kernel before it.
  const float* tile_sums;
  float* cross_parts;
};

// Column range [c0, c1) of part `part` of a row.
__device__ __forceinline__ void part_range(const RowParams& p, int part, int64_t& c0, int64_t& c1) {
  c0 = static_cast<int64_t>(part) * p.part_cols;
  c1 = c0 + p.part_cols < p.vocab ? c0 + p.part_cols : p.vocab;
}

__device__ __forceinline__ Partial warp_merge(Partial a, double inv_t, bool cross) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    Partial b;
    b.max_v = __shfl_down_sync(0xffffffffu, a.max_v, off);
    b.sum1 = __shfl_down_sync(0xffffffffu, a.sum1, off);
    b.sumt = __shfl_down_sync(0xffffffffu, a.sumt, off);
    b.cross = __shfl_down_sync(0xffffffffu, a.cross, off);
    merge_partial(a, b, inv_t, cross);
  }
  return a;
}

// gathered[world][rows][kRowStats] -> out[rows][kRowStats]
__global__ void merge_records_kernel(const float* gathered, int world, int64_t rows, float* out) {
  for (int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; row < rows; row += (int64_t)gridDim.x * blockDim.x) {
    const float* r0 = gathered + row * kRowStats;
    const bool cross_t = r0[10] != 0.f;
    const double inv_t = r0[11];
    Partial s{-CUDART_INF, 0.0, 0.0, 0.0}, t{-CUDART_INF, 0.0, 0.0, 0.0};
    float ls = 0.f, lt = 0.f, has = 0.f;
    for (int w = 0; w < world; ++w) {
      const float* r = gathered + ((int64_t)w * rows + row) * kRowStats;
      Partial ps{r[RS_MAX_S], r[RS_SUM1_S], r[RS_SUMT_S], cross_t ? 0.0 : (double)r[RS_CROSS]};
      Partial pt{r[RS_MAX_T], r[RS_SUM1_T], r[RS_SUMT_T], cross_t ? (double)r[RS_CROSS] : 0.0};
      merge_partial(s, ps, inv_t, !cross_t);
      merge_partial(t, pt, inv_t, cross_t);
      if (r[RS_HAS_LABEL] != 0.f) {
        ls = r[RS_LABEL_S];
        lt = r[RS_LABEL_T];
        has = 1.f;
      }
    }
    float* o = out + row * kRowStats;
    o[RS_MAX_S] = (float)s.max_v; o[RS_SUM1_S] = (float)s.sum1; o[RS_SUMT_S] = (float)s.sumt;
    o[RS_MAX_T] = (float)t.max_v; o[RS_SUM1_T] = (float)t.sum1; o[RS_SUMT_T] = (float)t.sumt;
    o[RS_CROSS] = (float)(cross_t ? t.cross : s.cross);
    o[RS_LABEL_S] = ls; o[RS_LABEL_T] = lt; o[RS_HAS_LABEL] = has;
    o[10] = cross_t ? 1.f : 0.f; o[11] = (float)inv_t;
    for (int k = 12; k < kRowStats; ++k) o[k] = 0.f;
  }
}

// Per-row losses from the (global) row record.
__device__ __forceinline__ void row_loss_one(const RowParams& p, int64_t row) {
  const float* r = p.row_stats + row * kRowStats;
  bool ignored;
  safe_label(p.labels[row], p.ignore_index, p.vocab_total, &ignored);
  double ce_s = 0.0, ce_t = 0.0, div = 0.0;
  if (!ignored) {
    const double lse_s = (double)r[RS_MAX_S] + log((double)r[RS_SUM1_S]);
    ce_s = lse_s - (double)r[RS_LABEL_S];
    if (p.flags & F_TEACHER_CE) {
      const double lse_t = (double)r[RS_MAX_T] + log((double)r[RS_SUM1_T]);
      ce_t = lse_t - (double)r[RS_LABEL_T];
    }
    if (p.flags & F_KL) {
      const double t = p.temperature, it = p.inv_t;
      if (p.cross_parts && (p.flags & (F_JSD | F_KL_REVERSE | F_T_NOT_ONE))) {
        // reverse KL (R), JSD (J), or at T != 1 forward KL, of the tempered distributions, summed
        // over the sweeps' parts
        for (int k = 0; k < p.parts; ++k) div += (double)p.cross_parts[(int64_t)k * p.rows + row];
        div *= t * t;
      } else if (p.flags & F_JSD) {
        div = p.row_sums[row * 2] * t * t;
      } else if (p.cross_parts) {
        // T = 1 forward KL: sum_j p_t (u_j - z_j) - lse_t + lse_s, the cross sum from the dlogits sweep
        double cr = 0.0;
        for (int k = 0; k < p.parts; ++k) cr += (double)p.cross_parts[(int64_t)k * p.rows + row];
        const double lse_t = (double)r[RS_MAX_T] + log((double)r[RS_SUM1_T]);
        div = cr - lse_t + lse_s;
      } else {
        const double lse_st = (double)r[RS_MAX_S] * it + log((double)r[RS_SUMT_S]);
        const double lse_tt = (double)r[RS_MAX_T] * it + log((double)r[RS_SUMT_T]);
        if (p.flags & F_KL_REVERSE) div = ((double)r[RS_CROSS] / r[RS_SUMT_S] - lse_st + lse_tt) * t * t;
        else div = ((double)r[RS_CROSS] / r[RS_SUMT_T] - lse_tt + lse_st) * t * t;
      }
    }
  }
  p.row_losses[row] = (float)ce_s;
  p.row_losses[p.ld_row_losses + row] = (float)ce_t;
  p.row_losses[2 * p.ld_row_losses + row] = (float)div;
}

// One thread per row.
__global__ void row_loss_kernel(RowParams p) {
  for (int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; row < p.rows; row += (int64_t)gridDim.x * blockDim.x)
    row_loss_one(p, row);
}

template <typename T>
__device__ __forceinline__ void load8(const T* src, float (&v)[8]) {
  if constexpr (sizeof(T) == 2) {
    const uint4 u = *reinterpret_cast<const uint4*>(src);
    const T* h = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = Conv<T>::to_f(h[j]);
  } else {
    const float4 a = reinterpret_cast<const float4*>(src)[0];
    const float4 b = reinterpret_cast<const float4*>(src)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* dst, const float (&v)[8]) {
  if constexpr (sizeof(T) == 2) {
    uint4 u;
    T* h = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int j = 0; j < 8; ++j) h[j] = Conv<T>::from_f(v[j]);
    *reinterpret_cast<uint4*>(dst) = u;
  } else {
    reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

// Eight teacher logits [j0, j0 + 8) of a row from the caller's buffer; columns at or past `cnt` get
// `fill`. Rows whose base and stride are 16-byte aligned (tg_vec) are read with two (fp32) or one
// (16-bit) 16-byte loads.
__device__ __forceinline__ float load_tg(const RowParams& p, int64_t row, int64_t col);
__device__ __forceinline__ void load_tg8(const RowParams& p, int64_t row, int64_t j0, int cnt, float fill,
                                         float (&u)[8]) {
  if (cnt >= 8 && p.tg_vec) {
    if (p.tg_dtype == ORDA_F32) {
      const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(p.t_gmem) + row * p.ld_tg + j0);
      const float4 a = __ldg(q), b = __ldg(q + 1);
      u[0] = a.x; u[1] = a.y; u[2] = a.z; u[3] = a.w; u[4] = b.x; u[5] = b.y; u[6] = b.z; u[7] = b.w;
    } else {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.t_gmem) + row * p.ld_tg + j0));
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (p.tg_dtype == ORDA_BF16) unpack2<__nv_bfloat16>(ws[q], u[2 * q], u[2 * q + 1]);
        else unpack2<__half>(ws[q], u[2 * q], u[2 * q + 1]);
      }
    }
    return;
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) u[j] = j < cnt ? load_tg(p, row, j0 + j) : fill;
}

__device__ __forceinline__ float load_tg(const RowParams& p, int64_t row, int64_t col) {
  if (p.tg_dtype == ORDA_F32) return __ldg(static_cast<const float*>(p.t_gmem) + row * p.ld_tg + col);
  if (p.tg_dtype == ORDA_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p.t_gmem)[row * p.ld_tg + col]);
  return __half2float(static_cast<const __half*>(p.t_gmem)[row * p.ld_tg + col]);
}

// Per-row constants of the sweep kernels.
struct RowConsts {
  float ms, log_s1, log_st;  // student row max, log sum exp at T=1, at T
  float mt, log_t1, log_tt;  // teacher
  bool ignored;
  int64_t label_local;       // label column in this shard, or -1
};

__device__ __forceinline__ RowConsts row_consts(const RowParams& p, int64_t row) {
  const float* r = p.row_stats + row * kRowStats;
  RowConsts c;
  c.ms = r[RS_MAX_S];
  c.log_s1 = logf(r[RS_SUM1_S]);
  c.log_st = logf(r[RS_SUMT_S]);
  c.mt = r[RS_MAX_T];
  c.log_t1 = logf(r[RS_SUM1_T]);
  c.log_tt = logf(r[RS_SUMT_T]);
  const int64_t ys = safe_label(p.labels[row], p.ignore_index, p.vocab_total, &c.ignored);
  c.label_local = (!c.ignored && ys >= p.vocab_offset && ys < p.vocab_offset + p.vocab) ? ys - p.vocab_offset : -1;
  return c;
}

// The sweep kernels run one warp per row (no block-wide synchronisation); each lane handles vectors
// of 8 consecutive vocabulary columns, 256 columns apart. Tile maxima are read from the [row][tile]
// float2 array through the read-only cache (a warp touches at most two tiles per step).
__device__ __forceinline__ const float2* row_tile_maxima(const RowParams& p, int64_t row) {
  return reinterpret_cast<const float2*>(p.tile_stats) + row * p.n_vtiles;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// Loads 8 consecutive (student, teacher) values as offsets from the ROW maxima:
//   ds = z - max_s ; dt = u - max_t
template <typename WsT>
__device__ __forceinline__ void load_row8(const RowParams& p, int64_t row, int64_t j0, const float2* tm,
                                          const RowConsts& c, bool need_t, float (&ds)[8], float (&dt)[8]) {
  const float2 m = __ldg(tm + j0 / kVocabTile);
  load8<WsT>(static_cast<const WsT*>(p.ws_s) + row * p.ld_ws + j0, ds);
  const float off_s = m.x - c.ms;
#pragma unroll
  for (int j = 0; j < 8; ++j) ds[j] = fmaf(ds[j], kLn2, off_s);
  if (need_t) {
    if (p.flags & F_TEACHER_GMEM) {
      // columns past the vocabulary read as the row maximum, i.e. offset 0 (they are never used)
      load_tg8(p, row, j0, static_cast<int>(p.vocab - j0 < 8 ? p.vocab - j0 : 8), c.mt, dt);
#pragma unroll
      for (int j = 0; j < 8; ++j) dt[j] -= c.mt;
    } else {
      load8<WsT>(static_cast<const WsT*>(p.ws_t) + row * p.ld_ws + j0, dt);
      const float off_t = m.y - c.mt;
#pragma unroll
      for (int j = 0; j < 8; ++j) dt[j] = fmaf(dt[j], kLn2, off_t);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) dt[j] = 0.f;
  }
}

// Teacher source of the row kernels (compile-time).
enum TeacherSrc { TS_NONE = 0, TS_WS = 1, TS_GMEM = 2 };
// Divergence kind of the gradient kernel (compile-time).
enum DivKind { DK_NONE = 0, DK_FWD = 1, DK_REV = 2, DK_JSD = 3 };

// One warp per row: softmax statistics of this shard's part of the row, streamed from the shifted
// logits in the workspace (and from the caller's teacher logits for a precomputed teacher):
//   sum exp(z - M) and sum exp((z - M)/T) for the student and the teacher, and the divergence cross
//   term (forward: sum exp((u - M_t)/T) (u - z)/T, reverse: sum exp((z - M_s)/T) (z - u)/T),
// plus the exact label logits kept by the GEMM epilogue. Writes the row record (shard-local maxima).
// Student / workspace-teacher maxima come from the epilogue's tile maxima; a caller-provided teacher
// row is normalised on the fly (running maximum, rescaled sums). Each lane keeps two sets of
// accumulators (even / odd columns) to shorten the dependency chains.
template <typename WsT, int TSRC, bool TNO>
__global__ void __launch_bounds__(256, 4) row_stats_kernel(RowParams p) {
  const uint32_t f = p.flags;
  constexpr bool teacher = TSRC != TS_NONE;
  const bool need_t1 = f & F_TEACHER_CE, kl = f & F_KL, rev = f & F_KL_REVERSE;
  const float it = p.inv_t;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const int64_t tasks = p.rows * p.parts;
  for (int64_t task = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; task < tasks; task += warps) {
    const int64_t row = task / p.parts;
    const int part = static_cast<int>(task - row * p.parts);
    int64_t c0, c1;
    part_range(p, part, c0, c1);
    const float2* tm = row_tile_maxima(p, row);
    float lms = -CUDART_INF_F, lmt = -CUDART_INF_F;
    const int t1 = static_cast<int>((c1 + kVocabTile - 1) / kVocabTile);
    for (int i = static_cast<int>(c0 / kVocabTile) + lane; i < t1; i += 32) {
      const float2 m = __ldg(tm + i);
      lms = fmaxf(lms, m.x);
      lmt = fmaxf(lmt, m.y);
    }
    const float Ms = warp_max(lms);
    float mt = (TSRC == TS_WS) ? warp_max(lmt) : -CUDART_INF_F;  // running maximum for a caller teacher
    float s1s[2] = {0.f, 0.f}, sts[2] = {0.f, 0.f}, s1t[2] = {0.f, 0.f}, stt[2] = {0.f, 0.f}, cross[2] = {0.f, 0.f};
    const WsT* rs = static_cast<const WsT*>(p.ws_s) + row * p.ld_ws;
    const WsT* rt = static_cast<const WsT*>(p.ws_t) + row * p.ld_ws;
    if constexpr (!TNO && TSRC == TS_GMEM) {
      // T = 1, the caller's teacher logits: everything in base 2. The student exponents are the
      // stored ones plus the tile offset; the teacher's are u log2 e against a per-lane running
      // maximum (its sums and its cross term rescaled when the maximum grows). The cross term is
      // accumulated as w * (log2 difference) and converted to natural units once per lane.
      float es[2] = {0.f, 0.f}, et[2] = {0.f, 0.f}, cr[2] = {0.f, 0.f};
      float mt2 = -CUDART_INF_F;
      const float msl = Ms * kLog2e;
      for (int64_t j0 = c0 + (int64_t)lane * 8; j0 < c1; j0 += 256) {
        const float2 m = __ldg(tm + j0 / kVocabTile);
        float ds[8], t2[8];
        load8<WsT>(rs + j0, ds);
        const int cnt = c1 - j0 < 8 ? static_cast<int>(c1 - j0) : 8;
        load_tg8(p, row, j0, cnt, -CUDART_INF_F, t2);
        float m8 = -CUDART_INF_F;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          t2[j] *= kLog2e;
          m8 = fmaxf(m8, t2[j]);
        }
        if (m8 > mt2) {  // rescale this lane's teacher sums to the new running maximum
          const float fac = ex2_approx(mt2 - m8);  // 0 while nothing was accumulated
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            et[q] *= fac;
            if (!rev) cr[q] *= fac;
          }
          mt2 = m8;
        }
        const float offs = (m.x - Ms) * kLog2e;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (j >= cnt) break;
          const int q = j & 1;
          const float dL = ds[j] + offs;  // log2 of exp(z - Ms)
          const float e = ex2_approx(dL);
          const float t = ex2_approx(t2[j] - mt2);
          es[q] += e;
          et[q] += t;
          if (kl) {
            const float diff = t2[j] - (dL + msl);  // (u - z) log2 e
            cr[q] = rev ? fmaf(-e, diff, cr[q]) : fmaf(t, diff, cr[q]);
          }
        }
      }
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        s1s[q] = sts[q] = es[q];
        s1t[q] = stt[q] = et[q];
        cross[q] = kl ? cr[q] * kLn2 : 0.f;
      }
      mt = mt2 * kLn2;
    } else if constexpr (!TNO && TSRC != TS_GMEM) {
      // T = 1: the tempered sums equal the plain ones. The stored base-2 exponents only need the
      // per-tile offset added; the cross term is accumulated as w * (log2 difference) and converted
      // once per lane: u - z = (tL - dL) / log2 e + (mt - Ms).
      const bool want_t = teacher && (need_t1 || kl);
      float es[2] = {0.f, 0.f}, et[2] = {0.f, 0.f}, cr[2] = {0.f, 0.f};
      for (int64_t j0 = c0 + (int64_t)lane * 8; j0 < c1; j0 += 256) {
        const float2 m = __ldg(tm + j0 / kVocabTile);
        float ds[8], dt[8];
        load8<WsT>(rs + j0, ds);
        if (want_t) load8<WsT>(rt + j0, dt);
        const int cnt = c1 - j0 < 8 ? static_cast<int>(c1 - j0) : 8;
        const float offs = (m.x - Ms) * kLog2e, offt = (m.y - mt) * kLog2e;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int q = j & 1;
          const bool valid = j < cnt;
          const float dL = ds[j] + offs;
          const float e = valid ? ex2_approx(dL) : 0.f;
          es[q] += e;
          if (want_t) {
            const float tL = dt[j] + offt;
            const float t = valid ? ex2_approx(tL) : 0.f;
            et[q] += t;
            if (kl) cr[q] += rev ? e * (dL - tL) : t * (tL - dL);
          }
        }
      }
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        s1s[q] = sts[q] = es[q];
        s1t[q] = stt[q] = et[q];
        cross[q] = !(want_t && kl) ? 0.f : rev ? cr[q] * kLn2 + (Ms - mt) * es[q] : cr[q] * kLn2 + (mt - Ms) * et[q];
      }
    } else
    for (int64_t j0 = c0 + (int64_t)lane * 8; j0 < c1; j0 += 256) {
      const float2 m = __ldg(tm + j0 / kVocabTile);
      float ds[8], u[8];
      load8<WsT>(rs + j0, ds);
      const int cnt = c1 - j0 < 8 ? static_cast<int>(c1 - j0) : 8;
      if constexpr (TSRC == TS_GMEM) {
        load_tg8(p, row, j0, cnt, -CUDART_INF_F, u);
        float m8 = -CUDART_INF_F;
#pragma unroll
        for (int j = 0; j < 8; ++j) m8 = fmaxf(m8, u[j]);
        if (m8 > mt) {  // rescale the teacher sums to the new running maximum
          const float d = mt - m8;
          const float f1 = __expf(d), ft = TNO ? __expf(d * it) : f1;
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            s1t[q] *= f1;
            stt[q] *= ft;
            if (!rev) cross[q] *= ft;
          }
          mt = m8;
        }
      } else if constexpr (TSRC == TS_WS) {
        load8<WsT>(rt + j0, u);
#pragma unroll
        for (int j = 0; j < 8; ++j) u[j] = fmaf(u[j], kLn2, m.y);  // raw teacher logit
      }
      const float off_s = m.x - Ms;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int q = j & 1;
        const bool valid = j < cnt;
        const float d = fmaf(ds[j], kLn2, off_s);  // z - M_s
        const float e1 = valid ? __expf(d) : 0.f;
        const float et = TNO ? (valid ? __expf(d * it) : 0.f) : e1;
        s1s[q] += e1;
        sts[q] += et;
        if constexpr (teacher) {
          const float dt = u[j] - mt;
          float e1t = 0.f, ett = 0.f;
          if (valid) {
            if (!TNO) {
              e1t = __expf(dt);
              ett = e1t;
            } else {
              if (need_t1) e1t = __expf(dt);
              if (kl) ett = __expf(dt * it);
            }
          }
          s1t[q] += e1t;
          stt[q] += ett;
          if (kl && valid) {
            const float z = d + Ms;
            cross[q] += rev ? et * (z - u[j]) * it : ett * (u[j] - z) * it;
          }
        }
      }
    }
    const float cr = cross[0] + cross[1];
    Partial ps{Ms, warp_sum(s1s[0] + s1s[1]), warp_sum(sts[0] + sts[1]), rev ? (double)warp_sum(cr) : 0.0};
    Partial T{-CUDART_INF, 0.0, 0.0, 0.0};
    if constexpr (TSRC == TS_GMEM) {
      Partial pt{mt, s1t[0] + s1t[1], stt[0] + stt[1], rev ? 0.0 : (double)cr};
      if (pt.max_v == -CUDART_INF) pt.sum1 = pt.sumt = pt.cross = 0.0;
      T = warp_merge(pt, it, !rev);  // lane 0 holds the merge of the lanes' running maxima
    } else if constexpr (TSRC == TS_WS) {
      T = Partial{mt, warp_sum(s1t[0] + s1t[1]), warp_sum(stt[0] + stt[1]), rev ? 0.0 : (double)warp_sum(cr)};
    }
    if (lane == 0) {
      float* out = p.parts == 1 ? p.row_stats + row * kRowStats
                                : p.part_records + (static_cast<int64_t>(part) * p.rows + row) * kRowStats;
      bool ignored;
      const int64_t ys = safe_label(p.labels[row], p.ignore_index, p.vocab_total, &ignored);
      const bool has = !ignored && ys >= p.vocab_offset + c0 && ys < p.vocab_offset + c1;
      if ((f & F_VALIDATE) && part == 0) {  // validate labels (debug profile): flag, never trap
        const int64_t y = p.labels[row];
        if (y != p.ignore_index && (y < 0 || y >= p.vocab_total)) atomicCAS(p.status, 0, ORDA_ERR_LABEL_RANGE);
      }
      out[RS_MAX_S] = (float)ps.max_v;
      out[RS_SUM1_S] = (float)ps.sum1;
      out[RS_SUMT_S] = (float)ps.sumt;
      out[RS_MAX_T] = (float)T.max_v;
      out[RS_SUM1_T] = (float)T.sum1;
      out[RS_SUMT_T] = (float)T.sumt;
      out[RS_CROSS] = (float)(rev ? ps.cross : T.cross);
      out[RS_LABEL_S] = has ? p.label_logits[row * 2] : 0.f;
      out[RS_LABEL_T] = has ? p.label_logits[row * 2 + 1] : 0.f;
      out[RS_HAS_LABEL] = has ? 1.f : 0.f;
      out[10] = rev ? 0.f : 1.f;  // cross term follows the teacher maxima
      out[11] = p.inv_t;
      for (int k = 12; k < kRowStats; ++k) out[k] = 0.f;
    }
  }
}

// Epilogue-statistics path, one warp per row: the row record from the per-tile maxima and softmax
// sums the logits epilogue wrote (sum exp(z - M) = sum_tiles S_tile 2^((m_tile - M) log2 e), and at
// T != 1 the tempered sums with the offsets divided by T). Reads 16 to 24 bytes per (row, tile)
// instead of the row's logits. The divergence's row sums are left to the sweeps.
__global__ void __launch_bounds__(256) tile_merge_kernel(RowParams p) {
  const uint32_t f = p.flags;
  const bool teacher = f & F_TEACHER;
  const bool tempered = f & F_T_NOT_ONE;
  const float it = p.inv_t;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; row < p.rows; row += warps) {
    const float2* tm = row_tile_maxima(p, row);
    float ms = -CUDART_INF_F, mt = -CUDART_INF_F;
    for (int i = lane; i < p.n_vtiles; i += 32) {
      const float2 m = __ldg(tm + i);
      ms = fmaxf(ms, m.x);
      mt = fmaxf(mt, m.y);
    }
    ms = warp_max(ms);
    mt = teacher ? warp_max(mt) : -CUDART_INF_F;
    const float ms_l = ms * kLog2e, mt_l = mt * kLog2e;
    float ss = 0.f, st = 0.f, sst = 0.f, stt = 0.f;
    for (int i = lane; i < p.n_vtiles; i += 32) {
      const float2 m = __ldg(tm + i);
      const float ds = fmaf(m.x, kLog2e, -ms_l), dt = fmaf(m.y, kLog2e, -mt_l);  // tile offsets, base 2
      if (tempered) {
        const float4 e = __ldg(reinterpret_cast<const float4*>(p.tile_sums) + row * p.n_vtiles + i);
        ss = fmaf(e.x, ex2_approx(ds), ss);
        sst = fmaf(e.y, ex2_approx(ds * it), sst);
        if (teacher) {
          st = fmaf(e.z, ex2_approx(dt), st);
          stt = fmaf(e.w, ex2_approx(dt * it), stt);
        }
      } else {
        const float2 e = __ldg(reinterpret_cast<const float2*>(p.tile_sums) + row * p.n_vtiles + i);
        ss = fmaf(e.x, ex2_approx(ds), ss);
        if (teacher) st = fmaf(e.y, ex2_approx(dt), st);
      }
    }
    ss = warp_sum(ss);
    st = teacher ? warp_sum(st) : 0.f;
    if (tempered) {
      sst = warp_sum(sst);
      stt = teacher ? warp_sum(stt) : 0.f;
    } else {
      sst = ss;
      stt = st;
    }
    if (lane == 0) {
      float* out = p.row_stats + row * kRowStats;
      bool ignored;
      const int64_t ys = safe_label(p.labels[row], p.ignore_index, p.vocab_total, &ignored);
      const bool has = !ignored && ys >= p.vocab_offset && ys < p.vocab_offset + p.vocab;
      if (f & F_VALIDATE) {  // validate labels (debug profile): flag, never trap
        const int64_t y = p.labels[row];
        if (y != p.ignore_index && (y < 0 || y >= p.vocab_total)) atomicCAS(p.status, 0, ORDA_ERR_LABEL_RANGE);
      }
      out[RS_MAX_S] = ms;
      out[RS_SUM1_S] = ss;
      out[RS_SUMT_S] = sst;
      out[RS_MAX_T] = mt;
      out[RS_SUM1_T] = st;
      out[RS_SUMT_T] = stt;
      out[RS_CROSS] = 0.f;
      out[RS_LABEL_S] = has ? p.label_logits[row * 2] : 0.f;
      out[RS_LABEL_T] = has ? p.label_logits[row * 2 + 1] : 0.f;
      out[RS_HAS_LABEL] = has ? 1.f : 0.f;
      out[10] = 1.f;
      out[11] = p.inv_t;
      for (int k = 12; k < kRowStats; ++k) out[k] = 0.f;
    }
  }
}

// Smallest mixture probability the JSD terms take a logarithm of (keeps 0 * log 0 at 0 where both
// distributions underflow).
constexpr float kTinyProb = 1e-37f;

__device__ __forceinline__ float lg2_approx(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Epilogue-statistics path (and precomputed teacher logits at T = 1, JSD), reverse KL or JSD: the
// per-row divergence sums that the dlogits need before they can be formed, one warp per (row, column
// part), from the stored base-2 exponents and the merged row records, with the tempered
// distributions p = softmax(z / T) (log2 p = stored / T + per-tile constant):
//   reverse: R = sum_j p_s,j (log p_s,j - log p_t,j) (= the row's KL(p_s || p_t))
//   JSD:     J = sum_j [b p_t (log p_t - log m) + (1 - b) p_s (log p_s - log m)] and
//            G = sum_j p_s g_j, g = (1 - b)(log p_s - log m), m = b p_t + (1 - b) p_s
// Part k of row r goes to cross_parts[k * rows + r] (R or J) and, for JSD,
// cross_parts[(parts + k) * rows + r] (G).
template <typename WsT, int DK, bool GMEM = false>
__global__ void __launch_bounds__(256, 4) div_sweep_kernel(RowParams p) {
  const float beta = p.jsd_beta;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const int64_t tasks = p.rows * p.parts;
  for (int64_t task = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; task < tasks; task += warps) {
    const int64_t row = task / p.parts;
    const int part = static_cast<int>(task - row * p.parts);
    int64_t c0, c1;
    part_range(p, part, c0, c1);
    const float2* tm = row_tile_maxima(p, row);
    const RowConsts c = row_consts(p, row);
    float a0 = 0.f, a1 = 0.f;
    if (!c.ignored) {
      const WsT* rs = static_cast<const WsT*>(p.ws_s) + row * p.ld_ws;
      const WsT* rt = static_cast<const WsT*>(p.ws_t) + row * p.ld_ws;
      // tempered base-2 log-probabilities: log2 p^T = (z log2 e) / T - (M / T + log S_T) log2 e, with
      // z log2 e = stored exponent + tile maximum * log2 e (T = 1: the plain ones)
      const float it = p.inv_t, itl = it * kLog2e;
      const float base_s = -(c.ms * it + c.log_st) * kLog2e, base_t = -(c.mt * it + c.log_tt) * kLog2e;
      for (int64_t j0 = c0 + (int64_t)lane * 8; j0 < c1; j0 += 256) {
        const float2 m = __ldg(tm + j0 / kVocabTile);
        float ds[8], dt[8];
        load8<WsT>(rs + j0, ds);
        if constexpr (GMEM) {
          // the caller's teacher logits in base 2, against the row's constant
          load_tg8(p, row, j0, static_cast<int>(c1 - j0 < 8 ? c1 - j0 : 8), 0.f, dt);
#pragma unroll
          for (int j = 0; j < 8; ++j) dt[j] *= kLog2e;
        } else {
          load8<WsT>(rt + j0, dt);
        }
        const float cs = fmaf(m.x, itl, base_s);
        const float ct = GMEM ? base_t : fmaf(m.y, itl, base_t);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (j0 + j >= c1) break;
          const float lps = fmaf(ds[j], it, cs), lpt = fmaf(dt[j], it, ct);
          const float ps = ex2_approx(lps);
          if constexpr (DK == DK_REV) {
            a0 = fmaf(ps, lps - lpt, a0);
          } else {
            const float pt = ex2_approx(lpt);
            const float lm = lg2_approx(fmaxf(fmaf(beta, pt - ps, ps), kTinyProb));
            const float tps = ps * (lps - lm);
            a0 = fmaf(beta * pt, lpt - lm, fmaf(1.f - beta, tps, a0));
            a1 += tps;
          }
        }
      }
    }
    a0 = warp_sum(a0);
    if (DK == DK_JSD) a1 = warp_sum(a1);
    if (lane == 0) {
      p.cross_parts[static_cast<int64_t>(part) * p.rows + row] = a0 * kLn2;
      if (DK == DK_JSD) p.cross_parts[static_cast<int64_t>(p.parts + part) * p.rows + row] = a1 * (1.f - beta) * kLn2;
    }
  }
}

// JSD (0 < beta < 1), one warp per row: sum_j [b p_t (log p_t - log m) + (1-b) p_s (log p_s - log m)]
// and sum_j p_s g_j with g = (1-b)(log p_s - log m); this shard's partial sums -> row_sums[row][0..1].
template <typename WsT>
__global__ void __launch_bounds__(256, 4) jsd_sweep_kernel(RowParams p, float* row_sums) {
  const float beta = p.jsd_beta, it = p.inv_t;
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; row < p.rows; row += warps) {
    const float2* tm = row_tile_maxima(p, row);
    const RowConsts c = row_consts(p, row);
    float acc_j = 0.f, acc_g = 0.f;
    if (!c.ignored) {
      for (int64_t j0 = (int64_t)lane * 8; j0 < p.vocab; j0 += 256) {
        float ds[8], dt[8];
        load_row8<WsT>(p, row, j0, tm, c, true, ds, dt);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (j0 + j >= p.vocab) break;
          const float lps = ds[j] * it - c.log_st;
          const float lpt = dt[j] * it - c.log_tt;
          const float ps = __expf(lps), pt = __expf(lpt);
          const float lm = __logf(fmaxf(fmaf(beta, pt - ps, ps), kTinyProb));  // log m, m = b p_t + (1-b) p_s
          acc_j += beta * pt * (lpt - lm) + (1.f - beta) * ps * (lps - lm);
          acc_g += ps * (1.f - beta) * (lps - lm);
        }
      }
    }
    const float sj = warp_sum(acc_j), sg = warp_sum(acc_g);
    if (lane == 0) {
      row_sums[row * 2] = sj;
      row_sums[row * 2 + 1] = sg;
    }
  }
}

// dlogits in place, one warp per row. Student:
//   w_s (softmax(z) - onehot) + w_kl * T * G,  G = p_s^T - p_t^T           (forward KL)
//                                              G = p_s^T (a - R)             (reverse KL)
//                                              G = p_s^T (g - sum p_s g)     (JSD)
// Teacher (teacher CE only; the divergence never reaches the teacher): w_t (softmax(u) - onehot).
// Ignored rows are zeroed.
template <typename WsT, int TSRC, int DK, bool TNO>
__global__ void __launch_bounds__(256, 4) grad_sweep_kernel(RowParams p) {
  const uint32_t f = p.flags;
  constexpr bool kl = DK != DK_NONE;
  const bool grad_t = f & F_GRAD_T, grad_s = f & F_GRAD_S;
  const float it = p.inv_t, kls = p.w_kl * p.temperature;
  const float beta = p.jsd_beta;
  const bool need_t = TSRC != TS_NONE && (kl || grad_t);
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const int64_t tasks = p.rows * p.parts;
  for (int64_t task = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; task < tasks; task += warps) {
    const int64_t row = task / p.parts;
    const int part = static_cast<int>(task - row * p.parts);
    int64_t c0, c1;
    part_range(p, part, c0, c1);
    const float2* tm = row_tile_maxima(p, row);
    const RowConsts c = row_consts(p, row);
    float rrev = 0.f, gsum = 0.f;
    if (DK == DK_REV) {
      if (p.cross_parts) {  // epilogue-statistics path: R summed over the divergence sweep's parts
        for (int k = 0; k < p.parts; ++k) rrev += p.cross_parts[static_cast<int64_t>(k) * p.rows + row];
      } else {
        const float* r = p.row_stats + row * kRowStats;
        rrev = r[RS_CROSS] / r[RS_SUMT_S] - c.log_st - c.ms * it + c.log_tt + c.mt * it;
      }
    }
    if (DK == DK_JSD) {
      if (p.cross_parts) {
        for (int k = 0; k < p.parts; ++k) gsum += p.cross_parts[static_cast<int64_t>(p.parts + k) * p.rows + row];
      } else {
        gsum = p.row_sums[row * 2 + 1];
      }
    }
    const float gscale = p.grad_scale ? *p.grad_scale : 1.f;
    WsT* rs = static_cast<WsT*>(p.ws_s) + row * p.ld_ws;
    WsT* rt = static_cast<WsT*>(p.ws_t) + row * p.ld_ws;
    if constexpr (sizeof(WsT) == 2 && !TNO) {
      if (c.ignored) {
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
        for (int64_t j0 = c0 + (int64_t)lane * 8; j0 < c1; j0 += 256) {
          if (grad_s) *reinterpret_cast<uint4*>(rs + j0) = z;
          if (grad_t) *reinterpret_cast<uint4*>(rt + j0) = z;
        }
        continue;  // next task
      }
      // T = 1: log2 p = stored exponent + per-tile constant, p = 2^(log2 p): one add + one ex2 per
      // distribution. Forward KL (or none): dZ_s = (w_s + w_kl) p_s - w_kl p_t - w_s [label];
      // reverse KL: dZ_s = w_s (p_s - [label]) + w_kl p_s (ln2 (log2 p_s - log2 p_t) - R);
      // JSD: dZ_s = w_s (p_s - [label]) + w_kl p_s ((1 - b) ln2 (log2 p_s - log2 m) - G),
      // m = b p_t + (1 - b) p_s. dZ_t = w_t (p_t - [label]). All scaled by gscale.
      const float kl_w = kl ? kls : 0.f;
      const float as = gscale * (p.w_s + kl_w), bs = gscale * kl_w, at = gscale * p.w_t;
      const float ys = gscale * p.w_s;
      const float kd = gscale * kls;                 // divergence weight x T (T = 1), scaled
      const float g_ln2 = (1.f - beta) * kLn2;       // JSD: g = (1 - b) ln2 (log2 p_s - log2 m)
      const float base_s = -(c.ms + c.log_s1) * kLog2e, base_t = -(c.mt + c.log_t1) * kLog2e;
      // epilogue-statistics path: also sum_j p_t (u_j - z_j) for the forward-KL loss, with
      // u - z = (stored_t - stored_s) ln 2 + (tile max_t - tile max_s)
      const bool want_cross = DK == DK_FWD && p.cross_parts != nullptr;
      float cross = 0.f;
      for (int64_t j0 = c0 + (int64_t)lane * 8; j0 < c1; j0 += 256) {
        const float2 m = __ldg(tm + j0 / kVocabTile);
        float ds[8], dt[8];
        load8<WsT>(rs + j0, ds);
        if (need_t) {
          if constexpr (TSRC == TS_GMEM) {
            // the caller's teacher logits in base 2; their constant is the row's, not a tile's
            load_tg8(p, row, j0, static_cast<int>(p.vocab - j0 < 8 ? p.vocab - j0 : 8), 0.f, dt);
#pragma unroll
            for (int j = 0; j < 8; ++j) dt[j] *= kLog2e;
          } else {
            load8<WsT>(rt + j0, dt);
          }
        }
        const float cs = fmaf(m.x, kLog2e, base_s);
        const float ct = TSRC == TS_GMEM ? base_t : fmaf(m.y, kLog2e, base_t);
        const float dm = m.y - m.x;
        float gs[8], gt[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float lps = ds[j] + cs, lpt = dt[j] + ct;  // base-2 log-probabilities
          const float ps = ex2_approx(lps);
          const float pt = need_t ? ex2_approx(lpt) : 0.f;
          if constexpr (DK == DK_REV) {
            gs[j] = fmaf(ys, ps, kd * ps * fmaf(lps - lpt, kLn2, -rrev));
          } else if constexpr (DK == DK_JSD) {
            const float lm = lg2_approx(fmaxf(fmaf(beta, pt - ps, ps), kTinyProb));
            gs[j] = fmaf(ys, ps, kd * ps * fmaf(lps - lm, g_ln2, -gsum));
          } else {
            gs[j] = fmaf(as, ps, -bs * pt);
          }
          gt[j] = at * pt;
          if (want_cross && j0 + j < c1) cross = fmaf(pt, fmaf(dt[j] - ds[j], kLn2, dm), cross);
        }
        const int64_t lc = c.label_local - j0;  // label column inside this vector of 8
        if (lc >= 0 && lc < 8) {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (j == lc) {
              gs[j] -= ys;
              gt[j] -= at;
            }
        }
        if (grad_s) {
          uint4 u;
          u.x = pack2<WsT>(gs[0], gs[1]); u.y = pack2<WsT>(gs[2], gs[3]);
          u.z = pack2<WsT>(gs[4], gs[5]); u.w = pack2<WsT>(gs[6], gs[7]);
          *reinterpret_cast<uint4*>(rs + j0) = u;
        }
        if (grad_t) {
          uint4 u;
          u.x = pack2<WsT>(gt[0], gt[1]); u.y = pack2<WsT>(gt[2], gt[3]);
          u.z = pack2<WsT>(gt[4], gt[5]); u.w = pack2<WsT>(gt[6], gt[7]);
          *reinterpret_cast<uint4*>(rt + j0) = u;
        }
      }
      if (want_cross) {
        cross = warp_sum(cross);
        if (lane == 0) p.cross_parts[static_cast<int64_t>(part) * p.rows + row] = cross;
      }
    } else {
    // epilogue-statistics path at T != 1, forward KL: this part's sum_j p_t (log p_t - log p_s) of
    // the tempered distributions, for the row loss
    const bool want_kl = DK == DK_FWD && p.cross_parts != nullptr;
    float klsum = 0.f;
    for (int64_t j0 = c0 + (int64_t)lane * 8; j0 < c1; j0 += 256) {
      float gs[8], gt[8];
      if (c.ignored) {
#pragma unroll
        for (int j = 0; j < 8; ++j) gs[j] = gt[j] = 0.f;
      } else {
        float ds[8], dt[8];
        load_row8<WsT>(p, row, j0, tm, c, need_t, ds, dt);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float onehot = (j0 + j == c.label_local) ? 1.f : 0.f;
          const float ps1 = __expf(ds[j] - c.log_s1);
          float g = p.w_s * (ps1 - onehot);
          // at T = 1 the tempered distributions are the CE softmaxes: reuse the exponentials
          float pt1 = 0.f;
          bool have_pt1 = false;
          if constexpr (kl) {
            const float lps = ds[j] * it - c.log_st;
            const float lpt = dt[j] * it - c.log_tt;
            const float ps = TNO ? __expf(lps) : ps1;
            float d;
            if constexpr (DK == DK_JSD) {
              const float pt = __expf(lpt);
              const float lm = __logf(fmaxf(fmaf(beta, pt - ps, ps), kTinyProb));
              d = ps * ((1.f - beta) * (lps - lm) - gsum);
            } else if constexpr (DK == DK_REV) {
              d = ps * ((lps - lpt) - rrev);
            } else {
              const float pt = __expf(lpt);
              if (!TNO) {
                pt1 = pt;
                have_pt1 = true;
              }
              d = ps - pt;
              if (want_kl && j0 + j < c1) klsum = fmaf(pt, lpt - lps, klsum);
            }
            g += kls * d;
          }
          gs[j] = g * gscale;
          if (TSRC != TS_NONE && grad_t) {
            if (!have_pt1) pt1 = __expf(dt[j] - c.log_t1);
            gt[j] = p.w_t * (pt1 - onehot) * gscale;
          } else {
            gt[j] = 0.f;
          }
        }
      }
      if (grad_s) store8<WsT>(rs + j0, gs);
      if (grad_t) store8<WsT>(rt + j0, gt);
    }
    if (want_kl) {
      klsum = warp_sum(klsum);
      if (lane == 0) p.cross_parts[static_cast<int64_t>(part) * p.rows + row] = klsum;
    }
    }
  }
}

// Launch helpers selecting the compile-time specialisation from the runtime flags.
template <typename WsT, int TSRC>
void launch_row_stats_t(const RowParams& r, int grid, cudaStream_t s) {
  if (r.flags & F_T_NOT_ONE) row_stats_kernel<WsT, TSRC, true><<<grid, 256, 0, s>>>(r);
  else row_stats_kernel<WsT, TSRC, false><<<grid, 256, 0, s>>>(r);
}

template <typename WsT>
void launch_row_stats(const RowParams& r, int grid, cudaStream_t s) {
  if (!(r.flags & F_TEACHER)) launch_row_stats_t<WsT, TS_NONE>(r, grid, s);
  else if (r.flags & F_TEACHER_GMEM) launch_row_stats_t<WsT, TS_GMEM>(r, grid, s);
  else launch_row_stats_t<WsT, TS_WS>(r, grid, s);
}

template <typename WsT, int TSRC, int DK>
void launch_grad_sweep_dk(const RowParams& r, int grid, cudaStream_t s) {
  if (r.flags & F_T_NOT_ONE) grad_sweep_kernel<WsT, TSRC, DK, true><<<grid, 256, 0, s>>>(r);
  else grad_sweep_kernel<WsT, TSRC, DK, false><<<grid, 256, 0, s>>>(r);
}

template <typename WsT, int TSRC>
void launch_grad_sweep_t(const RowParams& r, int grid, cudaStream_t s) {
  if (!(r.flags & F_KL)) launch_grad_sweep_dk<WsT, TSRC, DK_NONE>(r, grid, s);
  else if (r.flags & F_JSD) launch_grad_sweep_dk<WsT, TSRC, DK_JSD>(r, grid, s);
  else if (r.flags & F_KL_REVERSE) launch_grad_sweep_dk<WsT, TSRC, DK_REV>(r, grid, s);
  else launch_grad_sweep_dk<WsT, TSRC, DK_FWD>(r, grid, s);
}

template <typename WsT>
void launch_grad_sweep(const RowParams& r, int grid, cudaStream_t s) {
  if (!(r.flags & F_TEACHER)) launch_grad_sweep_t<WsT, TS_NONE>(r, grid, s);
  else if (r.flags & F_TEACHER_GMEM) launch_grad_sweep_t<WsT, TS_GMEM>(r, grid, s);
  else launch_grad_sweep_t<WsT, TS_WS>(r, grid, s);
}

// Single block: reduce per-row losses (double) into the reference's scalars
// (tied_teacher.py:500-516): sums, count of non-ignored labels, mean scale, weighted loss.
__global__ void finalize_kernel(const float* row_losses, int64_t ld, const int64_t* labels, int64_t n,
                                int64_t ignore_index, int32_t reduction, uint32_t flags, float w_s, float w_t,
                                float w_kl, float* out) {
  __shared__ double red[4][32];
  double a = 0, b = 0, c = 0, cnt = 0;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
    a += row_losses[i];
    b += row_losses[ld + i];
    c += row_losses[2 * ld + i];
    cnt += (labels[i] != ignore_index) ? 1.0 : 0.0;
  }
  double v[4] = {a, b, c, cnt};
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    for (int off = 16; off > 0; off >>= 1) v[k] += __shfl_down_sync(0xffffffffu, v[k], off);
    if (l == 0) red[k][w] = v[k];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double s[4] = {0, 0, 0, 0};
    for (int k = 0; k < 4; ++k)
      for (int i = 0; i < (int)(blockDim.x / 32); ++i) s[k] += red[k][i];
    const double denom = s[3] > 1.0 ? s[3] : 1.0;
    const double scale = reduction == ORDA_REDUCTION_MEAN ? 1.0 / denom : 1.0;
    // component values are rounded to fp32 first, as the reference combines fp32 scalars (:516)
    const float ce_s = (float)(s[0] * scale);
    const float ce_t = (flags & F_TEACHER_CE) ? (float)(s[1] * scale) : 0.f;
    const float kl = (flags & F_KL) ? (float)(s[2] * scale) : 0.f;
    out[ORDA_OUT_LOSS] = ce_s * w_s + ce_t * w_t + w_kl * kl;
    out[ORDA_OUT_STUDENT_CE] = ce_s;
    out[ORDA_OUT_TEACHER_CE] = ce_t;
    out[ORDA_OUT_KL] = kl;
    out[ORDA_OUT_MEAN_SCALE] = (float)scale;
    out[ORDA_OUT_SUM_STUDENT_CE] = (float)s[0];
    out[ORDA_OUT_SUM_TEACHER_CE] = (float)s[1];
    out[ORDA_OUT_SUM_KL] = (float)s[2];
    out[ORDA_OUT_COUNT] = (float)s[3];
  }
}

// out[ORDA_OUT_MEAN_SCALE] before any gradient is formed: 1/max(count of non-ignored labels, 1) for
// mean reduction, 1 for sum (tied_teacher.py:503-513). Single block.
__global__ void mean_scale_kernel(const int64_t* labels, int64_t n, int64_t ignore_index, int32_t reduction,
                                  float* out) {
  __shared__ int64_t red[32];
  int64_t c = 0;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) c += labels[i] != ignore_index;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) c += __shfl_down_sync(0xffffffffu, c, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t t = 0;
    for (int i = 0; i < (int)(blockDim.x / 32); ++i) t += red[i];
    out[ORDA_OUT_MEAN_SCALE] = reduction == ORDA_REDUCTION_MEAN ? 1.f / (float)(t > 1 ? t : 1) : 1.f;
  }
}

// out[r][c] = sum_k part[k][r][c] over the `splits` fp32 k-split partials of a GEMM (each rows x n
// contiguous, `stride` elements apart), added in order k = 0, 1, ... and rounded once to the 16-bit
// output type; n is a multiple of 8.
template <typename T>
__global__ void sum_split_kernel(const float* part, int splits, int64_t stride, T* out, int64_t count8) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count8; i += (int64_t)gridDim.x * blockDim.x) {
    float4 a0 = reinterpret_cast<const float4*>(part)[2 * i], a1 = reinterpret_cast<const float4*>(part)[2 * i + 1];
    for (int k = 1; k < splits; ++k) {
      const float4* q = reinterpret_cast<const float4*>(part + k * stride);
      const float4 b0 = q[2 * i], b1 = q[2 * i + 1];
      a0.x += b0.x; a0.y += b0.y; a0.z += b0.z; a0.w += b0.w;
      a1.x += b1.x; a1.y += b1.y; a1.z += b1.z; a1.w += b1.w;
    }
    uint4 u;
    u.x = pack2<T>(a0.x, a0.y);
    u.y = pack2<T>(a0.z, a0.w);
    u.z = pack2<T>(a1.x, a1.y);
    u.w = pack2<T>(a1.z, a1.w);
    reinterpret_cast<uint4*>(out)[i] = u;
  }
}

// Owner side of the peer-memory gradient exchange: rows [row0, row0 + rows) of the summed gradient
// are the sum over the `world` slots of this GPU's slot buffer ([world][slab_rows][hidden], slot k
// written by rank k), accumulated in fp32 and rounded once, then stored into every rank's gradient
// buffer (dst[k], peer addresses mapped here; dst[rank] is local). 16-byte vectors, grid-stride.
struct PeerReduceParams {
  int32_t world;
  int64_t rows, row0, slab_rows, hidden;
  const void* slots;
  void* dst[ORDA_MAX_PEERS];
};

template <typename T>
__global__ void __launch_bounds__(256) peer_reduce_broadcast_kernel(const __grid_constant__ PeerReduceParams q) {
  const int64_t per_row = q.hidden / 8;
  const int64_t n = q.rows * per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / per_row, c8 = i - r * per_row;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < q.world; ++k) {
      float v[8];
      load8<T>(static_cast<const T*>(q.slots) + ((int64_t)k * q.slab_rows + r) * q.hidden + c8 * 8, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += v[j];
    }
    uint4 u;
    u.x = pack2<T>(acc[0], acc[1]); u.y = pack2<T>(acc[2], acc[3]);
    u.z = pack2<T>(acc[4], acc[5]); u.w = pack2<T>(acc[6], acc[7]);
    const int64_t off = (q.row0 + r) * q.hidden + c8 * 8;
    for (int k = 0; k < q.world; ++k) *reinterpret_cast<uint4*>(static_cast<T*>(q.dst[k]) + off) = u;
  }
  // the broadcast stores are visible system-wide once this kernel has finished
  __threadfence_system();
}

// data *= *scale in place; every block returns at once when *scale == 1 (no memory traffic).
template <typename T>
__global__ void scale_grad_kernel(T* data, int64_t n, const float* scale) {
  const float s = *scale;
  if (s == 1.f) return;
  const int64_t n8 = n / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    float v[8];
    load8<T>(data + 8 * i, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] *= s;
    store8<T>(data + 8 * i, v);
  }
  for (int64_t i = 8 * n8 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    data[i] = Conv<T>::from_f(Conv<T>::to_f(data[i]) * s);
}

}  // namespace orda
