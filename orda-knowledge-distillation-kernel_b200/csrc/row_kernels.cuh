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
  int32_t* status;
};

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

// One warp per row.
__global__ void row_merge_kernel(RowParams p) {
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const int lane = threadIdx.x & 31;
  const bool teacher = p.flags & F_TEACHER;
  const bool rev = p.flags & F_KL_REVERSE;
  const double inv_t = p.inv_t;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; row < p.rows; row += warps) {
    Partial s{-CUDART_INF, 0.0, 0.0, 0.0}, t{-CUDART_INF, 0.0, 0.0, 0.0};
    const float* rec = p.tile_stats + row * p.n_vtiles * kTileStats;
    for (int tile = lane; tile < p.n_vtiles; tile += 32) {
      const float4 a = reinterpret_cast<const float4*>(rec + tile * kTileStats)[0];
      const float4 b = reinterpret_cast<const float4*>(rec + tile * kTileStats)[1];
      Partial ps{a.x, a.y, a.z, rev ? (double)b.z : 0.0};
      merge_partial(s, ps, inv_t, rev);
      if (teacher) {
        Partial pt{a.w, b.x, b.y, rev ? 0.0 : (double)b.z};
        merge_partial(t, pt, inv_t, !rev);
      }
    }
    s = warp_merge(s, inv_t, rev);
    if (teacher) t = warp_merge(t, inv_t, !rev);
    if (lane == 0) {
      float* out = p.row_stats + row * kRowStats;
      bool ignored;
      const int64_t ys = safe_label(p.labels[row], p.ignore_index, p.vocab_total, &ignored);
      const bool has = !ignored && ys >= p.vocab_offset && ys < p.vocab_offset + p.vocab;
      if (p.flags & F_VALIDATE) {  // validate labels (debug profile): flag, never trap
        const int64_t y = p.labels[row];
        if (y != p.ignore_index && (y < 0 || y >= p.vocab_total)) atomicCAS(p.status, 0, ORDA_ERR_LABEL_RANGE);
      }
      out[RS_MAX_S] = (float)s.max_v;
      out[RS_SUM1_S] = (float)s.sum1;
      out[RS_SUMT_S] = (float)s.sumt;
      out[RS_MAX_T] = (float)t.max_v;
      out[RS_SUM1_T] = (float)t.sum1;
      out[RS_SUMT_T] = (float)t.sumt;
      out[RS_CROSS] = (float)(rev ? s.cross : t.cross);
      out[RS_LABEL_S] = has ? p.label_logits[row * 2] : 0.f;
      out[RS_LABEL_T] = has ? p.label_logits[row * 2 + 1] : 0.f;
      out[RS_HAS_LABEL] = has ? 1.f : 0.f;
      out[10] = rev ? 0.f : 1.f;  // cross term follows the teacher maxima
      out[11] = p.inv_t;
      for (int k = 12; k < kRowStats; ++k) out[k] = 0.f;
    }
  }
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

// One thread per row: per-row losses from the (global) row record.
__global__ void row_loss_kernel(RowParams p) {
  for (int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; row < p.rows; row += (int64_t)gridDim.x * blockDim.x) {
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
        if (p.flags & F_JSD) {
          div = p.row_sums[row * 2] * t * t;
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

// Loads 8 consecutive (student, teacher) values as offsets from the ROW maxima:
//   ds = z - max_s ; dt = u - max_t
template <typename WsT>
__device__ __forceinline__ void load_row8(const RowParams& p, int64_t row, int64_t j0, const float* smax_s,
                                          const float* smax_t, const RowConsts& c, bool need_t, float (&ds)[8],
                                          float (&dt)[8]) {
  const int tile = static_cast<int>(j0 / kVocabTile);
  load8<WsT>(static_cast<const WsT*>(p.ws_s) + row * p.ld_ws + j0, ds);
  const float off_s = smax_s[tile] - c.ms;
#pragma unroll
  for (int j = 0; j < 8; ++j) ds[j] += off_s;
  if (need_t) {
    if (p.flags & F_TEACHER_GMEM) {
#pragma unroll
      for (int j = 0; j < 8; ++j) dt[j] = (j0 + j < p.vocab) ? load_tg(p, row, j0 + j) - c.mt : 0.f;
    } else {
      load8<WsT>(static_cast<const WsT*>(p.ws_t) + row * p.ld_ws + j0, dt);
      const float off_t = smax_t[tile] - c.mt;
#pragma unroll
      for (int j = 0; j < 8; ++j) dt[j] += off_t;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) dt[j] = 0.f;
  }
}

__device__ __forceinline__ void load_tile_maxima(const RowParams& p, int64_t row, float* smax_s, float* smax_t) {
  const float* rec = p.tile_stats + row * p.n_vtiles * kTileStats;
  for (int i = threadIdx.x; i < p.n_vtiles; i += blockDim.x) {
    smax_s[i] = rec[i * kTileStats + TS_MAX_S];
    smax_t[i] = rec[i * kTileStats + TS_MAX_T];
  }
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_down_sync(0xffffffffu, v, off);
  const int w = threadIdx.x / 32, l = threadIdx.x % 32;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  if (threadIdx.x < 32) {
    s = (l < (int)(blockDim.x / 32)) ? red[l] : 0.f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_down_sync(0xffffffffu, s, off);
  }
  return s;  // valid in thread 0
}

// log(exp(a) + exp(b)), stable.
__device__ __forceinline__ float log_add_exp(float a, float b) {
  const float m = fmaxf(a, b);
  if (m == -CUDART_INF_F) return m;
  return m + log1pf(__expf(-fabsf(a - b)));
}

// JSD (0 < beta < 1): per row, sum_j [b p_t (log p_t - log m) + (1-b) p_s (log p_s - log m)] and
// sum_j p_s g_j with g = (1-b)(log p_s - log m); this shard's partial sums -> row_sums[row][0..1].
template <typename WsT>
__global__ void jsd_sweep_kernel(RowParams p, float* row_sums) {
  extern __shared__ float sh[];
  float* smax_s = sh;
  float* smax_t = sh + p.n_vtiles;
  float* red = sh + 2 * p.n_vtiles;
  const float beta = p.jsd_beta, lb = logf(beta), l1b = log1pf(-beta), it = p.inv_t;
  for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
    __syncthreads();
    load_tile_maxima(p, row, smax_s, smax_t);
    __syncthreads();
    const RowConsts c = row_consts(p, row);
    float acc_j = 0.f, acc_g = 0.f;
    if (!c.ignored) {
      for (int64_t j0 = (int64_t)threadIdx.x * 8; j0 < p.vocab; j0 += (int64_t)blockDim.x * 8) {
        float ds[8], dt[8];
        load_row8<WsT>(p, row, j0, smax_s, smax_t, c, true, ds, dt);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (j0 + j >= p.vocab) break;
          const float lps = ds[j] * it - c.log_st;
          const float lpt = dt[j] * it - c.log_tt;
          const float ps = __expf(lps), pt = __expf(lpt);
          const float lm = log_add_exp(lb + lpt, l1b + lps);
          acc_j += beta * pt * (lpt - lm) + (1.f - beta) * ps * (lps - lm);
          acc_g += ps * (1.f - beta) * (lps - lm);
        }
      }
    }
    const float sj = block_sum(acc_j, red);
    const float sg = block_sum(acc_g, red);
    if (threadIdx.x == 0) {
      row_sums[row * 2] = sj;
      row_sums[row * 2 + 1] = sg;
    }
  }
}

// dlogits in place. Student:
//   w_s (softmax(z) - onehot) + w_kl * T * G,  G = p_s^T - p_t^T           (forward KL)
//                                              G = p_s^T (a - R)             (reverse KL)
//                                              G = p_s^T (g - sum p_s g)     (JSD)
// Teacher (teacher CE only; the divergence never reaches the teacher): w_t (softmax(u) - onehot).
// Ignored rows are zeroed.
template <typename WsT>
__global__ void grad_sweep_kernel(RowParams p) {
  extern __shared__ float sh[];
  float* smax_s = sh;
  float* smax_t = sh + p.n_vtiles;
  const uint32_t f = p.flags;
  const bool kl = f & F_KL, grad_t = f & F_GRAD_T, grad_s = f & F_GRAD_S;
  const bool rev = f & F_KL_REVERSE, jsd = f & F_JSD;
  const float it = p.inv_t, kls = p.w_kl * p.temperature;
  const float beta = p.jsd_beta, lb = logf(fmaxf(beta, 1e-30f)), l1b = log1pf(-fminf(beta, 0.999999f));
  for (int64_t row = blockIdx.x; row < p.rows; row += gridDim.x) {
    __syncthreads();
    load_tile_maxima(p, row, smax_s, smax_t);
    __syncthreads();
    const RowConsts c = row_consts(p, row);
    float rrev = 0.f, gsum = 0.f;
    if (kl && rev) {
      const float* r = p.row_stats + row * kRowStats;
      rrev = r[RS_CROSS] / r[RS_SUMT_S] - c.log_st - c.ms * it + c.log_tt + c.mt * it;
    }
    if (kl && jsd) gsum = p.row_sums[row * 2 + 1];
    WsT* rs = static_cast<WsT*>(p.ws_s) + row * p.ld_ws;
    WsT* rt = static_cast<WsT*>(p.ws_t) + row * p.ld_ws;
    for (int64_t j0 = (int64_t)threadIdx.x * 8; j0 < p.vocab; j0 += (int64_t)blockDim.x * 8) {
      float gs[8], gt[8];
      if (c.ignored) {
#pragma unroll
        for (int j = 0; j < 8; ++j) gs[j] = gt[j] = 0.f;
      } else {
        float ds[8], dt[8];
        load_row8<WsT>(p, row, j0, smax_s, smax_t, c, kl || grad_t, ds, dt);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float onehot = (j0 + j == c.label_local) ? 1.f : 0.f;
          const float ps1 = __expf(ds[j] - c.log_s1);
          float g = p.w_s * (ps1 - onehot);
          if (kl) {
            const float lps = ds[j] * it - c.log_st;
            const float lpt = dt[j] * it - c.log_tt;
            const float ps = __expf(lps);
            float d;
            if (jsd) {
              const float lm = log_add_exp(lb + lpt, l1b + lps);
              d = ps * ((1.f - beta) * (lps - lm) - gsum);
            } else if (rev) {
              d = ps * ((lps - lpt) - rrev);
            } else {
              d = ps - __expf(lpt);
            }
            g += kls * d;
          }
          gs[j] = g;
          gt[j] = grad_t ? p.w_t * (__expf(dt[j] - c.log_t1) - onehot) : 0.f;
        }
      }
      if (grad_s) store8<WsT>(rs + j0, gs);
      if (grad_t) store8<WsT>(rt + j0, gt);
    }
  }
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

}  // namespace orda
