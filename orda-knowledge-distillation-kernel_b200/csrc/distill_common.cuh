// Shared definitions of the fused distillation kernels: element conversions, the per-(row, vocab
// tile) statistics record written by the logits-GEMM epilogue, and the per-row record merged from it.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math_constants.h>
#include <stdint.h>

namespace orda {

constexpr int kTileRows = 128;   // rows of one GEMM tile (TMEM lanes)

// The chunk workspace holds every logit as a base-2 exponent relative to its 128-column tile
// maximum, y = (z - m_tile) * log2(e), in the compute dtype. exp(z - m) is then 2^y: one ex2 per
// element with no scaling multiply, and the bf16 rounding of y has the same relative precision as
// rounding z - m would have.
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// 2^x with the PTX ex2.approx instruction. Callers evaluate exp(x) through the identity
// exp(x) = 2^(x * log2 e), folding the log2 e factor into the arguments they already scale.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr int kVocabTile = 128;  // vocab columns covered by one statistics record
constexpr int kTileStats = 2;    // floats per (row, vocab tile) record
constexpr int kRowStats = 16;    // floats per merged row record (== ORDA_ROW_STATS)

// Tile record fields (one per row and 128-column vocab tile): the maxima the workspace logits are
// shifted by.
enum TileStat {
  TS_MAX_S = 0,   // max_j z_j of the tile (student)
  TS_MAX_T = 1,   // max_j u_j of the tile (teacher)
};

// Merged row record fields (the unit exchanged between vocab shards):
enum RowStat {
  RS_MAX_S = 0, RS_SUM1_S = 1, RS_SUMT_S = 2,
  RS_MAX_T = 3, RS_SUM1_T = 4, RS_SUMT_T = 5,
  RS_CROSS = 6,        // divergence cross term, relative to the row maxima
  RS_LABEL_S = 7,      // student logit at the label (valid when RS_HAS_LABEL == 1)
  RS_LABEL_T = 8,      // teacher logit at the label
  RS_HAS_LABEL = 9,    // 1 if this shard (or the merge) holds the label column
  RS_COUNT = 16
};

// Epilogue / row-kernel feature flags (runtime, warp-uniform).
enum DistillFlags : uint32_t {
  F_TEACHER = 1u << 0,          // teacher logits exist (KL or teacher CE)
  F_TEACHER_GMEM = 1u << 1,     // teacher logits are read from caller memory (precomputed logits)
  F_TEACHER_CE = 1u << 2,       // teacher CE term (teacher_ce_weight != 0)
  F_KL = 1u << 3,               // divergence term (kl_weight != 0)
  F_T_NOT_ONE = 1u << 4,        // temperature != 1
  F_KL_REVERSE = 1u << 5,       // cross term of the reverse KL instead of the forward KL
  F_WRITE_WS_S = 1u << 6,       // keep shifted student logits in the workspace
  F_WRITE_WS_T = 1u << 7,       // keep shifted teacher logits in the workspace
  F_JSD = 1u << 8,              // generalised JSD (needs an extra row sweep)
  F_GRAD_S = 1u << 9,           // student dlogits needed
  F_GRAD_T = 1u << 10,          // teacher dlogits needed (teacher CE gradients)
  F_VALIDATE = 1u << 31,        // flag labels outside [0, V) that are not ignore_index
};

template <typename T> struct Conv;
template <> struct Conv<float> {
  static __device__ __forceinline__ float to_f(float x) { return x; }
  static __device__ __forceinline__ float from_f(float x) { return x; }
};
template <> struct Conv<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Conv<__half> {
  static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};

// Two floats rounded to the 16-bit type in one conversion, low half = a (memory order a, b).
// The two 16-bit values of a packed word as floats (low half first, as pack2 stores them).
template <typename T> __device__ __forceinline__ void unpack2(uint32_t w, float& a, float& b);
template <> __device__ __forceinline__ void unpack2<__nv_bfloat16>(uint32_t w, float& a, float& b) {
  a = __uint_as_float(w << 16);
  b = __uint_as_float(w & 0xffff0000u);
}
template <> __device__ __forceinline__ void unpack2<__half>(uint32_t w, float& a, float& b) {
  const __half2 h = *reinterpret_cast<const __half2*>(&w);
  const float2 f = __half22float2(h);
  a = f.x;
  b = f.y;
}

template <typename T> __device__ __forceinline__ uint32_t pack2(float a, float b);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  const __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&v);
}

__device__ __forceinline__ float fast_exp(float x) { return __expf(x); }

// Label semantics of the reference row kernels (ops/tied_teacher.py:42-44): ignore_index rows are
// skipped; any other label outside [0, vocab_total) is read as label 0.
__device__ __forceinline__ int64_t safe_label(int64_t y, int64_t ignore_index, int64_t vocab_total, bool* ignored) {
  *ignored = (y == ignore_index);
  if (*ignored) return -1;
  return (y >= 0 && y < vocab_total) ? y : 0;
}

// Merge two (max, sum1, sumT, cross) partials of one distribution into the first.
// `a_max == -inf` marks an empty partial.
struct Partial {
  double max_v, sum1, sumt, cross;
};

__device__ __forceinline__ void merge_partial(Partial& a, const Partial& b, double inv_t, bool cross_follows) {
  if (b.max_v == -CUDART_INF) return;
  if (a.max_v == -CUDART_INF) { a = b; return; }
  const double m = a.max_v > b.max_v ? a.max_v : b.max_v;
  const double fa = exp(a.max_v - m), fb = exp(b.max_v - m);
  const double fat = exp((a.max_v - m) * inv_t), fbt = exp((b.max_v - m) * inv_t);
  a.sum1 = a.sum1 * fa + b.sum1 * fb;
  a.sumt = a.sumt * fat + b.sumt * fbt;
  if (cross_follows) a.cross = a.cross * fat + b.cross * fbt;
  a.max_v = m;
}

}  // namespace orda
