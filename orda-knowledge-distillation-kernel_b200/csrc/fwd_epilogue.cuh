// Fused statistics epilogue of the logits GEMM.
//
// One thread owns one logits row of a 128-row x 128-column tile (student accumulator, and the
// teacher accumulator or the caller's teacher logits). It computes, without ever writing the
// un-shifted logits to memory:
//   - the tile maxima (student and teacher),
//   - the label logit (exact fp32 accumulator value),
// and stores the logits shifted by the tile maximum, as base-2 exponents, into the bounded chunk
// workspace in the compute dtype (values near the row maximum, which dominate softmax, keep full relative precision).
//
// Together with row_stats_kernel this is the statistics half of the reference row kernels
// (ops/tied_teacher.py:54-141, ops/separate_teacher.py, ops/precomputed_teacher.py:53-101).
#pragma once

#include "distill_common.cuh"
#include "orda_b200.h"

namespace orda {

struct FwdEpiParams {
  int64_t rows;          // valid rows of this chunk
  int64_t vocab;         // valid vocab columns (this shard)
  int64_t vocab_offset;  // global id of column 0
  int64_t vocab_total;
  int64_t ignore_index;
  int32_t n_vtiles;      // vocab tiles per row (tile_stats stride)
  uint32_t flags;
  float inv_t;
  const int64_t* labels;          // chunk labels
  void* ws_s;                     // shifted student logits [rows, ld_ws]
  void* ws_t;                     // shifted teacher logits
  int64_t ld_ws;
  const void* t_gmem;             // caller's teacher logits (F_TEACHER_GMEM)
  int64_t ld_tg;
  int32_t tg_dtype;
  float* tile_stats;              // [rows][n_vtiles][kTileStats]
  float* label_logits;            // [rows][2]
  // Optional: per (row, vocab tile) sum of 2^y over the tile's stored base-2 exponents y, i.e.
  // sum exp(z - m_tile), as [rows][n_vtiles] float2 {student, teacher}; at T != 1 (F_T_NOT_ONE) also
  // the tempered sum exp((z - m_tile) / T), as float4 {student, student tempered, teacher, teacher
  // tempered}. The wide GEMM's epilogue forms it after releasing the accumulator, from the tile it
  // has just stored.
  float* tile_sums;
  int32_t plain_teacher;          // wide kernel, A_PLAIN: the accumulators hold teacher logits
};

template <typename WsT>
__device__ __forceinline__ void store_chunk32(WsT* dst, const float (&v)[32]) {
  if constexpr (sizeof(WsT) == 2) {
    uint32_t w[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      WsT lo = Conv<WsT>::from_f(v[2 * j]), hi = Conv<WsT>::from_f(v[2 * j + 1]);
      w[j] = static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&lo)) |
             (static_cast<uint32_t>(*reinterpret_cast<uint16_t*>(&hi)) << 16);
    }
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int j = 0; j < 4; ++j) d[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
  } else {
    float4* d = reinterpret_cast<float4*>(dst);
#pragma unroll
    for (int j = 0; j < 8; ++j) d[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
}

// `src.load(acc, chunk, v)` yields 32 fp32 logits of accumulator `acc` (0 student, 1 teacher) for
// columns [32*chunk, 32*chunk+32) of the tile. For TMEM sources the call is warp-collective, so
// every lane calls it the same number of times whatever its row.
//
// Per (row, 128-column vocab tile) the epilogue produces only what needs the fp32 accumulator:
// the tile maximum of each distribution, the logits shifted by that maximum in the compute dtype,
// and the exact label logit. The exponentials (softmax sums, divergence cross terms) are computed
// by the memory-bound row pass that streams the workspace anyway, which keeps the transcendental
// pipe out of the GEMM's critical path.
template <typename WsT, bool kTeacherAcc, class Src>
__device__ __forceinline__ void fwd_tile_stats(const FwdEpiParams& p, int64_t row, bool row_ok, int64_t n0,
                                               int tile, Src& src) {
  constexpr int kChunks = kVocabTile / 32;
  const uint32_t f = p.flags;
  const bool teacher = kTeacherAcc && (f & F_TEACHER) != 0;
  const int nvalid = static_cast<int>((p.vocab - n0 < (int64_t)kVocabTile ? p.vocab - n0 : (int64_t)kVocabTile));

  int label_col = -1;
  if (row_ok) {
    bool ignored;
    const int64_t ys = safe_label(p.labels[row], p.ignore_index, p.vocab_total, &ignored);
    if (!ignored) {
      const int64_t local = ys - p.vocab_offset - n0;
      if (local >= 0 && local < nvalid) label_col = static_cast<int>(local);
    }
  }

  // ---- pass 1: tile maxima
  float ms = -CUDART_INF_F, mt = -CUDART_INF_F;
#pragma unroll 1
  for (int c = 0; c < kChunks; ++c) {
    float v[32];
    src.load(0, c, v);
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (c * 32 + j < nvalid) ms = fmaxf(ms, v[j]);
    if (teacher) {
      src.load(1, c, v);
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (c * 32 + j < nvalid) mt = fmaxf(mt, v[j]);
    }
  }

  // ---- pass 2: shifted logits and the label logit
  float zy_s = 0.f, zy_t = 0.f;
  const int64_t ws_row = row * p.ld_ws + n0;
#pragma unroll 1
  for (int c = 0; c < kChunks; ++c) {
    float v[32];
    src.load(0, c, v);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (c * 32 + j == label_col) zy_s = v[j];
      v[j] = (v[j] - ms) * kLog2e;
    }
    if (row_ok && (f & F_WRITE_WS_S)) store_chunk32<WsT>(static_cast<WsT*>(p.ws_s) + ws_row + c * 32, v);
    if (teacher) {
      src.load(1, c, v);
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (c * 32 + j == label_col) zy_t = v[j];
        v[j] = (v[j] - mt) * kLog2e;
      }
      if (row_ok && (f & F_WRITE_WS_T)) store_chunk32<WsT>(static_cast<WsT*>(p.ws_t) + ws_row + c * 32, v);
    }
  }

  if (row_ok) {
    reinterpret_cast<float2*>(p.tile_stats)[row * p.n_vtiles + tile] = make_float2(ms, mt);
    if (label_col >= 0) {
      p.label_logits[row * 2 + 0] = zy_s;
      p.label_logits[row * 2 + 1] = zy_t;
    }
  }
}

}  // namespace orda
