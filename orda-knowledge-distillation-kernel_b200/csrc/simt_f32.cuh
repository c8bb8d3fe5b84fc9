// fp32 path (fp32 hidden and weights): CUDA-core GEMM and the statistics pass over
// materialised fp32 logits. The tensor-core kinds that take fp32 inputs (tf32) cannot hold the
// 1e-5 relative tolerance the fp32 reference path is held to, and the fp32 configurations are
// small, so this path trades speed for exact fp32 arithmetic. It shares the epilogue statistics
// code and every row kernel with the tensor-core path.
#pragma once

#include "distill_common.cuh"
#include "fwd_epilogue.cuh"

namespace orda {

// D[m, n] = sum_k A[m*sam + k*sak] * B[n*sbn + k*sbk];  out[m*ldo + n] (=|+=) D.
constexpr int kSimtTile = 64, kSimtK = 16;

__global__ void __launch_bounds__(256) simt_gemm_f32_kernel(const float* __restrict__ A, int64_t sam, int64_t sak,
                                                            const float* __restrict__ B, int64_t sbn, int64_t sbk,
                                                            float* __restrict__ out, int64_t ldo, int64_t M,
                                                            int64_t N, int64_t K, int accumulate) {
  __shared__ float As[kSimtK][kSimtTile + 4];
  __shared__ float Bs[kSimtK][kSimtTile + 4];
  const int64_t m0 = (int64_t)blockIdx.y * kSimtTile, n0 = (int64_t)blockIdx.x * kSimtTile;
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += kSimtK) {
    for (int i = threadIdx.x; i < kSimtK * kSimtTile; i += 256) {
      const int kk = i / kSimtTile, mm = i % kSimtTile;
      const int64_t gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < M && gk < K) ? A[gm * sam + gk * sak] : 0.f;
      const int64_t gn = n0 + mm;
      Bs[kk][mm] = (gn < N && gk < K) ? B[gn * sbn + gk * sbk] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kSimtK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        a[i] = As[kk][ty * 4 + i];
        b[i] = Bs[kk][tx * 4 + i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
      if (m < M && n < N) {
        float* o = out + m * ldo + n;
        *o = accumulate ? *o + acc[i][j] : acc[i][j];
      }
    }
}

// Source of logits chunks read from materialised fp32 rows (student row in ws_s, teacher in ws_t).
struct GmemRowSrc {
  const float* s;
  const float* t;
  int nvalid;
  bool ok;
  __device__ __forceinline__ void load(int acc, int chunk, float (&v)[32]) const {
    const float* q = (acc == 0 ? s : t) + chunk * 32;
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (ok && chunk * 32 + j < nvalid) ? q[j] : 0.f;
  }
};

// One thread per (row, vocab tile): tile statistics over raw fp32 logits, shifted in place.
template <bool kTeacherAcc>
__global__ void fwd_stats_gmem_kernel(FwdEpiParams p) {
  const int64_t total = p.rows * (int64_t)p.n_vtiles;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = i / p.n_vtiles;
    const int tile = static_cast<int>(i % p.n_vtiles);
    const int64_t n0 = (int64_t)tile * kVocabTile;
    GmemRowSrc src;
    src.s = static_cast<const float*>(p.ws_s) + row * p.ld_ws + n0;
    src.t = kTeacherAcc ? static_cast<const float*>(p.ws_t) + row * p.ld_ws + n0 : nullptr;
    src.nvalid = static_cast<int>((p.vocab - n0 < (int64_t)kVocabTile ? p.vocab - n0 : (int64_t)kVocabTile));
    src.ok = true;
    fwd_tile_stats<float, kTeacherAcc>(p, row, true, n0, tile, src);
  }
}

}  // namespace orda
