/*
 * orda_b200_testing.h - testing hook of the B200 distillation library (no counterpart in the
 * reference). It exposes the library's tcgen05 GEMM on its own so the GPU tests can check each
 * operand layout against a plain matrix product before the fused paths are checked.
 */
#ifndef ORDA_B200_TESTING_H_
#define ORDA_B200_TESTING_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* out[m*ldo + n] = sum_k A(m, k) * B(n, k) in fp32, with 16-bit A/B (ORDA_BF16 / ORDA_F16).
 * A(m, k) = A[m*lda + k] (a_mn == 0, K-major) or A[k*lda + m] (a_mn == 1, MN-major); B likewise.
 * Enqueued on `stream`; pipeline timeouts are reported in *status. */
int32_t orda_debug_gemm(int32_t dtype, int32_t a_mn, int32_t b_mn, const void* A, int64_t lda, const void* B,
                        int64_t ldb, int64_t M, int64_t N, int64_t K, float* out, int64_t ldo, int32_t* status,
                        void* stream);

/* Same contract, computed by the CTA-pair (cta_group::2) kernel with 256 x 256 tiles. */
int32_t orda_debug_gemm_pair(int32_t dtype, int32_t a_mn, int32_t b_mn, const void* A, int64_t lda, const void* B,
                             int64_t ldb, int64_t M, int64_t N, int64_t K, float* out, int64_t ldo, int32_t* status,
                             void* stream);

/* Same contract, computed by the wide CTA-pair kernel with 512 x 256 tiles (two accumulators). */
int32_t orda_debug_gemm_wide(int32_t dtype, int32_t a_mn, int32_t b_mn, const void* A, int64_t lda, const void* B,
                             int64_t ldb, int64_t M, int64_t N, int64_t K, float* out, int64_t ldo, int32_t* status,
                             void* stream);

/* Pipeline counters of the CTA-pair GEMMs, collected while the environment variable
 * ORDA_GEMM_PROFILE=1 was set when the library first launched one: out[slot*8 + i] for slot 0 logits
 * GEMM, 1 dHidden, 2 dW, 3 unused; i = 0 MMA issuer waiting for a free accumulator, 1 MMA issuer
 * waiting for a loaded stage, 2 MMA issuer total, 3 epilogue waiting for an accumulator, 4 epilogue
 * working, 5 producer waiting for a free stage, 6 producer total (SM clock cycles summed over CTAs),
 * 7 tiles. Synchronous; `reset` != 0 zeroes the counters afterwards. */
int32_t orda_debug_gemm_profile(uint64_t* out, int32_t reset);

/* Bounded-wait check: one thread waits on an mbarrier that nothing arrives at, with the same bounded
 * wait the GEMM pipelines use but a limit of limit_ns (<= the library's 2 s bound). The wait gives
 * up, writes ORDA_ERR_TIMEOUT to *status (device int32, zero on entry), stores the time it waited in
 * *waited_ns (device uint64) and the kernel returns, leaving the context usable. */
int32_t orda_debug_wait_timeout(int32_t* status, uint64_t limit_ns, uint64_t* waited_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ORDA_B200_TESTING_H_ */
