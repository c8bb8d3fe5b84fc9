// Host side of the C ABI (include/orda_b200.h): argument checks, workspace layout, TMA descriptor
// encoding and the per-chunk launch sequence
//
//   logits GEMM + statistics epilogue -> row merge -> row losses -> [JSD sweep] -> dlogits sweep
//   -> dH GEMM(s) -> dW GEMM(s)            ...per chunk, then one final reduction.
//
// It replaces the Python chunk loop of the reference autograd Functions
// (ops/tied_teacher.py:366-516, ops/separate_teacher.py:589-700 and 849-968,
// ops/precomputed_teacher.py:358-478).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "gemm_tc.cuh"
#include "gemm_tc2.cuh"
#include "gemm_tc2w.cuh"
#include "orda_b200.h"
#include "orda_b200_testing.h"
#include "row_kernels.cuh"
#include "simt_f32.cuh"

using namespace orda;

namespace {

std::atomic<uint64_t> g_launches{0};
inline void count_launch(uint64_t n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D tensor map over a row-major [outer, inner] array of 16-bit elements with a 128B-swizzled box.
int make_map(CUtensorMap* m, int dtype, const void* base, uint64_t inner, uint64_t outer, uint64_t ld_elems,
             uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return ORDA_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (ld_elems * 2) % 16 != 0) return ORDA_ERR_ALIGNMENT;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {ld_elems * 2};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, dtype == ORDA_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                        const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? ORDA_OK : ORDA_ERR_INVALID_ARGUMENT;
}

// Operand map: K-major [mn, k] (k contiguous) or MN-major [k, mn] (mn contiguous).
int make_operand_map(CUtensorMap* m, int dtype, const void* base, bool mn_major, int64_t mn, int64_t k, int64_t ld,
                     int tile_mn) {
  if (mn_major) return make_map(m, dtype, base, mn, k, ld, 64, 64);
  return make_map(m, dtype, base, k, mn, ld, 64, tile_mn);
}

int num_sms() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}


size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
size_t esize(int dtype) { return dtype == ORDA_F32 ? 4 : 2; }

// Bound of the default chunk's logits buffers: 2 GiB, so the logits of a whole Llama-3-8B-head batch
// (8192 tokens x 128256 x 2 distributions x 2 B = 4.2 GB) are never held at once; the chunk is 4096
// rows there. A one-chunk layout was measured 2.4% faster on that step (fewer dW accumulations) and
// stays available through chunk_rows.
constexpr int64_t kDefaultWorkspaceLogitBytes = int64_t(2) << 30;

struct Plan {
  // problem classification
  bool teacher;        // teacher logits exist
  bool teacher_gmem;   // from caller memory
  bool teacher_acc;    // from a second accumulator
  bool teacher_ce;
  bool kl, jsd, rev, t_not_one;
  bool grad_s, grad_t, any_grad;
  bool write_ws_s, write_ws_t;
  uint32_t flags;
  // layout
  int64_t C, n_vtiles, vpad;
  size_t off_row_losses, off_tile_stats, off_label, off_row_stats, off_row_sums, off_ws_s, off_ws_t, total;
  int32_t parts;       // column parts of the row sweeps
  int64_t part_cols;
  size_t off_part_records;
  int32_t dh_split;     // K (vocabulary) split of the dHidden GEMM: 4 for V >= 65536, else 2
  size_t off_dh_split;  // fp32 partials of the k-split dHidden GEMM: [dh_split][C][max(H, Ht)]
  // Epilogue-statistics path: the logits epilogue sums each stored tile, so the row records come
  // from the tile records (no statistics pass over the logits); the divergence row sums come from
  // the dlogits sweep (forward KL) or one base-2 divergence sweep before it (reverse KL, JSD).
  // 16-bit compute, teacher logits from an accumulator (or no teacher), gradients requested, one
  // GPU; at T != 1 the epilogue also sums the tempered exponentials.
  bool es;
  // Precomputed teacher logits, T = 1, JSD: the row sums come from the base-2 divergence sweep
  // (column parts, caller's teacher logits) instead of the one-warp-per-row JSD sweep.
  bool gmem_div;
  size_t off_tile_sums;    // [C][n_vtiles] float2 (T = 1) or float4 (T != 1: plain and tempered sums)
  size_t off_cross_parts;  // [parts][C] fp32
};

// ORDA_EPILOGUE_STATS=0 turns the epilogue-statistics path off (A/B measurements and tests of the
// statistics-pass path on the same inputs).
// The epilogue-statistics path at T != 1 (tempered tile sums, tempered divergence sweeps);
// ORDA_EPILOGUE_STATS_T=0 keeps T != 1 on the statistics-pass path (A/B measurements).
bool epilogue_stats_tempered() {
  static const bool on = [] {
    const char* e = getenv("ORDA_EPILOGUE_STATS_T");
    return !(e && e[0] == '0');
  }();
  return on;
}

bool epilogue_stats_enabled() {
  static const bool on = [] {
    const char* e = getenv("ORDA_EPILOGUE_STATS");
    return !(e && e[0] == '0');
  }();
  return on;
}

int check_args(const orda_distill_args_t* a) {
  if (!a || a->abi_version != ORDA_ABI_VERSION) return ORDA_ERR_INVALID_ARGUMENT;
  if (a->n_rows <= 0 || a->hidden <= 0 || a->vocab <= 0) return ORDA_ERR_INVALID_ARGUMENT;
  if (a->compute_dtype != ORDA_F32 && a->compute_dtype != ORDA_F16 && a->compute_dtype != ORDA_BF16)
    return ORDA_ERR_INVALID_ARGUMENT;
  if (!a->student_hidden || !a->weight || !a->labels || !a->out_reduced || !a->device_status)
    return ORDA_ERR_INVALID_ARGUMENT;
  if (a->teacher_mode < ORDA_TEACHER_TIED || a->teacher_mode > ORDA_TEACHER_HIDDEN) return ORDA_ERR_INVALID_ARGUMENT;
  if (a->vocab_offset < 0 || a->vocab_total < a->vocab_offset + a->vocab) return ORDA_ERR_INVALID_ARGUMENT;
  if (!(a->kl_temperature > 0.f) || a->student_ce_weight < 0.f || a->teacher_ce_weight < 0.f || a->kl_weight < 0.f)
    return ORDA_ERR_INVALID_ARGUMENT;
  if (a->divergence < ORDA_DIV_FORWARD || a->divergence > ORDA_DIV_JSD) return ORDA_ERR_INVALID_ARGUMENT;
  if (a->divergence == ORDA_DIV_JSD && !(a->jsd_beta >= 0.f && a->jsd_beta <= 1.f)) return ORDA_ERR_INVALID_ARGUMENT;
  if (a->teacher_mode == ORDA_TEACHER_LOGITS && a->teacher_ce_weight != 0.f) return ORDA_ERR_UNSUPPORTED;
  if (a->teacher_mode == ORDA_TEACHER_HIDDEN && a->teacher_ce_weight != 0.f) return ORDA_ERR_UNSUPPORTED;
  return ORDA_OK;
}

Plan make_plan(const orda_distill_args_t* a, int64_t chunk_override, bool allow_es = true) {
  Plan p{};
  const int mode = a->teacher_mode;
  p.teacher_ce = a->teacher_ce_weight != 0.f;
  p.kl = a->kl_weight != 0.f;
  p.teacher = p.kl || p.teacher_ce;
  p.teacher_gmem = p.teacher && mode == ORDA_TEACHER_LOGITS;
  p.teacher_acc = p.teacher && !p.teacher_gmem;
  p.t_not_one = a->kl_temperature != 1.f;
  const bool beta_edge0 = a->divergence == ORDA_DIV_JSD && a->jsd_beta == 0.f;
  const bool beta_edge1 = a->divergence == ORDA_DIV_JSD && a->jsd_beta == 1.f;
  p.jsd = p.kl && a->divergence == ORDA_DIV_JSD && !beta_edge0 && !beta_edge1;
  p.rev = p.kl && (a->divergence == ORDA_DIV_REVERSE || beta_edge1);
  p.grad_s = a->need_grad_student_hidden || a->need_grad_weight;
  const bool tied = mode == ORDA_TEACHER_TIED, sep = mode == ORDA_TEACHER_SEPARATE;
  p.grad_t = p.teacher_ce && ((tied && (a->need_grad_teacher_hidden || a->need_grad_weight)) ||
                              (sep && (a->need_grad_teacher_hidden || a->need_grad_teacher_weight)));
  p.any_grad = p.grad_s || p.grad_t;
  // the row statistics pass streams the shifted logits, so they are always kept
  p.write_ws_s = true;
  p.write_ws_t = p.teacher_acc;
  uint32_t f = 0;
  if (p.teacher) f |= F_TEACHER;
  if (p.teacher_gmem) f |= F_TEACHER_GMEM;
  if (p.teacher_ce) f |= F_TEACHER_CE;
  if (p.kl) f |= F_KL;
  if (p.t_not_one) f |= F_T_NOT_ONE;
  if (p.rev) f |= F_KL_REVERSE;
  if (p.jsd) f |= F_JSD;
  if (p.write_ws_s) f |= F_WRITE_WS_S;
  if (p.write_ws_t) f |= F_WRITE_WS_T;
  if (p.grad_s) f |= F_GRAD_S;
  if (p.grad_t) f |= F_GRAD_T;
  if (a->validate_labels) f |= F_VALIDATE;
  p.flags = f;
  p.es = allow_es && epilogue_stats_enabled() && a->compute_dtype != ORDA_F32 && !p.teacher_gmem &&
         (!p.t_not_one || epilogue_stats_tempered()) && p.any_grad;
  p.gmem_div = allow_es && epilogue_stats_enabled() && a->compute_dtype != ORDA_F32 && p.teacher_gmem &&
               !p.t_not_one && p.jsd;

  p.n_vtiles = cdiv(a->vocab, kVocabTile);
  p.vpad = p.n_vtiles * kVocabTile;
  const size_t es = esize(a->compute_dtype);
  const int64_t bufs = (p.write_ws_s || a->compute_dtype == ORDA_F32 ? 1 : 0) + (p.teacher_acc ? 1 : 0);
  int64_t C = chunk_override > 0 ? chunk_override : a->chunk_rows;
  if (C <= 0) {
    const int64_t per_row = std::max<int64_t>(1, bufs) * p.vpad * (int64_t)es;
    C = std::max<int64_t>(kTileRows, (kDefaultWorkspaceLogitBytes / per_row) / kTileRows * kTileRows);
  }
  p.C = std::min<int64_t>(C, a->n_rows);

  size_t off = 0;
  p.off_row_losses = off; off = align256(off + sizeof(float) * 3 * a->n_rows);
  p.off_tile_stats = off; off = align256(off + sizeof(float) * p.C * p.n_vtiles * kTileStats);
  p.off_label = off; off = align256(off + sizeof(float) * 2 * p.C);
  p.off_row_stats = off; off = align256(off + sizeof(float) * kRowStats * p.C);
  p.off_row_sums = off; off = align256(off + sizeof(float) * 2 * p.C);
  // Row sweeps split long rows into up to 4 column parts (>= 8192 columns each) so that the warp
  // tasks spread evenly over the SMs and each SM has enough rows streaming at once; the parts'
  // records are merged like vocab shards. The split depends on the vocabulary alone, so a row's
  // arithmetic does not depend on how many rows a call has.
  p.parts = static_cast<int32_t>(std::max<int64_t>(1, std::min<int64_t>(4, a->vocab / 8192)));
  p.part_cols = cdiv(cdiv(a->vocab, p.parts), 256) * 256;
  p.off_part_records = off;
  if (p.parts > 1) off = align256(off + sizeof(float) * kRowStats * p.parts * p.C);
  p.off_tile_sums = off;
  if (p.es) off = align256(off + sizeof(float) * (p.t_not_one ? 4 : 2) * p.C * p.n_vtiles);
  p.off_cross_parts = off;
  if (p.es || p.gmem_div) off = align256(off + sizeof(float) * (p.jsd ? 2 : 1) * p.parts * p.C);
  // The dHidden GEMM has few output tiles (C x H), so it splits K: a 4096 x 4096 chunk has 128 wide
  // tiles, 1.7 waves on 74 CTA pairs; a 4-way split gives 512 work units, 6.9 waves. The split
  // depends on the vocabulary alone, so a row's arithmetic does not depend on the chunking.
  p.dh_split = a->vocab >= 65536 ? 4 : 2;
  p.off_dh_split = off;
  if (a->compute_dtype != ORDA_F32 && (a->need_grad_student_hidden || a->need_grad_teacher_hidden))
    off = align256(off + sizeof(float) * p.dh_split * p.C * std::max(a->hidden, a->teacher_hidden));
  // the fp32 path materialises raw logits, so it always needs the student (and teacher) buffer
  const bool need_s = p.write_ws_s || a->compute_dtype == ORDA_F32;
  const bool need_t = p.teacher_acc && (p.write_ws_t || a->compute_dtype == ORDA_F32);
  p.off_ws_s = off; if (need_s) off = align256(off + es * p.C * p.vpad);
  p.off_ws_t = off; if (need_t) off = align256(off + es * p.C * p.vpad);
  p.total = off;
  return p;
}

template <typename Kernel>
void set_smem(Kernel k, uint32_t bytes) {
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
}

template <int BN, bool A_MN, bool B_MN, typename T16>
int launch_tc(TcGemmParams& prm, int64_t M, int64_t N, cudaStream_t stream, int group_m) {
  using S = GemmShape<BN>;
  prm.m_tiles = static_cast<int32_t>(cdiv(M, kTileRows));
  prm.n_tiles = static_cast<int32_t>(cdiv(N, BN));
  prm.group_m = group_m;
  const int64_t tiles = (int64_t)prm.m_tiles * prm.n_tiles;
  if (tiles <= 0) return ORDA_OK;
  if (tiles > INT32_MAX) return ORDA_ERR_UNSUPPORTED;
  auto k = tc_gemm_kernel<BN, A_MN, B_MN, T16>;
  set_smem(k, S::kSmemBytes);
  const int grid = static_cast<int>(std::min<int64_t>(tiles, num_sms()));
  count_launch();
  k<<<grid, kGemmThreads, S::kSmemBytes, stream>>>(prm);
  return cudaPeekAtLastError() == cudaSuccess ? ORDA_OK : ORDA_ERR_CUDA;
}

// Pipeline counters of the pair GEMMs are collected when ORDA_GEMM_PROFILE=1 (testing hook; read back
// with orda_debug_gemm_profile).
bool gemm_profiling() {
  static const bool on = [] {
    const char* e = getenv("ORDA_GEMM_PROFILE");
    return e && e[0] == '1';
  }();
  return on;
}

// Tile-raster grouping of the pair GEMMs (tile_coords: > 0 groups that many m tiles with m running
// fastest, < 0 groups n tiles). Testing knob: ORDA_GROUP_LOGITS / ORDA_GROUP_DH / ORDA_GROUP_DW
// replace the defaults, so the raster can be swept without a rebuild.
int group_for(int role, int dflt) {
  static int v[3] = {0, 0, 0};
  static std::once_flag once;
  std::call_once(once, [] {
    const char* names[3] = {"ORDA_GROUP_LOGITS", "ORDA_GROUP_DH", "ORDA_GROUP_DW"};
    for (int i = 0; i < 3; ++i) {
      const char* e = getenv(names[i]);
      v[i] = e ? atoi(e) : 0;
    }
  });
  return v[role] != 0 ? v[role] : dflt;
}
enum GemmRole { ROLE_LOGITS = 0, ROLE_DH = 1, ROLE_DW = 2 };

template <bool A_MN, bool B_MN, int AMODE, bool TWO_SEG, int EPI, typename T16>
int launch_tc2(TcGemmParams& prm, int64_t M_tiles, int64_t N, cudaStream_t stream, int group_m,
               int reserve_sms = 0) {
  using S = PairShape<AMODE>;
  prm.m_tiles = static_cast<int32_t>(M_tiles);
  prm.n_tiles = static_cast<int32_t>(cdiv(N, kPairBN));
  prm.group_m = group_m;
  const int64_t tiles = (int64_t)prm.m_tiles * prm.n_tiles;
  if (tiles <= 0) return ORDA_OK;
  if (tiles > INT32_MAX) return ORDA_ERR_UNSUPPORTED;
  auto k = tc2_gemm_kernel<A_MN, B_MN, AMODE, TWO_SEG, EPI, T16>;
  set_smem(k, S::kSmemBytes);
  prm.prof_slot = gemm_profiling() ? (EPI == EPI_FWD_STATS ? 0 : (A_MN ? 2 : 1)) : -1;
  const int usable = std::max(2, num_sms() - std::max(0, reserve_sms));
  const int pairs = static_cast<int>(std::min<int64_t>(tiles, usable / 2));
  count_launch();
  k<<<2 * pairs, kGemmThreads, S::kSmemBytes, stream>>>(prm);
  return cudaPeekAtLastError() == cudaSuccess ? ORDA_OK : ORDA_ERR_CUDA;
}


// Wide pair kernel (512 x 256 tiles); M_tiles counts 512-row (A_PLAIN) or 256-token (A_INTERLEAVE) tiles.
template <bool A_MN, bool B_MN, int AMODE, bool TWO_SEG, int EPI, typename T16>
int launch_tc2w(TcGemmParams& prm, int64_t M_tiles, int64_t N, cudaStream_t stream, int group_m,
                int reserve_sms = 0) {
  using S = WideShape<EPI>;
  prm.m_tiles = static_cast<int32_t>(M_tiles);
  prm.n_tiles = static_cast<int32_t>(cdiv(N, kPairBN));
  prm.group_m = group_m;
  const int64_t tiles = (int64_t)prm.m_tiles * prm.n_tiles * std::max<int32_t>(1, prm.ksplit);
  if (tiles <= 0) return ORDA_OK;
  if (tiles > INT32_MAX) return ORDA_ERR_UNSUPPORTED;
  auto k = tc2w_gemm_kernel<A_MN, B_MN, AMODE, TWO_SEG, EPI, T16>;
  set_smem(k, S::kSmemBytes);
  prm.prof_slot = gemm_profiling() ? (EPI == EPI_FWD_STATS ? 0 : (A_MN ? 2 : 1)) : -1;
  const int usable = std::max(2, num_sms() - std::max(0, reserve_sms));
  const int pairs = static_cast<int>(std::min<int64_t>(tiles, usable / 2));
  count_launch();
  k<<<2 * pairs, S::kThreads, S::kSmemBytes, stream>>>(prm);
  return cudaPeekAtLastError() == cudaSuccess ? ORDA_OK : ORDA_ERR_CUDA;
}


struct ChunkPtrs {
  const uint8_t* hs; const uint8_t* ht; const int64_t* labels;
  int64_t r0, rows;
  uint8_t* grad_hs; uint8_t* grad_ht;
  const uint8_t* tg;
};

RowParams row_params(const orda_distill_args_t* a, const Plan& P, uint8_t* ws, const ChunkPtrs& c) {
  RowParams r{};
  r.rows = c.rows;
  r.vocab = a->vocab; r.vocab_offset = a->vocab_offset; r.vocab_total = a->vocab_total;
  r.ignore_index = a->ignore_index;
  r.n_vtiles = static_cast<int32_t>(P.n_vtiles);
  r.flags = P.flags;
  r.temperature = a->kl_temperature; r.inv_t = 1.f / a->kl_temperature;
  r.jsd_beta = a->jsd_beta;
  r.w_s = a->student_ce_weight; r.w_t = a->teacher_ce_weight; r.w_kl = a->kl_weight;
  r.labels = c.labels;
  r.tile_stats = reinterpret_cast<float*>(ws + P.off_tile_stats);
  r.label_logits = reinterpret_cast<float*>(ws + P.off_label);
  r.row_stats = reinterpret_cast<float*>(ws + P.off_row_stats);
  r.row_sums = reinterpret_cast<float*>(ws + P.off_row_sums);
  float* rl = a->out_row_losses ? a->out_row_losses : reinterpret_cast<float*>(ws + P.off_row_losses);
  r.row_losses = rl + c.r0;
  r.ld_row_losses = a->n_rows;
  r.ws_s = ws + P.off_ws_s; r.ws_t = ws + P.off_ws_t; r.ld_ws = P.vpad;
  r.t_gmem = c.tg; r.ld_tg = a->ld_teacher_logits; r.tg_dtype = a->teacher_logits_dtype;
  r.tg_vec = c.tg && (reinterpret_cast<uintptr_t>(a->teacher_logits) & 15u) == 0 &&
             (a->ld_teacher_logits * static_cast<int64_t>(esize(a->teacher_logits_dtype))) % 16 == 0;
  r.status = a->device_status;
  r.grad_scale = a->grads_include_mean_scale ? a->out_reduced + ORDA_OUT_MEAN_SCALE : nullptr;
  r.parts = P.parts;
  r.part_cols = P.part_cols;
  r.part_records = reinterpret_cast<float*>(ws + P.off_part_records);
  r.tile_sums = P.es ? reinterpret_cast<const float*>(ws + P.off_tile_sums) : nullptr;
  r.cross_parts = (P.es && P.kl) || P.gmem_div ? reinterpret_cast<float*>(ws + P.off_cross_parts) : nullptr;
  return r;
}

FwdEpiParams fwd_params(const orda_distill_args_t* a, const Plan& P, uint8_t* ws, const ChunkPtrs& c) {
  FwdEpiParams f{};
  f.rows = c.rows;
  f.vocab = a->vocab; f.vocab_offset = a->vocab_offset; f.vocab_total = a->vocab_total;
  f.ignore_index = a->ignore_index;
  f.n_vtiles = static_cast<int32_t>(P.n_vtiles);
  f.flags = P.flags;
  f.inv_t = 1.f / a->kl_temperature;
  f.labels = c.labels;
  f.ws_s = ws + P.off_ws_s; f.ws_t = ws + P.off_ws_t; f.ld_ws = P.vpad;
  f.t_gmem = c.tg; f.ld_tg = a->ld_teacher_logits; f.tg_dtype = a->teacher_logits_dtype;
  f.tile_stats = reinterpret_cast<float*>(ws + P.off_tile_stats);
  f.label_logits = reinterpret_cast<float*>(ws + P.off_label);
  f.tile_sums = P.es ? reinterpret_cast<float*>(ws + P.off_tile_sums) : nullptr;
  return f;
}

// ------------------------------------------------------------------ 16-bit (tensor core) phases
// TMA store maps of the chunk's shifted-logit buffers ([rows, Vpad], 64 x 32 boxes) for the wide kernel.
int ws_store_maps(const orda_distill_args_t* a, const Plan& P, uint8_t* ws, const ChunkPtrs& c, TcGemmParams& prm) {
  int rc;
  if (P.write_ws_s &&
      (rc = make_map(&prm.ws_s_map, a->compute_dtype, ws + P.off_ws_s, P.vpad, c.rows, P.vpad, 64, 32)))
    return rc;
  if (P.teacher_acc && P.write_ws_t &&
      (rc = make_map(&prm.ws_t_map, a->compute_dtype, ws + P.off_ws_t, P.vpad, c.rows, P.vpad, 64, 32)))
    return rc;
  return ORDA_OK;
}

template <typename T16>
int forward_tc(const orda_distill_args_t* a, const Plan& P, uint8_t* ws, const ChunkPtrs& c, cudaStream_t s) {
  const int dt = a->compute_dtype;
  TcGemmParams prm{};
  prm.status = a->device_status;
  prm.fwd = fwd_params(a, P, ws, c);
  int rc;
  if ((rc = make_operand_map(&prm.a0, dt, c.hs, false, c.rows, a->hidden, a->ld_student_hidden, kTileRows))) return rc;
  if ((rc = make_operand_map(&prm.b0, dt, a->weight, false, a->vocab, a->hidden, a->ld_weight, kVocabTile))) return rc;
  prm.kb0 = static_cast<int32_t>(cdiv(a->hidden, kBK));
  if (P.teacher_acc && a->teacher_mode == ORDA_TEACHER_TIED) {
    // CTA-pair kernel: 64 student rows + the same 64 teacher rows per CTA, half the lm_head tile per CTA
    if ((rc = make_operand_map(&prm.a0, dt, c.hs, false, c.rows, a->hidden, a->ld_student_hidden, 64))) return rc;
    if ((rc = make_operand_map(&prm.a1, dt, c.ht, false, c.rows, a->hidden, a->ld_teacher_hidden, 64))) return rc;
    if ((rc = ws_store_maps(a, P, ws, c, prm))) return rc;
    return launch_tc2w<false, false, A_INTERLEAVE, false, EPI_FWD_STATS, T16>(prm, cdiv(c.rows, 256), a->vocab, s,
                                                                            group_for(ROLE_LOGITS, 8));
  }
  if ((rc = ws_store_maps(a, P, ws, c, prm))) return rc;
  if ((rc = launch_tc2w<false, false, A_PLAIN, false, EPI_FWD_STATS, T16>(prm, cdiv(c.rows, 512), a->vocab, s,
                                                                        group_for(ROLE_LOGITS, 4))))
    return rc;
  if (P.teacher_acc) {
    // separate teacher (or precomputed teacher hidden + weight): a second wide launch over (ht, Wt)
    // writes the teacher's tile maxima, shifted logits and label logits
    TcGemmParams pt = prm;
    if ((rc = make_operand_map(&pt.a0, dt, c.ht, false, c.rows, a->teacher_hidden, a->ld_teacher_hidden, kTileRows))) return rc;
    if ((rc = make_operand_map(&pt.b0, dt, a->teacher_weight, false, a->vocab, a->teacher_hidden, a->ld_teacher_weight, kVocabTile))) return rc;
    pt.kb0 = static_cast<int32_t>(cdiv(a->teacher_hidden, kBK));
    pt.fwd.plain_teacher = 1;
    return launch_tc2w<false, false, A_PLAIN, false, EPI_FWD_STATS, T16>(pt, cdiv(c.rows, 512), a->vocab, s,
                                                                         group_for(ROLE_LOGITS, 4));
  }
  return ORDA_OK;
}

// dH[rows, N] = dZ[rows, V] * Wm[V, N]
// dHidden has few output tiles (rows x H), so the wide pair kernel splits K (the vocabulary) into
// P.dh_split ranges: each accumulates an fp32 partial in the workspace and a sum kernel adds them
// in a fixed order into the 16-bit result. The split does not depend on the row count, so chunking
// leaves every row's arithmetic unchanged.
template <typename T16>
int dh_tc(const orda_distill_args_t* a, const Plan& P, uint8_t* ws, const void* dz, const void* wmat, int64_t ldw,
          int64_t n, void* out, int64_t rows, int32_t* status, cudaStream_t s) {
  const int reserve = a->dweight_first ? a->overlap_reserve_sms : 0;
  TcGemmParams prm{};
  prm.status = status;
  int rc;
  if ((rc = make_operand_map(&prm.a0, a->compute_dtype, dz, false, rows, a->vocab, P.vpad, kTileRows))) return rc;
  if ((rc = make_operand_map(&prm.b0, a->compute_dtype, wmat, true, n, a->vocab, ldw, 128))) return rc;
  prm.kb0 = static_cast<int32_t>(cdiv(a->vocab, kBK));
  if (prm.kb0 < 2 || n % 8 != 0) {
    prm.st = StoreEpiParams{out, n, rows, n, 0, 0};
    return launch_tc2<false, true, A_PLAIN, false, EPI_STORE, T16>(prm, cdiv(rows, 256), n, s, group_for(ROLE_DH, 8),
                                                                    reserve);
  }
  float* part = reinterpret_cast<float*>(ws + P.off_dh_split);
  prm.ksplit = P.dh_split;
  prm.kb_split = static_cast<int32_t>(cdiv(prm.kb0, P.dh_split));
  prm.split_bytes = static_cast<int64_t>(sizeof(float)) * rows * n;
  prm.st = StoreEpiParams{part, n, rows, n, 1, 0};
  if ((rc = launch_tc2w<false, true, A_PLAIN, false, EPI_STORE, T16>(prm, cdiv(rows, 512), n, s, group_for(ROLE_DH, 4),
                                                                     reserve)))
    return rc;
  const int64_t count8 = rows * n / 8;
  count_launch();
  sum_split_kernel<T16><<<static_cast<int>(std::min<int64_t>(cdiv(count8, 256), 4 * 148)), 256, 0, s>>>(
      part, P.dh_split, rows * n, static_cast<T16*>(out), count8);
  return cudaPeekAtLastError() == cudaSuccess ? ORDA_OK : ORDA_ERR_CUDA;
}

// dW[V, N] (+)= dZ0^T H0 (+ dZ1^T H1)
// With `route`, the rows of the result go to their owners' slots on the peer GPUs (accumulating the
// local partial in `out` when `accumulate`) instead of into `out`.
template <typename T16>
int dw_tc(const orda_distill_args_t* a, const Plan& P, const void* dz0, const void* h0, int64_t ldh0, const void* dz1,
          const void* h1, int64_t ldh1, int64_t n, void* out, int out_f32, int accumulate, int64_t rows,
          int32_t* status, cudaStream_t s, const orda_peer_slots_t* route = nullptr) {
  TcGemmParams prm{};
  prm.status = status;
  const int dt = a->compute_dtype;
  int rc;
  if ((rc = make_operand_map(&prm.a0, dt, dz0, true, a->vocab, rows, P.vpad, kTileRows))) return rc;
  if ((rc = make_operand_map(&prm.b0, dt, h0, true, n, rows, ldh0, 128))) return rc;
  prm.kb0 = static_cast<int32_t>(cdiv(rows, kBK));
  prm.st = StoreEpiParams{out, n, a->vocab, n, out_f32, accumulate};
  // 16-bit dW: stage the tiles in shared memory and store them by TMA, into `out` or, routed, into
  // the owners' slots (one map per owner; needs owner slabs of whole 512-row tiles)
  if (!out_f32 && n % 64 == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0 &&
      (!route || route->slab_rows % 512 == 0)) {
    if ((rc = make_map(&prm.out_map, dt, out, n, a->vocab, n, 64, 32))) return rc;
    if (route) {
      for (int k = 0; k < route->world; ++k) {
        const uint8_t* slot = static_cast<const uint8_t*>(route->slot_base[k]) +
                              static_cast<int64_t>(route->rank) * route->slab_rows * n * 2;
        if ((rc = make_map(&prm.peer_maps[k], dt, slot, n, route->slab_rows, n, 64, 32))) return rc;
      }
    }
    prm.st_tma = 1;
  }
  if (route) {
    prm.st.peers = route->world;
    prm.st.slot = route->rank;
    prm.st.slab_rows = route->slab_rows;
    prm.st.acc_src = accumulate ? out : nullptr;
    for (int k = 0; k < route->world; ++k) prm.st.peer_base[k] = route->slot_base[k];
  }
  if (dz1) {
    if ((rc = make_operand_map(&prm.a1, dt, dz1, true, a->vocab, rows, P.vpad, kTileRows))) return rc;
    if ((rc = make_operand_map(&prm.b1, dt, h1, true, n, rows, ldh1, 128))) return rc;
    prm.kb1 = prm.kb0;
    return launch_tc2w<true, true, A_PLAIN, true, EPI_STORE, T16>(prm, cdiv(a->vocab, 512), n, s, group_for(ROLE_DW, 4));
  }
  return launch_tc2w<true, true, A_PLAIN, false, EPI_STORE, T16>(prm, cdiv(a->vocab, 512), n, s, group_for(ROLE_DW, 4));
}

// ------------------------------------------------------------------ fp32 (SIMT) phases
void simt_gemm(const float* A, int64_t sam, int64_t sak, const float* B, int64_t sbn, int64_t sbk, float* out,
               int64_t ldo, int64_t M, int64_t N, int64_t K, int accumulate, cudaStream_t s) {
  dim3 grid(static_cast<unsigned>(cdiv(N, kSimtTile)), static_cast<unsigned>(cdiv(M, kSimtTile)));
  count_launch();
  simt_gemm_f32_kernel<<<grid, 256, 0, s>>>(A, sam, sak, B, sbn, sbk, out, ldo, M, N, K, accumulate);
}

int forward_f32(const orda_distill_args_t* a, const Plan& P, uint8_t* ws, const ChunkPtrs& c, cudaStream_t s) {
  float* ws_s = reinterpret_cast<float*>(ws + P.off_ws_s);
  float* ws_t = reinterpret_cast<float*>(ws + P.off_ws_t);
  simt_gemm(reinterpret_cast<const float*>(c.hs), a->ld_student_hidden, 1, static_cast<const float*>(a->weight),
            a->ld_weight, 1, ws_s, P.vpad, c.rows, a->vocab, a->hidden, 0, s);
  if (P.teacher_acc) {
    const bool tied = a->teacher_mode == ORDA_TEACHER_TIED;
    const float* wt = static_cast<const float*>(tied ? a->weight : a->teacher_weight);
    const int64_t ldwt = tied ? a->ld_weight : a->ld_teacher_weight;
    const int64_t kt = tied ? a->hidden : a->teacher_hidden;
    simt_gemm(reinterpret_cast<const float*>(c.ht), a->ld_teacher_hidden, 1, wt, ldwt, 1, ws_t, P.vpad, c.rows,
              a->vocab, kt, 0, s);
  }
  FwdEpiParams f = fwd_params(a, P, ws, c);
  f.flags |= F_WRITE_WS_S | (P.teacher_acc ? F_WRITE_WS_T : 0u);  // shift in place
  const int64_t total = c.rows * P.n_vtiles;
  const int grid = static_cast<int>(std::min<int64_t>(cdiv(total, 128), 8192));
  count_launch();
  if (P.teacher_acc) fwd_stats_gmem_kernel<true><<<grid, 128, 0, s>>>(f);
  else fwd_stats_gmem_kernel<false><<<grid, 128, 0, s>>>(f);
  return cudaPeekAtLastError() == cudaSuccess ? ORDA_OK : ORDA_ERR_CUDA;
}

// ------------------------------------------------------------------ shared row phases
template <typename WsT>
int row_phases(const orda_distill_args_t* a, const Plan& P, uint8_t* ws, const ChunkPtrs& c, cudaStream_t s,
               bool do_merge, bool do_loss_and_sweeps, const float* row_stats_ext, const float* row_sums_ext) {
  RowParams r = row_params(a, P, ws, c);
  // one warp per (row, column part), 8 per block; the JSD sweep runs one warp per row
  const int sweep_grid = static_cast<int>(std::min<int64_t>(cdiv(c.rows * P.parts, 8), 16 * num_sms()));
  const int row_grid = static_cast<int>(std::min<int64_t>(cdiv(c.rows, 8), 16 * num_sms()));
  if (P.es) {
    // row records from the epilogue's tile records -> dlogits sweep (+ cross term) -> row losses
    count_launch(3);
    tile_merge_kernel<<<row_grid, 256, 0, s>>>(r);
    if constexpr (sizeof(WsT) == 2) {
      if (P.rev || P.jsd) {
        count_launch();
        if (P.jsd) div_sweep_kernel<WsT, DK_JSD><<<sweep_grid, 256, 0, s>>>(r);
        else div_sweep_kernel<WsT, DK_REV><<<sweep_grid, 256, 0, s>>>(r);
      }
    }
    launch_grad_sweep<WsT>(r, sweep_grid, s);
    row_loss_kernel<<<static_cast<int>(cdiv(c.rows, 256)), 256, 0, s>>>(r);
    return cudaPeekAtLastError() == cudaSuccess ? ORDA_OK : ORDA_ERR_CUDA;
  }
  if (do_merge) {
    count_launch();
    launch_row_stats<WsT>(r, sweep_grid, s);
    if (P.parts > 1) {
      count_launch();
      merge_records_kernel<<<static_cast<int>(cdiv(c.rows, 256)), 256, 0, s>>>(r.part_records, P.parts, c.rows,
                                                                              r.row_stats);
    }
  }
  if (!do_loss_and_sweeps) return cudaPeekAtLastError() == cudaSuccess ? ORDA_OK : ORDA_ERR_CUDA;
  if (row_stats_ext) r.row_stats = const_cast<float*>(row_stats_ext);
  if (P.jsd && !row_sums_ext) {
    count_launch();
    bool done = false;
    if constexpr (sizeof(WsT) == 2) {
      if (P.gmem_div) {
        div_sweep_kernel<WsT, DK_JSD, true><<<sweep_grid, 256, 0, s>>>(r);
        done = true;
      }
    }
    if (!done) jsd_sweep_kernel<WsT><<<row_grid, 256, 0, s>>>(r, reinterpret_cast<float*>(ws + P.off_row_sums));
  }
  if (row_sums_ext) r.row_sums = row_sums_ext;
  count_launch();
  row_loss_kernel<<<static_cast<int>(cdiv(c.rows, 256)), 256, 0, s>>>(r);
  if (P.any_grad) {
    count_launch();
    launch_grad_sweep<WsT>(r, sweep_grid, s);
  }
  return cudaPeekAtLastError() == cudaSuccess ? ORDA_OK : ORDA_ERR_CUDA;
}

// Records the start / end event of a phase (instrumentation hook; no-op without events).
struct PhaseMark {
  const orda_distill_args_t* a;
  cudaStream_t s;
  bool on;
  void mark(int phase, int end) const {
    if (on && a->phase_events && a->phase_events[2 * phase + end])
      cudaEventRecord(static_cast<cudaEvent_t>(a->phase_events[2 * phase + end]), s);
  }
};

template <typename WsT>
int grad_gemms(const orda_distill_args_t* a, const Plan& P, uint8_t* ws, const ChunkPtrs& c, bool first_chunk,
               cudaStream_t s, const PhaseMark* pm = nullptr, bool last_chunk = true,
               const orda_peer_slots_t* peers = nullptr) {
  const bool tied = a->teacher_mode == ORDA_TEACHER_TIED;
  const bool sep = a->teacher_mode == ORDA_TEACHER_SEPARATE;
  void* ws_s = ws + P.off_ws_s;
  void* ws_t = ws + P.off_ws_t;
  const int acc = first_chunk ? 0 : 1;
  int rc = ORDA_OK;
  if constexpr (std::is_same<WsT, float>::value) {
    const float* zs = static_cast<const float*>(ws_s);
    const float* zt = static_cast<const float*>(ws_t);
    const float* W = static_cast<const float*>(a->weight);
    const float* Wt = static_cast<const float*>(a->teacher_weight);
    if (a->need_grad_student_hidden)
      simt_gemm(zs, P.vpad, 1, W, 1, a->ld_weight, reinterpret_cast<float*>(c.grad_hs), a->hidden, c.rows, a->hidden,
                a->vocab, 0, s);
    if (a->need_grad_weight) {
      simt_gemm(zs, 1, P.vpad, reinterpret_cast<const float*>(c.hs), 1, a->ld_student_hidden,
                static_cast<float*>(a->grad_weight), a->hidden, a->vocab, a->hidden, c.rows, acc, s);
      if (tied && P.grad_t)
        simt_gemm(zt, 1, P.vpad, reinterpret_cast<const float*>(c.ht), 1, a->ld_teacher_hidden,
                  static_cast<float*>(a->grad_weight), a->hidden, a->vocab, a->hidden, c.rows, 1, s);
    }
    if (P.grad_t && a->need_grad_teacher_hidden) {
      const float* wm = tied ? W : Wt;
      const int64_t ldm = tied ? a->ld_weight : a->ld_teacher_weight;
      simt_gemm(zt, P.vpad, 1, wm, 1, ldm, reinterpret_cast<float*>(c.grad_ht), a->teacher_hidden, c.rows,
                a->teacher_hidden, a->vocab, 0, s);
    }
    if (sep && P.grad_t && a->need_grad_teacher_weight)
      simt_gemm(zt, 1, P.vpad, reinterpret_cast<const float*>(c.ht), 1, a->ld_teacher_hidden,
                static_cast<float*>(a->grad_teacher_weight), a->teacher_hidden, a->vocab, a->teacher_hidden, c.rows,
                acc, s);
    if (last_chunk && a->dweight_done_event) cudaEventRecord(static_cast<cudaEvent_t>(a->dweight_done_event), s);
    rc = cudaPeekAtLastError() == cudaSuccess ? ORDA_OK : ORDA_ERR_CUDA;
  } else {
    int32_t* st = a->device_status;
    auto dhidden = [&]() -> int {
      int r = ORDA_OK;
      if (pm) pm->mark(ORDA_PHASE_DHIDDEN, 0);
      if (a->need_grad_student_hidden)
        if ((r = dh_tc<WsT>(a, P, ws, ws_s, a->weight, a->ld_weight, a->hidden, c.grad_hs, c.rows, st, s))) return r;
      if (P.grad_t && a->need_grad_teacher_hidden) {
        const void* wm = tied ? a->weight : a->teacher_weight;
        const int64_t ldm = tied ? a->ld_weight : a->ld_teacher_weight;
        if ((r = dh_tc<WsT>(a, P, ws, ws_t, wm, ldm, a->teacher_hidden, c.grad_ht, c.rows, st, s))) return r;
      }
      if (pm) pm->mark(ORDA_PHASE_DHIDDEN, 1);
      return r;
    };
    auto dweight = [&]() -> int {
      int r = ORDA_OK;
      if (pm) pm->mark(ORDA_PHASE_DWEIGHT, 0);
      if (a->need_grad_weight) {
        const bool two = tied && P.grad_t;
        if ((r = dw_tc<WsT>(a, P, ws_s, c.hs, a->ld_student_hidden, two ? ws_t : nullptr, two ? c.ht : nullptr,
                            a->ld_teacher_hidden, a->hidden, a->grad_weight, a->grad_weight_fp32, acc, c.rows, st, s,
                            last_chunk ? peers : nullptr)))
          return r;
      }
      if (sep && P.grad_t && a->need_grad_teacher_weight)
        if ((r = dw_tc<WsT>(a, P, ws_t, c.ht, a->ld_teacher_hidden, nullptr, nullptr, 0, a->teacher_hidden,
                            a->grad_teacher_weight, a->grad_weight_fp32, acc, c.rows, st, s)))
          return r;
      if (pm) pm->mark(ORDA_PHASE_DWEIGHT, 1);
      if (last_chunk && a->dweight_done_event) cudaEventRecord(static_cast<cudaEvent_t>(a->dweight_done_event), s);
      return r;
    };
    if (a->dweight_first) {
      if ((rc = dweight())) return rc;
      if ((rc = dhidden())) return rc;
    } else {
      if ((rc = dhidden())) return rc;
      if ((rc = dweight())) return rc;
    }
  }
  // tied teacher with teacher CE off: the reference returns an all-zero teacher-hidden gradient
  if (tied && a->need_grad_teacher_hidden && !P.grad_t)
    cudaMemsetAsync(c.grad_ht, 0, esize(a->compute_dtype) * c.rows * a->teacher_hidden, s);
  return rc;
}

ChunkPtrs chunk_ptrs(const orda_distill_args_t* a, int64_t r0, int64_t rows) {
  const size_t es = esize(a->compute_dtype);
  ChunkPtrs c{};
  c.r0 = r0;
  c.rows = rows;
  c.hs = static_cast<const uint8_t*>(a->student_hidden) + es * r0 * a->ld_student_hidden;
  c.ht = a->teacher_hidden_ptr ? static_cast<const uint8_t*>(a->teacher_hidden_ptr) + es * r0 * a->ld_teacher_hidden
                               : nullptr;
  c.labels = a->labels + r0;
  c.grad_hs = a->grad_student_hidden ? static_cast<uint8_t*>(a->grad_student_hidden) + es * r0 * a->hidden : nullptr;
  c.grad_ht = a->grad_teacher_hidden ? static_cast<uint8_t*>(a->grad_teacher_hidden) + es * r0 * a->teacher_hidden
                                     : nullptr;
  c.tg = a->teacher_logits
             ? static_cast<const uint8_t*>(a->teacher_logits) + esize(a->teacher_logits_dtype) * r0 * a->ld_teacher_logits
             : nullptr;
  return c;
}

int check_operands(const orda_distill_args_t* a, const Plan& P) {
  const bool needs_t_hidden = P.teacher_acc || (a->teacher_mode == ORDA_TEACHER_TIED && a->need_grad_teacher_hidden);
  if (needs_t_hidden && !a->teacher_hidden_ptr) return ORDA_ERR_INVALID_ARGUMENT;
  if (P.teacher_acc && a->teacher_mode != ORDA_TEACHER_TIED && !a->teacher_weight) return ORDA_ERR_INVALID_ARGUMENT;
  if (P.teacher_gmem && !a->teacher_logits) return ORDA_ERR_INVALID_ARGUMENT;
  if (a->need_grad_student_hidden && !a->grad_student_hidden) return ORDA_ERR_INVALID_ARGUMENT;
  if (a->need_grad_weight && !a->grad_weight) return ORDA_ERR_INVALID_ARGUMENT;
  if (a->need_grad_teacher_hidden && !a->grad_teacher_hidden) return ORDA_ERR_INVALID_ARGUMENT;
  if (a->need_grad_teacher_weight && !a->grad_teacher_weight) return ORDA_ERR_INVALID_ARGUMENT;
  if (a->compute_dtype != ORDA_F32) {
    if (a->hidden % 8 || a->ld_student_hidden % 8 || a->ld_weight % 8) return ORDA_ERR_ALIGNMENT;
    if (P.teacher_acc && (a->teacher_hidden % 8 || a->ld_teacher_hidden % 8)) return ORDA_ERR_ALIGNMENT;
    if (P.teacher_acc && a->teacher_mode != ORDA_TEACHER_TIED && a->ld_teacher_weight % 8) return ORDA_ERR_ALIGNMENT;
    if (a->grad_weight_fp32 == 0 && a->need_grad_weight == 0) { /* nothing */ }
  } else if (a->grad_weight_fp32 == 0 && (a->need_grad_weight || a->need_grad_teacher_weight)) {
    return ORDA_ERR_INVALID_ARGUMENT;  // fp32 path accumulates weight gradients in fp32
  }
  return ORDA_OK;
}

template <typename WsT>
int run_all(const orda_distill_args_t* a, const Plan& P, uint8_t* ws, cudaStream_t s,
            const orda_peer_slots_t* peers = nullptr) {
  int rc;
  if (a->grads_include_mean_scale) {
    count_launch();
    mean_scale_kernel<<<1, 1024, 0, s>>>(a->labels, a->n_rows, a->ignore_index, a->reduction, a->out_reduced);
  }
  for (int64_t r0 = 0; r0 < a->n_rows; r0 += P.C) {
    const int64_t rows = std::min<int64_t>(P.C, a->n_rows - r0);
    const ChunkPtrs c = chunk_ptrs(a, r0, rows);
    const PhaseMark pm{a, s, r0 + rows >= a->n_rows};
    pm.mark(ORDA_PHASE_LOGITS, 0);
    if constexpr (std::is_same<WsT, float>::value) rc = forward_f32(a, P, ws, c, s);
    else rc = forward_tc<WsT>(a, P, ws, c, s);
    if (rc) return rc;
    pm.mark(ORDA_PHASE_LOGITS, 1);
    pm.mark(ORDA_PHASE_ROWS, 0);
    if ((rc = row_phases<WsT>(a, P, ws, c, s, true, true, nullptr, nullptr))) return rc;
    pm.mark(ORDA_PHASE_ROWS, 1);
    if ((rc = grad_gemms<WsT>(a, P, ws, c, r0 == 0, s, &pm, pm.on, peers))) return rc;
  }
  const float* rl = a->out_row_losses ? a->out_row_losses : reinterpret_cast<const float*>(ws + P.off_row_losses);
  count_launch();
  finalize_kernel<<<1, 1024, 0, s>>>(rl, a->n_rows, a->labels, a->n_rows, a->ignore_index, a->reduction, P.flags,
                                     a->student_ce_weight, a->teacher_ce_weight, a->kl_weight, a->out_reduced);
  return cudaPeekAtLastError() == cudaSuccess ? ORDA_OK : ORDA_ERR_CUDA;
}

int dispatch_all(const orda_distill_args_t* a, const Plan& P, uint8_t* ws, cudaStream_t s) {
  switch (a->compute_dtype) {
    case ORDA_BF16: return run_all<__nv_bfloat16>(a, P, ws, s);
    case ORDA_F16: return run_all<__half>(a, P, ws, s);
    default: return run_all<float>(a, P, ws, s);
  }
}

}  // namespace

extern "C" {

int32_t orda_abi_version(void) { return ORDA_ABI_VERSION; }

uint64_t orda_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

size_t orda_args_struct_size(void) { return sizeof(orda_distill_args_t); }

int32_t orda_scale_grad(void* data, int64_t n, int32_t dtype, const float* scale, void* stream) {
  if (!data || !scale || n < 0) return ORDA_ERR_INVALID_ARGUMENT;
  if (n == 0) return ORDA_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = static_cast<int>(std::min<int64_t>(cdiv(n, 8 * 256), 8 * num_sms()));
  count_launch();
  switch (dtype) {
    case ORDA_BF16: scale_grad_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(static_cast<__nv_bfloat16*>(data), n, scale); break;
    case ORDA_F16: scale_grad_kernel<__half><<<grid, 256, 0, s>>>(static_cast<__half*>(data), n, scale); break;
    case ORDA_F32: scale_grad_kernel<float><<<grid, 256, 0, s>>>(static_cast<float*>(data), n, scale); break;
    default: return ORDA_ERR_INVALID_ARGUMENT;
  }
  return cudaPeekAtLastError() == cudaSuccess ? ORDA_OK : ORDA_ERR_CUDA;
}

const char* orda_status_string(int32_t status) {
  switch (status) {
    case ORDA_OK: return "ok";
    case ORDA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case ORDA_ERR_ALIGNMENT: return "16-bit operands need 16-byte aligned bases and row strides that are multiples of 8 elements";
    case ORDA_ERR_WORKSPACE: return "workspace too small";
    case ORDA_ERR_UNSUPPORTED: return "unsupported configuration";
    case ORDA_ERR_CUDA: return "CUDA launch error";
    case ORDA_ERR_TIMEOUT: return "device pipeline wait timed out";
    case ORDA_ERR_LABEL_RANGE: return "label outside [0, vocab) that is not ignore_index";
    case ORDA_ERR_NO_DEVICE: return "no CUDA device";
    default: return "unknown status";
  }
}

size_t orda_distill_workspace_bytes(const orda_distill_args_t* args) {
  if (check_args(args) != ORDA_OK) return 0;
  return make_plan(args, 0).total;
}

int32_t orda_distill_fwdbwd(const orda_distill_args_t* args, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_args(args);
  if (rc) return rc;
  const Plan P = make_plan(args, 0);
  if ((rc = check_operands(args, P))) return rc;
  if (!workspace || workspace_bytes < P.total) return ORDA_ERR_WORKSPACE;
  return dispatch_all(args, P, static_cast<uint8_t*>(workspace), static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------- token sharding over peer memory
int32_t orda_distill_fwdbwd_peer(const orda_distill_args_t* args, void* workspace, size_t workspace_bytes,
                                 const orda_peer_slots_t* peers, void* stream) {
  int rc = check_args(args);
  if (rc) return rc;
  if (!peers || peers->world < 1 || peers->world > ORDA_MAX_PEERS || peers->rank < 0 || peers->rank >= peers->world)
    return ORDA_ERR_INVALID_ARGUMENT;
  if (args->compute_dtype == ORDA_F32 || args->grad_weight_fp32 || !args->need_grad_weight || args->vocab_offset != 0)
    return ORDA_ERR_UNSUPPORTED;
  if (peers->slab_rows <= 0 || peers->slab_rows * peers->world < args->vocab) return ORDA_ERR_INVALID_ARGUMENT;
  for (int k = 0; k < peers->world; ++k)
    if (!peers->slot_base[k] || (reinterpret_cast<uintptr_t>(peers->slot_base[k]) & 15u) != 0)
      return ORDA_ERR_ALIGNMENT;
  const Plan P = make_plan(args, 0);
  if ((rc = check_operands(args, P))) return rc;
  if (!workspace || workspace_bytes < P.total) return ORDA_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  return args->compute_dtype == ORDA_BF16 ? run_all<__nv_bfloat16>(args, P, ws, s, peers)
                                          : run_all<__half>(args, P, ws, s, peers);
}

typedef CUresult (*MemGetAddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

int32_t orda_ipc_export(const void* ptr, orda_ipc_handle_t* out) {
  if (!ptr || !out) return ORDA_ERR_INVALID_ARGUMENT;
  static MemGetAddressRangeFn range_fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      range_fn = reinterpret_cast<MemGetAddressRangeFn>(p);
  });
  if (!range_fn) return ORDA_ERR_CUDA;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range_fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return ORDA_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return ORDA_ERR_CUDA;
  static_assert(sizeof(h) <= sizeof(out->handle), "IPC handle size");
  memset(out->handle, 0, sizeof(out->handle));
  memcpy(out->handle, &h, sizeof(h));
  out->offset = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return ORDA_OK;
}

int32_t orda_ipc_import(const orda_ipc_handle_t* handle, void** ptr_out) {
  if (!handle || !ptr_out) return ORDA_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle->handle, sizeof(h));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return ORDA_ERR_CUDA;
  *ptr_out = static_cast<uint8_t*>(base) + handle->offset;
  return ORDA_OK;
}

int32_t orda_ipc_close(void* ptr, const orda_ipc_handle_t* handle) {
  if (!ptr || !handle) return ORDA_ERR_INVALID_ARGUMENT;
  return cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - handle->offset) == cudaSuccess ? ORDA_OK : ORDA_ERR_CUDA;
}

int32_t orda_peer_reduce_broadcast(const orda_peer_slots_t* peers, int64_t vocab, int64_t hidden, int32_t dtype,
                                   int32_t ctas, void* stream) {
  if (!peers || peers->world < 1 || peers->world > ORDA_MAX_PEERS || peers->rank < 0 || peers->rank >= peers->world)
    return ORDA_ERR_INVALID_ARGUMENT;
  if (vocab <= 0 || hidden <= 0 || peers->slab_rows <= 0 || peers->slab_rows * peers->world < vocab)
    return ORDA_ERR_INVALID_ARGUMENT;
  if (dtype != ORDA_BF16 && dtype != ORDA_F16) return ORDA_ERR_INVALID_ARGUMENT;
  if (hidden % 8) return ORDA_ERR_ALIGNMENT;
  for (int k = 0; k < peers->world; ++k)
    if (!peers->slot_base[k] || !peers->grad_base[k] || (reinterpret_cast<uintptr_t>(peers->slot_base[k]) & 15u) ||
        (reinterpret_cast<uintptr_t>(peers->grad_base[k]) & 15u))
      return ORDA_ERR_ALIGNMENT;
  const int64_t r0 = static_cast<int64_t>(peers->rank) * peers->slab_rows;
  const int64_t rows = std::max<int64_t>(0, std::min<int64_t>(peers->slab_rows, vocab - r0));
  if (rows == 0) return ORDA_OK;
  PeerReduceParams q{};
  q.world = peers->world;
  q.rows = rows;
  q.row0 = r0;
  q.slab_rows = peers->slab_rows;
  q.hidden = hidden;
  q.slots = peers->slot_base[peers->rank];
  for (int k = 0; k < peers->world; ++k) q.dst[k] = peers->grad_base[k];
  const int64_t vecs = rows * (hidden / 8);
  const int grid = static_cast<int>(std::min<int64_t>(cdiv(vecs, 256), ctas > 0 ? ctas : 2 * num_sms()));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  count_launch();
  if (dtype == ORDA_BF16) peer_reduce_broadcast_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(q);
  else peer_reduce_broadcast_kernel<__half><<<grid, 256, 0, s>>>(q);
  return cudaPeekAtLastError() == cudaSuccess ? ORDA_OK : ORDA_ERR_CUDA;
}

// ---------------------------------------------------------------- vocab-sharded phases
size_t orda_shard_workspace_bytes(const orda_distill_args_t* args) {
  if (check_args(args) != ORDA_OK) return 0;
  return make_plan(args, args->n_rows, false).total;
}

int32_t orda_shard_forward(const orda_distill_args_t* args, void* workspace, size_t workspace_bytes,
                           float* row_stats, void* stream) {
  int rc = check_args(args);
  if (rc) return rc;
  const Plan P = make_plan(args, args->n_rows, false);
  if ((rc = check_operands(args, P))) return rc;
  if (!workspace || workspace_bytes < P.total || !row_stats) return ORDA_ERR_WORKSPACE;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const ChunkPtrs c = chunk_ptrs(args, 0, args->n_rows);
  switch (args->compute_dtype) {
    case ORDA_BF16: rc = forward_tc<__nv_bfloat16>(args, P, ws, c, s); if (!rc) rc = row_phases<__nv_bfloat16>(args, P, ws, c, s, true, false, nullptr, nullptr); break;
    case ORDA_F16: rc = forward_tc<__half>(args, P, ws, c, s); if (!rc) rc = row_phases<__half>(args, P, ws, c, s, true, false, nullptr, nullptr); break;
    default: rc = forward_f32(args, P, ws, c, s); if (!rc) rc = row_phases<float>(args, P, ws, c, s, true, false, nullptr, nullptr); break;
  }
  if (rc) return rc;
  cudaMemcpyAsync(row_stats, ws + P.off_row_stats, sizeof(float) * kRowStats * args->n_rows, cudaMemcpyDeviceToDevice, s);
  return cudaPeekAtLastError() == cudaSuccess ? ORDA_OK : ORDA_ERR_CUDA;
}

int32_t orda_merge_row_stats(const float* gathered, int32_t world, int64_t n_rows, float* row_stats, void* stream) {
  if (!gathered || !row_stats || world < 1 || n_rows <= 0) return ORDA_ERR_INVALID_ARGUMENT;
  const int grid = static_cast<int>(std::min<int64_t>(cdiv(n_rows, 256), 65535));
  count_launch();
  merge_records_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(gathered, world, n_rows, row_stats);
  return cudaPeekAtLastError() == cudaSuccess ? ORDA_OK : ORDA_ERR_CUDA;
}

int32_t orda_shard_jsd_partials(const orda_distill_args_t* args, void* workspace, size_t workspace_bytes,
                                const float* row_stats, float* row_sums, void* stream) {
  int rc = check_args(args);
  if (rc) return rc;
  const Plan P = make_plan(args, args->n_rows, false);
  if (!workspace || workspace_bytes < P.total || !row_stats || !row_sums) return ORDA_ERR_WORKSPACE;
  if (!P.jsd) return ORDA_OK;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const ChunkPtrs c = chunk_ptrs(args, 0, args->n_rows);
  RowParams r = row_params(args, P, ws, c);
  r.row_stats = const_cast<float*>(row_stats);
  const int grid = static_cast<int>(std::min<int64_t>(cdiv(c.rows, 8), 16 * num_sms()));
  count_launch();
  switch (args->compute_dtype) {
    case ORDA_BF16: jsd_sweep_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(r, row_sums); break;
    case ORDA_F16: jsd_sweep_kernel<__half><<<grid, 256, 0, s>>>(r, row_sums); break;
    default: jsd_sweep_kernel<float><<<grid, 256, 0, s>>>(r, row_sums); break;
  }
  return cudaPeekAtLastError() == cudaSuccess ? ORDA_OK : ORDA_ERR_CUDA;
}

int32_t orda_shard_backward(const orda_distill_args_t* args, void* workspace, size_t workspace_bytes,
                            const float* row_stats, const float* row_sums, void* stream) {
  int rc = check_args(args);
  if (rc) return rc;
  const Plan P = make_plan(args, args->n_rows, false);
  if ((rc = check_operands(args, P))) return rc;
  if (!workspace || workspace_bytes < P.total || !row_stats) return ORDA_ERR_WORKSPACE;
  if (P.jsd && !row_sums) return ORDA_ERR_INVALID_ARGUMENT;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const ChunkPtrs c = chunk_ptrs(args, 0, args->n_rows);
  if (args->grads_include_mean_scale) {
    count_launch();
    mean_scale_kernel<<<1, 1024, 0, s>>>(args->labels, args->n_rows, args->ignore_index, args->reduction,
                                         args->out_reduced);
  }
  switch (args->compute_dtype) {
    case ORDA_BF16:
      rc = row_phases<__nv_bfloat16>(args, P, ws, c, s, false, true, row_stats, row_sums);
      if (!rc) rc = grad_gemms<__nv_bfloat16>(args, P, ws, c, true, s);
      break;
    case ORDA_F16:
      rc = row_phases<__half>(args, P, ws, c, s, false, true, row_stats, row_sums);
      if (!rc) rc = grad_gemms<__half>(args, P, ws, c, true, s);
      break;
    default:
      rc = row_phases<float>(args, P, ws, c, s, false, true, row_stats, row_sums);
      if (!rc) rc = grad_gemms<float>(args, P, ws, c, true, s);
      break;
  }
  if (rc) return rc;
  const float* rl = args->out_row_losses ? args->out_row_losses : reinterpret_cast<const float*>(ws + P.off_row_losses);
  count_launch();
  finalize_kernel<<<1, 1024, 0, s>>>(rl, args->n_rows, args->labels, args->n_rows, args->ignore_index,
                                     args->reduction, P.flags, args->student_ce_weight, args->teacher_ce_weight,
                                     args->kl_weight, args->out_reduced);
  return cudaPeekAtLastError() == cudaSuccess ? ORDA_OK : ORDA_ERR_CUDA;
}

// ---------------------------------------------------------------- testing hook
int32_t orda_debug_gemm(int32_t dtype, int32_t a_mn, int32_t b_mn, const void* A, int64_t lda, const void* B,
                        int64_t ldb, int64_t M, int64_t N, int64_t K, float* out, int64_t ldo, int32_t* status,
                        void* stream) {
  if (dtype != ORDA_BF16 && dtype != ORDA_F16) return ORDA_ERR_INVALID_ARGUMENT;
  TcGemmParams prm{};
  prm.status = status;
  int rc;
  if ((rc = make_operand_map(&prm.a0, dtype, A, a_mn != 0, M, K, lda, kTileRows))) return rc;
  if ((rc = make_operand_map(&prm.b0, dtype, B, b_mn != 0, N, K, ldb, 256))) return rc;
  prm.kb0 = static_cast<int32_t>(cdiv(K, kBK));
  prm.st = StoreEpiParams{out, ldo, M, N, 1, 0};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define ORDA_DBG(T, AM, BM) return launch_tc<256, AM, BM, T>(prm, M, N, s, 8)
  if (dtype == ORDA_BF16) {
    if (a_mn && b_mn) ORDA_DBG(__nv_bfloat16, true, true);
    if (a_mn) ORDA_DBG(__nv_bfloat16, true, false);
    if (b_mn) ORDA_DBG(__nv_bfloat16, false, true);
    ORDA_DBG(__nv_bfloat16, false, false);
  }
  if (a_mn && b_mn) ORDA_DBG(__half, true, true);
  if (a_mn) ORDA_DBG(__half, true, false);
  if (b_mn) ORDA_DBG(__half, false, true);
  ORDA_DBG(__half, false, false);
#undef ORDA_DBG
}

int32_t orda_debug_gemm_pair(int32_t dtype, int32_t a_mn, int32_t b_mn, const void* A, int64_t lda, const void* B,
                             int64_t ldb, int64_t M, int64_t N, int64_t K, float* out, int64_t ldo, int32_t* status,
                             void* stream) {
  if (dtype != ORDA_BF16 && dtype != ORDA_F16) return ORDA_ERR_INVALID_ARGUMENT;
  TcGemmParams prm{};
  prm.status = status;
  int rc;
  if ((rc = make_operand_map(&prm.a0, dtype, A, a_mn != 0, M, K, lda, kTileRows))) return rc;
  if ((rc = make_operand_map(&prm.b0, dtype, B, b_mn != 0, N, K, ldb, 128))) return rc;
  prm.kb0 = static_cast<int32_t>(cdiv(K, kBK));
  prm.st = StoreEpiParams{out, ldo, M, N, 1, 0};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t mt = cdiv(M, 256);
#define ORDA_DBG2(T, AM, BM) return launch_tc2<AM, BM, A_PLAIN, false, EPI_STORE, T>(prm, mt, N, s, 8)
  if (dtype == ORDA_BF16) {
    if (a_mn && b_mn) ORDA_DBG2(__nv_bfloat16, true, true);
    if (a_mn) ORDA_DBG2(__nv_bfloat16, true, false);
    if (b_mn) ORDA_DBG2(__nv_bfloat16, false, true);
    ORDA_DBG2(__nv_bfloat16, false, false);
  }
  if (a_mn && b_mn) ORDA_DBG2(__half, true, true);
  if (a_mn) ORDA_DBG2(__half, true, false);
  if (b_mn) ORDA_DBG2(__half, false, true);
  ORDA_DBG2(__half, false, false);
#undef ORDA_DBG2
}

}  // extern "C"

// ---------------------------------------------------------------- allocation-free variant
// Library-owned scratch for callers that cannot allocate device memory. Host code must not pass
// the symbol itself to a kernel (on the host it is only a stand-in); the device address is looked
// up once per device with cudaGetSymbolAddress while that device is current.
static __device__ __align__(256) uint8_t g_orda_static_ws[ORDA_STATIC_WORKSPACE_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_static_ws_mutex;
// per device: the array's device address and the context it was looked up in
void* g_static_ws_ptr[kMaxDevices] = {};
void* g_static_ws_ctx[kMaxDevices] = {};

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

// The current driver context (null if none or the entry point is unavailable).
void* current_context() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  CUcontext ctx = nullptr;
  if (fn && fn(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  return ctx;
}

// Device address of the scratch array on the current device, looked up once per device (with that
// device current) and again whenever the device's context differs from the one it was looked up in
// (a reset context reloads the module, which moves the array).
int static_ws_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return ORDA_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_static_ws_mutex);
  // cudaGetSymbolAddress makes the primary context current if needed, so it runs before the
  // context is read
  if (!g_static_ws_ptr[dev] || g_static_ws_ctx[dev] != current_context()) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_orda_static_ws) != cudaSuccess || !p) return ORDA_ERR_CUDA;
    g_static_ws_ptr[dev] = p;
    g_static_ws_ctx[dev] = current_context();
  }
  *out = g_static_ws_ptr[dev];
  return ORDA_OK;
}
}  // namespace

extern "C" int32_t orda_distill_fwdbwd_static_ws(const orda_distill_args_t* args, void* stream) {
  int rc = check_args(args);
  if (rc) return rc;
  // largest chunk (a multiple of 128 rows, or all rows) whose workspace fits in the static array
  int64_t C = args->chunk_rows > 0 ? std::min<int64_t>(args->chunk_rows, args->n_rows) : args->n_rows;
  Plan P = make_plan(args, C);
  while (P.total > ORDA_STATIC_WORKSPACE_BYTES && C > kTileRows) {
    C = std::max<int64_t>(kTileRows, (C / 2) / kTileRows * kTileRows);
    P = make_plan(args, C);
  }
  if (P.total > ORDA_STATIC_WORKSPACE_BYTES) return ORDA_ERR_WORKSPACE;
  if ((rc = check_operands(args, P))) return rc;
  void* ws = nullptr;
  if ((rc = static_ws_address(&ws))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the array keeps the previous call's contents; the label-logit slots are cleared so no row can
  // read a value left behind by an earlier call
  if (cudaMemsetAsync(static_cast<uint8_t*>(ws) + P.off_label, 0, P.off_row_stats - P.off_label, s) != cudaSuccess)
    return ORDA_ERR_CUDA;
  return dispatch_all(args, P, static_cast<uint8_t*>(ws), s);
}

// Testing hook: one thread waits on an mbarrier that nothing ever arrives at, with the library's
// bounded wait and a caller-given limit. The wait must give up, flag ORDA_ERR_TIMEOUT in *status and
// let the kernel return normally.
namespace {
__global__ void wait_timeout_kernel(int32_t* status, uint64_t limit_ns, uint64_t* waited_ns) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = static_cast<uint32_t>(__cvta_generic_to_shared(&bar));
  mbar_init(b, 1);
  fence_barrier_init();
  const uint64_t t0 = global_timer_ns();
  const bool ok = mbar_wait(b, 0, status, limit_ns);  // phase 0 never completes
  *waited_ns = ok ? 0ull : global_timer_ns() - t0;
}
}  // namespace

extern "C" int32_t orda_debug_wait_timeout(int32_t* status, uint64_t limit_ns, uint64_t* waited_ns, void* stream) {
  if (!status || !waited_ns || limit_ns == 0 || limit_ns > ORDA_WAIT_TIMEOUT_NS) return ORDA_ERR_INVALID_ARGUMENT;
  count_launch();
  wait_timeout_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(status, limit_ns, waited_ns);
  return cudaPeekAtLastError() == cudaSuccess ? ORDA_OK : ORDA_ERR_CUDA;
}

extern "C" int32_t orda_debug_gemm_profile(uint64_t* out, int32_t reset) {
  if (!out) return ORDA_ERR_INVALID_ARGUMENT;
  unsigned long long host[orda::kProfSlots][8];
  if (cudaMemcpyFromSymbol(host, orda::g_tc2_prof, sizeof(host)) != cudaSuccess) return ORDA_ERR_CUDA;
  memcpy(out, host, sizeof(host));
  if (reset) {
    memset(host, 0, sizeof(host));
    if (cudaMemcpyToSymbol(orda::g_tc2_prof, host, sizeof(host)) != cudaSuccess) return ORDA_ERR_CUDA;
  }
  return ORDA_OK;
}

extern "C" int32_t orda_debug_gemm_wide(int32_t dtype, int32_t a_mn, int32_t b_mn, const void* A, int64_t lda,
                                        const void* B, int64_t ldb, int64_t M, int64_t N, int64_t K, float* out,
                                        int64_t ldo, int32_t* status, void* stream) {
  if (dtype != ORDA_BF16 && dtype != ORDA_F16) return ORDA_ERR_INVALID_ARGUMENT;
  TcGemmParams prm{};
  prm.status = status;
  int rc;
  if ((rc = make_operand_map(&prm.a0, dtype, A, a_mn != 0, M, K, lda, kTileRows))) return rc;
  if ((rc = make_operand_map(&prm.b0, dtype, B, b_mn != 0, N, K, ldb, 128))) return rc;
  prm.kb0 = static_cast<int32_t>(cdiv(K, kBK));
  prm.st = StoreEpiParams{out, ldo, M, N, 1, 0};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t mt = cdiv(M, 512);
#define ORDA_DBGW(T, AM, BM) return launch_tc2w<AM, BM, A_PLAIN, false, EPI_STORE, T>(prm, mt, N, s, 4)
  if (dtype == ORDA_BF16) {
    if (a_mn && b_mn) ORDA_DBGW(__nv_bfloat16, true, true);
    if (a_mn) ORDA_DBGW(__nv_bfloat16, true, false);
    if (b_mn) ORDA_DBGW(__nv_bfloat16, false, true);
    ORDA_DBGW(__nv_bfloat16, false, false);
  }
  if (a_mn && b_mn) ORDA_DBGW(__half, true, true);
  if (a_mn) ORDA_DBGW(__half, true, false);
  if (b_mn) ORDA_DBGW(__half, false, true);
  ORDA_DBGW(__half, false, false);
#undef ORDA_DBGW
}
