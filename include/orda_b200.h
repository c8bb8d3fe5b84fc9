/*
 * orda_b200.h - C ABI of the B200 (sm_100a) fused linear-cross-entropy + distillation loss.
 *
 * The library replaces the GPU work of the reference's per-mode autograd Functions
 * (hiwuhgds-pixel/ORDA-Knowledge-Distillation-Kernel):
 *   - TiedCEFunction.forward            src/orda_ce_kernel/ops/tied_teacher.py:287-527
 *   - SeparateStudentCEFunction.forward src/orda_ce_kernel/ops/separate_teacher.py:488-725
 *   - SeparateFullCEFunction.forward    src/orda_ce_kernel/ops/separate_teacher.py:743-1001
 *   - PrecomputedCEFunction.forward     src/orda_ce_kernel/ops/precomputed_teacher.py:239-486
 * i.e. the chunk loop "logits GEMM -> Triton row kernel -> dH GEMM -> dW GEMM" plus the loss
 * reduction (tied_teacher.py:367-516). Backward stays a scalar rescale done by the caller
 * (tied_teacher.py:529-564).
 *
 * Conventions
 *   - All pointers are device pointers unless stated; the caller owns every buffer.
 *   - The library never allocates device memory and never synchronises the stream; every
 *     entry point only enqueues work on `stream` (a cudaStream_t passed as void*).
 *   - 16-bit operands (student/teacher hidden and weights) share one dtype (compute_dtype);
 *     their row strides must be multiples of 8 elements and their base addresses 16-byte
 *     aligned (TMA requirements). ORDA_ERR_ALIGNMENT is returned otherwise.
 *   - Errors detected on the device (label out of range with validate_labels, a pipeline wait
 *     that timed out) are written to *device_status (int32, device memory, zero on entry); the
 *     caller reads it whenever it chooses. Kernels never trap.
 *   - Thread-safe and re-entrant. Global state: a per-process cache of the driver entry points
 *     used to encode TMA descriptors, an atomic launch counter, and one exception, the scratch
 *     array of orda_distill_fwdbwd_static_ws (32 MiB of device memory per GPU, shared by every
 *     call of that entry point; see its comment). No other entry point touches that array.
 */
#ifndef ORDA_B200_H_
#define ORDA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ORDA_ABI_VERSION 1

/* status codes */
#define ORDA_OK 0
#define ORDA_ERR_INVALID_ARGUMENT 1
#define ORDA_ERR_ALIGNMENT 2
#define ORDA_ERR_WORKSPACE 3
#define ORDA_ERR_UNSUPPORTED 4
#define ORDA_ERR_CUDA 5
#define ORDA_ERR_TIMEOUT 6      /* device: an mbarrier wait exceeded its bound            */
#define ORDA_ERR_LABEL_RANGE 7  /* device: a label outside [0, V) that is not ignore_index */
#define ORDA_ERR_NO_DEVICE 8

/* element types */
#define ORDA_F32 0
#define ORDA_F16 1
#define ORDA_BF16 2

/* teacher modes (api.py:126-135) */
#define ORDA_TEACHER_TIED 0            /* TiedTeacher: teacher hidden through the student lm_head      */
#define ORDA_TEACHER_SEPARATE 1        /* SeparateTeacher: own hidden and lm_head                       */
#define ORDA_TEACHER_LOGITS 2          /* PrecomputedTeacher(logits=...)                                */
#define ORDA_TEACHER_HIDDEN 3          /* PrecomputedTeacher(teacher_hidden, teacher_weight), no grads  */

/* distillation divergence (reference: forward only) */
#define ORDA_DIV_FORWARD 0  /* T^2 KL(p_t || p_s) - the reference's only variant                    */
#define ORDA_DIV_REVERSE 1  /* T^2 KL(p_s || p_t)                                                   */
#define ORDA_DIV_JSD 2      /* T^2 [b KL(p_t||m) + (1-b) KL(p_s||m)], m = b p_t + (1-b) p_s;
                               b = 0 -> forward KL, b = 1 -> reverse KL                             */

#define ORDA_REDUCTION_MEAN 0
#define ORDA_REDUCTION_SUM 1

/* out_reduced[] slots */
#define ORDA_OUT_LOSS 0
#define ORDA_OUT_STUDENT_CE 1
#define ORDA_OUT_TEACHER_CE 2
#define ORDA_OUT_KL 3
#define ORDA_OUT_MEAN_SCALE 4  /* 1/max(count,1) for mean, 1 for sum (tied_teacher.py:503-513)      */
#define ORDA_OUT_SUM_STUDENT_CE 5
#define ORDA_OUT_SUM_TEACHER_CE 6
#define ORDA_OUT_SUM_KL 7
#define ORDA_OUT_COUNT 8       /* number of rows whose label != ignore_index                         */
#define ORDA_OUT_SLOTS 9

typedef struct orda_distill_args {
  int32_t abi_version;      /* = ORDA_ABI_VERSION */
  int32_t teacher_mode;     /* ORDA_TEACHER_* */
  int32_t compute_dtype;    /* ORDA_F32 / ORDA_F16 / ORDA_BF16: dtype of hidden + weights            */
  int32_t teacher_logits_dtype; /* dtype of teacher_logits (ORDA_TEACHER_LOGITS only)                */

  int64_t n_rows;           /* BT                                                                    */
  int64_t hidden;           /* student hidden size H                                                 */
  int64_t teacher_hidden;   /* teacher hidden size (tied: == hidden)                                 */
  int64_t vocab;            /* vocab rows held by this call's weight(s)                              */
  int64_t vocab_offset;     /* first vocab id of `weight` (vocab sharding; 0 on one GPU)             */
  int64_t vocab_total;      /* full vocab size (labels index it); == vocab on one GPU                 */

  const void* student_hidden; int64_t ld_student_hidden;   /* [n_rows, hidden]                      */
  const void* weight;         int64_t ld_weight;           /* [vocab, hidden]                       */
  const void* teacher_hidden_ptr; int64_t ld_teacher_hidden; /* [n_rows, teacher_hidden] or NULL    */
  const void* teacher_weight; int64_t ld_teacher_weight;   /* [vocab, teacher_hidden] or NULL       */
  const void* teacher_logits; int64_t ld_teacher_logits;   /* [n_rows, vocab] or NULL               */
  const int64_t* labels;                                   /* [n_rows]                              */

  float student_ce_weight;
  float teacher_ce_weight;  /* already resolved (tied default 1.0, others 0.0: api.py:138-141)       */
  float kl_weight;
  float kl_temperature;
  float jsd_beta;
  int32_t divergence;       /* ORDA_DIV_* */
  int64_t ignore_index;
  int32_t reduction;        /* ORDA_REDUCTION_* */
  int32_t validate_labels;  /* flag out-of-range labels in *device_status (reference: debug profile) */

  int32_t need_grad_student_hidden;
  int32_t need_grad_weight;
  int32_t need_grad_teacher_hidden;
  int32_t need_grad_teacher_weight;
  int64_t chunk_rows;       /* rows per internal chunk; 0 = library default                          */

  /* outputs (device). Gradients are of the UNSCALED loss sum terms: the caller multiplies them by
     grad_output * out_reduced[ORDA_OUT_MEAN_SCALE] in backward, as tied_teacher.py:538-545 does. */
  float* out_reduced;           /* [ORDA_OUT_SLOTS] fp32                                             */
  float* out_row_losses;        /* optional [3, n_rows] fp32: student CE, teacher CE, divergence     */
  void* grad_student_hidden;    /* [n_rows, hidden], compute dtype, row stride = hidden              */
  void* grad_weight;            /* [vocab, hidden], compute dtype or fp32 (grad_weight_fp32)          */
  void* grad_teacher_hidden;    /* [n_rows, teacher_hidden], compute dtype                           */
  void* grad_teacher_weight;    /* [vocab, teacher_hidden], compute dtype or fp32                    */
  int32_t grad_weight_fp32;     /* grad_weight / grad_teacher_weight are fp32 accumulators            */
  int32_t* device_status;       /* int32 device word, zero on entry                                   */

  /* optional instrumentation / overlap hooks (host handles; NULL = off) */
  void* const* phase_events;    /* 2*ORDA_PHASES cudaEvent_t: start/end recorded around each phase of
                                   the LAST chunk (timing of the individual kernels)                  */
  void* dweight_done_event;     /* cudaEvent_t recorded once the weight gradients are complete, so a
                                   caller can start their all-reduce on another stream                 */
  int32_t dweight_first;        /* run the dW GEMMs before the dH GEMMs (overlap the dW all-reduce)  */
  int32_t grads_include_mean_scale; /* 1: gradients already include out_reduced[ORDA_OUT_MEAN_SCALE]
                                   (1/count for mean), so backward only multiplies by grad_output     */
  int32_t overlap_reserve_sms;  /* with dweight_first: the dHidden GEMMs, which run while the caller's
                                   dW all-reduce runs on another stream, leave this many SMs free for
                                   the collective's kernels (0 = use every SM)                        */
} orda_distill_args_t;

/* phases bracketed by phase_events */
#define ORDA_PHASE_LOGITS 0     /* logits GEMM(s) + statistics epilogue                              */
#define ORDA_PHASE_ROWS 1       /* row merge, losses, (JSD sweep), dlogits sweep                     */
#define ORDA_PHASE_DHIDDEN 2    /* dHidden GEMM(s)                                                    */
#define ORDA_PHASE_DWEIGHT 3    /* dWeight GEMM(s)                                                    */
#define ORDA_PHASES 4

/* Version of this ABI (ORDA_ABI_VERSION). */
int32_t orda_abi_version(void);

/* sizeof(orda_distill_args_t) as compiled into the library (lets FFI callers check their layout). */
size_t orda_args_struct_size(void);

/* Number of kernels this library has launched in this process (monotonic; for launch accounting). */
uint64_t orda_kernel_launches(void);

/* In-place backward rescale of a gradient buffer: data[i] *= *scale (device fp32 scalar), skipped
 * entirely on the device when *scale == 1. dtype: ORDA_F32 / ORDA_F16 / ORDA_BF16. Replaces the
 * elementwise rescale of the reference's backward (ops/tied_teacher.py:538-545). */
int32_t orda_scale_grad(void* data, int64_t n, int32_t dtype, const float* scale, void* stream);

/* Human-readable text for a status code. */
const char* orda_status_string(int32_t status);

/* Bytes of scratch `orda_distill_fwdbwd` needs for `args` (bounded by chunk_rows x vocab).
 * Replaces the reference's per-chunk temporaries (logits chunk, loss buffers:
 * tied_teacher.py:346-358, 444-445) and its OOM-driven chunk retry (utils/dispatcher.py:244-293). */
size_t orda_distill_workspace_bytes(const orda_distill_args_t* args);

/* Fused forward + backward of the distillation loss on one GPU.
 * Replaces: TiedCEFunction.forward (ops/tied_teacher.py:287-527),
 *           SeparateStudentCEFunction.forward / SeparateFullCEFunction.forward
 *           (ops/separate_teacher.py:488-725, 743-1001),
 *           PrecomputedCEFunction.forward (ops/precomputed_teacher.py:239-486).
 * Writes out_reduced[] (loss, components, mean scale, sums, count), optional per-row losses and the
 * requested gradients; workspace must hold orda_distill_workspace_bytes(args) bytes. */
int32_t orda_distill_fwdbwd(const orda_distill_args_t* args, void* workspace, size_t workspace_bytes,
                            void* stream);

/* Size of the library-owned scratch used by orda_distill_fwdbwd_static_ws (32 MiB per GPU). */
#define ORDA_STATIC_WORKSPACE_BYTES (32u << 20)

/* No counterpart in the reference. Same computation and outputs as orda_distill_fwdbwd, for callers
 * that cannot allocate device memory themselves (for example a host runtime that hands out only
 * pre-registered input/output buffers, or code running where a cudaMalloc would synchronise or is
 * forbidden). The scratch lives in a fixed 32 MiB array inside the library, which every GPU that loads
 * the library keeps until the process exits; the call allocates nothing. Rows are processed in
 * chunks small enough to fit; if even one 128-row chunk (or the per-row loss buffer, 3 x n_rows
 * floats) does not fit, it returns ORDA_ERR_WORKSPACE and launches nothing. The first call on each
 * device looks up the array's device address (make it before any stream capture); the address is
 * cached per device together with the CUDA context it was looked up in, and looked up again if the
 * device's context changed (for example after cudaDeviceReset). All calls share
 * the one array: calls that overlap on the GPU (other streams, other host threads) race and must be
 * serialised by the caller. */
int32_t orda_distill_fwdbwd_static_ws(const orda_distill_args_t* args, void* stream);

/* ---- token-sharded multi-GPU: lm_head gradient exchanged over peer memory ----
 * The reference has no multi-GPU code; this replaces the all-reduce of the lm_head gradient that
 * data parallelism needs after TiedCEFunction / SeparateFullCEFunction (ops/tied_teacher.py:481-495,
 * ops/separate_teacher.py:926-934 compute it per process). Every rank owns one slab of lm_head rows:
 * rows [r * slab_rows, (r + 1) * slab_rows) belong to rank r. Each rank exposes two buffers mapped
 * into every peer's address space (CUDA IPC / symmetric memory, set up by the caller):
 *   slots: [world * slab_rows, hidden] in the compute dtype - slot k receives rank k's partial
 *          gradient of this rank's slab;
 *   grad:  [vocab, hidden] in the compute dtype - the summed lm_head gradient, written by every owner.
 * No kernel of this library waits on another GPU: the caller orders the phases with its own
 * collective (e.g. a one-element NCCL all-reduce) between them. */
#define ORDA_MAX_PEERS 8

typedef struct orda_peer_slots {
  int32_t world;                        /* ranks (1..ORDA_MAX_PEERS)                                 */
  int32_t rank;                         /* this rank                                                 */
  int64_t slab_rows;                    /* lm_head rows owned per rank (>= ceil(vocab / world); a
                                           multiple of 512 lets the dW epilogue store by TMA)        */
  void* slot_base[ORDA_MAX_PEERS];      /* device address of rank k's slots buffer, as mapped here   */
  void* grad_base[ORDA_MAX_PEERS];      /* device address of rank k's grad buffer, as mapped here    */
} orda_peer_slots_t;

/* Mapping a buffer of one process into another process on the same node (plain CUDA IPC peer
 * mappings, no multicast objects), for the slots / grad buffers above. `ptr` may point anywhere
 * inside a device allocation (e.g. one made by a caching allocator); the handle carries the offset. */
typedef struct orda_ipc_handle {
  uint8_t handle[64];  /* cudaIpcMemHandle_t of the allocation that contains ptr */
  uint64_t offset;     /* ptr - allocation base                                  */
} orda_ipc_handle_t;

/* Describes `ptr` (device memory of the current device) for orda_ipc_import in another process. */
int32_t orda_ipc_export(const void* ptr, orda_ipc_handle_t* out);

/* Maps the exporter's allocation into this process (peer access over NVLink) and returns the
 * address of the exported pointer. Close it with orda_ipc_close when done. */
int32_t orda_ipc_import(const orda_ipc_handle_t* handle, void** ptr_out);

/* Unmaps an address returned by orda_ipc_import (with the handle it came from). */
int32_t orda_ipc_close(void* ptr, const orda_ipc_handle_t* handle);

/* orda_distill_fwdbwd with the student lm_head gradient routed to its owners: the dW GEMM of the
 * last row chunk stores row v of this rank's partial gradient into slot `rank` of the owner of v
 * (peer stores from the GEMM epilogue, overlapped with the GEMM's remaining tiles). Earlier chunks
 * accumulate in args->grad_weight, which the last chunk adds in; grad_weight may be this rank's own
 * grad buffer. 16-bit compute dtype, grad_weight_fp32 = 0, vocab_offset = 0. The routed stores are
 * complete and visible system-wide when the kernel that made them has finished (dweight_done_event
 * marks that point on `stream`). */
int32_t orda_distill_fwdbwd_peer(const orda_distill_args_t* args, void* workspace, size_t workspace_bytes,
                                 const orda_peer_slots_t* peers, void* stream);

/* Phase 2, after every rank's routed dW GEMM has finished (the caller's barrier): this rank sums
 * the `world` slots of its slab (fp32 accumulation, one rounding) and writes the sum into the grad
 * buffer of every rank (peer stores), so each grad buffer ends up holding the summed [vocab, hidden]
 * gradient once all ranks have run this (the caller's second barrier). dtype: ORDA_BF16 / ORDA_F16.
 * `ctas` bounds the grid (0 = library default) so the kernel can run beside a GEMM on another
 * stream. */
int32_t orda_peer_reduce_broadcast(const orda_peer_slots_t* peers, int64_t vocab, int64_t hidden, int32_t dtype,
                                   int32_t ctas, void* stream);

/* ---- vocab-sharded multi-GPU building blocks (one call per rank; NCCL stays with the caller) ----
 * Per-row statistics record exchanged between ranks: ORDA_ROW_STATS floats per row. */
#define ORDA_ROW_STATS 16

/* Bytes of scratch the shard entry points need (same layout as orda_distill_workspace_bytes with
 * chunk_rows = n_rows). */
size_t orda_shard_workspace_bytes(const orda_distill_args_t* args);

/* Phase 1: logits GEMMs over this rank's vocab shard with the fused statistics epilogue, then the
 * per-row merge over the shard. Writes row_stats[n_rows][ORDA_ROW_STATS] (device).
 * Replaces the stats half of the reference row kernels (ops/tied_teacher.py:70-141). */
int32_t orda_shard_forward(const orda_distill_args_t* args, void* workspace, size_t workspace_bytes,
                           float* row_stats, void* stream);

/* Merge `world` gathered records gathered[world][n_rows][ORDA_ROW_STATS] into row_stats (LSE merge). */
int32_t orda_merge_row_stats(const float* gathered, int32_t world, int64_t n_rows, float* row_stats,
                             void* stream);

/* Phase 1b (JSD only): per-row partial sums over this shard, row_sums[n_rows][2]; the caller sums
 * them over ranks before phase 2. */
int32_t orda_shard_jsd_partials(const orda_distill_args_t* args, void* workspace, size_t workspace_bytes,
                                const float* row_stats, float* row_sums, void* stream);

/* Phase 2: per-row losses from the global records (rank-independent), dlogits over this shard, the
 * partial dHidden (caller all-reduces it) and this shard's dW (complete, no communication).
 * Replaces the gradient half of the row kernels (ops/tied_teacher.py:143-189) and the dH / dW GEMMs
 * (tied_teacher.py:469-495). `row_sums` is the summed phase-1b output (JSD) or NULL. */
int32_t orda_shard_backward(const orda_distill_args_t* args, void* workspace, size_t workspace_bytes,
                            const float* row_stats, const float* row_sums, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ORDA_B200_H_ */
