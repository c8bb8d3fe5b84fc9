/* Host-only check of the C ABI from plain C (no Python, no GPU): the header compiles as C, the
 * library links, the argument struct size matches, the workspace of the benchmark config 3 shape is
 * bounded, and invalid arguments are rejected before anything is launched. Built and run by
 * tests/test_c_abi.py with gcc. */
#include <stdio.h>
#include <string.h>

#include "orda_b200.h"

static int fails = 0;
#define CHECK(cond, msg)                           \
  do {                                             \
    if (!(cond)) {                                 \
      fprintf(stderr, "FAIL: %s\n", msg);          \
      ++fails;                                     \
    }                                              \
  } while (0)

int main(void) {
  CHECK(orda_abi_version() == ORDA_ABI_VERSION, "ABI version");
  CHECK(orda_args_struct_size() == sizeof(orda_distill_args_t), "argument struct size");
  CHECK(strlen(orda_status_string(ORDA_ERR_WORKSPACE)) > 0, "status string");

  orda_distill_args_t a;
  memset(&a, 0, sizeof(a));
  a.abi_version = ORDA_ABI_VERSION;
  a.teacher_mode = ORDA_TEACHER_TIED;
  a.compute_dtype = ORDA_BF16;
  a.n_rows = 8192;
  a.hidden = a.teacher_hidden = 4096;
  a.vocab = a.vocab_total = 128256;
  a.student_ce_weight = a.teacher_ce_weight = a.kl_weight = 1.0f;
  a.kl_temperature = 1.0f;
  a.ignore_index = -100;
  a.reduction = ORDA_REDUCTION_MEAN;
  /* any non-null, 16-byte aligned value: nothing is dereferenced on the host */
  a.student_hidden = a.weight = a.teacher_hidden_ptr = (void*)(size_t)4096;
  a.labels = (const int64_t*)(size_t)4096;
  a.out_reduced = (float*)(size_t)4096;
  a.device_status = (int32_t*)(size_t)4096;
  a.ld_student_hidden = a.ld_weight = a.ld_teacher_hidden = 4096;
  a.need_grad_student_hidden = a.need_grad_weight = 1;
  a.grad_student_hidden = a.grad_weight = (void*)(size_t)4096;

  const size_t ws = orda_distill_workspace_bytes(&a);
  CHECK(ws > 0, "workspace bytes of config 3");
  CHECK(ws < ((size_t)5 << 30), "workspace bounded by the logits budget");

  a.kl_temperature = 0.0f; /* invalid: rejected without a launch */
  CHECK(orda_distill_fwdbwd(&a, (void*)(size_t)4096, ws, NULL) == ORDA_ERR_INVALID_ARGUMENT, "T = 0 rejected");
  a.kl_temperature = 1.0f;
  CHECK(orda_distill_fwdbwd(&a, (void*)(size_t)4096, 16, NULL) == ORDA_ERR_WORKSPACE, "small workspace rejected");

  if (fails == 0) printf("c abi ok: workspace %zu bytes\n", ws);
  return fails == 0 ? 0 : 1;
}
