"""``torch.ops.orda_b200.distill_fwdbwd``: the fused call as a ``torch.library`` custom op, so that
``torch.compile`` traces ``distillation_loss`` without a graph break (the reference breaks the graph at
``api.py:339`` and ``utils/dispatcher.py:156``).

The op runs the same library call as the eager path (forward and backward together) and returns the
reduced outputs plus the gradients of the loss sums, already scaled by the mean factor. Its fake
implementation gives the output shapes; its autograd formula multiplies the stored gradients by the
incoming gradient of the loss. Eager calls keep using ``FusedDistillFunction`` (which scales the stored
gradients in place); this op is selected while ``torch.compile`` traces.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _native
from ._fused import FusedSpec, launch_prepared, need_grad_flags, prepare_call


def _logical(g: torch.Tensor | None, cols: int, dtype: torch.dtype, like: torch.Tensor) -> torch.Tensor:
    """The gradient buffer as [rows, cols] in the parameter's dtype (empty when not requested)."""
    if g is None:
        return like.new_empty((0,), dtype=dtype)
    if g.shape[1] != cols:
        g = g[:, :cols]
    return g.to(dtype).contiguous()


@torch.library.custom_op("orda_b200::distill_fwdbwd", mutates_args=())
def distill_fwdbwd(student_hidden: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor,
                   teacher_hidden: Optional[torch.Tensor], teacher_weight: Optional[torch.Tensor],
                   teacher_logits: Optional[torch.Tensor], mode: str, student_ce_weight: float,
                   teacher_ce_weight: float, kl_weight: float, kl_temperature: float, ignore_index: int,
                   reduction: str, divergence: str, jsd_beta: float, chunk_rows: int, fp32_grad_weight: bool,
                   need: list[bool]) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Returns (out[ORDA_OUT_SLOTS] fp32, d student_hidden, d teacher_hidden, d weight, d teacher_weight);
    a gradient that ``need`` (hs, ht, w, wt) does not ask for is an empty tensor."""
    spec = FusedSpec(mode=mode, student_ce_weight=student_ce_weight, teacher_ce_weight=teacher_ce_weight,
                     kl_weight=kl_weight, kl_temperature=kl_temperature, ignore_index=ignore_index,
                     reduction=reduction, divergence=divergence, jsd_beta=jsd_beta, chunk_rows=chunk_rows,
                     fp32_grad_weight=fp32_grad_weight)
    pr = prepare_call(student_hidden, teacher_hidden, weight, teacher_weight, labels, teacher_logits, spec,
                      need=list(need))
    launch_prepared(pr, spec)
    h, h_t = student_hidden.shape[1], pr.h_t
    return (pr.out.clone(),
            _logical(pr.g_hs, h, student_hidden.dtype, student_hidden),
            _logical(pr.g_ht, h_t, teacher_hidden.dtype if teacher_hidden is not None else student_hidden.dtype,
                     student_hidden),
            _logical(pr.g_w, h, weight.dtype, weight),
            _logical(pr.g_wt, h_t, teacher_weight.dtype if teacher_weight is not None else weight.dtype, weight))


@distill_fwdbwd.register_fake
def _(student_hidden, weight, labels, teacher_hidden, teacher_weight, teacher_logits, mode, student_ce_weight,
      teacher_ce_weight, kl_weight, kl_temperature, ignore_index, reduction, divergence, jsd_beta, chunk_rows,
      fp32_grad_weight, need):
    def grad_like(t, flag):
        return t.new_empty(t.shape) if (flag and t is not None) else student_hidden.new_empty((0,))

    out = student_hidden.new_empty((_native.OUT_SLOTS,), dtype=torch.float32)
    return (out, grad_like(student_hidden, need[0]), grad_like(teacher_hidden, need[1]),
            grad_like(weight, need[2]), grad_like(teacher_weight, need[3]))


def _setup_context(ctx, inputs, output):
    _out, g_hs, g_ht, g_w, g_wt = output
    ctx.save_for_backward(g_hs, g_ht, g_w, g_wt)
    ctx.need = inputs[-1]


def _backward(ctx, d_out, _d_hs, _d_ht, _d_w, _d_wt):
    g_hs, g_ht, g_w, g_wt = ctx.saved_tensors
    go = d_out[_native.OUT_LOSS].float()

    def scale(g, flag):
        return (g.float() * go).to(g.dtype) if flag else None

    need = ctx.need
    # inputs: student_hidden, weight, labels, teacher_hidden, teacher_weight, teacher_logits, then 12 scalars
    return (scale(g_hs, need[0]), scale(g_w, need[2]), None, scale(g_ht, need[1]), scale(g_wt, need[3]), None,
            *([None] * 12))


distill_fwdbwd.register_autograd(_backward, setup_context=_setup_context)


def compiled_fused_distillation(student_hidden, teacher_hidden, weight, teacher_weight, labels, teacher_logits,
                                spec: FusedSpec):
    """Same outputs as ``FusedDistillFunction.apply`` through the custom op: (loss, student_ce,
    teacher_ce, kl), with only ``loss`` carrying gradients."""
    need = need_grad_flags(student_hidden, teacher_hidden, weight, teacher_weight, spec)
    out, *_ = torch.ops.orda_b200.distill_fwdbwd(
        student_hidden, weight, labels, teacher_hidden, teacher_weight, teacher_logits, spec.mode,
        spec.student_ce_weight, spec.teacher_ce_weight, spec.kl_weight, spec.kl_temperature, spec.ignore_index,
        spec.reduction, spec.divergence, spec.jsd_beta, spec.chunk_rows, spec.fp32_grad_weight, need)
    return (out[_native.OUT_LOSS], out[_native.OUT_STUDENT_CE].detach(), out[_native.OUT_TEACHER_CE].detach(),
            out[_native.OUT_KL].detach())
