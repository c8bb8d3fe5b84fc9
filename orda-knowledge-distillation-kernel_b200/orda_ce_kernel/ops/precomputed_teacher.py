"""Precomputed-teacher entry point: teacher logits given, or teacher (hidden, weight) recomputed
without gradients.

Signature and checks of ``precomputed_distillation_loss``
(``src/orda_ce_kernel/ops/precomputed_teacher.py:527-651``). Teacher logits of any float dtype are
read directly by the kernels (fp32 teacher log-probs are not rounded to the compute dtype first, which
the reference does at ``precomputed_teacher.py:342-348``).
"""
from __future__ import annotations

import torch

from .._fused import FusedSpec, fused_distillation
from ..utils.resolver import DEFAULT_MAX_FUSED_SIZE
from ._common import check_bt, check_labels_host, check_scalars, chunk_rows, require_kernels


def precomputed_distillation_loss(
    student_hidden: torch.Tensor,
    weight: torch.Tensor,
    logits_teacher: torch.Tensor | None = None,
    labels: torch.Tensor = None,
    student_ce_weight: float = 1.0,
    ignore_index: int = -100,
    reduction: str = "mean",
    chunk_size: str | int | None = None,
    use_fp32_accum: bool | None = None,
    kl_weight: float = 0.0,
    kl_temperature: float = 1.0,
    teacher_ce_weight: float | None = None,
    max_chunks: int | None = None,
    max_fused_size: int = DEFAULT_MAX_FUSED_SIZE,
    autotune: bool = False,
    teacher_hidden: torch.Tensor | None = None,
    teacher_weight: torch.Tensor | None = None,
    validate_labels: bool = True,
    *,
    kl_divergence: str = "forward",
    jsd_beta: float = 0.5,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    tce = 0.0 if teacher_ce_weight is None else float(teacher_ce_weight)
    require_kernels("precomputed_distillation_loss")
    if student_hidden.ndim != 2:
        raise ValueError(f"student_hidden must be 2D, got shape={tuple(student_hidden.shape)}")
    BT, H = student_hidden.shape
    device = student_hidden.device
    if weight.ndim != 2 or weight.shape[1] != H:
        raise ValueError(f"weight must have shape (V, {H}), got {tuple(weight.shape)}")
    V = weight.shape[0]
    has_hidden_weight = teacher_hidden is not None and teacher_weight is not None
    if logits_teacher is not None:
        if logits_teacher.shape != (BT, V):
            raise ValueError(f"logits_teacher must have shape ({BT}, {V}), got {tuple(logits_teacher.shape)}")
        if logits_teacher.requires_grad:
            raise ValueError(
                "precomputed_distillation_loss requires logits_teacher without gradients; "
                "use SeparateTeacher when the teacher path needs gradients"
            )
    elif has_hidden_weight:
        if teacher_hidden.ndim != 2 or teacher_hidden.shape[0] != BT:
            raise ValueError(f"teacher_hidden must have shape (BT, D_t), got {tuple(teacher_hidden.shape)}")
        if teacher_weight.shape != (V, teacher_hidden.shape[1]):
            raise ValueError(
                f"teacher_weight must have shape ({V}, {teacher_hidden.shape[1]}), got {tuple(teacher_weight.shape)}"
            )
        if teacher_hidden.requires_grad or teacher_weight.requires_grad:
            raise ValueError("teacher_hidden and teacher_weight must not require gradients")
    else:
        raise ValueError("precomputed_distillation_loss requires logits_teacher or (teacher_hidden, teacher_weight)")
    if labels is None:
        raise ValueError("labels is required")
    if labels.shape != (BT,):
        raise ValueError(f"labels must have shape ({BT},), got {tuple(labels.shape)}")
    if labels.dtype != torch.long:
        raise ValueError(f"labels must have dtype torch.long, got {labels.dtype}")
    if tce != 0.0:
        raise ValueError("precomputed_distillation_loss requires teacher_ce_weight=0.0")
    check_scalars(student_ce_weight=student_ce_weight, kl_weight=kl_weight, kl_temperature=kl_temperature,
                  teacher_ce_weight=tce, reduction=reduction, max_chunks=max_chunks,
                  max_fused_size=max_fused_size, kl_divergence=kl_divergence, jsd_beta=jsd_beta)
    if device.type != "cuda":
        raise ValueError(f"tensors must be CUDA/HIP tensors, got device={device}")
    others = [labels, weight] + ([logits_teacher] if logits_teacher is not None else []) + (
        [teacher_hidden, teacher_weight] if teacher_hidden is not None else [])
    if any(t.device != device for t in others):
        raise ValueError("all tensors must be on the same device as student_hidden")
    check_bt(BT)
    if validate_labels:
        check_labels_host(labels, V, ignore_index)
    mode = "precomputed_logits" if logits_teacher is not None else "precomputed_hidden"
    spec = FusedSpec(
        mode=mode, student_ce_weight=float(student_ce_weight), teacher_ce_weight=0.0,
        kl_weight=float(kl_weight), kl_temperature=float(kl_temperature), ignore_index=int(ignore_index),
        reduction=reduction, divergence=kl_divergence, jsd_beta=float(jsd_beta),
        chunk_rows=chunk_rows(chunk_size, BT), fp32_grad_weight=bool(use_fp32_accum),
    )
    th = teacher_hidden if logits_teacher is None else None
    tw = teacher_weight if logits_teacher is None else None
    return fused_distillation(student_hidden, th, weight, tw, labels, logits_teacher, spec)
