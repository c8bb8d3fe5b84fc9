"""Separate-teacher entry point: the teacher has its own hidden states and lm_head.

Signature and checks of ``separate_distillation_loss``
(``src/orda_ce_kernel/ops/separate_teacher.py:1024-1121``). ``teacher_ce_weight > 0`` selects the
"full" variant whose teacher-CE gradients reach the teacher hidden states and weight
(``SeparateFullCEFunction``); otherwise the teacher is KL-only and receives no gradient
(``SeparateStudentCEFunction``). The divergence never back-propagates into the teacher.
"""
from __future__ import annotations

import torch

from .._fused import FusedSpec, fused_distillation
from ..utils.resolver import DEFAULT_MAX_FUSED_SIZE
from ._common import check_bt, check_labels_host, check_scalars, chunk_rows, require_kernels


def separate_distillation_loss(
    student_hidden: torch.Tensor,
    teacher_hidden: torch.Tensor | None,
    weight: torch.Tensor,
    teacher_weight: torch.Tensor | None,
    labels: torch.Tensor,
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
    validate_labels: bool = True,
    *,
    kl_divergence: str = "forward",
    jsd_beta: float = 0.5,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    tce = 0.0 if teacher_ce_weight is None else float(teacher_ce_weight)
    require_kernels("separate_distillation_loss")
    if student_hidden.ndim != 2:
        raise ValueError(f"student_hidden must be 2D, got shape={tuple(student_hidden.shape)}")
    BT, H = student_hidden.shape
    device = student_hidden.device
    if teacher_hidden is None:
        raise ValueError("separate_distillation_loss requires teacher_hidden")
    if teacher_hidden.ndim != 2 or teacher_hidden.shape[0] != BT:
        raise ValueError(f"teacher_hidden must have shape (BT, teacher_hidden_dim), got {tuple(teacher_hidden.shape)}")
    H_t = teacher_hidden.shape[1]
    if weight.ndim != 2 or weight.shape[1] != H:
        raise ValueError(f"weight must have shape (V, {H}), got {tuple(weight.shape)}")
    V = weight.shape[0]
    if teacher_weight is None:
        raise ValueError("separate_distillation_loss requires teacher_weight")
    if teacher_weight.shape != (V, H_t):
        raise ValueError(f"teacher_weight must have shape ({V}, {H_t}), got {tuple(teacher_weight.shape)}")
    if labels.shape != (BT,):
        raise ValueError(f"labels must have shape ({BT},), got {tuple(labels.shape)}")
    if labels.dtype != torch.long:
        raise ValueError(f"labels must have dtype torch.long, got {labels.dtype}")
    check_scalars(student_ce_weight=student_ce_weight, kl_weight=kl_weight, kl_temperature=kl_temperature,
                  teacher_ce_weight=tce, reduction=reduction, max_chunks=max_chunks,
                  max_fused_size=max_fused_size, kl_divergence=kl_divergence, jsd_beta=jsd_beta)
    if device.type != "cuda":
        raise ValueError(f"tensors must be CUDA/HIP tensors, got device={device}")
    if labels.device != device or weight.device != device:
        raise ValueError("labels and weight must be on the same device as student_hidden")
    if teacher_hidden.device != device or teacher_weight.device != device:
        raise ValueError("teacher_hidden and teacher_weight must be on the same device as student_hidden")
    check_bt(BT)
    if validate_labels:
        check_labels_host(labels, V, ignore_index)
    spec = FusedSpec(
        mode="separate", student_ce_weight=float(student_ce_weight), teacher_ce_weight=tce,
        kl_weight=float(kl_weight), kl_temperature=float(kl_temperature), ignore_index=int(ignore_index),
        reduction=reduction, divergence=kl_divergence, jsd_beta=float(jsd_beta),
        chunk_rows=chunk_rows(chunk_size, BT), fp32_grad_weight=bool(use_fp32_accum),
    )
    return fused_distillation(student_hidden, teacher_hidden, weight, teacher_weight, labels, None, spec)
