"""``dynamic_chunk`` kept as the reference's dispatch entry (``src/orda_ce_kernel/utils/dispatcher.py:156-293``).

The reference picks a chunk count, runs the per-mode op and, on CUDA OOM, doubles the chunk count
and retries, remembering the working count in a locked cache. The fused kernels need only a bounded
workspace sized before launch (no large temporaries), so there is nothing to retry: this function
validates the chunk arguments exactly as the reference does and forwards to the per-mode op. The
cache functions stay importable and report an empty cache.
"""
from __future__ import annotations

import torch

from .resolver import DEFAULT_MAX_FUSED_SIZE, _is_auto_chunk_size, resolve_chunk_size


def clear_chunk_cache() -> None:
    """No-op: the fused path has no OOM-retry chunk cache."""


def get_chunk_cache() -> dict:
    return {}


def _resolve_kernel_fn(teacher_mode: str):
    if teacher_mode == "tied":
        from ..ops.tied_teacher import tied_distillation_loss

        return tied_distillation_loss
    if teacher_mode == "separate":
        from ..ops.separate_teacher import separate_distillation_loss

        return separate_distillation_loss
    if teacher_mode == "precomputed":
        from ..ops.precomputed_teacher import precomputed_distillation_loss

        return precomputed_distillation_loss
    raise ValueError(f"teacher_mode must be 'tied', 'separate', or 'precomputed', got {teacher_mode!r}")


def dynamic_chunk(
    student_hidden: torch.Tensor,
    teacher_hidden: torch.Tensor | None,
    weight: torch.Tensor,
    labels: torch.Tensor,
    student_ce_weight: float = 1.0,
    ignore_index: int = -100,
    reduction: str = "mean",
    chunk_size: str | int | None = None,
    num_chunks: int | None = None,
    use_fp32_accum: bool | None = None,
    kl_weight: float = 0.0,
    kl_temperature: float = 1.0,
    max_chunks: int | None = None,
    max_fused_size: int = DEFAULT_MAX_FUSED_SIZE,
    autotune: bool = False,
    teacher_mode: str | None = None,
    teacher_weight: torch.Tensor | None = None,
    logits_teacher: torch.Tensor | None = None,
    teacher_ce_weight: float | None = None,
    validate_labels: bool = True,
    kl_divergence: str = "forward",
    jsd_beta: float = 0.5,
):
    BT = student_hidden.shape[0]
    mode = "tied" if teacher_mode is None else teacher_mode
    kernel_fn = _resolve_kernel_fn(mode)
    if num_chunks is not None or not _is_auto_chunk_size(chunk_size):
        cs, _ = resolve_chunk_size(BT, chunk_size, max_chunks=max_chunks, num_chunks=num_chunks)
    else:
        resolve_chunk_size(BT, chunk_size, V=weight.shape[0], max_chunks=max_chunks)
        cs = None  # library default: bounded workspace
    common = dict(
        student_ce_weight=student_ce_weight,
        ignore_index=ignore_index,
        reduction=reduction,
        chunk_size=cs,
        use_fp32_accum=use_fp32_accum,
        kl_weight=kl_weight,
        kl_temperature=kl_temperature,
        teacher_ce_weight=teacher_ce_weight,
        max_chunks=max_chunks,
        max_fused_size=max_fused_size,
        autotune=autotune,
        validate_labels=validate_labels,
        kl_divergence=kl_divergence,
        jsd_beta=jsd_beta,
    )
    if mode == "tied":
        return kernel_fn(student_hidden, teacher_hidden, weight, labels, **common)
    if mode == "separate":
        return kernel_fn(student_hidden, teacher_hidden, weight, teacher_weight, labels, **common)
    return kernel_fn(
        student_hidden, weight, logits_teacher, labels,
        teacher_hidden=teacher_hidden, teacher_weight=teacher_weight, **common,
    )
