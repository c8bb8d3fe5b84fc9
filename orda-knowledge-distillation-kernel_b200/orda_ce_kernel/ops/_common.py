"""Argument checks shared by the per-mode entry points (same messages as the reference ops)."""
from __future__ import annotations

import torch

from .._runtime import cuda_kernels_available
from ..utils.resolver import _is_auto_chunk_size, is_power_of_two

DIVERGENCES = ("forward", "reverse", "jsd")


def require_kernels(name: str) -> None:
    # while torch.compile traces, the custom op loads the library (and fails loudly) when the graph runs
    if torch.compiler.is_compiling():
        return
    if not cuda_kernels_available():
        raise RuntimeError(
            f"{name} requires the sm_100a CUDA library (liborda_b200.so) and a B200 GPU; "
            "there is no CPU fallback."
        )


def check_scalars(*, student_ce_weight, kl_weight, kl_temperature, teacher_ce_weight, reduction, max_chunks,
                  max_fused_size, kl_divergence, jsd_beta) -> None:
    if student_ce_weight < 0.0:
        raise ValueError(f"student_ce_weight must be >= 0.0, got {student_ce_weight}")
    if kl_weight < 0.0:
        raise ValueError(f"kl_weight must be >= 0.0, got {kl_weight}")
    if kl_temperature <= 0.0:
        raise ValueError(f"kl_temperature must be > 0.0, got {kl_temperature}")
    if teacher_ce_weight < 0.0:
        raise ValueError(f"teacher_ce_weight must be >= 0.0, got {teacher_ce_weight}")
    if reduction not in ("mean", "sum"):
        raise ValueError(f"reduction must be 'mean' or 'sum', got {reduction!r}")
    if max_chunks is not None and max_chunks < 1:
        raise ValueError(f"max_chunks must be >= 1, got {max_chunks}")
    if max_fused_size < 1:
        raise ValueError(f"max_fused_size must be >= 1, got {max_fused_size}")
    if not is_power_of_two(int(max_fused_size)):
        raise ValueError(f"max_fused_size must be a power of two, got {max_fused_size}")
    check_divergence(kl_divergence, jsd_beta)


def check_divergence(kl_divergence, jsd_beta) -> None:
    if kl_divergence not in DIVERGENCES:
        raise ValueError(f"kl_divergence must be 'forward', 'reverse', or 'jsd', got {kl_divergence!r}")
    if not (0.0 <= float(jsd_beta) <= 1.0):
        raise ValueError(f"jsd_beta must be in [0, 1], got {jsd_beta}")


def chunk_rows(chunk_size, BT: int) -> int:
    """Rows per internal chunk for the library (0 = library default)."""
    if _is_auto_chunk_size(chunk_size):
        return 0
    if int(BT) == 0:
        raise ValueError("BT (batch x sequence length) must be > 0.")
    return min(int(chunk_size), int(BT))


def check_bt(BT: int) -> None:
    if int(BT) == 0:
        raise ValueError("BT (batch x sequence length) must be > 0.")


def check_labels_host(labels: torch.Tensor, V: int, ignore_index: int) -> None:
    valid = (labels == ignore_index) | ((labels >= 0) & (labels < V))
    if not bool(valid.all()):
        bad = labels[~valid].tolist()[:5]
        raise ValueError(
            f"labels contains values outside [0, {V}) and not equal to ignore_index={ignore_index}: {bad}"
        )
