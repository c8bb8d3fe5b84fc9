"""B200-native fused linear-cross-entropy + knowledge-distillation loss (sm_100a).

Drop-in for the ``orda_ce_kernel`` API of hiwuhgds-pixel/ORDA-Knowledge-Distillation-Kernel
(``src/orda_ce_kernel/__init__.py``); the GPU work runs in ``liborda_b200.so`` (C ABI in
``include/orda_b200.h``).
"""
from .api import (
    DistillationLoss,
    DistillationLossOutput,
    KernelConfig,
    PrecomputedTeacher,
    SeparateTeacher,
    TiedTeacher,
    distillation_loss,
)
from . import _op  # noqa: F401  (registers torch.ops.orda_b200.distill_fwdbwd for torch.compile)


def is_available() -> bool:
    """True when the sm_100a CUDA kernels can run (a B200 is visible and the library loads)."""
    from ._runtime import cuda_kernels_available

    return bool(cuda_kernels_available())


__all__ = [
    "DistillationLoss",
    "DistillationLossOutput",
    "KernelConfig",
    "PrecomputedTeacher",
    "SeparateTeacher",
    "TiedTeacher",
    "distillation_loss",
    "is_available",
]
