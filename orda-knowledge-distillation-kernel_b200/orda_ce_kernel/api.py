"""Public API of the B200 distillation loss - a drop-in for ``orda_ce_kernel``'s API
(``src/orda_ce_kernel/api.py``): the same teacher descriptors, config type, output tuple, argument
checks and error messages, with the GPU work running in the fused sm_100a kernels.

Differences from the reference, all deliberate:

* No CPU fallback. ``backend="auto"`` and ``backend="triton"`` both select the CUDA kernels and raise
  ``RuntimeError`` for CPU tensors; ``backend="torch"`` (the reference's CPU formula) is not part of
  this build and raises ``RuntimeError``.
* Two opt-in keywords select the divergence: ``kl_divergence`` = ``"forward"`` (default, the
  reference's only variant ``T^2 KL(p_t||p_s)``), ``"reverse"`` (``T^2 KL(p_s||p_t)``) or ``"jsd"``
  (``T^2 [b KL(p_t||m) + (1-b) KL(p_s||m)]`` with ``m = b p_t + (1-b) p_s`` and ``b = jsd_beta``;
  ``b = 0`` is forward KL and ``b = 1`` reverse KL, the TRL / Liger convention).
* ``KernelConfig.max_fused_size`` and ``autotune`` are validated and ignored (no Triton block sizes);
  chunk settings only bound the workspace, and there is no out-of-memory retry loop.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Literal, NamedTuple

import torch
from torch import nn

from ._runtime import cuda_kernels_available
from .ops._common import check_divergence
from .utils.dispatcher import dynamic_chunk
from .utils.resolver import DEFAULT_MAX_FUSED_SIZE, _is_auto_chunk_size, is_power_of_two

Reduction = Literal["mean", "sum"]
Profile = Literal["balanced", "debug"]
Backend = Literal["auto", "triton", "torch"]
Divergence = Literal["forward", "reverse", "jsd"]


# ---------------------------------------------------------------- teacher descriptors (api.py:20-52)
@dataclass(frozen=True)
class TiedTeacher:
    hidden: torch.Tensor


@dataclass(frozen=True)
class SeparateTeacher:
    hidden: torch.Tensor
    weight: torch.Tensor


@dataclass(frozen=True)
class PrecomputedTeacher:
    logits: torch.Tensor | None = None
    teacher_hidden: torch.Tensor | None = None
    teacher_weight: torch.Tensor | None = None

    def __post_init__(self):
        has_logits = self.logits is not None
        has_pair = self.teacher_hidden is not None or self.teacher_weight is not None
        if has_logits and has_pair:
            raise ValueError("PrecomputedTeacher: provide logits or (teacher_hidden, teacher_weight), not both")
        if not has_logits and not has_pair:
            raise ValueError("PrecomputedTeacher: must provide logits or (teacher_hidden, teacher_weight)")
        if has_pair and (self.teacher_hidden is None or self.teacher_weight is None):
            raise ValueError("PrecomputedTeacher: teacher_hidden and teacher_weight must both be provided")


# ---------------------------------------------------------------- config and output (api.py:55-76)
@dataclass(frozen=True)
class KernelConfig:
    fp32_grad_weight_accumulation: bool | None = None
    chunk_size: int | Literal["auto", "dynamic"] | None = None
    num_chunks: int | None = None
    max_chunks: int | None = None
    max_fused_size: int | None = None
    kl_weight: float | None = None
    kl_temperature: float | None = None
    autotune: bool | None = None

    @property
    def effective_fp32_grad_weight_accumulation(self) -> bool:
        return bool(self.fp32_grad_weight_accumulation)


class DistillationLossOutput(NamedTuple):
    loss: torch.Tensor
    student_ce: torch.Tensor
    teacher_ce: torch.Tensor
    kl: torch.Tensor


# ---------------------------------------------------------------- config resolution (api.py:79-141)
def _resolve_profile(profile: Profile) -> KernelConfig:
    if profile not in ("balanced", "debug"):
        raise ValueError(f"profile must be 'balanced' or 'debug', got {profile!r}")
    return KernelConfig(
        fp32_grad_weight_accumulation=profile == "debug",
        max_fused_size=DEFAULT_MAX_FUSED_SIZE,
        autotune=False,
    )


def _resolve_config(profile: Profile, config: KernelConfig | None) -> KernelConfig:
    base = _resolve_profile(profile)
    if config is None:
        return base

    def pick(name):
        value = getattr(config, name)
        return getattr(base, name) if value is None else value

    return KernelConfig(**{name: pick(name) for name in KernelConfig.__dataclass_fields__})


def _resolve_kl_config(config: KernelConfig, kl_weight: float, kl_temperature: float) -> tuple[float, float]:
    w = kl_weight if config.kl_weight is None else float(config.kl_weight)
    t = kl_temperature if config.kl_temperature is None else float(config.kl_temperature)
    return w, t


def _teacher_mode_and_tensors(teacher):
    if isinstance(teacher, TiedTeacher):
        return "tied", teacher.hidden, None, None
    if isinstance(teacher, SeparateTeacher):
        return "separate", teacher.hidden, teacher.weight, None
    if isinstance(teacher, PrecomputedTeacher):
        return "precomputed", teacher.teacher_hidden, teacher.teacher_weight, teacher.logits
    raise TypeError("teacher must be TiedTeacher, SeparateTeacher, or PrecomputedTeacher")


def _resolve_teacher_ce_weight(mode: str, teacher_ce_weight: float | None) -> float:
    if teacher_ce_weight is not None:
        return float(teacher_ce_weight)
    return 1.0 if mode == "tied" else 0.0


# ---------------------------------------------------------------- validation (api.py:144-265)
def _validate_public_args(*, student_hidden, weight, labels, student_ce_weight, teacher_ce_weight, kl_weight,
                          kl_temperature, reduction, backend, config: KernelConfig) -> None:
    if student_ce_weight < 0.0:
        raise ValueError(f"student_ce_weight must be >= 0.0, got {student_ce_weight}")
    if teacher_ce_weight is not None and teacher_ce_weight < 0.0:
        raise ValueError(f"teacher_ce_weight must be >= 0.0, got {teacher_ce_weight}")
    if kl_weight < 0.0:
        raise ValueError(f"kl_weight must be >= 0.0, got {kl_weight}")
    if kl_temperature <= 0.0:
        raise ValueError(f"kl_temperature must be > 0.0, got {kl_temperature}")
    if reduction not in ("mean", "sum"):
        raise ValueError(f"reduction must be 'mean' or 'sum', got {reduction!r}")
    if backend not in ("auto", "triton", "torch"):
        raise ValueError(f"backend must be 'auto', 'triton', or 'torch', got {backend!r}")
    if student_hidden.ndim != 2:
        raise ValueError(f"student_hidden must be 2D, got shape={tuple(student_hidden.shape)}")
    if weight.ndim != 2 or weight.shape[1] != student_hidden.shape[1]:
        raise ValueError(f"weight must have shape (vocab, {student_hidden.shape[1]}), got {tuple(weight.shape)}")
    if labels.shape != (student_hidden.shape[0],):
        raise ValueError(f"labels must have shape ({student_hidden.shape[0]},), got {tuple(labels.shape)}")
    if labels.dtype != torch.long:
        raise ValueError(f"labels must have dtype torch.long, got {labels.dtype}")
    if config.max_chunks is not None and config.max_chunks < 1:
        raise ValueError(f"config.max_chunks must be >= 1, got {config.max_chunks}")
    if config.num_chunks is not None and config.num_chunks < 1:
        raise ValueError(f"config.num_chunks must be >= 1, got {config.num_chunks}")
    if config.num_chunks is not None and not _is_auto_chunk_size(config.chunk_size):
        raise ValueError("config.chunk_size and config.num_chunks are mutually exclusive")
    eff_chunks = None if config.num_chunks is None else min(int(config.num_chunks), int(student_hidden.shape[0]))
    if eff_chunks is not None and config.max_chunks is not None and eff_chunks > config.max_chunks:
        raise ValueError(
            f"config.num_chunks must be <= config.max_chunks, got "
            f"num_chunks={config.num_chunks}, max_chunks={config.max_chunks}"
        )
    if config.max_fused_size < 1:
        raise ValueError(f"config.max_fused_size must be >= 1, got {config.max_fused_size}")
    if not is_power_of_two(int(config.max_fused_size)):
        raise ValueError(f"config.max_fused_size must be a power of two, got {config.max_fused_size}")


def _validate_teacher(*, mode, teacher_hidden, teacher_weight, teacher_logits, student_hidden, weight) -> None:
    bt, hidden = student_hidden.shape
    vocab = weight.shape[0]
    if mode == "tied":
        if teacher_hidden.shape != (bt, hidden):
            raise ValueError(f"TiedTeacher.hidden must have shape {(bt, hidden)}, got {tuple(teacher_hidden.shape)}")
    elif mode == "separate":
        if teacher_hidden.ndim != 2 or teacher_hidden.shape[0] != bt:
            raise ValueError(
                f"SeparateTeacher.hidden must have shape (BT, teacher_hidden_dim), got {tuple(teacher_hidden.shape)}"
            )
        if teacher_weight.shape != (vocab, teacher_hidden.shape[1]):
            raise ValueError(
                f"SeparateTeacher.weight must have shape {(vocab, teacher_hidden.shape[1])}, "
                f"got {tuple(teacher_weight.shape)}"
            )
    else:
        if teacher_logits is not None:
            if teacher_logits.shape != (bt, vocab):
                raise ValueError(
                    f"PrecomputedTeacher.logits must have shape {(bt, vocab)}, got {tuple(teacher_logits.shape)}"
                )
            if teacher_logits.requires_grad:
                raise ValueError(
                    "PrecomputedTeacher.logits must not require gradients; use SeparateTeacher "
                    "when the teacher path needs gradients"
                )
        elif teacher_hidden is not None and teacher_weight is not None:
            if teacher_hidden.ndim != 2 or teacher_hidden.shape[0] != bt:
                raise ValueError(
                    f"PrecomputedTeacher.teacher_hidden must have shape (BT, D_t), got {tuple(teacher_hidden.shape)}"
                )
            if teacher_weight.shape != (vocab, teacher_hidden.shape[1]):
                raise ValueError(
                    f"PrecomputedTeacher.teacher_weight must have shape {(vocab, teacher_hidden.shape[1])}, "
                    f"got {tuple(teacher_weight.shape)}"
                )
            if teacher_hidden.requires_grad or teacher_weight.requires_grad:
                raise ValueError("PrecomputedTeacher.teacher_hidden and teacher_weight must not require gradients")
        else:
            raise ValueError("PrecomputedTeacher requires logits or (teacher_hidden, teacher_weight)")


# ---------------------------------------------------------------- functional API (api.py:338-437)
def distillation_loss(
    student_hidden: torch.Tensor,
    weight: torch.Tensor,
    labels: torch.Tensor,
    teacher: TiedTeacher | SeparateTeacher | PrecomputedTeacher,
    *,
    student_ce_weight: float = 1.0,
    teacher_ce_weight: float | None = None,
    kl_weight: float = 0.0,
    kl_temperature: float = 1.0,
    ignore_index: int = -100,
    reduction: Reduction = "mean",
    profile: Profile = "balanced",
    backend: Backend = "auto",
    config: KernelConfig | None = None,
    kl_divergence: Divergence = "forward",
    jsd_beta: float = 0.5,
) -> DistillationLossOutput:
    """Fused linear cross-entropy + distillation loss; forward and backward run in one call and the
    returned ``loss`` back-propagates into the student (and, for teacher-CE modes, the teacher)."""
    resolved = _resolve_config(profile, config)
    eff_kl_weight, eff_kl_temperature = _resolve_kl_config(resolved, kl_weight, kl_temperature)
    _validate_public_args(
        student_hidden=student_hidden, weight=weight, labels=labels, student_ce_weight=student_ce_weight,
        teacher_ce_weight=teacher_ce_weight, kl_weight=eff_kl_weight, kl_temperature=eff_kl_temperature,
        reduction=reduction, backend=backend, config=resolved,
    )
    check_divergence(kl_divergence, jsd_beta)
    mode, teacher_hidden, teacher_weight, teacher_logits = _teacher_mode_and_tensors(teacher)
    _validate_teacher(mode=mode, teacher_hidden=teacher_hidden, teacher_weight=teacher_weight,
                      teacher_logits=teacher_logits, student_hidden=student_hidden, weight=weight)
    eff_teacher_ce = _resolve_teacher_ce_weight(mode, teacher_ce_weight)

    if mode == "precomputed" and eff_teacher_ce != 0.0:
        raise ValueError(f"backend={backend!r} with PrecomputedTeacher requires teacher_ce_weight=0.0")
    if backend == "torch":
        raise RuntimeError(
            "backend='torch' (the reference's CPU formula) is not part of this build; the distillation loss "
            "runs only in the sm_100a CUDA kernels (use backend='auto' with CUDA tensors)"
        )
    # (while torch.compile traces, the library is probed when the compiled graph first runs)
    if student_hidden.device.type != "cuda" or (not torch.compiler.is_compiling() and not cuda_kernels_available()):
        raise RuntimeError(
            f"backend={backend!r} requires CUDA tensors on a B200 (sm_100a) GPU and the built CUDA library; "
            "there is no CPU fallback"
        )

    loss, student_ce, teacher_ce, kl = dynamic_chunk(
        student_hidden, teacher_hidden, weight, labels,
        student_ce_weight=student_ce_weight, ignore_index=ignore_index, reduction=reduction,
        chunk_size=resolved.chunk_size, num_chunks=resolved.num_chunks,
        use_fp32_accum=resolved.effective_fp32_grad_weight_accumulation,
        kl_weight=eff_kl_weight, kl_temperature=eff_kl_temperature, max_chunks=resolved.max_chunks,
        max_fused_size=resolved.max_fused_size, autotune=resolved.autotune, teacher_mode=mode,
        teacher_weight=teacher_weight, logits_teacher=teacher_logits, teacher_ce_weight=eff_teacher_ce,
        validate_labels=profile == "debug", kl_divergence=kl_divergence, jsd_beta=jsd_beta,
    )
    return DistillationLossOutput(loss, student_ce, teacher_ce, kl)


# ---------------------------------------------------------------- module wrapper (api.py:440-487)
class DistillationLoss(nn.Module):
    def __init__(
        self,
        *,
        student_ce_weight: float = 1.0,
        teacher_ce_weight: float | None = None,
        kl_weight: float = 0.0,
        kl_temperature: float = 1.0,
        ignore_index: int = -100,
        reduction: Reduction = "mean",
        profile: Profile = "balanced",
        backend: Backend = "auto",
        config: KernelConfig | None = None,
        kl_divergence: Divergence = "forward",
        jsd_beta: float = 0.5,
    ) -> None:
        super().__init__()
        self.student_ce_weight = student_ce_weight
        self.teacher_ce_weight = teacher_ce_weight
        self.kl_weight = kl_weight
        self.kl_temperature = kl_temperature
        self.ignore_index = ignore_index
        self.reduction = reduction
        self.profile = profile
        self.backend = backend
        self.config = config
        self.kl_divergence = kl_divergence
        self.jsd_beta = jsd_beta

    def forward(self, student_hidden, weight, labels, teacher) -> DistillationLossOutput:
        return distillation_loss(
            student_hidden, weight, labels, teacher,
            student_ce_weight=self.student_ce_weight, teacher_ce_weight=self.teacher_ce_weight,
            kl_weight=self.kl_weight, kl_temperature=self.kl_temperature, ignore_index=self.ignore_index,
            reduction=self.reduction, profile=self.profile, backend=self.backend, config=self.config,
            kl_divergence=self.kl_divergence, jsd_beta=self.jsd_beta,
        )
