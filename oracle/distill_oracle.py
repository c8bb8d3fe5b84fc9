"""CPU oracle for the fused linear-CE + distillation loss (TEST INFRASTRUCTURE ONLY).

This module is the parity checker for the CUDA path. Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s ``cpu_baseline`` / ``--impl reference`` legs may import it. The product package
never imports it, and there is no CPU fallback in the product path.

It restates, in float64 numpy, the reference's PyTorch implementation of the hot path:

* ``_torch_reference`` in ``src/orda_ce_kernel/api.py:274-335`` (losses: CE via
  ``F.cross_entropy(..., reduction="none")`` at :302-313, forward KL with T^2 at :317-322,
  masked mean/sum at :314-331, the teacher-CE zeroing rule at :333 and the weighted total at :334);
* the gradients the reference's autograd Functions produce: the in-kernel dlogits of
  ``ops/tied_teacher.py:153-186`` (``w*(softmax - onehot)`` plus ``kl_weight*T*(p_s^T - p_t^T)``,
  zero on ignored rows), the teacher-CE-only teacher dlogits of ``ops/tied_teacher.py:158-163`` and
  ``ops/separate_teacher.py:265-269`` (the KL term never reaches the teacher), and the dH / dW GEMMs of
  ``ops/tied_teacher.py:469-495``, ``ops/separate_teacher.py:440-469``,
  ``ops/precomputed_teacher.py:441-457``, scaled by ``grad_output/denom`` in ``backward``
  (``ops/tied_teacher.py:538-545``).

Reverse KL and JSD have NO counterpart in the reference (parity unpinned by the reference). Their
restatement here follows the formulas:

* reverse KL:  ``T^2 * sum p_s^T (log p_s^T - log p_t^T)``; d/dz_s = ``T * p_s (a - sum p_s a)``
  with ``a = log p_s^T - log p_t^T``;
* generalised JSD (the TRL/Liger convention): ``m = beta*p_t + (1-beta)*p_s``,
  ``T^2 * [beta*KL(p_t||m) + (1-beta)*KL(p_s||m)]``; d/dz_s = ``T * p_s (g - sum p_s g)`` with
  ``g = (1-beta) log(p_s/m)``. beta == 0 is defined as forward KL and beta == 1 as reverse KL.

The reverse-KL value is partially pinned: it equals the reference's forward-KL formula with the
student and teacher logits swapped (checked in ``tests/test_oracle.py``).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

KL_FORWARD = "forward"
KL_REVERSE = "reverse"
KL_JSD = "jsd"


def _log_softmax(x: np.ndarray) -> np.ndarray:
    m = np.max(x, axis=-1, keepdims=True)
    s = x - m
    return s - np.log(np.sum(np.exp(s), axis=-1, keepdims=True))


@dataclass
class OracleResult:
    loss: float
    student_ce: float
    teacher_ce: float
    kl: float
    # per-row losses (unreduced; zero on ignored rows)
    ce_s_rows: np.ndarray
    ce_t_rows: np.ndarray
    kl_rows: np.ndarray
    # gradients of ``loss`` (None where the reference returns no gradient)
    d_student_hidden: np.ndarray | None
    d_weight: np.ndarray | None
    d_teacher_hidden: np.ndarray | None
    d_teacher_weight: np.ndarray | None
    denom: int


def _cross_entropy_rows(logits: np.ndarray, labels: np.ndarray, mask: np.ndarray) -> np.ndarray:
    """``F.cross_entropy(reduction="none", ignore_index)`` (api.py:302-313): lse - z[y], 0 if ignored."""
    n, v = logits.shape
    y = labels[mask]
    if y.size and (y.min() < 0 or y.max() >= v):
        raise IndexError(f"label out of range [0, {v}) (the reference's torch path raises here too)")
    lse = np.log(np.sum(np.exp(logits - logits.max(-1, keepdims=True)), -1)) + logits.max(-1)
    out = np.zeros(n, dtype=np.float64)
    rows = np.nonzero(mask)[0]
    out[rows] = lse[rows] - logits[rows, labels[rows]]
    return out


def _softmax_minus_onehot(logits: np.ndarray, labels: np.ndarray, mask: np.ndarray) -> np.ndarray:
    p = np.exp(_log_softmax(logits))
    rows = np.nonzero(mask)[0]
    p[rows, labels[rows]] -= 1.0
    p[~mask] = 0.0
    return p


def divergence_rows(
    z_s: np.ndarray,
    z_t: np.ndarray,
    temperature: float,
    kind: str = KL_FORWARD,
    jsd_beta: float = 0.5,
) -> tuple[np.ndarray, np.ndarray]:
    """Per-row divergence (times T^2) and its gradient w.r.t. the student logits (times 1/weight).

    Forward KL follows api.py:317-321 / ops/tied_teacher.py:182-183; reverse KL and JSD are the
    unpinned restatements described in the module docstring.
    """
    t = float(temperature)
    lps = _log_softmax(z_s / t)
    lpt = _log_softmax(z_t / t)
    ps = np.exp(lps)
    pt = np.exp(lpt)
    if kind == KL_JSD:
        beta = float(jsd_beta)
        if beta == 0.0:
            kind = KL_FORWARD
        elif beta == 1.0:
            kind = KL_REVERSE
    if kind == KL_FORWARD:
        rows = np.sum(pt * (lpt - lps), -1)
        grad = t * (ps - pt)
    elif kind == KL_REVERSE:
        a = lps - lpt
        rows = np.sum(ps * a, -1)
        r = rows[:, None]
        grad = t * ps * (a - r)
    elif kind == KL_JSD:
        beta = float(jsd_beta)
        # log m via a stable two-term logsumexp
        lm = np.logaddexp(np.log(beta) + lpt, np.log1p(-beta) + lps)
        rows = beta * np.sum(pt * (lpt - lm), -1) + (1.0 - beta) * np.sum(ps * (lps - lm), -1)
        g = (1.0 - beta) * (lps - lm)
        grad = t * ps * (g - np.sum(ps * g, -1, keepdims=True))
    else:
        raise ValueError(f"unknown divergence {kind!r}")
    return rows * (t * t), grad


def distill_reference(
    student_hidden: np.ndarray,
    weight: np.ndarray,
    labels: np.ndarray,
    *,
    mode: str,
    teacher_hidden: np.ndarray | None = None,
    teacher_weight: np.ndarray | None = None,
    teacher_logits: np.ndarray | None = None,
    student_ce_weight: float = 1.0,
    teacher_ce_weight: float | None = None,
    kl_weight: float = 0.0,
    kl_temperature: float = 1.0,
    ignore_index: int = -100,
    reduction: str = "mean",
    kl_divergence: str = KL_FORWARD,
    jsd_beta: float = 0.5,
    need_teacher_hidden_grad: bool = True,
    grad_output: float = 1.0,
) -> OracleResult:
    """Losses and gradients of ``distillation_loss`` for one call (float64).

    ``mode`` is ``"tied"``, ``"separate"`` or ``"precomputed"`` (api.py:126-135); the teacher-CE
    default follows api.py:138-141 (tied -> 1.0, others -> 0.0).
    """
    hs = np.asarray(student_hidden, dtype=np.float64)
    w = np.asarray(weight, dtype=np.float64)
    y = np.asarray(labels, dtype=np.int64)
    n = hs.shape[0]
    if teacher_ce_weight is None:
        teacher_ce_weight = 1.0 if mode == "tied" else 0.0
    w_t = float(teacher_ce_weight)

    z_s = hs @ w.T
    ht = wt = None
    if mode == "tied":
        ht = np.asarray(teacher_hidden, dtype=np.float64)
        z_t = ht @ w.T
    elif mode == "separate":
        ht = np.asarray(teacher_hidden, dtype=np.float64)
        wt = np.asarray(teacher_weight, dtype=np.float64)
        z_t = ht @ wt.T
    elif mode == "precomputed":
        if teacher_logits is not None:
            z_t = np.asarray(teacher_logits, dtype=np.float64)
        else:
            z_t = np.asarray(teacher_hidden, dtype=np.float64) @ np.asarray(teacher_weight, dtype=np.float64).T
    else:
        raise ValueError(f"unknown mode {mode!r}")

    mask = y != ignore_index
    denom = max(int(mask.sum()), 1)
    ce_s = _cross_entropy_rows(z_s, y, mask)
    ce_t = _cross_entropy_rows(z_t, y, mask)
    kl_rows, kl_grad = divergence_rows(z_s, z_t, kl_temperature, kl_divergence, jsd_beta)
    kl_rows = np.where(mask, kl_rows, 0.0)
    kl_grad[~mask] = 0.0

    scale = 1.0 / denom if reduction == "mean" else 1.0
    if reduction not in ("mean", "sum"):
        raise ValueError(f"reduction must be 'mean' or 'sum', got {reduction!r}")
    student_ce = ce_s.sum() * scale
    teacher_ce = ce_t.sum() * scale if w_t != 0.0 else 0.0
    kl = kl_rows.sum() * scale
    loss = student_ce_weight * student_ce + w_t * teacher_ce + kl_weight * kl

    g = grad_output * scale
    dz_s = (student_ce_weight * _softmax_minus_onehot(z_s, y, mask) + kl_weight * kl_grad) * g
    d_hs = dz_s @ w
    d_w = dz_s.T @ hs
    d_ht = d_wt = None
    if mode == "tied":
        dz_t = w_t * _softmax_minus_onehot(z_t, y, mask) * g
        if need_teacher_hidden_grad:
            d_ht = dz_t @ w  # exact zeros when teacher_ce_weight == 0 (tied_teacher.py:478-479)
        d_w = d_w + dz_t.T @ ht
    elif mode == "separate" and w_t != 0.0:
        dz_t = w_t * _softmax_minus_onehot(z_t, y, mask) * g
        d_ht = dz_t @ wt
        d_wt = dz_t.T @ ht

    return OracleResult(
        loss=float(loss),
        student_ce=float(student_ce),
        teacher_ce=float(teacher_ce),
        kl=float(kl),
        ce_s_rows=ce_s,
        ce_t_rows=ce_t if w_t != 0.0 else np.zeros_like(ce_t),
        kl_rows=kl_rows,
        d_student_hidden=d_hs,
        d_weight=d_w,
        d_teacher_hidden=d_ht,
        d_teacher_weight=d_wt,
        denom=denom,
    )


def synthetic_case(
    *,
    n: int,
    h: int,
    v: int,
    ht: int | None = None,
    seed: int = 0,
    ignore_frac: float = 0.05,
    ignore_index: int = -100,
    w_std: float = 0.02,
    teacher_logit_std: float | None = None,
) -> dict:
    """Seeded synthetic inputs with the benchmark configs' distributions (hidden ~ N(0,1), W ~ N(0, w_std),
    labels uniform with a fraction set to ignore_index, teacher logits ~ N(0, s) -> log_softmax)."""
    rng = np.random.default_rng(seed)
    out = {
        "student_hidden": rng.standard_normal((n, h), dtype=np.float32),
        "weight": (rng.standard_normal((v, h), dtype=np.float32) * w_std).astype(np.float32),
    }
    labels = rng.integers(0, v, size=n, dtype=np.int64)
    k = int(round(ignore_frac * n))
    if k:
        labels[rng.choice(n, size=k, replace=False)] = ignore_index
    out["labels"] = labels
    if ht is not None:
        out["teacher_hidden"] = rng.standard_normal((n, ht), dtype=np.float32)
        out["teacher_weight"] = (rng.standard_normal((v, ht), dtype=np.float32) * w_std).astype(np.float32)
    if teacher_logit_std is not None:
        t = rng.standard_normal((n, v)) * teacher_logit_std
        out["teacher_logits"] = _log_softmax(t).astype(np.float32)
    return out
