"""Chunked torch restatement of the oracle (TEST INFRASTRUCTURE ONLY), for sizes the float64 numpy
oracle cannot run in seconds.

It computes the same losses and gradients as ``oracle.distill_oracle.distill_reference`` (which
restates the reference's ``_torch_reference``, ``src/orda_ce_kernel/api.py:274-335``, and the
gradients of its autograd Functions, ``ops/tied_teacher.py:153-186,469-495``), block by block over
rows, in float32 (or float64) on whatever device the inputs are on. On a GPU this checks the full
benchmark configurations (config 3: N=8192, H=4096, V=128256; config 4: N=16384, Hs=3584, Ht=8192,
V=151936) in about a second. ``tests/test_fp32_checker.py`` pins it to the oracle on CPU.

TF32 is switched off while it runs, so its matrix products are true fp32.
"""
from __future__ import annotations

import contextlib
import math
from dataclasses import dataclass

import torch


@dataclass
class CheckerResult:
    loss: float
    student_ce: float
    teacher_ce: float
    kl: float
    d_student_hidden: torch.Tensor | None
    d_weight: torch.Tensor | None
    d_teacher_hidden: torch.Tensor | None
    d_teacher_weight: torch.Tensor | None


@contextlib.contextmanager
def _no_tf32():
    prev = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    try:
        yield
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = prev


def _softmax_minus_onehot(z, labels, mask):
    p = torch.softmax(z, dim=-1)
    rows = torch.nonzero(mask).flatten()
    p[rows, labels[rows]] -= 1.0
    p[~mask] = 0.0
    return p


def _ce_rows(z, labels, mask):
    lse = torch.logsumexp(z, dim=-1)
    out = torch.zeros_like(lse)
    rows = torch.nonzero(mask).flatten()
    out[rows] = lse[rows] - z[rows, labels[rows]]
    return out


def _divergence(zs, zt, t, kind, beta):
    """Per-row divergence (x T^2) and its gradient w.r.t. the student logits (/ weight), as
    ``oracle.distill_oracle.divergence_rows``."""
    lps = torch.log_softmax(zs / t, dim=-1)
    lpt = torch.log_softmax(zt / t, dim=-1)
    ps, pt = lps.exp(), lpt.exp()
    if kind == "jsd" and beta == 0.0:
        kind = "forward"
    elif kind == "jsd" and beta == 1.0:
        kind = "reverse"
    if kind == "forward":
        rows = (pt * (lpt - lps)).sum(-1)
        grad = t * (ps - pt)
    elif kind == "reverse":
        a = lps - lpt
        rows = (ps * a).sum(-1)
        grad = t * ps * (a - rows[:, None])
    else:
        lm = torch.logaddexp(math.log(beta) + lpt, math.log1p(-beta) + lps)
        rows = beta * (pt * (lpt - lm)).sum(-1) + (1.0 - beta) * (ps * (lps - lm)).sum(-1)
        g = (1.0 - beta) * (lps - lm)
        grad = t * ps * (g - (ps * g).sum(-1, keepdim=True))
    return rows * (t * t), grad


def check_reference(student_hidden, weight, labels, *, mode, teacher_hidden=None, teacher_weight=None,
                    teacher_logits=None, student_ce_weight=1.0, teacher_ce_weight=None, kl_weight=0.0,
                    kl_temperature=1.0, ignore_index=-100, reduction="mean", kl_divergence="forward",
                    jsd_beta=0.5, need_teacher_hidden_grad=False, dtype=torch.float32,
                    row_block=1024) -> CheckerResult:
    """Losses and gradients of one ``distillation_loss`` call (``mode``: tied / separate /
    precomputed). Inputs are upcast to ``dtype`` block by block; the weight gradients accumulate in
    ``dtype`` over the blocks."""
    if teacher_ce_weight is None:
        teacher_ce_weight = 1.0 if mode == "tied" else 0.0
    w_t = float(teacher_ce_weight)
    dev = student_hidden.device
    n = student_hidden.shape[0]
    w = weight.to(dtype)
    wt = teacher_weight.to(dtype) if teacher_weight is not None else None
    y = labels.to(dev)
    mask_all = y != ignore_index
    denom = max(int(mask_all.sum()), 1)
    scale = 1.0 / denom if reduction == "mean" else 1.0
    need_dwt = mode == "separate" and w_t != 0.0
    need_dht = (mode == "tied" and need_teacher_hidden_grad) or need_dwt
    d_hs = torch.empty((n, w.shape[1]), dtype=dtype, device=dev)
    d_w = torch.zeros_like(w)
    d_ht = torch.empty((n, teacher_hidden.shape[1]), dtype=dtype, device=dev) if need_dht else None
    d_wt = torch.zeros_like(wt) if need_dwt else None
    sums = torch.zeros(3, dtype=torch.float64, device=dev)
    with _no_tf32(), torch.no_grad():
        for r0 in range(0, n, row_block):
            r1 = min(n, r0 + row_block)
            hs = student_hidden[r0:r1].to(dtype)
            lab = y[r0:r1]
            mask = mask_all[r0:r1]
            zs = hs @ w.t()
            ht = None
            if mode == "tied":
                ht = teacher_hidden[r0:r1].to(dtype)
                zt = ht @ w.t()
            elif mode == "separate":
                ht = teacher_hidden[r0:r1].to(dtype)
                zt = ht @ wt.t()
            elif teacher_logits is not None:
                zt = teacher_logits[r0:r1].to(dtype)
            else:
                zt = teacher_hidden[r0:r1].to(dtype) @ wt.t()
            ce_s = _ce_rows(zs, lab, mask)
            ce_t = _ce_rows(zt, lab, mask)
            kl_rows, kl_grad = _divergence(zs, zt, float(kl_temperature), kl_divergence, float(jsd_beta))
            kl_rows = torch.where(mask, kl_rows, torch.zeros_like(kl_rows))
            kl_grad[~mask] = 0.0
            sums += torch.stack([ce_s.sum(), ce_t.sum(), kl_rows.sum()]).double()
            dzs = (student_ce_weight * _softmax_minus_onehot(zs, lab, mask) + kl_weight * kl_grad) * scale
            del kl_grad
            d_hs[r0:r1] = dzs @ w
            d_w += dzs.t() @ hs
            if mode == "tied":
                dzt = w_t * _softmax_minus_onehot(zt, lab, mask) * scale
                if need_dht:
                    d_ht[r0:r1] = dzt @ w
                if w_t != 0.0:
                    d_w += dzt.t() @ ht
            elif need_dwt:
                dzt = w_t * _softmax_minus_onehot(zt, lab, mask) * scale
                d_ht[r0:r1] = dzt @ wt
                d_wt += dzt.t() @ ht
            del zs, zt, dzs
    s = sums.cpu().tolist()
    student_ce, teacher_ce, kl = s[0] * scale, (s[1] * scale if w_t != 0.0 else 0.0), s[2] * scale
    loss = student_ce_weight * student_ce + w_t * teacher_ce + kl_weight * kl
    return CheckerResult(loss, student_ce, teacher_ce, kl, d_hs, d_w, d_ht, d_wt)


def row_rel_errors(actual: torch.Tensor, expected: torch.Tensor) -> tuple[float, int]:
    """Largest per-row relative error ||a_r - e_r|| / ||e_r|| over the rows whose expected norm is
    nonzero, and the number of rows whose expected value is exactly zero but whose actual value is
    not (ignored rows must be exact zeros)."""
    a = actual.detach().to(torch.float64)
    e = expected.detach().to(torch.float64)
    en = torch.linalg.vector_norm(e, dim=1)
    dn = torch.linalg.vector_norm(a - e, dim=1)
    nz = en > 0
    worst = float((dn[nz] / en[nz]).max()) if bool(nz.any()) else 0.0
    bad_zero = int(((~nz) & (torch.linalg.vector_norm(a, dim=1) > 0)).sum())
    return worst, bad_zero


def norm_rel_error(actual: torch.Tensor, expected: torch.Tensor) -> float:
    a = actual.detach().to(torch.float64)
    e = expected.detach().to(torch.float64)
    return float(torch.linalg.vector_norm(a - e) / torch.linalg.vector_norm(e).clamp(min=1e-300))
