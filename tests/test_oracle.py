"""Pins the numpy oracle to the reference's own outputs (golden fixtures from make_golden.py)."""
from __future__ import annotations

import ast
import glob
import os

import numpy as np
import pytest

from oracle.distill_oracle import KL_REVERSE, distill_reference, divergence_rows

GOLDEN = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))


def _run_oracle(d):
    meta = ast.literal_eval(str(d["meta"]))
    mode = meta.pop("mode")
    kw = dict(
        student_ce_weight=meta.get("student_ce_weight", 1.0),
        teacher_ce_weight=meta.get("teacher_ce_weight"),
        kl_weight=meta.get("kl_weight", 0.0),
        kl_temperature=meta.get("kl_temperature", 1.0),
        reduction=meta.get("reduction", "mean"),
    )
    base = dict(student_hidden=d["in_student_hidden"], weight=d["in_weight"], labels=d["in_labels"])
    if mode == "tied":
        return distill_reference(**base, mode="tied", teacher_hidden=d["in_teacher_hidden"], **kw)
    if mode == "separate":
        return distill_reference(**base, mode="separate", teacher_hidden=d["in_teacher_hidden"],
                                 teacher_weight=d["in_teacher_weight"], **kw)
    if mode == "precomputed_logits":
        return distill_reference(**base, mode="precomputed", teacher_logits=d["in_teacher_logits"], **kw)
    return distill_reference(**base, mode="precomputed", teacher_hidden=d["in_teacher_hidden"],
                             teacher_weight=d["in_teacher_weight"], **kw)


def test_golden_fixtures_present():
    assert len(GOLDEN) >= 10


@pytest.mark.parametrize("path", GOLDEN, ids=[os.path.basename(p)[:-4] for p in GOLDEN])
def test_oracle_matches_reference_golden(path):
    d = np.load(path)
    r = _run_oracle(d)
    tol = dict(rtol=1e-11, atol=1e-12)
    np.testing.assert_allclose(r.loss, d["out_loss"], **tol)
    np.testing.assert_allclose(r.student_ce, d["out_student_ce"], **tol)
    np.testing.assert_allclose(r.teacher_ce, d["out_teacher_ce"], **tol)
    np.testing.assert_allclose(r.kl, d["out_kl"], **tol)
    np.testing.assert_allclose(r.d_student_hidden, d["grad_student_hidden"], **tol)
    np.testing.assert_allclose(r.d_weight, d["grad_weight"], **tol)
    if "grad_teacher_hidden" in d:
        np.testing.assert_allclose(r.d_teacher_hidden, d["grad_teacher_hidden"], **tol)
    if "grad_teacher_weight" in d:
        np.testing.assert_allclose(r.d_teacher_weight, d["grad_teacher_weight"], **tol)


def test_reverse_kl_value_pinned_by_swapped_forward_kl():
    """Reverse KL has no reference code; its value equals the reference's forward KL with the
    student and teacher logits swapped."""
    d = np.load(os.path.join(os.path.dirname(__file__), "golden", "swapped_for_reverse_pin.npz"))
    z_model = d["in_student_hidden"] @ d["in_weight"].T
    z_given = d["in_teacher_logits"]
    mask = d["in_labels"] != -100
    rows, _ = divergence_rows(z_given, z_model, 1.5, KL_REVERSE)
    np.testing.assert_allclose(np.sum(rows[mask]), d["out_kl"], rtol=1e-11)


@pytest.mark.parametrize("kind,beta", [("reverse", 0.5), ("jsd", 0.5), ("jsd", 0.2), ("jsd", 0.0), ("jsd", 1.0)])
def test_divergence_grad_matches_finite_difference(kind, beta):
    rng = np.random.default_rng(3)
    zs = rng.standard_normal((3, 11))
    zt = rng.standard_normal((3, 11))
    t = 1.3
    rows, grad = divergence_rows(zs, zt, t, kind, beta)
    eps = 1e-6
    num = np.zeros_like(zs)
    for i in range(zs.shape[0]):
        for j in range(zs.shape[1]):
            zp = zs.copy(); zp[i, j] += eps
            zm = zs.copy(); zm[i, j] -= eps
            num[i, j] = (divergence_rows(zp, zt, t, kind, beta)[0][i] - divergence_rows(zm, zt, t, kind, beta)[0][i]) / (2 * eps)
    np.testing.assert_allclose(grad, num, rtol=1e-6, atol=1e-8)


def test_jsd_symmetry_at_half():
    rng = np.random.default_rng(4)
    a = rng.standard_normal((4, 9))
    b = rng.standard_normal((4, 9))
    r1, _ = divergence_rows(a, b, 1.0, "jsd", 0.5)
    r2, _ = divergence_rows(b, a, 1.0, "jsd", 0.5)
    np.testing.assert_allclose(r1, r2, rtol=1e-12)
