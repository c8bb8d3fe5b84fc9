"""Pins the chunked torch checker (tests/fp32_checker.py) to the float64 oracle on CPU, so the
full-size GPU parity tests that use it inherit the oracle's pin to the reference."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.distill_oracle import distill_reference
from tests.fp32_checker import check_reference, norm_rel_error, row_rel_errors


def _case(mode, seed, n=37, h=12, ht=20, v=53):
    g = torch.Generator().manual_seed(seed)
    d = {"hs": torch.randn(n, h, generator=g, dtype=torch.float64),
         "w": torch.randn(v, h, generator=g, dtype=torch.float64) * 0.5,
         "labels": torch.randint(0, v, (n,), generator=g)}
    d["labels"][::6] = -100
    if mode == "tied":
        d["ht"] = torch.randn(n, h, generator=g, dtype=torch.float64)
    elif mode in ("separate", "precomputed_hidden"):
        d["ht"] = torch.randn(n, ht, generator=g, dtype=torch.float64)
        d["wt"] = torch.randn(v, ht, generator=g, dtype=torch.float64) * 0.5
    else:
        d["tl"] = torch.log_softmax(torch.randn(n, v, generator=g, dtype=torch.float64) * 2.0, -1)
    return d


@pytest.mark.parametrize("mode", ["tied", "separate", "precomputed_logits", "precomputed_hidden"])
@pytest.mark.parametrize("div", ["forward", "reverse", "jsd"])
def test_checker_matches_oracle(mode, div):
    d = _case(mode, seed=hash((mode, div)) % 1000)
    sep_tce = 0.6 if mode == "separate" else None
    kw = dict(student_ce_weight=0.8, teacher_ce_weight=sep_tce, kl_weight=0.45, kl_temperature=1.3,
              kl_divergence=div, jsd_beta=0.3)
    m = "precomputed" if mode.startswith("precomputed") else mode
    tens = dict(teacher_hidden=d.get("ht"), teacher_weight=d.get("wt"), teacher_logits=d.get("tl"))
    got = check_reference(d["hs"], d["w"], d["labels"], mode=m, **tens, **kw, dtype=torch.float64, row_block=8,
                          need_teacher_hidden_grad=True)
    ref = distill_reference(d["hs"].numpy(), d["w"].numpy(), d["labels"].numpy(), mode=m,
                            **{k: (None if v is None else v.numpy()) for k, v in tens.items()}, **kw)
    for name in ("loss", "student_ce", "teacher_ce", "kl"):
        assert getattr(got, name) == pytest.approx(getattr(ref, name), rel=1e-12, abs=1e-14), name
    np.testing.assert_allclose(got.d_student_hidden.numpy(), ref.d_student_hidden, rtol=1e-10, atol=1e-14)
    np.testing.assert_allclose(got.d_weight.numpy(), ref.d_weight, rtol=1e-10, atol=1e-14)
    if ref.d_teacher_hidden is not None:
        np.testing.assert_allclose(got.d_teacher_hidden.numpy(), ref.d_teacher_hidden, rtol=1e-10, atol=1e-14)
    if ref.d_teacher_weight is not None:
        np.testing.assert_allclose(got.d_teacher_weight.numpy(), ref.d_teacher_weight, rtol=1e-10, atol=1e-14)


def test_row_errors_flag_one_bad_row_that_the_norm_dilutes():
    e = torch.randn(400, 16, dtype=torch.float64)
    a = e.clone()
    a[17] *= 1.05  # one row 5% off
    assert norm_rel_error(a, e) < 5e-3
    worst, bad_zero = row_rel_errors(a, e)
    assert worst == pytest.approx(0.05, rel=1e-9) and bad_zero == 0
    e[3] = 0.0
    a[3] = 1e-9
    assert row_rel_errors(a, e)[1] == 1
