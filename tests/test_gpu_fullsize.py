"""Full-size benchmark configurations against the chunked fp32 checker (tests/fp32_checker.py,
itself pinned to the float64 oracle on CPU).

The slices in test_gpu_parity.py check the math; these run the shapes the benchmark times, so that a
defect that appears only with many k blocks, many waves of the persistent GEMMs, large TMA
coordinates or the dHidden K split at V=128256 cannot pass:

* config 3: N=8192, H=4096, V=128256, tied teacher, T=1, teacher CE 1.0, forward / reverse / JSD,
  once as a single 8192-row chunk (the bench's layout) and once with the library's default chunks;
  reference kernels ops/tied_teacher.py:367-516;
* config 4: N=16384, Hs=3584, Ht=8192, V=151936, separate teacher, reverse KL, T=1.5, 10%
  ignore_index, plus a 128-row slice of the same shape against the float64 oracle itself;
  reference kernels ops/separate_teacher.py:743-1020.

Tolerances are north_star's: losses within 1e-3 relative; gradients within 2e-2 relative, both over
the whole tensor and for the worst single row of dHidden and the worst single vocabulary row of dW.
"""
from __future__ import annotations

import pytest
import torch

from tests.fp32_checker import check_reference, norm_rel_error, row_rel_errors

pytestmark = pytest.mark.gpu

ok = pytest.importorskip("orda_ce_kernel")
from orda_ce_kernel import KernelConfig, SeparateTeacher, TiedTeacher, distillation_loss  # noqa: E402

LOSS_RTOL = 1e-3
GRAD_RTOL = 2e-2


def _gen(seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return g


def _randn(shape, seed, std=1.0):
    return (torch.randn(shape, generator=_gen(seed), device="cuda") * std).to(torch.bfloat16)


def _labels(n, v, frac, seed):
    g = _gen(seed)
    lab = torch.randint(0, v, (n,), generator=g, device="cuda")
    return lab.masked_fill(torch.rand(n, generator=g, device="cuda") < frac, -100)


def _assert_grads(name, got, ref):
    norm = norm_rel_error(got, ref)
    worst, bad_zero = row_rel_errors(got, ref)
    assert bad_zero == 0, f"{name}: {bad_zero} rows should be exactly zero"
    assert norm < GRAD_RTOL, f"{name}: tensor relative error {norm:.3e}"
    assert worst < GRAD_RTOL, f"{name}: worst row relative error {worst:.3e}"


def _assert_losses(out, ref, with_teacher_ce=True):
    for name in ("loss", "student_ce", "kl") + (("teacher_ce",) if with_teacher_ce else ()):
        a, e = float(getattr(out, name)), getattr(ref, name)
        assert abs(a - e) <= LOSS_RTOL * abs(e), f"{name}: got {a:.8g} expected {e:.8g}"


@pytest.fixture(scope="module")
def config3():
    n, h, v = 8192, 4096, 128256
    return (_randn((n, h), 301), _randn((n, h), 302), _randn((v, h), 303, std=0.02), _labels(n, v, 0.05, 304))


@pytest.mark.parametrize("div", ["forward", "reverse", "jsd"])
@pytest.mark.parametrize("chunking", ["one 8192-row chunk", "library default"])
def test_config3_full_size(config3, div, chunking):
    hs0, ht, w0, labels = config3
    hs = hs0.clone().requires_grad_(True)
    w = w0.clone().requires_grad_(True)
    cfg = KernelConfig(chunk_size=8192) if chunking.startswith("one") else None
    out = distillation_loss(hs, w, labels, TiedTeacher(ht), kl_weight=1.0, kl_temperature=1.0, kl_divergence=div,
                            jsd_beta=0.5, config=cfg)
    out.loss.backward()
    torch.cuda.synchronize()
    ref = check_reference(hs0, w0, labels, mode="tied", teacher_hidden=ht, kl_weight=1.0, kl_temperature=1.0,
                          kl_divergence=div, jsd_beta=0.5)
    _assert_losses(out, ref)
    _assert_grads("dHidden", hs.grad, ref.d_student_hidden)
    _assert_grads("dW", w.grad, ref.d_weight)


@pytest.fixture(scope="module")
def config4():
    n, hs_, ht_, v = 16384, 3584, 8192, 151936
    return (_randn((n, hs_), 401), _randn((n, ht_), 402), _randn((v, hs_), 403, std=0.02),
            _randn((v, ht_), 404, std=0.02), _labels(n, v, 0.10, 405))


def test_config4_full_size(config4):
    hs0, ht, w0, wt, labels = config4
    hs = hs0.clone().requires_grad_(True)
    w = w0.clone().requires_grad_(True)
    out = distillation_loss(hs, w, labels, SeparateTeacher(ht, wt), kl_weight=1.0, kl_temperature=1.5,
                            kl_divergence="reverse")
    out.loss.backward()
    torch.cuda.synchronize()
    ref = check_reference(hs0, w0, labels, mode="separate", teacher_hidden=ht, teacher_weight=wt, kl_weight=1.0,
                          kl_temperature=1.5, kl_divergence="reverse")
    _assert_losses(out, ref, with_teacher_ce=False)
    assert float(out.teacher_ce) == 0.0
    _assert_grads("dHidden", hs.grad, ref.d_student_hidden)
    _assert_grads("dW", w.grad, ref.d_weight)


def test_config4_shape_slice_against_oracle(config4):
    """128 rows of config 4 against the float64 numpy oracle directly (no checker in between)."""
    import numpy as np

    from oracle.distill_oracle import distill_reference

    hs_all, ht_all, w0, wt, labels_all = config4
    rows = slice(1000, 1128)
    hs = hs_all[rows].clone().requires_grad_(True)
    w = w0.clone().requires_grad_(True)
    ht, labels = ht_all[rows].clone(), labels_all[rows].clone()
    out = distillation_loss(hs, w, labels, SeparateTeacher(ht, wt), kl_weight=1.0, kl_temperature=1.5,
                            kl_divergence="reverse")
    out.loss.backward()
    f64 = lambda t: t.detach().double().cpu().numpy()  # noqa: E731
    # With teacher CE 0 a separate teacher enters only through its logits, so the oracle gets those
    # logits (the exact fp64 product of the bf16 inputs, formed on the GPU) instead of the 10 GB fp64
    # copy of the teacher lm_head.
    zt = (ht.double() @ wt.double().t()).cpu().numpy()
    ref = distill_reference(f64(hs), f64(w0), labels.cpu().numpy(), mode="precomputed", teacher_logits=zt,
                            kl_weight=1.0, kl_temperature=1.5, kl_divergence="reverse")
    _assert_losses(out, ref, with_teacher_ce=False)
    g_ref = torch.tensor(ref.d_student_hidden, device="cuda")
    _assert_grads("dHidden", hs.grad, g_ref)
    _assert_grads("dW", w.grad, torch.tensor(ref.d_weight, device="cuda"))
    assert np.isfinite(float(out.loss))
