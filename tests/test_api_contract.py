"""Host-side contract of the public API (no GPU): exports, config resolution, argument errors with
the reference's messages, the chunk resolver, and the absence of any CPU fallback.
Mirrors the reference's test/unit/test_public_api.py and test_resolver.py where they apply."""
from __future__ import annotations

import pytest
import torch

import orda_ce_kernel
from orda_ce_kernel import api as public_api
from orda_ce_kernel.utils import clear_chunk_cache, get_chunk_cache, resolve_chunk_size
from orda_ce_kernel.utils.resolver import is_power_of_two


def _inputs():
    hs = torch.randn(4, 8, requires_grad=True)
    ht = torch.randn(4, 8, requires_grad=True)
    w = torch.randn(16, 8, requires_grad=True)
    labels = torch.randint(0, 16, (4,))
    return hs, ht, w, labels


def test_exports_are_the_reference_surface():
    expected = {"DistillationLoss", "DistillationLossOutput", "KernelConfig", "PrecomputedTeacher",
                "SeparateTeacher", "TiedTeacher", "distillation_loss", "is_available"}
    assert set(orda_ce_kernel.__all__) == expected
    for name in expected:
        assert hasattr(orda_ce_kernel, name)
    from orda_ce_kernel.ops import precomputed_distillation_loss, separate_distillation_loss, tied_distillation_loss  # noqa: F401
    from orda_ce_kernel.utils import DEFAULT_MAX_FUSED_SIZE, dynamic_chunk  # noqa: F401

    assert DEFAULT_MAX_FUSED_SIZE == 32768


def test_is_available_is_boolean_and_false_without_gpu():
    assert isinstance(orda_ce_kernel.is_available(), bool)
    if not torch.cuda.is_available():
        assert orda_ce_kernel.is_available() is False


def test_precomputed_teacher_descriptor_checks():
    logits = torch.randn(4, 16)
    th, tw = torch.randn(4, 8), torch.randn(16, 8)
    with pytest.raises(ValueError, match="logits or"):
        orda_ce_kernel.PrecomputedTeacher(logits=logits, teacher_hidden=th, teacher_weight=tw)
    with pytest.raises(ValueError, match="must provide"):
        orda_ce_kernel.PrecomputedTeacher()
    with pytest.raises(ValueError, match="both be provided"):
        orda_ce_kernel.PrecomputedTeacher(teacher_hidden=th)


def test_config_profile_merge():
    debug = public_api._resolve_profile("debug")
    assert debug.fp32_grad_weight_accumulation is True
    assert public_api._resolve_profile("balanced").fp32_grad_weight_accumulation is False
    merged = public_api._resolve_config("debug", orda_ce_kernel.KernelConfig(chunk_size=7))
    assert merged.fp32_grad_weight_accumulation is True and merged.chunk_size == 7
    over = public_api._resolve_config("debug", orda_ce_kernel.KernelConfig(fp32_grad_weight_accumulation=False))
    assert over.fp32_grad_weight_accumulation is False
    with pytest.raises(ValueError, match="profile"):
        public_api._resolve_profile("fast")
    assert public_api._resolve_kl_config(orda_ce_kernel.KernelConfig(kl_weight=0.5), 0.1, 2.0) == (0.5, 2.0)
    assert public_api._resolve_teacher_ce_weight("tied", None) == 1.0
    assert public_api._resolve_teacher_ce_weight("separate", None) == 0.0
    assert public_api._resolve_teacher_ce_weight("precomputed", None) == 0.0


@pytest.mark.parametrize("cfg,match", [
    (dict(max_chunks=0), "max_chunks"),
    (dict(num_chunks=0), "num_chunks"),
    (dict(chunk_size=2, num_chunks=2), "mutually exclusive"),
    (dict(max_fused_size=100), "power of two"),
    (dict(num_chunks=4, max_chunks=2), "num_chunks must be <="),
])
def test_config_validation_errors(cfg, match):
    hs, ht, w, labels = _inputs()
    with pytest.raises(ValueError, match=match):
        orda_ce_kernel.distillation_loss(hs, w, labels, orda_ce_kernel.TiedTeacher(ht),
                                         config=orda_ce_kernel.KernelConfig(**cfg))


@pytest.mark.parametrize("kwargs,match", [
    (dict(student_ce_weight=-1.0), "student_ce_weight"),
    (dict(teacher_ce_weight=-1.0), "teacher_ce_weight"),
    (dict(kl_weight=-0.5), "kl_weight"),
    (dict(kl_temperature=0.0), "kl_temperature"),
    (dict(reduction="max"), "reduction"),
    (dict(backend="cuda"), "backend"),
    (dict(kl_divergence="tvd"), "kl_divergence"),
    (dict(kl_divergence="jsd", jsd_beta=1.5), "jsd_beta"),
])
def test_argument_errors(kwargs, match):
    hs, ht, w, labels = _inputs()
    with pytest.raises(ValueError, match=match):
        orda_ce_kernel.distillation_loss(hs, w, labels, orda_ce_kernel.TiedTeacher(ht), **kwargs)


def test_shape_and_dtype_errors():
    hs, ht, w, labels = _inputs()
    with pytest.raises(ValueError, match="integer class-index|torch.long"):
        orda_ce_kernel.distillation_loss(hs, w, torch.tensor([True, False, True, False]), orda_ce_kernel.TiedTeacher(ht))
    with pytest.raises(ValueError, match="weight must have shape"):
        orda_ce_kernel.distillation_loss(hs, torch.randn(16, 5), labels, orda_ce_kernel.TiedTeacher(ht))
    with pytest.raises(ValueError, match="TiedTeacher.hidden must have shape"):
        orda_ce_kernel.distillation_loss(hs, w, labels, orda_ce_kernel.TiedTeacher(torch.randn(3, 8)))
    with pytest.raises(ValueError, match="SeparateTeacher.weight must have shape"):
        orda_ce_kernel.distillation_loss(hs, w, labels, orda_ce_kernel.SeparateTeacher(torch.randn(4, 6), torch.randn(15, 6)))
    with pytest.raises(ValueError, match="must not require gradients"):
        orda_ce_kernel.distillation_loss(hs, w, labels, orda_ce_kernel.PrecomputedTeacher(logits=torch.randn(4, 16, requires_grad=True)))
    with pytest.raises(ValueError, match="must not require gradients"):
        orda_ce_kernel.distillation_loss(
            hs, w, labels,
            orda_ce_kernel.PrecomputedTeacher(teacher_hidden=torch.randn(4, 8, requires_grad=True), teacher_weight=torch.randn(16, 8)))
    with pytest.raises(ValueError, match="teacher_ce_weight=0.0"):
        orda_ce_kernel.distillation_loss(hs, w, labels, orda_ce_kernel.PrecomputedTeacher(logits=torch.randn(4, 16)),
                                         teacher_ce_weight=0.5)


def test_no_cpu_fallback():
    hs, ht, w, labels = _inputs()
    for backend in ("auto", "triton"):
        with pytest.raises(RuntimeError, match="no CPU fallback"):
            orda_ce_kernel.distillation_loss(hs, w, labels, orda_ce_kernel.TiedTeacher(ht), backend=backend)
    with pytest.raises(RuntimeError, match="backend='torch'"):
        orda_ce_kernel.distillation_loss(hs, w, labels, orda_ce_kernel.TiedTeacher(ht), backend="torch")
    mod = orda_ce_kernel.DistillationLoss(kl_weight=0.2)
    with pytest.raises(RuntimeError):
        mod(hs, w, labels, orda_ce_kernel.TiedTeacher(ht))


def test_ops_fail_fast_without_kernels():
    from orda_ce_kernel.ops import tied_distillation_loss

    if torch.cuda.is_available():
        pytest.skip("GPU present")
    hs, ht, w, labels = _inputs()
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        tied_distillation_loss(hs, ht, w, labels)


def test_resolver_contract():
    assert is_power_of_two(32768) and not is_power_of_two(100) and not is_power_of_two(0)
    assert resolve_chunk_size(32768, "dynamic", V=131072) == (512, 64)
    assert resolve_chunk_size(100, 7) == (7, 15)
    assert resolve_chunk_size(10, None, num_chunks=3) == (4, 3)
    assert resolve_chunk_size(10, None) == (10, 1)
    with pytest.raises(ValueError, match="BT"):
        resolve_chunk_size(0, None)
    with pytest.raises(ValueError, match="mutually exclusive"):
        resolve_chunk_size(10, 5, num_chunks=2)
    with pytest.raises(ValueError, match="num_chunks must be <= max_chunks"):
        resolve_chunk_size(10, None, num_chunks=8, max_chunks=4)


def test_chunk_cache_is_empty_noop():
    clear_chunk_cache()
    assert get_chunk_cache() == {}


def test_core_modules_read_no_config_files():
    import ast
    import inspect

    from orda_ce_kernel import _fused, _native, api
    from orda_ce_kernel.utils import dispatcher, resolver

    for mod in (api, _fused, _native, dispatcher, resolver):
        tree = ast.parse(inspect.getsource(mod))
        names = {n.id for n in ast.walk(tree) if isinstance(n, ast.Name)}
        assert "open" not in names
        imported = {a.name for n in ast.walk(tree) if isinstance(n, (ast.Import, ast.ImportFrom)) for a in n.names}
        assert not imported & {"json", "yaml", "toml", "configparser"}
