"""``torch.ops.orda_b200.distill_fwdbwd``: the custom op that lets ``torch.compile`` trace
``distillation_loss`` without a graph break. CPU: the fake implementation's shapes and the op schema.
GPU: compiled loss / gradients equal the eager ones, and a student layer + loss compile as one graph."""
from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import orda_ce_kernel as ok

_SCALARS = ("tied", 1.0, 1.0, 0.5, 1.0, -100, "mean", "forward", 0.5, 0, False)


def test_fake_impl_shapes_follow_need_flags():
    with FakeTensorMode():
        hs = torch.empty(64, 40, dtype=torch.bfloat16)
        w = torch.empty(100, 40, dtype=torch.bfloat16)
        ht = torch.empty(64, 40, dtype=torch.bfloat16)
        lab = torch.empty(64, dtype=torch.long)
        out, g_hs, g_ht, g_w, g_wt = torch.ops.orda_b200.distill_fwdbwd(
            hs, w, lab, ht, None, None, *_SCALARS, [True, True, False, False])
    assert out.shape == (9,) and out.dtype == torch.float32
    assert g_hs.shape == hs.shape and g_hs.dtype == torch.bfloat16
    assert g_ht.shape == ht.shape
    assert g_w.numel() == 0 and g_wt.numel() == 0


def test_separate_teacher_fake_shapes():
    with FakeTensorMode():
        hs = torch.empty(8, 16, dtype=torch.float16)
        w = torch.empty(50, 16, dtype=torch.float16)
        ht = torch.empty(8, 24, dtype=torch.float16)
        wt = torch.empty(50, 24, dtype=torch.float16)
        lab = torch.empty(8, dtype=torch.long)
        res = torch.ops.orda_b200.distill_fwdbwd(hs, w, lab, ht, wt, None, "separate", 1.0, 0.5, 0.5, 1.5, -100,
                                                 "sum", "reverse", 0.5, 0, False, [True, True, True, True])
    assert [tuple(t.shape) for t in res[1:]] == [(8, 16), (8, 24), (50, 16), (50, 24)]


def _case(seed=3, n=300, h=256, v=3000):
    g = torch.Generator().manual_seed(seed)
    hs = torch.randn(n, h, generator=g).to(torch.bfloat16).cuda()
    ht = torch.randn(n, h, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(v, h, generator=g) * 0.02).to(torch.bfloat16).cuda()
    labels = torch.randint(0, v, (n,), generator=g).cuda()
    labels[::7] = -100
    return hs, ht, w, labels


@pytest.mark.gpu
def test_compiled_loss_matches_eager():
    hs0, ht0, w0, labels = _case()

    def loss_fn(hs, ht, w, labels):
        out = ok.distillation_loss(hs, w, labels, ok.TiedTeacher(ht), kl_weight=0.5, kl_temperature=1.5)
        return out.loss * 2.0, out.kl

    results = []
    for fn in (loss_fn, torch.compile(loss_fn, fullgraph=True)):
        hs = hs0.clone().requires_grad_(True)
        ht = ht0.clone().requires_grad_(True)
        w = w0.clone().requires_grad_(True)
        loss, kl = fn(hs, ht, w, labels)
        loss.backward()
        results.append((float(loss), float(kl), hs.grad.float(), ht.grad.float(), w.grad.float()))
    (l0, k0, *g0), (l1, k1, *g1) = results
    assert l1 == pytest.approx(l0, rel=1e-6) and k1 == pytest.approx(k0, rel=1e-6)
    for a, b in zip(g0, g1):
        torch.testing.assert_close(b, a, rtol=1e-2, atol=1e-6)


@pytest.mark.gpu
def test_student_layer_and_loss_compile_as_one_graph():
    hs0, ht0, w0, labels = _case(seed=4)
    proj = torch.nn.Linear(256, 256, dtype=torch.bfloat16).cuda()

    def step(x, ht, w, labels):
        h = torch.nn.functional.gelu(proj(x))
        return ok.distillation_loss(h, w, labels, ok.TiedTeacher(ht), kl_weight=1.0).loss

    explain = torch._dynamo.explain(step)(hs0, ht0, w0.clone().requires_grad_(True), labels)
    assert explain.graph_break_count == 0, explain.break_reasons
    w = w0.clone().requires_grad_(True)
    loss = torch.compile(step, fullgraph=True)(hs0, ht0, w, labels)
    loss.backward()
    assert torch.isfinite(loss) and w.grad is not None and proj.weight.grad is not None


def test_public_api_traces_to_one_custom_op_without_graph_break():
    """torch.export (strict dynamo capture, which fails on any graph break) of ``distillation_loss`` on
    fake CUDA tensors: the whole public path lowers to the custom op plus output selection."""
    class LossModule(torch.nn.Module):
        def forward(self, hs, ht, w, labels):
            out = ok.distillation_loss(hs, w, labels, ok.TiedTeacher(ht), kl_weight=0.5, kl_temperature=1.5,
                                       kl_divergence="jsd")
            return out.loss, out.kl

    with FakeTensorMode(allow_non_fake_inputs=True):
        hs = torch.empty(64, 32, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        ht = torch.empty(64, 32, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        w = torch.empty(100, 32, device="cuda", dtype=torch.bfloat16, requires_grad=True)
        labels = torch.zeros(64, device="cuda", dtype=torch.long)
    ep = torch.export.export(LossModule(), (hs, ht, w, labels), strict=True)
    calls = [n for n in ep.graph.nodes if n.op == "call_function" and "orda_b200" in str(n.target)]
    assert len(calls) == 1
    args = calls[0].args
    assert args[6] == "tied" and args[13] == "jsd" and list(args[-1]) == [True, True, True, False]
