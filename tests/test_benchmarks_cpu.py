"""Host-side checks of the user benchmarks (no GPU): the accuracy benchmark's fp32 baseline formula
agrees with the oracle, and the training benchmark's model and loss formula run on small shapes."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.distill_oracle import distill_reference
from orda_ce_kernel.benchmarks import accuracy, train_step


@pytest.mark.parametrize("mode", ["tied", "separate-full", "precomputed-logits"])
@pytest.mark.parametrize("component", ["ce", "kl"])
def test_accuracy_baseline_formula_matches_oracle(mode, component):
    g = torch.Generator().manual_seed(1)
    n, h, v = 24, 16, 50
    hs = torch.randn(n, h, generator=g, dtype=torch.float64) * 0.5
    w = torch.randn(v, h, generator=g, dtype=torch.float64) * 0.5
    ht = torch.randn(n, h, generator=g, dtype=torch.float64) * 0.5
    wt = torch.randn(v, h, generator=g, dtype=torch.float64) * 0.5
    tl = torch.randn(n, v, generator=g, dtype=torch.float64)
    labels = torch.randint(0, v, (n,), generator=g)
    labels[::5] = -100
    ws, wtce, wk = accuracy.component_weights(mode, component)
    kw = {"tied": dict(ht=ht), "separate-full": dict(ht=ht, wt=wt), "precomputed-logits": dict(tl=tl)}[mode]
    got = float(accuracy.formula(hs, w, labels, tce=accuracy.teacher_ce_weight(mode), component=component, **kw))
    okw = {"tied": dict(mode="tied", teacher_hidden=ht.numpy()),
           "separate-full": dict(mode="separate", teacher_hidden=ht.numpy(), teacher_weight=wt.numpy()),
           "precomputed-logits": dict(mode="precomputed", teacher_logits=tl.numpy())}[mode]
    ref = distill_reference(hs.numpy(), w.numpy(), labels.numpy(), student_ce_weight=ws, teacher_ce_weight=wtce,
                            kl_weight=wk, kl_temperature=accuracy.TEMP, **okw)
    exp = ref.student_ce + ref.teacher_ce if component == "ce" else ref.kl
    assert got == pytest.approx(float(exp), rel=1e-9, abs=1e-12)


def test_train_benchmark_model_and_formula_run_on_cpu():
    cfg = dict(dim=32, q_heads=4, kv_heads=2, n_layers=2, ffn_dim=64)
    lm = train_step.TinyLM(97, cfg, seq=8)
    ids = torch.randint(0, 97, (2, 8))
    h = lm.hidden(ids).view(-1, 32)
    labels = torch.randint(0, 97, (16,))
    loss = train_step.torch_loss(h, lm.head_weight, labels, "tied", h_t=h.detach(), w_t=lm.head_weight)
    loss.backward()
    assert np.isfinite(float(loss.detach())) and lm.embed.weight.grad is not None
