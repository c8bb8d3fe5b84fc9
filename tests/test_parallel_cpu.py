"""Host logic of the multi-GPU forms on CPU: two gloo ranks, the per-rank fused call replaced by a
torch restatement of the loss formula (the CUDA kernels need a GPU). Checks that token sharding
returns the single-process loss (global mean over all ranks' rows) and the same gradients."""
from __future__ import annotations

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from orda_ce_kernel import DistillationLossOutput, TiedTeacher


def _formula(hs, w, labels, teacher, *, reduction="sum", kl_weight=0.0, kl_temperature=1.0, ignore_index=-100,
             teacher_ce_weight=1.0, student_ce_weight=1.0):
    """Tied-teacher loss (forward KL) with the reference's formula (api.py:288-334)."""
    zs, zt = hs @ w.t(), teacher.hidden @ w.t()
    ce_s = F.cross_entropy(zs, labels, ignore_index=ignore_index, reduction="none")
    ce_t = F.cross_entropy(zt, labels, ignore_index=ignore_index, reduction="none")
    mask = labels != ignore_index
    t = kl_temperature
    lps, lpt = F.log_softmax(zs / t, -1), F.log_softmax(zt.detach() / t, -1)
    kl = ((lpt.exp() * (lpt - lps)).sum(-1) * t * t).masked_fill(~mask, 0.0)
    s, tc, k = ce_s.sum(), ce_t.sum(), kl.sum()
    if reduction == "mean":
        d = mask.sum().clamp(min=1)
        s, tc, k = s / d, tc / d, k / d
    loss = student_ce_weight * s + teacher_ce_weight * tc + kl_weight * k
    return DistillationLossOutput(loss, s.detach(), tc.detach(), k.detach())


def _worker(rank, world, port, inputs, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from orda_ce_kernel.parallel import allreduce_weight_grad, token_parallel_distillation_loss

    hs_all, ht_all, w0, labels_all = inputs
    rows = torch.arange(hs_all.shape[0]).chunk(world)[rank]
    hs = hs_all[rows].clone().requires_grad_(True)
    ht = ht_all[rows].clone().requires_grad_(True)
    w = w0.clone().requires_grad_(True)
    out = token_parallel_distillation_loss(hs, w, labels_all[rows], TiedTeacher(ht), kl_weight=0.3,
                                           kl_temperature=1.5, _local_loss=_formula)
    out.loss.backward()
    allreduce_weight_grad(w)
    results[rank] = (rows, [float(x) for x in out], hs.grad.clone(), ht.grad.clone(), w.grad.clone())
    dist.destroy_process_group()


def test_token_parallel_matches_single_process():
    g = torch.Generator().manual_seed(0)
    n, h, v = 21, 6, 13
    hs = torch.randn(n, h, generator=g, dtype=torch.float64)
    ht = torch.randn(n, h, generator=g, dtype=torch.float64)
    w = torch.randn(v, h, generator=g, dtype=torch.float64)
    labels = torch.randint(0, v, (n,), generator=g)
    labels[[1, 4, 15, 16]] = -100
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_worker, args=(2, 29531, (hs, ht, w, labels), results), nprocs=2, join=True)
        results = dict(results)
    a, b, c = hs.clone().requires_grad_(True), ht.clone().requires_grad_(True), w.clone().requires_grad_(True)
    ref = _formula(a, c, labels, TiedTeacher(b), reduction="mean", kl_weight=0.3, kl_temperature=1.5)
    ref.loss.backward()
    for rank in (0, 1):
        rows, vals, ghs, ght, gw = results[rank]
        for got, exp in zip(vals, ref):
            assert got == pytest.approx(float(exp), rel=1e-6)  # sums exchanged in fp32
        torch.testing.assert_close(ghs, a.grad[rows], rtol=1e-6, atol=1e-12)
        torch.testing.assert_close(ght, b.grad[rows], rtol=1e-6, atol=1e-12)
        torch.testing.assert_close(gw, c.grad, rtol=1e-6, atol=1e-12)
