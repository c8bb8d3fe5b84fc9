"""Host logic of the multi-GPU forms on CPU: two gloo ranks, the per-rank fused call replaced by a
torch restatement of the loss formula (the CUDA kernels need a GPU). Checks that token sharding
returns the single-process loss (global mean over all ranks' rows) and the same gradients."""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from orda_ce_kernel import DistillationLossOutput, TiedTeacher


def _free_port() -> int:
    """A port no other listener holds right now (bound to 0, then released), so parallel test runs
    do not collide at rendezvous."""
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


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
        mp.spawn(_worker, args=(2, _free_port(), (hs, ht, w, labels), results), nprocs=2, join=True)
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


# ------------------------------------------------------------------------------ vocab sharding on gloo
class _Pr:
    pass


class _TorchShardOps:
    """Torch (float64) restatement of the per-shard library phases for a tied teacher with CE and
    forward / reverse KL: the row-record layout and LSE merge of the C ABI (include/orda_b200.h,
    orda_shard_forward / orda_merge_row_stats / orda_shard_backward). Lets the CPU ranks run the
    collective choreography of ``vocab_parallel_distillation_loss``."""

    def prepare(self, hs, ht, w, wt, labels, tl, spec, vocab_offset=0, vocab_total=None):
        from orda_ce_kernel import _native

        pr = _Pr()
        pr.spec, pr.off, pr.vt, pr.labels = spec, vocab_offset, vocab_total, labels
        pr.hs, pr.ht, pr.w = hs.detach(), ht.detach(), w.detach()
        pr.zs, pr.zt = pr.hs @ pr.w.t(), pr.ht @ pr.w.t()
        pr.args = _Pr()
        pr.args.n_rows = hs.shape[0]
        pr.dev = hs.device
        pr.h_t = ht.shape[1]
        pr.g_hs = torch.zeros_like(pr.hs) if hs.requires_grad else None
        pr.g_ht = torch.zeros_like(pr.ht) if (ht.requires_grad and spec.teacher_ce_weight > 0) else None
        pr.g_w = torch.zeros_like(pr.w) if w.requires_grad else None
        pr.g_wt = None
        pr.out = torch.zeros(_native.OUT_SLOTS, dtype=torch.float64)
        pr.status = torch.zeros(1, dtype=torch.int32)
        return pr

    def _label_col(self, pr):
        local = pr.labels - pr.off
        has = (pr.labels != pr.spec.ignore_index) & (local >= 0) & (local < pr.w.shape[0])
        return local.clamp(0, pr.w.shape[0] - 1), has

    def forward(self, pr):
        it = 1.0 / pr.spec.kl_temperature
        rev = pr.spec.divergence == "reverse"
        ms, mt = pr.zs.max(-1).values, pr.zt.max(-1).values
        es1, et1 = (pr.zs - ms[:, None]).exp(), (pr.zt - mt[:, None]).exp()
        esT, etT = ((pr.zs - ms[:, None]) * it).exp(), ((pr.zt - mt[:, None]) * it).exp()
        cross = (esT * (pr.zs - pr.zt) * it).sum(-1) if rev else (etT * (pr.zt - pr.zs) * it).sum(-1)
        col, has = self._label_col(pr)
        rec = torch.zeros(pr.zs.shape[0], 16, dtype=torch.float64)
        rec[:, 0], rec[:, 1], rec[:, 2] = ms, es1.sum(-1), esT.sum(-1)
        rec[:, 3], rec[:, 4], rec[:, 5] = mt, et1.sum(-1), etT.sum(-1)
        rec[:, 6] = cross
        rec[:, 7] = torch.where(has, pr.zs.gather(1, col[:, None])[:, 0], torch.zeros(()))
        rec[:, 8] = torch.where(has, pr.zt.gather(1, col[:, None])[:, 0], torch.zeros(()))
        rec[:, 9] = has.double()
        rec[:, 10] = 0.0 if rev else 1.0
        rec[:, 11] = it
        return rec

    def merge(self, gathered, world, n):
        it = float(gathered[0, 0, 11])
        cross_t = bool(gathered[0, 0, 10] != 0)
        out = torch.zeros(n, 16, dtype=torch.float64)
        for side, (im, i1, iT) in enumerate(((0, 1, 2), (3, 4, 5))):
            m = gathered[:, :, im].max(0).values
            f1 = (gathered[:, :, im] - m).exp()
            fT = ((gathered[:, :, im] - m) * it).exp()
            out[:, im], out[:, i1], out[:, iT] = m, (gathered[:, :, i1] * f1).sum(0), (gathered[:, :, iT] * fT).sum(0)
            if (side == 1) == cross_t:
                out[:, 6] = (gathered[:, :, 6] * fT).sum(0)
        out[:, 7] = (gathered[:, :, 7] * gathered[:, :, 9]).sum(0)
        out[:, 8] = (gathered[:, :, 8] * gathered[:, :, 9]).sum(0)
        out[:, 9] = gathered[:, :, 9].max(0).values
        out[:, 10], out[:, 11] = gathered[0, :, 10], it
        return out

    def _log_probs(self, pr, rs):
        it = 1.0 / pr.spec.kl_temperature
        lse_sT, lse_tT = rs[:, 0] * it + rs[:, 2].log(), rs[:, 3] * it + rs[:, 5].log()
        return pr.zs * it - lse_sT[:, None], pr.zt * it - lse_tT[:, None]

    def _jsd_terms(self, pr, rs):
        b = pr.spec.jsd_beta
        lps, lpt = self._log_probs(pr, rs)
        lm = torch.logaddexp(torch.log(torch.tensor(b, dtype=torch.float64)) + lpt,
                             torch.log1p(torch.tensor(-b, dtype=torch.float64)) + lps)
        return lps, lpt, lm

    def jsd_partials(self, pr, row_stats):
        """This shard's [sum_v b p_t (log p_t - log m) + (1-b) p_s (log p_s - log m), sum_v p_s g]."""
        b = pr.spec.jsd_beta
        lps, lpt, lm = self._jsd_terms(pr, row_stats)
        ps, pt = lps.exp(), lpt.exp()
        valid = (pr.labels != pr.spec.ignore_index).double()
        sj = (b * pt * (lpt - lm) + (1 - b) * ps * (lps - lm)).sum(-1) * valid
        sg = (ps * (1 - b) * (lps - lm)).sum(-1) * valid
        return torch.stack([sj, sg], -1)

    def backward(self, pr, rs, row_sums):
        from orda_ce_kernel import _native

        sp, T = pr.spec, pr.spec.kl_temperature
        it = 1.0 / T
        valid = pr.labels != sp.ignore_index
        cnt = valid.sum().clamp(min=1).double()
        scale = 1.0 / cnt if sp.reduction == "mean" else torch.ones((), dtype=torch.float64)
        lse_s1, lse_t1 = rs[:, 0] + rs[:, 1].log(), rs[:, 3] + rs[:, 4].log()
        lse_sT, lse_tT = rs[:, 0] * it + rs[:, 2].log(), rs[:, 3] * it + rs[:, 5].log()
        ce_s, ce_t = (lse_s1 - rs[:, 7]) * valid, (lse_t1 - rs[:, 8]) * valid
        rev = sp.divergence == "reverse"
        if sp.divergence == "jsd":
            div = row_sums[:, 0] * T * T * valid
        else:
            div = (rs[:, 6] / (rs[:, 2] if rev else rs[:, 5]) + ((lse_tT - lse_sT) if rev else (lse_sT - lse_tT)))
            div = div * T * T * valid
        ps1, pt1 = (pr.zs - lse_s1[:, None]).exp(), (pr.zt - lse_t1[:, None]).exp()
        lpsT, lptT = pr.zs * it - lse_sT[:, None], pr.zt * it - lse_tT[:, None]
        psT, ptT = lpsT.exp(), lptT.exp()
        col, has = self._label_col(pr)
        onehot = torch.zeros_like(pr.zs).scatter_(1, col[:, None], 1.0) * has[:, None]
        if sp.divergence == "jsd":
            # g = (1 - b)(log p_s - log m); the row sum of p_s g comes all-reduced from jsd_partials
            _, _, lm = self._jsd_terms(pr, rs)
            dkl = psT * ((1 - sp.jsd_beta) * (lpsT - lm) - row_sums[:, 1:2])
        elif rev:
            # R = sum_v p_s (log p_s - log p_t) over the WHOLE vocabulary, from the merged record
            a = lpsT - lptT
            r = (rs[:, 6] / rs[:, 2] - lse_sT + lse_tT)[:, None]
            dkl = psT * (a - r)
        else:
            dkl = psT - ptT
        dzs = (sp.student_ce_weight * (ps1 - onehot) + sp.kl_weight * T * dkl) * valid[:, None] * scale
        dzt = sp.teacher_ce_weight * (pt1 - onehot) * valid[:, None] * scale
        if pr.g_hs is not None:
            pr.g_hs.copy_(dzs @ pr.w)
        if pr.g_ht is not None:
            pr.g_ht.copy_(dzt @ pr.w)
        if pr.g_w is not None:
            pr.g_w.copy_(dzs.t() @ pr.hs + dzt.t() @ pr.ht)
        s0, s1, s2 = ce_s.sum(), ce_t.sum(), div.sum()
        o = pr.out
        o[_native.OUT_STUDENT_CE], o[_native.OUT_TEACHER_CE], o[_native.OUT_KL] = s0 * scale, s1 * scale, s2 * scale
        o[_native.OUT_LOSS] = (sp.student_ce_weight * s0 + sp.teacher_ce_weight * s1 + sp.kl_weight * s2) * scale
        o[_native.OUT_MEAN_SCALE] = scale

    @staticmethod
    def rescale(ctx, grads, grad_output):
        return [None if g is None else (g[:, :cols] * grad_output).to(dt) for g, cols, dt in grads]


def _vocab_worker(rank, world, port, inputs, div, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from orda_ce_kernel.parallel import vocab_parallel_distillation_loss

    hs0, ht0, w_all, labels = inputs
    v = w_all.shape[0]
    lo, hi = rank * v // world, (rank + 1) * v // world
    hs = hs0.clone().requires_grad_(True)
    ht = ht0.clone().requires_grad_(True)
    w = w_all[lo:hi].clone().requires_grad_(True)
    out = vocab_parallel_distillation_loss(hs, w, labels, TiedTeacher(ht), vocab_offset=lo, vocab_total=v,
                                           kl_weight=0.4, kl_temperature=1.5, kl_divergence=div, jsd_beta=0.3,
                                           student_ce_weight=0.7, _shard_ops=_TorchShardOps)
    (2.0 * out.loss).backward()
    results[rank] = ((lo, hi), [float(x) for x in out], hs.grad.clone(), ht.grad.clone(), w.grad.clone())
    dist.destroy_process_group()


@pytest.mark.parametrize("div", ["forward", "reverse", "jsd"])
def test_vocab_parallel_matches_single_process(div):
    """Two gloo ranks each holding half of the lm_head rows: the record gather + LSE merge, the
    hidden-gradient all-reduce and the backward rescale reproduce the single-process loss and
    gradients (oracle)."""
    import numpy as np

    from oracle.distill_oracle import distill_reference

    g = torch.Generator().manual_seed(3)
    n, h, v = 17, 6, 29
    hs = torch.randn(n, h, generator=g, dtype=torch.float64)
    ht = torch.randn(n, h, generator=g, dtype=torch.float64)
    w = torch.randn(v, h, generator=g, dtype=torch.float64)
    labels = torch.randint(0, v, (n,), generator=g)
    labels[::5] = -100
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_vocab_worker, args=(2, _free_port(), (hs, ht, w, labels), div, results), nprocs=2, join=True)
        results = dict(results)
    ref = distill_reference(hs.numpy(), w.numpy(), labels.numpy(), mode="tied", teacher_hidden=ht.numpy(),
                            student_ce_weight=0.7, kl_weight=0.4, kl_temperature=1.5, kl_divergence=div,
                            jsd_beta=0.3)
    for rank in (0, 1):
        (lo, hi), vals, ghs, ght, gw = results[rank]
        exp = [ref.loss, ref.student_ce, ref.teacher_ce, ref.kl]
        assert vals == pytest.approx([float(x) for x in exp], rel=1e-9, abs=1e-12)
        np.testing.assert_allclose(ghs.numpy(), 2.0 * ref.d_student_hidden, rtol=1e-9, atol=1e-12)
        np.testing.assert_allclose(ght.numpy(), 2.0 * ref.d_teacher_hidden, rtol=1e-9, atol=1e-12)
        np.testing.assert_allclose(gw.numpy(), 2.0 * ref.d_weight[lo:hi], rtol=1e-9, atol=1e-12)


# ------------------------------------------------------------------------------ failure handling
class _FailingShardOps(_TorchShardOps):
    """Shard ops whose backward on rank 1 reports a device error in the status word, the way a
    bounded pipeline wait that ran out (ORDA_ERR_TIMEOUT) reports it from the kernels."""

    def backward(self, pr, rs, row_sums):
        from orda_ce_kernel import _native

        super().backward(pr, rs, row_sums)
        if dist.get_rank() == 1:
            pr.status.fill_(_native.ERR_TIMEOUT)


def _status_worker(rank, world, port, inputs, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    from orda_ce_kernel.parallel import vocab_parallel_distillation_loss

    hs0, ht0, w_all, labels = inputs
    v = w_all.shape[0]
    lo, hi = rank * v // world, (rank + 1) * v // world
    try:
        vocab_parallel_distillation_loss(hs0.clone().requires_grad_(True), w_all[lo:hi].clone().requires_grad_(True),
                                         labels, TiedTeacher(ht0.clone()), vocab_offset=lo, vocab_total=v,
                                         kl_weight=0.4, _shard_ops=_FailingShardOps)
        results[rank] = "returned"
    except RuntimeError as e:
        results[rank] = str(e)
    dist.destroy_process_group()


def test_vocab_parallel_device_status_raises_on_every_rank():
    """A device error reported by one rank's kernels makes every rank raise (the status words are
    MAX-all-reduced before any gradient is returned), instead of one rank raising while the other
    goes on with garbage gradients."""
    g = torch.Generator().manual_seed(5)
    n, h, v = 9, 4, 11
    inputs = (torch.randn(n, h, generator=g, dtype=torch.float64), torch.randn(n, h, generator=g, dtype=torch.float64),
              torch.randn(v, h, generator=g, dtype=torch.float64), torch.randint(0, v, (n,), generator=g))
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_status_worker, args=(2, _free_port(), inputs, results), nprocs=2, join=True)
        results = dict(results)
    for rank in (0, 1):
        assert "timed out" in results[rank], results[rank]


def _dead_rank_worker(rank, world, port, inputs, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    from orda_ce_kernel.parallel import vocab_parallel_distillation_loss

    hs0, ht0, w_all, labels = inputs
    v = w_all.shape[0]
    lo, hi = rank * v // world, (rank + 1) * v // world
    if rank == 1:
        # this rank fails on the host before its first collective and never joins it
        results[rank] = "failed before the collective"
        return
    try:
        vocab_parallel_distillation_loss(hs0.clone().requires_grad_(True), w_all[lo:hi].clone().requires_grad_(True),
                                         labels, TiedTeacher(ht0.clone()), vocab_offset=lo, vocab_total=v,
                                         kl_weight=0.4, _shard_ops=_TorchShardOps)
        results[rank] = "returned"
    except RuntimeError as e:
        results[rank] = "error: " + str(e).splitlines()[0]


def test_vocab_parallel_rank_failure_ends_the_collective_with_an_error():
    """A rank that fails before the record gather leaves the surviving rank's collective to end with
    an error (the process group's short timeout, or the closed connection), never to wait forever."""
    g = torch.Generator().manual_seed(6)
    n, h, v = 9, 4, 11
    inputs = (torch.randn(n, h, generator=g, dtype=torch.float64), torch.randn(n, h, generator=g, dtype=torch.float64),
              torch.randn(v, h, generator=g, dtype=torch.float64), torch.randint(0, v, (n,), generator=g))
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_dead_rank_worker, args=(2, _free_port(), inputs, results), nprocs=2, join=True)
        results = dict(results)
    assert results[1] == "failed before the collective"
    assert results[0].startswith("error:"), results[0]
