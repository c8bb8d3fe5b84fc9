"""Multi-GPU forms on 2 GPUs (NCCL): vocab-sharded and token-sharded losses must reproduce the
single-GPU result of ``distillation_loss`` on the same inputs. Skipped with fewer than 2 GPUs."""
from __future__ import annotations

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

CASES = [
    ("tied", "forward", 1.0),
    ("tied", "reverse", 1.5),
    ("tied", "jsd", 1.0),
    ("separate-full", "reverse", 1.5),
    ("precomputed-logits", "forward", 2.0),
]


def _inputs(mode, n=300, h=256, ht=384, v=3000, seed=5):
    g = torch.Generator().manual_seed(seed)
    d = {
        "hs": torch.randn(n, h, generator=g).to(torch.bfloat16),
        "w": (torch.randn(v, h, generator=g) * 0.02).to(torch.bfloat16),
        "labels": torch.randint(0, v, (n,), generator=g),
    }
    d["labels"][::11] = -100
    if mode == "tied":
        d["ht"] = torch.randn(n, h, generator=g).to(torch.bfloat16)
    elif mode == "separate-full":
        d["ht"] = torch.randn(n, ht, generator=g).to(torch.bfloat16)
        d["wt"] = (torch.randn(v, ht, generator=g) * 0.02).to(torch.bfloat16)
    else:
        d["tl"] = torch.log_softmax(torch.randn(n, v, generator=g) * 2.0, -1)
    return d


def _run(mode, div, temp, d, dev, *, vocab_slice=None, row_slice=None, group=None, parallel=None, exchange=None,
         config=None):
    import orda_ce_kernel as ok
    from orda_ce_kernel import _fused
    from orda_ce_kernel.parallel import token_parallel_distillation_loss, vocab_parallel_distillation_loss

    rows = row_slice if row_slice is not None else slice(None)
    cols = vocab_slice if vocab_slice is not None else slice(None)
    hs = d["hs"][rows].to(dev).requires_grad_(True)
    w = d["w"][cols].contiguous().to(dev).requires_grad_(True)
    labels = d["labels"][rows].to(dev)
    tce, extra = None, {}
    if mode == "tied":
        ht = d["ht"][rows].to(dev).requires_grad_(True)
        teacher = ok.TiedTeacher(ht)
    elif mode == "separate-full":
        ht = d["ht"][rows].to(dev).requires_grad_(True)
        wt = d["wt"][cols].contiguous().to(dev).requires_grad_(True)
        teacher, tce = ok.SeparateTeacher(ht, wt), 0.5
    else:
        teacher = ok.PrecomputedTeacher(logits=d["tl"][rows][:, cols].contiguous().to(dev))
    kw = dict(teacher_ce_weight=tce, student_ce_weight=0.5, kl_weight=0.5, kl_temperature=temp, kl_divergence=div)
    if config is not None:
        kw["config"] = config
    if parallel == "peer":
        # token sharding with the lm_head gradient summed through peer memory (no all-reduce of it)
        with _fused.instrument(peer_exchange=exchange):
            out = token_parallel_distillation_loss(hs, w, labels, teacher, group=group, **kw)
            out.loss.backward()
        if mode == "separate-full":
            dist.all_reduce(teacher.weight.grad, group=group)  # the teacher lm_head gradient stays per rank
    elif parallel == "vocab":
        out = vocab_parallel_distillation_loss(hs, w, labels, teacher, vocab_offset=cols.start,
                                               vocab_total=d["w"].shape[0], group=group, **kw)
    elif parallel == "tokens":
        out = token_parallel_distillation_loss(hs, w, labels, teacher, group=group, **kw)
    else:
        out = ok.distillation_loss(hs, w, labels, teacher, **kw)
    if parallel != "peer":
        out.loss.backward()
    if parallel == "tokens":
        dist.all_reduce(w.grad, group=group)
    res = {"vals": [float(x.detach()) for x in out], "ghs": hs.grad.float().cpu(), "gw": w.grad.float().cpu()}
    if mode != "precomputed-logits":
        res["ght"] = teacher.hidden.grad.float().cpu()
    if mode == "separate-full":
        res["gwt"] = teacher.weight.grad.float().cpu()
    return res


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    from orda_ce_kernel import KernelConfig
    from orda_ce_kernel.parallel import PeerGradientExchange

    out = {}
    exchange = PeerGradientExchange(_inputs("tied")["w"].to(dev), group=dist.group.WORLD)
    for mode, div, temp in CASES:
        d = _inputs(mode)
        v = d["w"].shape[0]
        vs = slice(rank * v // world, (rank + 1) * v // world)
        n = d["hs"].shape[0]
        rs = slice(rank * n // world, (rank + 1) * n // world)
        out[(mode, div, "vocab")] = (vs, _run(mode, div, temp, d, dev, vocab_slice=vs, parallel="vocab"))
        out[(mode, div, "tokens")] = (rs, _run(mode, div, temp, d, dev, row_slice=rs, parallel="tokens"))
        out[(mode, div, "peer")] = (rs, _run(mode, div, temp, d, dev, row_slice=rs, parallel="peer",
                                             exchange=exchange))
        # several row chunks: earlier chunks accumulate locally, the last one routes the sum
        out[(mode, div, "peer-chunked")] = (rs, _run(mode, div, temp, d, dev, row_slice=rs, parallel="peer",
                                                     exchange=exchange, config=KernelConfig(chunk_size=64)))
    results[rank] = out
    # every rank unmaps its peers' buffers before any rank frees its own
    exchange.close()
    dist.barrier()
    dist.destroy_process_group()


def _free_port() -> int:
    import socket

    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _rel(a, b):
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_vocab_and_token_parallel_match_single_gpu():
    with mp.Manager() as m:
        results = m.dict()
        mp.spawn(_worker, args=(2, _free_port(), results), nprocs=2, join=True)
        results = dict(results)
    dev = torch.device("cuda", 0)
    for mode, div, temp in CASES:
        d = _inputs(mode)
        ref = _run(mode, div, temp, d, dev)
        for rank in (0, 1):
            vs, vres = results[rank][(mode, div, "vocab")]
            rs, tres = results[rank][(mode, div, "tokens")]
            for got, exp in zip(vres["vals"] + tres["vals"], ref["vals"] * 2):
                assert got == pytest.approx(exp, rel=1e-3, abs=1e-5), (mode, div)
            # vocab sharding: full hidden gradients, this rank's slice of the lm_head gradient
            assert _rel(vres["ghs"], ref["ghs"]) < 2e-2
            assert _rel(vres["gw"], ref["gw"][vs]) < 2e-2
            # token sharding: this rank's rows, the summed lm_head gradient (NCCL all-reduce, or the
            # peer-memory exchange fused into the dW GEMM, in one or several row chunks)
            assert _rel(tres["ghs"], ref["ghs"][rs]) < 2e-2
            assert _rel(tres["gw"], ref["gw"]) < 2e-2
            for key in ("peer", "peer-chunked"):
                _, pres = results[rank][(mode, div, key)]
                for got, exp in zip(pres["vals"], ref["vals"]):
                    assert got == pytest.approx(exp, rel=1e-3, abs=1e-5), (mode, div, key)
                assert _rel(pres["ghs"], ref["ghs"][rs]) < 2e-2, (mode, div, key)
                assert _rel(pres["gw"], ref["gw"]) < 2e-2, (mode, div, key)
                # every rank holds the same summed gradient
                torch.testing.assert_close(pres["gw"], results[1 - rank][(mode, div, key)][1]["gw"], rtol=0, atol=0)
                if "gwt" in ref:
                    assert _rel(pres["gwt"], ref["gwt"]) < 2e-2
            if "ght" in ref:
                assert _rel(vres["ght"], ref["ght"]) < 2e-2
                assert _rel(tres["ght"], ref["ght"][rs]) < 2e-2
            if "gwt" in ref:
                assert _rel(vres["gwt"], ref["gwt"][vs]) < 2e-2
