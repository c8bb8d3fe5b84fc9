"""Peak extra device memory of one loss + backward: plain PyTorch, ``torch.compile`` and the fused kernels.

    python -m orda_ce_kernel.benchmarks.vram [--teacher tied|separate-student|separate-full|precomputed]
                                             [--dims 512 1024] [--vocabs 16384 32768 65536]
                                             [--seqs 256 512 1024 2048] [--json out.json]

Same protocol as the reference's VRAM benchmark (``test/benchmark/src/_vram.py:435-673``,
``bench_vram_*.py``): batch 16, T = 3.0, ``KernelConfig(num_chunks=16)`` for the fused call, inputs
N(0, 1) in the 16-bit dtype, the student hidden states and the student lm_head take gradients. The
figure is ``max_memory_allocated`` during one forward + backward minus the memory held before it (the
inputs), i.e. logits, workspace, saved tensors and the gradients. "OOM" marks a backend that ran out of
memory.
"""
from __future__ import annotations

import argparse
import gc
from itertools import product

import torch
import torch.nn.functional as F

from ._common import print_table, write_json

BATCH = 16
TEMP = 3.0
NUM_CHUNKS = 16
DIMS = [512, 1024]
VOCABS = [16_384, 32_768, 65_536]
SEQS = [256, 512, 1024, 2048]
BACKENDS = ["torch", "torch-compile", "orda_b200"]
TEACHERS = ["tied", "separate-student", "separate-full", "precomputed"]


def _torch_loss(teacher: str):
    """The unfused formula of each teacher mode (mean CE + batch-mean KL · T²)."""
    def loss_fn(h_s, w_s, labels, h_t, w_t):
        z_s = F.linear(h_s, w_s)
        z_t = F.linear(h_t, w_t if w_t is not None else w_s)
        ce = F.cross_entropy(z_s, labels)
        if teacher in ("tied", "separate-full"):
            ce = ce + F.cross_entropy(z_t, labels)
        log_p_s = F.log_softmax(z_s / TEMP, dim=-1)
        p_t = F.softmax((z_t / TEMP).detach(), dim=-1)
        return ce + F.kl_div(log_p_s, p_t, reduction="batchmean") * (TEMP * TEMP)
    return loss_fn


def _fused_loss(teacher: str):
    import orda_ce_kernel as ok

    def loss_fn(h_s, w_s, labels, h_t, w_t):
        if teacher == "tied":
            t, tce = ok.TiedTeacher(h_t), 1.0
        elif teacher == "precomputed":
            t, tce = ok.PrecomputedTeacher(teacher_hidden=h_t, teacher_weight=w_t), 0.0
        else:
            t, tce = ok.SeparateTeacher(h_t, w_t), (1.0 if teacher == "separate-full" else 0.0)
        return ok.distillation_loss(h_s, w_s, labels, t, student_ce_weight=1.0, teacher_ce_weight=tce,
                                    kl_weight=1.0, kl_temperature=TEMP,
                                    config=ok.KernelConfig(num_chunks=NUM_CHUNKS)).loss
    return loss_fn


def _inputs(teacher, vocab, dim, seq, dtype, device):
    n = BATCH * seq
    h_s = torch.randn(n, dim, device=device, dtype=dtype)
    w_s = torch.randn(vocab, dim, device=device, dtype=dtype, requires_grad=True)
    labels = torch.randint(0, vocab, (n,), device=device)
    h_t = torch.randn(n, dim, device=device, dtype=dtype)
    w_t = None if teacher == "tied" else torch.randn(vocab, dim, device=device, dtype=dtype)
    return h_s, w_s, labels, h_t, w_t


def _cleanup():
    torch._dynamo.reset()
    gc.collect()
    torch.cuda.empty_cache()


def measure_once(teacher, backend, vocab, dim, seq, *, dtype=torch.bfloat16, device="cuda") -> float:
    """Peak extra MB of one loss + backward after one warm-up call (inf on out-of-memory)."""
    _cleanup()
    fn = _fused_loss(teacher) if backend == "orda_b200" else _torch_loss(teacher)
    if backend == "torch-compile":
        fn = torch.compile(fn, mode="default")

    def run(inp):
        h_s, w_s, labels, h_t, w_t = inp
        h = h_s.detach().requires_grad_(True)
        w_s.grad = None
        fn(h, w_s, labels, h_t, w_t).backward()
        torch.cuda.synchronize(device)
        return h

    try:
        inp = _inputs(teacher, vocab, dim, seq, dtype, device)
        run(inp)  # warm-up (compilation, library load)
        inp[1].grad = None
        torch.cuda.synchronize(device)
        torch.cuda.reset_peak_memory_stats(device)
        base = torch.cuda.memory_allocated(device)
        h = run(inp)
        extra = (torch.cuda.max_memory_allocated(device) - base) / 1024 ** 2
        del h, inp
    except torch.cuda.OutOfMemoryError:
        extra = float("inf")
    _cleanup()
    return extra


def _mb(v: float) -> str:
    return "OOM" if v == float("inf") else f"{v:.1f} MB"


def _delta(base: float, ours: float) -> str:
    if base in (0.0, float("inf")) or ours == float("inf"):
        return "NA"
    return f"{(ours / base - 1) * 100:+.1f}%"


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--teacher", default="tied", choices=TEACHERS)
    p.add_argument("--dims", type=int, nargs="+", default=DIMS)
    p.add_argument("--vocabs", type=int, nargs="+", default=VOCABS)
    p.add_argument("--seqs", type=int, nargs="+", default=SEQS)
    p.add_argument("--backends", nargs="+", default=BACKENDS, choices=BACKENDS)
    p.add_argument("--json", default=None)
    a = p.parse_args(argv)
    if not torch.cuda.is_available():
        raise RuntimeError("the VRAM benchmark needs a CUDA device (B200)")
    records = []
    for dim in a.dims:
        rows = []
        for vocab, seq in product(a.vocabs, a.seqs):
            r = {"teacher": a.teacher, "dim": dim, "vocab": vocab, "seq": seq, "batch": BATCH}
            for b in a.backends:
                r[b] = measure_once(a.teacher, b, vocab, dim, seq)
            records.append(r)
            ours = r.get("orda_b200", float("inf"))
            rows.append([f"vocab={vocab // 1024}k seq={seq}", *(_mb(r[b]) for b in a.backends),
                         _delta(r.get("torch", 0.0), ours), _delta(r.get("torch-compile", 0.0), ours)])
        print_table(["config", *a.backends, "deltaTorch", "deltaCompile"], rows,
                    title=f"{a.teacher}  dim={dim}  batch={BATCH}  T={TEMP}  num_chunks={NUM_CHUNKS}")
    write_json(a.json, {"gpu": torch.cuda.get_device_name(), "records": [
        {k: (None if v == float("inf") else v) for k, v in r.items()} for r in records]})
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
