"""Training step of a small Transformer student distilled from a Transformer teacher: ms/step and
peak memory with the loss as a ``torch.compile``d PyTorch formula vs the fused kernels.

    python -m orda_ce_kernel.benchmarks.train_step [--teacher separate-student] [--vocabs 32768]
                                                   [--seqs 512 1024 2048] [--steps 50] [--json out.json]

Protocol of the reference's training benchmark (``test/benchmark/src/_train.py:102-452``,
``Train_*.py``, model of ``src/core.py:106-138``): a pre-norm decoder (RMSNorm, rotary position
embedding, grouped-query attention through SDPA, SwiGLU MLP, lm_head tied to the embedding), teacher
dim 1024 / 16 layers, student dim 1024 / 8 layers (8 query heads, 2 KV heads, FFN 2816), batch 16,
T = 3.0, bf16 weights, SGD lr 1e-3; 5 warm-up steps, then ``--steps`` timed steps per pass, two passes
in opposite order. A step is teacher forward (no grad) + student forward + loss + backward + optimizer
step on random token ids. Backends:
  torch-compile  - teacher, student and the PyTorch loss formula in one compiled function;
  orda_b200      - compiled teacher and student, the fused loss called eagerly;
  orda_b200-graph- the student forward and the fused loss compiled together (the loss is a custom op,
                   so the compiled region has no graph break).
"""
from __future__ import annotations

import argparse
import gc
import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from ._common import write_json

TEACHER_CFG = dict(dim=1024, q_heads=8, kv_heads=2, n_layers=16, ffn_dim=2816)
STUDENT_CFG = dict(dim=1024, q_heads=8, kv_heads=2, n_layers=8, ffn_dim=2816)
BATCH, TEMP, WARMUP = 16, 3.0, 5
BACKENDS = ["torch-compile", "orda_b200", "orda_b200-graph"]
TEACHERS = ["tied", "separate-student", "separate-full", "precomputed-logits", "precomputed-hidden"]


# ----------------------------------------------------------------------------------------- model
class RMSNorm(nn.Module):
    def __init__(self, d: int, eps: float = 1e-6):
        super().__init__()
        self.eps = eps
        self.scale = nn.Parameter(torch.ones(d))

    def forward(self, x):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + self.eps) * self.scale


def rotary_tables(head_dim: int, seq: int):
    inv = 1.0 / (10000.0 ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    ang = torch.outer(torch.arange(seq, dtype=torch.float32), inv)
    ang = torch.cat([ang, ang], dim=-1)
    return ang.cos(), ang.sin()


def rotate(x, cos, sin):
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos + rot * sin


class Attention(nn.Module):
    def __init__(self, d, q_heads, kv_heads, seq):
        super().__init__()
        self.hq, self.hkv, self.dh = q_heads, kv_heads, d // q_heads
        self.qkv = nn.Linear(d, (q_heads + 2 * kv_heads) * self.dh, bias=False)
        self.proj = nn.Linear(d, d, bias=False)
        cos, sin = rotary_tables(self.dh, seq)
        self.register_buffer("cos", cos, persistent=False)
        self.register_buffer("sin", sin, persistent=False)

    def forward(self, x):
        b, t, d = x.shape
        q, k, v = self.qkv(x).split([self.hq * self.dh, self.hkv * self.dh, self.hkv * self.dh], dim=-1)
        q = q.view(b, t, self.hq, self.dh).transpose(1, 2)
        k = k.view(b, t, self.hkv, self.dh).transpose(1, 2)
        v = v.view(b, t, self.hkv, self.dh).transpose(1, 2)
        cos, sin = self.cos[:t].to(x.dtype), self.sin[:t].to(x.dtype)
        q, k = rotate(q, cos, sin), rotate(k, cos, sin)
        rep = self.hq // self.hkv
        k = k.repeat_interleave(rep, dim=1)
        v = v.repeat_interleave(rep, dim=1)
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return self.proj(y.transpose(1, 2).reshape(b, t, d))


class MLP(nn.Module):
    def __init__(self, d, ff):
        super().__init__()
        self.gate = nn.Linear(d, ff, bias=False)
        self.up = nn.Linear(d, ff, bias=False)
        self.down = nn.Linear(ff, d, bias=False)

    def forward(self, x):
        return self.down(F.silu(self.gate(x)) * self.up(x))


class Block(nn.Module):
    def __init__(self, cfg, seq):
        super().__init__()
        d = cfg["dim"]
        self.n1, self.n2 = RMSNorm(d), RMSNorm(d)
        self.attn = Attention(d, cfg["q_heads"], cfg["kv_heads"], seq)
        self.mlp = MLP(d, cfg["ffn_dim"])

    def forward(self, x):
        x = x + self.attn(self.n1(x))
        return x + self.mlp(self.n2(x))


class TinyLM(nn.Module):
    """Decoder with the lm_head tied to the token embedding; ``hidden`` returns the final normed states."""

    def __init__(self, vocab, cfg, seq):
        super().__init__()
        self.embed = nn.Embedding(vocab, cfg["dim"])
        nn.init.normal_(self.embed.weight, std=0.02)
        self.blocks = nn.ModuleList(Block(cfg, seq) for _ in range(cfg["n_layers"]))
        self.norm = RMSNorm(cfg["dim"])

    @property
    def head_weight(self):
        return self.embed.weight

    def hidden(self, ids):
        h = self.embed(ids)
        for blk in self.blocks:
            h = blk(h)
        return self.norm(h)


# ------------------------------------------------------------------------------------------ loss
def torch_loss(h_s, w_s, labels, teacher, z_t=None, h_t=None, w_t=None):
    """PyTorch formula of the same objective: CE(student) [+ CE(teacher)] + T^2 KL(p_t || p_s)."""
    z_s = F.linear(h_s, w_s)
    if z_t is None:
        z_t = F.linear(h_t, w_t)
    ce = F.cross_entropy(z_s, labels)
    if teacher in ("tied", "separate-full"):
        ce = ce + F.cross_entropy(z_t, labels)
    log_p_s = F.log_softmax(z_s / TEMP, dim=-1)
    p_t = F.softmax((z_t / TEMP).detach(), dim=-1)
    return ce + F.kl_div(log_p_s, p_t, reduction="batchmean") * (TEMP * TEMP)


def fused_loss(h_s, w_s, labels, teacher, z_t=None, h_t=None, w_t=None):
    import orda_ce_kernel as ok

    if teacher == "tied":
        t, tce = ok.TiedTeacher(h_t), 1.0
    elif teacher in ("separate-student", "separate-full"):
        t, tce = ok.SeparateTeacher(h_t, w_t), (1.0 if teacher == "separate-full" else 0.0)
    elif teacher == "precomputed-logits":
        t, tce = ok.PrecomputedTeacher(logits=z_t), 0.0
    else:
        t, tce = ok.PrecomputedTeacher(teacher_hidden=h_t, teacher_weight=w_t), 0.0
    return ok.distillation_loss(h_s, w_s, labels, t, student_ce_weight=1.0, teacher_ce_weight=tce, kl_weight=1.0,
                                kl_temperature=TEMP).loss


# ------------------------------------------------------------------------------------------ step
def make_step(backend, teacher, vocab, seq, device, dtype=torch.bfloat16):
    torch.manual_seed(0)
    student = TinyLM(vocab, STUDENT_CFG, seq).to(device=device, dtype=dtype)
    teacher_lm = TinyLM(vocab, TEACHER_CFG, seq).to(device=device, dtype=dtype).requires_grad_(False)
    opt = torch.optim.SGD(student.parameters(), lr=1e-3)
    ids = torch.randint(0, vocab, (BATCH, seq), device=device)
    labels = torch.randint(0, vocab, (BATCH * seq,), device=device)
    d = STUDENT_CFG["dim"]
    pre = {}
    if teacher.startswith("precomputed"):
        with torch.no_grad():
            h_t = teacher_lm.hidden(ids).view(-1, TEACHER_CFG["dim"])
            if teacher == "precomputed-logits":
                pre["z_t"] = F.linear(h_t, teacher_lm.head_weight)
            else:
                pre["h_t"], pre["w_t"] = h_t, teacher_lm.head_weight
        del teacher_lm
        teacher_lm = None

    def teacher_args(ids_in):
        if teacher_lm is None:
            return dict(pre)
        with torch.no_grad():
            h_t = teacher_lm.hidden(ids_in).view(-1, TEACHER_CFG["dim"])
        if teacher == "tied":
            return dict(h_t=h_t)
        return dict(h_t=h_t, w_t=teacher_lm.head_weight)

    loss_fn = torch_loss if backend == "torch-compile" else fused_loss

    def forward_and_loss(ids_in, labels_in):
        h_s = student.hidden(ids_in).view(-1, d)
        kw = teacher_args(ids_in)
        if teacher == "tied":
            kw["w_t"] = student.head_weight
        return loss_fn(h_s, student.head_weight, labels_in, teacher, **kw)

    if backend in ("torch-compile", "orda_b200-graph"):
        run = torch.compile(forward_and_loss)
    else:
        student.hidden = torch.compile(student.hidden)
        if teacher_lm is not None:
            teacher_lm.hidden = torch.compile(teacher_lm.hidden)
        run = forward_and_loss

    def step():
        opt.zero_grad(set_to_none=True)
        loss = run(ids, labels)
        loss.backward()
        opt.step()
        return loss

    return step


def time_backend(backend, teacher, vocab, seq, steps, device="cuda"):
    """(ms per step, peak MB during the timed steps); inf on out-of-memory."""
    torch._dynamo.reset()
    gc.collect()
    torch.cuda.empty_cache()
    try:
        step = make_step(backend, teacher, vocab, seq, device)
        for _ in range(WARMUP):
            step()
        torch.cuda.synchronize()
        torch.cuda.reset_peak_memory_stats()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            loss = step()
        e.record()
        torch.cuda.synchronize()
        if not math.isfinite(float(loss)):
            raise RuntimeError(f"{backend}: non-finite loss")
        res = (s.elapsed_time(e) / steps, torch.cuda.max_memory_allocated() / 1024 ** 2)
    except torch.cuda.OutOfMemoryError:
        res = (float("inf"), float("inf"))
    del step
    torch._dynamo.reset()
    gc.collect()
    torch.cuda.empty_cache()
    return res


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--teacher", default="separate-student", choices=TEACHERS)
    p.add_argument("--vocabs", type=int, nargs="+", default=[32_768])
    p.add_argument("--seqs", type=int, nargs="+", default=[512, 1024, 2048])
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--passes", type=int, default=2)
    p.add_argument("--backends", nargs="+", default=BACKENDS, choices=BACKENDS)
    p.add_argument("--json", default=None)
    a = p.parse_args(argv)
    if not torch.cuda.is_available():
        raise RuntimeError("the training-step benchmark needs a CUDA device (B200)")
    records = []
    for vocab in a.vocabs:
        for seq in a.seqs:
            acc = {b: [] for b in a.backends}
            for ps in range(a.passes):
                order = a.backends if ps % 2 == 0 else list(reversed(a.backends))
                for b in order:
                    acc[b].append(time_backend(b, a.teacher, vocab, seq, a.steps))
            print(f"\n-- {a.teacher}  vocab={vocab // 1024}k  seq={seq}  batch={BATCH}")
            rec = {"teacher": a.teacher, "vocab": vocab, "seq": seq, "batch": BATCH}
            for b in a.backends:
                ms = sum(x[0] for x in acc[b]) / len(acc[b])
                mb = max(x[1] for x in acc[b])
                rec[b] = {"ms_per_step": ms, "peak_mb": mb}
                print(f"   {b:>16}  {ms:9.2f} ms  {mb:10.1f} MB")
            base = rec.get("torch-compile")
            for b in a.backends:
                if b != "torch-compile" and base and math.isfinite(base["ms_per_step"]):
                    r = rec[b]
                    print(f"   {b} vs torch-compile: {r['ms_per_step'] - base['ms_per_step']:+.2f} ms "
                          f"({(r['ms_per_step'] / base['ms_per_step'] - 1) * 100:+.1f}%)  "
                          f"{r['peak_mb'] - base['peak_mb']:+.1f} MB "
                          f"({(r['peak_mb'] / base['peak_mb'] - 1) * 100:+.1f}%)")
            records.append(rec)
    write_json(a.json, {"gpu": torch.cuda.get_device_name(), "records": records})
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
