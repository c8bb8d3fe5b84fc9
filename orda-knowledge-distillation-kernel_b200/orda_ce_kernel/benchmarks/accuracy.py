"""Loss and gradient accuracy of the fused bf16 kernels against an fp32 PyTorch formula.

    python -m orda_ce_kernel.benchmarks.accuracy [--component ce|kl|both] [--no-compile] [--json out.json]

Same protocol as the reference's accuracy benchmark (``test/benchmark/src/_accuracy.py:331-420``,
``bench_accuracy_ce.py``, ``bench_accuracy_kl.py``): vocab 32768, student and teacher dim 1024,
(batch, seq) in {(32, 256), (16, 512), (8, 1024)} (8192 rows each), T = 1.7, inputs N(0, 0.1^2),
every (rows / 8)-th label ignored, the five teacher modes. For each case the fp32 baseline is a plain
PyTorch formula on the fp32 inputs; the kernels (and, optionally, ``torch.compile`` of the same
formula) run on the bf16-rounded inputs. Component ``ce`` is ``student_ce + teacher_ce`` with weights
(1, teacher CE weight of the mode, KL 0); component ``kl`` is the KL term alone (weights 0, 0, 1).
Reported per case: the value, its absolute and relative error, and for the student-hidden gradient the
cosine similarity, mean and max absolute error against the baseline's.
"""
from __future__ import annotations

import argparse

import torch
import torch.nn.functional as F

from ._common import IGNORE_INDEX, fmt_float, print_table, seeded_labels, seeded_randn, write_json

TEMP = 1.7
VOCAB = 32_768
DIM = 1_024
BATCH_SEQS = [(32, 256), (16, 512), (8, 1_024)]
MODES = ["tied", "separate-student", "separate-full", "precomputed-logits", "precomputed-hidden"]

# Largest errors of the reference's fused kernels on a B200 with this protocol
# (logs/NVIDIA_B200/bench_accuracy_ce_20260705_201534.log, bench_accuracy_kl_20260705_201723.log).
REFERENCE_B200_MAX = {"ce": {"abs": 4.196167e-05, "rel": 2.007572e-06},
                      "kl": {"abs": 1.430511e-06, "rel": 1.396960e-05}}


def make_case(mode: str, bt: int, *, seed: int, device) -> dict:
    """fp32 tensors of one case (the bf16 inputs are their rounding)."""
    s = seed * 16
    c = {"labels": seeded_labels(bt, VOCAB, seed=s, device=device, ignore_every=bt // 8),
         "hs": seeded_randn((bt, DIM), seed=s + 1, device=device, scale=0.1),
         "w": seeded_randn((VOCAB, DIM), seed=s + 2, device=device, scale=0.1)}
    if mode == "tied":
        c["ht"] = seeded_randn((bt, DIM), seed=s + 3, device=device, scale=0.1)
    elif mode in ("separate-student", "separate-full", "precomputed-hidden"):
        c["ht"] = seeded_randn((bt, DIM), seed=s + 3, device=device, scale=0.1)
        c["wt"] = seeded_randn((VOCAB, DIM), seed=s + 4, device=device, scale=0.1)
    else:
        c["tl"] = seeded_randn((bt, VOCAB), seed=s + 5, device=device, scale=0.1)
    return c


def teacher_ce_weight(mode: str) -> float:
    return {"tied": 1.0, "separate-full": 1.0}.get(mode, 0.0)


def component_weights(mode: str, component: str) -> tuple[float, float, float]:
    return (1.0, teacher_ce_weight(mode), 0.0) if component == "ce" else (0.0, 0.0, 1.0)


def formula(hs, w, labels, *, ht=None, wt=None, tl=None, tce=0.0, component="ce"):
    """Plain PyTorch restatement of the loss components (mean over non-ignored rows)."""
    z_s = hs @ w.t()
    z_t = tl if tl is not None else ht @ (wt if wt is not None else w).t()
    valid = labels != IGNORE_INDEX
    denom = valid.sum().clamp_min(1)
    if component == "ce":
        loss = F.cross_entropy(z_s, labels, ignore_index=IGNORE_INDEX, reduction="sum") / denom
        if tce != 0.0:
            loss = loss + tce * F.cross_entropy(z_t, labels, ignore_index=IGNORE_INDEX, reduction="sum") / denom
        return loss
    log_p_s = F.log_softmax(z_s / TEMP, dim=-1)
    log_p_t = F.log_softmax(z_t.detach() / TEMP, dim=-1)
    kl_rows = (log_p_t.exp() * (log_p_t - log_p_s)).sum(-1) * (TEMP * TEMP)
    return kl_rows.masked_fill(~valid, 0.0).sum() / denom


def _formula_args(mode, c):
    if mode == "tied":
        return dict(ht=c["ht"])
    if mode == "precomputed-logits":
        return dict(tl=c["tl"])
    return dict(ht=c["ht"], wt=c["wt"])


def run_baseline(mode, c, component):
    hs = c["hs"].clone().requires_grad_(True)
    loss = formula(hs, c["w"], c["labels"], tce=teacher_ce_weight(mode), component=component, **_formula_args(mode, c))
    loss.backward()
    return float(loss.detach().double()), hs.grad.float()


def run_compiled(mode, c16, component, cache):
    key = component
    if key not in cache:
        cache[key] = torch.compile(formula, dynamic=False)
    hs = c16["hs"].clone().requires_grad_(True)
    loss = cache[key](hs, c16["w"], c16["labels"], tce=teacher_ce_weight(mode), component=component,
                      **_formula_args(mode, c16))
    loss.backward()
    return float(loss.detach().double()), hs.grad.float()


def run_kernels(mode, c16, component):
    import orda_ce_kernel as ok

    hs = c16["hs"].clone().requires_grad_(True)
    w = c16["w"].clone().requires_grad_(True)
    if mode == "tied":
        teacher = ok.TiedTeacher(c16["ht"])
    elif mode in ("separate-student", "separate-full"):
        teacher = ok.SeparateTeacher(c16["ht"], c16["wt"])
    elif mode == "precomputed-logits":
        teacher = ok.PrecomputedTeacher(logits=c16["tl"])
    else:
        teacher = ok.PrecomputedTeacher(teacher_hidden=c16["ht"], teacher_weight=c16["wt"])
    ws, wt, wk = component_weights(mode, component)
    out = ok.distillation_loss(hs, w, c16["labels"], teacher, student_ce_weight=ws, teacher_ce_weight=wt,
                               kl_weight=wk, kl_temperature=TEMP)
    out.loss.backward()
    value = out.student_ce + out.teacher_ce if component == "ce" else out.kl
    return float(value.double()), hs.grad.float()


def grad_metrics(expected: torch.Tensor, actual: torch.Tensor) -> tuple[float, float, float]:
    e, a = expected.flatten(), actual.flatten()
    cos = float(F.cosine_similarity(e.double(), a.double(), dim=0, eps=1e-30))
    d = (e - a).abs()
    return cos, float(d.mean()), float(d.max())


def measure(component: str, *, batch_seqs=BATCH_SEQS, modes=MODES, use_compile=True, device="cuda") -> list[dict]:
    """One record per (config, mode) with the baseline value and the errors of each backend."""
    rows, cache = [], {}
    for ci, (batch, seq) in enumerate(batch_seqs):
        bt = batch * seq
        for mi, mode in enumerate(modes):
            c = make_case(mode, bt, seed=10_000 + ci * 100 + mi, device=device)
            c16 = {k: (v.to(torch.bfloat16) if v.is_floating_point() else v) for k, v in c.items()}
            exp, exp_g = run_baseline(mode, c, component)
            rec = {"config": f"vocab={VOCAB // 1024}k seq={seq} batch={batch} dim={DIM}", "mode": mode, "fp32": exp}
            backends = [("orda_b200", run_kernels)]
            if use_compile:
                backends.insert(0, ("torch_compile", lambda m, cc, comp: run_compiled(m, cc, comp, cache)))
            for name, fn in backends:
                val, g = fn(mode, c16, component)
                cos, gmean, gmax = grad_metrics(exp_g, g)
                err = abs(val - exp)
                rec[name] = {"value": val, "abs_err": err, "rel_err": err / max(abs(exp), 1e-12),
                             "grad_cos": cos, "grad_mean_abs_err": gmean, "grad_max_abs_err": gmax}
            rows.append(rec)
            del c, c16
            torch.cuda.empty_cache()
    return rows


def print_report(component: str, rows: list[dict]) -> dict:
    names = [n for n in ("torch_compile", "orda_b200") if n in rows[0]]
    loss_rows, grad_rows = [], []
    for r in rows:
        lr, gr = [r["config"], r["mode"], fmt_float(r["fp32"])], [r["config"], r["mode"]]
        for n in names:
            b = r[n]
            lr += [fmt_float(b["value"]), fmt_float(b["abs_err"]), fmt_float(b["rel_err"])]
            gr += [f"{b['grad_cos']:.8f}", fmt_float(b["grad_mean_abs_err"]), fmt_float(b["grad_max_abs_err"])]
        loss_rows.append(lr)
        grad_rows.append(gr)
    lh, gh = ["config", "mode", "fp32"], ["config", "mode"]
    for n in names:
        lh += [n, f"{n}_abs_err", f"{n}_rel_err"]
        gh += [f"{n}_grad_cos", f"{n}_grad_mean", f"{n}_grad_max"]
    print_table(lh, loss_rows, title=f"loss ({component})")
    print_table(gh, grad_rows, title="grad student_hidden")
    summary = {}
    for n in names:
        summary[n] = {"max_abs_err": max(r[n]["abs_err"] for r in rows),
                      "max_rel_err": max(r[n]["rel_err"] for r in rows),
                      "min_grad_cos": min(r[n]["grad_cos"] for r in rows)}
        print(f"{n} max abs_err: {summary[n]['max_abs_err']:.6e}   max rel_err: {summary[n]['max_rel_err']:.6e}")
    ref = REFERENCE_B200_MAX[component]
    print(f"reference kernels on B200 (published log) max abs_err: {ref['abs']:.6e}   max rel_err: {ref['rel']:.6e}")
    summary["reference_b200_published"] = ref
    return summary


def main(argv=None) -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--component", default="both", choices=["ce", "kl", "both"])
    p.add_argument("--no-compile", action="store_true", help="skip the torch.compile column")
    p.add_argument("--json", default=None, help="write the records and the summary here")
    a = p.parse_args(argv)
    if not torch.cuda.is_available():
        raise RuntimeError("the accuracy benchmark needs a CUDA device (B200)")
    torch.backends.cuda.matmul.allow_tf32 = False  # the fp32 baseline uses full fp32 GEMMs
    out = {}
    for comp in (["ce", "kl"] if a.component == "both" else [a.component]):
        rows = measure(comp, use_compile=not a.no_compile)
        out[comp] = {"rows": rows, "summary": print_report(comp, rows)}
    out["gpu"] = torch.cuda.get_device_name()
    write_json(a.json, out)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
