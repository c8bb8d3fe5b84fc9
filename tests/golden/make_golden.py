"""Generate the golden fixtures that pin ``oracle/distill_oracle.py`` to the reference.

Run in a container where the reference package is importable (its ``src/`` directory, or an
installed copy) - it is not needed afterwards; the ``.npz`` files it writes are committed:

    PYTHONPATH=<reference>/src python tests/golden/make_golden.py

Every case calls the reference's own PyTorch implementation, ``orda_ce_kernel.api._torch_reference``
(``src/orda_ce_kernel/api.py:274-335``), on float64 leaves and back-propagates with autograd, so the
stored losses and gradients are the reference's outputs. Shapes, weights and seeds follow the
reference's CPU correctness tests (``test/correctness/test_torch_backend_cpu.py``: seeds 101-106,
weights 0.8/0.25/0.35, T=1.4/1.6/1.5/1.7, the all-ignored case) plus the small end of
benchmark config 1 (student-only CE) and config 2 (precomputed fp32 log-softmax teacher, T=2).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference():
    # the reference package: its source tree (ORDA_REFERENCE_SRC) or the copy installed in baseline/_ref
    for cand in (os.environ.get("ORDA_REFERENCE_SRC"), os.path.join(HERE, "..", "..", "baseline", "_ref")):
        if cand and os.path.isdir(os.path.join(cand, "orda_ce_kernel")):
            sys.path.insert(0, cand)
            break
    import orda_ce_kernel.api as ref_api  # noqa: E402

    return ref_api


def _inputs(seed, n, h, v, ht=None, ignore_every=None, logits=False, all_ignored=False):
    g = torch.Generator().manual_seed(seed)
    d = {
        "student_hidden": torch.randn(n, h, generator=g, dtype=torch.float64) * 0.1,
        "weight": torch.randn(v, h, generator=g, dtype=torch.float64) * 0.1,
    }
    if ht is not None:
        d["teacher_hidden"] = torch.randn(n, ht, generator=g, dtype=torch.float64) * 0.1
        d["teacher_weight"] = torch.randn(v, ht, generator=g, dtype=torch.float64) * 0.1
    if logits:
        d["teacher_logits"] = torch.log_softmax(torch.randn(n, v, generator=g, dtype=torch.float64) * 2.0, -1)
    labels = torch.randint(0, v, (n,), generator=g)
    if ignore_every:
        labels[::ignore_every] = -100
    if all_ignored:
        labels[:] = -100
    d["labels"] = labels
    return d


CASES = [
    # name, mode, inputs kwargs, loss kwargs
    ("tied_mean", "tied", dict(seed=101, n=9, h=7, v=17, ht=7, ignore_every=2),
     dict(student_ce_weight=0.8, teacher_ce_weight=0.25, kl_weight=0.35, kl_temperature=1.4, reduction="mean")),
    ("tied_sum", "tied", dict(seed=101, n=9, h=7, v=17, ht=7, ignore_every=2),
     dict(student_ce_weight=0.8, teacher_ce_weight=0.25, kl_weight=0.35, kl_temperature=1.4, reduction="sum")),
    ("tied_default_tce_t1", "tied", dict(seed=107, n=12, h=8, v=23, ht=8, ignore_every=4),
     dict(kl_weight=0.5, kl_temperature=1.0, reduction="mean")),
    ("separate_pure_kd", "separate", dict(seed=102, n=10, h=6, v=19, ht=8, ignore_every=2),
     dict(kl_weight=0.4, kl_temperature=1.6, reduction="mean")),
    ("separate_full", "separate", dict(seed=103, n=10, h=6, v=19, ht=8, ignore_every=2),
     dict(teacher_ce_weight=0.6, kl_weight=0.4, kl_temperature=1.6, reduction="mean")),
    ("precomputed_logits", "precomputed_logits", dict(seed=104, n=11, h=9, v=21, logits=True, ignore_every=3),
     dict(kl_weight=0.3, kl_temperature=2.0, student_ce_weight=0.5, reduction="mean")),
    ("precomputed_hidden", "precomputed_hidden", dict(seed=105, n=11, h=9, v=21, ht=5, ignore_every=3),
     dict(kl_weight=0.3, kl_temperature=1.5, reduction="sum")),
    ("all_ignored", "tied", dict(seed=106, n=8, h=6, v=13, ht=6, all_ignored=True),
     dict(kl_weight=0.5, kl_temperature=1.7, reduction="mean")),
    ("student_only_cfg1_small", "tied", dict(seed=0, n=64, h=32, v=96, ht=32, ignore_every=20),
     dict(teacher_ce_weight=0.0, kl_weight=0.0, reduction="mean")),
    ("swapped_for_reverse_pin", "precomputed_logits", dict(seed=108, n=7, h=5, v=15, logits=True, ignore_every=3),
     dict(kl_weight=1.0, kl_temperature=1.5, student_ce_weight=0.0, reduction="sum")),
]


def run_case(ref_api, mode, inp, kw):
    hs = inp["student_hidden"].clone().requires_grad_(True)
    w = inp["weight"].clone().requires_grad_(True)
    labels = inp["labels"]
    ht = wt = None
    if mode == "tied":
        ht = inp["teacher_hidden"].clone().requires_grad_(True)
        teacher = ref_api.TiedTeacher(ht)
    elif mode == "separate":
        full = kw.get("teacher_ce_weight") not in (None, 0.0)
        ht = inp["teacher_hidden"].clone().requires_grad_(full)
        wt = inp["teacher_weight"].clone().requires_grad_(full)
        teacher = ref_api.SeparateTeacher(ht, wt)
    elif mode == "precomputed_logits":
        teacher = ref_api.PrecomputedTeacher(logits=inp["teacher_logits"])
    else:
        teacher = ref_api.PrecomputedTeacher(teacher_hidden=inp["teacher_hidden"], teacher_weight=inp["teacher_weight"])
    tce = ref_api._resolve_teacher_ce_weight(mode.split("_")[0], kw.get("teacher_ce_weight"))
    out = ref_api._torch_reference(
        student_hidden=hs, weight=w, labels=labels, teacher=teacher,
        student_ce_weight=kw.get("student_ce_weight", 1.0), teacher_ce_weight=tce,
        kl_weight=kw.get("kl_weight", 0.0), kl_temperature=kw.get("kl_temperature", 1.0),
        ignore_index=-100, reduction=kw.get("reduction", "mean"),
    )
    out.loss.backward()
    res = {
        "out_loss": out.loss.detach().numpy(), "out_student_ce": out.student_ce.numpy(),
        "out_teacher_ce": out.teacher_ce.numpy(), "out_kl": out.kl.numpy(),
        "grad_student_hidden": hs.grad.numpy(), "grad_weight": w.grad.numpy(),
    }
    if ht is not None and ht.grad is not None:
        res["grad_teacher_hidden"] = ht.grad.numpy()
    if wt is not None and wt.grad is not None:
        res["grad_teacher_weight"] = wt.grad.numpy()
    return res


def main():
    ref_api = _import_reference()
    for name, mode, ikw, kw in CASES:
        inp = _inputs(**ikw)
        res = run_case(ref_api, mode, inp, kw)
        arrays = {f"in_{k}": v.numpy() for k, v in inp.items()}
        arrays.update(res)
        meta = dict(kw)
        meta["mode"] = mode
        arrays["meta"] = np.array(repr(meta))
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
        print(f"wrote {name}: loss={float(res['out_loss']):.10g}")


if __name__ == "__main__":
    main()
