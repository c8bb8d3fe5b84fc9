"""GPU smoke versions of the user benchmarks (the "next" rows): the accuracy benchmark's protocol on
one 8192-row configuration for every teacher mode, the VRAM benchmark on one shape against the
reference's published figure, and two steps of the training-step benchmark.

Reference protocols: test/benchmark/src/_accuracy.py:331-420 (accuracy), _vram.py:435-673 (VRAM),
_train.py:102-452 (training step).
"""
from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

pytest.importorskip("orda_ce_kernel")
from orda_ce_kernel.benchmarks import accuracy, train_step, vram  # noqa: E402


@pytest.mark.parametrize("component", ["ce", "kl"])
def test_accuracy_within_the_reference_b200_errors(component):
    """Every teacher mode at (batch 8, seq 1024): the relative error of the loss component against the
    fp32 formula is at most the largest one the reference's kernels showed on a B200
    (logs/NVIDIA_B200/bench_accuracy_{ce,kl}_*.log: 2.01e-6 CE, 1.40e-5 KL)."""
    rows = accuracy.measure(component, batch_seqs=[(8, 1024)], use_compile=False)
    assert len(rows) == len(accuracy.MODES)
    bound = accuracy.REFERENCE_B200_MAX[component]["rel"]
    for r in rows:
        rec = r["orda_b200"]
        assert rec["rel_err"] <= bound, (r["mode"], rec["rel_err"], bound)
        assert rec["grad_cos"] > 0.9999, (r["mode"], rec["grad_cos"])


def test_vram_below_the_reference_kernels():
    """Tied teacher, dim 1024, vocab 64k, seq 2048, batch 16: the reference's kernels need 1236.4 MB
    of extra memory for one loss + backward (logs/Tesla_T4/bench_vram_TiedTeacher_20260705_192312.log)."""
    extra = vram.measure_once("tied", "orda_b200", 65_536, 1024, 2048)
    assert math.isfinite(extra)
    assert extra < 1236.4, extra


def test_training_step_runs_and_updates():
    """Two steps of the training benchmark (own small decoder, separate teacher, the fused loss as
    its head): the losses are finite and the second differs from the first (the optimizer step used
    the fused gradients)."""
    step = train_step.make_step("orda_b200", "separate-student", 32_768, 256, "cuda")
    l1 = float(step())
    l2 = float(step())
    assert math.isfinite(l1) and math.isfinite(l2)
    assert l1 != l2
