"""Host-side pieces of bench.py (no GPU): the roofline peaks from the measured-peaks file or the
stated fallback, the SM reserve of the overlapped all-reduce, and the command-line defaults."""
from __future__ import annotations

import json
import sys

import bench


def test_peaks_from_file_and_fallback(tmp_path, monkeypatch):
    (tmp_path / "MEASURED_PEAKS.json").write_text(json.dumps(
        {"bf16_tflops": 1600.0, "bf16_tflops_sustained": 1400.0, "hbm_gbs": 6500.0}))
    monkeypatch.setattr(bench, "ROOT", str(tmp_path))
    assert bench._peaks() == (1600.0, 1400.0, 6500.0, "measured")
    monkeypatch.setattr(bench, "ROOT", str(tmp_path / "missing"))
    burst, sustained, hbm, src = bench._peaks()
    assert src == "fallback" and burst > sustained > 0 and hbm > 0


def test_reserve_and_cli_defaults(monkeypatch):
    assert bench.default_reserve_sms(1) == 16 and bench.default_reserve_sms(2) == 16
    assert bench.default_reserve_sms(8) == 32
    monkeypatch.setattr(sys, "argv", ["bench.py"])
    a = bench._args()
    assert (a.gpus, a.steps, a.impl, a.rows, a.reserve_sms) == (1, 10, "ours", 8192, -1)
    assert a.warmup >= 3
