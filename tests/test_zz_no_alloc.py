"""The allocation-free entry point ``orda_distill_fwdbwd_static_ws``.

Some callers cannot allocate device memory themselves (a host runtime that only hands out
pre-registered buffers, or code where a cudaMalloc is forbidden or would synchronise). For them the
library keeps its scratch in one fixed 32 MiB array. This test calls that entry point through the C
ABI, twice in a row (the array keeps the previous call's contents), and checks every output against
the regular ``orda_distill_fwdbwd`` with a caller-provided workspace. This file is named so pytest
collects it last.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(n, h, v, seed):
    g = torch.Generator().manual_seed(seed)
    hs = torch.randn(n, h, generator=g).to(torch.bfloat16).cuda()
    ht = torch.randn(n, h, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(v, h, generator=g) * 0.02).to(torch.bfloat16).cuda()
    labels = torch.randint(0, v, (n,), generator=g)
    labels[::17] = -100
    return hs, ht, w, labels.cuda()


def _run(lib, native, hs, ht, w, labels, static):
    n, h = hs.shape
    v = w.shape[0]
    out = torch.empty(native.OUT_SLOTS, dtype=torch.float32, device="cuda")
    g_hs = torch.empty_like(hs)
    g_w = torch.empty(v, h, dtype=torch.float32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    a = native.DistillArgs()
    a.abi_version = native.ABI_VERSION
    a.teacher_mode = native.TEACHER_TIED
    a.compute_dtype = native.BF16
    a.n_rows, a.hidden, a.teacher_hidden, a.vocab, a.vocab_offset, a.vocab_total = n, h, h, v, 0, v
    a.student_hidden, a.ld_student_hidden = hs.data_ptr(), h
    a.weight, a.ld_weight = w.data_ptr(), h
    a.teacher_hidden_ptr, a.ld_teacher_hidden = ht.data_ptr(), h
    a.labels = labels.data_ptr()
    a.student_ce_weight, a.teacher_ce_weight, a.kl_weight, a.kl_temperature = 1.0, 1.0, 0.5, 1.5
    a.divergence = native.DIV_FORWARD
    a.ignore_index = -100
    a.reduction = native.REDUCTION_MEAN
    a.need_grad_student_hidden = a.need_grad_weight = 1
    a.out_reduced = out.data_ptr()
    a.grad_student_hidden, a.grad_weight = g_hs.data_ptr(), g_w.data_ptr()
    a.grad_weight_fp32 = 1
    a.device_status = status.data_ptr()
    stream = torch.cuda.current_stream().cuda_stream
    if static:
        rc = lib.orda_distill_fwdbwd_static_ws(ctypes.byref(a), stream)
    else:
        ws_bytes = lib.orda_distill_workspace_bytes(ctypes.byref(a))
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        rc = lib.orda_distill_fwdbwd(ctypes.byref(a), ws.data_ptr(), ws_bytes, stream)
    assert rc == 0, native.status_string(rc)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out.clone(), g_hs.float(), g_w


def _rel(a, b):
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.parametrize("shape", [(300, 256, 3000), (600, 512, 32000)])  # the second needs several chunks
def test_static_workspace_matches_workspace_entry_point_twice(shape):
    from orda_ce_kernel import _native

    lib = _native.load()
    hs, ht, w, labels = _case(*shape, seed=7)
    ref_out, ref_hs, ref_w = _run(lib, _native, hs, ht, w, labels, static=False)
    for _ in range(2):
        out, g_hs, g_w = _run(lib, _native, hs, ht, w, labels, static=True)
        torch.testing.assert_close(out[:4], ref_out[:4], rtol=1e-5, atol=1e-6)
        assert _rel(g_hs, ref_hs) < 2e-2
        assert _rel(g_w, ref_w) < 2e-2


def test_static_workspace_rejects_problems_that_do_not_fit():
    from orda_ce_kernel import _native

    lib = _native.load()
    hs, ht, w, labels = _case(128, 64, 131072, seed=3)  # 128 rows x 2 x 128k vocab x 2 B > 32 MiB
    out = torch.empty(_native.OUT_SLOTS, dtype=torch.float32, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    a = _native.DistillArgs()
    a.abi_version = _native.ABI_VERSION
    a.teacher_mode = _native.TEACHER_TIED
    a.compute_dtype = _native.BF16
    a.n_rows, a.hidden, a.teacher_hidden, a.vocab, a.vocab_total = 128, 64, 64, 131072, 131072
    a.student_hidden, a.ld_student_hidden = hs.data_ptr(), 64
    a.weight, a.ld_weight = w.data_ptr(), 64
    a.teacher_hidden_ptr, a.ld_teacher_hidden = ht.data_ptr(), 64
    a.labels = labels.data_ptr()
    a.student_ce_weight, a.teacher_ce_weight, a.kl_weight, a.kl_temperature = 1.0, 1.0, 1.0, 1.0
    a.ignore_index = -100
    a.need_grad_student_hidden = 1  # gradients need the logits chunk buffers, which do not fit
    a.out_reduced = out.data_ptr()
    a.device_status = status.data_ptr()
    assert lib.orda_distill_fwdbwd_static_ws(ctypes.byref(a), torch.cuda.current_stream().cuda_stream) == _native.ERR_WORKSPACE
