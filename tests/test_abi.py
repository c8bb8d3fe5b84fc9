"""C ABI checks that need no GPU: the library loads, exports every declared symbol, and its
argument struct matches the Python mirror."""
from __future__ import annotations

import ctypes
import glob
import os
import re

import pytest

from orda_ce_kernel import _native

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*\s*\*?\s*(orda_[a-z0-9_]+)\s*\(", text, re.M):
            names.add(m.group(1))
    return names


def test_library_loads_and_version():
    lib = _native.load()
    assert lib.orda_abi_version() == _native.ABI_VERSION
    assert lib.orda_args_struct_size() == ctypes.sizeof(_native.DistillArgs)


def test_every_declared_symbol_is_exported():
    lib = _native.load()
    declared = _declared_functions()
    assert declared, "no declarations found in include/*.h"
    assert declared == set(_native.EXPORTED_SYMBOLS)
    for name in declared:
        assert hasattr(lib, name), name


def test_status_strings():
    lib = _native.load()
    for code in range(0, 9):
        assert lib.orda_status_string(code)
    assert b"unknown" in lib.orda_status_string(999)


def _args(**kw):
    a = _native.DistillArgs()
    a.abi_version = _native.ABI_VERSION
    a.teacher_mode = _native.TEACHER_TIED
    a.compute_dtype = _native.BF16
    a.n_rows, a.hidden, a.teacher_hidden, a.vocab = 8192, 4096, 4096, 128256
    a.vocab_offset, a.vocab_total = 0, 128256
    a.student_hidden = a.weight = a.labels = a.out_reduced = a.device_status = 16
    a.kl_temperature = 1.0
    a.student_ce_weight = 1.0
    a.teacher_ce_weight = 1.0
    a.kl_weight = 1.0
    a.need_grad_student_hidden = a.need_grad_weight = 1
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_workspace_is_bounded_and_host_only():
    lib = _native.load()
    a = _args()
    ws = lib.orda_distill_workspace_bytes(a)
    # two 16-bit logits chunks bounded by 2 GiB plus statistics
    assert 0 < ws < (2 << 30) + 512 * (1 << 20)
    a.chunk_rows = 1024
    ws_small = lib.orda_distill_workspace_bytes(a)
    assert ws_small < ws
    bad = _args(abi_version=99)
    assert lib.orda_distill_workspace_bytes(bad) == 0


@pytest.mark.parametrize("field,value", [("n_rows", 0), ("kl_temperature", 0.0), ("kl_weight", -1.0),
                                         ("compute_dtype", 7), ("teacher_mode", 9)])
def test_invalid_arguments_rejected_without_launch(field, value):
    lib = _native.load()
    a = _args(**{field: value})
    assert lib.orda_distill_fwdbwd(a, None, 0, None) == _native.ERR_INVALID_ARGUMENT


def test_precomputed_teacher_ce_unsupported():
    lib = _native.load()
    a = _args(teacher_mode=_native.TEACHER_LOGITS, teacher_ce_weight=1.0)
    assert lib.orda_distill_fwdbwd(a, None, 0, None) == _native.ERR_UNSUPPORTED


def test_workspace_too_small_rejected():
    lib = _native.load()
    a = _args(teacher_hidden_ptr=16, ld_student_hidden=4096, ld_weight=4096, ld_teacher_hidden=4096,
              grad_student_hidden=16, grad_weight=16)
    assert lib.orda_distill_fwdbwd(a, 256, 256, None) == _native.ERR_WORKSPACE
