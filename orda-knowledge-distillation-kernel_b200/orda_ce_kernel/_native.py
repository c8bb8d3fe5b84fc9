"""ctypes binding of the C ABI in ``include/orda_b200.h`` (``liborda_b200.so``).

The library is built in-tree (``orda-knowledge-distillation-kernel_b200/build.py``) and loaded from
this package directory. There is no fallback: if the library is missing or cannot be loaded, every
entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

LIB_NAME = "liborda_b200.so"
LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), LIB_NAME)

ABI_VERSION = 1

# status codes
OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_ALIGNMENT = 2
ERR_WORKSPACE = 3
ERR_UNSUPPORTED = 4
ERR_CUDA = 5
ERR_TIMEOUT = 6
ERR_LABEL_RANGE = 7

# dtypes
F32, F16, BF16 = 0, 1, 2
# teacher modes
TEACHER_TIED, TEACHER_SEPARATE, TEACHER_LOGITS, TEACHER_HIDDEN = 0, 1, 2, 3
# divergences
DIV_FORWARD, DIV_REVERSE, DIV_JSD = 0, 1, 2
REDUCTION_MEAN, REDUCTION_SUM = 0, 1

OUT_LOSS, OUT_STUDENT_CE, OUT_TEACHER_CE, OUT_KL, OUT_MEAN_SCALE = 0, 1, 2, 3, 4
OUT_SUM_STUDENT_CE, OUT_SUM_TEACHER_CE, OUT_SUM_KL, OUT_COUNT = 5, 6, 7, 8
OUT_SLOTS = 9
ROW_STATS = 16
STATIC_WORKSPACE_BYTES = 32 << 20
PHASE_LOGITS, PHASE_ROWS, PHASE_DHIDDEN, PHASE_DWEIGHT = 0, 1, 2, 3
PHASES = 4

_i32, _i64, _f32, _vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p


class DistillArgs(ctypes.Structure):
    """Mirror of ``orda_distill_args_t`` (field order and types must match the header)."""

    _fields_ = [
        ("abi_version", _i32), ("teacher_mode", _i32), ("compute_dtype", _i32), ("teacher_logits_dtype", _i32),
        ("n_rows", _i64), ("hidden", _i64), ("teacher_hidden", _i64), ("vocab", _i64),
        ("vocab_offset", _i64), ("vocab_total", _i64),
        ("student_hidden", _vp), ("ld_student_hidden", _i64),
        ("weight", _vp), ("ld_weight", _i64),
        ("teacher_hidden_ptr", _vp), ("ld_teacher_hidden", _i64),
        ("teacher_weight", _vp), ("ld_teacher_weight", _i64),
        ("teacher_logits", _vp), ("ld_teacher_logits", _i64),
        ("labels", _vp),
        ("student_ce_weight", _f32), ("teacher_ce_weight", _f32), ("kl_weight", _f32),
        ("kl_temperature", _f32), ("jsd_beta", _f32),
        ("divergence", _i32),
        ("ignore_index", _i64),
        ("reduction", _i32), ("validate_labels", _i32),
        ("need_grad_student_hidden", _i32), ("need_grad_weight", _i32),
        ("need_grad_teacher_hidden", _i32), ("need_grad_teacher_weight", _i32),
        ("chunk_rows", _i64),
        ("out_reduced", _vp), ("out_row_losses", _vp),
        ("grad_student_hidden", _vp), ("grad_weight", _vp),
        ("grad_teacher_hidden", _vp), ("grad_teacher_weight", _vp),
        ("grad_weight_fp32", _i32),
        ("device_status", _vp),
        ("phase_events", _vp),
        ("dweight_done_event", _vp),
        ("dweight_first", _i32),
        ("grads_include_mean_scale", _i32),
        ("overlap_reserve_sms", _i32),
    ]


MAX_PEERS = 8


class PeerSlots(ctypes.Structure):
    """Mirror of orda_peer_slots_t (include/orda_b200.h)."""

    _fields_ = [
        ("world", _i32), ("rank", _i32), ("slab_rows", _i64),
        ("slot_base", _vp * MAX_PEERS), ("grad_base", _vp * MAX_PEERS),
    ]


class IpcHandle(ctypes.Structure):
    """Mirror of orda_ipc_handle_t (include/orda_b200.h)."""

    _fields_ = [("handle", ctypes.c_uint8 * 64), ("offset", ctypes.c_uint64)]


# every symbol include/orda_b200.h and include/orda_b200_testing.h declare
EXPORTED_SYMBOLS = (
    "orda_abi_version",
    "orda_args_struct_size",
    "orda_kernel_launches",
    "orda_status_string",
    "orda_distill_workspace_bytes",
    "orda_distill_fwdbwd",
    "orda_distill_fwdbwd_static_ws",
    "orda_distill_fwdbwd_peer",
    "orda_peer_reduce_broadcast",
    "orda_ipc_export",
    "orda_ipc_import",
    "orda_ipc_close",
    "orda_scale_grad",
    "orda_shard_workspace_bytes",
    "orda_shard_forward",
    "orda_merge_row_stats",
    "orda_shard_jsd_partials",
    "orda_shard_backward",
    "orda_debug_gemm",
    "orda_debug_gemm_pair",
    "orda_debug_gemm_profile",
    "orda_debug_gemm_wide",
    "orda_debug_wait_timeout",
)

_lib = None
_lib_lock = threading.Lock()
_load_error: str | None = None


def _declare(lib):
    P = ctypes.POINTER(DistillArgs)
    lib.orda_abi_version.restype = _i32
    lib.orda_abi_version.argtypes = []
    lib.orda_args_struct_size.restype = ctypes.c_size_t
    lib.orda_args_struct_size.argtypes = []
    lib.orda_kernel_launches.restype = ctypes.c_uint64
    lib.orda_kernel_launches.argtypes = []
    lib.orda_status_string.restype = ctypes.c_char_p
    lib.orda_status_string.argtypes = [_i32]
    lib.orda_distill_workspace_bytes.restype = ctypes.c_size_t
    lib.orda_distill_workspace_bytes.argtypes = [P]
    lib.orda_distill_fwdbwd.restype = _i32
    lib.orda_distill_fwdbwd.argtypes = [P, _vp, ctypes.c_size_t, _vp]
    lib.orda_scale_grad.restype = _i32
    lib.orda_scale_grad.argtypes = [_vp, _i64, _i32, _vp, _vp]
    lib.orda_distill_fwdbwd_static_ws.restype = _i32
    lib.orda_distill_fwdbwd_static_ws.argtypes = [P, _vp]
    PP = ctypes.POINTER(PeerSlots)
    lib.orda_distill_fwdbwd_peer.restype = _i32
    lib.orda_distill_fwdbwd_peer.argtypes = [P, _vp, ctypes.c_size_t, PP, _vp]
    lib.orda_peer_reduce_broadcast.restype = _i32
    lib.orda_peer_reduce_broadcast.argtypes = [PP, _i64, _i64, _i32, _i32, _vp]
    PH = ctypes.POINTER(IpcHandle)
    lib.orda_ipc_export.restype = _i32
    lib.orda_ipc_export.argtypes = [_vp, PH]
    lib.orda_ipc_import.restype = _i32
    lib.orda_ipc_import.argtypes = [PH, ctypes.POINTER(_vp)]
    lib.orda_ipc_close.restype = _i32
    lib.orda_ipc_close.argtypes = [_vp, PH]
    lib.orda_shard_workspace_bytes.restype = ctypes.c_size_t
    lib.orda_shard_workspace_bytes.argtypes = [P]
    lib.orda_shard_forward.restype = _i32
    lib.orda_shard_forward.argtypes = [P, _vp, ctypes.c_size_t, _vp, _vp]
    lib.orda_merge_row_stats.restype = _i32
    lib.orda_merge_row_stats.argtypes = [_vp, _i32, _i64, _vp, _vp]
    lib.orda_shard_jsd_partials.restype = _i32
    lib.orda_shard_jsd_partials.argtypes = [P, _vp, ctypes.c_size_t, _vp, _vp, _vp]
    lib.orda_shard_backward.restype = _i32
    lib.orda_shard_backward.argtypes = [P, _vp, ctypes.c_size_t, _vp, _vp, _vp]
    lib.orda_debug_gemm.restype = _i32
    lib.orda_debug_gemm.argtypes = [_i32, _i32, _i32, _vp, _i64, _vp, _i64, _i64, _i64, _i64, _vp, _i64, _vp, _vp]
    lib.orda_debug_gemm_pair.restype = _i32
    lib.orda_debug_gemm_pair.argtypes = lib.orda_debug_gemm.argtypes
    lib.orda_debug_gemm_wide.restype = _i32
    lib.orda_debug_gemm_wide.argtypes = lib.orda_debug_gemm.argtypes
    lib.orda_debug_gemm_profile.restype = _i32
    lib.orda_debug_gemm_profile.argtypes = [ctypes.c_void_p, _i32]
    lib.orda_debug_wait_timeout.restype = _i32
    lib.orda_debug_wait_timeout.argtypes = [_vp, ctypes.c_uint64, _vp, _vp]


def load(path: str | None = None):
    """Load (once) and return the ctypes library; raises RuntimeError if it is missing or stale."""
    global _lib, _load_error
    if _lib is not None and path is None:
        return _lib
    with _lib_lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            _load_error = f"{p} is not built (run orda-knowledge-distillation-kernel_b200/build.py)"
            raise RuntimeError(_load_error)
        try:
            lib = ctypes.CDLL(p)
        except OSError as exc:  # pragma: no cover - depends on the host
            _load_error = f"cannot load {p}: {exc}"
            raise RuntimeError(_load_error) from exc
        _declare(lib)
        if lib.orda_abi_version() != ABI_VERSION:
            raise RuntimeError(f"{p}: ABI version {lib.orda_abi_version()} != {ABI_VERSION}")
        if lib.orda_args_struct_size() != ctypes.sizeof(DistillArgs):
            raise RuntimeError(
                f"{p}: orda_distill_args_t is {lib.orda_args_struct_size()} bytes, "
                f"the Python mirror is {ctypes.sizeof(DistillArgs)}"
            )
        if path is None:
            _lib = lib
        return lib


def status_string(code: int) -> str:
    try:
        return load().orda_status_string(int(code)).decode()
    except RuntimeError:
        return f"status {code}"


def check(code: int, what: str) -> None:
    if code != OK:
        raise RuntimeError(f"{what} failed: {status_string(code)} (status {code})")
