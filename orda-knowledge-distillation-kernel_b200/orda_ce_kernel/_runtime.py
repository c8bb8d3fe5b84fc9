"""Runtime helpers: CUDA availability of the sm_100a library and the compute-dtype rule.

``default_compute_dtype`` keeps the reference's rule (``src/orda_ce_kernel/_runtime.py:61-80``):
an active autocast dtype wins, else bf16 if any input is bf16, else fp16, else fp32.
"""
from __future__ import annotations

import torch


def cuda_kernels_available() -> bool:
    """True when a CUDA device of compute capability 10.0 (B200) is visible and the library loads."""
    if not torch.cuda.is_available():
        return False
    try:
        major, minor = torch.cuda.get_device_capability()
    except RuntimeError:
        return False
    if (major, minor) != (10, 0):
        return False
    from . import _native

    try:
        _native.load()
    except RuntimeError:
        return False
    return True


def _active_autocast_dtype(device: torch.device | None) -> torch.dtype | None:
    device_type = device.type if device is not None else "cuda"
    try:
        enabled = torch.is_autocast_enabled(device_type)
    except TypeError:  # older torch
        enabled = torch.is_autocast_enabled()
    if not enabled:
        return None
    try:
        dtype = torch.get_autocast_dtype(device_type)
    except (AttributeError, TypeError):
        dtype = torch.get_autocast_gpu_dtype()
    if dtype in (torch.bfloat16, torch.float16):
        return dtype
    return None


def default_compute_dtype(*tensors: torch.Tensor) -> torch.dtype:
    device = next((t.device for t in tensors if isinstance(t, torch.Tensor)), None)
    autocast_dtype = _active_autocast_dtype(device)
    if autocast_dtype is not None:
        return autocast_dtype
    dtypes = [t.dtype for t in tensors if isinstance(t, torch.Tensor) and t.is_floating_point()]
    if torch.bfloat16 in dtypes:
        return torch.bfloat16
    if torch.float16 in dtypes:
        return torch.float16
    if torch.float32 in dtypes:
        return torch.float32
    return torch.float16
