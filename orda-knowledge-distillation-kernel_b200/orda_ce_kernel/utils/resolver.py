"""Chunk-argument validation kept from the reference (``src/orda_ce_kernel/utils/resolver.py:1-62``).

The fused kernels tile rows and vocab internally, so the chunk count only bounds the size of the
workspace; the argument contract (and its error messages) is the reference's, which callers and the
reference's unit tests rely on.
"""
from __future__ import annotations

import math

DEFAULT_MAX_FUSED_SIZE = 32768  # reference utils/_autotune.py:32; accepted and ignored by the fused path


def is_power_of_two(value: int) -> bool:
    return value > 0 and (value & (value - 1)) == 0


def _is_auto_chunk_size(chunk_size) -> bool:
    """None, "auto", "dynamic", -2 and non-positive numbers mean "library default" (resolver.py:9-16)."""
    if chunk_size is None or chunk_size in ("auto", "dynamic"):
        return True
    if isinstance(chunk_size, bool):
        return False
    return isinstance(chunk_size, (int, float)) and chunk_size <= 0


def _chunks_from_raw(raw: float) -> int:
    if raw < 1.5:
        return 1
    return 1 << (math.floor(math.log2(raw / 1.5)) + 1)


def resolve_chunk_size(BT, chunk_size_arg, V=None, max_chunks=None, num_chunks=None):
    """(chunk_size, num_chunks) for BT rows: explicit num_chunks, explicit chunk_size, or the
    pressure heuristic (BT/1024)*(V/32768)^2 capped to 2*BT/512 chunks (resolver.py:28-62)."""
    if int(BT) == 0:
        raise ValueError("BT (batch x sequence length) must be > 0.")
    if num_chunks is not None:
        if not _is_auto_chunk_size(chunk_size_arg):
            raise ValueError("chunk_size and num_chunks are mutually exclusive.")
        requested = int(num_chunks)
        if requested < 1:
            raise ValueError(f"num_chunks must be >= 1, got {num_chunks}")
        effective = min(requested, int(BT))
        if max_chunks is not None and effective > int(max_chunks):
            raise ValueError(
                f"num_chunks must be <= max_chunks, got num_chunks={num_chunks}, max_chunks={max_chunks}"
            )
        return (BT + effective - 1) // effective, effective
    if _is_auto_chunk_size(chunk_size_arg):
        if V is None:
            return BT, 1
        useful = max(1, int(BT) // 512)
        if max_chunks is None:
            max_chunks = 2 * useful
        pressure = (float(BT) / 1024.0) * ((float(V) / 32768.0) ** 2)
        floor = float(BT) / 4096.0
        chunks = min(max_chunks, useful, _chunks_from_raw(max(pressure, floor)), int(BT))
        return (BT + chunks - 1) // chunks, chunks
    cs = min(int(chunk_size_arg), BT)
    return cs, (BT + cs - 1) // cs
