from .dispatcher import clear_chunk_cache, dynamic_chunk, get_chunk_cache
from .resolver import DEFAULT_MAX_FUSED_SIZE, resolve_chunk_size

__all__ = [
    "DEFAULT_MAX_FUSED_SIZE",
    "clear_chunk_cache",
    "dynamic_chunk",
    "get_chunk_cache",
    "resolve_chunk_size",
]
