"""kvq — B200-native quantized-KV attention for mlx-bun's hot path.

Python host layer over ``libkvq.so`` (the C ABI in include/kvq.h):
quantized KV caches (growing and rotating), quantize-on-append (uniform or
ragged per-sequence positions), flash decoding, chunked prefill,
context-split partials with their merge and peer exchange, dense ->
quantized conversion, MLXBUNKV1 persistence, and the fused K/V projection +
norms + RoPE + append.
"""
from ._lib import KvqError, lib
from .cache import Mask, QuantizedKVCache, QuantizedTensor, RotatingQuantizedKVCache
from .convert import DenseKVCache, DenseRotatingKVCache, KvQuantSpec, maybe_quantize_kv
from .project import KvProjection, QuantizedLinear, append_projected
from .sdpa import (debug_scores, decode_workspace_bytes, quantize, quantized_sdpa, sdpa_decode,
                   sdpa_decode_partial, sdpa_merge, sdpa_merge_packed, sdpa_prefill)
from .store import load_kv_cache, read_kv_header, save_kv_cache

__all__ = [
    "KvqError", "lib", "Mask", "QuantizedKVCache", "QuantizedTensor", "RotatingQuantizedKVCache",
    "debug_scores", "decode_workspace_bytes", "quantize", "quantized_sdpa", "sdpa_decode",
    "sdpa_decode_partial", "sdpa_merge", "sdpa_merge_packed", "sdpa_prefill", "DenseKVCache",
    "DenseRotatingKVCache", "KvQuantSpec", "maybe_quantize_kv", "load_kv_cache",
    "read_kv_header", "save_kv_cache", "KvProjection", "QuantizedLinear", "append_projected",
]
