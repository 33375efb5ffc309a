"""kvq — B200-native quantized-KV attention for mlx-bun's hot path.

Python host layer over ``libkvq.so`` (the C ABI in include/kvq.h):
quantized KV caches (growing and rotating), quantize-on-append, flash
decoding, chunked prefill, context-split partials and their merge.
"""
from ._lib import KvqError, lib
from .cache import Mask, QuantizedKVCache, QuantizedTensor, RotatingQuantizedKVCache
from .sdpa import (debug_scores, decode_workspace_bytes, quantize, quantized_sdpa, sdpa_decode,
                   sdpa_decode_partial, sdpa_merge, sdpa_merge_packed, sdpa_prefill)

__all__ = [
    "KvqError", "lib", "Mask", "QuantizedKVCache", "QuantizedTensor", "RotatingQuantizedKVCache",
    "debug_scores", "decode_workspace_bytes", "quantize", "quantized_sdpa", "sdpa_decode",
    "sdpa_decode_partial", "sdpa_merge", "sdpa_merge_packed", "sdpa_prefill",
]
