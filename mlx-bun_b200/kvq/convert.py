"""Dense -> quantized KV conversion: mlx-bun's maybeQuantizeKv on-ramp.

mlx-bun runs the first prompt prefill with dense bf16 / fp16 caches and
converts the populated caches to quantized ones before decode
(src/generate.ts:101-129), one layer at a time so the transient stays about
one layer: ``KVCache.toQuantized`` and ``RotatingKVCache.toQuantized``
(src/model/gemma4-base.ts:395-404, :892-902) quantize the whole buffer as
laid out (padding and ring order included) and carry offset and ring index
over.  Here a dense cache is its device buffers and state
(``DenseKVCache`` / ``DenseRotatingKVCache``), and each conversion is one
kvq_cache_from_dense call.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .cache import QuantizedKVCache, RotatingQuantizedKVCache


@dataclass
class KvQuantSpec:
    """Per-layer KV quantization (KvQuantSpec, src/config.ts:74-78)."""
    layer_idx: int
    bits: int
    group_size: int


@dataclass
class DenseKVCache:
    """A dense growing cache's state: keys / values [B, H, rows, D] (rows a
    multiple of 256, padding included) and the tokens written."""
    keys: torch.Tensor
    values: torch.Tensor
    offset: int

    def to_quantized(self, group_size: int, bits: int, reserve_rows: int = 0):
        return QuantizedKVCache.from_dense(self.keys, self.values, self.offset, group_size, bits,
                                           reserve_rows)


@dataclass
class DenseRotatingKVCache:
    """A dense ring's state: the buffer as laid out, offset, ring index and
    window size."""
    keys: torch.Tensor
    values: torch.Tensor
    offset: int
    ring_idx: int
    max_size: int

    def to_quantized(self, group_size: int, bits: int, reserve_rows: int = 0):
        return RotatingQuantizedKVCache.from_dense(self.keys, self.values, self.offset,
                                                   self.ring_idx, self.max_size, group_size,
                                                   bits, reserve_rows)


def maybe_quantize_kv(caches: list, kv_bits: int | None = None, kv_group_size: int | None = None,
                      quantized_kv_start: int | None = None, kv_config=None) -> list:
    """Convert the dense caches of `caches` in place, with maybeQuantizeKv's
    rules (src/generate.ts:101-129): nothing without kv_bits or kv_config;
    the start threshold defaults to 0 with a kv_config and 5000 otherwise;
    empty caches (offset 0) and caches below the threshold stay dense; with a
    kv_config only its layers convert, with their own bits / group size.
    Each layer's conversion completes (stream synchronized) before the next
    starts, so the dense source of one layer can be released first."""
    if not kv_bits and not kv_config:
        return caches
    start = quantized_kv_start if quantized_kv_start is not None else (0 if kv_config else 5000)
    by_layer = {e.layer_idx: e for e in kv_config} if kv_config else None
    for i, c in enumerate(caches):
        if not isinstance(c, (DenseKVCache, DenseRotatingKVCache)) or c.offset < start:
            continue
        if c.offset == 0:
            continue
        if by_layer is not None:
            e = by_layer.get(i)
            if e is None:
                continue
            caches[i] = c.to_quantized(e.group_size, e.bits)
        else:
            caches[i] = c.to_quantized(kv_group_size or 64, kv_bits)
        if c.keys.is_cuda:
            torch.cuda.current_stream(c.keys.device).synchronize()
    return caches
