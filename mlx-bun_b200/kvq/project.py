"""Fused K/V projection + norms + RoPE + quantize-on-append.

The K/V side of mlx-bun's Attention.forward (src/model/gemma4.ts:234-268),
and optionally its query side (:224-226 and q's rope), as one library call,
kvq_append_projected: the K (and V, and Q) projections from
MLX affine-quantized weights (QuantizedLinear, src/model/gemma4-base.ts:
76-158), K's RMSNorm with weight and V's without (:160-165, gemma4.ts:
174-177), RoPE of K at the cache offset (gemma4.ts:184-188, the default and
ProportionalRoPE frequency forms) and the quantize-on-append into the
cache, with the rows placed by the cache's own state machine.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import check, lib


@dataclass
class QuantizedLinear:
    """An MLX affine-quantized linear layer's weight triple: weight (uint32
    as int32 [out, in * bits / 32]), scales and biases ([out, in / group_size],
    the activation dtype; biases may be None)."""
    weight: torch.Tensor
    scales: torch.Tensor
    biases: torch.Tensor | None
    group_size: int
    bits: int

    @property
    def in_features(self) -> int:
        return self.scales.shape[1] * self.group_size

    @property
    def out_features(self) -> int:
        return self.scales.shape[0]

    def _struct(self) -> _lib.QLinear:
        for t in (self.weight, self.scales) + ((self.biases,) if self.biases is not None else ()):
            if not t.is_cuda or not t.is_contiguous():
                raise ValueError("quantized weights must be contiguous CUDA tensors")
        if self.weight.shape != (self.out_features, self.in_features * self.bits // 32):
            raise ValueError("weight shape does not match scales, group_size and bits")
        return _lib.QLinear(self.weight.data_ptr(), self.scales.data_ptr(),
                            self.biases.data_ptr() if self.biases is not None else None,
                            self.bits, self.group_size, self.in_features, self.out_features)


@dataclass
class KvProjection:
    """The K/V side of one attention layer: k_proj, v_proj (None: V is K's
    projection, attention_k_eq_v), the norms and the RoPE parameters
    (rope_dims 0: none; rope_freqs: a device f32 [rope_dims / 2] table
    replacing rope_base, as ProportionalRoPE and the scaled variants use;
    rope_pre_scale: yarn's / longrope's input scale on K's rotated part).
    q_proj (None: no query side) with q_heads heads: the query rows, normed
    by q_norm (weight q_norm_weight) and roped like K, go to the caller's
    q_out."""
    k_proj: QuantizedLinear
    v_proj: QuantizedLinear | None
    head_dim: int
    k_norm: bool = True
    k_norm_weight: torch.Tensor | None = None
    v_norm: bool = True
    v_norm_weight: torch.Tensor | None = None
    eps: float = 1e-6
    rope_dims: int = 0
    rope_traditional: bool = False
    rope_base: float = 10000.0
    rope_scale: float = 1.0
    rope_freqs: torch.Tensor | None = None
    rope_pre_scale: float = 1.0
    q_proj: QuantizedLinear | None = None
    q_heads: int = 0
    q_norm: bool = True
    q_norm_weight: torch.Tensor | None = None

    @property
    def kv_heads(self) -> int:
        return self.k_proj.out_features // self.head_dim

    def _struct(self) -> _lib.KvProjection:
        for t in (self.k_norm_weight, self.v_norm_weight, self.q_norm_weight):
            if t is not None and (not t.is_cuda or not t.is_contiguous()):
                raise ValueError("norm weights must be contiguous CUDA tensors")
        if self.rope_freqs is not None and (self.rope_freqs.dtype != torch.float32 or
                                            not self.rope_freqs.is_cuda):
            raise ValueError("rope_freqs must be a CUDA float32 tensor")
        s = _lib.KvProjection()
        s.k_proj = self.k_proj._struct()
        s.v_from_k = 1 if self.v_proj is None else 0
        if self.v_proj is not None:
            s.v_proj = self.v_proj._struct()
        s.k_norm, s.v_norm = int(self.k_norm), int(self.v_norm)
        s.k_norm_weight = self.k_norm_weight.data_ptr() if self.k_norm_weight is not None else None
        s.v_norm_weight = self.v_norm_weight.data_ptr() if self.v_norm_weight is not None else None
        s.norm_eps = self.eps
        s.rope_dims = self.rope_dims
        s.rope_traditional = int(self.rope_traditional)
        s.rope_base = self.rope_base
        s.rope_scale = self.rope_scale
        s.rope_pre_scale = self.rope_pre_scale
        s.rope_freqs = self.rope_freqs.data_ptr() if self.rope_freqs is not None else None
        if self.q_proj is not None:
            s.q_proj = self.q_proj._struct()
            s.q_heads = self.q_heads
            s.q_norm = int(self.q_norm)
            s.q_norm_weight = (self.q_norm_weight.data_ptr()
                               if self.q_norm_weight is not None else None)
        return s


def append_projected(cache, x: torch.Tensor, proj: KvProjection, k_out=None, v_out=None,
                     stream=None, q_out=None):
    """Project x [B, L, hidden] through `proj` and append the quantized rows
    to `cache` (a QuantizedKVCache or RotatingQuantizedKVCache); returns the
    active (keys, values) views like update_and_fetch_quantized.  k_out /
    v_out: optional [B, kv_heads, L, head_dim] tensors that receive the rows
    before quantisation.  q_out: the [B, q_heads, L, head_dim] query rows
    (required with a query projection)."""
    if x.dim() != 3 or not x.is_cuda or not x.is_contiguous():
        raise ValueError("x must be a contiguous CUDA tensor [B, L, hidden]")
    B, L, _ = x.shape
    shape = (B, proj.kv_heads, L, proj.head_dim)
    for t in (k_out, v_out):
        if t is not None and (tuple(t.shape) != shape or t.dtype != x.dtype or
                              not t.is_contiguous()):
            raise ValueError(f"k_out / v_out must be contiguous {x.dtype} {shape}")
    if proj.q_proj is not None:
        qshape = (B, proj.q_heads, L, proj.head_dim)
        if q_out is None or tuple(q_out.shape) != qshape or q_out.dtype != x.dtype or \
                not q_out.is_contiguous():
            raise ValueError(f"q_out must be a contiguous {x.dtype} {qshape} tensor")
    cache._ensure_shape(B, proj.kv_heads, proj.head_dim, x.dtype, x.device.index)
    st = torch.cuda.current_stream(x.device).cuda_stream if stream is None else stream
    s = proj._struct()
    check(lib().kvq_append_projected(
        cache._h, x.data_ptr(), L, ctypes.byref(s),
        q_out.data_ptr() if q_out is not None else None,
        k_out.data_ptr() if k_out is not None else None,
        v_out.data_ptr() if v_out is not None else None, None, 0, st))
    return cache.fetch()
