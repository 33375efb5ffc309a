"""Quantized-KV scaled dot-product attention over libkvq.

``quantized_sdpa`` mirrors mlx-bun's dispatch ``quantizedSdpa(q, kq, vq,
scale, mask, groupSize, bits)`` (src/model/gemma4-base.ts:1560-1578): an L = 1
step with no mask runs the flash-decoding kernel (the role of
``fusedDecodeSdpa``, src/model/fused-decode-kernel.ts:274-312); everything
else (chunked prefill, causal / sliding-window masks) runs the prefill
kernel (the role of ``quantizedSdpaTiled`` / ``quantizedSdpaUnfused``).  There
is no CPU path: every call launches libkvq's CUDA kernels.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, lib
from .cache import Mask, QuantizedTensor, dtype_code


def _stream(t: torch.Tensor, stream):
    return torch.cuda.current_stream(t.device).cuda_stream if stream is None else stream


def _check_q(q: torch.Tensor, keys: QuantizedTensor, L: int | None = None):
    if not q.is_cuda or not q.is_contiguous():
        raise ValueError("q must be a contiguous CUDA tensor [B, Hq, L, D]")
    B, Hq, Lq, D = q.shape
    if B != keys.qt.batch or D != keys.qt.head_dim:
        raise ValueError("q batch / head_dim do not match the cache")
    if dtype_code(q.dtype) != keys.qt.dtype:
        raise ValueError("q dtype must equal the cache dtype")
    return B, Hq, Lq, D


def decode_workspace_bytes(keys: QuantizedTensor, q_heads: int) -> int:
    n = ctypes.c_size_t()
    check(lib().kvq_sdpa_decode_workspace(ctypes.byref(keys.qt), q_heads, ctypes.byref(n)))
    return n.value


def sdpa_decode(q: torch.Tensor, keys: QuantizedTensor, values: QuantizedTensor, scale: float,
                seq_lens: torch.Tensor | None = None, out: torch.Tensor | None = None,
                workspace: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """L = 1 attention; q [B, Hq, 1, D] -> out [B, Hq, 1, D]."""
    B, Hq, L, D = _check_q(q, keys)
    if L != 1:
        raise ValueError("sdpa_decode takes one query row per head")
    if out is None:
        out = torch.empty_like(q)
    sl = 0
    if seq_lens is not None:
        if seq_lens.dtype != torch.int32 or not seq_lens.is_cuda or seq_lens.numel() != B:
            raise ValueError("seq_lens must be a CUDA int32 tensor of B entries")
        sl = seq_lens.data_ptr()
    ws, wsb = (workspace.data_ptr(), workspace.numel() * workspace.element_size()) \
        if workspace is not None else (None, 0)
    check(lib().kvq_sdpa_decode(ctypes.byref(keys.qt), ctypes.byref(values.qt), q.data_ptr(), Hq,
                                ctypes.c_float(scale), sl or None, out.data_ptr(), ws, wsb,
                                _stream(q, stream)))
    return out


def sdpa_decode_partial(q: torch.Tensor, keys: QuantizedTensor, values: QuantizedTensor,
                        scale: float, seq_lens: torch.Tensor | None = None,
                        packed_out: torch.Tensor | None = None, stream=None):
    """Log-sum-exp partials of this key range.

    Returns (m [B*Hq], l [B*Hq], o [B*Hq, D]) float32.  With `packed_out`
    (a float32 tensor of B*Hq*(D+2) elements) they are written into it as
    [m | l | o] — the per-part layout sdpa_merge_packed expects — and the
    returned tensors are views of it."""
    B, Hq, L, D = _check_q(q, keys)
    if L != 1:
        raise ValueError("partials are defined for one query row per head")
    R = B * Hq
    if packed_out is None:
        packed_out = torch.empty(R * (D + 2), dtype=torch.float32, device=q.device)
    if packed_out.numel() != R * (D + 2) or packed_out.dtype != torch.float32 or \
            not packed_out.is_contiguous():
        raise ValueError("packed_out must be a contiguous float32 tensor of B*Hq*(D+2) elements")
    flat = packed_out.view(-1)
    m, l, o = flat[:R], flat[R:2 * R], flat[2 * R:].view(R, D)
    sl = seq_lens.data_ptr() if seq_lens is not None else None
    check(lib().kvq_sdpa_decode_partial(ctypes.byref(keys.qt), ctypes.byref(values.qt),
                                        q.data_ptr(), Hq, ctypes.c_float(scale), sl, m.data_ptr(),
                                        l.data_ptr(), o.data_ptr(), None, 0, _stream(q, stream)))
    return m, l, o


def sdpa_merge(m: torch.Tensor, l: torch.Tensor, o: torch.Tensor, dtype: torch.dtype,
               stream=None) -> torch.Tensor:
    """Merge part-major partials m [P, R], l [P, R], o [P, R, D] -> [R, D]."""
    P, R, D = o.shape
    for t in (m, l, o):
        if t.dtype != torch.float32 or not t.is_contiguous() or not t.is_cuda:
            raise ValueError("partials must be contiguous CUDA float32 tensors")
    out = torch.empty(R, D, dtype=dtype, device=o.device)
    # three separate arrays: one stride per array is not expressible, so merge
    # through a packed copy [P, R*(D+2)]
    packed = torch.cat([m, l, o.reshape(P, R * D)], dim=1).contiguous()
    return sdpa_merge_packed(packed, R, D, dtype, out=out, stream=stream)


def sdpa_merge_packed(packed: torch.Tensor, rows: int, head_dim: int, dtype: torch.dtype,
                      out: torch.Tensor | None = None, stream=None) -> torch.Tensor:
    """Merge partials packed per part as [m (rows) | l (rows) | o (rows*D)]:
    packed [P, rows*(head_dim+2)] float32 -> out [rows, head_dim] dtype."""
    if packed.dtype != torch.float32 or not packed.is_contiguous() or not packed.is_cuda:
        raise ValueError("packed partials must be a contiguous CUDA float32 tensor")
    P = packed.shape[0]
    ps = rows * (head_dim + 2)
    if packed.numel() != P * ps:
        raise ValueError("packed partials have the wrong size")
    if out is None:
        out = torch.empty(rows, head_dim, dtype=dtype, device=packed.device)
    base = packed.data_ptr()
    check(lib().kvq_sdpa_merge(base, base + 4 * rows, base + 8 * rows, P, ps, rows, head_dim,
                               dtype_code(dtype), out.data_ptr(), _stream(packed, stream)))
    return out


def sdpa_prefill(q: torch.Tensor, keys: QuantizedTensor, values: QuantizedTensor, scale: float,
                 mask: Mask, out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                 stream=None) -> torch.Tensor:
    """L >= 1 query rows per head over the keys (bottom-right aligned).

    `workspace`: None (library-managed) or a zero-initialised device buffer.
    The tensor-core kernel's balanced grid needs 262,400 + SMs * 135,168
    bytes of it; with less it runs one CTA per (query block, kv head, batch
    entry)."""
    B, Hq, L, D = _check_q(q, keys)
    if out is None:
        out = torch.empty_like(q)
    mode, window = mask.codes()
    ws, wsb = (workspace.data_ptr(), workspace.numel() * workspace.element_size()) \
        if workspace is not None else (None, 0)
    check(lib().kvq_sdpa_prefill(ctypes.byref(keys.qt), ctypes.byref(values.qt), q.data_ptr(),
                                 Hq, L, ctypes.c_float(scale), mode, window, out.data_ptr(), ws,
                                 wsb, _stream(q, stream)))
    return out


def quantized_sdpa(q: torch.Tensor, keys: QuantizedTensor, values: QuantizedTensor, scale: float,
                   mask: Mask | None = None, group_size: int | None = None,
                   bits: int | None = None, stream=None) -> torch.Tensor:
    """Dispatch of quantizedSdpa (gemma4-base.ts:1560-1578)."""
    mask = mask or Mask("", 0)
    if group_size is not None and group_size != keys.group_size:
        raise ValueError("group_size differs from the cache's")
    if bits is not None and bits != keys.bits:
        raise ValueError("bits differ from the cache's")
    if q.shape[2] == 1 and mask.mode == "":
        return sdpa_decode(q, keys, values, scale, stream=stream)
    return sdpa_prefill(q, keys, values, scale, mask, stream=stream)


def debug_scores(q: torch.Tensor, keys: QuantizedTensor, scale: float, mask: Mask | None = None,
                 stream=None) -> torch.Tensor:
    """Scaled, masked logits [B, Hq, L, N] (f32 of dtype-rounded values)."""
    B, Hq, L, D = _check_q(q, keys)
    mask = mask or Mask("", 0)
    mode, window = mask.codes()
    out = torch.empty(B, Hq, L, keys.qt.len, dtype=torch.float32, device=q.device)
    check(lib().kvq_debug_scores(ctypes.byref(keys.qt), q.data_ptr(), Hq, L,
                                 ctypes.c_float(scale), mode, window, out.data_ptr(),
                                 _stream(q, stream)))
    return out


def quantize(x: torch.Tensor, group_size: int, bits: int, stream=None):
    """mx.quantize of the last axis (ops.ts:615-637) on the GPU:
    x [..., D] -> (packed int32-view [..., D*bits/32], scales, biases)."""
    if not x.is_cuda or not x.is_contiguous():
        raise ValueError("x must be a contiguous CUDA tensor")
    D = x.shape[-1]
    rows = x.numel() // D if D else 0
    packed = torch.empty(x.shape[:-1] + (D * bits // 32,), dtype=torch.int32, device=x.device)
    scales = torch.empty(x.shape[:-1] + (D // group_size,), dtype=x.dtype, device=x.device)
    biases = torch.empty_like(scales)
    check(lib().kvq_quantize(x.data_ptr(), rows, D, group_size, bits, dtype_code(x.dtype),
                             packed.data_ptr(), scales.data_ptr(), biases.data_ptr(),
                             _stream(x, stream)))
    return packed, scales, biases


def check_device(stream=None):
    """Synchronize and raise if a kernel reported a timed-out wait."""
    check(lib().kvq_check_device(None, stream))
