"""Quantized KV caches over libkvq — the Python mirror of mlx-bun's cache API.

Class and method names follow the reference's TypeScript classes
(src/model/gemma4-base.ts): ``QuantizedKVCache`` (:419-598) and
``RotatingQuantizedKVCache`` (:932-1261) with ``update_and_fetch_quantized``
(updateAndFetchQuantized), ``make_mask`` (makeMask), ``trim``,
``is_trimmable``, ``offset`` / ``ring_idx`` and ``state``.  The state machines
themselves live in the C library (kvq_append); this layer only converts torch
tensors to pointers and wraps the returned views.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from ._lib import QTensor, check, lib

_DT = {torch.float16: _lib.DTYPE_FLOAT16, torch.bfloat16: _lib.DTYPE_BFLOAT16}
_TORCH_DT = {v: k for k, v in _DT.items()}


def dtype_code(dt: torch.dtype) -> int:
    if dt not in _DT:
        raise TypeError(f"kvq supports float16 and bfloat16, not {dt}")
    return _DT[dt]


def torch_dtype(code: int) -> torch.dtype:
    return _TORCH_DT[code]


class _CudaArray:
    """__cuda_array_interface__ holder so torch can view library memory."""

    def __init__(self, ptr, shape, strides_elems, typestr, itemsize, device):
        self.__cuda_array_interface__ = {
            "shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
            "strides": tuple(s * itemsize for s in strides_elems), "version": 3,
        }
        self.device = device


@dataclass
class Mask:
    """mlx-bun's Mask (gemma4-base.ts:21-32) reduced to what the kernels need:
    mode "" (none) or "causal"; window > 0 adds the sliding-window bound of
    createCausalMask (:1595-1614) — the reference's "array" masks."""
    mode: str = ""
    window: int = 0

    def codes(self):
        if self.mode == "":
            return _lib.MASK_NONE, 0
        return _lib.MASK_CAUSAL, int(self.window or 0)


class QuantizedTensor:
    """A (packed, scales, biases) view [B, H, len, *] (ops.ts:607-611).

    Holds the C struct handed to the attention entry points and exposes the
    three components as zero-copy torch views (``packed``, ``scales``,
    ``biases``) for inspection.  The view is only valid until the next call
    that may re-lay out the owning cache (an append that grows or wraps).
    """

    def __init__(self, qt: QTensor, device: int, owner=None):
        self.qt = qt
        self.device = device
        self._owner = owner  # keep the cache alive while the view exists

    @property
    def shape(self):
        q = self.qt
        return (q.batch, q.heads, q.len, q.head_dim)

    @property
    def group_size(self):
        return self.qt.group_size

    @property
    def bits(self):
        return self.qt.bits

    def _view(self, ptr, width, typestr, itemsize, torch_dt):
        q = self.qt
        shape = (q.batch, q.heads, q.len, width)
        strides = (q.batch_stride * width, q.head_stride * width, width, 1)
        arr = _CudaArray(ptr, shape, strides, typestr, itemsize, self.device)
        with torch.cuda.device(self.device):
            t = torch.as_tensor(arr, device=f"cuda:{self.device}")
        return t.view(torch_dt) if torch_dt is not None else t

    @property
    def packed(self) -> torch.Tensor:
        q = self.qt
        t = self._view(q.packed, q.head_dim * q.bits // 32, "<i4", 4, None)
        return t

    @property
    def scales(self) -> torch.Tensor:
        q = self.qt
        return self._view(q.scales, q.head_dim // q.group_size, "<i2", 2, torch_dtype(q.dtype))

    @property
    def biases(self) -> torch.Tensor:
        q = self.qt
        return self._view(q.biases, q.head_dim // q.group_size, "<i2", 2, torch_dtype(q.dtype))

    def slice_rows(self, start: int, stop: int) -> "QuantizedTensor":
        """The view of key rows [start, stop) of every (batch, head) — one
        rank's range of a context split.  `start` must be a multiple of 16
        (the kernels' row tile), so every component stays 16-byte aligned."""
        q = self.qt
        if not (0 <= start <= stop <= q.len) or start % 16:
            raise ValueError("slice_rows: need 0 <= start <= stop <= len and start % 16 == 0")
        word_b = q.head_dim * q.bits // 8
        grp_b = q.head_dim // q.group_size * 2
        qt = QTensor(q.packed + start * word_b, q.scales + start * grp_b,
                     q.biases + start * grp_b, q.batch_stride, q.head_stride, q.batch, q.heads,
                     stop - start, q.head_dim, q.bits, q.group_size, q.dtype)
        return QuantizedTensor(qt, self.device, owner=self._owner if self._owner is not None
                               else self)

    @classmethod
    def from_tensors(cls, packed: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                     group_size: int, bits: int) -> "QuantizedTensor":
        """Wrap caller-owned [B, H, N, *] triples (row-contiguous per head)."""
        B, H, N, W = packed.shape
        for t in (packed, scales, biases):
            if not t.is_cuda or t.stride(3) != 1 or t.stride(2) != t.shape[3]:
                raise ValueError("triples must be CUDA tensors with contiguous rows")
        hs = packed.stride(1) // W
        bs = packed.stride(0) // W
        for t in (scales, biases):
            if t.stride(1) // t.shape[3] != hs or t.stride(0) // t.shape[3] != bs:
                raise ValueError("packed, scales and biases must share row strides")
        D = W * 32 // bits
        qt = QTensor(packed.data_ptr(), scales.data_ptr(), biases.data_ptr(), bs, hs, B, H, N, D,
                     bits, group_size, dtype_code(scales.dtype))
        return cls(qt, packed.device.index, owner=(packed, scales, biases))


def _strides4(x: torch.Tensor):
    arr = (ctypes.c_int64 * 4)(*[int(s) for s in x.stride()])
    return arr


class _CacheBase:
    def __init__(self, max_size: int, group_size: int, bits: int, reserve_rows: int = 0):
        self.max_size = max_size
        self.group_size = group_size
        self.bits = bits
        self.reserve_rows = reserve_rows
        self._h = ctypes.c_void_p(None)
        self._shape = None

    def _ensure(self, k: torch.Tensor):
        B, H, _, D = k.shape
        self._ensure_shape(B, H, D, k.dtype, k.device.index)

    def _ensure_shape(self, B, H, D, dtype, device):
        if self._h.value is None:
            d = _lib.Desc(B, H, D, self.bits, self.group_size, dtype_code(dtype),
                          self.max_size, self.reserve_rows, device)
            check(lib().kvq_cache_create(ctypes.byref(d), ctypes.byref(self._h)))
            self._shape = (B, H, D, dtype, device)
        elif (B, H, D, dtype, device) != self._shape:
            raise ValueError("k/v shape, dtype or device differ from the cache's")

    def update_and_fetch_projected(self, x: torch.Tensor, proj, k_out=None, v_out=None,
                                   stream=None, q_out=None):
        """Fused K/V (and Q) projection + norms + RoPE + append of x [B, L,
        hidden] (kvq_append_projected; see kvq.project)."""
        from .project import append_projected
        return append_projected(self, x, proj, k_out, v_out, stream, q_out)

    def update_and_fetch_quantized(self, k: torch.Tensor, v: torch.Tensor, stream=None):
        """Quantize k, v ([B, H, S, D], any strides with unit d stride) into the
        cache and return the active (keys, values) views."""
        if k.shape != v.shape:
            raise ValueError("k and v must have the same shape")
        if not k.is_cuda or not v.is_cuda:
            raise ValueError("k and v must be CUDA tensors")
        self._ensure(k)
        st = torch.cuda.current_stream(k.device).cuda_stream if stream is None else stream
        check(lib().kvq_append(self._h, k.data_ptr(), v.data_ptr(), k.shape[2], _strides4(k),
                               _strides4(v), st))
        return self.fetch()

    def fetch(self):
        kq, vq = QTensor(), QTensor()
        check(lib().kvq_cache_fetch(self._h, ctypes.byref(kq), ctypes.byref(vq)))
        dev = self._shape[4]
        return QuantizedTensor(kq, dev, self), QuantizedTensor(vq, dev, self)

    # ---- batched serving: per-sequence positions on the device ----

    def append_ragged(self, k: torch.Tensor, v: torch.Tensor, seq_lens: torch.Tensor,
                      counts: torch.Tensor | None = None, stream=None):
        """Entry b writes its first counts[b] (all S when None) rows of k / v
        [B, H, S, D] at rows seq_lens[b]..., then seq_lens[b] += counts[b] —
        on the device (kvq_append_ragged).  The cache must be a growing one
        created with reserve_rows (its capacity).  Returns fetch_all()."""
        if k.shape != v.shape or not k.is_cuda or not v.is_cuda:
            raise ValueError("k and v must be CUDA tensors of one shape")
        for t in (seq_lens,) + ((counts,) if counts is not None else ()):
            if t.dtype != torch.int32 or not t.is_cuda or t.numel() != k.shape[0] or \
                    not t.is_contiguous():
                raise ValueError("seq_lens / counts must be contiguous CUDA int32 [B]")
        if not self.reserve_rows:
            raise ValueError("ragged appends need reserve_rows (the capacity) at creation")
        self._ensure(k)
        st = torch.cuda.current_stream(k.device).cuda_stream if stream is None else stream
        check(lib().kvq_append_ragged(self._h, k.data_ptr(), v.data_ptr(), k.shape[2],
                                      _strides4(k), _strides4(v), seq_lens.data_ptr(),
                                      counts.data_ptr() if counts is not None else None, st))
        return self.fetch_all()

    def fetch_all(self):
        """Views over the whole capacity, for decode with per-sequence seq_lens."""
        kq, vq = QTensor(), QTensor()
        check(lib().kvq_cache_fetch_all(self._h, ctypes.byref(kq), ctypes.byref(vq)))
        dev = self._shape[4]
        return QuantizedTensor(kq, dev, self), QuantizedTensor(vq, dev, self)

    def check(self, stream=None):
        """Raise if a ragged append skipped an entry past the capacity."""
        if self._h.value is not None:
            check(lib().kvq_cache_check(self._h, stream))

    # ---- conversion and persistence ----

    @classmethod
    def _adopt(cls, h, shape, max_size, group_size, bits, reserve_rows=0):
        obj = cls.__new__(cls)
        _CacheBase.__init__(obj, max_size, group_size, bits, reserve_rows)
        obj._h = h
        obj._shape = shape
        return obj

    @classmethod
    def _from_dense(cls, keys, values, offset, ring_idx, max_size, group_size, bits,
                    reserve_rows=0, stream=None):
        if keys.shape[:3] != values.shape[:3] or keys.shape[3] != values.shape[3]:
            raise ValueError("keys and values must have one shape [B, H, rows, D]")
        if not keys.is_cuda or not values.is_cuda or keys.dtype != values.dtype:
            raise ValueError("keys and values must be CUDA tensors of one dtype")
        B, H, rows, D = keys.shape
        dev = keys.device.index
        d = _lib.Desc(B, H, D, bits, group_size, dtype_code(keys.dtype), max_size, reserve_rows,
                      dev)
        st = torch.cuda.current_stream(keys.device).cuda_stream if stream is None else stream
        h = ctypes.c_void_p()
        check(lib().kvq_cache_from_dense(ctypes.byref(d), keys.data_ptr(), values.data_ptr(),
                                         rows, _strides4(keys), _strides4(values), int(offset),
                                         int(ring_idx), st, ctypes.byref(h)))
        return cls._adopt(h, (B, H, D, keys.dtype, dev), max_size, group_size, bits, reserve_rows)

    def export(self):
        """Host copy of the saved region and the state, as mlx-bun persists a
        cache (src/kv-store.ts:54-123): a growing cache keeps its live
        [0:offset] rows, a ring its whole buffer and ring index.  Returns
        dict(kind, offset, idx, max_size, bits, group_size, dtype, shape,
        tensors = [k packed, k scales, k biases, v packed, v scales,
        v biases] as numpy arrays)."""
        import numpy as np
        if self._h.value is None:
            raise ValueError("cannot persist an empty cache")
        B, H, D, dt, dev = self._shape
        offset, ring_idx, seq_len, _ = self._state()
        rows = seq_len if self.max_size else offset
        G, W = D // self.group_size, D * self.bits // 32
        arrs = [np.empty((B, H, rows, W), np.uint32), np.empty((B, H, rows, G), np.uint16),
                np.empty((B, H, rows, G), np.uint16), np.empty((B, H, rows, W), np.uint32),
                np.empty((B, H, rows, G), np.uint16), np.empty((B, H, rows, G), np.uint16)]
        ptrs = (ctypes.c_void_p * 6)(*[a.ctypes.data for a in arrs])
        with torch.cuda.device(dev):
            torch.cuda.synchronize()
            check(lib().kvq_cache_export(self._h, rows, ptrs, None))
        return dict(kind="rotating-kvq" if self.max_size else "kvq", offset=offset,
                    idx=ring_idx if self.max_size else None,
                    max_size=self.max_size or None, bits=self.bits, group_size=self.group_size,
                    dtype=dtype_code(dt), shape=[B, H, rows, D], tensors=arrs)

    @staticmethod
    def from_export(state, device: int = 0, reserve_rows: int = 0):
        """The cache `export` described, on `device` (loadKvCache +
        restoreState, src/kv-store.ts:147-175)."""
        import numpy as np
        B, H, rows, D = state["shape"]
        max_size = state.get("max_size") or 0
        d = _lib.Desc(B, H, D, state["bits"], state["group_size"], state["dtype"], max_size,
                      reserve_rows, device)
        arrs = [np.ascontiguousarray(a) for a in state["tensors"]]
        ptrs = (ctypes.c_void_p * 6)(*[a.ctypes.data for a in arrs])
        h = ctypes.c_void_p()
        with torch.cuda.device(device):
            check(lib().kvq_cache_import(ctypes.byref(d), ptrs, rows, int(state["offset"]),
                                         int(state.get("idx") or 0), None, ctypes.byref(h)))
        cls = RotatingQuantizedKVCache if max_size else QuantizedKVCache
        return cls._adopt(h, (B, H, D, torch_dtype(state["dtype"]), device), max_size,
                          state["group_size"], state["bits"], reserve_rows)

    def _state(self):
        vals = [ctypes.c_int64() for _ in range(4)]
        if self._h.value is None:
            return 0, 0, 0, 0
        check(lib().kvq_cache_state(self._h, *[ctypes.byref(x) for x in vals]))
        return tuple(x.value for x in vals)

    @property
    def offset(self) -> int:
        return self._state()[0]

    @property
    def seq_len(self) -> int:
        return self._state()[2]

    @property
    def capacity(self) -> int:
        return self._state()[3]

    def make_mask(self, N: int, window_size=None) -> Mask:
        if self._h.value is None:  # empty cache: offset 0
            if N == 1:
                return Mask("", 0)
            if self.max_size:
                w = window_size or self.max_size
                return Mask("causal", w if N > w else 0)
            return Mask("causal", window_size or 0)
        mode, win = ctypes.c_int32(), ctypes.c_int32()
        check(lib().kvq_cache_make_mask(self._h, N, int(window_size or 0), ctypes.byref(mode),
                                        ctypes.byref(win)))
        return Mask("" if mode.value == _lib.MASK_NONE else "causal", win.value)

    def trim(self, n: int, bypass: bool = False):
        if self._h.value is not None:
            check(lib().kvq_cache_trim(self._h, n, 1 if bypass else 0))

    def state(self):
        """The six buffers as torch views [B, H, seq_len, *] (state(), :577-587)."""
        if self._h.value is None:
            return []
        k, v = self.fetch()
        n = self.seq_len
        out = []
        for qt in (k, v):
            qt.qt.len = n
            out += [qt.packed, qt.scales, qt.biases]
        return out

    def dispose(self):
        if self._h.value is not None:
            check(lib().kvq_cache_free(self._h))
            self._h = ctypes.c_void_p(None)

    def __del__(self):
        try:
            self.dispose()
        except Exception:
            pass


class QuantizedKVCache(_CacheBase):
    """Growing quantized cache (gemma4-base.ts:419-598)."""

    STEP = 256

    def __init__(self, group_size: int = 64, bits: int = 8, reserve_rows: int = 0):
        super().__init__(0, group_size, bits, reserve_rows)

    @classmethod
    def from_dense(cls, keys: torch.Tensor, values: torch.Tensor, offset: int,
                   group_size: int = 64, bits: int = 8, reserve_rows: int = 0, stream=None):
        """KVCache.toQuantized (gemma4-base.ts:395-404): quantize the whole
        dense buffer [B, H, rows, D] (padding included) and adopt offset."""
        return cls._from_dense(keys, values, offset, 0, 0, group_size, bits, reserve_rows, stream)

    def is_trimmable(self) -> bool:
        return True


class RotatingQuantizedKVCache(_CacheBase):
    """Sliding-window ring cache, keep = 0 (gemma4-base.ts:932-1261)."""

    STEP = 256

    def __init__(self, max_size: int, group_size: int = 64, bits: int = 8, reserve_rows: int = 0):
        if max_size <= 0:
            raise ValueError("max_size must be positive")
        super().__init__(max_size, group_size, bits, reserve_rows)

    @property
    def ring_idx(self) -> int:
        return self._state()[1]

    @classmethod
    def from_dense(cls, keys: torch.Tensor, values: torch.Tensor, offset: int, ring_idx: int,
                   max_size: int, group_size: int = 64, bits: int = 8, reserve_rows: int = 0,
                   stream=None):
        """RotatingKVCache.toQuantized (gemma4-base.ts:892-902): quantize the
        ring as laid out (ring order, not temporal) and adopt offset and
        ring index."""
        if max_size <= 0:
            raise ValueError("max_size must be positive")
        return cls._from_dense(keys, values, offset, ring_idx, max_size, group_size, bits,
                               reserve_rows, stream)

    def is_trimmable(self) -> bool:
        return self.offset < self.max_size
