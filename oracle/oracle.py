"""CPU oracle for the quantized-KV attention path (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this module, and only as the checker or the timed CPU baseline.
The product path (``mlx-bun_b200/kvq``) never imports it.

Two parts:

* ctypes bindings over ``kvq_oracle.c`` (quantize rule, packing, the unfused
  op graph ``quantizedSdpaUnfused`` with its dtype rounding points);
* a numpy restatement of the two quantized cache state machines of mlx-bun,
  line by line from ``src/model/gemma4-base.ts``:
    - ``QuantizedKVCache``        (:419-598)   growing, 256-row steps
    - ``RotatingQuantizedKVCache`` (:932-1261) sliding-window ring, keep=0
  and of their dense (bf16 / fp16) originals, whose mechanics the quantized
  classes port step for step, with ``to_quantized``:
    - ``KVCache``        (:255-404, toQuantized :395-404)
    - ``RotatingKVCache`` (:604-902, toQuantized :892-902)
* ``save_kv`` / ``load_kv``: the MLXBUNKV1 file layout of ``src/kv-store.ts``
  (magic, u32 header length, u32 data start, JSON header, 16 KiB-aligned
  tensors) over numpy arrays, for checking the product's writer and reader.

The oracle's quantize rule is pinned bit-exactly by
``tests/golden/rotating_kvq_mechanics.npz`` (bf16, gs 32, 8 bit), which was
extracted from mlx-bun's ``goldens/rotating-kvq.bin``.  fp16 inputs, gs 64,
4-bit codes and all SDPA outputs are pinned against this restatement only
(MLX itself cannot run here).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
F16 = 9
BF16 = 12
STEP = 256

_lib = None


def lib():
    global _lib
    if _lib is None:
        from . import build as _build  # noqa: F401  (package-relative when imported as oracle.oracle)
        path = _build.build()
        _lib = ctypes.CDLL(path)
        u16p = ctypes.POINTER(ctypes.c_uint16)
        u32p = ctypes.POINTER(ctypes.c_uint32)
        f32p = ctypes.POINTER(ctypes.c_float)
        _lib.kvqo_quantize_rows.argtypes = [u16p, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                            ctypes.c_int, ctypes.c_int, u32p, u16p, u16p]
        _lib.kvqo_dequantize_rows.argtypes = [u32p, u16p, u16p, ctypes.c_int64, ctypes.c_int,
                                              ctypes.c_int, ctypes.c_int, ctypes.c_int, f32p]
        _lib.kvqo_sdpa_unfused.argtypes = [u16p, ctypes.c_void_p, ctypes.c_void_p] + \
            [ctypes.c_int] * 9 + [ctypes.c_float, ctypes.c_int, ctypes.c_int,
                                   ctypes.POINTER(ctypes.c_int32), u16p, f32p, ctypes.c_int]
        _lib.kvqo_sdpa_unfused.restype = ctypes.c_int
        _lib.kvqo_max_threads.restype = ctypes.c_int
    return _lib


class _View(ctypes.Structure):
    _fields_ = [("packed", ctypes.c_void_p), ("scales", ctypes.c_void_p),
                ("biases", ctypes.c_void_p), ("batch_stride", ctypes.c_int64),
                ("head_stride", ctypes.c_int64)]


def _p(a, t):
    return a.ctypes.data_as(ctypes.POINTER(t))


# ---------------------------------------------------------------- dtypes ---

def to_dtype_bits(x: np.ndarray, dtype: int) -> np.ndarray:
    """f32 array -> uint16 bit patterns of fp16 (RNE) or bf16 (RNE)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if dtype == F16:
        return x.astype(np.float16).view(np.uint16)
    u = x.view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return r.astype(np.uint16)


def from_dtype_bits(h: np.ndarray, dtype: int) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    if dtype == F16:
        return h.view(np.float16).astype(np.float32)
    return (h.astype(np.uint32) << 16).view(np.float32)


# -------------------------------------------------------------- quantize ---

def quantize(x_bits: np.ndarray, group_size: int, bits: int, dtype: int):
    """MLX affine quantize of the last axis (ops.ts:615-637).

    x_bits: uint16 dtype bit patterns [..., D].  Returns (packed u32
    [..., D*bits/32], scales u16 [..., D/gs], biases u16 [..., D/gs]).
    """
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    D = x.shape[-1]
    rows = int(np.prod(x.shape[:-1])) if x.ndim > 1 else 1
    packed = np.zeros(x.shape[:-1] + (D * bits // 32,), np.uint32)
    scales = np.zeros(x.shape[:-1] + (D // group_size,), np.uint16)
    biases = np.zeros_like(scales)
    if rows:
        lib().kvqo_quantize_rows(_p(x, ctypes.c_uint16), rows, D, group_size, bits, dtype,
                                 _p(packed, ctypes.c_uint32), _p(scales, ctypes.c_uint16),
                                 _p(biases, ctypes.c_uint16))
    return packed, scales, biases


def dequantize(packed, scales, biases, group_size: int, bits: int, dtype: int) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.uint32)
    scales = np.ascontiguousarray(scales, dtype=np.uint16)
    biases = np.ascontiguousarray(biases, dtype=np.uint16)
    D = packed.shape[-1] * 32 // bits
    rows = int(np.prod(packed.shape[:-1]))
    out = np.zeros(packed.shape[:-1] + (D,), np.float32)
    if rows:
        lib().kvqo_dequantize_rows(_p(packed, ctypes.c_uint32), _p(scales, ctypes.c_uint16),
                                   _p(biases, ctypes.c_uint16), rows, D, group_size, bits, dtype,
                                   _p(out, ctypes.c_float))
    return out


# ---------------------------------------------------------- unfused SDPA ---

def sdpa_unfused(q_bits, kq, vq, scale: float, group_size: int, bits: int, dtype: int,
                 mask_mode: int = 0, window: int = 0, seq_lens=None, want_scores=False,
                 threads: int = 0):
    """quantizedSdpaUnfused (gemma4-base.ts:1273-1342) on contiguous triples.

    q_bits [B, Hq, L, D] uint16; kq / vq = (packed [B,Hkv,N,*], scales, biases).
    Returns out bits [B, Hq, L, D] (and f32 masked logits [B, Hq, L, N]).
    """
    q = np.ascontiguousarray(q_bits, dtype=np.uint16)
    B, Hq, L, D = q.shape
    kp, ks, kb = (np.ascontiguousarray(a) for a in kq)
    vp, vs, vb = (np.ascontiguousarray(a) for a in vq)
    Hkv, N = kp.shape[1], kp.shape[2]
    kv = _View(kp.ctypes.data, ks.ctypes.data, kb.ctypes.data, Hkv * N, N)
    vv = _View(vp.ctypes.data, vs.ctypes.data, vb.ctypes.data, Hkv * N, N)
    out = np.zeros((B, Hq, L, D), np.uint16)
    scores = np.full((B, Hq, L, N), np.nan, np.float32) if want_scores else None
    sl = None
    if seq_lens is not None:
        sl = np.ascontiguousarray(seq_lens, dtype=np.int32)
    rc = lib().kvqo_sdpa_unfused(
        _p(q, ctypes.c_uint16), ctypes.byref(kv), ctypes.byref(vv), B, Hq, Hkv, L, N, D,
        group_size, bits, dtype, ctypes.c_float(scale), mask_mode, window,
        _p(sl, ctypes.c_int32) if sl is not None else None, _p(out, ctypes.c_uint16),
        _p(scores, ctypes.c_float) if scores is not None else None, threads)
    if rc != 0:
        raise ValueError("oracle sdpa: bad arguments")
    return (out, scores) if want_scores else out


def max_threads() -> int:
    return lib().kvqo_max_threads()


# ------------------------------------------------------ cache mechanics ---

def _zeros(B, H, T, dim, dt):
    return np.zeros((B, H, T, dim), dt)


def _triple_zeros(B, H, T, D, group_size, bits):
    return [_zeros(B, H, T, D * bits // 32, np.uint32), _zeros(B, H, T, D // group_size, np.uint16),
            _zeros(B, H, T, D // group_size, np.uint16)]


def _cat(a, b):
    return np.concatenate([a, b], axis=2)


class QuantizedKVCache:
    """Restates QuantizedKVCache (gemma4-base.ts:419-598) over numpy triples."""

    def __init__(self, group_size: int, bits: int, dtype: int):
        self.group_size, self.bits, self.dtype = group_size, bits, dtype
        self.keys = None
        self.values = None
        self.offset = 0

    # the stored form of new rows and of appended zeros (a triple here, the
    # raw dtype bits in the dense subclasses)
    def _enc(self, x_bits):
        return list(quantize(x_bits, self.group_size, self.bits, self.dtype))

    def _blank(self, B, H, T, D):
        return _triple_zeros(B, H, T, D, self.group_size, self.bits)

    def update_and_fetch(self, k_bits: np.ndarray, v_bits: np.ndarray):
        """updateAndFetchQuantized (:452-507); k/v [B, H, L, D] uint16 bits."""
        B, H, L, kD = k_bits.shape
        vD = v_bits.shape[3]
        prev = self.offset
        if self.keys is None or prev + L > self.keys[0].shape[2]:
            new_steps = ((STEP + L - 1) // STEP) * STEP
            if self.keys is not None and prev % STEP != 0:
                self.keys = [a[:, :, :prev] for a in self.keys]
                self.values = [a[:, :, :prev] for a in self.values]
            nk = self._blank(B, H, new_steps, kD)
            nv = self._blank(B, H, new_steps, vD)
            if self.keys is None:
                self.keys, self.values = nk, nv
            else:
                self.keys = [_cat(a, z) for a, z in zip(self.keys, nk)]
                self.values = [_cat(a, z) for a, z in zip(self.values, nv)]
        self.offset += L
        kq = self._enc(k_bits)
        vq = self._enc(v_bits)
        for dst, src in ((self.keys, kq), (self.values, vq)):
            for a, s in zip(dst, src):
                a[:, :, prev:self.offset] = s
        return self.fetch()

    def fetch(self):
        return ([a[:, :, :self.offset] for a in self.keys],
                [a[:, :, :self.offset] for a in self.values])

    @property
    def seq_len(self):
        return 0 if self.keys is None else self.keys[0].shape[2]

    def trim(self, n: int):
        self.offset = max(0, self.offset - n)


class RotatingQuantizedKVCache:
    """Restates RotatingQuantizedKVCache (gemma4-base.ts:932-1261), keep=0."""

    def __init__(self, max_size: int, group_size: int, bits: int, dtype: int):
        self.max_size = max_size
        self.group_size, self.bits, self.dtype = group_size, bits, dtype
        self.keys = None
        self.values = None
        self.offset = 0
        self.ring_idx = 0

    def _enc(self, x_bits):
        return list(quantize(x_bits, self.group_size, self.bits, self.dtype))

    def _blank(self, B, H, T, D):
        return _triple_zeros(B, H, T, D, self.group_size, self.bits)

    @property
    def seq_len(self):
        return 0 if self.keys is None else self.keys[0].shape[2]

    def _temporal_order(self, t):  # :967-985
        S = t[0].shape[2]
        if self.ring_idx == S:
            return [a[:, :, :S] for a in t]
        if self.ring_idx < self.offset:
            return [_cat(a[:, :, self.ring_idx:S], a[:, :, :self.ring_idx]) for a in t]
        return [a[:, :, :self.ring_idx] for a in t]

    @staticmethod
    def _trim(trim_size, t, append):  # :987-1001
        base = [a[:, :, trim_size if trim_size > 0 else 0:] for a in t]
        if append is None:
            return base
        return [_cat(a, b) for a, b in zip(base, append)]

    def _update_concat(self, k, v):  # :1003-1024
        S = k.shape[2]
        kq = self._enc(k)
        vq = self._enc(v)
        if self.keys is None:
            self.keys, self.values = kq, vq
        else:
            tk = self._temporal_order(self.keys)
            tv = self._temporal_order(self.values)
            self.ring_idx = tk[0].shape[2]
            trim_size = self.ring_idx - self.max_size + 1
            self.keys = self._trim(trim_size, tk, kq)
            self.values = self._trim(trim_size, tv, vq)
        self.offset += S
        self.ring_idx = self.seq_len
        return self.active_slices()

    def _update_in_place(self, k, v):  # :1026-1086
        B, H, S, D = k.shape
        vD = v.shape[3]
        prev = self.offset
        if self.keys is None or (prev >= self.seq_len and self.seq_len < self.max_size):
            new_size = min(STEP, self.max_size - prev)
            if new_size <= 0:
                raise ValueError("rotating cache: non-positive growth")
            nk = self._blank(B, H, new_size, D)
            nv = self._blank(B, H, new_size, vD)
            if self.keys is None:
                self.keys, self.values = nk, nv
            else:
                self.keys = [_cat(a, z) for a, z in zip(self.keys, nk)]
                self.values = [_cat(a, z) for a, z in zip(self.values, nv)]
            self.ring_idx = prev
        trim_size = self.seq_len - self.max_size
        if trim_size > 0:
            self.keys = self._trim(trim_size, self.keys, None)
            self.values = self._trim(trim_size, self.values, None)
            self.ring_idx = self.max_size
        if self.ring_idx == self.max_size:
            self.ring_idx = 0
        kq = self._enc(k)
        vq = self._enc(v)
        self.keys = [a.copy() for a in self.keys]
        self.values = [a.copy() for a in self.values]
        for dst, src in ((self.keys, kq), (self.values, vq)):
            for a, s in zip(dst, src):
                a[:, :, self.ring_idx:self.ring_idx + S] = s
        self.offset += S
        self.ring_idx += S
        return self.active_slices()

    def active_slices(self):  # :1097-1104
        up_to = self.offset if self.offset < self.max_size else self.seq_len
        return ([a[:, :, :up_to] for a in self.keys], [a[:, :, :up_to] for a in self.values])

    def update_and_fetch(self, k_bits, v_bits):  # :1108-1110
        if k_bits.shape[2] == 1:
            return self._update_in_place(k_bits, v_bits)
        return self._update_concat(k_bits, v_bits)

    def is_trimmable(self):
        return self.offset < self.max_size

    def trim(self, n: int, bypass: bool = False):  # :1137-1163
        k = min(self.offset, n)
        if not bypass:
            self.offset -= k
            self.ring_idx -= k
            return
        self.offset -= k
        if k > 0 and self.keys is not None:
            S = self.seq_len
            self.keys = [a[:, :, :S - k] for a in self.keys]
            self.values = [a[:, :, :S - k] for a in self.values]
            self.ring_idx = self.seq_len
        else:
            self.ring_idx -= k


class KVCache(QuantizedKVCache):
    """Dense growing cache (gemma4-base.ts:255-404): the same mechanics with
    raw dtype rows; keys / values are one-element lists [B, H, T, D]."""

    def __init__(self, dtype: int):
        super().__init__(64, 8, dtype)

    def _enc(self, x_bits):
        return [np.ascontiguousarray(x_bits, dtype=np.uint16)]

    def _blank(self, B, H, T, D):
        return [_zeros(B, H, T, D, np.uint16)]

    def to_quantized(self, group_size: int, bits: int):
        """toQuantized (:395-404): the whole buffer, padding included."""
        q = QuantizedKVCache(group_size, bits, self.dtype)
        q.offset = self.offset
        if self.keys is not None:
            q.keys = list(quantize(self.keys[0], group_size, bits, self.dtype))
            q.values = list(quantize(self.values[0], group_size, bits, self.dtype))
        return q


class RotatingKVCache(RotatingQuantizedKVCache):
    """Dense sliding-window ring (gemma4-base.ts:604-902), keep = 0."""

    def __init__(self, max_size: int, dtype: int):
        super().__init__(max_size, 64, 8, dtype)

    def _enc(self, x_bits):
        return [np.ascontiguousarray(x_bits, dtype=np.uint16)]

    def _blank(self, B, H, T, D):
        return [_zeros(B, H, T, D, np.uint16)]

    def to_quantized(self, group_size: int, bits: int):
        """toQuantized (:892-902): the ring as laid out, state carried over."""
        q = RotatingQuantizedKVCache(self.max_size, group_size, bits, self.dtype)
        if self.keys is not None:
            q.keys = list(quantize(self.keys[0], group_size, bits, self.dtype))
            q.values = list(quantize(self.values[0], group_size, bits, self.dtype))
        q.offset = self.offset
        q.ring_idx = self.ring_idx
        return q


# ------------------------------------------------------- MLXBUNKV1 files ---

KV_MAGIC = b"MLXBUNKV1\n"
KV_ALIGN = 16384


def _align_up(n):
    return (n + KV_ALIGN - 1) // KV_ALIGN * KV_ALIGN


def save_kv(path, tokens, entries):
    """Write the MLXBUNKV1 layout of src/kv-store.ts:54-123: magic, u32 LE
    header length, u32 LE data start, JSON header, then each tensor at a
    16 KiB-aligned offset relative to the data start.  `entries`: list of
    (header dict without tensor offsets, list of (name, numpy array)); the
    writer adds {name}Offset / {name}Bytes keys per tensor."""
    import json
    hdr_entries, blobs, off = [], [], 0
    for meta, tensors in entries:
        e = dict(meta)
        for name, a in tensors:
            b = np.ascontiguousarray(a).tobytes()
            o = _align_up(off)
            e[name + "Offset"], e[name + "Bytes"] = o, len(b)
            blobs.append((o, b))
            off = o + len(b)
        hdr_entries.append(e)
    hj = json.dumps({"tokens": list(tokens), "caches": hdr_entries}).encode()
    start = _align_up(len(KV_MAGIC) + 8 + len(hj))
    with open(path, "wb") as f:
        pre = bytearray(start)
        pre[:len(KV_MAGIC)] = KV_MAGIC
        pre[len(KV_MAGIC):len(KV_MAGIC) + 4] = len(hj).to_bytes(4, "little")
        pre[len(KV_MAGIC) + 4:len(KV_MAGIC) + 8] = start.to_bytes(4, "little")
        pre[len(KV_MAGIC) + 8:len(KV_MAGIC) + 8 + len(hj)] = hj
        f.write(pre)
        for o, b in blobs:
            f.seek(start + o)
            f.write(b)


def load_kv(path):
    """Read an MLXBUNKV1 file: (header dict, data start, raw bytes)."""
    import json
    raw = open(path, "rb").read()
    if raw[:len(KV_MAGIC)] != KV_MAGIC:
        raise ValueError("not an mlx-bun KV cache file")
    n = int.from_bytes(raw[len(KV_MAGIC):len(KV_MAGIC) + 4], "little")
    start = int.from_bytes(raw[len(KV_MAGIC) + 4:len(KV_MAGIC) + 8], "little")
    hdr = json.loads(raw[len(KV_MAGIC) + 8:len(KV_MAGIC) + 8 + n])
    return hdr, start, raw


def make_mask(N: int, offset: int, window):
    """Mask decision of QuantizedKVCache.makeMask (:509-519) as (mode, window):
    mode 0 = none, 1 = bottom-right aligned causal (window 0 = unbounded)."""
    if N == 1:
        return 0, 0
    return 1, (window or 0)


def make_mask_rotating(N: int, offset: int, max_size: int, window):
    """RotatingQuantizedKVCache.makeMask (:1113-1122) as (mode, window)."""
    w = window if window is not None else max_size
    if N > 1:
        off = min(max_size - 1, offset)
        if off + N > w:
            return 1, w
        return 1, 0
    return 0, 0


# ------------------------------------------ K/V projection, norms, RoPE ---
# The K/V side of Attention.forward (src/model/gemma4.ts:234-268) ahead of
# the cache append: QuantizedLinear.forward (src/model/gemma4-base.ts:119-
# 124, mlx quantized_matmul with transpose: x @ dequantize(w).T accumulated
# in f32, the result in the activation dtype), RMSNorm (gemma4-base.ts:
# 160-165, mlx fast::rms_norm) and RoPE (src/mlx/ops.ts:100-134, mlx
# fast::rope), MLX 0.31.2.  Every dtype rounding point of those ops is kept;
# sums run in f64 here (the product accumulates in f32, in another order).

def round_dt(x: np.ndarray, dtype: int) -> np.ndarray:
    """f32 values rounded (RNE) to the dtype and back."""
    return from_dtype_bits(to_dtype_bits(x, dtype), dtype)


def quantized_linear(x: np.ndarray, packed, scales, biases, group_size: int, bits: int,
                     dtype: int) -> np.ndarray:
    """x [..., in] (dtype values as f32) @ dequantize(w).T -> [..., out] in the dtype."""
    if biases is None:
        biases = np.zeros_like(scales)
    w = dequantize(packed, scales, biases, group_size, bits, dtype).astype(np.float64)
    y = np.asarray(x, np.float64) @ w.T
    return round_dt(y.astype(np.float32), dtype)


def rms_norm(x: np.ndarray, weight, eps: float, dtype: int) -> np.ndarray:
    """mlx fast::rms_norm over the last axis: x / sqrt(mean(x^2) + eps)
    rounded to the dtype, then times the weight (dtype values), rounded."""
    x = np.asarray(x, np.float32)
    ms = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True).astype(np.float32)
    n = (np.float32(1.0) / np.sqrt(ms + np.float32(eps))).astype(np.float32)
    y = round_dt(x * n, dtype)
    if weight is not None:
        y = round_dt(y * np.asarray(weight, np.float32), dtype)
    return y


def rope(x: np.ndarray, dims: int, traditional: bool, base, scale: float, offset: int,
         freqs, dtype: int) -> np.ndarray:
    """mlx fast::rope of x [..., L, D] at positions offset + l: the first
    `dims` elements rotate in pairs (i, i + dims/2) (or (2i, 2i+1) when
    traditional) by theta = (scale * position) * inv_freq_i, inv_freq_i =
    2^(-(i / (dims/2)) * log2(base)) or 1 / freqs[i]; f32, rounded to the
    dtype.  Elements past `dims` pass through."""
    x = np.asarray(x, np.float32)
    L = x.shape[-2]
    half = dims // 2
    i = np.arange(half, dtype=np.float32)
    if freqs is None:
        inv = np.exp2(-(i / np.float32(half)) * np.float32(np.log2(base))).astype(np.float32)
    else:
        inv = (np.float32(1.0) / np.asarray(freqs, np.float32)).astype(np.float32)
    pos = (np.float32(scale) * (offset + np.arange(L)).astype(np.float32)).astype(np.float32)
    theta = (pos[:, None] * inv[None, :]).astype(np.float32)
    c, s = np.cos(theta).astype(np.float32), np.sin(theta).astype(np.float32)
    out = x.copy()
    if traditional:
        x1, x2 = x[..., 0:dims:2], x[..., 1:dims:2]
    else:
        x1, x2 = x[..., :half], x[..., half:dims]
    r1 = round_dt((x1 * c - x2 * s).astype(np.float32), dtype)
    r2 = round_dt((x1 * s + x2 * c).astype(np.float32), dtype)
    if traditional:
        out[..., 0:dims:2], out[..., 1:dims:2] = r1, r2
    else:
        out[..., :half], out[..., half:dims] = r1, r2
    return out


def project_kv(x: np.ndarray, proj: dict, offset: int, dtype: int):
    """K and V rows [B, H, L, D] (dtype values as f32) of x [B, L, hidden]:
    k = rope(k_norm(k_proj(x))), v = v_norm(v_proj(x) or k_proj(x)).

    proj: k_proj / v_proj = (packed, scales, biases, group_size, bits) (v_proj
    None: attention_k_eq_v), head_dim, k_norm / v_norm (bool), k_norm_weight /
    v_norm_weight (f32 or None), eps, rope_dims, rope_traditional, rope_base,
    rope_scale, rope_freqs (f32 or None), rope_pre_scale."""
    B, L, _ = x.shape
    D = proj["head_dim"]
    k = quantized_linear(x, *proj["k_proj"], dtype)
    v = k if proj.get("v_proj") is None else quantized_linear(x, *proj["v_proj"], dtype)
    H = k.shape[-1] // D
    k = k.reshape(B, L, H, D).transpose(0, 2, 1, 3)
    v = v.reshape(B, L, H, D).transpose(0, 2, 1, 3)
    if proj.get("k_norm"):
        k = rms_norm(k, proj.get("k_norm_weight"), proj["eps"], dtype)
    if proj.get("v_norm"):
        v = rms_norm(v, proj.get("v_norm_weight"), proj["eps"], dtype)
    if proj.get("rope_dims", 0):
        pre = proj.get("rope_pre_scale", 1.0)
        if pre not in (0.0, 1.0):  # UniversalRope.apply (rope.ts:51-75): a weak scalar
            dims = proj["rope_dims"]
            k = k.copy()
            k[..., :dims] = round_dt(k[..., :dims] * round_dt(np.array([pre], np.float32),
                                                              dtype)[0], dtype)
        k = rope(k, proj["rope_dims"], proj.get("rope_traditional", False),
                 proj.get("rope_base"), proj.get("rope_scale", 1.0), offset,
                 proj.get("rope_freqs"), dtype)
    return np.ascontiguousarray(k), np.ascontiguousarray(v)


def project_q(x: np.ndarray, proj: dict, offset: int, dtype: int) -> np.ndarray:
    """The query rows [B, Hq, L, D] of x [B, L, hidden] (Attention.forward,
    src/model/gemma4.ts:224-226 and q's rope, generated/gemma4-12b.ts:
    73-74): q = rope(q_norm(q_proj(x))) with K's RoPE parameters.  proj as
    for project_kv plus q_proj = (packed, scales, biases, group_size, bits),
    q_norm (bool), q_norm_weight (f32 or None)."""
    B, L, _ = x.shape
    D = proj["head_dim"]
    q = quantized_linear(x, *proj["q_proj"], dtype)
    H = q.shape[-1] // D
    q = q.reshape(B, L, H, D).transpose(0, 2, 1, 3)
    if proj.get("q_norm"):
        q = rms_norm(q, proj.get("q_norm_weight"), proj["eps"], dtype)
    if proj.get("rope_dims", 0):
        pre = proj.get("rope_pre_scale", 1.0)
        if pre not in (0.0, 1.0):
            dims = proj["rope_dims"]
            q = q.copy()
            q[..., :dims] = round_dt(q[..., :dims] * round_dt(np.array([pre], np.float32),
                                                              dtype)[0], dtype)
        q = rope(q, proj["rope_dims"], proj.get("rope_traditional", False),
                 proj.get("rope_base"), proj.get("rope_scale", 1.0), offset,
                 proj.get("rope_freqs"), dtype)
    return np.ascontiguousarray(q)
