"""ctypes binding of libkvq.so (the C ABI in include/kvq.h).

Loads ``libkvq.so`` from this package directory and fails loudly when it is
missing: there is no CPU fallback anywhere in the product path.  Every call
returns an int32 status; a non-zero status raises :class:`KvqError` carrying
``kvq_last_error()`` — the same convention the reference uses for mlx-c calls
(``outArray`` throwing with the recorded mlx message, src/mlx/ffi.ts:338-348).
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libkvq.so")

DTYPE_FLOAT16 = 9
DTYPE_BFLOAT16 = 12
MASK_NONE = 0
MASK_CAUSAL = 1

OK, ERR_ARG, ERR_CUDA, ERR_OOM, ERR_STATE, ERR_WORKSPACE = range(6)

EXPORTS = (
    "kvq_last_error", "kvq_version", "kvq_cache_create", "kvq_cache_free", "kvq_append",
    "kvq_cache_fetch", "kvq_cache_state", "kvq_cache_trim", "kvq_cache_make_mask",
    "kvq_quantize", "kvq_sdpa_decode_workspace", "kvq_sdpa_decode", "kvq_sdpa_decode_partial",
    "kvq_sdpa_merge", "kvq_sdpa_prefill", "kvq_debug_scores", "kvq_check_device",
    "kvq_sdpa_decode_noalloc", "kvq_debug_raise_flag", "kvq_peer_group_create",
    "kvq_peer_group_connect", "kvq_peer_exchange_merge", "kvq_peer_group_check",
    "kvq_peer_group_free", "kvq_append_ragged", "kvq_cache_fetch_all", "kvq_cache_check",
    "kvq_cache_from_dense", "kvq_cache_export", "kvq_cache_import", "kvq_append_projected",
    "kvq_append_projected_workspace",
)


class KvqError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"kvq error {code}: {msg}")
        self.code = code


class Desc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "batch", "kv_heads", "head_dim", "bits", "group_size", "dtype", "max_size",
        "reserve_rows", "device")]


class QTensor(ctypes.Structure):
    _fields_ = [("packed", ctypes.c_void_p), ("scales", ctypes.c_void_p),
                ("biases", ctypes.c_void_p), ("batch_stride", ctypes.c_int64),
                ("head_stride", ctypes.c_int64)] + \
        [(n, ctypes.c_int32) for n in ("batch", "heads", "len", "head_dim", "bits",
                                       "group_size", "dtype")]


class QLinear(ctypes.Structure):
    """kvq_qlinear: one MLX affine-quantized linear layer's weight triple."""
    _fields_ = [("packed", ctypes.c_void_p), ("scales", ctypes.c_void_p),
                ("biases", ctypes.c_void_p)] + \
        [(n, ctypes.c_int32) for n in ("bits", "group_size", "in_features", "out_features")]


class KvProjection(ctypes.Structure):
    """kvq_kv_projection: the K/V side of one attention layer."""
    _fields_ = [("k_proj", QLinear), ("v_proj", QLinear), ("v_from_k", ctypes.c_int32),
                ("k_norm", ctypes.c_int32), ("v_norm", ctypes.c_int32),
                ("k_norm_weight", ctypes.c_void_p), ("v_norm_weight", ctypes.c_void_p),
                ("norm_eps", ctypes.c_float), ("rope_dims", ctypes.c_int32),
                ("rope_traditional", ctypes.c_int32), ("rope_base", ctypes.c_float),
                ("rope_scale", ctypes.c_float), ("rope_pre_scale", ctypes.c_float),
                ("rope_freqs", ctypes.c_void_p), ("q_proj", QLinear), ("q_heads", ctypes.c_int32),
                ("q_norm", ctypes.c_int32), ("q_norm_weight", ctypes.c_void_p)]


_lib = None


def lib():
    """Load libkvq.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"libkvq.so not found at {LIB_PATH}; build it with "
                          "`python mlx-bun_b200/build.py` (no CPU fallback exists)")
    L = ctypes.CDLL(LIB_PATH)
    i32, i64, vp, f32 = ctypes.c_int32, ctypes.c_int64, ctypes.c_void_p, ctypes.c_float
    P = ctypes.POINTER
    sig = {
        "kvq_last_error": (ctypes.c_char_p, []),
        "kvq_version": (i32, []),
        "kvq_cache_create": (i32, [P(Desc), P(vp)]),
        "kvq_cache_free": (i32, [vp]),
        "kvq_append": (i32, [vp, vp, vp, i32, P(i64), P(i64), vp]),
        "kvq_cache_fetch": (i32, [vp, P(QTensor), P(QTensor)]),
        "kvq_cache_state": (i32, [vp, P(i64), P(i64), P(i64), P(i64)]),
        "kvq_cache_trim": (i32, [vp, i32, i32]),
        "kvq_cache_make_mask": (i32, [vp, i32, i32, P(i32), P(i32)]),
        "kvq_quantize": (i32, [vp, i64, i32, i32, i32, i32, vp, vp, vp, vp]),
        "kvq_sdpa_decode_workspace": (i32, [P(QTensor), i32, P(ctypes.c_size_t)]),
        "kvq_sdpa_decode": (i32, [P(QTensor), P(QTensor), vp, i32, f32, vp, vp, vp,
                                  ctypes.c_size_t, vp]),
        "kvq_sdpa_decode_partial": (i32, [P(QTensor), P(QTensor), vp, i32, f32, vp, vp, vp, vp,
                                          vp, ctypes.c_size_t, vp]),
        "kvq_sdpa_merge": (i32, [vp, vp, vp, i32, i64, i32, i32, i32, vp, vp]),
        "kvq_sdpa_prefill": (i32, [P(QTensor), P(QTensor), vp, i32, i32, f32, i32, i32, vp, vp,
                                   ctypes.c_size_t, vp]),
        "kvq_debug_scores": (i32, [P(QTensor), vp, i32, i32, f32, i32, i32, vp, vp]),
        "kvq_check_device": (i32, [vp, vp]),
        "kvq_sdpa_decode_noalloc": (i32, [P(QTensor), P(QTensor), vp, i32, f32, vp, vp, vp]),
        "kvq_debug_raise_flag": (i32, [vp, vp]),
        "kvq_peer_group_create": (i32, [i32, i32, i32, i32, vp, P(vp)]),
        "kvq_peer_group_connect": (i32, [vp, vp]),
        "kvq_peer_exchange_merge": (i32, [vp, vp, i32, vp, vp]),
        "kvq_peer_group_check": (i32, [vp, vp]),
        "kvq_peer_group_free": (i32, [vp]),
        "kvq_append_ragged": (i32, [vp, vp, vp, i32, P(i64), P(i64), vp, vp, vp]),
        "kvq_cache_fetch_all": (i32, [vp, P(QTensor), P(QTensor)]),
        "kvq_cache_check": (i32, [vp, vp]),
        "kvq_cache_from_dense": (i32, [P(Desc), vp, vp, i32, P(i64), P(i64), i64, i64, vp,
                                       P(vp)]),
        "kvq_cache_export": (i32, [vp, i64, P(vp), vp]),
        "kvq_cache_import": (i32, [P(Desc), P(vp), i32, i64, i64, vp, P(vp)]),
        "kvq_append_projected": (i32, [vp, vp, i32, P(KvProjection), vp, vp, vp, vp,
                                       ctypes.c_size_t, vp]),
        "kvq_append_projected_workspace": (i32, [vp, i32, P(KvProjection),
                                                 P(ctypes.c_size_t)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(status: int) -> None:
    if status != OK:
        msg = lib().kvq_last_error().decode("utf-8", "replace")
        raise KvqError(status, msg)


def exported_symbols():
    """Names the loaded library exports out of EXPORTS (for load tests)."""
    L = lib()
    return [n for n in EXPORTS if hasattr(L, n)]
