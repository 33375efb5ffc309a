"""kvq_sdpa_decode_noalloc against kvq_sdpa_decode, through the C ABI.

The no-allocation decode exists for callers that cannot have device memory
allocated on their behalf: serving processes whose own pool took all free
device memory at start-up, and latency-bound decode loops that must never
meet a cudaMalloc's implicit device synchronization.  Its scratch is a fixed
array inside libkvq.  These tests call it twice in a row on different
inputs — the second call finds the first call's leftovers in that shared
scratch — and require each result to match kvq_sdpa_decode on the same
inputs within the decode tolerance (2e-3 on fp16 outputs).  They also check
that shapes needing more scratch than the array holds are refused with
KVQ_ERR_WORKSPACE, that a query the balanced kernel cannot take (not 16-byte
aligned) still fits by running without a key split, and that a raised device
error flag in the scratch survives later calls until kvq_check_device
reports it.

This file is collected last, so a run that stops at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from helpers import F16, as_qtensor, from_torch, max_abs, quantized_inputs, to_torch_bits, \
    upload_triple

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _inputs(seed, B, Hq, Hkv, N, D, gs, bits):
    rng = np.random.default_rng(seed)
    q, kq, vq = quantized_inputs(rng, B, Hq, Hkv, N, D, gs, bits, F16)
    K = as_qtensor(*upload_triple(*kq, gs, bits)[:3], N, gs, bits, F16)
    V = as_qtensor(*upload_triple(*vq, gs, bits)[:3], N, gs, bits, F16)
    return to_torch_bits(q, F16), K, V


def _noalloc(q, K, V, scale, out):
    import torch
    from kvq import _lib
    st = torch.cuda.current_stream().cuda_stream
    return _lib.lib().kvq_sdpa_decode_noalloc(ctypes.byref(K.qt), ctypes.byref(V.qt),
                                              q.data_ptr(), q.shape[1], ctypes.c_float(scale),
                                              None, out.data_ptr(), st)


def test_noalloc_decode_matches_decode_two_calls():
    import torch
    import kvq
    from kvq import _lib
    # two different problems back to back; both split the keys across CTAs,
    # so both use the scratch's tickets and partials
    cases = [(11, 2, 32, 8, 3000, 128, 64, 4), (12, 1, 16, 4, 2048, 128, 64, 8)]
    for seed, B, Hq, Hkv, N, D, gs, bits in cases:
        q, K, V = _inputs(seed, B, Hq, Hkv, N, D, gs, bits)
        scale = 1.0 / np.sqrt(D)
        want = kvq.sdpa_decode(q, K, V, scale)
        got = torch.empty_like(q)
        _lib.check(_noalloc(q, K, V, scale, got))
        torch.cuda.synchronize()
        err = max_abs(from_torch(got, F16), from_torch(want, F16), F16)
        assert err <= TOL, (seed, err)


def test_noalloc_refuses_shapes_beyond_its_scratch():
    import torch
    from kvq import _lib
    # 64 (batch, kv head) pairs with 16 query heads each at D 256: the split
    # partials exceed the fixed scratch even when the decode runs on one CTA
    q, K, V = _inputs(13, 8, 128, 8, 512, 256, 64, 8)
    out = torch.zeros_like(q)
    rc = _noalloc(q, K, V, 0.0625, out)
    assert rc == _lib.ERR_WORKSPACE
    msg = _lib.lib().kvq_last_error().decode()
    assert "kvq_sdpa_decode_noalloc" in msg and "bytes" in msg
    torch.cuda.synchronize()
    assert not out.any()


def test_noalloc_unaligned_query_runs_without_key_split():
    """A q that is not 16-byte aligned takes the split kernel; at this shape
    its split partials exceed the scratch, so the call runs unsplit."""
    import torch
    import kvq
    from kvq import _lib
    q0, K, V = _inputs(14, 1, 8, 4, 32768, 256, 64, 8)
    buf = torch.zeros(q0.numel() + 8, dtype=q0.dtype, device=q0.device)
    q = buf[1:1 + q0.numel()].view(q0.shape)  # 2 bytes past a 16-byte boundary
    q.copy_(q0)
    assert q.data_ptr() % 16 == 2
    want = kvq.sdpa_decode(q, K, V, 0.0625)
    for _ in range(2):
        got = torch.empty_like(q0)
        _lib.check(_noalloc(q, K, V, 0.0625, got))
        torch.cuda.synchronize()
        err = max_abs(from_torch(got, F16), from_torch(want, F16), F16)
        assert err <= TOL, err


def test_noalloc_error_flag_kept_until_reported():
    """A raised error flag in the scratch is not cleared by the next call;
    kvq_check_device(NULL) reports it once and clears it."""
    import torch
    from kvq import _lib
    L = _lib.lib()
    q, K, V = _inputs(15, 1, 16, 4, 1024, 128, 64, 8)
    out = torch.empty_like(q)
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(_noalloc(q, K, V, 0.088, out))  # looks the scratch address up
    _lib.check(L.kvq_check_device(None, st))   # nothing raised so far
    _lib.check(L.kvq_debug_raise_flag(None, st))
    _lib.check(_noalloc(q, K, V, 0.088, out))  # must leave the flag raised
    assert L.kvq_check_device(None, st) == _lib.ERR_CUDA
    assert "error flag" in L.kvq_last_error().decode()
    _lib.check(L.kvq_check_device(None, st))   # reported once, then clear
