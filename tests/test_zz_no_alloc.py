"""kvq_sdpa_decode_noalloc against kvq_sdpa_decode, through the C ABI.

The no-allocation decode exists for callers that must not allocate device
memory (work recorded inside an open CUDA stream capture, serving processes
that own all device memory): its scratch is a fixed array inside libkvq.
These tests call it twice in a row on different inputs — the second call
finds the first call's leftovers in that shared scratch — and require each
result to match kvq_sdpa_decode on the same inputs within the decode
tolerance (2e-3 on fp16 outputs).  They also check that shapes needing more
scratch than the array holds are refused with KVQ_ERR_WORKSPACE.

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
