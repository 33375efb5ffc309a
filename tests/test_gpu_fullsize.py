"""The BASELINE configurations at their full sizes on the GPU, vs the oracle.

* config 4: B 1, Hq 32, Hkv 8, D 128, kv8 group 64: a 16,384-row prior and a
  512-row chunk appended through the growing cache, then the chunk's causal
  prefill (tensor-core kernel, balanced grid) through quantized_sdpa; keys
  with 4 outlier channels x8.  The appended codes are checked bit for bit
  against the oracle's quantize of the same fp16 rows.
* config 3: B 4, Hq 8, Hkv 4, D 256, kv8: five rotating window-1024 layers
  after 4,096 writes (the ring wraps 3 times) and one global layer over
  4,096 keys, each decoded through quantized_sdpa.
* config 5: B 64 ragged sequences, lengths U[1024, 32768] (numpy seed 5),
  Hq 32, Hkv 8, D 128, kv4, decoded with seq_lens; the oracle checks a
  seeded subset of six batch entries (all heads), named in the test.
* config 5's single sequence of 131,072 keys: the whole-sequence decode,
  eight contiguous-range partials merged, and the single-rank peer exchange
  of the whole range's partial, each against the oracle.

Configs 3 and 5 and the long sequence use ~N(0,1) inputs and the strict
2e-3 bar; config 4 has key outliers and uses helpers.check_outlier_parity.
The K/V of configs 5 and the long sequence are drawn on the GPU and
quantized there (bit-exactness of that quantize is covered by
test_gpu_quantize); the oracle reads the very triples the kernels read.
"""
import ctypes

import numpy as np
import pytest

from helpers import F16, check_outlier_parity, from_torch, ideal_sdpa, max_abs, record_parity, \
    to_torch_bits
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _np_triple(qt, entries=None):
    """Download a QuantizedTensor view (optionally batch entries `entries`)
    as contiguous oracle arrays (uint32 packed, uint16 scales / biases)."""
    import torch
    out = []
    for t in (qt.packed, qt.scales, qt.biases):
        if entries is not None:
            t = t[entries]
        a = t.contiguous().view(torch.int32 if t.dtype == torch.int32 else torch.int16).cpu().numpy()
        out.append(a.view(np.uint32) if a.dtype == np.int32 else a.view(np.uint16))
    return tuple(out)


def test_config4_full_size_prefill():
    import kvq
    import torch
    dt, B, Hq, Hkv, D, gs, bits, Np, L = F16, 1, 32, 8, 128, 64, 8, 16384, 512
    rng = np.random.default_rng(40)
    ch = np.random.default_rng(1234).choice(D, 4, replace=False)

    def rows(n, outl):
        x = rng.standard_normal((B, Hkv, n, D)).astype(np.float32)
        if outl:
            x[..., ch] *= 8.0
        return O.to_dtype_bits(x, dt)

    k0, v0, k1, v1 = rows(Np, True), rows(Np, False), rows(L, True), rows(L, False)
    q = O.to_dtype_bits(rng.standard_normal((B, Hq, L, D)).astype(np.float32), dt)
    cache = kvq.QuantizedKVCache(gs, bits)
    cache.update_and_fetch_quantized(to_torch_bits(k0, dt), to_torch_bits(v0, dt))
    qk, qv = cache.update_and_fetch_quantized(to_torch_bits(k1, dt), to_torch_bits(v1, dt))
    mask = cache.make_mask(L, None)
    assert (mask.mode, mask.window) == ("causal", 0)
    out = kvq.quantized_sdpa(to_torch_bits(q, dt), qk, qv, 1.0 / np.sqrt(D), mask)
    torch.cuda.synchronize()
    kvq.sdpa.check_device()
    kq, vq = _np_triple(qk), _np_triple(qv)
    for got, src in ((kq, np.concatenate([k0, k1], 2)), (vq, np.concatenate([v0, v1], 2))):
        want = O.quantize(src, gs, bits, dt)
        for a, b in zip(got, want):
            assert np.array_equal(a, b)
    scale = 1.0 / np.sqrt(D)
    want = O.sdpa_unfused(q, kq, vq, scale, gs, bits, dt, mask_mode=1)
    ideal = ideal_sdpa(q, kq, vq, scale, gs, bits, dt, mask_mode=1)
    check_outlier_parity(from_torch(out, dt), want, ideal, dt,
                         name="config 4 full size (16384 prior + 512 causal, kv8, key outliers)")
    cache.dispose()


def test_config3_full_size_window_and_global_layers():
    import kvq
    import torch
    dt, B, Hq, Hkv, D, W, gs, bits = F16, 4, 8, 4, 256, 1024, 64, 8
    scale = 1.0 / 16.0
    for layer in range(6):
        rng = np.random.default_rng(300 + layer)
        local = layer < 5
        if local:
            cache = kvq.RotatingQuantizedKVCache(W, gs, bits)
            ocache = O.RotatingQuantizedKVCache(W, gs, bits, dt)
            writes = [1024, 1024, 1024, 1023, 1]  # 4,096 rows: three wraps, then a decode write
        else:
            cache = kvq.QuantizedKVCache(gs, bits)
            ocache = O.QuantizedKVCache(gs, bits, dt)
            writes = [2048, 2047, 1]
        for S in writes:
            k = O.to_dtype_bits(rng.standard_normal((B, Hkv, S, D)).astype(np.float32), dt)
            v = O.to_dtype_bits(rng.standard_normal((B, Hkv, S, D)).astype(np.float32), dt)
            qk, qv = cache.update_and_fetch_quantized(to_torch_bits(k, dt), to_torch_bits(v, dt))
            ok, ov = ocache.update_and_fetch(k, v)
        assert cache.offset == 4096
        assert qk.shape[2] == (W if local else 4096)
        q = O.to_dtype_bits(rng.standard_normal((B, Hq, 1, D)).astype(np.float32), dt)
        want = O.sdpa_unfused(q, ok, ov, scale, gs, bits, dt)
        out = kvq.quantized_sdpa(to_torch_bits(q, dt), qk, qv, scale, cache.make_mask(1, None))
        torch.cuda.synchronize()
        got = from_torch(out, dt)
        name = f"config 3 full size, {'window' if local else 'global'} layer {layer}"
        record_parity(name, got, want, dt, f"<= {TOL}")
        assert max_abs(got, want, dt) <= TOL, name
        cache.dispose()


def _gpu_cache(B, Hkv, N, D, gs, bits, seed, chunk):
    """A growing cache of N rows per (b, kv head) drawn on the GPU (seeded)."""
    import kvq
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    cache = kvq.QuantizedKVCache(gs, bits, reserve_rows=(N + 255) // 256 * 256)
    views = None
    for s0 in range(0, N, chunk):
        S = min(chunk, N - s0)
        k = torch.randn(B, Hkv, S, D, generator=g, device="cuda").half()
        v = torch.randn(B, Hkv, S, D, generator=g, device="cuda").half()
        views = cache.update_and_fetch_quantized(k, v)
    torch.cuda.synchronize()
    return cache, views


# the batch entries of config 5 the oracle checks (all 32 query heads each):
# the longest and shortest sequences plus four fixed ones
CONFIG5_FIXED = (0, 17, 38, 63)


def test_config5_full_size_ragged_decode():
    import kvq
    import torch
    B, Hq, Hkv, D, gs, bits = 64, 32, 8, 128, 64, 4
    lens = np.random.default_rng(5).integers(1024, 32769, size=B)
    Nmax = int(lens.max())
    cache, (qk, qv) = _gpu_cache(B, Hkv, Nmax, D, gs, bits, seed=55, chunk=1024)
    g = torch.Generator(device="cuda")
    g.manual_seed(56)
    q = torch.randn(B, Hq, 1, D, generator=g, device="cuda").half()
    sl = torch.tensor(lens, dtype=torch.int32, device="cuda")
    scale = 1.0 / np.sqrt(D)
    out = kvq.sdpa_decode(q, qk, qv, scale, seq_lens=sl)
    torch.cuda.synchronize()
    kvq.sdpa.check_device()
    subset = sorted(set(CONFIG5_FIXED) | {int(np.argmax(lens)), int(np.argmin(lens))})
    idx = torch.tensor(subset, device="cuda")
    n_sub = int(lens[subset].max())
    kq = tuple(a[:, :, :n_sub] for a in _np_triple(qk, idx))
    vq = tuple(a[:, :, :n_sub] for a in _np_triple(qv, idx))
    qb = from_torch(q[idx], F16)
    want = O.sdpa_unfused(qb, kq, vq, scale, gs, bits, F16, seq_lens=lens[subset])
    got = from_torch(out[idx], F16)
    record_parity(f"config 5 full size (B64 ragged, kv4), entries {subset}", got, want, F16,
                  f"<= {TOL}")
    assert max_abs(got, want, F16) <= TOL
    assert np.isfinite(from_torch(out, F16).view(np.float16)).all()
    cache.dispose()


def test_config5_long_sequence_context_split():
    """131,072 keys: whole decode, 8 range partials + merge, and the
    single-rank peer exchange of one partial, all against the oracle."""
    import kvq
    import torch
    from kvq import _lib
    from kvq.parallel import context_ranges
    B, Hq, Hkv, D, gs, bits, N = 1, 32, 8, 128, 64, 4, 131072
    cache, (qk, qv) = _gpu_cache(B, Hkv, N, D, gs, bits, seed=57, chunk=8192)
    g = torch.Generator(device="cuda")
    g.manual_seed(58)
    q = torch.randn(B, Hq, 1, D, generator=g, device="cuda").half()
    scale = 1.0 / np.sqrt(D)
    whole = kvq.sdpa_decode(q, qk, qv, scale)
    # eight contiguous ranges, as eight ranks would hold them
    R = B * Hq
    parts = []
    for a, b in context_ranges(N, 8):
        K, V = qk.slice_rows(a, b), qv.slice_rows(a, b)
        packed = torch.empty(R * (D + 2), dtype=torch.float32, device="cuda")
        kvq.sdpa_decode_partial(q, K, V, scale, packed_out=packed)
        parts.append(packed)
    merged = kvq.sdpa_merge_packed(torch.stack(parts), R, D, torch.float16)
    # the peer exchange with a single rank: partial of the whole range, three
    # steps in a row (epoch parities 1, 0, 1)
    handle = (ctypes.c_uint8 * 64)()
    grp = ctypes.c_void_p()
    L = _lib.lib()
    _lib.check(L.kvq_peer_group_create(0, 1, R, D, handle, ctypes.byref(grp)))
    try:
        _lib.check(L.kvq_peer_group_connect(grp, bytes(handle)))
        packed = torch.empty(R * (D + 2), dtype=torch.float32, device="cuda")
        kvq.sdpa_decode_partial(q, qk, qv, scale, packed_out=packed)
        st = torch.cuda.current_stream().cuda_stream
        outs = []
        for _ in range(3):
            o = torch.empty(R, D, dtype=torch.float16, device="cuda")
            _lib.check(L.kvq_peer_exchange_merge(grp, packed.data_ptr(), _lib.DTYPE_FLOAT16,
                                                 o.data_ptr(), st))
            outs.append(o)
        _lib.check(L.kvq_peer_group_check(grp, st))
    finally:
        torch.cuda.synchronize()
        _lib.check(L.kvq_peer_group_free(grp))
    torch.cuda.synchronize()
    kq, vq = _np_triple(qk), _np_triple(qv)
    want = O.sdpa_unfused(from_torch(q, F16), kq, vq, scale, gs, bits, F16)
    for name, t in [("whole", whole), ("8 partials merged", merged)] + \
            [(f"peer exchange step {i}", o) for i, o in enumerate(outs)]:
        got = from_torch(t, F16).reshape(want.shape)
        record_parity(f"131072-key sequence, {name}", got, want, F16, f"<= {TOL}")
        assert max_abs(got, want, F16) <= TOL, name
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    cache.dispose()
