"""Quantized caches on the GPU: state machine + contents bit-exact.

1. The rotating cache replays mlx-bun's golden mechanics sequence
   (tests/rotating-kvq.test.ts:64-105) on the GPU and matches the golden
   triples and (offset, ring index) at every checkpoint.
2. Random append schedules (prefill chunks, decode steps, wraps, trims) on
   growing and rotating caches match the oracle restatement exactly: offset,
   ring index, buffer length and every active row.
"""
import numpy as np
import pytest

from helpers import BF16, F16, from_torch, gen, to_torch_bits
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def fetch_np(qt, dt):
    return (qt.packed.cpu().numpy().view(np.uint32), from_torch(qt.scales, dt),
            from_torch(qt.biases, dt))


def test_golden_ring_mechanics_on_gpu(golden_rotating):
    import kvq
    g = golden_rotating
    max_size, H, D, gs, bits = (int(x) for x in g["config"])
    cache = kvq.RotatingQuantizedKVCache(max_size, gs, bits)
    cps = set(int(c) for c in g["checkpoints"])
    for i, S in enumerate(g["steps_S"]):
        k = to_torch_bits(g[f"step{i}_k"], BF16)
        v = to_torch_bits(g[f"step{i}_v"], BF16)
        qk, qv = cache.update_and_fetch_quantized(k, v)
        if i in cps:
            off, idx = g[f"cp{i}_state"]
            assert (cache.offset, cache.ring_idx) == (off, idx)
            for name, got in (("k", qk), ("v", qv)):
                p, s, b = fetch_np(got, BF16)
                np.testing.assert_array_equal(p, g[f"cp{i}_{name}_packed"])
                np.testing.assert_array_equal(s, g[f"cp{i}_{name}_scales"])
                np.testing.assert_array_equal(b, g[f"cp{i}_{name}_biases"])
    cache.dispose()


def _compare(cache, ocache, qk, qv, oq, dt, ring):
    assert cache.offset == ocache.offset
    assert cache.seq_len == ocache.seq_len
    if ring:
        assert cache.ring_idx == ocache.ring_idx
    for got, want in zip((qk, qv), oq):
        p, s, b = fetch_np(got, dt)
        np.testing.assert_array_equal(p, want[0])
        np.testing.assert_array_equal(s, want[1])
        np.testing.assert_array_equal(b, want[2])


SCHEDULES = {
    "decode-growth": [300] + [1] * 40,
    "chunked": [100, 200, 1, 1, 513, 1],
    "ring-wrap": [48] + [1] * 30 + [16] + [1] * 10,
    "ring-big-prefill": [150, 1, 1, 70, 1, 1, 1],
    "ring-tiny": [1] * 70 + [5] + [1] * 5,
}


@pytest.mark.parametrize("name", list(SCHEDULES))
@pytest.mark.parametrize("dt,bits,gs", [(F16, 4, 64), (BF16, 8, 64), (F16, 8, 32), (BF16, 4, 128)])
def test_cache_matches_oracle(name, dt, bits, gs):
    import kvq
    ring = name.startswith("ring")
    B, H, D = 2, 3, 128
    max_size = 64
    rng = np.random.default_rng(11)
    if ring:
        cache = kvq.RotatingQuantizedKVCache(max_size, gs, bits)
        ocache = O.RotatingQuantizedKVCache(max_size, gs, bits, dt)
    else:
        cache = kvq.QuantizedKVCache(gs, bits)
        ocache = O.QuantizedKVCache(gs, bits, dt)
    for S in SCHEDULES[name]:
        k = O.to_dtype_bits(gen(rng, (B, H, S, D), outlier_channels=4), dt)
        v = O.to_dtype_bits(gen(rng, (B, H, S, D)), dt)
        qk, qv = cache.update_and_fetch_quantized(to_torch_bits(k, dt), to_torch_bits(v, dt))
        oq = ocache.update_and_fetch(k, v)
        _compare(cache, ocache, qk, qv, oq, dt, ring)
    cache.dispose()


def test_strided_bshd_input_and_trim():
    """[B, S, H, D] inputs (transposed view, no copy) and trim/bypass paths."""
    import kvq
    dt = F16
    B, H, D, gs, bits = 2, 4, 64, 32, 8
    rng = np.random.default_rng(5)
    cache = kvq.RotatingQuantizedKVCache(40, gs, bits)
    ocache = O.RotatingQuantizedKVCache(40, gs, bits, dt)
    for step, S in enumerate([20, 1, 1, 8, 1, 1]):
        k = O.to_dtype_bits(gen(rng, (B, S, H, D)), dt)
        v = O.to_dtype_bits(gen(rng, (B, S, H, D)), dt)
        kt = to_torch_bits(k, dt).transpose(1, 2)  # logical [B, H, S, D], strided
        vt = to_torch_bits(v, dt).transpose(1, 2)
        qk, qv = cache.update_and_fetch_quantized(kt, vt)
        oq = ocache.update_and_fetch(np.ascontiguousarray(k.transpose(0, 2, 1, 3)),
                                     np.ascontiguousarray(v.transpose(0, 2, 1, 3)))
        _compare(cache, ocache, qk, qv, oq, dt, True)
        if step == 3:  # speculative rollback right after a concat write
            cache.trim(2, bypass=True)
            ocache.trim(2, bypass=True)
            assert (cache.offset, cache.ring_idx, cache.seq_len) == \
                (ocache.offset, ocache.ring_idx, ocache.seq_len)
    g = kvq.QuantizedKVCache(64, 4)
    og = O.QuantizedKVCache(64, 4, dt)
    for S in (10, 5):
        k = O.to_dtype_bits(gen(rng, (1, 2, S, 128)), dt)
        g.update_and_fetch_quantized(to_torch_bits(k, dt), to_torch_bits(k, dt))
        og.update_and_fetch(k, k)
    g.trim(3)
    og.trim(3)
    k = O.to_dtype_bits(gen(rng, (1, 2, 1, 128)), dt)
    qk, qv = g.update_and_fetch_quantized(to_torch_bits(k, dt), to_torch_bits(k, dt))
    _compare(g, og, qk, qv, og.update_and_fetch(k, k), dt, False)


def test_reserved_capacity_no_relayout():
    import kvq
    dt = F16
    cache = kvq.QuantizedKVCache(64, 8, reserve_rows=4096)
    ocache = O.QuantizedKVCache(64, 8, dt)
    rng = np.random.default_rng(9)
    cap0 = None
    for S in (700, 1, 1, 300):
        k = O.to_dtype_bits(gen(rng, (1, 2, S, 128)), dt)
        qk, qv = cache.update_and_fetch_quantized(to_torch_bits(k, dt), to_torch_bits(k, dt))
        oq = ocache.update_and_fetch(k, k)
        _compare(cache, ocache, qk, qv, oq, dt, False)
        cap0 = cap0 or cache.capacity
        assert cache.capacity == cap0 == 4096
