"""Pins the CPU oracle against mlx-bun's rotating-KV-quant golden.

Mirrors tests/rotating-kvq.test.ts:64-105 of mlx-bun: drive the ring cache
through the scripted sequence (prefill 48 -> 20 decodes with a wrap ->
16-token concat over the wrapped ring -> 8 decodes) and compare the active
(packed, scales, biases) triples plus offset / ring index bit for bit at every
checkpoint.
"""
import numpy as np

from oracle import oracle as O


def test_ring_mechanics_bit_exact(golden_rotating):
    g = golden_rotating
    max_size, H, D, gs, bits = (int(x) for x in g["config"])
    cache = O.RotatingQuantizedKVCache(max_size, gs, bits, O.BF16)
    cps = set(int(c) for c in g["checkpoints"])
    checked = 0
    for i, S in enumerate(g["steps_S"]):
        k, v = g[f"step{i}_k"], g[f"step{i}_v"]
        assert k.shape == (1, H, S, D)
        qk, qv = cache.update_and_fetch(k, v)
        if i in cps:
            off, idx = g[f"cp{i}_state"]
            assert cache.offset == off and cache.ring_idx == idx, (i, cache.offset, cache.ring_idx)
            for name, got in (("k", qk), ("v", qv)):
                np.testing.assert_array_equal(got[0], g[f"cp{i}_{name}_packed"])
                np.testing.assert_array_equal(got[1], g[f"cp{i}_{name}_scales"])
                np.testing.assert_array_equal(got[2], g[f"cp{i}_{name}_biases"])
            checked += 1
    assert checked == 7


def test_half_conversions_match_numpy():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s
                        for s in (1e-8, 1e-6, 1e-4, 1, 100, 3e4, 7e4)])
    x = np.concatenate([x, np.array([0.0, -0.0, 65504, 65519.99, 65520, -65520,
                                     2.0 ** -25, 2.0 ** -24, 3 * 2.0 ** -26], np.float32)])
    import ctypes
    lib = O.lib()
    lib.kvqo_f32_to_half.restype = ctypes.c_uint16
    lib.kvqo_f32_to_half.argtypes = [ctypes.c_float]
    lib.kvqo_half_to_f32.restype = ctypes.c_float
    lib.kvqo_half_to_f32.argtypes = [ctypes.c_uint16]
    want = x.astype(np.float16).view(np.uint16)
    got = np.array([lib.kvqo_f32_to_half(float(v)) for v in x], np.uint16)
    np.testing.assert_array_equal(got, want)
    back = np.array([lib.kvqo_half_to_f32(int(h)) for h in want[::7]], np.float32)
    np.testing.assert_array_equal(back, want[::7].view(np.float16).astype(np.float32))
