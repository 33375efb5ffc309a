"""The oracle's unfused SDPA graph vs an independent numpy restatement.

Checks, on CPU, the pieces the GPU parity tests lean on: the GQA head
mapping, bottom-right aligned causal and sliding-window masks, ragged
sequence lengths, and the dtype rounding points of quantizedSdpaUnfused
(src/model/gemma4-base.ts:1273-1342).
"""
import numpy as np
import pytest

from oracle import oracle as O


def np_unfused(q_bits, kq, vq, scale, gs, bits, dt, mask_mode=0, window=0, seq_lens=None):
    r = lambda x: O.from_dtype_bits(O.to_dtype_bits(np.asarray(x, np.float32), dt), dt)
    q = O.from_dtype_bits(q_bits, dt)
    B, Hq, L, D = q.shape
    kd = O.dequantize(*kq, gs, bits, dt)
    vd = O.dequantize(*vq, gs, bits, dt)
    Hkv, N = kd.shape[1], kd.shape[2]
    nrep = Hq // Hkv
    out = np.zeros((B, Hq, L, D), np.float32)
    sdt = r(np.float32(scale))
    for b in range(B):
        Nb = N if seq_lens is None else seq_lens[b]
        for h in range(Hq):
            qs = r(q[b, h] * sdt)                                  # [L, D]
            s = r(qs.astype(np.float64) @ kd[b, h // nrep, :Nb].T.astype(np.float64))
            if mask_mode:
                pos = Nb - L + np.arange(L)[:, None]
                j = np.arange(Nb)[None, :]
                ok = j <= pos
                if window:
                    ok &= pos < j + window
                s = np.where(ok, s, -65504.0 if dt == O.F16 else -3.3895313892515355e38)
            e = np.exp(s - s.max(1, keepdims=True))
            p = r(e / e.sum(1, keepdims=True))
            out[b, h] = r(p.astype(np.float64) @ vd[b, h // nrep, :Nb].astype(np.float64))
    return O.to_dtype_bits(out, dt)


@pytest.mark.parametrize("dt", [O.F16, O.BF16])
@pytest.mark.parametrize("mask_mode,window,L", [(0, 0, 1), (1, 0, 7), (1, 5, 9), (0, 0, 3)])
def test_oracle_graph(dt, mask_mode, window, L):
    rng = np.random.default_rng(5)
    B, Hq, Hkv, N, D, gs, bits = 2, 6, 2, 40, 64, 32, 4
    q = O.to_dtype_bits(rng.standard_normal((B, Hq, L, D)).astype(np.float32), dt)
    k = O.to_dtype_bits(rng.standard_normal((B, Hkv, N, D)).astype(np.float32), dt)
    v = O.to_dtype_bits(rng.standard_normal((B, Hkv, N, D)).astype(np.float32), dt)
    kq, vq = O.quantize(k, gs, bits, dt), O.quantize(v, gs, bits, dt)
    got = O.sdpa_unfused(q, kq, vq, 0.125, gs, bits, dt, mask_mode=mask_mode, window=window)
    want = np_unfused(q, kq, vq, 0.125, gs, bits, dt, mask_mode, window)
    a, b = O.from_dtype_bits(got, dt), O.from_dtype_bits(want, dt)
    # identical rounding points; accumulation order differs (f32 vs f64 sums)
    ulp = 2.0 ** -10 if dt == O.F16 else 2.0 ** -7
    assert np.max(np.abs(a - b)) <= 2 * ulp * max(1.0, np.abs(b).max())


def test_oracle_ragged_and_scores():
    rng = np.random.default_rng(6)
    dt, B, Hq, Hkv, N, D, gs, bits = O.F16, 3, 4, 2, 50, 64, 64, 8
    q = O.to_dtype_bits(rng.standard_normal((B, Hq, 1, D)).astype(np.float32), dt)
    k = O.to_dtype_bits(rng.standard_normal((B, Hkv, N, D)).astype(np.float32), dt)
    kq = O.quantize(k, gs, bits, dt)
    lens = [50, 1, 17]
    got, sc = O.sdpa_unfused(q, kq, kq, 1.0, gs, bits, dt, seq_lens=lens, want_scores=True)
    want = np_unfused(q, kq, kq, 1.0, gs, bits, dt, seq_lens=lens)
    assert np.max(np.abs(O.from_dtype_bits(got, dt) - O.from_dtype_bits(want, dt))) <= 4e-3
    assert np.isnan(sc[1, :, 0, 1:]).all() and np.isfinite(sc[1, :, 0, :1]).all()
