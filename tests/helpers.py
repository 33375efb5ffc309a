"""Shared helpers of the parity tests: seeded inputs, oracle calls, uploads."""
from __future__ import annotations

import numpy as np

from oracle import oracle as O

F16, BF16 = O.F16, O.BF16


def torch_dt(dt):
    import torch
    return torch.float16 if dt == F16 else torch.bfloat16


def gen(rng, shape, outlier_channels=0, outlier_scale=8.0):
    """~N(0,1) f32; optionally `outlier_channels` fixed channels of the last
    axis scaled by `outlier_scale` (the key-outlier pattern of the configs)."""
    x = rng.standard_normal(shape).astype(np.float32)
    if outlier_channels:
        D = shape[-1]
        ch = np.random.default_rng(1234).choice(D, outlier_channels, replace=False)
        x[..., ch] *= outlier_scale
    return x


def to_torch_bits(bits, dt, device="cuda"):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).to(device)
    return t.view(torch_dt(dt))


def from_torch(t, dt):
    import torch
    a = t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    return a


def bits_to_f32(bits, dt):
    return O.from_dtype_bits(bits, dt)


def upload_triple(packed, scales, biases, group_size, bits, pad_to=16, device="cuda"):
    """Oracle triple [B, H, N, *] -> QuantizedTensor over padded CUDA buffers
    (row capacity rounded up to `pad_to`, as a kvq cache lays them out)."""
    import torch
    from kvq.cache import QuantizedTensor
    B, H, N, W = packed.shape
    Np = max(pad_to, (N + pad_to - 1) // pad_to * pad_to)
    G = scales.shape[3]
    pk = torch.zeros(B, H, Np, W, dtype=torch.int32, device=device)
    sc = torch.zeros(B, H, Np, G, dtype=torch.int16, device=device)
    bi = torch.zeros(B, H, Np, G, dtype=torch.int16, device=device)
    pk[:, :, :N] = torch.from_numpy(packed.view(np.int32)).to(device)
    sc[:, :, :N] = torch.from_numpy(scales.view(np.int16)).to(device)
    bi[:, :, :N] = torch.from_numpy(biases.view(np.int16)).to(device)
    return pk, sc, bi, (B, H, N, Np)


def as_qtensor(pk, sc, bi, N, group_size, bits, dt):
    from kvq.cache import QuantizedTensor
    tdt = torch_dt(dt)
    qt = QuantizedTensor.from_tensors(pk[:, :, :N], sc.view(tdt)[:, :, :N], bi.view(tdt)[:, :, :N],
                                      group_size, bits)
    return qt


def quantized_inputs(rng, B, Hq, Hkv, N, D, gs, bits, dt, L=1, k_outliers=0):
    """q bits [B,Hq,L,D], oracle triples for K and V, and their f32 sources."""
    q = O.to_dtype_bits(gen(rng, (B, Hq, L, D)), dt)
    k = O.to_dtype_bits(gen(rng, (B, Hkv, N, D), outlier_channels=k_outliers), dt)
    v = O.to_dtype_bits(gen(rng, (B, Hkv, N, D)), dt)
    kq = O.quantize(k, gs, bits, dt)
    vq = O.quantize(v, gs, bits, dt)
    return q, kq, vq


def max_abs(a_bits, b_bits, dt):
    a = bits_to_f32(a_bits, dt).astype(np.float64)
    b = bits_to_f32(b_bits, dt).astype(np.float64)
    return float(np.max(np.abs(a - b))) if a.size else 0.0


def ideal_sdpa(q_bits, kq, vq, scale, group_size, bits, dt, mask_mode=0, window=0):
    """float64 evaluation of the same attention on the same quantized K/V and
    dtype-rounded scaled q, with no intermediate rounding (the exact math the
    oracle's fp16 rounding points approximate)."""
    kd = O.dequantize(*kq, group_size, bits, dt).astype(np.float64)
    vd = O.dequantize(*vq, group_size, bits, dt).astype(np.float64)
    qf = O.from_dtype_bits(q_bits, dt).astype(np.float64)
    sdt = float(O.from_dtype_bits(O.to_dtype_bits(np.array([scale], np.float32), dt), dt)[0])
    qs = O.from_dtype_bits(O.to_dtype_bits((qf * sdt).astype(np.float32), dt), dt).astype(np.float64)
    B, Hq, L, D = qs.shape
    Hkv, N = kd.shape[1], kd.shape[2]
    nrep = Hq // Hkv
    out = np.zeros((B, Hq, L, D))
    pos = N - L + np.arange(L)[:, None]
    j = np.arange(N)[None]
    ok = np.ones((L, N), bool)
    if mask_mode:
        ok = j <= pos
        if window:
            ok &= pos < j + window
    for b in range(B):
        for h in range(Hq):
            s = np.where(ok, qs[b, h] @ kd[b, h // nrep].T, -np.inf)
            e = np.exp(s - s.max(1, keepdims=True))
            out[b, h] = (e / e.sum(1, keepdims=True)) @ vd[b, h // nrep]
    return out


# (test name, max |diff| vs oracle, fraction of outputs beyond 2e-3, bar) per
# parity check, printed in the terminal summary of the run (conftest.py)
PARITY_LOG = []


def record_parity(name, got_bits, want_bits, dt, bar):
    """Log how far the kernel's outputs sit from the oracle's."""
    g = bits_to_f32(got_bits, dt).astype(np.float64)
    w = bits_to_f32(want_bits, dt).astype(np.float64)
    d = np.abs(g - w)
    m = float(d.max()) if d.size else 0.0
    beyond = float((d > 2e-3).mean()) if d.size else 0.0
    PARITY_LOG.append((name, m, beyond, bar))
    return m, beyond


def check_outlier_parity(got_bits, want_bits, ideal, dt, tol=2e-3, frac=0.9999, hard=1e-2,
                         slack=5e-4, name=None):
    """Parity bar for inputs with key-outlier channels, where logits reach
    |s| ~ 30-50 and one fp16 ulp of a rounded logit (0.03) moves its
    probability by ~3%: any summation order different from the oracle's flips
    a few roundings.  Requires (a) >= `frac` of the outputs within `tol` of the
    oracle, (b) all within `hard`, and (c) the kernel no farther from the exact
    float64 result than the oracle is (plus `slack`)."""
    g = bits_to_f32(got_bits, dt).astype(np.float64)
    w = bits_to_f32(want_bits, dt).astype(np.float64)
    d = np.abs(g - w)
    e_ours = np.abs(g - ideal).max()
    e_ref = np.abs(w - ideal).max()
    PARITY_LOG.append((name or "outlier-input case", float(d.max()), float((d > tol).mean()),
                       f"outlier bar (kernel->f64 {e_ours:.2e}, oracle->f64 {e_ref:.2e})"))
    assert (d <= tol).mean() >= frac, (d > tol).mean()
    assert d.max() <= hard, d.max()
    assert e_ours <= e_ref + slack, (e_ours, e_ref)
    return d.max(), e_ours, e_ref
