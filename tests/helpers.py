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
