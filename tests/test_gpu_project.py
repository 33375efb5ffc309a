"""Fused K/V projection + norms + RoPE + quantize-on-append on the GPU.

* RoPE goldens: with identity projection weights (8-bit codes 0/1, scale 1,
  bias 0, exact) and the norms off, the rows the fused call produces before
  quantisation are mlx fast::rope of the input — checked against mlx-bun's
  RoPE golden vectors (MLX 0.31.2, seven variants — yarn's and longrope's
  pre-rope input scale applied by the kernel (rope_pre_scale) — offsets 0
  and 5, the offset-5 rows appended after five other rows) to at most one
  element per case, one bf16 ulp (the oracle's own bar against the same
  goldens).
* Projection parity: random inputs and oracle-quantized weights (4 / 8
  bit, group 32 / 64 / 128, with biases), K RMSNorm with weight, V RMSNorm
  without (gemma4.ts:174-177), default / proportional / partial-traditional
  RoPE, attention_k_eq_v, the query side (its projection, q_norm and RoPE
  into q_out; the decode then reads the fused query rows), fp16 and bf16,
  batch 1 / 4 / 2 / 1 / 1 / 3 with
  1 / 1 / 37 / 20 / 300 / 70 rows (the one-launch cluster path at 1 and 4
  rows; the tensor-core projection + epilogue pair beyond, with partial
  128-row and 64-token tiles): the rows before
  quantisation match the oracle's project_kv within 3 dtype ulps of the
  row's largest element (the product sums in f32, the oracle in f64), at
  least 90 % of them exactly; the cache rows are bit-exact with the oracle's
  quantize of those rows, placed as the oracle cache places them; and a
  decode over the cache matches the oracle's attention (2e-3 fp16, 2/128
  bf16, the attention tests' bars).
* bf16 inputs from 1e-6 to 3e5 in magnitude (beyond fp16's range) pass
  the same bar on the tensor-core path (its exact per-block power-of-two
  input scaling).
* Rotating caches: prefill, in-place decode steps past the wrap and a
  chunked append through the temporal re-layout — RoPE positions follow
  the logical offset, the ring matches the oracle's bit for bit.
* A caller workspace of the size kvq_append_projected_workspace reports
  gives the same rows; one byte less is refused (KVQ_ERR_WORKSPACE);
  decode-sized steps (the one-launch cluster path) need none.
"""
import ctypes
import os

import numpy as np
import pytest

from helpers import BF16, F16, from_torch, max_abs, record_parity, to_torch_bits
from oracle import oracle as O
from test_project_cpu import check_rope_golden, rope_case_inputs

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ULP = {F16: 2.0 ** -10, BF16: 2.0 ** -7}
TOL = {F16: 2e-3, BF16: 2.0 / 128}  # decode outputs, as the attention tests bound them


def _np(t):
    import torch
    if t.dtype == torch.int32:
        return t.contiguous().cpu().numpy().view(np.uint32)
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _dev_bits(a, dt):
    return to_torch_bits(np.ascontiguousarray(a), dt)


def _dev_u32(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).cuda()


def make_qlinear(rng, out, inn, gs, bits, dt, scale=1.0):
    """Oracle-quantized random weights: (kvq QuantizedLinear, oracle tuple)."""
    from kvq import QuantizedLinear
    w = (rng.uniform(-1, 1, (out, inn)) * scale / np.sqrt(inn)).astype(np.float32)
    packed, scales, biases = O.quantize(O.to_dtype_bits(w, dt), gs, bits, dt)
    ql = QuantizedLinear(_dev_u32(packed), _dev_bits(scales, dt), _dev_bits(biases, dt), gs, bits)
    return ql, (packed, scales, biases, gs, bits)


def identity_qlinear(n, dt):
    from kvq import QuantizedLinear
    gs = 32
    packed = np.zeros((n, n // 4), np.uint32)
    r = np.arange(n)
    packed[r, r // 4] = (1 << (8 * (r % 4))).astype(np.uint32)
    one = O.to_dtype_bits(np.ones((n, n // gs), np.float32), dt)
    zero = np.zeros_like(one)
    return QuantizedLinear(_dev_u32(packed), _dev_bits(one, dt), _dev_bits(zero, dt), gs, 8)


def check_rows(got_bits, want, dt, label):
    g = O.from_dtype_bits(got_bits, dt).astype(np.float64)
    w = want.astype(np.float64)
    rowmax = np.max(np.abs(w), axis=-1, keepdims=True)
    d = np.abs(g - w)
    lim = 3 * ULP[dt] * rowmax
    exact = float(np.mean(d == 0))
    record_parity(label, got_bits, O.to_dtype_bits(want, dt), dt,
                  f"<= 3 ulp of row max; exact {exact:.3f}")
    assert np.all(d <= lim), f"{label}: worst {np.max(d / np.maximum(lim, 1e-30)):.2f} x limit"
    assert exact >= 0.9, f"{label}: only {exact:.3f} exact"


def _cache_rows_match(K, V, oracle_cache, n, label):
    for got, want in zip((K.packed, K.scales, K.biases, V.packed, V.scales, V.biases),
                         oracle_cache.keys + oracle_cache.values):
        assert np.array_equal(_np(got[:, :, :n]), want[:, :, :n]), label


def test_rope_goldens_through_fused_append():
    import torch
    import kvq
    z = np.load(os.path.join(HERE, "golden", "universal_rope.npz"))
    for name in [str(n) for n in z["names"]]:
        # the raw input; the variant's pre-rope scale goes through the kernel
        x, dims, trad, base, scale, freqs, offsets = rope_case_inputs(z, name, prescale=False)
        pre = float(z[f"{name}/params"][4])
        _, H, L, D = x.shape
        ident = identity_qlinear(H * D, BF16)
        fr = torch.from_numpy(np.ascontiguousarray(freqs, np.float32)).cuda() \
            if freqs is not None else None
        proj = kvq.KvProjection(ident, None, D, k_norm=False, v_norm=False, rope_dims=dims,
                                rope_traditional=trad, rope_base=base, rope_scale=scale,
                                rope_freqs=fr, rope_pre_scale=pre)
        xin = O.to_dtype_bits(x.transpose(0, 2, 1, 3).reshape(1, L, H * D), BF16)
        for off in offsets:
            cache = kvq.QuantizedKVCache(32, 8)
            if off:
                pre = O.to_dtype_bits(np.ones((1, off, H * D), np.float32), BF16)
                cache.update_and_fetch_projected(_dev_bits(pre, BF16), proj)
            k_out = torch.empty(1, H, L, D, dtype=torch.bfloat16, device="cuda")
            cache.update_and_fetch_projected(_dev_bits(xin, BF16), proj, k_out=k_out)
            got = O.from_dtype_bits(from_torch(k_out, BF16), BF16)
            check_rope_golden(got, z[f"{name}/out{off}"], f"fused {name}@{off}")
            record_parity(f"fused append RoPE vs MLX golden {name}@{off}", from_torch(k_out, BF16),
                          O.to_dtype_bits(z[f"{name}/out{off}"], BF16), BF16,
                          "<= 1 element off by 1 ulp")
            cache.dispose()


def _proportional_freqs(D, base, factor=0.25):
    """ProportionalRoPE's table (gemma4.ts:131-165): base^(2i/D) for the
    rotated quarter, infinity for the rest, as f32."""
    rotated = int(D * factor)
    e = (np.arange(0, rotated, 2, dtype=np.float32) / np.float32(D)).astype(np.float32)
    rot = np.power(np.float32(base), e).astype(np.float32)
    return np.concatenate([rot, np.full(D // 2 - rotated // 2, np.inf, np.float32)])


CASES = [
    # dt, wbits, wgs, kv bits, kv gs, B, L, H, D, hidden, k_eq_v, rope
    (F16, 4, 64, 4, 64, 1, 1, 8, 256, 2048, False, "default"),
    (BF16, 4, 64, 8, 32, 4, 1, 4, 128, 1024, True, "proportional"),
    (F16, 8, 32, 8, 64, 2, 37, 2, 128, 512, False, "default"),
    (BF16, 8, 128, 4, 128, 1, 20, 2, 256, 1024, False, "partial-traditional"),
    (BF16, 4, 64, 4, 64, 1, 300, 4, 128, 1024, False, "default"),
    (F16, 4, 32, 8, 32, 3, 70, 2, 64, 2048, True, "proportional"),
    # decode launches whose threads hold more than 8 weight loads: the
    # Gemma-4-12B sliding layer (8-CTA clusters, 14-16 loads, the rest of
    # them staged in shared memory) and 8-bit group-128 weights over a
    # hidden of 8192 (32 loads: registers, shared memory, then plain loads;
    # two rows per launch)
    (F16, 4, 64, 4, 64, 1, 1, 8, 256, 3840, False, "default"),
    (BF16, 8, 128, 8, 64, 2, 1, 2, 128, 8192, False, "default"),
]
# query heads of the cases that also run the query side (the rest: none)
QHEADS = {0: 16, 1: 8, 2: 4, 4: 8, 5: 4, 6: 16, 7: 4}


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{'f16' if c[0] == F16 else 'bf16'}"
                         f"-w{c[1]}g{c[2]}-kv{c[3]}g{c[4]}-B{c[5]}L{c[6]}H{c[7]}D{c[8]}-{c[11]}")
def test_fused_projection_matches_oracle(case):
    import torch
    import kvq
    dt, wbits, wgs, kvbits, kvgs, B, L, H, D, hidden, keqv, rope = case
    tdt = torch.float16 if dt == F16 else torch.bfloat16
    rng = np.random.default_rng(300 + CASES.index(case))
    kq, k_or = make_qlinear(rng, H * D, hidden, wgs, wbits, dt)
    vq, v_or = (None, None) if keqv else make_qlinear(rng, H * D, hidden, wgs, wbits, dt)
    kw = O.round_dt(rng.uniform(0.5, 1.5, D).astype(np.float32), dt)
    spec = dict(head_dim=D, k_proj=k_or, v_proj=v_or, k_norm=True, k_norm_weight=kw, v_norm=True,
                v_norm_weight=None, eps=1e-6)
    kw_dev = _dev_bits(O.to_dtype_bits(kw, dt), dt)
    fr_dev = None
    if rope == "default":
        spec.update(rope_dims=D, rope_base=10000.0)
    elif rope == "proportional":
        fr = _proportional_freqs(D, 1e6)
        spec.update(rope_dims=D, rope_freqs=fr)
        fr_dev = torch.from_numpy(fr).cuda()
    else:
        spec.update(rope_dims=D // 2, rope_traditional=True, rope_base=500000.0)
    Hq = QHEADS.get(CASES.index(case), 0)
    qkw = {}
    if Hq:
        qq, q_or = make_qlinear(rng, Hq * D, hidden, wgs, wbits, dt)
        qw = O.round_dt(rng.uniform(0.5, 1.5, D).astype(np.float32), dt)
        spec.update(q_proj=q_or, q_norm=True, q_norm_weight=qw)
        qkw = dict(q_proj=qq, q_heads=Hq, q_norm=True,
                   q_norm_weight=_dev_bits(O.to_dtype_bits(qw, dt), dt))
    proj = kvq.KvProjection(kq, vq, D, k_norm=True, k_norm_weight=kw_dev, v_norm=True, eps=1e-6,
                            rope_dims=spec["rope_dims"],
                            rope_traditional=spec.get("rope_traditional", False),
                            rope_base=spec.get("rope_base", 10000.0), rope_freqs=fr_dev, **qkw)
    cache = kvq.QuantizedKVCache(kvgs, kvbits)
    oc = O.QuantizedKVCache(kvgs, kvbits, dt)
    offset = 0
    for step, n in enumerate((L, 1)):  # a chunk, then one decode row at the next position
        x = O.to_dtype_bits(rng.uniform(-1, 1, (B, n, hidden)).astype(np.float32), dt)
        k_out = torch.empty(B, H, n, D, dtype=tdt, device="cuda")
        v_out = torch.empty_like(k_out)
        q_out = torch.empty(B, Hq, n, D, dtype=tdt, device="cuda") if Hq else None
        K, V = cache.update_and_fetch_projected(_dev_bits(x, dt), proj, k_out=k_out, v_out=v_out,
                                                q_out=q_out)
        torch.cuda.synchronize()
        want_k, want_v = O.project_kv(O.from_dtype_bits(x, dt), spec, offset, dt)
        if Hq:
            want_q = O.project_q(O.from_dtype_bits(x, dt), spec, offset, dt)
            check_rows(from_torch(q_out, dt), want_q, dt, f"fused projection Q {case[11]} step {step}")
        kb, vb = from_torch(k_out, dt), from_torch(v_out, dt)
        check_rows(kb, want_k, dt, f"fused projection K {case[11]} step {step}")
        check_rows(vb, want_v, dt, f"fused projection V {case[11]} step {step}")
        oc.update_and_fetch(kb, vb)
        offset += n
        assert cache.offset == offset
        _cache_rows_match(K, V, oc, offset, f"cache rows step {step}")
    # attention over the cache the fused path filled: with the query side,
    # the last step's fused query rows (the oracle's own query for the oracle)
    scale = 1.0 / np.sqrt(D)
    if Hq:
        q = O.to_dtype_bits(want_q, dt)
        o = kvq.sdpa_decode(q_out, K, V, scale)
    else:
        q = O.to_dtype_bits(rng.standard_normal((B, 2 * H, 1, D)).astype(np.float32), dt)
        o = kvq.sdpa_decode(_dev_bits(q, dt), K, V, scale)
    want = O.sdpa_unfused(q, *oc.fetch(), scale, kvgs, kvbits, dt)
    got = from_torch(o, dt)
    record_parity(f"decode after fused append {case[11]}", got, want, dt, f"<= {TOL[dt]}")
    assert max_abs(got, want, dt) <= TOL[dt]
    cache.dispose()


def test_bf16_inputs_far_outside_fp16_range():
    """bf16 token rows from 1e-6 to 3e5 in magnitude (some beyond fp16's
    65504) through the tensor-core prefill path: every row within the bar
    of the oracle, nothing infinite."""
    import torch
    import kvq
    dt, B, L, H, D, hidden = BF16, 1, 70, 2, 128, 512
    rng = np.random.default_rng(77)
    kq, k_or = make_qlinear(rng, H * D, hidden, 64, 4, dt)
    vq, v_or = make_qlinear(rng, H * D, hidden, 64, 4, dt)
    spec = dict(head_dim=D, k_proj=k_or, v_proj=v_or, k_norm=True, k_norm_weight=None,
                v_norm=False, eps=1e-6, rope_dims=D, rope_base=10000.0)
    proj = kvq.KvProjection(kq, vq, D, v_norm=False, rope_dims=D, rope_base=10000.0)
    mag = 10.0 ** rng.uniform(-6, 5, (B, L, 1))
    mag[0, :4, 0] = [1e5, 3e5, 1e-6, 7e4]
    x = O.to_dtype_bits((rng.uniform(-1, 1, (B, L, hidden)) * mag).astype(np.float32), dt)
    cache = kvq.QuantizedKVCache(64, 4)
    k_out = torch.empty(B, H, L, D, dtype=torch.bfloat16, device="cuda")
    v_out = torch.empty_like(k_out)
    cache.update_and_fetch_projected(_dev_bits(x, dt), proj, k_out=k_out, v_out=v_out)
    torch.cuda.synchronize()
    assert torch.isfinite(k_out.float()).all() and torch.isfinite(v_out.float()).all()
    want_k, want_v = O.project_kv(O.from_dtype_bits(x, dt), spec, 0, dt)
    check_rows(from_torch(k_out, dt), want_k, dt, "bf16 wide-range inputs K")
    check_rows(from_torch(v_out, dt), want_v, dt, "bf16 wide-range inputs V")
    cache.dispose()


def test_rotating_cache_positions_follow_logical_offset():
    import torch
    import kvq
    dt, H, D, hidden, M = F16, 2, 128, 512, 16
    rng = np.random.default_rng(7)
    kq, k_or = make_qlinear(rng, H * D, hidden, 64, 4, dt)
    vq, v_or = make_qlinear(rng, H * D, hidden, 64, 4, dt)
    spec = dict(head_dim=D, k_proj=k_or, v_proj=v_or, k_norm=True, k_norm_weight=None,
                v_norm=True, eps=1e-6, rope_dims=D, rope_base=10000.0)
    proj = kvq.KvProjection(kq, vq, D, rope_dims=D, rope_base=10000.0)
    cache = kvq.RotatingQuantizedKVCache(M, 64, 8)
    oc = O.RotatingQuantizedKVCache(M, 64, 8, dt)
    offset = 0
    for step, n in enumerate([10] + [1] * 12 + [5, 1]):
        x = O.to_dtype_bits(rng.uniform(-1, 1, (1, n, hidden)).astype(np.float32), dt)
        k_out = torch.empty(1, H, n, D, dtype=torch.float16, device="cuda")
        v_out = torch.empty_like(k_out)
        K, V = cache.update_and_fetch_projected(_dev_bits(x, dt), proj, k_out=k_out, v_out=v_out)
        torch.cuda.synchronize()
        want_k, want_v = O.project_kv(O.from_dtype_bits(x, dt), spec, offset, dt)
        kb, vb = from_torch(k_out, dt), from_torch(v_out, dt)
        check_rows(kb, want_k, dt, f"rotating fused K step {step}")
        check_rows(vb, want_v, dt, f"rotating fused V step {step}")
        ok, ov = oc.update_and_fetch(kb, vb)
        offset += n
        for got, want in zip((K.packed, K.scales, K.biases, V.packed, V.scales, V.biases),
                             list(ok) + list(ov)):
            assert np.array_equal(_np(got), want), step
    cache.dispose()


def test_caller_workspace_sized_by_query():
    import torch
    import kvq
    from kvq import _lib
    dt, B, H, D, hidden, L = BF16, 1, 4, 128, 1024, 16
    rng = np.random.default_rng(9)
    kq, _ = make_qlinear(rng, H * D, hidden, 64, 4, dt)
    proj = kvq.KvProjection(kq, None, D, rope_dims=D)
    x = _dev_bits(O.to_dtype_bits(rng.uniform(-1, 1, (B, L, hidden)).astype(np.float32), dt), dt)
    ref = kvq.QuantizedKVCache(64, 8)
    k_ref = torch.empty(B, H, L, D, dtype=torch.bfloat16, device="cuda")
    ref.update_and_fetch_projected(x, proj, k_out=k_ref)
    cache = kvq.QuantizedKVCache(64, 8)
    cache._ensure_shape(B, H, D, torch.bfloat16, 0)
    lib = _lib.lib()
    s = proj._struct()
    n = ctypes.c_size_t()
    # decode-sized steps keep their partials on chip: no workspace
    _lib.check(lib.kvq_append_projected_workspace(cache._h, 1, ctypes.byref(s), ctypes.byref(n)))
    assert n.value == 0
    _lib.check(lib.kvq_append_projected_workspace(cache._h, L, ctypes.byref(s), ctypes.byref(n)))
    assert n.value > 0
    ws = torch.zeros(n.value, dtype=torch.uint8, device="cuda")
    k_out = torch.empty_like(k_ref)
    st = torch.cuda.current_stream().cuda_stream
    rc = lib.kvq_append_projected(cache._h, x.data_ptr(), L, ctypes.byref(s), None,
                                  k_out.data_ptr(), None, ws.data_ptr(), n.value - 1, st)
    assert rc == _lib.ERR_WORKSPACE
    _lib.check(lib.kvq_append_projected(cache._h, x.data_ptr(), L, ctypes.byref(s), None,
                                        k_out.data_ptr(), None, ws.data_ptr(), n.value, st))
    torch.cuda.synchronize()
    assert torch.equal(k_out.view(torch.int16), k_ref.view(torch.int16))
    K1, V1 = ref.fetch()
    K2, V2 = cache.fetch()
    for a, b in zip((K1.packed, K1.scales, V1.packed, V1.biases),
                    (K2.packed, K2.scales, V2.packed, V2.biases)):
        assert np.array_equal(_np(a), _np(b))
    ref.dispose()
    cache.dispose()
