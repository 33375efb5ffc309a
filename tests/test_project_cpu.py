"""The projection / RMSNorm / RoPE restatement, pinned on CPU, and the fused
entry point's argument checks (no GPU).

* RoPE: the oracle's mlx fast::rope restatement against mlx-bun's RoPE
  golden vectors (tests/fixtures/universal-rope, MLX 0.31.2: default,
  linear, llama3, yarn, yarn-noscale, longrope and traditional-partial at
  offsets 0 and 5, bf16) — bit-exact but for at most one element per case,
  by at most one bf16 ulp.  yarn and longrope apply their pre-rope input
  scale as UniversalRope.apply does (src/model/universal/rope.ts:51-75):
  x[..., :dims] times the scale rounded to bf16 (a weak scalar), rounded.
* RMSNorm and the quantized linear layer: known answers.
* kvq_append_projected_workspace refuses malformed projections with
  KVQ_ERR_ARG before any CUDA call.
"""
import ctypes
import os

import numpy as np
import pytest

from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
BF16_ULP = 2.0 ** -7


def _rope_cases():
    z = np.load(os.path.join(HERE, "golden", "universal_rope.npz"))
    return z, [str(n) for n in z["names"]]


def rope_case_inputs(z, name, prescale=True):
    """(x as bf16 values, dims, traditional, base, scale, freqs, offsets)
    with the variant's pre-rope input scale applied (unless `prescale` is
    False)."""
    p = z[f"{name}/params"]
    dims, base, scale, trad, pre, always = p[:6]
    dims = int(dims)
    x = O.round_dt(z[f"{name}/input"], O.BF16)
    if prescale and (always or pre != 1.0):
        s = O.round_dt(np.array([pre], np.float32), O.BF16)[0]
        x = x.copy()
        x[..., :dims] = O.round_dt(x[..., :dims] * s, O.BF16)
    freqs = z[f"{name}/freqs"] if f"{name}/freqs" in z else None
    return x, dims, bool(trad), float(base), float(scale), freqs, [int(o) for o in p[6:]]


def check_rope_golden(got, want, label):
    d = np.abs(got.astype(np.float64) - want.astype(np.float64))
    ulp = BF16_ULP * np.maximum(np.abs(want), 2.0 ** -126)
    bad = d > 0
    assert bad.sum() <= 1, f"{label}: {bad.sum()} elements differ"
    assert np.all(d <= ulp * 1.0001), f"{label}: max diff {d.max()}"


def test_rope_restatement_matches_mlx_goldens():
    z, names = _rope_cases()
    assert str(z["mlx_version"]) == "0.31.2"
    assert len(names) == 7
    for name in names:
        x, dims, trad, base, scale, freqs, offsets = rope_case_inputs(z, name)
        for off in offsets:
            got = O.rope(x, dims, trad, base, scale, off, freqs, O.BF16)
            check_rope_golden(got, z[f"{name}/out{off}"], f"{name}@{off}")


def test_rope_passes_through_past_dims_and_is_identity_at_zero():
    rng = np.random.default_rng(0)
    x = O.round_dt(rng.standard_normal((1, 2, 3, 128)).astype(np.float32), O.F16)
    y = O.rope(x, 64, False, 10000.0, 1.0, 0, None, O.F16)
    assert np.array_equal(y[..., 64:], x[..., 64:])
    assert np.array_equal(y[:, :, 0], x[:, :, 0])  # position 0: theta = 0
    # infinite frequencies (ProportionalRoPE's tail) leave their pairs unrotated
    fr = np.full(32, np.inf, np.float32)
    assert np.array_equal(O.rope(x, 64, False, None, 1.0, 7, fr, O.F16), x)


def test_project_kv_applies_pre_scale_like_the_goldens():
    """project_kv's rope_pre_scale (identity weights, no norms) reproduces
    the yarn and longrope goldens from the raw inputs."""
    z, _ = _rope_cases()
    for name in ("yarn", "longrope"):
        x, dims, trad, base, scale, freqs, offsets = rope_case_inputs(z, name, prescale=False)
        _, H, L, D = x.shape
        n = H * D
        packed = np.zeros((n, n // 4), np.uint32)
        r = np.arange(n)
        packed[r, r // 4] = (1 << (8 * (r % 4))).astype(np.uint32)
        one = O.to_dtype_bits(np.ones((n, n // 32), np.float32), O.BF16)
        spec = dict(head_dim=D, k_proj=(packed, one, np.zeros_like(one), 32, 8), v_proj=None,
                    k_norm=False, v_norm=False, eps=1e-6, rope_dims=dims,
                    rope_traditional=trad, rope_base=base, rope_scale=scale, rope_freqs=freqs,
                    rope_pre_scale=float(z[f"{name}/params"][4]))
        xin = x.transpose(0, 2, 1, 3).reshape(1, L, n)
        for off in offsets:
            k, _ = O.project_kv(xin, spec, off, O.BF16)
            check_rope_golden(k, z[f"{name}/out{off}"], f"project_kv {name}@{off}")


def test_struct_layout_matches_the_header(tmp_path):
    """ctypes' kvq_qlinear / kvq_kv_projection match the C header's."""
    import subprocess
    from kvq import _lib
    src = tmp_path / "sz.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "kvq.h"\n'
                   'int main(void){printf("%zu %zu %zu %zu %zu %zu %zu %zu\\n", sizeof(kvq_qlinear),'
                   ' sizeof(kvq_kv_projection), offsetof(kvq_kv_projection, k_norm_weight),'
                   ' offsetof(kvq_kv_projection, norm_eps), offsetof(kvq_kv_projection,'
                   ' rope_pre_scale), offsetof(kvq_kv_projection, rope_freqs),'
                   ' offsetof(kvq_kv_projection, q_proj), offsetof(kvq_kv_projection,'
                   ' q_norm_weight)); return 0;}\n')
    exe = tmp_path / "sz"
    inc = os.path.join(os.path.dirname(HERE), "include")
    subprocess.check_call(["gcc", "-I", inc, str(src), "-o", str(exe)])
    got = [int(v) for v in subprocess.check_output([str(exe)]).split()]
    P = _lib.KvProjection
    assert got == [ctypes.sizeof(_lib.QLinear), ctypes.sizeof(P), P.k_norm_weight.offset,
                   P.norm_eps.offset, P.rope_pre_scale.offset, P.rope_freqs.offset,
                   P.q_proj.offset, P.q_norm_weight.offset]


def test_rms_norm_known_answers():
    x = np.array([[3.0, -4.0, 0.0, 0.0]], np.float32)  # mean(x^2) = 6.25
    y = O.rms_norm(x, None, 0.0, O.F16)
    assert np.allclose(y, x / 2.5, rtol=0, atol=1e-3)
    w = np.array([2.0, 0.5, 1.0, 1.0], np.float32)
    y2 = O.rms_norm(x, w, 0.0, O.F16)
    assert np.array_equal(y2, O.round_dt(O.round_dt(x / 2.5, O.F16) * w, O.F16))


def test_quantized_linear_identity_weights_are_exact():
    D, gs = 64, 32
    codes = np.eye(D, dtype=np.uint32)  # 8-bit codes: word i//4, byte i%4
    packed = np.zeros((D, D // 4), np.uint32)
    for r in range(D):
        for c in range(D):
            packed[r, c // 4] |= codes[r, c] << (8 * (c % 4))
    one = O.to_dtype_bits(np.ones((D, D // gs), np.float32), O.BF16)
    zero = np.zeros_like(one)
    rng = np.random.default_rng(1)
    x = O.round_dt(rng.standard_normal((3, D)).astype(np.float32), O.BF16)
    y = O.quantized_linear(x, packed, one, zero, gs, 8, O.BF16)
    assert np.array_equal(y, x)


# ---- argument checks of the C ABI (no CUDA call is reached) ----

def _cache(lib, Desc, H=2, D=128):
    h = ctypes.c_void_p()
    d = Desc(1, H, D, 4, 64, O.BF16, 0, 0, 0)  # reserve_rows 0: no device memory
    assert lib.kvq_cache_create(ctypes.byref(d), ctypes.byref(h)) == 0
    return h


def _proj(_lib, hidden=256, out=256, bits=4, gs=64, rope_dims=128, packed=16):
    s = _lib.KvProjection()
    s.k_proj = _lib.QLinear(packed, 32, 0, bits, gs, hidden, out)
    s.v_from_k = 1
    s.rope_dims = rope_dims
    s.rope_base = 10000.0
    s.rope_scale = 1.0
    return s


@pytest.mark.parametrize("field,value,needle", [
    ("out", 200, "out_features"),
    ("bits", 3, "bits"),
    ("gs", 48, "group_size"),
    ("hidden", 100, "in_features"),
    ("rope_dims", 7, "rope_dims"),
    ("rope_dims", 130, "rope_dims"),
    ("packed", 8, "aligned"),
])
def test_append_projected_rejects_malformed_projection(field, value, needle):
    from kvq import _lib
    lib = _lib.lib()
    h = _cache(lib, _lib.Desc)
    try:
        s = _proj(_lib, **{field: value})
        n = ctypes.c_size_t()
        rc = lib.kvq_append_projected_workspace(h, 1, ctypes.byref(s), ctypes.byref(n))
        assert rc == _lib.ERR_ARG
        assert needle in lib.kvq_last_error().decode()
        rc = lib.kvq_append_projected(h, 64, 1, ctypes.byref(s), None, None, None, None, 0,
                                      None)
        assert rc == _lib.ERR_ARG
    finally:
        assert lib.kvq_cache_free(h) == 0


def test_append_projected_rejects_mismatched_v_proj_and_head_dim():
    from kvq import _lib
    lib = _lib.lib()
    h = _cache(lib, _lib.Desc)
    try:
        s = _proj(_lib)
        s.v_from_k = 0
        s.v_proj = _lib.QLinear(16, 32, 0, 8, 64, 256, 256)  # bit width differs from k_proj
        n = ctypes.c_size_t()
        assert lib.kvq_append_projected_workspace(h, 1, ctypes.byref(s), ctypes.byref(n)) == \
            _lib.ERR_ARG
        assert "bit width" in lib.kvq_last_error().decode()
        s.v_proj = _lib.QLinear(16, 32, 0, 4, 64, 512, 256)  # in_features differ
        assert lib.kvq_append_projected_workspace(h, 1, ctypes.byref(s), ctypes.byref(n)) == \
            _lib.ERR_ARG
        assert lib.kvq_append_projected(None, 64, 1, ctypes.byref(s), None, None, None, None, 0,
                                        None) == _lib.ERR_ARG
    finally:
        assert lib.kvq_cache_free(h) == 0
    h2 = _cache(lib, _lib.Desc, H=1, D=512)  # head_dim above the fused path's 256
    try:
        s = _proj(_lib, out=512, rope_dims=0)
        n = ctypes.c_size_t()
        assert lib.kvq_append_projected_workspace(h2, 1, ctypes.byref(s), ctypes.byref(n)) == \
            _lib.ERR_ARG
        assert "head_dim" in lib.kvq_last_error().decode()
    finally:
        assert lib.kvq_cache_free(h2) == 0


def test_append_projected_rejects_malformed_query_side():
    from kvq import _lib
    lib = _lib.lib()
    h = _cache(lib, _lib.Desc)  # 2 kv heads of 128
    try:
        n = ctypes.c_size_t()
        s = _proj(_lib)
        s.q_proj = _lib.QLinear(16, 32, 0, 4, 64, 256, 512)
        s.q_heads = 0  # a query projection needs its heads
        assert lib.kvq_append_projected_workspace(h, 1, ctypes.byref(s), ctypes.byref(n)) == \
            _lib.ERR_ARG
        assert "q_heads" in lib.kvq_last_error().decode()
        s.q_heads = 3  # 3 x 128 != 512 output features
        assert lib.kvq_append_projected_workspace(h, 1, ctypes.byref(s), ctypes.byref(n)) == \
            _lib.ERR_ARG
        assert "q_proj" in lib.kvq_last_error().decode()
        s.q_heads = 4
        s.q_proj = _lib.QLinear(16, 32, 0, 4, 64, 512, 512)  # in_features differ from k_proj's
        assert lib.kvq_append_projected_workspace(h, 1, ctypes.byref(s), ctypes.byref(n)) == \
            _lib.ERR_ARG
        s.q_proj = _lib.QLinear(16, 32, 0, 4, 64, 256, 512)
        # a well-formed query side, but no q_out: refused before any CUDA call
        assert lib.kvq_append_projected(h, 64, 1, ctypes.byref(s), None, None, None, None, 0,
                                        None) == _lib.ERR_ARG
        assert "q_out" in lib.kvq_last_error().decode()
    finally:
        assert lib.kvq_cache_free(h) == 0
