"""Decode / prefill / partial+merge / logits on the GPU vs the oracle op graph.

The oracle is the CPU restatement of quantizedSdpaUnfused
(src/model/gemma4-base.ts:1273-1342) on the same seeded, quantized inputs.
Tolerances (written per dtype below):
  * fp16 outputs: max |diff| <= 2e-3;
  * bf16 outputs: max |diff| <= 2/128, the reference's own bound for its
    online-softmax path vs the unfused graph (tests/fused-sdpa.test.ts:105-108);
  * logits: max |diff| <= 1e-2 (fp16) / 6e-2 (bf16, one bf16 ulp at 8).
  * inputs with key-outlier channels: see helpers.check_outlier_parity
    (>= 99.99% within 2e-3, all within 1e-2, and no farther from the exact
    float64 result than the oracle).
"""
import numpy as np
import pytest

from helpers import BF16, F16, as_qtensor, check_outlier_parity, from_torch, ideal_sdpa, max_abs, \
    quantized_inputs, record_parity, to_torch_bits, upload_triple
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = {F16: 2e-3, BF16: 2.0 / 128}
LOGIT_TOL = {F16: 1e-2, BF16: 6e-2}


def run_decode(B, Hq, Hkv, N, D, gs, bits, dt, seed=0, k_outliers=0, seq_lens=None, scale=None,
               inputs=False):
    import kvq
    import torch
    rng = np.random.default_rng(seed)
    q, kq, vq = quantized_inputs(rng, B, Hq, Hkv, N, D, gs, bits, dt, k_outliers=k_outliers)
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    want = O.sdpa_unfused(q, kq, vq, scale, gs, bits, dt, seq_lens=seq_lens)
    kt = upload_triple(*kq, gs, bits)
    vt = upload_triple(*vq, gs, bits)
    K = as_qtensor(*kt[:3], N, gs, bits, dt)
    V = as_qtensor(*vt[:3], N, gs, bits, dt)
    sl = None if seq_lens is None else torch.tensor(seq_lens, dtype=torch.int32, device="cuda")
    out = kvq.sdpa_decode(to_torch_bits(q, dt), K, V, scale, seq_lens=sl)
    torch.cuda.synchronize()
    if inputs:
        return from_torch(out, dt), want, (q, kq, vq, scale)
    return from_torch(out, dt), want


DECODE_CASES = [
    # B, Hq, Hkv, N, D, gs, bits, dt, outliers
    (1, 16, 4, 2048, 128, 64, 8, F16, 0),     # config 1 (full size)
    (2, 32, 8, 1000, 128, 64, 4, F16, 4),     # config 2 shape, shorter context
    (1, 8, 4, 1024, 256, 64, 8, F16, 0),      # config 3 local-layer shape
    (1, 4, 2, 333, 256, 64, 4, F16, 0),       # odd N (reference decode-kernel test site)
    (1, 4, 2, 333, 256, 64, 8, BF16, 0),
    (1, 16, 1, 777, 128, 64, 4, BF16, 0),     # GQA 16 (two query n-tiles)
    (3, 4, 4, 100, 64, 32, 8, F16, 0),        # no GQA, gs 32, short
    (2, 6, 2, 515, 128, 128, 8, F16, 0),      # nrep 3, gs 128
    (1, 2, 1, 17, 64, 64, 4, F16, 0),         # tiny
    (1, 8, 8, 1, 128, 32, 4, F16, 0),         # single key
]


@pytest.mark.parametrize("case", DECODE_CASES, ids=lambda c: "-".join(map(str, c)))
def test_decode_matches_oracle(case):
    B, Hq, Hkv, N, D, gs, bits, dt, outl = case
    got, want, (q, kq, vq, scale) = run_decode(B, Hq, Hkv, N, D, gs, bits, dt, k_outliers=outl,
                                               inputs=True)
    assert got.shape == want.shape
    name = "decode " + "-".join(map(str, case))
    if outl:
        check_outlier_parity(got, want, ideal_sdpa(q, kq, vq, scale, gs, bits, dt), dt, name=name)
    else:
        record_parity(name, got, want, dt, f"<= {TOL[dt]}")
        err = max_abs(got, want, dt)
        assert err <= TOL[dt], err
    assert np.abs(O.from_dtype_bits(want, dt)).mean() > 1e-3


def test_decode_config2_full_size():
    """Config 2 at its full size: B 8, Hq 32, Hkv 8, D 128, N 8193, kv4, key outliers."""
    got, want, (q, kq, vq, scale) = run_decode(8, 32, 8, 8193, 128, 64, 4, F16, seed=2,
                                               k_outliers=4, inputs=True)
    check_outlier_parity(got, want, ideal_sdpa(q, kq, vq, scale, 64, 4, F16), F16,
                         name="decode config 2 full size (B8 Hq32 Hkv8 N8193 kv4, key outliers)")


def test_decode_ragged_seq_lens():
    lens = [1000, 1, 517, 64]
    got, want = run_decode(4, 8, 2, 1000, 128, 64, 4, F16, seed=3, seq_lens=lens)
    assert max_abs(got, want, F16) <= TOL[F16]


@pytest.mark.parametrize("lens", [[0, 3000, 0, 17, 1, 0], [1, 17, 0], [0, 0], [2999, 3000, 5, 2048]])
def test_decode_ragged_with_empty_entries(lens):
    """Entries with no keys give zero rows; a batch with fewer key tiles than
    the launch has CTAs still covers every tile exactly once."""
    got, want = run_decode(len(lens), 8, 2, 3000, 128, 64, 8, F16, seed=5, seq_lens=lens)
    assert max_abs(got, want, F16) <= TOL[F16]
    for b, n in enumerate(lens):
        if n == 0:
            assert not np.any(O.from_dtype_bits(got[b], F16))


def test_decode_one_long_unit_many_holders():
    """One (batch, kv head) unit over 20000 keys: its tiles spread over more
    CTAs than one merge pass takes, so the merge runs in several passes."""
    got, want = run_decode(1, 8, 1, 20000, 128, 64, 4, F16, seed=6)
    assert max_abs(got, want, F16) <= TOL[F16]


@pytest.mark.parametrize("case", [
    (1, 8, 2, 20000, 64, 64, 4, F16),     # two row slices per merge row
    (1, 4, 1, 12000, 256, 64, 8, BF16),   # eight slices, bf16
    (1, 8, 1, 20000, 128, 32, 4, BF16),   # four slices, bf16, group 32
], ids=lambda c: "-".join(map(str, c)))
def test_decode_long_units_wide_merge(case):
    """Units with hundreds of partial slots each take the wide merge: D / 32
    blocks per (unit, query row), one-warp slot groups; every head size's
    slicing against the oracle."""
    B, Hq, Hkv, N, D, gs, bits, dt = case
    got, want = run_decode(B, Hq, Hkv, N, D, gs, bits, dt, seed=60 + D)
    record_parity(f"decode, long units, wide merge {case}", got, want, dt, f"<= {TOL[dt]}")
    assert max_abs(got, want, dt) <= TOL[dt]


def test_decode_through_ring_cache_config3():
    """Config 3 local layer: window 1024 ring after 4096 writes (3 wraps), kv8 D256."""
    import kvq
    import torch
    dt, B, Hq, Hkv, D, W, gs, bits = F16, 2, 8, 4, 256, 1024, 64, 8
    rng = np.random.default_rng(4)
    cache = kvq.RotatingQuantizedKVCache(W, gs, bits)
    ocache = O.RotatingQuantizedKVCache(W, gs, bits, dt)
    for S in [2048, 1024, 1023, 1]:
        k = O.to_dtype_bits(rng.standard_normal((B, Hkv, S, D)).astype(np.float32), dt)
        v = O.to_dtype_bits(rng.standard_normal((B, Hkv, S, D)).astype(np.float32), dt)
        qk, qv = cache.update_and_fetch_quantized(to_torch_bits(k, dt), to_torch_bits(v, dt))
        ok, ov = ocache.update_and_fetch(k, v)
    assert cache.offset == 4096
    q = O.to_dtype_bits(rng.standard_normal((B, Hq, 1, D)).astype(np.float32), dt)
    want = O.sdpa_unfused(q, ok, ov, 1 / 16, gs, bits, dt)
    out = kvq.quantized_sdpa(to_torch_bits(q, dt), qk, qv, 1 / 16, cache.make_mask(1, None))
    torch.cuda.synchronize()
    assert max_abs(from_torch(out, dt), want, dt) <= TOL[dt]


PREFILL_CASES = [
    # B, Hq, Hkv, N, L, D, gs, bits, dt, window, outliers
    (1, 32, 8, 1536, 512, 128, 64, 8, F16, 0, 4),   # config 4 shape, shorter prior
    (1, 8, 2, 1217, 96, 64, 64, 4, F16, 0, 0),      # reference multi-tile kv4 case
    (1, 4, 4, 700, 64, 64, 32, 8, BF16, 0, 0),      # reference no-gqa case
    (2, 8, 4, 900, 40, 128, 64, 8, F16, 256, 0),    # sliding window
    (1, 16, 1, 300, 48, 128, 64, 8, F16, 0, 0),     # GQA 16
    (1, 4, 2, 333, 333, 128, 64, 4, F16, 0, 0),     # full prefill (offset 0)
    # kv8 / D 128 / group 64 run on the tensor-core (tcgen05) prefill:
    (1, 32, 8, 1100, 256, 128, 64, 8, BF16, 0, 0),  # bf16 cache
    (1, 8, 2, 2000, 300, 128, 64, 8, F16, 64, 0),   # window 64: later rows' first tiles all masked
    (2, 8, 2, 650, 5, 128, 64, 8, F16, 0, 0),       # 20 query rows: one padded 128-row tile
    (1, 4, 1, 400, 400, 128, 64, 8, F16, 0, 0),     # offset 0, keys end mid-tile
    # fp16 D 128 shapes of the warp-specialised tcgen05 prefill (kv4, kv8 group 32 / 128):
    (1, 32, 8, 1536, 512, 128, 64, 4, F16, 0, 4),   # config 4 shape in kv4, key outliers
    (2, 8, 2, 1000, 200, 128, 32, 4, F16, 0, 0),    # kv4 group 32, two batch entries
    (1, 8, 2, 900, 130, 128, 128, 8, F16, 0, 0),    # kv8 group 128, 520 query rows: a padded block
    (1, 16, 4, 1200, 300, 128, 64, 4, F16, 200, 0), # kv4 sliding window 200
    (1, 4, 1, 77, 77, 128, 32, 8, F16, 0, 0),       # kv8 group 32, offset 0, one partial tile
]


@pytest.mark.parametrize("case", PREFILL_CASES, ids=lambda c: "-".join(map(str, c)))
def test_prefill_matches_oracle(case):
    import kvq
    import torch
    B, Hq, Hkv, N, L, D, gs, bits, dt, window, outl = case
    rng = np.random.default_rng(21)
    q, kq, vq = quantized_inputs(rng, B, Hq, Hkv, N, D, gs, bits, dt, L=L, k_outliers=outl)
    scale = 1.0 / np.sqrt(D)
    want = O.sdpa_unfused(q, kq, vq, scale, gs, bits, dt, mask_mode=1, window=window)
    K = as_qtensor(*upload_triple(*kq, gs, bits)[:3], N, gs, bits, dt)
    V = as_qtensor(*upload_triple(*vq, gs, bits)[:3], N, gs, bits, dt)
    out = kvq.sdpa_prefill(to_torch_bits(q, dt), K, V, scale, kvq.Mask("causal", window))
    torch.cuda.synchronize()
    name = "prefill " + "-".join(map(str, case))
    if outl:
        ideal = ideal_sdpa(q, kq, vq, scale, gs, bits, dt, mask_mode=1, window=window)
        check_outlier_parity(from_torch(out, dt), want, ideal, dt, name=name)
    else:
        record_parity(name, from_torch(out, dt), want, dt, f"<= {TOL[dt]}")
        assert max_abs(from_torch(out, dt), want, dt) <= TOL[dt]


def test_prefill_no_mask_and_single_row():
    import kvq
    import torch
    dt, B, Hq, Hkv, N, D, gs, bits = F16, 1, 8, 2, 400, 128, 64, 8
    rng = np.random.default_rng(8)
    for L, mode, window in ((16, 0, 0), (1, 1, 100)):
        q, kq, vq = quantized_inputs(rng, B, Hq, Hkv, N, D, gs, bits, dt, L=L)
        want = O.sdpa_unfused(q, kq, vq, 0.1, gs, bits, dt, mask_mode=mode, window=window)
        K = as_qtensor(*upload_triple(*kq, gs, bits)[:3], N, gs, bits, dt)
        V = as_qtensor(*upload_triple(*vq, gs, bits)[:3], N, gs, bits, dt)
        m = kvq.Mask("causal" if mode else "", window)
        out = kvq.sdpa_prefill(to_torch_bits(q, dt), K, V, 0.1, m)
        torch.cuda.synchronize()
        assert max_abs(from_torch(out, dt), want, dt) <= TOL[dt]


def test_prefill_small_workspace_runs_per_unit_grid():
    """A caller workspace too small for the balanced grid's partial slots
    runs the tensor-core prefill with one CTA per (query block, kv head,
    batch entry); both grids match the oracle and each other."""
    import kvq
    import torch
    dt, B, Hq, Hkv, N, L, D, gs, bits = F16, 2, 8, 2, 1500, 300, 128, 64, 8
    rng = np.random.default_rng(12)
    q, kq, vq = quantized_inputs(rng, B, Hq, Hkv, N, D, gs, bits, dt, L=L)
    scale = 1.0 / np.sqrt(D)
    want = O.sdpa_unfused(q, kq, vq, scale, gs, bits, dt, mask_mode=1)
    K = as_qtensor(*upload_triple(*kq, gs, bits)[:3], N, gs, bits, dt)
    V = as_qtensor(*upload_triple(*vq, gs, bits)[:3], N, gs, bits, dt)
    qt, m = to_torch_bits(q, dt), kvq.Mask("causal", 0)
    balanced = kvq.sdpa_prefill(qt, K, V, scale, m)
    small_ws = torch.zeros(262_400 + (1 << 20), dtype=torch.uint8, device="cuda")  # < 20 MB
    per_unit = kvq.sdpa_prefill(qt, K, V, scale, m, workspace=small_ws)
    torch.cuda.synchronize()
    kvq.sdpa.check_device()  # the library-managed workspace's error flag
    assert int(small_ws[:4].view(torch.int32).item()) == 0  # the caller workspace's flag
    got_b, got_u = from_torch(balanced, dt), from_torch(per_unit, dt)
    assert max_abs(got_b, want, dt) <= TOL[dt]
    assert max_abs(got_u, want, dt) <= TOL[dt]
    assert max_abs(got_b, got_u, dt) <= TOL[dt]


@pytest.mark.parametrize("dt", [F16, BF16])
def test_logits_match_oracle(dt):
    import kvq
    import torch
    B, Hq, Hkv, N, L, D, gs, bits = 1, 8, 2, 300, 4, 128, 64, 4
    rng = np.random.default_rng(12)
    q, kq, vq = quantized_inputs(rng, B, Hq, Hkv, N, D, gs, bits, dt, L=L, k_outliers=4)
    _, want = O.sdpa_unfused(q, kq, vq, 0.0883883, gs, bits, dt, mask_mode=1, want_scores=True)
    K = as_qtensor(*upload_triple(*kq, gs, bits)[:3], N, gs, bits, dt)
    got = kvq.debug_scores(to_torch_bits(q, dt), K, 0.0883883, kvq.Mask("causal", 0))
    torch.cuda.synchronize()
    got = got.cpu().numpy()
    finite = want > (-65504.0 if dt == F16 else -3.3e38)  # the oracle masks with finfo.min
    assert np.array_equal(np.isfinite(got), finite)
    assert np.max(np.abs(got[finite] - want[finite])) <= LOGIT_TOL[dt]


@pytest.mark.parametrize("parts", [2, 3, 4])
def test_context_split_partials_merge(parts):
    """Partials over contiguous key ranges + merge == one decode over all keys."""
    import kvq
    import torch
    dt, B, Hq, Hkv, N, D, gs, bits = F16, 2, 32, 8, 3000, 128, 64, 4
    rng = np.random.default_rng(30 + parts)
    q, kq, vq = quantized_inputs(rng, B, Hq, Hkv, N, D, gs, bits, dt)
    want = O.sdpa_unfused(q, kq, vq, 1 / np.sqrt(D), gs, bits, dt)
    bounds = np.linspace(0, N, parts + 1).astype(int)
    qt = to_torch_bits(q, dt)
    ms, ls, os_ = [], [], []
    for a, b in zip(bounds[:-1], bounds[1:]):
        sk = tuple(np.ascontiguousarray(x[:, :, a:b]) for x in kq)
        sv = tuple(np.ascontiguousarray(x[:, :, a:b]) for x in vq)
        K = as_qtensor(*upload_triple(*sk, gs, bits)[:3], b - a, gs, bits, dt)
        V = as_qtensor(*upload_triple(*sv, gs, bits)[:3], b - a, gs, bits, dt)
        m, l, o = kvq.sdpa_decode_partial(qt, K, V, 1 / np.sqrt(D))
        ms.append(m)
        ls.append(l)
        os_.append(o)
    out = kvq.sdpa_merge(torch.stack(ms), torch.stack(ls), torch.stack(os_), torch.float16)
    torch.cuda.synchronize()
    got = from_torch(out, dt).reshape(want.shape)
    assert max_abs(got, want, dt) <= TOL[dt]


def test_bad_arguments_raise():
    import kvq
    import torch
    dt = F16
    rng = np.random.default_rng(1)
    q, kq, vq = quantized_inputs(rng, 1, 6, 4, 64, 128, 64, 8, dt)
    K = as_qtensor(*upload_triple(*kq, 64, 8)[:3], 64, 64, 8, dt)
    with pytest.raises(kvq.KvqError):
        kvq.sdpa_decode(to_torch_bits(q, dt), K, K, 1.0)  # 6 query heads over 4 kv heads
    q2 = torch.zeros(1, 4, 1, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        kvq.sdpa_decode(q2, K, K, 1.0)  # dtype mismatch
