"""Batched serving, conversion and persistence on the GPU, against the oracle.

* Ragged appends (kvq_append_ragged): sequences at different lengths in one
  cache, positions in a device array.  A ragged prefill (per-entry row
  counts) and single-row decode steps leave every entry's rows bit-exact
  with a per-sequence oracle cache fed the same rows, and the decode over
  per-sequence seq_lens matches the oracle's attention (2e-3).  Recorded
  once in a CUDA graph, append + decode lands at the next row on every
  replay.  An entry that would pass the capacity is skipped and reported.
* Conversion (kvq_cache_from_dense): a dense bf16 ring driven past its wrap
  (tests/rotating-kvq.test.ts:107-167) and a dense growing buffer with
  padding convert bit-exactly to the oracle's to_quantized, with offset and
  ring index carried over, and keep working identically after the next
  appends.
* Persistence (MLXBUNKV1): growing and rotating quantized caches survive a
  save / load round trip bit for bit and continue identically; dense
  reference-kind entries convert on load.
"""
import numpy as np
import pytest

from helpers import BF16, F16, from_torch, max_abs, record_parity, to_torch_bits
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _np(t):
    import torch
    if t.dtype == torch.int32:
        return t.contiguous().cpu().numpy().view(np.uint32)
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _rows(rng, shape, dt):
    return O.to_dtype_bits(rng.standard_normal(shape).astype(np.float32), dt)


def _ragged_case(graph: bool):
    import torch
    import kvq
    dt, B, Hq, Hkv, D, gs, bits, cap = F16, 4, 8, 2, 128, 64, 4, 1024
    scale = 1.0 / np.sqrt(D)
    rng = np.random.default_rng(70 + graph)
    prompt = [300, 17, 512, 1]
    cache = kvq.QuantizedKVCache(gs, bits, reserve_rows=cap)
    oracles = [O.QuantizedKVCache(gs, bits, dt) for _ in range(B)]
    lens = torch.zeros(B, dtype=torch.int32, device="cuda")
    # ragged prefill: one padded [B, H, 512, D] input, per-entry row counts
    S = max(prompt)
    k, v = _rows(rng, (B, Hkv, S, D), dt), _rows(rng, (B, Hkv, S, D), dt)
    counts = torch.tensor(prompt, dtype=torch.int32, device="cuda")
    cache.append_ragged(to_torch_bits(k, dt), to_torch_bits(v, dt), lens, counts)
    for b in range(B):
        oracles[b].update_and_fetch(k[b:b + 1, :, :prompt[b]], v[b:b + 1, :, :prompt[b]])
    K, V = cache.fetch_all()
    steps = 4
    if graph:  # static inputs, one recorded step, replays with new contents
        sk = torch.empty(B, Hkv, 1, D, dtype=torch.float16, device="cuda")
        sv, sq = torch.empty_like(sk), torch.empty(B, Hq, 1, D, dtype=torch.float16, device="cuda")
        out = torch.empty_like(sq)
        sq.zero_()
        # size the decode workspace and cache the kernels' set-up before capture
        kvq.sdpa_decode(sq, K, V, scale, seq_lens=lens, out=out)
        torch.cuda.synchronize()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=side):
            cache.append_ragged(sk, sv, lens)
            kvq.sdpa_decode(sq, K, V, scale, seq_lens=lens, out=out)
    outs, wants = [], []
    for step in range(steps):
        kn, vn = _rows(rng, (B, Hkv, 1, D), dt), _rows(rng, (B, Hkv, 1, D), dt)
        q = _rows(rng, (B, Hq, 1, D), dt)
        if graph:
            sk.copy_(to_torch_bits(kn, dt))
            sv.copy_(to_torch_bits(vn, dt))
            sq.copy_(to_torch_bits(q, dt))
            g.replay()
            torch.cuda.synchronize()
            o = out.clone()
        else:
            cache.append_ragged(to_torch_bits(kn, dt), to_torch_bits(vn, dt), lens)
            o = kvq.sdpa_decode(to_torch_bits(q, dt), K, V, scale, seq_lens=lens)
        want = np.zeros((B, Hq, 1, D), np.uint16)
        for b in range(B):
            ok, ov = oracles[b].update_and_fetch(kn[b:b + 1], vn[b:b + 1])
            want[b] = O.sdpa_unfused(q[b:b + 1], ok, ov, scale, gs, bits, dt)[0]
        outs.append(from_torch(o, dt))
        wants.append(want)
    torch.cuda.synchronize()
    cache.check()
    n = [p + steps for p in prompt]
    assert lens.cpu().tolist() == n
    for b in range(B):
        for got, want in zip((K.packed, K.scales, K.biases, V.packed, V.scales, V.biases),
                             oracles[b].keys + oracles[b].values):
            assert np.array_equal(_np(got[b:b + 1, :, :n[b]]), want[:, :, :n[b]]), b
    for i, (got, want) in enumerate(zip(outs, wants)):
        record_parity(f"ragged append + decode ({'graph replay' if graph else 'eager'}) step {i}",
                      got, want, dt, f"<= {TOL}")
        assert max_abs(got, want, dt) <= TOL, i
    cache.dispose()


def test_ragged_append_decode_matches_per_sequence_oracles():
    _ragged_case(graph=False)


def test_ragged_append_in_cuda_graph_advances_positions():
    _ragged_case(graph=True)


def test_ragged_append_past_capacity_is_skipped_and_reported():
    import torch
    import kvq
    dt, B, Hkv, D, gs, bits, cap = F16, 3, 2, 64, 64, 8, 256
    cache = kvq.QuantizedKVCache(gs, bits, reserve_rows=cap)
    lens = torch.tensor([0, 250, 10], dtype=torch.int32, device="cuda")
    k = to_torch_bits(_rows(np.random.default_rng(3), (B, Hkv, 8, D), dt), dt)
    cache.append_ragged(k, k, lens)  # entry 1 would need rows 250..257
    torch.cuda.synchronize()
    assert lens.cpu().tolist() == [8, 250, 18]
    with pytest.raises(kvq.KvqError):
        cache.check()
    cache.check()  # reported once, then clear
    cache.dispose()


def _compare_triples(cache, oq, rows=None):
    K, V = cache.fetch()
    n = rows if rows is not None else K.shape[2]
    for got, want in zip((K.packed, K.scales, K.biases, V.packed, V.scales, V.biases),
                         list(oq[0]) + list(oq[1])):
        assert np.array_equal(_np(got[:, :, :n]), np.ascontiguousarray(want[:, :, :n]))


def test_from_dense_wrapped_ring_matches_oracle():
    import torch
    import kvq
    dt, MAX, H, D = BF16, 64, 2, 64
    rng = np.random.default_rng(9)
    ring = O.RotatingKVCache(MAX, dt)

    def uni(shape):  # U[-1, 1), the reference test's input range
        return O.to_dtype_bits(rng.uniform(-1, 1, shape).astype(np.float32), dt)

    for _ in range(70):
        ring.update_and_fetch(uni((1, H, 1, D)), uni((1, H, 1, D)))
    assert (ring.offset, ring.ring_idx, ring.seq_len) == (70, 6, 64)
    want = ring.to_quantized(64, 8)
    kd, vd = to_torch_bits(ring.keys[0], dt), to_torch_bits(ring.values[0], dt)
    q = kvq.RotatingQuantizedKVCache.from_dense(kd, vd, ring.offset, ring.ring_idx, MAX, 64, 8)
    torch.cuda.synchronize()
    assert (q.offset, q.ring_idx, q.seq_len) == (70, 6, 64)
    _compare_triples(q, (want.keys, want.values))
    # the reference's own check: dequantized ring within kv8 noise of the bf16 ring
    deq = O.dequantize(*want.keys, 64, 8, dt)
    assert np.abs(deq - O.from_dtype_bits(ring.keys[0], dt)).max() < 0.02
    # a post-conversion decode step on both
    kn, vn = uni((1, H, 1, D)), uni((1, H, 1, D))
    qk, qv = q.update_and_fetch_quantized(to_torch_bits(kn, dt), to_torch_bits(vn, dt))
    ok, ov = want.update_and_fetch(kn, vn)
    assert (q.offset, q.ring_idx, q.seq_len) == (want.offset, want.ring_idx, want.seq_len)
    _compare_triples(q, (ok, ov))
    qq = _rows(rng, (1, 4, 1, D), dt)
    out = kvq.quantized_sdpa(to_torch_bits(qq, dt), qk, qv, 0.125, q.make_mask(1, None))
    torch.cuda.synchronize()
    assert max_abs(from_torch(out, dt), O.sdpa_unfused(qq, ok, ov, 0.125, 64, 8, dt), dt) <= 2 / 128
    q.dispose()


def test_from_dense_growing_buffer_with_padding():
    import torch
    import kvq
    dt, B, H, D, gs, bits = F16, 2, 2, 128, 64, 4
    rng = np.random.default_rng(10)
    dense = O.KVCache(dt)
    for S in (300, 1, 5):
        k, v = _rows(rng, (B, H, S, D), dt), _rows(rng, (B, H, S, D), dt)
        dense.update_and_fetch(k, v)
    want = dense.to_quantized(gs, bits)
    kd = to_torch_bits(dense.keys[0], dt)
    vd = to_torch_bits(dense.values[0], dt)
    q = kvq.QuantizedKVCache.from_dense(kd, vd, dense.offset, gs, bits)
    torch.cuda.synchronize()
    assert (q.offset, q.seq_len) == (306, 512)
    K, V = q.fetch()
    for got, w in zip((K.packed, K.scales, K.biases), want.keys):
        assert np.array_equal(_np(got), w[:, :, :306])
    # continue: a short append inside the buffer, then one that re-grows it
    for S in (3, 300):
        k, v = _rows(rng, (B, H, S, D), dt), _rows(rng, (B, H, S, D), dt)
        q.update_and_fetch_quantized(to_torch_bits(k, dt), to_torch_bits(v, dt))
        want.update_and_fetch(k, v)
        assert (q.offset, q.seq_len) == (want.offset, want.seq_len)
        torch.cuda.synchronize()
        _compare_triples(q, want.fetch())
    q.dispose()


def test_save_load_roundtrip_growing_and_ring(tmp_path):
    import torch
    import kvq
    dt = F16
    rng = np.random.default_rng(11)
    g = kvq.QuantizedKVCache(64, 8)
    r = kvq.RotatingQuantizedKVCache(64, 64, 4)
    for S in (100, 1, 1):
        k = _rows(rng, (2, 2, S, 128), dt)
        g.update_and_fetch_quantized(to_torch_bits(k, dt), to_torch_bits(k, dt))
    for S in [1] * 70:
        k = _rows(rng, (2, 2, S, 128), dt)
        r.update_and_fetch_quantized(to_torch_bits(k, dt), to_torch_bits(k, dt))
    path = str(tmp_path / "prompt.kv")
    kvq.save_kv_cache(path, [1, 2, 3], [g, r])
    hdr, start, raw = O.load_kv(path)  # the oracle's reader of the layout
    assert hdr["tokens"] == [1, 2, 3] and start % 16384 == 0
    assert [e["kind"] for e in hdr["caches"]] == ["kvq", "rotating-kvq"]
    assert hdr["caches"][1]["idx"] == 6 and hdr["caches"][1]["maxSize"] == 64
    assert all(e[n + "Offset"] % 16384 == 0 for e in hdr["caches"]
               for n in ("kPacked", "kScales", "kBiases", "vPacked", "vScales", "vBiases"))
    tokens, (g2, r2) = kvq.load_kv_cache(path, device=0)
    assert tokens == [1, 2, 3]
    # a reloaded growing cache's buffer is its live rows (restoreState keeps
    # the saved [0:offset] region), so only offset and contents carry over
    assert (g2.offset, g2.seq_len) == (g.offset, g.offset)
    assert (r2.offset, r2.ring_idx, r2.seq_len) == (r.offset, r.ring_idx, r.seq_len) == (70, 6, 64)
    for a, b in ((g, g2), (r, r2)):
        ea, eb = a.export(), b.export()
        assert all(np.array_equal(x, y) for x, y in zip(ea["tensors"], eb["tensors"]))
    # both continue identically
    for S in (1, 300):
        k = _rows(rng, (2, 2, S, 128), dt)
        for c in (g, g2):
            c.update_and_fetch_quantized(to_torch_bits(k, dt), to_torch_bits(k, dt))
        k = _rows(rng, (2, 2, S, 128), dt)
        for c in (r, r2):
            c.update_and_fetch_quantized(to_torch_bits(k, dt), to_torch_bits(k, dt))
    torch.cuda.synchronize()
    assert r.ring_idx == r2.ring_idx and r.seq_len == r2.seq_len
    for a, b in ((g, g2), (r, r2)):
        assert a.offset == b.offset
        ea, eb = a.export(), b.export()
        assert all(np.array_equal(x, y) for x, y in zip(ea["tensors"], eb["tensors"]))


def test_load_dense_reference_kinds_converts(tmp_path):
    import torch
    import kvq
    dt = BF16
    rng = np.random.default_rng(12)
    grow = O.KVCache(dt)
    for S in (200, 1):
        k = _rows(rng, (1, 2, S, 64), dt)
        grow.update_and_fetch(k, k)
    ring = O.RotatingKVCache(32, dt)
    for _ in range(40):
        k = _rows(rng, (1, 2, 1, 64), dt)
        ring.update_and_fetch(k, _rows(rng, (1, 2, 1, 64), dt))
    path = tmp_path / "dense.kv"
    gk = grow.keys[0][:, :, :grow.offset]  # the reference saves a growing cache's live rows
    O.save_kv(path, [9], [
        ({"kind": "kv", "offset": grow.offset, "dtype": dt, "kShape": list(gk.shape),
          "vShape": list(gk.shape)}, [("k", gk), ("v", gk)]),
        ({"kind": "rotating", "offset": ring.offset, "idx": ring.ring_idx, "maxSize": 32,
          "dtype": dt, "kShape": list(ring.keys[0].shape), "vShape": list(ring.values[0].shape)},
         [("k", ring.keys[0]), ("v", ring.values[0])])])
    tokens, (g2, r2) = kvq.load_kv_cache(str(path), quantize_dense=(8, 64))
    torch.cuda.synchronize()
    wr = ring.to_quantized(64, 8)
    assert (r2.offset, r2.ring_idx, r2.seq_len) == (wr.offset, wr.ring_idx, wr.seq_len)
    _compare_triples(r2, (wr.keys, wr.values))
    wg = O.quantize(gk, 64, 8, dt)
    assert (g2.offset, g2.seq_len) == (201, 201)
    _compare_triples(g2, (wg, wg))
