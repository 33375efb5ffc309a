"""Host logic of conversion and persistence, on CPU.

* The dense cache restatements reproduce the bookkeeping the reference's
  wrapped-ring replay test expects (tests/rotating-kvq.test.ts:107-167):
  70 single-row writes into a 64-row ring leave offset 70, ring index 6 and a
  64-row buffer, carried over by to_quantized.
* maybe_quantize_kv follows maybeQuantizeKv's rules (src/generate.ts:101-129)
  on stand-in caches.
* The product's MLXBUNKV1 header reader parses a file written by the
  oracle's independent writer (src/kv-store.ts layout).
"""
import numpy as np

from oracle import oracle as O


def test_dense_ring_replay_bookkeeping():
    ring = O.RotatingKVCache(64, O.BF16)
    rng = np.random.default_rng(0)
    for _ in range(70):
        k = O.to_dtype_bits(rng.uniform(-1, 1, (1, 2, 1, 64)).astype(np.float32), O.BF16)
        ring.update_and_fetch(k, k)
    assert (ring.offset, ring.ring_idx, ring.seq_len) == (70, 6, 64)
    q = ring.to_quantized(64, 8)
    assert (q.offset, q.ring_idx, q.seq_len) == (70, 6, 64)
    deq = O.dequantize(*q.keys, 64, 8, O.BF16)
    assert np.abs(deq - O.from_dtype_bits(ring.keys[0], O.BF16)).max() < 0.02
    q.update_and_fetch(k, k)  # the converted cache keeps working
    assert (q.offset, q.seq_len) == (71, 64)


def test_dense_growing_to_quantized_keeps_padding():
    c = O.KVCache(O.F16)
    rng = np.random.default_rng(1)
    for S in (300, 1, 5):
        k = O.to_dtype_bits(rng.standard_normal((1, 2, S, 64)).astype(np.float32), O.F16)
        c.update_and_fetch(k, k)
    q = c.to_quantized(64, 4)
    assert (q.offset, q.seq_len) == (306, 512)
    zero = O.quantize(np.zeros((1, 2, 1, 64), np.uint16), 64, 4, O.F16)
    assert all(np.array_equal(a[:, :, 400:401], z) for a, z in zip(q.keys, zero))


class _Stub:
    def __init__(self, offset, keys=None):
        import torch
        self.offset = offset
        self.keys = torch.zeros(1) if keys is None else keys


def test_maybe_quantize_kv_rules():
    import kvq
    from kvq.convert import DenseKVCache, DenseRotatingKVCache

    class D(DenseKVCache):
        def to_quantized(self, group_size, bits, reserve_rows=0):
            return ("q", group_size, bits)

    class R(DenseRotatingKVCache):
        def to_quantized(self, group_size, bits, reserve_rows=0):
            return ("rq", group_size, bits)

    import torch
    z = torch.zeros(1)
    caches = [D(z, z, 0), D(z, z, 100), D(z, z, 6000), R(z, z, 7000, 3, 1024), "other"]
    out = kvq.maybe_quantize_kv(list(caches), kv_bits=8)
    assert out[0] is caches[0] and out[1] is caches[1]  # empty / below the 5000 default
    assert out[2] == ("q", 64, 8) and out[3] == ("rq", 64, 8) and out[4] == "other"
    out = kvq.maybe_quantize_kv(list(caches), kv_config=[kvq.KvQuantSpec(1, 4, 32)])
    assert out[1] == ("q", 32, 4)  # kv_config: start 0, only its layers
    assert all(out[i] is caches[i] for i in (0, 2, 3, 4))
    assert kvq.maybe_quantize_kv(list(caches)) == caches  # neither option: no-op


def test_header_reader_parses_reference_layout(tmp_path):
    import kvq
    p = tmp_path / "c.kv"
    k = np.arange(2 * 3 * 8, dtype=np.uint16).reshape(1, 2, 3, 8)
    O.save_kv(p, [5, 6, 7], [({"kind": "kv", "offset": 3, "dtype": 12, "kShape": [1, 2, 3, 8],
                               "vShape": [1, 2, 3, 8]}, [("k", k), ("v", k + 1)])])
    hdr = kvq.read_kv_header(str(p))
    assert hdr["tokens"] == [5, 6, 7] and hdr["dataStart"] % 16384 == 0
    e = hdr["caches"][0]
    assert e["kind"] == "kv" and e["kOffset"] % 16384 == 0 and e["vOffset"] % 16384 == 0
    raw = open(p, "rb").read()
    got = np.frombuffer(raw, np.uint16, count=k.size, offset=hdr["dataStart"] + e["vOffset"])
    assert np.array_equal(got.reshape(k.shape), k + 1)
