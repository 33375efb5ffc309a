"""Quantized-KV persistence in mlx-bun's MLXBUNKV1 file layout.

mlx-bun saves prompt caches to disk (src/kv-store.ts:1-46): the magic
``MLXBUNKV1\\n``, a u32 LE header length, a u32 LE data start, a JSON header
``{tokens, caches: [...]}`` and every tensor at a 16 KiB-aligned offset
(relative to the data start), so a file can be mapped and handed to the GPU
without copies.  Its header knows two kinds, ``"kv"`` and ``"rotating"``
(dense bf16 / fp16 caches).  This module keeps the layout and adds the two
quantized kinds the reference cannot persist:

  ``"kvq"``           growing cache: its live rows [0:offset];
  ``"rotating-kvq"``  ring: the whole buffer, with ``idx`` (ring index) and
                      ``maxSize``.

A quantized entry is ``{kind, offset, idx?, maxSize?, dtype, bits,
groupSize, shape: [B, H, rows, D]}`` plus ``{name}Offset`` / ``{name}Bytes``
for the six tensors kPacked, kScales, kBiases, vPacked, vScales, vBiases
(uint32 codes, dtype scales and biases, each [B, H, rows, *]).
``load_kv_cache`` also reads the reference's dense kinds and, given
``quantize_dense=(bits, group_size)``, converts them on load exactly as
toQuantized would (kvq_cache_from_dense).
"""
from __future__ import annotations

import json

import numpy as np

MAGIC = b"MLXBUNKV1\n"
ALIGN = 16384
TENSORS = ("kPacked", "kScales", "kBiases", "vPacked", "vScales", "vBiases")


def _align_up(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


def save_kv_cache(path: str, tokens, caches) -> None:
    """Write `caches` (kvq QuantizedKVCache / RotatingQuantizedKVCache, one
    per layer) and the prompt `tokens` to `path` (saveKvCache,
    src/kv-store.ts:54-123).  Synchronizes each cache's device."""
    entries, blobs, off = [], [], 0
    for c in caches:
        st = c.export()
        e = {"kind": st["kind"], "offset": int(st["offset"]), "dtype": int(st["dtype"]),
             "bits": int(st["bits"]), "groupSize": int(st["group_size"]),
             "shape": [int(x) for x in st["shape"]]}
        if st["kind"] == "rotating-kvq":
            e["idx"] = int(st["idx"])
            e["maxSize"] = int(st["max_size"])
        for name, a in zip(TENSORS, st["tensors"]):
            b = np.ascontiguousarray(a).tobytes()
            o = _align_up(off)
            e[name + "Offset"] = o
            e[name + "Bytes"] = len(b)
            blobs.append((o, b))
            off = o + len(b)
        entries.append(e)
    hj = json.dumps({"tokens": [int(t) for t in tokens], "caches": entries}).encode()
    start = _align_up(len(MAGIC) + 8 + len(hj))
    with open(path, "wb") as f:
        pre = bytearray(start)
        pre[:len(MAGIC)] = MAGIC
        pre[len(MAGIC):len(MAGIC) + 4] = len(hj).to_bytes(4, "little")
        pre[len(MAGIC) + 4:len(MAGIC) + 8] = start.to_bytes(4, "little")
        pre[len(MAGIC) + 8:len(MAGIC) + 8 + len(hj)] = hj
        f.write(pre)
        for o, b in blobs:
            f.seek(start + o)
            f.write(b)


def read_kv_header(path: str) -> dict:
    """Only the header (readKvHeader, src/kv-store.ts:126-143), plus
    ``dataStart``."""
    with open(path, "rb") as f:
        head = f.read(len(MAGIC) + 8)
        if head[:len(MAGIC)] != MAGIC:
            raise ValueError(f"{path}: not an mlx-bun KV cache file")
        n = int.from_bytes(head[len(MAGIC):len(MAGIC) + 4], "little")
        start = int.from_bytes(head[len(MAGIC) + 4:len(MAGIC) + 8], "little")
        hdr = json.loads(f.read(n))
    hdr["dataStart"] = start
    return hdr


def _tensor(mm, start, e, name, dtype, shape):
    o, nb = start + e[name + "Offset"], e[name + "Bytes"]
    a = np.frombuffer(mm, dtype=dtype, count=nb // np.dtype(dtype).itemsize, offset=o)
    return a.reshape(shape)


def load_kv_cache(path: str, device: int = 0, quantize_dense=None, reserve_rows: int = 0):
    """(tokens, caches) from `path` (loadKvCache, src/kv-store.ts:147-175).

    Quantized kinds come back as kvq caches on `device` holding the saved
    rows and state.  The reference's dense kinds ("kv", "rotating") need
    ``quantize_dense=(bits, group_size)``: they are uploaded and quantized as
    toQuantized does (whole buffer, ring order, state adopted)."""
    import torch
    from .cache import QuantizedKVCache, RotatingQuantizedKVCache, _CacheBase, torch_dtype
    hdr = read_kv_header(path)
    start = hdr["dataStart"]
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    caches = []
    for e in hdr["caches"]:
        kind = e["kind"]
        if kind in ("kvq", "rotating-kvq"):
            B, H, rows, D = e["shape"]
            W, G = D * e["bits"] // 32, D // e["groupSize"]
            shapes = [(B, H, rows, W), (B, H, rows, G), (B, H, rows, G)] * 2
            dts = [np.uint32, np.uint16, np.uint16] * 2
            tensors = [_tensor(mm, start, e, n, dt, sh) for n, dt, sh in zip(TENSORS, dts, shapes)]
            st = {"shape": [B, H, rows, D], "bits": e["bits"], "group_size": e["groupSize"],
                  "dtype": e["dtype"], "offset": e["offset"], "idx": e.get("idx"),
                  "max_size": e.get("maxSize"), "tensors": tensors}
            caches.append(_CacheBase.from_export(st, device=device, reserve_rows=reserve_rows))
        elif kind in ("kv", "rotating"):
            if quantize_dense is None:
                raise ValueError(f"{path}: dense '{kind}' entry; pass quantize_dense=(bits, "
                                 "group_size) to convert it on load")
            bits, gs = quantize_dense
            tdt = torch_dtype(e["dtype"])
            dev = torch.device("cuda", device)
            kv = []
            for n, shape in (("k", e["kShape"]), ("v", e["vShape"])):
                a = _tensor(mm, start, {"xOffset": e[n + "Offset"], "xBytes": e[n + "Bytes"]},
                            "x", np.uint16, tuple(shape))
                kv.append(torch.from_numpy(np.array(a).view(np.int16)).to(dev).view(tdt))
            if kind == "rotating":
                c = RotatingQuantizedKVCache.from_dense(kv[0], kv[1], e["offset"], e["idx"],
                                                        e["maxSize"], gs, bits, reserve_rows)
            else:
                c = QuantizedKVCache.from_dense(kv[0], kv[1], e["offset"], gs, bits, reserve_rows)
            torch.cuda.current_stream(dev).synchronize()
            caches.append(c)
        else:
            raise ValueError(f"{path}: unknown cache kind {kind!r}")
    return hdr["tokens"], caches
