"""Extract the cache-mechanics part of mlx-bun's rotating-KV-quant golden.

Source: mlx-bun ``goldens/rotating-kvq.{json,bin}`` (written by
``scripts/regen-rotating-kvq-goldens.ts:40-70`` from optiq's
RotatingQuantizedKVCache on MLX's GPU stream; config max_size 64, H 2, D 64,
group_size 32, bits 8, bf16 inputs).  The reference is not available where
tests run, so its mechanics section (30 update steps, 7 checkpoints) is
committed as ``rotating_kvq_mechanics.npz``; the end-to-end 12B logits are not
extracted (they need model weights).

All K/V inputs and scales/biases are bf16 values stored as f32 in the blob;
they are re-stored here as bf16 bit patterns (lossless: the low 16 bits of
every stored f32 are checked to be zero).

Usage: python tests/golden/make_rotating_kvq_fixture.py <mlx-bun checkout>
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref_root: str) -> None:
    man = json.load(open(os.path.join(ref_root, "goldens", "rotating-kvq.json")))
    blob = np.fromfile(os.path.join(ref_root, "goldens", "rotating-kvq.bin"), dtype=np.uint8)

    def take(t, kind):
        n = int(np.prod(t["shape"]))
        raw = blob[t["offset"] * 4:(t["offset"] + n) * 4].view(np.uint32).reshape(t["shape"])
        if kind == "u32":
            return raw.copy()
        assert not (raw & 0xFFFF).any(), "value is not a bf16"
        return (raw >> 16).astype(np.uint16)

    m = man["mechanics"]
    out = {"config": np.array([m["config"][k] for k in
                               ("max_size", "heads", "dim", "group_size", "bits")], np.int32)}
    out["steps_S"] = np.array([s["S"] for s in m["steps"]], np.int32)
    for i, s in enumerate(m["steps"]):
        out[f"step{i}_k"] = take(s["k"], "bf16")
        out[f"step{i}_v"] = take(s["v"], "bf16")
    cps = sorted(int(k) for k in m["checkpoints"])
    out["checkpoints"] = np.array(cps, np.int32)
    for c in cps:
        cp = m["checkpoints"][str(c)]
        out[f"cp{c}_state"] = np.array([cp["offset"], cp["idx"]], np.int64)
        for kv in "kv":
            out[f"cp{c}_{kv}_packed"] = take(cp[f"{kv}_packed"], "u32")
            out[f"cp{c}_{kv}_scales"] = take(cp[f"{kv}_scales"], "bf16")
            out[f"cp{c}_{kv}_biases"] = take(cp[f"{kv}_biases"], "bf16")
    np.savez_compressed(os.path.join(HERE, "rotating_kvq_mechanics.npz"), **out)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])
