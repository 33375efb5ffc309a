"""Extract mlx-bun's RoPE golden vectors into one committed fixture.

Source: mlx-bun ``tests/fixtures/universal-rope/`` (``manifest.json`` + raw
f32 blobs), dumped from MLX 0.31.2 on an Apple M1 Max by the reference's
``scripts/gen-universal-rope-fixtures.py`` and checked bit-exactly by its
``tests/universal-rope.test.ts:58-100``: for each rope variant, the input
(applied as bf16), the frequency table where the variant has one, the
pre-rope input scale (yarn mscale / longrope su scale, applied to
x[..., :dims] by UniversalRope.apply, src/model/universal/rope.ts:51-75),
and the mlx fast::rope output at offsets 0 and 5 (bf16 values as f32).

Stored per case ``<name>/input``, ``<name>/out<offset>``, ``<name>/freqs``
(cases with a table) and ``<name>/params`` = [dims, base, scale,
traditional, pre_scale, pre_scale_always, offset0, offset1] (f64).  The
fast_rope scale is 1 / factor for the "linear" variant and 1 otherwise
(rope.ts:40-41).  The gelu case is not extracted (not on this path).

Usage: python tests/golden/make_universal_rope_fixture.py <mlx-bun checkout>
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref_root: str) -> None:
    fix = os.path.join(ref_root, "tests", "fixtures", "universal-rope")
    man = json.load(open(os.path.join(fix, "manifest.json")))
    out = {}
    names = []
    for c in man["cases"]:
        if c.get("kind") == "gelu":
            continue
        name = c["name"]
        names.append(name)
        f32 = lambda fn: np.fromfile(os.path.join(fix, fn), dtype="<f4")  # noqa: E731
        shape = tuple(c["shape"])
        out[f"{name}/input"] = f32(f"{name}-input.bin").reshape(shape)
        for off in c["offsets"]:
            out[f"{name}/out{off}"] = f32(f"{name}-out{off}.bin").reshape(shape)
        if c.get("has_freqs"):
            out[f"{name}/freqs"] = f32(f"{name}-freqs.bin")
        sc = c.get("scaling_config") or {}
        scale = 1.0 / sc["factor"] if sc.get("rope_type") == "linear" else 1.0
        if "su_scale" in c:
            pre, always = c["su_scale"], 1.0
        else:
            pre, always = c.get("mscale", 1.0), 0.0
        out[f"{name}/params"] = np.array(
            [c["dims"], c["base"], scale, 1.0 if c.get("traditional") else 0.0, pre, always]
            + [float(o) for o in c["offsets"]], np.float64)
    out["names"] = np.array(names)
    out["mlx_version"] = np.array(man["oracle"]["mlx"])
    np.savez_compressed(os.path.join(HERE, "universal_rope.npz"), **out)
    print(f"wrote {len(names)} cases")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])
