#!/usr/bin/env python
"""Generate tests/golden/qk_norm_golden.npz: the Qwen TypeB Q/K prologue (LayerNorm over each
whole token row with a head_dim weight tiled over the heads, then ApplyRoPEFull;
Compute/Formats/QwenHybridFormat.cs:141-142) computed by the reference's own shaders compiled for
the CPU (oracle/ref_glsl). Needs the reference checkout and oracle/_ref built
(python oracle/ref_glsl/build_ref.py). Inputs are seeded numpy draws.

Usage: python tests/golden/make_qk_norm_golden.py
"""
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

# (seq, n_heads, head_dim, start_pos, theta, x std, weight mean)
CASES = [(5, 4, 64, 0, 1e4, 1.0, 1.0), (3, 16, 128, 777, 1e6, 2.5, 0.8), (4, 2, 256, 12345, 1e7, 0.3, 1.2),
         (1, 7, 64, 9, 5e5, 1.0, 1.0)]
EPS = 1e-5


def main():
    from oracle.ref_glsl import ref

    if not ref.available():
        raise SystemExit("oracle/_ref/libref_glsl.so is missing; run oracle/ref_glsl/build_ref.py first")
    rng = np.random.default_rng(20240611)
    arrays, meta = {}, []
    for i, (seq, h, d, start, theta, std, wmean) in enumerate(CASES):
        x = rng.normal(0, std, (seq, h * d)).astype(np.float32)
        w = rng.normal(wmean, 0.1, d).astype(np.float32)
        arrays[f"x{i}"], arrays[f"w{i}"] = x, w
        arrays[f"y{i}"] = ref.qk_norm_rope(x, w, start, h, d, theta, EPS)
        meta.append(dict(seq=seq, n_heads=h, head_dim=d, start=start, theta=theta, eps=EPS))
    arrays["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    out = Path(__file__).resolve().parent / "qk_norm_golden.npz"
    np.savez_compressed(out, **arrays)
    print(out)


if __name__ == "__main__":
    main()
