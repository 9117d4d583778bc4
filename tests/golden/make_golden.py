#!/usr/bin/env python
"""Generate tests/golden/attn_golden.npz from the reference's own shaders run on the CPU.

Each case is one attention-layer step exactly as AIHost's TransformerLayer runs it
(ComputeOps.cs:1282-1304: RoPE(Q), RoPE(K), KVCache.Add, MultiHeadAttention), evaluated by
oracle/_ref/libref_glsl.so (the reference GLSL compiled for the CPU by
oracle/ref_glsl/build_ref.py). Inputs come from aihost_b200.gen with the seeds below and are
not stored; a SHA-256 of them is, so a change of the generator is detected. Prefill cases use
fp16-representable inputs so the fp16 GPU path sees the same values.

Usage (needs the reference checkout): python oracle/ref_glsl/build_ref.py &&
                                      python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from aihost_b200 import gen  # noqa: E402

OUT = Path(__file__).resolve().parent / "attn_golden.npz"

# name: (S new rows, P cached rows, Hq, Hkv, d, theta, std, fp16-representable inputs)
CASES = {
    "decode_tinyllama": (1, 512, 32, 4, 64, 1e4, 0.5, False),
    "decode_gqa4_d128": (1, 700, 8, 2, 128, 5e5, 1.0, False),
    "decode_mha_at_4096": (1, 4095, 4, 4, 64, 1e4, 1.0, False),
    "decode_first_token": (1, 0, 8, 2, 64, 1e4, 1.0, False),
    "prefill_qwen_like": (48, 0, 4, 2, 64, 1e6, 1.0, True),
    "prefill_chunked_d128": (40, 24, 4, 1, 128, 5e5, 1.0, True),
    "prefill_ragged_gqa7": (21, 0, 7, 1, 64, 1e6, 1.0, True),
}


def case_inputs(name: str):
    S, P, hq, hkv, d, theta, std, fp16 = CASES[name]
    seed = int(hashlib.sha256(name.encode()).hexdigest()[:8], 16)
    dt = torch.float16 if fp16 else torch.float32
    arrs = {
        "q": gen.normal((S, hq * d), seed, "q", std=std, dtype=dt),
        "k_new": gen.normal((S, hkv * d), seed, "k_new", std=std, dtype=dt),
        "v_new": gen.normal((S, hkv * d), seed, "v_new", std=std, dtype=dt),
        "k_cached": gen.normal((P, hkv * d), seed, "k_cached", std=std, dtype=dt),
        "v_cached": gen.normal((P, hkv * d), seed, "v_cached", std=std, dtype=dt),
    }
    return {k: v.float().numpy() for k, v in arrs.items()}


def inputs_digest(arrs) -> str:
    h = hashlib.sha256()
    for k in sorted(arrs):
        h.update(k.encode())
        h.update(np.ascontiguousarray(arrs[k], dtype=np.float32).tobytes())
    return h.hexdigest()


def main():
    from oracle.ref_glsl import ref

    if not ref.available():
        raise SystemExit("oracle/_ref/libref_glsl.so missing: run oracle/ref_glsl/build_ref.py first")
    payload, meta = {}, {}
    for name, (S, P, hq, hkv, d, theta, std, fp16) in CASES.items():
        x = case_inputs(name)
        out, k_all, v_all = ref.layer_attention(x["q"], x["k_new"], x["v_new"], x["k_cached"], x["v_cached"], P, hq,
                                                hkv, d, theta)
        payload[f"{name}.out"] = out
        payload[f"{name}.k_rotated"] = k_all[P:]
        meta[name] = {"S": S, "P": P, "n_q_heads": hq, "n_kv_heads": hkv, "head_dim": d, "theta": theta, "std": std,
                      "fp16_inputs": fp16, "inputs_sha256": inputs_digest(x)}
        print(f"{name}: out {out.shape}, |out|max {np.abs(out).max():.3f}")
    payload["meta"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(OUT, **payload)
    print(OUT, OUT.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
