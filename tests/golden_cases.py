"""Loader for tests/golden/attn_golden.npz (outputs of the reference's own shaders on the CPU)."""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden" / "attn_golden.npz"


def load():
    z = np.load(GOLDEN)
    meta = json.loads(bytes(z["meta"]).decode())
    return z, meta


def case_layout(meta_case, x, kv_dtype_code, q_dtype_code, out_dtype_code):
    """Arguments of one fused call (batch 1) reproducing a golden case: desc fields and host arrays."""
    from aihost_b200 import ROPE_INTERLEAVED
    from aihost_b200.ops import LayerSpec

    S, P = meta_case["S"], meta_case["P"]
    hq, hkv, d = meta_case["n_q_heads"], meta_case["n_kv_heads"], meta_case["head_dim"]
    spec = LayerSpec(hq, hkv, d, rope_theta=meta_case["theta"], rope_mode=ROPE_INTERLEAVED, q_dtype=q_dtype_code,
                     kv_dtype=kv_dtype_code, out_dtype=out_dtype_code, kv_capacity=P + S)
    return spec, S, P, hq, hkv, d
