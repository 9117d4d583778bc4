"""The oracle against golden vectors produced by the reference's own shaders (CPU).

tests/golden/attn_golden.npz holds outputs of AIHost's GLSL attention shaders compiled for the
CPU (oracle/ref_glsl), driven in ComputeOps order. The oracle's faithful mode evaluates the
same fp32 operations in the same order and must reproduce them; glibc's expf/powf/cosf/sinf
may differ in the last bit between hosts, hence a 1e-6 bound instead of bit equality.
"""
import numpy as np
import pytest

from aihost_b200 import F32
from golden_cases import case_layout, load
from oracle import oracle as orc

import sys
from pathlib import Path
sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
from make_golden import CASES, case_inputs, inputs_digest  # noqa: E402

Z, META = load()


def run_oracle(name, mode):
    m = META[name]
    x = case_inputs(name)
    spec, S, P, hq, hkv, d = case_layout(m, x, F32, F32, F32)
    kc = np.zeros((P + S, hkv * d), np.float32)
    vc = np.zeros((P + S, hkv * d), np.float32)
    kc[:P], vc[:P] = x["k_cached"], x["v_cached"]
    kcb, vcb = kc.view(np.uint8).reshape(-1).copy(), vc.view(np.uint8).reshape(-1).copy()
    out = orc.attn_forward(spec.desc(), x["q"].reshape(1, S, hq, d), x["k_new"].reshape(1, S, hkv, d),
                           x["v_new"].reshape(1, S, hkv, d), kcb, vcb, np.array([P], np.int32), mode=mode)
    return out.reshape(S, hq * d), kcb.view(np.float32).reshape(P + S, -1)[P:]


@pytest.mark.parametrize("name", sorted(CASES))
def test_golden_inputs_unchanged(name):
    assert inputs_digest(case_inputs(name)) == META[name]["inputs_sha256"]


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_faithful_matches_reference_shaders(name):
    out, krot = run_oracle(name, orc.FAITHFUL)
    assert np.abs(out - Z[f"{name}.out"]).max() <= 1e-6
    assert np.abs(krot - Z[f"{name}.k_rotated"]).max() <= 1e-6


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_exact_close_to_reference_shaders(name):
    out, _ = run_oracle(name, orc.EXACT)
    assert np.abs(out - Z[f"{name}.out"]).max() <= 2e-5


def test_live_pin_against_reference_shaders():
    """When the reference checkout is present, re-run its shaders on fresh inputs: bit-exact."""
    from oracle.ref_glsl import ref

    if not ref.available():
        pytest.skip("oracle/_ref not built (no reference checkout)")
    rng = np.random.default_rng(11)
    for S, P, hq, hkv, d, theta in [(1, 77, 6, 2, 32, 1e4), (9, 5, 2, 1, 16, 1e6)]:
        q = rng.standard_normal((S, hq * d)).astype(np.float32)
        kn = rng.standard_normal((S, hkv * d)).astype(np.float32)
        vn = rng.standard_normal((S, hkv * d)).astype(np.float32)
        kc = rng.standard_normal((P, hkv * d)).astype(np.float32)
        vc = rng.standard_normal((P, hkv * d)).astype(np.float32)
        out, k_all, _ = ref.layer_attention(q, kn, vn, kc, vc, P, hq, hkv, d, theta)
        qr = orc.rope_full(q, P, hq, d, theta)
        kr = orc.rope_full(kn, P, hkv, d, theta)
        o2 = orc.mha(qr, np.concatenate([kc, kr]), np.concatenate([vc, vn]), hq, P, mode=orc.FAITHFUL)
        assert np.array_equal(k_all[P:], kr)
        assert np.array_equal(out, o2)


def _qk_golden():
    import json
    from pathlib import Path

    z = np.load(Path(__file__).resolve().parent / "golden" / "qk_norm_golden.npz")
    return z, json.loads(bytes(z["meta"]).decode())


def test_qk_norm_rope_oracle_matches_reference_shader_golden():
    """The oracle's Qwen TypeB prologue equals the reference's layer_norm + rope_full shaders bit for bit."""
    from oracle import oracle as orc

    z, meta = _qk_golden()
    for i, m in enumerate(meta):
        y = orc.qk_norm_rope(z[f"x{i}"], z[f"w{i}"], m["start"], m["n_heads"], m["head_dim"], m["theta"], m["eps"])
        assert np.array_equal(y, z[f"y{i}"]), (i, float(np.abs(y - z[f"y{i}"]).max()))


def test_qk_norm_rope_oracle_matches_live_reference_shader():
    from oracle import oracle as orc
    from oracle.ref_glsl import ref

    if not ref.available():
        pytest.skip("reference-shader harness not built (no reference checkout)")
    rng = np.random.default_rng(5)
    for seq, h, d, start in [(2, 3, 64, 4), (6, 8, 128, 100), (3, 5, 256, 2047), (2, 40, 128, 31)]:
        x = rng.normal(0, 2.0, (seq, h * d)).astype(np.float32)
        w = rng.normal(1.0, 0.3, d).astype(np.float32)
        assert np.array_equal(orc.qk_norm_rope(x, w, start, h, d, 1e6), ref.qk_norm_rope(x, w, start, h, d, 1e6))
