"""The weight products beside the op, without a GPU: the oracle's K-quant dequantisation and
MatMulWeights against golden vectors made by the reference's own shaders (CPU), the live pin when
the reference harness is built, and the C ABI's argument checks.

tests/golden/weights_golden.npz: QuantizationFormats.cs DequantizeQ2K..Q6K_Correct and
ComputeShaders.cs _inlineMatMulWeights compiled for the CPU (oracle/ref_glsl), on seeded inputs
(tests/golden/make_weights_golden.py). The oracle is compiled without contraction and evaluates
the same fp32 operations in the same order: bit-exact.
"""
import ctypes
import json
import sys
from pathlib import Path

import numpy as np
import pytest

import aihost_b200 as A
from aihost_b200.ops import MatMulDesc
from oracle import oracle as orc

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
from make_weights_golden import CASES, KINDS, case_inputs, digest  # noqa: E402

Z = np.load(Path(__file__).resolve().parent / "golden" / "weights_golden.npz")
META = json.loads(bytes(Z["meta"]).decode())


@pytest.mark.parametrize("i", range(len(CASES)))
def test_weights_golden_inputs_unchanged(i):
    assert digest(*case_inputs(i)) == META[i]["inputs_sha256"]


@pytest.mark.parametrize("i", range(len(CASES)))
def test_oracle_dequantize_matches_reference_shader(i):
    name, n_out, k, _ = CASES[i]
    blocks, _ = case_inputs(i)
    w = orc.dequantize(KINDS[name], blocks, n_out * k)
    assert np.array_equal(w.view(np.uint32), Z[f"w{i}"].view(np.uint32))


@pytest.mark.parametrize("i", range(len(CASES)))
def test_oracle_matmul_weights_matches_reference_shader(i):
    name, n_out, k, rows = CASES[i]
    _, a = case_inputs(i)
    c = orc.matmul_weights(a, Z[f"w{i}"].reshape(n_out, k), mode=orc.FAITHFUL)
    assert np.array_equal(c.view(np.uint32), Z[f"c{i}"].view(np.uint32))
    exact = orc.matmul_weights(a, Z[f"w{i}"].reshape(n_out, k), mode=orc.EXACT)
    assert np.abs(exact - c).max() <= 1e-5 * np.abs(c).max()


def test_live_pin_of_weight_shaders():
    """Fresh blocks of every K-quant type through the reference shaders and the oracle."""
    from oracle.ref_glsl import ref

    if not ref.available():
        pytest.skip("reference shader harness not built (no reference checkout)")
    from aihost_b200 import gen

    for kind in KINDS.values():
        blocks = gen.kquant_blocks(kind, 32, 99 + kind, "live").numpy()
        assert np.array_equal(orc.dequantize(kind, blocks, 32 * 256).view(np.uint32),
                              ref.dequantize(kind, blocks, 32 * 256).view(np.uint32))
    rng = np.random.default_rng(5)
    a = rng.standard_normal((9, 256)).astype(np.float32)
    w = (rng.standard_normal((24, 256)) * 0.05).astype(np.float32)
    assert np.array_equal(orc.matmul_weights(a, w, orc.FAITHFUL).view(np.uint32), ref.matmul_weights(a, w).view(np.uint32))


def _desc(**kw):
    base = dict(rows=64, k=4096, n_out=4096, n_parts=1, a_dtype=A.F16, w_dtype=A.Q4_K, out_dtype=A.F16)
    base.update(kw)
    return MatMulDesc(**base)


def _ws(d):
    need = ctypes.c_size_t()
    return A.lib().aihost_matmul_workspace_size(ctypes.byref(d), ctypes.byref(need)), need.value


def test_matmul_abi_validates_arguments():
    assert _ws(_desc())[0] == A.OK
    assert _ws(_desc(k=4000))[0] == A.EINVAL            # not a multiple of 64
    assert _ws(_desc(k=4096 + 64, w_dtype=A.Q4_K))[0] == A.EINVAL  # K-quant needs multiples of 256
    assert _ws(_desc(k=4096 + 64, w_dtype=A.F16))[0] == A.OK
    assert _ws(_desc(n_out=4100))[0] == A.EINVAL        # not a multiple of 8
    assert _ws(_desc(n_parts=3))[0] == A.EINVAL         # 4096 / 3 is not a multiple of 64
    assert _ws(_desc(n_parts=8))[0] == A.OK
    assert _ws(_desc(w_dtype=A.Q8_0))[0] == A.EINVAL    # the reference dequantises K-quants only
    assert _ws(_desc(a_dtype=A.Q4_K))[0] == A.EINVAL
    assert _ws(_desc(rows=0))[0] == A.EINVAL
    d = _desc()
    assert A.lib().aihost_matmul_weights(None, ctypes.byref(d), None, None, None, None) == A.EINVAL
    assert A.lib().aihost_dequantize(None, A.Q4_K, 256, None, A.F32, None) == A.EINVAL
    assert A.lib().aihost_dequantize(ctypes.c_void_p(16), A.F16, 256, ctypes.c_void_p(16), A.F32, None) == A.EINVAL


def test_matmul_workspace_covers_staging():
    """Scratch = fp16 copy of an fp32 A + fp16 copy of a non-fp16 weight (split K needs none)."""
    _, f16 = _ws(_desc(rows=8192, w_dtype=A.F16))  # tiles fill the SMs: no split, no staging
    assert f16 == 0
    _, q4 = _ws(_desc(rows=8192, w_dtype=A.Q4_K))
    assert q4 == 4096 * 4096 * 2
    _, both = _ws(_desc(rows=8192, a_dtype=A.F32, w_dtype=A.F32))
    assert both == 2 * 8192 * 4096 + 4096 * 4096 * 2


def test_matmul_workspace_in_gemm_dequantisation():
    """At most 128 rows of A with Q4_K / Q5_K weights: the GEMM dequantises the blocks itself, so
    no fp16 weight copy is staged; other K-quant types, fp32 weights and larger row counts stage it."""
    for kind in (A.Q4_K, A.Q5_K):
        for rows in (1, 64, 128):
            assert _ws(_desc(rows=rows, w_dtype=kind)) == (A.OK, 0)
        assert _ws(_desc(rows=129, w_dtype=kind))[1] == 4096 * 4096 * 2
    for kind in (A.Q2_K, A.Q3_K, A.Q6_K, A.F32):
        assert _ws(_desc(rows=64, w_dtype=kind))[1] == 4096 * 4096 * 2
    # an fp32 A is still converted, with the weight dequantised in the GEMM
    assert _ws(_desc(rows=64, a_dtype=A.F32, w_dtype=A.Q4_K))[1] == 64 * 4096 * 2
