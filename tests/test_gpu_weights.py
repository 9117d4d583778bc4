"""GPU parity of the weight products beside the op (aihost_dequantize, aihost_matmul_weights)
through the C ABI, against the reference's own shaders (golden vectors) and exact products.

Tolerances, stated per check:
  dequantisation to fp32: bit-exact against the reference shader (same fp32 operations, same
    order, no contraction); to fp16: that value rounded once, bit-exact;
  matmul against the reference's fp32 MatMulWeights (golden): max |gpu - ref| <= 2e-3 * max |ref|
    (the tensor cores take fp16 operands: A and the dequantised W are rounded to fp16 once;
    measured on the golden cases: <= 7.6e-4 * max |ref|);
  matmul against the exact (float64) product of the same fp16-rounded operands: per element
    |gpu - exact| <= 4e-6 * sum_k |a_k w_k| + (fp16 output: 2^-11 * |exact|) — fp32
    accumulation error only, which isolates the kernel from the operand rounding.
"""
import json
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import aihost_b200 as A
from aihost_b200 import gen
from aihost_b200.ops import WeightOps

pytestmark = pytest.mark.gpu
sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
from make_weights_golden import CASES, KINDS, case_inputs  # noqa: E402

Z = np.load(Path(__file__).resolve().parent / "golden" / "weights_golden.npz")
DEV = torch.device("cuda", 0)


def exact_bound_check(got, a16, w16, fp16_out):
    """got [M, N] against float64 a16 @ w16.T with the accumulation bound above."""
    a, w = a16.astype(np.float64), w16.astype(np.float64)
    exact = a @ w.T
    mag = np.abs(a) @ np.abs(w).T
    bound = 4e-6 * mag + (np.abs(exact) * 2.0 ** -11 if fp16_out else 0.0) + 1e-30
    err = np.abs(got.astype(np.float64) - exact)
    worst = float((err / bound).max())
    assert worst <= 1.0, f"max err / bound = {worst:.3g} (max err {err.max():.3g})"
    return float(err.max())


@pytest.mark.parametrize("i", range(len(CASES)))
def test_dequantize_matches_reference_shader(ctx, i):
    name, n_out, k, _ = CASES[i]
    blocks, _ = case_inputs(i)
    ops = WeightOps(ctx)
    wt = torch.from_numpy(blocks).to(DEV)
    w32 = ops.dequantize(wt, KINDS[name], n_out * k, torch.float32)
    w16 = ops.dequantize(wt, KINDS[name], n_out * k, torch.float16)
    torch.cuda.synchronize()
    ref = Z[f"w{i}"]
    assert np.array_equal(w32.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    assert np.array_equal(w16.cpu().numpy().view(np.uint16), ref.astype(np.float16).view(np.uint16))


@pytest.mark.parametrize("i", range(len(CASES)))
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
def test_matmul_kquant_matches_reference_shader(ctx, i, out_dtype):
    name, n_out, k, rows = CASES[i]
    blocks, a = case_inputs(i)
    ops = WeightOps(ctx)
    c = ops.mat_mul_weights(torch.from_numpy(a).to(DEV), torch.from_numpy(blocks).to(DEV), KINDS[name], n_out,
                            out_dtype=out_dtype)
    torch.cuda.synchronize()
    ctx.sync_status()
    got = c.float().cpu().numpy()
    ref = Z[f"c{i}"]
    assert np.abs(got - ref).max() <= 2e-3 * np.abs(ref).max()
    w16 = Z[f"w{i}"].astype(np.float16).reshape(n_out, k)
    exact_bound_check(got, a.astype(np.float16), w16, out_dtype == torch.float16)


@pytest.mark.parametrize("rows,k,n_out,kind", [
    (64, 4096, 4096, A.F16),      # decode-sized: 64-wide tiles, K split over CTAs
    (1, 2048, 1024, A.Q4_K),      # one token
    (77, 1536, 200, A.Q6_K),      # ragged rows and columns
    (4096, 2048, 2048, A.F16),    # 256-wide tiles fill the SMs: persistent, no split
    (300, 1024, 1032, A.Q5_K),    # 64-wide tiles, K split over a cluster of 5
    (16, 256, 512, A.F16),        # 4 K tiles: a cluster of 4, one K tile each
    (8, 64, 264, A.F16),          # one K tile: no split
    (64, 4096, 1024, A.Q5_K),     # Q5_K dequantised inside the GEMM, clusters of 8
    (128, 1536, 520, A.Q4_K),     # 128-row swapped tiles, ragged weight rows, 6 super-blocks: clusters of 2
    (16, 256, 264, A.Q5_K),       # one super-block: no split (clusters of one)
    (96, 2048, 4096, A.Q4_K),
])
def test_matmul_shapes_against_exact_product(ctx, rows, k, n_out, kind):
    ops = WeightOps(ctx)
    seed = rows * 7 + n_out
    a = gen.normal((rows, k), seed, "a", dtype=torch.float16)
    if kind == A.F16:
        w = gen.normal((n_out, k), seed, "w", std=0.02, dtype=torch.float16)
        w16 = w.numpy()
        wt = w.to(DEV)
    else:
        blocks = gen.kquant_blocks(kind, n_out * k // 256, seed, "w")
        w16 = ops.dequantize(blocks.to(DEV), kind, n_out * k, torch.float16).cpu().numpy().reshape(n_out, k)
        wt = blocks.to(DEV)
    c = ops.mat_mul_weights(a.to(DEV), wt, kind, n_out, out_dtype=torch.float32)
    torch.cuda.synchronize()
    ctx.sync_status()
    exact_bound_check(c.cpu().numpy(), a.numpy(), w16, False)


@pytest.mark.parametrize("n_parts", [2, 8])
def test_matmul_reads_rank_major_head_outputs_in_place(ctx, n_parts):
    """A as the KV-head-sharded all-gather leaves it, [N][B*S][Hq/N*d], gives bit for bit what
    the same product gives on the reference layout [B*S][Hq*d] (a permute of A)."""
    ops = WeightOps(ctx)
    rows, hq, d, n_out = 96, 32, 128, 4096
    g = gen.normal((n_parts, rows, hq // n_parts * d), 11, "heads", dtype=torch.float16).to(DEV)
    w = gen.normal((n_out, hq * d), 12, "wo", std=0.02, dtype=torch.float16).to(DEV)
    ref_layout = g.permute(1, 0, 2).reshape(rows, hq * d).contiguous()
    c_parts = ops.mat_mul_weights(g, w, A.F16, n_out, n_parts=n_parts, out_dtype=torch.float32)
    c_ref = ops.mat_mul_weights(ref_layout, w, A.F16, n_out, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.equal(c_parts, c_ref)
    exact_bound_check(c_ref.cpu().numpy(), ref_layout.cpu().numpy(), w.cpu().numpy(), False)


def test_matmul_repeated_calls_are_deterministic(ctx):
    """The K-split reduction sums the splits in a fixed order: repeated calls agree bit for bit."""
    ops = WeightOps(ctx)
    a = gen.normal((32, 4096), 3, "a", dtype=torch.float16).to(DEV)
    w = gen.normal((2048, 4096), 3, "w", std=0.02, dtype=torch.float16).to(DEV)
    outs = [ops.mat_mul_weights(a, w, A.F16, 2048, out_dtype=torch.float32) for _ in range(3)]
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
