"""GPU parity of the fused op (RoPE + KV append + attention) against the CPU oracle.

Every case runs libaihost_attn.so through its C ABI on cuda:0 and the oracle
(oracle/attn_oracle.c, ORACLE_EXACT: double accumulation) on the same seeded inputs.
Tolerances (max |gpu - oracle| over every output element):
  fp16 inputs / fp16 cache:  2e-3   (the north-star bound for fp16 inputs)
  fp32 inputs / fp32 cache:  2e-4
  Q8_0 cache:                2e-3   (against the dequantise-then-attend oracle)
  fp32 prefill:              1e-3   (the tensor-core prefill reads fp16 copies of fp32 operands
                                     and rounds P to fp16; accumulation stays fp32)
Appended cache rows: V rows are bit-exact (fp16 round-to-nearest-even, fp32 copy, Q8_0 bytes);
K rows go through RoPE, whose cos/sin come from CUDA's sincosf on the GPU and glibc on the CPU
(1-ulp differences), so they are compared within one unit of the stored format.
"""
import numpy as np
import pytest
import torch

from aihost_b200 import F16, F32, Q8_0, ROPE_INTERLEAVED, ROPE_NEOX, ROPE_NONE
from aihost_b200.configs import CONFIGS, make_inputs
from helpers import cache_rows, gpu_forward, max_abs, oracle_forward

pytestmark = pytest.mark.gpu

TOL = {F16: 2e-3, F32: 2e-4, Q8_0: 2e-3}


TOL_F32_PREFILL = 1e-3


def tol_for(cfg):
    if cfg.kv_dtype == Q8_0:
        return TOL[Q8_0]
    if cfg.n_new > 1 and (cfg.q_dtype == F32 or cfg.kv_dtype == F32):
        return TOL_F32_PREFILL
    return TOL[cfg.q_dtype]


def check_call(ctx, cfg, pass_host_len=True, part=None, inp=None, check_cache=True):
    inp = inp or make_inputs(cfg)
    out, kc, vc = gpu_forward(ctx, cfg, inp, pass_host_len=pass_host_len)
    ref, rkc, rvc = oracle_forward(cfg, inp, part=part)
    out = out.float().numpy()
    if part is not None:
        b0, b1, h0, h1 = part
        out, ref = out[b0:b1, :, h0:h1], ref[b0:b1, :, h0:h1]
    err = max_abs(out, ref)
    assert np.isfinite(out).all()
    assert err <= tol_for(cfg), f"max |gpu - oracle| = {err:.3g} > {tol_for(cfg)}"
    if check_cache:
        lengths = inp["lengths"]
        rows = [list(range(n, n + cfg.n_new)) for n in lengths]
        cap = inp["capacity"]
        bl = slice(None) if part is None else slice(part[0], part[1])
        gv, rv = cache_rows(vc.numpy(), cfg, cap, rows)[bl], cache_rows(rvc, cfg, cap, rows)[bl]
        assert np.array_equal(gv, rv), "appended V rows differ from the oracle"
        if cfg.kv_dtype == Q8_0:
            gvb = vc.numpy().reshape(cfg.batch, cap, -1)
            rvb = rvc.reshape(cfg.batch, cap, -1)
            for b in range(cfg.batch)[bl]:
                assert np.array_equal(gvb[b, rows[b]], rvb[b, rows[b]]), "Q8_0 V blocks differ byte-wise"
        gk, rk = cache_rows(kc.numpy(), cfg, cap, rows)[bl], cache_rows(rkc, cfg, cap, rows)[bl]
        unit = {F32: 1e-5, F16: 2e-3}.get(cfg.kv_dtype, 0.03)
        assert max_abs(gk, rk) <= unit * max(1.0, float(np.abs(rk).max())), "appended K rows differ"
        # rows outside the appended range are untouched
        before = kc.numpy().reshape(cfg.batch, cap, -1)
        orig = inp["k_cache"].numpy().reshape(cfg.batch, cap, -1)
        for b in range(cfg.batch)[bl]:
            assert np.array_equal(before[b, :lengths[b]], orig[b, :lengths[b]])
    return err


# ---------------------------------------------------------------- decode (n_new == 1)

def test_decode_cfg1_fp32_full(ctx):
    check_call(ctx, CONFIGS[1])


@pytest.mark.parametrize("hq,hkv", [(4, 4), (8, 2), (16, 2), (32, 2), (12, 4)])
def test_decode_f16_gqa_ratios(ctx, hq, hkv):
    cfg = CONFIGS[3].scaled(batch=3, n_q_heads=hq, n_kv_heads=hkv, cached_range=None, cached_list=[0, 700, 1999])
    check_call(ctx, cfg)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("kv", [F32, F16, Q8_0])
def test_decode_dtypes_dims(ctx, d, kv):
    qd = F32 if kv == F32 else F16
    cfg = CONFIGS[3].scaled(batch=2, n_q_heads=16, n_kv_heads=2, head_dim=d, q_dtype=qd, kv_dtype=kv, out_dtype=qd,
                            cached_range=None, cached_list=[33, 1500])
    check_call(ctx, cfg)


@pytest.mark.parametrize("mode", [ROPE_NEOX, ROPE_NONE])
def test_decode_rope_modes(ctx, mode):
    cfg = CONFIGS[3].scaled(batch=2, rope_mode=mode, cached_range=None, cached_list=[100, 4097])
    check_call(ctx, cfg)


def test_decode_without_host_lengths(ctx):
    cfg = CONFIGS[3].scaled(batch=4, cached_range=None, cached_list=[5, 300, 2048, 4095])
    check_call(ctx, cfg, pass_host_len=False)


def test_decode_cfg3_full_sample(ctx):
    # full 64-sequence call on the GPU; oracle on sequences 0-3 (all heads)
    check_call(ctx, CONFIGS[3], part=(0, 4, 0, 32))


def test_decode_cfg5_q8_full_sample(ctx):
    check_call(ctx, CONFIGS[5], part=(0, 2, 0, 64))


@pytest.mark.parametrize("batch,hq,hkv,lengths", [
    (1, 8, 1, [5]),                                   # fewer tiles than CTAs: ranges of a few tiles
    (3, 16, 2, [1, 700, 64]),                         # ragged: a 1-row unit, tile-aligned lengths
    (4, 32, 8, [4095, 17, 2049, 300]),                # groups of 4 query heads
    (64, 64, 8, None),                                # 512 (sequence, KV head) units
    (65, 16, 8, None),
    (513, 8, 1, "short"),                             # more sequences than the schedule takes: per-split kernel
])
def test_decode_q8_stream_k_partitions(ctx, batch, hq, hkv, lengths):
    """Q8_0 decode over the stream-K schedule (every CTA an equal share of the cache tiles laid
    end to end; units split between CTAs merged by the last part): every unit, whole or split,
    must match the dequantise-then-attend oracle; the appended blocks byte for byte."""
    import numpy as np

    if lengths is None or lengths == "short":
        hi = 1500 if lengths is None else 200
        lengths = [int(x) for x in np.random.default_rng(batch).integers(1, hi, batch)]
    cfg = CONFIGS[5].scaled(batch=batch, n_q_heads=hq, n_kv_heads=hkv, cached=None, cached_list=lengths)
    check_call(ctx, cfg, part=(0, min(batch, 6), 0, hq))


def test_decode_stale_nan_rows_ignored(ctx):
    """Cache rows past each sequence's length hold NaN bit patterns; they must not leak."""
    cfg = CONFIGS[3].scaled(batch=2, n_q_heads=8, n_kv_heads=2, cached_range=None, cached_list=[40, 300])
    inp = make_inputs(cfg, capacity=512)
    for name in ("k_cache", "v_cache"):
        c = inp[name].view(torch.float16).reshape(cfg.batch, 512, cfg.n_kv_heads, cfg.head_dim)
        for b, n in enumerate(inp["lengths"]):
            c[b, n + 1:] = float("nan")
    check_call(ctx, cfg, inp=inp, check_cache=False)


# ---------------------------------------------------------------- prefill (n_new > 1)

def test_prefill_cfg2_full(ctx):
    check_call(ctx, CONFIGS[2], part=(0, 1, 0, 14))


def test_prefill_cfg4_full_sample(ctx):
    """Config 4 at its real size: S = 32768, Hq 32 / Hkv 8, d 128 (up to 256 cache tiles per query
    tile, thousands of online-softmax steps, the pair schedule at full occupancy). The whole call
    runs on the GPU; the oracle checks query heads 0 and 31 (the first and the last KV head) on
    the first query tile, a middle block and the last 256 rows, which attend every cache tile;
    the appended V rows of those KV heads must equal the oracle's bit for bit."""
    cfg = CONFIGS[4]
    inp = make_inputs(cfg)
    out, _, vc = gpu_forward(ctx, cfg, inp)
    out = out.float().numpy()
    assert np.isfinite(out).all()
    S, cap, D = cfg.n_new, inp["capacity"], cfg.head_dim
    gv = vc.numpy().view(np.float16).reshape(cap, cfg.n_kv_heads, D)
    for h in (0, cfg.n_q_heads - 1):
        kvh = h // (cfg.n_q_heads // cfg.n_kv_heads)
        for r0, r1 in ((0, 128), (S // 2 - 64, S // 2 + 64), (S - 256, S)):
            ref, _, rvc = oracle_forward(cfg, inp, part=(0, 1, h, h + 1), rows=(r0, r1))
            err = max_abs(out[:, r0:r1, h], ref[:, r0:r1, h])
            assert err <= TOL[F16], f"head {h} rows [{r0}, {r1}): max |gpu - oracle| = {err:.3g}"
        rv = rvc.view(np.float16).reshape(cap, cfg.n_kv_heads, D)
        assert np.array_equal(gv[:S, kvh], rv[:S, kvh]), f"appended V rows of KV head {kvh} differ"


@pytest.mark.parametrize("s", [2, 37, 128, 129, 300])
@pytest.mark.parametrize("d", [64, 128])
def test_prefill_ragged(ctx, s, d):
    cfg = CONFIGS[2].scaled(n_new=s, head_dim=d, n_q_heads=4, n_kv_heads=2, cached=0)
    check_call(ctx, cfg)


@pytest.mark.parametrize("d", [64, 128])
def test_prefill_pair_schedule(ctx, d):
    """A grid of more than two waves of query-tile pairs: the kernel pairs adjacent query tiles
    (shared K/V tiles) instead of splitting each tile's cache range over its two groups."""
    cfg = CONFIGS[2].scaled(batch=2, n_new=1200, n_q_heads=32, n_kv_heads=8, head_dim=d, cached=None,
                            cached_list=[0, 64])
    # the partial oracle appends only the KV heads of its query heads: compare the output only
    check_call(ctx, cfg, part=(0, 2, 0, 3), check_cache=False)


@pytest.mark.parametrize("cached", [[100], [1, 257]])
def test_prefill_chunked(ctx, cached):
    """Prefill after cached rows (chunked prefill): causal rule j <= P + i with P > 0."""
    cfg = CONFIGS[2].scaled(batch=len(cached), n_new=150, n_q_heads=6, n_kv_heads=2, head_dim=128, cached=None,
                            cached_list=cached)
    check_call(ctx, cfg)


@pytest.mark.parametrize("mode", [ROPE_NEOX, ROPE_NONE])
def test_prefill_rope_modes(ctx, mode):
    cfg = CONFIGS[2].scaled(n_new=200, n_q_heads=4, n_kv_heads=1, rope_mode=mode)
    check_call(ctx, cfg)


def test_prefill_f32_out(ctx):
    cfg = CONFIGS[2].scaled(n_new=130, n_q_heads=2, n_kv_heads=1, out_dtype=F32)
    check_call(ctx, cfg)


@pytest.mark.parametrize("d", [64, 128])
@pytest.mark.parametrize("cached", [[0], [100, 7]])
def test_prefill_fp32_reference_dtypes(ctx, d, cached):
    """The reference's own dtypes (fp32 q, cache and output) through prefill and chunked prefill."""
    cfg = CONFIGS[1].scaled(batch=len(cached), n_new=150, head_dim=d, n_q_heads=8, n_kv_heads=2, cached=None,
                            cached_list=cached)
    check_call(ctx, cfg)


@pytest.mark.parametrize("mode", [ROPE_INTERLEAVED, ROPE_NEOX])
def test_prefill_fp32_rope_modes_without_host_lengths(ctx, mode):
    cfg = CONFIGS[1].scaled(batch=2, n_new=130, n_q_heads=4, n_kv_heads=1, cached=None, cached_list=[0, 33],
                            rope_mode=mode)
    check_call(ctx, cfg, pass_host_len=False)


@pytest.mark.parametrize("d", [64, 128])
def test_prefill_q8_cache(ctx, d):
    """Chunked prefill over a Q8_0 cache: the new rows are quantised into the cache and every row
    is attended dequantised."""
    cfg = CONFIGS[5].scaled(batch=2, n_new=140, n_q_heads=8, n_kv_heads=2, head_dim=d, cached=None,
                            cached_list=[0, 300])
    check_call(ctx, cfg)


def test_prefill_stale_nan_rows_ignored(ctx):
    cfg = CONFIGS[2].scaled(n_new=100, n_q_heads=2, n_kv_heads=1, head_dim=128)
    inp = make_inputs(cfg, capacity=256)
    for name in ("k_cache", "v_cache"):
        c = inp[name].view(torch.float16).reshape(1, 256, 1, 128)
        c[0, 100:] = float("nan")
    check_call(ctx, cfg, inp=inp, check_cache=False)


# ---------------------------------------------------------------- reference-shaped ops

def test_multi_head_attention_matches_reference_shapes(ctx):
    """ComputeOps.MultiHeadAttention(Q, K, V, numHeads, startPosition) with already-rotated inputs."""
    from aihost_b200 import gen
    from aihost_b200.ops import ComputeOps
    from oracle import oracle as orc

    ops = ComputeOps(ctx)
    for S, Lk, P, hq, hkv, d in [(1, 513, 512, 32, 4, 64), (96, 96, 0, 8, 2, 64), (64, 200, 136, 4, 4, 128)]:
        q = gen.normal((S, hq * d), 7, "mq", dtype=torch.float16)
        k = gen.normal((Lk, hkv * d), 7, "mk", dtype=torch.float16)
        v = gen.normal((Lk, hkv * d), 7, "mv", dtype=torch.float16)
        out = ops.multi_head_attention(q.cuda(), k.cuda(), v.cuda(), hq, P).cpu().float().numpy()
        ref = orc.mha(q.float().numpy(), k.float().numpy(), v.float().numpy(), hq, P)
        assert max_abs(out, ref) <= 2e-3


def test_multi_head_attention_fp32_prefill(ctx):
    """MultiHeadAttention with the reference's fp32 tensors (S > 1 goes through fp16 staging)."""
    from aihost_b200 import gen
    from aihost_b200.ops import ComputeOps
    from oracle import oracle as orc

    ops = ComputeOps(ctx)
    for S, Lk, P, hq, hkv, d in [(96, 96, 0, 8, 2, 64), (64, 200, 136, 4, 4, 128)]:
        q = gen.normal((S, hq * d), 8, "fq", std=0.5)
        k = gen.normal((Lk, hkv * d), 8, "fk", std=0.5)
        v = gen.normal((Lk, hkv * d), 8, "fv", std=0.5)
        out = ops.multi_head_attention(q.cuda(), k.cuda(), v.cuda(), hq, P).cpu().numpy()
        ref = orc.mha(q.numpy(), k.numpy(), v.numpy(), hq, P)
        assert max_abs(out, ref) <= TOL_F32_PREFILL


def test_fused_mha_generate_fp32(ctx):
    from aihost_b200 import gen
    from aihost_b200.ops import ComputeOps, default_scale
    from oracle import oracle as orc

    ops = ComputeOps(ctx)
    q = gen.normal((1, 32 * 64), 9, "gq", std=0.5)
    k = gen.normal((513, 4 * 64), 9, "gk", std=0.5)
    v = gen.normal((513, 4 * 64), 9, "gv", std=0.5)
    out = ops.fused_mha_generate(q.cuda(), k.cuda(), v.cuda(), 32, 4, 64, default_scale(64)).cpu().numpy()
    ref = orc.mha(q.numpy(), k.numpy(), v.numpy(), 32, 512)
    assert max_abs(out, ref) <= 2e-4


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("mode", [ROPE_INTERLEAVED, ROPE_NEOX])
def test_apply_rope_full(ctx, dtype, mode):
    from aihost_b200 import gen
    from aihost_b200.ops import ComputeOps
    from oracle import oracle as orc

    x = gen.normal((33, 6 * 128), 11, "rope", dtype=dtype)
    y = x.cuda()
    ComputeOps(ctx).apply_rope_full(y, 4000, 6, 128, theta=5e5, rope_mode=mode)
    ref = orc.rope_full(x.float().numpy(), 4000, 6, 128, 5e5, mode)
    tol = 2e-5 if dtype == torch.float32 else 4e-3
    assert max_abs(y.cpu().float().numpy(), ref) <= tol


@pytest.mark.parametrize("kv", [F32, F16, Q8_0])
def test_kv_append_exact(ctx, kv):
    """KVCache.Add without rotation: the stored bytes equal the oracle's conversion / quantiser."""
    from aihost_b200.ops import KVCache
    from oracle import oracle as orc

    cfg = CONFIGS[3].scaled(batch=2, n_new=5, n_q_heads=8, n_kv_heads=2, q_dtype=F32 if kv == F32 else F16,
                            kv_dtype=kv, cached_range=None, cached_list=[3, 10], rope_mode=ROPE_NONE)
    inp = make_inputs(cfg, capacity=32)
    spec = cfg.spec(32)
    cache = KVCache(ctx, spec, batch=2, device=torch.device("cuda", 0))
    cache.k[0].copy_(inp["k_cache"])
    cache.v[0].copy_(inp["v_cache"])
    cache.seq_len.copy_(inp["seq_len"])
    cache.host_len = list(inp["lengths"])
    cache.add(0, inp["k_new"].cuda(), inp["v_new"].cuda())
    torch.cuda.synchronize()
    ctx.sync_status()
    _, rk, rv = oracle_forward(cfg, inp)
    assert np.array_equal(cache.k[0].cpu().numpy(), rk)
    assert np.array_equal(cache.v[0].cpu().numpy(), rv)


def test_device_length_over_capacity_reports_status(ctx):
    """A device-side seq_len past kv_capacity is refused by the kernels and reported on sync."""
    from aihost_b200 import AttnError, EINVAL

    cfg = CONFIGS[3].scaled(batch=2, n_q_heads=8, n_kv_heads=2, cached_range=None, cached_list=[10, 20])
    inp = make_inputs(cfg, capacity=64)
    inp["seq_len"] = torch.tensor([10, 64], dtype=torch.int32)  # 64 + 1 > 64 rows
    with pytest.raises(AttnError) as ei:
        gpu_forward(ctx, cfg, inp, pass_host_len=False)
    assert ei.value.status == EINVAL


# ---------------------------------------------------------------- Qwen TypeB Q/K prologue

def test_qk_norm_rope_matches_reference_shader_golden(ctx):
    """aihost_qk_norm_rope (fp32) against the reference's layer_norm + rope_full shaders (golden)."""
    import json
    from pathlib import Path

    from aihost_b200.ops import ComputeOps

    z = np.load(Path(__file__).resolve().parent / "golden" / "qk_norm_golden.npz")
    meta = json.loads(bytes(z["meta"]).decode())
    dev = torch.device("cuda", 0)
    for i, m in enumerate(meta):
        x = torch.from_numpy(z[f"x{i}"]).to(dev)
        w = torch.from_numpy(z[f"w{i}"]).to(dev)
        ComputeOps(ctx).qk_norm_rope(x, w, m["start"], m["n_heads"], m["head_dim"], m["theta"], m["eps"])
        torch.cuda.synchronize()
        ref = z[f"y{i}"]
        err = float(np.abs(x.cpu().numpy() - ref).max())
        assert err <= 2e-5 * max(1.0, float(np.abs(ref).max())), (i, err)


@pytest.mark.parametrize("mode", [ROPE_INTERLEAVED, ROPE_NEOX, ROPE_NONE])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_qk_norm_rope_matches_oracle(ctx, mode, dtype):
    from aihost_b200.ops import ComputeOps
    from oracle import oracle as orc

    rng = np.random.default_rng(11)
    dev = torch.device("cuda", 0)
    # register-resident kernel with 1, 2 and 4 units per thread, and the scalar kernel (head_dim 40)
    for seq, h, d, start in [(33, 14, 64, 0), (5, 32, 128, 4000), (300, 2, 64, 17), (3, 16, 256, 99), (4, 64, 128, 7),
                             (2, 64, 256, 5), (9, 6, 40, 3)]:
        x = rng.normal(0, 1.5, (seq, h * d)).astype(np.float32)
        w = rng.normal(1.0, 0.2, d).astype(np.float32)
        xt = torch.from_numpy(x).to(dtype).to(dev)
        x_in = xt.float().cpu().numpy()  # the input as the kernel sees it (fp16-rounded for fp16), before the in-place call
        ComputeOps(ctx).qk_norm_rope(xt, torch.from_numpy(w).to(dev), start, h, d, 1e6, 1e-5, mode)
        torch.cuda.synchronize()
        ref = orc.qk_norm_rope(x_in, w, start, h, d, 1e6, 1e-5, mode)
        tol = 2e-5 if dtype == torch.float32 else 2e-3
        err = float(np.abs(xt.float().cpu().numpy() - ref).max())
        assert err <= tol * max(1.0, float(np.abs(ref).max())), (seq, h, d, err)
