"""CPU checks of the oracle itself (oracle/attn_oracle.c): formats, RoPE, softmax, causality."""
import numpy as np
import pytest

from aihost_b200 import F16, F32, Q8_0, ROPE_INTERLEAVED, ROPE_NEOX, ROPE_NONE
from aihost_b200.configs import CONFIGS, make_inputs
from oracle import oracle as orc


def test_f16_to_f32_all_values():
    h = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    out = np.empty(65536, dtype=np.float32)
    orc.lib().oracle_f16_to_f32_n(h.ctypes.data, out.ctypes.data, 65536)
    ref = h.view(np.float16).astype(np.float32)
    both_nan = np.isnan(out) & np.isnan(ref)
    assert np.array_equal(out[~both_nan], ref[~both_nan])
    assert np.array_equal(np.isnan(out), np.isnan(ref))


def test_f32_to_f16_round_to_nearest_even():
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(200000).astype(np.float32) * np.float32(10.0) ** rng.integers(-9, 5, 200000),
        np.array([65504, 65519, 65520, 1e9, -1e9, 6e-8, 2.98e-8, 2 ** -25, 2 ** -24, 5.96e-8, 0.0, -0.0],
                 dtype=np.float32),
        (np.arange(1, 2049, dtype=np.float32) + np.float32(0.5)),  # exact ties at integer/2 steps
    ]).astype(np.float32)
    got = orc.f32_to_f16(x)
    with np.errstate(over="ignore"):
        ref = x.astype(np.float16)
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))


def ggml_q8_0_ref(x: np.ndarray) -> np.ndarray:
    """ggml quantize_row_q8_0_ref restated independently in numpy (float32 arithmetic)."""
    x = x.astype(np.float32).reshape(-1, 32)
    amax = np.abs(x).max(axis=1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    xs = (x * idv[:, None]).astype(np.float32)
    q = np.where(xs >= 0, np.floor(xs + np.float32(0.5)), -np.floor(-xs + np.float32(0.5))).astype(np.int8)
    out = np.empty((x.shape[0], 34), dtype=np.uint8)
    out[:, :2] = d.astype(np.float16).view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.reshape(-1)


def test_q8_0_quantize_matches_ggml_rule():
    rng = np.random.default_rng(1)
    x = rng.standard_normal(32 * 4096).astype(np.float32)
    x[:32] = 0.0  # all-zero block: d = 0, id = 0
    x[32:64] = np.linspace(-1, 1, 32, dtype=np.float32)
    got = orc.q8_0_quantize(x)
    ref = ggml_q8_0_ref(x)
    # roundf vs floor(x+0.5) differ only on exact .5 ties of x*id, which the data avoid
    assert np.array_equal(got, ref)
    back = orc.q8_0_dequantize(got, x.size)
    d = got.reshape(-1, 34)[:, :2].copy().view(np.float16).astype(np.float32).reshape(-1)
    assert np.all(np.abs(back - x).reshape(-1, 32).max(axis=1) <= d * 0.5 + np.abs(x).reshape(-1, 32).max(axis=1) * 1e-3)


def test_rope_identity_at_position_zero_and_norm_preserved():
    rng = np.random.default_rng(2)
    x = rng.standard_normal((5, 4 * 64)).astype(np.float32)
    y0 = orc.rope_full(x[:1], 0, 4, 64, 1e4)
    assert np.array_equal(y0, x[:1])
    for mode in (ROPE_INTERLEAVED, ROPE_NEOX):
        y = orc.rope_full(x, 1000, 4, 64, 1e4, mode)
        nx = np.linalg.norm(x.reshape(5, 4, 64), axis=-1)
        ny = np.linalg.norm(y.reshape(5, 4, 64), axis=-1)
        assert np.allclose(nx, ny, rtol=1e-5)


def test_rope_interleaved_matches_formula():
    rng = np.random.default_rng(3)
    d, theta, pos = 64, 10000.0, 37
    x = rng.standard_normal((1, d)).astype(np.float32)
    y = orc.rope_full(x, pos, 1, d, theta, ROPE_INTERLEAVED)
    i = np.arange(d // 2)
    freq = 1.0 / np.power(theta, 2 * i / d)
    ang = pos * freq
    x1, x2 = x[0, 0::2].astype(np.float64), x[0, 1::2].astype(np.float64)
    ref = np.empty(d)
    ref[0::2] = x1 * np.cos(ang) - x2 * np.sin(ang)
    ref[1::2] = x1 * np.sin(ang) + x2 * np.cos(ang)
    assert np.allclose(y[0], ref, atol=1e-5)


def _np_attention(q, k, v, hq, start):
    """float64 numpy attention (causal j <= start + i for S > 1)."""
    S, dq = q.shape
    d = dq // hq
    hkv = k.shape[1] // d
    out = np.zeros((S, dq))
    for h in range(hq):
        kh = h // (hq // hkv)
        Q = q[:, h * d:(h + 1) * d].astype(np.float64)
        K = k[:, kh * d:(kh + 1) * d].astype(np.float64)
        V = v[:, kh * d:(kh + 1) * d].astype(np.float64)
        s = Q @ K.T * float(np.float32(1) / np.sqrt(np.float32(d)))
        if S > 1:
            mask = np.arange(k.shape[0])[None, :] > (start + np.arange(S))[:, None]
            s[mask] = -np.inf
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[:, h * d:(h + 1) * d] = p @ V
    return out


@pytest.mark.parametrize("S,Lk,P,hq,hkv,d", [(1, 300, 299, 8, 2, 64), (40, 40, 0, 4, 2, 32), (20, 70, 50, 6, 3, 16)])
def test_mha_exact_and_faithful_agree_with_numpy(S, Lk, P, hq, hkv, d):
    rng = np.random.default_rng(4)
    q = rng.standard_normal((S, hq * d)).astype(np.float32)
    k = rng.standard_normal((Lk, hkv * d)).astype(np.float32)
    v = rng.standard_normal((Lk, hkv * d)).astype(np.float32)
    ref = _np_attention(q, k, v, hq, P)
    ex = orc.mha(q, k, v, hq, P, mode=orc.EXACT)
    fa = orc.mha(q, k, v, hq, P, mode=orc.FAITHFUL)
    assert np.abs(ex - ref).max() < 1e-6
    assert np.abs(fa - ref).max() < 2e-5


def test_prefill_is_causal():
    rng = np.random.default_rng(5)
    S, hq, d = 30, 2, 16
    q = rng.standard_normal((S, hq * d)).astype(np.float32)
    k = rng.standard_normal((S, hq * d)).astype(np.float32)
    v = rng.standard_normal((S, hq * d)).astype(np.float32)
    a = orc.mha(q, k, v, hq, 0, mode=orc.FAITHFUL)
    k2, v2 = k.copy(), v.copy()
    k2[20:] += 5.0
    v2[20:] -= 3.0
    b = orc.mha(q, k2, v2, hq, 0, mode=orc.FAITHFUL)
    assert np.array_equal(a[:20], b[:20])
    assert not np.array_equal(a[20:], b[20:])


def test_constant_values_give_constant_output():
    rng = np.random.default_rng(6)
    q = rng.standard_normal((1, 4 * 64)).astype(np.float32)
    k = rng.standard_normal((500, 64)).astype(np.float32)
    v = np.full((500, 64), 0.75, dtype=np.float32)
    out = orc.mha(q, k, v, 4, 499, mode=orc.EXACT)
    assert np.allclose(out, 0.75, atol=1e-6)


@pytest.mark.parametrize("kv", [F32, F16, Q8_0])
def test_forward_appends_rows_and_keeps_others(kv):
    cfg = CONFIGS[3].scaled(batch=2, n_new=3, n_q_heads=4, n_kv_heads=2, head_dim=64, q_dtype=F32 if kv == F32 else F16,
                            kv_dtype=kv, out_dtype=F32, cached_range=None, cached_list=[5, 9], rope_mode=ROPE_NONE)
    inp = make_inputs(cfg, capacity=16)
    desc = cfg.spec(16).desc()
    kc, vc = inp["k_cache"].numpy().copy(), inp["v_cache"].numpy().copy()
    orc.attn_forward(desc, inp["q"].numpy(), inp["k_new"].numpy(), inp["v_new"].numpy(), kc, vc,
                     inp["seq_len"].numpy())
    rb = {F32: 256, F16: 128, Q8_0: 68}[kv] * 2
    orig = inp["v_cache"].numpy().reshape(2, 16, rb)
    new = vc.reshape(2, 16, rb)
    for b, n in enumerate(inp["lengths"]):
        assert np.array_equal(new[b, :n], orig[b, :n])
        assert np.array_equal(new[b, n + 3:], orig[b, n + 3:])
        vn = inp["v_new"].numpy()[b].reshape(3, -1).astype(np.float32)
        if kv == F32:
            assert np.array_equal(new[b, n:n + 3].view(np.float32).reshape(3, -1), vn)
        elif kv == F16:
            assert np.array_equal(new[b, n:n + 3].view(np.float16).reshape(3, -1), vn.astype(np.float16))
        else:
            assert np.array_equal(new[b, n:n + 3].reshape(-1), orc.q8_0_quantize(vn))


def test_faithful_forward_close_to_exact():
    cfg = CONFIGS[1]
    inp = make_inputs(cfg)
    desc = cfg.spec(inp["capacity"]).desc()
    outs = []
    for mode in (orc.FAITHFUL, orc.EXACT):
        kc, vc = inp["k_cache"].numpy().copy(), inp["v_cache"].numpy().copy()
        outs.append(orc.attn_forward(desc, inp["q"].numpy(), inp["k_new"].numpy(), inp["v_new"].numpy(), kc, vc,
                                     inp["seq_len"].numpy(), mode=mode))
    assert np.abs(outs[0] - outs[1]).max() < 1e-5


def test_num_threads_positive():
    assert orc.num_threads() >= 1


def test_oracle_row_range_equals_full_rows():
    """oracle_attn_forward_rows (samples of long prefills) computes exactly the full call's rows."""
    from helpers import oracle_forward

    cfg = CONFIGS[2].scaled(n_new=300, n_q_heads=4, n_kv_heads=2, cached=None, cached_list=[37])
    inp = make_inputs(cfg)
    full, fk, fv = oracle_forward(cfg, inp)
    sub, sk, sv = oracle_forward(cfg, inp, part=(0, 1, 1, 3), rows=(100, 250))
    assert np.array_equal(full[:, 100:250, 1:3], sub[:, 100:250, 1:3])
    assert not sub[:, :100].any() and not sub[:, 250:].any()
    assert np.array_equal(fv, sv)  # query heads 1-2 use both KV heads: every new row is appended
