"""ctypes wrapper of oracle/liboracle.so — TEST INFRASTRUCTURE ONLY.

The CPU restatement of the reference's attention path (attn_oracle.c). Imported by tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg only, as the checker and the timed CPU
reference; the product (aihost_b200, libaihost_attn.so) never imports it.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
FAITHFUL, EXACT = 0, 1

_LIB = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        vp, i32, i64, f32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float
        L.oracle_num_threads.restype = i32
        L.oracle_set_num_threads.argtypes = [i32]
        L.oracle_f16_to_f32.argtypes, L.oracle_f16_to_f32.restype = [ctypes.c_uint16], f32
        L.oracle_f32_to_f16.argtypes, L.oracle_f32_to_f16.restype = [f32], ctypes.c_uint16
        L.oracle_f16_to_f32_n.argtypes = [vp, vp, i64]
        L.oracle_f32_to_f16_n.argtypes = [vp, vp, i64]
        L.oracle_q8_0_quantize.argtypes = [vp, i64, vp]
        L.oracle_q8_0_dequantize.argtypes = [vp, i64, vp]
        L.oracle_rope_freq.argtypes, L.oracle_rope_freq.restype = [f32, i32, i32], f32
        L.oracle_rope_full.argtypes = [vp, i32, i32, i32, i32, f32, i32]
        L.oracle_qk_norm_rope.argtypes = [vp, i32, i32, i32, vp, f32, i32, f32, i32]
        L.oracle_mha.argtypes = [vp, vp, vp, i64, i32, i32, i32, i32, i32, i32, f32, i32, vp]
        L.oracle_mha.restype = i32
        L.oracle_attn_forward.argtypes = [vp, i32, i32, vp, vp, vp, vp, vp, vp, vp, i32]
        L.oracle_attn_forward.restype = i32
        L.oracle_attn_forward_part.argtypes = [vp, i32, i32, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32]
        L.oracle_attn_forward_part.restype = i32
        L.oracle_attn_forward_rows.argtypes = [vp, i32, i32, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32,
                                               i32]
        L.oracle_attn_forward_rows.restype = i32
        L.oracle_kquant_block_bytes.argtypes, L.oracle_kquant_block_bytes.restype = [i32], i32
        L.oracle_dequantize.argtypes, L.oracle_dequantize.restype = [i32, vp, i64, vp], i32
        L.oracle_matmul_weights.argtypes, L.oracle_matmul_weights.restype = [vp, i32, i32, vp, i32, vp, i32], i32
        _LIB = L
    return _LIB


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def num_threads() -> int:
    return lib().oracle_num_threads()


def set_num_threads(n: int) -> None:
    """OpenMP threads of later oracle calls."""
    lib().oracle_set_num_threads(int(n))


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().oracle_f32_to_f16_n(_p(x), _p(out), x.size)
    return out.view(np.float16)


def q8_0_quantize(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    out = np.empty(x.size // 32 * 34, dtype=np.uint8)
    lib().oracle_q8_0_quantize(_p(x), x.size, _p(out))
    return out


def q8_0_dequantize(blocks: np.ndarray, n: int) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty(n, dtype=np.float32)
    lib().oracle_q8_0_dequantize(_p(blocks), n, _p(out))
    return out


def rope_full(x: np.ndarray, start_pos: int, n_heads: int, head_dim: int, theta: float, mode: int = 0) -> np.ndarray:
    """ApplyRoPEFull on a copy of x [seq, n_heads*head_dim] (fp32)."""
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    lib().oracle_rope_full(_p(y), y.shape[0], n_heads, head_dim, start_pos, theta, mode)
    return y


def qk_norm_rope(x: np.ndarray, w: np.ndarray, start_pos: int, n_heads: int, head_dim: int, theta: float,
                 eps: float = 1e-5, mode: int = 0) -> np.ndarray:
    """Qwen TypeB prologue on a copy of x [seq, n_heads*head_dim] (fp32): RMS over each whole
    row with the per-head weight w [head_dim] tiled over the heads, then ApplyRoPEFull."""
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    wf = np.ascontiguousarray(w, dtype=np.float32)
    lib().oracle_qk_norm_rope(_p(y), y.shape[0], n_heads, head_dim, _p(wf), eps, start_pos, theta, mode)
    return y


def mha(q: np.ndarray, k: np.ndarray, v: np.ndarray, n_q_heads: int, start_pos: int = 0, scale: float | None = None,
        mode: int = EXACT) -> np.ndarray:
    """MultiHeadAttention over rotated fp32 q [S, Hq*d], k/v [Lk, Hkv*d]."""
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    S, dq = q.shape
    d = dq // n_q_heads
    hkv = k.shape[1] // d
    if scale is None:
        scale = float(np.float32(1.0) / np.sqrt(np.float32(d)))
    out = np.empty_like(q)
    rc = lib().oracle_mha(_p(q), _p(k), _p(v), k.shape[1], S, k.shape[0], n_q_heads, hkv, d, start_pos, scale, mode,
                          _p(out))
    if rc:
        raise RuntimeError(f"oracle_mha failed ({rc})")
    return out


def attn_forward(desc, q: np.ndarray, k_new: np.ndarray, v_new: np.ndarray, k_cache: np.ndarray,
                 v_cache: np.ndarray, seq_len: np.ndarray, mode: int = EXACT, part=None, rows=None) -> np.ndarray:
    """The fused forward on host arrays; k_cache / v_cache (uint8 bytes) are appended in place.

    desc is an aihost_b200.AttnDesc (the same struct the C ABI takes). part = (b0, b1, h0, h1)
    restricts the sequences and query heads computed (bounded CPU-baseline samples); rows =
    (r0, r1) further restricts the attended query rows (the other rows of `out` stay zero)."""
    B, S = q.shape[0], q.shape[1]
    out_dt = np.float32 if desc.out_dtype == 0 else np.float16
    out = np.zeros((B, S, desc.n_q_heads, desc.head_dim), dtype=out_dt)
    arrs = [np.ascontiguousarray(a) for a in (q, k_new, v_new)]
    for c in (k_cache, v_cache):
        assert c.flags["C_CONTIGUOUS"] and c.dtype == np.uint8
    sl = np.ascontiguousarray(seq_len, dtype=np.int32)
    if rows is not None:
        p = part if part is not None else (0, B, 0, desc.n_q_heads)
        rc = lib().oracle_attn_forward_rows(ctypes.addressof(desc), B, S, *(_p(a) for a in arrs), _p(k_cache),
                                            _p(v_cache), _p(sl), _p(out), mode, *p, *rows)
    elif part is None:
        rc = lib().oracle_attn_forward(ctypes.addressof(desc), B, S, *(_p(a) for a in arrs), _p(k_cache),
                                       _p(v_cache), _p(sl), _p(out), mode)
    else:
        rc = lib().oracle_attn_forward_part(ctypes.addressof(desc), B, S, *(_p(a) for a in arrs), _p(k_cache),
                                            _p(v_cache), _p(sl), _p(out), mode, *part)
    if rc:
        raise RuntimeError(f"oracle_attn_forward failed ({rc})")
    return out


def dequantize(kind: int, blocks: np.ndarray, n: int) -> np.ndarray:
    """n values of GGUF K-quant blocks (bytes) -> fp32, the reference shaders' formulas."""
    blk = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty(n, dtype=np.float32)
    if lib().oracle_dequantize(kind, _p(blk), n, _p(out)):
        raise ValueError(f"oracle_dequantize: bad kind {kind} or n {n}")
    return out


def matmul_weights(a: np.ndarray, w_nk: np.ndarray, mode: int = EXACT) -> np.ndarray:
    """ComputeOps.MatMulWeights: a [M, K] times the GGUF column-major weight given as w_nk [N, K]."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    w = np.ascontiguousarray(w_nk, dtype=np.float32)
    c = np.empty((a.shape[0], w.shape[0]), dtype=np.float32)
    if lib().oracle_matmul_weights(_p(a), a.shape[0], a.shape[1], _p(w), w.shape[0], _p(c), mode):
        raise ValueError("oracle_matmul_weights: bad shape")
    return c
