"""ctypes wrapper of oracle/_ref/libref_glsl.so — the reference's own shaders on the CPU.

TEST INFRASTRUCTURE ONLY (pins the oracle; generates tests/golden fixtures). The library is
built from the reference checkout by oracle/ref_glsl/build_ref.py and is absent when the
checkout is; callers skip in that case.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

LIB_PATH = Path(__file__).resolve().parent.parent / "_ref" / "libref_glsl.so"
_LIB = None


def available() -> bool:
    return LIB_PATH.exists()


def lib():
    global _LIB
    if _LIB is None:
        L = ctypes.CDLL(str(LIB_PATH))
        vp, i32, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        L.ref_rope_full.argtypes = [vp, i32, i32, i32, i32, f32]
        L.ref_qk_norm_rope.argtypes = [vp, i32, i32, i32, vp, f32, i32, f32]
        L.ref_mha.argtypes = [vp, i32, vp, vp, i32, i32, i32, i32, i32, vp]
        L.ref_layer_attention.argtypes = [vp, vp, vp, i32, vp, vp, i32, i32, i32, i32, f32, vp, vp, vp]
        L.ref_dequantize.argtypes = [i32, vp, i32, vp]
        L.ref_matmul_weights.argtypes = [vp, i32, i32, vp, i32, vp]
        _LIB = L
    return _LIB


def _f(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def rope_full(x, start, n_heads, head_dim, theta):
    y = _f(x).copy()
    lib().ref_rope_full(y.ctypes.data, y.shape[0], n_heads, head_dim, start, theta)
    return y


def qk_norm_rope(x, w, start, n_heads, head_dim, theta, eps=1e-5):
    y = _f(x).copy()
    wf = _f(w)
    lib().ref_qk_norm_rope(y.ctypes.data, y.shape[0], n_heads, head_dim, wf.ctypes.data, eps, start, theta)
    return y


def mha(q, k, v, n_q_heads, start):
    q, k, v = _f(q), _f(k), _f(v)
    d = q.shape[1] // n_q_heads
    out = np.empty_like(q)
    lib().ref_mha(q.ctypes.data, q.shape[0], k.ctypes.data, v.ctypes.data, k.shape[0], n_q_heads, k.shape[1] // d, d,
                  start, out.ctypes.data)
    return out


def layer_attention(q, k_new, v_new, k_cached, v_cached, pos, n_q_heads, n_kv_heads, head_dim, theta):
    """q [S, Hq*d], k_new/v_new [S, Hkv*d], caches [pos, Hkv*d] -> (out, k_all, v_all)."""
    q, k_new, v_new = _f(q), _f(k_new), _f(v_new)
    S = q.shape[0]
    dkv = n_kv_heads * head_dim
    kc = _f(k_cached) if pos else np.zeros((1, dkv), np.float32)
    vc = _f(v_cached) if pos else np.zeros((1, dkv), np.float32)
    out = np.empty_like(q)
    k_all = np.empty((pos + S, dkv), np.float32)
    v_all = np.empty((pos + S, dkv), np.float32)
    lib().ref_layer_attention(q.ctypes.data, k_new.ctypes.data, v_new.ctypes.data, S, kc.ctypes.data, vc.ctypes.data,
                              pos, n_q_heads, n_kv_heads, head_dim, theta, out.ctypes.data, k_all.ctypes.data,
                              v_all.ctypes.data)
    return out, k_all, v_all


def dequantize(kind: int, blocks: np.ndarray, n: int) -> np.ndarray:
    """ComputeOps.Dequantize of n values (GGUF K-quant blocks as bytes) -> fp32."""
    blk = np.ascontiguousarray(blocks, dtype=np.uint8)
    out = np.empty(n, dtype=np.float32)
    if lib().ref_dequantize(kind, blk.ctypes.data, n, out.ctypes.data):
        raise ValueError(f"unsupported kind {kind}")
    return out


def matmul_weights(a: np.ndarray, w_nk: np.ndarray) -> np.ndarray:
    """ComputeOps.MatMulWeights: a [M, K] fp32 times a GGUF column-major weight given as
    w_nk [N, K] (element (k, n) at n * K + k) -> [M, N] fp32."""
    a = _f(a)
    w = _f(w_nk)
    M, K = a.shape
    N = w.shape[0]
    c = np.empty((M, N), dtype=np.float32)
    lib().ref_matmul_weights(a.ctypes.data, M, K, w.ctypes.data, N, c.ctypes.data)
    return c
