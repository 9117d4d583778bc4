"""aihost_b200 — B200-native attention hot path for AIHost, behind the libaihost_attn.so C ABI.

`lib()` loads the in-tree library (built by `python -m aihost_b200.build`) and raises if it is
missing: there is no CPU or fallback path. `ops` mirrors the reference's C# operator surface
(ComputeOps.MultiHeadAttention / ApplyRoPEFull / KVCache) on top of the C ABI.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libaihost_attn.so"

# aihost_status
OK, EINVAL, ENOMEM, ECUDA, ETIMEOUT, EUNSUPPORTED, ENCCL = range(7)
STATUS_NAMES = {0: "OK", 1: "EINVAL", 2: "ENOMEM", 3: "ECUDA", 4: "ETIMEOUT", 5: "EUNSUPPORTED", 6: "ENCCL"}
# aihost_dtype (AIHost DataType ordinals)
F32, F16, Q8_0 = 0, 1, 6
Q2_K, Q3_K, Q4_K, Q5_K, Q6_K = 8, 9, 10, 11, 12
# aihost_rope_mode
ROPE_INTERLEAVED, ROPE_NEOX, ROPE_NONE = 0, 1, 2

# Every symbol include/aihost_attn.h declares.
EXPORTS = (
    "aihost_attn_abi_version", "aihost_attn_last_error", "aihost_attn_create", "aihost_attn_destroy",
    "aihost_attn_workspace_size", "aihost_attn_reserve", "aihost_attn_forward", "aihost_attn_mha",
    "aihost_rope_full", "aihost_kv_append", "aihost_attn_sync_status", "aihost_attn_profiler_enable",
    "aihost_attn_profiler_read", "aihost_attn_profiler_reset", "aihost_attn_decode_noalloc",
    "aihost_attn_dist_unique_id", "aihost_attn_dist_init", "aihost_attn_dist_destroy", "aihost_attn_forward_sharded",
    "aihost_attn_decode_partial", "aihost_attn_merge_partials", "aihost_qk_norm_rope", "aihost_attn_forward_paged",
    "aihost_attn_noalloc_sync_status", "aihost_attn_dist_init_bounded", "aihost_attn_dist_sync",
    "aihost_matmul_workspace_size", "aihost_matmul_weights", "aihost_dequantize",
)
# aihost_kernel ids of the device-time profiler
KERNEL_APPEND, KERNEL_DECODE, KERNEL_COMBINE, KERNEL_PREFILL, KERNEL_CONVERT, KERNEL_MATMUL = range(6)


class AttnDesc(ctypes.Structure):
    """aihost_attn_desc."""

    _fields_ = [
        ("n_q_heads", ctypes.c_int32), ("n_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
        ("rope_theta", ctypes.c_float), ("rope_mode", ctypes.c_int32), ("scale", ctypes.c_float),
        ("q_dtype", ctypes.c_int32), ("kv_dtype", ctypes.c_int32), ("out_dtype", ctypes.c_int32),
        ("kv_capacity", ctypes.c_int32),
        ("kv_seq_stride", ctypes.c_int64), ("kv_token_stride", ctypes.c_int64), ("kv_head_stride", ctypes.c_int64),
    ]


class AttnError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")
        self.status = status


_LIB = None


def lib() -> ctypes.CDLL:
    """Load libaihost_attn.so (raises FileNotFoundError when it has not been built)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise FileNotFoundError(f"{LIB_PATH} is missing; build it with `python -m aihost_b200.build`")
    L = ctypes.CDLL(str(LIB_PATH))
    vp, i32, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_size_t
    dp = ctypes.POINTER(AttnDesc)
    L.aihost_attn_abi_version.restype = i32
    L.aihost_attn_last_error.restype = ctypes.c_char_p
    L.aihost_attn_create.argtypes = [i32, ctypes.POINTER(vp)]
    L.aihost_attn_destroy.argtypes = [vp]
    L.aihost_attn_workspace_size.argtypes = [dp, i32, i32, ctypes.POINTER(sz)]
    L.aihost_attn_reserve.argtypes = [vp, sz]
    L.aihost_attn_forward.argtypes = [vp, dp, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp]
    L.aihost_attn_mha.argtypes = [vp, dp, i32, i32, i32, vp, vp, vp, vp, vp]
    L.aihost_rope_full.argtypes = [vp, i32, i32, i32, i32, i32, ctypes.c_float, i32, vp]
    L.aihost_kv_append.argtypes = [vp, dp, i32, i32, vp, vp, vp, vp, vp, vp]
    L.aihost_attn_sync_status.argtypes = [vp, ctypes.POINTER(i32)]
    L.aihost_attn_profiler_enable.argtypes = [vp, i32]
    L.aihost_attn_profiler_read.argtypes = [vp, i32, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_double)]
    L.aihost_attn_profiler_reset.argtypes = [vp]
    L.aihost_attn_decode_noalloc.argtypes = [dp, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp]
    L.aihost_attn_noalloc_sync_status.argtypes = [vp, ctypes.POINTER(i32)]
    L.aihost_attn_dist_unique_id.argtypes = [vp]
    L.aihost_attn_dist_init.argtypes = [i32, i32, vp, i32, ctypes.POINTER(vp)]
    L.aihost_attn_dist_init_bounded.argtypes = [i32, i32, vp, i32, i32, ctypes.POINTER(vp)]
    L.aihost_attn_dist_destroy.argtypes = [vp]
    L.aihost_attn_dist_sync.argtypes = [vp, vp, i32]
    L.aihost_matmul_workspace_size.argtypes = [vp, ctypes.POINTER(sz)]
    L.aihost_matmul_weights.argtypes = [vp, vp, vp, vp, vp, vp]
    L.aihost_dequantize.argtypes = [vp, i32, ctypes.c_int64, vp, i32, vp]
    L.aihost_attn_forward_sharded.argtypes = [vp, vp, dp, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp]
    L.aihost_attn_decode_partial.argtypes = [vp, dp, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]
    L.aihost_attn_merge_partials.argtypes = [vp, i32, i32, i32, i32, vp, vp, vp, vp, vp]
    L.aihost_attn_forward_paged.argtypes = [vp, dp, i32, i32, vp, vp, vp, vp, vp, i32, i32, vp, i32, vp, vp, vp, vp]
    L.aihost_qk_norm_rope.argtypes = [vp, i32, i32, i32, i32, vp, ctypes.c_float, i32, ctypes.c_float, i32, vp]
    for name in EXPORTS:
        fn = getattr(L, name)
        if name not in ("aihost_attn_abi_version", "aihost_attn_last_error"):
            fn.restype = i32
    _LIB = L
    return L


def check(status: int) -> None:
    """Raise AttnError carrying aihost_attn_last_error() when status != OK."""
    if status != OK:
        msg = lib().aihost_attn_last_error()
        raise AttnError(status, msg.decode() if msg else "")


__all__ = ["lib", "check", "AttnDesc", "AttnError", "F32", "F16", "Q8_0", "Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "ROPE_INTERLEAVED", "ROPE_NEOX",
           "ROPE_NONE", "EXPORTS", "LIB_PATH"]
