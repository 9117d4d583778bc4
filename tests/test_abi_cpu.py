"""The C ABI without a GPU: the library loads, exports what include/aihost_attn.h declares, and
rejects bad arguments with status codes and messages before touching the device."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

import aihost_b200 as A
from aihost_b200.ops import LayerSpec

HEADER = Path(__file__).resolve().parent.parent / "include" / "aihost_attn.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(aihost_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = A.lib()
    names = declared_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(L, n), f"{n} declared in aihost_attn.h but not exported"
    assert sorted(A.EXPORTS) == names


def test_abi_version():
    assert A.lib().aihost_attn_abi_version() == 1


def _ws(spec: LayerSpec, batch=1, n_new=1):
    need = ctypes.c_size_t()
    d = spec.desc()
    return A.lib().aihost_attn_workspace_size(ctypes.byref(d), batch, n_new, ctypes.byref(need)), need.value


def test_validation_status_codes():
    base = dict(n_q_heads=32, n_kv_heads=8, head_dim=128, kv_capacity=4096)
    assert _ws(LayerSpec(**base))[0] == A.OK
    assert _ws(LayerSpec(**{**base, "n_q_heads": 30}))[0] == A.EINVAL
    assert b"multiple" in A.lib().aihost_attn_last_error()
    assert _ws(LayerSpec(**{**base, "head_dim": 96}))[0] == A.EUNSUPPORTED
    assert _ws(LayerSpec(**{**base, "kv_dtype": 3}))[0] == A.EINVAL
    assert _ws(LayerSpec(**{**base, "rope_theta": -1.0}))[0] == A.EINVAL
    assert _ws(LayerSpec(**{**base, "kv_capacity": 0}))[0] == A.EINVAL
    assert _ws(LayerSpec(**{**base, "kv_head_stride": 8}))[0] == A.EINVAL  # smaller than a row
    assert _ws(LayerSpec(**base), batch=0)[0] == A.EINVAL


def test_workspace_scales_with_capacity():
    small = _ws(LayerSpec(32, 8, 128, kv_capacity=1024), batch=4)[1]
    big = _ws(LayerSpec(32, 8, 128, kv_capacity=65536), batch=4)[1]
    assert big > small
    assert _ws(LayerSpec(32, 8, 128, kv_capacity=1024), batch=4, n_new=16)[1] == 0  # fp16 prefill needs none


def test_workspace_covers_fp16_staging_of_fp32_and_q8_prefill():
    """fp32 q -> fp16 copy of q; fp32 / Q8_0 cache -> fp16 copies of K and V (kv_capacity rows)."""
    q_bytes = 4 * 16 * 32 * 128 * 2
    kv_bytes = 2 * 4 * 1024 * 8 * 128 * 2
    assert _ws(LayerSpec(32, 8, 128, kv_capacity=1024, q_dtype=A.F32, kv_dtype=A.F16), 4, 16)[1] == q_bytes
    assert _ws(LayerSpec(32, 8, 128, kv_capacity=1024, q_dtype=A.F16, kv_dtype=A.Q8_0), 4, 16)[1] == kv_bytes
    assert _ws(LayerSpec(32, 8, 128, kv_capacity=1024, q_dtype=A.F32, kv_dtype=A.F32), 4, 16)[1] == q_bytes + kv_bytes


def test_null_context_and_pointers_rejected():
    L = A.lib()
    d = LayerSpec(8, 2, 64, kv_capacity=64).desc()
    st = L.aihost_attn_forward(None, ctypes.byref(d), 1, 1, None, None, None, None, None, None, None, None, None)
    assert st == A.EINVAL
    assert L.aihost_rope_full(None, 0, 1, 1, 64, 0, 1e4, 0, None) == A.EINVAL
    assert L.aihost_rope_full(ctypes.c_void_p(16), 0, 1, 1, 63, 0, 1e4, 0, None) == A.EINVAL
    assert L.aihost_attn_sync_status(None, None) == A.EINVAL


def test_dist_calls_validate_arguments_before_nccl():
    """The bounded NCCL set-up and wait reject bad arguments without loading NCCL or a device."""
    L = A.lib()
    nid = ctypes.create_string_buffer(128)
    h = ctypes.c_void_p()
    assert L.aihost_attn_dist_init_bounded(2, 0, nid, 0, 1000, None) == A.EINVAL
    assert L.aihost_attn_dist_init_bounded(2, 0, None, 0, 1000, ctypes.byref(h)) == A.EINVAL
    assert L.aihost_attn_dist_init_bounded(2, 2, nid, 0, 1000, ctypes.byref(h)) == A.EINVAL
    assert L.aihost_attn_dist_init_bounded(2, 0, nid, 0, 0, ctypes.byref(h)) == A.EINVAL
    assert b"timeout_ms" in L.aihost_attn_last_error()
    assert not h
    assert L.aihost_attn_dist_sync(None, None, 1000) == A.EINVAL
    d = LayerSpec(8, 2, 64, kv_capacity=64).desc()
    assert L.aihost_attn_forward_sharded(None, None, ctypes.byref(d), 1, 1, None, None, None, None, None, None, None,
                                         None, None) == A.EINVAL
    assert L.aihost_attn_noalloc_sync_status is not None


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_create_without_device_fails_cleanly():
    h = ctypes.c_void_p()
    st = A.lib().aihost_attn_create(0, ctypes.byref(h))
    assert st in (A.ECUDA, A.EINVAL)
    assert not h
    assert A.lib().aihost_attn_last_error()
