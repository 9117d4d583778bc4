"""aihost_attn_decode_noalloc: the decode step for hosts that cannot allocate device memory.

Some callers of this library cannot call cudaMalloc while they decode (an engine whose device
memory is already carved up by its own pool, or a host that must not enter the allocator on the
token path). For them, aihost_attn_decode_noalloc runs the same one-token step as
aihost_attn_forward with its split scratch in a static device array instead of a context's
reserved buffer. These tests call both entry points through the C ABI on the same inputs:
each config is decoded by the no-alloc call, then by aihost_attn_forward, then by the no-alloc
call again (the static array keeps the previous call's contents, and the context call in
between advances its own merge counters, not the array's). Both no-alloc calls must give
bit-identical outputs and cache rows, and equal aihost_attn_forward's within the parity bound
the other fp16 tests use (2e-3). Device-side errors of no-alloc calls must reach the caller
through aihost_attn_noalloc_sync_status, which needs no context either.

The file name puts it last in collection order, so a run that stops at the first failure has run
every other test before it; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from aihost_b200 import EINVAL, ENOMEM, OK, check, lib
from aihost_b200.configs import CONFIGS, make_inputs

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _regular(ctx, cfg, inp):
    """aihost_attn_forward with a context and reserved scratch; returns (out, k_cache, v_cache)."""
    dev = torch.device("cuda", 0)
    spec = cfg.spec(inp["capacity"])
    ctx.reserve_for(spec, cfg.batch, 1)
    d = spec.desc()
    q, kn, vn = (inp[n].to(dev) for n in ("q", "k_new", "v_new"))
    kc, vc = inp["k_cache"].to(dev).clone(), inp["v_cache"].to(dev).clone()
    sl = inp["seq_len"].to(dev)
    out = torch.empty(cfg.batch, 1, cfg.n_q_heads, cfg.head_dim, dtype=torch.float16, device=dev)
    hl = (ctypes.c_int32 * cfg.batch)(*inp["lengths"])
    check(lib().aihost_attn_forward(ctx.handle, ctypes.byref(d), cfg.batch, 1, q.data_ptr(), kn.data_ptr(),
                                    vn.data_ptr(), kc.data_ptr(), vc.data_ptr(), sl.data_ptr(),
                                    ctypes.cast(hl, ctypes.c_void_p), out.data_ptr(), _stream()))
    torch.cuda.synchronize()
    return out.cpu(), kc.cpu(), vc.cpu()


def _noalloc(cfg, inp, seq_len=None):
    """aihost_attn_decode_noalloc on the current device; no context, no reservation. Returns
    (out, k_cache, v_cache, status of aihost_attn_noalloc_sync_status, its raw bits)."""
    dev = torch.device("cuda", 0)
    d = cfg.spec(inp["capacity"]).desc()
    q, kn, vn = (inp[n].to(dev) for n in ("q", "k_new", "v_new"))
    kc, vc = inp["k_cache"].to(dev).clone(), inp["v_cache"].to(dev).clone()
    sl = (inp["seq_len"] if seq_len is None else seq_len).to(dev)
    out = torch.zeros(cfg.batch, 1, cfg.n_q_heads, cfg.head_dim, dtype=torch.float16, device=dev)
    check(lib().aihost_attn_decode_noalloc(ctypes.byref(d), cfg.batch, q.data_ptr(), kn.data_ptr(), vn.data_ptr(),
                                           kc.data_ptr(), vc.data_ptr(), sl.data_ptr(), None, out.data_ptr(),
                                           _stream()))
    bits = ctypes.c_int32(-1)
    st = lib().aihost_attn_noalloc_sync_status(ctypes.c_void_p(_stream()), ctypes.byref(bits))
    return out.cpu(), kc.cpu(), vc.cpu(), st, bits.value


def test_noalloc_matches_forward_on_two_calls_in_a_row(ctx):
    torch.cuda.set_device(0)
    calls = [
        CONFIGS[3].scaled(batch=8, cached_range=None, cached_list=[300, 4095, 17, 2048, 999, 1, 3333, 640]),
        CONFIGS[5].scaled(batch=2, n_q_heads=16, n_kv_heads=2, cached=None, cached_list=[513, 2700]),
    ]
    for cfg in calls:
        inp = make_inputs(cfg)
        first = _noalloc(cfg, inp)
        ref_out, ref_k, ref_v = _regular(ctx, cfg, inp)
        second = _noalloc(cfg, inp)
        for out, k, v, st, bits in (first, second):
            assert st == OK and bits == 0, f"{cfg.name}: no-alloc status {st} bits {bits}"
            assert torch.isfinite(out.float()).all()
            err = float((out.float() - ref_out.float()).abs().max())
            assert err <= TOL, f"{cfg.name}: max |noalloc - forward| = {err:.3g}"
            assert np.array_equal(k.numpy(), ref_k.numpy()) and np.array_equal(v.numpy(), ref_v.numpy())
        assert torch.equal(first[0], second[0]), f"{cfg.name}: two no-alloc calls on the same inputs differ"


def test_noalloc_reports_device_length_past_capacity():
    """A device-side seq_len whose new row would not fit (seq_len == kv_capacity, no host copy to
    check it against) is refused by the kernels and reported by aihost_attn_noalloc_sync_status;
    the word is cleared by that read, so the next good call reports OK."""
    torch.cuda.set_device(0)
    cfg = CONFIGS[3].scaled(batch=2, n_q_heads=8, n_kv_heads=2, cached_range=None, cached_list=[10, 20])
    inp = make_inputs(cfg, capacity=64)
    _, _, _, st, bits = _noalloc(cfg, inp, seq_len=torch.tensor([10, 64], dtype=torch.int32))
    assert st == EINVAL and bits & 2, f"status {st}, bits {bits}"
    assert b"kv_capacity" in lib().aihost_attn_last_error()
    out, _, _, st, bits = _noalloc(cfg, inp)
    assert st == OK and bits == 0
    assert torch.isfinite(out.float()).all()


def test_noalloc_refuses_requests_past_its_static_scratch():
    torch.cuda.set_device(0)
    # 1024 sequences x 32 query heads need 1024 * 32 * (128 + 2) * 4 bytes = 17 MB of partials even
    # with a single split: more than the 8 MiB array under any split plan. The size is checked
    # before the pointers, and the pointers are NULL, so no kernel can be launched either way.
    d = CONFIGS[3].scaled(batch=1024).spec(8193).desc()
    st = lib().aihost_attn_decode_noalloc(ctypes.byref(d), 1024, None, None, None, None, None, None, None, None,
                                          None)
    assert st == ENOMEM
    assert b"8 MiB" in lib().aihost_attn_last_error()
    assert st != OK
