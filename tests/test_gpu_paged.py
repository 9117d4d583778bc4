"""Paged fp32 / fp16 / Q8_0 KV cache (aihost_attn_forward_paged, PagedKVCache).

Each sequence's cached rows are scattered over pages of a shared pool in shuffled order. A decode
step and a chunked prefill over the paged cache must give the contiguous path's output bit for
bit (the same kernels read the same data), the oracle's within 2e-3, and the same cache rows
after the append. A block-table entry outside the pool is refused by the kernels with a status
(the row is not written; reads of it return zeros), reported on sync.
"""
import numpy as np
import pytest
import torch

from aihost_b200.configs import CONFIGS, make_inputs

pytestmark = pytest.mark.gpu


def _paged(ctx, cfg, inp, page_rows, seed=0):
    """A PagedKVCache holding inp's cached rows in shuffled pages."""
    from aihost_b200.ops import PagedKVCache, row_bytes

    cap = inp["capacity"]
    spec = cfg.spec(cap)
    max_pages = -(-cap // page_rows)
    n_pages = cfg.batch * max_pages + 3
    cache = PagedKVCache(ctx, spec, n_pages=n_pages, page_rows=page_rows, batch=cfg.batch)
    cache.free = list(np.random.default_rng(seed).permutation(n_pages))
    rb = row_bytes(cfg.kv_dtype, cfg.head_dim) * cfg.n_kv_heads
    for name, pool in (("k_cache", cache.k[0]), ("v_cache", cache.v[0])):
        full = inp[name].view(cfg.batch, cap, rb)
        host_pool = torch.zeros(n_pages * page_rows, rb, dtype=torch.uint8)
        for b, length in enumerate(inp["lengths"]):
            if name == "k_cache":
                cache.reserve(b, length)
            for i, pg in enumerate(cache.pages[b]):
                lo, hi = i * page_rows, min((i + 1) * page_rows, length)
                host_pool[pg * page_rows: pg * page_rows + hi - lo] = full[b, lo:hi]
        pool.copy_(host_pool.reshape(-1).to(pool.device))
    cache.seq_len = inp["seq_len"].to(pool.device)
    cache.host_len = list(inp["lengths"])
    return cache, rb


def _gather(cache, rb, b, rows):
    pool = cache.k[0].view(-1, rb).cpu(), cache.v[0].view(-1, rb).cpu()
    pr = cache.page_rows
    idx = [cache.pages[b][t // pr] * pr + t % pr for t in range(rows)]
    return pool[0][idx].numpy(), pool[1][idx].numpy()


CASES = {
    "decode": (CONFIGS[3].scaled(batch=3, n_q_heads=8, n_kv_heads=2, cached_range=None, cached_list=[300, 1029, 64]),
               128),
    "prefill_chunked": (CONFIGS[2].scaled(batch=2, n_new=300, n_q_heads=4, n_kv_heads=2, cached=None,
                                          cached_list=[0, 77]), 256),
    "prefill_d128": (CONFIGS[4].scaled(batch=1, n_new=200, n_q_heads=8, n_kv_heads=2, cached=None, cached_list=[390]),
                     128),
    # Q8_0 pools: head groups of 8 (K-direct kernel) and 16, and a prefill through the fp16 staging
    "q8_decode_g8": (CONFIGS[5].scaled(batch=2, n_q_heads=16, n_kv_heads=2, cached=None, cached_list=[777, 130]), 128),
    "q8_decode_g16": (CONFIGS[5].scaled(batch=2, n_q_heads=32, n_kv_heads=2, cached=None, cached_list=[300, 1500]),
                      256),
    "q8_prefill": (CONFIGS[5].scaled(batch=2, n_new=150, n_q_heads=8, n_kv_heads=2, cached=None, cached_list=[0, 260]),
                   128),
    # fp32 pools (the reference's dtype): CUDA-core decode and a staged prefill
    "fp32_decode": (CONFIGS[1].scaled(batch=2, cached=None, cached_list=[512, 200]), 128),
    "fp32_prefill": (CONFIGS[1].scaled(batch=2, n_new=150, n_q_heads=8, n_kv_heads=2, cached=None,
                                       cached_list=[0, 100]), 128),
}
TOL = {"fp32_decode": 2e-4, "fp32_prefill": 1e-3}


@pytest.mark.parametrize("case", list(CASES))
def test_paged_equals_contiguous_and_oracle(ctx, case):
    from helpers import gpu_forward, max_abs, oracle_forward
    from aihost_b200.ops import ComputeOps

    cfg, page_rows = CASES[case]
    inp = make_inputs(cfg)
    dev = torch.device("cuda", 0)
    cache, rb = _paged(ctx, cfg, inp, page_rows)
    out = ComputeOps(ctx).attention_layer_paged(inp["q"].to(dev), inp["k_new"].to(dev), inp["v_new"].to(dev), cache)
    torch.cuda.synchronize()
    ctx.sync_status()
    out_c, kc_c, vc_c = gpu_forward(ctx, cfg, inp)
    assert torch.equal(out.cpu(), out_c), case
    ref, _, _ = oracle_forward(cfg, inp)
    assert max_abs(out.cpu().float().numpy(), ref) <= TOL.get(case, 2e-3)
    cap = inp["capacity"]
    for b, length in enumerate(inp["lengths"]):
        rows = length + cfg.n_new
        k_p, v_p = _gather(cache, rb, b, rows)
        assert np.array_equal(k_p, kc_c.view(torch.uint8).numpy().reshape(cfg.batch, cap, rb)[b, :rows])
        assert np.array_equal(v_p, vc_c.view(torch.uint8).numpy().reshape(cfg.batch, cap, rb)[b, :rows])


def test_paged_block_table_outside_pool_reports_status(ctx):
    from aihost_b200 import EINVAL, AttnError
    from aihost_b200.ops import ComputeOps

    cfg, page_rows = CASES["decode"]
    inp = make_inputs(cfg)
    dev = torch.device("cuda", 0)
    cache, _ = _paged(ctx, cfg, inp, page_rows)
    for b, length in enumerate(inp["lengths"]):
        cache.reserve(b, length + 1)
    # sequence 0's new row (row 300) lives in its third page: point that page outside the pool
    cache.table_host[0, 300 // page_rows] = cache.n_pages
    cache.block_table.copy_(cache.table_host)
    hl = list(cache.host_len)
    from aihost_b200 import lib
    import ctypes

    spec = cache.spec
    out = torch.empty(cfg.batch, 1, spec.n_q_heads, spec.head_dim, dtype=torch.float16, device=dev)
    ctx.reserve_for(spec, cfg.batch, 1)
    d = spec.desc()
    h = (ctypes.c_int32 * cfg.batch)(*hl)
    st = lib().aihost_attn_forward_paged(ctx.handle, ctypes.byref(d), cfg.batch, 1, inp["q"].to(dev).data_ptr(),
                                         inp["k_new"].to(dev).data_ptr(), inp["v_new"].to(dev).data_ptr(),
                                         cache.k[0].data_ptr(), cache.v[0].data_ptr(), cache.n_pages, page_rows,
                                         cache.block_table.data_ptr(), cache.max_pages, cache.seq_len.data_ptr(),
                                         ctypes.cast(h, ctypes.c_void_p), out.data_ptr(), None)
    assert st == 0
    with pytest.raises(AttnError) as ei:
        ctx.sync_status()
    assert ei.value.status == EINVAL
    ComputeOps(ctx)  # the context stays usable


def test_paged_arguments_are_validated(ctx):
    import ctypes

    from aihost_b200 import EINVAL, EUNSUPPORTED, lib

    cfg, _ = CASES["decode"]
    spec = cfg.spec(1030)
    d = spec.desc()
    z = ctypes.c_void_p(16)
    assert lib().aihost_attn_forward_paged(ctx.handle, ctypes.byref(d), 1, 1, z, z, z, z, z, 4, 100, z, 9, z, None, z,
                                           None) == EINVAL  # page_rows not a multiple of 128
    assert lib().aihost_attn_forward_paged(ctx.handle, ctypes.byref(d), 1, 1, z, z, z, z, z, 4, 128, z, 2, z, None, z,
                                           None) == EINVAL  # kv_capacity beyond max_pages * page_rows
    import dataclasses

    d9 = dataclasses.replace(spec, kv_dtype=9).desc()
    assert lib().aihost_attn_forward_paged(ctx.handle, ctypes.byref(d9), 1, 1, z, z, z, z, z, 4, 128, z, 9, z, None,
                                           z, None) == EUNSUPPORTED
