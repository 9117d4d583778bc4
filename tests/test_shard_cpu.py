"""KV-head sharding host logic on CPU: two gloo ranks each compute their heads (with the CPU
oracle standing in for the GPU kernels) and the all-gather must rebuild the unsharded result."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from aihost_b200 import F16, F32, Q8_0, ROPE_INTERLEAVED
from aihost_b200.configs import CONFIGS, make_inputs
from aihost_b200.ops import row_bytes
from aihost_b200.shard import HeadShard


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _local_cache(full_cache: torch.Tensor, cfg, shard: HeadShard, capacity: int) -> torch.Tensor:
    """The rank's slice of a full token-major cache, re-laid with the local token stride."""
    rb = row_bytes(cfg.kv_dtype, cfg.head_dim)
    full = full_cache.view(cfg.batch, capacity, cfg.n_kv_heads * rb)
    part = full[:, :, shard.kv0 * rb:(shard.kv0 + shard.kv_per_rank) * rb]
    tok = shard.local_spec().kv_token_stride
    out = torch.zeros(cfg.batch, capacity, tok, dtype=torch.uint8)
    out[:, :, :part.shape[2]] = part
    return out.reshape(-1)


def _worker(rank, world, port, cfg_num, kv, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle as orc

        cfg = CONFIGS[cfg_num].scaled(batch=2, n_q_heads=8, n_kv_heads=4, head_dim=64, kv_dtype=kv,
                                      q_dtype=F32 if kv == F32 else F16, out_dtype=F32, cached_range=None,
                                      cached=None, cached_list=[37, 90], rope_mode=ROPE_INTERLEAVED)
        inp = make_inputs(cfg, capacity=96)
        shard = HeadShard(cfg.spec(96), rank, world)
        ls = shard.local_spec()
        kc = _local_cache(inp["k_cache"], cfg, shard, 96).numpy()
        vc = _local_cache(inp["v_cache"], cfg, shard, 96).numpy()
        out_l = orc.attn_forward(ls.desc(), shard.slice_q(inp["q"]).numpy(), shard.slice_kv(inp["k_new"]).numpy(),
                                 shard.slice_kv(inp["v_new"]).numpy(), kc, vc, inp["seq_len"].numpy())
        gathered = shard.gather(torch.from_numpy(out_l))
        full = HeadShard.to_reference_layout(gathered)
        if rank == 0:
            ref = orc.attn_forward(cfg.spec(96).desc(), inp["q"].numpy(), inp["k_new"].numpy(),
                                   inp["v_new"].numpy(), inp["k_cache"].numpy().copy(),
                                   inp["v_cache"].numpy().copy(), inp["seq_len"].numpy())
            result_q.put(float(np.abs(full.numpy() - ref).max()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("kv", [F32, Q8_0])
def test_head_sharded_gather_matches_unsharded(kv):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, 3, kv, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    err = q.get(timeout=5)
    assert err == 0.0, err


def test_local_spec_pads_q8_token_stride():
    spec = CONFIGS[5].spec(16385)
    sh = HeadShard(spec, 3, 8)
    ls = sh.local_spec()
    assert (ls.n_q_heads, ls.n_kv_heads) == (8, 1)
    assert ls.kv_head_stride == 136 and ls.kv_token_stride == 144
    with pytest.raises(ValueError):
        HeadShard(CONFIGS[2].spec(2048), 0, 4)  # 2 KV heads over 4 ranks


# ---------------------------------------------------------------- query-row sharding (Hkv < N)

def test_row_boundaries_cover_rows_and_balance_causal_work():
    from aihost_b200.shard import RowShard

    for n_new, cached, world in [(2048, 0, 2), (2048, 0, 8), (32768, 0, 8), (1000, 3000, 4), (150, 100, 2)]:
        bounds = [RowShard(n_new, cached, 0, world).boundary(k) for k in range(world + 1)]
        assert bounds[0] == 0 and bounds[-1] == n_new and bounds == sorted(bounds)
        assert all(b % 128 == 0 for b in bounds[:-1])
        work = [sum(cached + i + 1 for i in range(bounds[k], bounds[k + 1])) for k in range(world)]
        if n_new >= 128 * world * 4:  # enough tiles for the rounding to stay small
            assert max(work) <= 1.25 * sum(work) / world, work


def _row_worker(rank, world, port, result_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from aihost_b200.shard import RowShard
        from oracle import oracle as orc

        cfg = CONFIGS[2].scaled(n_new=300, n_q_heads=4, n_kv_heads=2, head_dim=64, q_dtype=F32, kv_dtype=F32,
                                out_dtype=F32, cached=None, cached_list=[77])
        cap = 400
        inp = make_inputs(cfg, capacity=cap)
        S, hq, hkv, d, P = cfg.n_new, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, 77
        theta = cfg.spec(cap).rope_theta
        sh = RowShard(S, P, rank, world)
        # the CPU oracle stands in for the kernels: RoPE(K) + append on every rank, then this rank's rows
        k = orc.rope_full(inp["k_new"].numpy()[0].reshape(S, hkv * d), P, hkv, d, theta)
        kc = inp["k_cache"].numpy().view(np.float32).reshape(cap, hkv * d).copy()
        vc = inp["v_cache"].numpy().view(np.float32).reshape(cap, hkv * d).copy()
        kc[P:P + S] = k
        vc[P:P + S] = inp["v_new"].numpy()[0].reshape(S, hkv * d)
        a, b = sh.rows
        out_t = torch.zeros(S, hq * d)
        if b > a:
            qa = orc.rope_full(inp["q"].numpy()[0, a:b].reshape(b - a, hq * d), P + a, hq, d, theta)
            out_t[a:b] = torch.from_numpy(orc.mha(qa, kc[:P + b], vc[:P + b], hq, P + a))
        for r in range(world):  # each block broadcast from its owner, as RowShard.forward does
            a_r, b_r = sh.boundary(r), sh.boundary(r + 1)
            if b_r > a_r:
                dist.broadcast(out_t[a_r:b_r], src=r)
        out = out_t.numpy()
        if rank == 0:
            ref = orc.attn_forward(cfg.spec(cap).desc(), inp["q"].numpy(), inp["k_new"].numpy(), inp["v_new"].numpy(),
                                   inp["k_cache"].numpy().copy(), inp["v_cache"].numpy().copy(), inp["seq_len"].numpy())
            result_q.put(float(np.abs(out - ref.reshape(S, hq * d)).max()))
    finally:
        dist.destroy_process_group()


def test_row_sharded_gather_matches_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_row_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    err = q.get(timeout=5)
    assert err <= 1e-5, err


def test_context_chunks_cover_rows_and_balance():
    from aihost_b200.shard import ContextShard

    for length in (1, 2, 7, 512, 513, 16384):
        for world in (1, 2, 4, 8):
            if length < world:
                continue
            spans = [ContextShard(r, world).chunk(length) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == length
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            sizes = [hi - lo for lo, hi in spans]
            assert min(sizes) >= 1 and max(sizes) - min(sizes) <= 1
    assert ContextShard(3, 4).appends and not ContextShard(0, 4).appends


def test_context_merge_of_partials_equals_full_softmax():
    """The merge the kernel implements: out = sum_p o_p exp(lse_p - lse), lse = ln sum_p exp(lse_p)."""
    from aihost_b200.shard import ContextShard

    rng = np.random.default_rng(7)
    for n_rows, world in ((513, 2), (1000, 4), (9, 8)):
        s = rng.normal(0, 3, n_rows)
        v = rng.normal(0, 1, (n_rows, 16))
        full = (np.exp(s - s.max()) / np.exp(s - s.max()).sum()) @ v
        o, lse = [], []
        for r in range(world):
            lo, hi = ContextShard(r, world).chunk(n_rows)
            m = s[lo:hi].max()
            e = np.exp(s[lo:hi] - m)
            o.append(e @ v[lo:hi] / e.sum())
            lse.append(m + np.log(e.sum()))
        lse = np.array(lse)
        w = np.exp(lse - lse.max())
        merged = (w[:, None] * np.array(o)).sum(0) / w.sum()
        assert np.abs(merged - full).max() < 1e-12


def test_paged_cache_allocator_host_logic():
    """PagedKVCache's page bookkeeping (host side; pools in host memory, no kernels)."""
    from aihost_b200 import EINVAL, ENOMEM, F16, AttnError
    from aihost_b200.ops import LayerSpec, PagedKVCache

    spec = LayerSpec(8, 2, 128, kv_dtype=F16, q_dtype=F16, out_dtype=F16, kv_capacity=1000)
    cache = PagedKVCache(None, spec, n_pages=10, page_rows=128, batch=3, device=torch.device("cpu"))
    assert cache.max_pages == 8 and cache.k[0].numel() == 10 * 128 * 2 * 128 * 2
    cache.reserve(0, 300)   # 3 pages
    cache.reserve(1, 128)   # 1 page
    cache.reserve(0, 300)   # nothing new
    assert cache.pages[0] == [0, 1, 2] and cache.pages[1] == [3]
    assert cache.block_table[0, :4].tolist() == [0, 1, 2, -1] and cache.block_table[1, 0] == 3
    with pytest.raises(AttnError) as ei:
        cache.reserve(2, 1001)   # beyond kv_capacity
    assert ei.value.status == EINVAL
    cache.reserve(2, 6 * 128)    # the last 6 pages
    with pytest.raises(AttnError) as ei:
        cache.reserve(1, 2 * 128)  # pool exhausted
    assert ei.value.status == ENOMEM
    cache.release(0)
    assert sorted(cache.free) == [0, 1, 2] and cache.block_table[0].tolist() == [-1] * 8
    cache.reserve(1, 2 * 128)
    assert cache.pages[1] == [3, 0]
    with pytest.raises(AttnError):
        PagedKVCache(None, spec, n_pages=4, page_rows=100, device=torch.device("cpu"))
