"""KV-head sharding through the C ABI (aihost_attn_dist_* / aihost_attn_forward_sharded).

World of 1 (any GPU box): the sharded call must equal aihost_attn_forward on the same inputs.
World of 2 (boxes with two or more GPUs, else skipped): two processes, one GPU each, run their
heads and the library's NCCL all-gather; rank 0 compares the gathered output with the CPU oracle
on the unsharded layer (tolerance 2e-3, fp16 inputs). NVLS is switched off for the test's NCCL.
"""
import os

import numpy as np
import pytest
import torch

from aihost_b200 import F16, Q8_0, ROPE_INTERLEAVED
from aihost_b200.configs import CONFIGS, make_inputs

pytestmark = pytest.mark.gpu


def _local_cache(full_cache, cfg, shard, capacity, device):
    from aihost_b200.ops import row_bytes

    rb = row_bytes(cfg.kv_dtype, cfg.head_dim)
    full = full_cache.view(cfg.batch, capacity, cfg.n_kv_heads * rb)
    part = full[:, :, shard.kv0 * rb:(shard.kv0 + shard.kv_per_rank) * rb]
    tok = shard.local_spec().kv_token_stride
    out = torch.zeros(cfg.batch, capacity, tok, dtype=torch.uint8)
    out[:, :, :part.shape[2]] = part
    return out.reshape(-1).to(device)


def _run_rank(rank, world, nccl_id, cfg, capacity, device):
    from aihost_b200.ops import ComputeOps, Context, KVCache
    from aihost_b200.shard import HeadShard, NcclDist

    torch.cuda.set_device(device)
    ctx = Context(device)
    inp = make_inputs(cfg, capacity=capacity)
    shard = HeadShard(cfg.spec(capacity), rank, world)
    cache = KVCache(ctx, shard.local_spec(), batch=cfg.batch, device=torch.device("cuda", device))
    cache.k[0] = _local_cache(inp["k_cache"], cfg, shard, capacity, device)
    cache.v[0] = _local_cache(inp["v_cache"], cfg, shard, capacity, device)
    cache.seq_len = inp["seq_len"].to(device)
    cache.host_len = list(inp["lengths"])
    dist = NcclDist(world, rank, nccl_id, device)
    try:
        dev = torch.device("cuda", device)
        out = shard.forward(dist, ComputeOps(ctx), shard.slice_q(inp["q"]).to(dev), shard.slice_kv(inp["k_new"]).to(dev),
                            shard.slice_kv(inp["v_new"]).to(dev), cache)
        dist.sync(timeout_ms=60000)  # bounded wait for the kernels and the all-gather
        torch.cuda.synchronize()
        ctx.sync_status()
        return HeadShard.to_reference_layout(out.cpu()).float().numpy(), inp
    finally:
        dist.close()
        ctx.close()


def _cfg(kv):
    return CONFIGS[3].scaled(batch=2, n_q_heads=8, n_kv_heads=4, head_dim=128, kv_dtype=kv, q_dtype=F16,
                             out_dtype=F16, cached_range=None, cached=None, cached_list=[300, 1029],
                             rope_mode=ROPE_INTERLEAVED)


@pytest.mark.parametrize("kv", [F16, Q8_0])
def test_sharded_world_one_equals_forward(ctx, kv):
    from aihost_b200.shard import NcclDist
    from helpers import gpu_forward

    cfg = _cfg(kv)
    got, inp = _run_rank(0, 1, NcclDist.unique_id(), cfg, 1056, 0)
    ref, _, _ = gpu_forward(ctx, cfg, make_inputs(cfg, capacity=1056))
    assert np.array_equal(got, ref.float().numpy())


def _worker(rank, world, nccl_id, kv, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        got, inp = _run_rank(rank, world, nccl_id, _cfg(kv), 1056, rank)
        if rank == 0:
            from helpers import max_abs, oracle_forward

            ref, _, _ = oracle_forward(_cfg(kv), make_inputs(_cfg(kv), capacity=1056))
            q.put(max_abs(got, ref))
    except Exception as e:  # report instead of hanging the parent
        q.put(f"rank {rank}: {e!r}")
        raise


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("kv", [F16, Q8_0])
def test_sharded_two_gpus_match_oracle(kv):
    import torch.multiprocessing as mp

    from aihost_b200.shard import NcclDist

    nccl_id = NcclDist.unique_id()
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    procs = [mpc.Process(target=_worker, args=(r, 2, nccl_id, kv, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    err = q.get(timeout=5)
    assert isinstance(err, float) and err <= 2e-3, err


# ---------------------------------------------------------------- query-row sharding (Hkv < N)

def _row_cfg():
    return CONFIGS[2].scaled(n_new=700, n_q_heads=4, n_kv_heads=2, head_dim=64, cached=None, cached_list=[200])


def _row_run(rank, world, device, group=None):
    from aihost_b200.ops import ComputeOps, Context, KVCache
    from aihost_b200.shard import RowShard

    torch.cuda.set_device(device)
    dev = torch.device("cuda", device)
    cfg = _row_cfg()
    inp = make_inputs(cfg, capacity=1024)
    ctx = Context(device)
    try:
        cache = KVCache(ctx, cfg.spec(1024), batch=1, device=dev)
        cache.k[0] = inp["k_cache"].to(dev).clone()
        cache.v[0] = inp["v_cache"].to(dev).clone()
        cache.seq_len = inp["seq_len"].to(dev)
        cache.host_len = list(inp["lengths"])
        out = RowShard(cfg.n_new, 200, rank, world).forward(ComputeOps(ctx), inp["q"].to(dev), inp["k_new"].to(dev),
                                                            inp["v_new"].to(dev), cache, group=group)
        torch.cuda.synchronize()
        ctx.sync_status()
        return out.cpu().float().numpy(), inp
    finally:
        ctx.close()


def test_row_shard_world_one_matches_oracle():
    from helpers import max_abs, oracle_forward

    got, inp = _row_run(0, 1, 0)
    ref, _, _ = oracle_forward(_row_cfg(), inp)
    assert max_abs(got, ref) <= 2e-3


def _row_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        got, inp = _row_run(rank, world, rank)
        if rank == 0:
            from helpers import max_abs, oracle_forward

            ref, _, _ = oracle_forward(_row_cfg(), inp)
            q.put(max_abs(got, ref))
    except Exception as e:
        q.put(f"rank {rank}: {e!r}")
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_row_shard_two_gpus_match_oracle():
    import socket

    import torch.multiprocessing as mp

    sock = socket.socket()
    sock.bind(("127.0.0.1", 0))
    port = sock.getsockname()[1]
    sock.close()
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    procs = [mpc.Process(target=_row_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    err = q.get(timeout=5)
    assert isinstance(err, float) and err <= 2e-3, err
