"""Context-parallel decode (aihost_attn_decode_partial + aihost_attn_merge_partials, ContextShard).

One GPU: the ranks of a context-parallel decode are emulated in one process. Each emulated rank
gets its own local cache holding its chunk of every sequence's rows, runs its part
(ContextShard.partial, which goes through aihost_attn_decode_partial), and the library's merge
kernel combines the parts. The result must match the CPU oracle's unsharded fused decode step
(config 1 shape in fp32, fp16 and Q8_0 caches with batch > 1). The log-sum-exp output is
checked against a float64 restatement over the oracle's final cache rows.
Two GPUs (else skipped): two processes run ContextShard.forward with NCCL all-gathers.
"""
import os

import numpy as np
import pytest
import torch

from aihost_b200 import F16, F32, Q8_0
from aihost_b200.configs import CONFIGS, make_inputs

pytestmark = pytest.mark.gpu

TOL = {F32: 2e-4, F16: 2e-3, Q8_0: 2e-3}


def _cases():
    return {
        "cfg1_fp32": CONFIGS[1],
        "fp16_b3": CONFIGS[3].scaled(batch=3, n_q_heads=8, n_kv_heads=2, cached_range=None, cached=None,
                                     cached_list=[300, 1029, 64]),
        "q8_b2": CONFIGS[5].scaled(batch=2, n_q_heads=16, n_kv_heads=2, cached=None, cached_list=[777, 130]),
    }


def _local_cache(ctx, cfg, inp, shard, dev):
    """KVCache holding rank `shard.rank`'s chunk of every sequence's rows (local row 0 = global row lo)."""
    from aihost_b200.ops import KVCache, row_bytes

    cap = inp["capacity"]
    rb = row_bytes(cfg.kv_dtype, cfg.head_dim) * cfg.n_kv_heads
    cache = KVCache(ctx, cfg.spec(cap), batch=cfg.batch, device=dev)
    rows = []
    for name, dst in (("k_cache", cache.k[0]), ("v_cache", cache.v[0])):
        full = inp[name].view(cfg.batch, cap, rb)
        local = torch.zeros(cfg.batch, cap, rb, dtype=torch.uint8)
        rows = []
        for b, length in enumerate(inp["lengths"]):
            lo, hi = shard.chunk(length)
            local[b, : hi - lo] = full[b, lo:hi]
            rows.append(hi - lo)
        dst.copy_(local.reshape(-1).to(dev))
    cache.seq_len = torch.tensor(rows, dtype=torch.int32, device=dev)
    cache.host_len = rows
    return cache


def _emulated(ctx, cfg, world):
    from aihost_b200.ops import ComputeOps
    from aihost_b200.shard import ContextShard

    dev = torch.device("cuda", 0)
    inp = make_inputs(cfg)
    ops = ComputeOps(ctx)
    q, kn, vn = (inp[n].to(dev) for n in ("q", "k_new", "v_new"))
    q_pos = inp["seq_len"].to(dev)
    parts = []
    for r in range(world):
        sh = ContextShard(r, world)
        cache = _local_cache(ctx, cfg, inp, sh, dev)
        parts.append(sh.partial(ops, q, kn, vn, cache, q_pos))
    o_all = torch.stack([o for o, _ in parts])
    lse_all = torch.stack([lse for _, lse in parts])
    out = ops.merge_partials(o_all, lse_all)
    torch.cuda.synchronize()
    ctx.sync_status()
    return out.cpu().float().numpy(), inp, parts


@pytest.mark.parametrize("world", [1, 2, 4])
@pytest.mark.parametrize("case", ["cfg1_fp32", "fp16_b3", "q8_b2"])
def test_context_parallel_decode_matches_oracle(ctx, case, world):
    from helpers import max_abs, oracle_forward

    cfg = _cases()[case]
    got, inp, _ = _emulated(ctx, cfg, world)
    ref, _, _ = oracle_forward(cfg, inp)
    err = max_abs(got, ref.reshape(got.shape))
    assert err <= TOL[cfg.kv_dtype], (case, world, err)


def test_decode_partial_lse_matches_float64(ctx):
    """lse of one part holding every row equals ln sum_j exp(scale * q_rot . k_j) over the final cache."""
    from helpers import cache_rows, oracle_forward
    from oracle import oracle as orc

    cfg = _cases()["cfg1_fp32"]
    _, inp, parts = _emulated(ctx, cfg, 1)
    lse = parts[0][1].cpu().numpy()  # [B, Hq]
    _, kc, _ = oracle_forward(cfg, inp)
    B, Hq, Hkv, d = cfg.batch, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    G = Hq // Hkv
    for b, L in enumerate(inp["lengths"]):
        krows = cache_rows(kc, cfg, inp["capacity"], [list(range(L + 1))] * B)[b].astype(np.float64)
        qr = orc.rope_full(inp["q"].numpy()[b, 0].reshape(1, Hq * d).astype(np.float32), L, Hq, d,
                           cfg.spec().rope_theta).reshape(Hq, d).astype(np.float64)
        for h in range(Hq):
            s = krows[:, h // G, :] @ qr[h] / np.sqrt(d)
            m = s.max()
            ref = m + np.log(np.exp(s - m).sum())
            assert abs(lse[b, h] - ref) <= 1e-4, (b, h, lse[b, h], ref)


def _cp_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from aihost_b200.ops import ComputeOps, Context
        from aihost_b200.shard import ContextShard

        cfg = _cases()["fp16_b3"]
        dev = torch.device("cuda", rank)
        ctx = Context(rank)
        try:
            inp = make_inputs(cfg)
            sh = ContextShard(rank, world)
            cache = _local_cache(ctx, cfg, inp, sh, dev)
            out = sh.forward(ComputeOps(ctx), inp["q"].to(dev), inp["k_new"].to(dev), inp["v_new"].to(dev), cache,
                             inp["seq_len"].to(dev))
            torch.cuda.synchronize()
            ctx.sync_status()
            if rank == 0:
                from helpers import max_abs, oracle_forward

                ref, _, _ = oracle_forward(cfg, inp)
                q.put(max_abs(out.cpu().float().numpy(), ref.reshape(tuple(out.shape))))
        finally:
            ctx.close()
    except Exception as e:
        q.put(f"rank {rank}: {e!r}")
        raise
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_context_parallel_two_gpus_match_oracle():
    import socket

    import torch.multiprocessing as mp

    sock = socket.socket()
    sock.bind(("127.0.0.1", 0))
    port = sock.getsockname()[1]
    sock.close()
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    procs = [mpc.Process(target=_cp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    err = q.get(timeout=5)
    assert isinstance(err, float) and err <= 2e-3, err
