"""CUDA-graph replay of the fused decode step (one launch per step for fp16 / Q8_0 caches, with
the split merge done by the last split to finish): every replay must reproduce the direct call,
which needs the merge counters to return to zero after each launch."""
import numpy as np
import pytest
import torch

from aihost_b200 import F16, Q8_0
from aihost_b200.configs import CONFIGS, make_inputs
from helpers import gpu_forward

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kv", [F16, Q8_0])
def test_decode_graph_replays_match_direct_call(ctx, kv):
    from aihost_b200.ops import ComputeOps, KVCache

    cfg = CONFIGS[3].scaled(batch=4, kv_dtype=kv, cached_range=None, cached=None, cached_list=[4000, 100, 2500, 3000])
    inp = make_inputs(cfg)
    ref, _, _ = gpu_forward(ctx, cfg, inp)  # several splits per long sequence, merged in-kernel
    dev = torch.device("cuda", 0)
    cache = KVCache(ctx, cfg.spec(inp["capacity"]), batch=cfg.batch, device=dev)
    cache.k[0] = inp["k_cache"].to(dev).clone()
    cache.v[0] = inp["v_cache"].to(dev).clone()
    cache.seq_len = inp["seq_len"].to(dev)
    cache.host_len = list(inp["lengths"])
    q, kn, vn = (inp[n].to(dev) for n in ("q", "k_new", "v_new"))
    ops = ComputeOps(ctx)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        out = ops.attention_layer(q, kn, vn, cache)  # reserves scratch outside the capture
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ops.attention_layer(q, kn, vn, cache, out=out)
    for _ in range(3):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().float().numpy(), ref.float().numpy())
    ctx.sync_status()
