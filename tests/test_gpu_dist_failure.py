"""Failure detection on the sharded path, made on the host: a rank that never joins.

Rank 0 of a world of 2 calls aihost_attn_dist_init_bounded with a 3 s limit and rank 1 never
calls it. The set-up must come back with AIHOST_ETIMEOUT within the limit (plus polling slack),
having aborted the half-built communicator, and the process must still be able to build a
working communicator afterwards. Nothing runs on the GPU while the set-up waits (NCCL's
bootstrap is host sockets), so no kernel or collective is ever left in flight. The test runs in a
child process under a wall-clock limit, with NVLS off, so even a hang would only end that child.
The reference has no bound on any wait (ICompute/Vulkan/VulkanComputeCommandQueue.cs:287).
"""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent

CHILD = r"""
import ctypes, json, os, sys, time
sys.path.insert(0, sys.argv[1])
import torch
torch.cuda.set_device(0)
torch.zeros(1, device="cuda")
import aihost_b200 as A
from aihost_b200.shard import NcclDist
nid = ctypes.create_string_buffer(NcclDist.unique_id(), 128)
h = ctypes.c_void_p()
t0 = time.monotonic()
st = A.lib().aihost_attn_dist_init_bounded(2, 0, nid, 0, 3000, ctypes.byref(h))
elapsed = time.monotonic() - t0
msg = A.lib().aihost_attn_last_error().decode()
# the process stays usable: a fresh one-rank communicator, a sharded-path wait on an idle stream
d = NcclDist(1, 0, NcclDist.unique_id(), 0, timeout_ms=60000)
d.sync(timeout_ms=10000)
d.close()
print(json.dumps({"status": st, "elapsed": elapsed, "msg": msg, "handle": bool(h.value)}), flush=True)
"""


def test_rank_that_never_joins_times_out_on_the_host():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", NCCL_DEBUG="WARN")
    res = subprocess.run([sys.executable, "-c", CHILD, str(ROOT)], capture_output=True, text=True, timeout=240,
                         env=env)
    assert res.returncode == 0, res.stderr[-2000:]
    line = [ln for ln in res.stdout.splitlines() if ln.startswith("{")][-1]
    r = json.loads(line)
    from aihost_b200 import ETIMEOUT

    assert r["status"] == ETIMEOUT, r
    assert not r["handle"]
    assert "3000 ms" in r["msg"]
    assert 2.9 <= r["elapsed"] <= 30.0, r


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_call_refuses_context_and_communicator_on_different_devices():
    import ctypes

    from aihost_b200 import EINVAL, lib
    from aihost_b200.ops import Context, LayerSpec
    from aihost_b200.shard import NcclDist

    ctx = Context(1)
    dist = NcclDist(1, 0, NcclDist.unique_id(), 0, timeout_ms=60000)
    try:
        d = LayerSpec(8, 2, 64, kv_capacity=64).desc()
        buf = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda:1")
        sl = torch.zeros(1, dtype=torch.int32, device="cuda:1")
        p = buf.data_ptr()
        st = lib().aihost_attn_forward_sharded(dist.handle, ctx.handle, ctypes.byref(d), 1, 1, p, p, p, p, p,
                                               sl.data_ptr(), None, p, None)
        assert st == EINVAL
        assert b"device" in lib().aihost_attn_last_error()
    finally:
        dist.close()
        ctx.close()
