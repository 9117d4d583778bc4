"""GPU kernels against the golden vectors of the reference's own shaders.

Decode cases run the fp32 path (fp32 q / cache / out; bound 2e-4). Prefill cases use
fp16-representable inputs and run the fp16 tcgen05 path (fp16 cache, fp32 out; bound 2e-3).
"""
import numpy as np
import pytest
import torch

from aihost_b200 import F16, F32
from aihost_b200.ops import ComputeOps, KVCache
from golden_cases import case_layout, load

import sys
from pathlib import Path
sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
from make_golden import CASES, case_inputs  # noqa: E402

pytestmark = pytest.mark.gpu
Z, META = load()


@pytest.mark.parametrize("name", sorted(CASES))
def test_gpu_matches_reference_shaders(ctx, name):
    m = META[name]
    x = case_inputs(name)
    decode = m["S"] == 1
    dt = F32 if decode else F16
    tdt = torch.float32 if decode else torch.float16
    spec, S, P, hq, hkv, d = case_layout(m, x, dt, dt, F32)
    dev = torch.device("cuda", 0)
    cache = KVCache(ctx, spec, batch=1, device=dev)
    kc = torch.zeros(P + S, hkv * d, dtype=tdt)
    vc = torch.zeros(P + S, hkv * d, dtype=tdt)
    kc[:P], vc[:P] = torch.from_numpy(x["k_cached"]).to(tdt), torch.from_numpy(x["v_cached"]).to(tdt)
    cache.k[0] = kc.view(torch.uint8).reshape(-1).to(dev)
    cache.v[0] = vc.view(torch.uint8).reshape(-1).to(dev)
    cache.seq_len = torch.tensor([P], dtype=torch.int32, device=dev)
    cache.host_len = [P]
    q = torch.from_numpy(x["q"]).to(tdt).reshape(1, S, hq, d).to(dev)
    kn = torch.from_numpy(x["k_new"]).to(tdt).reshape(1, S, hkv, d).to(dev)
    vn = torch.from_numpy(x["v_new"]).to(tdt).reshape(1, S, hkv, d).to(dev)
    out = ComputeOps(ctx).attention_layer(q, kn, vn, cache)
    torch.cuda.synchronize()
    ctx.sync_status()
    got = out.cpu().numpy().reshape(S, hq * d)
    tol = 2e-4 if decode else 2e-3
    assert np.abs(got - Z[f"{name}.out"]).max() <= tol
