"""Helpers shared by the parity tests: run one fused-op call on the GPU and on the oracle."""
from __future__ import annotations

import numpy as np
import torch

from aihost_b200 import F16, F32, Q8_0
from aihost_b200.configs import AttnConfig, make_inputs
from aihost_b200.ops import ComputeOps, KVCache


def gpu_forward(ctx, cfg: AttnConfig, inp: dict, pass_host_len: bool = True):
    """Fused RoPE + append + attention on cuda:0 through the C ABI. Returns CPU tensors."""
    dev = torch.device("cuda", 0)
    spec = cfg.spec(inp["capacity"])
    cache = KVCache(ctx, spec, batch=cfg.batch, n_layers=1, device=dev)
    cache.k[0] = inp["k_cache"].to(dev).clone()
    cache.v[0] = inp["v_cache"].to(dev).clone()
    cache.seq_len = inp["seq_len"].to(dev)
    cache.host_len = list(inp["lengths"]) if pass_host_len else None
    ops = ComputeOps(ctx)
    out = ops.attention_layer(inp["q"].to(dev), inp["k_new"].to(dev), inp["v_new"].to(dev), cache, 0)
    torch.cuda.synchronize()
    ctx.sync_status()
    return out.cpu(), cache.k[0].cpu(), cache.v[0].cpu()


def oracle_forward(cfg: AttnConfig, inp: dict, mode=None, part=None, rows=None):
    """The same call on the CPU oracle (part = (b0, b1, h0, h1) sequences and query heads, rows =
    (r0, r1) query rows; None = all). Returns (out, k_cache, v_cache) as numpy arrays."""
    from oracle import oracle as orc

    mode = orc.EXACT if mode is None else mode
    desc = cfg.spec(inp["capacity"]).desc()
    kc = inp["k_cache"].numpy().copy()
    vc = inp["v_cache"].numpy().copy()
    q, kn, vn = (inp[n].numpy() for n in ("q", "k_new", "v_new"))
    out = orc.attn_forward(desc, q, kn, vn, kc, vc, inp["seq_len"].numpy(), mode=mode, part=part, rows=rows)
    return out, kc, vc


def max_abs(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.max(np.abs(a - b))) if a.size else 0.0


def cache_rows(cache_bytes, cfg: AttnConfig, capacity: int, rows):
    """Dequantised fp32 view [B, len(rows), Hkv, d] of selected cache rows (per-sequence row lists)."""
    from oracle import oracle as orc

    B, H, D = cfg.batch, cfg.n_kv_heads, cfg.head_dim
    c = np.asarray(cache_bytes)
    if cfg.kv_dtype == Q8_0:
        rb = 34 * (D // 32)
        c = c.reshape(B, capacity, H, rb)
        sel = np.stack([c[b, rows[b]] for b in range(B)])
        return orc.q8_0_dequantize(sel.reshape(-1), sel.size // 34 * 32).reshape(B, -1, H, D)
    dt = np.float32 if cfg.kv_dtype == F32 else np.float16
    c = c.view(dt).reshape(B, capacity, H, D)
    return np.stack([c[b, rows[b]] for b in range(B)]).astype(np.float32)


__all__ = ["gpu_forward", "oracle_forward", "max_abs", "cache_rows", "make_inputs", "F16", "F32", "Q8_0"]
