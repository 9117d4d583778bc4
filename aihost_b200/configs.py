"""The five workloads of the attention hot path and their seeded inputs.

Each config is one call of the fused op (RoPE + KV append + attention) on synthetic data with
the shapes and distributions below; seed = 1234 + config number. No model weights or datasets
are involved.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import F16, F32, Q8_0, ROPE_INTERLEAVED
from . import gen
from .ops import LayerSpec, row_bytes


@dataclass
class AttnConfig:
    number: int
    name: str
    batch: int
    n_q_heads: int
    n_kv_heads: int
    head_dim: int
    n_new: int
    theta: float
    q_dtype: int
    kv_dtype: int
    out_dtype: int
    cached: int | None = None          # fixed cached rows per sequence (None: seeded uniform range)
    cached_range: tuple | None = None  # (lo, hi) inclusive
    cached_list: list | None = None    # explicit cached rows per sequence
    std: float = 1.0
    rope_mode: int = ROPE_INTERLEAVED
    note: str = ""
    extra: dict = field(default_factory=dict)

    @property
    def seed(self) -> int:
        return 1234 + self.number

    def lengths(self) -> list[int]:
        if self.cached_list is not None:
            return list(self.cached_list)
        if self.cached is not None:
            return [self.cached] * self.batch
        lo, hi = self.cached_range
        return gen.randint((self.batch,), lo, hi, self.seed, "lengths").tolist()

    def capacity(self) -> int:
        return max(self.lengths()) + self.n_new

    def spec(self, capacity: int | None = None) -> LayerSpec:
        return LayerSpec(self.n_q_heads, self.n_kv_heads, self.head_dim, rope_theta=self.theta,
                         rope_mode=self.rope_mode, q_dtype=self.q_dtype, kv_dtype=self.kv_dtype,
                         out_dtype=self.out_dtype, kv_capacity=capacity or self.capacity())

    def scaled(self, **kw) -> "AttnConfig":
        """A copy with some fields replaced (smaller parity-test variants)."""
        d = dict(self.__dict__)
        d.update(kw)
        return AttnConfig(**d)


CONFIGS = {
    1: AttnConfig(1, "decode_tinyllama", batch=1, n_q_heads=32, n_kv_heads=4, head_dim=64, n_new=1, theta=1e4,
                  q_dtype=F32, kv_dtype=F32, out_dtype=F32, cached=512, std=0.5,
                  note="single-layer decode, fp32, 512 cached + 1 new at position 512"),
    2: AttnConfig(2, "prefill_qwen2_0.5b", batch=1, n_q_heads=14, n_kv_heads=2, head_dim=64, n_new=2048, theta=1e6,
                  q_dtype=F16, kv_dtype=F16, out_dtype=F16, cached=0,
                  note="causal prefill, fp16 in, fp32 accumulate, fp16 out"),
    3: AttnConfig(3, "decode_batched_llama3_8b", batch=64, n_q_heads=32, n_kv_heads=8, head_dim=128, n_new=1,
                  theta=5e5, q_dtype=F16, kv_dtype=F16, out_dtype=F16, cached_range=(256, 8192),
                  note="batched decode, fp16 cache, lengths uniform in [256, 8192]"),
    4: AttnConfig(4, "prefill_long_llama3_8b", batch=1, n_q_heads=32, n_kv_heads=8, head_dim=128, n_new=32768,
                  theta=5e5, q_dtype=F16, kv_dtype=F16, out_dtype=F16, cached=0,
                  note="long causal prefill, 1 KV-head group per GPU across 8"),
    5: AttnConfig(5, "decode_q8_0_llama3_70b", batch=32, n_q_heads=64, n_kv_heads=8, head_dim=128, n_new=1,
                  theta=5e5, q_dtype=F16, kv_dtype=Q8_0, out_dtype=F16, cached=16384,
                  note="batched decode, GGUF Q8_0 cache, 16384 cached rows each"),
}


def torch_dtype(code: int) -> torch.dtype:
    return torch.float32 if code == F32 else torch.float16


def make_inputs(cfg: AttnConfig, device="cpu", capacity: int | None = None) -> dict:
    """q, k_new, v_new, k_cache, v_cache (uint8 bytes), seq_len (int32) for one call of `cfg`."""
    B, S, Hq, Hkv, D = cfg.batch, cfg.n_new, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    lengths = cfg.lengths()
    cap = capacity or (max(lengths) + S)
    qdt = torch_dtype(cfg.q_dtype)
    s = cfg.seed
    q = gen.normal((B, S, Hq, D), s, "q", std=cfg.std, dtype=qdt, device=device)
    k_new = gen.normal((B, S, Hkv, D), s, "k_new", std=cfg.std, dtype=qdt, device=device)
    v_new = gen.normal((B, S, Hkv, D), s, "v_new", std=cfg.std, dtype=qdt, device=device)
    rb = row_bytes(cfg.kv_dtype, D)
    caches = []
    for name in ("k_cache", "v_cache"):
        if cfg.kv_dtype == Q8_0:
            c = gen.q8_0_blocks(B * cap * Hkv * (D // 32), s, name, device=device)
        else:
            c = gen.normal((B, cap, Hkv, D), s, name, std=cfg.std, dtype=torch_dtype(cfg.kv_dtype),
                           device=device).view(torch.uint8).reshape(-1)
        caches.append(c)
    assert caches[0].numel() == B * cap * Hkv * rb
    seq_len = torch.tensor(lengths, dtype=torch.int32, device=device)
    return dict(q=q, k_new=k_new, v_new=v_new, k_cache=caches[0], v_cache=caches[1], seq_len=seq_len,
                lengths=lengths, capacity=cap)


__all__ = ["AttnConfig", "CONFIGS", "make_inputs", "torch_dtype"]
