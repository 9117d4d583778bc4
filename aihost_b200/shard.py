"""KV-head-sharded execution of the fused attention op, one process per GPU.

Heads are independent: Q head h only reads KV head h / (Hq/Hkv). Rank r of N owns KV heads
[r*Hkv/N, (r+1)*Hkv/N) and their Q heads [r*Hq/N, (r+1)*Hq/N). Each rank keeps only its own
heads' KV cache (a local slice, no remote reads), runs RoPE + append + attention on them, and
one NCCL all-gather over NVLink assembles the head outputs. The reference splits layers across
GPUs and stages activations through the host (Inference/MultiGPUTransformer.cs:48-183); this
module shards one layer's attention instead.

The gather is rank-major ([N][B][S][Hq/N][d], a contiguous concat of the ranks' outputs);
`to_reference_layout` turns it into [B][S][Hq][d] (the reference's [S, Hq*d] per sequence).
"""
from __future__ import annotations

import dataclasses

import torch

from . import Q8_0
from .ops import LayerSpec, row_bytes


@dataclasses.dataclass
class HeadShard:
    """Rank `rank` of `world`'s share of a layer described by `spec` (the full layer)."""

    spec: LayerSpec
    rank: int
    world: int

    def __post_init__(self):
        if self.spec.n_kv_heads % self.world:
            raise ValueError(f"{self.spec.n_kv_heads} KV heads do not split over {self.world} ranks")
        self.kv_per_rank = self.spec.n_kv_heads // self.world
        self.q_per_rank = self.spec.n_q_heads // self.world
        self.kv0 = self.rank * self.kv_per_rank
        self.q0 = self.rank * self.q_per_rank

    def local_spec(self) -> LayerSpec:
        """The layer as this rank sees it: its heads only, with a token-major local cache whose
        token stride is padded to 16 bytes (so TMA can stream it, also for one Q8_0 head)."""
        rb = row_bytes(self.spec.kv_dtype, self.spec.head_dim)
        tok = self.kv_per_rank * rb
        if self.spec.kv_dtype == Q8_0:
            tok = (tok + 15) // 16 * 16
        return dataclasses.replace(self.spec, n_q_heads=self.q_per_rank, n_kv_heads=self.kv_per_rank,
                                   kv_head_stride=rb, kv_token_stride=tok, kv_seq_stride=0)

    def local_cache_bytes(self, batch: int) -> int:
        ls = self.local_spec()
        return batch * ls.kv_capacity * ls.kv_token_stride

    def slice_q(self, q: torch.Tensor) -> torch.Tensor:
        """This rank's Q heads of q [B, S, Hq, d] (contiguous copy)."""
        return q[:, :, self.q0:self.q0 + self.q_per_rank].contiguous()

    def slice_kv(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's KV heads of k_new / v_new [B, S, Hkv, d] (contiguous copy)."""
        return x[:, :, self.kv0:self.kv0 + self.kv_per_rank].contiguous()

    def gather(self, out_local: torch.Tensor, group=None) -> torch.Tensor:
        """All-gather every rank's [B, S, Hq/N, d] output into a rank-major [N, B, S, Hq/N, d] buffer."""
        import torch.distributed as dist

        buf = torch.empty((self.world,) + tuple(out_local.shape), dtype=out_local.dtype, device=out_local.device)
        dist.all_gather_into_tensor(buf.view(-1), out_local.contiguous().view(-1), group=group)
        return buf

    @staticmethod
    def to_reference_layout(gathered: torch.Tensor) -> torch.Tensor:
        """[N, B, S, Hq/N, d] -> [B, S, Hq, d]."""
        n, b, s, hq_l, d = gathered.shape
        return gathered.permute(1, 2, 0, 3, 4).reshape(b, s, n * hq_l, d)


__all__ = ["HeadShard"]
