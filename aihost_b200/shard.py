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

    def forward(self, dist: "NcclDist", ops, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, cache,
                out: torch.Tensor | None = None, layer: int = 0) -> torch.Tensor:
        """This rank's heads of the fused layer step through aihost_attn_forward_sharded: RoPE,
        append into the local cache, attention, then one NCCL all-gather of the head outputs.
        q [B, S, Hq/N, d], k_new / v_new [B, S, Hkv/N, d] (this rank's slices), `cache` a
        KVCache built with local_spec(). Returns the rank-major [N, B, S, Hq/N, d] buffer."""
        import ctypes

        from . import check, lib
        from .ops import _ptr, _stream

        ls = cache.spec
        B, S = q.shape[0], q.shape[1]
        if out is None:
            odt = torch.float32 if ls.out_dtype == 0 else torch.float16
            out = torch.empty((self.world, B, S, ls.n_q_heads, ls.head_dim), dtype=odt, device=q.device)
        ops.ctx.reserve_for(ls, B, S)
        d = ls.desc()
        hl = (ctypes.c_int32 * B)(*cache.host_len) if cache.host_len is not None else None
        check(lib().aihost_attn_forward_sharded(dist.handle, ops.ctx.handle, ctypes.byref(d), B, S, _ptr(q),
                                                _ptr(k_new), _ptr(v_new), _ptr(cache.k[layer]), _ptr(cache.v[layer]),
                                                _ptr(cache.seq_len),
                                                ctypes.cast(hl, ctypes.c_void_p) if hl is not None else None,
                                                _ptr(out), _stream(ops.stream)))
        return out

    @staticmethod
    def to_reference_layout(gathered: torch.Tensor) -> torch.Tensor:
        """[N, B, S, Hq/N, d] -> [B, S, Hq, d]."""
        n, b, s, hq_l, d = gathered.shape
        return gathered.permute(1, 2, 0, 3, 4).reshape(b, s, n * hq_l, d)


@dataclasses.dataclass
class RowShard:
    """Rank `rank` of `world`'s query rows of one sequence's causal prefill: n_new new rows after
    `cached` rows. For layers with fewer KV heads than ranks (Hkv < N), where head sharding runs
    out of heads: every rank appends all new K/V rows (replicated, a small fraction of the work),
    each rank attends its own contiguous block of query rows over the cache, and each block is
    broadcast from its owner into every rank's output. Block boundaries split the causal work, sum over rows i of (cached + i + 1)
    keys, into equal parts, rounded to the prefill kernel's 128-row tiles."""

    n_new: int
    cached: int
    rank: int
    world: int
    tile: int = 128

    def pairs(self, k: int) -> float:
        """Causal (query, key) pairs of rank k's block."""
        a, b = self.boundary(k), self.boundary(k + 1)
        return float(sum(self.cached + i + 1 for i in range(a, b)))

    def boundary(self, k: int) -> int:
        """First row of rank k's block (k = world gives n_new)."""
        if k <= 0:
            return 0
        if k >= self.world:
            return self.n_new
        p, s = float(self.cached), float(self.n_new)
        total = s * p + s * (s + 1) / 2
        target = total * k / self.world
        r = -(p + 0.5) + ((p + 0.5) ** 2 + 2 * target) ** 0.5  # r*p + r(r+1)/2 = target
        r = int(round(r / self.tile)) * self.tile
        return max(0, min(self.n_new, r))

    @property
    def rows(self) -> tuple[int, int]:
        return self.boundary(self.rank), self.boundary(self.rank + 1)

    @property
    def max_rows(self) -> int:
        return max(self.boundary(k + 1) - self.boundary(k) for k in range(self.world))

    def forward(self, ops, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, cache, layer: int = 0,
                group=None, out: torch.Tensor | None = None) -> torch.Tensor:
        """The fused step for batch-1 inputs q [1, S, Hq, d], k_new / v_new [1, S, Hkv, d], with
        `cache` holding `cached` rows (device and host lengths), split over the ranks by query
        rows. Every rank appends all S new rows (RoPE'd K) to its cache, runs the fused op
        (aihost_attn_forward: RoPE of its Q rows in the kernel, causal attention) on its block
        [a, b) as a call that starts at row cached + a, and the blocks are then broadcast from
        their owners into `out` [1, S, Hq, d] (allocated when None) on every rank. `group` must
        list the ranks 0..world-1 in order (None: the default group). The cache lengths are not
        advanced."""
        import torch.distributed as dist

        spec = cache.spec
        if spec.kv_dtype not in (0, 1):
            raise ValueError("row sharding supports fp32 / fp16 caches")
        S, hq, hkv, d = q.shape[1], q.shape[2], k_new.shape[2], q.shape[3]
        if S != self.n_new or q.shape[0] != 1:
            raise ValueError(f"expected q [1, {self.n_new}, Hq, d], got {tuple(q.shape)}")
        P = self.cached
        if out is None:
            odt = torch.float32 if spec.out_dtype == 0 else torch.float16
            out = torch.empty(1, S, hq, d, dtype=odt, device=q.device)
        a, b = self.rows
        if self.world > 1:
            # rows outside this rank's block: rotated and appended here (the block's own rows are
            # appended again, to the same bits, by the fused call below)
            kr = k_new.contiguous().clone()
            if spec.rope_mode != 2:  # ROPE_NONE
                ops.apply_rope_full(kr.view(S, hkv * d), P, hkv, d, spec.rope_theta, spec.rope_mode)
            cache.add(layer, kr, v_new.contiguous())
        if b > a:
            view = _CacheAt(cache, P + a, q.device)
            ops.attention_layer(q[:, a:b].contiguous(), k_new[:, a:b].contiguous(), v_new[:, a:b].contiguous(), view,
                                layer=layer, out=out[:, a:b])
        if self.world > 1:
            for k in range(self.world):
                a_k, b_k = self.boundary(k), self.boundary(k + 1)
                if b_k > a_k:
                    dist.broadcast(out[0, a_k:b_k], src=k, group=group)
        return out


class _CacheAt:
    """A KVCache seen as holding `start` rows: the fused call for one rank's query block."""

    _starts: dict = {}

    def __init__(self, cache, start: int, device):
        self.spec, self.k, self.v = cache.spec, cache.k, cache.v
        key = (str(device), start)
        if key not in _CacheAt._starts:
            _CacheAt._starts[key] = torch.full((1,), start, dtype=torch.int32, device=device)
        self.seq_len = _CacheAt._starts[key]
        self.host_len = [start]


@dataclasses.dataclass
class ContextShard:
    """Rank `rank` of `world`'s share of a decode step split by cache rows (context parallelism),
    for layers with fewer KV heads than ranks (e.g. 4 KV heads on 8 GPUs: each head group's rows
    over 2 ranks). Rank r holds rows [r*L/N, (r+1)*L/N) of every sequence's cache in its own local
    cache (local row i = global row r*L/N + i); the last rank also appends the new token. Each rank
    attends its rows (aihost_attn_decode_partial: q rotated at the global position), the ranks
    all-gather (out, lse), and aihost_attn_merge_partials combines them."""

    rank: int
    world: int

    def chunk(self, length: int, k: int | None = None) -> tuple[int, int]:
        """Global rows [lo, hi) of a sequence of `length` cached rows held by rank k (default: this rank)."""
        k = self.rank if k is None else k
        return length * k // self.world, length * (k + 1) // self.world

    @property
    def appends(self) -> bool:
        return self.rank == self.world - 1

    def partial(self, ops, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, cache, q_pos: torch.Tensor,
                layer: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
        """This rank's part of one decode step: q [B, 1, Hq, d], k_new / v_new [B, 1, Hkv, d];
        `cache` holds this rank's rows (device and host lengths = local rows, each >= 1); q_pos
        (device int32 [B]) = each sequence's cached rows over all ranks, the new token's position.
        The last rank appends the new rows in the same call (K rotated at q_pos). Returns
        (out [B, Hq, d] normalised over this rank's rows, lse [B, Hq]). Cache lengths are not
        advanced."""
        spec = cache.spec
        B, d = q.shape[0], q.shape[3]
        if self.appends and any(n + 1 > spec.kv_capacity for n in cache.host_len):
            raise ValueError("KV cache capacity exceeded")
        kn = k_new.reshape(B, k_new.shape[2], d) if self.appends else None
        vn = v_new.reshape(B, v_new.shape[2], d) if self.appends else None
        return ops.decode_partial(spec, q.reshape(B, spec.n_q_heads, d), cache.k[layer], cache.v[layer],
                                  cache.seq_len, q_pos, k_new=kn, v_new=vn)

    def forward(self, ops, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, cache, q_pos: torch.Tensor,
                layer: int = 0, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
        """One decode step (arguments as `partial`): every rank's part, all-gathered over `group`
        and merged. Returns the full output [B, Hq, d] on every rank."""
        import torch.distributed as dist

        o, lse = self.partial(ops, q, k_new, v_new, cache, q_pos, layer)
        if self.world == 1:
            o_all, lse_all = o.unsqueeze(0), lse.unsqueeze(0)
        else:
            o_all = torch.empty((self.world,) + tuple(o.shape), dtype=o.dtype, device=o.device)
            lse_all = torch.empty((self.world,) + tuple(lse.shape), dtype=lse.dtype, device=lse.device)
            dist.all_gather_into_tensor(o_all.view(-1), o.view(-1), group=group)
            dist.all_gather_into_tensor(lse_all.view(-1), lse.view(-1), group=group)
        return ops.merge_partials(o_all, lse_all, out=out)


class NcclDist:
    """aihost_attn_dist: the library's NCCL communicator for one rank (one process per GPU).
    Set-up waits at most `timeout_ms` for the other ranks (AttnError ETIMEOUT otherwise)."""

    def __init__(self, world: int, rank: int, nccl_id: bytes, device: int, timeout_ms: int = 300000):
        import ctypes

        from . import check, lib

        if len(nccl_id) != 128:
            raise ValueError("an NCCL unique id is 128 bytes")
        self._id = ctypes.create_string_buffer(nccl_id, 128)
        self._h = ctypes.c_void_p()
        check(lib().aihost_attn_dist_init_bounded(world, rank, self._id, device, int(timeout_ms),
                                                  ctypes.byref(self._h)))
        self.world, self.rank = world, rank

    @staticmethod
    def unique_id() -> bytes:
        """A fresh NCCL id (made by one rank and handed to the others by the host)."""
        import ctypes

        from . import check, lib

        buf = ctypes.create_string_buffer(128)
        check(lib().aihost_attn_dist_unique_id(buf))
        return buf.raw

    @property
    def handle(self):
        return self._h

    def sync(self, stream=None, timeout_ms: int = 60000) -> None:
        """Wait at most timeout_ms for the stream's kernels and collectives (aborts the
        communicator and raises AttnError ETIMEOUT / ENCCL when they do not finish)."""
        from . import check, lib
        from .ops import _stream

        check(lib().aihost_attn_dist_sync(self._h, _stream(stream), int(timeout_ms)))

    def close(self) -> None:
        from . import lib

        if self._h:
            lib().aihost_attn_dist_destroy(self._h)
            self._h = None


__all__ = ["HeadShard", "RowShard", "ContextShard", "NcclDist"]
