"""Reference-shaped operator surface over libaihost_attn.so.

Mirrors the C# calls the reference's transformer formats make for attention
(AIHost/AIHost/Compute/ComputeOps.cs and Inference/InferenceEngine.cs):

  ComputeOps.ApplyRoPEFull(tensor, startPosition, numHeads, headDim, theta)  -> apply_rope_full
  ComputeOps.MultiHeadAttention(Q, K, V, numHeads, startPosition)            -> multi_head_attention
  ComputeOps.FusedMHAGenerate(Q, K, V, numQHeads, numKvHeads, headDim, scale) -> fused_mha_generate
  KVCache.Add(layer, K, V) / KVCache.Get(layer) / KVCache.SequenceLength     -> KVCache
  TransformerLayer's RoPE(Q), RoPE(K), Add, Get, MultiHeadAttention sequence
  (ComputeOps.cs:1282-1304)                                                  -> attention_layer

Tensors are torch CUDA tensors used only as device memory; every computation runs in the
library's CUDA kernels. Argument errors surface as AttnError (the C# side throws
ArgumentException / CudaException for the same cases).
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from . import (F16, F32, Q8_0, ROPE_INTERLEAVED, ROPE_NONE, AttnDesc, AttnError, EINVAL, ENOMEM, check, lib)

_TORCH_CODES = {torch.float32: F32, torch.float16: F16}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _TORCH_CODES[t.dtype]
    except KeyError:
        raise AttnError(EINVAL, f"unsupported tensor dtype {t.dtype} (float32 or float16)") from None


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream) -> int | None:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def row_bytes(kv_dtype: int, head_dim: int) -> int:
    return {F32: 4 * head_dim, F16: 2 * head_dim, Q8_0: 34 * (head_dim // 32)}[kv_dtype]


@dataclass
class LayerSpec:
    """One attention layer's description (aihost_attn_desc)."""

    n_q_heads: int
    n_kv_heads: int
    head_dim: int
    rope_theta: float = 10000.0
    rope_mode: int = ROPE_INTERLEAVED
    scale: float = 0.0
    q_dtype: int = F16
    kv_dtype: int = F16
    out_dtype: int = F16
    kv_capacity: int = 1
    kv_seq_stride: int = 0
    kv_token_stride: int = 0
    kv_head_stride: int = 0

    def desc(self) -> AttnDesc:
        return AttnDesc(self.n_q_heads, self.n_kv_heads, self.head_dim, self.rope_theta, self.rope_mode, self.scale,
                        self.q_dtype, self.kv_dtype, self.out_dtype, self.kv_capacity, self.kv_seq_stride,
                        self.kv_token_stride, self.kv_head_stride)


class Context:
    """aihost_attn_ctx: device binding plus split-K scratch."""

    def __init__(self, device: int = 0):
        self._h = ctypes.c_void_p()
        check(lib().aihost_attn_create(int(device), ctypes.byref(self._h)))
        self.device = device

    @property
    def handle(self) -> ctypes.c_void_p:
        if not self._h:
            raise AttnError(EINVAL, "context is closed")
        return self._h

    def reserve_for(self, spec: LayerSpec, batch: int, n_new: int) -> None:
        need = ctypes.c_size_t()
        d = spec.desc()
        check(lib().aihost_attn_workspace_size(ctypes.byref(d), batch, n_new, ctypes.byref(need)))
        if need.value:
            check(lib().aihost_attn_reserve(self.handle, need.value))

    def sync_status(self) -> int:
        bits = ctypes.c_int32()
        check(lib().aihost_attn_sync_status(self.handle, ctypes.byref(bits)))
        return bits.value

    def profiler(self, enable: bool) -> None:
        """Bracket every kernel launch with CUDA events (device time per kernel kind)."""
        check(lib().aihost_attn_profiler_enable(self.handle, int(enable)))

    def profiler_read(self, kernel: int) -> tuple[int, float]:
        """(launches, total device ms) of one aihost_kernel kind since the last reset (synchronises)."""
        n, ms = ctypes.c_int64(), ctypes.c_double()
        check(lib().aihost_attn_profiler_read(self.handle, kernel, ctypes.byref(n), ctypes.byref(ms)))
        return n.value, ms.value

    def profiler_reset(self) -> None:
        check(lib().aihost_attn_profiler_reset(self.handle))

    def close(self) -> None:
        if self._h:
            lib().aihost_attn_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class KVCache:
    """Preallocated KV cache for `n_layers` layers and `batch` sequences.

    Layout per layer (the reference's token-major [rows, Hkv*d], InferenceEngine.cs:582-625):
    [batch][capacity][n_kv_heads][head_dim] in `kv_dtype` (Q8_0: GGUF blocks, stored as bytes).
    `add` copies new rows in place instead of the reference's Concat of old and new rows.
    """

    def __init__(self, ctx: Context, spec: LayerSpec, batch: int = 1, n_layers: int = 1, device=None):
        self.ctx, self.spec, self.batch = ctx, spec, batch
        dev = device if device is not None else torch.device("cuda", ctx.device)
        nbytes = batch * spec.kv_capacity * spec.n_kv_heads * row_bytes(spec.kv_dtype, spec.head_dim)
        self.k = [torch.zeros(nbytes, dtype=torch.uint8, device=dev) for _ in range(n_layers)]
        self.v = [torch.zeros(nbytes, dtype=torch.uint8, device=dev) for _ in range(n_layers)]
        self.seq_len = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.host_len = [0] * batch

    @property
    def sequence_length(self) -> int:
        """KVCache.SequenceLength of sequence 0."""
        return self.host_len[0]

    def add(self, layer: int, k: torch.Tensor, v: torch.Tensor, stream=None) -> None:
        """KVCache.Add: append k, v [batch, n_new, Hkv, d] (already rotated) after the cached rows."""
        n_new = k.shape[1]
        if any(n + n_new > self.spec.kv_capacity for n in self.host_len):
            raise AttnError(EINVAL, "KV cache capacity exceeded")
        spec = LayerSpec(**{**self.spec.__dict__, "q_dtype": dtype_code(k)})
        d = spec.desc()
        check(lib().aihost_kv_append(self.ctx.handle, ctypes.byref(d), self.batch, n_new, _ptr(k), _ptr(v),
                                      _ptr(self.k[layer]), _ptr(self.v[layer]), _ptr(self.seq_len), _stream(stream)))

    def advance(self, n_new: int) -> None:
        """Commit n_new appended rows for every sequence (after the last layer of a step)."""
        self.host_len = [n + n_new for n in self.host_len]
        self.seq_len += n_new

    def get(self, layer: int):
        """KVCache.Get: the raw K and V byte buffers of one layer."""
        return self.k[layer], self.v[layer]


class PagedKVCache:
    """Preallocated paged KV cache (fp32, fp16 or Q8_0): one pool of `n_pages` pages of `page_rows` rows per layer
    for K and one for V, shared by all sequences, and a block table mapping each sequence's row
    blocks to pages. Replaces KVCache.Add's per-token Concat (InferenceEngine.cs:598-622) with a
    page allocation every `page_rows` tokens; memory follows the sequences' actual lengths.

    `reserve(b, rows)` takes pages from the free list until sequence b can hold `rows` rows;
    `release(b)` returns its pages. Lengths advance as in KVCache (`advance`). Both update the
    device block table with a copy enqueued on `stream` (default: torch's current stream): pass
    the stream the attention calls run on, so the copy is ordered after the steps that read the
    old table and before the next one."""

    def __init__(self, ctx: Context, spec: LayerSpec, n_pages: int, page_rows: int = 128, batch: int = 1,
                 n_layers: int = 1, device=None):
        if spec.kv_dtype not in (F32, F16, Q8_0):
            raise AttnError(EINVAL, "unsupported kv_dtype for a paged cache")
        if page_rows < 128 or page_rows % 128:
            raise AttnError(EINVAL, "page_rows must be a positive multiple of 128")
        self.ctx, self.spec, self.batch, self.n_pages, self.page_rows = ctx, spec, batch, n_pages, page_rows
        self.max_pages = -(-spec.kv_capacity // page_rows)
        dev = device if device is not None else torch.device("cuda", ctx.device)
        nbytes = n_pages * page_rows * spec.n_kv_heads * row_bytes(spec.kv_dtype, spec.head_dim)
        self.k = [torch.zeros(nbytes, dtype=torch.uint8, device=dev) for _ in range(n_layers)]
        self.v = [torch.zeros(nbytes, dtype=torch.uint8, device=dev) for _ in range(n_layers)]
        self.table_host = torch.full((batch, self.max_pages), -1, dtype=torch.int32)
        self.block_table = self.table_host.to(dev)
        self.pages = [[] for _ in range(batch)]
        self.free = list(range(n_pages))
        self.seq_len = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.host_len = [0] * batch

    def _upload_table(self, stream) -> None:
        if self.block_table.device.type != "cuda":
            self.block_table.copy_(self.table_host)
            return
        with torch.cuda.stream(stream if stream is not None else torch.cuda.current_stream(self.block_table.device)):
            self.block_table.copy_(self.table_host)

    def reserve(self, b: int, rows: int, stream=None) -> None:
        if rows > self.spec.kv_capacity:
            raise AttnError(EINVAL, f"{rows} rows exceed kv_capacity {self.spec.kv_capacity}")
        need = -(-rows // self.page_rows)
        if need - len(self.pages[b]) > len(self.free):
            raise AttnError(ENOMEM, "the page pool is exhausted")
        if len(self.pages[b]) >= need:
            return
        while len(self.pages[b]) < need:
            pg = self.free.pop(0)
            self.table_host[b, len(self.pages[b])] = pg
            self.pages[b].append(pg)
        self._upload_table(stream)

    def release(self, b: int, stream=None) -> None:
        self.free.extend(self.pages[b])
        self.pages[b] = []
        self.table_host[b] = -1
        self._upload_table(stream)
        self.host_len[b] = 0
        self.seq_len[b] = 0

    def advance(self, n_new: int) -> None:
        self.host_len = [n + n_new for n in self.host_len]
        self.seq_len += n_new


class ComputeOps:
    """The attention subset of the reference's ComputeOps, executed by libaihost_attn."""

    def __init__(self, ctx: Context, stream=None):
        self.ctx, self.stream = ctx, stream

    def apply_rope_full(self, tensor: torch.Tensor, start_position: int, num_heads: int, head_dim: int,
                        theta: float = 10000.0, rope_mode: int = ROPE_INTERLEAVED) -> None:
        """ApplyRoPEFull (ComputeOps.cs:959-979): rotate tensor [seq, num_heads*head_dim] in place."""
        seq = tensor.shape[0]
        check(lib().aihost_rope_full(_ptr(tensor), dtype_code(tensor), seq, num_heads, head_dim, int(start_position),
                                     float(theta), rope_mode, _stream(self.stream)))

    def qk_norm_rope(self, tensor: torch.Tensor, weight: torch.Tensor, start_position: int, num_heads: int,
                     head_dim: int, theta: float = 10000.0, eps: float = 1e-5,
                     rope_mode: int = ROPE_INTERLEAVED) -> None:
        """Qwen TypeB prologue (QwenHybridFormat.cs:141-142) in place on tensor [seq, num_heads*head_dim]:
        LayerNorm over each whole row with weight [head_dim] (fp32) tiled over the heads, then RoPE."""
        seq = tensor.shape[0]
        check(lib().aihost_qk_norm_rope(_ptr(tensor), dtype_code(tensor), seq, num_heads, head_dim, _ptr(weight),
                                        float(eps), int(start_position), float(theta), rope_mode, _stream(self.stream)))

    def multi_head_attention(self, Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, num_heads: int,
                             start_position: int = 0, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        """MultiHeadAttention (ComputeOps.cs:1055-1102) over rotated Q [S, Hq*d], K/V [Lk, Hkv*d]."""
        seq, dq = Q.shape
        head_dim = dq // num_heads
        n_kv_heads = K.shape[1] // head_dim
        out_dtype = out_dtype or Q.dtype
        out = torch.empty(seq, dq, dtype=out_dtype, device=Q.device)
        spec = LayerSpec(num_heads, n_kv_heads, head_dim, rope_mode=ROPE_NONE, q_dtype=dtype_code(Q),
                         kv_dtype=dtype_code(K), out_dtype=dtype_code(out), kv_capacity=K.shape[0])
        self.ctx.reserve_for(spec, 1, seq)
        d = spec.desc()
        check(lib().aihost_attn_mha(self.ctx.handle, ctypes.byref(d), seq, K.shape[0], int(start_position), _ptr(Q),
                                    _ptr(K), _ptr(V), _ptr(out), _stream(self.stream)))
        return out

    def decode_partial(self, spec: LayerSpec, q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                       seq_len: torch.Tensor, q_pos: torch.Tensor | None = None, k_new: torch.Tensor | None = None,
                       v_new: torch.Tensor | None = None,
                       out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
        """One query row per sequence (q [B, Hq, d]) over this part's cache rows [0, seq_len[b]),
        plus the new rows k_new / v_new [B, Hkv, d] appended at row seq_len[b] (K rotated at
        q_pos[b]) when given; q rotated at q_pos[b] when given (spec.rope_mode), else used as is.
        Returns (out [B, Hq, d] normalised over these rows, lse [B, Hq] fp32 =
        ln sum_j exp(scale * q.k_j)). Cache lengths are not advanced."""
        B = q.shape[0]
        if out is None:
            odt = torch.float32 if spec.out_dtype == F32 else torch.float16
            out = torch.empty(B, spec.n_q_heads, spec.head_dim, dtype=odt, device=q.device)
        lse = torch.empty(B, spec.n_q_heads, dtype=torch.float32, device=q.device)
        self.ctx.reserve_for(spec, B, 1)
        d = spec.desc()
        check(lib().aihost_attn_decode_partial(self.ctx.handle, ctypes.byref(d), B, _ptr(q), _ptr(k_new),
                                               _ptr(v_new), _ptr(k_cache), _ptr(v_cache), _ptr(seq_len), _ptr(q_pos),
                                               _ptr(out), _ptr(lse), _stream(self.stream)))
        return out, lse

    def merge_partials(self, o_parts: torch.Tensor, lse_parts: torch.Tensor,
                       out: torch.Tensor | None = None) -> torch.Tensor:
        """Combine n partial results o_parts [n, ..., d] / lse_parts [n, ...] of the same query rows
        over disjoint key sets into the result over all of them."""
        n, d = o_parts.shape[0], o_parts.shape[-1]
        rows = o_parts[0].numel() // d
        if out is None:
            out = torch.empty(o_parts.shape[1:], dtype=o_parts.dtype, device=o_parts.device)
        check(lib().aihost_attn_merge_partials(self.ctx.handle, n, rows, d, dtype_code(o_parts), _ptr(o_parts),
                                               _ptr(lse_parts), _ptr(out), None, _stream(self.stream)))
        return out

    def fused_mha_generate(self, Q, K, V, num_q_heads: int, num_kv_heads: int, head_dim: int,
                           scale: float) -> torch.Tensor:
        """FusedMHAGenerate (ComputeOps.cs:1015-1043): one query row, every cached row visible."""
        out = torch.empty(1, num_q_heads * head_dim, dtype=Q.dtype, device=Q.device)
        spec = LayerSpec(num_q_heads, num_kv_heads, head_dim, rope_mode=ROPE_NONE, scale=scale, q_dtype=dtype_code(Q),
                         kv_dtype=dtype_code(K), out_dtype=dtype_code(out), kv_capacity=K.shape[0])
        self.ctx.reserve_for(spec, 1, 1)
        d = spec.desc()
        check(lib().aihost_attn_mha(self.ctx.handle, ctypes.byref(d), 1, K.shape[0], 0, _ptr(Q), _ptr(K), _ptr(V),
                                    _ptr(out), _stream(self.stream)))
        return out

    def attention_layer_paged(self, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, cache: PagedKVCache,
                              layer: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
        """attention_layer over a PagedKVCache: pages for the new rows are reserved first."""
        B, S = q.shape[0], q.shape[1]
        spec = cache.spec
        for b in range(B):
            cache.reserve(b, cache.host_len[b] + S, stream=self.stream)
        if out is None:
            odt = torch.float32 if spec.out_dtype == F32 else torch.float16
            out = torch.empty(B, S, spec.n_q_heads, spec.head_dim, dtype=odt, device=q.device)
        self.ctx.reserve_for(spec, B, S)
        d = spec.desc()
        hl = (ctypes.c_int32 * B)(*cache.host_len)
        check(lib().aihost_attn_forward_paged(self.ctx.handle, ctypes.byref(d), B, S, _ptr(q), _ptr(k_new), _ptr(v_new),
                                              _ptr(cache.k[layer]), _ptr(cache.v[layer]), cache.n_pages,
                                              cache.page_rows, _ptr(cache.block_table), cache.max_pages,
                                              _ptr(cache.seq_len), ctypes.cast(hl, ctypes.c_void_p), _ptr(out),
                                              _stream(self.stream)))
        return out

    def attention_layer(self, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, cache: KVCache,
                        layer: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
        """The fused layer step (ComputeOps.cs:1282-1304): RoPE(Q), RoPE(K), KVCache.Add, MultiHeadAttention.

        q [B, S, Hq, d], k_new / v_new [B, S, Hkv, d]. Rows are appended to `cache` for this layer;
        call cache.advance(S) once all layers of the step ran.
        """
        B, S = q.shape[0], q.shape[1]
        spec = cache.spec
        if out is None:
            odt = torch.float32 if spec.out_dtype == F32 else torch.float16
            out = torch.empty(B, S, spec.n_q_heads, spec.head_dim, dtype=odt, device=q.device)
        self.ctx.reserve_for(spec, B, S)
        d = spec.desc()
        # host copy of the lengths (sizes the grid); None -> the library plans from kv_capacity
        hl = (ctypes.c_int32 * B)(*cache.host_len) if cache.host_len is not None else None
        check(lib().aihost_attn_forward(self.ctx.handle, ctypes.byref(d), B, S, _ptr(q), _ptr(k_new), _ptr(v_new),
                                        _ptr(cache.k[layer]), _ptr(cache.v[layer]), _ptr(cache.seq_len),
                                        ctypes.cast(hl, ctypes.c_void_p) if hl is not None else None, _ptr(out),
                                        _stream(self.stream)))
        return out


class MatMulDesc(ctypes.Structure):
    """aihost_matmul_desc."""

    _fields_ = [("rows", ctypes.c_int32), ("k", ctypes.c_int32), ("n_out", ctypes.c_int32), ("n_parts", ctypes.c_int32),
                ("a_dtype", ctypes.c_int32), ("w_dtype", ctypes.c_int32), ("out_dtype", ctypes.c_int32)]


class WeightOps:
    """The weight products beside the attention op, executed by libaihost_attn:

      ComputeOps.MatMulWeights(a, w) (ComputeOps.cs:275-313)   -> mat_mul_weights
      ComputeOps.Dequantize / DequantizeInto (ComputeOps.cs:733-861) -> dequantize

    Weights are GGUF tensors as stored (column-major: n_out rows of k values; K-quant blocks
    as raw bytes in a uint8 tensor)."""

    def __init__(self, ctx: Context, stream=None):
        self.ctx, self.stream = ctx, stream

    def mat_mul_weights(self, a: torch.Tensor, w: torch.Tensor, w_dtype: int, n_out: int, n_parts: int = 1,
                        out_dtype: torch.dtype = torch.float16, out: torch.Tensor | None = None) -> torch.Tensor:
        """C [rows, n_out] = A . W. `a` is [rows, k] (n_parts = 1) or n_parts column blocks
        stored one after another, [n_parts, rows, k / n_parts] (e.g. the rank-major output of
        a KV-head-sharded attention call viewed as [N, B*S, Hq/N*d])."""
        if n_parts == 1:
            rows, k = a.shape[-2], a.shape[-1]
        else:
            rows, k = a.shape[1], a.shape[0] * a.shape[2]
        d = MatMulDesc(rows, k, n_out, n_parts, dtype_code(a), w_dtype, _TORCH_CODES[out_dtype])
        need = ctypes.c_size_t()
        check(lib().aihost_matmul_workspace_size(ctypes.byref(d), ctypes.byref(need)))
        if need.value:
            check(lib().aihost_attn_reserve(self.ctx.handle, need.value))
        if out is None:
            out = torch.empty(rows, n_out, dtype=out_dtype, device=a.device)
        check(lib().aihost_matmul_weights(self.ctx.handle, ctypes.byref(d), _ptr(a), _ptr(w), _ptr(out),
                                          _stream(self.stream)))
        return out

    def dequantize(self, w: torch.Tensor, w_dtype: int, n: int, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """K-quant blocks -> n values (DequantizeInto writes fp32; fp16 is that value rounded once)."""
        out = torch.empty(n, dtype=out_dtype, device=w.device)
        check(lib().aihost_dequantize(_ptr(w), w_dtype, n, _ptr(out), _TORCH_CODES[out_dtype], _stream(self.stream)))
        return out


def default_scale(head_dim: int) -> float:
    """1.0f / MathF.Sqrt(headDim) in fp32 (ComputeOps.cs:1065)."""
    import numpy as np

    return float(np.float32(1.0) / np.sqrt(np.float32(head_dim)))


__all__ = ["Context", "LayerSpec", "KVCache", "ComputeOps", "WeightOps", "MatMulDesc", "dtype_code", "row_bytes",
           "default_scale", "math"]
