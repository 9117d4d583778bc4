"""Seeded synthetic inputs, identical on CPU and GPU.

Counter-based SplitMix64 (Steele, Lea & Flood, "Fast splittable pseudorandom number
generators", OOPSLA 2014) gives 53-bit uniforms; Box-Muller turns pairs into normals. Written
with torch integer ops so the same call produces the same bits on any device (int64 products
wrap modulo 2^64; right shifts are made logical with a mask). Normal variates go through
float64 transcendental functions whose last bit may differ between CPU and GPU libraries, so
tests generate on the CPU and copy to the device.
"""
from __future__ import annotations

import math

import torch

_M64 = (1 << 64) - 1


def _s64(x: int) -> int:
    x &= _M64
    return x - (1 << 64) if x >= (1 << 63) else x


_GAMMA = _s64(0x9E3779B97F4A7C15)
_MUL1 = _s64(0xBF58476D1CE4E5B9)
_MUL2 = _s64(0x94D049BB133111EB)


def _lsr(z: torch.Tensor, k: int) -> torch.Tensor:
    return (z >> k) & ((1 << (64 - k)) - 1)


def _mix(z: torch.Tensor) -> torch.Tensor:
    z = (z ^ _lsr(z, 30)) * _MUL1
    z = (z ^ _lsr(z, 27)) * _MUL2
    return z ^ _lsr(z, 31)


def _mix_int(x: int) -> int:
    z = (x + 0x9E3779B97F4A7C15) & _M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return z ^ (z >> 31)


def stream_key(seed: int, stream: str) -> int:
    """64-bit key of a named stream (each tensor gets its own)."""
    h = seed & _M64
    for ch in stream.encode():
        h = _mix_int(h ^ ch)
    return h


def uniform(n: int, seed: int, stream: str, device="cpu") -> torch.Tensor:
    """n float64 uniforms in [0, 1)."""
    base = _s64(stream_key(seed, stream))
    idx = torch.arange(1, n + 1, dtype=torch.int64, device=device)
    z = _mix(idx * _GAMMA + base)
    return _lsr(z, 11).to(torch.float64) * (1.0 / (1 << 53))


def normal(shape, seed: int, stream: str, mean: float = 0.0, std: float = 1.0, dtype=torch.float32,
           device="cpu") -> torch.Tensor:
    n = math.prod(shape)
    m = (n + 1) // 2
    u = uniform(2 * m, seed, stream, device)
    r = torch.sqrt(-2.0 * torch.log1p(-u[:m]))
    t = 2.0 * math.pi * u[m:]
    z = torch.cat([r * torch.cos(t), r * torch.sin(t)])[:n]
    return (z * std + mean).to(dtype).reshape(shape)


def randint(shape, lo: int, hi: int, seed: int, stream: str, device="cpu") -> torch.Tensor:
    """Integers uniform in [lo, hi] inclusive (int64)."""
    n = math.prod(shape)
    u = uniform(n, seed, stream, device)
    return (lo + torch.floor(u * (hi - lo + 1))).to(torch.int64).clamp_(lo, hi).reshape(shape)


def q8_0_blocks(n_blocks: int, seed: int, stream: str, scale_lo: float = 0.001, scale_hi: float = 0.02,
                device="cpu") -> torch.Tensor:
    """GGUF Q8_0 blocks (34 bytes: fp16 scale ~ U(lo, hi), 32 int8 ~ U{-127..127}) as uint8 [n_blocks*34]."""
    q = randint((n_blocks, 32), -127, 127, seed, stream + ".qs", device).to(torch.int8)
    d = (scale_lo + uniform(n_blocks, seed, stream + ".d", device) * (scale_hi - scale_lo)).to(torch.float16)
    out = torch.empty(n_blocks, 34, dtype=torch.uint8, device=device)
    out[:, :2] = d.view(torch.uint8).reshape(n_blocks, 2)
    out[:, 2:] = q.view(torch.uint8)
    return out.reshape(-1)


# GGUF K-quant block sizes (bytes per 256 values) and where each block keeps its fp16 super-scales
KQUANT_BLOCK_BYTES = {8: 84, 9: 110, 10: 144, 11: 176, 12: 210}
_KQUANT_F16 = {8: (80, 82), 9: (108,), 10: (0, 2), 11: (0, 2), 12: (208,)}


def kquant_blocks(kind: int, n_blocks: int, seed: int, stream: str, scale_lo: float = 0.001, scale_hi: float = 0.01,
                  device="cpu") -> torch.Tensor:
    """GGUF K-quant weight blocks (kind = AIHost DataType ordinal, Q2_K 8 .. Q6_K 12) as uint8
    [n_blocks * bytes]: every quant and sub-block scale byte uniform in [0, 255], the fp16
    super-scales (d, and dmin where the format has one) uniform in [scale_lo, scale_hi]."""
    nb = KQUANT_BLOCK_BYTES[kind]
    out = randint((n_blocks, nb), 0, 255, seed, stream + ".bytes", device).to(torch.uint8)
    for i, off in enumerate(_KQUANT_F16[kind]):
        d = (scale_lo + uniform(n_blocks, seed, f"{stream}.d{i}", device) * (scale_hi - scale_lo)).to(torch.float16)
        out[:, off:off + 2] = d.view(torch.uint8).reshape(n_blocks, 2)
    return out.reshape(-1)


__all__ = ["uniform", "normal", "randint", "q8_0_blocks", "kquant_blocks", "KQUANT_BLOCK_BYTES", "stream_key"]
