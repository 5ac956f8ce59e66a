"""Counter-based synthetic inputs: every element is a function of (seed, tensor
tag, global element index) alone.

A shard therefore generates exactly its own slice of the global tensor: rows
[r0, r1) of an N-GPU job hold the same values whichever GPU, and however many
GPUs, produce them, and a CPU check can regenerate any slice.

    key     = splitmix64(seed * 0x9E3779B97F4A7C15 + tag)
    bits_i  = splitmix64(key ^ splitmix64(i))            (64-bit wraparound)
    normal  : u1, u2 from two such streams (i -> 2i, 2i + 1), 53-bit uniforms in
              (0, 1]; z = sqrt(-2 ln u1) cos(2 pi u2) in float64 (Box-Muller);
              value = bf16_rne(f32_rne(mean + std * z))
    ids     : bits_i mod vocab

The device path (torch, integer ops on int64 with explicit logical shifts, float64
transcendentals) and the host path (numpy uint64 / float64) compute the same
bits; the float64 logarithm and cosine of the two libraries agree far below the
bf16 rounding step (tests check the two paths bit for bit).
"""

from __future__ import annotations

import zlib
from typing import Sequence

import numpy as np

M64 = (1 << 64) - 1
GOLDEN = 0x9E3779B97F4A7C15
C1, C2 = 0xBF58476D1CE4E5B9, 0x94D049BB133111EB
CHUNK = 1 << 24


def tag_of(name: str) -> int:
    """Stable 32-bit tag of a tensor name."""
    return zlib.crc32(name.encode())


# --------------------------------------------------------------------- host
def _mix_np(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = z + np.uint64(GOLDEN)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(C1)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(C2)
        return z ^ (z >> np.uint64(31))


def _key(seed: int, tag: int) -> int:
    return int(_mix_np(np.array([(seed * GOLDEN + tag) & M64], np.uint64))[0])


def bits_np(seed: int, tag: int, start: int, n: int) -> np.ndarray:
    i = np.arange(start, start + n, dtype=np.uint64)
    return _mix_np(np.uint64(_key(seed, tag)) ^ _mix_np(i))


def _unit_np(b: np.ndarray) -> np.ndarray:
    return ((b >> np.uint64(11)).astype(np.float64) + 1.0) * (2.0 ** -53)


def normal_f32_np(seed: int, tag: int, start: int, n: int, std: float = 1.0, mean: float = 0.0) -> np.ndarray:
    b = bits_np(seed, tag, 2 * start, 2 * n)
    u1, u2 = _unit_np(b[0::2]), _unit_np(b[1::2])
    z = np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)
    return (mean + std * z).astype(np.float32)


def normal_bf16_np(seed: int, tag: int, start: int, n: int, std: float = 1.0, mean: float = 0.0) -> np.ndarray:
    """bf16 bit patterns (uint16) of elements [start, start + n)."""
    u = normal_f32_np(seed, tag, start, n, std, mean).view(np.uint32)
    u = u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    return (u >> np.uint32(16)).astype(np.uint16)


def ids_np(seed: int, tag: int, start: int, n: int, vocab: int) -> np.ndarray:
    return (bits_np(seed, tag, start, n) % np.uint64(vocab)).astype(np.uint32)


# ------------------------------------------------------------------- device
def _i64(c: int) -> int:
    """A 64-bit pattern as a signed int64 value."""
    return c - (1 << 64) if c >= 1 << 63 else c


def _shr(z, k: int):
    """Logical right shift of int64 tensors."""
    return (z >> k) & ((1 << (64 - k)) - 1)


def _mix_t(z):
    z = z + _i64(GOLDEN)
    z = (z ^ _shr(z, 30)) * _i64(C1)
    z = (z ^ _shr(z, 27)) * _i64(C2)
    return z ^ _shr(z, 31)


def _fill_chunks(out_flat, n: int, fn):
    for c0 in range(0, n, CHUNK):
        c1 = min(n, c0 + CHUNK)
        out_flat[c0:c1] = fn(c0, c1 - c0)


def normal_bf16(shape: Sequence[int], seed: int, tag: int, start: int = 0, std: float = 1.0, mean: float = 0.0,
                device=None):
    """torch bf16 tensor of `shape` holding elements [start, start + numel) of
    the (seed, tag) stream; equal bit for bit to normal_bf16_np."""
    import torch

    n = int(np.prod(shape)) if len(shape) else 1
    out = torch.empty(n, dtype=torch.bfloat16, device=device)

    def gen(c0, m):
        k = _key(seed, tag)
        i1 = torch.arange(m, dtype=torch.int64, device=device) * 2 + 2 * (start + c0)
        b1 = _mix_t(_mix_t(i1) ^ _i64(k))
        b2 = _mix_t(_mix_t(i1 + 1) ^ _i64(k))
        u1 = (_shr(b1, 11).to(torch.float64) + 1.0) * (2.0 ** -53)
        u2 = (_shr(b2, 11).to(torch.float64) + 1.0) * (2.0 ** -53)
        z = torch.sqrt(-2.0 * torch.log(u1)) * torch.cos(2.0 * np.pi * u2)
        return (mean + std * z).to(torch.float32).to(torch.bfloat16)

    _fill_chunks(out, n, gen)
    return out.view(*shape)


def ids(n: int, seed: int, tag: int, vocab: int, start: int = 0, device=None):
    """int32 token ids (bits mod vocab) of elements [start, start + n)."""
    import torch

    out = torch.empty(n, dtype=torch.int32, device=device)

    def gen(c0, m):
        k = _key(seed, tag)
        i = torch.arange(m, dtype=torch.int64, device=device) + (start + c0)
        b = _mix_t(_mix_t(i) ^ _i64(k))
        # unsigned 64-bit modulo from two non-negative halves: b = hi * 2^32 + lo
        hi, lo = _shr(b, 32), b & 0xFFFFFFFF
        return ((((hi % vocab) * ((1 << 32) % vocab)) % vocab + lo % vocab) % vocab).to(torch.int32)

    _fill_chunks(out, n, gen)
    return out
