"""Seeded synthetic inputs for the quantized-matmul workloads.

The reference's benchmark configurations use fp32 weights drawn N(0, 0.02)
and activations drawn N(0, 1) from a seed.  This module defines the
generator exactly, so every run and every test sees the same numbers:

* a splitmix64 stream (Steele, Lea, Flood 2014) seeded with ``seed``;
  draw i is splitmix64 applied to ``seed + (i + 1) * 0x9E3779B97F4A7C15``;
* two consecutive draws -> two doubles in (0, 1] from their top 53 bits;
* Box-Muller in float64, rounded once to float32 at the end.

It is plain numpy (vectorised uint64 arithmetic), so generation of a
hundred-million-element matrix takes a few seconds.
"""
from __future__ import annotations

import numpy as np

_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _splitmix64(idx: np.ndarray, seed: int) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = np.uint64(seed & 0xFFFFFFFFFFFFFFFF) + (idx + np.uint64(1)) * _GOLDEN
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
        return z ^ (z >> np.uint64(31))


def normal(shape, seed: int, std: float = 1.0, chunk: int = 1 << 24) -> np.ndarray:
    """float32 array of the given shape, N(0, std^2), deterministic in seed."""
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.float32)
    npairs = (n + 1) // 2
    for p0 in range(0, npairs, chunk):
        p1 = min(npairs, p0 + chunk)
        k = np.arange(p0, p1, dtype=np.uint64)
        a = _splitmix64(k * np.uint64(2), seed)
        b = _splitmix64(k * np.uint64(2) + np.uint64(1), seed)
        u1 = ((a >> np.uint64(11)).astype(np.float64) + 1.0) * (1.0 / 9007199254740992.0)
        u2 = (b >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)
        r = np.sqrt(-2.0 * np.log(u1)) * std
        t = 2.0 * np.pi * u2
        z = np.empty(2 * (p1 - p0), dtype=np.float64)
        z[0::2] = r * np.cos(t)
        z[1::2] = r * np.sin(t)
        lo = 2 * p0
        hi = min(n, 2 * p1)
        out[lo:hi] = z[: hi - lo].astype(np.float32)
    return out.reshape(shape)


def _splitmix64_torch(idx, seed: int):
    """_splitmix64 on int64 torch tensors: two's-complement wrap-around is
    the uint64 arithmetic; right shifts are made logical with a mask."""
    import torch
    g = torch.tensor(0x9E3779B97F4A7C15 - (1 << 64), dtype=torch.int64, device=idx.device)
    m1 = torch.tensor(0xBF58476D1CE4E5B9 - (1 << 64), dtype=torch.int64, device=idx.device)
    m2 = torch.tensor(0x94D049BB133111EB - (1 << 64), dtype=torch.int64, device=idx.device)
    s = seed & 0xFFFFFFFFFFFFFFFF
    s = s - (1 << 64) if s >= (1 << 63) else s

    def shr(z, k):
        return (z >> k) & ((1 << (64 - k)) - 1)

    z = (idx + 1) * g + s
    z = (z ^ shr(z, 30)) * m1
    z = (z ^ shr(z, 27)) * m2
    return z ^ shr(z, 31)


def normal_torch(shape, seed: int, std: float = 1.0, device="cpu", offset: int = 0,
                 chunk: int = 1 << 24):
    """normal() computed with torch on `device`: elements [offset, offset +
    prod(shape)) of the same stream (offset even), so a row range of a
    matrix is drawn without drawing the rows before it.  On the CPU it is
    bit-identical to normal(); on a GPU the float64 log/cos/sin may differ
    from the host's in the last bit of a float64, which rarely survives the
    final rounding to float32."""
    import torch
    if offset % 2:
        raise ValueError("offset must be even (values come in Box-Muller pairs)")
    n = 1
    for d in shape:
        n *= int(d)
    out = torch.empty(n, dtype=torch.float32, device=device)
    npairs = (n + 1) // 2
    p_base = offset // 2
    mant = (1 << 53) - 1
    for p0 in range(0, npairs, chunk):
        p1 = min(npairs, p0 + chunk)
        k = torch.arange(p_base + p0, p_base + p1, dtype=torch.int64, device=device)
        a = _splitmix64_torch(k * 2, seed)
        b = _splitmix64_torch(k * 2 + 1, seed)
        u1 = (((a >> 11) & mant).to(torch.float64) + 1.0) * (1.0 / 9007199254740992.0)
        u2 = ((b >> 11) & mant).to(torch.float64) * (1.0 / 9007199254740992.0)
        r = torch.sqrt(-2.0 * torch.log(u1)) * std
        t = 2.0 * np.pi * u2
        z = torch.stack((r * torch.cos(t), r * torch.sin(t)), dim=1).reshape(-1)
        lo = 2 * p0
        hi = min(n, 2 * p1)
        out[lo:hi] = z[: hi - lo].to(torch.float32)
    return out.reshape(tuple(shape))
