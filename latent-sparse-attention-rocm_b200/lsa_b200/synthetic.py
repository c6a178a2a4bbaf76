"""Seeded synthetic inputs of the benchmark configurations (no dataset is involved).

Keys carry a per-position low-rank drift so buckets are non-uniform:
k[t, h] = n[t, h] + amp * sum_r c_r(t) U_r, with a rank-8 Gaussian basis U ~ N(0,1)/sqrt(8)
per KV head, c_r(t) = sin(2 pi t / P_r + phi_r), P_r log-spaced over [256, T] and
phi_r ~ U(0, 2 pi); n, q and v are N(0, 1). Generated on the device with a seeded torch
generator, in fp32, then cast.
"""

from __future__ import annotations

import math

import torch


def drift_keys(T: int, Hkv: int, D: int, gen: torch.Generator, device, amp: float = 0.5, rank: int = 8,
               batch: int = 1) -> torch.Tensor:
    """[batch, T, Hkv, D] fp32 keys with the rank-8 drift."""
    U = torch.randn(batch, Hkv, rank, D, generator=gen, device=device) / math.sqrt(rank)
    periods = torch.logspace(math.log10(256), math.log10(max(T, 257)), rank, device=device)
    phase = torch.rand(batch, rank, generator=gen, device=device) * (2 * math.pi)
    t = torch.arange(T, device=device, dtype=torch.float32)[:, None]
    keys = torch.randn(batch, T, Hkv, D, generator=gen, device=device)
    for b in range(batch):
        c = torch.sin(2 * math.pi * t / periods[None, :] + phase[b][None, :])  # [T, rank]
        keys[b] += amp * torch.einsum("tr,hrd->thd", c, U[b])
    return keys


def qkv(T: int, Hq: int, Hkv: int, D: int, seed: int, device, dtype=torch.bfloat16, drift: bool = True,
        batch: int = 1):
    """(q, k, v) [batch, T, H, D] in ``dtype``."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    k = drift_keys(T, Hkv, D, gen, device, batch=batch) if drift else torch.randn(batch, T, Hkv, D, generator=gen,
                                                                                   device=device)
    q = torch.randn(batch, T, Hq, D, generator=gen, device=device)
    v = torch.randn(batch, T, Hkv, D, generator=gen, device=device)
    return q.to(dtype), k.to(dtype), v.to(dtype)
