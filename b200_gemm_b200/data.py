"""Seeded synthetic operands for the benchmark configurations.

The reference fills A and B with N(0,1) samples from
std::default_random_engine(69) converted float -> bf16 (round to nearest
even) on the host (include/utils.cuh:22-29).  Its generator stream is not
reproduced; what carries over is the distribution and the rounding.  The
configurations in use:
  "normal"   A, B ~ N(0, 1)
  "uniform"  A, B ~ U[-1, 1]
  "mlp"      A ~ N(0, 1) (activations), B ~ N(0, 0.02) (weights)
Host arrays come from numpy's PCG64 (identical on every machine); device
arrays from torch's CUDA generator.  bf16 values are carried as raw uint16
bit patterns on the host.
"""
from __future__ import annotations

import numpy as np

DISTS = ("normal", "uniform", "mlp")


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even (NaN kept quiet)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7F800000) == 0x7F800000
    nan &= (u & 0x007FFFFF) != 0
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def host_operands(M: int, N: int, K: int, dist: str = "normal", seed: int = 0):
    """(A_bits [M,K], B_bits [N,K]) as uint16 bf16 patterns."""
    if dist not in DISTS:
        raise ValueError(f"unknown distribution {dist!r}; expected one of {DISTS}")
    rng = np.random.Generator(np.random.PCG64(seed))
    if dist == "uniform":
        a = rng.uniform(-1.0, 1.0, size=(M, K)).astype(np.float32)
        b = rng.uniform(-1.0, 1.0, size=(N, K)).astype(np.float32)
    else:
        a = rng.standard_normal(size=(M, K), dtype=np.float32)
        b = rng.standard_normal(size=(N, K), dtype=np.float32)
        if dist == "mlp":
            b *= np.float32(0.02)
    return f32_to_bf16_bits(a), f32_to_bf16_bits(b)


def device_operands(M: int, N: int, K: int, dist: str = "normal", seed: int = 0, device="cuda"):
    """(A [M,K], B [N,K]) torch.bfloat16 tensors generated on the device."""
    import torch

    if dist not in DISTS:
        raise ValueError(f"unknown distribution {dist!r}; expected one of {DISTS}")
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    if dist == "uniform":
        a = torch.empty(M, K, device=device, dtype=torch.float32).uniform_(-1.0, 1.0, generator=g)
        b = torch.empty(N, K, device=device, dtype=torch.float32).uniform_(-1.0, 1.0, generator=g)
    else:
        a = torch.randn(M, K, device=device, dtype=torch.float32, generator=g)
        b = torch.randn(N, K, device=device, dtype=torch.float32, generator=g)
        if dist == "mlp":
            b.mul_(0.02)
    return a.to(torch.bfloat16), b.to(torch.bfloat16)
