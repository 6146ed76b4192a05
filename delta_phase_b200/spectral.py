"""Spectral bases of the Lerp FFN (drop-in for ``delta_phase.spectral``).

The matrices are the FFN's registered buffers, so they are built with the reference's
exact values (float32) to keep ``state_dict`` interchangeable; the forward pass itself
never multiplies by them densely except for the DCT-II (the FWHT and the Haar recursion
run as fast transforms in the CUDA library).

Reference: delta_phase/spectral.py:4-35 (mcarbonell/delta-phase v1.3.0).
"""
from __future__ import annotations

import math

import torch


def create_hadamard_matrix(n: int) -> torch.Tensor:
    """Sylvester Hadamard matrix / sqrt(n) (spectral.py:4-12).  As in the reference, a
    non-power-of-two n yields the next power-of-two size, scaled by 1/sqrt(n)."""
    size = 1
    while size < n:
        size *= 2
    idx = torch.arange(size)
    bits = idx[:, None] & idx[None, :]
    parity = torch.zeros_like(bits)
    while bool(bits.any()):
        parity ^= bits & 1
        bits = bits >> 1
    H = (1 - 2 * parity).to(torch.float32)
    return H / math.sqrt(n)


def create_dct2_matrix(n: int) -> torch.Tensor:
    """Orthonormal DCT-II matrix, row k = frequency (spectral.py:14-23)."""
    k = torch.arange(n, dtype=torch.float64)[:, None]
    i = torch.arange(n, dtype=torch.float64)[None, :]
    C = math.sqrt(2.0 / n) * torch.cos(math.pi * k * (2 * i + 1) / (2.0 * n))
    C[0, :] = 1.0 / math.sqrt(n)
    return C.to(torch.float32)


def create_haar_matrix(n: int) -> torch.Tensor:
    """The reference's recursive "Haar" matrix (spectral.py:25-35): low rows
    [H_{n/2}, H_{n/2}] / sqrt(2), high row i = (e_{2i} - e_{2i+1}) / sqrt(2).  Not
    orthogonal; n must be a power of two (the reference raises otherwise)."""
    if n == 1:
        return torch.ones(1, 1, dtype=torch.float32)
    if n % 2:
        raise RuntimeError("Sizes of tensors must match: Haar matrix needs a power-of-two size")
    sub = create_haar_matrix(n // 2)
    low = torch.cat([sub, sub], dim=1) / math.sqrt(2)
    high = torch.zeros(n // 2, n, dtype=torch.float32)
    idx = torch.arange(n // 2)
    high[idx, 2 * idx] = 1.0 / math.sqrt(2)
    high[idx, 2 * idx + 1] = -1.0 / math.sqrt(2)
    return torch.cat([low, high], dim=0)
