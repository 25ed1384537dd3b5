"""Weight-layout helpers of the tile-GEMM formats (host side, numpy or torch).

The tile layout (micro_kernel/session_vm.nim:384-387, backends/cpu/cpu_vm.c:612-617): row n of
W takes K/2 bytes; the 16 bytes of 32-value block g start at byte 16g; byte j of a block holds
element 32g + j in its low nibble and element 32g + 16 + j in its high nibble.  Q4B32 stores the
signed int4 value q in [-8, 7] as its two's-complement nibble and one IEEE-half scale per block,
[N, K/32] row-major.
"""
from __future__ import annotations

import numpy as np


def pack_q4b32(q):
    """Signed int4 values [N, K] (numpy int8 or torch int8, any device) -> nibble bytes
    [N, K/2] in the tile layout."""
    N, K = q.shape
    if K % 32:
        raise ValueError(f"unsupported tile GEMM shape K={K} N={N}")
    if isinstance(q, np.ndarray):
        u = (q.astype(np.int16) & 15).astype(np.uint8).reshape(N, K // 32, 2, 16)
        return (u[:, :, 0, :] | (u[:, :, 1, :] << 4)).reshape(N, K // 2)
    import torch
    u = (q.to(torch.int16) & 15).to(torch.uint8).reshape(N, K // 32, 2, 16)
    return (u[:, :, 0, :] | (u[:, :, 1, :] << 4)).reshape(N, K // 2)


def unpack_q4b32(nibbles):
    """Nibble bytes [N, K/2] in the tile layout -> signed int4 values [N, K] (int8)."""
    N, half = nibbles.shape
    K = half * 2
    if isinstance(nibbles, np.ndarray):
        b = nibbles.reshape(N, K // 32, 16)
        lo = (b & 15).astype(np.int8)
        hi = (b >> 4).astype(np.int8)
        u = np.stack([lo, hi], axis=2).reshape(N, K)
        return np.where(u >= 8, u - 16, u).astype(np.int8)
    import torch
    b = nibbles.reshape(N, K // 32, 16)
    u = torch.stack([(b & 15), (b >> 4)], dim=2).reshape(N, K).to(torch.int8)
    return torch.where(u >= 8, u - 16, u)


def synthetic_q4b32(N: int, K: int, *, seed: int, device):
    """Seeded synthetic Q4B32 weights on `device`, with the benchmark configurations'
    distributions: q uniform over [-8, 7]; scales |N(0, 0.02)| rounded to fp16, an exact zero
    replaced by 2^-24.  Returns (nibbles uint8 [N, K/2], scales float16 [N, K/32])."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    nib = torch.randint(0, 256, (N, K // 2), generator=g, device=device, dtype=torch.int32).to(torch.uint8)
    s = (torch.randn(N, K // 32, generator=g, device=device, dtype=torch.float32).abs() * 0.02).to(torch.float16)
    s = torch.where(s == 0, torch.tensor(2.0 ** -24, dtype=torch.float16, device=device), s)
    return nib, s


def synthetic_x(M: int, K: int, *, seed: int, device, dtype=None):
    """Seeded N(0, 1) activations [M, K] (bf16 unless `dtype` is given)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.randn(M, K, generator=g, device=device, dtype=torch.float32)
    return x.to(dtype or torch.bfloat16)


def q4b32_weight_bytes(N: int, K: int) -> int:
    """Algorithmic bytes of Q4B32 weights: 0.5 B of nibble + 2/32 B of scale per weight."""
    return N * (K // 2) + N * (K // 32) * 2
