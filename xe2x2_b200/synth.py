"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (no checkpoint or dataset is available offline).

GPTQ: codes uniform over 0..15 packed eight per int32 along K (checkpoint
layout), zeros uniform 0..15 packed along N (or none = symmetric),
scales fp16 = |N(0, 0.02)| + 1e-3 per (group, column), activations ~N(0, sigma).
NVFP4: codes uniform over the 16 E2M1 values, two per byte; E4M3 block scales
= e4m3(2^u), u ~ U[-6, 2]; fp32 tensor scale 1/448; activations bf16 ~N(0, 1).
Uniform random 32-bit words have uniform independent nibbles, so packed
tensors are drawn directly as random words / bytes.
"""
from __future__ import annotations

import torch


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def gptq_weights(K: int, N: int, group_size: int = 128, asym: bool = True, seed: int = 0,
                 device="cpu", act_order: bool = False):
    g = _gen(seed, device)
    qweight = torch.randint(-2**31, 2**31, (K // 8, N), dtype=torch.int64, generator=g, device=device).to(torch.int32)
    ngrp = K // group_size
    qzeros = None
    if asym:
        qzeros = torch.randint(-2**31, 2**31, (ngrp, N // 8), dtype=torch.int64, generator=g,
                               device=device).to(torch.int32)
    scales = (torch.randn((ngrp, N), generator=g, device=device) * 0.02).abs_().add_(1e-3).to(torch.float16)
    g_idx = None
    if act_order:
        perm = torch.randperm(K, generator=g, device=device)
        g_idx = torch.empty(K, dtype=torch.int32, device=device)
        g_idx[perm] = (torch.arange(K, device=device, dtype=torch.int32) // group_size)
    return qweight, qzeros, scales, g_idx


def activations(M: int, K: int, dtype=torch.bfloat16, sigma: float = 1.0, seed: int = 1, device="cpu"):
    g = _gen(seed, device)
    return (torch.randn((M, K), generator=g, device=device) * sigma).to(dtype)


def nvfp4_weights(K: int, N: int, seed: int = 0, device="cpu"):
    """-> (w u8 [K/2, N] stored K-contiguous (stride(0) == 1), block scales e4m3 [K/16, N], global f32[1])."""
    g = _gen(seed, device)
    w_nk = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, generator=g, device=device)
    u = torch.rand((K // 16, N), generator=g, device=device) * 8.0 - 6.0
    scale = torch.exp2(u).to(torch.float8_e4m3fn)
    gscale = torch.full((1,), 1.0 / 448.0, dtype=torch.float32, device=device)
    return w_nk.t(), scale, gscale


def gptq_s4_tile(rows: int, k: int, cols: int, seed: int = 0, device="cpu"):
    """Inputs of the reference s4-activation kernel: s4 A, s4 B (as int8), a_scale, f16 group scales."""
    g = _gen(seed, device)
    a = torch.randint(-8, 8, (rows, k), dtype=torch.int8, generator=g, device=device)
    b = torch.randint(-8, 8, (k, cols), dtype=torch.int8, generator=g, device=device)
    a_scale = torch.full((rows,), 0.02, dtype=torch.float32, device=device)
    s = ((torch.rand((k // 128, cols), generator=g, device=device) * 0.0074) + 0.0028).to(torch.float16)
    return a, b, a_scale, s
