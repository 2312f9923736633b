"""Seeded synthetic inputs for the five benchmark configurations, and their algorithmic byte counts.

No public dataset is involved: every input is drawn from a seeded torch generator with the shapes, value
distributions and sizes the benchmark configurations state. Generation runs on the given device (fast on a
GPU); the same seed always gives the same tensors on the same device type.
"""
from __future__ import annotations

import dataclasses

import torch

SEED = 20261201


def _gen(device, seed):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


# ---- config 1: row-wise f32 sum ----
ROWSUM = dict(rows=8192, cols=8192)


def rowsum_input(rows=8192, cols=8192, seed=SEED, device="cuda"):
    return torch.randn(rows, cols, generator=_gen(device, seed), device=device, dtype=torch.float32)


def rowsum_bytes(rows=8192, cols=8192) -> int:
    return rows * cols * 4 + rows * 4


# ---- config 2: int32 scans ----
SCAN_N = 1 << 28


def scan_input(n=SCAN_N, seed=SEED + 2, device="cuda"):
    return torch.randint(0, 16, (n,), generator=_gen(device, seed), device=device, dtype=torch.int32)


def scan_bytes(n=SCAN_N) -> int:
    return 2 * n * 4


# ---- config 3: Zipf row gather ----
GATHER = dict(rows=1 << 20, dim=256, n=1 << 24, s=1.1)


def gather_inputs(rows=1 << 20, dim=256, n=1 << 24, s=1.1, seed=SEED + 3, device="cuda"):
    """table bf16 [rows, dim] = RNE(N(0, 0.02)); ids int32 [n] Zipf(s) over ranks 1..rows (inverse CDF),
    mapped through a seeded permutation of the rows."""
    g = _gen(device, seed)
    table = (torch.randn(rows, dim, generator=g, device=device, dtype=torch.float32) * 0.02).to(torch.bfloat16)
    ranks = torch.arange(1, rows + 1, device=device, dtype=torch.float64)
    cdf = torch.cumsum(ranks.pow(-s), 0)
    cdf /= cdf[-1].clone()
    u = torch.rand(n, generator=g, device=device, dtype=torch.float64)
    r = torch.searchsorted(cdf, u).clamp_(max=rows - 1)
    perm = torch.randperm(rows, generator=g, device=device)
    ids = perm[r].to(torch.int32)
    return table, ids


def zipf_ids(n: int, rows: int, s: float, seed: int, device="cuda") -> torch.Tensor:
    """int32 [n] Zipf(s) over ranks 1..rows (inverse CDF), mapped through a seeded permutation of the rows."""
    g = _gen(device, seed)
    ranks = torch.arange(1, rows + 1, device=device, dtype=torch.float64)
    cdf = torch.cumsum(ranks.pow(-s), 0)
    cdf /= cdf[-1].clone()
    u = torch.rand(n, generator=g, device=device, dtype=torch.float64)
    r = torch.searchsorted(cdf, u).clamp_(max=rows - 1)
    return torch.randperm(rows, generator=g, device=device)[r].to(torch.int32)


def gather_bytes(ids: torch.Tensor, dim=256, elem=2):
    """(compulsory, logical) bytes: ids + output + each distinct table row once; logical reads every row."""
    n = ids.numel()
    row = dim * elem
    uniq = int(torch.unique(ids).numel())
    return 4 * n + row * n + uniq * row, 4 * n + 2 * row * n, uniq


# ---- config 4: max + argmax ----
ARGMAX = dict(rows=32768, cols=32000)


def argmax_input(rows=32768, cols=32000, seed=SEED + 4, device="cuda"):
    """bf16 = RNE(N(0,1) + u_r), u_r ~ U[-5, 5] per row."""
    g = _gen(device, seed)
    x = torch.randn(rows, cols, generator=g, device=device, dtype=torch.float32)
    off = torch.rand(rows, 1, generator=g, device=device, dtype=torch.float32) * 10.0 - 5.0
    x += off
    return x.to(torch.bfloat16)


def argmax_bytes(rows=32768, cols=32000) -> int:
    return rows * cols * 2 + rows * (4 + 4)


# ---- config 5: int4 group dequant + W4A16 ----
W4A16 = dict(n=28672, k=8192, m=16, group=128)


@dataclasses.dataclass
class W4A16Inputs:
    w_packed: torch.Tensor  # uint8 [n, k/2], low nibble = even k
    scale: torch.Tensor     # float16 [n, k/group]
    x: torch.Tensor         # bfloat16 [m, k]
    n: int
    k: int
    m: int
    group: int


def w4a16_inputs(n=28672, k=8192, m=16, group=128, seed=SEED + 5, device="cuda") -> W4A16Inputs:
    """W int4 uniform [-8, 7] packed two per byte; scale f16 ~ U(0.005, 0.02); x bf16 ~ N(0, 1)."""
    g = _gen(device, seed)
    w = torch.randint(-8, 8, (n, k), generator=g, device=device, dtype=torch.int32)
    packed = ((w[:, 0::2] & 0xF) | ((w[:, 1::2] & 0xF) << 4)).to(torch.uint8)
    scale = (torch.rand(n, k // group, generator=g, device=device, dtype=torch.float32) * 0.015 + 0.005).to(
        torch.float16)
    x = torch.randn(m, k, generator=g, device=device, dtype=torch.float32).to(torch.bfloat16)
    return W4A16Inputs(packed, scale, x, n, k, m, group)


def w4a16_bytes(n=28672, k=8192, m=16, group=128) -> int:
    return n * k // 2 + n * (k // group) * 2 + m * k * 2 + m * n * 2


def w4a16_flops(n=28672, k=8192, m=16) -> int:
    return 2 * m * n * k


def dequant_bytes(n=28672, k=8192, group=128) -> int:
    return n * k // 2 + n * (k // group) * 2 + n * k * 2
