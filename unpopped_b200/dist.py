"""Sharding the lifted kernel families over the GPUs of one node: one process per GPU, torch.distributed over
NCCL for the plumbing, NCCL only where the path has a real exchange step.

* row sum, max+argmax, gather, dequant: independent rows / output rows — each rank runs its shard, no
  collective on the data path (`gather_outputs` is an optional all-gather of the results, timed apart);
* scan: one exchange — each rank folds its shard (`reduce_i32`), the ranks all-gather the G shard totals
  (4 bytes each), and each rank scans its shard seeded with the fold of the lower ranks' totals (the higher
  ranks' for a reverse scan). Integer combines are exact and associative, so the concatenated shards equal
  the single-GPU scan of the concatenated array bit for bit;
* W4A16: the weight rows (N) are split; each rank computes its [M, N/G] slice and the slices are all-gathered
  into the [M, N] output.

The per-rank kernels come from `ops` (libunpopped_sm100.so). `Local` lets the CPU tests of this module run the
exchange logic on gloo ranks with a CPU stand-in for the kernels; the product path never substitutes them.
"""
from __future__ import annotations

import dataclasses
from typing import Callable

import torch
import torch.distributed as dist


@dataclasses.dataclass
class Local:
    """The per-rank kernels the sharded paths call."""
    reduce_i32: Callable  # (x, op) -> 1-element int32 tensor
    scan: Callable        # (x, op, exclusive, reverse, carry) -> tensor
    w4a16: Callable = None  # (w_packed, scale, x, group) -> [M, N_local] bf16


def cuda_local() -> Local:
    from . import ops

    return Local(
        reduce_i32=lambda x, op: ops.reduce_i32(x, op),
        scan=lambda x, op, ex, rev, carry: ops.scan(x, op, ex, rev, carry=carry),
        w4a16=lambda w, s, x, g: ops.w4a16(w, s, x, g),
    )


def _world(group):
    return dist.get_world_size(group), dist.get_rank(group)


def shard_carry(totals: torch.Tensor, rank: int, op: str, reverse: bool, local: Local) -> torch.Tensor:
    """The carry of shard `rank`: the fold of the totals of the shards before it in scan order."""
    part = totals[rank + 1:] if reverse else totals[:rank]
    return local.reduce_i32(part.contiguous(), op)


def sharded_scan(x_local: torch.Tensor, op: str = "sum", exclusive: bool = False, reverse: bool = False,
                 group=None, local: Local | None = None) -> torch.Tensor:
    """Scan of the array formed by concatenating every rank's 1-D int32 shard in rank order; returns this
    rank's shard of the result."""
    local = local or cuda_local()
    world, rank = _world(group)
    total = local.reduce_i32(x_local, op).reshape(1)
    totals = torch.empty(world, dtype=total.dtype, device=total.device)
    dist.all_gather_into_tensor(totals, total, group=group)
    carry = shard_carry(totals, rank, op, reverse, local)
    return local.scan(x_local, op, exclusive, reverse, carry)


def gather_outputs(y_local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather of equally sized row shards (dim 0) into the full result on every rank."""
    world, _ = _world(group)
    out = torch.empty((world * y_local.shape[0],) + tuple(y_local.shape[1:]), dtype=y_local.dtype,
                      device=y_local.device)
    dist.all_gather_into_tensor(out, y_local.contiguous(), group=group)
    return out


def row_slice(n_rows: int, world: int, rank: int) -> slice:
    """This rank's contiguous block of rows (the first n % world ranks take one more)."""
    base, extra = divmod(n_rows, world)
    lo = rank * base + min(rank, extra)
    return slice(lo, lo + base + (1 if rank < extra else 0))


def sharded_w4a16(w_local: torch.Tensor, scale_local: torch.Tensor, x: torch.Tensor, group_size: int,
                  group=None, local: Local | None = None) -> torch.Tensor:
    """W4A16 with the weight rows split evenly over the ranks; returns the full [M, N] output on every rank."""
    local = local or cuda_local()
    world, _ = _world(group)
    y = local.w4a16(w_local, scale_local, x, group_size)  # [M, N/G]
    m, nl = y.shape
    parts = torch.empty((world * m, nl), dtype=y.dtype, device=y.device)
    dist.all_gather_into_tensor(parts, y.contiguous(), group=group)
    return parts.reshape(world, m, nl).permute(1, 0, 2).reshape(m, world * nl)
