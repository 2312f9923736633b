"""Sharding the lifted kernel families over the GPUs of one node: one process per GPU, and the exchange steps the
path has, run inside libunpopped_sm100 through its communicator (`up_comm`, `up_sm100_launch_multi`).

* row sum, max+argmax, gather, dequant: independent rows / output rows: each rank runs its shard, no collective on
  the data path (`gather_outputs` is an optional all-gather of the results, timed apart);
* scan, layout "contiguous": the global array is the shards in rank order. Each rank folds its shard, the ranks
  all-gather the G shard totals (NCCL, 4 bytes each), and each scans its shard seeded with the fold of the lower
  ranks' totals (the higher ranks' for a reverse scan). Two passes over the data;
* scan, layout "block_cyclic": the global array is a sequence of stripes of 148 x 8192 elements dealt round-robin
  over the ranks (stripe s on rank s % G). One pass: the scan kernel's look-back adds the stripe aggregates the
  other ranks store into this rank's memory over NVLink. Integer combines are exact and associative, so either
  layout equals the single-GPU scan of the global array bit for bit;
* W4A16: the weight rows (N) are split; each rank computes its [M, N/G] slice and the slices are all-gathered
  (NCCL) into the [M, N] output on every rank.

`Comm` joins the ranks of a torch.distributed process group (which only carries the NCCL unique id) into a C-ABI
communicator, so the path a Rust host takes through the FFI is the one measured here. `Local` lets the CPU tests run
the exchange logic on gloo ranks with a CPU stand-in for the kernels; the product path never substitutes them.
"""
from __future__ import annotations

import ctypes
import dataclasses
from typing import Callable

import torch
import torch.distributed as dist

STRIPE_ELEMS = 148 * 8192  # the block-cyclic layout's stripe: one 8192-element tile per CTA of the scan's grid
LAYOUTS = {"contiguous": 0, "block_cyclic": 1}


@dataclasses.dataclass
class Local:
    """The per-rank kernels of the CPU stand-in path."""
    reduce_i32: Callable  # (x, op) -> 1-element int32 tensor
    scan: Callable        # (x, op, exclusive, reverse, carry) -> tensor
    w4a16: Callable = None  # (w_packed, scale, x, group) -> [M, N_local] bf16


def _world(group):
    return dist.get_world_size(group), dist.get_rank(group)


class Comm:
    """A communicator of libunpopped_sm100 over the ranks of `group`, one GPU per rank (the current device)."""

    def __init__(self, group=None):
        from . import _lib

        self._lib = _lib
        L = _lib.load()
        self.world, self.rank = _world(group)
        uid = (ctypes.c_ubyte * 128)()
        if self.rank == 0:
            _lib.check(L.up_sm100_comm_unique_id(uid), "comm_unique_id")
        box = [bytes(uid)]
        dist.broadcast_object_list(box, src=0, group=group)
        uid = (ctypes.c_ubyte * 128).from_buffer_copy(box[0])
        self.ptr = ctypes.c_void_p()
        _lib.check(L.up_sm100_comm_init_rank(self.world, self.rank, uid, ctypes.byref(self.ptr)), "comm_init_rank")
        self._ws = {}

    def close(self):
        if self.ptr:
            self._ws.clear()
            self._lib.check(self._lib.load().up_sm100_comm_destroy(self.ptr), "comm_destroy")
            self.ptr = ctypes.c_void_p()

    def workspace(self, kernel_id, ins, outs, scalars, device) -> torch.Tensor:
        """A zero-filled workspace for this call's shape, kept per kernel and grown on demand (the kernels leave it
        ready for the next call)."""
        from ._lib import UpTensor

        L = self._lib.load()
        cin = (UpTensor * len(ins))(*ins)
        cout = (UpTensor * len(outs))(*outs)
        sc = (ctypes.c_int64 * max(1, len(scalars)))(*scalars)
        n = ctypes.c_size_t(0)
        self._lib.check(L.up_sm100_workspace_bytes_multi(kernel_id, cin, len(ins), cout, len(outs), sc, len(scalars),
                                                         self.ptr, ctypes.byref(n)), "workspace_bytes_multi")
        ws = self._ws.get(kernel_id)
        if ws is None or ws.numel() < max(1, n.value):
            ws = torch.zeros(max(1, n.value), dtype=torch.uint8, device=device)
            self._ws[kernel_id] = ws
        return ws

    def launch(self, kernel_id: int, ins: list, outs: list, scalars: list, device) -> torch.Tensor:
        """up_sm100_launch_multi on `UpTensor` descriptors; returns the workspace it used."""
        from ._lib import UpTensor

        L = self._lib.load()
        ws = self.workspace(kernel_id, ins, outs, scalars, device)
        cin = (UpTensor * len(ins))(*ins)
        cout = (UpTensor * len(outs))(*outs)
        sc = (ctypes.c_int64 * max(1, len(scalars)))(*scalars)
        stream = torch.cuda.current_stream(device).cuda_stream
        self._lib.check(L.up_sm100_launch_multi(kernel_id, cin, len(ins), cout, len(outs), sc, len(scalars),
                                                ws.data_ptr(), ws.numel(), stream, self.ptr), "launch_multi")
        return ws


def _desc(t: torch.Tensor, ek: str, shape=None):
    from .backend import Operand

    shape = tuple(t.shape) if shape is None else tuple(shape)
    return Operand(ek, shape, ptr=t.data_ptr()).to_c()


def block_cyclic_index(n_local: int, world: int, rank: int | None = None, device="cpu") -> torch.Tensor:
    """The global positions of a rank's n_local elements under the block-cyclic layout (int64 [n_local]), or of
    every rank's ([world, n_local]) when `rank` is None. Local stripe k of rank r is global stripe k * world + r;
    every stripe of a round has the same size (full, or the shards' common remainder in the last round), so it starts
    at k * world * S + r * size_k."""
    pos = torch.arange(n_local, dtype=torch.int64, device=device)
    k, off = pos // STRIPE_ELEMS, pos % STRIPE_ELEMS
    last = (n_local - 1) // STRIPE_ELEMS if n_local > 0 else 0
    size_k = torch.where(k == last, torch.full_like(k, n_local - last * STRIPE_ELEMS), torch.full_like(k, STRIPE_ELEMS))
    if rank is not None:
        return k * world * STRIPE_ELEMS + rank * size_k + off
    return torch.stack([k * world * STRIPE_ELEMS + r * size_k + off for r in range(world)])


def shard_carry(totals: torch.Tensor, rank: int, op: str, reverse: bool, local: Local) -> torch.Tensor:
    """The carry of shard `rank`: the fold of the totals of the shards before it in scan order."""
    part = totals[rank + 1:] if reverse else totals[:rank]
    return local.reduce_i32(part.contiguous(), op)


def _cpu_block_cyclic(x_local, op, exclusive, world, rank, group, local):
    """The block-cyclic layout's semantics with the CPU stand-in: stripe totals all-gathered, each local stripe
    scanned with the fold of every global stripe before it."""
    n = x_local.numel()
    ns = (n + STRIPE_ELEMS - 1) // STRIPE_ELEMS
    stripes = [x_local[k * STRIPE_ELEMS:(k + 1) * STRIPE_ELEMS] for k in range(ns)]
    mine = torch.stack([local.reduce_i32(s.contiguous(), op).reshape(()) for s in stripes])
    allt = torch.empty(world * ns, dtype=torch.int32)
    dist.all_gather_into_tensor(allt, mine, group=group)
    allt = allt.reshape(world, ns).t().reshape(-1)  # global stripe order: stripe k * world + r
    outs = []
    for k, s in enumerate(stripes):
        carry = local.reduce_i32(allt[:k * world + rank].contiguous(), op)
        outs.append(local.scan(s.contiguous(), op, exclusive, False, carry))
    return torch.cat(outs)


def sharded_scan(x_local: torch.Tensor, op: str = "sum", exclusive: bool = False, reverse: bool = False,
                 group=None, local: Local | None = None, comm: Comm | None = None,
                 layout: str = "contiguous", out: torch.Tensor | None = None) -> torch.Tensor:
    """This rank's shard of the scan of the global array the ranks' 1-D int32 shards form under `layout`
    ("contiguous": shards in rank order; "block_cyclic": 148 x 8192-element stripes dealt round-robin)."""
    world, rank = _world(group)
    if local is not None:  # the CPU stand-in path
        if layout == "block_cyclic":
            if reverse:
                raise ValueError("the block-cyclic scan runs forward")
            return _cpu_block_cyclic(x_local, op, exclusive, world, rank, group, local)
        total = local.reduce_i32(x_local, op).reshape(1)
        totals = torch.empty(world, dtype=total.dtype, device=total.device)
        dist.all_gather_into_tensor(totals, total, group=group)
        carry = shard_carry(totals, rank, op, reverse, local)
        return local.scan(x_local, op, exclusive, reverse, carry)
    from ._lib import KERNEL, OP

    comm = comm or Comm(group)
    if out is None:
        out = torch.empty_like(x_local)
    comm.launch(KERNEL["SCAN_I32"], [_desc(x_local, "I32")], [_desc(out, "I32")],
                [OP[op.upper()], int(exclusive), int(reverse), LAYOUTS[layout]], x_local.device)
    return out


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
                  group=None, local: Local | None = None, comm: Comm | None = None) -> torch.Tensor:
    """W4A16 with the weight rows split evenly over the ranks; returns the full [M, N] output on every rank."""
    world, _ = _world(group)
    if local is not None:  # the CPU stand-in path
        y = local.w4a16(w_local, scale_local, x, group_size)  # [M, N/G]
        m, nl = y.shape
        parts = torch.empty((world * m, nl), dtype=y.dtype, device=y.device)
        dist.all_gather_into_tensor(parts, y.contiguous(), group=group)
        return parts.reshape(world, m, nl).permute(1, 0, 2).reshape(m, world * nl)
    from ._lib import KERNEL

    comm = comm or Comm(group)
    nl, kh = w_local.shape
    out = torch.empty(x.shape[0], world * nl, dtype=torch.bfloat16, device=x.device)
    comm.launch(KERNEL["W4A16_GEMM"],
                [_desc(w_local, "I4", (nl, 2 * kh)), _desc(scale_local, "F16"), _desc(x, "BF16")],
                [_desc(out, "BF16")], [group_size], x.device)
    return out


def sharded_rows(kernel: str, ins: list, outs: list, scalars: list, comm: Comm, device) -> None:
    """A row-parallel lift (ROW_SUM_F32, ROW_MAX_ARGMAX_BF16, GATHER_ROWS, DEQUANT_I4) on this rank's shard through
    up_sm100_launch_multi: no collective on the data path. `ins`/`outs` are (tensor, element kind) pairs."""
    from ._lib import KERNEL

    comm.launch(KERNEL[kernel], [_desc(t, ek) for t, ek in ins], [_desc(t, ek) for t, ek in outs], scalars, device)
