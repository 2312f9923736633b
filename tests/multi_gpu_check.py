"""Multi-GPU parity of up_sm100_launch_multi, one process per GPU (run by tests/test_gpu_multi.py under torchrun).

Each rank builds the same seeded global inputs, takes its shard, runs the sharded lift through the C-ABI
communicator, and compares with the single-GPU kernel on the global array (itself held to the oracle by the other
GPU tests), bit for bit:
  * the scan over contiguous shards (inclusive / exclusive add, max, reverse) and over block-cyclic stripes
    (inclusive / exclusive add, max, min; a partial last stripe; the full 2^28-per-rank configuration);
  * the W4A16 GEMM with the weight rows split, against the single-GPU kernel on each slice;
  * the row-parallel lifts (row sum, max + argmax, gather) on their row shards;
  * failure detection: rank 1 withholds one look-back flag (a flag nothing sets) under a short wait limit; every
    rank's bounded waits run out, the error reaches the other rank through an "aborted" stripe word, both report
    UP_ERR_DEVICE_TIMEOUT, and the next launch is exact again. No fault, no hang;
  * a wrap of the communicator's 30-bit launch tag.
Rank 0 prints one JSON line with every check and exits non-zero if any failed.
"""
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    from unpopped_b200 import _lib, dist as udist, ops, workloads as wl

    L = _lib.load()
    comm = udist.Comm()
    checks = {}

    def gen(seed):  # the same stream on every rank (same device type, same seed)
        return torch.Generator(device=dev).manual_seed(seed)

    def agree(name, ok):
        t = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        checks[name] = bool(t.item())

    # ---- scan over contiguous shards ----
    n = (1 << 22) + 12
    full = torch.randint(-(2 ** 31), 2 ** 31 - 1, (world * n,), generator=gen(1), dtype=torch.int32, device=dev)
    mine = full[rank * n:(rank + 1) * n].contiguous()
    for op, ex, rev in (("sum", False, False), ("sum", True, False), ("max", False, False), ("sum", False, True),
                        ("min", True, True)):
        y = udist.sharded_scan(mine, op, ex, rev, comm=comm)
        want = ops.scan(full, op, ex, rev)[rank * n:(rank + 1) * n]
        agree(f"contiguous_{op}_{'excl' if ex else 'incl'}_{'rev' if rev else 'fwd'}", torch.equal(y, want))

    # ---- block-cyclic scan ----
    for n_local, seed in ((3 * udist.STRIPE_ELEMS + 8192 * 5 + 4, 2), (1 << 28, 3)):
        glob = torch.randint(0, 16, (world * n_local,), generator=gen(seed), dtype=torch.int32, device=dev)
        idx = udist.block_cyclic_index(n_local, world, rank, dev)
        x = glob[idx].contiguous()
        cases = (("sum", False), ("sum", True), ("max", False), ("min", True)) if n_local < (1 << 28) else \
            (("sum", False),)
        for op, ex in cases:
            y = udist.sharded_scan(x, op, ex, layout="block_cyclic", comm=comm)
            ws = comm._ws[_lib.KERNEL["SCAN_I32"]]
            st = L.up_sm100_workspace_status(ws.data_ptr(), torch.cuda.current_stream().cuda_stream)
            want = ops.scan(glob, op, ex)[idx]
            agree(f"block_cyclic_{n_local}_{op}_{'excl' if ex else 'incl'}", st == _lib.UP_OK and torch.equal(y, want))
        del glob, idx, x

    # ---- W4A16 with the weight rows split ----
    d = wl.w4a16_inputs(n=2048 * world, k=4096, m=16, device="cpu", seed=5)
    nl = 2048
    sl = slice(rank * nl, (rank + 1) * nl)
    out = udist.sharded_w4a16(d.w_packed[sl].contiguous().to(dev), d.scale[sl].contiguous().to(dev), d.x.to(dev), 128,
                              comm=comm)
    want = torch.cat([ops.w4a16(d.w_packed[g * nl:(g + 1) * nl].contiguous().to(dev),
                                d.scale[g * nl:(g + 1) * nl].contiguous().to(dev), d.x.to(dev), 128)
                      for g in range(world)], dim=1)
    agree("w4a16_split_rows", torch.equal(out.view(torch.int16), want.view(torch.int16)))

    # ---- row-parallel lifts on row shards ----
    xs = torch.randn(4096 * world, 8192, generator=gen(6), device=dev)[rank * 4096:(rank + 1) * 4096].contiguous()
    rs = torch.empty(4096, device=dev)
    udist.sharded_rows("ROW_SUM_F32", [(xs, "F32")], [(rs, "F32")], [1, 256], comm, dev)
    agree("row_sum_shard", torch.equal(rs.view(torch.int32), ops.row_sum(xs, "f32").view(torch.int32)))
    xb = wl.argmax_input(rows=2048, cols=32000, seed=7 + rank, device="cuda")
    mx = torch.empty(2048, device=dev)
    am = torch.empty(2048, dtype=torch.int32, device=dev)
    udist.sharded_rows("ROW_MAX_ARGMAX_BF16", [(xb, "BF16")], [(mx, "F32"), (am, "I32")], [], comm, dev)
    m2, a2 = ops.row_max_argmax(xb, torch.int32)
    agree("max_argmax_shard", torch.equal(mx.view(torch.int32), m2.view(torch.int32)) and torch.equal(am, a2))
    table, ids = wl.gather_inputs(rows=1 << 16, n=1 << 20, seed=8, device="cuda")
    ids = ids[rank * (1 << 19):(rank + 1) * (1 << 19)].contiguous()
    go = torch.empty(ids.numel(), 256, dtype=torch.bfloat16, device=dev)
    udist.sharded_rows("GATHER_ROWS", [(table, "BF16"), (ids, "I32")], [(go, "BF16")], [2], comm, dev)
    agree("gather_shard", torch.equal(go.view(torch.int16), ops.gather_rows(table, ids, "zero_fill").view(torch.int16)))

    # ---- failure detection across GPUs: a withheld flag, bounded waits, the error reported on every rank ----
    n_local = 2 * udist.STRIPE_ELEMS
    glob = torch.randint(0, 16, (world * n_local,), generator=gen(9), dtype=torch.int32, device=dev)
    idx = udist.block_cyclic_index(n_local, world, rank, dev)
    x = glob[idx].contiguous()
    udist.sharded_scan(x, "sum", layout="block_cyclic", comm=comm)  # the workspace for this shape exists
    ws = comm._ws[_lib.KERNEL["SCAN_I32"]]
    stream = torch.cuda.current_stream().cuda_stream
    L.up_sm100_workspace_status(ws.data_ptr(), stream)
    L.up_sm100_set_wait_limit_ns(20_000_000)
    try:
        if rank == 1:
            L.up_sm100_set_test_withhold_flag(1)
        torch.cuda.synchronize()
        dist.barrier()
        udist.sharded_scan(x, "sum", layout="block_cyclic", comm=comm)
        st = L.up_sm100_workspace_status(ws.data_ptr(), stream)
        agree("timeout_reported_on_every_rank", st == _lib.UP_ERR_DEVICE_TIMEOUT)
    finally:
        L.up_sm100_set_test_withhold_flag(0)
        L.up_sm100_set_wait_limit_ns(1_000_000_000)
    torch.cuda.synchronize()
    dist.barrier()
    y = udist.sharded_scan(x, "sum", layout="block_cyclic", comm=comm)
    st = L.up_sm100_workspace_status(ws.data_ptr(), stream)
    agree("exact_after_timeout", st == _lib.UP_OK and torch.equal(y, ops.scan(glob)[idx]))

    # ---- a wrap of the communicator's 30-bit launch tag ----
    L.up_sm100_comm_set_test_launches(comm.ptr, (1 << 30) - 2)
    ok = True
    for op in ("sum", "max", "sum", "min"):
        y = udist.sharded_scan(x, op, layout="block_cyclic", comm=comm)
        st = L.up_sm100_workspace_status(ws.data_ptr(), stream)
        ok = ok and st == _lib.UP_OK and torch.equal(y, ops.scan(glob, op)[idx])
    agree("tag_wrap", ok)

    torch.cuda.synchronize()
    dist.barrier()
    comm.close()
    if rank == 0:
        print(json.dumps({"world": world, "checks": checks}), flush=True)
    ok = all(checks.values())
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
