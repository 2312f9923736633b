"""The multi-GPU exchange logic (unpopped_b200/dist.py) on world_size-2 and -3 gloo ranks on the CPU.

The per-rank kernels are stood in by the CPU oracle (test infrastructure): what is under test is the sharding,
the all-gather of shard totals, the carry each rank derives from them and the reassembly of outputs. Also a
rank that leaves before the exchange: the other rank's collective ends with an error within the short
process-group timeout instead of waiting forever.
"""
import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
OPS = {"sum": 0, "max": 2, "min": 3}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def cpu_local():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc

    from unpopped_b200.dist import Local

    def reduce_i32(x, op):
        return torch.tensor([orc.reduce_i32(x.numpy(), OPS[op])], dtype=torch.int32)

    def scan(x, op, ex, rev, carry):
        c = int(carry.item()) if carry is not None else None
        return torch.from_numpy(orc.scan_i32(x.numpy(), OPS[op], ex, rev, carry=c))

    def w4a16(w, s, x, g):
        n, kh = w.shape
        out, _, _ = orc.w4a16(w.numpy(), s.view(torch.int16).numpy().view(np.uint16),
                              x.view(torch.int16).numpy().view(np.uint16), x.shape[0], n, 2 * kh, g)
        return torch.from_numpy(out.view(np.int16)).view(torch.bfloat16)

    return Local(reduce_i32=reduce_i32, scan=scan, w4a16=w4a16)


def _init(rank, world, port, timeout_s=30):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    sys.path.insert(0, ROOT)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))


def _scan_worker(rank, world, port, n_per, q):
    try:
        _init(rank, world, port)
        from unpopped_b200.dist import sharded_scan

        rng = np.random.default_rng(123)
        full = rng.integers(-(2 ** 31), 2 ** 31 - 1, size=n_per * world, dtype=np.int64).astype(np.int32)
        mine = torch.from_numpy(full[rank * n_per:(rank + 1) * n_per].copy())
        res = {}
        for op in OPS:
            for ex in (False, True):
                for rev in (False, True):
                    res[(op, ex, rev)] = sharded_scan(mine, op, ex, rev, local=cpu_local()).numpy()
        q.put((rank, res))
        dist.destroy_process_group()
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_scan_equals_global_scan(world):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc

    n_per = 5000
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_scan_worker, args=(r, world, port, n_per, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    rng = np.random.default_rng(123)
    full = rng.integers(-(2 ** 31), 2 ** 31 - 1, size=n_per * world, dtype=np.int64).astype(np.int32)
    for r in range(world):
        assert isinstance(got[r], dict), got[r]
    for key in got[0]:
        op, ex, rev = key
        want = orc.scan_i32(full, OPS[op], ex, rev)
        cat = np.concatenate([got[r][key] for r in range(world)])
        assert np.array_equal(cat, want), key


def _w4_worker(rank, world, port, q):
    try:
        _init(rank, world, port)
        from unpopped_b200.dist import gather_outputs, row_slice, sharded_w4a16

        g = torch.Generator().manual_seed(7)
        n, k, m, grp = 64 * world, 256, 3, 128
        w = torch.randint(0, 256, (n, k // 2), generator=g, dtype=torch.int32).to(torch.uint8)
        s = (torch.rand(n, k // grp, generator=g) * 0.015 + 0.005).to(torch.float16)
        x = torch.randn(m, k, generator=g).to(torch.bfloat16)
        sl = row_slice(n, world, rank)
        y = sharded_w4a16(w[sl].contiguous(), s[sl].contiguous(), x, grp, local=cpu_local())
        rows = gather_outputs(torch.arange(rank * 4, rank * 4 + 4, dtype=torch.int32).reshape(4, 1))
        q.put((rank, (y.view(torch.int16).numpy(), rows.numpy())))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, repr(e)))


def test_sharded_w4a16_and_output_gather():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_w4_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert isinstance(got[r], tuple), got[r]
    g = torch.Generator().manual_seed(7)
    n, k, m, grp = 64 * world, 256, 3, 128
    w = torch.randint(0, 256, (n, k // 2), generator=g, dtype=torch.int32).to(torch.uint8)
    s = (torch.rand(n, k // grp, generator=g) * 0.015 + 0.005).to(torch.float16)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    want, _, _ = orc.w4a16(w.numpy(), s.view(torch.int16).numpy().view(np.uint16),
                           x.view(torch.int16).numpy().view(np.uint16), m, n, k, grp)
    for r in range(world):
        assert np.array_equal(got[r][0].view(np.uint16), want)
        assert got[r][1].reshape(-1).tolist() == list(range(4 * world))


def test_row_slice_covers_every_row_once():
    from unpopped_b200.dist import row_slice

    for n in (0, 1, 7, 8192, 8193):
        for world in (1, 2, 3, 8):
            covered = []
            for r in range(world):
                s = row_slice(n, world, r)
                covered.extend(range(s.start, s.stop))
            assert covered == list(range(n))


def _leaving_worker(rank, world, port, q):
    try:
        _init(rank, world, port, timeout_s=5)
        if rank == 1:
            q.put((rank, "left"))
            q.close()
            q.join_thread()  # flush the message before the abrupt exit
            os._exit(0)  # leaves between steps, before the exchange
        from unpopped_b200.dist import sharded_scan

        try:
            sharded_scan(torch.arange(10, dtype=torch.int32), "sum", local=cpu_local())
            q.put((rank, "completed"))
        except Exception as e:
            q.put((rank, "error:" + type(e).__name__))
    except Exception as e:
        q.put((rank, "setup:" + repr(e)))


def test_a_rank_that_leaves_ends_the_exchange_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert got[1] == "left"
    assert got[0].startswith("error:"), got[0]


def _block_cyclic_worker(rank, world, port, n_local, q):
    try:
        _init(rank, world, port)
        from unpopped_b200.dist import block_cyclic_index, sharded_scan

        g = torch.Generator().manual_seed(11)
        glob = torch.randint(-(2 ** 31), 2 ** 31 - 1, (world * n_local,), generator=g, dtype=torch.int32)
        x = glob[block_cyclic_index(n_local, world)[rank]].contiguous()
        res = {}
        for op in OPS:
            for ex in (False, True):
                res[(op, ex)] = sharded_scan(x, op, ex, layout="block_cyclic", local=cpu_local()).numpy()
        q.put((rank, res))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world", [2, 3])
def test_block_cyclic_layout_is_the_global_scan(world):
    """The block-cyclic layout (stripes of 148 x 8192 elements dealt round-robin, a partial last stripe): every
    rank's result, put back at its global positions, is the scan of the global array."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc

    from unpopped_b200.dist import STRIPE_ELEMS, block_cyclic_index

    n_local = 2 * STRIPE_ELEMS + 8192 * 3 + 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_block_cyclic_worker, args=(r, world, port, n_local, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        assert isinstance(got[r], dict), got[r]
    g = torch.Generator().manual_seed(11)
    glob = torch.randint(-(2 ** 31), 2 ** 31 - 1, (world * n_local,), generator=g, dtype=torch.int32).numpy()
    idx = block_cyclic_index(n_local, world).numpy()
    for (op, ex) in got[0]:
        want = orc.scan_i32(glob, OPS[op], ex)
        for r in range(world):
            assert np.array_equal(got[r][(op, ex)], want[idx[r]]), (op, ex, r)


def test_block_cyclic_index_is_a_permutation_in_stripes():
    from unpopped_b200.dist import STRIPE_ELEMS, block_cyclic_index

    for world in (1, 2, 3, 8):
        n_local = STRIPE_ELEMS + 17 * 4
        idx = block_cyclic_index(n_local, world)
        assert sorted(idx.reshape(-1).tolist()[:0]) == []
        flat = idx.reshape(-1)
        assert torch.unique(flat).numel() == flat.numel()
        # rank r's first stripe is global stripe r
        for r in range(world):
            assert int(idx[r, 0]) == r * STRIPE_ELEMS


def _comm_args_worker(rank, world, port, q):
    """A communicator cannot form without a GPU: every entry point answers with a status, none crashes."""
    try:
        _init(rank, world, port)
        import ctypes

        from unpopped_b200 import _lib

        L = _lib.load()
        uid = (ctypes.c_ubyte * 128)()
        out = {"uid": L.up_sm100_comm_unique_id(uid) if rank == 0 else 0}
        box = [bytes(uid)]
        dist.broadcast_object_list(box, src=0)
        uid = (ctypes.c_ubyte * 128).from_buffer_copy(box[0])
        c = ctypes.c_void_p()
        out["init_bad_rank"] = L.up_sm100_comm_init_rank(world, world, uid, ctypes.byref(c))
        out["init_bad_size"] = L.up_sm100_comm_init_rank(0, 0, uid, ctypes.byref(c))
        out["init_too_many"] = L.up_sm100_comm_init_rank(9, 0, uid, ctypes.byref(c))
        out["init_null"] = L.up_sm100_comm_init_rank(world, rank, uid, None)
        out["init_no_gpu"] = L.up_sm100_comm_init_rank(world, rank, uid, ctypes.byref(c))
        t = _lib.UpTensor()
        out["launch_no_comm"] = L.up_sm100_launch_multi(_lib.KERNEL["SCAN_I32"], ctypes.byref(t), 1, ctypes.byref(t),
                                                        1, None, 0, None, 0, None, None)
        n = ctypes.c_size_t(0)
        out["ws_no_comm"] = L.up_sm100_workspace_bytes_multi(_lib.KERNEL["SCAN_I32"], ctypes.byref(t), 1,
                                                             ctypes.byref(t), 1, None, 0, None, ctypes.byref(n))
        out["rank_null"] = L.up_sm100_comm_rank(None, None, None)
        out["destroy_null"] = L.up_sm100_comm_destroy(None)
        out["uid_null"] = L.up_sm100_comm_unique_id(None)
        q.put((rank, out))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, repr(e)))


def test_communicator_argument_errors_on_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_comm_args_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    for r in range(world):
        out = got[r]
        assert isinstance(out, dict), out
        for key in ("init_bad_rank", "init_bad_size", "init_too_many", "init_null", "launch_no_comm", "ws_no_comm",
                    "rank_null", "destroy_null", "uid_null"):
            assert out[key] == 7, (key, out[key])  # UP_ERR_INVALID
        assert out["init_no_gpu"] in (5, 6), out  # UP_ERR_CUDA or UP_ERR_COMM: no device in this container
    assert got[0]["uid"] in (0, 6)  # NCCL may or may not make an id without a network interface
