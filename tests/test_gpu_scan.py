"""GPU parity of the int32 scans (decoupled look-back) against the oracle: bit-exact, every op, inclusive and
exclusive, forward and reverse, on the reference's corpora, odd sizes, multi-row inputs and the full 2^28
configuration; plus the bounded-wait error path (a flag nothing sets) and workspace re-arming."""
import json
import os

import numpy as np
import pytest
import torch

import oracle as orc
from unpopped_b200 import _lib, ops, workloads

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
OPS = {"sum": orc.OP_SUM, "max": orc.OP_MAX, "min": orc.OP_MIN}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "these tests need the B200"


def run(x_np, op, excl, rev, carry=None):
    x = torch.from_numpy(np.ascontiguousarray(x_np)).cuda()
    c = None if carry is None else torch.tensor([carry], dtype=torch.int32, device="cuda")
    y = ops.scan(x, op, excl, rev, carry=c)
    ops.check_workspace("scan", x.device)
    return y.cpu().numpy()


@pytest.mark.parametrize("case", ["int_reduce_scan_5x6", "parallel_scan_4x45"])
def test_golden_corpora_every_variant(case):
    with open(os.path.join(GOLDEN, "scan_i32.json")) as f:
        g = json.load(f)["cases"][case]
    x = np.array(g["x"], dtype=np.int32)
    for key, exp in g["expected"].items():
        op, mode, direction = key.split("_")
        assert run(x, op, mode == "excl", direction == "rev").tolist() == exp, key


SIZES = [1, 2, 31, 512, 4095, 4096, 4097, 8191, 8192, 8196, 16383, 16384, 16385, 2 * 16384 + 8, 100_003,
         (1 << 20) + 12, 160 * 8192 + 4]


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("op", ["sum", "max", "min"])
def test_one_row_bit_exact(n, op):
    rng = np.random.default_rng(n)
    x = rng.integers(-(2 ** 31), 2 ** 31 - 1, size=n, dtype=np.int64).astype(np.int32)  # wraps often
    for excl in (False, True):
        for rev in (False, True):
            got = run(x, op, excl, rev)
            assert np.array_equal(got, orc.scan_i32(x, OPS[op], excl, rev)), (excl, rev)


@pytest.mark.parametrize("rows,k", [(3, 10_000), (1000, 45), (7, 4096), (2, 12_289), (3, 40_000), (2, 16_384 * 3 + 2)])
def test_many_rows(rows, k):
    rng = np.random.default_rng(rows + k)
    x = rng.integers(-50, 50, size=(rows, k)).astype(np.int32)
    for op in OPS:
        for excl in (False, True):
            for rev in (False, True):
                assert np.array_equal(run(x, op, excl, rev), orc.scan_i32(x, OPS[op], excl, rev))


def test_carry_in_is_combined_in_front():
    rng = np.random.default_rng(9)
    x = rng.integers(0, 16, size=50_000).astype(np.int32)
    for op, carry in (("sum", 123456), ("max", 20), ("min", -5)):
        for excl in (False, True):
            got = run(x, op, excl, False, carry=carry)
            assert np.array_equal(got, orc.scan_i32(x, OPS[op], excl, False, carry=carry))


def test_unaligned_input_takes_the_scalar_path():
    rng = np.random.default_rng(3)
    base = torch.from_numpy(rng.integers(-9, 9, size=20_001).astype(np.int32)).cuda()
    x = base[1:]  # 4-byte offset: no 16-byte vector access
    y = ops.scan(x, "sum")
    assert np.array_equal(y.cpu().numpy(), orc.scan_i32(x.cpu().numpy(), orc.OP_SUM, False))


def test_full_config_three_variants():
    x = workloads.scan_input(device="cuda")
    xn = x.cpu().numpy()
    for op, excl in (("sum", False), ("sum", True), ("max", False)):
        y = ops.scan(x, op, excl)
        ops.check_workspace("scan", x.device)
        want = orc.scan_i32_chunked(xn, OPS[op], excl, threads=orc.max_threads())
        assert np.array_equal(y.cpu().numpy(), want), (op, excl)


def test_workspace_rearms_across_launches_and_shapes():
    rng = np.random.default_rng(5)
    ws = torch.zeros(_lib.load().up_sm100_scan_workspace_bytes(1, 1 << 20), dtype=torch.uint8, device="cuda")
    for n in (1 << 20, 5000, 1 << 20, 77, 300_000):
        x = torch.from_numpy(rng.integers(-3, 3, size=n).astype(np.int32)).cuda()
        for _ in range(2):
            y = ops.scan(x, "sum", ws=ws)
            assert ops.workspace_status(ws) == _lib.UP_OK
            assert np.array_equal(y.cpu().numpy(), orc.scan_i32(x.cpu().numpy(), orc.OP_SUM, False))


def test_bounded_wait_reports_timeout_and_recovers():
    """Tile 0 withholds its flag (a flag nothing sets): every other tile's look-back gives up after the wait
    limit, the status comes back as UP_ERR_DEVICE_TIMEOUT, and the next launch works. No fault, no hang."""
    L = _lib.load()
    x = torch.ones(1 << 18, dtype=torch.int32, device="cuda")  # 32 tiles
    ws = torch.zeros(L.up_sm100_scan_workspace_bytes(1, x.numel()), dtype=torch.uint8, device="cuda")
    L.up_sm100_set_wait_limit_ns(2_000_000)  # 2 ms
    try:
        L.up_sm100_set_test_withhold_flag(1)
        ops.scan(x, "sum", ws=ws)
        assert ops.workspace_status(ws) == _lib.UP_ERR_DEVICE_TIMEOUT
        # the error word was cleared and the workspace re-armed: a normal scan works
        y = ops.scan(x, "sum", ws=ws)
        assert ops.workspace_status(ws) == _lib.UP_OK
        assert np.array_equal(y.cpu().numpy(), np.arange(1, x.numel() + 1, dtype=np.int32))
    finally:
        L.up_sm100_set_test_withhold_flag(0)
        L.up_sm100_set_wait_limit_ns(1_000_000_000)


def test_reduce_i32_matches_oracle():
    rng = np.random.default_rng(11)
    for n in (1, 100, 8191, 8192, 1 << 20, (1 << 22) + 3):
        x = rng.integers(-(2 ** 31), 2 ** 31 - 1, size=n, dtype=np.int64).astype(np.int32)
        xt = torch.from_numpy(x).cuda()
        for op in OPS:
            assert int(ops.reduce_i32(xt, op).item()) == orc.reduce_i32(x, OPS[op]), (n, op)
    assert int(ops.reduce_i32(torch.empty(0, dtype=torch.int32, device="cuda"), "max").item()) == -(2 ** 31)


def test_epoch_wrap_clears_flags_left_by_the_earlier_cycle():
    """The flags carry the low 30 bits of the launch count. A launch exactly 2^30 launches after another one has
    the same tag, so the first launch on a workspace after the wrap must clear what the earlier cycle left: here
    a large scan writes flags at tag T, the count jumps to T + 2^30, and a smaller scan on the same workspace
    must leave every flag it does not write at zero, and every scan stays exact."""
    L = _lib.load()
    rng = np.random.default_rng(21)
    big, small = (1 << 22) + 16, (1 << 20) + 4  # 513 and 129 tiles of 8192
    ws = torch.zeros(L.up_sm100_scan_workspace_bytes(1, big), dtype=torch.uint8, device="cuda")
    tag = (1 << 30) - 3
    xb = torch.from_numpy(rng.integers(-9, 9, size=big).astype(np.int32)).cuda()
    xs = torch.from_numpy(rng.integers(-9, 9, size=small).astype(np.int32)).cuda()
    L.up_sm100_set_test_scan_epoch(tag)
    y = ops.scan(xb, "sum", ws=ws)
    assert ops.workspace_status(ws) == _lib.UP_OK
    assert np.array_equal(y.cpu().numpy(), orc.scan_i32(xb.cpu().numpy(), orc.OP_SUM, False))
    flags = ws[64:].view(torch.int64)
    assert int((flags != 0).sum()) == 513
    L.up_sm100_set_test_scan_epoch(tag + (1 << 30))  # the same 30-bit tag, one cycle later
    y = ops.scan(xs, "max", ws=ws)
    assert ops.workspace_status(ws) == _lib.UP_OK
    assert np.array_equal(y.cpu().numpy(), orc.scan_i32(xs.cpu().numpy(), orc.OP_MAX, False))
    flags = ws[64:].view(torch.int64)
    assert int((flags[129:] != 0).sum()) == 0  # cleared before the scan, and not written by it
    for _ in range(2):  # later launches of the new cycle do not clear again, and stay exact
        y = ops.scan(xb, "sum", True, ws=ws)
        assert ops.workspace_status(ws) == _lib.UP_OK
        assert np.array_equal(y.cpu().numpy(), orc.scan_i32(xb.cpu().numpy(), orc.OP_SUM, True))


def test_general_form_takes_tiles_by_ticket_and_resets_the_ticket():
    """Unaligned input takes the one-tile-per-CTA form, whose CTAs take their tiles from a ticket counter in the
    workspace header; the CTA with the last ticket sets it back to zero for the next launch."""
    L = _lib.load()
    rng = np.random.default_rng(8)
    base = torch.from_numpy(rng.integers(-(2 ** 31), 2 ** 31 - 1, size=(1 << 21) + 3, dtype=np.int64)
                            .astype(np.int32)).cuda()
    x = base[1:]  # a 4-byte offset
    ws = torch.zeros(L.up_sm100_scan_workspace_bytes(1, x.numel()), dtype=torch.uint8, device="cuda")
    for op, excl, rev in (("sum", False, False), ("min", True, True), ("max", False, True)):
        y = ops.scan(x, op, excl, rev, ws=ws)
        assert ops.workspace_status(ws) == _lib.UP_OK
        assert int(ws[:4].view(torch.int32).item()) == 0
        assert np.array_equal(y.cpu().numpy(), orc.scan_i32(x.cpu().numpy(), OPS[op], excl, rev))
