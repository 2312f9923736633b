"""up_sm100_scan_i32_noalloc, the scan whose scratch is a built-in device array, called through the C ABI.

Each case runs two calls in a row and compares each one with up_sm100_scan_i32, the entry point that takes
a caller's workspace, and with the oracle. Covered: the largest shape the array holds, the refusal of a
larger shape, the timeout report, and device free memory staying the same across calls once the first call
has done its set-up. This file is named to be collected last, and it also passes when run alone.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle as orc
from unpopped_b200 import _lib

pytestmark = pytest.mark.gpu
OPS = {"sum": orc.OP_SUM, "max": orc.OP_MAX, "min": orc.OP_MIN}
MAX_TILES = 32768
TILE = 8192


@pytest.fixture(scope="module")
def L():
    assert torch.cuda.is_available(), "these tests need the B200"
    return _lib.load()


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def noalloc(L, x, op, excl, rev, carry=None, sync=1):
    rows, k = (1, x.numel()) if x.dim() == 1 else x.shape
    y = torch.empty_like(x)
    st = L.up_sm100_scan_i32_noalloc(x.data_ptr(), y.data_ptr(), rows, k, OPS[op], int(excl), int(rev),
                                     carry.data_ptr() if carry is not None else None, sync, _stream())
    return st, y


def with_workspace(L, x, op, excl, rev, carry=None):
    rows, k = (1, x.numel()) if x.dim() == 1 else x.shape
    y = torch.empty_like(x)
    nb = L.up_sm100_scan_workspace_bytes(rows, k)
    ws = torch.zeros(nb, dtype=torch.uint8, device=x.device)
    _lib.check(L.up_sm100_scan_i32(x.data_ptr(), y.data_ptr(), rows, k, OPS[op], int(excl), int(rev),
                                   carry.data_ptr() if carry is not None else None, ws.data_ptr(), nb, _stream()),
               "up_sm100_scan_i32")
    assert L.up_sm100_workspace_status(ws.data_ptr(), _stream()) == _lib.UP_OK
    return y


CASES = [
    # (rows, k, op, exclusive, reverse, carry)
    (1, (1 << 20) + 7, "sum", False, False, None),
    (1, 100_003, "max", True, True, None),
    (3, 40_000, "min", False, True, 5),
    (MAX_TILES, 45, "sum", True, False, -3),             # every tile of the array, one per row
    (1, MAX_TILES * TILE, "sum", False, False, None),    # every tile of the array, one row of 2^28
]


@pytest.mark.parametrize("rows,k,op,excl,rev,carry", CASES)
def test_two_calls_in_a_row_match_the_workspace_entry(L, rows, k, op, excl, rev, carry):
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + k)
    xs = [torch.randint(-(2 ** 31), 2 ** 31 - 1, (rows, k), generator=g, dtype=torch.int32, device="cuda")
          for _ in range(2)]
    c = None if carry is None else torch.tensor([carry], dtype=torch.int32, device="cuda")
    got = []
    for x in xs:  # back to back on one stream, no synchronization in between
        st, y = noalloc(L, x, op, excl, rev, c, sync=0)
        assert st == _lib.UP_OK, L.up_sm100_last_error()
        got.append(y)
    st, _ = noalloc(L, xs[0][:1, :1].contiguous(), op, excl, rev, sync=1)  # reports any timeout
    assert st == _lib.UP_OK
    for x, y in zip(xs, got):
        want = with_workspace(L, x, op, excl, rev, c)
        assert torch.equal(y, want)
    if rows * k <= 200_000:  # the oracle as well, where it is quick
        xn = xs[1].cpu().numpy()
        want = np.stack([orc.scan_i32(r, OPS[op], excl, rev, carry=carry) for r in xn])
        assert np.array_equal(got[1].cpu().numpy(), want)


def test_larger_shapes_are_refused_before_any_device_work(L):
    x = torch.zeros(MAX_TILES + 1, dtype=torch.int32, device="cuda")
    before = L.up_sm100_launch_count()
    st, _ = noalloc(L, x.view(MAX_TILES + 1, 1), "sum", False, False)
    assert st == _lib.UP_ERR_UNSUPPORTED
    assert b"32768" in L.up_sm100_last_error()
    st, _ = noalloc(L, torch.zeros(2, TILE * (MAX_TILES // 2) + 1, dtype=torch.int32, device="cuda"), "max",
                    False, False)
    assert st == _lib.UP_ERR_UNSUPPORTED
    assert L.up_sm100_launch_count() == before
    # the empty scan is a no-op, argument errors come back as such
    st, _ = noalloc(L, torch.zeros(0, dtype=torch.int32, device="cuda"), "sum", False, False)
    assert st == _lib.UP_OK
    assert L.up_sm100_scan_i32_noalloc(None, None, 1, 10, OPS["sum"], 0, 0, None, 1, _stream()) == \
        _lib.UP_ERR_INVALID


def test_a_timeout_is_reported_once_and_the_next_call_works(L):
    """The bounded-wait test hook: tile 0 withholds its flag, so every later tile's look-back gives up after
    the (shortened) limit. The sync report returns UP_ERR_DEVICE_TIMEOUT and clears the flag."""
    x = torch.ones(1 << 18, dtype=torch.int32, device="cuda")  # 32 tiles
    L.up_sm100_set_wait_limit_ns(2_000_000)
    try:
        L.up_sm100_set_test_withhold_flag(1)
        st, _ = noalloc(L, x, "sum", False, False, sync=0)
        assert st == _lib.UP_OK
        st, _ = noalloc(L, x, "sum", False, False, sync=1)  # a later call reports the earlier timeout
        assert st == _lib.UP_ERR_DEVICE_TIMEOUT
    finally:
        L.up_sm100_set_test_withhold_flag(0)
        L.up_sm100_set_wait_limit_ns(1_000_000_000)
    st, y = noalloc(L, x, "sum", False, False, sync=1)
    assert st == _lib.UP_OK
    assert np.array_equal(y.cpu().numpy(), np.arange(1, x.numel() + 1, dtype=np.int32))


def test_calls_leave_device_free_memory_unchanged(L):
    x = torch.randint(-100, 100, (3, 70_000), dtype=torch.int32, device="cuda")
    y = torch.empty_like(x)
    for op in OPS:  # set-up, and the first launch of each kernel variant
        assert L.up_sm100_scan_i32_noalloc(x.data_ptr(), y.data_ptr(), 3, 70_000, OPS[op], 0, 0, None, 1,
                                           _stream()) == _lib.UP_OK
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for op in OPS:
        for excl in (0, 1):
            assert L.up_sm100_scan_i32_noalloc(x.data_ptr(), y.data_ptr(), 3, 70_000, OPS[op], excl, 1, None, 1,
                                               _stream()) == _lib.UP_OK
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
