"""GPU parity of the host-memory scan (up_sm100_scan_i32_host) against the CPU oracle restatement.

The entry streams host buffers through a ring of 2^23-element device slots: rows longer than a slot are cut
into chunks whose carries are derived on the device, shorter rows travel in groups. Integer scans are exact,
so every case is bit-exact.
"""
import numpy as np
import pytest
import torch

import oracle as orc
from unpopped_b200 import ops
from unpopped_b200._lib import OP

pytestmark = pytest.mark.gpu
SLOT = 1 << 23
OPS = {"sum": OP["SUM"], "max": OP["MAX"], "min": OP["MIN"]}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "these tests need the B200"


def _data(shape, op, seed):
    rng = np.random.default_rng(seed)
    if op == "sum":
        return rng.integers(-2**31, 2**31, shape, dtype=np.int64).astype(np.int32)  # wraps
    return rng.integers(-1000, 1000, shape, dtype=np.int64).astype(np.int32)


@pytest.mark.parametrize("op", ["sum", "max", "min"])
@pytest.mark.parametrize("exclusive", [False, True])
@pytest.mark.parametrize("reverse", [False, True])
def test_row_longer_than_a_slot(op, exclusive, reverse):
    """One row of two slots and a ragged tail: the second and third chunks start from device-derived carries."""
    k = 2 * SLOT + 12345
    x = _data((1, k), op, k + exclusive + 2 * reverse)
    carry = 17 if op == "sum" else None
    got = ops.scan_host(x, op, exclusive, reverse, carry)
    want = orc.scan_i32(x, OPS[op], exclusive, reverse, carry)
    assert np.array_equal(got, want)


def test_several_long_rows_pinned():
    """Three rows of 2.5 slots each from a pinned tensor: a row's chunks chain, the next row starts fresh."""
    rows, k = 3, SLOT * 5 // 2 + 3
    x = torch.from_numpy(_data((rows, k), "sum", 3)).pin_memory()
    for exclusive, reverse in [(False, False), (True, True)]:
        got = ops.scan_host(x, "sum", exclusive, reverse, carry=-5)
        want = orc.scan_i32(x.numpy(), OPS["sum"], exclusive, reverse, -5)
        assert np.array_equal(got.numpy(), want)


@pytest.mark.parametrize("rows,k", [(100000, 100), (70001, 1), (5, 8192 * 3 + 1), (1, SLOT), (2, SLOT - 4)])
def test_short_rows_travel_in_groups(rows, k):
    x = _data((rows, k), "sum", rows + k)
    for op, exclusive, reverse in [("sum", False, False), ("max", True, True), ("min", False, True)]:
        xx = x if op == "sum" else _data((rows, k), op, rows)
        got = ops.scan_host(xx, op, exclusive, reverse)
        want = orc.scan_i32(xx, OPS[op], exclusive, reverse)
        assert np.array_equal(got, want), (op, exclusive, reverse)


def test_headline_size_pinned():
    """2^28 elements in one row (the benchmark's configs[1]) through pinned buffers: 32 chunks."""
    n = 1 << 28
    x = torch.randint(0, 16, (n,), dtype=torch.int32, generator=torch.Generator().manual_seed(9)).pin_memory()
    got = ops.scan_host(x, "sum")
    want = orc.scan_i32_chunked(x.numpy(), OPS["sum"], False, orc.max_threads())
    assert np.array_equal(got.numpy(), want)


def test_empty_and_errors():
    x = np.zeros((0, 5), np.int32)
    assert ops.scan_host(x).shape == (0, 5)
    x = np.zeros((4, 0), np.int32)
    assert ops.scan_host(x).shape == (4, 0)
    with pytest.raises(ValueError):
        ops.scan_host(np.zeros(8, np.int64))
