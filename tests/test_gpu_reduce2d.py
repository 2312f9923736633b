"""GPU parity of the reduction breadth (f32 Mean/Max/Min, i32 Sum/Prod/Max/Min/And/Or/Xor, last and outer axis)
against the CPU oracle restatement and the reference corpora. Every result is bit-exact (an f32 Mean of an empty
row is NaN on both sides)."""
import json
import os

import numpy as np
import pytest
import torch

import oracle as orc
from unpopped_b200 import ops

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
INT_OPS = ("sum", "prod", "max", "min", "and", "or", "xor")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "these tests need the B200"


def golden(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def test_int_corpus_every_op_both_axes():
    g = golden("scan_i32.json")
    x = torch.tensor(g["cases"]["int_reduce_scan_5x6"]["x"], dtype=torch.int32, device="cuda")
    for op, exp in g["reductions_5x6_both_axes"].items():
        assert ops.reduce2d(x, op, 1).tolist() == exp["axis1"], op
        assert ops.reduce2d(x, op, 0).tolist() == exp["axis0"], op


def test_float_corpus_mean_max_min_columns():
    g = golden("float_sum_documented.json")
    xn = np.array(g["x_f32_bits"], dtype=np.uint32).view(np.float32).reshape(g["rows"], g["cols"])
    x = torch.from_numpy(xn).cuda()
    for b in g["blocks"]:
        assert bits(ops.reduce2d(x, "mean", 1, block=b).cpu()).tolist() == g["documented_mean_f32_bits"][str(b)]
    assert bits(ops.reduce2d(x, "max", 1).cpu()).tolist() == g["max_f32_bits"]
    assert bits(ops.reduce2d(x, "min", 1).cpu()).tolist() == g["min_f32_bits"]
    assert bits(ops.reduce2d(x, "sum", 0).cpu()).tolist() == g["col_sum_f32_bits"]
    assert bits(ops.reduce2d(x, "max", 0).cpu()).tolist() == g["col_max_f32_bits"]
    xt = torch.from_numpy(np.ascontiguousarray(xn.T)).cuda()  # the corpus's rows as columns
    for b in g["col_documented_blocks"]:
        assert bits(ops.reduce2d(xt, "sum", 0, block=b).cpu()).tolist() == g["documented_f32_bits"][str(b)], b


SHAPES = [(1, 1), (3, 7), (17, 96), (64, 4097), (33, 8192), (1000, 5), (5, 1000), (300, 1024), (9, 12000)]


@pytest.mark.parametrize("rows,cols", SHAPES)
@pytest.mark.parametrize("axis", [0, 1])
def test_int_ops_vs_oracle(rows, cols, axis):
    rng = np.random.default_rng(rows * 7 + cols + axis)
    xn = rng.integers(-2**31, 2**31, (rows, cols), dtype=np.int64).astype(np.int32)
    xn[:, ::3] = rng.integers(-3, 4, (rows, (cols + 2) // 3))  # small values keep Prod and And/Or informative
    x = torch.from_numpy(xn).cuda()
    for op in INT_OPS:
        got = ops.reduce2d(x, op, axis).cpu().numpy()
        assert np.array_equal(got, orc.reduce2d_i32(xn, op, axis)), op


def _specials(rng, rows, cols):
    x = (rng.standard_normal((rows, cols)) * 10.0 ** rng.integers(-3, 4, (rows, 1))).astype(np.float32)
    pick = rng.random((rows, cols))
    x[pick < 0.02] = 0.0
    x[(pick >= 0.02) & (pick < 0.04)] = -0.0
    x[(pick >= 0.04) & (pick < 0.045)] = np.inf
    x[(pick >= 0.045) & (pick < 0.05)] = -np.inf
    nan_at = pick > 0.995
    payload = rng.integers(1, 1 << 22, (rows, cols)).astype(np.uint32) | np.uint32(0x7f800000)
    payload |= (rng.integers(0, 2, (rows, cols)).astype(np.uint32) << 31)
    xb = x.view(np.uint32)
    xb[nan_at] = payload[nan_at]
    return x


@pytest.mark.parametrize("rows,cols", SHAPES)
@pytest.mark.parametrize("axis", [0, 1])
def test_float_max_min_vs_oracle_with_specials(rows, cols, axis):
    rng = np.random.default_rng(rows + 13 * cols + axis)
    xn = _specials(rng, rows, cols)
    x = torch.from_numpy(xn).cuda()
    for op in ("max", "min"):
        got = bits(ops.reduce2d(x, op, axis).cpu())
        assert np.array_equal(got, bits(orc.reduce2d_f32(xn, op, axis))), op


@pytest.mark.parametrize("rows,cols", SHAPES)
def test_float_sum_mean_vs_oracle(rows, cols):
    rng = np.random.default_rng(rows * 3 + cols)
    xn = (rng.standard_normal((rows, cols)) * 10.0 ** rng.integers(-3, 4, (rows, 1))).astype(np.float32)
    x = torch.from_numpy(xn).cuda()
    # outer axis: the serial order per column (block 1) and the documented order of larger blocks
    assert np.array_equal(bits(ops.reduce2d(x, "sum", 0).cpu()), bits(orc.reduce2d_f32(xn, "sum", 0)))
    assert np.array_equal(bits(ops.reduce2d(x, "mean", 0).cpu()), bits(orc.reduce2d_f32(xn, "mean", 0)))
    for b in (2, 16, 64, 128, 256):
        assert np.array_equal(bits(ops.reduce2d(x, "sum", 0, block=b).cpu()),
                              bits(orc.col_sum_f32_documented(xn, b))), b
        assert np.array_equal(bits(ops.reduce2d(x, "mean", 0, block=b).cpu()),
                              bits(orc.col_sum_f32_documented(xn, b, mean=True))), b
    # last axis: the documented order for each block (block 1 is the serial order)
    for b in (1, 4, 256, 1024):
        assert np.array_equal(bits(ops.reduce2d(x, "mean", 1, block=b).cpu()),
                              bits(orc.row_mean_f32_documented(xn, b))), b
    assert np.array_equal(bits(ops.reduce2d(x, "mean", 1, block=1).cpu()), bits(orc.reduce2d_f32(xn, "mean", 1)))


def _serial_columns(rng, rows, cols):
    """Columns for the outer-axis Sum in the serial order, one kind per column in turn: N(0,1) and U[0,1) (chunks
    stay exact), a few values near 2^-40 among N(0,1) ones, sums of ones with tiny and large values (partial sums
    at full precision that cross binades), exponents over 40 binades, subnormals beside normals, NaN/±Inf/±0
    specials, and all -0 (the sum is +0)."""
    kinds = []
    for c in range(cols):
        k = c % 8
        if k == 0:
            v = rng.standard_normal(rows)
        elif k == 1:
            v = rng.random(rows)
        elif k == 2:
            v = rng.standard_normal(rows)
            v[rng.random(rows) < 0.01] = rng.choice([2.0 ** -40, -3.0 * 2.0 ** -45, 2.0 ** -30], 1)[0]
        elif k == 3:
            v = np.where(rng.random(rows) < 0.7, 1.0, rng.choice([2.0 ** -28, 2.0 ** -52, 3.0 * 2.0 ** 24], rows))
        elif k == 4:
            v = (rng.random(rows) - 0.5) * 2.0 ** rng.integers(-20, 20, rows)
        elif k == 5:
            v = rng.standard_normal(rows) * np.where(rng.random(rows) < 0.5, 2.0 ** -135, 1.0)
        elif k == 6:
            v = _specials(rng, rows, 1)[:, 0]  # kept in f32: the NaN payloads stay as drawn
        else:
            v = np.full(rows, -0.0)
        kinds.append(v if v.dtype == np.float32 else v.astype(np.float32))
    return np.ascontiguousarray(np.stack(kinds, axis=1))


@pytest.mark.parametrize("rows,cols", [(1, 33), (63, 40), (64, 32), (65, 31), (1023, 70), (1024, 64), (1025, 96),
                                       (3000, 257), (8192, 100), (8193, 16), (20000, 12), (20000, 9)])
def test_outer_sum_serial_order_exact_and_rounding_chunks(rows, cols):
    """The outer-axis Sum/Mean in the serial order, bit for bit, on columns whose chunks are added out of order (no
    add rounds) and columns that round and take the value-by-value fold, at row counts on both sides of the 64-row
    chunk, the 1,024-row segment and the 8,192-row round of the cluster form (widths that are a multiple of 4 on
    16-byte aligned rows); NaN results match as NaN. A strided, unaligned view takes the 32-column form."""
    rng = np.random.default_rng(rows * 7 + cols)
    xn = _serial_columns(rng, rows, cols)
    wide = np.zeros((rows, cols + 5), np.float32)
    wide[:, 3:3 + cols] = xn
    wt = torch.from_numpy(wide).cuda()
    for x in (torch.from_numpy(xn).cuda(), wt[:, 3:3 + cols]):
        for op in ("sum", "mean"):
            got = ops.reduce2d(x, op, 0).cpu().numpy()
            want = orc.reduce2d_f32(xn, op, 0)
            nan = np.isnan(want)
            assert np.array_equal(np.isnan(got), nan), op
            assert np.array_equal(bits(got)[~nan], bits(want)[~nan]), op


@pytest.mark.parametrize("dist", ["normal", "uniform", "ones_and_tiny"])
def test_outer_sum_serial_order_full_strips(dist):
    """8,192 x 8,192 in the cluster form: N(0,1) (the all-exact round), U[0,1) (a few chunks round) and unit values
    with a tiny one in every 50 (most rounds fall back to rank order), bit for bit against the serial fold."""
    rng = np.random.default_rng(5)
    if dist == "normal":
        xn = rng.standard_normal((8192, 8192), dtype=np.float32)
    elif dist == "uniform":
        xn = rng.random((8192, 8192), dtype=np.float32)
    else:
        xn = np.where(rng.random((8192, 8192)) < 0.02, np.float32(2.0 ** -35), np.float32(1.0)).astype(np.float32)
    x = torch.from_numpy(xn).cuda()
    t = orc.max_threads()
    for op in ("sum", "mean"):
        assert np.array_equal(bits(ops.reduce2d(x, op, 0).cpu()), bits(orc.reduce2d_f32(xn, op, 0, t))), op


@pytest.mark.parametrize("cols", [96, 8192, 12000])
def test_float_max_min_structured_rows(cols):
    """Rows built to hit each branch of the chunked fold: all -inf / +inf, all NaN, +0 and -0 ties in either order,
    the extreme value first, last and repeated, one NaN at the start or the end, and an extreme beside a NaN."""
    rng = np.random.default_rng(cols)
    rows = []
    inf = np.float32(np.inf)
    for fill in (-inf, inf, np.float32(np.nan), np.float32(0.0), np.float32(-0.0)):
        rows.append(np.full(cols, fill, np.float32))
    z = np.zeros(cols, np.float32)
    z[::2] = -0.0
    rows.append(z)
    rows.append(-z)
    for pos in (0, cols - 1, cols // 2, 3, cols - 4):
        for v in (1e30, -1e30):
            r = rng.standard_normal(cols).astype(np.float32)
            r[pos] = v
            rows.append(r)
    r = rng.standard_normal(cols).astype(np.float32)
    r[[5, cols // 3, cols - 2]] = 7.0
    r[[9, cols // 2]] = -7.0
    rows.append(r)
    for pos in (0, cols - 1):
        r = rng.standard_normal(cols).astype(np.float32)
        r.view(np.uint32)[pos] = 0xffa00001  # a signalling-looking NaN with the sign bit
        rows.append(r)
    r = rng.standard_normal(cols).astype(np.float32)
    r[10], r[11] = np.nan, 1e30
    rows.append(r)
    xn = np.stack(rows)
    x = torch.from_numpy(xn).cuda()
    for op in ("max", "min"):
        for axis in (0, 1):
            got = bits(ops.reduce2d(x, op, axis).cpu())
            assert np.array_equal(got, bits(orc.reduce2d_f32(xn, op, axis))), (op, axis)


def test_strided_views():
    rng = np.random.default_rng(5)
    full = rng.integers(-50, 50, (40, 130)).astype(np.int32)
    xv = torch.from_numpy(full).cuda()[:, 3:99]  # row stride 130, unaligned start
    sub = np.ascontiguousarray(full[:, 3:99])
    for axis in (0, 1):
        for op in INT_OPS:
            assert np.array_equal(ops.reduce2d(xv, op, axis).cpu().numpy(), orc.reduce2d_i32(sub, op, axis))
    ff = _specials(rng, 40, 130)
    fv = torch.from_numpy(ff).cuda()[:, 1:97]
    fsub = np.ascontiguousarray(ff[:, 1:97])
    for axis in (0, 1):
        for op in ("max", "min"):
            assert np.array_equal(bits(ops.reduce2d(fv, op, axis).cpu()), bits(orc.reduce2d_f32(fsub, op, axis)))
    assert np.array_equal(bits(ops.reduce2d(fv, "sum", 0).cpu()), bits(orc.reduce2d_f32(fsub, "sum", 0)))


def test_empty_reductions():
    for rows, cols, axis in ((4, 0, 1), (0, 4, 0)):
        xi = torch.zeros((rows, cols), dtype=torch.int32, device="cuda")
        for op in INT_OPS:
            got = ops.reduce2d(xi, op, axis).cpu().numpy()
            assert (got == (1 if op == "prod" else 0)).all(), op
        xf = torch.zeros((rows, cols), dtype=torch.float32, device="cuda")
        for op in ("sum", "max", "min"):
            assert (ops.reduce2d(xf, op, axis).cpu().numpy() == 0).all()
        assert torch.isnan(ops.reduce2d(xf, "mean", axis)).all()


def test_full_config_rows():
    """cfg 1's 8192 x 8192 f32 (Mean, Max, Min) and the same shape as i32 (every op), against the oracle."""
    rng = np.random.default_rng(11)
    xn = rng.standard_normal((8192, 8192), dtype=np.float32)
    x = torch.from_numpy(xn).cuda()
    t = orc.max_threads()
    assert np.array_equal(bits(ops.reduce2d(x, "mean", 1, block=1024).cpu()),
                          bits(orc.row_mean_f32_documented(xn, 1024, threads=t)))
    for op in ("max", "min"):
        for axis in (0, 1):
            assert np.array_equal(bits(ops.reduce2d(x, op, axis).cpu()), bits(orc.reduce2d_f32(xn, op, axis, t)))
    assert np.array_equal(bits(ops.reduce2d(x, "sum", 0, block=256).cpu()),
                          bits(orc.col_sum_f32_documented(xn, 256, threads=t)))
    for op in ("sum", "mean"):  # the serial order per column (block 1)
        assert np.array_equal(bits(ops.reduce2d(x, op, 0).cpu()), bits(orc.reduce2d_f32(xn, op, 0, t))), op
    xi = rng.integers(-2**31, 2**31, (8192, 8192), dtype=np.int64).astype(np.int32)
    xit = torch.from_numpy(xi).cuda()
    for op in INT_OPS:
        for axis in (0, 1):
            assert np.array_equal(ops.reduce2d(xit, op, axis).cpu().numpy(), orc.reduce2d_i32(xi, op, axis, t)), op


def test_refusals():
    x = torch.zeros((4, 4), dtype=torch.float32, device="cuda")
    from unpopped_b200._lib import UpError
    with pytest.raises(UpError):
        ops.reduce2d(x, "prod", 1)  # a float Prod is not lowered (the launched lift declines it too)
    with pytest.raises(UpError):
        ops.reduce2d(x, "mean", 1, accum="f32")
    with pytest.raises(UpError):
        ops.reduce2d(x, "sum", 0, accum="f32")
