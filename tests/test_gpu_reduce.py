"""GPU parity of the row reductions against the CPU oracle restatement and the reference's golden corpora.

Row sum, UP_ACCUM_AUTO: bit-exact against the documented order (the reference test's `documented`).
Row sum, UP_ACCUM_F32: |got - exact| <= gamma_d * sum|x| with u = 2^-24 and d the kernel's tree depth
  (13 for rows of at most 8192), which is below the 2^-20 * sum|x| the benchmark configuration states.
Max / argmax (bf16): bit-exact (a max never rounds; an index is an integer).
"""
import json
import os

import numpy as np
import pytest
import torch

import oracle as orc
from unpopped_b200 import ops, workloads

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
U32 = 2.0 ** -24


def gamma(d, u=U32):
    return d * u / (1 - d * u)


def golden(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "these tests need the B200"


def _f32(bits):
    return np.array(bits, dtype=np.uint32).view(np.float32)


# ---------------- row sum, documented f64 order ----------------

def test_auto_sum_matches_golden_documented_order():
    g = golden("float_sum_documented.json")
    x = torch.from_numpy(_f32(g["x_f32_bits"]).reshape(g["rows"], g["cols"])).cuda()
    for b in g["blocks"]:
        got = ops.row_sum(x, accum="auto", block=b).cpu().numpy().view(np.uint32)
        assert got.tolist() == g["documented_f32_bits"][str(b)], f"block {b}"
    # block 1 is the serial (plan-oracle) order
    assert ops.row_sum(x, accum="auto", block=1).cpu().numpy().view(np.uint32).tolist() == g["serial_f32_bits"]


def _serial_rows(rng, rows, cols):
    """Rows for the serial-order row sum (block 1), one kind per row in turn: N(0,1) and U[0,1) (chunks stay
    exact), a few values near 2^-40 among N(0,1) ones, ones with tiny and large values (partial sums at full
    precision that cross binades), exponents over 40 binades, subnormals beside normals, NaN/±Inf/±0 specials, and
    all -0 (the sum is +0)."""
    out = np.empty((rows, cols), np.float32)
    for r in range(rows):
        k = r % 8
        if k == 0:
            v = rng.standard_normal(cols)
        elif k == 1:
            v = rng.random(cols)
        elif k == 2:
            v = rng.standard_normal(cols)
            v[rng.random(cols) < 0.01] = rng.choice([2.0 ** -40, -3.0 * 2.0 ** -45, 2.0 ** -30], 1)[0]
        elif k == 3:
            v = np.where(rng.random(cols) < 0.7, 1.0, rng.choice([2.0 ** -28, 2.0 ** -52, 3.0 * 2.0 ** 24], cols))
        elif k == 4:
            v = (rng.random(cols) - 0.5) * 2.0 ** rng.integers(-20, 20, cols)
        elif k == 5:
            v = rng.standard_normal(cols) * np.where(rng.random(cols) < 0.5, 2.0 ** -135, 1.0)
        elif k == 6:
            v = rng.standard_normal(cols).astype(np.float32)
            pick = rng.random(cols)
            v[pick < 0.02] = 0.0
            v[(pick >= 0.02) & (pick < 0.04)] = -0.0
            v[(pick >= 0.04) & (pick < 0.045)] = np.inf
            v[(pick >= 0.045) & (pick < 0.05)] = -np.inf
            nan_at = pick > 0.995
            vb = v.view(np.uint32)
            vb[nan_at] = (rng.integers(1, 1 << 22, cols).astype(np.uint32) | np.uint32(0x7f800000))[nan_at]
        else:
            v = np.full(cols, -0.0)
        out[r] = v if v.dtype == np.float32 else v.astype(np.float32)
    return out


def _same_or_both_nan(got, want):
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    assert np.array_equal(got.view(np.uint32)[~nan], want.view(np.uint32)[~nan])


@pytest.mark.parametrize("rows,cols", [(8, 1), (8, 63), (8, 64), (16, 65), (16, 2047), (16, 2048), (16, 2049),
                                       (24, 8192), (9, 20000), (3, 100003)])
def test_auto_sum_serial_order_exact_and_rounding_chunks(rows, cols):
    """Block 1 (the serial order) bit for bit against the oracle's serial fold, on rows whose chunks are added out
    of order (no add rounds) and rows that round and take the value-by-value fold, at lengths on both sides of the
    64-value chunk and the 2,048-value segment; Sum and Mean; a view one column in (unaligned rows) as well."""
    rng = np.random.default_rng(rows * 11 + cols)
    xn = _serial_rows(rng, rows, cols)
    wide = np.zeros((rows, cols + 3), np.float32)
    wide[:, 1:1 + cols] = xn
    wt = torch.from_numpy(wide).cuda()
    for x in (torch.from_numpy(xn).cuda(), wt[:, 1:1 + cols]):
        _same_or_both_nan(ops.row_sum(x, accum="auto", block=1).cpu().numpy(), orc.row_sum_f32(xn))
        _same_or_both_nan(ops.reduce2d(x, "mean", 1, block=1).cpu().numpy(), orc.reduce2d_f32(xn, "mean", 1))


@pytest.mark.parametrize("dist", ["normal", "uniform", "ones_and_tiny"])
def test_auto_sum_serial_order_full_rows(dist):
    """8,192 rows of 8,192: N(0,1), U[0,1) and unit values with a tiny one in every 50, bit for bit."""
    rng = np.random.default_rng(6)
    if dist == "normal":
        xn = rng.standard_normal((8192, 8192), dtype=np.float32)
    elif dist == "uniform":
        xn = rng.random((8192, 8192), dtype=np.float32)
    else:
        xn = np.where(rng.random((8192, 8192)) < 0.02, np.float32(2.0 ** -35), np.float32(1.0)).astype(np.float32)
    got = ops.row_sum(torch.from_numpy(xn).cuda(), accum="auto", block=1).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), orc.row_sum_f32(xn, orc.max_threads()).view(np.uint32))


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 7), (17, 96), (5, 1000), (64, 4097), (33, 8192)])
@pytest.mark.parametrize("block", [1, 2, 4, 32, 128, 256, 1024])
def test_auto_sum_bit_exact_vs_oracle(rows, cols, block):
    rng = np.random.default_rng(rows * 131 + cols + block)
    x = (rng.standard_normal((rows, cols)) * 10.0 ** rng.integers(-3, 4, (rows, 1))).astype(np.float32)
    want = orc.row_sum_f32_documented(x, block)
    got = ops.row_sum(torch.from_numpy(x).cuda(), accum="auto", block=block).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("rows,cols,stride", [(7, 9000, 9000), (5, 1000, 1004), (1, 4096, 4096),
                                              (3000, 520, 520), (611, 20000, 20480)])
@pytest.mark.parametrize("block", [128, 256, 512, 1024])
def test_auto_sum_row_sets_bit_exact(rows, cols, stride, block):
    """Float4 rows at every block of 128 and up: rows shorter and longer than 8 * block (a thread's group
    of eight loads partial or repeated), row counts that leave a CTA's row set partial, row strides wider
    than the row."""
    rng = np.random.default_rng(rows + cols + block)
    full = (rng.standard_normal((rows, stride)) * 10.0 ** rng.integers(-3, 4, (rows, 1))).astype(np.float32)
    x = full[:, :cols]
    want = orc.row_sum_f32_documented(np.ascontiguousarray(x), block)
    got = ops.row_sum(torch.from_numpy(full).cuda()[:, :cols], accum="auto", block=block).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("block", [1, 4, 128, 256, 512, 1024])
def test_auto_sum_extreme_magnitudes_and_specials(block):
    """Denormals, cancelling tiny values, magnitudes near the f32 limit, signed zeros, every finite bit
    pattern, and rows holding Inf or NaN all match the documented order bit for bit (NaN results match as
    NaN)."""
    rng = np.random.default_rng(block + 7)
    rows, cols = 12, 2048
    x = np.zeros((rows, cols), dtype=np.float32)
    x[0] = (rng.standard_normal(cols) * 2.0 ** -140).astype(np.float32)            # denormals
    tiny = (rng.standard_normal(cols // 2) * 2.0 ** rng.integers(-149, -110, cols // 2)).astype(np.float32)
    x[1] = np.concatenate([tiny, -tiny[::-1]])                                       # cancels to ~0
    x[2] = (rng.uniform(-1.9, 1.9, cols) * 2.0 ** rng.integers(-149, 128, cols)).astype(np.float32)
    x[3] = (rng.standard_normal(cols) * 2.0 ** 126).astype(np.float32)              # f32 result overflows
    x[4] = -0.0                                                                      # all negative zeros
    x[5] = rng.integers(0, 2**32, cols, dtype=np.uint64).astype(np.uint32).view(np.float32)
    x[5][~np.isfinite(x[5])] = 1.0                                                   # every finite bit pattern
    x[6] = rng.standard_normal(cols)
    x[6, 1500] = np.inf
    x[7] = rng.standard_normal(cols)
    x[7, 3] = np.inf
    x[7, 2000] = -np.inf
    x[8] = rng.standard_normal(cols)
    x[8, 77] = np.nan
    x[9] = rng.standard_normal(cols)                                                 # shares a CTA with row 8
    x[10] = (rng.uniform(-1.9, 1.9, cols) * 2.0 ** 127).astype(np.float32)
    x[10, 5] = -np.inf
    x[11] = rng.standard_normal(cols).astype(np.float32)
    x[11, -1] = np.float32(3.4e38)
    want = orc.row_sum_f32_documented(x, block)
    got = ops.row_sum(torch.from_numpy(x).cuda(), accum="auto", block=block).cpu().numpy()
    both_nan = np.isnan(got) & np.isnan(want)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    assert np.array_equal(got.view(np.uint32)[~both_nan], want.view(np.uint32)[~both_nan])


def test_auto_sum_full_config_and_strided_rows():
    x = workloads.rowsum_input(device="cuda")
    for b in (256, 1024):
        got = ops.row_sum(x, accum="auto", block=b).cpu().numpy()
        want = orc.row_sum_f32_documented(x.cpu().numpy(), b, threads=orc.max_threads())
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), b
    # a row stride wider than the row (a view of every other column block)
    xv = x[:, :4000]
    got = ops.row_sum(xv, accum="auto", block=64).cpu().numpy()
    want = orc.row_sum_f32_documented(np.ascontiguousarray(xv.cpu().numpy()), 64)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# ---------------- row sum, f32 accumulation ----------------

def _check_f32_bound(x_np, got, depth):
    x64 = x_np.astype(np.float64)
    exact = x64.sum(axis=1)  # pairwise f64: its own error is far below the f32 bound
    sum_abs = np.abs(x64).sum(axis=1)
    err = np.abs(got.astype(np.float64) - exact)
    bound = gamma(depth) * sum_abs + 1e-300
    assert np.all(err <= bound), float(np.max(err / bound))
    return err, sum_abs


def test_f32_sum_full_config_meets_the_stated_tolerance():
    x = workloads.rowsum_input(device="cuda")
    got = ops.row_sum(x, accum="f32").cpu().numpy()
    xn = x.cpu().numpy()
    err, sum_abs = _check_f32_bound(xn, got, 13)
    assert np.all(err <= 2.0 ** -20 * sum_abs)
    # deterministic: same bytes on a second run
    assert np.array_equal(ops.row_sum(x, accum="f32").cpu().numpy().view(np.uint32), got.view(np.uint32))


def test_f32_sum_golden_corpus_bound():
    g = golden("float_sum_documented.json")
    x = _f32(g["x_f32_bits"]).reshape(g["rows"], g["cols"])
    got = ops.row_sum(torch.from_numpy(x).cuda(), accum="f32").cpu().numpy()
    _check_f32_bound(x, got, 13)


@pytest.mark.parametrize("rows,cols", [(1, 1), (7, 3), (9, 1023), (4, 4096), (2, 65536), (3, 100001)])
def test_f32_sum_odd_shapes(rows, cols):
    rng = np.random.default_rng(cols)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    got = ops.row_sum(torch.from_numpy(x).cuda(), accum="f32").cpu().numpy()
    # depth: 5 (tree of 8 float4 / 8 scalars) + sequential groups + 5 (warp) + 3 (block)
    groups = max(1, -(-cols // (256 * 8 * (4 if cols % 4 == 0 else 1))))
    _check_f32_bound(x, got, 13 + groups)


def test_empty_rows_and_columns():
    assert ops.row_sum(torch.empty(0, 5, device="cuda")).numel() == 0
    z = ops.row_sum(torch.empty(3, 0, device="cuda"), accum="auto", block=32)
    assert z.cpu().tolist() == [0.0, 0.0, 0.0]


# ---------------- max + argmax ----------------

def test_argmax_golden_corpus_and_tuple_fixture():
    g = golden("argmax.json")
    x = torch.from_numpy(np.array(g["x_bf16_bits"], np.uint16).view(np.int16)).cuda().view(torch.bfloat16)
    mx, am = ops.row_max_argmax(x, torch.int64)
    assert am.cpu().tolist() == g["argmax"]
    assert mx.cpu().numpy().view(np.uint32).tolist() == g["max_f32_bits"]
    t = torch.from_numpy(np.array([g["tuple_x_bf16_bits"]], np.uint16).view(np.int16)).cuda().view(torch.bfloat16)
    mx, am = ops.row_max_argmax(t)
    assert am.cpu().tolist() == [g["tuple_argmax"]] and mx.cpu().tolist() == [g["tuple_max"]]


def _bf16_rows(rng, rows, cols, kind):
    if kind == "ties":
        v = rng.integers(-3, 4, (rows, cols)).astype(np.float32)  # many exact ties
    elif kind == "normal":
        v = (rng.standard_normal((rows, cols)) + rng.uniform(-5, 5, (rows, 1))).astype(np.float32)
    else:  # specials: NaNs (both signs, payloads), infinities, signed zeros
        v = rng.standard_normal((rows, cols)).astype(np.float32)
        pick = rng.random((rows, cols))
        v[pick < 0.02] = np.inf
        v[(pick >= 0.02) & (pick < 0.04)] = -np.inf
        v[(pick >= 0.04) & (pick < 0.1)] = 0.0
        v[(pick >= 0.1) & (pick < 0.15)] = -0.0
    bits = torch.from_numpy(v).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16).copy()
    if kind == "specials":
        nan_at = rng.random((rows, cols)) < 0.01
        payload = rng.choice(np.array([0x7FC0, 0xFFC0, 0x7F81, 0xFF85, 0x7FFF], np.uint16), size=(rows, cols))
        bits[nan_at] = payload[nan_at]
        bits[0, :] = 0x8000  # a row of -0 only
        if rows > 1:
            bits[1, :] = 0xFF80  # all -inf
    return bits


@pytest.mark.parametrize("rows,cols", [(1, 1), (5, 7), (8, 8), (13, 1000), (64, 32000), (3, 65536), (2, 70000)])
@pytest.mark.parametrize("kind", ["ties", "normal", "specials"])
def test_max_argmax_bit_exact_vs_oracle(rows, cols, kind):
    rng = np.random.default_rng(rows * 7 + cols)
    bits = _bf16_rows(rng, rows, cols, kind)
    want_mx, want_am = orc.row_max_argmax_bf16(bits)
    x = torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)
    for idt in (torch.int32, torch.int64):
        mx, am = ops.row_max_argmax(x, idt)
        assert np.array_equal(am.cpu().numpy().astype(np.int64), want_am)
        assert np.array_equal(mx.cpu().numpy().view(np.uint32), want_mx.view(np.uint32))


def test_max_argmax_full_config():
    x = workloads.argmax_input(device="cuda")
    mx, am = ops.row_max_argmax(x, torch.int32)
    bits = x.view(torch.int16).cpu().numpy().view(np.uint16)
    want_mx, want_am = orc.row_max_argmax_bf16(bits, threads=orc.max_threads())
    assert np.array_equal(am.cpu().numpy().astype(np.int64), want_am)
    assert np.array_equal(mx.cpu().numpy().view(np.uint32), want_mx.view(np.uint32))


def test_max_argmax_unaligned_view_uses_general_path():
    rng = np.random.default_rng(1)
    bits = _bf16_rows(rng, 9, 801, "normal")
    x = torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)[:, 1:]  # 2-byte offset rows
    want_mx, want_am = orc.row_max_argmax_bf16(np.ascontiguousarray(bits[:, 1:]))
    mx, am = ops.row_max_argmax(x, torch.int64)
    assert np.array_equal(am.cpu().numpy(), want_am)
    assert np.array_equal(mx.cpu().numpy().view(np.uint32), want_mx.view(np.uint32))


def test_max_argmax_outputs_are_optional():
    x = workloads.argmax_input(64, 320, device="cuda")
    mx, _ = ops.row_max_argmax(x, want_argmax=False)
    _, am = ops.row_max_argmax(x, want_max=False)
    mx2, am2 = ops.row_max_argmax(x)
    assert torch.equal(mx, mx2) and torch.equal(am, am2)
