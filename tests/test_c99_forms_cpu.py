"""The C99-emitter restatements (oracle/c99_forms.c), timed as a CPU baseline, agree with the oracle.

They serialize the KernelFns of the lifts the way the reference's C99 emitter spells them (one loop over the threads
of a block per barrier-free run), so they must produce the oracle's bytes: the serial reduction lift is the oracle's
f64 fold, the launched block-tree lift is the documented order, both scan forms are the serial scan bit for bit,
the gather and argmax loops are the oracle's, and the W4A16 cell loop lies inside the f32-accumulation bound.
"""
import numpy as np
import pytest

import oracle as orc


def test_row_sum_forms():
    rng = np.random.default_rng(1)
    for shape in ((37, 1000), (1, 1), (5, 8192), (64, 3)):
        x = (rng.standard_normal(shape) * 1e3).astype(np.float32)
        assert np.array_equal(orc.c99_row_sum(x).view(np.uint32), orc.row_sum_f32(x).view(np.uint32))
        for b in (1, 32, 256, 1024):
            assert np.array_equal(orc.c99_row_sum(x, b).view(np.uint32),
                                  orc.row_sum_f32_documented(x, b).view(np.uint32)), (shape, b)


@pytest.mark.parametrize("n", [1, 5, 1000, 100_003])
def test_scan_forms(n):
    rng = np.random.default_rng(n)
    x = rng.integers(-(2 ** 31), 2 ** 31 - 1, n, dtype=np.int64).astype(np.int32)
    for op in (orc.OP_SUM, orc.OP_MAX):
        for ex in (False, True):
            want = orc.scan_i32(x, op, ex)
            assert np.array_equal(orc.c99_scan(x, op, ex), want)
            for b in (1, 64, 1024):
                assert np.array_equal(orc.c99_scan(x, op, ex, b), want), (op, ex, b)


@pytest.mark.parametrize("oob", [orc.OOB_SKIP, orc.OOB_CLAMP, orc.OOB_ZERO_FILL])
def test_gather_form(oob):
    rng = np.random.default_rng(oob)
    table = rng.integers(0, 2 ** 16, (300, 64), dtype=np.uint16)
    ids = rng.integers(-20, 320, 1000).astype(np.int32)
    pre = rng.integers(0, 2 ** 16, (1000, 64), dtype=np.uint16)
    got = orc.c99_gather(table, ids, oob, pre.copy())
    want = orc.gather_rows(table, ids, oob, out=pre.copy())
    assert np.array_equal(got, want)


def test_argmax_form():
    rng = np.random.default_rng(4)
    x = rng.standard_normal((50, 777)).astype(np.float32)
    bits = (x.view(np.uint32) >> 16).astype(np.uint16)
    bits[3, 10] = 0x7FC0   # a NaN wins
    bits[4, 7] = bits[4, 9] = 0x4300  # a tie goes to the lower index
    mx, am = orc.c99_row_max_argmax(bits)
    wmx, wam = orc.row_max_argmax_bf16(bits)
    assert np.array_equal(am, wam)
    assert np.array_equal(mx.view(np.uint32)[~np.isnan(mx)], wmx.view(np.uint32)[~np.isnan(wmx)])
    assert np.isnan(mx[3]) and np.isnan(wmx[3])


def test_w4a16_form_within_the_f32_bound():
    rng = np.random.default_rng(6)
    m, n, k, g = 3, 40, 512, 128
    w = rng.integers(0, 256, (n, k // 2), dtype=np.uint8)
    s = np.array([orc.f32_to_f16(v) for v in rng.uniform(0.005, 0.02, n * k // g)], np.uint16).reshape(n, k // g)
    x = np.array([orc.f32_to_bf16(v) for v in rng.standard_normal(m * k)], np.uint16).reshape(m, k)
    got = orc.c99_w4a16(w, s, x, m, n, k, g)
    _, exact, abs_sum = orc.w4a16(w, s, x, m, n, k, g)
    gv = (got.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    u = 2.0 ** -24
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(exact), 2.0 ** -126))) - 7)
    assert np.all(np.abs(gv - exact) <= 0.5 * ulp + (k + 2) * u * abs_sum * 1.01)
