"""Pins the CPU oracle restatement (oracle/up_oracle.c) to the reference tests' own corpora and expectations
(tests/golden/*.json, written by tests/golden/make_golden.py). CPU only."""
import json
import os
import struct

import numpy as np
import pytest

import oracle as orc

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def bits_to_f32(bits):
    return np.array(bits, dtype=np.uint32).view(np.float32)


def test_documented_float_sum_order_matches_reference_rule():
    g = load("float_sum_documented.json")
    x = bits_to_f32(g["x_f32_bits"]).reshape(g["rows"], g["cols"])
    for b in g["blocks"]:
        got = orc.row_sum_f32_documented(x, b).view(np.uint32)
        assert got.tolist() == g["documented_f32_bits"][str(b)], f"block {b}"
    # block 1 is the serial order, which is the plan oracle's fold (plan_eval.rs:566-645).
    assert orc.row_sum_f32(x).view(np.uint32).tolist() == g["serial_f32_bits"]


def test_documented_order_threads_do_not_change_bytes():
    g = load("float_sum_documented.json")
    x = bits_to_f32(g["x_f32_bits"]).reshape(g["rows"], g["cols"])
    for b in g["blocks"]:
        assert np.array_equal(orc.row_sum_f32_documented(x, b, threads=4).view(np.uint32),
                              orc.row_sum_f32_documented(x, b).view(np.uint32))


def test_argmax_corpus_and_tuple_fixture():
    g = load("argmax.json")
    x = np.array(g["x_bf16_bits"], dtype=np.uint16)
    mx, am = orc.row_max_argmax_bf16(x)
    assert am.tolist() == g["argmax"]
    assert mx.view(np.uint32).tolist() == g["max_f32_bits"]
    t = np.array([g["tuple_x_bf16_bits"]], dtype=np.uint16)
    mx, am = orc.row_max_argmax_bf16(t)
    assert am.tolist() == [g["tuple_argmax"]] and mx.tolist() == [g["tuple_max"]]


@pytest.mark.parametrize("case", ["int_reduce_scan_5x6", "parallel_scan_4x45"])
def test_scan_corpora(case):
    g = load("scan_i32.json")["cases"][case]
    x = np.array(g["x"], dtype=np.int32)
    ops = {"sum": orc.OP_SUM, "max": orc.OP_MAX, "min": orc.OP_MIN}
    for key, exp in g["expected"].items():
        op, mode, direction = key.split("_")
        got = orc.scan_i32(x, ops[op], mode == "excl", direction == "rev")
        assert got.tolist() == exp, key


def test_int_row_reductions_wrap():
    g = load("scan_i32.json")
    x = np.array(g["cases"]["int_reduce_scan_5x6"]["x"], dtype=np.int32)
    for name, op in (("sum", orc.OP_SUM), ("max", orc.OP_MAX), ("min", orc.OP_MIN)):
        assert [orc.reduce_i32(r, op) for r in x] == g["row_reductions_5x6"][name]


def test_int_reductions_every_op_both_axes():
    """reduce2d_i32 against the reference corpus's Sum/Prod/Max/Min/And/Or/Xor over both axes."""
    g = load("scan_i32.json")
    x = np.array(g["cases"]["int_reduce_scan_5x6"]["x"], dtype=np.int32)
    for op, exp in g["reductions_5x6_both_axes"].items():
        assert orc.reduce2d_i32(x, op, 1).tolist() == exp["axis1"], op
        assert orc.reduce2d_i32(x, op, 0).tolist() == exp["axis0"], op


def test_float_mean_max_min_and_columns():
    """Documented-order Mean for every block, serial Max/Min, and the serial column Sum/Max of the float corpus."""
    g = load("float_sum_documented.json")
    x = np.array(g["x_f32_bits"], dtype=np.uint32).view(np.float32).reshape(g["rows"], g["cols"])
    bits = lambda a: np.asarray(a, dtype=np.float32).view(np.uint32).tolist()
    for b in g["blocks"]:
        assert bits(orc.row_mean_f32_documented(x, b)) == g["documented_mean_f32_bits"][str(b)], b
    assert bits(orc.reduce2d_f32(x, "mean", 1)) == g["documented_mean_f32_bits"]["1"]
    assert bits(orc.reduce2d_f32(x, "max", 1)) == g["max_f32_bits"]
    assert bits(orc.reduce2d_f32(x, "min", 1)) == g["min_f32_bits"]
    assert bits(orc.reduce2d_f32(x, "sum", 0)) == g["col_sum_f32_bits"]
    assert bits(orc.reduce2d_f32(x, "max", 0)) == g["col_max_f32_bits"]
    xt = np.ascontiguousarray(x.T)  # the corpus's rows as the columns of a [96, 5] input
    for b in g["col_documented_blocks"]:
        assert bits(orc.col_sum_f32_documented(xt, b)) == g["documented_f32_bits"][str(b)], b


def test_float_extremum_nan_and_zero_rules():
    """extremum_fold's rules on the oracle: the last NaN (quiet bit set) wins, and of +0/-0 the first is kept."""
    nan_a = np.array([0x7f800001], np.uint32).view(np.float32)[0]  # signalling payload 1
    nan_b = np.array([0xffc00002], np.uint32).view(np.float32)[0]
    x = np.array([[1.0, nan_a, 5.0, nan_b, 2.0], [-0.0, 0.0, -1.0, -0.0, -1.0], [0.0, -0.0, 3.0, 3.0, 0.0]],
                 np.float32)
    mx = orc.reduce2d_f32(x, "max", 1).view(np.uint32).tolist()
    mn = orc.reduce2d_f32(x, "min", 1).view(np.uint32).tolist()
    assert mx[0] == 0xffc00002 and mn[0] == 0xffc00002
    assert mx[1] == 0x80000000  # -0 first, +0 not strictly greater
    assert mn[2] == 0x00000000  # +0 first
    assert np.isnan(orc.reduce2d_f32(np.zeros((3, 0), np.float32), "mean", 1)).all()


def test_scatter_corpus_and_bincount():
    """The scatter store against the launched-scatter corpus (duplicates, out-of-range targets, a pre-filled
    destination) for Add/Max/Min, and bincount's data."""
    g = load("scatter.json")
    src, dst = g["src"], g["dst"]
    upd = np.array(g["updates"], np.int32).reshape(src)
    idx = np.array(g["index"], np.int32).reshape(src)
    init = np.array(g["init"], np.int32).reshape(dst)
    for combine, exp in g["expected"].items():
        assert orc.scatter(upd, idx, init, combine).reshape(-1).tolist() == exp, combine
    b = g["bincount"]
    for dt in (np.int32, np.int64):
        assert orc.bincount(np.array(b["x"], dt), np.zeros(b["bins"], np.int32)).tolist() == b["counts"]


def test_float_scatter_serial_sum_is_in_the_band():
    """The serial f32 scatter-add of the band corpus lies inside gamma_(n-1) * sum|terms| of each cell's exact sum."""
    f = load("scatter.json")["float_band"]
    upd = np.array(f["updates_f32_bits"], np.uint32).view(np.float32).reshape(f["src"])
    tgt = np.array(f["targets"], np.int32).reshape(f["src"])
    init = np.array(f["init_f32_bits"], np.uint32).view(np.float32).reshape(f["dst"])
    got = orc.scatter(upd, tgt, init, "add").reshape(-1)
    u = 2.0 ** -24
    for c, (total, mag, n) in enumerate(f["cell_sum_abs_n"]):
        k = (n - 1) * u
        assert abs(float(got[c]) - total) <= k / (1 - k) * mag, c


def test_chunked_scan_equals_serial_scan():
    rng = np.random.default_rng(7)
    x = rng.integers(-(2**31), 2**31 - 1, size=100_003, dtype=np.int64).astype(np.int32)
    for op in (orc.OP_SUM, orc.OP_MAX, orc.OP_MIN):
        for excl in (False, True):
            assert np.array_equal(orc.scan_i32_chunked(x, op, excl, threads=5), orc.scan_i32(x, op, excl))


@pytest.mark.parametrize("policy,code", [("skip", orc.OOB_SKIP), ("clamp", orc.OOB_CLAMP),
                                         ("zero_fill", orc.OOB_ZERO_FILL)])
def test_gather_oob_pool(policy, code):
    g = load("gather_oob.json")
    table = np.array(g["table_f32_bits"], dtype=np.uint32)
    ids = np.array(g["ids_i32"], dtype=np.int32)
    out = np.full((ids.size, table.shape[1]), 0xABABABAB, dtype=np.uint32)
    orc.gather_rows(table, ids, code, out=out)
    assert out.tolist() == g["expected_f32_bits"][policy]


def test_gather_index_dtypes_agree_on_nonnegative_ids():
    rng = np.random.default_rng(3)
    table = rng.integers(0, 2**16, size=(50, 8), dtype=np.uint16)
    ids = rng.integers(0, 50, size=200)
    outs = [orc.gather_rows(table, ids.astype(dt), orc.OOB_SKIP) for dt in (np.int32, np.int64, np.uint32)]
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])
    assert np.array_equal(outs[0], table[ids])


def test_dequant_gemm_kat_and_packing():
    g = load("dequant_kat.json")
    packed = np.array(g["packed"], dtype=np.uint8)
    for signed, key in ((True, "expected_signed"), (False, "expected_unsigned")):
        got = orc.dequant_gemm_kat(packed, signed, g["zero"], g["scale"], g["x"], g["R"], g["K"], g["C"], g["GROUP"])
        assert got.tolist() == g[key]
    kat = g["packing_kat"]
    assert orc.i4_value(np.array([kat["i4_1_2"]], np.uint8), 0) == 1
    assert orc.i4_value(np.array([kat["i4_1_2"]], np.uint8), 1) == 2
    b = np.array([kat["i4_m1_m8"]], np.uint8)
    assert (orc.i4_value(b, 0), orc.i4_value(b, 1)) == (-1, -8)
    for v in range(-8, 8):
        byte = np.array([(v & 0xF) | ((v & 0xF) << 4)], np.uint8)
        assert orc.i4_value(byte, 0) == v and orc.i4_value(byte, 1) == v


def test_bf16_codec_matches_rne_and_quiet_nan_rule():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(11)
    vals = np.concatenate([rng.standard_normal(2000).astype(np.float32),
                           np.array([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, 3.0e38, 1e-40], np.float32),
                           # exact ties at the bf16 rounding point, both parities
                           np.array([1.0 + 2**-8, 1.0 + 3 * 2**-8], np.float32)])
    got = np.array([orc.f32_to_bf16(float(v)) for v in vals], np.uint16)
    want = torch.from_numpy(vals).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(got, want)
    # float_codec.rs:262-264: a NaN keeps its top half and gets the quiet bit.
    snan = struct.unpack("<f", struct.pack("<I", 0x7F810000))[0]
    assert orc.f32_to_bf16(snan) == 0x7FC1


def test_f16_codec_round_trips_every_finite_half():
    for h in range(0, 0x10000, 7):
        if (h & 0x7C00) == 0x7C00:
            continue
        v = orc.f16_to_f64(h)
        assert orc.f32_to_f16(v) == h, hex(h)


def test_w4a16_oracle_matches_direct_f64_sum():
    rng = np.random.default_rng(5)
    m, n, k, group = 3, 4, 256, 128
    w = rng.integers(-8, 8, size=(n, k))
    packed = ((w[:, 0::2] & 0xF) | ((w[:, 1::2] & 0xF) << 4)).astype(np.uint8)
    scale = rng.uniform(0.005, 0.02, size=(n, k // group)).astype(np.float16)
    x = rng.standard_normal((m, k)).astype(np.float32)
    xb = np.array([[orc.f32_to_bf16(float(v)) for v in row] for row in x], np.uint16)
    out, exact, abs_sum = orc.w4a16(packed, scale.view(np.uint16), xb, m, n, k, group)
    xf = (xb.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    sf = np.repeat(scale.astype(np.float64), group, axis=1)
    direct = xf @ (w * sf).T
    assert np.allclose(exact, direct, rtol=1e-14, atol=1e-14)
    assert np.allclose(abs_sum, np.abs(xf) @ np.abs(w * sf).T, rtol=1e-14)
    assert out.tolist() == [[orc.f64_to_bf16(v) for v in row] for row in exact]


def _ulps(a, b):
    """The f32 ulp distance between two arrays (the ordering key of row_reduce_agrees.rs:226-240)."""
    ka = a.view(np.int32).astype(np.int64)
    kb = b.view(np.int32).astype(np.int64)
    ka = np.where(ka < 0, -(1 << 31) - ka, ka)
    kb = np.where(kb < 0, -(1 << 31) - kb, kb)
    return int(np.abs(ka - kb).max())


def test_row_reduce_oracle_matches_the_reference_written_orders():
    """The centred quotient in the written order is bit-exact for every block
    (a_two_stage_op_follows_the_written_order_bit_for_bit); softmax and RMS norm equal the serial lift at block 1
    and stay within the reference's few-ulp band at every other block."""
    g = load("row_reduce.json")
    x = np.array(g["gentle_f32_bits"], np.uint32).view(np.float32)
    for b in g["blocks"]:
        want = np.array(g["centred_f32_bits"][str(b)], np.uint32)
        assert np.array_equal(orc.row_reduce_f32(x, "centred", b).view(np.uint32), want), b
    for form, key in (("softmax", "softmax_serial_f32_bits"), ("rms_norm", "rms_norm_serial_f32_bits")):
        want = np.array(g[key], np.uint32).view(np.float32)
        assert np.array_equal(orc.row_reduce_f32(x, form, 1).view(np.uint32), want.view(np.uint32)), form
        for b in g["blocks"]:
            assert _ulps(orc.row_reduce_f32(x, form, b), want) <= g["ulp_band"], (form, b)


def _splitk_harness_corpus():
    """splitk_validate.cu:53-61: rows 100, cols 64, in[i] = ((i % 37) - 18) * 0.25, column 0 all -0.0."""
    rows, cols = 100, 64
    x = np.array([((i % 37) - 18) * 0.25 for i in range(rows * cols)], np.float32).reshape(rows, cols)
    x[:, 0] = -0.0
    return x


def test_splitk_oracle_meets_the_reference_harness():
    """The split-K harness's checks (splitk_validate.cu:53-125): ragged chunks against the f64 sum, the zero-seeded
    fold maps an all -0 column to +0, and n_chunks = 1 is the serial fold bit for bit."""
    x = _splitk_harness_corpus()
    exact = x.astype(np.float64).sum(axis=0)
    got = orc.col_sum_f32_splitk(x, 3)
    denom = np.maximum(np.abs(exact), 1.0)
    assert (np.abs(got.astype(np.float64) - exact) / denom).max() < 1e-5
    assert got.view(np.uint32)[0] == 0x00000000
    rng = np.random.default_rng(4)
    y = (rng.standard_normal((333, 40)) * 10.0 ** rng.integers(-3, 4, (333, 1))).astype(np.float32)
    for mean in (False, True):
        serial = orc.reduce2d_f32(y, "mean" if mean else "sum", 0)
        assert np.array_equal(orc.col_sum_f32_splitk(y, 1, mean).view(np.uint32), serial.view(np.uint32))


def test_window_oracle_matches_the_reference_corpora():
    """kernel_window_agrees.rs and kernel_int_window_agrees.rs: every pool over the padded, strided and dilated
    geometries, the two Mean divisors, a NaN kept by Max/Min, the ascending f64 accumulator, wrapping integer sums."""
    g = load("window.json")
    vals = np.array(g["values_f32_bits"], np.uint32).view(np.float32)
    for name, c in g["cases"].items():
        rows, k_in, size, stride, dil, pad, inc, k_out = c["geometry"]
        x = np.resize(vals, rows * k_in).reshape(rows, k_in)
        for op, want in c["expected_f32_bits"].items():
            got = orc.window(x, op, size, stride, dil, pad, k_out, bool(inc))
            assert np.array_equal(got.view(np.uint32), np.array(want, np.uint32)), (name, op)
    x = np.array(g["nan_row_f32_bits"], np.uint32).view(np.float32)[None]
    for op, want in g["nan_row_expected"].items():
        assert np.array_equal(orc.window(x, op, 3, 3).view(np.uint32)[0], np.array(want, np.uint32)), op
    x = np.array(g["ascending_row_f32_bits"], np.uint32).view(np.float32)[None]
    assert orc.window(x, "sum", 9).view(np.uint32)[0].tolist() == g["ascending_sum_f32_bits"]
    ints = np.array(g["int_values"], np.int64).astype(np.int32)
    for name, c in g["int_cases"].items():
        rows, k_in, size, stride, dil, pad, _, k_out = c["geometry"]
        x = np.resize(ints, rows * k_in).reshape(rows, k_in)
        for op, want in c["expected"].items():
            assert orc.window(x, op, size, stride, dil, pad, k_out).tolist() == want, (name, op)


def test_im2col_oracle_matches_the_definition():
    """kernel_im2col_agrees.rs: distinct values with a NaN and a -0 planted, over padding, batch and channels,
    stride, dilation and a rectangular window."""
    for name, c in load("im2col.json").items():
        x = np.array(c["x_f32_bits"], np.uint32).view(np.float32).reshape(c["shape"])
        got = orc.im2col(x, c["kernel"], c["stride"], c["pad"], c["dilation"])
        assert got.view(np.uint32).reshape(-1).tolist() == c["expected_f32_bits"], name
