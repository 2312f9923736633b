"""Writes the golden fixtures under tests/golden/ from the reference's own test corpora.

The reference (Unpopped, Rust) cannot be built here, so its tests' corpora and the expectation rules those
tests compute *independently of the oracle* are restated below in plain Python, one function per
reference test, each citing the test it follows (paths relative to the Unpopped repository). The C oracle
restatement (oracle/up_oracle.c) is then pinned against these fixtures by tests/test_oracle_golden.py.

Run: python tests/golden/make_golden.py   (deterministic; rewrites the JSON files beside it)
"""
from __future__ import annotations

import functools
import json
import math
import os
import struct

HERE = os.path.dirname(os.path.abspath(__file__))
M64 = (1 << 64) - 1
I32_MIN, I32_MAX = -(1 << 31), (1 << 31) - 1


def f32(x: float) -> float:
    return struct.unpack("<f", struct.pack("<f", x))[0]


def f32_bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


def bf16_bits_exact(x: float) -> int:
    """bf16 bits of a value that bf16 holds exactly (the corpora below only hold such values)."""
    b = f32_bits(x)
    if math.isnan(x):
        return 0x7FC0
    assert b & 0xFFFF == 0, f"{x} is not exact in bf16"
    return b >> 16


def wrap32(v: int) -> int:
    v &= 0xFFFFFFFF
    return v - (1 << 32) if v >= (1 << 31) else v


# --- crates/unpopped/tests/kernel_parallel_reduction_float_sum_bound.rs -------------------------------

def lcg(state: list) -> float:
    """`lcg` (float_sum_bound.rs:40-46): a u64 LCG, the top 53 bits as a fraction in [0, 1)."""
    state[0] = (state[0] * 6364136223846793005 + 1442695040888963407) & M64
    return (state[0] >> 11) / float(1 << 53)


def float_sum_corpus() -> list:
    """`corpus` (float_sum_bound.rs:48-72): five rows of 96 values, interleaved then regrouped row-major."""
    rows, cols = 5, 96
    s = [0x9E3779B97F4A7C15]
    v = []
    for c in range(cols):
        v.append(1.0e-3 + 1.0e3 * lcg(s))
        big = 1.0e8 if c % 2 == 0 else -1.0e8
        v.append(1.0 + lcg(s) if c % 7 == 0 else big)
        huge = 1.0e30 if c % 2 == 0 else -1.0e30 * (1.0 + 1e-3 * lcg(s))
        v.append(huge * 1.0e-20)
        v.append(0.1)
        v.append((lcg(s) - 0.5) * 2.0e5)
    return [[v[c * rows + r] for c in range(cols)] for r in range(rows)]


def documented(xs: list, block: int, mean: bool = False) -> float:
    """`documented` (float_sum_bound.rs:147-170) at F32, Sum: thread t folds t, t+B, ... into an f64, then
    acc[t] += acc[t+s] for s = B/2 .. 1, one rounding to f32. Mean divides the f64 total by the extent before
    that rounding (kernel_lift/block_reduce.rs:13-23)."""
    acc = []
    for t in range(block):
        a = 0.0
        for x in xs[t::block]:
            a = a + x
        acc.append(a)
    s = block // 2
    while s > 0:
        for t in range(s):
            acc[t] = acc[t] + acc[t + s]
        s //= 2
    return f32(acc[0] / len(xs) if mean else acc[0])


def serial_extremum(xs: list, is_max: bool) -> float:
    """extremum_fold (oracle/plan_contract.rs:179-210) on finite values: the first element, replaced by a strictly
    better one."""
    acc = xs[0]
    for x in xs[1:]:
        if (x > acc) if is_max else (x < acc):
            acc = x
    return acc


def golden_float_sum() -> dict:
    rows = [[f32(x) for x in r] for r in float_sum_corpus()]  # `values(F32)`: the f32 roundings
    blocks = [1, 2, 8, 32, 128, 16]  # GEOMETRIES' block sizes (float_sum_bound.rs:37)
    return {
        "source": "crates/unpopped/tests/kernel_parallel_reduction_float_sum_bound.rs:37-170",
        "rows": 5, "cols": 96,
        "x_f32_bits": [[f32_bits(x) for x in r] for r in rows],
        "blocks": blocks,
        "documented_f32_bits": {str(b): [f32_bits(documented(r, b)) for r in rows] for b in blocks},
        "serial_f32_bits": [f32_bits(documented(r, 1)) for r in rows],
        "documented_mean_f32_bits": {str(b): [f32_bits(documented(r, b, True)) for r in rows] for b in blocks},
        "max_f32_bits": [f32_bits(serial_extremum(r, True)) for r in rows],
        "min_f32_bits": [f32_bits(serial_extremum(r, False)) for r in rows],
        "col_sum_f32_bits": [f32_bits(documented([r[c] for r in rows], 1)) for c in range(96)],
        # the corpus's transpose as a [96, 5] input reduced over its outer axis: each column of that input is a row
        # of the corpus, so the documented order over the outer axis gives the row sums above
        "col_documented_blocks": [1, 2, 8, 32, 16],
        "col_max_f32_bits": [f32_bits(serial_extremum([r[c] for r in rows], True)) for c in range(96)],
    }


# --- crates/unpopped/tests/reduce_argmax.rs + kernel_collective_tuple.rs --------------------------------

def argmax_corpus() -> list:
    """`corpus` (reduce_argmax.rs:31-41): ties, a NaN first, a NaN in the middle, all negative, signed
    zeros, all NaN."""
    n = float("nan")
    return [
        [3.0, 9.0, 9.0, 1.0, 1.0, 2.0],
        [n, 1.0, 2.0, 3.0, -4.0, 5.0],
        [1.0, 4.0, n, 7.0, n, 2.0],
        [-1.0, -2.0, -3.0, -4.0, -5.0, -6.0],
        [0.0, -0.0, 0.0, -0.0, 0.0, -0.0],
        [n, n, n, n, n, n],
    ]


def greater(x: float, y: float) -> bool:
    """`greater` (reduce_argmax.rs:76-78): NaN is the greatest value and equal to NaN."""
    return (math.isnan(x) and not math.isnan(y)) or (not math.isnan(x) and not math.isnan(y) and x > y)


def arg_of(xs: list) -> int:
    """`arg_of` for ArgMax (reduce_argmax.rs:80-95): only a strictly greater element replaces."""
    best = 0
    for i in range(1, len(xs)):
        if greater(xs[i], xs[best]):
            best = i
    return best


def max_of(xs: list):
    """The Max fold's rule (ReduceOp::Max, ir.rs:1700-1748; extremum_fold, plan_contract.rs:179-210): a NaN
    propagates, and of equal maxima the first is kept (so a row of signed zeros keeps the first zero's
    sign). Returns f32 bits; a NaN row gives the canonical quiet NaN the corpus holds."""
    have, acc = False, 0.0
    for v in xs:
        if not have or math.isnan(v) or v > acc:
            acc = v
        have = True
    return 0x7FC00000 if math.isnan(acc) else f32_bits(acc)


def golden_argmax() -> dict:
    rows = argmax_corpus()
    tup = [3.0, 7.0, -1.0, 7.0, 0.0, 9.0, 9.0, 2.0]
    return {
        "source": "crates/unpopped/tests/reduce_argmax.rs:31-100; kernel_collective_tuple.rs:6-12",
        "x_bf16_bits": [[bf16_bits_exact(v) for v in r] for r in rows],
        "argmax": [arg_of(r) for r in rows],
        "max_f32_bits": [max_of(r) for r in rows],
        "tuple_x_bf16_bits": [bf16_bits_exact(v) for v in tup],
        "tuple_argmax": 5,  # hand-derived in kernel_collective_tuple.rs:8-9: (9, 5)
        "tuple_max": 9.0,
    }


# --- crates/unpopped/tests/kernel_int_reduce_scan_agrees.rs + kernel_parallel_scan_agrees.rs ---------------

def int_corpus_i32() -> list:
    """`corpus(I32)` (kernel_int_reduce_scan_agrees.rs:28-45): wrap-around, all negative, ties, big."""
    hi, lo, big = I32_MAX, I32_MIN, 100_000
    return [
        [hi, 1, -1, 2, hi, 3],
        [-1, -2, -3, -4, -5, -6],
        [7, 7, 7, -7, lo, 0],
        [big, big, 3, 1, -1, 2],
        [4, 9, 2, 8, 6, 5],
    ]


def parallel_scan_ints() -> list:
    """`int_values` (kernel_parallel_scan_agrees.rs:60-64): ((i*37+11) % 41) - 20 over 4 x 45."""
    vals = [((i * 37 + 11) % 41) - 20 for i in range(4 * 45)]
    return [vals[r * 45:(r + 1) * 45] for r in range(4)]


def scan_def(row: list, op: str, exclusive: bool, reverse: bool) -> list:
    """Access::Scan's definition (ir.rs:2153-2195): the running combine along the row (from its end when
    reversed); exclusive shifts by one with the monoid identity first (Sum 0, Max the type minimum, Min the
    type maximum); an integer Sum wraps at 32 bits."""
    ident = {"sum": 0, "max": I32_MIN, "min": I32_MAX}[op]
    comb = {"sum": lambda a, b: wrap32(a + b), "max": max, "min": min}[op]
    k = len(row)
    out = [0] * k
    acc = ident
    for jj in range(k):
        j = k - 1 - jj if reverse else jj
        if exclusive:
            out[j] = acc
            acc = comb(acc, row[j])
        else:
            acc = comb(acc, row[j])
            out[j] = acc
    return out


def golden_scan() -> dict:
    cases = {}
    for name, rows in (("int_reduce_scan_5x6", int_corpus_i32()), ("parallel_scan_4x45", parallel_scan_ints())):
        exp = {}
        for op in ("sum", "max", "min"):
            for excl in (False, True):
                for rev in (False, True):
                    key = f"{op}_{'excl' if excl else 'incl'}_{'rev' if rev else 'fwd'}"
                    exp[key] = [scan_def(r, op, excl, rev) for r in rows]
        cases[name] = {"x": rows, "expected": exp}
    # Reductions of the wrap corpus along the last axis (fold_step / extremum_fold with wrap at the store).
    red = {
        "sum": [wrap32(sum(r)) for r in int_corpus_i32()],
        "max": [max(r) for r in int_corpus_i32()],
        "min": [min(r) for r in int_corpus_i32()],
    }
    # Every integer ReduceOp (ir.rs:1700-1748) over both axes of the corpus, as reduce_both runs them
    # (kernel_int_reduce_scan_agrees.rs:80-110): Sum and Prod wrap at the dtype's width, Max/Min exact, the bit
    # folds seeded by the first element.
    folds = {
        "sum": lambda v: wrap32(sum(v)),
        "prod": lambda v: wrap32(functools.reduce(lambda a, b: a * b, v, 1)),
        "max": max, "min": min,
        "and": lambda v: functools.reduce(lambda a, b: a & b, v),
        "or": lambda v: functools.reduce(lambda a, b: a | b, v),
        "xor": lambda v: functools.reduce(lambda a, b: a ^ b, v),
    }
    ic = int_corpus_i32()
    axes = {op: {"axis1": [f(r) for r in ic], "axis0": [f([r[c] for r in ic]) for c in range(len(ic[0]))]}
            for op, f in folds.items()}
    return {
        "source": "crates/unpopped/tests/kernel_int_reduce_scan_agrees.rs:28-45; "
                  "kernel_parallel_scan_agrees.rs:60-64",
        "cases": cases,
        "row_reductions_5x6": red,
        "reductions_5x6_both_axes": axes,
    }


# --- crates/unpopped/tests/kernel_parallel_gather_agrees.rs ---------------------------------------------------

def golden_gather() -> dict:
    """The 1-D-ids case (kernel_parallel_gather_agrees.rs:22-105): data [5, 6] f32 = i*1.5 - 7, out [9, 6]
    pre-filled with 0xAB, ids from the OOB pool; the expectation is the gather's definition (clamped load,
    OOB as a store predicate; plan_eval.rs:363-385)."""
    data = [[f32((r * 6 + c) * 1.5 - 7.0) for c in range(6)] for r in range(5)]
    extent = 5
    pool = [0, extent - 1, 1, extent, extent + 7, 2, -1, I32_MIN, I32_MAX, -3]
    n = 9
    ids = [pool[(i * 3 + i // 4) % len(pool)] for i in range(n)]
    prefill = struct.unpack("<I", bytes([0xAB] * 4))[0]
    exp = {}
    for pol in ("skip", "clamp", "zero_fill"):
        out = []
        for i in range(n):
            raw = ids[i]
            g = min(max(raw, 0), extent - 1)
            if raw < 0 or raw >= extent:
                if pol == "skip":
                    out.append([prefill] * 6)
                    continue
                if pol == "zero_fill":
                    out.append([0] * 6)
                    continue
            out.append([f32_bits(v) for v in data[g]])
        exp[pol] = out
    return {
        "source": "crates/unpopped/tests/kernel_parallel_gather_agrees.rs:22-105",
        "table_f32_bits": [[f32_bits(v) for v in r] for r in data],
        "ids_i32": ids,
        "prefill_byte": 0xAB,
        "expected_f32_bits": exp,
    }


# --- crates/unpopped/tests/support/dequant.rs + sub_byte_packing.rs --------------------------------------------

def golden_dequant() -> dict:
    """The dequant GEMM KAT (support/dequant.rs:13-20,146-178): R=4, K=8, C=4, GROUP=4; nibble(r,k) =
    (r*5 + k*3 + 1) % 16 packed low nibble first; zero = (i % 3) - 1, scale = 1 + (i*2 % 3),
    x = (i*7 % 9) - 4 laid out x[k*C + c]; out[r][c] = sum_k (w - zero) * scale * x."""
    R, K, C, GROUP = 4, 8, 4, 4
    G = K // GROUP
    nib = [[(r * 5 + k * 3 + 1) % 16 for k in range(K)] for r in range(R)]
    flat = [v for row in nib for v in row]
    packed = [flat[i] | (flat[i + 1] << 4) for i in range(0, len(flat), 2)]
    zero = [(i % 3) - 1 for i in range(R * G)]
    scale = [1 + (i * 2 % 3) for i in range(R * G)]
    x = [(i * 7 % 9) - 4 for i in range(K * C)]

    def ref(signed: bool):
        def w(r, k):
            v = nib[r][k]
            return v - 16 if signed and v >= 8 else v
        out = []
        for r in range(R):
            for c in range(C):
                out.append(sum((w(r, k) - zero[r * G + k // GROUP]) * scale[r * G + k // GROUP] * x[k * C + c]
                               for k in range(K)))
        return out

    return {
        "source": "crates/unpopped/tests/support/dequant.rs:13-20,146-178; tests/sub_byte_packing.rs:24-60",
        "R": R, "K": K, "C": C, "GROUP": GROUP,
        "packed": packed, "zero": zero, "scale": scale, "x": x,
        "expected_signed": ref(True), "expected_unsigned": ref(False),
        # sub_byte_packing.rs: [1, 2] -> 0x21; i4 [-1, -8] and u4 [15, 8] share the byte 0x8F.
        "packing_kat": {"i4_1_2": 0x21, "i4_m1_m8": 0x8F, "u4_15_8": 0x8F},
    }


# --- crates/unpopped/tests/kernel_parallel_scatter_agrees.rs, kernel_bincount_agrees.rs,
#     kernel_parallel_float_scatter_band.rs -----------------------------------------------------------------------

def golden_scatter() -> dict:
    """The launched-scatter corpus (kernel_parallel_scatter_agrees.rs:19-56): updates [9, 4] = (i*7 % 11) - 5, a
    full-shape index with duplicates and out-of-range targets, a destination [5, 4] pre-filled with i - 3; expected
    by the scatter store's definition (oracle/plan_eval.rs:430-490): serial, skip targets outside [0, 5), integer
    add/max/min. bincount's data (kernel_bincount_agrees.rs:26-34) into 6 zeroed bins. The float band corpus
    (kernel_parallel_float_scatter_band.rs:24-100): updates, targets and initial values, with each cell's exact sum,
    sum of magnitudes and term count."""
    src, dst = (9, 4), (5, 4)
    upd = [(i * 7 % 11) - 5 for i in range(src[0] * src[1])]
    targets = [0, 4, 4, 1, 7, -2, 0, 2, 4, 3, 0, 1, 9, 2, 2, 4, 0, 1]
    idx = [targets[(i * 5 + i // 4) % len(targets)] for i in range(src[0] * src[1])]
    init = [i - 3 for i in range(dst[0] * dst[1])]
    exp = {}
    for name, f in (("add", lambda a, b: wrap32(a + b)), ("max", max), ("min", min)):
        out = list(init)
        for i in range(src[0] * src[1]):
            t = idx[i]
            if 0 <= t < dst[0]:
                c = t * dst[1] + i % src[1]
                out[c] = f(out[c], upd[i])
        exp[name] = out
    bc_data = [0, 2, 2, 0, 5, 1, 0, -1, 6, 9, 2, 1, -7, 0]
    counts = [0] * 6
    for v in bc_data:
        if 0 <= v < 6:
            counts[v] += 1
    fsrc, fdst = (12, 3), (4, 3)

    def f_update(i):
        sign = -1.0 if (i * 7 + i // 5) % 3 == 0 else 1.0
        return f32(sign * f32(1.0000001) * 2.0 ** (((i * 11) % 26) - 3))

    def f_target(i):
        return [0, 0, 1, 0, 0, 5, 1, 0, -1, 0, 1, 0][(i // fsrc[1]) % 12]

    def f_init(i):
        return f32(i * 0.375 - 2.0)

    fu = [f_update(i) for i in range(fsrc[0] * fsrc[1])]
    ft = [f_target(i) for i in range(fsrc[0] * fsrc[1])]
    fi = [f_init(i) for i in range(fdst[0] * fdst[1])]
    truth = []
    for c in range(fdst[0] * fdst[1]):
        total, mag, n = fi[c], abs(fi[c]), 1
        for i in range(fsrc[0] * fsrc[1]):
            t = ft[i]
            if 0 <= t < fdst[0] and t * fdst[1] + i % fsrc[1] == c:
                total += fu[i]
                mag += abs(fu[i])
                n += 1
        truth.append([total, mag, n])
    return {
        "source": "crates/unpopped/tests/kernel_parallel_scatter_agrees.rs:19-56; kernel_bincount_agrees.rs:26-34; "
                  "kernel_parallel_float_scatter_band.rs:24-107",
        "src": list(src), "dst": list(dst), "updates": upd, "index": idx, "init": init, "expected": exp,
        "bincount": {"x": bc_data, "bins": 6, "counts": counts},
        "float_band": {"src": list(fsrc), "dst": list(fdst), "updates_f32_bits": [f32_bits(v) for v in fu],
                       "targets": ft, "init_f32_bits": [f32_bits(v) for v in fi], "cell_sum_abs_n": truth},
    }


# --- crates/unpopped/tests/kernel_parallel_row_reduce_agrees.rs ---------------------------------------

def row_reduce_corpus() -> list:
    """`corpus` (row_reduce_agrees.rs:36-55): benign positives, a cancelling row, huge/tiny alternation, 0.1,
    mixed signs; five rows of 96, generated column by column."""
    rows, cols = 5, 96
    s = [0x9E3779B97F4A7C15]
    per_col = []
    for c in range(cols):
        big = 1.0e8 if c % 2 == 0 else -1.0e8
        huge = 1.0e10 if c % 2 == 0 else -1.0e10
        a = 1.0e-3 + 1.0e3 * lcg(s)
        b = 1.0 + lcg(s) if c % 7 == 0 else big
        h = huge * (1.0 + 1e-3 * lcg(s))
        e = (lcg(s) - 0.5) * 2.0e5
        per_col.append([a, b, h, 0.1, e])
    return [[per_col[c][r] for c in range(cols)] for r in range(rows)]


def row_reduce_gentle() -> list:
    """`gentle` (row_reduce_agrees.rs:58-63): values in [-2, 4] for the transcendental epilogues."""
    rows, cols = 5, 96
    v = [((i * 7 + 3) % 19) * 0.37 - 2.0 for i in range(rows * cols)]
    return [v[r * cols:(r + 1) * cols] for r in range(rows)]


def centred_documented(xs: list, block: int) -> list:
    """`centred_documented` (row_reduce_agrees.rs:330-339): stage 0 a documented mean, stage 1 the max of x - r0,
    the epilogue (x - r0) / r1; stage values and the output are rounded to f32, the expressions between them are
    not."""
    r0 = documented(xs, block, mean=True)
    r1 = f32(max(x - r0 for x in xs))
    return [f32((x - r0) / r1) for x in xs]


def serial_softmax(xs: list) -> list:
    """The serial lift of `softmax` (row_reduce_agrees.rs:113-123; kernel_lift/row_reduce.rs:1-11): Max then an
    ascending f64 Sum of exp(x - r0), each stage rounded once to f32; the epilogue in f64, rounded on the store."""
    r0 = f32(max(xs))
    e = [math.exp(x - r0) for x in xs]
    acc = 0.0
    for v in e:
        acc = acc + v
    r1 = f32(acc)
    return [f32(v / r1) for v in e]


def serial_rms_norm(xs: list, eps: float = 1.0e-3) -> list:
    """The serial lift of `rms_norm` (row_reduce_agrees.rs:125-131): an ascending f64 Mean of x * x rounded to
    f32, then x / sqrt(r0 + 1e-3) in f64, rounded on the store."""
    acc = 0.0
    for x in xs:
        acc = acc + x * x
    r0 = f32(acc / len(xs))
    den = math.sqrt(r0 + eps)
    return [f32(x / den) for x in xs]


def golden_row_reduce() -> dict:
    gentle = [[f32(x) for x in r] for r in row_reduce_gentle()]  # `at(F32, ...)`
    corpus = [[f32(x) for x in r] for r in row_reduce_corpus()]
    blocks = [1, 2, 8, 32, 128, 16]  # GEOMETRIES' block sizes (row_reduce_agrees.rs:29)
    return {
        "rows": 5, "cols": 96, "blocks": blocks,
        "gentle_f32_bits": [[f32_bits(x) for x in r] for r in gentle],
        "corpus_f32_bits": [[f32_bits(x) for x in r] for r in corpus],
        "centred_f32_bits": {str(b): [[f32_bits(v) for v in centred_documented(r, b)] for r in gentle] for b in blocks},
        "softmax_serial_f32_bits": [[f32_bits(v) for v in serial_softmax(r)] for r in gentle],
        "rms_norm_serial_f32_bits": [[f32_bits(v) for v in serial_rms_norm(r)] for r in gentle],
        "ulp_band": 4,  # transcendental_epilogues_stay_within_a_few_ulps_of_the_serial_lift (:371-392)
    }


# --- crates/unpopped/tests/kernel_window_agrees.rs, kernel_int_window_agrees.rs ------------------------

WINDOW_VALUES = [1.0e8, 1.0, -1.0e8, 0.5, float("nan"), 2.0, -0.0, float("inf"), -3.0, 0.1, 0.25]  # VALUES (:52-64)


def window_fold(row: list, op: str, size: int, stride: int, dilation: int, pad: int, include_pad: bool,
                k_out: int, is_int: bool = False, bits: int = 32) -> list:
    """The oracle's window fold (oracle/plan_window.rs:320-475): valid taps ascending; f64 Sum/Mean (Mean over size
    or the valid taps), Max/Min take = !have || NaN || better; integer Sum wraps at the dtype's width."""
    out = []
    for o in range(k_out):
        acc, cnt, have, best = 0, 0, False, 0
        for kk in range(size):
            p = o * stride - pad + kk * dilation
            if p < 0 or p >= len(row):
                continue
            v = row[p]
            if op in ("sum", "mean"):
                acc = acc + v
                cnt += 1
            else:
                better = (v > best) if op == "max" else (v < best)
                if not have or (not is_int and v != v) or better:
                    best = v
                have = True
        if op == "sum":
            out.append(wrap_int(acc, bits) if is_int else acc)
        elif op == "mean":
            out.append(acc / (size if include_pad else cnt))
        else:
            out.append(best)
    return out


def wrap_int(v: int, bits: int) -> int:
    v &= (1 << bits) - 1
    return v - (1 << bits) if v >> (bits - 1) else v


def golden_window() -> dict:
    cases = {  # (rows, k_in, size, stride, dilation, pad, include_pad)
        "base": (3, 9, 3, 2, 1, 1, False),             # BASE (:45-53)
        "base_include_pad": (3, 9, 3, 2, 1, 1, True),  # the_two_mean_divisors_agree_and_differ (:140-150)
        "dilated_strided": (2, 12, 3, 3, 2, 2, False),  # dilation_and_stride_agree (:152-166)
        "no_padding": (3, 9, 3, 1, 1, 0, False),       # no_padding_agrees (:168-178)
    }
    res = {"values_f32_bits": [f32_bits(v) for v in WINDOW_VALUES], "cases": {}}
    for name, (rows, k_in, size, stride, dil, pad, inc) in cases.items():
        span = dil * (size - 1) + 1
        k_out = (k_in + 2 * pad - span) // stride + 1
        data = [[f32(WINDOW_VALUES[(r * k_in + c) % len(WINDOW_VALUES)]) for c in range(k_in)] for r in range(rows)]
        res["cases"][name] = {
            "geometry": [rows, k_in, size, stride, dil, pad, int(inc), k_out],
            "expected_f32_bits": {op: [[f32_bits(v) for v in window_fold(r, op, size, stride, dil, pad, inc, k_out)]
                                       for r in data] for op in ("sum", "mean", "max", "min")},
        }
    # a_nan_is_kept_by_max_and_min (:180-200) and the_accumulator_is_f64_and_ascending (:202-230, f32 part)
    nan_row = [1.0, float("nan"), 5.0, 4.0, 3.0, 2.0, 7.0, 6.0, 8.0]
    res["nan_row_f32_bits"] = [f32_bits(v) for v in nan_row]
    res["nan_row_expected"] = {op: [f32_bits(v) for v in window_fold(nan_row, op, 3, 3, 1, 0, False, 3)]
                               for op in ("max", "min")}
    acc_row = [f32(v) for v in [1.0e16, 1.0, -1.0e16, 1.0, 0.1, 0.2, 0.3, 0.4, 0.5]]
    res["ascending_row_f32_bits"] = [f32_bits(v) for v in acc_row]
    res["ascending_sum_f32_bits"] = [f32_bits(v) for v in window_fold(acc_row, "sum", 9, 1, 1, 0, False, 1)]
    # the integer corpus (kernel_int_window_agrees.rs:52-80): I32 values [hi, 1, -1, 2, hi, 3, lo, -5, -7, -7, 4]
    ints = [I32_MAX, 1, -1, 2, I32_MAX, 3, I32_MIN, -5, -7, -7, 4]
    res["int_values"] = ints
    res["int_cases"] = {}
    for name, (rows, k_in, size, stride, dil, pad) in {"base": (3, 9, 3, 2, 1, 1), "dilated": (3, 11, 3, 1, 2, 2)}.items():
        span = dil * (size - 1) + 1
        k_out = (k_in + 2 * pad - span) // stride + 1
        data = [[ints[(r * k_in + c) % len(ints)] for c in range(k_in)] for r in range(rows)]
        res["int_cases"][name] = {
            "geometry": [rows, k_in, size, stride, dil, pad, 0, k_out],
            "expected": {op: [window_fold(r, op, size, stride, dil, pad, False, k_out, True) for r in data]
                         for op in ("sum", "max", "min")},
        }
    return res


# --- crates/unpopped/tests/kernel_im2col_agrees.rs -----------------------------------------------------

def im2col_value(i: int) -> float:
    """`value` (kernel_im2col_agrees.rs:70-77): i + 1, with a NaN at 2 and a negative zero at 5."""
    return float("nan") if i == 2 else (-0.0 if i == 5 else float(i + 1))


def im2col_def(x: list, shape, kernel, stride, pad, dilation) -> list:
    """The Im2Col definition (ir.rs:2286-2324): cell (n, c*kh*kw + ki*kw + kj, oh*oW + ow) copies input
    (n, c, oh*sh - ph + ki*dh, ow*sw - pw + kj*dw), zero outside."""
    n, c, h, w = shape
    (kh, kw), (sh, sw), (ph, pw), (dh, dw) = kernel, stride, pad, dilation
    oh_n = (h + 2 * ph - dh * (kh - 1) - 1) // sh + 1
    ow_n = (w + 2 * pw - dw * (kw - 1) - 1) // sw + 1
    out = []
    for nn in range(n):
        for cc in range(c):
            for ki in range(kh):
                for kj in range(kw):
                    for oh in range(oh_n):
                        for ow in range(ow_n):
                            ih, iw = oh * sh - ph + ki * dh, ow * sw - pw + kj * dw
                            ok = 0 <= ih < h and 0 <= iw < w
                            out.append(x[((nn * c + cc) * h + ih) * w + iw] if ok else 0.0)
    return out


def golden_im2col() -> dict:
    square = dict(shape=[1, 1, 3, 3], kernel=[3, 3], stride=[1, 1], pad=[1, 1], dilation=[1, 1])  # SQUARE (:123-130)
    cases = {
        "padded_3x3": square,
        "batch_and_channels": dict(square, shape=[2, 3, 4, 4]),           # :142-150
        "stride_two": dict(square, shape=[1, 2, 5, 5], stride=[2, 2]),      # :152-161
        "dilation": dict(square, shape=[1, 1, 6, 6], dilation=[2, 2], pad=[2, 2]),  # :163-173
        "rectangular": dict(shape=[1, 2, 5, 7], kernel=[2, 3], stride=[1, 2], pad=[0, 2], dilation=[2, 1]),  # :175-188
    }
    res = {}
    for name, cs in cases.items():
        n = 1
        for d in cs["shape"]:
            n *= d
        x = [f32(im2col_value(i)) for i in range(n)]
        out = im2col_def(x, cs["shape"], cs["kernel"], cs["stride"], cs["pad"], cs["dilation"])
        res[name] = dict(cs, x_f32_bits=[f32_bits(v) for v in x], expected_f32_bits=[f32_bits(v) for v in out])
    return res


def main() -> None:
    out = {
        "float_sum_documented.json": golden_float_sum(),
        "argmax.json": golden_argmax(),
        "scan_i32.json": golden_scan(),
        "gather_oob.json": golden_gather(),
        "dequant_kat.json": golden_dequant(),
        "scatter.json": golden_scatter(),
        "row_reduce.json": golden_row_reduce(),
        "window.json": golden_window(),
        "im2col.json": golden_im2col(),
    }
    for name, obj in out.items():
        with open(os.path.join(HERE, name), "w") as f:
            json.dump(obj, f, indent=1, sort_keys=True)
            f.write("\n")
        print("wrote", name)


if __name__ == "__main__":
    main()
