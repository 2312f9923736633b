"""ctypes wrapper of the CPU oracle restatement (``up_oracle.c``).

TEST INFRASTRUCTURE ONLY: the parity tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg use it as the checker (and the timed CPU baseline). The product library never imports it.
All arrays are numpy; raw bf16/f16 travel as ``uint16``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liborc.so")

OP_SUM, OP_MAX, OP_MIN = 0, 2, 3
OOB_SKIP, OOB_CLAMP, OOB_ZERO_FILL = 0, 1, 2
EK_I32, EK_I64, EK_U32 = 9, 10, 23

_lib = None


def build(force: bool = False) -> str:
    """Compile liborc.so with the committed Makefile (gcc, strict FP, OpenMP)."""
    srcs = [os.path.join(_HERE, f) for f in ("up_oracle.c", "c99_forms.c", "Makefile")]
    if force or not os.path.exists(_LIB_PATH) or any(os.path.getmtime(_LIB_PATH) < os.path.getmtime(f) for f in srcs):
        subprocess.run(["make", "-s", "-C", _HERE, "liborc.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.orc_row_sum_f32.argtypes = [P, I64, I64, I64, P, I]
        L.orc_row_sum_f32_documented.argtypes = [P, I64, I64, I64, I64, P, I]
        L.orc_row_max_argmax_bf16.argtypes = [P, I64, I64, I64, P, P, I]
        L.orc_reduce2d_f32.argtypes = [P, I64, I64, I64, I, I, P, I]
        L.orc_row_mean_f32_documented.argtypes = [P, I64, I64, I64, I64, P, I]
        L.orc_reduce2d_i32.argtypes = [P, I64, I64, I64, I, I, P, I]
        L.orc_col_sum_f32_documented.argtypes = [P, I64, I64, I64, I64, I, P, I]
        L.orc_row_reduce_f32.argtypes = [P, I64, I64, I64, I, I64, ctypes.c_double, P, I64, I]
        L.orc_col_sum_f32_splitk.argtypes = [P, I64, I64, I64, I64, I, P, I]
        L.orc_window.argtypes = [P, I, I64, I64, I64, I, I64, I64, I64, I64, I, P, I64]
        L.orc_im2col.argtypes = [P, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64, I64, P]
        L.orc_scatter.argtypes = [P, I64, I64, I, P, I, I64, I, P, I64]
        L.orc_bincount.argtypes = [P, I64, I, P, I64]
        L.orc_scan_i32.argtypes = [P, P, I64, I64, I, I, I, ctypes.c_int32, I]
        L.orc_scan_i32_chunked.argtypes = [P, P, I64, I, I, I]
        L.orc_reduce_i32.argtypes = [P, I64, I]
        L.orc_reduce_i32.restype = ctypes.c_int32
        L.orc_scan_identity_i32.argtypes = [I]
        L.orc_scan_identity_i32.restype = ctypes.c_int32
        L.orc_gather_rows.argtypes = [P, I64, I64, P, I, I64, I, P, I]
        L.orc_dequant_i4_bf16.argtypes = [P, P, I64, I64, I64, P, I]
        L.orc_w4a16.argtypes = [P, P, P, I64, I64, I64, I64, P, P, P, I]
        L.orc_dequant_gemm_kat.argtypes = [P, I, P, P, P, I64, I64, I64, I64, P]
        L.orc_f32_to_bf16.argtypes = [ctypes.c_float]
        L.orc_f32_to_bf16.restype = ctypes.c_uint16
        L.orc_f64_to_bf16.argtypes = [ctypes.c_double]
        L.orc_f64_to_bf16.restype = ctypes.c_uint16
        L.orc_f32_to_f16.argtypes = [ctypes.c_float]
        L.orc_f32_to_f16.restype = ctypes.c_uint16
        L.orc_f16_to_f64.argtypes = [ctypes.c_uint16]
        L.orc_f16_to_f64.restype = ctypes.c_double
        L.orc_bf16_to_f64.argtypes = [ctypes.c_uint16]
        L.orc_bf16_to_f64.restype = ctypes.c_double
        L.orc_f64_to_f32_odd.argtypes = [ctypes.c_double]
        L.orc_f64_to_f32_odd.restype = ctypes.c_float
        L.orc_i4_value.argtypes = [P, I64]
        L.orc_i4_value.restype = I
        L.orc_max_threads.restype = I
        # c99_forms.c: (pointer, shape array, stride array, base) per buffer, as the C99 emitter passes them
        B4 = [P, P, P, ctypes.c_longlong]
        L.c99_row_sum_serial.argtypes = B4 + B4
        L.c99_row_sum_launched.argtypes = B4 + B4 + [ctypes.c_uint, ctypes.c_uint]
        L.c99_scan_serial.argtypes = B4 + B4 + [I, I]
        L.c99_scan_launched.argtypes = B4 + B4 + [I, I, ctypes.c_uint]
        L.c99_gather_rows_u16.argtypes = B4 + B4 + B4 + [I]
        L.c99_row_max_argmax_bf16.argtypes = B4 + [P, ctypes.c_longlong, P, ctypes.c_longlong]
        L.c99_w4a16.argtypes = [P, P, P, I64, I64, I64, I64, P]
        for f in ("c99_row_sum_serial", "c99_row_sum_launched", "c99_scan_serial", "c99_scan_launched",
                  "c99_gather_rows_u16", "c99_row_max_argmax_bf16", "c99_w4a16"):
            getattr(L, f).restype = I
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def max_threads() -> int:
    """Host threads this process may run on. Taken from the CPU affinity rather than OpenMP's default, which
    launchers such as torchrun pin to 1 through OMP_NUM_THREADS; every parallel region names its count."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return max(1, os.cpu_count() or int(lib().orc_max_threads()))


def row_sum_f32(x: np.ndarray, threads: int = 1) -> np.ndarray:
    """Serial f64 fold, one rounding (oracle/plan_eval.rs:501-651)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    out = np.empty(rows, np.float32)
    lib().orc_row_sum_f32(_p(x), rows, cols, cols, _p(out), threads)
    return out


def row_sum_f32_documented(x: np.ndarray, block: int, threads: int = 1) -> np.ndarray:
    """The launched lift's documented f64 order for a block of ``block`` threads."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    out = np.empty(rows, np.float32)
    lib().orc_row_sum_f32_documented(_p(x), rows, cols, cols, block, _p(out), threads)
    return out


REDUCE_OPS = {"sum": 0, "mean": 1, "max": 2, "min": 3, "prod": 4, "and": 5, "or": 6, "xor": 7}


def reduce2d_f32(x: np.ndarray, op: str, axis: int, threads: int = 1) -> np.ndarray:
    """Serial-order f64 fold of a [rows, cols] f32 array over one axis (oracle/plan_eval.rs:501-651)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    out = np.empty(rows if axis == 1 else cols, np.float32)
    lib().orc_reduce2d_f32(_p(x), rows, cols, cols, axis, REDUCE_OPS[op], _p(out), threads)
    return out


def row_mean_f32_documented(x: np.ndarray, block: int, threads: int = 1) -> np.ndarray:
    """Mean over the last axis in the launched lift's documented order (kernel_lift/block_reduce.rs:13-23)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    out = np.empty(rows, np.float32)
    lib().orc_row_mean_f32_documented(_p(x), rows, cols, cols, block, _p(out), threads)
    return out


def col_sum_f32_documented(x: np.ndarray, block: int, mean: bool = False, threads: int = 1) -> np.ndarray:
    """Sum/Mean over the outer axis in the launched lift's documented order (kernel_lift/block_reduce.rs:13-30)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    out = np.empty(cols, np.float32)
    lib().orc_col_sum_f32_documented(_p(x), rows, cols, cols, block, int(mean), _p(out), threads)
    return out


_SCATTER_EK = {np.dtype(np.int32): 9, np.dtype(np.int64): 10, np.dtype(np.uint32): 23, np.dtype(np.float32): 2,
               np.dtype(np.float64): 4}
_INDEX_EK = {np.dtype(np.int32): 9, np.dtype(np.int64): 10, np.dtype(np.uint32): 23}
COMBINE = {"add": 1, "max": 2, "min": 3}


def scatter(updates: np.ndarray, ids: np.ndarray, out: np.ndarray, combine: str) -> np.ndarray:
    """The scatter store over axis 0 in the serial source order (oracle/plan_eval.rs:430-490); `ids` is either
    full-shape [n, cols] (scatter) or 1-D [n] (index_add). Returns a new array: `out` with the updates combined in."""
    upd = np.ascontiguousarray(updates)
    idx = np.ascontiguousarray(ids)
    res = np.array(out, dtype=upd.dtype, copy=True, order="C")
    n, cols = upd.shape
    ids_stride = cols if idx.ndim == 2 else 0
    lib().orc_scatter(_p(upd), n, cols, _SCATTER_EK[upd.dtype], _p(idx), _INDEX_EK[idx.dtype], ids_stride,
                      COMBINE[combine], _p(res), res.shape[0])
    return res


def bincount(x: np.ndarray, counts: np.ndarray) -> np.ndarray:
    """counts[x[i]] += 1 for every in-range x[i] (kernel_bincount_agrees.rs:1-10); returns a new array."""
    xx = np.ascontiguousarray(x)
    res = np.array(counts, dtype=np.int32, copy=True)
    lib().orc_bincount(_p(xx), xx.size, _INDEX_EK[xx.dtype], _p(res), res.size)
    return res


WINDOW_OPS = {"sum": 0, "mean": 1, "max": 2, "min": 3}


def window(x: np.ndarray, op: str, size: int, stride: int = 1, dilation: int = 1, pad_lo: int = 0,
           k_out: int | None = None, count_include_pad: bool = False, axis: int = -1) -> np.ndarray:
    """Window pooling along `axis` of a float32 or int32 array (oracle/plan_window.rs:249-475); k_out defaults to
    the symmetric-padding extent."""
    x = np.ascontiguousarray(x)
    assert x.dtype in (np.float32, np.int32)
    axis = axis % x.ndim
    k_in = x.shape[axis]
    if k_out is None:
        k_out = (k_in + 2 * pad_lo - dilation * (size - 1) - 1) // stride + 1
    shape = list(x.shape)
    shape[axis] = k_out
    out = np.empty(shape, x.dtype)
    outer = int(np.prod(x.shape[:axis], dtype=np.int64))
    inner = int(np.prod(x.shape[axis + 1:], dtype=np.int64))
    lib().orc_window(_p(x), 2 if x.dtype == np.float32 else 9, outer, k_in, inner, WINDOW_OPS[op], size, stride,
                     dilation, pad_lo, int(count_include_pad), _p(out), k_out)
    return out


def im2col(x: np.ndarray, kernel, stride=(1, 1), pad=(0, 0), dilation=(1, 1)) -> np.ndarray:
    """The 2-D unfold of an NCHW array into [N, C*kh*kw, oH*oW], raw bits (oracle/plan_window.rs:483-535)."""
    x = np.ascontiguousarray(x)
    n, c, h, w = x.shape
    (kh, kw), (sh, sw), (ph, pw), (dh, dw) = kernel, stride, pad, dilation
    oh = (h + 2 * ph - dh * (kh - 1) - 1) // sh + 1
    ow = (w + 2 * pw - dw * (kw - 1) - 1) // sw + 1
    out = np.empty((n, c * kh * kw, oh * ow), x.dtype)
    lib().orc_im2col(_p(x), x.itemsize, n, c, h, w, kh, kw, sh, sw, ph, pw, dh, dw, _p(out))
    return out


def col_sum_f32_splitk(x: np.ndarray, n_chunks: int, mean: bool = False, threads: int = 1) -> np.ndarray:
    """The split-K variant of the outer-axis Sum/Mean (ondevice/README.md:185-218): f64 chunk partials added in
    chunk order."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    out = np.empty(cols, np.float32)
    lib().orc_col_sum_f32_splitk(_p(x), rows, cols, cols, n_chunks, int(mean), _p(out), threads)
    return out


ROW_REDUCE_FORMS = {"softmax": 1, "rms_norm": 2, "centred": 3}


def row_reduce_f32(x: np.ndarray, form: str, block: int, eps: float = 1e-3, threads: int = 1) -> np.ndarray:
    """A RowReduce form (softmax, rms_norm, centred) over the last axis of a [rows, cols] f32 array, in the
    launched lift's written order for a logical block of ``block`` (kernel_lift/row_reduce_launched.rs:1-24)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, cols = x.shape
    out = np.empty_like(x)
    lib().orc_row_reduce_f32(_p(x), rows, cols, cols, ROW_REDUCE_FORMS[form], block, ctypes.c_double(eps), _p(out),
                             cols, threads)
    return out


def reduce2d_i32(x: np.ndarray, op: str, axis: int, threads: int = 1) -> np.ndarray:
    """Fold of a [rows, cols] i32 array over one axis (oracle/plan_eval.rs:501-651, bit_fold)."""
    x = np.ascontiguousarray(x, dtype=np.int32)
    rows, cols = x.shape
    out = np.empty(rows if axis == 1 else cols, np.int32)
    lib().orc_reduce2d_i32(_p(x), rows, cols, cols, axis, REDUCE_OPS[op], _p(out), threads)
    return out


def row_max_argmax_bf16(x_bits: np.ndarray, threads: int = 1):
    """(max as f32, argmax as i64) per row of a bf16 matrix given as uint16 bits."""
    x = np.ascontiguousarray(x_bits, dtype=np.uint16)
    rows, cols = x.shape
    mx = np.empty(rows, np.float32)
    am = np.empty(rows, np.int64)
    lib().orc_row_max_argmax_bf16(_p(x), rows, cols, cols, _p(mx), _p(am), threads)
    return mx, am


def scan_i32(x: np.ndarray, op: int, exclusive: bool, reverse: bool = False, carry=None,
             threads: int = 1) -> np.ndarray:
    """Row scans of an int32 [rows, k] (or 1-D) array (oracle/plan_window.rs:10-238)."""
    x = np.ascontiguousarray(x, dtype=np.int32)
    shape = x.shape
    x2 = x.reshape(1, -1) if x.ndim == 1 else x.reshape(-1, shape[-1])
    y = np.empty_like(x2)
    c = lib().orc_scan_identity_i32(op) if carry is None else int(np.int32(carry))
    lib().orc_scan_i32(_p(x2), _p(y), x2.shape[0], x2.shape[1], op, int(exclusive), int(reverse),
                       c, threads)
    return y.reshape(shape)


def scan_i32_chunked(x: np.ndarray, op: int, exclusive: bool, threads: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.int32).reshape(-1)
    y = np.empty_like(x)
    lib().orc_scan_i32_chunked(_p(x), _p(y), x.size, op, int(exclusive), threads)
    return y


def reduce_i32(x: np.ndarray, op: int) -> int:
    x = np.ascontiguousarray(x, dtype=np.int32).reshape(-1)
    return int(lib().orc_reduce_i32(_p(x), x.size, op))


def scan_identity_i32(op: int) -> int:
    return int(lib().orc_scan_identity_i32(op))


def gather_rows(table: np.ndarray, ids: np.ndarray, oob: int, out: np.ndarray | None = None,
                threads: int = 1) -> np.ndarray:
    """Row gather with an OOB policy; ``out`` (pre-filled) is updated in place for Skip."""
    table = np.ascontiguousarray(table)
    ids = np.ascontiguousarray(ids)
    ek = {np.dtype(np.int32): EK_I32, np.dtype(np.int64): EK_I64, np.dtype(np.uint32): EK_U32}[ids.dtype]
    V = table.shape[0]
    row_bytes = table.nbytes // max(V, 1) if V > 0 else table.dtype.itemsize * int(np.prod(table.shape[1:]))
    n = ids.shape[0]
    if out is None:
        out = np.zeros((n,) + table.shape[1:], table.dtype)
    assert out.flags["C_CONTIGUOUS"]
    lib().orc_gather_rows(_p(table), V, row_bytes, _p(ids), ek, n, oob, _p(out), threads)
    return out


def dequant_i4_bf16(w_packed: np.ndarray, scale_f16_bits: np.ndarray, n: int, k: int, group: int,
                    threads: int = 1) -> np.ndarray:
    w = np.ascontiguousarray(w_packed, dtype=np.uint8)
    s = np.ascontiguousarray(scale_f16_bits, dtype=np.uint16)
    out = np.empty((n, k), np.uint16)
    lib().orc_dequant_i4_bf16(_p(w), _p(s), n, k, group, _p(out), threads)
    return out


def w4a16(w_packed, scale_f16_bits, x_bf16_bits, m, n, k, group, threads: int = 1):
    """(out bf16 bits [m, n], exact f64 [m, n], sum|w*s*x| [m, n])."""
    w = np.ascontiguousarray(w_packed, dtype=np.uint8)
    s = np.ascontiguousarray(scale_f16_bits, dtype=np.uint16)
    x = np.ascontiguousarray(x_bf16_bits, dtype=np.uint16)
    out = np.empty((m, n), np.uint16)
    exact = np.empty((m, n), np.float64)
    abs_sum = np.empty((m, n), np.float64)
    lib().orc_w4a16(_p(w), _p(s), _p(x), m, n, k, group, _p(out), _p(exact), _p(abs_sum), threads)
    return out, exact, abs_sum


def dequant_gemm_kat(packed, signed, zero, scale, x, R, K, C, group) -> np.ndarray:
    """The reference's integer dequant-GEMM KAT form (zero points, I32 scales and activations)."""
    w = np.ascontiguousarray(packed, dtype=np.uint8)
    z = np.ascontiguousarray(zero, dtype=np.int32)
    s = np.ascontiguousarray(scale, dtype=np.int32)
    xx = np.ascontiguousarray(x, dtype=np.int32)
    out = np.empty(R * C, np.int32)
    lib().orc_dequant_gemm_kat(_p(w), int(signed), _p(z), _p(s), _p(xx), R, K, C, group, _p(out))
    return out


def f32_to_bf16(x: float) -> int:
    return int(lib().orc_f32_to_bf16(float(x)))


def f64_to_bf16(x: float) -> int:
    return int(lib().orc_f64_to_bf16(float(x)))


def f32_to_f16(x: float) -> int:
    return int(lib().orc_f32_to_f16(float(x)))


def f16_to_f64(b: int) -> float:
    return float(lib().orc_f16_to_f64(int(b)))


def bf16_to_f64(b: int) -> float:
    return float(lib().orc_bf16_to_f64(int(b)))


def i4_value(packed: np.ndarray, idx: int) -> int:
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    return int(lib().orc_i4_value(_p(p), idx))


# ---- the C99 emitter's serial forms (c99_forms.c): a timed CPU baseline, checked against the oracle ----

def _buf(a: np.ndarray):
    """(pointer, shape array, stride array, base 0) of a C-contiguous array, in the emitter's argument ABI; the
    arrays are returned too so that they outlive the call."""
    assert a.flags["C_CONTIGUOUS"]
    shape = np.array(a.shape, np.int64)
    stride = np.array([st // a.itemsize for st in a.strides], np.int64)
    return (_p(a), _p(shape), _p(stride), 0), (shape, stride)


def c99_row_sum(x: np.ndarray, block: int | None = None) -> np.ndarray:
    """The serial reduction lift's C (block None) or the launched block-tree lift's serialized C (a block B)."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape[0], np.float32)
    a, keep_a = _buf(x)
    b, keep_b = _buf(out)
    if block is None:
        st = lib().c99_row_sum_serial(*a, *b)
    else:
        st = lib().c99_row_sum_launched(*a, *b, block, max(1, x.shape[0]))
    assert st == 0
    return out


def c99_scan(x: np.ndarray, op: int, exclusive: bool, block: int | None = None) -> np.ndarray:
    """The serial scan lift's C (block None) or the launched three-phase lift's serialized C, over a 1-D row."""
    x = np.ascontiguousarray(x, np.int32).reshape(-1)
    y = np.empty_like(x)
    a, keep_a = _buf(x)
    b, keep_b = _buf(y)
    if block is None:
        st = lib().c99_scan_serial(*a, *b, op, int(exclusive))
    else:
        st = lib().c99_scan_launched(*a, *b, op, int(exclusive), block)
    assert st == 0
    return y


def c99_gather(table_u16: np.ndarray, ids: np.ndarray, oob: int, out: np.ndarray) -> np.ndarray:
    """The gather lift's per-cell C over 2-byte elements and i32 ids; `out` (pre-filled) is updated in place."""
    t = np.ascontiguousarray(table_u16).view(np.uint16)
    i = np.ascontiguousarray(ids, np.int32)
    assert out.dtype.itemsize == 2 and out.flags["C_CONTIGUOUS"]
    o = out.view(np.uint16)
    a, ka = _buf(t)
    b, kb = _buf(i)
    c, kc = _buf(o)
    assert lib().c99_gather_rows_u16(*a, *b, *c, oob) == 0
    return out


def c99_row_max_argmax(x_bits: np.ndarray):
    """The kernel-layer arg loop's C over bf16 rows: (max f32, argmax i64)."""
    x = np.ascontiguousarray(x_bits, np.uint16)
    mx = np.empty(x.shape[0], np.float32)
    am = np.empty(x.shape[0], np.int64)
    a, ka = _buf(x)
    assert lib().c99_row_max_argmax_bf16(*a, _p(mx), 0, _p(am), 0) == 0
    return mx, am


def c99_w4a16(w_packed, scale_f16_bits, x_bf16_bits, m, n, k, group) -> np.ndarray:
    """The dequant GEMM KernelFn's serialized C (one thread per output cell, f32 accumulator): bf16 bits [m, n]."""
    w = np.ascontiguousarray(w_packed, np.uint8)
    s = np.ascontiguousarray(scale_f16_bits, np.uint16)
    x = np.ascontiguousarray(x_bf16_bits, np.uint16)
    out = np.empty((m, n), np.uint16)
    assert lib().c99_w4a16(_p(w), _p(s), _p(x), m, n, k, group, _p(out)) == 0
    return out
