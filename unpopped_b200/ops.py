"""Tensor-level entry points over the C ABI: each lifted kernel family on torch CUDA tensors.

torch supplies device memory and the current stream only; every computation runs in libunpopped_sm100.so.
Inputs must already be on a CUDA device; nothing here moves data to the host or computes on it. The one
exception is `scan_host`, whose buffers are in host memory: the library itself streams them through the device.
"""
from __future__ import annotations

import ctypes
import threading

import numpy as np
import torch

from . import _lib
from ._lib import ACCUM, COMBINE, EK, OOB, OP, check

_OPS = {"sum": OP["SUM"], "max": OP["MAX"], "min": OP["MIN"]}
_OOBS = {"skip": OOB["SKIP"], "clamp": OOB["CLAMP"], "zero_fill": OOB["ZERO_FILL"]}
_IDX = {torch.int32: EK["I32"], torch.int64: EK["I64"], torch.uint32: EK["U32"]}


def _stream(t: torch.Tensor):
    return ctypes_ptr(torch.cuda.current_stream(t.device).cuda_stream)


def ctypes_ptr(v):
    return None if v in (0, None) else v


def _cuda(t: torch.Tensor, name: str):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")


# ---- workspaces: zero-filled once per (device, stream, kind); the kernels re-arm them after every launch ----
_ws_lock = threading.Lock()
_ws_cache: dict = {}


def workspace(kind: str, nbytes: int, device: torch.device) -> torch.Tensor:
    """A zero-filled device workspace for `kind`, reused by later calls on the same stream."""
    stream = torch.cuda.current_stream(device).cuda_stream
    key = (kind, device.index, stream)
    with _ws_lock:
        ws = _ws_cache.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
            _ws_cache[key] = ws
        return ws


def workspace_status(ws: torch.Tensor) -> int:
    """Waits for the stream and returns UP_OK or UP_ERR_DEVICE_TIMEOUT (clearing the error word)."""
    return _lib.load().up_sm100_workspace_status(ws.data_ptr(), _stream(ws))


def check_workspace(kind: str, device: torch.device):
    ws = _ws_cache.get((kind, device.index, torch.cuda.current_stream(device).cuda_stream))
    if ws is not None:
        check(workspace_status(ws), f"{kind} device wait")


# ---- row sum ----
def row_sum(x: torch.Tensor, accum: str = "f32", block: int = 256, out: torch.Tensor | None = None) -> torch.Tensor:
    """Sum of each row of a 2-D f32 tensor (last axis). accum='f32' (fixed-order f32 tree) or 'auto' (f64 in
    the launched lift's documented order for a block of `block` threads, bit-exact)."""
    _cuda(x, "x")
    if x.dtype != torch.float32 or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("row_sum takes a 2-D float32 tensor with contiguous rows")
    rows, cols = x.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.float32, device=x.device)
    check(_lib.load().up_sm100_row_sum_f32(x.data_ptr(), rows, cols, x.stride(0), out.data_ptr(),
                                           ACCUM[accum.upper()], block, _stream(x)), "row_sum")
    return out


# ---- max + argmax ----
def reduce2d(x: torch.Tensor, op: str, axis: int = 1, accum: str = "auto", block: int | None = None,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """Reduction of a [rows, cols] f32 or i32 tensor with contiguous rows over axis 1 (the last; one value per
    row) or axis 0 (the outer; one per column). f32: sum, mean, max, min; i32: sum, prod, max, min, and, or, xor."""
    _cuda(x, "x")
    if x.dim() != 2 or x.stride(1) != 1 or x.dtype not in (torch.float32, torch.int32):
        raise ValueError("reduce2d takes a 2-D float32 or int32 tensor with contiguous rows")
    if axis not in (0, 1):
        raise ValueError("axis is 0 or 1")
    rows, cols = x.shape
    n = rows if axis == 1 else cols
    if out is None:
        out = torch.empty(n, dtype=x.dtype, device=x.device)
    L = _lib.load()
    if x.dtype == torch.float32:
        b = block if block is not None else (256 if axis == 1 else 1)
        check(L.up_sm100_reduce2d_f32(x.data_ptr(), rows, cols, x.stride(0), axis, OP[op.upper()],
                                      ACCUM[accum.upper()], b, out.data_ptr(), _stream(x)), "reduce2d_f32")
    else:
        check(L.up_sm100_reduce2d_i32(x.data_ptr(), rows, cols, x.stride(0), axis, OP[op.upper()], out.data_ptr(),
                                      _stream(x)), "reduce2d_i32")
    return out


def row_reduce(x: torch.Tensor, form: str, block: int = 256, eps: float = 1e-3,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """A RowReduce form over the rows of a [rows, cols] f32 tensor (contiguous rows): "softmax", "rms_norm"
    (x / sqrt(mean(x * x) + eps)) or "centred" ((x - mean) / max(x - mean)), for logical block `block`."""
    _cuda(x, "x")
    if x.dim() != 2 or x.stride(1) != 1 or x.dtype != torch.float32:
        raise ValueError("row_reduce takes a 2-D float32 tensor with contiguous rows")
    if out is None:
        out = torch.empty_like(x, memory_format=torch.contiguous_format)
    if out.shape != x.shape or out.stride(1) != 1 or out.dtype != torch.float32:
        raise ValueError("out has x's shape with contiguous rows")
    L = _lib.load()
    check(L.up_sm100_row_reduce_f32(x.data_ptr(), x.shape[0], x.shape[1], x.stride(0),
                                    _lib.ROW_REDUCE_FORM[form.upper()], block, eps, out.data_ptr(), out.stride(0),
                                    _stream(x)), "row_reduce_f32")
    return out


def col_sum_splitk(x: torch.Tensor, n_chunks: int, mean: bool = False,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """The split-K variant of the outer-axis f32 Sum (Mean) of a [rows, cols] tensor with contiguous rows: f64
    partials over n_chunks row chunks, added in chunk order. Allocates its workspace."""
    _cuda(x, "x")
    if x.dim() != 2 or x.stride(1) != 1 or x.dtype != torch.float32:
        raise ValueError("col_sum_splitk takes a 2-D float32 tensor with contiguous rows")
    rows, cols = x.shape
    if out is None:
        out = torch.empty(cols, dtype=torch.float32, device=x.device)
    L = _lib.load()
    nb = L.up_sm100_col_sum_splitk_workspace_bytes(rows, cols, n_chunks)
    ws = torch.empty(max(8, nb), dtype=torch.uint8, device=x.device)
    check(L.up_sm100_col_sum_f32_splitk(x.data_ptr(), rows, cols, x.stride(0), n_chunks, int(mean), ws.data_ptr(),
                                        ws.numel(), out.data_ptr(), _stream(x)), "col_sum_f32_splitk")
    return out


def window(x: torch.Tensor, op: str, size: int, stride: int = 1, dilation: int = 1, pad_lo: int = 0,
           pad_hi: int | None = None, count_include_pad: bool = False, axis: int = -1,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """1-D window pooling (sum, mean, max, min) of a dense f32 or i32 tensor along `axis`; the output extent is
    (k_in + pad_lo + pad_hi - dilation*(size-1) - 1) // stride + 1 (pad_hi defaults to pad_lo)."""
    _cuda(x, "x")
    if not x.is_contiguous() or x.dtype not in (torch.float32, torch.int32):
        raise ValueError("window takes a contiguous float32 or int32 tensor")
    axis = axis % x.dim()
    k_in = x.shape[axis]
    ph = pad_lo if pad_hi is None else pad_hi
    k_out = (k_in + pad_lo + ph - dilation * (size - 1) - 1) // stride + 1
    shape = list(x.shape)
    shape[axis] = max(k_out, 0)
    if out is None:
        out = torch.empty(shape, dtype=x.dtype, device=x.device)
    outer = int(np.prod(x.shape[:axis], dtype=np.int64))
    inner = int(np.prod(x.shape[axis + 1:], dtype=np.int64))
    L = _lib.load()
    check(L.up_sm100_window(x.data_ptr(), EK["F32"] if x.dtype == torch.float32 else EK["I32"], outer, k_in, inner,
                            OP[op.upper()], size, stride, dilation, pad_lo, int(count_include_pad), out.data_ptr(),
                            shape[axis], _stream(x)), "window")
    return out


def im2col(x: torch.Tensor, kernel: tuple, stride: tuple = (1, 1), pad: tuple = (0, 0), dilation: tuple = (1, 1),
           out: torch.Tensor | None = None) -> torch.Tensor:
    """The 2-D unfold of a contiguous NCHW tensor into [N, C*kh*kw, oH*oW], raw bits, zeros outside the input."""
    _cuda(x, "x")
    if x.dim() != 4 or not x.is_contiguous():
        raise ValueError("im2col takes a contiguous NCHW tensor")
    n, c, h, w = x.shape
    (kh, kw), (sh, sw), (ph, pw), (dh, dw) = kernel, stride, pad, dilation
    oh = (h + 2 * ph - dh * (kh - 1) - 1) // sh + 1
    ow = (w + 2 * pw - dw * (kw - 1) - 1) // sw + 1
    if out is None:
        out = torch.empty((n, c * kh * kw, max(oh, 0) * max(ow, 0)), dtype=x.dtype, device=x.device)
    L = _lib.load()
    check(L.up_sm100_im2col(x.data_ptr(), x.element_size(), n, c, h, w, kh, kw, sh, sw, ph, pw, dh, dw,
                            out.data_ptr(), _stream(x)), "im2col")
    return out


def reduce3d(x: torch.Tensor, op: str, accum: str = "auto", block: int = 1,
             out: torch.Tensor | None = None) -> torch.Tensor:
    """Reduction of an [outer, rows, cols] f32 or i32 tensor over its middle axis into [outer, cols]; the rows and
    the output rows are contiguous. Each output cell is the outer-axis fold of reduce2d over its batch."""
    _cuda(x, "x")
    if x.dim() != 3 or x.stride(2) != 1 or x.dtype not in (torch.float32, torch.int32):
        raise ValueError("reduce3d takes a 3-D float32 or int32 tensor with contiguous rows")
    outer, rows, cols = x.shape
    if out is None:
        out = torch.empty((outer, cols), dtype=x.dtype, device=x.device)
    if out.dim() != 2 or tuple(out.shape) != (outer, cols) or out.stride(1) != 1:
        raise ValueError("out is [outer, cols] with contiguous rows")
    L = _lib.load()
    if x.dtype == torch.float32:
        check(L.up_sm100_reduce3d_f32(x.data_ptr(), outer, rows, cols, x.stride(0), x.stride(1), OP[op.upper()],
                                      ACCUM[accum.upper()], block, out.data_ptr(), out.stride(0), _stream(x)),
              "reduce3d_f32")
    else:
        check(L.up_sm100_reduce3d_i32(x.data_ptr(), outer, rows, cols, x.stride(0), x.stride(1), OP[op.upper()],
                                      out.data_ptr(), out.stride(0), _stream(x)), "reduce3d_i32")
    return out


_SC_EK = {torch.int32: EK["I32"], torch.int64: EK["I64"], torch.uint32: EK["U32"], torch.float32: EK["F32"],
          torch.float64: EK["F64"]}


def scatter(updates: torch.Tensor, ids: torch.Tensor, out: torch.Tensor, combine: str = "add") -> torch.Tensor:
    """out[t][j] (combine)= updates[i][j] with t = ids[i][j] (a full-shape index, scatter) or ids[i] (1-D, index_add),
    over axis 0; targets outside [0, out.shape[0]) are skipped. Updates `out` in place and returns it."""
    for t, name in ((updates, "updates"), (ids, "ids"), (out, "out")):
        _cuda(t, name)
    if updates.dim() != 2 or out.dim() != 2 or updates.stride(1) != 1 or out.stride(1) != 1:
        raise ValueError("scatter takes rank-2 updates and destination with contiguous rows")
    if updates.dtype != out.dtype or updates.dtype not in _SC_EK or ids.dtype not in _IDX:
        raise ValueError("scatter dtypes: updates/out I32, U32, I64, F32 or F64; ids I32, I64 or U32")
    if ids.dim() == 2:
        if ids.shape != updates.shape or ids.stride(1) != 1:
            raise ValueError("a full-shape index has the updates' shape and contiguous rows")
        ids_stride = ids.stride(0)
    else:
        if ids.dim() != 1 or ids.shape[0] != updates.shape[0] or ids.stride(0) != 1:
            raise ValueError("a row index is 1-D, one per update row, contiguous")
        ids_stride = 0
    check(_lib.load().up_sm100_scatter(updates.data_ptr(), updates.shape[0], updates.shape[1], updates.stride(0),
                                       _SC_EK[updates.dtype], ids.data_ptr(), _IDX[ids.dtype], ids_stride,
                                       COMBINE[combine.upper()], out.data_ptr(), out.shape[0], out.stride(0),
                                       _stream(out)), "scatter")
    return out


def bincount(x: torch.Tensor, counts: torch.Tensor) -> torch.Tensor:
    """counts[x[i]] += 1 for every in-range x[i]; `counts` (int32) keeps its prior contents."""
    _cuda(x, "x")
    _cuda(counts, "counts")
    if counts.dtype != torch.int32 or not counts.is_contiguous() or not x.is_contiguous() or x.dtype not in _IDX:
        raise ValueError("bincount takes contiguous I32/I64/U32 values and contiguous int32 counts")
    check(_lib.load().up_sm100_bincount(x.data_ptr(), x.numel(), _IDX[x.dtype], counts.data_ptr(), counts.numel(),
                                        _stream(counts)), "bincount")
    return counts


def row_max_argmax(x: torch.Tensor, index_dtype=torch.int32, want_max: bool = True, want_argmax: bool = True):
    """(max as f32, argmax) of each row of a 2-D bf16 tensor: NaN-propagating max, first index of the maximum
    with NaN the greatest value."""
    _cuda(x, "x")
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("row_max_argmax takes a 2-D bfloat16 tensor with contiguous rows")
    rows, cols = x.shape
    mx = torch.empty(rows, dtype=torch.float32, device=x.device) if want_max else None
    am = torch.empty(rows, dtype=index_dtype, device=x.device) if want_argmax else None
    p32 = am.data_ptr() if (am is not None and index_dtype == torch.int32) else None
    p64 = am.data_ptr() if (am is not None and index_dtype == torch.int64) else None
    check(_lib.load().up_sm100_row_max_argmax_bf16(x.data_ptr(), rows, cols, x.stride(0),
                                                   mx.data_ptr() if mx is not None else None, p32, p64,
                                                   _stream(x)), "row_max_argmax")
    return mx, am


# ---- scans ----
def scan(x: torch.Tensor, op: str = "sum", exclusive: bool = False, reverse: bool = False,
         carry: torch.Tensor | None = None, out: torch.Tensor | None = None,
         ws: torch.Tensor | None = None) -> torch.Tensor:
    """Scan of int32 rows along the last axis (decoupled look-back, one pass)."""
    _cuda(x, "x")
    if x.dtype != torch.int32 or not x.is_contiguous():
        raise ValueError("scan takes a contiguous int32 tensor")
    k = x.shape[-1] if x.dim() > 0 else 1
    rows = x.numel() // k if k > 0 else 0
    if out is None:
        out = torch.empty_like(x)
    L = _lib.load()
    nbytes = L.up_sm100_scan_workspace_bytes(rows, k)
    if ws is None:
        ws = workspace("scan", nbytes, x.device)
    check(L.up_sm100_scan_i32(x.data_ptr(), out.data_ptr(), rows, k, _OPS[op], int(exclusive), int(reverse),
                              carry.data_ptr() if carry is not None else None, ws.data_ptr(), ws.numel(),
                              _stream(x)), "scan")
    return out


def scan_host(x, op: str = "sum", exclusive: bool = False, reverse: bool = False, carry: int | None = None,
              out=None):
    """Scan of int32 rows held in HOST memory (a numpy array or a CPU tensor, pinned for the full copy rate),
    streamed through the device with the copies overlapped; returns the output in host memory."""
    is_t = isinstance(x, torch.Tensor)
    if is_t:
        if x.device.type != "cpu" or x.dtype != torch.int32 or not x.is_contiguous():
            raise ValueError("scan_host takes a contiguous int32 tensor in host memory")
        if out is None:
            out = torch.empty_like(x, pin_memory=x.is_pinned())
        xp, yp = x.data_ptr(), out.data_ptr()
    else:
        x = np.ascontiguousarray(x)
        if x.dtype != np.int32:
            raise ValueError("scan_host takes an int32 array")
        if out is None:
            out = np.empty_like(x)
        xp, yp = x.ctypes.data, out.ctypes.data
    k = x.shape[-1] if x.ndim > 0 else 1
    rows = (x.size if not is_t else x.numel()) // k if k > 0 else 0
    c = ctypes.c_int32(carry) if carry is not None else None
    check(_lib.load().up_sm100_scan_i32_host(xp, yp, rows, k, _OPS[op], int(exclusive), int(reverse),
                                             ctypes.byref(c) if c is not None else None), "scan_host")
    return out


def reduce_i32(x: torch.Tensor, op: str = "sum", out: torch.Tensor | None = None) -> torch.Tensor:
    """Fold of a whole int32 tensor to one int32 (SUM wraps)."""
    _cuda(x, "x")
    if x.dtype != torch.int32 or not x.is_contiguous():
        raise ValueError("reduce_i32 takes a contiguous int32 tensor")
    if out is None:
        out = torch.empty(1, dtype=torch.int32, device=x.device)
    check(_lib.load().up_sm100_reduce_i32(x.data_ptr(), x.numel(), _OPS[op], out.data_ptr(), _stream(x)),
          "reduce_i32")
    return out


# ---- gather ----
def gather_rows(table: torch.Tensor, ids: torch.Tensor, oob: str = "skip",
                out: torch.Tensor | None = None) -> torch.Tensor:
    """out[n] = table[ids[n]] (rows copied bit for bit); out-of-range ids per `oob`."""
    _cuda(table, "table")
    _cuda(ids, "ids")
    if not table.is_contiguous() or ids.dim() != 1 or not ids.is_contiguous():
        raise ValueError("gather_rows takes a contiguous table and 1-D contiguous ids")
    if ids.dtype not in _IDX:
        raise ValueError("ids must be int32, int64 or uint32")
    V = table.shape[0]
    row_bytes = (table[0].numel() if V > 0 else int(torch.Size(table.shape[1:]).numel())) * table.element_size()
    n = ids.shape[0]
    if out is None:
        out = (torch.zeros if oob == "skip" else torch.empty)((n,) + tuple(table.shape[1:]), dtype=table.dtype,
                                                              device=table.device)
    check(_lib.load().up_sm100_gather_rows(table.data_ptr() if V > 0 else None, V, row_bytes, ids.data_ptr(),
                                           _IDX[ids.dtype], n, _OOBS[oob], out.data_ptr(), _stream(table)),
          "gather_rows")
    return out


# ---- int4 dequant and W4A16 ----
def dequant_i4(w_packed: torch.Tensor, scale: torch.Tensor, group: int, out: torch.Tensor | None = None):
    """bf16 [N, K] from int4 [N, K] packed two per byte ([N, K/2] uint8) and f16 scales [N, K/group]."""
    _cuda(w_packed, "w")
    _cuda(scale, "scale")
    n, kh = w_packed.shape
    k = 2 * kh
    if out is None:
        out = torch.empty((n, k), dtype=torch.bfloat16, device=w_packed.device)
    check(_lib.load().up_sm100_dequant_i4_bf16(w_packed.data_ptr(), scale.data_ptr(), n, k, group, out.data_ptr(),
                                               _stream(w_packed)), "dequant_i4")
    return out


def w4a16(w_packed: torch.Tensor, scale: torch.Tensor, x: torch.Tensor, group: int,
          out: torch.Tensor | None = None, ws: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 [M, N] = x [M, K] (bf16) times the dequantized int4 weights [N, K], f32 accumulation on tcgen05."""
    for t, nm in ((w_packed, "w"), (scale, "scale"), (x, "x")):
        _cuda(t, nm)
    n, kh = w_packed.shape
    k = 2 * kh
    m = x.shape[0]
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=x.device)
    L = _lib.load()
    if ws is None:
        ws = workspace("w4a16", L.up_sm100_w4a16_workspace_bytes(m, n, k, group), x.device)
    check(L.up_sm100_w4a16_gemm(w_packed.data_ptr(), scale.data_ptr(), x.data_ptr(), m, n, k, group, out.data_ptr(),
                                ws.data_ptr(), ws.numel(), _stream(x)), "w4a16")
    return out


def launch_count() -> int:
    return int(_lib.load().up_sm100_launch_count())
