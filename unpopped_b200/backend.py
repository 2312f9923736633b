"""The reference's `Backend` seam, as this library answers it (crates/unpopped/src/backend.rs:668-835).

`CudaSm100` mirrors the trait's methods over the C ABI: `name`, `provider`, `supports_dtype(dtype, target)`
(backend.rs:779, answering a `DtypeSupport`, :645-666) and `lower(plan)` (backend.rs:708), which returns a
`GeneratedKernel`-like record (entry symbol + launch scalars) or raises `LowerError` with the reference's
variant name (backend.rs:386-440). `launch` runs what `lower` chose, on device tensors, through
`up_sm100_launch`. The plan is described by `Plan`, the fields of a reference `KernelPlan`
(plan/types.rs:170-270) that the classifier reads.
"""
from __future__ import annotations

import ctypes
import dataclasses

from . import _lib
from ._lib import COMBINE, EK, KERNEL, LOWER_ERROR, OOB, OP, ROW_REDUCE_FORM, SCHED, UpLowered, UpPlanDesc, UpTensor

DTYPE_SUPPORT = {0: "Supported", 1: "Unsupported", 2: "NotExpressible"}
TARGET = "cuda:sm_100a"


@dataclasses.dataclass
class Operand:
    """An `OperandDesc` / `TypedBuffer` (oracle/buffers.rs:16): dtype, shape, strides (elements), base."""
    dtype: str
    shape: tuple
    strides: tuple | None = None
    base: int = 0
    ptr: int = 0

    def to_c(self) -> UpTensor:
        t = UpTensor()
        t.ptr = self.ptr or None
        t.dtype = EK[self.dtype]
        t.rank = len(self.shape)
        strides = self.strides
        if strides is None:
            strides, s = [], 1
            for d in reversed(self.shape):
                strides.insert(0, s)
                s *= d
        for i, (d, s) in enumerate(zip(self.shape, strides)):
            t.shape[i] = d
            t.stride[i] = s
        t.base = self.base
        return t


@dataclasses.dataclass
class Plan:
    schedule: str
    operands: list
    dtype: str = "F32"
    out_dtype: str | None = None
    op: str = "SUM"
    axes_mask: int = 0
    keepdim: bool = False
    identity_body: bool = True
    accum: str = "F32"
    block: int = 0
    scan_axis: int = 0
    exclusive: bool = False
    reverse: bool = False
    read_index: bool = False
    write_index: bool = False  # a scatter store (WriteIndex::ScatterIndexed)
    scatter_axis: int = 0
    combine: str = "ADD"
    count: bool = False  # bincount
    row_reduce_form: str = "NONE"  # a RowReduce plan's named form: SOFTMAX, RMS_NORM or CENTRED
    eps: float = 1e-3
    splitk_chunks: int = 0  # > 0: the split-K variant of an outer-axis f32 Sum/Mean
    window: tuple = (0, 1, 1, 1, 0, 0)  # Schedule::Window: (axis, size, stride, dilation, pad_lo, pad_hi)
    count_include_pad: bool = False
    im2col: tuple = ((1, 1), (1, 1), (0, 0), (1, 1))  # Schedule::Im2Col: kernel, stride, pad, dilation (h, w)
    gather_axis: int = 0
    oob: str = "SKIP"
    index_dtype: str = "I32"
    target: str = TARGET

    def to_c(self) -> UpPlanDesc:
        p = UpPlanDesc()
        p.schedule = SCHED[self.schedule]
        p.op = OP[self.op]
        p.dtype = EK[self.dtype]
        p.out_dtype = EK[self.out_dtype or self.dtype]
        p.axes_mask = self.axes_mask
        p.keepdim = int(self.keepdim)
        p.identity_body = int(self.identity_body)
        p.accum = 0 if self.accum == "AUTO" else 1
        p.block = self.block
        p.scan_axis = self.scan_axis
        p.exclusive = int(self.exclusive)
        p.reverse = int(self.reverse)
        p.has_read_index = int(self.read_index)
        p.has_write_index = int(self.write_index)
        p.scatter_axis = self.scatter_axis
        p.combine = COMBINE[self.combine]
        p.count = int(self.count)
        p.row_reduce_form = ROW_REDUCE_FORM[self.row_reduce_form]
        p.eps = self.eps
        p.splitk_chunks = self.splitk_chunks
        (p.window_axis, p.window_size, p.window_stride, p.window_dilation, p.window_pad_lo,
         p.window_pad_hi) = self.window
        p.count_include_pad = int(self.count_include_pad)
        for field, pair in zip(("im2col_kernel", "im2col_stride", "im2col_pad", "im2col_dilation"), self.im2col):
            getattr(p, field)[0], getattr(p, field)[1] = pair
        p.gather_axis = self.gather_axis
        p.oob = OOB[self.oob]
        p.index_dtype = EK[self.index_dtype]
        p.n_operands = len(self.operands)
        for i, o in enumerate(self.operands):
            p.operands[i] = o.to_c()
        p.target = self.target.encode()
        return p


class LowerError(Exception):
    def __init__(self, variant: str, detail: str):
        self.variant = variant
        self.detail = detail
        super().__init__(f"{variant}: {detail}")


@dataclasses.dataclass
class GeneratedKernel:
    name: str
    kernel_id: int
    scalars: tuple


class CudaSm100:
    """`impl Backend for CudaSm100` over libunpopped_sm100.so."""

    def name(self) -> str:
        return _lib.load().up_sm100_name().decode()

    def provider(self) -> str:
        return _lib.load().up_sm100_provider().decode()

    def supports_dtype(self, dtype: str, target: str = TARGET) -> str:
        return DTYPE_SUPPORT[_lib.load().up_sm100_supports_dtype(EK[dtype], target.encode())]

    def lower(self, plan: Plan) -> GeneratedKernel:
        desc = plan.to_c()
        out = UpLowered()
        st = _lib.load().up_sm100_classify(ctypes.byref(desc), ctypes.byref(out))
        if st != _lib.UP_OK:
            raise LowerError(LOWER_ERROR.get(out.lower_error, str(out.lower_error)), out.detail.decode())
        return GeneratedKernel(out.name.decode(), out.kernel_id, tuple(out.scalars[i] for i in range(out.n_scalars)))

    def launch(self, k: GeneratedKernel, ins: list, outs: list, workspace=None, stream=None) -> None:
        """Runs a lowered kernel on device buffers described by `Operand`s (ptr set)."""
        L = _lib.load()
        cin = (UpTensor * max(1, len(ins)))(*[o.to_c() for o in ins])
        cout = (UpTensor * max(1, len(outs)))(*[o.to_c() for o in outs])
        sc = (ctypes.c_int64 * max(1, len(k.scalars)))(*k.scalars)
        ws_ptr, ws_bytes = (None, 0)
        if workspace is not None:
            ws_ptr, ws_bytes = workspace.data_ptr(), workspace.numel()
        _lib.check(L.up_sm100_launch(k.kernel_id, cin, len(ins), cout, len(outs), sc, len(k.scalars), ws_ptr,
                                     ws_bytes, stream), f"launch {k.name}")

    def workspace_bytes(self, k: GeneratedKernel, ins: list, outs: list) -> int:
        L = _lib.load()
        cin = (UpTensor * max(1, len(ins)))(*[o.to_c() for o in ins])
        cout = (UpTensor * max(1, len(outs)))(*[o.to_c() for o in outs])
        sc = (ctypes.c_int64 * max(1, len(k.scalars)))(*k.scalars)
        n = ctypes.c_size_t(0)
        _lib.check(L.up_sm100_workspace_bytes(k.kernel_id, cin, len(ins), cout, len(outs), sc, len(k.scalars),
                                              ctypes.byref(n)), "workspace_bytes")
        return int(n.value)


__all__ = ["CudaSm100", "Plan", "Operand", "LowerError", "GeneratedKernel", "KERNEL"]
