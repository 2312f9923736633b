"""ctypes binding of libunpopped_sm100.so (the C ABI declared in include/up_sm100.h).

The library is loaded from this package directory. There is no fallback: if it is missing or fails to load,
every entry point raises, because a silent substitute would void the parity and performance claims.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libunpopped_sm100.so")

# status codes (up_status)
UP_OK, UP_ERR_OOB, UP_ERR_ZERO_STEP, UP_ERR_UNSUPPORTED = 0, 1, 2, 3
UP_ERR_DEVICE_TIMEOUT, UP_ERR_CUDA, UP_ERR_COMM, UP_ERR_INVALID = 4, 5, 6, 7
STATUS_NAMES = {0: "UP_OK", 1: "UP_ERR_OOB", 2: "UP_ERR_ZERO_STEP", 3: "UP_ERR_UNSUPPORTED",
                4: "UP_ERR_DEVICE_TIMEOUT", 5: "UP_ERR_CUDA", 6: "UP_ERR_COMM", 7: "UP_ERR_INVALID"}

# ElementKind ordinals (crates/unpopped-vocab/src/element.rs:1052-1206)
EK = dict(F16=0, BF16=1, F32=2, F32_STRICT=3, F64=4, I8=5, I16=6, U8=7, U16=8, I32=9, I64=10, BOOL=11,
          FP8_E4M3FN=12, FP8_E4M3FNUZ=13, FP8_E5M2=14, F8_E8M0=15, F8_E6M2=16, FP8_E5M2FNUZ=17, I4=18, U4=19,
          B1=20, COMPLEX64=21, COMPLEX128=22, U32=23, U64=24, F4_E2M1=25, F6_E2M3=26, F6_E3M2=27)
# ReduceOp ordinals (crates/unpopped/src/ir.rs:1700-1742)
OP = dict(SUM=0, MEAN=1, MAX=2, MIN=3, PROD=4, AND=5, OR=6, XOR=7, MAXNUM=8, MINNUM=9, ARGMAX=10, ARGMIN=11)
OOB = dict(SKIP=0, CLAMP=1, ZERO_FILL=2)
ACCUM = dict(AUTO=0, F32=1)
SCHED = dict(VECTORIZED=0, SCALAR=1, STRIDED=2, REDUCTION=3, ROW_REDUCE=4, CONTRACTION=5, SCAN=6, WINDOW=7, IM2COL=8,
             KERNEL_FN=100)
KERNEL = dict(NONE=-1, ROW_SUM_F32=1, ROW_MAX_ARGMAX_BF16=2, SCAN_I32=3, GATHER_ROWS=4, DEQUANT_I4=5,
              W4A16_GEMM=6, REDUCE2D_F32=7, REDUCE2D_I32=8, SCATTER=9, BINCOUNT=10, REDUCE_F32=11, REDUCE_I32=12,
              ROW_REDUCE_F32=13, COL_SUM_SPLITK=14, WINDOW=15, IM2COL=16)
ROW_REDUCE_FORM = dict(NONE=0, SOFTMAX=1, RMS_NORM=2, CENTRED=3)
# WriteCombine ordinals (crates/unpopped/src/ir.rs:2723-2732)
COMBINE = dict(ASSIGN=0, ADD=1, MAX=2, MIN=3)
LOWER_ERROR = {0: "Ok", 1: "UnsupportedDtype", 2: "UnsupportedSchedule", 3: "UnsupportedOp",
               4: "UnsupportedPlanShape", 5: "InadmissiblePlan", 6: "UnsupportedKernel"}

MAX_RANK = 8


class UpTensor(ctypes.Structure):
    _fields_ = [("ptr", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("shape", ctypes.c_int64 * MAX_RANK), ("stride", ctypes.c_int64 * MAX_RANK),
                ("base", ctypes.c_int64)]


class UpPlanDesc(ctypes.Structure):
    _fields_ = [("schedule", ctypes.c_int32), ("op", ctypes.c_int32), ("dtype", ctypes.c_int32),
                ("out_dtype", ctypes.c_int32), ("axes_mask", ctypes.c_uint32), ("keepdim", ctypes.c_int32),
                ("identity_body", ctypes.c_int32), ("accum", ctypes.c_int32), ("block", ctypes.c_int32),
                ("scan_axis", ctypes.c_int32), ("exclusive", ctypes.c_int32), ("reverse", ctypes.c_int32),
                ("has_read_index", ctypes.c_int32), ("gather_axis", ctypes.c_int32), ("oob", ctypes.c_int32),
                ("index_dtype", ctypes.c_int32), ("n_operands", ctypes.c_int32), ("operands", UpTensor * 8),
                ("target", ctypes.c_char * 32), ("has_write_index", ctypes.c_int32), ("scatter_axis", ctypes.c_int32),
                ("combine", ctypes.c_int32), ("count", ctypes.c_int32), ("row_reduce_form", ctypes.c_int32),
                ("eps", ctypes.c_double), ("splitk_chunks", ctypes.c_int64),
                ("window_axis", ctypes.c_int32), ("window_size", ctypes.c_int32), ("window_stride", ctypes.c_int32),
                ("window_dilation", ctypes.c_int32), ("window_pad_lo", ctypes.c_int32),
                ("window_pad_hi", ctypes.c_int32), ("count_include_pad", ctypes.c_int32),
                ("im2col_kernel", ctypes.c_int32 * 2), ("im2col_stride", ctypes.c_int32 * 2),
                ("im2col_pad", ctypes.c_int32 * 2), ("im2col_dilation", ctypes.c_int32 * 2)]


class UpLowered(ctypes.Structure):
    _fields_ = [("kernel_id", ctypes.c_int32), ("lower_error", ctypes.c_int32), ("name", ctypes.c_char * 64),
                ("detail", ctypes.c_char * 160), ("scalars", ctypes.c_int64 * 8), ("n_scalars", ctypes.c_int32)]


class UpError(RuntimeError):
    def __init__(self, status: int, where: str, detail: str = ""):
        self.status = status
        super().__init__(f"{where}: {STATUS_NAMES.get(status, status)}{(' — ' + detail) if detail else ''}")


# Every symbol include/up_sm100.h declares, with its ctypes signature.
_P, _I, _I64, _U64, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_uint64, ctypes.c_size_t
SIGNATURES = {
    "up_sm100_version": ([], _I),
    "up_sm100_name": ([], ctypes.c_char_p),
    "up_sm100_provider": ([], ctypes.c_char_p),
    "up_sm100_supports_dtype": ([_I, ctypes.c_char_p], _I),
    "up_sm100_classify": ([ctypes.POINTER(UpPlanDesc), ctypes.POINTER(UpLowered)], _I),
    "up_sm100_workspace_bytes": ([ctypes.POINTER(UpTensor), _I, ctypes.POINTER(UpTensor), _I,
                                  ctypes.POINTER(ctypes.c_int64), _I, ctypes.POINTER(_SZ)], _I),
    "up_sm100_launch": ([_I, ctypes.POINTER(UpTensor), _I, ctypes.POINTER(UpTensor), _I,
                         ctypes.POINTER(ctypes.c_int64), _I, _P, _SZ, _P], _I),
    "up_sm100_workspace_status": ([_P, _P], _I),
    "up_sm100_row_sum_f32": ([_P, _I64, _I64, _I64, _P, _I, _I, _P], _I),
    "up_sm100_row_max_argmax_bf16": ([_P, _I64, _I64, _I64, _P, _P, _P, _P], _I),
    "up_sm100_scan_i32": ([_P, _P, _I64, _I64, _I, _I, _I, _P, _P, _SZ, _P], _I),
    "up_sm100_scan_workspace_bytes": ([_I64, _I64], _SZ),
    "up_sm100_scan_i32_noalloc": ([_P, _P, _I64, _I64, _I, _I, _I, _P, _I, _P], _I),
    "up_sm100_scan_i32_host": ([_P, _P, _I64, _I64, _I, _I, _I, _P], _I),
    "up_sm100_reduce2d_f32": ([_P, _I64, _I64, _I64, _I, _I, _I, _I, _P, _P], _I),
    "up_sm100_reduce2d_i32": ([_P, _I64, _I64, _I64, _I, _I, _P, _P], _I),
    "up_sm100_reduce3d_f32": ([_P, _I64, _I64, _I64, _I64, _I64, _I, _I, _I, _P, _I64, _P], _I),
    "up_sm100_reduce3d_i32": ([_P, _I64, _I64, _I64, _I64, _I64, _I, _P, _I64, _P], _I),
    "up_sm100_row_reduce_f32": ([_P, _I64, _I64, _I64, _I, _I, ctypes.c_double, _P, _I64, _P], _I),
    "up_sm100_col_sum_f32_splitk": ([_P, _I64, _I64, _I64, _I64, _I, _P, ctypes.c_size_t, _P, _P], _I),
    "up_sm100_col_sum_splitk_workspace_bytes": ([_I64, _I64, _I64], ctypes.c_size_t),
    "up_sm100_kernel_interface": ([_I, ctypes.c_char_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)], _I),
    "up_sm100_revision_hash": ([_I], ctypes.c_uint64),
    "up_sm100_window": ([_P, _I, _I64, _I64, _I64, _I, _I, _I, _I, _I, _I, _P, _I64, _P], _I),
    "up_sm100_im2col": ([_P, _I, _I64, _I64, _I64, _I64, _I, _I, _I, _I, _I, _I, _I, _I, _P, _P], _I),
    "up_sm100_scatter": ([_P, _I64, _I64, _I64, _I, _P, _I, _I64, _I, _P, _I64, _I64, _P], _I),
    "up_sm100_bincount": ([_P, _I64, _I, _P, _I64, _P], _I),
    "up_sm100_reduce_i32": ([_P, _I64, _I, _P, _P], _I),
    "up_sm100_gather_rows": ([_P, _I64, _I64, _P, _I, _I64, _I, _P, _P], _I),
    "up_sm100_dequant_i4_bf16": ([_P, _P, _I64, _I64, _I64, _P, _P], _I),
    "up_sm100_w4a16_gemm": ([_P, _P, _P, _I64, _I64, _I64, _I64, _P, _P, _SZ, _P], _I),
    "up_sm100_w4a16_workspace_bytes": ([_I64, _I64, _I64, _I64], _SZ),
    "up_sm100_set_wait_limit_ns": ([_U64], None),
    "up_sm100_set_test_withhold_flag": ([_I], None),
    "up_sm100_set_test_scan_epoch": ([_U64], None),
    "up_sm100_comm_unique_id": ([_P], _I),
    "up_sm100_comm_init_rank": ([_I, _I, _P, ctypes.POINTER(ctypes.c_void_p)], _I),
    "up_sm100_comm_init": ([_I, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_void_p)], _I),
    "up_sm100_comm_destroy": ([_P], _I),
    "up_sm100_comm_rank": ([_P, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)], _I),
    "up_sm100_workspace_bytes_multi": ([_I, ctypes.POINTER(UpTensor), _I, ctypes.POINTER(UpTensor), _I,
                                        ctypes.POINTER(ctypes.c_int64), _I, _P, ctypes.POINTER(_SZ)], _I),
    "up_sm100_launch_multi": ([_I, ctypes.POINTER(UpTensor), _I, ctypes.POINTER(UpTensor), _I,
                               ctypes.POINTER(ctypes.c_int64), _I, _P, _SZ, _P, _P], _I),
    "up_sm100_comm_set_test_launches": ([_P, _U64], None),
    "up_sm100_launch_count": ([], _U64),
    "up_sm100_last_error": ([], ctypes.c_char_p),
}
# up_sm100_workspace_bytes' first parameter is the kernel id
SIGNATURES["up_sm100_workspace_bytes"] = ([_I] + SIGNATURES["up_sm100_workspace_bytes"][0], _I)

_lib = None


def load():
    """Load libunpopped_sm100.so (raises if it is absent: there is no substitute implementation)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m unpopped_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = res
        _lib = L
    return _lib


def check(status: int, where: str):
    if status != UP_OK:
        detail = ""
        if status == UP_ERR_CUDA:
            detail = (load().up_sm100_last_error() or b"").decode()
        raise UpError(status, where, detail)
