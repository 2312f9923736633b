"""The C-ABI library loads, exports every symbol include/up_sm100.h declares, and answers the Backend seam
(name, provider, supports_dtype, lower) on the CPU. No kernel is launched here."""
import ctypes
import os
import re

import pytest

from unpopped_b200 import _lib
from unpopped_b200._lib import COMBINE, OP
from unpopped_b200.backend import CudaSm100, LowerError, Operand, Plan

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "up_sm100.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^UP_API [^(]*?\b(up_sm100_\w+)\(", text, flags=re.M)))


def test_header_declares_the_entry_points():
    syms = declared_symbols()
    assert "up_sm100_launch" in syms and "up_sm100_classify" in syms and len(syms) >= 20


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    for s in declared_symbols():
        assert hasattr(L, s), s
    # and the ctypes binding covers exactly the declared set
    assert set(_lib.SIGNATURES) == set(declared_symbols())


def test_name_provider_version():
    b = CudaSm100()
    assert b.name() == "cuda_sm100"
    assert b.provider() == "unpopped-cuda-sm100"
    assert _lib.load().up_sm100_version() == 1


@pytest.mark.parametrize("target", ["cuda:sm_100a", "cuda:sm100a", "cuda:sm100"])
def test_supports_dtype_on_our_targets(target):
    b = CudaSm100()
    for dt in ("F32", "BF16", "F16", "I32", "I64", "U32", "I4", "U8", "F64"):
        assert b.supports_dtype(dt, target) == "Supported", dt
    for dt in ("FP8_E4M3FNUZ", "FP8_E5M2FNUZ", "U4", "B1", "F4_E2M1"):
        assert b.supports_dtype(dt, target) == "Unsupported", dt


def test_supports_dtype_declines_other_targets():
    b = CudaSm100()
    for target in ("cuda:sm89", "cuda:sm90a", "vulkan:spirv1.6", "rocm:gfx942"):
        assert b.supports_dtype("F32", target) == "Unsupported"


def _red(op, dtype, out_dtype=None, shape=(64, 96), **kw):
    return Plan("REDUCTION", [Operand(dtype, shape), Operand(out_dtype or dtype, shape[:1])], dtype=dtype,
                out_dtype=out_dtype, op=op, **kw)


def test_dispatch_table_maps_the_reduction_breadth():
    b = CudaSm100()
    k = b.lower(_red("MEAN", "F32", accum="AUTO", block=64))
    assert (k.name, k.scalars) == ("up_sm100_reduce2d_f32", (OP["MEAN"], 1, 0, 64))
    for op in ("MAX", "MIN"):
        k = b.lower(_red(op, "F32"))
        assert (k.name, k.scalars[:2]) == ("up_sm100_reduce2d_f32", (OP[op], 1))
        k = b.lower(_red(op, "F32", axes_mask=1))
        assert (k.name, k.scalars[:2]) == ("up_sm100_reduce2d_f32", (OP[op], 0))
    k = b.lower(_red("SUM", "F32", axes_mask=1, accum="AUTO"))
    assert (k.name, k.scalars) == ("up_sm100_reduce2d_f32", (OP["SUM"], 0, 0, 1))
    for op in ("SUM", "PROD", "MAX", "MIN", "AND", "OR", "XOR"):
        for mask, axis in ((0, 1), (2, 1), (1, 0)):
            k = b.lower(_red(op, "I32", axes_mask=mask))
            assert (k.name, k.scalars) == ("up_sm100_reduce2d_i32", (OP[op], axis)), (op, mask)


def test_dispatch_table_maps_middle_and_multi_axis_reductions():
    """Any rank, any one run of adjacent reduced axes: flattened to [A, R, C] at launch."""
    b = CudaSm100()
    for shape, mask in (((4, 8, 16), 2), ((4, 8, 16), 4), ((4, 8, 16), 3), ((2, 3, 4, 5), 6), ((2, 3, 4, 5), 12)):
        k = b.lower(_red("SUM", "F32", shape=shape, axes_mask=mask, accum="AUTO"))
        assert (k.name, k.scalars[:2]) == ("up_sm100_reduce3d_f32", (OP["SUM"], mask)), (shape, mask)
        for op in ("MAX", "XOR"):
            dt = "F32" if op == "MAX" else "I32"
            k = b.lower(_red(op, dt, shape=shape, axes_mask=mask))
            assert k.name == f"up_sm100_reduce3d_{dt.lower()}" and k.scalars[:2] == (OP[op], mask)


def test_dispatch_table_maps_row_reduce_forms():
    b = CudaSm100()
    for form in ("SOFTMAX", "RMS_NORM", "CENTRED"):
        for shape in ((64, 96), (3, 4, 96)):
            k = b.lower(Plan("ROW_REDUCE", [Operand("F32", shape), Operand("F32", shape)], row_reduce_form=form,
                             block=128, eps=0.25))
            assert k.name == "up_sm100_row_reduce_f32"
            assert k.scalars[:2] == (_lib.ROW_REDUCE_FORM[form], 128)
            assert ctypes.c_int64(k.scalars[2]).value == ctypes.cast(ctypes.pointer(ctypes.c_double(0.25)),
                                                                      ctypes.POINTER(ctypes.c_int64)).contents.value


def test_splitk_variant_is_selected_only_for_the_outer_axis_sum():
    b = CudaSm100()
    k = b.lower(_red("SUM", "F32", axes_mask=1, accum="AUTO", splitk_chunks=16))
    assert (k.name, k.scalars) == ("up_sm100_col_sum_f32_splitk", (0, 16))
    k = b.lower(_red("MEAN", "F32", axes_mask=1, accum="AUTO", splitk_chunks=3))
    assert (k.name, k.scalars) == ("up_sm100_col_sum_f32_splitk", (1, 3))
    for plan in (_red("MAX", "F32", axes_mask=1, splitk_chunks=4), _red("SUM", "F32", accum="AUTO", splitk_chunks=4)):
        with pytest.raises(LowerError) as e:
            b.lower(plan)
        assert e.value.variant == "UnsupportedPlanShape"
    assert _lib.load().up_sm100_col_sum_splitk_workspace_bytes(100, 64, 3) == 3 * 64 * 8
    assert _lib.load().up_sm100_col_sum_splitk_workspace_bytes(2, 64, 30) == 2 * 64 * 8  # at most one chunk per row


def test_dispatch_table_maps_window_and_im2col():
    b = CudaSm100()
    k = b.lower(Plan("WINDOW", [Operand("F32", (3, 9)), Operand("F32", (3, 5))], op="MEAN", window=(1, 3, 2, 1, 1, 1),
                     count_include_pad=True))
    assert (k.name, k.scalars) == ("up_sm100_window", (OP["MEAN"], 3, 2, 1, 1, 1, 1))
    k = b.lower(Plan("WINDOW", [Operand("I32", (4, 9, 5)), Operand("I32", (4, 3, 5))], dtype="I32", op="MAX",
                     window=(1, 3, 3, 1, 0, 0)))
    assert (k.name, k.scalars) == ("up_sm100_window", (OP["MAX"], 3, 3, 1, 0, 0, 1))
    k = b.lower(Plan("IM2COL", [Operand("BF16", (2, 3, 5, 7)), Operand("BF16", (2, 18, 12))],
                     im2col=((2, 3), (1, 2), (0, 2), (2, 1))))
    assert (k.name, k.scalars) == ("up_sm100_im2col", (2, 3, 1, 2, 0, 2, 2, 1))


def _scatter(dtype, index_shape, index_strides, combine="ADD", shape=(9, 4), out_rows=5, **kw):
    return Plan("STRIDED", [Operand(dtype, shape), Operand("I32", index_shape, index_strides),
                            Operand(dtype, (out_rows, shape[1]))], dtype=dtype, write_index=True, combine=combine, **kw)


def test_dispatch_table_maps_scatter_and_bincount():
    b = CudaSm100()
    for combine in ("ADD", "MAX", "MIN"):
        k = b.lower(_scatter("I32", (9, 4), (4, 1), combine))
        assert (k.name, k.scalars) == ("up_sm100_scatter", (COMBINE[combine], 1))
    k = b.lower(_scatter("I64", (9,), (1,)))  # index_add: one target per update row
    assert (k.name, k.scalars) == ("up_sm100_scatter", (COMBINE["ADD"], 0))
    assert b.lower(_scatter("F32", (9, 4), (4, 1))).name == "up_sm100_scatter"
    bc = Plan("STRIDED", [Operand("I32", (14,)), Operand("I32", (6,))], dtype="I32", write_index=True, count=True)
    assert b.lower(bc).name == "up_sm100_bincount"
    for plan, variant in ((_scatter("I32", (9, 4), (4, 1), "ASSIGN"), "UnsupportedOp"),
                          (_scatter("F32", (9, 4), (4, 1), "MAX"), "UnsupportedOp"),
                          (_scatter("F16", (9, 4), (4, 1)), "UnsupportedDtype"),
                          (_scatter("I32", (9, 4), (4, 1), scatter_axis=1), "UnsupportedPlanShape"),
                          (_scatter("I32", (3, 4), (4, 1)), "UnsupportedPlanShape")):
        with pytest.raises(LowerError) as e:
            b.lower(plan)
        assert e.value.variant == variant


def test_dispatch_table_maps_each_lift():
    b = CudaSm100()
    k = b.lower(_red("SUM", "F32"))
    assert (k.name, k.scalars) == ("up_sm100_row_sum_f32", (1, 256))
    k = b.lower(_red("SUM", "F32", accum="AUTO", block=128))
    assert k.scalars == (0, 128)
    assert b.lower(_red("MAX", "BF16", "F32")).name == "up_sm100_row_max_argmax_bf16"
    assert b.lower(_red("ARGMAX", "BF16", "I64")).name == "up_sm100_row_max_argmax_bf16"
    for op in ("SUM", "MAX", "MIN"):
        for excl in (False, True):
            for rev in (False, True):
                k = b.lower(Plan("SCAN", [Operand("I32", (1 << 28,)), Operand("I32", (1 << 28,))], dtype="I32",
                                 op=op, exclusive=excl, reverse=rev))
                assert k.name == "up_sm100_scan_i32" and k.scalars == (_lib.OP[op], int(excl), int(rev))
    g = Plan("STRIDED", [Operand("BF16", (1 << 20, 256)), Operand("I32", (1 << 24, 256), (1, 0)),
                         Operand("BF16", (1 << 24, 256))], dtype="BF16", read_index=True, oob="ZERO_FILL")
    k = b.lower(g)
    assert k.name == "up_sm100_gather_rows" and k.scalars == (_lib.OOB["ZERO_FILL"],)
    w = Plan("KERNEL_FN", [Operand("I4", (28672, 8192)), Operand("F16", (28672, 64)), Operand("BF16", (16, 8192)),
                           Operand("BF16", (16, 28672))])
    k = b.lower(w)
    assert k.name == "up_sm100_w4a16_gemm" and k.scalars == (128,)
    d = Plan("KERNEL_FN", [Operand("I4", (256, 512)), Operand("F16", (256, 4)), Operand("BF16", (256, 512))])
    assert b.lower(d).name == "up_sm100_dequant_i4_bf16"


@pytest.mark.parametrize("plan,variant", [
    (_red("SUM", "F64"), "UnsupportedDtype"),
    (_red("PROD", "F32"), "UnsupportedOp"),
    (_red("SUM", "F32", shape=(4, 8, 16), axes_mask=2), "UnsupportedOp"),  # a middle axis: Auto only
    (_red("MAX", "F32", shape=(4, 8, 16), axes_mask=5), "UnsupportedPlanShape"),  # axes 0 and 2: not one run
    (_red("MAX", "I32", shape=(4, 8, 16), axes_mask=8), "UnsupportedPlanShape"),  # no such axis
    (_red("SUM", "F32", axes_mask=1), "UnsupportedOp"),  # outer axis under the F32 policy: Auto only
    (_red("SUM", "F32", axes_mask=1, accum="AUTO", block=512), "UnsupportedPlanShape"),  # outer block <= 256
    (_red("MEAN", "I32"), "UnsupportedOp"),  # the oracle has no integer Mean
    (_red("AND", "F32"), "UnsupportedOp"),  # bit folds are integer-only
    (_red("ARGMAX", "F32", "I64"), "UnsupportedDtype"),
    (_red("ARGMAX", "BF16", "F32"), "InadmissiblePlan"),
    (_red("SUM", "F32", accum="AUTO", block=3), "UnsupportedPlanShape"),
    (Plan("SCAN", [Operand("F32", (8,)), Operand("F32", (8,))], dtype="F32"), "UnsupportedDtype"),
    (Plan("ROW_REDUCE", [Operand("F32", (4, 8)), Operand("F32", (4, 8))]), "UnsupportedOp"),  # not a named form
    (Plan("ROW_REDUCE", [Operand("I32", (4, 8)), Operand("I32", (4, 8))], dtype="I32", row_reduce_form="SOFTMAX"),
     "UnsupportedDtype"),
    (Plan("ROW_REDUCE", [Operand("F32", (8,)), Operand("F32", (8,))], row_reduce_form="SOFTMAX"),
     "UnsupportedPlanShape"),  # no leading axis to stride blocks over
    (Plan("ROW_REDUCE", [Operand("F32", (4, 8)), Operand("F32", (4, 8))], row_reduce_form="SOFTMAX", block=6),
     "UnsupportedPlanShape"),
    (Plan("SCAN", [Operand("I32", (4, 8)), Operand("I32", (4, 8))], dtype="I32", scan_axis=0), "UnsupportedPlanShape"),
    (Plan("STRIDED", [Operand("F32", (8,)), Operand("F32", (8,))]), "UnsupportedSchedule"),
    (Plan("WINDOW", [Operand("F32", (8,)), Operand("F32", (8,))], op="PROD"), "UnsupportedOp"),  # Prod refused
    (Plan("WINDOW", [Operand("I32", (8,)), Operand("I32", (8,))], dtype="I32", op="MEAN"), "UnsupportedOp"),
    (Plan("WINDOW", [Operand("F64", (8,)), Operand("F64", (8,))], dtype="F64"), "UnsupportedDtype"),
    (Plan("IM2COL", [Operand("F32", (1, 1, 4, 4)), Operand("F32", (9, 16))]), "UnsupportedPlanShape"),  # rank-2 out
    (Plan("IM2COL", [Operand("I4", (1, 1, 4, 4)), Operand("I4", (1, 1, 16))]), "UnsupportedDtype"),
    (Plan("CONTRACTION", [Operand("F32", (8, 8)), Operand("F32", (8, 8))]), "UnsupportedSchedule"),
    (Plan("KERNEL_FN", [Operand("F32", (8,))]), "UnsupportedKernel"),
    (_red("SUM", "F32", target="cuda:sm90a"), "UnsupportedSchedule"),
])
def test_refuses_rather_than_approximates(plan, variant):
    with pytest.raises(LowerError) as e:
        CudaSm100().lower(plan)
    assert e.value.variant == variant


def test_argument_errors_return_before_any_device_work():
    L = _lib.load()
    # negative extents, unknown ops and policies are refused on the host
    assert L.up_sm100_row_sum_f32(None, -1, 4, 4, None, 1, 256, None) == _lib.UP_ERR_INVALID
    assert L.up_sm100_row_sum_f32(None, 0, 4, 4, None, 1, 256, None) == _lib.UP_OK  # empty: nothing to do
    assert L.up_sm100_scan_i32(None, None, 1, 8, 7, 0, 0, None, None, 0, None) == _lib.UP_ERR_UNSUPPORTED
    assert L.up_sm100_scan_i32(None, None, 0, 8, 0, 0, 0, None, None, 0, None) == _lib.UP_OK
    assert L.up_sm100_gather_rows(None, 4, 16, None, _lib.EK["F32"], 4, 0, None, None) == _lib.UP_ERR_UNSUPPORTED
    assert L.up_sm100_gather_rows(None, 4, 16, None, _lib.EK["I32"], 4, 9, None, None) == _lib.UP_ERR_UNSUPPORTED
    assert L.up_sm100_dequant_i4_bf16(None, None, 4, 100, 64, None, None) == _lib.UP_ERR_UNSUPPORTED
    assert L.up_sm100_w4a16_gemm(None, None, None, 17, 128, 128, 128, None, None, 0, None) == _lib.UP_ERR_UNSUPPORTED
    assert L.up_sm100_w4a16_gemm(None, None, None, 16, 128, 100, 128, None, None, 0, None) == _lib.UP_ERR_UNSUPPORTED
    assert L.up_sm100_reduce_i32(None, 4, 4, None, None) == _lib.UP_ERR_INVALID


def test_workspace_sizes():
    L = _lib.load()
    assert L.up_sm100_scan_workspace_bytes(1, 1 << 28) == 64 + 8 * ((1 << 28) // 8192)  # one flag per 8192-tile
    assert L.up_sm100_scan_workspace_bytes(3, 40000) == 64 + 8 * 3 * 5
    assert L.up_sm100_w4a16_workspace_bytes(16, 28672, 8192, 128) > 64
    n = ctypes.c_size_t(0)
    ins = (_lib.UpTensor * 1)(Operand("I32", (4, 40000)).to_c())
    assert L.up_sm100_workspace_bytes(_lib.KERNEL["SCAN_I32"], ins, 1, ins, 1, None, 0, ctypes.byref(n)) == 0
    assert n.value == 64 + 8 * 4 * 5


# The reference's cross-emitter corpus (crates/unpopped/src/launch_cases.rs:140-180): four launched elementwise kernels,
# each with two inputs and one output of one dtype. This backend's kernel layer takes only the dequant-GEMM function,
# so its conformance answer for every case is the typed UnsupportedKernel decline, never an approximation.
LAUNCH_CASES = [("fma_shape_f32", "F32", (5, 7)), ("div_f32", "F32", (6, 5)), ("sub_i32", "I32", (3, 11)),
                ("add_u32", "U32", (37,))]


@pytest.mark.parametrize("name,dtype,shape", LAUNCH_CASES)
def test_launch_cases_corpus_is_declined_with_unsupported_kernel(name, dtype, shape):
    b = CudaSm100()
    plan = Plan("KERNEL_FN", [Operand(dtype, shape), Operand(dtype, shape), Operand(dtype, shape)], dtype=dtype)
    with pytest.raises(LowerError) as e:
        b.lower(plan)
    assert e.value.variant == "UnsupportedKernel", name
