"""GPU parity of the launched RowReduce forms (softmax, RMS norm, the centred quotient) against the CPU oracle
restatement and the reference test's corpora (crates/unpopped/tests/kernel_parallel_row_reduce_agrees.rs).

The tolerance is the reference's own: a launched softmax or RMS norm stays within 4 f32 ulps of the written order
(`transcendental_epilogues_stay_within_a_few_ulps_of_the_serial_lift`). The kernel evaluates exp in f64 with
CUDA's function and the oracle with the C library's, so the f64 values can differ in their last bit; after the
f32 rounding they are almost always identical, and the tests also require that of all but a tiny fraction of
cells. The centred quotient has no transcendental step and is bit-exact (`a_two_stage_op_follows_the_written_
order_bit_for_bit`)."""
import json
import os

import numpy as np
import pytest
import torch

import oracle as orc
from unpopped_b200 import ops
from unpopped_b200._lib import UpError
from unpopped_b200.backend import CudaSm100, Operand, Plan

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ULP_BAND = 4


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "these tests need the B200"


def golden():
    with open(os.path.join(GOLDEN, "row_reduce.json")) as f:
        return json.load(f)


def ulps(a, b):
    """Per-cell f32 ulp distance; NaN against NaN is 0, NaN against a number is huge."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    ka = a.view(np.int32).astype(np.int64)
    kb = b.view(np.int32).astype(np.int64)
    ka = np.where(ka < 0, -(1 << 31) - ka, ka)
    kb = np.where(kb < 0, -(1 << 31) - kb, kb)
    d = np.abs(ka - kb)
    na, nb = np.isnan(a), np.isnan(b)
    d = np.where(na & nb, 0, d)
    return np.where(na != nb, 1 << 40, d)


def check(got, want, exact=False):
    d = ulps(got, want)
    assert d.max() <= (0 if exact else ULP_BAND), int(d.max())
    if not exact:
        assert (d > 0).mean() <= 1e-3, (d > 0).mean()  # the f32 rounding hides the f64 exp's last bit


def test_reference_corpus_written_orders():
    g = golden()
    x = torch.from_numpy(np.array(g["gentle_f32_bits"], np.uint32).view(np.float32)).cuda()
    for b in g["blocks"]:
        want = np.array(g["centred_f32_bits"][str(b)], np.uint32).view(np.float32)
        check(ops.row_reduce(x, "centred", block=b).cpu().numpy(), want, exact=True)
        for form, key in (("softmax", "softmax_serial_f32_bits"), ("rms_norm", "rms_norm_serial_f32_bits")):
            want = np.array(g[key], np.uint32).view(np.float32)
            d = ulps(ops.row_reduce(x, form, block=b).cpu().numpy(), want)
            assert d.max() <= g["ulp_band"], (form, b, int(d.max()))


def test_reference_stress_corpus():
    """The huge/cancelling corpus: the centred quotient bit-exact, RMS norm within the band."""
    g = golden()
    xn = np.array(g["corpus_f32_bits"], np.uint32).view(np.float32)
    x = torch.from_numpy(xn).cuda()
    for b in g["blocks"]:
        check(ops.row_reduce(x, "centred", block=b).cpu().numpy(), orc.row_reduce_f32(xn, "centred", b), exact=True)
        check(ops.row_reduce(x, "rms_norm", block=b).cpu().numpy(), orc.row_reduce_f32(xn, "rms_norm", b))


SHAPES = [(1, 1), (3, 7), (17, 96), (64, 4097), (33, 8192), (1000, 5), (5, 1000), (300, 1024), (9, 12000), (2, 40000)]


@pytest.mark.parametrize("rows,cols", SHAPES)
@pytest.mark.parametrize("block", [1, 4, 32, 64, 256, 512, 1024])
def test_forms_vs_oracle(rows, cols, block):
    rng = np.random.default_rng(rows * 131 + cols + block)
    xn = (rng.standard_normal((rows, cols)) * 3).astype(np.float32)
    x = torch.from_numpy(xn).cuda()
    for form in ("softmax", "rms_norm"):
        check(ops.row_reduce(x, form, block=block).cpu().numpy(), orc.row_reduce_f32(xn, form, block))
    check(ops.row_reduce(x, "centred", block=block).cpu().numpy(), orc.row_reduce_f32(xn, "centred", block),
          exact=True)


def test_specials_and_eps():
    rng = np.random.default_rng(2)
    xn = rng.standard_normal((8, 300)).astype(np.float32)
    xn[0] = -np.inf          # softmax: -inf - -inf is NaN everywhere
    xn[1, 7] = np.nan        # NaN propagates through every form
    xn[2, 3] = np.inf
    xn[3] = 0.0              # RMS norm of zeros is 0 / sqrt(eps); the centred quotient is 0/0
    xn[4, ::2] = -0.0
    xn[5] *= 1e30            # x * x overflows f32 but not the f64 accumulator
    x = torch.from_numpy(xn).cuda()
    for form in ("softmax", "rms_norm", "centred"):
        for b in (1, 64, 256):
            d = ulps(ops.row_reduce(x, form, block=b).cpu().numpy(), orc.row_reduce_f32(xn, form, b))
            assert d.max() <= ULP_BAND, (form, b, int(d.max()))
    for eps in (0.0, 1e-6, 0.5):
        check(ops.row_reduce(x[6:], "rms_norm", eps=eps).cpu().numpy(), orc.row_reduce_f32(xn[6:], "rms_norm", 256, eps))


def test_strided_rows_and_output():
    rng = np.random.default_rng(5)
    full = rng.standard_normal((40, 130)).astype(np.float32)
    xv = torch.from_numpy(full).cuda()[:, 3:99]
    o_full = torch.full((40, 120), 7.0, device="cuda")
    ov = o_full[:, 10:106]
    ops.row_reduce(xv, "softmax", block=32, out=ov)
    check(ov.cpu().numpy(), orc.row_reduce_f32(np.ascontiguousarray(full[:, 3:99]), "softmax", 32))
    assert (o_full[:, :10] == 7).all() and (o_full[:, 106:] == 7).all()


def test_full_config_softmax_and_rms_norm():
    """cfg 1's 8192 x 8192 f32 rows."""
    rng = np.random.default_rng(11)
    xn = rng.standard_normal((8192, 8192), dtype=np.float32)
    x = torch.from_numpy(xn).cuda()
    t = orc.max_threads()
    for form in ("softmax", "rms_norm"):
        check(ops.row_reduce(x, form, block=256).cpu().numpy(), orc.row_reduce_f32(xn, form, 256, threads=t))


def test_plan_through_the_backend_rank3():
    rng = np.random.default_rng(8)
    xn = rng.standard_normal((4, 6, 200)).astype(np.float32)
    x = torch.from_numpy(xn).cuda()
    y = torch.empty_like(x)
    be = CudaSm100()
    plan = Plan("ROW_REDUCE", [Operand("F32", xn.shape), Operand("F32", xn.shape)], row_reduce_form="RMS_NORM",
                block=64, eps=1e-5)
    k = be.lower(plan)
    be.launch(k, [Operand("F32", xn.shape, ptr=x.data_ptr())], [Operand("F32", xn.shape, ptr=y.data_ptr())])
    check(y.cpu().numpy().reshape(24, 200), orc.row_reduce_f32(xn.reshape(24, 200), "rms_norm", 64, 1e-5))


def test_refusals():
    x = torch.zeros((4, 8), device="cuda")
    with pytest.raises(UpError):
        ops.row_reduce(x, "softmax", block=6)
    with pytest.raises(UpError):
        ops.row_reduce(x, "softmax", block=2048)
