"""GPU parity of the split-K variant of the outer-axis f32 Sum/Mean (crates/unpopped/ondevice/README.md:185-218)
against the CPU oracle restatement: bit-exact for every chunk count (the association is fixed by n_chunks), the
serial fold at n_chunks = 1, and the reference harness's corpus and zero-sign check (splitk_validate.cu:53-125)."""
import numpy as np
import pytest
import torch

import oracle as orc
from unpopped_b200 import _lib, ops
from unpopped_b200.backend import CudaSm100, Operand, Plan

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "these tests need the B200"


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def test_reference_harness_corpus():
    rows, cols = 100, 64
    x = np.array([((i % 37) - 18) * 0.25 for i in range(rows * cols)], np.float32).reshape(rows, cols)
    x[:, 0] = -0.0
    got = ops.col_sum_splitk(torch.from_numpy(x).cuda(), 3).cpu().numpy()
    assert np.array_equal(bits(got), bits(orc.col_sum_f32_splitk(x, 3)))
    assert bits(got)[0] == 0x00000000  # the zero-seeded fold: an all -0 column sums to +0
    serial = ops.reduce2d(torch.from_numpy(x).cuda(), "sum", 0).cpu().numpy()
    assert np.array_equal(bits(ops.col_sum_splitk(torch.from_numpy(x).cuda(), 1).cpu()), bits(serial))


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 7), (17, 96), (64, 4097), (1000, 5), (5, 1000), (4096, 256)])
def test_vs_oracle_every_chunk_count(rows, cols):
    rng = np.random.default_rng(rows * 17 + cols)
    xn = (rng.standard_normal((rows, cols)) * 10.0 ** rng.integers(-3, 4, (rows, 1))).astype(np.float32)
    x = torch.from_numpy(xn).cuda()
    for n in (1, 2, 3, 7, 64, rows, rows + 5):
        for mean in (False, True):
            got = ops.col_sum_splitk(x, n, mean).cpu().numpy()
            assert np.array_equal(bits(got), bits(orc.col_sum_f32_splitk(xn, n, mean))), (n, mean)


def test_strided_empty_and_full_size():
    rng = np.random.default_rng(6)
    full = rng.standard_normal((300, 130)).astype(np.float32)
    xv = torch.from_numpy(full).cuda()[:, 3:99]
    want = orc.col_sum_f32_splitk(np.ascontiguousarray(full[:, 3:99]), 9)
    assert np.array_equal(bits(ops.col_sum_splitk(xv, 9).cpu()), bits(want))
    e = torch.zeros((0, 8), device="cuda")
    assert (ops.col_sum_splitk(e, 4).cpu().numpy() == 0).all()
    assert torch.isnan(ops.col_sum_splitk(e, 4, mean=True)).all()
    xn = rng.standard_normal((8192, 8192), dtype=np.float32)
    got = ops.col_sum_splitk(torch.from_numpy(xn).cuda(), 64).cpu().numpy()
    assert np.array_equal(bits(got), bits(orc.col_sum_f32_splitk(xn, 64, threads=orc.max_threads())))


def test_plan_selects_the_variant_with_a_workspace():
    rng = np.random.default_rng(2)
    xn = rng.standard_normal((500, 64)).astype(np.float32)
    x = torch.from_numpy(xn).cuda()
    y = torch.empty(64, device="cuda")
    be = CudaSm100()
    plan = Plan("REDUCTION", [Operand("F32", xn.shape), Operand("F32", (64,))], op="MEAN", axes_mask=1,
                accum="AUTO", splitk_chunks=12)
    k = be.lower(plan)
    assert k.kernel_id == _lib.KERNEL["COL_SUM_SPLITK"]
    ins, outs = [Operand("F32", xn.shape, ptr=x.data_ptr())], [Operand("F32", (64,), ptr=y.data_ptr())]
    ws = torch.zeros(be.workspace_bytes(k, ins, outs), dtype=torch.uint8, device="cuda")
    be.launch(k, ins, outs, workspace=ws)
    assert np.array_equal(bits(y.cpu()), bits(orc.col_sum_f32_splitk(xn, 12, True)))
