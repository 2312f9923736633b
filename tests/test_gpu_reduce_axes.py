"""GPU parity of reductions over a middle axis and over several adjacent axes (`ReduceAxisClass::Middle` and
`Multi`, plan/types.rs:150-165) against the CPU oracle. The oracle folds every output cell over the reduced
coordinates in row-major order (oracle/plan_eval.rs:565-605), so a run of adjacent reduced axes is one flattened
axis: [A, R, C] with A the kept leading axes and C the kept trailing ones. Every result is bit-exact."""
import numpy as np
import pytest
import torch

import oracle as orc
from unpopped_b200 import ops
from unpopped_b200.backend import CudaSm100, Operand, Plan

pytestmark = pytest.mark.gpu
INT_OPS = ("sum", "prod", "max", "min", "and", "or", "xor")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "these tests need the B200"


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _floats(rng, shape):
    x = (rng.standard_normal(shape) * 10.0 ** rng.integers(-3, 4, shape[:-1] + (1,))).astype(np.float32)
    pick = rng.random(shape)
    x[pick < 0.02] = -0.0
    x[(pick >= 0.02) & (pick < 0.03)] = np.inf
    x.view(np.uint32)[pick > 0.997] = 0x7fa00001  # a NaN with a payload
    return x


def _middle_oracle(x3, op, block=1):
    """[A, R, C] -> [A, C]: the outer-axis fold of each batch."""
    out = []
    for a in range(x3.shape[0]):
        if x3.dtype == np.int32:
            out.append(orc.reduce2d_i32(x3[a], op, 0))
        elif op in ("sum", "mean") and block > 1:
            out.append(orc.col_sum_f32_documented(x3[a], block, mean=op == "mean"))
        else:
            out.append(orc.reduce2d_f32(x3[a], op, 0))
    return np.stack(out) if out else np.zeros((0, x3.shape[2]), x3.dtype)


@pytest.mark.parametrize("shape", [(3, 17, 96), (5, 1000, 36), (2, 33, 8192), (70, 9, 4), (4, 40, 7), (1, 64, 256)])
def test_middle_axis_f32_vs_oracle(shape):
    rng = np.random.default_rng(sum(shape))
    xn = _floats(rng, shape)
    x = torch.from_numpy(xn).cuda()
    for op in ("max", "min"):
        assert np.array_equal(bits(ops.reduce3d(x, op).cpu()), bits(_middle_oracle(xn, op))), op
    xs = np.nan_to_num(xn, nan=1.0, posinf=2.0).astype(np.float32)  # sums of finite values
    x = torch.from_numpy(xs).cuda()
    for op in ("sum", "mean"):
        for b in (1, 2, 64, 128, 256):
            got = bits(ops.reduce3d(x, op, block=b).cpu())
            assert np.array_equal(got, bits(_middle_oracle(xs, op, b))), (op, b)


@pytest.mark.parametrize("shape", [(3, 17, 96), (5, 1000, 36), (70, 9, 4), (4, 40, 7)])
def test_middle_axis_i32_vs_oracle(shape):
    rng = np.random.default_rng(7 * sum(shape))
    xn = rng.integers(-2**31, 2**31, shape, dtype=np.int64).astype(np.int32)
    xn[..., ::3] = rng.integers(-3, 4, xn[..., ::3].shape)
    x = torch.from_numpy(xn).cuda()
    for op in INT_OPS:
        assert np.array_equal(ops.reduce3d(x, op).cpu().numpy(), _middle_oracle(xn, op)), op


def test_middle_axis_strided_batches_and_empty():
    rng = np.random.default_rng(3)
    full = _floats(rng, (6, 20, 40))
    x = torch.from_numpy(full).cuda()[::2, 1:18, 4:36]  # batch stride 1600, row stride 40, unaligned start
    sub = np.ascontiguousarray(full[::2, 1:18, 4:36])
    for op in ("max", "min"):
        assert np.array_equal(bits(ops.reduce3d(x, op).cpu()), bits(_middle_oracle(sub, op)))
    e = torch.zeros((3, 0, 8), dtype=torch.int32, device="cuda")
    for op in INT_OPS:
        assert (ops.reduce3d(e, op).cpu().numpy() == (1 if op == "prod" else 0)).all()
    assert torch.isnan(ops.reduce3d(torch.zeros((2, 0, 8), device="cuda"), "mean")).all()


def _geometry(shape, mask):
    i = (mask & -mask).bit_length() - 1
    j = mask.bit_length()
    a = int(np.prod(shape[:i], dtype=np.int64))
    r = int(np.prod(shape[i:j], dtype=np.int64))
    c = int(np.prod(shape[j:], dtype=np.int64))
    return a, r, c


@pytest.mark.parametrize("shape,mask", [((4, 8, 16), 2), ((4, 8, 16), 3), ((4, 8, 16), 6), ((2, 3, 4, 5), 6),
                                        ((2, 3, 4, 5), 12), ((2, 3, 4, 8), 7), ((3, 5, 64), 4), ((6, 1, 5, 12), 2)])
def test_plans_of_any_rank_through_the_backend(shape, mask):
    """Lower a Reduction plan with an axes mask and launch it through the C ABI on device buffers."""
    rng = np.random.default_rng(mask * 31 + len(shape))
    be = CudaSm100()
    a, r, c = _geometry(shape, mask)
    kept = tuple(d for k, d in enumerate(shape) if not (mask >> k) & 1)
    for dt, op in (("F32", "MAX"), ("F32", "SUM"), ("F32", "MEAN"), ("I32", "XOR"), ("I32", "PROD")):
        if dt == "F32":
            xn = (rng.standard_normal(shape) * 100).astype(np.float32)
        else:
            xn = rng.integers(-2**31, 2**31, shape, dtype=np.int64).astype(np.int32)
        x = torch.from_numpy(xn).cuda()
        y = torch.empty(kept, dtype=x.dtype, device="cuda")
        plan = Plan("REDUCTION", [Operand(dt, shape), Operand(dt, kept)], dtype=dt, op=op, axes_mask=mask,
                    accum="AUTO")
        k = be.lower(plan)
        be.launch(k, [Operand(dt, shape, ptr=x.data_ptr())], [Operand(dt, kept, ptr=y.data_ptr())])
        x3 = xn.reshape(a, r, c)
        if c == 1:  # a last-axis reduction: rows of r
            x2 = x3.reshape(a, r)
            if dt == "I32":
                want = orc.reduce2d_i32(x2, op.lower(), 1)
            elif op == "SUM":
                want = orc.row_sum_f32_documented(x2, 256)
            elif op == "MEAN":
                want = orc.row_mean_f32_documented(x2, 256)
            else:
                want = orc.reduce2d_f32(x2, op.lower(), 1)
        else:
            want = _middle_oracle(x3, op.lower())
        got = y.cpu().numpy().reshape(-1)
        if dt == "F32":
            assert np.array_equal(bits(got), bits(want.reshape(-1))), (dt, op)
        else:
            assert np.array_equal(got, want.reshape(-1)), (dt, op)


def test_full_size_middle_axis():
    """[64, 1024, 1024] f32 (268 MB) over the middle axis: Max and the documented Sum against the oracle."""
    rng = np.random.default_rng(12)
    xn = rng.standard_normal((64, 1024, 1024), dtype=np.float32)
    x = torch.from_numpy(xn).cuda()
    t = orc.max_threads()
    want_max = np.stack([orc.reduce2d_f32(xn[a], "max", 0, t) for a in range(64)])
    assert np.array_equal(bits(ops.reduce3d(x, "max").cpu()), bits(want_max))
    want_sum = np.stack([orc.col_sum_f32_documented(xn[a], 256, threads=t) for a in range(64)])
    assert np.array_equal(bits(ops.reduce3d(x, "sum", block=256).cpu()), bits(want_sum))


def test_more_batches_than_one_launch_holds():
    """70,000 batches run as two launches of at most 65,535 (the grid's z extent)."""
    rng = np.random.default_rng(21)
    xf = rng.standard_normal((70000, 3, 4)).astype(np.float32)
    xi = rng.integers(-1000, 1000, (70000, 3, 4)).astype(np.int32)
    for op in ("max", "sum"):
        got = ops.reduce3d(torch.from_numpy(xf).cuda(), op).cpu().numpy()
        assert np.array_equal(bits(got), bits(_middle_oracle(xf, op))), op
    for op in ("xor", "min"):
        assert np.array_equal(ops.reduce3d(torch.from_numpy(xi).cuda(), op).cpu().numpy(), _middle_oracle(xi, op)), op
