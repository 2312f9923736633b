"""GPU parity of the Window lift (1-D pooling: Sum, Mean, Max, Min along one axis) and the Im2Col lift against the
CPU oracle restatement and the reference tests' corpora (kernel_window_agrees.rs, kernel_int_window_agrees.rs,
kernel_im2col_agrees.rs). Every result is bit-exact: the window folds its taps in the oracle's order in f64, and
im2col is a raw-bit copy."""
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


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "these tests need the B200"


def load(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


def test_reference_window_corpora():
    g = load("window.json")
    vals = np.array(g["values_f32_bits"], np.uint32).view(np.float32)
    for name, c in g["cases"].items():
        rows, k_in, size, stride, dil, pad, inc, k_out = c["geometry"]
        x = torch.from_numpy(np.resize(vals, rows * k_in).reshape(rows, k_in)).cuda()
        for op, want in c["expected_f32_bits"].items():
            got = ops.window(x, op, size, stride, dil, pad, pad, bool(inc)).cpu().numpy()
            assert np.array_equal(bits(got), np.array(want, np.uint32)), (name, op)
    x = torch.from_numpy(np.array(g["nan_row_f32_bits"], np.uint32).view(np.float32)[None]).cuda()
    for op, want in g["nan_row_expected"].items():
        assert bits(ops.window(x, op, 3, 3).cpu().numpy())[0].tolist() == want, op
    x = torch.from_numpy(np.array(g["ascending_row_f32_bits"], np.uint32).view(np.float32)[None]).cuda()
    assert bits(ops.window(x, "sum", 9).cpu().numpy())[0].tolist() == g["ascending_sum_f32_bits"]
    ints = np.array(g["int_values"], np.int64).astype(np.int32)
    for name, c in g["int_cases"].items():
        rows, k_in, size, stride, dil, pad, _, k_out = c["geometry"]
        x = torch.from_numpy(np.resize(ints, rows * k_in).reshape(rows, k_in)).cuda()
        for op, want in c["expected"].items():
            assert ops.window(x, op, size, stride, dil, pad).cpu().numpy().tolist() == want, (name, op)


GEOMS = [(3, 1, 1, 0), (3, 2, 1, 1), (5, 3, 2, 2), (1, 1, 1, 0), (7, 4, 3, 3), (2, 2, 1, 0), (9, 1, 1, 4),
         (2, 1, 1, 1), (3, 1, 1, 2)]


# Inner extents that are a multiple of 4 floats take the staged kernel when a tile of 8 outputs fits its 32 KiB
# buffer ((2, 3000, 4), (3, 37, 8), (2, 10, 16), (2, 4, 3, 64), and (2, 21, 768) at stride 1), else the column
# kernel for sizes 2 and 3 at strides 1 and 2 ((2, 9, 4096), and (2, 21, 768) at stride 2): short axes whose output
# count is not a multiple of the tile, and padding in the first and last windows
@pytest.mark.parametrize("shape,axis", [((4, 1000), 1), ((6, 50, 33), 1), ((3, 40, 7, 5), 2), ((200,), 0),
                                        ((2, 3000, 4), 1), ((3, 37, 8), 1), ((2, 10, 16), 1), ((2, 4, 3, 64), 1),
                                        ((2, 21, 768), 1), ((2, 9, 4096), 1)])
@pytest.mark.parametrize("geom", GEOMS)
def test_window_vs_oracle(shape, axis, geom):
    size, stride, dil, pad = geom
    rng = np.random.default_rng(sum(shape) + 10 * size + stride + dil + pad)
    xf = (rng.standard_normal(shape) * 10.0 ** rng.integers(-3, 4, shape)).astype(np.float32)
    xf.reshape(-1)[rng.random(xf.size) < 0.01] = np.nan
    xf.reshape(-1)[rng.random(xf.size) < 0.01] = -0.0
    xi = rng.integers(-2**31, 2**31, shape, dtype=np.int64).astype(np.int32)
    k_in = shape[axis]
    if (k_in + 2 * pad - dil * (size - 1) - 1) // stride + 1 <= 0:
        pytest.skip("the window does not fit")
    for x in (xf, xi):
        t = torch.from_numpy(x).cuda()
        for op in (("sum", "mean", "max", "min") if x.dtype == np.float32 else ("sum", "max", "min")):
            for inc in ((False, True) if op == "mean" else (False,)):
                got = ops.window(t, op, size, stride, dil, pad, pad, inc, axis=axis).cpu().numpy()
                want = orc.window(x, op, size, stride, dil, pad, None, inc, axis=axis)
                assert np.array_equal(bits(got), bits(want)), (op, inc, x.dtype)


def test_window_with_no_real_tap_is_refused():
    """window_without_real_tap_declines.rs: a window made only of padding is refused, not filled."""
    x = torch.zeros((2, 4), device="cuda")
    with pytest.raises(UpError):
        ops.window(x, "max", 2, 1, 1, 3, 0)  # pad 3 > span: the first window lies wholly in the padding
    with pytest.raises(UpError):
        ops.window(x.to(torch.int32), "mean", 2)  # an integer Mean is not defined


def test_reference_im2col_corpus():
    for name, c in load("im2col.json").items():
        x = torch.from_numpy(np.array(c["x_f32_bits"], np.uint32).view(np.float32).reshape(c["shape"])).cuda()
        got = ops.im2col(x, c["kernel"], c["stride"], c["pad"], c["dilation"]).cpu().numpy()
        assert bits(got).reshape(-1).tolist() == c["expected_f32_bits"], name


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float64, torch.uint8, torch.int64])
@pytest.mark.parametrize("case", [((2, 3, 9, 11), (3, 3), (1, 1), (1, 1), (1, 1)),
                                  ((1, 4, 16, 16), (5, 5), (2, 2), (2, 2), (1, 1)),
                                  ((3, 2, 7, 13), (2, 3), (1, 2), (0, 2), (2, 1)),
                                  ((1, 1, 1, 1), (1, 1), (1, 1), (0, 0), (1, 1)),
                                  # output rows of 12 and 16 cells: the 16-byte-store path for the types they divide
                                  ((2, 3, 10, 12), (3, 3), (1, 1), (1, 1), (1, 1)),
                                  ((1, 2, 9, 16), (3, 3), (1, 1), (2, 2), (2, 2))])
def test_im2col_vs_oracle(dtype, case):
    shape, k, s, p, d = case
    rng = np.random.default_rng(sum(shape))
    raw = rng.integers(0, 256, int(np.prod(shape)) * torch.tensor([], dtype=dtype).element_size(), dtype=np.uint8)
    x = torch.from_numpy(raw).cuda().view(dtype).reshape(shape)
    got = ops.im2col(x, k, s, p, d)
    xn = raw.view({1: np.uint8, 2: np.uint16, 4: np.uint32, 8: np.uint64}[x.element_size()]).reshape(shape)
    want = orc.im2col(xn, k, s, p, d)
    g = got.cpu().contiguous().view(torch.uint8).numpy().view(want.dtype).reshape(want.shape)
    assert np.array_equal(g, want)


def test_full_size_pooling_and_unfold():
    """A 64 x 8192 x 128 f32 pool along the middle axis (268 MB) and a ResNet-stem im2col of 32 x 64 x 56 x 56."""
    rng = np.random.default_rng(3)
    xn = rng.standard_normal((64, 8192, 128), dtype=np.float32)
    x = torch.from_numpy(xn).cuda()
    for op in ("max", "mean"):
        got = ops.window(x, op, 3, 2, 1, 1, axis=1).cpu().numpy()
        assert np.array_equal(bits(got), bits(orc.window(xn, op, 3, 2, 1, 1, axis=1))), op
    im = torch.from_numpy(rng.standard_normal((32, 64, 56, 56), dtype=np.float32)).cuda()
    got = ops.im2col(im, (3, 3), (1, 1), (1, 1), (1, 1)).cpu().numpy()
    assert np.array_equal(bits(got), bits(orc.im2col(im.cpu().numpy(), (3, 3), (1, 1), (1, 1), (1, 1))))


def test_plans_through_the_backend():
    be = CudaSm100()
    rng = np.random.default_rng(1)
    xn = rng.standard_normal((4, 30, 6)).astype(np.float32)
    x = torch.from_numpy(xn).cuda()
    y = torch.empty((4, 15, 6), device="cuda")
    k = be.lower(Plan("WINDOW", [Operand("F32", xn.shape), Operand("F32", (4, 15, 6))], op="MEAN",
                      window=(1, 3, 2, 1, 1, 1), count_include_pad=True))
    be.launch(k, [Operand("F32", xn.shape, ptr=x.data_ptr())], [Operand("F32", (4, 15, 6), ptr=y.data_ptr())])
    assert np.array_equal(bits(y.cpu().numpy()), bits(orc.window(xn, "mean", 3, 2, 1, 1, 15, True, axis=1)))
    im = torch.from_numpy(rng.standard_normal((2, 3, 8, 8)).astype(np.float32)).cuda()
    o = torch.empty((2, 27, 64), device="cuda")
    k = be.lower(Plan("IM2COL", [Operand("F32", (2, 3, 8, 8)), Operand("F32", (2, 27, 64))],
                      im2col=((3, 3), (1, 1), (1, 1), (1, 1))))
    be.launch(k, [Operand("F32", (2, 3, 8, 8), ptr=im.data_ptr())], [Operand("F32", (2, 27, 64), ptr=o.data_ptr())])
    assert np.array_equal(bits(o.cpu().numpy()), bits(orc.im2col(im.cpu().numpy(), (3, 3), (1, 1), (1, 1), (1, 1))))


def test_unstaged_paths():
    """Rows longer than the shared-memory stage (innermost windows) and planes larger than it (im2col) take the
    unstaged kernels."""
    rng = np.random.default_rng(13)
    xn = rng.standard_normal((3, 20000)).astype(np.float32)
    x = torch.from_numpy(xn).cuda()
    for op in ("max", "mean", "sum"):
        got = ops.window(x, op, 3, 2, 1, 1).cpu().numpy()
        assert np.array_equal(bits(got), bits(orc.window(xn, op, 3, 2, 1, 1))), op
    im = rng.standard_normal((1, 2, 200, 200)).astype(np.float32)  # 160 KB planes
    got = ops.im2col(torch.from_numpy(im).cuda(), (3, 3), (2, 2), (1, 1), (1, 1)).cpu().numpy()
    assert np.array_equal(bits(got), bits(orc.im2col(im, (3, 3), (2, 2), (1, 1), (1, 1))))
