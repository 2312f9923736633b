"""GPU parity of the int4 dequant (bit-exact) and of the tcgen05 W4A16 GEMM (within the stated bound) against
the oracle restatement, from small shapes that exercise split tiles up to the full 16 x 28672 x 8192 config.

W4A16 tolerance (f32 accumulation against the exact f64 sum, one bf16 rounding):
  |got - exact| <= 1/2 ulp_bf16(|exact|) + C * u * sum_k |x * w * s|,  u = 2^-24, C = 2,
and at least 99 % of the outputs are the correctly rounded bf16 of the exact sum. The a-priori bound of an f32
accumulation in this order, gamma_(K + 2G + 2) (one rounding per tensor-core accumulate step, the scale multiply and
add per k-block, and the split-tile partial sum; about 8,322 u at K = 8192), is far looser than what the kernel does:
measured, the error beyond the half ulp is at most 0.107 u * sum|x w s| on the full 16 x 28672 x 8192 config and
0.133 u on 7 x 38400 x 256, and 99.99 % of outputs are correctly rounded. C = 2 leaves a 15x margin over that and still
fails any change that loses f32 accumulation (a bf16 partial alone is 2^-9 relative, 32768 u).
"""
import numpy as np
import pytest
import torch

import oracle as orc
from unpopped_b200 import _lib, ops, workloads

pytestmark = pytest.mark.gpu
U32 = 2.0 ** -24
ACC_C = 2.0  # the accumulation allowance, in units of u * sum|x w s| (see the module docstring)


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "these tests need the B200"


def ulp_bf16(v):
    """Unit in the last place of the bf16 at |v| (for |v| in the normal range)."""
    a = np.abs(v).astype(np.float64)
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -126)))
    return 2.0 ** (e - 7)


def _np(t, dt):
    return t.cpu().contiguous().view({np.uint16: torch.int16, np.uint8: torch.uint8}[dt]).numpy().view(dt)


@pytest.mark.parametrize("n,k,group", [(128, 256, 128), (300, 512, 64), (64, 40, 8), (33, 24, 24), (1, 8, 8), (3, 6, 2),
                                       (5, 12, 4), (7, 16448, 64), (9000, 64, 64)])  # rows past 8192 k; many rows per CTA
def test_dequant_bit_exact(n, k, group):
    d = workloads.w4a16_inputs(n=n, k=k, m=1, group=group, seed=n + k)
    got = ops.dequant_i4(d.w_packed, d.scale, group)
    want = orc.dequant_i4_bf16(_np(d.w_packed, np.uint8), _np(d.scale.view(torch.int16), np.uint16), n, k, group)
    assert np.array_equal(_np(got.view(torch.int16), np.uint16), want)


def test_dequant_full_config():
    d = workloads.w4a16_inputs(device="cuda")
    got = ops.dequant_i4(d.w_packed, d.scale, d.group)
    # the oracle over a band of 1024 rows from several places
    for r0 in (0, 9000, 28672 - 1024):
        sl = slice(r0, r0 + 1024)
        want = orc.dequant_i4_bf16(_np(d.w_packed[sl], np.uint8), _np(d.scale[sl].view(torch.int16), np.uint16),
                                   1024, d.k, d.group)
        assert np.array_equal(_np(got[sl].view(torch.int16), np.uint16), want), r0


def _check_w4a16(d, got, threads=1):
    out, exact, abs_sum = orc.w4a16(_np(d.w_packed, np.uint8), _np(d.scale.view(torch.int16), np.uint16),
                                    _np(d.x.view(torch.int16), np.uint16), d.m, d.n, d.k, d.group, threads=threads)
    g = _np(got.view(torch.int16), np.uint16).astype(np.uint32)
    gv = (g << 16).view(np.float32).astype(np.float64)
    bound = 0.5 * ulp_bf16(exact) + ACC_C * U32 * abs_sum
    err = np.abs(gv - exact)
    bad = err > bound
    assert not bad.any(), (int(bad.sum()), float((err / bound).max()))
    # and nearly every output is the correctly rounded value itself
    assert np.mean(g == out) >= 0.99


@pytest.mark.parametrize("m,n,k", [(16, 128, 128), (16, 256, 1024), (1, 384, 512), (5, 1024, 2048),
                                   (16, 2048, 4096), (16, 200, 256), (7, 128 * 300, 256),
                                   (16, 1000, 640), (3, 512, 384),  # odd k-block counts: one-k-block units
                                   # many units a CTA (about 8), so every ring wraps several times per issuer
                                   (16, 9216, 4096), (5, 4096, 128 * 33)])
def test_w4a16_vs_oracle(m, n, k):
    d = workloads.w4a16_inputs(n=n, k=k, m=m, group=128, seed=m * n + k)
    got = ops.w4a16(d.w_packed, d.scale, d.x, 128)
    ops.check_workspace("w4a16", d.x.device)
    _check_w4a16(d, got, threads=orc.max_threads())


def test_w4a16_group_256_and_repeatability():
    d = workloads.w4a16_inputs(n=1024, k=2048, m=16, group=256, seed=3)
    a = ops.w4a16(d.w_packed, d.scale, d.x, 256)
    b = ops.w4a16(d.w_packed, d.scale, d.x, 256)
    ops.check_workspace("w4a16", d.x.device)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))  # split-tile fix-up order is fixed
    _check_w4a16(d, a, threads=orc.max_threads())


def test_w4a16_full_config():
    d = workloads.w4a16_inputs(device="cuda")
    got = ops.w4a16(d.w_packed, d.scale, d.x, d.group)
    ops.check_workspace("w4a16", d.x.device)
    _check_w4a16(d, got, threads=orc.max_threads())
    again = ops.w4a16(d.w_packed, d.scale, d.x, d.group)
    assert torch.equal(got.view(torch.int16), again.view(torch.int16))


def test_w4a16_refuses_unsupported_shapes():
    d = workloads.w4a16_inputs(n=128, k=256, m=1, group=128, seed=1)
    with pytest.raises(_lib.UpError) as e:
        ops.w4a16(d.w_packed, d.scale, torch.zeros(17, 256, dtype=torch.bfloat16, device="cuda"), 128)
    assert e.value.status == _lib.UP_ERR_UNSUPPORTED
