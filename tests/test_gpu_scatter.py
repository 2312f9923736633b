"""GPU parity of the launched scatter (scatter / index_add with Add, Max, Min over axis 0) and bincount against the
CPU oracle restatement and the reference corpora. Integer results are bit-exact (the combines are
order-independent); an f32 add is checked against the reassociation band the reference states for its launched
float scatter, |got - exact| <= gamma_(n-1) * sum|terms|, u = 2^-24, and bit-exactly on integer-valued data."""
import json
import os

import numpy as np
import pytest
import torch

import oracle as orc
from unpopped_b200 import ops
from unpopped_b200._lib import UpError

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "these tests need the B200"


def golden():
    with open(os.path.join(GOLDEN, "scatter.json")) as f:
        return json.load(f)


def test_reference_corpus_every_integer_combine():
    g = golden()
    upd = torch.tensor(g["updates"], dtype=torch.int32).reshape(g["src"]).cuda()
    idx = torch.tensor(g["index"], dtype=torch.int32).reshape(g["src"]).cuda()
    for combine, exp in g["expected"].items():
        out = torch.tensor(g["init"], dtype=torch.int32).reshape(g["dst"]).cuda()
        ops.scatter(upd, idx, out, combine)
        assert out.reshape(-1).tolist() == exp, combine


def test_reference_bincount():
    b = golden()["bincount"]
    for dt in (torch.int32, torch.int64):
        counts = torch.zeros(b["bins"], dtype=torch.int32, device="cuda")
        ops.bincount(torch.tensor(b["x"], dtype=dt, device="cuda"), counts)
        assert counts.tolist() == b["counts"]


def test_reference_float_band():
    f = golden()["float_band"]
    upd = np.array(f["updates_f32_bits"], np.uint32).view(np.float32).reshape(f["src"])
    tgt = np.array(f["targets"], np.int32).reshape(f["src"])
    init = np.array(f["init_f32_bits"], np.uint32).view(np.float32).reshape(f["dst"])
    u = 2.0 ** -24
    for _ in range(5):  # several launches: the atomics may land in different orders
        out = torch.from_numpy(init.copy()).cuda()
        ops.scatter(torch.from_numpy(upd).cuda(), torch.from_numpy(tgt).cuda(), out, "add")
        got = out.cpu().numpy().reshape(-1)
        for c, (total, mag, n) in enumerate(f["cell_sum_abs_n"]):
            k = (n - 1) * u
            assert abs(float(got[c]) - total) <= k / (1 - k) * mag, c
            if n == 1:
                assert got[c] == init.reshape(-1)[c]  # an untouched cell is exactly its initial value


@pytest.mark.parametrize("dtype", [np.int32, np.uint32, np.int64])
@pytest.mark.parametrize("index_dtype", [np.int32, np.int64])
@pytest.mark.parametrize("form", ["full", "row"])
def test_integer_scatter_vs_oracle(dtype, index_dtype, form):
    rng = np.random.default_rng(hash((np.dtype(dtype).str, np.dtype(index_dtype).str, form)) % 2**32)
    n, cols, rows = 5000, 37, 300
    if dtype == np.uint32:
        upd = rng.integers(0, 2**32, (n, cols), dtype=np.uint64).astype(np.uint32)
        init = rng.integers(0, 2**32, (rows, cols), dtype=np.uint64).astype(np.uint32)
    else:
        info = np.iinfo(dtype)
        upd = rng.integers(info.min, info.max, (n, cols), dtype=dtype, endpoint=True)
        init = rng.integers(info.min, info.max, (rows, cols), dtype=dtype, endpoint=True)
    shape = (n, cols) if form == "full" else (n,)
    ids = rng.integers(-5, rows + 5, shape).astype(index_dtype)  # duplicates and out-of-range targets
    tu = torch.from_numpy(upd.view(np.int32) if dtype == np.uint32 else upd).cuda()
    ti = torch.from_numpy(ids).cuda()
    for combine in ("add", "max", "min"):
        out = torch.from_numpy((init.view(np.int32) if dtype == np.uint32 else init).copy()).cuda()
        if dtype == np.uint32:
            tu_, out_ = tu.view(torch.uint32), out.view(torch.uint32)
            ops.scatter(tu_, ti, out_, combine)
            got = out.cpu().numpy().view(np.uint32)
        else:
            ops.scatter(tu, ti, out, combine)
            got = out.cpu().numpy()
        assert np.array_equal(got, orc.scatter(upd, ids, init, combine)), combine


@pytest.mark.parametrize("dtype", [np.int32, np.uint32])
@pytest.mark.parametrize("cols", [4, 64, 256, 260])
def test_index_add_whole_rows(dtype, cols):
    """index_add of whole rows (one target per source row): duplicates, a hot row, out-of-range targets."""
    rng = np.random.default_rng(cols * 7 + (dtype == np.uint32))
    n, rows = 20000, 200
    if dtype == np.uint32:
        upd = rng.integers(0, 2**32, (n, cols), dtype=np.uint64).astype(np.uint32)
        init = rng.integers(0, 2**32, (rows, cols), dtype=np.uint64).astype(np.uint32)
    else:
        upd = rng.integers(-2**31, 2**31, (n, cols), dtype=np.int64).astype(np.int32)
        init = rng.integers(-2**31, 2**31, (rows, cols), dtype=np.int64).astype(np.int32)
    ids = rng.integers(-5, rows + 5, n).astype(np.int32)
    ids[::3] = 7  # a third of the rows go to one target
    for combine in ("add", "max", "min"):
        out = torch.from_numpy(init.view(np.int32).copy()).cuda()
        tu = torch.from_numpy(upd.view(np.int32)).cuda()
        if dtype == np.uint32:
            ops.scatter(tu.view(torch.uint32), torch.from_numpy(ids).cuda(), out.view(torch.uint32), combine)
        else:
            ops.scatter(tu, torch.from_numpy(ids).cuda(), out, combine)
        got = out.cpu().numpy().view(dtype)
        assert np.array_equal(got, orc.scatter(upd, ids, init, combine)), combine


def test_float_scatter_integer_valued_is_exact():
    """f32 and f64 adds of integer-valued data inside 2^24 are exact in every order."""
    rng = np.random.default_rng(3)
    for dt in (np.float32, np.float64):
        upd = rng.integers(-1000, 1000, (20000, 16)).astype(dt)
        init = rng.integers(-1000, 1000, (64, 16)).astype(dt)
        ids = rng.integers(-3, 67, (20000,)).astype(np.int32)
        out = torch.from_numpy(init.copy()).cuda()
        ops.scatter(torch.from_numpy(upd).cuda(), torch.from_numpy(ids).cuda(), out, "add")
        assert np.array_equal(out.cpu().numpy(), orc.scatter(upd, ids, init, "add"))


def test_bincount_large_and_prefilled():
    rng = np.random.default_rng(9)
    x = rng.integers(-100, 5100, 1 << 22).astype(np.int64)
    counts = rng.integers(0, 10, 5000).astype(np.int32)
    got = ops.bincount(torch.from_numpy(x).cuda(), torch.from_numpy(counts.copy()).cuda()).cpu().numpy()
    assert np.array_equal(got, orc.bincount(x, counts))


def test_strided_views_and_empty():
    rng = np.random.default_rng(4)
    full = rng.integers(-50, 50, (40, 20)).astype(np.int32)
    upd = torch.from_numpy(full).cuda()[:, 2:14]  # row stride 20
    ids = torch.from_numpy(rng.integers(-2, 9, 40).astype(np.int32)).cuda()
    dst_full = torch.zeros((8, 30), dtype=torch.int32, device="cuda")
    dst = dst_full[:, 5:17]  # row stride 30
    ops.scatter(upd, ids, dst, "add")
    want = orc.scatter(np.ascontiguousarray(full[:, 2:14]), ids.cpu().numpy(), np.zeros((8, 12), np.int32), "add")
    assert np.array_equal(dst.cpu().numpy(), want)
    assert (dst_full[:, :5] == 0).all() and (dst_full[:, 17:] == 0).all()  # nothing outside the view
    e = torch.zeros((0, 4), dtype=torch.int32, device="cuda")
    out = torch.ones((3, 4), dtype=torch.int32, device="cuda")
    ops.scatter(e, torch.zeros((0,), dtype=torch.int32, device="cuda"), out, "add")
    assert (out == 1).all()


def test_refusals():
    u = torch.zeros((4, 4), dtype=torch.int32, device="cuda")
    i = torch.zeros((4,), dtype=torch.int32, device="cuda")
    with pytest.raises(UpError):
        ops.scatter(u, i, u.clone(), "assign")
    f = torch.zeros((4, 4), dtype=torch.float32, device="cuda")
    with pytest.raises(UpError):
        ops.scatter(f, i, f.clone(), "max")
