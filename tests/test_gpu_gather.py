"""GPU parity of the row gather: bit-exact against the oracle and the reference's OOB pool (Skip leaves the
pre-filled bytes, ZeroFill writes zeros, Clamp stores the clamped row), every index dtype, odd row sizes,
and the full Zipf configuration (checked against torch's own indexing and, on a sample, the oracle)."""
import json
import os

import numpy as np
import pytest
import torch

import oracle as orc
from unpopped_b200 import ops, workloads

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
POLICIES = {"skip": orc.OOB_SKIP, "clamp": orc.OOB_CLAMP, "zero_fill": orc.OOB_ZERO_FILL}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "these tests need the B200"


@pytest.mark.parametrize("policy", list(POLICIES))
def test_golden_oob_pool(policy):
    with open(os.path.join(GOLDEN, "gather_oob.json")) as f:
        g = json.load(f)
    table = torch.from_numpy(np.array(g["table_f32_bits"], np.uint32).view(np.int32)).cuda()
    ids = torch.tensor(g["ids_i32"], dtype=torch.int32, device="cuda")
    out = torch.full((ids.numel(), table.shape[1]), -0x54545455, dtype=torch.int32, device="cuda")  # 0xABABABAB
    ops.gather_rows(table, ids, policy, out=out)
    assert out.cpu().numpy().view(np.uint32).tolist() == g["expected_f32_bits"][policy]


def _pool_ids(rng, n, V):
    pool = np.array([0, V - 1, 1, V, V + 7, 2, -1, -(2 ** 31), 2 ** 31 - 1, -3], dtype=np.int64)
    ids = rng.integers(0, V, size=n)
    bad = rng.random(n) < 0.2
    ids[bad] = pool[rng.integers(0, len(pool), size=int(bad.sum()))]
    return ids


@pytest.mark.parametrize("dim,dtype", [(256, np.uint16), (8, np.uint16), (3, np.uint16), (7, np.uint8),
                                       (64, np.uint32), (5, np.uint64)])
@pytest.mark.parametrize("idx", ["i32", "i64", "u32"])
@pytest.mark.parametrize("policy", list(POLICIES))
def test_random_rows_every_policy_and_index_dtype(dim, dtype, idx, policy):
    rng = np.random.default_rng(dim * 3 + len(idx))
    V, n = 1000, 3001
    table = rng.integers(0, np.iinfo(dtype).max, size=(V, dim), dtype=np.uint64).astype(dtype)
    ids = _pool_ids(rng, n, V)
    if idx == "u32":
        ids = np.where(ids < 0, 2 ** 32 - 5, ids).astype(np.uint32)  # no negatives: large values are OOB
    else:
        ids = ids.astype(np.int32 if idx == "i32" else np.int64)
    prefill = np.full((n, dim * np.dtype(dtype).itemsize), 0xAB, dtype=np.uint8).view(dtype)
    want = orc.gather_rows(table, ids, POLICIES[policy], out=prefill.copy())
    tdt = {np.uint8: torch.uint8, np.uint16: torch.int16, np.uint32: torch.int32, np.uint64: torch.int64}[dtype]
    t_table = torch.from_numpy(table.view(tdt_np(tdt))).cuda()
    t_ids = torch.from_numpy(ids).cuda()
    out = torch.from_numpy(prefill.view(tdt_np(tdt)).copy()).cuda()
    ops.gather_rows(t_table, t_ids, policy, out=out)
    assert np.array_equal(out.cpu().numpy().view(dtype), want)


def tdt_np(tdt):
    return {torch.uint8: np.uint8, torch.int16: np.int16, torch.int32: np.int32, torch.int64: np.int64}[tdt]


def test_empty_table_zero_fill_and_skip():
    table = torch.empty(0, 256, dtype=torch.bfloat16, device="cuda")
    ids = torch.tensor([0, 5, -1], dtype=torch.int32, device="cuda")
    z = ops.gather_rows(table, ids, "zero_fill", out=torch.full((3, 256), 7.0, dtype=torch.bfloat16, device="cuda"))
    assert torch.count_nonzero(z.view(torch.int16)) == 0
    s = ops.gather_rows(table, ids, "skip", out=torch.full((3, 256), 7.0, dtype=torch.bfloat16, device="cuda"))
    assert torch.all(s == 7.0)


def test_full_zipf_config():
    table, ids = workloads.gather_inputs(device="cuda")
    out = ops.gather_rows(table, ids, "zero_fill")
    # every id is in range: the result is plain row indexing, compared as raw bits
    assert torch.equal(out.view(torch.int16), table.view(torch.int16)[ids.long()])
    # and the oracle on a sample of 65536 ids (its host copy of the whole output would be 8 GiB)
    sel = torch.randint(0, ids.numel(), (65536,), device="cuda", generator=torch.Generator("cuda").manual_seed(1))
    t_np = table.view(torch.int16).cpu().numpy().view(np.uint16)
    want = orc.gather_rows(t_np, ids[sel].cpu().numpy(), orc.OOB_ZERO_FILL)
    assert np.array_equal(out[sel].view(torch.int16).cpu().numpy().view(np.uint16), want)


# Many runs of 32 rows per warp over a multi-wave grid: 16-byte aligned rows of 16 B to 8 KiB (one chunk per lane
# and fewer, one, two and sixteen), n leaving a partial last run, and 20 % of the ids out of range (negative, past
# the end, extreme).
@pytest.mark.parametrize("row_bytes", [16, 48, 512, 1024, 8192])
@pytest.mark.parametrize("policy", list(POLICIES))
def test_large_n_every_policy(row_bytes, policy):
    rng = np.random.default_rng(row_bytes + len(policy))
    V = 3000
    n = 148 * 4 * 16 * 3 + 5 if row_bytes <= 1024 else 148 * 4 * 16 + 3
    words = row_bytes // 4
    table = rng.integers(0, 2 ** 32, size=(V, words), dtype=np.uint64).astype(np.uint32)
    for idx in ("i32", "i64", "u32"):
        ids = _pool_ids(rng, n, V)
        if idx == "u32":
            ids = np.where(ids < 0, 2 ** 32 - 5, ids).astype(np.uint32)
        else:
            ids = ids.astype(np.int32 if idx == "i32" else np.int64)
        prefill = rng.integers(0, 2 ** 32, size=(n, words), dtype=np.uint64).astype(np.uint32)
        want = orc.gather_rows(table, ids, POLICIES[policy], out=prefill.copy())
        out = torch.from_numpy(prefill.view(np.int32).copy()).cuda()
        ops.gather_rows(torch.from_numpy(table.view(np.int32)).cuda(), torch.from_numpy(ids).cuda(), policy, out=out)
        assert np.array_equal(out.cpu().numpy().view(np.uint32), want), idx


def test_zipf_2p20_all_in_range_and_repeat():
    """Zipf ids of the benchmark's distribution at 2^20 ids: plain row indexing, the same bits on a second call."""
    table, ids = workloads.gather_inputs(n=1 << 20, device="cuda")
    a = ops.gather_rows(table, ids, "skip")
    b = ops.gather_rows(table, ids, "zero_fill")
    assert torch.equal(a.view(torch.int16), table.view(torch.int16)[ids.long()])
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
