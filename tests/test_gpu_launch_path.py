"""The path a Rust host takes through the Backend seam, on the GPU, for each of the five config lifts.

`Backend::lower` (crates/unpopped/src/backend.rs:708) becomes `up_sm100_classify`; the host then sizes the workspace
(`up_sm100_workspace_bytes`) and runs the kernel on `TypedBuffer`-shaped descriptors (`up_sm100_launch`;
crates/unpopped/src/oracle/buffers.rs:16: a pointer, a `base` element offset and per-axis strides). Each case builds
the plan for a lift, lowers it, launches it on buffers that sit at a non-zero `base` inside a larger allocation (and,
where the kernel takes one, a row stride wider than the row), and compares the result with the oracle: bit for bit
for the integer, index, gather, dequant and Auto-sum results, within the stated bounds for the F32 sum and W4A16. At
the full config sizes the launch path is compared bit for bit with the typed entry point, which the other GPU tests
hold to the oracle at those sizes.
"""
import numpy as np
import pytest
import torch

import oracle as orc
from unpopped_b200 import _lib, ops, workloads
from unpopped_b200.backend import CudaSm100, LowerError, Operand, Plan

pytestmark = pytest.mark.gpu
U32 = 2.0 ** -24


@pytest.fixture(scope="module")
def be():
    assert torch.cuda.is_available(), "these tests need the B200"
    return CudaSm100()


def placed(t: torch.Tensor, lead: int, row_pad: int = 0):
    """A copy of 2-D (or 1-D) `t` inside a larger zeroed buffer: `lead` elements in front, rows `row_pad` elements
    wider than they are. Returns (buffer, base, strides)."""
    if t.dim() == 1:
        buf = torch.zeros(lead + t.numel() + 5, dtype=t.dtype, device=t.device)
        buf[lead:lead + t.numel()] = t
        return buf, lead, (1,)
    rows, cols = t.shape
    rs = cols + row_pad
    buf = torch.zeros(lead + rows * rs + 5, dtype=t.dtype, device=t.device)
    buf[lead:lead + rows * rs].view(rows, rs)[:, :cols] = t
    return buf, lead, (rs, 1)


def run(be, plan, ins, outs):
    k = be.lower(plan)
    nb = be.workspace_bytes(k, ins, outs)
    ws = torch.zeros(max(nb, 1), dtype=torch.uint8, device="cuda") if nb else None
    be.launch(k, ins, outs, workspace=ws)
    if ws is not None:
        assert ops.workspace_status(ws) == _lib.UP_OK
    torch.cuda.synchronize()
    return k


def bits32(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


# ---- config 1: row sum (F32 and the Auto documented order) ----

@pytest.mark.parametrize("rows,cols,pad,lead", [(64, 1000, 24, 7), (300, 8192, 4, 4), (5, 3, 1, 1)])
def test_row_sum_through_launch(be, rows, cols, pad, lead):
    rng = np.random.default_rng(rows + cols)
    xn = rng.standard_normal((rows, cols)).astype(np.float32)
    buf, base, strides = placed(torch.from_numpy(xn).cuda(), lead, pad)
    for accum, block in (("AUTO", 1024), ("AUTO", 256), ("F32", 0)):
        out = torch.full((rows + 3,), np.nan, dtype=torch.float32, device="cuda")
        plan = Plan("REDUCTION", [Operand("F32", (rows, cols), strides), Operand("F32", (rows,))], dtype="F32",
                    op="SUM", axes_mask=0b10, accum=accum, block=block)
        k = run(be, plan, [Operand("F32", (rows, cols), strides, base, buf.data_ptr())],
                [Operand("F32", (rows,), (1,), 2, out.data_ptr())])
        assert k.name == "up_sm100_row_sum_f32"
        got = out[2:2 + rows].cpu().numpy()
        assert np.isnan(out[0].item()) and np.isnan(out[-1].item())  # nothing outside the view is written
        if accum == "AUTO":
            assert np.array_equal(bits32(got), bits32(orc.row_sum_f32_documented(xn, block)))
        else:
            exact = xn.astype(np.float64).sum(axis=1)
            assert np.all(np.abs(got - exact) <= 2.0 ** -20 * np.abs(xn).astype(np.float64).sum(axis=1))


# ---- config 4: max + argmax over bf16 rows ----

@pytest.mark.parametrize("rows,cols,pad,lead", [(40, 32000, 8, 8), (17, 1001, 3, 5)])
def test_max_argmax_through_launch(be, rows, cols, pad, lead):
    x = workloads.argmax_input(rows=rows, cols=cols, seed=rows * cols, device="cuda")
    x[0, 5] = x[0, 9] = 60.0  # a tie: the lower index wins
    buf, base, strides = placed(x.view(torch.int16), lead, pad)
    mx = torch.zeros(rows + 1, dtype=torch.float32, device="cuda")
    for out_dt, tdt in (("I64", torch.int64), ("I32", torch.int32)):
        am = torch.full((rows + 1,), -7, dtype=tdt, device="cuda")
        plan = Plan("REDUCTION", [Operand("BF16", (rows, cols), strides), Operand(out_dt, (rows,))], dtype="BF16",
                    out_dtype=out_dt, op="ARGMAX", axes_mask=0b10)
        k = run(be, plan, [Operand("BF16", (rows, cols), strides, base, buf.data_ptr())],
                [Operand("F32", (rows,), (1,), 1, mx.data_ptr()), Operand(out_dt, (rows,), (1,), 1, am.data_ptr())])
        assert k.name == "up_sm100_row_max_argmax_bf16"
        want_mx, want_am = orc.row_max_argmax_bf16(x.view(torch.int16).cpu().numpy().view(np.uint16))
        assert np.array_equal(bits32(mx[1:].cpu().numpy()), bits32(want_mx))
        assert np.array_equal(am[1:].cpu().numpy().astype(np.int64), want_am)
        assert int(am[0].item()) == -7
        assert want_am[0] == 5


def test_argmax_full_config_launch_matches_typed_entry(be):
    x = workloads.argmax_input(device="cuda")
    rows, cols = x.shape
    mx = torch.empty(rows, dtype=torch.float32, device="cuda")
    am = torch.empty(rows, dtype=torch.int32, device="cuda")
    plan = Plan("REDUCTION", [Operand("BF16", (rows, cols)), Operand("I32", (rows,))], dtype="BF16", out_dtype="I32",
                op="ARGMAX", axes_mask=0b10)
    run(be, plan, [Operand("BF16", (rows, cols), ptr=x.data_ptr())],
        [Operand("F32", (rows,), ptr=mx.data_ptr()), Operand("I32", (rows,), ptr=am.data_ptr())])
    m2, a2 = ops.row_max_argmax(x, torch.int32)
    assert torch.equal(mx.view(torch.int32), m2.view(torch.int32)) and torch.equal(am, a2)


# ---- config 2: the three scan variants ----

SCAN_VARIANTS = [("SUM", False), ("SUM", True), ("MAX", False)]


@pytest.mark.parametrize("rows,k,lead", [(1, (1 << 20) + 8, 4), (3, 40_000, 1), (1000, 45, 3), (1, 77_777, 0)])
def test_scan_through_launch(be, rows, k, lead):
    rng = np.random.default_rng(rows * k)
    xn = rng.integers(0, 16, size=(rows, k)).astype(np.int32)
    buf, base, _ = placed(torch.from_numpy(xn.reshape(-1)).cuda(), lead)
    for op, excl in SCAN_VARIANTS:
        out = torch.full((rows * k + 2 * lead + 1,), -1, dtype=torch.int32, device="cuda")
        shape = (rows, k)
        plan = Plan("SCAN", [Operand("I32", shape), Operand("I32", shape)], dtype="I32", op=op, scan_axis=1,
                    exclusive=excl)
        k_ = run(be, plan, [Operand("I32", shape, None, base, buf.data_ptr())],
                 [Operand("I32", shape, None, 2 * lead, out.data_ptr())])
        assert k_.name == "up_sm100_scan_i32"
        got = out[2 * lead:2 * lead + rows * k].cpu().numpy().reshape(rows, k)
        assert np.array_equal(got, orc.scan_i32(xn, orc.OP_SUM if op == "SUM" else orc.OP_MAX, excl)), (op, excl)
        assert int(out[2 * lead + rows * k].item()) == -1


def test_scan_full_config_launch_matches_typed_entry(be):
    x = workloads.scan_input(device="cuda")
    n = x.numel()
    for op, excl in SCAN_VARIANTS:
        y = torch.empty_like(x)
        plan = Plan("SCAN", [Operand("I32", (n,)), Operand("I32", (n,))], dtype="I32", op=op, scan_axis=0,
                    exclusive=excl)
        run(be, plan, [Operand("I32", (n,), ptr=x.data_ptr())], [Operand("I32", (n,), ptr=y.data_ptr())])
        assert torch.equal(y, ops.scan(x, op.lower(), excl)), (op, excl)


def test_scan_plans_the_kernel_cannot_take_are_refused(be):
    strided = Operand("I32", (4, 100), (200, 1))
    with pytest.raises(LowerError) as e:
        be.lower(Plan("SCAN", [strided, Operand("I32", (4, 100))], dtype="I32", scan_axis=1))
    assert e.value.variant == "UnsupportedPlanShape"
    with pytest.raises(LowerError) as e:
        be.lower(Plan("SCAN", [Operand("I32", (4, 100)), Operand("I32", (4, 100))], dtype="I32", scan_axis=0))
    assert e.value.variant == "UnsupportedPlanShape"
    # a launch whose output is smaller than its input is refused before any device work
    L = _lib.load()
    x = torch.zeros(1000, dtype=torch.int32, device="cuda")
    k = be.lower(Plan("SCAN", [Operand("I32", (1000,)), Operand("I32", (1000,))], dtype="I32", scan_axis=0))
    before = L.up_sm100_launch_count()
    with pytest.raises(_lib.UpError):
        be.launch(k, [Operand("I32", (1000,), ptr=x.data_ptr())], [Operand("I32", (999,), ptr=x.data_ptr())],
                  workspace=torch.zeros(1 << 16, dtype=torch.uint8, device="cuda"))
    assert L.up_sm100_launch_count() == before


# ---- config 3: row gather with each OOB policy ----

@pytest.mark.parametrize("policy", ["SKIP", "CLAMP", "ZERO_FILL"])
def test_gather_through_launch(be, policy):
    V, D, N = 5000, 256, 20_000
    g = torch.Generator(device="cuda").manual_seed(7)
    table = (torch.randn(V, D, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    ids = workloads.zipf_ids(N, V, 1.1, seed=8)
    ids[::97] = V + 3  # past the end
    ids[5::101] = -2   # negative is out of range too
    tbuf, tbase, _ = placed(table.view(torch.int16), 3 * D)  # whole rows in front
    ibuf, ibase, _ = placed(ids, 9)
    prefill = torch.full((N + 2, D), 0x1234, dtype=torch.int16, device="cuda")
    out = prefill.clone()
    plan = Plan("STRIDED", [Operand("BF16", (V, D)), Operand("I32", (N,)), Operand("BF16", (N, D))], dtype="BF16",
                read_index=True, gather_axis=0, oob=policy, index_dtype="I32")
    k = run(be, plan, [Operand("BF16", (V, D), None, tbase, tbuf.data_ptr()),
                       Operand("I32", (N,), None, ibase, ibuf.data_ptr())],
            [Operand("BF16", (N, D), None, D, out.data_ptr())])
    assert k.name == "up_sm100_gather_rows"
    want = prefill[1:N + 1].cpu().numpy().copy()
    orc.gather_rows(table.view(torch.int16).cpu().numpy(), ids.cpu().numpy(), _lib.OOB[policy], out=want)
    assert np.array_equal(out[1:N + 1].cpu().numpy(), want)
    assert torch.equal(out[0], prefill[0]) and torch.equal(out[-1], prefill[-1])


def test_gather_full_config_launch_matches_typed_entry(be):
    table, ids = workloads.gather_inputs(device="cuda")
    V, D = table.shape
    N = ids.numel()
    out = torch.empty(N, D, dtype=torch.bfloat16, device="cuda")
    plan = Plan("STRIDED", [Operand("BF16", (V, D)), Operand("I32", (N,)), Operand("BF16", (N, D))], dtype="BF16",
                read_index=True, oob="ZERO_FILL")
    run(be, plan, [Operand("BF16", (V, D), ptr=table.data_ptr()), Operand("I32", (N,), ptr=ids.data_ptr())],
        [Operand("BF16", (N, D), ptr=out.data_ptr())])
    want = ops.gather_rows(table, ids, "zero_fill")
    assert torch.equal(out.view(torch.int16), want.view(torch.int16))
    del out, want


# ---- config 5: int4 dequant and the W4A16 GEMM, through the kernel-layer route ----

def _nibble_buffer(packed: torch.Tensor, lead_bytes: int):
    n, kb = packed.shape
    buf = torch.zeros(lead_bytes + n * kb + 16, dtype=torch.uint8, device="cuda")
    buf[lead_bytes:lead_bytes + n * kb] = packed.reshape(-1)
    return buf, 2 * lead_bytes  # base counts nibbles


def test_dequant_through_launch(be):
    n, k, group = 300, 1024, 128
    d = workloads.w4a16_inputs(n=n, k=k, m=1, group=group, seed=4)
    wbuf, wbase = _nibble_buffer(d.w_packed, 6)
    out = torch.zeros(n + 1, k, dtype=torch.int16, device="cuda")
    plan = Plan("KERNEL_FN", [Operand("I4", (n, k)), Operand("F16", (n, k // group)), Operand("BF16", (n, k))])
    kk = run(be, plan, [Operand("I4", (n, k), None, wbase, wbuf.data_ptr()),
                        Operand("F16", (n, k // group), ptr=d.scale.data_ptr())],
             [Operand("BF16", (n, k), None, k, out.data_ptr())])
    assert kk.name == "up_sm100_dequant_i4_bf16" and kk.scalars == (group,)
    want = orc.dequant_i4_bf16(d.w_packed.cpu().numpy(), d.scale.view(torch.int16).cpu().numpy().view(np.uint16),
                               n, k, group)
    assert np.array_equal(out[1:].cpu().numpy().view(np.uint16), want)
    assert int(out[0].abs().sum().item()) == 0


def _w4a16_bound_check(d, got_bits):
    out, exact, abs_sum = orc.w4a16(d.w_packed.cpu().numpy(), d.scale.view(torch.int16).cpu().numpy().view(np.uint16),
                                    d.x.view(torch.int16).cpu().numpy().view(np.uint16), d.m, d.n, d.k, d.group,
                                    threads=orc.max_threads())
    gv = (got_bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    a = np.abs(exact)
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(a, 2.0 ** -126))) - 7)
    bound = 0.5 * ulp + 2.0 * U32 * abs_sum  # the bar of tests/test_gpu_w4a16.py
    assert np.all(np.abs(gv - exact) <= bound)


@pytest.mark.parametrize("m,n,k", [(16, 1024, 2048), (5, 384, 512)])
def test_w4a16_through_launch(be, m, n, k):
    d = workloads.w4a16_inputs(n=n, k=k, m=m, group=128, seed=m + n)
    wbuf, wbase = _nibble_buffer(d.w_packed, 32)
    xbuf, xbase, _ = placed(d.x.view(torch.int16), 8 * k)
    out = torch.zeros(m + 1, n, dtype=torch.int16, device="cuda")
    ops_ = [Operand("I4", (n, k)), Operand("F16", (n, k // 128)), Operand("BF16", (m, k)), Operand("BF16", (m, n))]
    kk = run(be, Plan("KERNEL_FN", ops_),
             [Operand("I4", (n, k), None, wbase, wbuf.data_ptr()),
              Operand("F16", (n, k // 128), ptr=d.scale.data_ptr()),
              Operand("BF16", (m, k), None, xbase, xbuf.data_ptr())],
             [Operand("BF16", (m, n), None, n, out.data_ptr())])
    assert kk.name == "up_sm100_w4a16_gemm"
    _w4a16_bound_check(d, out[1:].cpu().numpy().view(np.uint16))
    assert int(out[0].abs().sum().item()) == 0


def test_w4a16_full_config_launch_matches_typed_entry(be):
    d = workloads.w4a16_inputs(device="cuda")
    out = torch.empty(d.m, d.n, dtype=torch.bfloat16, device="cuda")
    ops_ = [Operand("I4", (d.n, d.k)), Operand("F16", (d.n, d.k // d.group)), Operand("BF16", (d.m, d.k)),
            Operand("BF16", (d.m, d.n))]
    run(be, Plan("KERNEL_FN", ops_),
        [Operand("I4", (d.n, d.k), ptr=d.w_packed.data_ptr()),
         Operand("F16", (d.n, d.k // d.group), ptr=d.scale.data_ptr()),
         Operand("BF16", (d.m, d.k), ptr=d.x.data_ptr())],
        [Operand("BF16", (d.m, d.n), ptr=out.data_ptr())])
    want = ops.w4a16(d.w_packed, d.scale, d.x, d.group)
    assert torch.equal(out.view(torch.int16), want.view(torch.int16))


def test_w4a16_launch_refuses_mismatched_operands(be):
    d = workloads.w4a16_inputs(n=128, k=256, m=2, group=128, seed=2)
    ops_ = [Operand("I4", (128, 256)), Operand("F16", (128, 2)), Operand("BF16", (2, 256)), Operand("BF16", (2, 128))]
    k = be.lower(Plan("KERNEL_FN", ops_))
    out = torch.empty(2, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.UpError) as e:  # an output narrower than N
        be.launch(k, [Operand("I4", (128, 256), ptr=d.w_packed.data_ptr()),
                      Operand("F16", (128, 2), ptr=d.scale.data_ptr()), Operand("BF16", (2, 256), ptr=d.x.data_ptr())],
                  [Operand("BF16", (2, 64), ptr=out.data_ptr())],
                  workspace=torch.zeros(1 << 20, dtype=torch.uint8, device="cuda"))
    assert e.value.status == _lib.UP_ERR_UNSUPPORTED
