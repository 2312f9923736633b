"""Benchmark of the lifted kernel families on B200: achieved HBM GB/s per lift, one JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--lifts all|none]

Headline (`value`): the inclusive add-scan over 2^28 int32 (the benchmark's configs[1]), one decoupled
look-back pass per step, inputs resident in HBM, L2 flushed between steps, CUDA events on the launching
stream, max over ranks. With N GPUs every rank scans its own 2^28 shard of an N x 2^28 array (weak scaling):
local fold, an NCCL all-gather of the N shard totals, then the single-pass scan seeded with the carry.
`e2e`: the same scan through the C ABI from pinned host memory, copies inside the timed region: at N=1 the
host-buffer entry (up_sm100_scan_i32_host, copy-in, scan and copy-out overlapped chunk by chunk); at N>1 the
shard is copied in whole (the carry needs every shard's total), scanned, and copied back. `lifts`: every other configuration (row sum, max+argmax, Zipf gather, int4
dequant, W4A16) measured the same way in the same run. `roofline`: the scan kernel's algorithmic bytes over
its event-timed duration against the measured copy bandwidth. `cpu_baseline`: the oracle restatement timed
on the host cores (rank 0, N=1 only).
`--impl reference`: the reference's own CPU implementation of the path (the oracle restatement — the
reference is Rust and has no GPU code) on all host cores, same metric and config.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "oracle")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "achieved HBM GB/s per lift (reduce/scan/gather/dequant) at 1/2/4/8 B200 vs 8 TB/s"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
SCAN_N = 1 << 28


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d.get("bf16_tflops", FALLBACK_BF16_TFLOPS)), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def ncu_traffic(name):
    """DRAM bytes per launch of a kernel from its committed ncu summary (`dram_bytes_per_launch: N`)."""
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("dram_bytes_per_launch:"):
            try:
                return int(float(line.split(":", 1)[1].strip().split()[0]))
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while the timed regions run."""
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.t.join(timeout=5)
        sm, smax, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                smax = max(smax, float(parts[1]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(nm)
        if not sm:
            return None
        loaded = [s for s in sm if s > 0.5 * smax] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


class Ctx:
    def __init__(self, args):
        import torch
        import torch.distributed as dist

        self.torch, self.dist = torch, dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.args = args
        if self.world > 1:
            import datetime
            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
        else:
            torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        self.sleep_cycles = 1_000_000  # ~0.5 ms at the B200's 1.9 GHz SM clock
        self.comm = None
        if self.world > 1:
            from unpopped_b200 import dist as udist

            self.comm = udist.Comm()  # the library's communicator (NCCL inside libunpopped_sm100)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier(device_ids=[self.local])

    def max_over_ranks(self, v: float) -> float:
        if self.world == 1:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def timed(self, step, K, W, inner=False, head_start=True):
        """W warm-up steps, then EXACTLY K steps between one pair of events on the launching stream, with a
        barrier + synchronize on both sides. `step(i, kin)` runs step i; callers rotate through enough input
        copies that every step's inputs are colder than the 126 MB L2 (no flush inside the timed region). A GPU
        sleep before the start event lets the host enqueue all K steps ahead of the device, so the events time
        device work only; a step that blocks the host (a host-buffer call) takes head_start=False, so the events
        bracket its whole duration. With `inner`, the step appends (start, end) events of its dominant kernel to
        `kin`.
        Returns (ms per step, max over ranks; mean inner-kernel ms; our kernel launches in the timed region)."""
        from unpopped_b200 import ops

        torch = self.torch
        for i in range(W):
            step(i, None)
        torch.cuda.synchronize()
        self.barrier()
        torch.cuda.synchronize()
        kin = [] if inner else None
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        l0 = ops.launch_count()
        if head_start:
            torch.cuda._sleep(self.sleep_cycles + K * 200_000)  # ~0.1 ms per step of head start for the host
        a.record()
        for i in range(K):
            step(i, kin)
        b.record()
        torch.cuda.synchronize()
        launches = ops.launch_count() - l0
        self.barrier()
        torch.cuda.synchronize()
        ms = self.max_over_ranks(a.elapsed_time(b)) / K
        kms = None
        if kin:
            kms = self.max_over_ranks(sum(x.elapsed_time(y) for x, y in kin)) / len(kin)
        return ms, kms, launches


def copies_for(nbytes: int, l2_bytes: int = 126 << 20) -> int:
    """Input copies to rotate through so that each step's inputs were last touched >= 2 x L2 bytes ago."""
    return max(1, -(-(2 * l2_bytes) // max(1, nbytes)) + 1) if nbytes < 4 * l2_bytes else 1


def make_scan_step(ctx, x, y, layout="block_cyclic"):
    """One step of the (possibly sharded) inclusive add-scan. At N > 1 it goes through the library's communicator
    (up_sm100_launch_multi): "block_cyclic" is one kernel per step (the cross-GPU look-back over NVLink),
    "contiguous" folds the shard, all-gathers the totals and scans."""
    from unpopped_b200 import dist as udist, ops

    if ctx.world == 1:
        def step(i, kin):  # one kernel: the step time is the kernel time
            ops.scan(x, "sum", out=y)
        return step

    def step(i, kin):
        udist.sharded_scan(x, "sum", layout=layout, comm=ctx.comm, out=y)
    return step


def bench_lifts(ctx, K, W, hbm, bf16):
    """Every other configuration, each in its own timed region (same rules as the headline)."""
    from unpopped_b200 import _lib, ops, workloads as wl

    torch = ctx.torch
    res = {}

    def record(name, nbytes, ms, kernel, copies, extra=None):
        gbs = ctx.world * nbytes / (ms * 1e-3) / 1e9
        r = {"value": round(gbs, 1), "unit": "GB/s", "ms_per_step": round(ms, 4), "bytes_per_gpu": nbytes,
             "frac_of_hbm": round(gbs / (ctx.world * hbm), 4), "kernel": kernel, "input_copies_rotated": copies}
        if extra:
            r.update(extra)
        res[name] = r

    # config 1: row sum f32 8192 x 8192 (f32 accumulation, and the documented f64 order)
    R = copies_for(wl.rowsum_bytes())
    xs = [wl.rowsum_input(device=ctx.dev, seed=wl.SEED + 10 * c) for c in range(R)]
    out = torch.empty(xs[0].shape[0], dtype=torch.float32, device=ctx.dev)
    ms, _, _ = ctx.timed(lambda i, kin: ops.row_sum(xs[i % R], "f32", out=out), K, W)
    record("rowsum_f32_8192x8192", wl.rowsum_bytes(), ms, "row_sum_f32_kernel", R)
    ms, _, _ = ctx.timed(lambda i, kin: ops.row_sum(xs[i % R], "auto", 1024, out=out), K, W)
    record("rowsum_f32_auto_f64order_B1024", wl.rowsum_bytes(), ms, "row_sum_auto_kernel", R)
    # block 1, the serial order: runs of values added out of order where no add can round
    ms, _, _ = ctx.timed(lambda i, kin: ops.row_sum(xs[i % R], "auto", 1, out=out), K, W)
    record("rowsum_f32_serial", wl.rowsum_bytes(), ms, "row_sum_serial_spec_kernel", R)
    # the reduction breadth on the same input: f32 Max over the last axis, and Max over the outer axis
    ms, _, _ = ctx.timed(lambda i, kin: ops.reduce2d(xs[i % R], "max", 1, out=out), K, W)
    record("rowmax_f32_8192x8192", wl.rowsum_bytes(), ms, "row_extremum_f32_kernel", R)
    ms, _, _ = ctx.timed(lambda i, kin: ops.reduce2d(xs[i % R], "max", 0, out=out), K, W)
    record("colmax_f32_8192x8192", wl.rowsum_bytes(), ms, "col_extremum_f32_vec_kernel", R)
    ms, _, _ = ctx.timed(lambda i, kin: ops.reduce2d(xs[i % R], "sum", 0, block=256, out=out), K, W)
    record("colsum_f32_documented_B256", wl.rowsum_bytes(), ms, "col_sum_f32_doc_vec4_kernel", R)
    # the serial order per column (block 1, the default): runs of rows added out of order where no add can round
    ms, _, _ = ctx.timed(lambda i, kin: ops.reduce2d(xs[i % R], "sum", 0, out=out), K, W)
    record("colsum_f32_serial", wl.rowsum_bytes(), ms, "col_sum_f32_serial_strip_kernel", R)
    # its split-K variant (64 row chunks of f64 partials, added in chunk order): the parallel association
    L = _lib.load()
    ws = torch.empty(L.up_sm100_col_sum_splitk_workspace_bytes(8192, 8192, 64), dtype=torch.uint8,
                     device=ctx.dev)
    ms, _, _ = ctx.timed(lambda i, kin: _lib.check(L.up_sm100_col_sum_f32_splitk(
        xs[i % R].data_ptr(), 8192, 8192, 8192, 64, 0, ws.data_ptr(), ws.numel(), out.data_ptr(),
        torch.cuda.current_stream().cuda_stream), "splitk"), K, W)
    record("colsum_f32_splitk64", wl.rowsum_bytes() + ws.numel() * 2, ms, "splitk_partial_kernel", R)
    del ws
    # the RowReduce lift on the same rows (a read and a write of every element)
    o2 = torch.empty_like(xs[0])
    for form in ("softmax", "rms_norm"):
        ms, _, _ = ctx.timed(lambda i, kin: ops.row_reduce(xs[i % R], form, block=256, out=o2), K, W)
        record(f"row_{form}_f32_B256", 2 * wl.rowsum_bytes(), ms, "row_reduce_f32_held_kernel", R)
    del o2
    # the Window lift (max pool 3/2, pad 1, along the last axis) and Im2Col (a 3x3 unfold of 32 x 64 x 56 x 56)
    ow = torch.empty((8192, 4096), device=ctx.dev)
    ms, _, _ = ctx.timed(lambda i, kin: ops.window(xs[i % R], "max", 3, 2, 1, 1, out=ow), K, W)
    record("window_maxpool3s2_f32_8192x8192", wl.rowsum_bytes() + ow.numel() * 4, ms, "window_f32_staged_kernel", R)
    del ow
    # the same bytes as 64 x 8192 x 128, pooled along the middle axis (the column kernel)
    om = torch.empty((64, 4096, 128), device=ctx.dev)
    ms, _, _ = ctx.timed(lambda i, kin: ops.window(xs[i % R].view(64, 8192, 128), "max", 3, 2, 1, 1, axis=1, out=om),
                         K, W)
    record("window_maxpool3s2_f32_middle_64x8192x128", wl.rowsum_bytes() + om.numel() * 4, ms,
           "window_f32_lines_staged_kernel", R)
    del om
    # Im2Col: the 3x3, pad 1 unfold of 32 x 64 x 56 x 56 f32 (a ResNet stem's first layer), 9x its input in writes
    ximg = [torch.randn(32, 64, 56, 56, device=ctx.dev) for _ in range(R)]
    oimg = torch.empty((32, 64 * 9, 56 * 56), device=ctx.dev)
    ms, _, _ = ctx.timed(lambda i, kin: ops.im2col(ximg[i % R], (3, 3), (1, 1), (1, 1), out=oimg), K, W)
    record("im2col_3x3_f32_32x64x56x56", ximg[0].numel() * 4 + oimg.numel() * 4, ms, "im2col_plane_kernel", R)
    del ximg, oimg
    xi = [x.view(torch.int32) for x in xs]  # the same bytes read as i32
    oi = out.view(torch.int32)
    ms, _, _ = ctx.timed(lambda i, kin: ops.reduce2d(xi[i % R], "xor", 1, out=oi), K, W)
    record("rowxor_i32_8192x8192", wl.rowsum_bytes(), ms, "row_fold_i32_kernel", R)
    ms, _, _ = ctx.timed(lambda i, kin: ops.reduce2d(xi[i % R], "sum", 0, out=oi), K, W)
    record("colsum_i32_8192x8192", wl.rowsum_bytes() + 8192 * 4, ms, "col_fold_i32_vec_kernel", R)
    del xi, oi
    del xs, out

    # config 2 variants: exclusive add and inclusive max (the headline is the inclusive add)
    x = wl.scan_input(device=ctx.dev)
    y = torch.empty_like(x)
    for name, op, ex in (("scan_excl_add_i32_2p28", "sum", True), ("scan_incl_max_i32_2p28", "max", False)):
        ms, _, _ = ctx.timed(lambda i, kin, op=op, ex=ex: ops.scan(x, op, ex, out=y), K, W)
        record(name, wl.scan_bytes(), ms, "scan_i32_persist_kernel", 1)
    ops.check_workspace("scan", ctx.dev)
    del x, y

    # config 4: max + argmax bf16 32768 x 32000
    x = wl.argmax_input(device=ctx.dev)
    mx = torch.empty(x.shape[0], dtype=torch.float32, device=ctx.dev)
    am = torch.empty(x.shape[0], dtype=torch.int32, device=ctx.dev)
    L = _lib.load()

    def am_step(i, kin):
        _lib.check(L.up_sm100_row_max_argmax_bf16(x.data_ptr(), x.shape[0], x.shape[1], x.shape[1], mx.data_ptr(),
                                                  am.data_ptr(), None, torch.cuda.current_stream().cuda_stream),
                   "argmax")
    ms, _, _ = ctx.timed(am_step, K, W)
    record("max_argmax_bf16_32768x32000", wl.argmax_bytes(), ms, "row_max_argmax_vec_kernel", 1)
    del x, mx, am

    # config 3: Zipf gather, table 2^20 x 256 bf16, 2^24 ids
    table, ids = wl.gather_inputs(device=ctx.dev)
    comp, logical, uniq = wl.gather_bytes(ids)
    g_out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=ctx.dev)
    ms, _, _ = ctx.timed(lambda i, kin: ops.gather_rows(table, ids, "zero_fill", out=g_out), K, W)
    record("gather_rows_bf16_zipf1.1", comp, ms, "gather_rows_vec_kernel", 1,
           {"bytes_basis": "compulsory (ids + output + each distinct row once)", "unique_rows": uniq,
            "logical_GBps": round(ctx.world * logical / (ms * 1e-3) / 1e9, 1)})
    del table, ids, g_out

    # the scatter lift: index_add of 2^20 i32 rows of 64 into 2^16 rows with uniform targets (atomic adds)
    g = torch.Generator(device="cpu").manual_seed(wl.SEED + 7)
    upd = torch.randint(-1000, 1000, (1 << 20, 64), dtype=torch.int32, generator=g).to(ctx.dev)
    tid = torch.randint(0, 1 << 16, (1 << 20,), dtype=torch.int32, generator=g).to(ctx.dev)
    dst = torch.zeros((1 << 16, 64), dtype=torch.int32, device=ctx.dev)
    sc_bytes = upd.numel() * 4 + tid.numel() * 4 + 2 * dst.numel() * 4
    ms, _, _ = ctx.timed(lambda i, kin: ops.scatter(upd, tid, dst, "add"), K, W)
    record("index_add_i32_2p20x64_into_2p16_uniform", sc_bytes, ms, "scatter_kernel", 1,
           {"bytes_basis": "updates + ids read once, destination read and written once"})
    del upd, tid, dst

    # config 5: int4 group-128 dequant (standalone) and the W4A16 GEMM 16 x 28672 x 8192
    R = copies_for(wl.w4a16_bytes())
    ds = [wl.w4a16_inputs(device=ctx.dev, seed=wl.SEED + 5 + 10 * c) for c in range(R)]
    Rd = min(R, 2)
    dq = torch.empty(ds[0].n, ds[0].k, dtype=torch.bfloat16, device=ctx.dev)
    ms, _, _ = ctx.timed(lambda i, kin: ops.dequant_i4(ds[i % Rd].w_packed, ds[i % Rd].scale, ds[0].group, out=dq),
                         K, W)
    record("dequant_i4_g128_bf16_28672x8192", wl.dequant_bytes(), ms, "dequant_i4_rows_kernel", Rd)
    del dq
    o = torch.empty(ds[0].m, ds[0].n, dtype=torch.bfloat16, device=ctx.dev)
    ms, _, _ = ctx.timed(lambda i, kin: ops.w4a16(ds[i % R].w_packed, ds[i % R].scale, ds[i % R].x, ds[0].group,
                                                  out=o), K, W)
    ops.check_workspace("w4a16", ctx.dev)
    tflops = ctx.world * wl.w4a16_flops() / (ms * 1e-3) / 1e12
    record("w4a16_gemm_16x28672x8192_g128", wl.w4a16_bytes(), ms, "w4a16_kernel (tcgen05, TMEM A operand)", R,
           {"tflops": round(tflops, 1), "frac_of_bf16_peak": round(tflops / (ctx.world * bf16), 4)})
    del ds, o
    torch.cuda.empty_cache()
    return res


def cpu_scan_baseline():
    """The oracle restatement's serial scan (1 thread) on the full 2^28 config, timed on the host."""
    import numpy as np

    import oracle as orc

    rng = np.random.default_rng(20261201)
    x = rng.integers(0, 16, size=SCAN_N, dtype=np.int32)
    orc.scan_i32(x[:1 << 20], orc.OP_SUM, False)  # warm the code path
    reps, t0 = 0, time.perf_counter()
    while reps < 2 or time.perf_counter() - t0 < 3.0:
        orc.scan_i32(x, orc.OP_SUM, False)
        reps += 1
    dt = (time.perf_counter() - t0) / reps
    return {"value": round(2 * SCAN_N * 4 / dt / 1e9, 2), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"full config: 2^28 int32 inclusive add-scan, serial C restatement of eval_scan, {reps} passes"}


def _best_time(fn, min_s=0.4, max_reps=5):
    """Best wall time of `fn` over a few repetitions (at least two, or `min_s` seconds)."""
    best, reps, t_all = float("inf"), 0, time.perf_counter()
    while reps < 2 or (time.perf_counter() - t_all < min_s and reps < max_reps):
        t0 = time.perf_counter()
        fn()
        best = min(best, time.perf_counter() - t0)
        reps += 1
    return best


def cpu_baselines():
    """Each config lift's CPU baselines, timed on this host on a bounded sample of the config's own workload
    (seeded, same distributions): the oracle restatement on 1 core and with OpenMP on every core, and the serial C
    the reference's C99 emitter writes for the lift (oracle/c99_forms.c) on 1 core: the serial lift, and for the
    row sum and the scan also the launched lift's serialized thread loop. GB/s over the algorithmic bytes of the
    sample, as on the GPU. Returns ({config: {baseline: GB/s}}, {config: sample description}, threads)."""
    import numpy as np
    import torch

    import oracle as orc
    from unpopped_b200 import workloads as wl

    T = orc.max_threads()
    res, samples = {}, {}

    def gbs(nbytes, secs):
        return round(nbytes / secs / 1e9, 2)

    # config 1: the full 8192 x 8192 row sum
    x = wl.rowsum_input(device="cpu").numpy()
    nb = wl.rowsum_bytes()
    res["cfg1"] = {"oracle_1c": gbs(nb, _best_time(lambda: orc.row_sum_f32(x, 1))),
                   f"omp_{T}c": gbs(nb, _best_time(lambda: orc.row_sum_f32(x, T))),
                   "c99_1c": gbs(nb, _best_time(lambda: orc.c99_row_sum(x))),
                   "c99_launched_1c": gbs(nb, _best_time(lambda: orc.c99_row_sum(x, 256)))}
    samples["cfg1"] = "full 8192x8192 f32; c99_launched = the block-tree lift at B=256, serialized"
    del x
    # config 2: 2^26 of the 2^28 scan elements
    n = 1 << 26
    x = wl.scan_input(n=n, device="cpu").numpy()
    y = np.empty_like(x)
    nb = wl.scan_bytes(n)
    res["cfg2"] = {"oracle_1c": gbs(nb, _best_time(lambda: orc.lib().orc_scan_i32(
                       orc._p(x), orc._p(y), 1, n, orc.OP_SUM, 0, 0, 0, 1))),
                   f"omp_{T}c": gbs(nb, _best_time(lambda: orc.scan_i32_chunked(x, orc.OP_SUM, False, T))),
                   "c99_1c": gbs(nb, _best_time(lambda: orc.c99_scan(x, orc.OP_SUM, False))),
                   "c99_launched_1c": gbs(nb, _best_time(lambda: orc.c99_scan(x, orc.OP_SUM, False, 1024)))}
    samples["cfg2"] = "2^26 int32 inclusive add (1/4 of the config); c99_launched = the 3-phase lift at B=1024"
    del x, y
    # config 3: the first 2^20 of the 2^24 Zipf ids into the full 2^20 x 256 table
    table, ids = wl.gather_inputs(device="cpu")
    tb = table.view(torch.int16).numpy().view(np.uint16)
    ids = ids[:1 << 20].contiguous().numpy()
    comp, _, _ = wl.gather_bytes(torch.from_numpy(ids))
    out = np.zeros((ids.size, 256), np.uint16)
    res["cfg3"] = {"oracle_1c": gbs(comp, _best_time(lambda: orc.gather_rows(tb, ids, orc.OOB_ZERO_FILL, out, 1))),
                   f"omp_{T}c": gbs(comp, _best_time(lambda: orc.gather_rows(tb, ids, orc.OOB_ZERO_FILL, out, T))),
                   "c99_1c": gbs(comp, _best_time(lambda: orc.c99_gather(tb, ids, orc.OOB_ZERO_FILL, out)))}
    samples["cfg3"] = "2^20 of the 2^24 Zipf ids, full table; compulsory bytes of the sample"
    del table, tb, ids, out
    # config 4: 2048 of the 32768 rows
    rows = 2048
    xb = wl.argmax_input(rows=rows, device="cpu").view(torch.int16).numpy().view(np.uint16)
    nb = wl.argmax_bytes(rows=rows)
    res["cfg4"] = {"oracle_1c": gbs(nb, _best_time(lambda: orc.row_max_argmax_bf16(xb, 1))),
                   f"omp_{T}c": gbs(nb, _best_time(lambda: orc.row_max_argmax_bf16(xb, T))),
                   "c99_1c": gbs(nb, _best_time(lambda: orc.c99_row_max_argmax(xb)))}
    samples["cfg4"] = "2048 of the 32768 rows x 32000 bf16"
    del xb
    # config 5: 256 of the 28672 weight rows (all 16 activation rows, full K)
    nr = 256
    d = wl.w4a16_inputs(n=nr, device="cpu")
    w = d.w_packed.numpy()
    sc = d.scale.view(torch.int16).numpy().view(np.uint16)
    xa = d.x.view(torch.int16).numpy().view(np.uint16)
    nb = wl.w4a16_bytes(n=nr)
    res["cfg5"] = {"oracle_1c": gbs(nb, _best_time(lambda: orc.w4a16(w, sc, xa, d.m, nr, d.k, d.group, 1))),
                   f"omp_{T}c": gbs(nb, _best_time(lambda: orc.w4a16(w, sc, xa, d.m, nr, d.k, d.group, T))),
                   "c99_1c": gbs(nb, _best_time(lambda: orc.c99_w4a16(w, sc, xa, d.m, nr, d.k, d.group)))}
    samples["cfg5"] = "256 of the 28672 weight rows, M=16, K=8192; the oracle's products are exact f64"
    return res, samples, T


def scan_ws_status(ctx):
    """The sharded scan's workspace status on this rank (a bounded wait that ran out shows here)."""
    from unpopped_b200 import _lib

    ws = ctx.comm._ws.get(_lib.KERNEL["SCAN_I32"])
    if ws is not None:
        _lib.check(_lib.load().up_sm100_workspace_status(ws.data_ptr(), ctx.torch.cuda.current_stream().cuda_stream),
                   "sharded scan")


# The config lifts, by their names in `bench_lifts`, in the order of BASELINE.json's configs.
CONFIG_LIFTS = {
    "rowsum_f32_8192x8192": ("cfg1_rowsum_f32", "cfg1"),
    "rowsum_f32_auto_f64order_B1024": ("cfg1_rowsum_auto_B1024", None),
    "scan_excl_add_i32_2p28": ("cfg2_scan_excl_add", None),
    "scan_incl_max_i32_2p28": ("cfg2_scan_incl_max", None),
    "gather_rows_bf16_zipf1.1": ("cfg3_gather_zipf", "cfg3"),
    "max_argmax_bf16_32768x32000": ("cfg4_max_argmax", "cfg4"),
    "dequant_i4_g128_bf16_28672x8192": ("cfg5_dequant", None),
    "w4a16_gemm_16x28672x8192_g128": ("cfg5_w4a16", "cfg5"),
}


def config_block(lifts, head, cpu_cfg):
    """The five configurations, compact, for the end of the JSON line: GB/s (aggregate), ms per step, fraction of
    measured HBM per GPU, and the CPU baselines (GB/s) where measured."""
    out = {}

    def put(key, rec, cfg):
        e = {"GBps": rec["value"], "ms": rec["ms_per_step"], "frac": rec["frac_of_hbm"]}
        if "tflops" in rec:
            e["TFLOPs"] = rec["tflops"]
        if cfg and cfg in cpu_cfg:
            e["cpu"] = cpu_cfg[cfg]
        out[key] = e

    for name in ("rowsum_f32_8192x8192", "rowsum_f32_auto_f64order_B1024"):
        if name in lifts:
            put(CONFIG_LIFTS[name][0], lifts[name], CONFIG_LIFTS[name][1])
    put("cfg2_scan_incl_add", dict(value=head["value"], ms_per_step=head["ms_per_step"],
                                   frac_of_hbm=head["frac_of_hbm"]), "cfg2")
    for name, (key, cfg) in CONFIG_LIFTS.items():
        if name in lifts and not key.startswith("cfg1"):
            put(key, lifts[name], cfg)
    return out


def scan_config(world):
    """The headline workload's `config`, shared by both arms of the bench."""
    return {"workload": "configs[1]: inclusive add-scan over 2^28 int32 per GPU (1 GiB in, 1 GiB out)"
                        + ("; block-cyclic shards (148 x 8192-element stripes round-robin over the GPUs), one "
                           "pass with the cross-GPU look-back over NVLink" if world > 1 else ""),
            "lift": "scan_incl_add_i32", "elements_per_gpu": SCAN_N,
            "l2": "input (1 GiB per GPU) larger than the 126 MB L2; no flush", "parallelism": f"sharded x{world}"}


def run_reference(args):
    """The reference's CPU implementation of the path on all host cores (OpenMP chunked scan)."""
    import numpy as np

    import oracle as orc

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    threads = orc.max_threads()
    rng = np.random.default_rng(20261201)
    x = rng.integers(0, 16, size=SCAN_N, dtype=np.int32)
    y = np.empty_like(x)
    for _ in range(max(1, args.warmup)):
        orc.lib().orc_scan_i32_chunked(orc._p(x), orc._p(y), x.size, orc.OP_SUM, 0, threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        orc.lib().orc_scan_i32_chunked(orc._p(x), orc._p(y), x.size, orc.OP_SUM, 0, threads)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * sum(times) / len(times)
    gbs = 2 * SCAN_N * 4 / (ms * 1e-3) / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int32", "data": "synthetic (seeded, uniform [0,16))",
            "config": scan_config(world),
            "cpu_baseline": {"value": round(gbs, 2), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": "full config per step: OpenMP chunked scan (chunk totals, carry, rescan) "
                                       "restating eval_scan (oracle/plan_window.rs:10-238); the reference is Rust "
                                       "with no GPU path and no toolchain here"},
            "e2e": {"value": round(gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def profile_cases(which: str):
    """Small cases of each kernel for ncu (inputs above the 126 MB L2, a few GB on the device at most), each
    launched 3 times with an L2 flush in between. `which`: a lift name or "all"."""
    import torch

    from unpopped_b200 import ops, workloads as wl

    dev = torch.device("cuda", 0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    cases = {}

    def case(name):
        def deco(f):
            cases[name] = f
            return f
        return deco

    @case("scan")
    def _():
        x = wl.scan_input(n=1 << 26, device=dev)
        y = torch.empty_like(x)
        return lambda: ops.scan(x, "sum", out=y)

    @case("rowsum")
    def _():
        x = wl.rowsum_input(device=dev)
        o = torch.empty(x.shape[0], device=dev)
        return lambda: ops.row_sum(x, "f32", out=o)

    @case("rowsum_auto")
    def _():
        x = wl.rowsum_input(device=dev)
        o = torch.empty(x.shape[0], device=dev)
        return lambda: ops.row_sum(x, "auto", block=1024, out=o)

    @case("rowmax_f32")
    def _():
        x = wl.rowsum_input(device=dev)
        o = torch.empty(x.shape[0], device=dev)
        return lambda: ops.reduce2d(x, "max", 1, out=o)

    @case("colmax_f32")
    def _():
        x = wl.rowsum_input(device=dev)
        o = torch.empty(x.shape[1], device=dev)
        return lambda: ops.reduce2d(x, "max", 0, out=o)

    @case("row_softmax")
    def _():
        x = wl.rowsum_input(device=dev)
        o = torch.empty_like(x)
        return lambda: ops.row_reduce(x, "softmax", block=256, out=o)

    @case("row_rms_norm")
    def _():
        x = wl.rowsum_input(device=dev)
        o = torch.empty_like(x)
        return lambda: ops.row_reduce(x, "rms_norm", block=256, out=o)

    @case("window")
    def _():
        x = wl.rowsum_input(device=dev)
        o = torch.empty((x.shape[0], x.shape[1] // 2), device=dev)
        return lambda: ops.window(x, "max", 3, 2, 1, 1, out=o)

    @case("window_mid")
    def _():
        x = torch.randn(64, 8192, 128, device=dev)
        o = torch.empty(64, 4096, 128, device=dev)
        return lambda: ops.window(x, "max", 3, 2, 1, 1, axis=1, out=o)

    @case("im2col")
    def _():
        x = torch.randn(32, 64, 56, 56, device=dev)
        o = torch.empty(32, 64 * 9, 56 * 56, device=dev)
        return lambda: ops.im2col(x, (3, 3), (1, 1), (1, 1), out=o)

    @case("colsum_doc")
    def _():
        x = wl.rowsum_input(device=dev)
        o = torch.empty(x.shape[1], device=dev)
        return lambda: ops.reduce2d(x, "sum", 0, block=256, out=o)

    @case("rowsum_serial")
    def _():
        x = wl.rowsum_input(device=dev)
        o = torch.empty(x.shape[0], device=dev)
        return lambda: ops.row_sum(x, "auto", 1, out=o)

    @case("colsum_serial")
    def _():
        x = wl.rowsum_input(device=dev)
        o = torch.empty(x.shape[1], device=dev)
        return lambda: ops.reduce2d(x, "sum", 0, out=o)

    @case("argmax")
    def _():
        x = wl.argmax_input(rows=8192, device=dev)
        return lambda: ops.row_max_argmax(x, torch.int32)

    @case("gather")
    def _():
        t, i = wl.gather_inputs(n=1 << 22, device=dev)
        o = torch.empty(i.numel(), t.shape[1], dtype=t.dtype, device=dev)
        return lambda: ops.gather_rows(t, i, "zero_fill", out=o)

    @case("dequant")
    def _():
        d = wl.w4a16_inputs(device=dev)
        o = torch.empty(d.n, d.k, dtype=torch.bfloat16, device=dev)
        return lambda: ops.dequant_i4(d.w_packed, d.scale, d.group, out=o)

    @case("w4a16")
    def _():
        d = wl.w4a16_inputs(device=dev)
        o = torch.empty(d.m, d.n, dtype=torch.bfloat16, device=dev)
        return lambda: ops.w4a16(d.w_packed, d.scale, d.x, d.group, out=o)

    for name in (cases if which == "all" else which.split(",")):
        run = cases[name]()
        for _ in range(3):
            flush.zero_()
            run()
        torch.cuda.synchronize()
        print("profiled case", name, flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--lifts", default="all", choices=["all", "none"])
    ap.add_argument("--profile", default=None,
                    help="run only the small ncu cases of these lifts, comma-separated (scan, rowsum, rowsum_auto, "
                         "rowsum_serial, rowmax_f32, colmax_f32, colsum_doc, colsum_serial, im2col, row_softmax, row_rms_norm, window, window_mid, argmax, gather, dequant, w4a16, all)")
    args = ap.parse_args()
    if args.profile:
        profile_cases(args.profile)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    K, W = args.steps, max(3, args.warmup)

    ctx = Ctx(args)
    torch = ctx.torch
    from unpopped_b200 import ops, workloads as wl

    hbm, bf16, peak_src = peaks()
    clk = ClockSampler(ctx.local)
    clk.start()

    # ---- headline: inclusive add-scan over 2^28 int32 per GPU ----
    x = wl.scan_input(device=ctx.dev, seed=wl.SEED + 2 + ctx.rank)
    y = torch.empty_like(x)
    step = make_scan_step(ctx, x, y)
    ms, kms, launches = ctx.timed(step, K, W)
    kms = ms  # one kernel per step at any N
    if ctx.world == 1:
        ops.check_workspace("scan", ctx.dev)
    else:
        scan_ws_status(ctx)
    nbytes = wl.scan_bytes()
    value = ctx.world * nbytes / (ms * 1e-3) / 1e9
    achieved = nbytes / (kms * 1e-3) / 1e9

    # ---- e2e through the C ABI from pinned host memory (copies inside the timed region) ----
    xh = x.cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    if ctx.world == 1:
        # the host-buffer entry: chunks stream through the device with copy-in, scan and copy-out overlapped
        def e2e_step(i, kin):
            ops.scan_host(xh, "sum", out=yh)
        api = "up_sm100_scan_i32_host (pinned host buffers, copies overlapped with the scan)"
    else:
        # sharded: every rank copies its shard in, runs the block-cyclic scan and copies its result out
        def e2e_step(i, kin):
            x.copy_(xh, non_blocking=True)
            step(i, None)
            yh.copy_(y, non_blocking=True)
        api = "copy in, up_sm100_launch_multi block-cyclic scan (one pass, cross-GPU look-back), copy out"
    e_ms, _, _ = ctx.timed(e2e_step, max(3, K // 4), 3, head_start=ctx.world > 1)
    e2e = {"value": round(ctx.world * nbytes / (e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
           "h2d_bytes_per_step": xh.numel() * 4, "d2h_bytes_per_step": yh.numel() * 4, "api": api}
    contiguous = None
    if ctx.world > 1:
        # the two-pass layout over contiguous shards (fold, all-gather of totals, scan), for comparison
        c_ms, _, _ = ctx.timed(make_scan_step(ctx, x, y, "contiguous"), K, W)
        scan_ws_status(ctx)
        contiguous = {"value": round(ctx.world * nbytes / (c_ms * 1e-3) / 1e9, 1), "ms_per_step": round(c_ms, 4),
                      "frac_of_hbm": round(nbytes / (c_ms * 1e-3) / 1e9 / hbm, 4)}
    del xh, yh, x, y
    torch.cuda.empty_cache()

    lifts = bench_lifts(ctx, K, W, hbm, bf16) if args.lifts == "all" else {}
    clocks = clk.stop()

    cpu = cpu_scan_baseline() if (ctx.rank == 0 and ctx.world == 1) else None
    cpu_cfg, cpu_samples, cpu_threads = ({}, {}, None)
    if ctx.rank == 0 and ctx.world == 1 and args.lifts == "all":
        cpu_cfg, cpu_samples, cpu_threads = cpu_baselines()
    traffic = ncu_traffic("scan_i32_persist_kernel_incl_add.md")
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": ctx.world, "steps": K, "warmup": W,
        "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int32", "data": "synthetic (seeded torch generator, uniform [0,16))",
        "config": scan_config(ctx.world),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": traffic, "peak_source": peak_src,
                     "kernel": "scan_i32_persist_kernel<SUM>", "algorithmic_bytes_per_launch": nbytes,
                     "kernel_ms": round(kms, 4)},
        "e2e": e2e,
        "gpu_launches": launches,
        "clocks": clocks,
        "cpu_baseline": cpu,
    }
    if lifts:
        line["lifts"] = {k: [v["value"], v["frac_of_hbm"]] for k, v in lifts.items() if k not in CONFIG_LIFTS}
        line["lifts_unit"] = "[GB/s aggregate, fraction of measured HBM per GPU]"
        if cpu_samples:
            line["cpu_samples"] = dict(cpu_samples, threads=cpu_threads, unit="GB/s of the sample's algorithmic bytes")
        head = {"value": round(value, 1), "ms_per_step": round(ms, 4), "frac_of_hbm": round(achieved / hbm, 4)}
        line["configs"] = config_block(lifts, head, cpu_cfg)
    if contiguous is not None:
        line["scan_contiguous_two_pass"] = contiguous
    if ctx.rank == 0:
        print(json.dumps(line, separators=(",", ":")), flush=True)
    if ctx.world > 1:
        torch.cuda.synchronize()
        ctx.barrier()
        ctx.comm.close()
        ctx.dist.destroy_process_group()


if __name__ == "__main__":
    main()
