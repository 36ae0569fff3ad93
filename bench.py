"""Benchmark of the B200 strict-tensor provider (driver contract: one JSON line on rank 0).

Workload (the headline): strict checked F32 MatMul 8192^3, row-major,
entries dyadic U[-1,1) from a seed, fault-free.  A "step" is one strict MatMul call (exponent
prescan + ordered-K kernel).  N GPUs: the output rows are sharded across ranks (K is never split,
so the strict order is untouched), every rank's rows go into every rank's C inside the MatMul
kernel (NVLink stores), and the per-rank fault words are combined into the global first fault
every step (strong scaling: the 8192^3 product is fixed).  After the timed region, at N > 1,
sampled rows of the gathered C (both sides of every shard boundary) are compared bit for bit with
a one-device MatMul of the same rows.

Secondary keys of the same line: BASELINE configs[4] (strict MSE + SGD on 2^28 F32 elements, HBM
GB/s; element-sharded at N > 1 with its own parity check), and at N = 1 configs[2] (F64 4096^3),
configs[0] (single-layer train step), configs[3] (4-layer MLP step; column-sharded at N > 1), the
underflow-policy variants, and the measured FP32/FP64 non-FMA issue peak.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
  python bench.py --case matmul|sgd|mse|msesgd|binary|train1|mlp|probe [...]   (one timed case,
         for profilers; see run_case)

--impl reference times the reference's strict CPU path restated in C (oracle/; the reference is
Rust and cannot be built here) on ONE host thread, as the reference's CPU provider runs it, over
a bounded sample of the 8192^3 product's cells.
"""
import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "strict F32 MatMul TFLOP/s @8192^3 at 1/2/4/8 B200; MSE+SGD HBM GB/s"
WORKLOAD = "strict checked F32 MatMul 8192^3 (BASELINE configs[1]), dyadic U[-1,1) seeded"
N = 8192
FLOPS = 2.0 * N * N * N
MSE_SGD_ELEMS = 1 << 28
MATMUL_TRAFFIC_BYTES = 3378593536 + 266733056  # measured DRAM bytes of one 8192^3 strict MatMul launch
REFERENCE_CELLS = 1024  # output cells of the 8192^3 product per reference step (one thread)
MLP_DIMS, MLP_BATCH, MLP_RATE = [1024, 4096, 4096, 4096, 256], 8192, 1e-3


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-secondary", action="store_true", help="skip the MSE+SGD line item")
    ap.add_argument("--no-extras", action="store_true", help="skip the other configurations and policy variants")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    # --case: one timed case for profilers
    ap.add_argument("--case", choices=["matmul", "sgd", "mse", "msesgd", "binary", "train1", "mlp", "probe"])
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=8192)
    ap.add_argument("--k", type=int, default=1024)
    ap.add_argument("--count", type=int, default=1 << 26)
    ap.add_argument("--dtype", default="f32", choices=["f32", "f64"])
    ap.add_argument("--layout", default="nn", choices=["nn", "tn", "nt", "tt"])
    ap.add_argument("--policy", type=int, default=0)
    ap.add_argument("--repeat", type=int, default=2)
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            d = json.load(fh)
        return d.get("hbm_gbs", 6557.1), d.get("sm_max_mhz", 1965.0), "MEASURED_PEAKS.json"
    return 6650.0, 1965.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.device_index = device_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100", "-i",
                 str(self.device_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
            deadline = time.time() + 5.0  # the timed region starts once sampling has begun
            while not self.lines and time.time() < deadline and self.proc.poll() is None:
                time.sleep(0.02)
        except (OSError, ValueError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def dyadic(torch, shape, seed, device, dtype=None):
    """Seeded exact dyadic U[-1,1): k * 2^-23 (binary32) or k * 2^-52 (binary64).  A block of a
    seeded tensor is always cut from the whole draw (a draw in pieces need not give the same
    numbers)."""
    dtype = dtype or torch.float32
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    frac = 23 if dtype == torch.float32 else 52
    it = torch.int32 if dtype == torch.float32 else torch.int64
    k = torch.randint(-(1 << frac), 1 << frac, shape, generator=g, device=device, dtype=it)
    return k.to(dtype) * (2.0 ** -frac)


def dyadic_rows(torch, shape, seed, device, rows):
    """Rows `rows` (a slice or an index list) of the seeded tensor dyadic(shape, seed)."""
    full = dyadic(torch, shape, seed, device)
    part = full[rows].contiguous()
    del full
    return part


def host_dyadic(rng, shape, low=-1):
    return (rng.integers(low * (1 << 23), 1 << 23, size=shape, dtype=np.int64) * 2.0 ** -23).astype(np.float32)


def time_calls(torch, fn, reps, stream, warm=1):
    """Mean milliseconds per call of fn() on `stream` (CUDA events, after `warm` calls)."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def matmul_launches(rows, columns, sms, bm=128, bn=128):
    """Kernels one strict MatMul call launches under a rejecting policy: the two exponent
    prescans, then the TMA kernel (plus the half-tile launch that fills its last wave when that
    wave would be at most half full) or, for a product of few tiles, the 16 x 16-tile kernel."""
    tiles = -(-rows // bm) * -(-columns // bn)
    if tiles * 4 < sms:
        return 3
    rem = tiles % sms
    split = tiles > sms and rem != 0 and 2 * rem <= sms
    return 2 + (2 if split else 1)


# --------------------------------------------------------------------------- reference arm
def reference_cells(step):
    """The flat cells of the 8192^3 product one reference step computes: REFERENCE_CELLS
    consecutive cells of one output row (rows and column offsets vary by step)."""
    row = (step * 977) % N
    col0 = (step * 3 * REFERENCE_CELLS) % N
    return row * N + col0 + np.arange(REFERENCE_CELLS, dtype=np.uint64)


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle

    rng = np.random.default_rng(20261201)
    a = host_dyadic(rng, (N, N))
    b = host_dyadic(rng, (N, N))
    times = []
    for step in range(args.warmup + args.steps):
        cells = reference_cells(step)
        t0 = time.perf_counter()
        status, _ = oracle.matmul_cells(a, b, cells)
        dt = time.perf_counter() - t0
        assert status == oracle.STATUS_OK
        if step >= args.warmup:
            times.append(dt)
    per_cell = statistics.mean(times) / REFERENCE_CELLS
    value = 2.0 * N / per_cell / 1e12
    # the same law on every host thread (rows split across threads), reported beside it
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    status, _ = oracle.matmul(a, b, rows=(0, threads), threads=threads)
    all_dt = time.perf_counter() - t0
    assert status == oracle.STATUS_OK
    sample = (f"{REFERENCE_CELLS} consecutive output cells of one row per step (full K = {N} ordered loop "
              f"each; row and columns vary by step), soft-float law, 1 thread; extrapolated per cell")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.mean(times) * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample": sample,
                   "kind": "oracle port of Crates/backends/cpu/prepared_tensor/execution/execution.rs:243-281, "
                           "single-threaded like Crates/backends/cpu/prepared_tensor/prepared_tensor.rs:258-270"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": 1, "kind": "port", "sample": sample},
        "all_cores": {"value": 2.0 * threads * N * N / all_dt / 1e12, "unit": "TFLOP/s", "threads": threads,
                      "sample": f"{threads} full output rows, one per thread (not the reference's own path, "
                                f"which runs on one thread)"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_sample():
    """The reference's strict CPU path (its C restatement), one thread, on a bounded cell sample."""
    import oracle

    rng = np.random.default_rng(7)
    a = host_dyadic(rng, (N, N))
    b = host_dyadic(rng, (N, N))
    steps, t0 = 12, time.perf_counter()
    for step in range(steps):
        status, _ = oracle.matmul_cells(a, b, reference_cells(step))
        assert status == oracle.STATUS_OK
    dt = time.perf_counter() - t0
    value = 2.0 * N * steps * REFERENCE_CELLS / dt / 1e12
    return {"value": value, "unit": "TFLOP/s", "cores": 1, "kind": "port",
            "sample": f"{steps} x {REFERENCE_CELLS} output cells of the 8192^3 product ({dt:.1f} s), soft-float "
                      "law, 1 thread, extrapolated per cell"}


# --------------------------------------------------------------------------- provider arm
def main():
    args = parse()
    if args.case:
        run_case(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist

    pcu = importlib.import_module("fusion-pcu_b200")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world and world != 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    stream = torch.cuda.current_stream()
    hbm_gbs, sm_max_mhz, peak_src = peaks()
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    peak_tflops = sms * 128 * sm_max_mhz * 1e6 / 1e12

    # ---- data: this rank's row block of A and all of B (each rank owns a row block of C)
    rows_per = N // world
    r0 = rank * rows_per
    a = dyadic_rows(torch, (N, N), 1, device, slice(r0, r0 + rows_per))
    b = dyadic(torch, (N, N), 2, device)
    c_local = torch.empty((rows_per, N), dtype=torch.float32, device=device)
    status = pcu.new_status(device=device)
    lib = pcu.library()
    ws_bytes = lib.pcu_b200_strict_matmul_workspace_size(rows_per, N, N)
    workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=device)

    sharded = importlib.import_module("fusion-pcu_b200.sharded") if world > 1 else None
    shared_c = sharded.PeerRows(N, N, torch.float32) if world > 1 else None

    def fused_call():
        # this rank's rows with global fault events, written into every rank's C by the same
        # kernel (peer stores over NVLink, after each peer has entered the call)
        sharded.strict_matmul_rows_allgather(a, b, r0, shared_c, status, workspace=workspace, stream=stream)

    def step():
        if world > 1:
            fused_call()
            # the global first fault; also orders every rank's stores before C is read
            sharded.all_reduce_min_status(status)
        else:
            pcu.strict_matmul(a, b, out=c_local, status=status, workspace=workspace, stream=stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    word = int(status.cpu().numpy().view(np.uint64)[0])
    assert word == pcu.STATUS_OK, f"unexpected fault {word:#x}"

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        # the barrier comes after every rank's sampler is running (their start-up times differ),
        # so that all ranks enter the timed region together: the per-step collective would
        # otherwise charge the early ranks with waiting for the late ones
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        start.record(stream)
        for _ in range(args.steps):
            step()
        end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end) / args.steps
    assert int(status.cpu().numpy().view(np.uint64)[0]) == pcu.STATUS_OK

    # ---- parity of the gathered C (N > 1, untimed)
    parity = matmul_parity(torch, pcu, shared_c, b, rows_per, world, device) if world > 1 else None

    # kernel-only time of the MatMul call on this rank's shard (prescan + ordered-K kernel, no
    # peers), for the roofline; at N > 1 also the fused all-gather call alone (no collective)
    kernel_ms = time_calls(torch, lambda: pcu.strict_matmul(a, b, out=c_local, status=status, workspace=workspace,
                                                            stream=stream), args.steps, stream, warm=0)
    fused_ms = None
    if world > 1:
        dist.barrier()
        fused_ms = time_calls(torch, fused_call, args.steps, stream, warm=0)
        sharded.all_reduce_min_status(status)
        torch.cuda.synchronize()
        dist.barrier()

    # ---- end to end from page-locked host memory, every step: A's rows and B go up, C's rows and
    # the status word come back.  N = 1: the host-boundary call (pcu_b200_strict_matmul_host, B
    # uploaded in column pieces, A and C by row blocks, all overlapped with the arithmetic).
    # N > 1: each rank uploads its rows of A and only its 1/N slice of B's rows; the slices are
    # all-gathered over NVLink and pcu_b200_strict_matmul_host_left computes the rank's rows.
    a_h = a.cpu().pin_memory()
    k0, k1 = rank * N // world, (rank + 1) * N // world
    b_h = b[k0:k1].cpu().pin_memory()
    c_h = torch.empty((rows_per, N), dtype=torch.float32).pin_memory()
    s_h = torch.empty(1, dtype=torch.int64).pin_memory()
    del workspace
    if world == 1:
        host_scratch = pcu.matmul_host_scratch(a_h, b_h, device=device)

        def e2e_step():
            pcu.strict_matmul_host(a_h, b_h, out=c_h, status=s_h, scratch=host_scratch, stream=stream)
    else:
        b_gathered = torch.empty((N, N), dtype=torch.float32, device=device)
        host_scratch = torch.empty(lib.pcu_b200_strict_matmul_host_left_scratch_size(0, rows_per, N, N),
                                   dtype=torch.uint8, device=device)

        def e2e_step():
            sharded.strict_matmul_rows_host(a_h, b_h, k0, b_gathered, c_h, s_h, scratch=host_scratch, stream=stream)

    e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e2e_ms = time_calls(torch, e2e_step, args.steps, stream, warm=0)
    assert int(s_h.numpy().view(np.uint64)[0]) == pcu.STATUS_OK
    del host_scratch, a_h, b_h, c_h
    if world > 1:
        del b_gathered

    times = torch.tensor([ms, kernel_ms, e2e_ms, fused_ms or 0.0], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms, kernel_ms, e2e_ms, fused_ms = times.tolist()
    del a, b, c_local
    torch.cuda.empty_cache()

    secondary = None
    if not args.no_secondary:
        secondary = mse_sgd(torch, pcu, device, stream, hbm_gbs, args, rank, world)
        torch.cuda.empty_cache()
    extras = {}
    if not args.no_extras:
        extras = other_configs(torch, pcu, device, stream, hbm_gbs, sm_max_mhz, sms, args, rank, world)
        torch.cuda.empty_cache()

    if world > 1:
        torch.cuda.synchronize()
        shared_c.close()  # barriers inside: no rank frees its C while a peer may still map it
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    value = FLOPS / (ms * 1e-3) / 1e12
    kernel_tflops = FLOPS / world / (kernel_ms * 1e-3) / 1e12
    clk = clocks.summary()
    run_peak = sms * 128 * clk["sm_mhz"] * 1e6 / 1e12 if clk["sm_mhz"] else None
    launches = matmul_launches(rows_per, N, sms)
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD,
                   "parallelism": f"row-sharded x{world}" + (
                       " + all-gather of C inside the MatMul kernel (peer stores over NVLink)" if world > 1 else ""),
                   "l2": "inputs (2 x 256 MiB) exceed the 126 MB L2; no flush needed"},
        # per rank: its rows of A and its slice of B's rows in, its rows of C and its status out
        "e2e": {"value": FLOPS / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": (rows_per + N // world) * N * 4, "d2h_bytes_per_step": rows_per * N * 4 + 8,
                "bytes_per": "rank",
                "call": ("pcu_b200_strict_matmul_host (page-locked host buffers; uploads and read-backs "
                         "overlapped with the arithmetic by row blocks)") if world == 1 else
                        ("each rank: its rows of A and 1/N of B's rows up from page-locked memory, B's slices "
                         "all-gathered over NVLink (NCCL), pcu_b200_strict_matmul_host_left for its rows of C, "
                         "C's rows and the status word back")},
        "roofline": {"bound": "fp32-issue", "achieved": kernel_tflops, "peak": peak_tflops, "unit": "TFLOP/s",
                     "frac": kernel_tflops / peak_tflops,
                     "peak_source": f"{sms} SMs x 128 FP32 lanes x sm_max_mhz {sm_max_mhz} ({peak_src}); "
                                    "non-FMA: 1 FMUL + 1 FADD per (cell,k); tensor cores are excluded by the "
                                    "strict contract",
                     "frac_at_run_clock": (kernel_tflops / run_peak) if run_peak else None,
                     "kernel_ms": kernel_ms,
                     # dram__bytes_read.sum + dram__bytes_write.sum of one 8192^3 launch (ncu,
                     # profiles/strict_matmul_f32_8192cubed_traffic.md); not captured for the
                     # row blocks of N > 1
                     "traffic": MATMUL_TRAFFIC_BYTES if world == 1 else None, "traffic_unit": "bytes per launch"},
        "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"]},
        "gpu_launches": launches * args.steps,
    }
    if world > 1:
        line["fused_allgather"] = {
            "kernel_ms_no_peers": kernel_ms, "fused_call_ms": fused_ms, "step_ms": ms,
            "note": "the same shard: the MatMul call alone, the call with the in-kernel all-gather (peer stores "
                    "and entry flags), and the whole step (plus the status all-reduce)"}
        line["parity"] = parity
    if "issue_peak" in extras:
        probe = extras["issue_peak"]["f32_tflops"]
        line["roofline"]["peak_probe"] = probe
        line["roofline"]["frac_of_probe"] = kernel_tflops / probe
    if secondary:
        line["mse_sgd"] = secondary
    line.update(extras)
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline_sample()
    print(json.dumps(line), flush=True)


def matmul_parity(torch, pcu, shared_c, b, rows_per, world, device):
    """Sampled rows of this rank's gathered C -- both sides of every shard boundary, the first and
    last row and four seeded rows -- bit for bit against a one-device strict MatMul of the same
    rows of A; the verdict is all-reduced (every rank checks its own copy of C)."""
    import torch.distributed as dist

    rng = np.random.default_rng(99)
    rows = {0, N - 1} | {r * rows_per + d for r in range(1, world) for d in (-1, 0)}
    rows |= set(int(x) for x in rng.integers(0, N, 4))
    rows = sorted(rows)
    a_rows = dyadic_rows(torch, (N, N), 1, device, rows)
    st = pcu.new_status(device=device)
    want = pcu.strict_matmul(a_rows, b, status=st)
    got = shared_c.local[rows]
    ok = bool(torch.equal(want.view(torch.int32), got.view(torch.int32)))
    ok = ok and int(st.cpu().numpy().view(np.uint64)[0]) == pcu.STATUS_OK
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    return {"matmul_rows": len(rows), "matmul_cells": len(rows) * N, "matmul_ok": bool(flag.item()),
            "against": "one-device pcu_b200_strict_matmul of the same rows of A", "ranks_checked": world}


def mse_sgd(torch, pcu, device, stream, hbm_gbs, args, rank, world):
    """strict MSE + SGD on four 2^28-element F32 tensors, the two independent
    nodes run in one pass (pcu_b200_strict_mse_sgd: the SGD streams in dedicated CTAs of the MSE's
    integer-bound chunk launch).  With N ranks each holds a contiguous element block (strong
    scaling); SGD needs no exchange, MSE hands its running sum from rank to rank in order
    (fusion-pcu_b200/sharded.py).  The two nodes are also timed one after the other.  At N > 1 the
    sharded mean and SGD output are compared with one-device calls afterwards (untimed)."""
    import torch.distributed as dist

    n = MSE_SGD_ELEMS
    sharded = importlib.import_module("fusion-pcu_b200.sharded") if world > 1 else None
    e0, e1 = sharded.shard_bounds(n, rank, world, align=8192) if world > 1 else (0, n)
    m = e1 - e0

    def block(seed):  # this rank's block of the seeded full tensor
        return dyadic_rows(torch, (n,), seed, device, slice(e0, e1))

    w, g_, p, t = block(11), block(12), block(13), block(14)
    out_w = torch.empty_like(w)
    loss = torch.empty((), dtype=torch.float32, device=device)
    s12 = pcu.new_status(2, device=device)  # the two nodes' words, all-reduced together
    s1, s2 = s12[0:1], s12[1:2]
    if world > 1:
        # device hand-off: the segment walks chain through IPC-mapped blocks and one exchange
        # kernel leaves both global first faults and the mean on every rank
        smse = sharded.ShardedMse(p, t, e0, n)
        rider = {"weights": w, "gradient": g_, "rate": 0.01, "first_index": e0, "out": out_w, "status": s2}
        fused_call = lambda: smse.run(s1, stream=stream, sgd=rider)  # noqa: E731
        mse_call = lambda: smse.run(s1, stream=stream)  # noqa: E731
        sgd_call = lambda: (sharded.strict_sgd_block(w, g_, 0.01, e0, s2, out=out_w, stream=stream),  # noqa: E731
                            sharded.all_reduce_min_status(s2))
    else:
        ws = pcu.mse_workspace(p)
        fused_call = lambda: pcu.strict_mse_sgd(p, t, w, g_, 0.01, loss=loss, updated=out_w, mse_status=s1,  # noqa
                                                sgd_status=s2, workspace=ws, stream=stream)
        mse_call = lambda: pcu.strict_mse(p, t, out=loss, status=s1, workspace=ws, stream=stream)  # noqa: E731
        sgd_call = lambda: pcu.strict_sgd(w, g_, 0.01, out=out_w, status=s2, stream=stream)  # noqa: E731

    for _ in range(max(3, min(args.warmup, 3))):
        fused_call()
        mse_call()
        sgd_call()
    torch.cuda.synchronize()
    steps = max(1, min(args.steps, 5))
    times = {}
    for name, fn in (("fused", fused_call), ("mse", mse_call), ("sgd", sgd_call)):
        if world > 1:
            dist.barrier()
        times[name] = time_calls(torch, fn, steps, stream, warm=0)
    tt = torch.tensor([times["fused"], times["mse"], times["sgd"]], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    times["fused"], times["mse"], times["sgd"] = tt.tolist()
    ok = all(int(s.cpu().numpy().view(np.uint64)[0]) == pcu.STATUS_OK for s in (s1, s2))
    mse_bytes, sgd_bytes = 2 * n * 4, 3 * n * 4
    total = mse_bytes + sgd_bytes
    gbs = total / (times["fused"] * 1e-3) / 1e9
    result = {"value": gbs, "unit": "GB/s", "elements": n, "ms": times["fused"],
              "scaling": "strong", "parallelism": f"element blocks x{world}" + (
                  " + ordered MSE hand-off on the device (NVLink stores)" if world > 1 else ""),
              "call": "pcu_b200_strict_mse_sgd" + ("_split" if world > 1 else ""),
              "separate_ms": times["mse"] + times["sgd"], "mse_ms": times["mse"], "sgd_ms": times["sgd"],
              "separate_gbs": total / ((times["mse"] + times["sgd"]) * 1e-3) / 1e9,
              "sgd_gbs": sgd_bytes / (times["sgd"] * 1e-3) / 1e9,
              "mse_gbs": mse_bytes / (times["mse"] * 1e-3) / 1e9,
              "hbm_peak_gbs": hbm_gbs * world, "frac": gbs / (hbm_gbs * world),
              "mse_frac": mse_bytes / (times["mse"] * 1e-3) / 1e9 / (hbm_gbs * world), "fault_free": ok}
    if world > 1:
        fused_call()
        torch.cuda.synchronize()
        result["parity"] = mse_sgd_parity(torch, pcu, device, smse.mean, out_w, s12, e0, e1, n, rank, world)
        smse.close()
    return result


def mse_sgd_parity(torch, pcu, device, mean, out_w, s12, e0, e1, n, rank, world):
    """The sharded mean, status words and SGD output against one-device calls on the whole
    tensors (rank 0): the mean bit for bit, and the first and last 4096 updated weights of every
    rank's block (gathered to rank 0) against the same elements of the one-device update."""
    import torch.distributed as dist

    edge = 4096
    sample = torch.cat([out_w[:edge], out_w[-edge:]]).contiguous()
    gathered = torch.empty((world, 2 * edge), dtype=torch.float32, device=device)
    dist.all_gather_into_tensor(gathered, sample)
    bounds = torch.tensor([e0, e1], dtype=torch.int64, device=device)
    all_bounds = torch.empty((world, 2), dtype=torch.int64, device=device)
    dist.all_gather_into_tensor(all_bounds, bounds)
    flag = torch.tensor([1], dtype=torch.int32, device=device)
    result = {"mse_mean_ok": None, "sgd_cells": 2 * edge * world, "sgd_ok": None, "status_ok": None}
    if rank == 0:
        p, t = dyadic(torch, (n,), 13, device), dyadic(torch, (n,), 14, device)
        st = pcu.new_status(2, device=device)
        want_mean = pcu.strict_mse(p, t, status=st[0:1])
        del p, t
        w, g_ = dyadic(torch, (n,), 11, device), dyadic(torch, (n,), 12, device)
        want_w = pcu.strict_sgd(w, g_, 0.01, status=st[1:2])
        del w, g_
        mean_ok = bool(torch.equal(want_mean.reshape(1).view(torch.int32), mean.reshape(1).view(torch.int32)))
        sgd_ok = True
        for r, (b0, b1) in enumerate(all_bounds.tolist()):
            want = torch.cat([want_w[b0:b0 + edge], want_w[b1 - edge:b1]])
            sgd_ok = sgd_ok and bool(torch.equal(want.view(torch.int32), gathered[r].view(torch.int32)))
        status_ok = bool(torch.equal(st, s12))
        result.update(mse_mean_ok=mean_ok, sgd_ok=sgd_ok, status_ok=status_ok)
        flag.fill_(1 if (mean_ok and sgd_ok and status_ok) else 0)
        del want_w
    dist.broadcast(flag, src=0)
    result["ok"] = bool(flag.item())
    result["against"] = "one-device pcu_b200_strict_mse and pcu_b200_strict_sgd over all 2^28 elements"
    return result


# --------------------------------------------------------------------------- other configurations
def other_configs(torch, pcu, device, stream, hbm_gbs, sm_max_mhz, sms, args, rank, world):
    """N = 1: the issue-peak probe, configs[2] (F64 4096^3), configs[0] (train step), configs[3]
    (MLP step) and the underflow-policy variants.  N > 1: the column-sharded configs[3] step."""
    out = {}
    if world > 1:
        out["mlp"] = mlp_sharded(torch, pcu, device, world)
        return out
    out["issue_peak"] = issue_peak(torch, pcu, stream, sms, sm_max_mhz)
    out["f64_4096"] = f64_4096(torch, pcu, device, stream, out["issue_peak"]["f64_tflops"])
    out["train1"] = train1(torch, args)
    out["mlp"] = mlp_one_gpu(torch)
    out["policy_variants"] = policy_variants(torch, pcu, device, stream, hbm_gbs)
    return out


def issue_peak(torch, pcu, stream, sms, sm_max_mhz):
    """The measured FP32 and FP64 non-FMA issue rate (pcu_b200_issue_probe: independent,
    separately rounded multiplies and adds at full occupancy), against lanes x SMs x clock."""
    lib = pcu.library()
    res = {}
    for code, name, iters in ((0, "f32", 1 << 16), (1, "f64", 1 << 15)):
        ops = lib.pcu_b200_issue_probe_ops(code, iters)
        ms = time_calls(torch, lambda: pcu._check(lib.pcu_b200_issue_probe(code, iters, pcu._stream(stream))), 3,
                        stream, warm=1)
        res[f"{name}_tflops"] = ops / (ms * 1e-3) / 1e12
        res[f"{name}_lanes_per_sm_at_max_clock"] = ops / (ms * 1e-3) / (sms * sm_max_mhz * 1e6)
    res["how"] = "pcu_b200_issue_probe: 8 multiply + 8 add chains per thread, 2048 threads per SM, CUDA events"
    return res


def f64_4096(torch, pcu, device, stream, f64_peak):
    """strict F64 MatMul 4096^3, dyadic U[-1,1) (2^-52 grid), fault-free."""
    n = 4096
    a, b = dyadic(torch, (n, n), 21, device, torch.float64), dyadic(torch, (n, n), 22, device, torch.float64)
    out = torch.empty((n, n), dtype=torch.float64, device=device)
    st = pcu.new_status(device=device)
    ms = time_calls(torch, lambda: pcu.strict_matmul(a, b, out=out, status=st, stream=stream), 5, stream, warm=2)
    assert int(st.cpu().numpy().view(np.uint64)[0]) == pcu.STATUS_OK
    tflops = 2.0 * n ** 3 / (ms * 1e-3) / 1e12
    return {"value": tflops, "unit": "TFLOP/s", "ms": ms, "peak_probe": f64_peak, "frac_of_probe": tflops / f64_peak,
            "workload": "strict checked F64 MatMul 4096^3 (BASELINE configs[2]), dyadic U[-1,1) seeded"}


def train1(torch, args):
    """the single-layer strict train step (X 256x512, W 512x256, bias and
    target 256x256, lr 0.5) through the graph layer, 10 steps with the updated weights fed back
    (device copy) before each next step; milliseconds per step in each execution mode."""
    graph = importlib.import_module("fusion-pcu_b200.graph")
    sharded_mod = importlib.import_module("fusion-pcu_b200.sharded")
    rng = np.random.default_rng(1)
    g = graph.Graph(32, 0)
    x, w, b, t = g.input((256, 512)), g.input((512, 256)), g.input((256, 256)), g.input((256, 256))
    y = g.relu(g.add(g.matmul(x, w), b))
    loss = g.mean_squared_error(y, t)
    upd = g.sgd_update(w, g.backward_mse_for(loss, w), 0.5)
    prepared = g.prepare([upd, loss])
    feed = {x: host_dyadic(rng, (256, 512)), w: host_dyadic(rng, (512, 256)), b: host_dyadic(rng, (256, 256)),
            t: (rng.integers(0, 1 << 24, (256, 256)) * 2.0 ** -24).astype(np.float32)}
    view = lambda v: torch.as_tensor(sharded_mod._CudaArray(prepared.buffer(v), (512, 256), torch.float32),  # noqa
                                     device="cuda")
    w_in, w_out = view(w), view(upd)
    s = torch.cuda.Stream()
    res = {"workload": "BASELINE configs[0] single-layer strict train step, 10 steps, weights fed back"}
    with torch.cuda.stream(s):
        for mode in ("each_node", "chained", "graph"):
            prepared.execute(feed, mode=mode, stream=s)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(10):
                prepared.execute({}, mode=mode, stream=s)  # status read (host) included
                w_in.copy_(w_out)
            e1.record(s)
            torch.cuda.synchronize()
            res[f"{mode}_ms"] = e0.elapsed_time(e1) / 10
    return res


def mlp_inputs():
    rng = np.random.default_rng(5)
    dims = MLP_DIMS
    x, t = host_dyadic(rng, (MLP_BATCH, dims[0])), host_dyadic(rng, (MLP_BATCH, dims[-1]), 0)
    ws = [(host_dyadic(rng, (dims[k], dims[k + 1])) * np.float32(np.sqrt(6.0 / dims[k]))).astype(np.float32)
          for k in range(4)]
    return x, ws, t


def mlp_flops():
    d, bsz = MLP_DIMS, MLP_BATCH
    return sum(2.0 * bsz * d[k] * d[k + 1] for k in range(4)) * 2 + sum(2.0 * bsz * d[k] * d[k + 1] for k in range(1, 4))


def mlp_one_gpu(torch, repeat=3):
    """BASELINE configs[3] on one GPU: the 4-layer strict MLP step (1024 -> 4096 x 3 -> 256, batch
    8192, lr binary32(1e-3), He-uniform weights) through the graph layer in CUDA-graph mode."""
    graph = importlib.import_module("fusion-pcu_b200.graph")
    x, ws, t = mlp_inputs()
    g = graph.Graph(32, 0)
    gx, gt = g.input(x.shape), g.input(t.shape)
    gws = [g.input(w.shape) for w in ws]
    h = gx
    for k, w in enumerate(gws):
        h = g.matmul(h, w)
        if k < 3:
            h = g.relu(h)
    loss = g.mean_squared_error(h, gt)
    ups = [g.sgd_update(w, d, MLP_RATE) for w, d in zip(gws, g.backward_mse_for_targets(loss, gws))]
    prepared = g.prepare(ups + [loss])
    fused = sum(prepared.fused(v) for v in range(len(g)))
    s = torch.cuda.Stream()
    prepared.execute({gx: x, gt: t, **dict(zip(gws, ws))}, mode="graph", stream=s)
    ms = time_calls(torch, lambda: prepared.execute({}, mode="graph", stream=s), repeat, s, warm=1)
    chained_ms = time_calls(torch, lambda: prepared.execute({}, mode="chained", stream=s), repeat, s, warm=1)
    del prepared, g
    return {"ms_per_step": ms, "tflops": mlp_flops() / (ms * 1e-3) / 1e12, "n_gpus": 1,
            "chained_fused_ms": chained_ms, "fused_nodes": fused,
            "workload": "BASELINE configs[3] 4-layer strict MLP step, graph layer, CUDA-graph mode (the guarded "
                        "chain replayed); chained_fused_ms: the chained mode, the forward ReLUs in their MatMul's "
                        "epilogue (fused_nodes), one host launch per node"}


def mlp_sharded(torch, pcu, device, world, repeat=3):
    """BASELINE configs[3] column-sharded over the ranks (fusion-pcu_b200/sharded.ColumnShardedMlp)."""
    import torch.distributed as dist

    sharded = importlib.import_module("fusion-pcu_b200.sharded")
    x, ws, t = mlp_inputs()
    mlp = sharded.ColumnShardedMlp(MLP_DIMS, MLP_BATCH, MLP_RATE, device=device)
    mlp.load(x, ws, t)
    mlp.step()
    torch.cuda.synchronize()
    dist.barrier()
    ms = time_calls(torch, mlp.step, repeat, torch.cuda.current_stream(), warm=0)
    tt = torch.tensor([ms], dtype=torch.float64, device=device)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    ms = float(tt.item())
    del mlp
    return {"ms_per_step": ms, "tflops": mlp_flops() / (ms * 1e-3) / 1e12, "n_gpus": world,
            "workload": "BASELINE configs[3] 4-layer strict MLP step, weights column-sharded, activations "
                        "all-gathered (NCCL)"}


def policy_variants(torch, pcu, device, stream, hbm_gbs):
    """The RejectSubnormalResult (1) and AllowGradualUnderflow (2) kernels at the headline sizes:
    MatMul 8192^3 (TFLOP/s) and SGD 2^28 F32 (GB/s), beside IeeeAfterRounding (0)."""
    res = {"matmul_8192_tflops": {}, "sgd_2p28_gbs": {}}
    a, b = dyadic(torch, (N, N), 1, device), dyadic(torch, (N, N), 2, device)
    c = torch.empty((N, N), dtype=torch.float32, device=device)
    st = pcu.new_status(device=device)
    for policy in (0, 1, 2):
        ms = time_calls(torch, lambda: pcu.strict_matmul(a, b, False, False, policy, out=c, status=st, stream=stream),
                        2, stream, warm=1)
        res["matmul_8192_tflops"][str(policy)] = FLOPS / (ms * 1e-3) / 1e12
    del a, b, c
    n = MSE_SGD_ELEMS
    w, g_ = dyadic(torch, (n,), 11, device), dyadic(torch, (n,), 12, device)
    out = torch.empty_like(w)
    for policy in (0, 1, 2):
        ms = time_calls(torch, lambda: pcu.strict_sgd(w, g_, 0.01, policy, out=out, status=st, stream=stream), 3,
                        stream, warm=1)
        res["sgd_2p28_gbs"][str(policy)] = 3.0 * n * 4 / (ms * 1e-3) / 1e9
    assert int(st.cpu().numpy().view(np.uint64)[0]) == pcu.STATUS_OK
    res["hbm_peak_gbs"] = hbm_gbs
    return res


# --------------------------------------------------------------------------- --case (profilers)
def run_case(args):
    """One provider call on a fixed seeded case, repeated; prints the CUDA-event time per call and
    checks the status word stayed clean.  For ncu captures (small, few launches) and sweeps."""
    import torch

    pcu = importlib.import_module("fusion-pcu_b200")
    dt = torch.float32 if args.dtype == "f32" else torch.float64
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream()
    if args.case == "train1":
        print(json.dumps(train1(torch, args)))
        return
    if args.case == "mlp":
        print(json.dumps(mlp_one_gpu(torch, args.repeat)))
        return
    if args.case == "probe":
        sms = torch.cuda.get_device_properties(dev).multi_processor_count
        print(json.dumps(issue_peak(torch, pcu, stream, sms, peaks()[1])))
        return
    status, status2 = pcu.new_status(), pcu.new_status()
    if args.case == "matmul":
        tl, tr = args.layout[0] == "t", args.layout[1] == "t"
        a = dyadic(torch, (args.k, args.m) if tl else (args.m, args.k), 1, dev, dt)
        b = dyadic(torch, (args.n, args.k) if tr else (args.k, args.n), 2, dev, dt)
        out = torch.empty((args.m, args.n), dtype=dt, device=dev)
        ws = torch.empty(pcu.library().pcu_b200_strict_matmul_workspace_size(args.m, args.k, args.n),
                         dtype=torch.uint8, device=dev)
        call = lambda: pcu.strict_matmul(a, b, tl, tr, args.policy, out=out, status=status, workspace=ws)  # noqa
        work, unit = 2.0 * args.m * args.n * args.k, "TFLOP/s"
    elif args.case == "sgd":
        w, g = dyadic(torch, (args.count,), 1, dev, dt), dyadic(torch, (args.count,), 2, dev, dt)
        out = torch.empty_like(w)
        call = lambda: pcu.strict_sgd(w, g, 0.01, args.policy, out=out, status=status)  # noqa
        work, unit = 3.0 * args.count * w.element_size(), "GB/s"
    elif args.case == "binary":
        x, y = dyadic(torch, (args.count,), 1, dev, dt), dyadic(torch, (args.count,), 2, dev, dt)
        out = torch.empty_like(x)
        call = lambda: pcu.checked_binary("add", x, y, args.policy, out=out, status=status)  # noqa
        work, unit = 3.0 * args.count * x.element_size(), "GB/s"
    elif args.case == "msesgd":
        p, t = dyadic(torch, (args.count,), 1, dev, dt), dyadic(torch, (args.count,), 2, dev, dt)
        w, g = dyadic(torch, (args.count,), 3, dev, dt), dyadic(torch, (args.count,), 4, dev, dt)
        out, upd = torch.empty((), dtype=dt, device=dev), torch.empty_like(w)
        ws = pcu.mse_workspace(p)
        call = lambda: pcu.strict_mse_sgd(p, t, w, g, 0.01, args.policy, loss=out, updated=upd,  # noqa
                                          mse_status=status, sgd_status=status2, workspace=ws)
        work, unit = 5.0 * args.count * p.element_size(), "GB/s"
    else:  # mse
        p, t = dyadic(torch, (args.count,), 1, dev, dt), dyadic(torch, (args.count,), 2, dev, dt)
        out = torch.empty((), dtype=dt, device=dev)
        ws = pcu.mse_workspace(p)
        call = lambda: pcu.strict_mse(p, t, args.policy, out=out, status=status, workspace=ws)  # noqa
        work, unit = 2.0 * args.count * p.element_size(), "GB/s"
    ms = time_calls(torch, call, args.repeat, stream, warm=1)
    for s in (status, status2):
        word = int(s.cpu().item()) & ((1 << 64) - 1)
        assert word == pcu.STATUS_OK, hex(word)
    scale = 1e12 if unit == "TFLOP/s" else 1e9
    print(json.dumps({"case": args.case, "dtype": args.dtype, "ms_per_call": ms,
                      "rate": work / (ms * 1e-3) / scale, "unit": unit}))


if __name__ == "__main__":
    main()
