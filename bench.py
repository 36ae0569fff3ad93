"""Benchmark of the B200 strict-tensor provider (driver contract: one JSON line on rank 0).

Workload (the headline): strict checked F32 MatMul 8192^3, row-major,
entries dyadic U[-1,1) from a seed, fault-free.  A "step" is one pcu_b200_strict_matmul call
(exponent prescan + ordered-K kernel).  N GPUs: the output rows are sharded across ranks (K is
never split, so the strict order is untouched) and the row blocks are all-gathered with NCCL
(strong scaling: the 8192^3 product is fixed), and the per-rank fault words are combined into
the global first fault every step.  Secondary line item: BASELINE configs[4] (strict MSE + SGD
on 2^28 F32 elements, HBM GB/s), element-sharded at N > 1.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

--impl reference times the reference's strict CPU path restated in C (oracle/, the reference
itself is Rust and cannot be built here) on all host cores over a bounded row sample.
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
N = 8192
FLOPS = 2.0 * N * N * N
MSE_SGD_ELEMS = 1 << 28
MATMUL_TRAFFIC_BYTES = 3378593536 + 266733056  # measured DRAM bytes of one 8192^3 strict MatMul launch


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-secondary", action="store_true", help="skip the MSE+SGD line item")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            d = json.load(fh)
        return d.get("hbm_gbs", 6557.1), d.get("sm_max_mhz", 1965.0), "MEASURED_PEAKS.json"
    return 6650.0, 1965.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""

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


def dyadic(torch, shape, seed, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    k = torch.randint(-(1 << 23), 1 << 23, shape, generator=g, device=device, dtype=torch.int32)
    return k.to(torch.float32) * (2.0 ** -23)


# --------------------------------------------------------------------------- reference arm
def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle

    threads = os.cpu_count() or 1
    rng = np.random.default_rng(20261201)
    a = (rng.integers(-(1 << 23), 1 << 23, size=(N, N), dtype=np.int64) * 2.0 ** -23).astype(np.float32)
    b = (rng.integers(-(1 << 23), 1 << 23, size=(N, N), dtype=np.int64) * 2.0 ** -23).astype(np.float32)
    rows = max(threads, 8)  # bounded sample: `rows` full output rows of the 8192^3 product per step
    times = []
    for step in range(args.warmup + args.steps):
        r0 = (step * rows) % N
        t0 = time.perf_counter()
        status, _ = oracle.matmul(a, b, rows=(r0, r0 + rows), threads=threads)
        dt = time.perf_counter() - t0
        assert status == oracle.STATUS_OK
        if step >= args.warmup:
            times.append(dt)
    per_row = statistics.mean(times) / rows
    value = 2.0 * N * N / per_row / 1e12
    sample = f"{rows} full output rows (of {N}) of the 8192^3 product per step, soft-float law, {threads} threads"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": statistics.mean(times) * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "strict F32 MatMul 8192^3 (BASELINE configs[1]), row sample extrapolated",
                   "kind": "oracle port of Crates/backends/cpu/prepared_tensor/execution/execution.rs:243-281"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- provider arm
def cpu_baseline_sample():
    """Single-thread soft-float port (the reference CPU provider is single-threaded) on 2 rows."""
    import oracle

    rng = np.random.default_rng(7)
    a = (rng.integers(-(1 << 23), 1 << 23, size=(2, N), dtype=np.int64) * 2.0 ** -23).astype(np.float32)
    b = (rng.integers(-(1 << 23), 1 << 23, size=(N, N), dtype=np.int64) * 2.0 ** -23).astype(np.float32)
    t0 = time.perf_counter()
    status, _ = oracle.matmul(a, b, rows=(0, 2))
    dt = time.perf_counter() - t0
    assert status == oracle.STATUS_OK
    value = 2.0 * 2 * N * N / dt / 1e12
    return {"value": value, "unit": "TFLOP/s", "cores": 1, "kind": "port",
            "sample": f"2 of {N} output rows of the 8192^3 product ({dt:.1f} s), soft-float law, 1 thread, "
                      "extrapolated per row"}


def main():
    args = parse()
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

    # ---- data: full A and B on every rank (each rank owns a row block of C)
    rows_per = N // world
    r0 = rank * rows_per
    a_full = dyadic(torch, (N, N), 1, device)
    b = dyadic(torch, (N, N), 2, device)
    a = a_full[r0:r0 + rows_per].contiguous()
    del a_full
    c_local = torch.empty((rows_per, N), dtype=torch.float32, device=device)
    status = pcu.new_status(device=device)
    lib = pcu.library()
    ws_bytes = lib.pcu_b200_strict_matmul_workspace_size(rows_per, N, N)
    workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=device)

    sharded = importlib.import_module("fusion-pcu_b200.sharded") if world > 1 else None

    shared_c = sharded.PeerRows(N, N, torch.float32) if world > 1 else None

    def step():
        if world > 1:
            # this rank's rows with global fault events, written into every rank's C by the same
            # kernel (peer stores over NVLink); the status all-reduce gives the global first fault
            # and orders every rank's writes before the next use of C
            sharded.strict_matmul_rows_allgather(a, b, r0, shared_c, status, workspace=workspace, stream=stream)
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
    # kernel-only time of the matmul call (prescan + ordered-K kernel), for the roofline
    k_start, k_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k_start.record(stream)
    for _ in range(args.steps):
        pcu.strict_matmul(a, b, out=c_local, status=status, workspace=workspace, stream=stream)
    k_end.record(stream)
    torch.cuda.synchronize()
    kernel_ms = k_start.elapsed_time(k_end) / args.steps

    # ---- end to end through the host-boundary call (pcu_b200_strict_matmul_host): A's rows and
    # B from page-locked host memory, C's rows and the status word back to it, every step; the
    # uploads and read-backs overlap the arithmetic by row blocks inside the call
    a_h = a.cpu().pin_memory()
    b_h = b.cpu().pin_memory()
    c_h = torch.empty((rows_per, N), dtype=torch.float32).pin_memory()
    s_h = torch.empty(1, dtype=torch.int64).pin_memory()
    del workspace
    host_scratch = pcu.matmul_host_scratch(a_h, b_h, device=device)

    def e2e_step():
        pcu.strict_matmul_host(a_h, b_h, out=c_h, status=s_h, scratch=host_scratch, stream=stream)

    e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e_end.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e_start.elapsed_time(e_end) / args.steps
    assert int(s_h.numpy().view(np.uint64)[0]) == pcu.STATUS_OK

    times = torch.tensor([ms, kernel_ms, e2e_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms, kernel_ms, e2e_ms = times.tolist()

    secondary = None
    if not args.no_secondary:
        secondary = mse_sgd(torch, pcu, device, stream, hbm_gbs, args, rank, world)

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
    line = {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "strict checked F32 MatMul 8192^3 (BASELINE configs[1]), dyadic U[-1,1) seeded",
                   "parallelism": f"row-sharded x{world}" + (
                       " + all-gather of C inside the MatMul kernel (peer stores over NVLink)" if world > 1 else ""),
                   "l2": "inputs (2 x 256 MiB) exceed the 126 MB L2; no flush needed"},
        # every rank copies its A row block and all of B in, its C row block and status out
        "e2e": {"value": FLOPS / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": (rows_per + N) * N * 4, "d2h_bytes_per_step": rows_per * N * 4 + 8,
                "call": "pcu_b200_strict_matmul_host (page-locked host buffers; uploads and read-backs "
                        "overlapped with the arithmetic by row blocks)"},
        "roofline": {"bound": "fp32-issue", "achieved": kernel_tflops, "peak": peak_tflops, "unit": "TFLOP/s",
                     "frac": kernel_tflops / peak_tflops,
                     "peak_source": f"{sms} SMs x 128 FP32 lanes x sm_max_mhz {sm_max_mhz} ({peak_src}); "
                                    "non-FMA: 1 FMUL + 1 FADD per (cell,k); tensor cores are excluded by the "
                                    "strict contract",
                     "frac_at_run_clock": (kernel_tflops / run_peak) if run_peak else None,
                     # dram__bytes_read.sum + dram__bytes_write.sum of one 8192^3 launch (ncu,
                     # profiles/strict_matmul_f32_8192cubed_traffic.md); not captured for the
                     # row blocks of N > 1
                     "traffic": MATMUL_TRAFFIC_BYTES if world == 1 else None, "traffic_unit": "bytes per launch"},
        "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"]},
        "gpu_launches": 3 * args.steps,
    }
    if secondary:
        line["mse_sgd"] = secondary
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline_sample()
    print(json.dumps(line), flush=True)


def mse_sgd(torch, pcu, device, stream, hbm_gbs, args, rank, world):
    """strict MSE + SGD on four 2^28-element F32 tensors, the two independent
    nodes run in one pass (pcu_b200_strict_mse_sgd: the SGD streams in dedicated CTAs of the MSE's
    integer-bound chunk launch).  With N ranks each holds a contiguous element block (strong
    scaling); SGD needs no exchange, MSE hands its running sum from rank to rank in order
    (fusion-pcu_b200/sharded.py).  The two nodes are also timed one after the other."""
    import torch.distributed as dist

    n = MSE_SGD_ELEMS
    sharded = importlib.import_module("fusion-pcu_b200.sharded") if world > 1 else None
    e0, e1 = sharded.shard_bounds(n, rank, world, align=8192) if world > 1 else (0, n)
    m = e1 - e0

    def block(seed):  # this rank's block of the seeded full tensor
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        if e0:
            torch.randint(-(1 << 23), 1 << 23, (e0,), generator=g, device=device, dtype=torch.int32)
        k = torch.randint(-(1 << 23), 1 << 23, (m,), generator=g, device=device, dtype=torch.int32)
        return k.to(torch.float32) * (2.0 ** -23)

    w, g_, p, t = block(11), block(12), block(13), block(14)
    out_w = torch.empty_like(w)
    loss = torch.empty((), dtype=torch.float32, device=device)
    s12 = pcu.new_status(2, device=device)  # the two nodes' words, all-reduced together
    s1, s2 = s12[0:1], s12[1:2]
    if world > 1:
        smse = sharded.ShardedMse(p, t, e0, n)
        rider = {"weights": w, "gradient": g_, "rate": 0.01, "first_index": e0, "out": out_w, "status": s2}
        fused_call = lambda: (smse.run(s1, stream=stream, sgd=rider, reduce_status=False),  # noqa: E731
                              sharded.all_reduce_min_status(s12))
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
        torch.cuda.synchronize()
        e_0, e_1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_0.record(stream)
        for _ in range(steps):
            fn()
        e_1.record(stream)
        torch.cuda.synchronize()
        times[name] = e_0.elapsed_time(e_1) / steps
    tt = torch.tensor([times["fused"], times["mse"], times["sgd"]], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    times["fused"], times["mse"], times["sgd"] = tt.tolist()
    ok = all(int(s.cpu().numpy().view(np.uint64)[0]) == pcu.STATUS_OK for s in (s1, s2))
    mse_bytes, sgd_bytes = 2 * n * 4, 3 * n * 4
    total = mse_bytes + sgd_bytes
    gbs = total / (times["fused"] * 1e-3) / 1e9
    return {"value": gbs, "unit": "GB/s", "elements": n, "ms": times["fused"],
            "scaling": "strong", "parallelism": f"element blocks x{world}" + (
                " + ordered MSE hand-off" if world > 1 else ""),
            "call": "pcu_b200_strict_mse_sgd" + ("_segment_prepare + ordered walks" if world > 1 else ""),
            "separate_ms": times["mse"] + times["sgd"], "mse_ms": times["mse"], "sgd_ms": times["sgd"],
            "separate_gbs": total / ((times["mse"] + times["sgd"]) * 1e-3) / 1e9,
            "sgd_gbs": sgd_bytes / (times["sgd"] * 1e-3) / 1e9, "mse_gbs": mse_bytes / (times["mse"] * 1e-3) / 1e9,
            "hbm_peak_gbs": hbm_gbs * world, "frac": gbs / (hbm_gbs * world), "fault_free": ok}


if __name__ == "__main__":
    main()
