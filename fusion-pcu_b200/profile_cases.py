"""Run one provider kernel on a fixed seeded case, for profilers (ncu) and quick timing.

  python fusion-pcu_b200/profile_cases.py matmul --m 8192 --n 8192 --k 1024 [--dtype f32|f64]
         [--layout nn|tn|nt|tt] [--policy 0|1|2] [--repeat R]
  python fusion-pcu_b200/profile_cases.py sgd --count 67108864 [--repeat R]
  python fusion-pcu_b200/profile_cases.py mse --count 67108864 [--repeat R] [--phases]

Each run prints the CUDA-event time per call; it checks that the status word stayed clean.
"""
import argparse
import importlib
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))


def dyadic(torch, shape, seed, dtype):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    frac = 23 if dtype == torch.float32 else 52
    hi = 1 << min(frac, 30)
    k = torch.randint(-hi, hi, shape, generator=g, device="cuda", dtype=torch.int64)
    return (k.to(torch.float64) / hi).to(dtype)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["matmul", "sgd", "mse", "msesgd", "binary", "train1", "mlp"])
    ap.add_argument("--m", type=int, default=8192)
    ap.add_argument("--n", type=int, default=8192)
    ap.add_argument("--k", type=int, default=1024)
    ap.add_argument("--count", type=int, default=1 << 26)
    ap.add_argument("--dtype", default="f32", choices=["f32", "f64"])
    ap.add_argument("--layout", default="nn", choices=["nn", "tn", "nt", "tt"])
    ap.add_argument("--policy", type=int, default=0)
    ap.add_argument("--repeat", type=int, default=2)
    ap.add_argument("--phases", action="store_true", help="mse: also time the prepare and walk phases")
    args = ap.parse_args()

    import torch

    pcu = importlib.import_module("fusion-pcu_b200")
    dt = torch.float32 if args.dtype == "f32" else torch.float64
    if args.case == "train1":
        train_step(args)
        return
    if args.case == "mlp":
        mlp_step(args)
        return
    status = pcu.new_status()
    if args.case == "matmul":
        tl, tr = args.layout[0] == "t", args.layout[1] == "t"
        a = dyadic(torch, (args.k, args.m) if tl else (args.m, args.k), 1, dt)
        b = dyadic(torch, (args.n, args.k) if tr else (args.k, args.n), 2, dt)
        out = torch.empty((args.m, args.n), dtype=dt, device="cuda")
        ws = torch.empty(pcu.library().pcu_b200_strict_matmul_workspace_size(args.m, args.k, args.n),
                         dtype=torch.uint8, device="cuda")
        call = lambda: pcu.strict_matmul(a, b, tl, tr, args.policy, out=out, status=status, workspace=ws)  # noqa
        work, unit = 2.0 * args.m * args.n * args.k, "TFLOP/s"
    elif args.case == "sgd":
        w, g = dyadic(torch, (args.count,), 1, dt), dyadic(torch, (args.count,), 2, dt)
        out = torch.empty_like(w)
        call = lambda: pcu.strict_sgd(w, g, 0.01, args.policy, out=out, status=status)  # noqa
        work, unit = 3.0 * args.count * w.element_size(), "GB/s"
    elif args.case == "binary":
        x, y = dyadic(torch, (args.count,), 1, dt), dyadic(torch, (args.count,), 2, dt)
        out = torch.empty_like(x)
        call = lambda: pcu.checked_binary("add", x, y, args.policy, out=out, status=status)  # noqa
        work, unit = 3.0 * args.count * x.element_size(), "GB/s"
    elif args.case == "msesgd":
        # MSE over (p, t) and SGD over (w, g), fused in one pass
        p, t = dyadic(torch, (args.count,), 1, dt), dyadic(torch, (args.count,), 2, dt)
        w, g = dyadic(torch, (args.count,), 3, dt), dyadic(torch, (args.count,), 4, dt)
        out, upd = torch.empty((), dtype=dt, device="cuda"), torch.empty_like(w)
        ws = pcu.mse_workspace(p)
        status2 = pcu.new_status()
        call = lambda: pcu.strict_mse_sgd(p, t, w, g, 0.01, args.policy, loss=out, updated=upd,  # noqa
                                          mse_status=status, sgd_status=status2, workspace=ws)
        work, unit = 5.0 * args.count * p.element_size(), "GB/s"
    else:
        p, t = dyadic(torch, (args.count,), 1, dt), dyadic(torch, (args.count,), 2, dt)
        out = torch.empty((), dtype=dt, device="cuda")
        ws = torch.empty(pcu.library().pcu_b200_strict_mse_workspace_size(0 if dt == torch.float32 else 1,
                                                                           args.count),
                         dtype=torch.uint8, device="cuda")
        call = lambda: pcu.strict_mse(p, t, args.policy, out=out, status=status, workspace=ws)  # noqa
        work, unit = 2.0 * args.count * p.element_size(), "GB/s"
    call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.repeat):
        call()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.repeat
    word = int(status.cpu().item()) & ((1 << 64) - 1)
    assert word == pcu.STATUS_OK, hex(word)
    scale = 1e12 if unit == "TFLOP/s" else 1e9
    print(f"{args.case} {args.dtype} {ms:.3f} ms/call  {work / (ms * 1e-3) / scale:.2f} {unit}")
    if args.case == "msesgd":
        assert int(status2.cpu().item()) & ((1 << 64) - 1) == pcu.STATUS_OK
        for name, fn in (("separate", lambda: (pcu.strict_mse(p, t, args.policy, out=out, status=status, workspace=ws),
                                               pcu.strict_sgd(w, g, 0.01, args.policy, out=upd, status=status2))),):
            fn()
            e0.record()
            for _ in range(args.repeat):
                fn()
            e1.record()
            torch.cuda.synchronize()
            sep = e0.elapsed_time(e1) / args.repeat
            print(f"  {name} {sep:.3f} ms/call  {work / (sep * 1e-3) / 1e9:.2f} GB/s")
    if args.case == "mse" and args.phases:
        # the two phases through the segment form: bandwidth-bound maps, then the ordered walk
        carry = torch.zeros(1, dtype=dt, device="cuda")
        for name, fn in (("prepare", lambda: pcu.strict_mse_segment_prepare(p, t, 0, args.policy, status=status,
                                                                             workspace=ws)),
                         ("walk", lambda: pcu.strict_mse_segment_walk(p, t, 0, args.count, carry.zero_(), ws,
                                                                      status, args.policy, out=out))):
            e0.record()
            for _ in range(args.repeat):
                fn()
            e1.record()
            torch.cuda.synchronize()
            print(f"  {name} {e0.elapsed_time(e1) / args.repeat:.3f} ms/call")


def train_step(args):
    """The single-layer strict train step of BASELINE configs[0] (X 256x512, W 512x256, bias and
    target 256x256, lr 0.5) through the graph layer: milliseconds per step in each execution mode,
    the weights fed back from the device buffer between steps."""
    import numpy as np
    import torch

    graph = importlib.import_module("fusion-pcu_b200.graph")
    rng = np.random.default_rng(1)
    g = graph.Graph(32, 0)
    x, w, b, t = g.input((256, 512)), g.input((512, 256)), g.input((256, 256)), g.input((256, 256))
    y = g.relu(g.add(g.matmul(x, w), b))
    loss = g.mean_squared_error(y, t)
    upd = g.sgd_update(w, g.backward_mse_for(loss, w), 0.5)
    prepared = g.prepare([upd, loss])
    feed = {x: (rng.integers(-2**23, 2**23, (256, 512)) * 2.0**-23).astype(np.float32),
            w: (rng.integers(-2**23, 2**23, (512, 256)) * 2.0**-23).astype(np.float32),
            b: (rng.integers(-2**23, 2**23, (256, 256)) * 2.0**-23).astype(np.float32),
            t: (rng.integers(0, 2**24, (256, 256)) * 2.0**-24).astype(np.float32)}
    stream = torch.cuda.Stream()
    for mode in ("each_node", "chained", "graph"):
        with torch.cuda.stream(stream):
            prepared.execute(feed, mode=mode, stream=stream)
            torch.cuda.synchronize()
            import time
            t0 = time.perf_counter()
            for _ in range(args.repeat):
                prepared.execute({}, mode=mode, stream=stream)  # inputs stay on the device
            dt = (time.perf_counter() - t0) / args.repeat
        print(f"train1 {mode} {dt * 1e3:.3f} ms/step (host-observed, status read included)")


def mlp_step(args):
    """the 4-layer strict MLP step (1024 -> 4096 x 3 -> 256, batch 8192,
    lr binary32(1e-3)), He-uniform weights.  One GPU: the graph layer in CUDA-graph mode.  Under
    torchrun: the column-sharded step of fusion-pcu_b200/sharded.py.  Prints TFLOP/s of checked
    flops (forward, dW and dH MatMuls: 1.838e12 per step)."""
    import os

    import numpy as np
    import torch
    import torch.distributed as dist

    dims, batch, rate = [1024, 4096, 4096, 4096, 256], 8192, 1e-3
    flops = sum(2.0 * batch * dims[k] * dims[k + 1] for k in range(4)) * 2 + \
        sum(2.0 * batch * dims[k] * dims[k + 1] for k in range(1, 4))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    rng = np.random.default_rng(5)
    dy = lambda shape, lo=-1: ((rng.integers(lo * 2**23, 2**23, shape)) * 2.0**-23).astype(np.float32)  # noqa: E731
    x, t = dy((batch, dims[0])), dy((batch, dims[-1]), 0)
    ws = [(dy((dims[k], dims[k + 1])) * np.float32(np.sqrt(6.0 / dims[k]))).astype(np.float32) for k in range(4)]
    if world == 1:
        graph = importlib.import_module("fusion-pcu_b200.graph")
        g = graph.Graph(32, 0)
        gx, gt = g.input(x.shape), g.input(t.shape)
        gws = [g.input(w.shape) for w in ws]
        h = gx
        for k, w in enumerate(gws):
            h = g.matmul(h, w)
            if k < 3:
                h = g.relu(h)
        loss = g.mean_squared_error(h, gt)
        ups = [g.sgd_update(w, d, rate) for w, d in zip(gws, g.backward_mse_for_targets(loss, gws))]
        prepared = g.prepare(ups + [loss])
        stream = torch.cuda.Stream()
        prepared.execute({gx: x, gt: t, **dict(zip(gws, ws))}, mode="graph", stream=stream)
        prepared.execute({}, mode="graph", stream=stream)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.repeat):
            prepared.execute({}, mode="graph", stream=stream)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.repeat
    else:
        import datetime

        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        sharded = importlib.import_module("fusion-pcu_b200.sharded")
        mlp = sharded.ColumnShardedMlp(dims, batch, rate)
        mlp.load(x, ws, t)
        mlp.step()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.repeat):
            mlp.step()
        e1.record()
        torch.cuda.synchronize()
        tt = torch.tensor([e0.elapsed_time(e1) / args.repeat], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
        dist.destroy_process_group()
    if rank == 0:
        print(f"mlp {world} GPU(s) {ms:.2f} ms/step  {flops / (ms * 1e-3) / 1e12:.2f} TFLOP/s")


if __name__ == "__main__":
    main()
