"""The column-sharded MLP training step (fusion-pcu_b200/sharded.py) on 2+ B200s against the
same step through the one-device graph layer: updated weights and loss bit for bit."""
import importlib
import os
import socket

import numpy as np
import pytest

from gpu_util import dyadic_uniform

pytestmark = pytest.mark.gpu

DIMS = [64, 128, 128, 128, 32]
BATCH = 96


def _data():
    rng = np.random.default_rng(31)
    x = dyadic_uniform(rng, (BATCH, DIMS[0]), 32)
    ws = [(dyadic_uniform(rng, (DIMS[k], DIMS[k + 1]), 32) * np.float32(0.125)).astype(np.float32) for k in range(4)]
    t = dyadic_uniform(rng, (BATCH, DIMS[-1]), 32, low=0.0)
    return x, ws, t


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        sharded = importlib.import_module("fusion-pcu_b200.sharded")
        pcu = importlib.import_module("fusion-pcu_b200")
        x, ws, t = _data()
        mlp = sharded.ColumnShardedMlp(DIMS, BATCH, 1e-3)
        mlp.load(x, ws, t)
        loss = mlp.step()
        full = mlp.full_weights()
        torch.cuda.synchronize()
        words = mlp.status.cpu().numpy().view(np.uint64)
        assert all(int(w) == pcu.STATUS_OK for w in words)
        queue.put((rank, loss.cpu().numpy().reshape(1).view(np.uint32)[0],
                   [w.cpu().numpy().view(np.uint32) for w in full]))
    finally:
        dist.destroy_process_group()


def test_column_sharded_mlp_step_matches_one_device():
    import torch

    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    # one device, through the graph layer
    graph = importlib.import_module("fusion-pcu_b200.graph")
    x, ws, t = _data()
    g = graph.Graph(32, 0)
    gx = g.input(x.shape)
    gws = [g.input(w.shape) for w in ws]
    gt = g.input(t.shape)
    h = gx
    for k, w in enumerate(gws):
        h = g.matmul(h, w)
        if k < 3:
            h = g.relu(h)
    loss = g.mean_squared_error(h, gt)
    grads = g.backward_mse_for_targets(loss, gws)
    ups = [g.sgd_update(w, d, 1e-3) for w, d in zip(gws, grads)]
    feed = {gx: x, gt: t, **{w: a for w, a in zip(gws, ws)}}
    want = g.prepare(ups + [loss]).run(feed, ups + [loss], mode="chained")
    del g

    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict((r[0], r[1:]) for r in (queue.get(timeout=300) for _ in range(world)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in range(world):
        loss_bits, weights = got[rank]
        assert loss_bits == want[loss].reshape(1).view(np.uint32)[0]
        for k, u in enumerate(ups):
            assert np.array_equal(weights[k], want[u].view(np.uint32)), (rank, k)
