"""Split strict MSE (segment prepare + ordered walk) and the multi-GPU sharded path on B200s.

* On one GPU: a reduction cut into segments and walked in order with the carried running sum
  must give the bits and the first fault of the one-call strict MSE and of the oracle, for cuts
  inside chunks, on chunk edges and of length zero.
* On 2+ GPUs (skipped with fewer): MatMul rows, SGD elements and MSE segments sharded over NCCL
  ranks must reproduce the one-device results and first faults exactly.
"""
import importlib
import os
import socket

import numpy as np
import pytest

import oracle
from gpu_util import bits, dyadic_uniform, status_word, to_device, to_host

pytestmark = pytest.mark.gpu

pcu = importlib.import_module("fusion-pcu_b200")


def _segments(p, t, cuts, width):
    import torch

    n = p.numel()
    edges = [0] + list(cuts) + [n]
    status = pcu.new_status()
    carry = torch.zeros((), dtype=p.dtype, device=p.device)
    mean = torch.zeros((), dtype=p.dtype, device=p.device)
    for a, b in zip(edges, edges[1:]):
        ps, ts = p[a:b].contiguous(), t[a:b].contiguous()
        _, ws = pcu.strict_mse_segment_prepare(ps, ts, a, status=status)
        pcu.strict_mse_segment_walk(ps, ts, a, n, carry, ws, status, out=mean if b == n else None)
    torch.cuda.synchronize()
    return status_word(status), bits(to_host(mean).reshape(1))[0]


@pytest.mark.parametrize("width", [32, 64])
@pytest.mark.parametrize("case", ["clean", "nan_mid", "inf_late", "overflow_by_carry"])
def test_segments_match_one_call_and_oracle(width, case):
    import torch

    rng = np.random.default_rng(31 + width)
    n = 3 * 8192 + 777
    p = dyadic_uniform(rng, n, width)
    t = dyadic_uniform(rng, n, width)
    if case == "nan_mid":
        p[20000] = np.nan
    elif case == "inf_late":
        t[n - 3] = np.inf
    elif case == "overflow_by_carry":
        big = 1.5e19 if width == 32 else 1e154
        p[9000:] = big
        t[9000:] = 0
    st_o, out_o = oracle.mse(p, t)
    pd, td = to_device(p), to_device(t)
    status = pcu.new_status()
    whole = pcu.strict_mse(pd, td, status=status)
    torch.cuda.synchronize()
    assert status_word(status) == st_o
    # the one-call form on operands that are not 16-byte aligned (element offset 1)
    st_u, out_u = oracle.mse(p[1:], t[1:])
    status_u = pcu.new_status()
    got_u = pcu.strict_mse(pd[1:], td[1:], status=status_u)
    torch.cuda.synchronize()
    assert status_word(status_u) == st_u
    if st_u == oracle.STATUS_OK:
        assert bits(to_host(got_u).reshape(1))[0] == bits(out_u)[0]
    for cuts in ([8192], [100, 8192 * 2 + 5], [5000, 5000, 20001], [1, 2, 3, n - 1]):
        word, got = _segments(pd, td, cuts, width)
        assert word == st_o, (cuts, hex(word), hex(st_o))
        if st_o == oracle.STATUS_OK:
            assert got == bits(out_o)[0] == bits(to_host(whole).reshape(1))[0], cuts


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, queue):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        sharded = importlib.import_module("fusion-pcu_b200.sharded")
        rng = np.random.default_rng(77)
        m, k, n = 512, 384, 256
        a = dyadic_uniform(rng, (m, k), 32)
        b = dyadic_uniform(rng, (k, n), 32)
        a[300, 17] = np.nan
        rows = m // world
        r0 = rank * rows
        status = pcu.new_status()
        local = torch.empty((rows, n), dtype=torch.float32, device="cuda")
        full = torch.empty((m, n), dtype=torch.float32, device="cuda")
        sharded.strict_matmul_rows(to_device(a[r0:r0 + rows]), to_device(b), r0, local, status, gathered=full)
        sharded.all_reduce_min_status(status)
        mm_word = status_word(status)
        mm_bits = bits(to_host(full)) if mm_word == pcu.STATUS_OK else None

        e = 5 * 8192 + 123
        p = dyadic_uniform(rng, e, 32)
        t = dyadic_uniform(rng, e, 32)
        e0, e1 = sharded.shard_bounds(e, rank, world, align=4)
        st2 = pcu.new_status()
        sgd_out = sharded.strict_sgd_block(to_device(p[e0:e1]), to_device(t[e0:e1]), 0.25, e0, st2)
        sharded.all_reduce_min_status(st2)
        st3 = pcu.new_status()
        mse = sharded.ShardedMse(to_device(p[e0:e1]), to_device(t[e0:e1]), e0, e, handoff="nccl")
        mean = mse.run(st3)
        torch.cuda.synchronize()
        # the device hand-off on the same segments: twice in a row (the exchange banks alternate)
        # and then with an SGD node riding along, whose word is MIN-reduced with the MSE's
        dev = sharded.ShardedMse(to_device(p[e0:e1]), to_device(t[e0:e1]), e0, e)
        dev_words, dev_means = [], []
        for _ in range(2):
            st4 = pcu.new_status()
            dev_means.append(bits(to_host(dev.run(st4)).reshape(1))[0])
            torch.cuda.synchronize()
            dev_words.append(status_word(st4))
        st5, st6 = pcu.new_status(), pcu.new_status()
        w_out = torch.empty(e1 - e0, dtype=torch.float32, device="cuda")
        rider = {"weights": to_device(p[e0:e1]), "gradient": to_device(t[e0:e1]), "rate": 0.25, "first_index": e0,
                 "out": w_out, "status": st6}
        dev_means.append(bits(to_host(dev.run(st5, sgd=rider)).reshape(1))[0])
        torch.cuda.synchronize()
        dev_words += [status_word(st5), status_word(st6)]
        dev.close()
        queue.put((rank, mm_word, mm_bits, status_word(st2), bits(to_host(sgd_out)), status_word(st3),
                   bits(to_host(mean).reshape(1))[0], dev_words, dev_means, bits(to_host(w_out))))
    finally:
        dist.destroy_process_group()


def test_nccl_sharded_matches_one_device():
    import torch

    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict((r[0], r[1:]) for r in (queue.get(timeout=300) for _ in range(world)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rng = np.random.default_rng(77)
    a = dyadic_uniform(rng, (512, 384), 32)
    b = dyadic_uniform(rng, (384, 256), 32)
    a[300, 17] = np.nan
    mm_st, _ = oracle.matmul(a, b, fast=True)
    e = 5 * 8192 + 123
    p = dyadic_uniform(rng, e, 32)
    t = dyadic_uniform(rng, e, 32)
    sgd_st, sgd_out = oracle.sgd(p, t, 0.25)
    mse_st, mse_out = oracle.mse(p, t)
    for rank in range(world):
        mm_word, _, sgd_word, sgd_bits, mse_word, mean_bits, dev_words, dev_means, _ = got[rank]
        assert mm_word == mm_st
        assert sgd_word == sgd_st and mse_word == mse_st
        assert mean_bits == bits(mse_out)[0]
        assert dev_words == [mse_st, mse_st, mse_st, sgd_st], (rank, [hex(w) for w in dev_words])
        assert all(m == bits(mse_out)[0] for m in dev_means), rank
    sgd_all = np.concatenate([got[r][3] for r in range(world)])
    assert np.array_equal(sgd_all, bits(sgd_out))
    rider_all = np.concatenate([got[r][8] for r in range(world)])
    assert np.array_equal(rider_all, bits(sgd_out))


def _FUSED_CASES(world):
    return ((2048, 256, 1536, None), (256, 100, 96, None), (2048, 128, 1024, (1900, 5)),
            (1024 * world, 32, 8192, None))


def _fused_worker(rank, world, port, queue):
    """Row-sharded MatMul with the all-gather inside the kernel (peer stores into every rank's C)."""
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    shared = []
    try:
        sharded = importlib.import_module("fusion-pcu_b200.sharded")
        results = []
        # (m, k, n, fault): a TMA-path product (many 128-wide tiles), a small one (16x16 tiles),
        # a fault in a late rank's rows, and rows of 8 x 128 per rank x 8192 columns (512 tiles: the
        # last wave in half tiles, peer stores from both launches)
        for m, k, n, fault in _FUSED_CASES(world):
            rng = np.random.default_rng(m + k + n)
            a = dyadic_uniform(rng, (m, k), 32)
            b = dyadic_uniform(rng, (k, n), 32)
            if fault:
                a[fault] = np.nan
            rows = m // world
            r0 = rank * rows
            sh = sharded.PeerRows(m, n, torch.float32)
            shared.append(sh)
            sh.local.fill_(-7.0)
            torch.cuda.synchronize()
            dist.barrier()  # every rank's C is filled before any peer writes into it
            status = pcu.new_status()
            sharded.strict_matmul_rows_allgather(to_device(a[r0:r0 + rows]), to_device(b), r0, sh, status)
            sharded.all_reduce_min_status(status)
            torch.cuda.synchronize()
            results.append((status_word(status), bits(to_host(sh.local))))
        queue.put((rank, results))
    finally:
        for sh in shared:
            sh.close()
        dist.destroy_process_group()


def test_fused_rows_allgather_matches_one_device():
    import torch

    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(queue.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for case, (m, k, n, fault) in enumerate(_FUSED_CASES(world)):
        rng = np.random.default_rng(m + k + n)
        a = dyadic_uniform(rng, (m, k), 32)
        b = dyadic_uniform(rng, (k, n), 32)
        if fault:
            a[fault] = np.nan
        status = pcu.new_status()
        want = pcu.strict_matmul(to_device(a), to_device(b), status=status)
        torch.cuda.synchronize()
        want_word = status_word(status)
        for rank in range(world):
            word, c_bits = got[rank][case]
            assert word == want_word, (case, rank, hex(word), hex(want_word))
            if want_word == pcu.STATUS_OK:  # every rank holds the whole product
                assert np.array_equal(c_bits, bits(to_host(want))), (case, rank)


_RACE_CASE = (2048, 128, 1024, 10)  # m, k, n, back-to-back calls


def _race_worker(rank, world, port, queue):
    """Ten row-sharded calls in a row, each followed by a reader of C on the same stream; rank 0's
    reader first spins for about a millisecond, long enough for the other ranks' next call to
    finish its tiles.  Nothing but the library's own ordering keeps their stores out of rank 0's
    C until its reader is done."""
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    sh = None
    try:
        sharded = importlib.import_module("fusion-pcu_b200.sharded")
        m, k, n, calls = _RACE_CASE
        rows = m // world
        r0 = rank * rows
        b = to_device(dyadic_uniform(np.random.default_rng(900), (k, n), 32))
        lefts = [to_device(dyadic_uniform(np.random.default_rng(901 + i), (m, k), 32)[r0:r0 + rows])
                 for i in range(calls)]
        sh = sharded.PeerRows(m, n, torch.float32)
        status = pcu.new_status(calls)
        torch.cuda.synchronize()
        dist.barrier()
        snaps = []
        for i in range(calls):
            sharded.strict_matmul_rows_allgather(lefts[i], b, r0, sh, status[i:i + 1])
            sharded.all_reduce_min_status(status[i:i + 1])
            if rank == 0:
                torch.cuda._sleep(2_000_000)
            snaps.append(sh.local.clone())
        torch.cuda.synchronize()
        words = [int(w) & ((1 << 64) - 1) for w in status.cpu().tolist()]
        queue.put((rank, words, [bits(to_host(s)) for s in snaps]))
    finally:
        if sh is not None:
            sh.close()
        dist.destroy_process_group()


def test_fused_rows_allgather_readers_are_not_overwritten():
    import torch

    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_race_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict((r[0], r[1:]) for r in (queue.get(timeout=300) for _ in range(world)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    m, k, n, calls = _RACE_CASE
    b = to_device(dyadic_uniform(np.random.default_rng(900), (k, n), 32))
    for i in range(calls):
        a = to_device(dyadic_uniform(np.random.default_rng(901 + i), (m, k), 32))
        status = pcu.new_status()
        want = bits(to_host(pcu.strict_matmul(a, b, status=status)))
        torch.cuda.synchronize()
        assert status_word(status) == pcu.STATUS_OK
        for rank in range(world):
            words, snaps = got[rank]
            assert words[i] == pcu.STATUS_OK, (rank, i, hex(words[i]))
            assert np.array_equal(snaps[i], want), (rank, i)


def _mse_cases(world):
    """(width, p, t) cases for the device hand-off: clean, a NaN in the last segment, squares whose
    running sum overflows only once the carry from the earlier segments is added, and faults in
    the first and the last segment (the first one wins)."""
    e = 3 * 8192 + 515
    out = []
    for width in (32, 64):
        rng = np.random.default_rng(4000 + width)
        p, t = dyadic_uniform(rng, e, width), dyadic_uniform(rng, e, width)
        out.append((width, "clean", p, t))
        q = p.copy()
        q[e - 7] = np.nan
        out.append((width, "nan_last", q, t))
        # one huge square at the end of segment 0 and one at the start of segment 1: each is
        # finite, their sum is not, so rank 1's walk overflows on the carried sum
        sharded = importlib.import_module("fusion-pcu_b200.sharded")
        b1 = sharded.shard_bounds(e, 0, world, align=4)[1]
        big = 1.5e19 if width == 32 else 1e154
        q, r = p.copy(), t.copy()
        q[b1 - 1:b1 + 1] = big
        r[b1 - 1:b1 + 1] = 0
        out.append((width, "overflow_by_carry", q, r))
        q = p.copy()
        q[5] = np.inf
        q[e - 3] = np.nan
        out.append((width, "first_wins", q, t))
    return out


def _device_mse_worker(rank, world, port, queue):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    import datetime

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        sharded = importlib.import_module("fusion-pcu_b200.sharded")
        results = []
        for width, name, p, t in _mse_cases(world):
            e = p.size
            e0, e1 = sharded.shard_bounds(e, rank, world, align=4)
            mse = sharded.ShardedMse(to_device(p[e0:e1]), to_device(t[e0:e1]), e0, e)
            st = pcu.new_status()
            mean = mse.run(st)
            torch.cuda.synchronize()
            results.append((status_word(st), bits(to_host(mean).reshape(1))[0]))
            mse.close()
        queue.put((rank, results))
    finally:
        dist.destroy_process_group()


def test_device_mse_handoff_faults_match_one_device():
    import torch

    world = min(torch.cuda.device_count(), 4)
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_device_mse_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(queue.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for i, (width, name, p, t) in enumerate(_mse_cases(world)):
        st_o, out_o = oracle.mse(p, t)
        for rank in range(world):
            word, mean_bits = got[rank][i]
            assert word == st_o, (name, width, rank, oracle.decode(word), oracle.decode(st_o))
            if st_o == oracle.STATUS_OK:
                assert mean_bits == bits(out_o)[0], (name, width, rank)
