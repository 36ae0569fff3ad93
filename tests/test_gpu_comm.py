"""The C ABI's own communicator (pcu_b200_comm_*, fusion-pcu_b200/comm.py) on 2+ B200s.

Every rank runs the split paths through the communicator alone (no torch.distributed):
* the unsigned status MIN, a send/recv pair and a broadcast;
* the row-sharded MatMul with the all-gather in the kernel, into peer buffers exchanged by the
  communicator, on the generic and the TMA kernel, F32 and F64, with first faults on either side;
* the split strict MSE with its ordered hand-off, ragged cuts, first faults on either side.
Every rank's C, mean and status word must equal the one-device call (and, for the MSE, the
oracle) bit for bit.  Skipped with fewer than 2 GPUs.
"""
import importlib
import traceback

import numpy as np
import pytest

import oracle
from gpu_util import bits, dyadic_uniform, status_word, to_device, to_host

pytestmark = pytest.mark.gpu

OK = (1 << 64) - 1
# (rows, inner, columns, width, NaN position in A or None)
MM_CASES = [(512, 256, 384, 32, None), (512, 256, 384, 32, (400, 7)), (256, 64, 96, 64, None),
            (2048, 128, 1536, 32, None), (2048, 128, 1536, 32, (100, 3)), (1024, 96, 640, 64, (1000, 50))]
# (elements, width, NaN position in the target or None)
# (the last case is shorter than the cuts' 12345-element shift, so every rank after the first gets
# an empty segment, whatever the number of ranks)
MSE_CASES = [((1 << 20) + 7, 32, None), ((1 << 20) + 7, 32, 900000), (300001, 64, 1000), (70000, 64, None),
             (10000, 32, 4000)]


def _cuts(n, world):
    return [0] + [min(n, n * r // world + 12345 * r) for r in range(1, world)] + [n]


def _mm_inputs(case):
    m, k, n, width, fault = MM_CASES[case]
    rng = np.random.default_rng(m + k + n + width)
    a = dyadic_uniform(rng, (m, k), width)
    b = dyadic_uniform(rng, (k, n), width)
    if fault:
        a[fault] = np.nan
    return a, b


def _mse_inputs(case):
    n, width, fault = MSE_CASES[case]
    rng = np.random.default_rng(n + width)
    p = dyadic_uniform(rng, n, width)
    t = dyadic_uniform(rng, n, width, low=0.0)
    if fault is not None:
        t[fault] = np.nan
    return p, t


def _worker(rank, world, uid_queue, queue):
    try:
        import torch

        torch.cuda.set_device(rank)
        cm = importlib.import_module("fusion-pcu_b200.comm")
        pcu = importlib.import_module("fusion-pcu_b200")
        if rank == 0:
            uid = cm.Communicator.unique_id()
            for _ in range(world - 1):
                uid_queue.put(uid)
        else:
            uid = uid_queue.get(timeout=120)
        comm = cm.Communicator(uid, world, rank)
        res = {}
        words = np.array([OK, (1 << 63) | 0x15, ((rank + 3) << 3) | 3, OK if rank else (9 << 3) | 5], dtype=np.uint64)
        st = torch.from_numpy(words.view(np.int64).copy()).cuda()
        comm.status_min(st)
        x = torch.full((4,), float(rank + 1), dtype=torch.float64, device="cuda")
        if rank == 0:
            comm.send(x, 1)
        elif rank == 1:
            comm.recv(x, 0)
        comm.broadcast(x, 1)
        torch.cuda.synchronize()
        res["min"] = st.cpu().numpy().view(np.uint64).copy()
        res["bcast"] = x.cpu().numpy()
        for case in range(len(MM_CASES)):
            a, b = _mm_inputs(case)
            m, n = a.shape[0], b.shape[1]
            r0, r1 = rank * m // world, (rank + 1) * m // world
            ad, bd = to_device(a[r0:r1]), to_device(b)
            shared = comm.peer_matrix(m, n, ad.dtype)
            status = pcu.new_status()
            comm.strict_matmul_rows(ad, bd, r0, shared, status)
            torch.cuda.synchronize()
            res[("mm", case)] = (status_word(status), bits(to_host(shared.local)).copy())
            shared.close()
        for case in range(len(MSE_CASES)):
            p, t = _mse_inputs(case)
            c = _cuts(p.size, world)
            pd, td = to_device(p[c[rank]:c[rank + 1]]), to_device(t[c[rank]:c[rank + 1]])
            out = torch.zeros((), dtype=pd.dtype, device="cuda")
            status = pcu.new_status()
            comm.strict_mse(pd, td, c[rank], p.size, out, status)
            torch.cuda.synchronize()
            res[("mse", case)] = (status_word(status), int(bits(to_host(out).reshape(1))[0]))
        comm.close()
        # a second communicator, torn down with abort (the path a host takes after a failed peer)
        if rank == 0:
            uid = cm.Communicator.unique_id()
            for _ in range(world - 1):
                uid_queue.put(uid)
        else:
            uid = uid_queue.get(timeout=120)
        cm.Communicator(uid, world, rank).abort()
        queue.put((rank, res))
    except Exception:
        queue.put((rank, traceback.format_exc()))


def test_communicator_split_paths_match_one_device():
    import torch

    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    uid_queue, queue = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, uid_queue, queue)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    try:
        # a rank that fails reports its traceback at once; the others may then wait for it in a
        # collective, so stop at the first failure instead of waiting for every rank
        while len(got) < world:
            rank, res = queue.get(timeout=300)
            got[rank] = res
            assert isinstance(res, dict), f"rank {rank} failed:\n{res}"
    finally:
        for p in procs:
            p.join(timeout=60 if len(got) == world else 1)
            if p.exitcode is None:
                p.kill()
    pcu = importlib.import_module("fusion-pcu_b200")
    for rank in range(world):
        assert list(got[rank]["min"]) == [OK, (1 << 63) | 0x15, (3 << 3) | 3, (9 << 3) | 5]
        assert np.all(got[rank]["bcast"] == 1.0)
    for case in range(len(MM_CASES)):
        a, b = _mm_inputs(case)
        status = pcu.new_status()
        want = pcu.strict_matmul(to_device(a), to_device(b), status=status)
        want_bits, want_word = bits(to_host(want)), status_word(status)
        assert (want_word != OK) == (MM_CASES[case][4] is not None)
        for rank in range(world):
            word, c_bits = got[rank][("mm", case)]
            assert word == want_word, (case, rank, hex(word), hex(want_word))
            if want_word == OK:
                assert np.array_equal(c_bits, want_bits), (case, rank)
    for case in range(len(MSE_CASES)):
        p, t = _mse_inputs(case)
        status = pcu.new_status()
        mean = pcu.strict_mse(to_device(p), to_device(t), status=status)
        want_word, want_bits = status_word(status), int(bits(to_host(mean).reshape(1))[0])
        st_o, out_o = oracle.mse(p, t)
        assert want_word == st_o
        for rank in range(world):
            word, out_bits = got[rank][("mse", case)]
            assert word == want_word, (case, rank, hex(word), hex(want_word))
            if want_word == OK:
                assert out_bits == want_bits == int(bits(out_o)[0]), (case, rank)


def test_one_rank_communicator_matches_one_device():
    """A communicator of one rank (runs on one GPU): NCCL loaded at run time, the status MIN and
    broadcast as identities, the peer-buffer exchange with no peers, the row-sharded MatMul as the
    whole product and the split MSE as one segment, then abort."""
    import torch

    cm = importlib.import_module("fusion-pcu_b200.comm")
    pcu = importlib.import_module("fusion-pcu_b200")
    comm = cm.Communicator(cm.Communicator.unique_id(), 1, 0)
    try:
        words = np.array([OK, (7 << 3) | 4], dtype=np.uint64)
        st = torch.from_numpy(words.view(np.int64).copy()).cuda()
        comm.status_min(st)
        x = torch.arange(5, dtype=torch.float64, device="cuda")
        comm.broadcast(x, 0)
        torch.cuda.synchronize()
        assert list(st.cpu().numpy().view(np.uint64)) == list(words)
        assert np.array_equal(to_host(x), np.arange(5.0))
        for case in (0, 1, 3, 5):
            a, b = _mm_inputs(case)
            ad, bd = to_device(a), to_device(b)
            shared = comm.peer_matrix(a.shape[0], b.shape[1], ad.dtype)
            status = pcu.new_status()
            comm.strict_matmul_rows(ad, bd, 0, shared, status)
            want_status = pcu.new_status()
            want = pcu.strict_matmul(ad, bd, status=want_status)
            torch.cuda.synchronize()
            assert status_word(status) == status_word(want_status), case
            if status_word(status) == OK:
                assert np.array_equal(bits(to_host(shared.local)), bits(to_host(want))), case
            shared.close()
        for case in range(len(MSE_CASES)):
            p, t = _mse_inputs(case)
            pd, td = to_device(p), to_device(t)
            out = torch.zeros((), dtype=pd.dtype, device="cuda")
            status = pcu.new_status()
            comm.strict_mse(pd, td, 0, p.size, out, status)
            torch.cuda.synchronize()
            st_o, out_o = oracle.mse(p, t)
            assert status_word(status) == st_o, case
            if st_o == OK:
                assert int(bits(to_host(out).reshape(1))[0]) == int(bits(out_o)[0]), case
    finally:
        comm.abort()
