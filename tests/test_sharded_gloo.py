"""Host logic of the multi-GPU strict path, on CPU ranks over gloo (no GPU).

fusion-pcu_b200/sharded.py shards MatMul rows, SGD elements and MSE segments across ranks and
recombines the per-rank fault words into the one-device first fault.  Here each rank computes
its block with the CPU oracle (test infrastructure standing in for the device kernels, which
the GPU tests cover) and the real exchange helpers do the rest; the recombined result must be
the oracle's single-pass result bit for bit: same value, same first fault.
"""
import importlib
import os
import socket

import numpy as np
import pytest

import oracle

sharded = importlib.import_module("fusion-pcu_b200.sharded")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_bounds_cover_in_order():
    for total in (0, 1, 7, 64, 1000, 8192):
        for world in (1, 2, 3, 8):
            for align in (1, 4, 128):
                spans = [sharded.shard_bounds(total, r, world, align) for r in range(world)]
                assert spans[0][0] == 0 and spans[-1][1] == total
                for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                    assert a1 == b0 and a0 <= a1
                assert all(s % align == 0 or s == total for s, _ in spans)
                units = [-(-(e - s) // align) for s, e in spans]  # the last block may be partial
                assert max(units) - min(units) <= 1


def test_rebase_status_keeps_the_sentinel():
    import torch

    words = torch.tensor([-1, (5 << 3) | 3, (0 << 3) | 5], dtype=torch.int64)
    sharded.rebase_status(words, 100)
    assert words.tolist() == [-1, (105 << 3) | 3, (100 << 3) | 5]


# ---------------------------------------------------------------------------- rank programs
def _matmul_cases():
    rng = np.random.default_rng(5)
    m, k, n = 12, 9, 7
    a = (rng.integers(-(1 << 23), 1 << 23, (m, k)) * 2.0 ** -23).astype(np.float32)
    b = (rng.integers(-(1 << 23), 1 << 23, (k, n)) * 2.0 ** -23).astype(np.float32)
    cases = [(a, b)]
    for spots in ([(9, 4)], [(1, 7), (10, 0)], [(11, 8)]):
        a2 = a.copy()
        for r, c in spots:
            a2[r, c] = np.nan
        cases.append((a2, b))
    a3 = a.copy()
    a3[6, :] = 3e38  # overflow on the Add of a later cell
    cases.append((a3, b))
    return cases


def _mse_cases():
    rng = np.random.default_rng(9)
    n = 301
    p = (rng.integers(-(1 << 23), 1 << 23, n) * 2.0 ** -23).astype(np.float32)
    t = (rng.integers(-(1 << 23), 1 << 23, n) * 2.0 ** -23).astype(np.float32)
    cases = [(p, t)]
    p2 = p.copy(); p2[250] = np.inf
    cases.append((p2, t))
    p3 = p.copy(); p3[40] = np.nan; p3[260] = np.inf
    cases.append((p3, t))
    big = np.full(n, 1.5e19, np.float32)  # squares 2.25e38: the running sum overflows at element 1
    cases.append((big, np.zeros(n, np.float32)))
    late = p.copy(); late[140:] = 1.5e19  # overflow driven by the carry across a segment edge
    cases.append((late, t))
    return cases


def _rank_program(rank, world):
    import torch

    out = {"matmul": [], "sgd": [], "mse": []}
    for a, b in _matmul_cases():
        r0, r1 = sharded.shard_bounds(a.shape[0], rank, world)
        st, _ = oracle.matmul(a[r0:r1], b)
        word = torch.tensor([np.uint64(st).astype(np.int64)], dtype=torch.int64)
        sharded.rebase_status(word, sharded.matmul_event_offset(r0, b.shape[1], a.shape[1]))
        sharded.all_reduce_min_status(word)
        out["matmul"].append(int(word.item()) & ((1 << 64) - 1))
    for p, t in _mse_cases():
        # SGD over the same elements (weights p, gradient t, rate 0.5)
        e0, e1 = sharded.shard_bounds(p.size, rank, world, align=4)
        st, _ = oracle.sgd(p[e0:e1], t[e0:e1], 0.5)
        word = torch.tensor([np.uint64(st).astype(np.int64)], dtype=torch.int64)
        sharded.rebase_status(word, 2 * e0)
        sharded.all_reduce_min_status(word)
        out["sgd"].append(int(word.item()) & ((1 << 64) - 1))
        # MSE: ordered hand-off of the running sum's bits, last rank divides, mean broadcast
        carry = torch.zeros(1, dtype=torch.int64)
        status = torch.full((1,), -1, dtype=torch.int64)
        mean = torch.zeros(1, dtype=torch.int64)
        last = e1 == p.size

        def walk(c):
            st, bits, m = oracle.mse_segment(p[e0:e1], t[e0:e1], e0, p.size, int(c.item()), last=last)
            if st != oracle.STATUS_OK:
                status.fill_(int(np.uint64(st).astype(np.int64)))
            c.fill_(bits)
            if last and m is not None and st == oracle.STATUS_OK:
                mean.fill_(int(m.view(np.uint32)[0]))

        sharded.ordered_handoff(carry, walk)
        import torch.distributed as dist

        dist.broadcast(mean, src=world - 1)
        sharded.all_reduce_min_status(status)
        out["mse"].append((int(status.item()) & ((1 << 64) - 1), int(mean.item())))
    return out


def _worker(rank, world, port, queue):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        queue.put((rank, _rank_program(rank, world)))
    finally:
        dist.destroy_process_group()


def _expected():
    exp = {"matmul": [], "sgd": [], "mse": []}
    for a, b in _matmul_cases():
        exp["matmul"].append(oracle.matmul(a, b)[0])
    for p, t in _mse_cases():
        exp["sgd"].append(oracle.sgd(p, t, 0.5)[0])
        st, out = oracle.mse(p, t)
        exp["mse"].append((st, int(out.view(np.uint32)[0]) if st == oracle.STATUS_OK else 0))
    return exp


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_faults_and_mse_handoff_match_one_pass(world):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    exp = _expected()
    # the cases must exercise faults in several blocks, and a clean run
    assert any(s == oracle.STATUS_OK for s in exp["matmul"]) and any(s != oracle.STATUS_OK for s in exp["matmul"])
    assert len({s for s, _ in exp["mse"]}) >= 4
    for rank in range(world):
        assert results[rank]["matmul"] == exp["matmul"], rank
        assert results[rank]["sgd"] == exp["sgd"], rank
        assert results[rank]["mse"] == exp["mse"], rank


def _lost_rank_worker(rank, world, port, queue):
    """Rank 1 leaves before the MSE hand-off (an exception between steps); the others must end with
    an error from their next exchange within the process group's short timeout, not hang."""
    import datetime

    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    import time

    t0 = time.time()
    try:
        if rank == 1:
            raise RuntimeError("rank 1 lost")
        carry = torch.zeros(1, dtype=torch.int64)
        sharded.ordered_handoff(carry, lambda c: c.add_(1))
        mean = torch.zeros(1, dtype=torch.int64)
        dist.broadcast(mean, src=world - 1)
        status = torch.full((1,), -1, dtype=torch.int64)
        sharded.all_reduce_min_status(status)
        queue.put((rank, "completed", time.time() - t0))
    except RuntimeError as e:
        queue.put((rank, "error" if rank != 1 else "lost", time.time() - t0))
        del e
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001 - the group is already broken
            pass


def test_lost_rank_ends_the_handoff_with_an_error():
    import torch.multiprocessing as mp

    world = 3
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_lost_rank_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict((r, (what, dt)) for r, what, dt in (queue.get(timeout=120) for _ in range(world)))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert results[1][0] == "lost"
    for rank in (0, 2):
        what, dt = results[rank]
        assert what == "error", (rank, what)
        assert dt < 60, (rank, dt)


# ------------------------------------------------------------------ peer buffer set-up
class _FakePeerLibrary:
    """Stands in for libpcu_b200.so's IPC entry points on CPU ranks: a buffer is an address, its
    handle carries the address, and a mapping is the address plus an offset.  `fail_alloc` and
    `fail_open` name the ranks whose allocation or mapping returns an error code."""

    def __init__(self, rank, fail_alloc=(), fail_open=()):
        self.rank, self.fail_alloc, self.fail_open = rank, set(fail_alloc), set(fail_open)
        self.live, self.mapped = set(), set()

    def pcu_b200_peer_alloc(self, nbytes, pptr, handle):
        if self.rank in self.fail_alloc:
            return 2
        addr = 0x10000 * (self.rank + 1)
        pptr._obj.value = addr
        for i, b in enumerate(addr.to_bytes(8, "little")):
            handle[i] = b
        self.live.add(addr)
        return 0

    def pcu_b200_peer_open(self, handle, pptr):
        if self.rank in self.fail_open:
            return 2
        addr = int.from_bytes(bytes(handle)[:8], "little") + 0x100 * (self.rank + 1)
        pptr._obj.value = addr
        self.mapped.add(addr)
        return 0

    def pcu_b200_peer_close(self, ptr):
        self.mapped.discard(ptr)
        return 0

    def pcu_b200_peer_free(self, ptr):
        self.live.discard(ptr)
        return 0

    def pcu_b200_error_string(self, rc):
        return b"CUDA runtime failure"


def _peer_buffer_worker(rank, world, port, queue):
    """Three set-ups in a row on the same ranks: all succeed; one rank cannot allocate; one rank
    cannot map a peer's buffer.  Each rank reports what it returned or raised and what it still
    holds."""
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    out = []
    for fail_alloc, fail_open in (((), ()), ((1,), ()), ((), (0,))):
        fake = _FakePeerLibrary(rank, fail_alloc, fail_open)
        sharded.pcu.library = lambda fake=fake: fake
        try:
            own, ptrs = sharded._map_peer_buffer(64, None)
            out.append(("ok", own, ptrs, sorted(fake.live), sorted(fake.mapped)))
        except sharded.pcu.ProviderFailure as e:
            out.append(("raised", str(e), None, sorted(fake.live), sorted(fake.mapped)))
    dist.destroy_process_group()
    queue.put((rank, out))


def test_peer_buffer_setup_fails_on_every_rank_together():
    """sharded._map_peer_buffer is collective even when it fails: a rank that cannot allocate its
    buffer, or cannot map a peer's, makes every rank release what it holds and raise the same
    error, instead of leaving the others waiting in a later collective."""
    import torch.multiprocessing as mp

    world = 3
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_buffer_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in range(world):
        ok, alloc_fail, open_fail = results[rank]
        # all succeed: this rank's own buffer, every peer's mapped at its own address
        assert ok[0] == "ok"
        own = 0x10000 * (rank + 1)
        assert ok[1] == own and ok[2][rank] == own
        peers = [0x10000 * (r + 1) + 0x100 * (rank + 1) for r in range(world) if r != rank]
        assert [q for r, q in enumerate(ok[2]) if r != rank] == peers
        assert ok[3] == [own] and ok[4] == peers
        # rank 1 cannot allocate: every rank raises naming it and holds nothing
        assert alloc_fail[0] == "raised" and "rank 1 could not allocate" in alloc_fail[1], alloc_fail
        assert alloc_fail[3] == [] and alloc_fail[4] == []
        # rank 0 cannot map: every rank raises naming it, unmaps and frees
        assert open_fail[0] == "raised" and "rank 0 could not map" in open_fail[1], open_fail
        assert open_fail[3] == [] and open_fail[4] == []
