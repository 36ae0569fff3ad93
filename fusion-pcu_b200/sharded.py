"""Multi-GPU strict path: one process per GPU, torch.distributed (NCCL over NVLink) as plumbing.

Sharding never reorders a strict reduction:
  * MatMul: the rows of op(A) (so the rows of C) are split into contiguous blocks; every cell is
    computed by one GPU over its whole ordered K loop, then C is all-gathered.  K is never split,
    because a sum across GPUs would change the order of the additions.
  * SGD: contiguous element blocks; no exchange.
  * MSE: contiguous element segments.  The bandwidth-bound phase (squares and per-chunk maps)
    runs on every GPU at once; then the running sum is handed from rank r to rank r + 1 (one
    scalar per rank, in rank order), the last rank divides, and the mean is broadcast.
Faults: each rank's status word holds global event ordinals (the events of its block shifted
by the block's first event), and an all-reduce MIN over the unsigned words yields exactly the
one-device first fault (lowest event wins, as with the reference's atomicMin,
tensor/strict_matmul/strict_matmul.rs:253-256 in the Fusion-PCU checkout).

The exchange helpers (shard_bounds, rebase_status, all_reduce_min_status, ordered_handoff) work
on tensors of any device and with the gloo backend too, which is how the host logic is tested
without GPUs; the arithmetic itself is always the CUDA provider's.
"""
import importlib

import torch
import torch.distributed as dist

pcu = importlib.import_module("fusion-pcu_b200")

_SIGN = -(1 << 63)  # int64 bit pattern 0x8000000000000000


def shard_bounds(total, rank, world, align=1):
    """[start, end) of `rank`'s contiguous block of `total` items.  Blocks start at multiples of
    `align`, are as even as that allows, and follow rank order."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    units = -(-total // align)
    base, extra = divmod(units, world)
    start = (rank * base + min(rank, extra)) * align
    end = ((rank + 1) * base + min(rank + 1, extra)) * align
    return min(start, total), min(end, total)


def rebase_status(status, event_offset):
    """Shift the event of every faulted word in `status` (int64 storage of the unsigned words)
    by `event_offset`, in place, on the tensor's device (no host synchronisation)."""
    if event_offset:
        faulted = status != -1
        rebased = ((status >> 3) + int(event_offset)) * 8 + (status & 7)
        status.copy_(torch.where(faulted, rebased, status))
    return status


def all_reduce_min_status(status, group=None):
    """All-reduce MIN of unsigned status words.  Flipping the top bit maps unsigned order onto
    the signed order of the int64 storage, so the sentinel (all ones) stays the largest."""
    flipped = torch.bitwise_xor(status, _SIGN)
    dist.all_reduce(flipped, op=dist.ReduceOp.MIN, group=group)
    status.copy_(torch.bitwise_xor(flipped, _SIGN))
    return status


def _ranks(group):
    return dist.get_process_group_ranks(group) if group is not None else list(range(dist.get_world_size()))


def ordered_handoff(carry, step, group=None):
    """Run step(carry) on every rank in rank order: rank r receives the carry from rank r - 1,
    updates it in place and sends it on to rank r + 1.  Device work stays stream-ordered."""
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    ranks = _ranks(group)
    if rank > 0:
        dist.recv(carry, src=ranks[rank - 1], group=group)
    step(carry)
    if rank < world - 1:
        dist.send(carry, dst=ranks[rank + 1], group=group)
    return carry


# ------------------------------------------------------------------------------- MatMul
def matmul_event_offset(row0, columns, inner):
    """Events in front of output row row0: row0 * columns cells, 2 events per (cell, k)."""
    return row0 * columns * inner * 2


def strict_matmul_rows(left_rows, right, row0, out_local, status, gathered=None, transpose_right=False, policy=0,
                       workspace=None, stream=None, group=None):
    """Rows [row0, row0 + m) of C = A . op(B) from this rank's rows of A, with global fault
    events; when `gathered` (world * m rows) is given, C's row blocks are all-gathered into it."""
    pcu.strict_matmul(left_rows, right, False, transpose_right, policy, out=out_local, status=status,
                      workspace=workspace, stream=stream)
    rebase_status(status, matmul_event_offset(row0, out_local.shape[1], left_rows.shape[1]))
    if gathered is not None:
        dist.all_gather_into_tensor(gathered, out_local, group=group)
    return out_local


# ------------------------------------------------------------------------------- SGD
def strict_sgd_block(weights, gradient, rate, first_index, status, out=None, policy=0, stream=None):
    """SGD on this rank's element block [first_index, first_index + n) with global events."""
    out = pcu.strict_sgd(weights, gradient, rate, policy, out=out, status=status, stream=stream)
    rebase_status(status, 2 * first_index)
    return out


# ------------------------------------------------------------------------------- MSE
class ShardedMse:
    """Strict MSE over a tensor split into contiguous segments, one per rank (ordered hand-off).

    prediction/target: this rank's segment, the global elements [first_index, first_index + n)
    of `total`.  run() returns the mean (a device scalar, the same on every rank) and leaves the
    all-reduced first fault in `status`."""

    def __init__(self, prediction, target, first_index, total, policy=0, group=None):
        self.p, self.t = prediction, target
        self.first, self.total, self.policy, self.group = first_index, total, policy, group
        self.workspace = pcu.mse_workspace(prediction)
        self.carry = torch.zeros(1, dtype=prediction.dtype, device=prediction.device)
        self.mean = torch.zeros(1, dtype=prediction.dtype, device=prediction.device)
        self.last = first_index + prediction.numel() == total

    def run(self, status, stream=None, reduce_status=True):
        pcu.strict_mse_segment_prepare(self.p, self.t, self.first, self.policy, status=status,
                                       workspace=self.workspace, stream=stream)
        self.carry.zero_()

        def walk(carry):
            pcu.strict_mse_segment_walk(self.p, self.t, self.first, self.total, carry, self.workspace, status,
                                        self.policy, out=self.mean if self.last else None, stream=stream)

        ordered_handoff(self.carry, walk, self.group)
        dist.broadcast(self.mean, src=_ranks(self.group)[-1], group=self.group)
        if reduce_status:
            all_reduce_min_status(status, self.group)
        return self.mean.reshape(())
