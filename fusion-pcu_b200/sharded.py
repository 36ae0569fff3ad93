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

import numpy as np
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


def strict_matmul_rows_host(left_rows, right_rows, k0, right_device, out_rows, status, scratch=None, stream=None,
                            group=None, policy=0):
    """The row-sharded product end to end from host memory: this rank's rows of A (host,
    left_rows) and its slice of B's rows [k0, k0 + len) (host, right_rows) go up, the slices are
    all-gathered over NVLink into `right_device` (the whole of B on every rank), and the rank's
    rows of C come back to `out_rows` (host) with its status word (rank-local events) in `status`
    (a host int64 tensor).  Every rank uploads its own slice of B only, so the PCIe traffic of the
    whole job is A + B in and C out, each once.  B's row count must divide evenly by the ranks."""
    k1 = k0 + right_rows.shape[0]
    right_device[k0:k1].copy_(right_rows, non_blocking=True)
    dist.all_gather_into_tensor(right_device, right_device[k0:k1], group=group)
    return pcu.strict_matmul_host_left(left_rows, right_device, policy, out=out_rows, status=status, scratch=scratch,
                                       stream=stream)


# ------------------------------------------------------------------------------- SGD
def strict_sgd_block(weights, gradient, rate, first_index, status, out=None, policy=0, stream=None):
    """SGD on this rank's element block [first_index, first_index + n) with global events."""
    out = pcu.strict_sgd(weights, gradient, rate, policy, out=out, status=status, stream=stream)
    rebase_status(status, 2 * first_index)
    return out


class _CudaArray:
    """A view of raw device memory that torch.as_tensor accepts (__cuda_array_interface__)."""

    def __init__(self, ptr, shape, dtype):
        typestr = {torch.float32: "<f4", torch.float64: "<f8"}[dtype]
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3}


def _raise_collective(what, failed):
    """Raise the same ProviderFailure on every rank: the first rank in `failed` ((rank, code) pairs,
    as every rank received them) could not do `what`."""
    r, code = failed[0]
    msg = pcu.library().pcu_b200_error_string(code).decode()
    raise pcu.ProviderFailure(f"rank {r} could not {what}: pcu_b200 error {code}: {msg}")


def _map_peer_buffer(nbytes, group):
    """Allocate `nbytes` of zero-filled device memory with an IPC handle on every rank and map every
    peer's: (this rank's pointer, every rank's pointer in rank order as this process sees it).

    Collective even when it fails.  Every rank takes part in both exchanges (the handles, then
    whether each rank mapped every peer's buffer).  If any rank could not allocate its buffer or
    map a peer's, every rank releases what it holds and raises the same ProviderFailure, so no
    rank is left waiting in a later collective for one that gave up."""
    import ctypes

    L = pcu.library()
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    ptr, handle = ctypes.c_void_p(), (ctypes.c_ubyte * 64)()
    rc = L.pcu_b200_peer_alloc(nbytes, ctypes.byref(ptr), handle)
    entries = [None] * world
    dist.all_gather_object(entries, (rc, bytes(handle)), group=group)
    failed = [(r, code) for r, (code, _) in enumerate(entries) if code != 0]
    if failed:
        if rc == 0:
            L.pcu_b200_peer_free(ptr.value)  # no peer has mapped it
        _raise_collective("allocate its peer buffer", failed)
    ptrs, rc = [], 0
    for r, (_, h) in enumerate(entries):
        if r == rank:
            ptrs.append(ptr.value)
            continue
        q = ctypes.c_void_p()
        if rc == 0:
            rc = L.pcu_b200_peer_open((ctypes.c_ubyte * 64).from_buffer_copy(h), ctypes.byref(q))
        ptrs.append(q.value if rc == 0 else None)
    codes = [None] * world
    dist.all_gather_object(codes, rc, group=group)
    failed = [(r, code) for r, code in enumerate(codes) if code != 0]
    if failed:
        for r, q in enumerate(ptrs):
            if r != rank and q:
                L.pcu_b200_peer_close(q)
        dist.barrier(group=group)  # no rank still maps this rank's buffer when it is freed
        L.pcu_b200_peer_free(ptr.value)
        _raise_collective("map a peer's buffer", failed)
    return ptr.value, ptrs


def _unmap_peer_buffer(own, ptrs, group):
    """Unmap the peers' buffers, wait for every rank to do the same, free this rank's own."""
    L = pcu.library()
    dist.barrier(group=group)
    for q in ptrs:
        if q != own:
            L.pcu_b200_peer_close(q)
    dist.barrier(group=group)
    L.pcu_b200_peer_free(own)


class PeerRows:
    """A rows x columns matrix of which every rank holds a copy that all ranks write into (CUDA IPC,
    pcu_b200_peer_alloc / _open): the destination of the fused row-sharded MatMul + all-gather.
    `local` is this rank's copy (a torch view); `peer_ptrs` the peers' copies mapped here, in rank
    order without this rank.  Only the provider's own kernels touch the peer copies.  `calls`
    numbers the MatMuls made into this matrix (the same on every rank): the kernel stores into a
    peer's copy only once that peer has entered the same call."""

    def __init__(self, rows, columns, dtype=torch.float32, group=None):
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        L = pcu.library()
        code = 0 if dtype == torch.float32 else 1
        self._ptr, ptrs = _map_peer_buffer(L.pcu_b200_peer_rows_bytes(code, rows, columns), group)
        self.calls = 0
        self.peer_ptrs = [q for r, q in enumerate(ptrs) if r != self.rank]
        self.rows, self.columns, self.dtype = rows, columns, dtype
        self.local = torch.as_tensor(_CudaArray(self._ptr, (rows, columns), dtype), device="cuda")

    def close(self):
        """Unmap the peers' copies and free this one (every rank, after its last use)."""
        L = pcu.library()
        dist.barrier(group=self.group)
        for q in self.peer_ptrs:
            L.pcu_b200_peer_close(q)
        self.peer_ptrs = []
        dist.barrier(group=self.group)
        if self._ptr:
            L.pcu_b200_peer_free(self._ptr)
            self._ptr = None


def strict_matmul_rows_allgather(left_rows, right, row0, shared, status, transpose_right=False, policy=0,
                                 workspace=None, stream=None):
    """Rows [row0, row0 + m) of C = A . op(B) in one kernel with their all-gather: written into
    `shared.local` and every peer's copy (PeerRows), events global.

    Ordering: follow with a collective (all_reduce_min_status) before reading C; it orders every
    rank's stores before the read.  The other direction needs nothing from the caller as long as
    every reader of C runs on `stream` (or is joined into it) before the next call: the kernel
    stores into a peer's C only after that peer's kernel of the same call has started."""
    import ctypes

    L = pcu.library()
    rows, inner = left_rows.shape
    cols = right.shape[0] if transpose_right else right.shape[1]
    if workspace is None:
        workspace = torch.empty(max(L.pcu_b200_strict_matmul_workspace_size(rows, inner, cols), 1), dtype=torch.uint8,
                                device=left_rows.device)
    peers = (ctypes.c_void_p * max(len(shared.peer_ptrs), 1))(*shared.peer_ptrs)
    pcu._check(L.pcu_b200_strict_matmul_rows_allgather(
        pcu._dtype_code(left_rows), policy, pcu._ptr(left_rows), pcu._ptr(right), ctypes.c_void_p(shared._ptr), row0,
        rows, shared.rows, inner, cols, left_rows.stride(0), right.stride(0), int(transpose_right), peers,
        len(shared.peer_ptrs), shared.rank, shared.calls + 1, pcu._ptr(workspace), workspace.numel(),
        pcu._ptr(status), pcu._stream(stream)))
    shared.calls += 1
    return shared.local


# ------------------------------------------------------------------------------- MSE
class ShardedMse:
    """Strict MSE over a tensor split into contiguous segments, one per rank (ordered hand-off).

    prediction/target: this rank's segment, the global elements [first_index, first_index + n)
    of `total`.  run() returns the mean (a device scalar, the same on every rank) and leaves the
    global first fault in `status`.

    handoff="device" (the default on GPUs): pcu_b200_strict_mse_sgd_split -- every rank's segment
    is one launch whose walker takes the running sum from rank r - 1 and hands its own to rank
    r + 1 through IPC-mapped hand-off blocks, and a one-warp exchange leaves the MIN of the status
    words and the mean on every rank; no NCCL call and no host round trip.  handoff="nccl": the
    same hand-off with torch.distributed send/recv, broadcast and all-reduce (any backend)."""

    def __init__(self, prediction, target, first_index, total, policy=0, group=None, handoff="device"):
        self.p, self.t = prediction, target
        self.first, self.total, self.policy, self.group = first_index, total, policy, group
        self.workspace = pcu.mse_workspace(prediction)
        self.carry = torch.zeros(1, dtype=prediction.dtype, device=prediction.device)
        self.mean = torch.zeros(1, dtype=prediction.dtype, device=prediction.device)
        self.last = first_index + prediction.numel() == total
        self.handoff = handoff
        self.calls = 0
        if handoff == "device":
            self._own, self._blocks = _map_peer_buffer(pcu.library().pcu_b200_mse_handoff_bytes(), group)

    def close(self):
        """Release the hand-off blocks (every rank, after its last call)."""
        if self.handoff == "device" and self._own:
            _unmap_peer_buffer(self._own, self._blocks, self.group)
            self._own = None

    def _run_device(self, status, stream, sgd):
        import ctypes

        L = pcu.library()
        rank, world = dist.get_rank(self.group), dist.get_world_size(self.group)
        blocks = (ctypes.c_void_p * world)(*self._blocks)
        if sgd is None:
            sgd_args = (None, None, None, 0, 0, 0, None)
        else:
            rate_bits = int(np.array([sgd["rate"]], dtype=np.float32).view(np.uint32)[0])
            sgd_args = (pcu._ptr(sgd["weights"]), pcu._ptr(sgd["gradient"]), pcu._ptr(sgd["out"]),
                        sgd["weights"].numel(), sgd["first_index"], rate_bits, pcu._ptr(sgd["status"]))
        pcu._check(L.pcu_b200_strict_mse_sgd_split(
            pcu._dtype_code(self.p), self.policy, pcu._ptr(self.p), pcu._ptr(self.t), self.p.numel(), self.first,
            self.total, pcu._ptr(self.mean), pcu._ptr(self.workspace), self.workspace.numel(), pcu._ptr(status),
            *sgd_args, blocks, rank, world, self.calls + 1, pcu._stream(stream)))
        self.calls += 1
        return self.mean.reshape(())

    def run(self, status, stream=None, reduce_status=True, sgd=None):
        """`sgd`: optionally an independent strict SGD block carried by the bandwidth-bound phase,
        a dict with weights, gradient, rate, first_index (its global first element), out and
        status (its own word, global events; MIN-reduced with the MSE's in the device hand-off,
        left to the caller in the NCCL one).

        The first segment's running sum starts at +0, so its rank walks at once, in the same
        launch as its maps; the others build their maps at once and walk when the carry arrives."""
        if self.handoff == "device":
            return self._run_device(status, stream, sgd)
        first = dist.get_rank(self.group) == 0
        if first:
            pcu.strict_mse_sgd_segment(self.p, self.t, self.first, self.total, None, self.carry, self.workspace, status,
                                       self.policy, out=self.mean if self.last else None, sgd=sgd, stream=stream)
        elif sgd is None:
            pcu.strict_mse_segment_prepare(self.p, self.t, self.first, self.policy, status=status,
                                           workspace=self.workspace, stream=stream)
        else:
            pcu.strict_mse_sgd_segment_prepare(self.p, self.t, self.first, sgd["weights"], sgd["gradient"],
                                               sgd["rate"], sgd["first_index"], self.policy, updated=sgd["out"],
                                               mse_status=status, sgd_status=sgd["status"],
                                               workspace=self.workspace, stream=stream)

        def walk(carry):
            if not first:
                pcu.strict_mse_segment_walk(self.p, self.t, self.first, self.total, carry, self.workspace, status,
                                            self.policy, out=self.mean if self.last else None, stream=stream)

        ordered_handoff(self.carry, walk, self.group)
        dist.broadcast(self.mean, src=_ranks(self.group)[-1], group=self.group)
        if reduce_status:
            all_reduce_min_status(status, self.group)
        return self.mean.reshape(())


# ------------------------------------------------------------------------------- MLP
def gather_columns(shard, full, group=None):
    """All-gather the column blocks of a row-major (rows x n_r) tensor into `full` (rows x
    world * n_r): NCCL gathers whole blocks, a strided copy interleaves them."""
    world = dist.get_world_size(group)
    rows, n_r = shard.shape
    blocks = torch.empty((world, rows, n_r), dtype=shard.dtype, device=shard.device)
    dist.all_gather_into_tensor(blocks, shard.contiguous(), group=group)
    full.view(rows, world, n_r).copy_(blocks.permute(1, 0, 2))
    return full


class ColumnShardedMlp:
    """A strict MLP training step with every weight's output columns split over the ranks.

    Layers dims[0] -> ... -> dims[-1], ReLU after all but the last, strict MSE against the
    target, the reverse mode of the strict graph layer (MSE gradient (p - t) * 2/n, ReLU
    backward, dW = H^T G, dH = G W^T) and strict SGD.  Rank r owns columns [c0, c1) of every
    weight and computes those columns of every activation and gradient; each cell still runs
    its whole ordered reduction on one GPU, so the results are bit for bit those of one device.
    Exchanges: the activations (forward), the output gradients and the weights (backward, for
    dH = G W^T) are all-gathered.  Every dims[k >= 1] must be a multiple of the world size.
    Status words (one per kernel call, rank-local event ordinals) stay in `self.status`.
    """

    def __init__(self, dims, batch, rate, dtype=None, policy=0, group=None, device=None):
        self.dims, self.batch, self.rate, self.policy, self.group = list(dims), batch, rate, policy, group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.dtype = dtype or torch.float32
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        for d in self.dims[1:]:
            if d % self.world:
                raise ValueError(f"layer width {d} is not a multiple of {self.world} ranks")
        self.cols = [(self.rank * d // self.world, (self.rank + 1) * d // self.world) for d in self.dims]
        self.status = pcu.new_status(8 * len(dims) + 4, device=self.device)
        self._next = 0

    def _st(self):
        s = self.status[self._next:self._next + 1]
        self._next += 1
        return s

    def load(self, x, weights, target):
        """Full host or device tensors; each rank keeps its column blocks of the weights."""
        to = lambda a: torch.as_tensor(a).to(device=self.device, dtype=self.dtype)  # noqa: E731
        self.x = to(x).contiguous()
        self.t_full = to(target).contiguous()
        c0, c1 = self.cols[-1]
        self.t = self.t_full[:, c0:c1].contiguous()
        self.w = []
        for k, w in enumerate(weights):
            c0, c1 = self.cols[k + 1]
            self.w.append(to(w)[:, c0:c1].contiguous())

    def full_weights(self):
        out = []
        for k, w in enumerate(self.w):
            full = torch.empty((self.dims[k], self.dims[k + 1]), dtype=self.dtype, device=self.device)
            out.append(gather_columns(w, full, self.group))
        return out

    def step(self, stream=None):
        """One training step; returns the loss (a device scalar, the same on every rank)."""
        self._next = 0
        self.status.fill_(-1)
        L, P, st, g = len(self.w), self.policy, self._st, self.group
        dev, dt = self.device, self.dtype
        zs, hs = [], [self.x]
        for k in range(L):  # forward: column blocks of every layer, all-gathered
            z = pcu.strict_matmul(hs[-1], self.w[k], False, False, P, status=st(), stream=stream)
            zs.append(z)
            a = pcu.checked_relu(z, P, status=st(), stream=stream) if k + 1 < L else z
            full = torch.empty((self.batch, self.dims[k + 1]), dtype=dt, device=dev)
            hs.append(gather_columns(a, full, g))
        y = hs[-1]
        loss = pcu.strict_mse(y, self.t_full, P, status=st(), stream=stream)
        # d loss / d y = (y - t) * 2/n on this rank's columns
        c0, c1 = self.cols[-1]
        diff = pcu.checked_binary("sub", zs[-1], self.t, P, status=st(), stream=stream)
        # 2 / n correctly rounded in the element type (n itself is exact: below 2^24 elements)
        n = self.batch * self.dims[-1]
        two_over_n = float(np.float32(2.0) / np.float32(n)) if dt == torch.float32 else 2.0 / float(n)
        scale = torch.full((1,), two_over_n, dtype=dt, device=dev)
        grad = pcu.checked_binary("mul", diff, scale, P, right_uniform=True, status=st(), stream=stream)
        weights_full = self.full_weights()
        for k in range(L - 1, -1, -1):
            dw = pcu.strict_matmul(hs[k], grad, True, False, P, status=st(), stream=stream)
            if k > 0:
                gfull = torch.empty((self.batch, self.dims[k + 1]), dtype=dt, device=dev)
                gather_columns(grad, gfull, g)
                i0, i1 = self.cols[k]
                rows = weights_full[k][i0:i1].contiguous()  # this rank's rows of W_k
                dh = pcu.strict_matmul(gfull, rows, False, True, P, status=st(), stream=stream)
                grad = pcu.checked_relu_backward(zs[k - 1], dh, P, status=st(), stream=stream)
            self.w[k] = pcu.strict_sgd(self.w[k], dw, self.rate, P, status=st(), stream=stream)
        return loss
