"""The C ABI's own communicator (pcu_b200_comm_*): the multi-GPU exchange steps for a host without
torch.distributed.  One process per GPU; the NCCL unique id made by rank 0 is handed to the other
ranks by the host (any channel: a file, a pipe, a store).

    comm = Communicator(uid, nranks, rank)        # uid = Communicator.unique_id() on rank 0
    c = comm.peer_matrix(rows_total, columns)     # every rank's copy of C, mapped into the others
    comm.strict_matmul_rows(a_rows, b, row0, c, status)
    comm.strict_mse(pred_seg, target_seg, first_index, total, out, status)
"""
import ctypes
import importlib

import torch

pcu = importlib.import_module("fusion-pcu_b200")
_cuda_array = importlib.import_module("fusion-pcu_b200.sharded")._CudaArray


class Communicator:
    """pcu_b200_comm_init on the current device; close() (or abort() after a failed peer)."""

    ID_BYTES = 128

    @staticmethod
    def unique_id():
        uid = (ctypes.c_ubyte * Communicator.ID_BYTES)()
        pcu._check(pcu.library().pcu_b200_comm_unique_id(uid))
        return bytes(uid)

    def __init__(self, uid, nranks, rank):
        self.nranks, self.rank = nranks, rank
        handle = ctypes.c_void_p()
        buf = (ctypes.c_ubyte * self.ID_BYTES).from_buffer_copy(uid)
        pcu._check(pcu.library().pcu_b200_comm_init(buf, nranks, rank, ctypes.byref(handle)))
        self._c = handle

    def close(self):
        if self._c:
            pcu._check(pcu.library().pcu_b200_comm_free(self._c))
            self._c = None

    def abort(self):
        if self._c:
            pcu._check(pcu.library().pcu_b200_comm_abort(self._c))
            self._c = None

    def status_min(self, status, stream=None):
        pcu._check(pcu.library().pcu_b200_comm_status_min(self._c, pcu._ptr(status), status.numel(),
                                                           pcu._stream(stream)))
        return status

    def send(self, tensor, peer, stream=None):
        pcu._check(pcu.library().pcu_b200_comm_send(self._c, pcu._ptr(tensor), tensor.numel() * tensor.element_size(),
                                                     peer, pcu._stream(stream)))

    def recv(self, tensor, peer, stream=None):
        pcu._check(pcu.library().pcu_b200_comm_recv(self._c, pcu._ptr(tensor), tensor.numel() * tensor.element_size(),
                                                     peer, pcu._stream(stream)))
        return tensor

    def broadcast(self, tensor, root, stream=None):
        pcu._check(pcu.library().pcu_b200_comm_broadcast(self._c, pcu._ptr(tensor),
                                                          tensor.numel() * tensor.element_size(), root,
                                                          pcu._stream(stream)))
        return tensor

    def peer_matrix(self, rows, columns, dtype=torch.float32, stream=None):
        return PeerMatrix(self, rows, columns, dtype, stream)

    def strict_matmul_rows(self, left_rows, right, row0, shared, status, transpose_right=False, policy=0,
                           workspace=None, stream=None):
        """Rows [row0, row0 + m) of C = A . op(B) into every rank's copy of `shared`, then the
        status MIN (pcu_b200_comm_strict_matmul_rows).  Returns this rank's whole C."""
        L = pcu.library()
        rows, inner = left_rows.shape
        cols = right.shape[0] if transpose_right else right.shape[1]
        if workspace is None:
            workspace = torch.empty(max(L.pcu_b200_strict_matmul_workspace_size(rows, inner, cols), 1),
                                    dtype=torch.uint8, device=left_rows.device)
        pcu._check(L.pcu_b200_comm_strict_matmul_rows(
            self._c, pcu._dtype_code(left_rows), policy, pcu._ptr(left_rows), pcu._ptr(right), shared.buffers, row0,
            rows, shared.rows, inner, cols, left_rows.stride(0), right.stride(0), int(transpose_right),
            pcu._ptr(workspace), workspace.numel(), pcu._ptr(status), pcu._stream(stream)))
        return shared.local

    def strict_mse(self, prediction, target, first_index, total_count, out, status, policy=0, workspace=None,
                   stream=None):
        """The split strict MSE (pcu_b200_comm_strict_mse): this rank's segment holds the global
        elements [first_index, first_index + n).  `out` (a device scalar) gets the mean on every rank."""
        assert prediction.is_contiguous() and target.is_contiguous() and prediction.numel() == target.numel()
        if workspace is None:
            workspace = pcu.mse_workspace(prediction)
        pcu._check(pcu.library().pcu_b200_comm_strict_mse(
            self._c, pcu._dtype_code(prediction), policy, pcu._ptr(prediction), pcu._ptr(target), prediction.numel(),
            first_index, total_count, pcu._ptr(out), pcu._ptr(workspace), workspace.numel(), pcu._ptr(status),
            pcu._stream(stream)))
        return out


class PeerMatrix:
    """A rows x columns matrix of which every rank holds a copy that every rank writes into
    (pcu_b200_comm_peer_buffers).  `local` is this rank's copy as a torch view."""

    def __init__(self, comm, rows, columns, dtype, stream=None):
        self.comm, self.rows, self.columns, self.dtype = comm, rows, columns, dtype
        L = pcu.library()
        self.buffers = (ctypes.c_void_p * comm.nranks)()
        nbytes = L.pcu_b200_peer_rows_bytes(0 if dtype == torch.float32 else 1, rows, columns)
        pcu._check(L.pcu_b200_comm_peer_buffers(comm._c, nbytes, self.buffers, pcu._stream(stream)))
        self.local = torch.as_tensor(_cuda_array(self.buffers[comm.rank], (rows, columns), dtype), device="cuda")

    def close(self, stream=None):
        if self.buffers[self.comm.rank]:
            self.local = None
            pcu._check(pcu.library().pcu_b200_comm_peer_buffers_free(self.comm._c, self.buffers, pcu._stream(stream)))
