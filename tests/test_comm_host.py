"""The communicator entry points (pcu_b200_comm_*) check their arguments before any NCCL or CUDA
call, and the library does not depend on NCCL at load time (it is loaded when a communicator is
made).  No GPU needed; the collective calls themselves are in tests/test_gpu_comm.py."""
import ctypes
import os

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_no_load_time_nccl_dependency():
    out = os.popen(f"ldd {os.path.join(ROOT, 'fusion-pcu_b200', 'libpcu_b200.so')}").read()
    assert "nccl" not in out, out


def test_arguments_are_checked_first(provider):
    lib = provider.library()
    uid = (ctypes.c_ubyte * 128)()
    comm = ctypes.c_void_p(123)
    assert lib.pcu_b200_comm_init(uid, 2, 0, None) == 1
    assert lib.pcu_b200_comm_init(None, 2, 0, ctypes.byref(comm)) == 1 and comm.value is None
    for nranks, rank in ((0, 0), (9, 0), (2, 2), (2, -1)):
        assert lib.pcu_b200_comm_init(uid, nranks, rank, ctypes.byref(comm)) == 1
    assert lib.pcu_b200_comm_unique_id(None) == 1
    assert lib.pcu_b200_comm_free(None) == 0 and lib.pcu_b200_comm_abort(None) == 0
    assert lib.pcu_b200_comm_status_min(None, None, 1, None) == 1
    assert lib.pcu_b200_comm_send(None, None, 0, 1, None) == 1
    assert lib.pcu_b200_comm_recv(None, None, 0, 1, None) == 1
    assert lib.pcu_b200_comm_broadcast(None, None, 0, 0, None) == 1
    bufs = (ctypes.c_void_p * 2)()
    assert lib.pcu_b200_comm_peer_buffers(None, 64, bufs, None) == 1
    assert lib.pcu_b200_comm_peer_buffers_free(None, bufs, None) == 1
    assert lib.pcu_b200_comm_strict_matmul_rows(None, 0, 0, None, None, bufs, 0, 1, 1, 1, 1, 1, 1, 0, None, 0, None,
                                                None) == 1
    assert lib.pcu_b200_comm_strict_mse(None, 0, 0, None, None, 1, 0, 1, None, None, 0, None, None) == 1
    assert lib.pcu_b200_error_string(7).decode().startswith("communicator failure")
    assert lib.pcu_b200_last_comm_error() == 0
