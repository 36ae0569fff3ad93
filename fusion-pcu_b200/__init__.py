"""fusion-pcu_b200: B200-native (sm_100a) strict-tensor CUDA provider for Fusion-PCU.

Python front end over the C ABI in include/pcu_b200.h (libpcu_b200.so, built in-tree by
fusion-pcu_b200/build.py).  PyTorch is used only as plumbing: CUDA device memory, streams
and torch.distributed.  There is no CPU fallback: if the shared library is missing or no
CUDA device is present the calls raise ProviderUnavailable.

Fault lifting mirrors the reference's per-node decoding (paths relative to the Fusion-PCU
checkout): Profile::fault of Crates/backends/cuda/tensor/strict_matmul/strict_matmul.rs:191-215,
strict_sgd.rs:198-219, strict_mse.rs:189-222 and the element faults of relu_backward.rs:259-281,
producing the TensorError variants of Crates/core/dialect/tensor.rs:234-251.
"""
import ctypes
import os

import numpy as np

__all__ = [
    "ProviderUnavailable", "TensorError", "ArithmeticFault", "CompoundArithmeticFault", "ProviderFailure",
    "library", "POLICY", "OPS", "STATUS_OK", "new_status", "decode_status", "strict_matmul", "strict_matmul_host",
    "matmul_host_scratch", "strict_matmul_host_left", "strict_matmul_epilogue", "EpilogueStage", "strict_sgd",
    "strict_mse", "mse_workspace", "strict_mse_segment_prepare", "strict_mse_segment_walk", "strict_mse_sgd",
    "strict_mse_sgd_segment_prepare", "strict_mse_sgd_segment", "checked_binary", "checked_relu", "checked_relu_backward", "matmul_fault", "sgd_fault",
    "mse_fault", "element_fault", "GuardedChain", "CHAIN_OUTCOMES", "chain_validate", "wait",
]

_HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY = os.path.join(_HERE, "libpcu_b200.so")
STATUS_OK = (1 << 64) - 1
POLICY = {"IeeeAfterRounding": 0, "RejectSubnormalResult": 1, "AllowGradualUnderflow": 2}
OPS = {"add": 0, "sub": 1, "mul": 2, "div": 3}
KIND_NAMES = {1: "DivideByZero", 2: "SignedDivisionOverflow", 3: "ArithmeticOverflow", 4: "ArithmeticUnderflow",
              5: "InvalidFloatingOperand"}
WATCHDOG = 7


class ProviderUnavailable(RuntimeError):
    """The CUDA provider cannot run here (library not built, or no CUDA device)."""


class ProviderFailure(RuntimeError):
    """A host-side error code from the C ABI or a malformed / watchdog status word."""


class TensorError(Exception):
    pass


class ArithmeticFault(TensorError):
    """TensorError::ArithmeticFault { value, element_index, kind }."""

    def __init__(self, value, element_index, kind):
        super().__init__(f"ArithmeticFault(value={value}, element_index={element_index}, kind={kind})")
        self.value, self.element_index, self.kind = value, element_index, kind


class CompoundArithmeticFault(TensorError):
    """TensorError::CompoundArithmeticFault { value, element_index, reduction_index, step, kind }."""

    def __init__(self, value, element_index, reduction_index, step, kind):
        super().__init__(f"CompoundArithmeticFault(value={value}, element_index={element_index}, "
                         f"reduction_index={reduction_index}, step={step}, kind={kind})")
        self.value, self.element_index, self.reduction_index = value, element_index, reduction_index
        self.step, self.kind = step, kind


class EpilogueStage(ctypes.Structure):
    """pcu_b200_epilogue_stage: one elementwise node fused into a MatMul's epilogue."""
    _fields_ = [("op", ctypes.c_int), ("operand", ctypes.c_void_p), ("operand_uniform", ctypes.c_int),
                ("operand_left", ctypes.c_int), ("out", ctypes.c_void_p), ("status", ctypes.c_void_p)]


EPILOGUE_OPS = {"add": 0, "sub": 1, "mul": 2, "div": 3, "relu": 4, "relu_backward": 5}

_lib = None


def library():
    """Load libpcu_b200.so (raises ProviderUnavailable; never substitutes another path)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIBRARY):
            raise ProviderUnavailable(f"{LIBRARY} is not built (run fusion-pcu_b200/build.py)")
        lib = ctypes.CDLL(LIBRARY)
        _declare(lib)
        _lib = lib
    return _lib


def _declare(L):
    i32, u32, u64, vp, sz = ctypes.c_int, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_size_t
    L.pcu_b200_abi_version.restype = i32
    L.pcu_b200_error_string.argtypes = [i32]
    L.pcu_b200_error_string.restype = ctypes.c_char_p
    L.pcu_b200_last_cuda_error.restype = i32
    L.pcu_b200_status_reset.argtypes = [vp, u64, vp]
    L.pcu_b200_strict_matmul_workspace_size.argtypes = [u64, u64, u64]
    L.pcu_b200_strict_matmul_workspace_size.restype = sz
    L.pcu_b200_strict_matmul.argtypes = [i32, i32, vp, vp, vp, u64, u64, u64, u64, u64, i32, i32, vp, sz, vp, vp]
    L.pcu_b200_strict_matmul_host_scratch_size.argtypes = [i32, u64, u64, u64]
    L.pcu_b200_strict_matmul_host_scratch_size.restype = sz
    L.pcu_b200_strict_matmul_epilogue.argtypes = [i32, i32, vp, vp, vp, u64, u64, u64, u64, u64, i32, i32,
                                                  ctypes.POINTER(EpilogueStage), i32, vp, sz, vp, vp]
    L.pcu_b200_strict_matmul_static_scratch.argtypes = [i32, i32, vp, vp, vp, u64, u64, u64, u64, u64, i32, i32, vp,
                                                        vp]
    L.pcu_b200_strict_matmul_host.argtypes = [i32, i32, vp, vp, vp, u64, u64, u64, vp, sz, vp, vp]
    L.pcu_b200_strict_matmul_host_left_scratch_size.argtypes = [i32, u64, u64, u64]
    L.pcu_b200_strict_matmul_host_left_scratch_size.restype = sz
    L.pcu_b200_strict_matmul_host_left.argtypes = [i32, i32, vp, vp, u64, vp, u64, u64, u64, vp, sz, vp, vp]
    L.pcu_b200_issue_probe_ops.argtypes = [i32, u64]
    L.pcu_b200_issue_probe_ops.restype = u64
    L.pcu_b200_issue_probe.argtypes = [i32, u64, vp]
    L.pcu_b200_mse_handoff_bytes.restype = sz
    L.pcu_b200_strict_mse_sgd_split.argtypes = [i32, i32, vp, vp, u64, u64, u64, vp, vp, sz, vp, vp, vp, vp, u64, u64,
                                                u32, vp, ctypes.POINTER(vp), i32, i32, u64, vp]
    L.pcu_b200_peer_rows_bytes.argtypes = [i32, u64, u64]
    L.pcu_b200_peer_rows_bytes.restype = sz
    L.pcu_b200_strict_matmul_rows_allgather.argtypes = [i32, i32, vp, vp, vp, u64, u64, u64, u64, u64, u64, u64, i32,
                                                        ctypes.POINTER(vp), i32, i32, u64, vp, sz, vp, vp]
    L.pcu_b200_peer_alloc.argtypes = [sz, ctypes.POINTER(vp), vp]
    L.pcu_b200_peer_open.argtypes = [vp, ctypes.POINTER(vp)]
    L.pcu_b200_peer_close.argtypes = [vp]
    L.pcu_b200_peer_free.argtypes = [vp]
    L.pcu_b200_strict_sgd.argtypes = [i32, i32, vp, vp, vp, u64, u32, vp, vp]
    L.pcu_b200_strict_mse_workspace_size.argtypes = [i32, u64]
    L.pcu_b200_strict_mse_workspace_size.restype = sz
    L.pcu_b200_strict_mse.argtypes = [i32, i32, vp, vp, vp, u64, vp, sz, vp, vp]
    L.pcu_b200_strict_mse_segment_prepare.argtypes = [i32, i32, vp, vp, u64, u64, vp, sz, vp, vp]
    L.pcu_b200_strict_mse_segment_walk.argtypes = [i32, i32, vp, vp, u64, u64, u64, vp, vp, vp, vp, sz, vp, vp]
    L.pcu_b200_strict_mse_sgd.argtypes = [i32, i32, vp, vp, vp, u64, vp, sz, vp, vp, vp, vp, u64, u32, vp, vp]
    L.pcu_b200_strict_mse_sgd_segment_prepare.argtypes = [i32, i32, vp, vp, u64, u64, vp, sz, vp, vp, vp, vp, u64,
                                                          u64, u32, vp, vp]
    L.pcu_b200_strict_mse_sgd_segment.argtypes = [i32, i32, vp, vp, u64, u64, u64, vp, vp, vp, vp, sz, vp, vp, vp, vp,
                                                  u64, u64, u32, vp, vp]
    L.pcu_b200_checked_binary.argtypes = [i32, i32, i32, vp, vp, vp, u64, i32, i32, vp, vp]
    L.pcu_b200_checked_relu.argtypes = [i32, i32, vp, vp, u64, vp, vp]
    L.pcu_b200_checked_relu_backward.argtypes = [i32, i32, vp, vp, vp, u64, vp, vp]
    L.pcu_b200_chain_reset.argtypes = [vp, u32, vp]
    L.pcu_b200_guarded_strict_matmul.argtypes = [i32, i32, vp, vp, vp, u64, u64, u64, u64, u64, i32, i32, vp, sz, vp,
                                                 u32, vp]
    L.pcu_b200_guarded_strict_sgd.argtypes = [i32, i32, vp, vp, vp, u64, u32, vp, u32, vp]
    L.pcu_b200_guarded_strict_mse.argtypes = [i32, i32, vp, vp, vp, u64, vp, sz, vp, u32, vp]
    L.pcu_b200_guarded_checked_binary.argtypes = [i32, i32, i32, vp, vp, vp, u64, i32, i32, vp, u32, vp]
    L.pcu_b200_guarded_checked_relu.argtypes = [i32, i32, vp, vp, u64, vp, u32, vp]
    L.pcu_b200_guarded_checked_relu_backward.argtypes = [i32, i32, vp, vp, vp, u64, vp, u32, vp]
    L.pcu_b200_chain_validate.argtypes = [vp, u32, vp, ctypes.POINTER(i32), ctypes.POINTER(u32)]
    L.pcu_b200_wait.argtypes = [vp, u32]
    L.pcu_b200_last_comm_error.restype = i32
    L.pcu_b200_comm_unique_id.argtypes = [vp]
    L.pcu_b200_comm_init.argtypes = [vp, i32, i32, ctypes.POINTER(vp)]
    L.pcu_b200_comm_free.argtypes = [vp]
    L.pcu_b200_comm_abort.argtypes = [vp]
    L.pcu_b200_comm_status_min.argtypes = [vp, vp, u64, vp]
    L.pcu_b200_comm_send.argtypes = [vp, vp, sz, i32, vp]
    L.pcu_b200_comm_recv.argtypes = [vp, vp, sz, i32, vp]
    L.pcu_b200_comm_broadcast.argtypes = [vp, vp, sz, i32, vp]
    L.pcu_b200_comm_peer_buffers.argtypes = [vp, sz, ctypes.POINTER(vp), vp]
    L.pcu_b200_comm_peer_buffers_free.argtypes = [vp, ctypes.POINTER(vp), vp]
    L.pcu_b200_comm_strict_matmul_rows.argtypes = [vp, i32, i32, vp, vp, ctypes.POINTER(vp), u64, u64, u64, u64, u64,
                                                   u64, u64, i32, vp, sz, vp, vp]
    L.pcu_b200_comm_strict_mse.argtypes = [vp, i32, i32, vp, vp, u64, u64, u64, vp, vp, sz, vp, vp]


def _torch():
    import torch

    if not torch.cuda.is_available():
        raise ProviderUnavailable("no CUDA device: the strict provider has no CPU fallback")
    return torch


def _check(rc):
    if rc != 0:
        L = library()
        msg = L.pcu_b200_error_string(rc).decode()
        raise ProviderFailure(f"pcu_b200 error {rc}: {msg} (cuda error {L.pcu_b200_last_cuda_error()}, "
                              f"nccl error {L.pcu_b200_last_comm_error()})")


def _dtype_code(t):
    torch = _torch()
    if t.dtype == torch.float32:
        return 0
    if t.dtype == torch.float64:
        return 1
    raise TypeError(f"strict provider handles float32/float64, got {t.dtype}")


def _stream(stream):
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _node(name, args, status, chain, stream):
    """pcu_b200_<name>(*args, status, stream); with chain=(records, stage), the guarded form
    pcu_b200_guarded_<name>(*args, records, stage, stream) as one stage of a GuardedChain."""
    L = library()
    if chain is None:
        return getattr(L, "pcu_b200_" + name)(*args, _ptr(status), _stream(stream))
    records, stage = chain
    return getattr(L, "pcu_b200_guarded_" + name)(*args, _ptr(records), int(stage), _stream(stream))


def new_status(count=1, device=None, stream=None):
    """Device status words initialised to the no-fault sentinel (int64 storage, read as unsigned)."""
    torch = _torch()
    return torch.full((count,), -1, dtype=torch.int64, device=device or "cuda")


def decode_status(word):
    """Unsigned status word -> None (no fault) or (event, kind)."""
    word = int(word) & STATUS_OK
    if word == STATUS_OK:
        return None
    return word >> 3, word & 7


def _kind(kind):
    if kind not in KIND_NAMES:
        raise ProviderFailure("device watchdog expired" if kind == WATCHDOG else f"malformed status kind {kind}")
    return KIND_NAMES[kind]


def matmul_fault(word, inner, cells, value=None):
    """Profile::fault for MatMul (strict_matmul.rs:191-215)."""
    d = decode_status(word)
    if d is None:
        return None
    event, kind = d
    pair = event // 2
    if inner == 0 or pair // inner >= cells:
        raise ProviderFailure(f"status {word:#x} outside the MatMul event domain")
    return CompoundArithmeticFault(value, pair // inner, pair % inner, "Multiply" if event % 2 == 0 else "Add",
                                   _kind(kind))


def sgd_fault(word, count, value=None):
    d = decode_status(word)
    if d is None:
        return None
    event, kind = d
    if event // 2 >= count:
        raise ProviderFailure(f"status {word:#x} outside the SGD event domain")
    return CompoundArithmeticFault(value, event // 2, 0, "Multiply" if event % 2 == 0 else "Subtract", _kind(kind))


def mse_fault(word, count, value=None):
    d = decode_status(word)
    if d is None:
        return None
    event, kind = d
    if event > 3 * count:
        raise ProviderFailure(f"status {word:#x} outside the MSE event domain")
    if event == 3 * count:
        return CompoundArithmeticFault(value, 0, count, "Divide", _kind(kind))
    return CompoundArithmeticFault(value, 0, event // 3, ("Subtract", "Multiply", "Add")[event % 3], _kind(kind))


def element_fault(word, count, value=None):
    d = decode_status(word)
    if d is None:
        return None
    event, kind = d
    if event >= count:
        raise ProviderFailure(f"status {word:#x} outside the element domain")
    return ArithmeticFault(value, event, _kind(kind))


# ------------------------------------------------------------------ kernel-level calls
# Each returns the output tensor; faults stay in `status` (device) until the caller reads it,
# exactly like the reference's one-status-word-per-node protocol.  `chain=GuardedChain.stage(s)`
# runs the call as stage s of a guarded chain instead (its status word is in the chain's slab).

def strict_matmul(left, right, transpose_left=False, transpose_right=False, policy=0, out=None, status=None,
                  workspace=None, stream=None, chain=None):
    torch = _torch()
    assert left.dim() == 2 and right.dim() == 2 and left.dtype == right.dtype
    assert (left.numel() == 0 or left.stride(1) == 1) and (right.numel() == 0 or right.stride(1) == 1), \
        "operands must be row-major"
    rows, inner = (left.shape[1], left.shape[0]) if transpose_left else (left.shape[0], left.shape[1])
    inner2, cols = (right.shape[1], right.shape[0]) if transpose_right else (right.shape[0], right.shape[1])
    if inner != inner2:
        raise ValueError(f"MatMulShape {tuple(left.shape)} {tuple(right.shape)}")
    L = library()
    if out is None:
        out = torch.empty((rows, cols), dtype=left.dtype, device=left.device)
    if status is None and chain is None:
        status = new_status(device=left.device)
    need = L.pcu_b200_strict_matmul_workspace_size(rows, inner, cols)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=left.device)
    _check(_node("strict_matmul", (_dtype_code(left), policy, _ptr(left), _ptr(right), _ptr(out), rows, inner, cols,
                                   max(left.stride(0), left.shape[1]), max(right.stride(0), right.shape[1]),
                                   int(transpose_left), int(transpose_right), _ptr(workspace), workspace.numel()),
                 status, chain, stream))
    return out


def strict_matmul_epilogue(left, right, stages, transpose_left=False, transpose_right=False, policy=0, out=None,
                           status=None, workspace=None, stream=None):
    """op(left) . op(right) with elementwise nodes fused into the epilogue (at most two).  `stages`
    is a list of dicts: op ("add", "sub", "mul", "div", "relu", "relu_backward"), operand (a tensor
    shaped like the product, or one element for a uniform operand; none for relu), operand_left
    (the operand is the node's left argument: for relu_backward, the forward input x), out and
    status (the node's own output and status word).  Returns the MatMul's own output."""
    torch = _torch()
    rows, inner = (left.shape[1], left.shape[0]) if transpose_left else (left.shape[0], left.shape[1])
    cols = right.shape[0] if transpose_right else right.shape[1]
    L = library()
    if out is None:
        out = torch.empty((rows, cols), dtype=left.dtype, device=left.device)
    if status is None:
        status = new_status(device=left.device)
    need = L.pcu_b200_strict_matmul_workspace_size(rows, inner, cols)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=left.device)
    arr = (EpilogueStage * max(len(stages), 1))()
    for k, st in enumerate(stages):
        operand = st.get("operand")
        arr[k].op = EPILOGUE_OPS[st["op"]]
        arr[k].operand = operand.data_ptr() if operand is not None else None
        arr[k].operand_uniform = int(operand is not None and operand.numel() == 1 and rows * cols > 1)
        arr[k].operand_left = int(st.get("operand_left", False))
        arr[k].out = st["out"].data_ptr()
        arr[k].status = st["status"].data_ptr()
    _check(L.pcu_b200_strict_matmul_epilogue(_dtype_code(left), policy, _ptr(left), _ptr(right), _ptr(out), rows,
                                             inner, cols, max(left.stride(0), left.shape[1]),
                                             max(right.stride(0), right.shape[1]), int(transpose_left),
                                             int(transpose_right), arr, len(stages), _ptr(workspace),
                                             workspace.numel(), _ptr(status), _stream(stream)))
    return out


def matmul_host_scratch(left, right, device=None):
    """A device scratch sized for strict_matmul_host over host operands `left` (rows x inner) and
    `right` (inner x columns)."""
    torch = _torch()
    need = library().pcu_b200_strict_matmul_host_scratch_size(_dtype_code(left), left.shape[0], left.shape[1],
                                                               right.shape[1])
    return torch.empty(need, dtype=torch.uint8, device=device or torch.device("cuda", torch.cuda.current_device()))


def strict_matmul_host(left, right, policy=0, out=None, status=None, scratch=None, stream=None):
    """C = A . B with A, B and C in host memory (page-locked for overlap), uploads and read-backs
    pipelined with the arithmetic by row blocks.  `status` is a host int64 tensor of one element
    (the unsigned word's bits).  Asynchronous: synchronise the stream before reading the results."""
    torch = _torch()
    assert left.device.type == "cpu" and right.device.type == "cpu" and left.dtype == right.dtype
    assert left.dim() == 2 and right.dim() == 2 and left.is_contiguous() and right.is_contiguous()
    rows, inner = left.shape
    if right.shape[0] != inner:
        raise ValueError(f"MatMulShape {tuple(left.shape)} {tuple(right.shape)}")
    if out is None:
        out = torch.empty((rows, right.shape[1]), dtype=left.dtype).pin_memory()
    if status is None:
        status = torch.empty(1, dtype=torch.int64).pin_memory()
    if scratch is None:
        scratch = matmul_host_scratch(left, right)
    _check(library().pcu_b200_strict_matmul_host(_dtype_code(left), policy, _ptr(left), _ptr(right), _ptr(out), rows,
                                                 inner, right.shape[1], _ptr(scratch), scratch.numel(), _ptr(status),
                                                 _stream(stream)))
    return out, status


def strict_matmul_host_left(left, right, policy=0, out=None, status=None, scratch=None, stream=None):
    """C = A . B with A and C in host memory and B already on the device (row-major, unit column
    stride): A's rows go up and C's rows come back by row blocks, overlapped with the arithmetic.
    `status` is a host int64 tensor of one element.  Asynchronous, as strict_matmul_host."""
    torch = _torch()
    assert left.device.type == "cpu" and right.device.type == "cuda" and left.dtype == right.dtype
    assert left.dim() == 2 and right.dim() == 2 and left.is_contiguous() and (right.numel() == 0 or right.stride(1) == 1)
    rows, inner = left.shape
    if right.shape[0] != inner:
        raise ValueError(f"MatMulShape {tuple(left.shape)} {tuple(right.shape)}")
    cols = right.shape[1]
    L = library()
    if out is None:
        out = torch.empty((rows, cols), dtype=left.dtype).pin_memory()
    if status is None:
        status = torch.empty(1, dtype=torch.int64).pin_memory()
    if scratch is None:
        need = L.pcu_b200_strict_matmul_host_left_scratch_size(_dtype_code(left), rows, inner, cols)
        scratch = torch.empty(need, dtype=torch.uint8, device=right.device)
    _check(L.pcu_b200_strict_matmul_host_left(_dtype_code(left), policy, _ptr(left), _ptr(right),
                                              max(right.stride(0), cols), _ptr(out), rows, inner, cols, _ptr(scratch),
                                              scratch.numel(), _ptr(status), _stream(stream)))
    return out, status


def strict_sgd(weights, gradient, rate, policy=0, out=None, status=None, stream=None, chain=None):
    torch = _torch()
    assert weights.is_contiguous() and gradient.is_contiguous() and weights.numel() == gradient.numel()
    if out is None:
        out = torch.empty_like(weights)
    if status is None and chain is None:
        status = new_status(device=weights.device)
    rate_bits = int(np.array([rate], dtype=np.float32).view(np.uint32)[0])
    _check(_node("strict_sgd", (_dtype_code(weights), policy, _ptr(weights), _ptr(gradient), _ptr(out),
                                weights.numel(), rate_bits), status, chain, stream))
    return out


def strict_mse(prediction, target, policy=0, out=None, status=None, workspace=None, stream=None, chain=None):
    torch = _torch()
    assert prediction.is_contiguous() and target.is_contiguous() and prediction.numel() == target.numel()
    L = library()
    n = prediction.numel()
    if out is None:
        out = torch.empty((), dtype=prediction.dtype, device=prediction.device)
    if status is None and chain is None:
        status = new_status(device=prediction.device)
    need = L.pcu_b200_strict_mse_workspace_size(_dtype_code(prediction), n)
    if workspace is None or workspace.numel() < need:
        workspace = torch.empty(max(need, 1), dtype=torch.uint8, device=prediction.device)
    _check(_node("strict_mse", (_dtype_code(prediction), policy, _ptr(prediction), _ptr(target), _ptr(out), n,
                                _ptr(workspace), workspace.numel()), status, chain, stream))
    return out


def mse_workspace(prediction):
    """A device workspace sized for strict_mse / the segment calls over `prediction`."""
    torch = _torch()
    need = library().pcu_b200_strict_mse_workspace_size(_dtype_code(prediction), prediction.numel())
    return torch.empty(max(need, 1), dtype=torch.uint8, device=prediction.device)


def strict_mse_segment_prepare(prediction, target, first_index, policy=0, status=None, workspace=None, stream=None):
    """Bandwidth-bound phase of one segment [first_index, first_index + n) of a split strict MSE."""
    assert prediction.is_contiguous() and target.is_contiguous() and prediction.numel() == target.numel()
    if status is None:
        status = new_status(device=prediction.device)
    if workspace is None:
        workspace = mse_workspace(prediction)
    _check(library().pcu_b200_strict_mse_segment_prepare(
        _dtype_code(prediction), policy, _ptr(prediction), _ptr(target), prediction.numel(), first_index,
        _ptr(workspace), workspace.numel(), _ptr(status), _stream(stream)))
    return status, workspace


def strict_mse_segment_walk(prediction, target, first_index, total_count, carry, workspace, status, policy=0,
                            out=None, stream=None):
    """Ordered walk of one segment: `carry` (a device scalar) holds the running sum entering the
    segment and receives the sum after it; for the last segment `out` receives the checked mean."""
    _check(library().pcu_b200_strict_mse_segment_walk(
        _dtype_code(prediction), policy, _ptr(prediction), _ptr(target), prediction.numel(), first_index,
        total_count, _ptr(carry), _ptr(carry), _ptr(out), _ptr(workspace), workspace.numel(), _ptr(status),
        _stream(stream)))
    return out


def _rate_bits(rate):
    return int(np.array([rate], dtype=np.float32).view(np.uint32)[0])


def strict_mse_sgd(prediction, target, weights, gradient, rate, policy=0, loss=None, updated=None, mse_status=None,
                   sgd_status=None, workspace=None, stream=None):
    """The strict MSE of (prediction, target) and the strict SGD update of `weights` in one pass
    (two independent nodes, each with its own status word).  Returns (loss, updated)."""
    torch = _torch()
    for t in (prediction, target, weights, gradient):
        assert t.is_contiguous() and t.dtype == prediction.dtype
    assert prediction.numel() == target.numel() and weights.numel() == gradient.numel()
    if loss is None:
        loss = torch.empty((), dtype=prediction.dtype, device=prediction.device)
    if updated is None:
        updated = torch.empty_like(weights)
    if mse_status is None:
        mse_status = new_status(device=prediction.device)
    if sgd_status is None:
        sgd_status = new_status(device=prediction.device)
    if workspace is None:
        workspace = mse_workspace(prediction)
    _check(library().pcu_b200_strict_mse_sgd(
        _dtype_code(prediction), policy, _ptr(prediction), _ptr(target), _ptr(loss), prediction.numel(),
        _ptr(workspace), workspace.numel(), _ptr(mse_status), _ptr(weights), _ptr(gradient), _ptr(updated),
        weights.numel(), _rate_bits(rate), _ptr(sgd_status), _stream(stream)))
    return loss, updated


def strict_mse_sgd_segment_prepare(prediction, target, first_index, weights, gradient, rate, sgd_first_index,
                                   policy=0, updated=None, mse_status=None, sgd_status=None, workspace=None,
                                   stream=None):
    """strict_mse_segment_prepare carrying an SGD share (global SGD elements
    [sgd_first_index, sgd_first_index + weights.numel())).  Returns (mse_status, workspace, updated)."""
    torch = _torch()
    assert prediction.is_contiguous() and target.is_contiguous() and prediction.numel() == target.numel()
    assert weights.is_contiguous() and gradient.is_contiguous() and weights.numel() == gradient.numel()
    if updated is None:
        updated = torch.empty_like(weights)
    if mse_status is None:
        mse_status = new_status(device=prediction.device)
    if sgd_status is None:
        sgd_status = new_status(device=prediction.device)
    if workspace is None:
        workspace = mse_workspace(prediction)
    _check(library().pcu_b200_strict_mse_sgd_segment_prepare(
        _dtype_code(prediction), policy, _ptr(prediction), _ptr(target), prediction.numel(), first_index,
        _ptr(workspace), workspace.numel(), _ptr(mse_status), _ptr(weights), _ptr(gradient), _ptr(updated),
        weights.numel(), sgd_first_index, _rate_bits(rate), _ptr(sgd_status), _stream(stream)))
    return mse_status, workspace, updated


def strict_mse_sgd_segment(prediction, target, first_index, total_count, carry_in, carry_out, workspace, mse_status,
                           policy=0, out=None, sgd=None, stream=None):
    """A whole MSE segment in one call (one launch for binary32): maps and the walk from `carry_in`
    (a device scalar, None = +0); the running sum after it goes to `carry_out`, the checked mean
    to `out` for the last segment.  `sgd`: optionally an SGD block carried along, a dict with
    weights, gradient, rate, first_index, out and status."""
    assert prediction.is_contiguous() and target.is_contiguous() and prediction.numel() == target.numel()
    if sgd is None:
        w = g = upd = None
        n_sgd, sgd_first, rate_bits, sgd_status = 0, 0, _rate_bits(0.0), new_status(device=prediction.device)
    else:
        w, g, upd, sgd_status = sgd["weights"], sgd["gradient"], sgd["out"], sgd["status"]
        n_sgd, sgd_first, rate_bits = w.numel(), sgd["first_index"], _rate_bits(sgd["rate"])
    _check(library().pcu_b200_strict_mse_sgd_segment(
        _dtype_code(prediction), policy, _ptr(prediction), _ptr(target), prediction.numel(), first_index, total_count,
        _ptr(carry_in), _ptr(carry_out), _ptr(out), _ptr(workspace), workspace.numel(), _ptr(mse_status), _ptr(w),
        _ptr(g), _ptr(upd), n_sgd, sgd_first, rate_bits, _ptr(sgd_status), _stream(stream)))
    return out


def checked_binary(op, left, right, policy=0, left_uniform=False, right_uniform=False, out=None, status=None,
                   stream=None, chain=None):
    torch = _torch()
    n = max(1 if left_uniform else left.numel(), 1 if right_uniform else right.numel())
    shape = right.shape if left_uniform else left.shape
    if out is None:
        out = torch.empty(shape, dtype=left.dtype, device=left.device)
    if status is None and chain is None:
        status = new_status(device=left.device)
    _check(_node("checked_binary", (_dtype_code(left), policy, OPS.get(op, op), _ptr(left), _ptr(right), _ptr(out), n,
                                    int(left_uniform), int(right_uniform)), status, chain, stream))
    return out


def checked_relu(x, policy=0, out=None, status=None, stream=None, chain=None):
    torch = _torch()
    if out is None:
        out = torch.empty_like(x)
    if status is None and chain is None:
        status = new_status(device=x.device)
    _check(_node("checked_relu", (_dtype_code(x), policy, _ptr(x), _ptr(out), x.numel()), status, chain, stream))
    return out


def checked_relu_backward(x, upstream, policy=0, out=None, status=None, stream=None, chain=None):
    torch = _torch()
    if out is None:
        out = torch.empty_like(x)
    if status is None and chain is None:
        status = new_status(device=x.device)
    _check(_node("checked_relu_backward", (_dtype_code(x), policy, _ptr(x), _ptr(upstream), _ptr(out), x.numel()),
                 status, chain, stream))
    return out


# ------------------------------------------------------------------ guarded chains

CHAIN_OUTCOMES = {0: "succeeded", 1: "fault", 2: "stage_decode", 3: "unexpected_skip", 4: "executed_after_fault"}


def chain_validate(records, extents=None):
    """Checks a chain's record slab read back to the host (uint64 array, [word, disposition] per
    stage), as validate_guarded_execution does (Crates/core/runtime/execution/guarded/guarded.rs:
    107-140).  Returns (outcome, stage), outcome one of CHAIN_OUTCOMES's names; host code only."""
    recs = np.ascontiguousarray(np.asarray(records, dtype=np.uint64).reshape(-1))
    if recs.size % 2:
        raise ValueError("a chain slab holds two words per stage")
    stages = recs.size // 2
    ext = None
    if extents is not None:
        ext = np.ascontiguousarray(np.asarray(extents, dtype=np.uint64).reshape(-1))
        if ext.size != stages:
            raise ValueError("one event extent per stage")
    outcome, stage = ctypes.c_int(-1), ctypes.c_uint32(0)
    _check(library().pcu_b200_chain_validate(recs.ctypes.data_as(ctypes.c_void_p), stages,
                                             ext.ctypes.data_as(ctypes.c_void_p) if ext is not None else None,
                                             ctypes.byref(outcome), ctypes.byref(stage)))
    return CHAIN_OUTCOMES[outcome.value], stage.value


class GuardedChain:
    """The record slab of one ordered, stop-on-fault chain of node calls on one stream
    (Crates/backends/cuda/tensor/guarded/guarded.rs:355-400): [fault word, disposition] per stage.
    Pass `chain=g.stage(s)` to the node calls in stage order; `validate()` reads the slab once."""

    def __init__(self, stages, device=None):
        torch = _torch()
        self.stages = int(stages)
        self.records = torch.empty(2 * max(self.stages, 1), dtype=torch.int64, device=device or "cuda")

    def reset(self, stream=None):
        _check(library().pcu_b200_chain_reset(_ptr(self.records), self.stages, _stream(stream)))
        return self

    def stage(self, s):
        if not 0 <= s < self.stages:
            raise IndexError(f"stage {s} of a {self.stages}-stage chain")
        return (self.records, s)

    def read(self, stream=None):
        """The slab as uint64 on the host (waits for the stream)."""
        torch = _torch()
        s = stream if stream is not None else torch.cuda.current_stream()
        with torch.cuda.stream(s):
            host = self.records[:2 * self.stages].cpu()
        return host.numpy().view(np.uint64)

    def validate(self, extents=None, stream=None):
        """(outcome, stage, fault word of that stage)."""
        recs = self.read(stream)
        outcome, stage = chain_validate(recs, extents)
        return outcome, stage, int(recs[2 * stage]) if self.stages else STATUS_OK


def wait(stream=None, timeout_ms=1000):
    """True when all work on `stream` has completed within timeout_ms, False if it has not."""
    rc = library().pcu_b200_wait(_stream(stream), int(timeout_ms))
    if rc == 6:
        return False
    _check(rc)
    return True
