"""CPU oracle for the strict tensor path -- TEST INFRASTRUCTURE ONLY.

A ctypes front end over oracle/liboracle.so, the C restatement of the
reference's strict CPU provider (see pcu_oracle.h for the file:line map).  Only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference legs
import this package, and only as the checker; the CUDA provider never does.

Parity pin: the reference is Rust and cannot be built here; the restatement is
pinned by tests/test_oracle_kats.py against the reference's own known-answer
tests (tests/golden/reference_kats.json) and its randomized host-RNE checks.
"""
import ctypes
import os

import numpy as np

from . import build as _build

STATUS_OK = (1 << 64) - 1

KIND_NAMES = {
    1: "DivideByZero",
    2: "SignedDivisionOverflow",
    3: "ArithmeticOverflow",
    4: "ArithmeticUnderflow",
    5: "InvalidFloatingOperand",
}
KIND_BY_NAME = {v: k for k, v in KIND_NAMES.items()}
POLICIES = {"IeeeAfterRounding": 0, "RejectSubnormalResult": 1, "AllowGradualUnderflow": 2}
OPS = {"add": 0, "sub": 1, "mul": 2, "div": 3}

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.LIBRARY
        if not os.path.exists(path):
            path = _build.build()
        _lib = ctypes.CDLL(path)
        _declare(_lib)
    return _lib


def _declare(L):
    u32, u64, i32, vp = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int, ctypes.c_void_p
    P32, P64 = ctypes.POINTER(u32), ctypes.POINTER(u64)
    L.pcu_oracle_f32_binary.argtypes = [u32, u32, i32, i32, P32]
    L.pcu_oracle_f64_binary.argtypes = [u64, u64, i32, i32, P64]
    for name, t, p in (("f32", u32, P32), ("f64", u64, P64)):
        getattr(L, f"pcu_oracle_{name}_relu").argtypes = [t, i32, p]
        getattr(L, f"pcu_oracle_{name}_neg").argtypes = [t, i32, p]
        getattr(L, f"pcu_oracle_{name}_relu_backward").argtypes = [t, t, i32, p]
    L.pcu_oracle_count_f32.argtypes = [u64]
    L.pcu_oracle_count_f32.restype = u32
    L.pcu_oracle_count_f64.argtypes = [u64]
    L.pcu_oracle_count_f64.restype = u64
    L.pcu_oracle_f32_bits_to_f64_bits.argtypes = [u32]
    L.pcu_oracle_f32_bits_to_f64_bits.restype = u64
    mm = [i32, vp, vp, vp, u64, u64, u64, u64, u64, i32, i32, i32]
    L.pcu_oracle_matmul.argtypes = mm + [u64, u64]
    L.pcu_oracle_matmul.restype = u64
    L.pcu_oracle_matmul_cells.argtypes = mm + [vp, u64]
    L.pcu_oracle_matmul_cells.restype = u64
    L.pcu_oracle_fast_matmul.argtypes = mm + [u64, u64, i32]
    L.pcu_oracle_fast_matmul.restype = u64
    L.pcu_oracle_soft_matmul_threads.argtypes = mm + [u64, u64, i32]
    L.pcu_oracle_soft_matmul_threads.restype = u64
    L.pcu_oracle_mse.argtypes = [i32, vp, vp, u64, i32, vp]
    L.pcu_oracle_mse.restype = u64
    L.pcu_oracle_mse_segment.argtypes = [i32, vp, vp, u64, u64, u64, i32, ctypes.POINTER(u64), vp]
    L.pcu_oracle_mse_segment.restype = u64
    L.pcu_oracle_sgd.argtypes = [i32, vp, vp, u32, u64, i32, vp]
    L.pcu_oracle_sgd.restype = u64
    L.pcu_oracle_binary.argtypes = [i32, i32, vp, vp, u64, i32, i32, i32, vp]
    L.pcu_oracle_binary.restype = u64
    L.pcu_oracle_relu.argtypes = [i32, vp, u64, i32, vp]
    L.pcu_oracle_relu.restype = u64
    L.pcu_oracle_relu_backward.argtypes = [i32, vp, vp, u64, i32, vp]
    L.pcu_oracle_relu_backward.restype = u64


# ------------------------------------------------------------------ scalar law

def f32_binary(a_bits, b_bits, op, policy=0):
    out = ctypes.c_uint32(0)
    kind = lib().pcu_oracle_f32_binary(a_bits & 0xFFFFFFFF, b_bits & 0xFFFFFFFF, OPS.get(op, op), policy,
                                       ctypes.byref(out))
    return kind, out.value


def f64_binary(a_bits, b_bits, op, policy=0):
    out = ctypes.c_uint64(0)
    kind = lib().pcu_oracle_f64_binary(a_bits, b_bits, OPS.get(op, op), policy, ctypes.byref(out))
    return kind, out.value


def unary(name, width, x_bits, policy=0, upstream=None):
    fn = getattr(lib(), f"pcu_oracle_f{width}_{name}")
    out = (ctypes.c_uint32 if width == 32 else ctypes.c_uint64)(0)
    if upstream is None:
        kind = fn(x_bits, policy, ctypes.byref(out))
    else:
        kind = fn(x_bits, upstream, policy, ctypes.byref(out))
    return kind, out.value


def count_f32(n):
    return lib().pcu_oracle_count_f32(n)


def count_f64(n):
    return lib().pcu_oracle_count_f64(n)


def f32_bits_to_f64_bits(bits):
    return lib().pcu_oracle_f32_bits_to_f64_bits(bits)


# ------------------------------------------------------------------ tensors

def _elem(array):
    if array.dtype == np.float32:
        return 4
    if array.dtype == np.float64:
        return 8
    raise TypeError(f"oracle handles float32/float64 only, got {array.dtype}")


def _ptr(array):
    return array.ctypes.data_as(ctypes.c_void_p)


def matmul(left, right, transpose_left=False, transpose_right=False, policy=0, rows=None,
           fast=False, threads=None):
    """Ordered strict MatMul of op(left) . op(right); returns (status, out).

    `rows` = (begin, end) restricts the computed output rows (others stay 0).
    fast=True uses the hardware-IEEE checker with exact soft-float fallback.
    """
    left = np.ascontiguousarray(left)
    right = np.ascontiguousarray(right)
    elem = _elem(left)
    assert right.dtype == left.dtype and left.ndim == 2 and right.ndim == 2
    m, k = (left.shape[1], left.shape[0]) if transpose_left else left.shape
    k2, n = (right.shape[1], right.shape[0]) if transpose_right else right.shape
    assert k == k2, (left.shape, right.shape)
    out = np.zeros((m, n), dtype=left.dtype)
    begin, end = rows if rows is not None else (0, m)
    args = (elem, _ptr(left), _ptr(right), _ptr(out), m, k, n, left.shape[1], right.shape[1],
            int(transpose_left), int(transpose_right), policy, begin, end)
    if fast:
        status = lib().pcu_oracle_fast_matmul(*args, threads or os.cpu_count() or 1)
    elif threads:
        status = lib().pcu_oracle_soft_matmul_threads(*args, threads)
    else:
        status = lib().pcu_oracle_matmul(*args)
    return status, out


def matmul_cells(left, right, cells, transpose_left=False, transpose_right=False, policy=0):
    """Strict values of selected flat output cells; returns (min status over them, values)."""
    left = np.ascontiguousarray(left)
    right = np.ascontiguousarray(right)
    elem = _elem(left)
    m, k = (left.shape[1], left.shape[0]) if transpose_left else left.shape
    n = right.shape[0] if transpose_right else right.shape[1]
    cells = np.ascontiguousarray(cells, dtype=np.uint64)
    out = np.zeros(len(cells), dtype=left.dtype)
    status = lib().pcu_oracle_matmul_cells(elem, _ptr(left), _ptr(right), _ptr(out), m, k, n, left.shape[1],
                                           right.shape[1], int(transpose_left), int(transpose_right), policy,
                                           _ptr(cells), len(cells))
    return status, out


def mse(prediction, target, policy=0):
    prediction = np.ascontiguousarray(prediction)
    target = np.ascontiguousarray(target)
    out = np.zeros(1, dtype=prediction.dtype)
    status = lib().pcu_oracle_mse(_elem(prediction), _ptr(prediction), _ptr(target), prediction.size, policy,
                                  _ptr(out))
    return status, out


def mse_segment(prediction, target, first_index, total_count, carry_bits=0, policy=0, last=False):
    """One segment of a split ordered MSE: returns (status, carry bits after it, mean or None)."""
    prediction = np.ascontiguousarray(prediction)
    target = np.ascontiguousarray(target)
    carry = ctypes.c_uint64(carry_bits)
    out = np.zeros(1, dtype=prediction.dtype) if last else None
    status = lib().pcu_oracle_mse_segment(_elem(prediction), _ptr(prediction), _ptr(target), prediction.size,
                                          first_index, total_count, policy, ctypes.byref(carry),
                                          _ptr(out) if last else None)
    return status, carry.value, out


def sgd(weights, gradient, rate, policy=0):
    weights = np.ascontiguousarray(weights)
    gradient = np.ascontiguousarray(gradient)
    out = np.zeros_like(weights)
    rate_bits = int(np.float32(rate).view(np.uint32))
    status = lib().pcu_oracle_sgd(_elem(weights), _ptr(weights), _ptr(gradient), rate_bits, weights.size, policy,
                                  _ptr(out))
    return status, out


def binary(op, left, right, policy=0, left_uniform=False, right_uniform=False):
    left = np.ascontiguousarray(left)
    right = np.ascontiguousarray(right)
    count = max(left.size if not left_uniform else 1, right.size if not right_uniform else 1)
    shape = left.shape if not left_uniform else right.shape
    out = np.zeros(shape, dtype=left.dtype)
    status = lib().pcu_oracle_binary(_elem(left), OPS.get(op, op), _ptr(left), _ptr(right), count,
                                     int(left_uniform), int(right_uniform), policy, _ptr(out))
    return status, out


def relu(x, policy=0):
    x = np.ascontiguousarray(x)
    out = np.zeros_like(x)
    return lib().pcu_oracle_relu(_elem(x), _ptr(x), x.size, policy, _ptr(out)), out


def relu_backward(x, upstream, policy=0):
    x = np.ascontiguousarray(x)
    upstream = np.ascontiguousarray(upstream)
    out = np.zeros_like(x)
    return lib().pcu_oracle_relu_backward(_elem(x), _ptr(x), _ptr(upstream), x.size, policy, _ptr(out)), out


# ------------------------------------------------------------------ status words

def decode(status):
    """(event, kind) of a status word, or None for the no-fault sentinel."""
    if status == STATUS_OK:
        return None
    return status >> 3, status & 7


def matmul_location(status, inner):
    """(element_index, reduction_index, step) per fault_domain.rs:131-142."""
    event, kind = decode(status)
    pair = event // 2
    return pair // inner, pair % inner, "Multiply" if event % 2 == 0 else "Add", KIND_NAMES[kind]


def sgd_location(status):
    event, kind = decode(status)
    return event // 2, 0, "Multiply" if event % 2 == 0 else "Subtract", KIND_NAMES[kind]


def mse_location(status, count):
    event, kind = decode(status)
    if event == 3 * count:
        return 0, count, "Divide", KIND_NAMES[kind]
    return 0, event // 3, ("Subtract", "Multiply", "Add")[event % 3], KIND_NAMES[kind]
