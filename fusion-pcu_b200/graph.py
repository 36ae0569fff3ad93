"""Strict tensor graph over the C++ host layer of include/pcu_b200_graph.h.

The Python surface follows the reference's tensor dialect (paths relative to the Fusion-PCU
checkout): Graph::input / add / sub / mul / div / relu / relu_backward / matmul_transposed /
mean_squared_error / sgd_update (Crates/core/dialect/tensor.rs:3925-4345),
Graph::backward_mse_for (tensor.rs:4359 over gradients/gradients.rs:31-444), and prepared
execution that reports the first faulting node as a TensorError (tensor.rs:234-304).

Capture, reverse mode and planning are native (libpcu_b200.so) and need no GPU; prepare and
execute run the sm_100a node kernels on the current CUDA device.  There is no CPU fallback.
"""
import ctypes

import numpy as np

from . import (KIND_NAMES, POLICY, ArithmeticFault, CompoundArithmeticFault, ProviderFailure, ProviderUnavailable,
               TensorError, library)

NODE_OPS = ["input", "uniform", "add", "sub", "mul", "div", "relu", "relu_backward", "matmul", "mean_squared_error",
            "sgd_update"]
STEPS = ["Multiply", "Add", "Subtract", "Divide"]
EXEC_MODES = {"chained": 0, "each_node": 1, "graph": 2, "guarded": 3}
DISPOSITIONS = {0: "pending", 1: "executed", 2: "skipped"}
CODES = {1: "ArithmeticFault", 2: "CompoundArithmeticFault", 3: "ShapeMismatch", 4: "MatMulShape", 5: "UnknownValue",
         6: "InvalidLearningRate", 7: "GradientRootNotMse", 8: "UnsupportedGradient", 9: "EmptyOutputs",
         10: "DataLength", 11: "Backend", 12: "FailedCompletion"}


class TensorErrorStruct(ctypes.Structure):
    _fields_ = [("code", ctypes.c_int32), ("value", ctypes.c_int32), ("element_index", ctypes.c_uint64),
                ("reduction_index", ctypes.c_uint64), ("step", ctypes.c_int32), ("kind", ctypes.c_int32),
                ("backend", ctypes.c_int32)]


class GraphError(TensorError):
    """A non-arithmetic TensorError variant (shape, unknown value, gradient support, ...)."""

    def __init__(self, code, value):
        self.code, self.value = CODES.get(code, str(code)), value
        super().__init__(f"{self.code}(value={value})")


_declared = False


def _lib():
    global _declared
    L = library()
    if not _declared:
        i32, u32, u64, vp, sz = ctypes.c_int32, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_size_t
        err = ctypes.POINTER(TensorErrorStruct)
        shape = ctypes.POINTER(ctypes.c_uint64)
        L.pcu_b200_graph_new.argtypes = [i32, i32]
        L.pcu_b200_graph_new.restype = vp
        L.pcu_b200_graph_free.argtypes = [vp]
        L.pcu_b200_graph_input.argtypes = [vp, shape, i32, err]
        L.pcu_b200_graph_uniform.argtypes = [vp, shape, i32, u64, err]
        L.pcu_b200_graph_binary.argtypes = [vp, i32, i32, i32, err]
        L.pcu_b200_graph_relu.argtypes = [vp, i32, err]
        L.pcu_b200_graph_relu_backward.argtypes = [vp, i32, i32, err]
        L.pcu_b200_graph_matmul.argtypes = [vp, i32, i32, i32, i32, err]
        L.pcu_b200_graph_mean_squared_error.argtypes = [vp, i32, i32, err]
        L.pcu_b200_graph_sgd_update.argtypes = [vp, i32, i32, u32, err]
        L.pcu_b200_graph_gradient.argtypes = [vp, i32, i32, err]
        L.pcu_b200_graph_gradients.argtypes = [vp, i32, ctypes.POINTER(i32), ctypes.c_int, ctypes.POINTER(i32), err]
        L.pcu_b200_graph_gradients.restype = ctypes.c_int
        for name in ("input", "uniform", "binary", "relu", "relu_backward", "matmul", "mean_squared_error",
                     "sgd_update", "gradient"):
            getattr(L, f"pcu_b200_graph_{name}").restype = i32
        L.pcu_b200_graph_node_count.argtypes = [vp]
        L.pcu_b200_graph_node_count.restype = i32
        p32 = ctypes.POINTER(i32)
        L.pcu_b200_graph_describe.argtypes = [vp, i32, p32, p32, p32, p32, p32, shape, p32, ctypes.POINTER(u64)]
        L.pcu_b200_graph_describe.restype = ctypes.c_int
        L.pcu_b200_graph_prepare.argtypes = [vp, ctypes.POINTER(i32), ctypes.c_int, err]
        L.pcu_b200_graph_prepare.restype = vp
        L.pcu_b200_prepared_free.argtypes = [vp]
        L.pcu_b200_prepared_input_count.argtypes = [vp]
        L.pcu_b200_prepared_input_count.restype = i32
        L.pcu_b200_prepared_input_value.argtypes = [vp, i32]
        L.pcu_b200_prepared_input_value.restype = i32
        L.pcu_b200_prepared_buffer.argtypes = [vp, i32]
        L.pcu_b200_prepared_buffer.restype = vp
        L.pcu_b200_prepared_fused.argtypes = [vp, i32]
        L.pcu_b200_prepared_fused.restype = ctypes.c_int
        L.pcu_b200_prepared_execute.argtypes = [vp, ctypes.POINTER(vp), ctypes.c_int, vp, err]
        L.pcu_b200_prepared_execute.restype = ctypes.c_int
        L.pcu_b200_prepared_read.argtypes = [vp, i32, vp, sz, vp]
        L.pcu_b200_prepared_read.restype = ctypes.c_int
        L.pcu_b200_prepared_stage.argtypes = [vp, i32, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64),
                                              vp]
        L.pcu_b200_prepared_stage.restype = ctypes.c_int
        _declared = True
    return L


def _raise(e):
    """TensorError for a filled pcu_b200_tensor_error (never returns)."""
    if e.code == 1:
        raise ArithmeticFault(e.value, e.element_index, KIND_NAMES[e.kind])
    if e.code == 2:
        raise CompoundArithmeticFault(e.value, e.element_index, e.reduction_index, STEPS[e.step], KIND_NAMES[e.kind])
    if e.code == 11:
        raise ProviderFailure(f"backend failure at value {e.value} (code {e.backend})")
    raise GraphError(e.code, e.value)


def _shape(shape):
    shape = tuple(int(d) for d in shape)
    if len(shape) > 2:
        raise ValueError("tensors have rank 0, 1 or 2")
    return shape, (ctypes.c_uint64 * max(len(shape), 1))(*shape)


class Graph:
    """One captured strict tensor function (one element type, one underflow policy).

    Values are the integer ids the native layer assigns in append order."""

    def __init__(self, width=32, policy=0):
        if width not in (32, 64):
            raise ValueError("width is 32 or 64")
        self.width = width
        self.policy = POLICY.get(policy, policy)
        self.dtype = np.float32 if width == 32 else np.float64
        self._L = _lib()
        self._h = self._L.pcu_b200_graph_new(0 if width == 32 else 1, self.policy)
        if not self._h:
            raise ValueError(f"bad graph parameters ({width}, {policy})")

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h:
            self._L.pcu_b200_graph_free(h)

    def _call(self, fn, *args):
        e = TensorErrorStruct()
        v = fn(self._h, *args, ctypes.byref(e))
        if v < 0:
            _raise(e)
        return v

    def _bits(self, value):
        arr = np.array([value], dtype=self.dtype)
        return int(arr.view(np.uint32 if self.width == 32 else np.uint64)[0])

    def input(self, shape):
        shape, arr = _shape(shape)
        return self._call(self._L.pcu_b200_graph_input, arr, len(shape))

    def uniform(self, shape, value=None, bits=None):
        shape, arr = _shape(shape)
        return self._call(self._L.pcu_b200_graph_uniform, arr, len(shape), self._bits(value) if bits is None else bits)

    def add(self, a, b):
        return self._call(self._L.pcu_b200_graph_binary, 0, a, b)

    def sub(self, a, b):
        return self._call(self._L.pcu_b200_graph_binary, 1, a, b)

    def mul(self, a, b):
        return self._call(self._L.pcu_b200_graph_binary, 2, a, b)

    def div(self, a, b):
        return self._call(self._L.pcu_b200_graph_binary, 3, a, b)

    def binary(self, op, a, b):
        return getattr(self, op)(a, b)

    def relu(self, x):
        return self._call(self._L.pcu_b200_graph_relu, x)

    def relu_backward(self, x, upstream):
        return self._call(self._L.pcu_b200_graph_relu_backward, x, upstream)

    def matmul(self, a, b):
        return self._call(self._L.pcu_b200_graph_matmul, a, b, 0, 0)

    def matmul_transposed(self, a, b, transpose_left, transpose_right):
        return self._call(self._L.pcu_b200_graph_matmul, a, b, int(transpose_left), int(transpose_right))

    def mean_squared_error(self, prediction, target):
        return self._call(self._L.pcu_b200_graph_mean_squared_error, prediction, target)

    def sgd_update(self, weights, gradient, rate):
        rate_bits = int(np.array([rate], dtype=np.float32).view(np.uint32)[0])
        return self._call(self._L.pcu_b200_graph_sgd_update, weights, gradient, rate_bits)

    def backward_mse_for(self, loss, target):
        return self._call(self._L.pcu_b200_graph_gradient, loss, target)

    def backward_mse_for_targets(self, loss, targets):
        targets = [int(t) for t in targets]
        out = (ctypes.c_int32 * max(len(targets), 1))()
        e = TensorErrorStruct()
        rc = self._L.pcu_b200_graph_gradients(self._h, loss, (ctypes.c_int32 * max(len(targets), 1))(*targets),
                                              len(targets), out, ctypes.byref(e))
        if rc:
            _raise(e)
        return list(out[:len(targets)])

    def __len__(self):
        return self._L.pcu_b200_graph_node_count(self._h)

    def describe(self, value):
        """(op, left, right, transpose_left, transpose_right, shape, scalar_bits) of one value."""
        i = [ctypes.c_int32() for _ in range(6)]
        shape = (ctypes.c_uint64 * 2)()
        bits = ctypes.c_uint64()
        rc = self._L.pcu_b200_graph_describe(self._h, value, *(ctypes.byref(x) for x in i[:5]), shape,
                                             ctypes.byref(i[5]), ctypes.byref(bits))
        if rc:
            raise GraphError(rc, value)
        op, left, right, tl, tr, rank = (x.value for x in i)
        return NODE_OPS[op], left, right, bool(tl), bool(tr), tuple(shape[:rank]), bits.value

    def prepare(self, outputs):
        try:
            import torch

            if not torch.cuda.is_available():
                raise ProviderUnavailable("no CUDA device: the strict provider has no CPU fallback")
        except ImportError:
            pass
        outputs = [int(o) for o in outputs]
        e = TensorErrorStruct()
        h = self._L.pcu_b200_graph_prepare(self._h, (ctypes.c_int32 * max(len(outputs), 1))(*outputs), len(outputs),
                                           ctypes.byref(e))
        if not h:
            _raise(e)
        return PreparedGraph(self, h)


class PreparedGraph:
    """Device buffers, status words and workspace for one graph's plan."""

    def __init__(self, graph, handle):
        self.graph, self._h, self._L = graph, handle, graph._L
        n = self._L.pcu_b200_prepared_input_count(handle)
        self.inputs = [self._L.pcu_b200_prepared_input_value(handle, i) for i in range(n)]

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h:
            self._L.pcu_b200_prepared_free(h)

    def buffer(self, value):
        """Device address of a planned value's buffer (0 if the value is not planned)."""
        return self._L.pcu_b200_prepared_buffer(self._h, value) or 0

    def fused(self, value):
        """How many of the nodes after MatMul `value` the chained mode runs in its epilogue."""
        return self._L.pcu_b200_prepared_fused(self._h, value)

    def execute(self, inputs=None, wait_each_node=True, stream=None, mode=None):
        """Copy the host `inputs` ({input value: array}) in, run the plan and raise the first fault.

        mode: "chained" (one status read at the end), "each_node" (the reference's per-node wait),
        "guarded" (the guarded stage chain: nothing runs after the first fault; one read at the
        end) or "graph" (the guarded chain as a CUDA-graph replay); by default wait_each_node
        picks the first two."""
        inputs = inputs or {}
        held = []
        ptrs = (ctypes.c_void_p * max(len(self.inputs), 1))()
        for i, v in enumerate(self.inputs):
            if v in inputs:
                arr = np.ascontiguousarray(inputs[v], dtype=self.graph.dtype)
                shape = self.graph.describe(v)[5]
                if arr.size != int(np.prod(shape)):
                    raise GraphError(10, v)
                held.append(arr)
                ptrs[i] = arr.ctypes.data
        e = TensorErrorStruct()
        s = ctypes.c_void_p(stream.cuda_stream) if stream is not None else None
        code = EXEC_MODES[mode] if mode is not None else (1 if wait_each_node else 0)
        rc = self._L.pcu_b200_prepared_execute(self._h, ptrs, code, s, ctypes.byref(e))
        del held
        if rc:
            _raise(e)

    def read(self, value, stream=None):
        shape = self.graph.describe(value)[5]
        out = np.empty(shape if shape else (), dtype=self.graph.dtype)
        s = ctypes.c_void_p(stream.cuda_stream) if stream is not None else None
        rc = self._L.pcu_b200_prepared_read(self._h, value, out.ctypes.data, max(out.nbytes, out.itemsize), s)
        if rc:
            raise GraphError(rc, value)
        return out

    def stage(self, value, stream=None):
        """The last execution's record of a planned node: (fault word, disposition name)."""
        word, disp = ctypes.c_uint64(), ctypes.c_uint64()
        s = ctypes.c_void_p(stream.cuda_stream) if stream is not None else None
        rc = self._L.pcu_b200_prepared_stage(self._h, value, ctypes.byref(word), ctypes.byref(disp), s)
        if rc:
            raise GraphError(rc, value)
        return word.value, DISPOSITIONS.get(disp.value, disp.value)

    def run(self, inputs, outputs, wait_each_node=True, mode=None):
        self.execute(inputs, wait_each_node, mode=mode)
        return {o: self.read(o) for o in outputs}


def from_program(program):
    """Build a Graph from a reference_kats.json-style program: (graph, {name: value id})."""
    g = Graph(program["width"], program["policy"])
    ids = {}
    for name, spec in program["inputs"].items():
        ids[name] = g.input(spec["shape"])
    for entry in program["nodes"]:
        name, op, *rest = entry
        if op == "matmul":
            ids[name] = g.matmul_transposed(ids[rest[0]], ids[rest[1]], rest[2], rest[3])
        elif op == "sgd":
            ids[name] = g.sgd_update(ids[rest[0]], ids[rest[1]], rest[2])
        elif op == "mse":
            ids[name] = g.mean_squared_error(ids[rest[0]], ids[rest[1]])
        elif op == "relu":
            ids[name] = g.relu(ids[rest[0]])
        elif op == "relu_backward":
            ids[name] = g.relu_backward(ids[rest[0]], ids[rest[1]])
        elif op == "gradient":
            ids[name] = g.backward_mse_for(ids[rest[0]], ids[rest[1]])
        else:
            ids[name] = g.binary(op, ids[rest[0]], ids[rest[1]])
    return g, ids
