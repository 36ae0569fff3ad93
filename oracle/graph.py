"""Strict tensor program evaluator on the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Restates, in plain Python over the C oracle primitives:
  * reverse-mode construction for an MSE root
      Crates/core/dialect/tensor/gradients/gradients.rs:31-252 (node rules),
      :310-364 (requested-path selection), :366-444 (reverse sweep);
  * plan selection: dependency closure of the outputs plus every checked
    binary / compound node with its dependencies
      Crates/core/dialect/tensor.rs:3234-3285;
  * evaluation in append order, the first faulting node wins and nothing is
    published on failure
      Crates/backends/cpu/prepared_tensor/prepared_tensor.rs:258-270.

A program is a list of nodes [name, op, *operands] as in
tests/golden/reference_kats.json; "gradient" nodes are expanded in place.
"""
import numpy as np

from . import (STATUS_OK, KIND_NAMES, binary, count_f32, count_f64, decode, f32_binary, f64_binary,
               matmul, mse, relu, relu_backward, sgd)

COMPOUND = {"matmul", "mse", "sgd"}
CHECKED_BINARY = {"add", "sub", "mul", "div"}


class Node:
    __slots__ = ("name", "op", "args", "shape", "tl", "tr", "rate", "value")

    def __init__(self, name, op, args, shape, tl=False, tr=False, rate=None, value=None):
        self.name, self.op, self.args, self.shape = name, op, list(args), tuple(shape)
        self.tl, self.tr, self.rate, self.value = tl, tr, rate, value

    def __repr__(self):
        return f"Node({self.name}={self.op}{tuple(self.args)})"


class Graph:
    def __init__(self, width):
        self.width = width
        self.dtype = np.float32 if width == 32 else np.float64
        self.nodes = []
        self.index = {}
        self._auto = 0

    def _push(self, op, args, shape, name=None, **kw):
        if name is None:
            self._auto += 1
            name = f"%{self._auto}"
        node = Node(name, op, args, shape, **kw)
        self.index[name] = len(self.nodes)
        self.nodes.append(node)
        return name

    def shape(self, name):
        return self.nodes[self.index[name]].shape

    # builders mirroring Graph::{input, add, sub, mul, div, relu, relu_backward, matmul_transposed,
    # mean_squared_error, sgd_update, uniform}
    def input(self, name, shape):
        return self._push("input", [], shape, name)

    def uniform(self, shape, value_bits):
        return self._push("uniform", [], shape, value=value_bits)

    def binary(self, op, a, b, name=None):
        if self.shape(a) != self.shape(b):
            raise ValueError(f"ShapeMismatch {self.shape(a)} {self.shape(b)}")
        return self._push(op, [a, b], self.shape(a), name)

    def relu(self, x, name=None):
        return self._push("relu", [x], self.shape(x), name)

    def relu_backward(self, x, upstream, name=None):
        if self.shape(x) != self.shape(upstream):
            raise ValueError("ShapeMismatch")
        return self._push("relu_backward", [x, upstream], self.shape(x), name)

    def matmul(self, a, b, tl=False, tr=False, name=None):
        sa, sb = self.shape(a), self.shape(b)
        rows, inner = (sa[1], sa[0]) if tl else (sa[0], sa[1])
        inner2, cols = (sb[1], sb[0]) if tr else (sb[0], sb[1])
        if inner != inner2:
            raise ValueError(f"MatMulShape {sa} {sb}")
        return self._push("matmul", [a, b], (rows, cols), name, tl=tl, tr=tr)

    def mse(self, p, t, name=None):
        if self.shape(p) != self.shape(t) or int(np.prod(self.shape(p))) == 0:
            raise ValueError("ShapeMismatch")
        return self._push("mse", [p, t], (), name)

    def sgd(self, w, g, rate, name=None):
        if self.shape(w) != self.shape(g):
            raise ValueError("ShapeMismatch")
        return self._push("sgd", [w, g], self.shape(w), name, rate=rate)

    # ---------------------------------------------------------------- reverse mode
    def gradient(self, loss, target, name=None):
        """Graph::backward_mse_for(loss, target) (gradients.rs:279-287)."""
        result = self.gradients(loss, [target])[0]
        if name is not None:
            # give the final gradient value the requested name as an alias
            self.index[name] = self.index[result]
        return result

    def gradients(self, loss, targets):
        """Graph::backward_mse_for_targets(loss, targets): one shared reverse sweep (gradients.rs:289-303)."""
        if not targets:
            raise ValueError("EmptyOutputs")
        root = self.nodes[self.index[loss]]
        if root.op != "mse":
            raise ValueError("GradientRootNotMse")
        n_orig = len(self.nodes)
        loss_i = self.index[loss]
        visited = [False] * n_orig
        pending = [loss_i]
        while pending:
            i = pending.pop()
            if visited[i]:
                continue
            visited[i] = True
            node = self.nodes[i]
            if i != loss_i and node.op == "mse":
                raise ValueError("UnsupportedGradient (nested MSE)")
            if node.op in ("div", "relu_backward"):
                raise ValueError("UnsupportedGradient")
            pending.extend(self.index[a] for a in node.args)
        needed = [False] * n_orig
        for target in targets:
            t_i = self.index[target]
            if not visited[t_i]:
                raise ValueError("UnsupportedGradient")
            needed[t_i] = True
        for i in range(loss_i + 1):
            needed[i] = needed[i] or any(needed[self.index[a]] for a in self.nodes[i].args)
        grads = [None] * n_orig
        if any(self.index[t] == loss_i for t in targets):
            grads[loss_i] = self.uniform((), self._one())
        else:
            self._mse_grad(grads, root.args[0], root.args[1], needed)
        for i in range(loss_i, -1, -1):
            g = grads[i]
            if g is None:
                continue
            node = self.nodes[i]
            self._node_grad(grads, node, g, needed)
        results = [grads[self.index[t]] for t in targets]
        if any(r is None for r in results):
            raise ValueError("UnsupportedGradient")
        return results

    def _one(self):
        return 0x3F800000 if self.width == 32 else 0x3FF0000000000000

    def _accumulate(self, grads, target, addition):
        t = self.index[target]
        grads[t] = addition if grads[t] is None else self.binary("add", grads[t], addition)

    def _mse_grad(self, grads, prediction, target, needed):
        pi, ti = self.index[prediction], self.index[target]
        if not needed[pi] and not needed[ti]:
            return
        count = int(np.prod(self.shape(prediction)))
        if self.width == 32:
            kind, scale_bits = f32_binary(0x40000000, count_f32(count), "div")
        else:
            kind, scale_bits = f64_binary(0x4000000000000000, count_f64(count), "div")
        if kind:
            raise ArithmeticError(f"ArithmeticFault at capture: {KIND_NAMES[kind]}")
        scale = self.uniform(self.shape(prediction), scale_bits)
        pdiff = self.binary("sub", prediction, target) if needed[pi] else None
        tdiff = self.binary("sub", target, prediction) if needed[ti] else None
        pgrad = self.binary("mul", pdiff, scale) if pdiff is not None else None
        tgrad = self.binary("mul", tdiff, scale) if tdiff is not None else None
        if pgrad is not None:
            self._accumulate(grads, prediction, pgrad)
        if tgrad is not None:
            self._accumulate(grads, target, tgrad)

    def _filled_like(self, value, scalar_bits):
        return self.uniform(self.shape(value), scalar_bits)

    def _node_grad(self, grads, node, g, needed):
        op, args = node.op, node.args
        nd = lambda name: needed[self.index[name]]  # noqa: E731
        if op in ("input", "uniform"):
            return
        if op == "add":
            if nd(args[0]):
                self._accumulate(grads, args[0], g)
            if nd(args[1]):
                self._accumulate(grads, args[1], g)
        elif op == "sub":
            if nd(args[0]):
                self._accumulate(grads, args[0], g)
            if nd(args[1]):
                neg = self._filled_like(args[1], 0xBF800000 if self.width == 32 else 0xBFF0000000000000)
                self._accumulate(grads, args[1], self.binary("mul", g, neg))
        elif op == "mul":
            lg = self.binary("mul", g, args[1]) if nd(args[0]) else None
            rg = self.binary("mul", g, args[0]) if nd(args[1]) else None
            if lg is not None:
                self._accumulate(grads, args[0], lg)
            if rg is not None:
                self._accumulate(grads, args[1], rg)
        elif op == "matmul":
            left, right, tl, tr = args[0], args[1], node.tl, node.tr
            lg = rg = None
            if nd(left):
                lg = self.matmul(right, g, tr, True) if tl else self.matmul(g, right, False, not tr)
            if nd(right):
                rg = self.matmul(g, left, True, tl) if tr else self.matmul(left, g, not tl, False)
            if lg is not None:
                self._accumulate(grads, left, lg)
            if rg is not None:
                self._accumulate(grads, right, rg)
        elif op == "relu":
            if nd(args[0]):
                self._accumulate(grads, args[0], self.relu_backward(args[0], g))
        elif op == "sgd":
            w, upd = args
            ig = None
            if nd(upd):
                neg_rate = np.float32(node.rate)
                bits32 = int(neg_rate.view(np.uint32)) ^ 0x80000000
                from . import f32_bits_to_f64_bits
                scaled_bits = bits32 if self.width == 32 else f32_bits_to_f64_bits(bits32)
                ig = self.binary("mul", g, self._filled_like(upd, scaled_bits))
            if nd(w):
                self._accumulate(grads, w, g)
            if ig is not None:
                self._accumulate(grads, upd, ig)
        elif op == "mse":
            # only the root reaches here (nested MSE is rejected up front): an explicit
            # d loss / d loss seeds the root with Uniform(1), then the MSE rule runs
            # (gradients.rs:123-125, 384-397)
            self._mse_grad(grads, args[0], args[1], needed)
        else:
            raise ValueError(f"UnsupportedGradient ({op})")

    # ---------------------------------------------------------------- plan + evaluation
    def plan(self, outputs):
        selected = [False] * len(self.nodes)

        def close(i):
            stack = [i]
            while stack:
                at = stack.pop()
                if selected[at]:
                    continue
                selected[at] = True
                stack.extend(self.index[a] for a in self.nodes[at].args)

        for out in outputs:
            close(self.index[out])
        for i, node in enumerate(self.nodes):
            if node.op in CHECKED_BINARY or node.op in COMPOUND:
                close(i)
        return [i for i, s in enumerate(selected) if s]

    def evaluate(self, inputs, outputs, policy=0, fast=False):
        """Returns ({output: array}, None) or (None, fault dict) for the first faulting node.

        fast=True evaluates MatMul nodes with the multi-threaded hardware-IEEE checker
        (exact soft-float fallback), which the oracle tests hold to the scalar law."""
        values = {}
        for i in self.plan(outputs):
            node = self.nodes[i]
            status, value, fault = self._run(node, values, inputs, policy, fast)
            if status != STATUS_OK:
                return None, fault
            values[node.name] = value
        return {o: values[self.nodes[self.index[o]].name] for o in outputs}, None

    def _uniform_array(self, node):
        bits = np.array([node.value], dtype=np.uint32 if self.width == 32 else np.uint64)
        return np.broadcast_to(bits.view(self.dtype), node.shape if node.shape else (1,)).copy()

    def _run(self, node, values, inputs, policy, fast=False):
        op = node.op
        if op == "input":
            return STATUS_OK, np.ascontiguousarray(inputs[node.name], dtype=self.dtype).reshape(node.shape), None
        if op == "uniform":
            return STATUS_OK, self._uniform_array(node), None
        args = [values[self.nodes[self.index[a]].name] for a in node.args]
        if op in CHECKED_BINARY:
            status, out = binary(op, args[0].ravel(), args[1].ravel(), policy)
            out = out.reshape(node.shape)
        elif op == "relu":
            status, out = relu(args[0].ravel(), policy)
            out = out.reshape(node.shape)
        elif op == "relu_backward":
            status, out = relu_backward(args[0].ravel(), args[1].ravel(), policy)
            out = out.reshape(node.shape)
        elif op == "matmul":
            status, out = matmul(args[0], args[1], node.tl, node.tr, policy, fast=fast)
        elif op == "mse":
            status, out = mse(args[0].ravel(), args[1].ravel(), policy)
            out = out.reshape(())
        elif op == "sgd":
            status, out = sgd(args[0].ravel(), args[1].ravel(), node.rate, policy)
            out = out.reshape(node.shape)
        else:
            raise ValueError(op)
        if status == STATUS_OK:
            return status, out, None
        return status, None, self._fault(node, status, args)

    def _fault(self, node, status, args):
        event, kind = decode(status)
        fault = {"node": node.name, "kind": KIND_NAMES[kind]}
        if node.op == "matmul":
            inner = node_inner = (args[0].shape[0] if node.tl else args[0].shape[1])
            pair = event // 2
            fault.update(element_index=pair // inner, reduction_index=pair % node_inner,
                         step="Multiply" if event % 2 == 0 else "Add")
        elif node.op == "sgd":
            fault.update(element_index=event // 2, reduction_index=0,
                         step="Multiply" if event % 2 == 0 else "Subtract")
        elif node.op == "mse":
            n = args[0].size
            if event == 3 * n:
                fault.update(element_index=0, reduction_index=n, step="Divide")
            else:
                fault.update(element_index=0, reduction_index=event // 3,
                             step=("Subtract", "Multiply", "Add")[event % 3])
        else:
            fault.update(element_index=event)
        return fault


def from_program(program):
    """Build a Graph from a reference_kats.json program; returns (graph, inputs dict)."""
    width = program["width"]
    g = Graph(width)
    inputs = {}
    utype = np.uint32 if width == 32 else np.uint64
    for name, spec in program["inputs"].items():
        g.input(name, spec["shape"])
        data = [int(b, 16) for b, n in spec["runs"] for _ in range(n)]
        inputs[name] = np.array(data, dtype=utype).view(g.dtype).reshape(spec["shape"])
    for entry in program["nodes"]:
        name, op, *rest = entry
        if op == "matmul":
            g.matmul(rest[0], rest[1], rest[2], rest[3], name=name)
        elif op == "sgd":
            g.sgd(rest[0], rest[1], rest[2], name=name)
        elif op == "mse":
            g.mse(rest[0], rest[1], name=name)
        elif op == "relu":
            g.relu(rest[0], name=name)
        elif op == "relu_backward":
            g.relu_backward(rest[0], rest[1], name=name)
        elif op == "gradient":
            g.gradient(rest[0], rest[1], name=name)
        else:
            g.binary(op, rest[0], rest[1], name=name)
    return g, inputs
