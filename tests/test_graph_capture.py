"""The native graph layer's capture, reverse mode and plan against the oracle's restatement.

Capture and reverse mode are host code in libpcu_b200.so (no GPU is touched), so these run on
the CPU: every program of tests/golden/reference_kats.json, plus hand-built graphs that reach
each reverse-mode rule of gradients.rs (transposed MatMuls, Sub on the right, SGD on both
operands, shared values), must produce the oracle's node list node for node.
"""
import importlib

import numpy as np
import pytest

from oracle import graph as ograph

graph_mod = importlib.import_module("fusion-pcu_b200.graph")

OP_NAMES = {"input": "input", "uniform": "uniform", "add": "add", "sub": "sub", "mul": "mul", "div": "div",
            "relu": "relu", "relu_backward": "relu_backward", "matmul": "matmul", "mse": "mean_squared_error",
            "sgd": "sgd_update"}


def _rate_bits(rate):
    return int(np.array([rate], dtype=np.float32).view(np.uint32)[0])


def assert_same_nodes(native, oracle_graph):
    assert len(native) == len(oracle_graph.nodes)
    for i, node in enumerate(oracle_graph.nodes):
        op, left, right, tl, tr, shape, bits = native.describe(i)
        args = [oracle_graph.index[a] for a in node.args]
        assert op == OP_NAMES[node.op], (i, node, op)
        assert [a for a in (left, right) if a >= 0] == args, (i, node, left, right)
        assert shape == tuple(node.shape), (i, node, shape)
        if node.op == "matmul":
            assert (tl, tr) == (bool(node.tl), bool(node.tr)), (i, node)
        if node.op == "uniform":
            assert bits == node.value, (i, node, hex(bits), hex(node.value))
        if node.op == "sgd":
            assert bits == _rate_bits(node.rate), (i, node)


def test_reference_programs_capture_like_the_oracle(kats):
    for program in kats["programs"]:
        native, ids = graph_mod.from_program(program)
        og, _ = ograph.from_program(program)
        assert_same_nodes(native, og)
        for name, v in ids.items():
            assert og.index[name] == v, (program["cite"], name)


class Both:
    """Builds the same graph in the native layer and in the oracle."""

    def __init__(self, width):
        self.n = graph_mod.Graph(width, 0)
        self.o = ograph.Graph(width)
        self.names = []

    def _name(self, v):
        while len(self.names) < len(self.o.nodes):
            self.names.append(self.o.nodes[len(self.names)].name)
        return self.names[v]

    def input(self, shape):
        v = self.n.input(shape)
        self.o.input(f"in{v}", shape)
        return v

    def op(self, kind, *args, **kw):
        nv = {
            "matmul": lambda: self.n.matmul_transposed(args[0], args[1], kw.get("tl", False), kw.get("tr", False)),
            "relu": lambda: self.n.relu(args[0]),
            "mse": lambda: self.n.mean_squared_error(*args),
            "sgd": lambda: self.n.sgd_update(args[0], args[1], kw["rate"]),
            "gradient": lambda: self.n.backward_mse_for(*args),
        }.get(kind, lambda: self.n.binary(kind, *args))()
        names = [self._name(a) for a in args]
        if kind == "matmul":
            self.o.matmul(names[0], names[1], kw.get("tl", False), kw.get("tr", False))
        elif kind == "relu":
            self.o.relu(names[0])
        elif kind == "mse":
            self.o.mse(*names)
        elif kind == "sgd":
            self.o.sgd(names[0], names[1], kw["rate"])
        elif kind == "gradient":
            result = self.o.gradient(*names)
            assert self.o.index[result] == nv
        else:
            self.o.binary(kind, *names)
        assert_same_nodes(self.n, self.o)
        return nv


@pytest.mark.parametrize("width", [32, 64])
@pytest.mark.parametrize("tl,tr", [(False, False), (True, False), (False, True), (True, True)])
def test_matmul_gradients_every_transpose(width, tl, tr):
    b = Both(width)
    x = b.input((6, 4) if tl else (4, 6))
    w = b.input((3, 6) if tr else (6, 3))
    t = b.input((4, 3))
    y = b.op("matmul", x, w, tl=tl, tr=tr)
    h = b.op("relu", y)
    loss = b.op("mse", h, t)
    b.op("gradient", loss, w)
    b.op("gradient", loss, x)
    b.op("gradient", loss, t)


@pytest.mark.parametrize("width", [32, 64])
def test_sub_sgd_and_shared_values(width):
    b = Both(width)
    x = b.input((5,))
    w = b.input((5,))
    g = b.input((5,))
    t = b.input((5,))
    s = b.op("sgd", w, g, rate=0.1)
    d = b.op("sub", x, s)
    m = b.op("mul", d, d)
    a = b.op("add", m, x)
    loss = b.op("mse", a, t)
    for target in (w, g, x, t, s, d, m, a, loss):
        b.op("gradient", loss, target)


def test_capture_errors():
    g = graph_mod.Graph(32, 0)
    a = g.input((2, 3))
    c = g.input((3, 2))
    with pytest.raises(graph_mod.GraphError, match="ShapeMismatch"):
        g.add(a, c)
    with pytest.raises(graph_mod.GraphError, match="MatMulShape"):
        g.matmul(a, a)
    with pytest.raises(graph_mod.GraphError, match="UnknownValue"):
        g.relu(99)
    with pytest.raises(graph_mod.GraphError, match="InvalidLearningRate"):
        g.sgd_update(a, a, float("inf"))
    with pytest.raises(graph_mod.GraphError, match="GradientRootNotMse"):
        g.backward_mse_for(a, a)
    q = g.div(a, a)
    loss = g.mean_squared_error(q, a)
    with pytest.raises(graph_mod.GraphError, match="UnsupportedGradient"):
        g.backward_mse_for(loss, a)
    other = g.input((2, 3))
    loss2 = g.mean_squared_error(g.relu(a), a)
    with pytest.raises(graph_mod.GraphError, match="UnsupportedGradient"):
        g.backward_mse_for(loss2, other)


@pytest.mark.parametrize("width", [32, 64])
def test_shared_sweep_for_several_targets(width):
    """backward_mse_for_targets: a 3-layer MLP differentiated once for all weights."""
    n = graph_mod.Graph(width, 0)
    o = ograph.Graph(width)
    x = n.input((8, 6)); o.input("x", (8, 6))
    ws, names = [], []
    h, hn = x, "x"
    for k, (a, b) in enumerate([(6, 5), (5, 4), (4, 3)]):
        w = n.input((a, b)); o.input(f"w{k}", (a, b))
        ws.append(w); names.append(f"w{k}")
        h = n.matmul(h, w); hn = o.matmul(hn, f"w{k}")
        if k < 2:
            h = n.relu(h); hn = o.relu(hn)
    t = n.input((8, 3)); o.input("t", (8, 3))
    loss = n.mean_squared_error(h, t); lo = o.mse(hn, "t")
    got = n.backward_mse_for_targets(loss, ws + [ws[0]])
    want = o.gradients(lo, names + [names[0]])
    assert got == [o.index[w] for w in want]
    assert got[0] == got[-1]
    assert_same_nodes(n, o)
    with pytest.raises(graph_mod.GraphError, match="EmptyOutputs"):
        n.backward_mse_for_targets(loss, [])
