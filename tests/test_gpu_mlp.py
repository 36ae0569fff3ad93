"""The full-size 4-layer MLP training step of the benchmark's fourth configuration on a B200.

Configuration: input 1024 -> 4096 -> 4096 -> 4096 -> 256, batch 8192, ReLU after the hidden
layers, strict MSE against a U[0,1) target, one shared reverse sweep for the four weights and a
strict SGD update of each (rate binary32(1e-3)); He-uniform weights (bound binary32(sqrt(6 /
fan_in)) times a dyadic U[-1,1)) and dyadic U[-1,1) inputs from a seed.  About 1.8e12 checked
flops, far beyond the CPU oracle, so parity is checked node by node: every node of the plan is
run on the device, its inputs and output are read back, and the oracle recomputes a seeded
sample of its outputs (MatMul cells, elementwise elements; the MSE in full) from the device
inputs.  Every sampled output must match bit for bit and every status word must be clean.
"""
import importlib

import numpy as np
import pytest

import oracle
from gpu_util import dyadic_uniform

pytestmark = pytest.mark.gpu

graph_mod = importlib.import_module("fusion-pcu_b200.graph")

DIMS = [1024, 4096, 4096, 4096, 256]
BATCH = 8192


def _bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint32 if a.dtype == np.float32 else np.uint64)


def _mlp_graph():
    g = graph_mod.Graph(32, 0)
    x = g.input((BATCH, DIMS[0]))
    ws = [g.input((DIMS[k], DIMS[k + 1])) for k in range(4)]
    t = g.input((BATCH, DIMS[-1]))
    h = x
    for k, w in enumerate(ws):
        h = g.matmul(h, w)
        if k < 3:
            h = g.relu(h)
    loss = g.mean_squared_error(h, t)
    grads = g.backward_mse_for_targets(loss, ws)
    updates = [g.sgd_update(w, d, 1e-3) for w, d in zip(ws, grads)]
    return g, x, ws, t, loss, updates


def test_mlp_step_full_size_node_parity():
    rng = np.random.default_rng(2026)
    g, x, ws, t, loss, updates = _mlp_graph()
    feed = {x: dyadic_uniform(rng, (BATCH, DIMS[0]), 32), t: dyadic_uniform(rng, (BATCH, DIMS[-1]), 32, low=0.0)}
    for k, w in enumerate(ws):
        bound = np.float32(np.sqrt(6.0 / DIMS[k]))
        feed[w] = (dyadic_uniform(rng, (DIMS[k], DIMS[k + 1]), 32) * bound).astype(np.float32)
    prepared = g.prepare(updates + [loss])
    prepared.execute(feed, wait_each_node=False)  # raises on any fault

    values = {}

    def value(v):
        if v not in values:
            values[v] = prepared.read(v)
        return values[v]

    sample = np.random.default_rng(7)
    checked = {"matmul": 0, "elementwise": 0, "mse": 0, "sgd": 0}
    for v in range(len(g)):
        op, left, right, tl, tr, shape, bits = g.describe(v)
        if op in ("input", "uniform") or not prepared.buffer(v):
            continue
        out = value(v)
        if op == "matmul":
            a, b = value(left), value(right)
            cells = sample.choice(out.size, size=48, replace=False)
            st, want = oracle.matmul_cells(a, b, cells, tl, tr)
            assert st == oracle.STATUS_OK, (v, op)
            assert np.array_equal(_bits(out.ravel()[cells]), _bits(want)), (v, op, shape)
            checked["matmul"] += 1
        elif op == "mean_squared_error":
            st, want = oracle.mse(value(left).ravel(), value(right).ravel())
            assert st == oracle.STATUS_OK
            assert _bits(out.reshape(1))[0] == _bits(want)[0]
            checked["mse"] += 1
        else:
            idx = np.sort(sample.choice(out.size, size=min(4096, out.size), replace=False))
            a = value(left).ravel()
            b = value(right).ravel() if right >= 0 else None
            if op == "sgd_update":
                rate = np.array([bits], dtype=np.uint32).view(np.float32)[0]
                st, want = oracle.sgd(a[idx], b[idx], rate)
                checked["sgd"] += 1
            elif op == "relu":
                st, want = oracle.relu(a[idx])
                checked["elementwise"] += 1
            elif op == "relu_backward":
                st, want = oracle.relu_backward(a[idx], b[idx])
                checked["elementwise"] += 1
            else:
                uni_b = g.describe(right)[0] == "uniform"
                st, want = oracle.binary(op, a[idx], b[:1] if uni_b else b[idx], right_uniform=uni_b)
                checked["elementwise"] += 1
            assert st == oracle.STATUS_OK, (v, op)
            assert np.array_equal(_bits(out.ravel()[idx]), _bits(want)), (v, op, shape)
        if len(values) > 12:  # keep host memory bounded: drop what later nodes no longer read
            for key in list(values)[:-8]:
                del values[key]
    # forward 4 MatMuls, backward 3 for the hidden gradients and 4 for the weights
    assert checked["matmul"] == 11 and checked["mse"] == 1 and checked["sgd"] == 4
    assert checked["elementwise"] >= 8
    # the weights moved
    for w, u in zip(ws, updates):
        assert not np.array_equal(_bits(value(u)), _bits(feed[w]))
