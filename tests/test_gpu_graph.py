"""Strict tensor graphs executed on the B200 through the native graph layer (pcu_b200_graph.h).

* every program of tests/golden/reference_kats.json (the reference's own end-to-end programs:
  training steps, gradients, first-fault cases) in both execution modes;
* the single-layer train step of the benchmark's first configuration (X 256x512, W 512x256,
  bias 256x256, target 256x256, lr 0.5, 10 steps) bit-exact against the oracle's graph;
* a scaled-down 4-layer MLP step (shared reverse sweep for all weights) against the oracle;
* first-fault-wins across nodes and fault locations lifted from MatMul / MSE / SGD nodes.
"""
import importlib

import numpy as np
import pytest

from gpu_util import FT, UT, dyadic_uniform
from oracle import graph as ograph

pytestmark = pytest.mark.gpu

graph_mod = importlib.import_module("fusion-pcu_b200.graph")
pcu = importlib.import_module("fusion-pcu_b200")


def _bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint32 if a.dtype == np.float32 else np.uint64)


def _expect_runs(expect):
    return [b for b, n in expect["runs"] for _ in range(n)]


@pytest.mark.parametrize("mode", ["each_node", "chained", "guarded", "graph"])
def test_reference_programs(kats, mode):
    for program in kats["programs"]:
        g, ids = graph_mod.from_program(program)
        _, inputs = ograph.from_program(program)
        prepared = g.prepare([ids[program["output"]]])
        feed = {ids[name]: arr for name, arr in inputs.items()}
        expect = program["expect"]
        if "runs" in expect:
            out = prepared.run(feed, [ids[program["output"]]], mode=mode)[ids[program["output"]]]
            assert [hex(v) for v in _bits(out).ravel()] == _expect_runs(expect), program["cite"]
            continue
        with pytest.raises(pcu.TensorError) as info:
            prepared.execute(feed, mode=mode)
        err = info.value
        if "fault" in expect:
            f = expect["fault"]
            assert err.value == ids[f["node"]], (program["cite"], err)
            assert (err.element_index, err.reduction_index, err.step, err.kind) == (
                f["element_index"], f["reduction_index"], f["step"], f["kind"]), (program["cite"], err)
        else:
            assert err.kind == expect["fault_kind"] and err.element_index == expect["element_index"], (
                program["cite"], err)


def _single_layer(width, policy=0):
    """Config 1's graph in the native layer and the oracle (same append order)."""
    n, o = graph_mod.Graph(width, policy), ograph.Graph(width)
    names = {}
    for name, shape in (("x", (256, 512)), ("w", (512, 256)), ("bias", (256, 256)), ("target", (256, 256))):
        names[name] = n.input(shape)
        o.input(name, shape)
    pre = n.matmul(names["x"], names["w"]); o.matmul("x", "w", name="pre")
    z = n.add(pre, names["bias"]); o.binary("add", "pre", "bias", name="z")
    y = n.relu(z); o.relu("z", name="y")
    loss = n.mean_squared_error(y, names["target"]); o.mse("y", "target", name="loss")
    gw = n.backward_mse_for(loss, names["w"]); o.gradient("loss", "w", name="gw")
    upd = n.sgd_update(names["w"], gw, 0.5); o.sgd("w", "gw", 0.5, name="updated")
    return n, o, names, loss, upd


@pytest.mark.parametrize("mode", ["each_node", "chained", "guarded", "graph"])
def test_single_layer_train_ten_steps_bit_exact(mode):
    rng = np.random.default_rng(20260101)
    x = dyadic_uniform(rng, (256, 512), 32)
    w = dyadic_uniform(rng, (512, 256), 32)
    bias = dyadic_uniform(rng, (256, 256), 32)
    target = dyadic_uniform(rng, (256, 256), 32, low=0.0)
    n, o, ids, loss, upd = _single_layer(32)
    prepared = n.prepare([upd, loss])
    w_dev, w_ref = w.copy(), w.copy()
    for step in range(10):
        got = prepared.run({ids["x"]: x, ids["w"]: w_dev, ids["bias"]: bias, ids["target"]: target}, [upd, loss],
                           mode=mode)
        want, fault = o.evaluate({"x": x, "w": w_ref, "bias": bias, "target": target}, ["updated", "loss"], 0,
                                 fast=True)
        assert fault is None
        assert np.array_equal(_bits(got[loss]), _bits(want["loss"])), step
        assert np.array_equal(_bits(got[upd]), _bits(want["updated"])), step
        w_dev, w_ref = got[upd], want["updated"]
    assert not np.array_equal(_bits(w_dev), _bits(w))


@pytest.mark.parametrize("width", [32, 64])
def test_mlp_step_shared_backward(width):
    """4 layers (64 -> 128 -> 128 -> 128 -> 32), batch 96: forward, one shared reverse sweep for
    all four weights, four SGD updates; every updated weight bit-exact."""
    rng = np.random.default_rng(404 + width)
    dims = [64, 128, 128, 128, 32]
    batch = 96
    n, o = graph_mod.Graph(width, 0), ograph.Graph(width)
    x = n.input((batch, dims[0])); o.input("x", (batch, dims[0]))
    feed_n, feed_o = {x: dyadic_uniform(rng, (batch, dims[0]), width)}, {}
    feed_o["x"] = feed_n[x]
    ws, wn = [], []
    h, hn = x, "x"
    for k in range(4):
        w = n.input((dims[k], dims[k + 1])); o.input(f"w{k}", (dims[k], dims[k + 1]))
        feed_n[w] = (dyadic_uniform(rng, (dims[k], dims[k + 1]), width) * FT[width](2.0 ** -3)).astype(FT[width])
        feed_o[f"w{k}"] = feed_n[w]
        ws.append(w); wn.append(f"w{k}")
        h = n.matmul(h, w); hn = o.matmul(hn, f"w{k}")
        if k < 3:
            h = n.relu(h); hn = o.relu(hn)
    t = n.input((batch, dims[-1])); o.input("t", (batch, dims[-1]))
    feed_n[t] = dyadic_uniform(rng, (batch, dims[-1]), width, low=0.0)
    feed_o["t"] = feed_n[t]
    loss = n.mean_squared_error(h, t); lo = o.mse(hn, "t")
    grads = n.backward_mse_for_targets(loss, ws)
    ogr = o.gradients(lo, wn)
    upd = [n.sgd_update(w, g, 1e-3) for w, g in zip(ws, grads)]
    oupd = [o.sgd(w, g, 1e-3) for w, g in zip(wn, ogr)]
    prepared = n.prepare(upd + [loss])
    for wait in (True, False):
        got = prepared.run(feed_n, upd + [loss], wait)
        want, fault = o.evaluate(feed_o, oupd + [lo], 0, fast=True)
        assert fault is None
        for a, b in zip(upd + [loss], oupd + [lo]):
            assert np.array_equal(_bits(got[a]), _bits(want[b])), (a, b)


@pytest.mark.parametrize("mode", ["each_node", "chained", "guarded", "graph"])
def test_first_faulting_node_wins(mode):
    """A later node that faults at a smaller element must not hide the earlier node's fault."""
    g = graph_mod.Graph(32, 0)
    a = g.input((64,))
    b = g.input((64,))
    c = g.input((64,))
    q = g.div(a, b)         # DivideByZero at element 40
    m = g.mul(c, c)         # ArithmeticOverflow at element 0 (a later node)
    prepared = g.prepare([m])
    av = np.ones(64, np.float32)
    bv = np.ones(64, np.float32)
    bv[40] = 0.0
    cv = np.ones(64, np.float32)
    cv[0] = 3e38
    with pytest.raises(pcu.ArithmeticFault) as info:
        prepared.execute({a: av, b: bv, c: cv}, mode=mode)
    assert (info.value.value, info.value.element_index, info.value.kind) == (q, 40, "DivideByZero")
    bv[40] = 1.0
    with pytest.raises(pcu.ArithmeticFault) as info:
        prepared.execute({a: av, b: bv, c: cv}, mode=mode)
    assert (info.value.value, info.value.element_index, info.value.kind) == (m, 0, "ArithmeticOverflow")
    cv[0] = 1.0
    prepared.execute({a: av, b: bv, c: cv}, mode=mode)
    bv[40] = 0.0  # a replay after a clean run reports the fault again
    with pytest.raises(pcu.ArithmeticFault) as info:
        prepared.execute({a: av, b: bv, c: cv}, mode=mode)
    assert (info.value.value, info.value.element_index, info.value.kind) == (q, 40, "DivideByZero")


@pytest.mark.parametrize("width", [32, 64])
@pytest.mark.parametrize("case", ["nan_in_x", "huge_in_w", "tiny_x", "inf_target"])
def test_train_step_fault_location_matches_oracle(width, case):
    rng = np.random.default_rng(7 + width)
    n, o = graph_mod.Graph(width, 1), ograph.Graph(width)
    shapes = {"x": (48, 40), "w": (40, 24), "t": (48, 24)}
    ids = {}
    for name, shape in shapes.items():
        ids[name] = n.input(shape)
        o.input(name, shape)
    pre = n.matmul(ids["x"], ids["w"]); o.matmul("x", "w", name="pre")
    y = n.relu(pre); o.relu("pre", name="y")
    loss = n.mean_squared_error(y, ids["t"]); o.mse("y", "t", name="loss")
    gw = n.backward_mse_for(loss, ids["w"]); o.gradient("loss", "w", name="gw")
    upd = n.sgd_update(ids["w"], gw, 0.25); o.sgd("w", "gw", 0.25, name="upd")
    data = {k: dyadic_uniform(rng, s, width) for k, s in shapes.items()}
    if case == "nan_in_x":
        data["x"][17, 9] = np.nan
    elif case == "huge_in_w":
        data["w"][5, 3] = FT[width](1e38 if width == 32 else 1e300)
        data["x"][:, 5] = FT[width](4.0)
    elif case == "tiny_x":
        data["x"] *= FT[width](2.0 ** (-120 if width == 32 else -1016))
    else:
        data["t"][5, 3] = np.inf
    prepared = n.prepare([upd])
    _, fault = o.evaluate({k: v for k, v in data.items()}, ["upd"], 1, fast=True)
    assert fault is not None
    for wait in (True, False):
        with pytest.raises(pcu.TensorError) as info:
            prepared.execute({ids[k]: v for k, v in data.items()}, wait)
        err = info.value
        assert o.index[fault["node"]] == err.value, (err, fault)
        assert err.kind == fault["kind"] and err.element_index == fault["element_index"], (err, fault)
        if "step" in fault:
            assert (err.reduction_index, err.step) == (fault["reduction_index"], fault["step"]), (err, fault)


@pytest.mark.parametrize("mode", ["guarded", "graph"])
def test_guarded_chain_skips_every_stage_after_the_first_fault(mode):
    """Guarded chain (owned_dispatch/guarded/guarded.rs:15-38): after a faulting stage, every
    later stage is skipped and touches nothing, so the outputs of a clean run stay in place even
    though the inputs changed; the records validate as the reference requires (stages in front
    executed, the faulting stage executed with its fault word, later stages skipped and clear)."""
    rng = np.random.default_rng(11)
    g = graph_mod.Graph(32, 0)
    a, b, c, t = g.input((16, 16)), g.input((16, 16)), g.input((16, 16)), g.input((16, 16))
    e = g.add(a, c)          # stage 0: clean
    q = g.div(e, b)          # stage 1: DivideByZero in the second run
    m = g.matmul(q, c)       # stage 2: depends on the fault
    r = g.relu(m)            # stage 3
    loss = g.mean_squared_error(r, t)  # stage 4
    z = g.mul(c, c)          # stage 5: independent of the fault, but later in the chain
    prepared = g.prepare([loss, z])
    feed = {v: dyadic_uniform(rng, (16, 16), 32) for v in (a, b, c, t)}
    feed[b] = np.abs(feed[b]) + np.float32(0.5)
    prepared.execute(feed, mode=mode)
    clean = {v: prepared.read(v) for v in (m, r, loss, z)}
    for v in (e, q, m, r, loss, z):
        assert prepared.stage(v) == (pcu.STATUS_OK, "executed")
    feed2 = dict(feed)
    feed2[c] = dyadic_uniform(rng, (16, 16), 32)
    feed2[b] = feed[b].copy()
    feed2[b][3, 5] = 0.0
    with pytest.raises(pcu.ArithmeticFault) as info:
        prepared.execute(feed2, mode=mode)
    assert (info.value.value, info.value.element_index, info.value.kind) == (q, 3 * 16 + 5, "DivideByZero")
    assert prepared.stage(e) == (pcu.STATUS_OK, "executed")
    word, disp = prepared.stage(q)
    assert disp == "executed" and word == ((3 * 16 + 5) << 3 | 1)
    for v in (m, r, loss, z):
        assert prepared.stage(v) == (pcu.STATUS_OK, "skipped"), v
        assert np.array_equal(_bits(prepared.read(v)), _bits(clean[v])), v
    # the chained mode runs every node: the later outputs move with the new inputs
    with pytest.raises(pcu.ArithmeticFault):
        prepared.execute(feed2, mode="chained")
    assert not np.array_equal(_bits(prepared.read(z)), _bits(clean[z]))
    # and a clean guarded run afterwards executes every stage again
    prepared.execute(feed, mode=mode)
    assert np.array_equal(_bits(prepared.read(z)), _bits(clean[z]))
    for v in (e, q, m, r, loss, z):
        assert prepared.stage(v) == (pcu.STATUS_OK, "executed")
