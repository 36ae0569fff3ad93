"""MatMul with elementwise nodes fused into its epilogue (pcu_b200_strict_matmul_epilogue) and the
chained graph mode that uses it.

Every fused node keeps its own output and status word, so the result of a fused call must equal,
bit for bit and word for word, the MatMul followed by the same nodes run one by one: every output
when nothing faults, and the first faulting node's word when something does (a fault in the
MatMul is reported before one in a fused node; a fault in the Add before one in the ReLU).  The
graph tests check that the chained mode really fuses the single-layer step's Add and ReLU into the
MatMul and still reports a fault in them as the unfused node and element.
"""
import importlib

import numpy as np
import pytest

import oracle
from gpu_util import FT, bits, dyadic_uniform, status_word, to_device, to_host

pytestmark = pytest.mark.gpu

pcu = importlib.import_module("fusion-pcu_b200")
graph_mod = importlib.import_module("fusion-pcu_b200.graph")


def _unfused(a, b, tl, tr, plan, policy):
    """The MatMul, then each node in `plan` one by one; (outputs, status words)."""
    st = [pcu.new_status() for _ in range(len(plan) + 1)]
    z = pcu.strict_matmul(a, b, tl, tr, policy, status=st[0])
    outs, value = [z], z
    for k, (op, operand, left) in enumerate(plan):
        if op == "relu":
            value = pcu.checked_relu(value, policy, status=st[k + 1])
        elif op == "relu_backward":
            x, dy = (operand, value) if left else (value, operand)
            value = pcu.checked_relu_backward(x, dy, policy, status=st[k + 1])
        else:
            uniform = operand.numel() == 1
            lhs, rhs = (operand, value) if left else (value, operand)
            value = pcu.checked_binary(op, lhs, rhs, policy, left_uniform=uniform and left,
                                       right_uniform=uniform and not left, status=st[k + 1])
        outs.append(value)
    return outs, st


def _fused(a, b, tl, tr, plan, policy):
    import torch

    st = [pcu.new_status() for _ in range(len(plan) + 1)]
    rows = a.shape[1] if tl else a.shape[0]
    cols = b.shape[0] if tr else b.shape[1]
    outs = [torch.full((rows, cols), 7.0, dtype=a.dtype, device="cuda") for _ in range(len(plan))]
    stages = [{"op": op, "operand": operand, "operand_left": left, "out": outs[k], "status": st[k + 1]}
              for k, (op, operand, left) in enumerate(plan)]
    z = pcu.strict_matmul_epilogue(a, b, stages, tl, tr, policy, status=st[0])
    return [z] + outs, st


def _compare(a, b, tl, tr, plan, policy=0):
    import torch

    want, ws = _unfused(a, b, tl, tr, plan, policy)
    got, gs = _fused(a, b, tl, tr, plan, policy)
    torch.cuda.synchronize()
    words_w, words_g = [status_word(s) for s in ws], [status_word(s) for s in gs]
    # the first faulting node (in order) and its word are the same
    first_w = next((i for i, w in enumerate(words_w) if w != pcu.STATUS_OK), None)
    first_g = next((i for i, w in enumerate(words_g) if w != pcu.STATUS_OK), None)
    assert first_w == first_g, (words_w, words_g)
    if first_w is None:
        for w, g in zip(want, got):
            assert np.array_equal(bits(to_host(w)), bits(to_host(g)))
    else:
        assert words_w[first_w] == words_g[first_w], (first_w, hex(words_w[first_w]), hex(words_g[first_w]))
        for i in range(first_w):  # nodes in front of the fault are complete and equal
            assert np.array_equal(bits(to_host(want[i])), bits(to_host(got[i])))
    return first_w


@pytest.mark.parametrize("width", [32, 64])
@pytest.mark.parametrize("shape", [(256, 512, 256), (1024, 96, 1024), (300, 40, 200)])
def test_bias_relu_epilogue_matches_the_nodes_one_by_one(width, shape):
    """The forward layer of the single-layer step: Add(bias) then ReLU, on the 16x16-tile kernel
    (256 x 256 output), the TMA kernel (1024 x 1024) and a ragged shape."""
    m, k, n = shape
    rng = np.random.default_rng(m + k + n + width)
    a = to_device(dyadic_uniform(rng, (m, k), width))
    b = to_device(dyadic_uniform(rng, (k, n), width))
    bias = dyadic_uniform(rng, (m, n), width)
    assert _compare(a, b, False, False, [("add", to_device(bias), False), ("relu", None, False)]) is None
    # faults: the Add (a NaN bias element, and an overflow against a huge bias), the MatMul (a NaN
    # in A, with a NaN in the bias too: the MatMul is reported)
    for case in ("bias_nan", "bias_overflow", "matmul_first"):
        bb = bias.copy()
        aa, b2 = to_host(a).copy(), to_host(b).copy()
        if case == "bias_nan":
            bb[m // 2, n - 1] = np.nan
        elif case == "bias_overflow":
            # one product cell of at least half an ulp of MAX, positive, beside a MAX bias: the
            # MatMul is finite, the Add overflows
            bb[m - 1, 3] = np.finfo(FT[width]).max
            aa[m - 1, :] = FT[width](2.0 ** (105 if width == 32 else 980))
            b2[:, 3] = 0.5
        else:
            aa[m // 3, 5] = np.nan
            bb[1, 1] = np.nan
        first = _compare(to_device(aa), to_device(b2), False, False,
                         [("add", to_device(bb), False), ("relu", None, False)])
        assert first == (0 if case == "matmul_first" else 1), case


@pytest.mark.parametrize("width", [32, 64])
@pytest.mark.parametrize("tl,tr", [(False, True), (True, False)])
def test_relu_backward_epilogue(width, tl, tr):
    """The backward pattern: dH = G . W^T (NT) then ReLU-backward against the forward
    pre-activation, with the product as the upstream gradient (and the reverse operand order);
    a NaN in the forward input faults the fused node at its element."""
    rng = np.random.default_rng(77 + width + 2 * tl + tr)
    m, k, n = 512, 64, 768
    a = dyadic_uniform(rng, (k, m) if tl else (m, k), width)
    b = dyadic_uniform(rng, (n, k) if tr else (k, n), width)
    x = dyadic_uniform(rng, (m, n), width)
    ad, bd = to_device(a), to_device(b)
    assert _compare(ad, bd, tl, tr, [("relu_backward", to_device(x), True)]) is None
    assert _compare(ad, bd, tl, tr, [("relu_backward", to_device(x), False)]) is None
    x[100, 700] = np.nan
    assert _compare(ad, bd, tl, tr, [("relu_backward", to_device(x), True)]) == 1


@pytest.mark.parametrize("policy", [0, 1, 2])
def test_uniform_operand_and_policies(policy):
    """A uniform left operand (Sub with a constant on the left), then Mul by a uniform scale, under
    each underflow policy, with values near the smallest normal."""
    import torch

    rng = np.random.default_rng(900 + policy)
    a = dyadic_uniform(rng, (200, 48), 32) * np.float32(2.0 ** -60)
    b = dyadic_uniform(rng, (48, 136), 32) * np.float32(2.0 ** -60)
    c = torch.tensor([np.float32(2.0 ** -125)], device="cuda")
    s = torch.tensor([np.float32(0.75)], device="cuda")
    _compare(to_device(a), to_device(b), False, False, [("sub", c, True), ("mul", s, False)], policy)


def test_rejects_bad_epilogues(provider):
    import ctypes

    lib = provider.library()
    st = pcu.new_status()
    dev = ctypes.c_void_p(256)
    stages = (pcu.EpilogueStage * 3)()
    for i in range(3):
        stages[i].op, stages[i].operand, stages[i].out, stages[i].status = 0, 256, 256, st.data_ptr()
    args = (0, 0, dev, dev, dev, 4, 4, 4, 4, 4, 0, 0)
    assert lib.pcu_b200_strict_matmul_epilogue(*args, stages, 3, None, 0, st.data_ptr(), None) == 1  # too many
    stages[0].op = 9
    assert lib.pcu_b200_strict_matmul_epilogue(*args, stages, 1, None, 0, st.data_ptr(), None) == 1  # bad op
    stages[0].op, stages[0].operand = 0, None
    assert lib.pcu_b200_strict_matmul_epilogue(*args, stages, 1, None, 0, st.data_ptr(), None) == 1  # no operand


def _single_layer_graph(bias_fault=None):
    rng = np.random.default_rng(20260101)
    x = dyadic_uniform(rng, (256, 512), 32)
    w = dyadic_uniform(rng, (512, 256), 32)
    bias = dyadic_uniform(rng, (256, 256), 32)
    target = dyadic_uniform(rng, (256, 256), 32, low=0.0)
    if bias_fault:
        bias[bias_fault] = np.inf
    g = graph_mod.Graph(32, 0)
    gx, gw, gb, gt = g.input(x.shape), g.input(w.shape), g.input(bias.shape), g.input(target.shape)
    pre = g.matmul(gx, gw)
    z = g.add(pre, gb)
    y = g.relu(z)
    loss = g.mean_squared_error(y, gt)
    upd = g.sgd_update(gw, g.backward_mse_for(loss, gw), 0.5)
    return g, {gx: x, gw: w, gb: bias, gt: target}, pre, z, y, loss, upd


def test_chained_mode_fuses_the_single_layer_step():
    g, feed, pre, z, y, loss, upd = _single_layer_graph()
    prepared = g.prepare([upd, loss])
    assert prepared.fused(pre) == 2  # the Add and the ReLU run in the MatMul's epilogue
    results = {}
    for mode in ("each_node", "chained", "graph"):
        results[mode] = prepared.run(feed, [upd, loss, y, z], mode=mode)
    for v in (upd, loss, y, z):
        assert np.array_equal(_bits(results["chained"][v]), _bits(results["each_node"][v]))
        assert np.array_equal(_bits(results["chained"][v]), _bits(results["graph"][v]))


def _bits(arr):
    arr = np.ascontiguousarray(arr)
    return arr.view(np.uint32 if arr.dtype == np.float32 else np.uint64)


@pytest.mark.parametrize("where", [(3, 7), (255, 0), (128, 255)])
def test_fault_in_fused_add_reports_the_unfused_node(where):
    g, feed, pre, z, y, loss, upd = _single_layer_graph(bias_fault=where)
    prepared = g.prepare([upd, loss])
    assert prepared.fused(pre) == 2
    errors = {}
    for mode in ("each_node", "chained", "guarded"):
        with pytest.raises(pcu.TensorError) as info:
            prepared.execute(feed, mode=mode)
        e = info.value
        errors[mode] = (e.value, e.element_index, e.kind)
    assert errors["chained"] == errors["each_node"] == errors["guarded"] == (z, where[0] * 256 + where[1],
                                                                               "InvalidFloatingOperand")
