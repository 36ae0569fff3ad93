"""MSE and SGD in one pass (pcu_b200_strict_mse_sgd and its segment form) on a B200.

The two nodes are independent. Each keeps its own status word. The fused call must give exactly
what the oracle gives for each node run alone: the loss bits, every updated weight's bits and
both first faults. The SGD elements are split between the MSE chunk warps (a capped share per
warp) and the walker launch (at most a quarter of the node), so the cases cover:
* both shares, with faults in either;
* an SGD node far larger than the MSE (capped chunk-warp shares) and far smaller;
* no SGD at all;
* ragged sizes;
* operands that are not 16-byte aligned.
"""
import importlib

import numpy as np
import pytest

import oracle
from gpu_util import bits, dyadic_uniform, status_word, to_device, to_host

pytestmark = pytest.mark.gpu

pcu = importlib.import_module("fusion-pcu_b200")
RATE = 0.01


def _data(width, n_mse, n_sgd, seed):
    rng = np.random.default_rng(seed)
    p, t = dyadic_uniform(rng, n_mse, width), dyadic_uniform(rng, n_mse, width)
    w, g = dyadic_uniform(rng, n_sgd, width), dyadic_uniform(rng, n_sgd, width)
    return p, t, w, g


def _fused(p, t, w, g, offset=0):
    """Runs the fused call on device copies; `offset` elements in front make every operand
    start off the 16-byte grid."""
    import torch

    dev = [to_device(np.concatenate([np.zeros(offset, a.dtype), a]))[offset:] for a in (p, t, w, g)]
    upd_full = torch.empty(len(w) + offset, dtype=dev[2].dtype, device="cuda")
    upd = upd_full[offset:]
    ms, ss = pcu.new_status(), pcu.new_status()
    loss, _ = pcu.strict_mse_sgd(dev[0], dev[1], dev[2], dev[3], RATE, updated=upd, mse_status=ms, sgd_status=ss)
    torch.cuda.synchronize()
    return status_word(ms), bits(to_host(loss).reshape(1))[0], status_word(ss), bits(to_host(upd))


def _check(p, t, w, g, offset=0):
    mse_st, mse_out = oracle.mse(p, t)
    sgd_st, sgd_out = oracle.sgd(w, g, RATE)
    ms, loss, ss, upd = _fused(p, t, w, g, offset)
    assert ms == mse_st, (hex(ms), hex(mse_st))
    assert ss == sgd_st, (hex(ss), hex(sgd_st))
    if mse_st == oracle.STATUS_OK:
        assert loss == bits(mse_out)[0]
    if sgd_st == oracle.STATUS_OK:
        assert np.array_equal(upd, bits(sgd_out))
    return mse_st, sgd_st


SIZES = [
    (1000, 3000),
    (1 << 20, 1 << 20),
    (3 * 8192 + 777, 5 * 4096 + 13),
    (1 << 16, 1 << 24),   # chunk-warp shares capped, the rest beside the walker
    (1 << 22, 1 << 10),
    (4096, 0),
]


@pytest.mark.parametrize("width", [32, 64])
@pytest.mark.parametrize("sizes", SIZES, ids=[f"{a}x{b}" for a, b in SIZES])
def test_fused_clean_matches_oracle(width, sizes):
    p, t, w, g = _data(width, *sizes, seed=sizes[0] ^ sizes[1] ^ width)
    assert _check(p, t, w, g) == (oracle.STATUS_OK, oracle.STATUS_OK)


@pytest.mark.parametrize("width", [32, 64])
@pytest.mark.parametrize("case", ["sgd_early", "sgd_late", "sgd_both_steps", "mse_nan", "both_nodes", "unaligned"])
def test_fused_faults_match_oracle(width, case):
    n_mse, n_sgd = 1 << 20, (1 << 20) + 3
    p, t, w, g = _data(width, n_mse, n_sgd, seed=7 + width)
    offset = 0
    if case == "sgd_early":  # chunk-warp share; a later fault in the walker's share must lose
        g[1000] = np.inf
        w[n_sgd - 5] = np.nan
    elif case == "sgd_late":  # the walker's share only
        g[n_sgd - 2] = np.nan
    elif case == "sgd_both_steps":  # the multiply of one element against the subtract of an earlier one
        w[4096] = np.inf
        g[4097] = np.inf
    elif case == "mse_nan":
        p[123457] = np.nan
    elif case == "both_nodes":
        t[999999] = np.inf
        g[250000] = np.inf
        w[249999] = np.finfo(w.dtype).max
        g[249999] = -np.finfo(w.dtype).max  # w - rate * g overflows at the Subtract
    elif case == "unaligned":
        offset = 1
        g[77777] = np.inf
    mse_st, sgd_st = _check(p, t, w, g, offset)
    if case not in ("unaligned",):
        assert mse_st != oracle.STATUS_OK or sgd_st != oracle.STATUS_OK


@pytest.mark.parametrize("width", [32, 64])
def test_fused_segments_match_oracle(width):
    """Segment form: the MSE cut in three segments walked in order, the SGD cut in three blocks
    carried by the segments' chunk warps, one SGD status word shared (global events)."""
    import torch

    n_mse, n_sgd = 3 * 8192 + 777, 200003
    p, t, w, g = _data(width, n_mse, n_sgd, seed=99 + width)
    g[150001] = np.inf
    g[190000] = np.nan
    mse_st, mse_out = oracle.mse(p, t)
    sgd_st, _ = oracle.sgd(w, g, RATE)
    pd, td, wd, gd = (to_device(a) for a in (p, t, w, g))
    upd = torch.empty_like(wd)
    ms, ss = pcu.new_status(), pcu.new_status()
    carry = torch.zeros((), dtype=pd.dtype, device="cuda")
    mean = torch.zeros((), dtype=pd.dtype, device="cuda")
    mse_edges = [0, 5000, 8192 * 2 + 5, n_mse]
    sgd_edges = [0, 100000, 150000, n_sgd]
    for (a, b), (c, d) in zip(zip(mse_edges, mse_edges[1:]), zip(sgd_edges, sgd_edges[1:])):
        ps, ts = pd[a:b].contiguous(), td[a:b].contiguous()
        _, ws, _ = pcu.strict_mse_sgd_segment_prepare(ps, ts, a, wd[c:d], gd[c:d], RATE, c, updated=upd[c:d],
                                                      mse_status=ms, sgd_status=ss)
        pcu.strict_mse_segment_walk(ps, ts, a, n_mse, carry, ws, ms, out=mean if b == n_mse else None)
    torch.cuda.synchronize()
    assert status_word(ms) == mse_st == oracle.STATUS_OK
    assert bits(to_host(mean).reshape(1))[0] == bits(mse_out)[0]
    assert status_word(ss) == sgd_st != oracle.STATUS_OK
    # the elements in front of the first fault are updated exactly
    first = oracle.sgd_location(sgd_st)[0]
    _, ok_out = oracle.sgd(w[:first], g[:first], RATE)
    assert np.array_equal(bits(to_host(upd[:first])), bits(ok_out))


def test_large_mse_and_fused_match_oracle():
    """2^27 + 3 elements: the one-launch MSE then gives each chunk CTA several groups of chunks
    (one publication per 32 chunks), a path only large reductions take; the fused call carries an
    SGD node of the same size."""
    import torch

    n = (1 << 27) + 3
    p, t, w, g = _data(32, n, n, seed=271)
    mse_st, mse_out = oracle.mse(p, t)
    sgd_st, sgd_out = oracle.sgd(w, g, RATE)
    assert mse_st == sgd_st == oracle.STATUS_OK
    pd, td = to_device(p), to_device(t)
    status = pcu.new_status()
    loss = pcu.strict_mse(pd, td, status=status)
    torch.cuda.synchronize()
    assert status_word(status) == oracle.STATUS_OK
    assert bits(to_host(loss).reshape(1))[0] == bits(mse_out)[0]
    del p, t
    ms, loss2, ss, upd = _fused(*(a for a in (to_host(pd), to_host(td), w, g)))
    assert ms == ss == oracle.STATUS_OK
    assert loss2 == bits(mse_out)[0]
    assert np.array_equal(upd, bits(sgd_out))


@pytest.mark.parametrize("width", [32, 64])
@pytest.mark.parametrize("case", ["clean", "mse_fault_first_segment", "mse_fault_later", "sgd_fault"])
def test_one_call_first_segment_then_walks(width, case):
    """The first segment in one call (pcu_b200_strict_mse_sgd_segment: maps and walk together,
    from +0), the others prepared and walked with the carried sum, SGD blocks riding along: the
    split reduction must give the oracle's mean and first faults."""
    import torch

    n_mse, n_sgd = 5 * 8192 + 321, 120007
    p, t, w, g = _data(width, n_mse, n_sgd, seed=311 + width)
    if case == "mse_fault_first_segment":
        p[7000] = np.nan
    elif case == "mse_fault_later":
        t[30000] = np.inf
    elif case == "sgd_fault":
        g[100] = np.inf
    mse_st, mse_out = oracle.mse(p, t)
    sgd_st, sgd_out = oracle.sgd(w, g, RATE)
    pd, td, wd, gd = (to_device(a) for a in (p, t, w, g))
    upd = torch.empty_like(wd)
    ms, ss = pcu.new_status(), pcu.new_status()
    carry = torch.zeros((), dtype=pd.dtype, device="cuda")
    mean = torch.zeros((), dtype=pd.dtype, device="cuda")
    mse_edges, sgd_edges = [0, 9000, 8192 * 3 + 7, n_mse], [0, 50000, 50001, n_sgd]
    for k, ((a, b), (c, d)) in enumerate(zip(zip(mse_edges, mse_edges[1:]), zip(sgd_edges, sgd_edges[1:]))):
        ps, ts = pd[a:b].contiguous(), td[a:b].contiguous()
        ws = pcu.mse_workspace(ps)
        rider = {"weights": wd[c:d], "gradient": gd[c:d], "rate": RATE, "first_index": c, "out": upd[c:d],
                 "status": ss}
        if k == 0:
            pcu.strict_mse_sgd_segment(ps, ts, a, n_mse, None, carry, ws, ms, sgd=rider)
        else:
            pcu.strict_mse_sgd_segment_prepare(ps, ts, a, wd[c:d], gd[c:d], RATE, c, updated=upd[c:d],
                                               mse_status=ms, sgd_status=ss, workspace=ws)
            pcu.strict_mse_segment_walk(ps, ts, a, n_mse, carry, ws, ms, out=mean if b == n_mse else None)
    torch.cuda.synchronize()
    assert status_word(ms) == mse_st, (hex(status_word(ms)), hex(mse_st))
    assert status_word(ss) == sgd_st
    if mse_st == oracle.STATUS_OK:
        assert bits(to_host(mean).reshape(1))[0] == bits(mse_out)[0]
    if sgd_st == oracle.STATUS_OK:
        assert np.array_equal(bits(to_host(upd)), bits(sgd_out))


def test_bench_workload_matches_oracle():
    """BASELINE configuration 5 exactly as bench.py times it: 2^28 binary32 elements per array,
    drawn on the device by the bench's generator (seeds 11..14: weights, gradient, prediction,
    target; k * 2^-23 with k uniform in [-2^23, 2^23)), lr = f32(0.01).  The fused call's mean and
    updated weights equal the oracle's bit for bit."""
    import torch

    n = 1 << 28

    def block(seed):
        gen = torch.Generator(device="cuda")
        gen.manual_seed(seed)
        k = torch.randint(-(1 << 23), 1 << 23, (n,), generator=gen, device="cuda", dtype=torch.int32)
        return k.to(torch.float32) * (2.0 ** -23)

    w, g, p, t = block(11), block(12), block(13), block(14)
    ms, ss = pcu.new_status(), pcu.new_status()
    loss, upd = pcu.strict_mse_sgd(p, t, w, g, RATE, mse_status=ms, sgd_status=ss)
    torch.cuda.synchronize()
    assert status_word(ms) == status_word(ss) == oracle.STATUS_OK
    loss_bits, upd_bits = bits(to_host(loss).reshape(1))[0], bits(to_host(upd))
    del upd
    mse_st, mse_out = oracle.mse(to_host(p), to_host(t))
    assert mse_st == oracle.STATUS_OK and loss_bits == bits(mse_out)[0]
    del p, t
    sgd_st, sgd_out = oracle.sgd(to_host(w), to_host(g), RATE)
    assert sgd_st == oracle.STATUS_OK and np.array_equal(upd_bits, bits(sgd_out))
