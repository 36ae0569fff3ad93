"""Guarded chains of node calls (pcu_b200_guarded_*, pcu_b200_chain_reset/_validate) and
pcu_b200_wait on the B200.

The guarded kernel ABI is the reference's (Crates/backends/cuda/owned_dispatch/guarded/guarded.rs,
guarded_source): stage s is admitted when s == 0 or record s-1 is [clear word, executed]; an
admitted stage computes exactly what the unguarded call computes, and a skipped one writes nothing.
The unguarded calls are pinned to the oracle by the parity tests; here the guarded ones must equal
them bit for bit, fault words included.
"""
import numpy as np
import pytest

from gpu_util import bits, dyadic_uniform, status_word, to_device, to_host

pytestmark = pytest.mark.gpu

ROWS, INNER, COLS = 64, 48, 32
RATE = 0.5


def _inputs(width, seed):
    rng = np.random.default_rng(seed)
    return {
        "x": dyadic_uniform(rng, (ROWS, INNER), width),
        "w": dyadic_uniform(rng, (INNER, COLS), width),
        "bias": dyadic_uniform(rng, (ROWS, COLS), width),
        "t": dyadic_uniform(rng, (ROWS, COLS), width, low=0.0),
        "sw": dyadic_uniform(rng, (INNER, COLS), width),
        "sg": dyadic_uniform(rng, (INNER, COLS), width),
    }


EXTENTS = [ROWS * COLS * INNER * 2, ROWS * COLS, ROWS * COLS, 3 * ROWS * COLS + 1, 2 * INNER * COLS, 0]


def _unguarded(pcu, d):
    """The six stages as plain node calls: (outputs, status words)."""
    outs, words = [], []

    def run(fn, *a, **k):
        st = pcu.new_status()
        outs.append(fn(*a, status=st, **k))
        words.append(status_word(st))
        return outs[-1]

    z = run(pcu.strict_matmul, d["x"], d["w"])
    a = run(pcu.checked_relu, z)
    y = run(pcu.checked_binary, "add", a, d["bias"])
    run(pcu.strict_mse, y, d["t"])
    run(pcu.strict_sgd, d["sw"], d["sg"], RATE)
    run(pcu.checked_relu, d["x"][:0])
    return outs, words


def _guarded(pcu, d, sentinel):
    """The same six stages as one guarded chain; every output pre-filled with `sentinel`."""
    import torch

    chain = pcu.GuardedChain(6).reset()
    dt = d["x"].dtype
    outs = [torch.full((ROWS, COLS), sentinel, dtype=dt, device="cuda"),
            torch.full((ROWS, COLS), sentinel, dtype=dt, device="cuda"),
            torch.full((ROWS, COLS), sentinel, dtype=dt, device="cuda"),
            torch.full((), sentinel, dtype=dt, device="cuda"),
            torch.full((INNER, COLS), sentinel, dtype=dt, device="cuda"),
            torch.empty((0, INNER), dtype=dt, device="cuda")]
    pcu.strict_matmul(d["x"], d["w"], out=outs[0], chain=chain.stage(0))
    pcu.checked_relu(outs[0], out=outs[1], chain=chain.stage(1))
    pcu.checked_binary("add", outs[1], d["bias"], out=outs[2], chain=chain.stage(2))
    pcu.strict_mse(outs[2], d["t"], out=outs[3], chain=chain.stage(3))
    pcu.strict_sgd(d["sw"], d["sg"], RATE, out=outs[4], chain=chain.stage(4))
    pcu.checked_relu(d["x"][:0], out=outs[5], chain=chain.stage(5))
    return chain, outs


@pytest.mark.parametrize("width", [32, 64])
def test_clean_chain_equals_the_unguarded_calls(provider, width):
    pcu = provider
    d = {k: to_device(v) for k, v in _inputs(width, 5).items()}
    ref, words = _unguarded(pcu, d)
    assert all(w == pcu.STATUS_OK for w in words)
    chain, outs = _guarded(pcu, d, 7.0)
    outcome, stage, word = chain.validate(EXTENTS)
    assert (outcome, stage, word) == ("succeeded", 0, pcu.STATUS_OK)
    recs = chain.read()
    assert list(recs[1::2]) == [1] * 6 and all(int(w) == pcu.STATUS_OK for w in recs[0::2])
    for got, want in zip(outs, ref):
        assert np.array_equal(bits(to_host(got)), bits(to_host(want)))


def _poison(d, stage, width):
    """Inputs whose first fault is at `stage` (NaN operand -> InvalidFloatingOperand)."""
    h = {k: to_host(v).copy() for k, v in d.items()}
    if stage == 0:
        h["x"][5, 7] = np.nan
    elif stage == 2:
        h["bias"][9, 3] = np.inf
    elif stage == 3:
        h["t"][12, 30] = np.nan
    return {k: to_device(v) for k, v in h.items()}


@pytest.mark.parametrize("width", [32, 64])
@pytest.mark.parametrize("stage", [0, 2, 3])
def test_first_fault_skips_every_later_stage(provider, width, stage):
    pcu = provider
    d = _poison({k: to_device(v) for k, v in _inputs(width, 9).items()}, stage, width)
    ref, words = _unguarded(pcu, d)
    assert words[stage] != pcu.STATUS_OK and all(w == pcu.STATUS_OK for w in words[:stage])
    sentinel = 1234.5
    chain, outs = _guarded(pcu, d, sentinel)
    outcome, got_stage, word = chain.validate(EXTENTS)
    assert (outcome, got_stage, word) == ("fault", stage, words[stage])
    recs = chain.read()
    assert list(recs[1::2]) == [1] * (stage + 1) + [2] * (5 - stage)
    assert all(int(w) == pcu.STATUS_OK for w in recs[2 * stage + 2::2])
    for s in range(stage):  # stages in front ran as usual
        assert np.array_equal(bits(to_host(outs[s])), bits(to_host(ref[s])))
    for s in range(stage + 1, 5):  # skipped stages wrote nothing
        assert np.all(to_host(outs[s]) == sentinel), s


def test_an_empty_stage_is_skipped_after_a_fault_too(provider):
    import torch

    pcu = provider
    chain = pcu.GuardedChain(2).reset()
    x = torch.tensor([1.0, float("nan"), 2.0], device="cuda")
    pcu.checked_relu(x, chain=chain.stage(0))
    pcu.checked_relu(x[:0], chain=chain.stage(1))
    recs = chain.read()
    assert int(recs[0]) == (1 << 3) | 5 and list(recs[1::2]) == [1, 2]
    assert chain.validate()[:2] == ("fault", 0)


def test_wait_times_out_on_running_work_then_completes(provider):
    import torch

    pcu = provider
    rng = np.random.default_rng(3)
    a = to_device(dyadic_uniform(rng, (4096, 4096), 32))
    out = torch.empty_like(a)
    pcu.strict_matmul(a, a, out=out)  # one-time host set-up outside the measured part
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    for _ in range(3):  # about 14 ms of device work
        pcu.strict_matmul(a, a, out=out, stream=stream)
    assert pcu.wait(stream, timeout_ms=0) is False
    assert pcu.wait(stream, timeout_ms=60000) is True
    assert pcu.wait(stream, timeout_ms=0) is True
