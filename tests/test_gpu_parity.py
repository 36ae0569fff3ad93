"""Seeded parity of every CUDA kernel against the CPU oracle (bit-exact, same status word).

Sizes are chosen so the oracle finishes in seconds; full BASELINE sizes are covered by
sampled cells plus size-independent checks.  Inputs include the exceptional values the
reference tests use (signed zeros, subnormals, MAX, NaN, infinities) and ragged shapes
that exercise partial tiles on both the TMA and the plain kernel paths.
"""
import numpy as np
import pytest

import oracle
from gpu_util import FT, UT, bits, dyadic_uniform, specials, sprinkle, status_word, to_device, to_host

pytestmark = pytest.mark.gpu


def _sync():
    import torch

    torch.cuda.synchronize()


# ------------------------------------------------------------------ scalar law, all ops

def _random_bits(rng, n, width):
    lo = rng.integers(0, 1 << 32, size=n, dtype=np.uint64)
    if width == 32:
        return lo.astype(np.uint32)
    hi = rng.integers(0, 1 << 32, size=n, dtype=np.uint64)
    return (hi << np.uint64(32)) | lo


@pytest.mark.parametrize("width", [32, 64])
@pytest.mark.parametrize("policy", [0, 1, 2])
@pytest.mark.parametrize("op", ["add", "sub", "mul", "div"])
def test_checked_binary_random_bits(provider, width, policy, op):
    """Random bit patterns (all exponents, subnormals, NaN/Inf) through the exact and fast paths."""
    rng = np.random.default_rng(7 + width + 11 * policy + 101 * list(provider.OPS).index(op))
    n = 20000
    a = _random_bits(rng, n, width)
    b = _random_bits(rng, n, width)
    av, bv = a.view(FT[width]), b.view(FT[width])
    fn = oracle.f32_binary if width == 32 else oracle.f64_binary
    expect = [fn(int(x), int(y), op, policy) for x, y in zip(a, b)]
    ok = np.array([k == 0 for k, _ in expect])
    # fault-free subset in one launch: bit-exact, no status
    status = provider.new_status()
    out = provider.checked_binary(op, to_device(av[ok]), to_device(bv[ok]), policy, status=status)
    _sync()
    assert status_word(status) == provider.STATUS_OK
    got = bits(to_host(out))
    want = np.array([r for k, r in expect if k == 0], dtype=UT[width])
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, [(hex(int(a[ok][i])), hex(int(b[ok][i])), hex(int(got[i])), hex(int(want[i])))
                           for i in bad[:5]]
    # faulting elements: each one alone must report its kind at element 0
    fidx = np.nonzero(~ok)[0][:300]
    for i in fidx:
        status = provider.new_status()
        provider.checked_binary(op, to_device(av[i:i + 1]), to_device(bv[i:i + 1]), policy, status=status)
        _sync()
        f = provider.element_fault(status_word(status), 1)
        assert f is not None and f.kind == oracle.KIND_NAMES[expect[i][0]], (hex(int(a[i])), hex(int(b[i])))


@pytest.mark.parametrize("width", [32, 64])
def test_checked_binary_near_underflow(provider, width):
    """Dense sampling of products/quotients around the smallest normal for all policies."""
    rng = np.random.default_rng(99 + width)
    n = 40000
    fi = np.finfo(FT[width])
    emin = -126 if width == 32 else -1022
    ea = rng.integers(emin // 2 - 30, emin // 2 + 30, size=n)
    a = (rng.uniform(1, 2, size=n) * 2.0 ** ea).astype(FT[width])
    b = (rng.uniform(1, 2, size=n) * 2.0 ** (emin - ea)).astype(FT[width]) * rng.choice([-1, 1], size=n)
    b = b.astype(FT[width])
    for policy in (0, 1, 2):
        for op in ("mul", "div", "add", "sub"):
            y = b if op != "div" else (1 / b).astype(FT[width])
            fn = oracle.f32_binary if width == 32 else oracle.f64_binary
            expect = [fn(int(x), int(z), op, policy) for x, z in zip(bits(a), bits(y))]
            ok = np.array([k == 0 for k, _ in expect])
            status = provider.new_status()
            out = provider.checked_binary(op, to_device(a[ok]), to_device(y[ok]), policy, status=status)
            _sync()
            assert status_word(status) == provider.STATUS_OK, (op, policy)
            want = np.array([r for k, r in expect if k == 0], dtype=UT[width])
            assert np.array_equal(bits(to_host(out)), want), (op, policy)
            for i in np.nonzero(~ok)[0][:50]:
                status = provider.new_status()
                provider.checked_binary(op, to_device(a[i:i + 1]), to_device(y[i:i + 1]), policy, status=status)
                _sync()
                f = provider.element_fault(status_word(status), 1)
                assert f is not None and f.kind == oracle.KIND_NAMES[expect[i][0]]
    assert fi.tiny > 0


# ------------------------------------------------------------------ streaming ops, first fault

@pytest.mark.parametrize("width", [32, 64])
@pytest.mark.parametrize("policy", [0, 1, 2])
def test_streaming_ops_first_fault(provider, width, policy):
    rng = np.random.default_rng(1000 + width * 3 + policy)
    for n in (1, 3, 1000, 65537, 1 << 18):
        x = dyadic_uniform(rng, n, width)
        y = dyadic_uniform(rng, n, width)
        for inject in (False, True):
            if inject:
                sprinkle(rng, x, specials(width), 7)
                sprinkle(rng, y, specials(width), 5)
            # SGD
            rate = np.float32(0.01)
            s_o, o_o = oracle.sgd(x, y, rate, policy)
            status = provider.new_status()
            out = provider.strict_sgd(to_device(x), to_device(y), rate, policy, status=status)
            _sync()
            assert status_word(status) == s_o, (n, inject, hex(status_word(status)), hex(s_o))
            # every element in front of the first fault is written, as by the reference's loop
            first = n if s_o == oracle.STATUS_OK else oracle.decode(s_o)[0] // 2
            assert np.array_equal(bits(to_host(out)[:first]), bits(o_o[:first]))
            # binary ops (including a uniform right operand)
            for op in ("add", "sub", "mul", "div"):
                s_o, o_o = oracle.binary(op, x, y, policy)
                status = provider.new_status()
                out = provider.checked_binary(op, to_device(x), to_device(y), policy, status=status)
                _sync()
                assert status_word(status) == s_o, (op, n, inject)
                first = n if s_o == oracle.STATUS_OK else oracle.decode(s_o)[0]
                assert np.array_equal(bits(to_host(out)[:first]), bits(o_o[:first]))
            u = np.array([FT[width](2.0 ** -15)])
            s_o, o_o = oracle.binary("mul", x, u, policy, right_uniform=True)
            status = provider.new_status()
            out = provider.checked_binary("mul", to_device(x), to_device(u), policy, right_uniform=True,
                                          status=status)
            _sync()
            assert status_word(status) == s_o
            if s_o == oracle.STATUS_OK:
                assert np.array_equal(bits(to_host(out)), bits(o_o))
            # relu / relu backward
            s_o, o_o = oracle.relu(x, policy)
            status = provider.new_status()
            out = provider.checked_relu(to_device(x), policy, status=status)
            _sync()
            assert status_word(status) == s_o
            if s_o == oracle.STATUS_OK:
                assert np.array_equal(bits(to_host(out)), bits(o_o))
            s_o, o_o = oracle.relu_backward(x, y, policy)
            status = provider.new_status()
            out = provider.checked_relu_backward(to_device(x), to_device(y), policy, status=status)
            _sync()
            assert status_word(status) == s_o
            if s_o == oracle.STATUS_OK:
                assert np.array_equal(bits(to_host(out)), bits(o_o))


def test_sgd_in_place_and_unaligned(provider):
    import torch

    rng = np.random.default_rng(5)
    x = dyadic_uniform(rng, 4099, 32)
    g = dyadic_uniform(rng, 4099, 32)
    s_o, o_o = oracle.sgd(x, g, np.float32(0.5))
    w = to_device(x)
    provider.strict_sgd(w, to_device(g), np.float32(0.5), out=w)
    _sync()
    assert np.array_equal(bits(to_host(w)), bits(o_o))
    # offset views break 16-byte alignment and take the scalar path
    big = to_device(np.concatenate([[0], x]).astype(np.float32))
    gg = to_device(np.concatenate([[0], g]).astype(np.float32))
    out = torch.empty(4100, dtype=torch.float32, device="cuda")
    provider.strict_sgd(big[1:], gg[1:], np.float32(0.5), out=out[1:])
    _sync()
    assert np.array_equal(bits(to_host(out[1:])), bits(o_o))


# ------------------------------------------------------------------ MatMul

SHAPES = [(1, 1, 1), (1, 2, 1), (3, 5, 7), (16, 16, 16), (65, 2, 1), (129, 67, 131), (136, 68, 132),
          (128, 32, 128), (200, 100, 72), (257, 300, 260)]


def _matmul_case(provider, a, b, tl, tr, policy, fast_oracle=False):
    s_o, o_o = oracle.matmul(a, b, tl, tr, policy, fast=fast_oracle)
    status = provider.new_status()
    out = provider.strict_matmul(to_device(a), to_device(b), tl, tr, policy, status=status)
    _sync()
    word = status_word(status)
    assert word == s_o, (a.shape, b.shape, tl, tr, policy, oracle.decode(word), oracle.decode(s_o))
    if s_o == oracle.STATUS_OK:
        got, want = bits(to_host(out)), bits(o_o)
        diff = np.argwhere(got != want)
        assert diff.size == 0, (a.shape, b.shape, tl, tr, policy, diff[:5])


@pytest.mark.parametrize("width", [32, 64])
@pytest.mark.parametrize("tl,tr", [(False, False), (True, False), (False, True), (True, True)])
def test_matmul_random_shapes(provider, width, tl, tr):
    rng = np.random.default_rng(31 + width + 2 * tl + tr)
    for (m, k, n) in SHAPES:
        a = dyadic_uniform(rng, (k, m) if tl else (m, k), width)
        b = dyadic_uniform(rng, (n, k) if tr else (k, n), width)
        for policy in (0, 1, 2):
            _matmul_case(provider, a, b, tl, tr, policy)


@pytest.mark.parametrize("width", [32, 64])
@pytest.mark.parametrize("policy", [0, 1, 2])
def test_matmul_exceptional_values(provider, width, policy):
    rng = np.random.default_rng(500 + width + policy)
    for (m, k, n) in ((33, 40, 36), (136, 96, 140), (64, 256, 64)):
        for tl, tr in ((False, False), (True, False), (False, True)):
            for trial in range(4):
                a = dyadic_uniform(rng, (k, m) if tl else (m, k), width)
                b = dyadic_uniform(rng, (n, k) if tr else (k, n), width)
                if trial == 0:
                    sprinkle(rng, a, specials(width), 5)
                elif trial == 1:
                    a *= FT[width](2.0 ** (-70 if width == 32 else -520))
                    b *= FT[width](2.0 ** (-70 if width == 32 else -520))
                elif trial == 2:
                    sprinkle(rng, b, [np.finfo(FT[width]).tiny, np.finfo(FT[width]).smallest_subnormal], 3)
                else:
                    a *= FT[width](np.finfo(FT[width]).max / 8)
                _matmul_case(provider, a, b, tl, tr, policy)


@pytest.mark.parametrize("width", [32, 64])
def test_matmul_ordering_and_cancellation(provider, width):
    """Order-sensitive sums: any reassociation or FMA changes these bits."""
    rng = np.random.default_rng(77 + width)
    m, k, n = 96, 512, 80
    scale = 2.0 ** (24 if width == 32 else 53)
    a = rng.choice([scale, 1.0, -scale, 0.5, 3.0], size=(m, k)).astype(FT[width])
    b = rng.choice([1.0, -1.0, 1.0 + 2.0 ** -20, 0.75], size=(k, n)).astype(FT[width])
    for policy in (0, 2):
        _matmul_case(provider, a, b, False, False, policy)


@pytest.mark.parametrize("width", [32, 64])
def test_matmul_1024_full(provider, width):
    rng = np.random.default_rng(1024 + width)
    a = dyadic_uniform(rng, (1024, 1024), width)
    b = dyadic_uniform(rng, (1024, 1024), width)
    _matmul_case(provider, a, b, False, False, 0, fast_oracle=True)
    _matmul_case(provider, a, b, True, False, 0, fast_oracle=True)
    _matmul_case(provider, a, b, False, True, 0, fast_oracle=True)


def _split_launch(m, n, width, sms=148):
    """True when the product's last wave of 128-row tiles runs as a separate half-tile launch
    (the schedule of strict_matmul.cu's whole_tile_launch)."""
    bn = 128 if width == 32 else 64
    tiles = -(-m // 128) * -(-n // bn)
    return tiles > sms and tiles % sms != 0 and 2 * (tiles % sms) <= sms


@pytest.mark.parametrize("width", [32, 64])
@pytest.mark.parametrize("tl,tr", [(False, False), (True, False), (False, True), (True, True)])
def test_matmul_half_tile_tail_launch(provider, width, tl, tr):
    """Products whose last wave is cut into half tiles (a second launch of 64-row CTAs), the shape of
    an 8192 x 8192 product's row block on 8 GPUs, and a ragged one whose last tile row ends inside a
    half; every cell bit-exact and the first fault where the oracle puts it."""
    import torch

    sms = torch.cuda.get_device_properties(0).multi_processor_count
    rng = np.random.default_rng(640 + width + 2 * tl + tr)
    cols = 8192 if width == 32 else 4096
    for m, k, n, fault in ((1024, 48, cols, None), (1000, 40, cols - 24, None), (1024, 24, cols, 3)):
        assert sms != 148 or _split_launch(m, n, width, sms), (m, n)
        a = dyadic_uniform(rng, (k, m) if tl else (m, k), width)
        b = dyadic_uniform(rng, (n, k) if tr else (k, n), width)
        if fault is not None:  # a NaN in op(B)'s last column: its tiles are in the half-tile launch
            if tr:
                b[n - 1, fault] = np.nan
            else:
                b[fault, n - 1] = np.nan
        _matmul_case(provider, a, b, tl, tr, 0, fast_oracle=True)


@pytest.mark.parametrize("tl,tr", [(False, False), (True, False), (False, True), (True, True)])
def test_matmul_narrow_output_on_the_tma_kernel(provider, tl, tr):
    """Enough row tiles for the TMA kernel but an output only 32 (or 40) columns wide, so every
    128-column tile is mostly outside the matrix: the per-rank shapes of the 4-layer MLP's last
    layer column-sharded over 8 GPUs, forward (K = 512 here) and backward (K = 32).  Every cell
    bit-exact, and a NaN in op(B)'s last column reported where the oracle puts it."""
    rng = np.random.default_rng(7000 + 2 * tl + tr)
    for m, k, n, fault in ((8192, 512, 32, None), (8192, 32, 512, None), (8192, 200, 40, 7)):
        a = dyadic_uniform(rng, (k, m) if tl else (m, k), 32)
        b = dyadic_uniform(rng, (n, k) if tr else (k, n), 32)
        if fault is not None:
            if tr:
                b[n - 1, fault] = np.nan
            else:
                b[fault, n - 1] = np.nan
        _matmul_case(provider, a, b, tl, tr, 0, fast_oracle=True)


@pytest.mark.parametrize("m,k,n", [(8192, 8192, 8192), (2048, 2048, 2048), (4096, 4096, 4096), (8192, 1024, 16384)])
def test_matmul_sweep_sampled_cells(provider, m, k, n):
    """BASELINE config 2 at full size (the square sweep and the 8192x1024 . 1024x16384 case):
    512 random cells of each product re-derived by the soft-float law."""
    import torch

    rng = np.random.default_rng(8192 if (m, k, n) == (8192, 8192, 8192) else m + 3 * k + 7 * n)
    a = dyadic_uniform(rng, (m, k), 32)
    b = dyadic_uniform(rng, (k, n), 32)
    status = provider.new_status()
    out = provider.strict_matmul(to_device(a), to_device(b), status=status)
    torch.cuda.synchronize()
    assert status_word(status) == provider.STATUS_OK
    cells = rng.choice(m * n, size=512, replace=False).astype(np.uint64)
    s_o, vals = oracle.matmul_cells(a, b, cells)
    assert s_o == oracle.STATUS_OK
    got = to_host(out).reshape(-1)[cells.astype(np.int64)]
    assert np.array_equal(bits(got), bits(vals))


def test_matmul_f64_4096_fault_variants(provider):
    """BASELINE config 3 fault variants (NaN, 1e300, 1e-160 scaling) match the oracle's outcome."""
    import torch

    rng = np.random.default_rng(4096)
    n = 4096
    a = dyadic_uniform(rng, (n, n), 64)
    b = dyadic_uniform(rng, (n, n), 64)
    da, db = to_device(a), to_device(b)
    # NaN in A[r][k] -> first fault at cell r*n + 0, reduction k, Multiply, Invalid
    r, k = 1234, 777
    a2 = a.copy()
    a2[r, k] = np.nan
    status = provider.new_status()
    provider.strict_matmul(to_device(a2), db, status=status)
    torch.cuda.synchronize()
    f = provider.matmul_fault(status_word(status), n, n * n)
    assert (f.element_index, f.reduction_index, f.step, f.kind) == (r * n, k, "Multiply", "InvalidFloatingOperand")
    cells = np.arange(r * n, r * n + 4, dtype=np.uint64)
    s_o, _ = oracle.matmul_cells(a2, b, cells)
    assert status_word(status) == s_o
    # 1e300 entry: the oracle decides (products stay finite against |b| < 1)
    a3 = a.copy()
    a3[5, 9] = 1e300
    status = provider.new_status()
    out = provider.strict_matmul(to_device(a3), db, status=status)
    torch.cuda.synchronize()
    row_status, row_vals = oracle.matmul(a3, b, rows=(5, 6))
    assert status_word(status) == row_status
    if row_status == oracle.STATUS_OK:
        assert np.array_equal(bits(to_host(out)[5]), bits(row_vals[5]))
    # both operands scaled to 1e-160: products ~1e-320 are tiny and inexact
    status = provider.new_status()
    provider.strict_matmul(to_device(a * 1e-160), to_device(b * 1e-160), status=status)
    torch.cuda.synchronize()
    s_o, _ = oracle.matmul_cells(a * 1e-160, b * 1e-160, np.arange(0, 8, dtype=np.uint64))
    assert status_word(status) == s_o
    f = provider.matmul_fault(status_word(status), n, n * n)
    assert f.kind == "ArithmeticUnderflow"


# ------------------------------------------------------------------ MSE

@pytest.mark.parametrize("width", [32, 64])
@pytest.mark.parametrize("policy", [0, 1, 2])
def test_mse_random(provider, width, policy):
    rng = np.random.default_rng(300 + width + policy)
    for n in (1, 2, 1023, 1024, 1025, 100000, 1 << 20):
        p = dyadic_uniform(rng, n, width)
        t = dyadic_uniform(rng, n, width)
        for inject in (False, True):
            if inject:
                sprinkle(rng, p, specials(width), 3)
            s_o, o_o = oracle.mse(p, t, policy)
            status = provider.new_status()
            out = provider.strict_mse(to_device(p), to_device(t), policy, status=status)
            _sync()
            assert status_word(status) == s_o, (n, inject, oracle.decode(status_word(status)), oracle.decode(s_o))
            if s_o == oracle.STATUS_OK:
                assert bits(to_host(out).reshape(1))[0] == bits(o_o)[0]


def _mse_case(provider, p, t, policy=0):
    s_o, o_o = oracle.mse(p, t, policy)
    status = provider.new_status()
    out = provider.strict_mse(to_device(p), to_device(t), policy, status=status)
    _sync()
    word = status_word(status)
    assert word == s_o, (p.size, oracle.decode(word), oracle.decode(s_o))
    if s_o == oracle.STATUS_OK:
        assert bits(to_host(out).reshape(1))[0] == bits(o_o)[0], (p.size, to_host(out), o_o)


@pytest.mark.parametrize("width", [32, 64])
def test_mse_tie_heavy_and_wide_range(provider, width):
    """Squares with few significant bits make round-to-even ties at many binades of the running
    sum; powers of two spread the squares over many exponents; partial chunks at the end."""
    rng = np.random.default_rng(900 + width)
    ft = FT[width]
    for n in (5000, 8192 * 3 + 17, 1 << 19, (1 << 21) + 333):
        # small integers scaled by a power of two: d^2 has at most ~12 significant bits
        p = (rng.integers(-64, 64, size=n) * 2.0 ** -3).astype(ft)
        t = (rng.integers(-64, 64, size=n) * 2.0 ** -3).astype(ft)
        _mse_case(provider, p, t)
        # powers of two over a wide exponent range: every square is a tie somewhere
        e = rng.integers(-30, 30, size=n)
        p2 = (2.0 ** e * rng.choice([-1.0, 1.0], size=n)).astype(ft)
        _mse_case(provider, p2, np.zeros(n, ft), policy=2)
        # mostly tiny with rare large values (sum dominated by a few elements)
        p3 = dyadic_uniform(rng, n, width) * ft(2.0 ** -12)
        p3[rng.integers(0, n, size=5)] = ft(1000.0)
        _mse_case(provider, p3, np.zeros(n, ft), policy=2)
    # exactly representable halves: q = 0.25 everywhere -> ties whenever the sum's ulp is 0.5
    n = 1 << 20
    _mse_case(provider, np.full(n, ft(0.5)), np.zeros(n, ft))
    _mse_case(provider, np.full(n, ft(1.5)), np.zeros(n, ft))


@pytest.mark.parametrize("width", [32, 64])
def test_mse_late_faults(provider, width):
    rng = np.random.default_rng(950 + width)
    ft = FT[width]
    n = (1 << 20) + 11
    p = dyadic_uniform(rng, n, width)
    t = dyadic_uniform(rng, n, width)
    big = np.sqrt(np.finfo(ft).max / 4).astype(ft)
    for where in (0, 8191, 8192, 700001, n - 1):
        q = p.copy()
        q[where] = np.nan
        _mse_case(provider, q, t)
        q = p.copy()
        q[where:where + 8] = big  # the running sum overflows a few elements after `where`
        _mse_case(provider, q, t)


@pytest.mark.parametrize("width", [32, 64])
def test_mse_stop_inside_superblocks(provider, width):
    """A Subtract fault past the first superblock stops the walk in front of it: the walk takes
    superblock maps, then block maps and chunk maps up to the fault (and its rounds mix all three
    levels).  Faults at a superblock boundary, a block boundary, and inside a chunk."""
    rng = np.random.default_rng(970 + width)
    chunk = 1024 if width == 32 else 512
    block, sup = chunk * 64, chunk * 4096
    n = 3 * sup + 5000
    p = dyadic_uniform(rng, n, width)
    t = dyadic_uniform(rng, n, width)
    for where in (sup + 7 * block + 5 * chunk + 7, 2 * sup, 2 * sup + 3 * block, 3 * sup + 4999):
        q = p.copy()
        q[where] = np.nan
        _mse_case(provider, q, t)
    _mse_case(provider, p, t)


def test_mse_overflow_and_tiny_mean(provider):
    import torch

    big = np.full(64, np.float32(1e19))
    zero = np.zeros(64, np.float32)
    for p, t in ((big, zero), (np.full(3, np.float32(2.0 ** -70)), np.zeros(3, np.float32))):
        s_o, _ = oracle.mse(p, t)
        status = provider.new_status()
        provider.strict_mse(to_device(p), to_device(t), status=status)
        torch.cuda.synchronize()
        assert status_word(status) == s_o
