"""Pin the CPU oracle against the reference's own known answers (CPU only).

The oracle is the checker for every GPU parity test, so it is validated first:
every transcribed scalar/tensor/program known answer from the reference tests,
the reference's randomized host-RNE streams, and the fast CPU checker against
the soft-float law on random and exceptional data.
"""
import numpy as np
import pytest

import oracle
from oracle import graph as ograph

KIND = oracle.KIND_BY_NAME


def test_scalar_known_answers(kats):
    for case in kats["scalar"]:
        width, op, policy = case["width"], case["op"], case["policy"]
        a = int(case["a"], 16)
        if op in ("add", "sub", "mul", "div"):
            b = int(case["b"], 16)
            fn = oracle.f32_binary if width == 32 else oracle.f64_binary
            kind, out = fn(a, b, op, policy)
        else:
            kind, out = oracle.unary(op, width, a, policy)
        if "fault" in case:
            assert kind == KIND[case["fault"]], case
        else:
            assert kind == 0, case
            assert out == int(case["bits"], 16), (case, hex(out))


def _xorshift32(state):
    state ^= (state << 13) & 0xFFFFFFFF
    state ^= state >> 17
    state ^= (state << 5) & 0xFFFFFFFF
    return state


def _xorshift64(state):
    m = (1 << 64) - 1
    state ^= (state << 13) & m
    state ^= state >> 7
    state ^= (state << 17) & m
    return state


def _stream_pairs(spec):
    state = int(spec["seed"], 16)
    pairs = []
    for _ in range(spec["pairs"]):
        if spec["rng"] == "xorshift32":
            state = _xorshift32(state)
            a = state
            state = _xorshift32(state)
            b = state
        else:
            vals = []
            for _ in range(2):
                state = _xorshift64(state)
                v = state
                if spec["rng"] == "xorshift64_finite" and (v & 0x7FF0000000000000) == 0x7FF0000000000000:
                    v ^= 1 << 52
                vals.append(v)
            a, b = vals
        pairs.append((a, b))
    return pairs


@pytest.mark.parametrize("index", range(4))
def test_randomized_streams_match_host_rne(kats, index):
    """Reference tests.rs:306-353 / f64_tests.rs:274-344: law == host IEEE on finite pairs."""
    spec = kats["random_streams"][index]
    width = spec["width"]
    pairs = _stream_pairs(spec)
    ut = np.uint32 if width == 32 else np.uint64
    ft = np.float32 if width == 32 else np.float64
    emask = 0x7F800000 if width == 32 else 0x7FF0000000000000
    a = np.array([p[0] for p in pairs], dtype=ut)
    b = np.array([p[1] for p in pairs], dtype=ut)
    keep = ((a & emask) != emask) & ((b & emask) != emask)
    if spec.get("skip_zero_divisor"):
        keep &= (b << ut(1)) != 0
    a, b = a[keep], b[keep]
    af, bf = a.view(ft), b.view(ft)
    with np.errstate(all="ignore"):
        host = {"add": af + bf, "sub": af - bf, "mul": af * bf, "div": af / bf}
    fn = oracle.f32_binary if width == 32 else oracle.f64_binary
    checked = 0
    for op in spec["ops"]:
        expect = host[op]
        ebits = expect.view(ut)
        for i in range(len(a)):
            kind, out = fn(int(a[i]), int(b[i]), op, spec["policy"])
            if np.isinf(expect[i]):
                assert kind == KIND["ArithmeticOverflow"], (op, hex(a[i]), hex(b[i]))
            else:
                assert kind == 0 and out == int(ebits[i]), (op, hex(a[i]), hex(b[i]), hex(out))
            checked += 1
    assert checked > 0.9 * len(spec["ops"]) * len(a)


def _arr(width, hexes, shape=None):
    ut = np.uint32 if width == 32 else np.uint64
    ft = np.float32 if width == 32 else np.float64
    a = np.array([int(h, 16) for h in hexes], dtype=ut).view(ft)
    return a.reshape(shape) if shape is not None else a


def test_matmul_known_answers(kats):
    for case in kats["matmul"]:
        w = case["width"]
        left = _arr(w, case["left"], case["left_shape"])
        right = _arr(w, case["right"], case["right_shape"])
        inner = case["left_shape"][0] if case["transpose_left"] else case["left_shape"][1]
        for fast in (False, True):
            status, out = oracle.matmul(left, right, case["transpose_left"], case["transpose_right"],
                                        case["policy"], fast=fast, threads=2 if fast else None)
            if "fault" in case:
                f = case["fault"]
                assert oracle.matmul_location(status, inner) == (
                    f["element_index"], f["reduction_index"], f["step"], f["kind"]), case
            else:
                assert status == oracle.STATUS_OK, (case, oracle.decode(status))
                ut = np.uint32 if w == 32 else np.uint64
                assert [hex(v) for v in out.ravel().view(ut)] == case["out"], case


def test_mse_known_answers(kats):
    for case in kats["mse"]:
        w = case["width"]
        status, out = oracle.mse(_arr(w, case["prediction"]), _arr(w, case["target"]), case["policy"])
        if "fault" in case:
            f = case["fault"]
            assert oracle.mse_location(status, len(case["prediction"])) == (
                f["element_index"], f["reduction_index"], f["step"], f["kind"]), case
        else:
            ut = np.uint32 if w == 32 else np.uint64
            assert status == oracle.STATUS_OK and hex(int(out.view(ut)[0])) == case["out"], case


def test_sgd_known_answers(kats):
    for case in kats["sgd"]:
        w = case["width"]
        rate = np.array([int(case["rate"], 16)], dtype=np.uint32).view(np.float32)[0]
        status, out = oracle.sgd(_arr(w, case["weights"]), _arr(w, case["gradient"]), rate, case["policy"])
        if "fault" in case:
            f = case["fault"]
            assert oracle.sgd_location(status) == (f["element_index"], f["reduction_index"], f["step"],
                                                   f["kind"]), case
        else:
            ut = np.uint32 if w == 32 else np.uint64
            assert status == oracle.STATUS_OK, (case, oracle.decode(status))
            assert [hex(v) for v in out.view(ut)] == case["out"], case


def test_program_known_answers(kats):
    for program in kats["programs"]:
        g, inputs = ograph.from_program(program)
        outputs, fault = g.evaluate(inputs, [program["output"]], program["policy"])
        expect = program["expect"]
        if "runs" in expect:
            assert fault is None, (program["cite"], fault)
            ut = np.uint32 if program["width"] == 32 else np.uint64
            got = [hex(v) for v in outputs[program["output"]].ravel().view(ut)]
            want = [b for b, n in expect["runs"] for _ in range(n)]
            assert got == want, program["cite"]
        elif "fault" in expect:
            f = expect["fault"]
            assert fault is not None and fault["node"] == f["node"], (program["cite"], fault)
            for key in ("element_index", "reduction_index", "step", "kind"):
                assert fault[key] == f[key], (program["cite"], fault)
        else:
            assert fault is not None and fault["kind"] == expect["fault_kind"], (program["cite"], fault)
            assert fault["element_index"] == expect["element_index"]


def _edge_matrix(rng, shape, dtype, specials):
    x = rng.uniform(-1, 1, size=shape).astype(dtype)
    flat = x.ravel()
    idx = rng.choice(flat.size, size=min(len(specials) * 3, flat.size), replace=False)
    for j, i in enumerate(idx):
        flat[i] = specials[j % len(specials)]
    return x


@pytest.mark.parametrize("width", [32, 64])
@pytest.mark.parametrize("policy", [0, 1, 2])
def test_fast_checker_equals_soft_law(width, policy):
    rng = np.random.default_rng(1234 + width + policy)
    dtype = np.float32 if width == 32 else np.float64
    fi = np.finfo(dtype)
    tiny = fi.tiny
    specials = [0.0, -0.0, tiny, -tiny, tiny * 0.5, fi.max, -fi.max, np.nan, np.inf, 2.0 ** -70, 1e-20]
    for (m, k, n) in ((7, 13, 9), (33, 17, 65), (16, 64, 16)):
        for tl in (False, True):
            for tr in (False, True):
                a = _edge_matrix(rng, (k, m) if tl else (m, k), dtype, specials if m > 10 else [])
                b = _edge_matrix(rng, (n, k) if tr else (k, n), dtype, specials[:5])
                s1, o1 = oracle.matmul(a, b, tl, tr, policy)
                s2, o2 = oracle.matmul(a, b, tl, tr, policy, fast=True, threads=3)
                assert s1 == s2
                if s1 == oracle.STATUS_OK:
                    assert np.array_equal(o1.view(np.uint8), o2.view(np.uint8))
    # tiny-scaled operands force the exact path everywhere
    a = (rng.uniform(-1, 1, size=(9, 11)) * (1e-20 if width == 32 else 1e-160)).astype(dtype)
    b = (rng.uniform(-1, 1, size=(11, 5)) * (1e-20 if width == 32 else 1e-160)).astype(dtype)
    s1, o1 = oracle.matmul(a, b, policy=policy)
    s2, o2 = oracle.matmul(a, b, policy=policy, fast=True, threads=2)
    assert s1 == s2
    if s1 == oracle.STATUS_OK:
        assert np.array_equal(o1.view(np.uint8), o2.view(np.uint8))


def test_count_conversions():
    assert oracle.count_f32(65536) == 0x47800000
    assert oracle.count_f32((1 << 24) + 1) == 0x4B800000          # tie to even
    assert oracle.count_f32((1 << 24) + 3) == 0x4B800002
    assert oracle.count_f64(1 << 28) == 0x41B0000000000000
    assert oracle.f32_bits_to_f64_bits(0x3DCCCCCD) == np.float64(np.float32(0.1)).view(np.uint64)
    assert oracle.f32_bits_to_f64_bits(1) == np.float64(np.float32(1.4e-45)).view(np.uint64)
