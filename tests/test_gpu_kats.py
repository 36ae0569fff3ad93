"""The reference's known answers, run through the CUDA provider's C ABI on a B200.

Every case of tests/golden/reference_kats.json (transcribed from the reference's own
tests, each with its file:line) must give the same bits, or the same fault kind and
location, on the device.
"""
import numpy as np
import pytest

from gpu_util import bits, from_hex, status_word, to_device, to_host

pytestmark = pytest.mark.gpu


def _run_scalar(pcu, case):
    import torch

    width = case["width"]
    a = to_device(from_hex(width, [case["a"]]))
    status = pcu.new_status()
    if case["op"] in ("add", "sub", "mul", "div"):
        b = to_device(from_hex(width, [case["b"]]))
        out = pcu.checked_binary(case["op"], a, b, case["policy"], status=status)
    elif case["op"] == "relu":
        out = pcu.checked_relu(a, case["policy"], status=status)
    else:
        raise AssertionError(case)
    torch.cuda.synchronize()
    return status_word(status), bits(to_host(out))[0]


def test_scalar_kats(provider, kats):
    for case in kats["scalar"]:
        word, out = _run_scalar(provider, case)
        if "fault" in case:
            f = provider.element_fault(word, 1)
            assert f is not None and f.kind == case["fault"] and f.element_index == 0, case
        else:
            assert word == provider.STATUS_OK, (case, hex(word))
            assert int(out) == int(case["bits"], 16), (case, hex(int(out)))


def test_matmul_kats(provider, kats):
    import torch

    for case in kats["matmul"]:
        w = case["width"]
        left = to_device(from_hex(w, case["left"], case["left_shape"]))
        right = to_device(from_hex(w, case["right"], case["right_shape"]))
        status = provider.new_status()
        out = provider.strict_matmul(left, right, case["transpose_left"], case["transpose_right"], case["policy"],
                                     status=status)
        torch.cuda.synchronize()
        word = status_word(status)
        inner = case["left_shape"][0] if case["transpose_left"] else case["left_shape"][1]
        if "fault" in case:
            f = provider.matmul_fault(word, inner, out.numel())
            exp = case["fault"]
            assert f is not None, case
            assert (f.element_index, f.reduction_index, f.step, f.kind) == (
                exp["element_index"], exp["reduction_index"], exp["step"], exp["kind"]), case
        else:
            assert word == provider.STATUS_OK, (case, hex(word))
            assert [hex(v) for v in bits(to_host(out)).ravel()] == case["out"], case


def test_mse_kats(provider, kats):
    import torch

    for case in kats["mse"]:
        w = case["width"]
        p = to_device(from_hex(w, case["prediction"]))
        t = to_device(from_hex(w, case["target"]))
        status = provider.new_status()
        out = provider.strict_mse(p, t, case["policy"], status=status)
        torch.cuda.synchronize()
        word = status_word(status)
        if "fault" in case:
            f = provider.mse_fault(word, len(case["prediction"]))
            exp = case["fault"]
            assert f is not None and (f.element_index, f.reduction_index, f.step, f.kind) == (
                exp["element_index"], exp["reduction_index"], exp["step"], exp["kind"]), case
        else:
            assert word == provider.STATUS_OK, (case, hex(word))
            assert hex(int(bits(to_host(out).reshape(1))[0])) == case["out"], case


def test_sgd_kats(provider, kats):
    import torch

    for case in kats["sgd"]:
        w = case["width"]
        weights = to_device(from_hex(w, case["weights"]))
        gradient = to_device(from_hex(w, case["gradient"]))
        rate = np.array([int(case["rate"], 16)], dtype=np.uint32).view(np.float32)[0]
        status = provider.new_status()
        out = provider.strict_sgd(weights, gradient, rate, case["policy"], status=status)
        torch.cuda.synchronize()
        word = status_word(status)
        if "fault" in case:
            f = provider.sgd_fault(word, len(case["weights"]))
            exp = case["fault"]
            assert f is not None and (f.element_index, f.reduction_index, f.step, f.kind) == (
                exp["element_index"], exp["reduction_index"], exp["step"], exp["kind"]), case
        else:
            assert word == provider.STATUS_OK, (case, hex(word))
            assert [hex(v) for v in bits(to_host(out))] == case["out"], case
