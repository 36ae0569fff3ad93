"""pcu_b200_strict_matmul_static_scratch: the MatMul entry point for callers that cannot allocate.

Such callers (for example an FFI caller that was handed only its operand, output and status
buffers and does not own the device allocator) call this variant, which uses a fixed scratch
array inside the library instead of a caller workspace.  This test calls it through the C ABI
twice in a row -- with different data, so stale scratch from the first call would show -- and
requires results and status words bit-identical to pcu_b200_strict_matmul on the same inputs.
The file is collected last so that a failure here never hides the other GPU tests.
"""
import ctypes

import numpy as np
import pytest

from gpu_util import bits, dyadic_uniform, status_word, to_device, to_host

pytestmark = pytest.mark.gpu


def _bind(lib):
    fn = lib.pcu_b200_strict_matmul_static_scratch
    fn.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64,
                   ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int, ctypes.c_int,
                   ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    return fn


def _call_static(fn, pcu, a, b, out, status, transpose_left, transpose_right, policy):
    import torch

    rows, inner = (a.shape[1], a.shape[0]) if transpose_left else a.shape
    columns = b.shape[0] if transpose_right else b.shape[1]
    dtype = 0 if a.dtype == torch.float32 else 1
    return fn(dtype, policy, a.data_ptr(), b.data_ptr(), out.data_ptr(), rows, inner, columns, a.stride(0),
              b.stride(0), int(transpose_left), int(transpose_right), status.data_ptr(),
              torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("width", [32, 64])
def test_static_scratch_matches_workspace_entry_point_twice(provider, width):
    import torch

    fn = _bind(provider.library())
    rng = np.random.default_rng(4242 + width)
    tiny = 2.0 ** (-110 if width == 32 else -1000)
    cases = [
        # first call: one tiny power of two puts row 3's exponent minimum (held in the scratch)
        # below the underflow bound, so row 3 takes the exact path; its products are exact
        # subnormals, so nothing faults and every output must match
        (dyadic_uniform(rng, (300, 96), width), dyadic_uniform(rng, (96, 260), width), False, False, 0),
        # second call: different shapes and one NaN; stale minima from call one would change the path
        (dyadic_uniform(rng, (260, 128), width), dyadic_uniform(rng, (96, 128), width), False, True, 1),
        # third call: fault-free again, transposed left operand
        (dyadic_uniform(rng, (64, 200), width), dyadic_uniform(rng, (64, 72), width), True, False, 0),
    ]
    cases[0][0][3, 7] = tiny
    cases[1][0][17, 5] = np.nan
    for a_h, b_h, tl, tr, policy in cases:
        a, b = to_device(a_h), to_device(b_h)
        rows = a.shape[1] if tl else a.shape[0]
        columns = b.shape[0] if tr else b.shape[1]
        ref_status = provider.new_status()
        ref = provider.strict_matmul(a, b, tl, tr, policy, status=ref_status)
        out = torch.empty((rows, columns), dtype=a.dtype, device="cuda")
        status = provider.new_status()
        assert _call_static(fn, provider, a, b, out, status, tl, tr, policy) == 0
        torch.cuda.synchronize()
        assert status_word(status) == status_word(ref_status)
        if status_word(ref_status) == provider.STATUS_OK:
            assert np.array_equal(bits(to_host(out)), bits(to_host(ref)))


def test_static_scratch_rejects_shapes_beyond_its_limit(provider):
    import torch

    fn = _bind(provider.library())
    a = torch.zeros((40000, 4), dtype=torch.float32, device="cuda")
    b = torch.zeros((4, 30000), dtype=torch.float32, device="cuda")
    out = torch.empty((1, 1), dtype=torch.float32, device="cuda")
    status = provider.new_status()
    rc = fn(0, 0, a.data_ptr(), b.data_ptr(), out.data_ptr(), 40000, 4, 30000, 4, 30000, 0, 0, status.data_ptr(),
            torch.cuda.current_stream().cuda_stream)
    assert rc == 3  # PCU_B200_ERROR_WORKSPACE: rows + columns exceeds 65536
    torch.cuda.synchronize()
    assert status_word(status) == provider.STATUS_OK


def test_static_scratch_limit_applies_only_when_the_scratch_is_used(provider):
    """Calls that need no exponent minima (empty shapes, AllowGradualUnderflow) are not limited:
    they return exactly what the workspace entry point returns."""
    import torch

    fn = _bind(provider.library())
    status = provider.new_status()
    dummy = torch.zeros(16, dtype=torch.float32, device="cuda")
    # rows == 0: an empty product, whatever the column count
    assert fn(0, 0, dummy.data_ptr(), dummy.data_ptr(), dummy.data_ptr(), 0, 4, 70000, 4, 70000, 0, 0,
              status.data_ptr(), torch.cuda.current_stream().cuda_stream) == 0
    # AllowGradualUnderflow (policy 2) with rows + columns above the limit, twice in a row
    rng = np.random.default_rng(77)
    for seed in (0, 1):
        a = to_device(dyadic_uniform(rng, (65000, 4), 32))
        b = to_device(dyadic_uniform(rng, (4, 600), 32))
        ref_status = provider.new_status()
        ref = provider.strict_matmul(a, b, False, False, 2, status=ref_status)
        out = torch.empty((65000, 600), dtype=torch.float32, device="cuda")
        st = provider.new_status()
        assert _call_static(fn, provider, a, b, out, st, False, False, 2) == 0
        torch.cuda.synchronize()
        assert status_word(st) == status_word(ref_status) == provider.STATUS_OK
        assert np.array_equal(bits(to_host(out)), bits(to_host(ref)))
    torch.cuda.synchronize()
    assert status_word(status) == provider.STATUS_OK
