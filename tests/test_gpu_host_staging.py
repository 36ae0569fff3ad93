"""Strict MatMul with host operands (pcu_b200_strict_matmul_host), pipelined by row blocks.

Every result bit and the status word must equal those of the device call on the same operands
(itself checked against the oracle elsewhere), for 1 to 4 row blocks, ragged block sizes, an
empty inner dimension, faults placed in a late block (the block's events are shifted to the whole
product's ordinals) and in B (the first block wins), page-locked and pageable host memory; a small
case is also checked against the oracle directly.
"""
import importlib

import numpy as np
import pytest

import oracle
from gpu_util import bits, dyadic_uniform, status_word, to_device, to_host

pytestmark = pytest.mark.gpu

pcu = importlib.import_module("fusion-pcu_b200")


def _host(a, pinned):
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.pin_memory() if pinned else t


def _run_host(a, b, pinned=True, policy=0):
    import torch

    out, st = pcu.strict_matmul_host(_host(a, pinned), _host(b, pinned), policy)
    torch.cuda.synchronize()
    return out.numpy(), int(st.numpy().view(np.uint64)[0])


def _run_device(a, b, policy=0):
    import torch

    status = pcu.new_status()
    out = pcu.strict_matmul(to_device(a), to_device(b), policy=policy, status=status)
    torch.cuda.synchronize()
    return to_host(out), status_word(status)


@pytest.mark.parametrize("shape", [(100, 50, 70), (4100, 64, 96), (6150, 32, 40), (9000, 16, 24), (3000, 0, 5),
                                   (4200, 40, 2100), (4096, 8, 4096)])
@pytest.mark.parametrize("pinned", [True, False])
def test_host_matmul_matches_device_call(shape, pinned):
    rows, inner, cols = shape
    rng = np.random.default_rng(rows + inner + cols)
    a = dyadic_uniform(rng, (rows, inner), 32)
    b = dyadic_uniform(rng, (inner, cols), 32)
    got, st = _run_host(a, b, pinned)
    want, st_d = _run_device(a, b)
    assert st == st_d == oracle.STATUS_OK
    assert np.array_equal(bits(got), bits(want))


def test_host_matmul_small_against_oracle():
    rng = np.random.default_rng(5)
    a = dyadic_uniform(rng, (40, 33), 64)
    b = dyadic_uniform(rng, (33, 21), 64)
    got, st = _run_host(a, b)
    st_o, want = oracle.matmul(a, b)
    assert st == st_o == oracle.STATUS_OK
    assert np.array_equal(bits(got), bits(want))


@pytest.mark.parametrize("where", ["late_block", "b_column", "two_blocks", "first_block_last_columns",
                                   "first_block_two_column_pieces"])
def test_host_matmul_first_fault_matches_device_call(where):
    # four row blocks of 2250 rows; the first is computed in four column pieces of 528 columns
    rows, inner, cols = 9000, 24, 2100
    rng = np.random.default_rng(77)
    a = dyadic_uniform(rng, (rows, inner), 32)
    b = dyadic_uniform(rng, (inner, cols), 32)
    if where == "late_block":
        a[5000, 7] = np.nan
    elif where == "b_column":
        b[3, 11] = np.inf
    elif where == "two_blocks":
        a[8000, 2] = np.nan
        a[2500, 20] = np.float32(3e38)
        b[20, :] = np.float32(4.0)
    elif where == "first_block_last_columns":  # only the last column piece of the first block
        b[9, 1900] = np.nan
        a[:, 9] = np.float32(0.5)
    else:  # a fault in piece 3 at row 3 against one in piece 1 at row 7: the row decides
        b[4, 1700] = np.inf
        a[:3, 4] = 0.0
        b[11, 600] = np.nan
    got, st = _run_host(a, b)
    _, st_d = _run_device(a, b)
    assert st == st_d != oracle.STATUS_OK, (hex(st), hex(st_d))


@pytest.mark.parametrize("shape", [(1024, 96, 8192), (4100, 64, 96), (9000, 24, 2100), (3000, 0, 5)])
@pytest.mark.parametrize("strided", [False, True])
def test_host_left_matches_device_call(shape, strided):
    """pcu_b200_strict_matmul_host_left: A and C in host memory, B already on the device (dense or
    with a row stride wider than its columns); the result and status word of the device call."""
    import torch

    rows, inner, cols = shape
    rng = np.random.default_rng(rows + 3 * inner + 7 * cols)
    a = dyadic_uniform(rng, (rows, inner), 32)
    b = dyadic_uniform(rng, (inner, cols), 32)
    if inner:
        a[rows - 1, inner // 2] = np.nan if rows > 4000 else a[rows - 1, inner // 2]
    bd = to_device(b)
    if strided:
        wide = torch.zeros((inner, cols + 8), dtype=torch.float32, device="cuda")
        wide[:, :cols] = bd
        bd = wide[:, :cols]
    out, st = pcu.strict_matmul_host_left(_host(a, True), bd)
    torch.cuda.synchronize()
    got, word = out.numpy(), int(st.numpy().view(np.uint64)[0])
    want, st_d = _run_device(a, b)
    assert word == st_d, (hex(word), hex(st_d))
    if st_d == oracle.STATUS_OK:
        assert np.array_equal(bits(got), bits(want))
