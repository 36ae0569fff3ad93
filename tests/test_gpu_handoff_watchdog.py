"""The device-side MSE hand-off gives up instead of hanging when a predecessor never hands over.

pcu_b200_strict_mse_sgd_split's walker on rank r > 0 waits for rank r - 1 to store the running
sum into this rank's hand-off block.  Here nothing ever sets that flag (one GPU, both blocks in
this process, the call made as rank 1 of 2): the bounded wait must run out, leave the watchdog
word (kind 7, event 0) in the status word, and return, and the device must stay usable.  Rank
0's exchange slot is filled in beforehand, so the exchange step does not wait as well.  Takes
about 10 s (the wait's limit).
"""
import ctypes
import importlib
import time

import numpy as np
import pytest

import oracle
from gpu_util import bits, dyadic_uniform, status_word, to_device, to_host

pytestmark = pytest.mark.gpu

pcu = importlib.import_module("fusion-pcu_b200")

# HandoffBlock (strict_mse.cu): carry, carry_epoch, 6 pad words, then slot[2][8] of
# {mse, sgd, mean, epoch} (32 bytes each)
_SLOT0 = 64


def _slot(bank, rank):
    return _SLOT0 + (bank * 8 + rank) * 32


def test_missing_carry_reports_watchdog_and_the_device_stays_usable():
    import torch

    L = pcu.library()
    nbytes = L.pcu_b200_mse_handoff_bytes()
    blocks = [torch.zeros(nbytes, dtype=torch.uint8, device="cuda") for _ in range(2)]
    # rank 0's exchange word for call 1 (bank 1) is already in rank 1's block: clean, no mean
    words = blocks[1][_slot(1, 0):_slot(1, 0) + 32].view(torch.int64)
    words.copy_(torch.tensor([-1, -1, 0, 1], dtype=torch.int64))
    rng = np.random.default_rng(11)
    total, first = 10000, 5000
    p, t = dyadic_uniform(rng, total, 32), dyadic_uniform(rng, total, 32)
    pd, td = to_device(p[first:]), to_device(t[first:])
    mean = torch.zeros(1, dtype=torch.float32, device="cuda")
    status = pcu.new_status()
    ws = pcu.mse_workspace(pd)
    ptrs = (ctypes.c_void_p * 2)(blocks[0].data_ptr(), blocks[1].data_ptr())
    t0 = time.time()
    pcu._check(L.pcu_b200_strict_mse_sgd_split(0, 0, pcu._ptr(pd), pcu._ptr(td), total - first, first, total,
                                                pcu._ptr(mean), pcu._ptr(ws), ws.numel(), pcu._ptr(status), None, None,
                                                None, 0, 0, 0, None, ptrs, 1, 2, 1, pcu._stream(None)))
    torch.cuda.synchronize()
    waited = time.time() - t0
    assert status_word(status) == pcu.WATCHDOG, hex(status_word(status))
    assert waited > 5.0, waited  # it did wait, for about its limit
    # the context is intact: a plain strict MSE still gives the oracle's bits
    st2 = pcu.new_status()
    got = pcu.strict_mse(to_device(p), to_device(t), status=st2)
    torch.cuda.synchronize()
    st_o, out_o = oracle.mse(p, t)
    assert status_word(st2) == st_o
    assert bits(to_host(got).reshape(1))[0] == bits(out_o)[0]
