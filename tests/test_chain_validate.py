"""Guarded-chain record validation (pcu_b200_chain_validate), host code only: no GPU needed.

The cases follow the reference's own tests of validate_guarded_execution
(Crates/core/runtime/execution/guarded/tests/tests.rs) and of the record decoding
(Crates/backends/rocm/owned_dispatch/guarded/guarded.rs, tests module): an empty or clean chain
succeeds; the first fault wins and every later stage must be skipped; a bad record after a fault
is still reported; a skip without an earlier fault, or an execution after one, is a protocol
error; pending and unknown dispositions never decode.
"""
import ctypes

import numpy as np
import pytest

OK = (1 << 64) - 1
EXECUTED, SKIPPED, PENDING = 1, 2, 0
OVERFLOW, DIV0, UNDERFLOW, INVALID = 3, 1, 4, 5


def word(event, kind):
    return (event << 3) | kind


def slab(*records):
    return np.array([w for rec in records for w in rec], dtype=np.uint64)


def test_empty_and_clean_chains_succeed(provider):
    assert provider.chain_validate(np.zeros(0, dtype=np.uint64)) == ("succeeded", 0)
    assert provider.chain_validate(slab(*[(OK, EXECUTED)] * 4)) == ("succeeded", 0)


def test_first_fault_wins_and_successors_are_skipped(provider):
    records = slab((OK, EXECUTED), (word(900, OVERFLOW), EXECUTED), (OK, SKIPPED), (OK, SKIPPED))
    assert provider.chain_validate(records) == ("fault", 1)


def test_a_later_bad_record_is_not_hidden_by_an_earlier_fault(provider):
    records = slab((word(7, OVERFLOW), EXECUTED), (OK, SKIPPED), (OK, PENDING))
    assert provider.chain_validate(records) == ("stage_decode", 2)


@pytest.mark.parametrize("successor", [(OK, EXECUTED), (word(2, OVERFLOW), EXECUTED)])
def test_execution_after_a_fault_is_a_protocol_error(provider, successor):
    records = slab((word(900, OVERFLOW), EXECUTED), successor)
    assert provider.chain_validate(records) == ("executed_after_fault", 1)


@pytest.mark.parametrize("skipped", [0, 1, 2])
def test_a_skip_without_an_earlier_fault_is_not_success(provider, skipped):
    records = slab(*[(OK, SKIPPED) if s == skipped else (OK, EXECUTED) for s in range(3)])
    assert provider.chain_validate(records) == ("unexpected_skip", skipped)


@pytest.mark.parametrize("disposition", [PENDING, 3, 256, OK])
def test_pending_and_unknown_dispositions_never_decode(provider, disposition):
    assert provider.chain_validate(slab((OK, EXECUTED), (OK, disposition))) == ("stage_decode", 1)


def test_a_fault_word_on_a_skipped_stage_does_not_decode(provider):
    records = slab((word(3, INVALID), EXECUTED), (word(7, OVERFLOW), SKIPPED))
    assert provider.chain_validate(records) == ("stage_decode", 1)


@pytest.mark.parametrize("kind", [0, 2, 6, 7])
def test_kinds_no_node_call_writes_do_not_decode(provider, kind):
    # 2 = SignedDivisionOverflow (integer only); 7 = the device watchdog (no completed result)
    assert provider.chain_validate(slab((word(5, kind), EXECUTED))) == ("stage_decode", 0)


@pytest.mark.parametrize("kind", [DIV0, OVERFLOW, UNDERFLOW, INVALID])
def test_every_arithmetic_kind_decodes(provider, kind):
    assert provider.chain_validate(slab((word(5, kind), EXECUTED), (OK, SKIPPED))) == ("fault", 0)


def test_events_outside_the_stage_domain_do_not_decode(provider):
    # extent 65: event 64 is the last one inside (guarded.rs tests: (65 << 3) | 3 with extent 65)
    assert provider.chain_validate(slab((word(64, OVERFLOW), EXECUTED)), extents=[65]) == ("fault", 0)
    assert provider.chain_validate(slab((word(65, OVERFLOW), EXECUTED)), extents=[65]) == ("stage_decode", 0)
    # without extents only the kind is checked
    assert provider.chain_validate(slab((word(65, OVERFLOW), EXECUTED))) == ("fault", 0)


def test_malformed_arguments(provider):
    with pytest.raises(ValueError):
        provider.chain_validate(np.zeros(3, dtype=np.uint64))
    with pytest.raises(ValueError):
        provider.chain_validate(slab((OK, EXECUTED)), extents=[1, 2])
    lib = provider.library()
    out, stage = ctypes.c_int(), ctypes.c_uint32()
    assert lib.pcu_b200_chain_validate(None, 2, None, ctypes.byref(out), ctypes.byref(stage)) == 1
    assert lib.pcu_b200_chain_validate(None, 0, None, None, ctypes.byref(stage)) == 1
    assert lib.pcu_b200_chain_validate(None, 0, None, ctypes.byref(out), ctypes.byref(stage)) == 0
    assert (out.value, stage.value) == (0, 0)


def test_guarded_calls_reject_a_missing_slab_before_any_device_work(provider):
    lib = provider.library()
    assert lib.pcu_b200_chain_reset(None, 0, None) == 0
    assert lib.pcu_b200_chain_reset(None, 3, None) == 1
    assert lib.pcu_b200_guarded_strict_sgd(0, 0, None, None, None, 4, 0x3F000000, None, 0, None) == 1
    assert lib.pcu_b200_guarded_checked_relu(0, 0, None, None, 4, None, 0, None) == 1
    assert lib.pcu_b200_guarded_checked_relu_backward(0, 0, None, None, None, 4, None, 0, None) == 1
    assert lib.pcu_b200_guarded_checked_binary(0, 0, 0, None, None, None, 4, 0, 0, None, 0, None) == 1
    assert lib.pcu_b200_guarded_strict_mse(0, 0, None, None, None, 4, None, 0, None, 0, None) == 1
    assert lib.pcu_b200_guarded_strict_matmul(0, 0, None, None, None, 4, 4, 4, 4, 4, 0, 0, None, 0, None, 0,
                                              None) == 1
    assert lib.pcu_b200_error_string(6).decode().startswith("the stream's work")
