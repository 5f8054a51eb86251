"""The mbarrier hand-offs of the tensor-core kernels on the QLoRA step's path, checked over every
interleaving of their roles on a model (tests/protocol_model.py): no wait that can never
complete (on the GPU, a bounded wait that gives up and raises the device error flag), no
shared-memory stage or TMEM accumulator reused or read out of order. Small stage / k-block /
tile counts cover every phase-parity wrap of the rings (two passes over each ring and over both
accumulator buffers). The planted mistakes are made in the model, and the checker must find
each of them."""

import os
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import protocol_model as pm  # noqa: E402


@pytest.mark.parametrize("args", [(2, 2, 3, 2, True), (2, 3, 3, 2, False)])
def test_lora_xa_masking_ring_and_xd_store(args):
    """csrc/lora_xa.cu: TMA -> masking threads -> MMA (and the xd store) -> refill."""
    n, how = pm.explore(pm.lora_xa(*args))
    assert how == "complete" and n > 1000


def test_one_cta_gemm_ring_and_double_buffered_accumulators():
    """csrc/tc_gemm.cuh: producer / MMA issuer / epilogue warps, two TMEM accumulators."""
    n, how = pm.explore(pm.gemm1(2, 2, 4, 2))
    assert how == "complete" and n > 1000


def test_two_sm_gemm_cross_cta_handoffs():
    """csrc/tc_gemm_pair.cuh: both CTAs' loads complete on the leader's barrier, which only the
    leader arms (the follower's bytes may land first: a negative transaction count); the
    leader's commits arrive in both CTAs; both CTAs' epilogues arrive on the leader."""
    n, how = pm.explore(pm.gemm_pair(2, 2, 3, 1))
    assert how == "complete" and n > 1000


def test_masked_input_gradient_dx_tile_ring():
    """csrc/lora_dx.cu: the dx tile loaded by TMA, rewritten by the epilogue threads, stored by
    one of them, whose arrival lets the producer reload the buffer."""
    n, how = pm.explore(pm.lora_dx(2, 2, 4, 2))
    assert how == "complete" and n > 1000


def test_planted_mistake_refill_before_the_xd_store_read_is_found():
    # the stage is refilled once the MMAs are done, without waiting for the xd store's read
    with pytest.raises(pm.Hazard, match="store|arrival beyond"):
        pm.explore(pm.lora_xa(2, 2, 3, 1, True, empty_count=1))


def test_planted_mistake_leader_arming_only_its_own_bytes_is_found():
    # the phase completes when the leader's half lands: the MMA may read the follower's half early
    with pytest.raises(pm.Hazard, match="before it landed"):
        pm.explore(pm.gemm_pair(2, 1, 2, 1, leader_bytes=2))


def test_planted_mistake_wrong_epilogue_parity_is_found():
    with pytest.raises(pm.Hazard, match="DEADLOCK|before its MMAs"):
        pm.explore(pm.gemm1(2, 1, 3, 1, epi_parity_flip=1))


def test_fused_nf4_kernel_rings_and_alternating_dequant_groups():
    """csrc/tc_nf4_gemm.cuh: activations and codes by TMA, the A operand written by two dequant
    groups taking alternate k-blocks (a stage's generations alternate between the groups), the
    LoRA segment without codes, one accumulator set drained before the next tile."""
    n, how = pm.explore(pm.nf4_gemm(1, 3, 2, 3, 1, 2, warps_per_group=1))
    assert how == "complete" and n > 1000


def test_planted_mistake_codes_ring_shorter_than_the_group_count_is_found():
    # one codes stage for two alternating groups: a parity wait two generations ahead
    with pytest.raises(pm.Hazard, match="before it is complete"):
        pm.explore(pm.nf4_gemm(1, 3, 1, 3, 0, 2, warps_per_group=1))
