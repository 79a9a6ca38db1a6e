"""The bench's algorithmic byte accounting (the roofline numerator) against the
per-unit figures of the hot path: config 2 layer, E4M3 shared expert, FP4
routed experts with per-32 UE8M0 scales (architecture.py:137-168)."""

import numpy as np

import bench as B


def test_unit_bytes_of_config2():
    w13 = 2 * B.I * (B.D // 2 + B.D // 32)
    w2 = B.D * (B.I // 2 + B.I // 32)
    assert w13 + w2 == 13_369_344                     # one routed expert
    s13 = 2 * B.I * B.D + 2 * (B.I // 128) * (B.D // 128)
    s2 = B.D * B.I + (B.D // 128) * (B.I // 128)
    assert s13 + s2 == 25_167_360                     # shared expert
    assert B.ROUTER_BYTES == 2_098_176                # gate weight + bias


def test_step_bytes_counts_distinct_local_experts_and_pairs():
    idx = np.array([[0, 1, 2, 3, 4, 5], [5, 6, 7, 8, 9, 10], [0, 0, 1, 300 % 256, 2, 3]])
    b = B.step_bytes(idx, 3, 0, 256)
    assert b["experts"] == len(np.unique(idx))
    # a token listing an expert twice keeps one pair (index-put semantics)
    assert b["pairs"] == 6 + 6 + 5
    half = B.step_bytes(idx, 3, 0, 4)                 # shard [0, 4)
    assert half["experts"] == 4 and half["pairs"] == 4 + 0 + 4


def test_ep_phase_bytes_are_per_rank():
    idx = np.tile(np.arange(6), (32, 1))
    b = B.ep_step_bytes(idx, 16, 2, 0, 128)
    assert b["experts_touched"] == 6
    assert b["all_gather"] == 16 * (2 * B.D + 12 * B.K_TOP)
    assert b["combine"] == 16 * B.D * 4
