"""The serving harness's host-side rules against the reference's own harness (CPU only).

tests/golden/cluster_sched.json holds the outputs of the reference's python/bz_ggml/cluster.py
(estimate_speech_profile, select_burst_steps, a TieredSlotPool acquire/release trace) on seeded
inputs, written by tests/golden/make_golden.py.
"""
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def cluster(pkg):
    import importlib
    return importlib.import_module(pkg.__name__ + ".cluster")


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(HERE, "golden", "cluster_sched.json")) as f:
        return json.load(f)


def test_speech_profile_matches_reference(cluster, golden):
    for case in golden["profiles"]:
        got = cluster.estimate_speech_profile(case["text"], case["instruction"], case["ref_frames"], case["cfg_scale"])
        assert got == case["out"], case


def test_burst_size_matches_reference(cluster, golden):
    for case in golden["bursts"]:
        sess = {i: {"expected_eos": e, "total_frames": t} for i, (e, t) in enumerate(case["sessions"])}
        assert cluster.select_burst_steps(sess, case["max_burst"]) == case["out"], case


def test_slot_pool_trace_matches_reference(cluster, golden):
    pool = cluster.TieredSlotPool(*golden["pool"]["tiers"])
    for step in golden["pool"]["trace"]:
        if step[0] == "release":
            pool.release(step[1])
            assert pool.active_count() == step[2]
        else:
            got = pool.acquire(step[1])
            assert (list(got) if got else None) == step[2], step
            assert pool.active_count() == step[3]
    assert pool.total_slots() == sum(golden["pool"]["tiers"])


def test_token_wire_round_trip(cluster):
    rng = np.random.default_rng(5)
    frames = rng.integers(0, 2051, (7, 32)).astype(np.int32)
    packet = cluster.pack_frames(frames)
    assert len(packet) == 7 * 32  # 16 codes x 2 bytes per frame
    assert np.array_equal(cluster.unpack_frames(packet), frames[:, :16])
    wide = cluster.pack_frames(frames, width=32)
    assert np.array_equal(cluster.unpack_frames(wide, width=32), frames)
    assert cluster.unpack_frames(b"").shape == (0, 16)
    with pytest.raises(ValueError):
        cluster.unpack_frames(packet[:-2])
    with pytest.raises(ValueError):
        cluster.pack_frames(frames[:, :8])
    with pytest.raises(ValueError):
        cluster.pack_frames(np.full((1, 16), -1))
