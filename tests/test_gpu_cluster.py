"""The N-island serving harness on the GPU (needs a B200): two islands on one GPU share a job
queue of staggered arrivals, admit them through the tiered slot pool in batched creations, and
deliver token-mode requests as 32-byte-per-frame packets and the others as server-side PCM
(streamed in chunks, or in one pass at the end), as the reference's cluster.py worker does.
"""
import importlib

import numpy as np
import pytest

from parity_helpers import snr_db

pytestmark = pytest.mark.gpu


def test_islands_serve_tokens_and_audio(pkg, tiny_model):
    cl = importlib.import_module(pkg.__name__ + ".cluster")
    rng = np.random.default_rng(12)
    tasks = []
    for i in range(7):
        text = pkg.ids_to_text(list(range(400 + 10 * i, 403 + 10 * i + i))) + " request"
        t = cl.UserTask(id=100 + i, text=text, seed=7 * i, max_steps=5 + i,
                        client_has_vocoder=(i % 2 == 0), stream_pcm=(i in (1, 5)),
                        cfg_scale=2.0 if i == 3 else 1.0)
        if i == 5:
            t.ref_text = pkg.ids_to_text([301, 302])
            t.ref_frames = 2
            t.ref_codes = rng.integers(0, 2048, (2, 8)).astype(np.int32).reshape(-1).tolist()
        tasks.append(t)
    packets, pcm_chunks, finals = {}, {}, {}

    def on_tokens(tid, packet, final):
        packets.setdefault(tid, []).append(packet)
        finals[tid] = finals.get(tid, 0) + int(final)

    def on_pcm(tid, pcm, final):
        pcm_chunks.setdefault(tid, []).append(np.asarray(pcm))
        finals[tid] = finals.get(tid, 0) + int(final)

    with cl.IslandCluster(tiny_model, devices=(0, 0), max_slots=3, chunk_size=4, slot_tiers=(2, 1, 1),
                          keep_tokens=True, keep_pcm=True) as cluster:
        results = cluster.run_workload(tasks, arrival_offsets=[0, 0, 0.01, 0.02, 0.05, 0.05, 0.1],
                                       on_tokens=on_tokens, on_pcm_chunk=on_pcm)
        assert all(g.active_session_count() == 0 for g in cluster.gens)
        nc, wc = cluster.gens[0].nc, cluster.wire_codes
    assert [r.id for r in results] == [t.id for t in tasks]
    voc = pkg.VocoderHandle(tiny_model, 0)
    try:
        for t, r in zip(tasks, results):
            n = r.frames.shape[0]
            assert 0 < n <= t.max_steps and r.frames.shape[1] == nc
            assert (r.frames[:, 0] >= 0).all() and (r.frames[:, 0] < 2048).all()
            assert finals[t.id] == 1, t.id
            if t.client_has_vocoder:
                assert "client tokens" in r.worker
                assert len(r.tokens) == n * wc
                wire = cl.unpack_frames(b"".join(packets[t.id]), width=wc)
                assert np.array_equal(wire, np.asarray(r.tokens).reshape(n, wc))
                assert np.array_equal(wire, r.frames[:, :wc])
                assert abs(r.audio_s - n * cl.FRAME_S) < 1e-6
                assert t.id not in pcm_chunks
            else:
                assert "server vocoder" in r.worker and r.tokens is None
                assert r.pcm.size == n * 1920 and abs(r.audio_s - n * 0.08) < 1e-3
                assert np.array_equal(np.concatenate(pcm_chunks[t.id]), r.pcm)
                # the same frames through a standalone vocoder session (one pass; the streamed
                # chunks see the same causal history)
                ref = voc.session_decode(9000 + t.id, r.frames)
                voc.session_free(9000 + t.id)
                assert snr_db(ref, r.pcm) > 60.0, (t.id, snr_db(ref, r.pcm))
            assert r.turnaround_s >= r.compute_wall_s >= 0 and r.ttfa_s <= r.turnaround_s + 1e-3
    finally:
        voc.close()


def test_islands_on_every_gpu(pkg, tiny_model):
    """One island per visible GPU on one shared job queue (the reference's DualInstanceCluster
    generalised, python/bz_ggml/cluster.py:402-414, 744-750): every request is served once, by
    some island, and every island takes part. Runs where the process sees two or more GPUs."""
    import torch
    n_gpu = torch.cuda.device_count()
    if n_gpu < 2:
        pytest.skip("needs two or more GPUs in the process")
    cl = importlib.import_module(pkg.__name__ + ".cluster")
    tasks = [cl.UserTask(id=500 + i, text=pkg.ids_to_text([600 + i, 700 + 3 * i, 800 + i]) + " spread", seed=i,
                         max_steps=12 + (i % 5), client_has_vocoder=(i % 3 == 0))
             for i in range(6 * n_gpu)]
    with cl.IslandCluster(tiny_model, devices=tuple(range(n_gpu)), max_slots=4, chunk_size=4, slot_tiers=(2, 1, 1),
                          keep_tokens=True, keep_pcm=True) as cluster:
        results = cluster.run_workload(tasks)
        assert all(g.active_session_count() == 0 for g in cluster.gens)
    assert sorted(r.id for r in results) == sorted(t.id for t in tasks)
    islands = {}
    for t, r in zip(tasks, results):
        n = r.frames.shape[0]
        assert 0 < n <= t.max_steps
        if not t.client_has_vocoder:
            assert r.pcm.size == n * 1920
        gpu = int(r.worker.split("GPU ")[1].split(" ")[0])
        islands[gpu] = islands.get(gpu, 0) + 1
    assert set(islands) == set(range(n_gpu)), islands
