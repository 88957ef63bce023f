"""Streaming PCM through the C ABI (needs a B200).

A vocoder stream carries the codec decoder's causal state between calls, so the PCM of a stream
decoded a few frames at a time must equal one decode of all its frames: the oracle's
`Vocoder.decode` of the whole history is the reference (SNR >= 40 dB). Several streams decoded
in one call run as one batch; their PCM must not depend on which other streams share the call.
The serving step (`bzb_generator_sessions_step_pcm`) decodes each session's new frame on the
session's stream; the device-resident variant must give the same PCM as the host-buffer one.
"""
import numpy as np
import pytest

import breeze_oracle as bo
from parity_helpers import snr_db

pytestmark = pytest.mark.gpu

SNR_MIN_DB = 40.0


def _codes(nc, T, seed):
    return np.random.default_rng(seed).integers(0, 2051, (T, nc)).astype(np.int32)


@pytest.fixture(scope="module")
def voc(pkg, tiny_model):
    v = pkg.VocoderHandle(tiny_model, 0)
    yield v
    v.close()


@pytest.fixture(scope="module")
def ovoc(tiny_oracle):
    return bo.Vocoder(tiny_oracle)


def test_stream_chunks_equal_one_decode_of_the_history(voc, ovoc, tiny_oracle):
    nc = tiny_oracle.cfg.nc
    chunks = [1, 3, 1, 7, 2, 1, 12, 5]   # 32 frames, past the tiny model's attention window of 8
    total = sum(chunks)
    codes = {sid: _codes(nc, total, sid) for sid in (11, 12, 13)}
    got = {sid: [] for sid in codes}
    t = 0
    for n in chunks:
        ids = list(codes)
        pcm = voc.streams_decode(ids, np.stack([codes[s][t:t + n] for s in ids]))
        assert pcm.shape == (3, n * 1920)
        for i, s in enumerate(ids):
            got[s].append(pcm[i])
        t += n
    for s in codes:
        ref = ovoc.decode(codes[s], total)
        out = np.concatenate(got[s])
        assert np.abs(out).max() <= 1.0
        assert snr_db(ref, out) > SNR_MIN_DB, (s, snr_db(ref, out))
    for s in codes:
        assert voc.stream_close(s)
    assert not voc.stream_close(11)


def test_streams_independent_of_batch_company(voc, tiny_oracle):
    """A stream decoded alone and decoded in a batch with other streams gives the same PCM."""
    nc = tiny_oracle.cfg.nc
    a, b, c = _codes(nc, 6, 1), _codes(nc, 6, 2), _codes(nc, 6, 3)
    solo = np.concatenate([voc.streams_decode([21], a[None, t:t + 2])[0] for t in (0, 2, 4)])
    voc.stream_close(21)
    mixed = []
    for t in (0, 2, 4):
        pcm = voc.streams_decode([22, 21, 23], np.stack([b[t:t + 2], a[t:t + 2], c[t:t + 2]]))
        mixed.append(pcm[1])
    mixed = np.concatenate(mixed)
    assert snr_db(solo, mixed) > 100.0, snr_db(solo, mixed)
    for s in (21, 22, 23):
        voc.stream_close(s)


def test_stream_reopen_restarts(voc, tiny_oracle):
    nc = tiny_oracle.cfg.nc
    a = _codes(nc, 4, 7)
    first = voc.streams_decode([31], a[None])
    voc.streams_decode([31], a[None])          # the stream moves on
    voc.stream_open(31)                         # and starts over
    again = voc.streams_decode([31], a[None])
    assert np.array_equal(first, again)
    voc.stream_close(31)


def test_stream_rejects_duplicate_ids(voc, tiny_oracle):
    nc = tiny_oracle.cfg.nc
    with pytest.raises(RuntimeError, match="twice"):
        voc.streams_decode([41, 41], np.stack([_codes(nc, 1, 1), _codes(nc, 1, 2)]))


def test_batched_windowed_sessions_match_oracle(pkg, tiny_model, tiny_oracle):
    """breeze_vocoder_session_decode_batch decodes entries of equal window length together; each
    entry's PCM still equals the reference's windowed decode of its own history."""
    v = pkg.VocoderHandle(tiny_model, 0)
    ov = bo.Vocoder(tiny_oracle)
    try:
        nc = tiny_oracle.cfg.nc
        rng = np.random.default_rng(4)
        ids = [51, 52, 53, 54, 55]
        for rnd, sizes in enumerate([(2, 2, 3, 2, 1), (4, 4, 4, 1, 4), (30, 30, 2, 30, 30), (3, 3, 3, 3, 3)]):
            frames = [rng.integers(0, 2051, (n, nc)).astype(np.int32) for n in sizes]
            out = v.session_decode_batch(ids, frames)
            for sid, f, o in zip(ids, frames, out):
                ref = ov.session_decode(sid, f, f.shape[0])
                assert snr_db(ref, o) > SNR_MIN_DB, (rnd, sid, snr_db(ref, o))
    finally:
        v.close()


def test_full_size_streams_match_oracle(pkg, model_dir):
    """The full-size decoder (1536-channel conv stack, 8 layers, window 72) streamed frame by frame
    for 4 streams, against one oracle decode of each stream's frames."""
    path = pkg.synth_model(str(model_dir / "depth_voc.gguf"), preset="depth", nc=32, seed=1)
    v = pkg.VocoderHandle(path, 0)
    try:
        m = bo.Model(path)
        nc = m.cfg.nc
        T = 6
        codes = np.stack([_codes(nc, T, 100 + i) for i in range(4)])
        got = [[] for _ in range(4)]
        for t, n in ((0, 1), (1, 1), (2, 3), (5, 1)):
            pcm = v.streams_decode([0, 1, 2, 3], codes[:, t:t + n])
            for i in range(4):
                got[i].append(pcm[i])
        ov = bo.Vocoder(m)
        for i in range(4):
            ref = ov.decode(codes[i], T)
            out = np.concatenate(got[i])
            assert snr_db(ref, out) > SNR_MIN_DB, (i, snr_db(ref, out))
    finally:
        v.close()


def test_step_pcm_streams_each_session(pkg, tiny_model, tiny_oracle):
    """bzb_generator_sessions_step_pcm: frames as sessions_step_burst gives them, and the PCM of
    each session's frames so far equals one decode of them; a session created again under the
    same id starts a new stream."""
    cfg = tiny_oracle.cfg
    gen = pkg.GeneratorHandle(tiny_model, 0)
    voc = pkg.VocoderHandle(generator=gen)
    ov = bo.Vocoder(tiny_oracle)
    try:
        ids = [61, 62, 63]
        budgets = {61: 9, 62: 4, 63: 9}
        for sid in ids:
            gen.session_create_ext(sid, pkg.ids_to_text([sid, 3 * sid, 7 * sid]), seed=sid, max_new_tokens=budgets[sid])
        frames = {sid: [] for sid in ids}
        pcms = {sid: [] for sid in ids}
        for step in range(6):
            live, fr, nxt, pcm = gen.step_pcm(voc, ids, seeds=[step + s for s in ids])
            for i, sid in enumerate(ids):
                if fr[i, 0] >= 0:
                    frames[sid].append(fr[i])
                    pcms[sid].append(pcm[i])
                else:
                    assert (pcm[i] == 0).all()
        assert len(frames[62]) == 4 and len(frames[61]) == 6
        for sid in ids:
            f = np.stack(frames[sid])
            ref = ov.decode(f, f.shape[0])
            out = np.concatenate(pcms[sid])
            assert snr_db(ref, out) > SNR_MIN_DB, (sid, snr_db(ref, out))
        # session 62 again under the same id: its first frame decodes as a new stream
        gen.session_create_ext(62, pkg.ids_to_text([5, 6]), seed=3, max_new_tokens=3)
        _, fr, _, pcm = gen.step_pcm(voc, [62], seeds=[1])
        ref = ov.decode(fr[0][None], 1)
        assert snr_db(ref, pcm[0]) > SNR_MIN_DB
    finally:
        voc.close()
        gen.close()


def test_step_pcm_device_equals_host_path(pkg, tiny_model):
    """The device-resident serving steps leave the same PCM as the host-buffer call (identical
    sessions on two generators; the steps are deterministic)."""
    outs = []
    for mode in ("host", "device"):
        gen = pkg.GeneratorHandle(tiny_model, 0)
        voc = pkg.VocoderHandle(generator=gen)
        try:
            ids = [71, 72, 73, 74, 75]
            for sid in ids:
                gen.session_create_ext(sid, pkg.ids_to_text([sid, sid + 9]), seed=sid, max_new_tokens=20)
            for step in range(4):
                seeds = [10 * step + s for s in ids]
                if mode == "host":
                    _, _, _, pcm = gen.step_pcm(voc, ids, seeds=seeds)
                else:
                    gen.step_pcm_device(voc, ids, seeds=seeds)
            if mode == "device":
                pcm = voc.last_pcm(len(ids) * 1920).reshape(len(ids), 1920)
            outs.append(pcm)
        finally:
            voc.close()
            gen.close()
    assert np.array_equal(outs[0], outs[1])
