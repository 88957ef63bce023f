"""The CUDA codec decoder against the oracle's restatement of the reference's decode graph
(src/codec_decoder.cpp:65-98) and vocoder session semantics (src/c_api.cpp:952-1229), through
the C ABI (needs a B200). Bar: PCM SNR >= 40 dB against the oracle."""
import numpy as np
import pytest

import breeze_oracle as bo

pytestmark = pytest.mark.gpu

SNR_MIN_DB = 40.0


def snr_db(ref, out):
    ref = np.asarray(ref, np.float64)
    err = ref - np.asarray(out, np.float64)
    return 10.0 * np.log10((ref @ ref) / max(err @ err, 1e-30))


@pytest.fixture(scope="module")
def voc(pkg, tiny_model):
    v = pkg.VocoderHandle(tiny_model, 0)
    yield v
    v.close()


@pytest.fixture(scope="module")
def ovoc(tiny_oracle):
    return bo.Vocoder(tiny_oracle)


def _codes(nc, T, seed):
    return np.random.default_rng(seed).integers(0, 2051, (T, nc)).astype(np.int32)


@pytest.mark.parametrize("T", [1, 3, 17])
def test_stream_decode_matches_oracle(voc, ovoc, tiny_oracle, T):
    codes = _codes(tiny_oracle.cfg.nc, T, T)
    pcm = voc.stream_decode(codes)
    ref = ovoc.decode(codes, T)
    assert pcm.shape == ref.shape == (T * 1920,)
    assert np.abs(pcm).max() <= 1.0
    assert snr_db(ref, pcm) > SNR_MIN_DB, snr_db(ref, pcm)


def test_session_windows_match_oracle(pkg, tiny_model, tiny_oracle):
    """Chunks of 5, 1, 20 and 9 frames: each decode covers the kept history (at most 32 frames)
    plus the new frames and returns only the new frames' samples."""
    v = pkg.VocoderHandle(tiny_model, 0)
    ov = bo.Vocoder(tiny_oracle)
    try:
        assert v.session_create(4) == 0
        rng = np.random.default_rng(9)
        for n in (5, 1, 20, 9):
            frames = rng.integers(0, 2051, (n, tiny_oracle.cfg.nc)).astype(np.int32)
            pcm = v.session_decode(4, frames)
            ref = ov.session_decode(4, frames, n)
            assert pcm.shape == (n * 1920,)
            assert snr_db(ref, pcm) > SNR_MIN_DB, (n, snr_db(ref, pcm))
        assert v.session_free(4) == 0
        assert v.session_free(4) == -1
    finally:
        v.close()


def test_session_decode_batch_and_unknown_session(pkg, tiny_model, tiny_oracle):
    v = pkg.VocoderHandle(tiny_model, 0)
    ov = bo.Vocoder(tiny_oracle)
    try:
        nc = tiny_oracle.cfg.nc
        a, b = _codes(nc, 3, 1), _codes(nc, 2, 2)
        # session 8 was never created: decoding creates it (src/c_api.cpp:1011-1018)
        out = v.session_decode_batch([7, 8], [a, b])
        assert [o.shape[0] for o in out] == [3 * 1920, 2 * 1920]
        assert snr_db(ov.session_decode(7, a, 3), out[0]) > SNR_MIN_DB
        assert snr_db(ov.session_decode(8, b, 2), out[1]) > SNR_MIN_DB
        # the second call sees each session's history
        a2 = _codes(nc, 2, 3)
        out2 = v.session_decode_batch([7], [a2])
        assert snr_db(ov.session_decode(7, a2, 2), out2[0]) > SNR_MIN_DB
    finally:
        v.close()


def test_vocoder_from_generator_matches_standalone(pkg, tiny_model, voc, tiny_oracle):
    g = pkg.GeneratorHandle(tiny_model, 0)
    try:
        v2 = pkg.VocoderHandle(generator=g)
        codes = _codes(tiny_oracle.cfg.nc, 4, 5)
        assert np.array_equal(v2.stream_decode(codes), voc.stream_decode(codes))
        v2.close()
    finally:
        g.close()


def test_full_size_vocoder_matches_oracle(pkg, model_dir):
    """The full-size decoder shapes (1536-channel conv stack, 8-layer transformer) on a few frames."""
    path = pkg.synth_model(str(model_dir / "depth_voc.gguf"), preset="depth", nc=32, seed=1)
    v = pkg.VocoderHandle(path, 0)
    try:
        m = bo.Model(path)
        codes = _codes(m.cfg.nc, 3, 11)
        pcm = v.stream_decode(codes)
        ref = bo.Vocoder(m).decode(codes, 3)
        assert snr_db(ref, pcm) > SNR_MIN_DB, snr_db(ref, pcm)
    finally:
        v.close()
