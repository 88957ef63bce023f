"""breeze_generate / breeze_generate_wav on the GPU against the oracle (needs a B200).

The reference's streaming loop (src/generation.cpp:83-273) is checked piece by piece:
- Prompts: the instruction and, from the second piece on, the first piece's frames and text as
  the reference voice.
- Sampler: the request's values, zero keeping the GGUF's. The depth codes come from the GGUF's
  depth sampler.
- Budget: exactly max_new_tokens frames per piece. The model has no EOS row, so no piece ends early.
- Streaming: chunks ramp c -> c + c//3 + 1 from 4 to 25 frames. Each vocoder window decodes
  sliding_window + 16 frames of left context.
- WAV: the file holds the same PCM.

Tokens follow the engine (teacher forcing). Each draw must be reachable from the oracle's logits
with the same uniform. PCM must reach SNR >= 40 dB against the oracle's vocoder on the same frames.
"""
import numpy as np
import pytest

import breeze_oracle as bo
from parity_helpers import check_depth, flip_budget, reconcile_cb0, snr_db

pytestmark = pytest.mark.gpu

SNR_MIN_DB = 40.0
SPF = 1920


@pytest.fixture(scope="module")
def noeos_model(pkg, model_dir):
    return pkg.synth_model(str(model_dir / "tiny_noeos.gguf"), preset="tiny", seed=3, eos_off=True)


@pytest.fixture(scope="module")
def noeos_oracle(noeos_model):
    return bo.Model(noeos_model)


@pytest.fixture(scope="module")
def ctx(pkg, noeos_model):
    c = pkg.ContextHandle(noeos_model)
    yield c
    c.close()


def _params(cfg, top_k=0, temperature=0.0, rep=0.0):
    return bo.SamplerParams(temperature if temperature > 0 else cfg.temperature, top_k if top_k > 0 else cfg.top_k,
                            cfg.top_p, rep if rep > 0 else cfg.rep, cfg.depth_temperature, cfg.depth_top_k,
                            cfg.depth_top_p)


def _follow_piece(ref, m, sid, text, codes, seed, max_new, params, scale=1.0, ref_text=None, ref_codes=None):
    """Replays one piece on the oracle with the engine's frames; returns (tolerated flips, draws)."""
    nc = m.cfg.nc
    cb0, _ = ref.session_create(sid, text, ref_text=ref_text, ref_codes=ref_codes, seed=seed, max_new_tokens=max_new,
                                params=params, cfg_scale=scale, clamp_total=False)
    flips = 0
    if cb0 != int(codes[0, 0]):
        flips += reconcile_cb0(ref, sid, int(codes[0, 0]), cb0, scale, "first")
    for f in range(codes.shape[0]):
        dl = {}
        rf, rn = ref.step_batched([sid], forced_depth=codes[f:f + 1, 1:nc], depth_logits_out=dl, sampled_depth=True)
        assert rf[0][0] == codes[f, 0], f
        flips += check_depth(ref, nc, sid, codes[f, 1:nc], dl, scale, f)
        engine_next = int(codes[f + 1, 0]) if f + 1 < codes.shape[0] else -1
        flips += reconcile_cb0(ref, sid, engine_next, int(rn[0]), scale, f)
    assert not ref.sessions[sid].active  # the budget ends the piece
    return flips, codes.shape[0] * nc + 1


def _check_pcm(m, codes, pcm, sizes):
    want = bo.stream_chunks(bo.Vocoder(m), codes)
    assert [w.size for w in want] == sizes
    got = np.split(pcm, np.cumsum(sizes)[:-1])
    for w, g in zip(want, got):
        assert snr_db(w, g) > SNR_MIN_DB, snr_db(w, g)


def test_generate_one_piece_matches_oracle(pkg, ctx, noeos_oracle):
    m = noeos_oracle
    text = pkg.ids_to_text([300, 301, 4000, 77]) + " speak now"
    req = ctx.request(text, seed=5, max_new_tokens=12, split_chars=-1, top_k=1)
    pcm, sizes, codes, n, tm = ctx.generate(req)
    assert n == 12 and codes.shape == (12, m.cfg.nc)
    assert sizes == [4 * SPF, 6 * SPF, 2 * SPF]          # chunks 4, then 6 (4 + 1 + 1), then the rest
    assert tm["pieces"] == 1 and tm["frames"] == 12 and tm["flushes"] == 3 and tm["first_audio_ms"] > 0
    ref = bo.Generator(m)
    flips, draws = _follow_piece(ref, m, 0, text, codes, 5, 12, _params(m.cfg, top_k=1))
    assert flips <= flip_budget(draws)
    _check_pcm(m, codes, pcm, sizes)


def test_generate_pieces_carry_the_first_as_reference(pkg, ctx, noeos_oracle):
    m = noeos_oracle
    s1 = "The first sentence has quite a few words in it to weigh enough. "
    s2 = "A second sentence follows right after the first one with more words. "
    s3 = "The third sentence closes the text and ends up in a piece of its own."
    text = s1 + s2 + s3 + s1 + s2
    pieces = bo.split_text(text, 150, 200)
    assert len(pieces) == 3 and pkg.split_text(text, 150, 200) == pieces
    req = ctx.request(text, seed=11, max_new_tokens=5, split_chars=150, top_k=1, temperature=0.7)
    pcm, sizes, codes, n, tm = ctx.generate(req)
    assert n == 15 and tm["pieces"] == 3
    assert sizes == [4 * SPF, 1 * SPF] * 3
    ref = bo.Generator(m)
    p = _params(m.cfg, top_k=1, temperature=0.7)
    flips = draws = 0
    for i, piece in enumerate(pieces):
        # pieces after the first condition on the first piece's frames and text
        # (src/generation.cpp:228-242): the voice is kept across the seams
        anchor = dict(ref_text=pieces[0], ref_codes=codes[:5]) if i else {}
        f, d = _follow_piece(ref, m, i, piece, codes[5 * i:5 * i + 5], 11 + i, 5, p, **anchor)
        flips, draws = flips + f, draws + d
        _check_pcm(m, codes[5 * i:5 * i + 5], pcm[5 * i * SPF:5 * (i + 1) * SPF], sizes[2 * i:2 * i + 2])
    assert flips <= flip_budget(draws)


def test_generate_with_guidance_and_reference_codes(pkg, ctx, noeos_oracle):
    m = noeos_oracle
    nc = m.cfg.nc
    ref_codes = np.random.default_rng(3).integers(0, 2048, (3, nc)).astype(np.int32)
    text = pkg.ids_to_text([900, 901]) + " guided"
    req = ctx.request(text, ref_text=pkg.ids_to_text([10, 11, 12]), cfg_scale=2.0, seed=21, max_new_tokens=7,
                      split_chars=-1)
    pcm, sizes, codes, n, tm = ctx.generate(req, ref_codes=ref_codes)
    assert n == 7 and sizes == [4 * SPF, 3 * SPF]
    ref = bo.Generator(m)
    flips, draws = _follow_piece(ref, m, 0, text, codes, 21, 7, _params(m.cfg), scale=2.0,
                                 ref_text=pkg.ids_to_text([10, 11, 12]), ref_codes=ref_codes)
    assert flips <= flip_budget(draws)
    _check_pcm(m, codes, pcm, sizes)


def test_generate_stops_when_the_callback_says_so_and_wav_holds_the_pcm(pkg, ctx, noeos_oracle, tmp_path):
    text = pkg.ids_to_text([42, 43, 44]) + " stop early"
    req = ctx.request(text, seed=8, max_new_tokens=30, split_chars=-1)
    pcm, sizes, codes, n, tm = ctx.generate(req, stop_after_chunks=2)
    assert sizes == [4 * SPF, 6 * SPF] and n == 10        # frames made before the stop, no more
    full, fsizes, fcodes, fn, _ = ctx.generate(req)
    assert fn == 30 and np.array_equal(fcodes[:10], codes)  # same seed, same frames
    assert np.array_equal(full[:pcm.size], pcm)
    path = tmp_path / "out.wav"
    ctx.generate_wav(req, str(path))
    assert ctx.sample_rate == 24000
    assert path.read_bytes() == bo.wav_bytes(full, ctx.sample_rate)
