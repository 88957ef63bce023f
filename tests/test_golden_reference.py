"""Pins against the reference itself: the committed fixtures in tests/golden (made by
tests/golden/make_golden.py from the reference's Python serializer and its compiled C++
sampler) and, where oracle/_ref is built, the reference's compiled host code live. CPU only."""
import ctypes
import importlib.util
import os

import numpy as np
import pytest

import breeze_oracle as bo

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
ROOT = os.path.dirname(HERE)


def _golden_module():
    spec = importlib.util.spec_from_file_location("make_golden", os.path.join(GOLDEN, "make_golden.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


MG = _golden_module()


def _ref_lib():
    path = os.path.join(ROOT, "oracle", "_ref", "libref_host.so")
    if not os.path.exists(path):
        import subprocess
        r = subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "ref"], capture_output=True)
        if r.returncode != 0 or not os.path.exists(path):
            pytest.skip("the reference's host code is not built here")
    return ctypes.CDLL(path)


def _save_ours(lib, path, text, codes, frames, ncb, sr):
    return lib.breeze_voice_save_file(path.encode(), b"x", text.encode("utf-8"),
                                      codes.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), frames, ncb, sr)


def _load_ours(lib, path, max_codes):
    name = ctypes.create_string_buffer(256)
    text = ctypes.create_string_buffer(4096)
    out = np.zeros(max_codes, np.int32)
    nf, ncb, sr = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    n = lib.breeze_voice_load_file(path.encode(), name, 256, text, 4096, out.ctypes.data_as(ctypes.POINTER(ctypes.c_int)),
                                   ctypes.byref(nf), ctypes.byref(ncb), ctypes.byref(sr))
    return n, name.value.decode(), text.value.decode("utf-8"), out[:max(n, 0)], nf.value, ncb.value, sr.value


@pytest.mark.parametrize("case", MG.VOICES, ids=[v[0] for v in MG.VOICES])
def test_voice_writer_matches_reference_fixture_bytes(pkg, tmp_path, case):
    name, text, frames, ncb, sr, seed = case
    codes = MG.voice_codes(frames, ncb, seed)
    lib = pkg.lib().lib
    path = str(tmp_path / f"{name}.breeze")
    assert _save_ours(lib, path, text, codes, frames, ncb, sr) == 0
    assert open(path, "rb").read() == open(os.path.join(GOLDEN, f"voice_{name}.breeze"), "rb").read()


@pytest.mark.parametrize("case", MG.VOICES, ids=[v[0] for v in MG.VOICES])
def test_voice_loader_reads_reference_fixture(pkg, case):
    name, text, frames, ncb, sr, seed = case
    n, got_name, got_text, codes, nf, nc, rate = _load_ours(pkg.lib().lib, os.path.join(GOLDEN, f"voice_{name}.breeze"),
                                                           frames * ncb)
    assert n == frames * ncb and (nf, nc, rate) == (frames, ncb, sr)
    assert got_name == f"voice_{name}" and got_text == text
    assert np.array_equal(codes, MG.voice_codes(frames, ncb, seed))


def test_reference_voice_codec_round_trips_with_ours(pkg, tmp_path):
    ref = _ref_lib()
    lib = pkg.lib().lib
    codes = MG.voice_codes(7, 16, 9)
    ours = str(tmp_path / "ours.breeze")
    theirs = str(tmp_path / "theirs.breeze")
    assert _save_ours(lib, ours, "abc déf", codes, 7, 16, 24000) == 0
    assert ref.ref_voice_save(theirs.encode(), "abc déf".encode(), codes.ctypes.data_as(ctypes.c_void_p), 7, 16, 24000) == 0
    assert open(ours, "rb").read() == open(theirs, "rb").read()
    out = np.zeros(7 * 16, np.int32)
    f, c, r = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    assert ref.ref_voice_load(ours.encode(), None, 0, None, 0, out.ctypes.data_as(ctypes.c_void_p), out.size,
                              ctypes.byref(f), ctypes.byref(c), ctypes.byref(r)) == 7 * 16
    assert np.array_equal(out, codes)
    # a header the reference rejects (codebooks > 64) is rejected by ours too
    bad = tmp_path / "bad.breeze"
    bad.write_bytes(open(ours, "rb").read()[:12] + (65).to_bytes(4, "little") + open(ours, "rb").read()[16:])
    assert ref.ref_voice_load(str(bad).encode(), None, 0, None, 0, out.ctypes.data_as(ctypes.c_void_p), out.size,
                              ctypes.byref(f), ctypes.byref(c), ctypes.byref(r)) == -1
    assert _load_ours(lib, str(bad), out.size)[0] == -1


def _fixture():
    return np.load(os.path.join(GOLDEN, "sampler_mt.npz"))


def test_reference_sampler_reproduces_fixture():
    ref = _ref_lib()
    fx = _fixture()
    for name, seed, temp, k, p, rep, hist, sup, n in MG.SAMPLER_CASES:
        logits = fx[name + "_logits"]
        assert np.array_equal(logits, MG.sampler_logits(seed))
        h = np.asarray(hist if hist else [0], np.int32)
        toks = np.zeros(n, np.int32)
        ref.ref_sample_tokens(logits.ctypes.data_as(ctypes.c_void_p), ctypes.c_int(logits.size), ctypes.c_float(temp),
                              ctypes.c_int(k), ctypes.c_float(p), ctypes.c_float(rep), h.ctypes.data_as(ctypes.c_void_p),
                              ctypes.c_int(len(hist)), ctypes.c_int(sup[0]), ctypes.c_int(sup[1]), ctypes.c_uint(seed),
                              ctypes.c_int(n), toks.ctypes.data_as(ctypes.c_void_p))
        assert np.array_equal(toks, fx[name + "_tokens"]), name


def _hist_counts(hist):
    out = {}
    for t in hist:
        out[t] = out.get(t, 0) + 1
    return out


@pytest.mark.parametrize("case", MG.SAMPLER_CASES, ids=[c[0] for c in MG.SAMPLER_CASES])
def test_philox_sampler_matches_reference_draws(case):
    """The engine's sampler semantics (oracle Philox mode) against the reference's own
    std::mt19937 draws: the same support, and the same distribution by a chi-square two-sample
    homogeneity test; a greedy case must agree draw for draw."""
    name, seed, temp, k, p, rep, hist, sup, n = case
    fx = _fixture()
    ref_toks = fx[name + "_tokens"]
    logits = bo.apply_penalties(fx[name + "_logits"], rep, _hist_counts(hist), sup[0], sup[1])
    ours = np.array([bo.sample_philox(logits, temp, k, p, bo.philox_uniform(seed, d)) for d in range(n)])
    if k == 1:
        assert np.array_equal(ours, ref_toks)
        return
    assert not (set(range(sup[0], sup[1])) & set(ours))
    if k > 0:
        top = set(np.lexsort((np.arange(logits.size), -logits.astype(np.float64)))[:k].tolist())
        assert set(ours.tolist()) <= top and set(ref_toks.tolist()) <= top
    cats = sorted(set(ref_toks) | set(ours))
    ca = np.array([np.sum(ref_toks == c) for c in cats], float)
    cb = np.array([np.sum(ours == c) for c in cats], float)
    keep = (ca + cb) >= 10
    # categories too rare to test are pooled into one
    ca = np.append(ca[keep], ca[~keep].sum())
    cb = np.append(cb[keep], cb[~keep].sum())
    m = (ca + cb) > 0
    ca, cb = ca[m], cb[m]
    e = (ca + cb) / 2
    chi2 = np.sum((ca - e) ** 2 / e + (cb - e) ** 2 / e)
    dof = len(ca) - 1
    assert chi2 < dof + 6 * np.sqrt(2 * dof), (chi2, dof)
    # and the support: every id the reference drew at least 1% of the time appears in ours
    frequent = {c for c in cats if np.sum(ref_toks == c) > n // 100}
    assert frequent <= set(ours)


def test_reference_bindings_bind_this_library(pkg, reference_bindings, tiny_model, tmp_path):
    """The drop-in check: the reference's unmodified ctypes bindings load libbreeze.so, bind
    every symbol they declare, and see the reference's error conventions."""
    rb = reference_bindings
    lib = rb.BreezeLib(pkg.LIB_PATH)
    assert lib.lib_path == pkg.LIB_PATH
    import torch
    if not torch.cuda.is_available():
        with pytest.raises(RuntimeError, match="Failed to initialize Generator"):
            rb.GeneratorHandle(lib, tiny_model, 0)
        assert "CUDA" in pkg.lib().last_error()
    # the reference's Python voice files and this library's C reader/writer interoperate
    codes = MG.voice_codes(4, 16, 5)
    path = str(tmp_path / "v" / "bob.breeze")
    rb.save_breeze_voice(path, "hi there", codes.tolist(), 4)
    n, name, text, got, nf, ncb, sr = _load_ours(lib.lib, path, 64)
    assert (n, name, text, nf, ncb, sr) == (64, "bob", "hi there", 4, 16, 24000)
    assert np.array_equal(got, codes)
    ours = str(tmp_path / "ours.breeze")
    assert _save_ours(lib.lib, ours, "hi there", codes, 4, 16, 24000) == 0
    v = rb.load_breeze_voice(ours)
    assert v["codes"] == codes.tolist() and v["text"] == "hi there" and v["name"] == "ours"


def _split_cases():
    import json
    with open(os.path.join(GOLDEN, "split_text.json"), encoding="utf-8") as f:
        return json.load(f)


def test_split_text_matches_reference_fixture(pkg):
    """The long-text splitter of breeze_generate, the library's (C++) and the oracle's, against
    the pieces the reference's own src/text_split.cpp returned for the same texts and budgets."""
    cases = _split_cases()
    assert len(cases) >= 200
    for c in cases:
        assert bo.split_text(c["text"], c["budget"], c["first_budget"]) == c["pieces"], c["name"]
        assert pkg.split_text(c["text"], c["budget"], c["first_budget"]) == c["pieces"], c["name"]


def test_split_text_matches_reference_live(pkg):
    ref = _ref_lib()
    rng = np.random.default_rng(2024)
    for _ in range(500):
        text = "".join(MG.FUZZ_ALPHABET[j] for j in rng.integers(0, len(MG.FUZZ_ALPHABET), int(rng.integers(0, 200))))
        budget, first = int(rng.integers(-1, 60)), int(rng.integers(-1, 30))
        raw = text.encode("utf-8")
        buf = ctypes.create_string_buffer(-ref.ref_split_text(raw, budget, first, None, 0))
        n = ref.ref_split_text(raw, budget, first, buf, len(buf))
        want = [p.decode("utf-8") for p in buf.raw.split(b"\0")[:n]]
        assert pkg.split_text(text, budget, first) == want, (text, budget, first)


def test_wav_writer_matches_reference_fixture(pkg, tmp_path):
    """breeze_generate_wav's file layout: the library's writer and the oracle's restatement give the
    bytes the reference's src/audio.cpp wrote for the same samples (clamping and truncation)."""
    with open(os.path.join(GOLDEN, "wav_ref.wav"), "rb") as f:
        want = f.read()
    x = MG.wav_samples()
    out = tmp_path / "ours.wav"
    pkg.write_wav(str(out), x, 24000)
    assert out.read_bytes() == want
    assert bo.wav_bytes(x, 24000) == want
