"""Host-side checks that need no GPU: the C ABI library loads and exports every declared
symbol, GGUF parsing and its errors, the tokenizer, voice files, the sampler semantics of
the oracle, and generator construction failing loudly without a device."""
import ctypes
import os
import re
import struct

import numpy as np
import pytest

import breeze_oracle as bo

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in ("breeze.h", "bzb_ext.h"):
        src = open(os.path.join(ROOT, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = "\n".join(l for l in src.splitlines() if not l.lstrip().startswith("#"))
        names |= set(re.findall(r"BREEZE_API[^;(]*?\b(\w+)\s*\(", src))
    return names


def test_library_exports_every_declared_symbol(pkg):
    lib = ctypes.CDLL(pkg.LIB_PATH)
    names = declared_symbols()
    assert len(names) >= 45
    for n in names:
        assert hasattr(lib, n), n
    assert names == set(pkg.SIGNATURES), names ^ set(pkg.SIGNATURES)


def test_reference_binding_names_are_all_exported(pkg):
    # the reference bindings bind these at load; a missing one makes BreezeLib() raise
    ref = ["breeze_generator_init", "breeze_generator_free", "breeze_generator_prefill", "breeze_generator_step_frame",
           "breeze_generator_session_create", "breeze_generator_session_create_ext", "breeze_generator_session_step",
           "breeze_generator_session_free", "breeze_generator_load_q4_depth", "breeze_generator_session_set_q4",
           "breeze_generator_session_count", "breeze_generator_sessions_step_round",
           "breeze_generator_sessions_step_batched", "breeze_generator_sessions_step_burst",
           "breeze_generator_convert_voice", "breeze_generator_encode_audio", "breeze_vocoder_init",
           "breeze_vocoder_create_from_generator", "breeze_vocoder_free", "breeze_vocoder_session_create",
           "breeze_vocoder_session_decode", "breeze_vocoder_session_decode_batch", "breeze_vocoder_session_free",
           "breeze_vocoder_stream_decode", "breeze_vocoder_stream_decode_batch", "breeze_init", "breeze_free",
           "breeze_sample_rate", "breeze_generate", "breeze_generate_wav", "breeze_last_error",
           "breeze_voice_save_file", "breeze_voice_load_file"]
    lib = ctypes.CDLL(pkg.LIB_PATH)
    for n in ref:
        assert hasattr(lib, n), n


def test_gguf_inspect_and_config(pkg, tiny_model, tiny_oracle):
    hidden, nc, nt = pkg.gguf_inspect(tiny_model)
    assert hidden == tiny_oracle.cfg.hidden and nc == tiny_oracle.cfg.nc
    assert nt == len(tiny_oracle.g.tensors)


def test_gguf_errors_are_reported(pkg, tiny_model, tmp_path):
    with pytest.raises(RuntimeError, match="cannot open"):
        pkg.gguf_inspect(str(tmp_path / "missing.gguf"))
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOPE" + b"\0" * 64)
    with pytest.raises(RuntimeError, match="magic"):
        pkg.gguf_inspect(str(bad))
    trunc = tmp_path / "trunc.gguf"
    trunc.write_bytes(open(tiny_model, "rb").read()[: 1 << 20])
    with pytest.raises(RuntimeError, match="past the end|truncated"):
        pkg.gguf_inspect(str(trunc))


@pytest.mark.parametrize("text", [
    "[S0]<ins_bos>Speak clearly and naturally.<ins_eos><|t300|><|t5000|> hi there",
    "héllo wörld ▁x <bos><|t128255|><|t264|>",
    "",
    "[S0][S0]<ins_eos>  double  spaces ",
])
def test_tokenizer_matches_oracle(pkg, tiny_model, tiny_oracle, text):
    assert pkg.tokenize(tiny_model, text) == tiny_oracle.tok.encode(text)
    assert pkg.tokenize(tiny_model, text, add_bos=False) == tiny_oracle.tok.encode(text, add_bos=False)


def test_ids_round_trip_through_text(pkg, tiny_model):
    ids = list(np.random.default_rng(0).integers(264, 128000, 200))
    assert pkg.tokenize(tiny_model, pkg.ids_to_text(ids), add_bos=False) == ids


def _brzv_bytes(text, codes, sr, ncb):
    # layout of the reference's voice files: magic, five u32 (version, rate, codebooks,
    # frames, text length), text, then i32 codes
    codes = np.asarray(codes, np.int32).reshape(-1)
    frames = codes.size // ncb
    tb = text.encode("utf-8")
    return b"BRZV" + struct.pack("<5I", 1, sr, ncb, frames, len(tb)) + tb + codes.astype("<i4").tobytes()


def test_voice_file_round_trip_and_layout(pkg, tmp_path):
    lib = pkg.lib().lib
    codes = np.random.default_rng(0).integers(-1, 2048, (125, 16)).astype(np.int32)
    path = str(tmp_path / "voices" / "alice.breeze")
    rc = lib.breeze_voice_save_file(path.encode(), b"alice", "héllo".encode(), codes.ctypes.data_as(ctypes.POINTER(ctypes.c_int)),
                                    125, 16, 24000)
    assert rc == 0
    assert open(path, "rb").read() == _brzv_bytes("héllo", codes, 24000, 16)
    name = ctypes.create_string_buffer(64)
    text = ctypes.create_string_buffer(64)
    out = np.zeros(125 * 16, np.int32)
    nf, ncb, sr = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    n = lib.breeze_voice_load_file(path.encode(), name, 64, text, 64, out.ctypes.data_as(ctypes.POINTER(ctypes.c_int)),
                                   ctypes.byref(nf), ctypes.byref(ncb), ctypes.byref(sr))
    assert n == 125 * 16 and name.value == b"alice" and text.value.decode() == "héllo"
    assert (nf.value, ncb.value, sr.value) == (125, 16, 24000)
    assert np.array_equal(out, codes.reshape(-1))


def test_corrupt_voice_file_rejected(pkg, tmp_path):
    lib = pkg.lib().lib
    bad = tmp_path / "bad.breeze"
    bad.write_bytes(b"BRZV" + struct.pack("<5I", 1, 24000, 9999, 10, 0))
    out = np.zeros(16, np.int32)
    nf, ncb = ctypes.c_int(), ctypes.c_int()
    assert lib.breeze_voice_load_file(str(bad).encode(), None, 0, None, 0, out.ctypes.data_as(ctypes.POINTER(ctypes.c_int)),
                                      ctypes.byref(nf), ctypes.byref(ncb), None) == -1


def test_generator_without_gpu_fails_loudly(pkg, tiny_model):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    with pytest.raises(RuntimeError, match="CUDA"):
        pkg.GeneratorHandle(tiny_model, 0)
    with pytest.raises(RuntimeError, match="CUDA"):
        pkg.VocoderHandle(tiny_model, 0)


def test_oracle_conv_ops_follow_their_definitions():
    """The restated conv ops against their defining sums on small random inputs: causal conv
    (zero history, dilation), transposed conv truncated to L * stride, causal depthwise."""
    rng = np.random.default_rng(4)
    x = rng.standard_normal((3, 11)).astype(np.float32)
    w = rng.standard_normal((5, 3, 4)).astype(np.float32)
    b = rng.standard_normal(5).astype(np.float32)
    y = bo.conv1d_causal(x, w, b, 1, 2)
    ref = np.zeros((5, 11))
    for o in range(5):
        for t in range(11):
            ref[o, t] = b[o] + sum(w[o, i, k] * x[i, t - (3 - k) * 2] for i in range(3) for k in range(4) if t - (3 - k) * 2 >= 0)
    assert np.allclose(y, ref, atol=1e-4)
    wt = rng.standard_normal((3, 5, 6)).astype(np.float32)
    y = bo.convtr1d_causal(x, wt, b, 3)
    ref = np.zeros((5, 33))
    for o in range(5):
        for u in range(33):
            ref[o, u] = b[o] + sum(wt[i, o, k] * x[i, (u - k) // 3] for i in range(3) for k in range(6)
                                   if u - k >= 0 and (u - k) % 3 == 0 and (u - k) // 3 < 11)
    assert np.allclose(y, ref, atol=1e-4)
    wd = rng.standard_normal((7, 3)).astype(np.float32)
    y = bo.depthwise1d_causal(x, wd, b[:3])
    ref = np.array([[b[c] + sum(wd[k, c] * x[c, t - 6 + k] for k in range(7) if t - 6 + k >= 0) for t in range(11)] for c in range(3)])
    assert np.allclose(y, ref, atol=1e-4)


# ---- sampler semantics (src/sampling.cpp:9-60) on the CPU ---------------------------------
def _ref_lib():
    """The reference's own sampler and voice codec, compiled from its sources into oracle/_ref
    (`make -C oracle ref`); skips where neither the build nor the reference checkout exists."""
    path = os.path.join(ROOT, "oracle", "_ref", "libref_host.so")
    if not os.path.exists(path):
        import subprocess
        r = subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "ref"], capture_output=True)
        if r.returncode != 0 or not os.path.exists(path):
            pytest.skip("the reference's host code is not built here")
    lib = ctypes.CDLL(path)
    lib.ref_sample_tokens.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.c_int, ctypes.c_float, ctypes.c_int,
                                      ctypes.c_float, ctypes.c_float, ctypes.POINTER(ctypes.c_int), ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int, ctypes.c_uint, ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
    return lib


def mt_draws(logits, n, temp=0.9, top_k=50, top_p=1.0, rep=1.0, hist=(), sup=(2048, 2051), seed=1):
    lib = _ref_lib()
    l = np.ascontiguousarray(logits, np.float32)
    h = np.asarray(hist, np.int32) if len(hist) else np.zeros(1, np.int32)
    out = np.zeros(n, np.int32)
    lib.ref_sample_tokens(l.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), l.size, temp, top_k, top_p, rep,
                          h.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), len(hist), sup[0], sup[1], seed, n,
                          out.ctypes.data_as(ctypes.POINTER(ctypes.c_int)))
    return out


def philox_draws(logits, n, temp=0.9, top_k=50, top_p=1.0, rep=1.0, hist=None, sup=(2048, 2051), seed=1):
    l = bo.apply_penalties(logits, rep, hist, sup[0], sup[1])
    return np.array([bo.sample_philox(l, temp, top_k, top_p, bo.philox_uniform(seed, d)) for d in range(n)])


def test_philox_sampler_matches_mt19937_distribution():
    rng = np.random.default_rng(5)
    logits = (rng.standard_normal(2052) * 1.5).astype(np.float32)
    n = 3000
    a = mt_draws(logits, n)
    b = philox_draws(logits, n)
    # both only ever draw from the same top-50 set
    top = set(np.argsort(-logits[:2048])[:50])
    assert set(a) <= top and set(b) <= top
    # chi-square two-sample homogeneity over the top-50 categories
    cats = sorted(top)
    ca = np.array([np.sum(a == c) for c in cats], float)
    cb = np.array([np.sum(b == c) for c in cats], float)
    keep = (ca + cb) >= 10
    tot = ca[keep] + cb[keep]
    ea, eb = tot * n / (2 * n), tot * n / (2 * n)
    chi2 = np.sum((ca[keep] - ea) ** 2 / ea + (cb[keep] - eb) ** 2 / eb)
    dof = keep.sum() - 1
    assert chi2 < dof + 6 * np.sqrt(2 * dof), (chi2, dof)


def test_sampler_greedy_suppression_and_repetition_penalty():
    logits = np.zeros(2052, np.float32)
    logits[2049] = 50.0          # suppressed [2048, 2051)
    logits[10] = 3.0
    logits[11] = 2.5
    for draws in (mt_draws(logits, 20, top_k=1), philox_draws(logits, 20, top_k=1)):
        assert set(draws) == {10}
    # the penalty is applied once per history occurrence: 3.0 / 1.1 > 2.5 > 3.0 / 1.1^2
    assert set(mt_draws(logits, 10, top_k=1, rep=1.1, hist=[10, 10])) == {11}
    assert set(philox_draws(logits, 10, top_k=1, rep=1.1, hist={10: 2})) == {11}
    assert set(philox_draws(logits, 10, top_k=1, rep=1.1, hist={10: 1})) == {10}
    # EOS (2051) is not suppressed
    logits[2051] = 60.0
    assert set(philox_draws(logits, 5, top_k=1)) == {2051}


def test_session_budget_semantics(tiny_oracle):
    """max_new_tokens <= 0 estimates ceil(1.5*words)+30 capped at 1000; the total is clamped
    to 2040 with a floor of 64 frames (src/c_api.cpp:354-364, 398-405)."""
    g = bo.Generator(tiny_oracle)
    text = "one two three four"
    e = np.zeros((10, tiny_oracle.cfg.hidden), np.float32)
    _, alloc = g.session_create(1, text, embeds=e, max_new_tokens=0)
    assert alloc == 10 + (int(np.ceil(4 * 1.5)) + 30) + 8
    e = np.zeros((2000, tiny_oracle.cfg.hidden), np.float32)
    _, alloc = g.session_create(2, text, embeds=e, max_new_tokens=500)
    assert alloc == 2000 + 64 + 8


def test_sample_reachable_bounds():
    """The parity tests' tolerance for sampled cb0 ids: the oracle's own draw is always
    reachable, a draw far from the uniform's CDF position never is, and a boundary token
    becomes reachable once the logit tolerance covers the gap."""
    rng = np.random.default_rng(8)
    logits = (rng.standard_normal(2052) * 2).astype(np.float32)
    for d in range(50):
        u = bo.philox_uniform(3, d)
        tok = bo.sample_philox(logits, 0.9, 50, 1.0, u)
        assert bo.sample_reachable(logits, 0.9, 50, u, tok, 0.0)
    order = np.lexsort((np.arange(2052), -logits.astype(np.float64)))
    u = np.float32(0.001)                     # the top token's interval
    assert not bo.sample_reachable(logits, 0.9, 50, u, int(order[30]), 0.02)
    assert not bo.sample_reachable(logits, 0.9, 50, u, int(order[200]), 0.02)
    # two equal top logits: u just past the first interval reaches the first token only with a tolerance
    l2 = np.full(2052, -10.0, np.float32)
    l2[5] = l2[6] = 1.0
    u = np.float32(0.51)
    assert bo.sample_philox(l2, 0.9, 50, 1.0, u) == 6
    assert not bo.sample_reachable(l2, 0.9, 50, u, 5, 0.0)
    assert bo.sample_reachable(l2, 0.9, 50, u, 5, 0.02)
