"""Generates the golden fixtures in this folder from the reference itself (run where the
reference checkout is present; the fixtures are committed so that the tests need neither).

  voice_*.breeze   BRZV bytes written by the reference's own Python serializer
                   (python/bz_ggml/bindings.py:606-611, serialize_breeze_voice)
  sampler_mt.npz   logits and the token sequences drawn from them by the reference's own C++
                   sampler (src/sampling.cpp:9-60, compiled unmodified into oracle/_ref by
                   `make -C oracle ref`), std::mt19937 seeded per case

usage: python tests/golden/make_golden.py [reference checkout, default /root/reference]
"""
import ctypes
import importlib.util
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

VOICES = [
    # name, text, frames, n_codebooks, sample_rate, code seed
    ("alice", "héllo wörld, this is a reference clip.", 3, 16, 24000, 1),
    ("wide32", "thirty-two codebooks", 5, 32, 24000, 2),
    ("empty_text", "", 1, 16, 16000, 3),
]

# name, seed, temperature, top_k, top_p, repetition penalty, history, suppress range, draws
SAMPLER_CASES = [
    ("topk50_t09", 11, 0.9, 50, 1.0, 1.0, [], (2048, 2051), 4000),
    ("rep11_hist", 12, 0.9, 50, 1.0, 1.1, [5, 5, 17, 900, 2047], (2048, 2051), 4000),
    ("topp08", 13, 0.7, 0, 0.8, 1.0, [], (2048, 2051), 4000),
    ("greedy", 14, 0.9, 1, 1.0, 1.1, [3, 3], (2048, 2051), 64),
]


def voice_codes(frames, ncb, seed):
    return np.random.default_rng(seed).integers(-1, 2051, frames * ncb).astype(np.int32)


def sampler_logits(seed):
    x = (np.random.default_rng(seed).standard_normal(2052) * 2.0).astype(np.float32)
    x[2049] = 40.0          # a suppressed id with the largest logit
    return x


def main(ref):
    spec = importlib.util.spec_from_file_location("ref_bindings", os.path.join(ref, "python", "bz_ggml", "bindings.py"))
    rb = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(rb)
    for name, text, frames, ncb, sr, seed in VOICES:
        data = rb.serialize_breeze_voice(text, voice_codes(frames, ncb, seed).tolist(), frames, sr, ncb)
        with open(os.path.join(HERE, f"voice_{name}.breeze"), "wb") as f:
            f.write(data)

    subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "ref", f"REF={ref}"], check=True)
    lib = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref_host.so"))
    out = {}
    for name, seed, temp, k, p, rep, hist, sup, n in SAMPLER_CASES:
        logits = sampler_logits(seed)
        h = np.asarray(hist if hist else [0], np.int32)
        toks = np.zeros(n, np.int32)
        lib.ref_sample_tokens(logits.ctypes.data_as(ctypes.c_void_p), ctypes.c_int(logits.size), ctypes.c_float(temp),
                              ctypes.c_int(k), ctypes.c_float(p), ctypes.c_float(rep), h.ctypes.data_as(ctypes.c_void_p),
                              ctypes.c_int(len(hist)), ctypes.c_int(sup[0]), ctypes.c_int(sup[1]), ctypes.c_uint(seed),
                              ctypes.c_int(n), toks.ctypes.data_as(ctypes.c_void_p))
        out[name + "_logits"] = logits
        out[name + "_tokens"] = toks
    np.savez_compressed(os.path.join(HERE, "sampler_mt.npz"), **out)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
