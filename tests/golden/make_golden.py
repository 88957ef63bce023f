"""Generates the golden fixtures in this folder from the reference itself (run where the
reference checkout is present; the fixtures are committed so that the tests need neither).

  voice_*.breeze   BRZV bytes written by the reference's own Python serializer
                   (python/bz_ggml/bindings.py:606-611, serialize_breeze_voice)
  sampler_mt.npz   logits and the token sequences drawn from them by the reference's own C++
                   sampler (src/sampling.cpp:9-60, compiled unmodified into oracle/_ref by
                   `make -C oracle ref`), std::mt19937 seeded per case
  split_text.json  texts, budgets and the pieces the reference's long-text splitter returns
                   (src/text_split.cpp:89-111, compiled into oracle/_ref)
  wav_ref.wav      a WAV the reference's writer (src/audio.cpp:80-107) makes of wav_samples()
  cluster_sched.json  the serving harness's scheduling rules evaluated by the reference's own
                   python/bz_ggml/cluster.py: estimate_speech_profile, select_burst_steps and
                   a TieredSlotPool acquire/release trace

usage: python tests/golden/make_golden.py <reference checkout>
"""
import ctypes
import importlib.util
import json
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


# name, text, budget, first budget
SPLIT_CASES = [
    ("short", "Short enough to stay whole.", 600, 200),
    ("sentences", "One sentence here. Another one follows! Does a third? Yes; a fourth.", 20, 0),
    ("first_budget", "Alpha beta gamma. Delta epsilon zeta. Eta theta iota. Kappa lambda mu.", 30, 45),
    ("decimals", "Pi is 3.14 and Dr. Who said \"hi.\" (quietly.) Then left.\nNew line here.", 12, 0),
    ("clauses", "a long clause, with commas, and colons: and plenty of spaces between the words that go on", 25, 0),
    ("cjk", "你好。今天天气很好！你呢？我们一起去吧；好的…再见．", 6, 0),
    ("cjk_commas", "这是一个很长的句子，里面有很多逗号、顿号，还有更多的文字需要分开", 12, 0),
    ("mixed", "Hello 世界. Mixed text, 中文，and English; together! 结束。", 10, 4),
    ("no_budget", "Stays whole. Even with stops.", 0, 0),
    ("empty", "", 10, 0),
]
FUZZ_ALPHABET = list("abc de f. ! ? ; , : \n\"')]") + ["你", "好", "。", "！", "，", "、", "…", "．", "é"]


def fuzz_split_cases(n=200, seed=7):
    rng = np.random.default_rng(seed)
    cases = []
    for i in range(n):
        text = "".join(FUZZ_ALPHABET[j] for j in rng.integers(0, len(FUZZ_ALPHABET), int(rng.integers(0, 120))))
        cases.append((f"fuzz{i}", text, int(rng.choice([0, 5, 10, 17, 40, 600])), int(rng.choice([0, 3, 8, 200]))))
    return cases


def wav_samples():
    t = np.arange(600, dtype=np.float32)
    x = (np.sin(t * np.float32(0.05)) * np.float32(1.3)).astype(np.float32)
    x[:6] = [1.0, -1.0, 0.99999, -0.99999, 2.0, -2.0]
    return x


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

    split = []
    for name, text, budget, first in SPLIT_CASES + fuzz_split_cases():
        raw = text.encode("utf-8")
        need = -lib.ref_split_text(raw, budget, first, None, 0)
        buf = ctypes.create_string_buffer(max(need, 1))
        n = lib.ref_split_text(raw, budget, first, buf, len(buf))
        pieces = [p.decode("utf-8") for p in buf.raw.split(b"\0")[:n]]
        split.append(dict(name=name, text=text, budget=budget, first_budget=first, pieces=pieces))
    with open(os.path.join(HERE, "split_text.json"), "w", encoding="utf-8") as f:
        json.dump(split, f, ensure_ascii=False, indent=0)

    x = wav_samples()
    lib.ref_write_wav(os.path.join(HERE, "wav_ref.wav").encode(), x.ctypes.data_as(ctypes.c_void_p), x.size, 24000)

    with open(os.path.join(HERE, "cluster_sched.json"), "w") as f:
        json.dump(cluster_cases(ref), f, indent=0)


def cluster_cases(ref):
    """The reference harness's pure scheduling functions on seeded inputs."""
    pkg_dir = os.path.join(ref, "python", "bz_ggml")
    spec = importlib.util.spec_from_file_location("ref_bz_ggml", os.path.join(pkg_dir, "__init__.py"),
                                                  submodule_search_locations=[pkg_dir])
    pkg = importlib.util.module_from_spec(spec)
    sys.modules["ref_bz_ggml"] = pkg
    cspec = importlib.util.spec_from_file_location("ref_bz_ggml.cluster", os.path.join(pkg_dir, "cluster.py"))
    cl = importlib.util.module_from_spec(cspec)
    sys.modules["ref_bz_ggml.cluster"] = cl
    cspec.loader.exec_module(cl)
    rng = np.random.default_rng(21)
    words = ["alpha", "beta", "gamma", "delta", "epsilon", "zeta", "eta", "theta"]
    profiles = []
    for i in range(60):
        n = int(rng.integers(0, 120))
        text = " ".join(rng.choice(words, n)) if n else ""
        ins = [None, "", "Speak clearly and naturally.", "Whisper softly please"][i % 4]
        ref_frames = int(rng.integers(0, 200)) if i % 3 else 0
        cfg = [1.0, 1.5, 0.5, 2.0][i % 4]
        profiles.append(dict(text=text, instruction=ins, ref_frames=ref_frames, cfg_scale=cfg,
                             out=cl.estimate_speech_profile(text, ins, ref_frames, cfg_scale=cfg)))
    bursts = []
    for i in range(200):
        n = int(rng.integers(0, 12))
        sess = {j: {"expected_eos": int(rng.integers(0, 120)), "total_frames": int(rng.integers(0, 120))} for j in range(n)}
        mb = [16, 8, 4, 32][i % 4]
        bursts.append(dict(sessions=[[s["expected_eos"], s["total_frames"]] for s in sess.values()], max_burst=mb,
                           out=cl.select_burst_steps(sess, max_burst=mb)))
    pool = cl.TieredSlotPool(short_slots=3, standard_slots=2, long_slots=2)
    held, trace = [], []
    for i in range(120):
        if held and rng.random() < 0.4:
            slot = held.pop(int(rng.integers(0, len(held))))
            pool.release(slot)
            trace.append(["release", slot, pool.active_count()])
        else:
            need = int(rng.integers(50, 2600))
            got = pool.acquire(need)
            if got is not None:
                held.append(got[0])
            trace.append(["acquire", need, list(got) if got else None, pool.active_count()])
    return dict(profiles=profiles, bursts=bursts, pool=dict(tiers=[3, 2, 2], trace=trace))


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])
