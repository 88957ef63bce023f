#!/usr/bin/env python
"""Aggregate real-time factor of Breeze-TTS-2 serving on B200: audio seconds of PCM produced per
second, 64 live sessions per GPU.

The metric is the reference's (python/benchmark_40burst.py:103-113): the sum of the audio
seconds every session received, divided by the time taken. One bench step is one serving step
of continuous batching (configuration 3: ragged sessions, admission each step):
- sessions that produced their last frame in the previous step retire and the next arrivals
  take their places in the same step (their text-encoder and backbone prefill, first cb0 and
  vocoder stream start inside the timed region);
- every live session advances one frame: the depth decoder's nc-1 argmax sub-steps, the audio
  embedding, the 16-layer backbone over its paged KV cache and the cb0 sampler;
- the codec decoder turns every new frame into its 1920 PCM samples (80 ms at 24 kHz), each
  session on its own vocoder stream (the decoder's causal state carried across steps).

Workload: arrivals drawn from configuration 3's distributions (text prompts U[16,512] tokens,
voice contexts 0-125 frames, generation lengths U[50,400] frames, top-k 50 / T 0.9, greedy
depth per the batched ABI), on a seeded random-init Q8_0 model of the stated architecture
(nc = 32). The loop is closed at 64 live sessions per GPU -- a retiring session is replaced at
once -- and runs untimed from a cold start until the population is in steady state (ramp) before
the W warm-up and K timed steps. Sessions are independent: each GPU runs its own 64 (weak
scaling, no collective on the data path); rank times are combined as the max.

Prints one JSON line (rank 0):
- `value`: the serving steps resident on the device (bzb_generator_step_pcm_device: frames and PCM
  stay in HBM; admissions are host calls between steps), CUDA events on the engine's stream;
- `e2e`: the same loop through the C ABI with host buffers (bzb_generator_sessions_step_pcm:
  session ids and seeds up, frames, next cb0 and every session's PCM down, each step), over
  `--long-steps` steps (100) so that it meets the closed loop's steady admission rate;
  `steady_state`: the device-resident loop over as many steps, its like-for-like partner;
- `decode_only`: the frame step alone on the final batch (no vocoder, no admission);
- `ttfa`: time to first audio of the sessions admitted in the timed loop (prefill + first step
  with its PCM), and an open-loop run with Poisson arrivals at 4/s (configuration 3 as stated);
- `configs`: configuration 1 (one session through breeze_generate, greedy, 100 frames),
  configuration 2 (16 equal sessions, 200 frames, 63-frame voice prompts), configuration 4
  (Q4_K model, 40 sessions arriving at once) and configuration 5 (this GPU's share of elastic
  waves of streaming sessions, generation U[200,1500] frames; and 64 sessions at contexts near the
  2040-position clamp), each with PCM, and the reference ABI's own calls (sessions_step_burst,
  windowed session_decode_batch) on the same batch.
The per-step working set (~5 GB of weights and KV) exceeds the 126 MB L2: no flush is needed.

`--impl reference` times the reference's algorithm for the same path on the host cores: the
oracle (a CPU restatement, numpy on every core; the reference's ggml build cannot be compiled
here) running the reference's serving loop -- frame bursts, then its windowed vocoder sessions
(32 frames of history re-decoded with every call) -- on a bounded sample of the same sessions.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

if "reference" in sys.argv:
    # the CPU arm uses every host core (torchrun's ranks start with OMP_NUM_THREADS=1)
    for _k in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[_k] = str(os.cpu_count() or 1)

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FRAME_S = 1920 / 24000.0  # 80 ms of audio per frame
METRIC = "aggregate realtime factor @64 sessions/GPU"
CHUNK_FIRST = 4  # frames in the reference's first streamed chunk (src/generation.h GenRequest::chunk_first)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--sessions", type=int, default=64)
    ap.add_argument("--nc", type=int, default=32)
    ap.add_argument("--ramp", type=int, default=300, help="untimed serving steps from a cold start to steady state")
    ap.add_argument("--model-dir", default=os.environ.get("BZB_MODEL_DIR", "/tmp/bzb_models"))
    ap.add_argument("--cpu-sample-sessions", type=int, default=2)
    ap.add_argument("--poisson-s", type=float, default=6.0, help="seconds of the open-loop Poisson run (0: skip)")
    ap.add_argument("--configs", default="1,2,4,5,abi", help="other configurations to measure (comma list, or none)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--long-steps", type=int, default=100,
                    help="steps of the end-to-end (C ABI) loop and of the long device-resident loop beside it: "
                         "enough admissions for the closed loop's steady rate (about 0.28 per step)")
    ap.add_argument("--profile", action="store_true",
                    help="after the ramp, run one device-resident serving step between cudaProfilerStart/Stop and exit (ncu)")
    ap.add_argument("--profile-admit", action="store_true",
                    help="after the ramp, run one admission (a retired session replaced: batched create of one "
                         "arrival) between cudaProfilerStart/Stop and exit (ncu)")
    ap.add_argument("--profile-create", action="store_true",
                    help="after the ramp, run one batched creation of --sessions new arrivals between "
                         "cudaProfilerStart/Stop and exit (ncu)")
    ap.add_argument("--prompt-cap", type=int, default=512,
                    help="upper end of the text prompt lengths (tokens); smaller values make small profiling captures")
    ap.add_argument("--model-preset", default="full", choices=["full", "depth"],
                    help="'depth': the full-size depth decoder behind a one-layer backbone (small profiling captures)")
    return ap.parse_args()


def model_path(args, rank_local: int, barrier=None, quant: str = "q8_0", nc: int = 0) -> str:
    """The seeded random-init model (written once per box): greedy depth sampler (the batched ABI's
    depth is the argmax anyway; breeze_generate then decodes greedily, as configuration 1 asks)."""
    import __graft_entry__ as graft
    pkg = graft.load_package()
    nc = nc or args.nc
    os.makedirs(args.model_dir, exist_ok=True)
    path = os.path.join(args.model_dir, f"breeze_{args.model_preset}_nc{nc}_{quant}_seed0_eosoff.gguf")
    if rank_local == 0 and not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        pkg.synth_model(tmp, preset=args.model_preset, nc=nc, quant=quant, seed=0, eos_off=True, depth_top_k=1)
        os.replace(tmp, path)
    if barrier:
        barrier()
    return path


class Arrivals:
    """Seeded arrivals with configuration 3's shapes: text prompts U[lo,hi] tokens, voice contexts
    of U[v_lo,v_hi] frames (codes U[0,2048)) with an 8-token transcript, generation lengths
    U[g_lo,g_hi] frames (the session budget, max_new_tokens)."""

    def __init__(self, pkg, nc, seed, prompt=(16, 512), voice=(0, 125), gen=(50, 400), first_id=0):
        self.pkg, self.nc = pkg, nc
        self.rng = np.random.default_rng(seed)
        self.prompt, self.voice, self.gen = prompt, voice, gen
        self.next_id = first_id
        self.ready = []

    def prefill(self, n):
        """Draws the next n arrivals ahead of time: producing the synthetic request (the text and
        voice a client would send) is not the server's work, so timed loops take ready ones."""
        while len(self.ready) < n:
            self.ready.append(self._draw())

    def take(self):
        return self.ready.pop(0) if self.ready else self._draw()

    def _draw(self):
        rng = self.rng
        plen = int(rng.integers(self.prompt[0], self.prompt[1] + 1))
        vframes = int(rng.integers(self.voice[0], self.voice[1] + 1))
        glen = int(rng.integers(self.gen[0], self.gen[1] + 1))
        sid = self.next_id
        self.next_id += 1
        spec = dict(session_id=sid, text=self.pkg.ids_to_text(rng.integers(264, 128000, plen)), seed=sid,
                    max_new_tokens=glen)
        if vframes > 0:
            spec.update(ref_codes=rng.integers(0, 2048, (vframes, self.nc)).astype(np.int32),
                        ref_text=self.pkg.ids_to_text(rng.integers(264, 128000, 8)), ref_frames=vframes)
        return spec


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""
    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown," \
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, uuid: str):
        self.uuid = uuid
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", self.uuid], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in self.rows:
            for nm, v in zip(names, r[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows)}


class Server:
    """Closed-loop continuous batching on one GPU: `n_live` sessions; a session that has produced its
    budget of frames retires before the next step and the next arrival takes its place (one
    batched creation per step for all of that step's arrivals). Every step produces one frame and
    its PCM for every live session, each session on its own vocoder stream."""

    def __init__(self, gen, voc, arrivals, n_live):
        self.gen, self.voc, self.arr, self.n = gen, voc, arrivals, n_live
        self.live = []   # session ids in row order
        self.left = {}   # frames each session still produces
        self.ctx = {}    # cached backbone positions of each session (prompt + frames so far)
        self.frames = 0  # frames of audio produced
        self.admitted = 0
        self.admit_h2d = 0  # prompt bytes sent up by admissions (token text, voice codes)

    def admit(self):
        """Retires finished sessions and fills their places; returns the number admitted."""
        for sid in [s for s in self.live if self.left[s] == 0]:
            self.gen.session_free(sid)
            self.voc.stream_close(sid)
            self.live.remove(sid)
            del self.left[sid], self.ctx[sid]
        need = self.n - len(self.live)
        if need <= 0:
            return 0
        specs = [self.arr.take() for _ in range(need)]
        _, alloc = self.gen.sessions_create_batch(specs)
        for sp, a in zip(specs, alloc):
            sid = sp["session_id"]
            self.live.append(sid)
            self.left[sid] = sp["max_new_tokens"]
            self.ctx[sid] = a - sp["max_new_tokens"] - 8   # prompt + budget + 8, no 2040 clamp at these sizes
            # token ids of the prompt text (one per synthetic-vocabulary token) and the voice codes
            self.admit_h2d += 4 * sp["text"].count("<|t") + (sp["ref_codes"].nbytes if "ref_codes" in sp else 0)
        self.admitted += need
        return need

    def seeds(self):
        return [(sid * 7919 + self.left[sid]) & 0xFFFFFFFF for sid in self.live]

    def _advance(self):
        for sid in self.live:
            self.left[sid] -= 1
            self.ctx[sid] += 1
        self.frames += len(self.live)

    def step_device(self):
        """One serving step resident on the device (frames and PCM stay in HBM)."""
        self.gen.step_pcm_device(self.voc, self.live, self.seeds())
        self._advance()

    def step_abi(self):
        """One serving step through the C ABI with host buffers; returns (h2d, d2h) bytes."""
        n = len(self.live)
        _, fr, nx, pcm = self.gen.step_pcm(self.voc, self.live, self.seeds())
        if (fr[:, 0] < 0).any():
            raise RuntimeError("a live session produced no frame")
        self._advance()
        return n * 8, fr.nbytes + nx.nbytes + pcm.nbytes


def poisson_run(pkg, gen, voc, nc, seed, rate, duration, max_live):
    """Configuration 3 as stated: Poisson arrivals at `rate`/s admitted into the running batch as
    they come, through the C ABI (bzb_generator_sessions_step_pcm); time to first audio = the
    first PCM of a session (its first step's return) minus its arrival time (python/bz_ggml/
    cluster.py:636-637, 661), host wall clock."""
    arr = Arrivals(pkg, nc, seed, first_id=2_000_000)
    arr.prefill(int(2 * rate * duration) + 16)  # the clients' requests exist before they arrive
    rng = np.random.default_rng(seed + 1)
    live, left, arrived, first = [], {}, {}, {}
    ttfa, conc, frames = [], [], 0
    t0 = time.perf_counter()
    next_t = t0 + rng.exponential(1.0 / rate)
    while True:
        now = time.perf_counter()
        if now - t0 >= duration:
            break
        specs = []
        while next_t <= now and len(live) + len(specs) < max_live:
            sp = arr.take()
            arrived[sp["session_id"]] = next_t
            specs.append(sp)
            next_t += rng.exponential(1.0 / rate)
        if specs:
            gen.sessions_create_batch(specs)
            for sp in specs:
                live.append(sp["session_id"])
                left[sp["session_id"]] = sp["max_new_tokens"]
        if not live:
            time.sleep(max(0.0, min(next_t - time.perf_counter(), 0.01)))
            continue
        gen.step_pcm(voc, live, [(s * 31 + left[s]) & 0xFFFFFFFF for s in live], want_frames=False)
        t = time.perf_counter()
        for sid in live:
            if sid not in first:
                first[sid] = t
                ttfa.append((t - arrived[sid]) * 1e3)
            left[sid] -= 1
        frames += len(live)
        conc.append(len(live))
        for sid in [s for s in live if left[s] == 0]:
            gen.session_free(sid)
            voc.stream_close(sid)
            live.remove(sid)
    wall = time.perf_counter() - t0
    for sid in live:
        gen.session_free(sid)
        voc.stream_close(sid)
    return {"arrival_rate_per_s": rate, "seconds": wall, "arrivals": len(arrived), "first_audio": len(ttfa),
            "p50_ms": statistics.median(ttfa) if ttfa else None,
            "p90_ms": float(np.percentile(ttfa, 90)) if ttfa else None,
            "mean_concurrency": float(np.mean(conc)) if conc else 0.0,
            "aggregate_rtf": frames * FRAME_S / wall,
            "method": "open loop: Poisson arrivals admitted into the running batch as they come (one batched "
                      "create per step), one frame plus its PCM per live session per step through "
                      "bzb_generator_sessions_step_pcm; TTFA = first PCM returned minus arrival, host wall clock"}


def config1(pkg, path):
    """Configuration 1: one session through breeze_generate (the reference's single-request route,
    src/generation.cpp:83-273): a 64-token prompt, greedy (top_k 1, repetition penalty 1; the
    model's depth sampler is top-1), exactly 100 frames (EOS unreachable), PCM streamed through
    the callback in the reference's chunk schedule. Host wall clock."""
    ctx = pkg.ContextHandle(path)
    try:
        text = pkg.ids_to_text(np.random.default_rng(1).integers(264, 128000, 64))
        req = pkg.ContextHandle.request(text, seed=0, max_new_tokens=100, top_k=1, repetition_penalty=1.0,
                                        split_chars=100000)
        ctx.generate(req)  # warm-up: buffers, graphs
        t0 = time.perf_counter()
        pcm, chunks, codes, n, tm = ctx.generate(req)
        wall = time.perf_counter() - t0
    finally:
        ctx.close()
    return {"frames": int(n), "audio_s": pcm.size / 24000.0, "wall_s": wall, "rtf": pcm.size / 24000.0 / wall,
            "ttfa_ms": tm["first_audio_ms"], "chunks": len(chunks),
            "route": "breeze_generate (bzb_generate_codes), one request, chunked windowed vocoder"}


def config2(pkg, gen, voc, nc):
    """Configuration 2: 16 sessions arriving together, equal lengths: 128-token prompts, a 63-frame
    voice context each, 200 frames, top-k 50 / T 0.9, per-session seed = session index. One batched
    create, then 200 serving steps (frame + PCM) through the C ABI. Host wall clock."""
    rng = np.random.default_rng(2)
    specs = []
    for i in range(16):
        specs.append(dict(session_id=3_000_000 + i, text=pkg.ids_to_text(rng.integers(264, 128000, 128)), seed=i,
                          max_new_tokens=200, ref_codes=rng.integers(0, 2048, (63, nc)).astype(np.int32),
                          ref_text=pkg.ids_to_text(rng.integers(264, 128000, 8)), ref_frames=63))
    ids = [sp["session_id"] for sp in specs]
    gen.sync()
    t0 = time.perf_counter()
    gen.sessions_create_batch(specs)
    t1 = time.perf_counter()
    frames = 0
    first = None
    for k in range(200):
        _, fr, _, _ = gen.step_pcm(voc, ids, [i + k for i in range(16)])
        frames += int((fr[:, 0] >= 0).sum())
        if first is None:
            first = time.perf_counter()
    t2 = time.perf_counter()
    for sid in ids:
        gen.session_free(sid)
        voc.stream_close(sid)
    return {"sessions": 16, "frames": frames, "audio_s": frames * FRAME_S, "create_ms": (t1 - t0) * 1e3,
            "steps_s": t2 - t1, "rtf_steps": frames * FRAME_S / (t2 - t1), "rtf_total": frames * FRAME_S / (t2 - t0),
            "ttfa_ms": (first - t0) * 1e3,
            "route": "bzb_generator_sessions_create_batch + 200 x bzb_generator_sessions_step_pcm"}


def config5(pkg, gen, voc, nc, seed, elastic_s=10.0, n_gpus_share=8, long_steps=30):
    """Configuration 5, streaming PCM with elastic load, on this GPU's share of it. Two parts:
    - elastic: waves of 20 sessions every 2 s spread over 8 GPUs (this GPU takes waves of 2 and 3
      alternately), generation lengths U[200,1500] frames, prompts and voices as configuration 3;
      arrivals join the running batch at the next step (one batched create), every live session
      makes one frame and its 1920 PCM samples per step through the C ABI; aggregate RTF, time to
      first audio (first PCM returned minus arrival) and concurrency, host wall clock;
    - long_context: 64 sessions whose contexts start at 1300-1850 positions (text prompts
      U[1300,1700] tokens plus 0-125 voice frames) and grow towards the 2040-position clamp:
      `long_steps` device-resident serving steps with PCM timed by CUDA events, then as many
      through the C ABI (the paged decode attention over its longest spans)."""
    import torch
    out = {}
    # elastic waves
    arr = Arrivals(pkg, nc, seed, gen=(200, 1500), first_id=8_000_000)
    arr.prefill(int(elastic_s / 2 + 2) * (20 // n_gpus_share + 1))
    live, left, arrived, first = [], {}, {}, {}
    ttfa, conc, frames, steps = [], [], 0, 0
    wave, next_wave = 0, 0.0
    t0 = time.perf_counter()
    while True:
        now = time.perf_counter() - t0
        if now >= elastic_s:
            break
        specs = []
        while next_wave <= now:
            k = 20 // n_gpus_share + (1 if wave % 2 and 20 % n_gpus_share else 0)
            for _ in range(k):
                sp = arr.take()
                arrived[sp["session_id"]] = t0 + next_wave
                specs.append(sp)
            wave += 1
            next_wave += 2.0
        if specs:
            gen.sessions_create_batch(specs)
            for sp in specs:
                live.append(sp["session_id"])
                left[sp["session_id"]] = sp["max_new_tokens"]
        if not live:
            time.sleep(0.005)
            continue
        gen.step_pcm(voc, live, [(s * 13 + left[s]) & 0xFFFFFFFF for s in live], want_frames=False)
        t = time.perf_counter()
        for sid in live:
            if sid not in first:
                first[sid] = t
                ttfa.append((t - arrived[sid]) * 1e3)
            left[sid] -= 1
        frames += len(live)
        steps += 1
        conc.append(len(live))
        for sid in [x for x in live if left[x] == 0]:
            gen.session_free(sid)
            voc.stream_close(sid)
            live.remove(sid)
    wall = time.perf_counter() - t0
    for sid in live:
        gen.session_free(sid)
        voc.stream_close(sid)
    out["elastic"] = {
        "seconds": wall, "waves": wave, "arrivals": len(arrived), "steps": steps,
        "ms_per_step": wall / max(steps, 1) * 1e3, "aggregate_rtf": frames * FRAME_S / wall,
        "ttfa_p50_ms": statistics.median(ttfa) if ttfa else None,
        "ttfa_p90_ms": float(np.percentile(ttfa, 90)) if ttfa else None,
        "mean_concurrency": float(np.mean(conc)) if conc else 0.0, "peak_concurrency": max(conc) if conc else 0,
        "method": f"this GPU's share of 20 arrivals per 2 s over {n_gpus_share} GPUs, generation U[200,1500] frames; "
                  "bzb_generator_sessions_create_batch per step with arrivals, bzb_generator_sessions_step_pcm "
                  "per step; host wall clock"}
    # long contexts
    arr = Arrivals(pkg, nc, seed + 1, prompt=(1300, 1700), gen=(100, 100), first_id=9_000_000)
    specs = [arr.take() for _ in range(64)]
    gen.sessions_create_batch(specs)
    ids = [sp["session_id"] for sp in specs]
    stream = torch.cuda.ExternalStream(gen.stream_ptr())
    for k in range(3):
        gen.step_pcm_device(voc, ids, [i + k for i in range(64)])
    gen.sync()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for k in range(long_steps):
        gen.step_pcm_device(voc, ids, [i + 3 + k for i in range(64)])
    e1.record(stream)
    e1.synchronize()
    ms_dev = e0.elapsed_time(e1)
    t1 = time.perf_counter()
    for k in range(long_steps):
        gen.step_pcm(voc, ids, [i + 3 + long_steps + k for i in range(64)], want_frames=False)
    ms_abi = (time.perf_counter() - t1) * 1e3
    for sid in ids:
        gen.session_free(sid)
        voc.stream_close(sid)
    prompt = [sp["text"].count("<|t") + sp.get("ref_frames", 0) for sp in specs]
    out["long_context"] = {
        "sessions": 64, "prompt_positions_mean": float(np.mean(prompt)), "prompt_positions_max": int(max(prompt)),
        "context_at_end_max": int(max(prompt)) + 3 + 2 * long_steps,
        "ms_per_step": ms_dev / long_steps, "rtf": 64 * long_steps * FRAME_S / (ms_dev / 1e3),
        "e2e_ms_per_step": ms_abi / long_steps, "e2e_rtf": 64 * long_steps * FRAME_S / (ms_abi / 1e3),
        "method": "64 sessions prefilled to long contexts (text and voice prompt positions as shown, plus the "
                  "instruction), then serving steps with PCM: bzb_generator_step_pcm_device timed by CUDA events, "
                  "then bzb_generator_sessions_step_pcm with host buffers (host wall clock)"}
    return out


def config4(pkg, args, local, barrier=None, n_sessions=40):
    """Configuration 4: a Q4_K model (backbone and depth linears Q4_K); 40 sessions per GPU arrive
    at t = 0 (prompts U[32,256] tokens, 5 s voice contexts of 63 frames, generation U[100,300]
    frames); one batched create, then serving steps (frame + PCM, C ABI) until every session has
    finished. Aggregate RTF = all audio / wall; TTFA = the first step's return (host wall clock)."""
    path = model_path(args, local, barrier, quant="q4_k")  # written once per node, by local rank 0
    gen = pkg.GeneratorHandle(path, local)
    voc = pkg.VocoderHandle(generator=gen)
    try:
        arr = Arrivals(pkg, gen.nc, 40 + local, prompt=(32, 256), voice=(63, 63), gen=(100, 300), first_id=4_000_000)
        warm = [arr.take() for _ in range(4)]
        gen.sessions_create_batch(warm)
        for k in range(3):
            gen.step_pcm(voc, [w["session_id"] for w in warm], [k] * 4)
        for w in warm:
            gen.session_free(w["session_id"])
            voc.stream_close(w["session_id"])
        specs = [arr.take() for _ in range(n_sessions)]
        left = {sp["session_id"]: sp["max_new_tokens"] for sp in specs}
        live = list(left)
        gen.sync()
        t0 = time.perf_counter()
        gen.sessions_create_batch(specs)
        t1 = time.perf_counter()
        frames, first, steps = 0, None, 0
        while live:
            _, fr, _, _ = gen.step_pcm(voc, live, [(s + left[s]) & 0xFFFFFFFF for s in live])
            frames += int((fr[:, 0] >= 0).sum())
            steps += 1
            if first is None:
                first = time.perf_counter()
            for s in live:
                left[s] -= 1
            live = [s for s in live if left[s] > 0]
        t2 = time.perf_counter()
    finally:
        voc.close()
        gen.close()
    return {"quant": "Q4_K", "sessions_per_gpu": n_sessions, "frames": frames, "audio_s": frames * FRAME_S,
            "create_ms": (t1 - t0) * 1e3, "steps": steps, "wall_s": t2 - t0, "rtf": frames * FRAME_S / (t2 - t0),
            "burst_ttfa_ms": (first - t0) * 1e3,
            "route": "one bzb_generator_sessions_create_batch for the burst, then bzb_generator_sessions_step_pcm "
                     "until every session has finished"}


def abi_path(pkg, gen, srv, nc, burst=8):
    """The reference ABI's own serving calls (python/bz_ggml/cluster.py:851-867, 625-648) on the
    live batch: frame bursts through breeze_generator_sessions_step_burst (16 codes per frame),
    and the reference vocoder semantics -- breeze_vocoder_session_decode_batch re-decoding each
    session's kept 32 frames of history with its new frames -- on full-width frames
    (bzb_generator_sessions_step_frames). Host wall clock per burst."""
    ids = [s for s in srv.live if srv.left[s] > 6 * burst]
    if not ids:
        return None
    seeds = [s & 0xFFFFFFFF for s in ids]
    gen.sync()
    t0 = time.perf_counter()
    gen.sessions_step_burst(ids, burst, seeds)
    t_burst = time.perf_counter() - t0
    voc = pkg.VocoderHandle(generator=gen)
    try:
        vids = [5_000_000 + s for s in ids]
        times = []
        for rep in range(5):   # the kept history fills up to 32 frames
            _, frames, _ = gen.step_frames(ids, burst, seeds)
            t0 = time.perf_counter()
            voc.session_decode_batch(vids, [frames[:, i, :] for i in range(len(ids))])
            times.append(time.perf_counter() - t0)
        for v in vids:
            voc.session_free(v)
    finally:
        voc.close()
    for s in ids:
        srv.left[s] -= 6 * burst
        srv.ctx[s] += 6 * burst
    audio = len(ids) * burst * FRAME_S
    return {"sessions": len(ids), "burst_frames": burst, "step_burst_ms": t_burst * 1e3,
            "step_burst_rtf": audio / t_burst, "windowed_vocoder_ms": times[-1] * 1e3,
            "serving_rtf": audio / (t_burst + times[-1]),
            "route": "breeze_generator_sessions_step_burst (16 codes/frame) timed; then full-width bursts and "
                     "breeze_vocoder_session_decode_batch with 32 frames of kept history, the last of 5 timed"}


def cluster_config(pkg, args, per_gpu=40):
    """The N-island harness (bz-ggml_b200/cluster.py) over every GPU this process sees, one island
    per GPU on one shared job queue: configuration 4's burst (Q4_K model, `per_gpu` requests per
    GPU at t = 0, prompts U[32,256] tokens, 63-frame voice contexts, U[100,300] frames, PCM made on
    the server). Aggregate RTF = all audio / wall; per-island request counts show the balance."""
    import importlib
    import torch
    cl = importlib.import_module(pkg.__name__ + ".cluster")
    n_gpu = torch.cuda.device_count()
    path = model_path(args, 0, quant="q4_k")
    arr = Arrivals(pkg, args.nc, 44, prompt=(32, 256), voice=(63, 63), gen=(100, 300), first_id=6_000_000)
    tasks = []
    for i in range(per_gpu * n_gpu):
        sp = arr.take()
        tasks.append(cl.UserTask(id=sp["session_id"], text=sp["text"], seed=sp["seed"], max_steps=sp["max_new_tokens"],
                                 ref_text=sp.get("ref_text"), ref_codes=sp["ref_codes"].reshape(-1).tolist(),
                                 ref_frames=sp["ref_frames"]))
    with cl.IslandCluster(path, devices=tuple(range(n_gpu)), max_slots=per_gpu, chunk_size=8, max_burst=16) as cluster:
        warm = [cl.UserTask(id=7_000_000 + i, text=tasks[i].text, max_steps=4) for i in range(n_gpu)]
        cluster.run_workload(warm)
        t0 = time.perf_counter()
        results = cluster.run_workload(tasks)
        wall = time.perf_counter() - t0
    per_island, audio = {}, 0.0
    for r in results:
        gpu = int(r.worker.split("GPU ")[1].split(" ")[0])
        d = per_island.setdefault(gpu, {"requests": 0, "audio_s": 0.0})
        d["requests"] += 1
        d["audio_s"] += r.audio_s
        audio += r.audio_s
    ttfa = [r.ttfa_s * 1e3 for r in results]
    return {"islands": n_gpu, "requests": len(results), "audio_s": audio, "wall_s": wall,
            "aggregate_rtf": audio / wall, "ttfa_p50_ms": statistics.median(ttfa),
            "ttfa_p90_ms": float(np.percentile(ttfa, 90)), "per_island": per_island,
            "route": "IslandCluster.run_workload: one process, one island (generator + vocoder) per GPU, shared "
                     "job queue, tiered slot pool, batched creation, burst steps, server-side PCM"}


def cpu_reference_rtf(path, n_sessions, bursts, warm_bursts, burst=8, seed=7):
    """The reference's serving loop on the host cores, with the oracle for the path: n sessions of
    the workload (prefill untimed), then bursts of `burst` batched frame steps, each followed by the
    reference's windowed vocoder decode (src/c_api.cpp:1066-1162: each session's last 32 frames
    re-decoded with its new ones). Returns (aggregate RTF, seconds, BLAS threads)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import breeze_oracle as bo
    import __graft_entry__ as graft
    from threadpoolctl import threadpool_info, threadpool_limits
    pkg = graft.load_package()
    cores = os.cpu_count() or 1
    with threadpool_limits(limits=cores):
        threads = max([p.get("num_threads", 1) for p in threadpool_info()] or [1])
        m = bo.Model(path)
        g = bo.Generator(m)
        v = bo.Vocoder(m)
        arr = Arrivals(pkg, m.cfg.nc, seed)
        ids = []
        rng = np.random.default_rng(seed)
        for _ in range(n_sessions):
            sp = arr.take()
            kw = {k: sp[k] for k in ("ref_text", "ref_codes") if k in sp}
            g.session_create(sp["session_id"], sp["text"], seed=sp["seed"], max_new_tokens=400, **kw)
            ids.append(sp["session_id"])
            # a session in steady state: the vocoder keeps its full 32 frames of history
            v.history[sp["session_id"]] = rng.integers(0, 2048, 32 * m.cfg.nc).astype(np.int64)
        dt = 0.0
        for b in range(warm_bursts + bursts):
            t0 = time.perf_counter()
            frames = []
            for k in range(burst):
                fr, _ = g.step_batched(ids, seeds=[s + 8 * b + k for s in ids])
                frames.append(fr)
            for i, sid in enumerate(ids):
                v.session_decode(sid, np.stack([f[i] for f in frames]), burst)
            if b >= warm_bursts:
                dt += time.perf_counter() - t0
    return n_sessions * bursts * burst * FRAME_S / dt, dt, threads


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    path = model_path(args, 0)
    bursts, warm = 2, 1
    value, dt, cores = cpu_reference_rtf(path, args.cpu_sample_sessions, bursts, warm)
    sample = (f"{args.cpu_sample_sessions} sessions of the 64-session workload (same prompt, voice and generation "
              f"distributions; prefill untimed), {bursts} timed bursts of 8 frame steps after {warm} untimed, each "
              f"followed by the reference's windowed vocoder decode (32 frames of history re-decoded per call); oracle "
              f"numpy on {cores} BLAS threads. Per-session work is independent, so the aggregate RTF of the sample "
              f"stands for the 64-session batch (normalised per session)")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "x realtime", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / (bursts * 8) * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "64 ragged sessions/GPU serving with PCM (configuration 3 shapes), bounded CPU "
                                   "sample normalised per session", "nc": args.nc, "quant": "Q8_0",
                       "sessions": args.cpu_sample_sessions, "same_config": True},
            "cpu_baseline": {"value": value, "unit": "x realtime", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "x realtime", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist
    import __graft_entry__ as graft

    pkg = graft.load_package()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900), device_id=torch.device("cuda", local))
    barrier = (lambda: dist.barrier()) if world > 1 else None
    path = model_path(args, local, barrier)

    t_load = time.perf_counter()
    gen = pkg.GeneratorHandle(path, local)
    voc = pkg.VocoderHandle(generator=gen)
    t_load = time.perf_counter() - t_load
    nc = gen.nc
    cap = max(1, args.prompt_cap)
    srv = Server(gen, voc, Arrivals(pkg, nc, 1000 + rank, prompt=(min(16, cap), cap)), args.sessions)
    # ramp: from a cold start to the steady state of the closed loop (ages and contexts mixed)
    t_ramp = time.perf_counter()
    for _ in range(args.ramp):
        srv.admit()
        srv.step_device()
    gen.sync()
    t_ramp = time.perf_counter() - t_ramp
    if args.profile_admit:
        srv.left[srv.live[0]] = 0
        gen.sync()
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        n = srv.admit()
        gen.sync()
        torch.cuda.profiler.stop()
        print(json.dumps({"profiled_admissions": n}))
        voc.close()
        gen.close()
        return
    if args.profile_create:
        specs = [srv.arr.take() for _ in range(args.sessions)]
        gen.sync()
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        gen.sessions_create_batch(specs)
        gen.sync()
        torch.cuda.profiler.stop()
        print(json.dumps({"profiled_creations": len(specs)}))
        voc.close()
        gen.close()
        return
    if args.profile:
        srv.admit()
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        srv.step_device()
        gen.sync()
        torch.cuda.profiler.stop()
        print(json.dumps({"profiled_steps": 1, "launches_per_step": gen.launches_per_step(), "sessions": args.sessions}))
        voc.close()
        gen.close()
        return
    for _ in range(args.warmup):
        srv.admit()
        srv.step_device()
    gen.sync()

    stream = torch.cuda.ExternalStream(gen.stream_ptr())
    uuid = "GPU-" + str(torch.cuda.get_device_properties(local).uuid)

    def ev():
        e = torch.cuda.Event(enable_timing=True)
        e.record(stream)
        return e

    def max_over_ranks(ms):
        if world > 1:
            t = torch.tensor([ms], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    def begin():
        if barrier:
            barrier()
        torch.cuda.synchronize()
        gen.sync()

    # timed: device-resident serving steps, admissions included (the arrivals' synthetic requests
    # drawn beforehand)
    srv.arr.prefill(4 * args.steps + args.sessions)
    admits_before, frames_before = srv.admitted, srv.frames
    ttfa_ev = []
    begin()
    # clocks sampled through the K timed steps and the long windows after them
    clk = ClockSampler(uuid)
    clk.__enter__()
    e0 = ev()
    for _ in range(args.steps):
        ea = ev()
        k = srv.admit()
        srv.step_device()
        if k:
            ttfa_ev.append((ea, ev(), k))
    e1 = ev()
    e1.synchronize()
    ms_dev = max_over_ranks(e0.elapsed_time(e1))
    frames_dev = srv.frames - frames_before
    admits_timed = srv.admitted - admits_before
    ttfa_closed = []
    for ea, eb, k in ttfa_ev:
        ttfa_closed += [ea.elapsed_time(eb)] * k
    mean_ctx = float(np.mean(list(srv.ctx.values())))

    # long windows at the closed loop's steady admission rate: the device-resident loop, then the
    # same loop through the C ABI with host buffers (e2e)
    n_long = max(args.steps, args.long_steps)
    srv.arr.prefill(n_long + args.sessions)
    admits_before, frames_before = srv.admitted, srv.frames
    begin()
    e0 = ev()
    for _ in range(n_long):
        srv.admit()
        srv.step_device()
    e1 = ev()
    e1.synchronize()
    ms_long = max_over_ranks(e0.elapsed_time(e1))
    frames_long, admits_long = srv.frames - frames_before, srv.admitted - admits_before
    srv.arr.prefill(n_long + args.sessions)
    frames_before, admit_h2d_before, admits_before = srv.frames, srv.admit_h2d, srv.admitted
    h2d = d2h = 0
    begin()
    e0 = ev()
    for _ in range(n_long):
        srv.admit()
        hb, db = srv.step_abi()
        h2d += hb
        d2h += db
    e1 = ev()
    e1.synchronize()
    ms_e2e = max_over_ranks(e0.elapsed_time(e1))
    clk.__exit__(None, None, None)
    frames_e2e, admits_e2e = srv.frames - frames_before, srv.admitted - admits_before
    h2d += srv.admit_h2d - admit_h2d_before

    # the frame step alone on the last batch, and one profiled eager step (roofline)
    begin()
    e0 = ev()
    gen.step_device(args.steps)
    e1 = ev()
    e1.synchronize()
    ms_decode = max_over_ranks(e0.elapsed_time(e1))
    prof = gen.profile_step()
    for sid in srv.live:  # the sessions moved on by those steps
        srv.left[sid] = max(0, srv.left[sid] - args.steps - 1)
        srv.ctx[sid] += args.steps + 1
    launches = gen.launches_per_step()
    voc_kernels = voc.kernels_per_decode(args.sessions, 1)
    ctx_mid = np.asarray(list(srv.ctx.values()), np.float64)
    b_step = gen.weight_bytes_per_step() + float(gen.kv_bytes_per_position() * ctx_mid.sum())

    poisson = None
    if args.poisson_s > 0:
        poisson = poisson_run(pkg, gen, voc, nc, 6000 + rank, 4.0, args.poisson_s, 256)
    configs = {}
    want = set(c.strip() for c in args.configs.split(",")) if args.configs != "none" else set()
    if "abi" in want:
        configs["abi_path"] = abi_path(pkg, gen, srv, nc)
    if "2" in want:
        configs["c2_16_equal_sessions"] = config2(pkg, gen, voc, nc)
    # the main generator's sessions are done with: free them before other workloads
    for sid in list(srv.live):
        gen.session_free(sid)
        voc.stream_close(sid)
    if "5" in want:
        configs["c5_streaming_elastic"] = config5(pkg, gen, voc, nc, 5000 + rank)
    voc.close()
    gen.close()
    if "1" in want:
        configs["c1_single_session_generate"] = config1(pkg, path)
    if "cluster" in want and world == 1:
        configs["cluster_islands"] = cluster_config(pkg, args)
    if "4" in want:
        if barrier:
            barrier()
        configs["c4_q4k_burst"] = config4(pkg, args, local, barrier)
        if world > 1:
            t = torch.tensor([configs["c4_q4k_burst"]["wall_s"]], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            c4 = configs["c4_q4k_burst"]
            c4["wall_s_max_over_ranks"] = float(t.item())
            c4["aggregate_rtf_all_gpus"] = world * c4["audio_s"] / c4["wall_s_max_over_ranks"]

    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    traffic = None
    if prof["depth_ms"] > 0:
        dom_gbs = prof["depth_bytes"] / (prof["depth_ms"] / 1e3) / 1e9
        if nc == 32 and args.sessions == 64:
            # dram__bytes_read.sum + dram__bytes_write.sum of one launch, from an ncu capture of the
            # same depth decode (64 sessions, nc 32) on the depth-sized model: 3.868 GB + 34.3 MB
            traffic = 3.868159e9 + 34.275840e6
        dom_name = "depth_persist_kernel (persistent tcgen05 depth decoder, 31 sub-steps)"
        dom_share = prof["depth_ms"] / prof["step_ms"]
    else:
        dom_gbs = prof["gemm_bytes"] / (prof["gemm_ms"] / 1e3) / 1e9
        dom_name = "umma_gemm_kernel (Q8_0 dequant-GEMM, all launches of one step)"
        dom_share = prof["gemm_ms"] / prof["step_ms"]
    cpu = None
    if barrier:
        barrier()  # every rank's GPU work is done: the CPU port gets the host's cores to itself
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            v, dt, cores = cpu_reference_rtf(path, 1, 1, 1)
            cpu = {"value": v, "unit": "x realtime", "cores": cores, "kind": "port",
                   "sample": "1 session of the workload, 1 timed burst of 8 frame steps after 1 untimed, each burst "
                             "followed by the reference's windowed vocoder decode (32 frames of history); oracle numpy "
                             "on all host cores; normalised per session"}
        except Exception as e:  # the baseline is reported, not the target
            cpu = {"value": None, "unit": "x realtime", "cores": os.cpu_count(), "kind": "port", "sample": f"failed: {e}"}
    if rank == 0:
        step_ms = ms_dev / args.steps
        value = world * frames_dev * FRAME_S / (ms_dev / 1e3)
        e2e = world * frames_e2e * FRAME_S / (ms_e2e / 1e3)
        line = {
            "metric": METRIC, "value": value, "unit": "x realtime", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded random-init Q8_0 GGUF, seeded arrivals)",
            "config": {"workload": "64 live sessions/GPU, closed-loop continuous batching with PCM: each step every "
                                   "live session makes one frame and its 1920 PCM samples (streaming vocoder); sessions "
                                   "retire at their length and the next arrival is prefilled in the same step "
                                   "(prompts U[16,512] tok, voice 0-125 frames, gen U[50,400] frames, page 16, top-k 50 "
                                   "T 0.9, greedy depth per the batched ABI)",
                       "sessions_per_gpu": args.sessions, "nc": nc, "quant": "Q8_0", "parallelism": f"replicas x{world}",
                       "l2": "per-step working set > 126 MB L2 (no flush needed)", "ramp_steps": args.ramp,
                       "ramp_s": t_ramp, "admissions_in_timed_steps": admits_timed, "mean_context": mean_ctx,
                       "model_load_s": t_load},
            "e2e": {"value": e2e, "unit": "x realtime", "h2d_bytes_per_step": h2d / n_long,
                    "d2h_bytes_per_step": d2h / n_long, "steps": n_long, "admissions": admits_e2e,
                    "route": "per step: admissions (bzb_generator_sessions_create_batch, prompt text and voice codes "
                             "up) and bzb_generator_sessions_step_pcm (ids and seeds up; frames, next cb0 and PCM down)"},
            "steady_state": {"value": world * frames_long * FRAME_S / (ms_long / 1e3), "unit": "x realtime",
                             "steps": n_long, "admissions": admits_long, "ms_per_step": ms_long / n_long,
                             "method": "the device-resident loop over as many steps as e2e (the K-step value sees "
                                       "fewer admissions than the steady rate of about 0.28 per step)"},
            "decode_only": {"value": world * args.sessions * args.steps * FRAME_S / (ms_decode / 1e3),
                            "ms_per_step": ms_decode / args.steps,
                            "method": "the frame step's graph alone on the last batch (no vocoder, no admission)"},
            "roofline": {"bound": "hbm", "achieved": dom_gbs, "peak": hbm, "unit": "GB/s", "frac": dom_gbs / hbm,
                         "traffic": traffic, "kernel": dom_name, "peak_source": peak_src,
                         "kernel_share_of_decode_step": dom_share},
            "step_roofline": {"bytes_per_step": b_step, "achieved": b_step / (ms_decode / args.steps / 1e3) / 1e9,
                              "peak": hbm, "unit": "GB/s",
                              "frac": b_step / (ms_decode / args.steps / 1e3) / 1e9 / hbm,
                              "note": "decode step: weights (depth re-read per sub-step) + live KV, over decode_only"},
            "cpu_baseline": cpu,
            "ttfa": {"closed_loop": {"p50_ms": statistics.median(ttfa_closed) if ttfa_closed else None,
                                     "p90_ms": float(np.percentile(ttfa_closed, 90)) if ttfa_closed else None,
                                     "n": len(ttfa_closed),
                                     "method": "sessions admitted in the timed steps: prefill + their first serving "
                                               "step with its PCM, CUDA events on the engine's stream"},
                     "poisson": poisson},
            "configs": configs,
            "gpu_launches": args.steps * (launches + voc_kernels),
            "gpu_launches_note": f"{launches} frame-step graph nodes + {voc_kernels} vocoder kernels per step; the "
                                 "admissions' prefill kernels come on top",
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
