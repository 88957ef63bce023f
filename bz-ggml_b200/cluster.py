"""N-island serving harness over the generator and vocoder handles: one island (generator, and
vocoder when a request wants server-side audio) per GPU, all pulling from one job queue.

It restates the scheduling of the reference's python/bz_ggml/cluster.py for any number of GPUs
(the reference's DualInstanceCluster drives exactly two): the speech-length estimate
(cluster.py:143-176), the tiered slot pool that caps each island's admissions (cluster.py:179-229),
the burst-size choice (cluster.py:232-261), per-step reseeding with the task seed plus the
frames already made (cluster.py:857-860), and the two delivery modes of a request (cluster.py:819,
887-895, 943-967):

- client_has_vocoder: the frames go back as codes. `pack_frames` gives them a wire form of
  little-endian uint16 codes, 16 per frame by default (the ABI frame width), 32 bytes per 80 ms
  frame (3.2 kbit/s); `on_tokens(task_id, packet, final)` receives one packet per burst.
- otherwise the island's vocoder decodes them: in chunks of `chunk_size` frames as they arrive
  when the task asks for streaming (`stream_pcm`), else in one pass at the end; `on_pcm_chunk`
  receives the PCM.

Unlike the reference worker, an island admits every waiting arrival that fits in one batched
creation call (bzb_generator_sessions_create_batch), and it steps full-width frames
(bzb_generator_sessions_step_frames).
"""
import math
import os
import queue
import threading
import time
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import GeneratorHandle, VocoderHandle, write_wav

FRAME_S = 0.08
SAMPLE_RATE = 24000
WIRE_CODES = 16  # codes per frame on the token wire (the generator ABI's frame width)
# cb0 values that end a stream in a burst's frames: -1 (retired), the backbone EOS and the
# out-of-vocabulary marker the reference also checks (cluster.py:876-879)
_STOP_CB0 = (2051, 4096)


@dataclass
class UserTask:
    """One synthesis request (cluster.py:13-27)."""
    id: int
    text: str
    instruction: str = "Speak clearly and naturally."
    cfg_scale: float = 1.0
    temperature: float = 0.25
    seed: int = 42
    max_steps: int = 2040
    ref_text: Optional[str] = None
    ref_codes: Optional[Sequence[int]] = None
    ref_frames: int = 0
    client_has_vocoder: bool = False  # True: codes on the wire; False: server-side PCM
    stream_pcm: bool = False          # server-side PCM in chunks as frames arrive, else one pass at the end


@dataclass
class ClusterResult:
    """Per-request outcome (cluster.py:47-63); `tokens` holds a token-mode request's codes,
    frame-major, WIRE_CODES per frame. `frames` and `pcm` are filled when the cluster keeps them."""
    id: int
    words: int
    audio_s: float
    queue_wait_s: float
    compute_wall_s: float
    turnaround_s: float
    ttfa_s: float
    rtf: float
    worker: str
    wav_path: str
    tokens: Optional[List[int]] = None
    frames: Optional[np.ndarray] = field(default=None, repr=False)  # [n][num_codebooks], when kept
    pcm: Optional[np.ndarray] = field(default=None, repr=False)     # server-side audio, when kept

    @property
    def audio_path(self) -> str:
        return self.wav_path


def estimate_speech_profile(text: str, instruction: Optional[str] = None, ref_frames: int = 0,
                            cfg_scale: float = 1.0) -> Dict[str, int]:
    """Token and frame bounds of a request (cluster.py:143-176): 1.3 prompt tokens per word plus
    reference frames plus 20; output between 3.75 (fast speech) and 6.8 frames per word + 25
    (slow speech with pauses), 5.35 + 12 expected; a guided request needs both branches."""
    words = max(1, len(text.split()))
    ins_words = len(instruction.split()) if instruction else 0
    prefix = math.ceil(words * 1.30) + math.ceil(ins_words * 1.30) + ref_frames + 20
    conservative = math.ceil(words * 6.80) + 25
    return {
        "words": words,
        "prefix_tokens": prefix,
        "earliest_eos": max(16, math.floor(words * 3.75)),
        "expected_eos": math.ceil(words * 5.35) + 12,
        "conservative_max": conservative,
        "total_needed": (prefix + conservative) * (2 if cfg_scale > 1.0 else 1),
    }


class TieredSlotPool:
    """Admission slots in three capacity tiers (cluster.py:179-229): short (600 tokens), standard
    (1000) and long (2040). A request takes the first free slot of the smallest tier that holds
    it, falling back to larger tiers; slot ids are numbered across the tiers from 1."""

    TIERS = (("short", 600), ("standard", 1000), ("long", 2040))

    def __init__(self, short_slots: int = 16, standard_slots: int = 24, long_slots: int = 56):
        counts = (short_slots, standard_slots, long_slots)
        self.capacity = {name: cap for name, cap in self.TIERS}
        self.total = dict(zip(self.capacity, counts))
        self.free: Dict[str, List[int]] = {}
        self.tier_of: Dict[int, str] = {}
        first = 1
        for (name, _), n in zip(self.TIERS, counts):
            self.free[name] = list(range(first, first + n))
            for s in self.free[name]:
                self.tier_of[s] = name
            first += n
        self.lock = threading.Lock()

    def acquire(self, needed_tokens: int) -> Optional[Tuple[int, str, int]]:
        with self.lock:
            for name, cap in self.TIERS:
                if needed_tokens <= cap or name == "long":
                    if self.free[name]:
                        return self.free[name].pop(0), name, cap
            return None

    def release(self, slot_id: int) -> None:
        with self.lock:
            name = self.tier_of.get(slot_id)
            if name:
                self.free[name].append(slot_id)

    def active_count(self) -> int:
        with self.lock:
            return sum(self.total.values()) - sum(len(v) for v in self.free.values())

    def total_slots(self) -> int:
        return sum(self.total.values())


def select_burst_steps(active_sessions: dict, max_burst: int = 16) -> int:
    """Frames per burst in {16, 8, 4, 2, 1} from the quartiles of the live sessions' expected
    remaining frames (cluster.py:232-261): large bursts while three quarters of the streams have
    16 or more frames to go, shorter ones as streams near their expected end."""
    if not active_sessions:
        return 1
    rem = sorted(max(0, s.get("expected_eos", 200) - s.get("total_frames", 0)) for s in active_sessions.values())
    p25, p50 = rem[len(rem) // 4], rem[len(rem) // 2]
    if p25 >= 16:
        k = 16
    elif p25 >= 8 or p50 >= 16:
        k = 8
    elif p50 >= 8 or p25 >= 4:
        k = 4
    elif p50 >= 2:
        k = 2
    else:
        return 1
    return min(max_burst, k)


def pack_frames(frames: np.ndarray, width: int = WIRE_CODES) -> bytes:
    """Frames [n][>= width] of codes (0..65535) -> the wire form: `width` little-endian uint16
    per frame, frame-major."""
    f = np.asarray(frames)
    if f.ndim != 2 or f.shape[1] < width:
        raise ValueError("frames must be [n][>= width]")
    c = f[:, :width]
    if c.size and (c.min() < 0 or c.max() > 0xFFFF):
        raise ValueError("codes must fit in 16 bits")
    return np.ascontiguousarray(c, dtype="<u2").tobytes()


def unpack_frames(packet: bytes, width: int = WIRE_CODES) -> np.ndarray:
    """The wire form back to frames [n][width] int32."""
    if len(packet) % (2 * width):
        raise ValueError("packet length is not a whole number of frames")
    return np.frombuffer(packet, dtype="<u2").astype(np.int32).reshape(-1, width)


class IslandCluster:
    """One island per entry of `devices` (a GPU index; an index may repeat, which runs several
    islands on one GPU). `run_workload` feeds the tasks (optionally at arrival offsets in seconds)
    to a shared queue and returns one ClusterResult per task."""

    def __init__(self, model_path: str, devices: Sequence[int] = (0, 1), max_slots: int = 64, chunk_size: int = 32,
                 max_burst: int = 16, slot_tiers: Tuple[int, int, int] = (16, 24, 56), wire_codes: int = WIRE_CODES,
                 q4_depth_path: Optional[str] = None, q4_threshold: int = 48, keep_tokens: bool = False,
                 keep_pcm: bool = False):
        if not devices:
            raise ValueError("at least one island")
        self.model_path = model_path
        self.devices = list(devices)
        self.max_slots, self.chunk_size, self.max_burst = max_slots, chunk_size, max_burst
        self.slot_tiers, self.wire_codes = slot_tiers, wire_codes
        self.q4_threshold, self.keep_tokens, self.keep_pcm = q4_threshold, keep_tokens, keep_pcm
        self.gens = [GeneratorHandle(model_path, d) for d in self.devices]
        self.wire_codes = min(wire_codes, self.gens[0].nc)
        self.has_q4 = False
        if q4_depth_path:
            self.has_q4 = all(g.load_q4_depth(q4_depth_path) for g in self.gens)
        self.vocs: List[Optional[VocoderHandle]] = [None] * len(self.gens)

    def close(self) -> None:
        for v in self.vocs:
            if v is not None:
                v.close()
        for g in self.gens:
            g.close()
        self.vocs, self.gens = [], []

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def run_workload(self, tasks: Sequence[UserTask], arrival_offsets: Optional[Sequence[float]] = None,
                     on_tokens: Optional[Callable[[int, bytes, bool], None]] = None,
                     on_pcm_chunk: Optional[Callable[[int, np.ndarray, bool], None]] = None,
                     on_progress: Optional[Callable[[ClusterResult], None]] = None,
                     return_tokens: bool = False, out_dir: Optional[str] = None) -> List[ClusterResult]:
        """Serve `tasks`; `return_tokens` puts every request in token mode (cluster.py:562)."""
        jobs: "queue.Queue[Tuple[UserTask, float]]" = queue.Queue()
        results: List[ClusterResult] = []
        lock = threading.Lock()
        fed = threading.Event()
        errors: List[BaseException] = []
        if any(not (return_tokens or t.client_has_vocoder) for t in tasks):
            for i, g in enumerate(self.gens):
                if self.vocs[i] is None:
                    self.vocs[i] = VocoderHandle(generator=g)
        t0 = time.time()

        def feed():
            order = sorted(range(len(tasks)), key=lambda i: arrival_offsets[i] if arrival_offsets else 0.0)
            for i in order:
                if arrival_offsets:
                    delay = t0 + arrival_offsets[i] - time.time()
                    if delay > 0:
                        time.sleep(delay)
                jobs.put((tasks[i], time.time()))
            fed.set()

        def emit(res: ClusterResult):
            with lock:
                results.append(res)
            if on_progress:
                on_progress(res)

        def island(idx: int):
            try:
                self._island_loop(idx, jobs, fed, emit, on_tokens, on_pcm_chunk, return_tokens, out_dir)
            except BaseException as e:  # surfaced by run_workload
                errors.append(e)
                fed.set()

        feeder = threading.Thread(target=feed, daemon=True)
        workers = [threading.Thread(target=island, args=(i,), daemon=True) for i in range(len(self.gens))]
        feeder.start()
        for w in workers:
            w.start()
        feeder.join()
        for w in workers:
            w.join()
        if errors:
            raise errors[0]
        return sorted(results, key=lambda r: r.id)

    # ------------------------------------------------------------------------------- one island
    def _island_loop(self, idx, jobs, fed, emit, on_tokens, on_pcm_chunk, return_tokens, out_dir):
        gen, voc = self.gens[idx], self.vocs[idx]
        tag = f"GPU {self.devices[idx]} (island {idx})"
        pool = TieredSlotPool(*self.slot_tiers)
        active: Dict[int, dict] = {}
        pending: Optional[Tuple[UserTask, float]] = None
        while True:
            # A. admissions: every waiting arrival that has a slot, created in one call
            admit = []
            while len(active) + len(admit) < self.max_slots:
                if pending is not None:
                    item, pending = pending, None
                else:
                    try:
                        item = jobs.get_nowait()
                    except queue.Empty:
                        break
                task, arrival = item
                prof = estimate_speech_profile(task.text, task.instruction, task.ref_frames, task.cfg_scale)
                slot = pool.acquire(prof["prefix_tokens"] + prof["conservative_max"])
                if slot is None:
                    pending = item
                    break
                cap_out = max(64, slot[2] - prof["prefix_tokens"])
                budget = min(cap_out, task.max_steps if task.max_steps > 0 else prof["conservative_max"])
                admit.append((task, arrival, prof, slot, budget))
            if admit:
                t_exec = time.time()
                specs = []
                for task, _, _, _, budget in admit:
                    sp = dict(session_id=task.id, text=task.text, instruction=task.instruction, cfg_scale=task.cfg_scale,
                              seed=(task.seed + task.id) & 0xFFFFFFFF, max_new_tokens=budget)
                    if task.ref_codes is not None and task.ref_frames > 0:
                        sp.update(ref_text=task.ref_text, ref_codes=np.asarray(task.ref_codes, np.int32), ref_frames=task.ref_frames)
                    specs.append(sp)
                try:
                    gen.sessions_create_batch(specs)
                except RuntimeError:
                    for _, _, _, slot, _ in admit:
                        pool.release(slot[0])
                    raise
                for task, arrival, prof, slot, budget in admit:
                    # surge tiering (cluster.py:788-792): the Q4_K depth weights once the island is busy
                    if self.has_q4 and len(active) >= self.q4_threshold:
                        gen.session_set_q4(task.id, True)
                    active[task.id] = dict(task=task, arrival=arrival, t_exec=t_exec, words=prof["words"],
                                           expected_eos=prof["expected_eos"], slot=slot[0], max_steps=budget,
                                           total_frames=0, frames=[], emitted=0, first=None, pcm=[],
                                           tokens_mode=return_tokens or task.client_has_vocoder)
            if not active:
                if fed.is_set() and jobs.empty() and pending is None:
                    return
                time.sleep(0.002)
                continue
            # B. one burst over every live session
            ids = list(active)
            k = select_burst_steps(active, self.max_burst)
            seeds = [(active[s]["task"].seed + active[s]["total_frames"]) & 0xFFFFFFFF for s in ids]
            _, frames, nxt = gen.step_frames(ids, k, seeds)
            now = time.time()
            finished = []
            for i, sid in enumerate(ids):
                s = active[sid]
                new = []
                stop = False
                for step in range(k):
                    f = frames[step, i]
                    if f[0] < 0 or int(f[0]) in _STOP_CB0:
                        stop = True
                        break
                    new.append(f)
                    s["total_frames"] += 1
                    if s["total_frames"] >= s["max_steps"]:
                        stop = True
                        break
                if new:
                    s["frames"].extend(new)
                    if s["first"] is None and s["tokens_mode"]:
                        s["first"] = now
                if s["tokens_mode"] and on_tokens and (new or stop):
                    on_tokens(sid, pack_frames(np.asarray(new, np.int32).reshape(-1, frames.shape[2]), self.wire_codes)
                              if new else b"", stop or nxt[i] < 0)
                if stop or nxt[i] < 0:
                    finished.append(sid)
            # C. server-side audio: full chunks of streaming requests, batched in one decode
            if voc is not None:
                ready = []
                for sid, s in active.items():
                    if s["tokens_mode"] or not s["task"].stream_pcm:
                        continue
                    whole = (len(s["frames"]) - s["emitted"]) // self.chunk_size * self.chunk_size
                    if whole:  # every complete chunk of this burst in one span
                        ready.append((sid, s["emitted"], s["emitted"] + whole))
                self._vocode(voc, active, ready, on_pcm_chunk, final=False)
            # D. retirements: last audio, result, slot and session back
            tail = [(sid, active[sid]["emitted"], len(active[sid]["frames"])) for sid in finished
                    if not active[sid]["tokens_mode"]]
            if voc is not None and tail:
                self._vocode(voc, active, tail, on_pcm_chunk, final=True)
            for sid in finished:
                s = active.pop(sid)
                gen.session_free(sid)
                pool.release(s["slot"])
                emit(self._result(s, tag, out_dir))
                if voc is not None and not s["tokens_mode"]:
                    voc.session_free(sid)

    def _vocode(self, voc, active, spans, on_pcm_chunk, final):
        """Decodes frames [a, b) of each (session, a, b) in one batched vocoder call; `final`
        also tells `on_pcm_chunk` that each of these streams has ended."""
        work = [(sid, a, b) for sid, a, b in spans if b > a]
        if work:
            pcms = voc.session_decode_batch([sid for sid, _, _ in work],
                                            [np.asarray(active[sid]["frames"][a:b], np.int32) for sid, a, b in work])
            now = time.time()
            for (sid, a, b), pcm in zip(work, pcms):
                s = active[sid]
                s["emitted"] = b
                s["pcm"].append(pcm)
                if s["first"] is None:
                    s["first"] = now
                if on_pcm_chunk:
                    on_pcm_chunk(sid, pcm, False)
        if final and on_pcm_chunk:
            for sid, _, _ in spans:
                on_pcm_chunk(sid, np.zeros(0, np.float32), True)

    def _result(self, s, tag, out_dir) -> ClusterResult:
        t_end = time.time()
        task = s["task"]
        if s["tokens_mode"]:
            audio_s = s["total_frames"] * FRAME_S
            worker = tag + " [client tokens]"
        else:
            audio_s = sum(p.size for p in s["pcm"]) / SAMPLE_RATE
            worker = tag + " [server vocoder]"
        wall = t_end - s["t_exec"]
        turnaround = t_end - s["arrival"]
        first = s["first"] if s["first"] is not None else t_end
        wav = ""
        pcm = np.concatenate(s["pcm"]) if s["pcm"] else np.zeros(0, np.float32)
        if out_dir and not s["tokens_mode"]:
            os.makedirs(out_dir, exist_ok=True)
            wav = os.path.join(out_dir, f"island_user_{task.id:04d}.wav")
            write_wav(wav, pcm, SAMPLE_RATE)
        frames = np.asarray(s["frames"], np.int32).reshape(len(s["frames"]), -1) if s["frames"] else np.zeros((0, 0), np.int32)
        tokens = frames[:, :self.wire_codes].reshape(-1).tolist() if s["tokens_mode"] else None
        return ClusterResult(id=task.id, words=s["words"], audio_s=round(audio_s, 3),
                             queue_wait_s=round(s["t_exec"] - s["arrival"], 3), compute_wall_s=round(wall, 3),
                             turnaround_s=round(turnaround, 3), ttfa_s=round(first - s["arrival"], 3),
                             rtf=round(wall / (audio_s if audio_s > 0 else 1.0), 3), worker=worker, wav_path=wav,
                             tokens=tokens, frames=frames if self.keep_tokens else None,
                             pcm=pcm if self.keep_pcm else None)


# the reference's two-GPU cluster is the two-island case
def DualInstanceCluster(model_path: str, **kw) -> IslandCluster:
    return IslandCluster(model_path, devices=kw.pop("devices", (0, 1)), **kw)
