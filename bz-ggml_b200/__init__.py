"""Python host side of the B200 Breeze-TTS-2 generation library.

`libbreeze.so` (built from `csrc/` by `make`) exports the reference's C ABI
(sharjeel103/bz-ggml include/breeze/breeze.h); this module binds it with ctypes and mirrors
the reference's `python/bz_ggml/bindings.py` GeneratorHandle (same method names, argument
meaning and error behaviour: a failed create/load raises RuntimeError, step calls return
the C ABI's values). It adds the `bzb_*` extension entry points used by the benchmark and
the parity tests. There is no CPU fallback: without the built library, or without a CUDA
device, generator construction fails.

The directory name is not an importable identifier; load it with `load_package()` of the
repository's `__graft_entry__` or `importlib` under the name `bz_ggml_b200`.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import List, Optional, Sequence, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libbreeze.so")
SYNTH_BIN = os.path.join(HERE, "bin", "breeze-synth")

_c_int_p = ctypes.POINTER(ctypes.c_int)
_c_uint_p = ctypes.POINTER(ctypes.c_uint)
_c_float_p = ctypes.POINTER(ctypes.c_float)
_c_double_p = ctypes.POINTER(ctypes.c_double)


class BreezeRequest(ctypes.Structure):
    """breeze_request of include/breeze.h (reference include/breeze/breeze.h:25-45)."""
    _fields_ = [("text", ctypes.c_char_p), ("instruction", ctypes.c_char_p), ("ref_text", ctypes.c_char_p),
                ("ref_audio", _c_float_p), ("ref_audio_len", ctypes.c_int), ("cfg_scale", ctypes.c_float),
                ("seed", ctypes.c_int), ("max_new_tokens", ctypes.c_int), ("split_chars", ctypes.c_int),
                ("temperature", ctypes.c_float), ("top_k", ctypes.c_int), ("top_p", ctypes.c_float),
                ("repetition_penalty", ctypes.c_float)]


AUDIO_CB = ctypes.CFUNCTYPE(ctypes.c_int, _c_float_p, ctypes.c_int, ctypes.c_void_p)

# every symbol include/breeze.h and include/bzb_ext.h declare: name -> (restype, argtypes)
SIGNATURES = {
    "breeze_init": (ctypes.c_void_p, [ctypes.c_char_p, ctypes.c_int]),
    "breeze_free": (None, [ctypes.c_void_p]),
    "breeze_sample_rate": (ctypes.c_int, [ctypes.c_void_p]),
    "breeze_generate": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "breeze_generate_wav": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p]),
    "breeze_last_error": (ctypes.c_char_p, []),
    "breeze_generator_init": (ctypes.c_void_p, [ctypes.c_char_p, ctypes.c_int]),
    "breeze_generator_free": (None, [ctypes.c_void_p]),
    "breeze_generator_prefill": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_uint, _c_int_p]),
    "breeze_generator_step_frame": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_uint, _c_int_p]),
    "breeze_vocoder_init": (ctypes.c_void_p, [ctypes.c_char_p, ctypes.c_int]),
    "breeze_vocoder_free": (None, [ctypes.c_void_p]),
    "breeze_vocoder_create_from_generator": (ctypes.c_void_p, [ctypes.c_void_p]),
    "breeze_vocoder_session_create": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "breeze_vocoder_session_decode": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, _c_int_p, ctypes.c_int, _c_float_p]),
    "breeze_vocoder_session_decode_batch": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, _c_int_p, _c_int_p, _c_int_p,
                                                           _c_int_p, _c_float_p, _c_int_p, _c_int_p]),
    "breeze_vocoder_session_free": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "breeze_vocoder_stream_decode": (ctypes.c_int, [ctypes.c_void_p, _c_int_p, ctypes.c_int, _c_float_p]),
    "breeze_vocoder_stream_decode_batch": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, _c_int_p, _c_int_p, _c_int_p,
                                                          _c_float_p, _c_int_p, _c_int_p]),
    "breeze_generator_session_create": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_char_p,
                                                       ctypes.c_float, ctypes.c_uint, _c_int_p]),
    "breeze_generator_session_create_ext": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_char_p,
                                                           ctypes.c_char_p, _c_int_p, ctypes.c_int, ctypes.c_float,
                                                           ctypes.c_uint, ctypes.c_int, _c_int_p, _c_int_p]),
    "breeze_generator_session_step": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_uint, _c_int_p]),
    "breeze_generator_session_free": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "breeze_generator_load_q4_depth": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p]),
    "breeze_generator_session_set_q4": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]),
    "breeze_generator_session_count": (ctypes.c_int, [ctypes.c_void_p]),
    "breeze_generator_sessions_step_round": (ctypes.c_int, [ctypes.c_void_p, _c_int_p, ctypes.c_int, ctypes.c_uint,
                                                            _c_int_p, _c_int_p]),
    "breeze_generator_sessions_step_batched": (ctypes.c_int, [ctypes.c_void_p, _c_int_p, ctypes.c_int, _c_uint_p,
                                                              _c_int_p, _c_int_p]),
    "breeze_generator_sessions_step_burst": (ctypes.c_int, [ctypes.c_void_p, _c_int_p, ctypes.c_int, ctypes.c_int,
                                                            _c_uint_p, _c_int_p, _c_int_p]),
    "breeze_generator_convert_voice": (ctypes.c_int, [ctypes.c_void_p, _c_int_p, ctypes.c_int, _c_float_p, ctypes.c_int,
                                                      _c_int_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_char_p,
                                                      ctypes.c_float, ctypes.c_int, ctypes.c_int, ctypes.c_uint,
                                                      _c_int_p, _c_float_p, ctypes.c_int]),
    "breeze_generator_encode_audio": (ctypes.c_int, [ctypes.c_void_p, _c_float_p, ctypes.c_int, _c_int_p, _c_int_p]),
    "breeze_voice_save_file": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_char_p, _c_int_p, ctypes.c_int,
                                              ctypes.c_int, ctypes.c_int]),
    "breeze_voice_load_file": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_char_p,
                                              ctypes.c_int, _c_int_p, _c_int_p, _c_int_p, _c_int_p]),
    "bzb_generator_num_codebooks": (ctypes.c_int, [ctypes.c_void_p]),
    "bzb_generator_sessions_step_frames": (ctypes.c_int, [ctypes.c_void_p, _c_int_p, ctypes.c_int, ctypes.c_int,
                                                          _c_uint_p, _c_int_p, _c_int_p]),
    "bzb_generator_step_device": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "bzb_generator_sync": (ctypes.c_int, [ctypes.c_void_p]),
    "bzb_generator_stream": (ctypes.c_void_p, [ctypes.c_void_p]),
    "bzb_generator_weight_bytes_per_step": (ctypes.c_longlong, [ctypes.c_void_p]),
    "bzb_generator_kv_bytes_per_position": (ctypes.c_longlong, [ctypes.c_void_p]),
    "bzb_generator_launches_per_step": (ctypes.c_int, [ctypes.c_void_p]),
    "bzb_generator_profile_step": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_double)]),
    "bzb_generator_debug_hidden": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, _c_float_p]),
    "bzb_generator_debug_depth": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, _c_float_p, _c_int_p, _c_int_p,
                                                 _c_int_p, _c_float_p]),
    "bzb_generator_debug_gemv": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_int,
                                                _c_float_p, _c_float_p]),
    "bzb_generator_debug_gemm": (ctypes.c_longlong, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int, _c_float_p,
                                                     _c_float_p, ctypes.c_int, ctypes.c_int, _c_int_p, ctypes.c_int]),
    "bzb_vocoder_stream_open": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "bzb_vocoder_stream_close": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "bzb_vocoder_streams_decode": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, _c_int_p, _c_int_p, ctypes.c_int,
                                                  _c_float_p]),
    "bzb_vocoder_last_pcm": (ctypes.c_int, [ctypes.c_void_p, _c_float_p, ctypes.c_int]),
    "bzb_vocoder_kernels_per_decode": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]),
    "bzb_generator_sessions_step_pcm": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, _c_int_p, ctypes.c_int,
                                                       _c_uint_p, _c_int_p, _c_int_p, _c_float_p]),
    "bzb_generator_step_pcm_device": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, _c_int_p, ctypes.c_int,
                                                     _c_uint_p, ctypes.c_int]),
    "bzb_generator_debug_grid_spin": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_longlong]),
    "bzb_generator_debug_sample": (ctypes.c_int, [ctypes.c_void_p, _c_float_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                  ctypes.c_float, ctypes.c_float, ctypes.c_uint, ctypes.c_int,
                                                  ctypes.c_int, _c_int_p]),
    "bzb_debug_mbar_timeout": (ctypes.c_int, [ctypes.c_int, ctypes.c_longlong]),
    "bzb_generator_bench_gemv": (ctypes.c_double, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_int,
                                                    ctypes.c_int, ctypes.c_int]),
    "bzb_generator_depth_trace": (ctypes.c_int, [ctypes.c_void_p, _c_double_p, ctypes.c_int]),
    "bzb_generator_gemm_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_int, ctypes.c_void_p,
                                                  ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "bzb_gguf_inspect": (ctypes.c_int, [ctypes.c_char_p, _c_int_p, _c_int_p, _c_int_p]),
    "bzb_tokenize": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, _c_int_p, ctypes.c_int]),
    "bzb_generate_codes": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, _c_int_p, ctypes.c_int, ctypes.c_void_p,
                                          ctypes.c_void_p, _c_int_p, ctypes.c_int, _c_int_p, _c_double_p]),
    "bzb_split_text": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_char_p, ctypes.c_int]),
    "bzb_write_wav": (ctypes.c_int, [ctypes.c_char_p, _c_float_p, ctypes.c_int, ctypes.c_int]),
    "bzb_generator_sessions_create_batch": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, _c_int_p, ctypes.c_void_p,
                                                           ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, _c_int_p,
                                                           _c_float_p, _c_uint_p, _c_int_p, _c_int_p, _c_int_p]),
    "bzb_generator_encode_audio_full": (ctypes.c_int, [ctypes.c_void_p, _c_float_p, ctypes.c_int, _c_int_p, ctypes.c_int,
                                                       _c_int_p]),
}


def build(jobs: int = 8) -> None:
    """Compile libbreeze.so (sm_100a) and the breeze-synth tool in place."""
    subprocess.run(["make", "-C", HERE, f"-j{jobs}"], check=True)


class BreezeLib:
    """ctypes binding of libbreeze.so (mirrors bz_ggml.bindings.BreezeLib)."""

    def __init__(self, lib_path: Optional[str] = None):
        self.lib_path = lib_path or os.environ.get("BREEZE_LIB_PATH") or LIB_PATH
        if not os.path.exists(self.lib_path):
            raise FileNotFoundError(f"libbreeze.so not found at {self.lib_path}; run `make -C {HERE}`")
        self.lib = ctypes.CDLL(self.lib_path, mode=ctypes.RTLD_GLOBAL)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(self.lib, name)
            fn.restype = res
            fn.argtypes = args

    def last_error(self) -> str:
        e = self.lib.breeze_last_error()
        return e.decode("utf-8", "replace") if e else ""


_LIB: Optional[BreezeLib] = None


def lib() -> BreezeLib:
    global _LIB
    if _LIB is None:
        _LIB = BreezeLib()
    return _LIB


def _ip(a: np.ndarray):
    return a.ctypes.data_as(_c_int_p)


def _up(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(_c_uint_p)


def _fp(a: np.ndarray):
    return a.ctypes.data_as(_c_float_p)


class GeneratorHandle:
    """One generator on one CUDA device (mirrors bz_ggml.bindings.GeneratorHandle)."""

    def __init__(self, model_path: str, cuda_device: int = 0, breeze_lib: Optional[BreezeLib] = None):
        self.lib = breeze_lib or lib()
        self.device = cuda_device
        self.handle = self.lib.lib.breeze_generator_init(model_path.encode("utf-8"), cuda_device)
        if not self.handle:
            raise RuntimeError(f"Failed to initialize Generator on CUDA device {cuda_device}: {self.lib.last_error()}")
        self.nc = self.lib.lib.bzb_generator_num_codebooks(self.handle)

    def close(self):
        if self.handle:
            self.lib.lib.breeze_generator_free(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # --- reference-mirroring API -------------------------------------------------------
    def session_create(self, session_id: int, text: str, instruction: str = "Speak clearly and naturally.",
                       cfg_scale: float = 1.0, seed: int = 42, max_new_tokens: int = 0) -> Tuple[int, int]:
        return self.session_create_ext(session_id, text, instruction, None, None, 0, cfg_scale, seed, max_new_tokens)

    def session_create_ext(self, session_id: int, text: str, instruction: Optional[str] = "Speak clearly and naturally.",
                           ref_text: Optional[str] = None, ref_codes: Optional[Sequence[int]] = None, ref_frames: int = 0,
                           cfg_scale: float = 1.0, seed: int = 42, max_new_tokens: int = 0) -> Tuple[int, int]:
        cb0 = ctypes.c_int()
        alloc = ctypes.c_int()
        c_codes = None
        if ref_codes is not None and ref_frames > 0:
            arr = np.ascontiguousarray(np.asarray(ref_codes, dtype=np.int32).reshape(-1))
            c_codes = _ip(arr)
        res = self.lib.lib.breeze_generator_session_create_ext(
            self.handle, session_id, text.encode("utf-8"),
            instruction.encode("utf-8") if instruction else None,
            ref_text.encode("utf-8") if ref_text else None, c_codes, ref_frames,
            ctypes.c_float(cfg_scale), ctypes.c_uint(seed & 0xFFFFFFFF), max_new_tokens,
            ctypes.byref(cb0), ctypes.byref(alloc))
        if res != 0:
            raise RuntimeError(f"Session create ext failed (session {session_id}): {self.lib.last_error()}")
        return cb0.value, alloc.value

    def sessions_create_batch(self, specs: Sequence[dict]) -> Tuple[List[int], List[int]]:
        """session_create_ext for every spec (dicts of its keyword arguments plus session_id and
        text) in one call, the prompts prefilled as packed rows. Returns (cb0s, allocations)."""
        n = len(specs)
        keep = []

        def strs(key, default=None):
            arr = (ctypes.c_char_p * max(n, 1))()
            for i, sp in enumerate(specs):
                v = sp.get(key, default)
                arr[i] = v.encode("utf-8") if v else None
            keep.append(arr)
            return ctypes.cast(arr, ctypes.c_void_p)

        codes = (ctypes.POINTER(ctypes.c_int) * max(n, 1))()
        frames = np.zeros(max(n, 1), np.int32)
        for i, sp in enumerate(specs):
            rc, rf = sp.get("ref_codes"), int(sp.get("ref_frames", 0))
            if rc is not None and rf > 0:
                arr = np.ascontiguousarray(np.asarray(rc, dtype=np.int32).reshape(-1))
                keep.append(arr)
                codes[i] = _ip(arr)
                frames[i] = rf
        ids = np.asarray([sp["session_id"] for sp in specs] or [0], np.int32)
        scales = np.asarray([sp.get("cfg_scale", 1.0) for sp in specs] or [1.0], np.float32)
        seeds = np.asarray([sp.get("seed", 42) & 0xFFFFFFFF for sp in specs] or [0], np.uint32)
        budgets = np.asarray([sp.get("max_new_tokens", 0) for sp in specs] or [0], np.int32)
        cb0 = np.zeros(max(n, 1), np.int32)
        alloc = np.zeros(max(n, 1), np.int32)
        res = self.lib.lib.bzb_generator_sessions_create_batch(
            self.handle, n, _ip(ids), strs("text"), strs("instruction", "Speak clearly and naturally."),
            strs("ref_text"), ctypes.cast(codes, ctypes.c_void_p), _ip(frames), _fp(scales),
            seeds.ctypes.data_as(_c_uint_p), _ip(budgets), _ip(cb0), _ip(alloc))
        if res != 0:
            raise RuntimeError(f"Batched session create failed: {self.lib.last_error()}")
        return cb0[:n].tolist(), alloc[:n].tolist()

    def session_step(self, session_id: int, seed: int) -> Tuple[int, List[int]]:
        fr = np.zeros(16, np.int32)
        nxt = self.lib.lib.breeze_generator_session_step(self.handle, session_id, ctypes.c_uint(seed & 0xFFFFFFFF), _ip(fr))
        return nxt, fr.tolist()

    def session_free(self, session_id: int) -> int:
        return self.lib.lib.breeze_generator_session_free(self.handle, session_id)

    def active_session_count(self) -> int:
        return self.lib.lib.breeze_generator_session_count(self.handle)

    def sessions_step_round(self, session_ids: Sequence[int], seed: int = 42) -> Tuple[List[int], List[List[int]]]:
        """One session_step per listed session with seed + i (reference bindings.py:307-319): returns
        (next cb0 per session, -1 at EOS, budget or unknown session; frames [n][16], rows of sessions
        that did not step left zero)."""
        n = len(session_ids)
        if n == 0:
            return [], []
        ids = np.asarray(session_ids, np.int32)
        fr = np.zeros((n, 16), np.int32)
        nx = np.zeros(n, np.int32)
        self.last_round_completed = self.lib.lib.breeze_generator_sessions_step_round(
            self.handle, _ip(ids), n, ctypes.c_uint(seed & 0xFFFFFFFF), _ip(fr), _ip(nx))
        return nx.tolist(), fr.tolist()

    def sessions_step_batched(self, session_ids: Sequence[int], seeds: Optional[Sequence[int]] = None):
        n = len(session_ids)
        ids = np.asarray(session_ids, np.int32)
        fr = np.zeros((n, 16), np.int32)
        nx = np.zeros(n, np.int32)
        sd = None if seeds is None else np.asarray(seeds, np.uint32)
        rc = self.lib.lib.breeze_generator_sessions_step_batched(self.handle, _ip(ids), n, _up(sd), _ip(fr), _ip(nx))
        if rc < 0:
            raise RuntimeError(f"sessions_step_batched failed: {self.lib.last_error()}")
        return nx.tolist(), fr.tolist()

    def sessions_step_burst(self, session_ids: Sequence[int], burst_steps: int, seeds: Optional[Sequence[int]] = None):
        """Returns (next_cb0 per session, frames [session][step][16]) like the reference binding."""
        n = len(session_ids)
        ids = np.asarray(session_ids, np.int32)
        fr = np.zeros((burst_steps, n, 16), np.int32)
        nx = np.zeros(n, np.int32)
        sd = None if seeds is None else np.asarray(seeds, np.uint32)
        rc = self.lib.lib.breeze_generator_sessions_step_burst(self.handle, _ip(ids), n, burst_steps, _up(sd), _ip(fr), _ip(nx))
        if rc < 0:
            raise RuntimeError(f"sessions_step_burst failed: {self.lib.last_error()}")
        return nx.tolist(), fr.transpose(1, 0, 2).tolist()

    # --- extensions ----------------------------------------------------------------------
    def step_frames(self, session_ids: Sequence[int], burst_steps: int, seeds: Optional[Sequence[int]] = None):
        """Full-width burst: returns (steps executed, frames [K, n, nc] int32, next_cb0 [n])."""
        n = len(session_ids)
        ids = np.ascontiguousarray(np.asarray(session_ids, np.int32))
        fr = np.zeros((burst_steps, n, self.nc), np.int32)
        nx = np.zeros(n, np.int32)
        sd = None if seeds is None else np.ascontiguousarray(np.asarray(seeds, np.uint32))
        rc = self.lib.lib.bzb_generator_sessions_step_frames(self.handle, _ip(ids), n, burst_steps, _up(sd), _ip(fr), _ip(nx))
        if rc < 0:
            raise RuntimeError(f"step_frames failed: {self.lib.last_error()}")
        return rc, fr, nx

    def step_pcm(self, voc: "VocoderHandle", session_ids: Sequence[int], seeds: Optional[Sequence[int]] = None,
                 want_frames: bool = True, want_pcm: bool = True):
        """One frame step of the listed sessions plus the PCM of every new frame, decoded on each
        session's vocoder stream (bzb_generator_sessions_step_pcm). Returns (still active, frames
        [n][nc] or None, next cb0 [n], pcm [n][1920] or None)."""
        n = len(session_ids)
        ids = np.ascontiguousarray(np.asarray(session_ids, np.int32))
        fr = np.zeros((n, self.nc), np.int32) if want_frames else None
        nx = np.zeros(n, np.int32)
        pcm = np.zeros((n, VocoderHandle.SAMPLES_PER_FRAME), np.float32) if want_pcm else None
        sd = None if seeds is None else np.ascontiguousarray(np.asarray(seeds, np.uint32))
        rc = self.lib.lib.bzb_generator_sessions_step_pcm(self.handle, voc.handle, _ip(ids), n, _up(sd),
                                                          None if fr is None else _ip(fr), _ip(nx),
                                                          None if pcm is None else _fp(pcm))
        if rc < 0:
            raise RuntimeError(f"sessions_step_pcm failed: {self.lib.last_error()}")
        return rc, fr, nx, pcm

    def step_pcm_device(self, voc: "VocoderHandle", session_ids: Sequence[int], seeds: Optional[Sequence[int]] = None,
                        burst_steps: int = 1) -> None:
        """burst_steps device-resident frame steps, each followed by the streaming decode of its frames
        (bzb_generator_step_pcm_device); asynchronous on the generator's stream."""
        ids = np.ascontiguousarray(np.asarray(session_ids, np.int32))
        sd = None if seeds is None else np.ascontiguousarray(np.asarray(seeds, np.uint32))
        if self.lib.lib.bzb_generator_step_pcm_device(self.handle, voc.handle, _ip(ids), len(ids), _up(sd), burst_steps) != 0:
            raise RuntimeError(self.lib.last_error())

    def step_device(self, burst_steps: int) -> None:
        if self.lib.lib.bzb_generator_step_device(self.handle, burst_steps) != 0:
            raise RuntimeError(self.lib.last_error())

    def sync(self) -> None:
        if self.lib.lib.bzb_generator_sync(self.handle) != 0:
            raise RuntimeError(self.lib.last_error())

    def stream_ptr(self) -> int:
        return int(self.lib.lib.bzb_generator_stream(self.handle) or 0)

    def weight_bytes_per_step(self) -> int:
        return int(self.lib.lib.bzb_generator_weight_bytes_per_step(self.handle))

    def kv_bytes_per_position(self) -> int:
        return int(self.lib.lib.bzb_generator_kv_bytes_per_position(self.handle))

    def launches_per_step(self) -> int:
        return int(self.lib.lib.bzb_generator_launches_per_step(self.handle))

    def profile_step(self) -> dict:
        out = (ctypes.c_double * 7)()
        if self.lib.lib.bzb_generator_profile_step(self.handle, out) != 0:
            raise RuntimeError(self.lib.last_error())
        return dict(step_ms=out[0], gemm_ms=out[1], gemm_launches=int(out[2]), gemm_bytes=out[3],
                    depth_ms=out[5], depth_bytes=out[6])

    def bench_gemv(self, tensor: str, rows: int, iters: int = 50, epilogue: int = 0, sub: int = -1) -> float:
        us = self.lib.lib.bzb_generator_bench_gemv(self.handle, tensor.encode(), sub, rows, iters, epilogue)
        if us < 0:
            raise RuntimeError(self.lib.last_error())
        return us

    def depth_trace(self):
        """Timeline of one persistent depth launch: (phase types [n], times [n][grid][slots] in
        microseconds, -1 where a slot was not reached), or None without the persistent path."""
        need = self.lib.lib.bzb_generator_depth_trace(self.handle, None, 0)
        if need < 0:
            raise RuntimeError(self.lib.last_error())
        if need == 0:
            return None
        out = np.zeros(need, np.float64)
        if self.lib.lib.bzb_generator_depth_trace(self.handle, out.ctypes.data_as(_c_double_p), need) < 0:
            raise RuntimeError(self.lib.last_error())
        n, g, k = int(out[0]), int(out[1]), int(out[2])
        return out[3:3 + n].astype(int), out[3 + n:].reshape(n, g, k)

    def gemm_noalloc(self, tensor: str, rows: int, x16_ptr: int, ldx: int, y_ptr: int, ldy: int,
                     stream_ptr: int = 0) -> None:
        """Allocation-free dequant-GEMM on caller-owned device buffers (pointers as ints);
        asynchronous on `stream_ptr` (0 = the generator's stream)."""
        if self.lib.lib.bzb_generator_gemm_noalloc(self.handle, tensor.encode(), rows, x16_ptr, ldx, y_ptr, ldy,
                                                    stream_ptr or None) != 0:
            raise RuntimeError(self.lib.last_error())

    def debug_hidden(self, session_id: int, hidden: int) -> np.ndarray:
        out = np.zeros(hidden, np.float32)
        if self.lib.lib.bzb_generator_debug_hidden(self.handle, session_id, _fp(out)) != 0:
            raise RuntimeError(self.lib.last_error())
        return out

    def debug_depth(self, hidden: np.ndarray, cb0: Sequence[int], vs: int, forced: Optional[np.ndarray] = None):
        n = hidden.shape[0]
        h = np.ascontiguousarray(hidden, np.float32)
        c = np.ascontiguousarray(np.asarray(cb0, np.int32))
        codes = np.zeros((n, self.nc - 1), np.int32)
        logits = np.zeros((n, self.nc - 1, vs), np.float32)
        f = None if forced is None else np.ascontiguousarray(np.asarray(forced, np.int32))
        rc = self.lib.lib.bzb_generator_debug_depth(self.handle, n, _fp(h), _ip(c), None if f is None else _ip(f),
                                                    _ip(codes), _fp(logits))
        if rc != 0:
            raise RuntimeError(self.lib.last_error())
        return codes, logits

    def convert_voice(self, src_codes: Sequence[int], src_T: int, ref_audio=None, ref_codes: Optional[Sequence[int]] = None,
                      ref_frames: int = 0, ref_text: Optional[str] = None, src_text: Optional[str] = None,
                      cfg_scale: float = 1.5, keep_acoustic: int = 0, feed_source: bool = True, seed: int = 42,
                      return_pcm: bool = True):
        """Voice conversion of encoded source frames into the reference voice (mirrors
        bz_ggml.bindings.GeneratorHandle.convert_voice): returns (pcm or None, codes)."""
        src = np.ascontiguousarray(np.asarray(src_codes, np.int32))
        ra = None if ref_audio is None or len(ref_audio) == 0 else np.ascontiguousarray(np.asarray(ref_audio, np.float32))
        rc = None if not ref_codes or ref_frames <= 0 else np.ascontiguousarray(np.asarray(ref_codes, np.int32))
        out_codes = np.zeros(src_T * 16, np.int32)
        pcm = np.zeros(src_T * 1920 + 32000, np.float32) if return_pcm else None
        res = self.lib.lib.breeze_generator_convert_voice(
            self.handle, _ip(src), src_T, None if ra is None else _fp(ra), 0 if ra is None else ra.size,
            None if rc is None else _ip(rc), 0 if rc is None else ref_frames,
            ref_text.encode("utf-8") if ref_text else None, src_text.encode("utf-8") if src_text else None,
            ctypes.c_float(cfg_scale), keep_acoustic, 1 if feed_source else 0, ctypes.c_uint(seed & 0xFFFFFFFF),
            _ip(out_codes), None if pcm is None else _fp(pcm), 0 if pcm is None else pcm.size)
        if res < 0:
            raise RuntimeError(f"Voice conversion failed on Generator (device {self.device}): {self.lib.last_error()}")
        return (pcm[:res].tolist() if return_pcm else None), out_codes.tolist()

    def encode_audio(self, pcm_samples) -> Tuple[List[int], int]:
        """24 kHz mono PCM -> (codes, n_frames), min(num_codebooks, 16) codes per frame
        (mirrors bz_ggml.bindings.GeneratorHandle.encode_audio)."""
        x = np.ascontiguousarray(np.asarray(pcm_samples, np.float32))
        if x.size == 0:
            return [], 0
        w = min(self.nc, 16)
        out = np.zeros((x.size // 1920 + 64) * w, np.int32)
        nf = ctypes.c_int(0)
        res = self.lib.lib.breeze_generator_encode_audio(self.handle, _fp(x), x.size, _ip(out), ctypes.byref(nf))
        if res < 0:
            raise RuntimeError(f"Audio encoding failed on Generator (device {self.device}): {self.lib.last_error()}")
        return out[: nf.value * w].tolist(), nf.value

    def encode_audio_full(self, pcm_samples) -> np.ndarray:
        """All num_codebooks codes per frame: [n_frames][num_codebooks] int32."""
        x = np.ascontiguousarray(np.asarray(pcm_samples, np.float32))
        mf = x.size // 1920
        out = np.zeros((max(mf, 1), self.nc), np.int32)
        nf = ctypes.c_int(0)
        if self.lib.lib.bzb_generator_encode_audio_full(self.handle, _fp(x), x.size, _ip(out), mf, ctypes.byref(nf)) < 0:
            raise RuntimeError(self.lib.last_error())
        return out[: nf.value]

    def load_q4_depth(self, q4_model_path: str) -> bool:
        """The Q4_K depth override (dd.* of a second GGUF) for flagged sessions."""
        if self.lib.lib.breeze_generator_load_q4_depth(self.handle, q4_model_path.encode("utf-8")) != 0:
            raise RuntimeError(f"Failed to load modular Q4 depth decoder on Generator (device {self.device}): "
                               f"{self.lib.last_error()}")
        return True

    def session_set_q4(self, session_id: int, use_q4: bool = True) -> bool:
        return self.lib.lib.breeze_generator_session_set_q4(self.handle, session_id, 1 if use_q4 else 0) == 0

    def debug_gemm(self, name: str, x: np.ndarray, out_dim: int, repeats: int = 0, pdl: bool = True,
                   where_cap: int = 0):
        """One launch of a resident (step-layout) matrix on x [rows][K]: returns (y [rows][out_dim],
        32-bit words that differed over `repeats` captured re-launches); with where_cap > 0 also the
        first differences as an array of (word index, repeat index) rows."""
        xx = np.ascontiguousarray(x, np.float32)
        y = np.zeros((xx.shape[0], out_dim), np.float32)
        where = np.zeros((max(where_cap, 1), 2), np.int32)
        n = self.lib.lib.bzb_generator_debug_gemm(self.handle, name.encode(), xx.shape[0], _fp(xx), _fp(y), repeats,
                                                  0 if pdl else 1, _ip(where) if where_cap else None, where_cap)
        if n < 0:
            raise RuntimeError(self.lib.last_error())
        if where_cap:
            return y, int(n), where[:min(int(n), where_cap)]
        return y, int(n)

    def debug_sample(self, logits: np.ndarray, top_k: int, temp: float, top_p: float = 1.0, seed: int = 0,
                     draws: int = 1, force_sort: bool = False) -> np.ndarray:
        """cb0 sampler picks [draws][rows] on logits [rows][V] (bzb_generator_debug_sample)."""
        lg = np.ascontiguousarray(np.asarray(logits, np.float32))
        rows, V = lg.shape
        out = np.zeros((draws, rows), np.int32)
        if self.lib.lib.bzb_generator_debug_sample(self.handle, _fp(lg), V, rows, top_k, temp, top_p, seed & 0xFFFFFFFF,
                                                   draws, 1 if force_sort else 0, _ip(out)) != 0:
            raise RuntimeError(self.lib.last_error())
        return out

    def set_debug_grid_spin(self, polls: int) -> None:
        """Grid-barrier poll limit of the persistent depth launches debug_depth makes (0: default)."""
        if self.lib.lib.bzb_generator_debug_grid_spin(self.handle, int(polls)) != 0:
            raise RuntimeError(self.lib.last_error())

    def debug_gemv(self, tensor: str, x: np.ndarray, out_dim: int, sub: int = -1) -> np.ndarray:
        xx = np.ascontiguousarray(x, np.float32)
        y = np.zeros((xx.shape[0], out_dim), np.float32)
        if self.lib.lib.bzb_generator_debug_gemv(self.handle, tensor.encode(), sub, xx.shape[0], _fp(xx), _fp(y)) != 0:
            raise RuntimeError(self.lib.last_error())
        return y


class VocoderHandle:
    """Codec decoder sessions (mirror of the reference's python/bz_ggml/bindings.py
    VocoderHandle): frames are [n_frames][num_codebooks] ints, PCM is 1920 f32 samples per frame
    at 24 kHz."""

    SAMPLES_PER_FRAME = 1920

    def __init__(self, model_path: str = "", cuda_device: int = 0, generator: Optional["GeneratorHandle"] = None):
        self.lib = lib()
        if generator is not None:
            self.handle = self.lib.lib.breeze_vocoder_create_from_generator(generator.handle)
            self._gen = generator
        else:
            self.handle = self.lib.lib.breeze_vocoder_init(model_path.encode(), cuda_device)
        if not self.handle:
            raise RuntimeError(f"vocoder init failed: {self.lib.last_error()}")

    def session_create(self, session_id: int) -> int:
        return self.lib.lib.breeze_vocoder_session_create(self.handle, session_id)

    def session_decode(self, session_id: int, frames: np.ndarray) -> np.ndarray:
        f = np.ascontiguousarray(frames, np.int32)
        n = f.shape[0]
        out = np.zeros(n * self.SAMPLES_PER_FRAME, np.float32)
        got = self.lib.lib.breeze_vocoder_session_decode(self.handle, session_id, _ip(f), n, _fp(out))
        if got <= 0:
            raise RuntimeError(f"session_decode failed: {self.lib.last_error()}")
        return out[:got]

    def session_decode_batch(self, session_ids: Sequence[int], batch_frames: Sequence[np.ndarray]) -> List[np.ndarray]:
        nf = np.array([np.asarray(b).shape[0] for b in batch_frames], np.int32)
        flat = np.ascontiguousarray(np.concatenate([np.asarray(b, np.int32).reshape(-1) for b in batch_frames]))
        ids = np.asarray(session_ids, np.int32)
        pcm = np.zeros(int(nf.sum()) * self.SAMPLES_PER_FRAME, np.float32)
        ns = np.zeros(len(ids), np.int32)
        got = self.lib.lib.breeze_vocoder_session_decode_batch(self.handle, len(ids), _ip(ids), _ip(flat), None, _ip(nf),
                                                               _fp(pcm), None, _ip(ns))
        if got != len(ids):
            raise RuntimeError(f"session_decode_batch failed: {self.lib.last_error()}")
        offs = np.concatenate([[0], np.cumsum(ns)])
        return [pcm[offs[i]:offs[i + 1]] for i in range(len(ids))]

    def session_free(self, session_id: int) -> int:
        return self.lib.lib.breeze_vocoder_session_free(self.handle, session_id)

    def stream_open(self, stream_id: int) -> None:
        if self.lib.lib.bzb_vocoder_stream_open(self.handle, stream_id) != 0:
            raise RuntimeError(self.lib.last_error())

    def stream_close(self, stream_id: int) -> bool:
        return self.lib.lib.bzb_vocoder_stream_close(self.handle, stream_id) == 0

    def streams_decode(self, stream_ids: Sequence[int], codes: np.ndarray) -> np.ndarray:
        """codes [n][T][nc] new frames of n distinct streams -> PCM [n][T * 1920], each stream
        continuing its carried decoder state (bzb_vocoder_streams_decode)."""
        c = np.ascontiguousarray(codes, np.int32)
        n, T = c.shape[0], c.shape[1]
        ids = np.ascontiguousarray(np.asarray(stream_ids, np.int32))
        out = np.zeros((n, T * self.SAMPLES_PER_FRAME), np.float32)
        if self.lib.lib.bzb_vocoder_streams_decode(self.handle, n, _ip(ids), _ip(c), T, _fp(out)) != n:
            raise RuntimeError(f"streams_decode failed: {self.lib.last_error()}")
        return out

    def kernels_per_decode(self, n_streams: int, n_frames: int) -> int:
        n = self.lib.lib.bzb_vocoder_kernels_per_decode(self.handle, n_streams, n_frames)
        if n < 0:
            raise RuntimeError(self.lib.last_error())
        return n

    def last_pcm(self, n_samples: int) -> np.ndarray:
        """The PCM the last device-resident step left in the vocoder (synchronises)."""
        out = np.zeros(n_samples, np.float32)
        if self.lib.lib.bzb_vocoder_last_pcm(self.handle, _fp(out), n_samples) != n_samples:
            raise RuntimeError(self.lib.last_error())
        return out

    def stream_decode(self, frames: np.ndarray) -> np.ndarray:
        f = np.ascontiguousarray(frames, np.int32)
        out = np.zeros(f.shape[0] * self.SAMPLES_PER_FRAME, np.float32)
        got = self.lib.lib.breeze_vocoder_stream_decode(self.handle, _ip(f), f.shape[0], _fp(out))
        if got <= 0:
            raise RuntimeError(f"stream_decode failed: {self.lib.last_error()}")
        return out[:got]

    def close(self):
        if getattr(self, "handle", None):
            self.lib.lib.breeze_vocoder_free(self.handle)
            self.handle = None

    def __del__(self):
        self.close()


class ContextHandle:
    """breeze_init / breeze_generate / breeze_generate_wav (reference src/c_api.cpp:50-108): one
    request at a time, PCM streamed through a callback."""

    def __init__(self, model_path: str, use_gpu: int = 1):
        self.lib = lib()
        self.handle = self.lib.lib.breeze_init(model_path.encode(), use_gpu)
        if not self.handle:
            raise RuntimeError(f"breeze_init failed: {self.lib.last_error()}")
        self.nc = gguf_inspect(model_path)[1]

    @property
    def sample_rate(self) -> int:
        return self.lib.lib.breeze_sample_rate(self.handle)

    @staticmethod
    def request(text: str, instruction: Optional[str] = None, ref_text: Optional[str] = None, cfg_scale: float = 0.0,
                seed: int = 42, max_new_tokens: int = 0, split_chars: int = 0, temperature: float = 0.0,
                top_k: int = 0, top_p: float = 0.0, repetition_penalty: float = 0.0,
                ref_audio: Optional[np.ndarray] = None) -> BreezeRequest:
        enc = lambda x: None if x is None else x.encode("utf-8")
        ra = None if ref_audio is None else np.ascontiguousarray(ref_audio, np.float32)
        r = BreezeRequest(enc(text), enc(instruction), enc(ref_text), None if ra is None else _fp(ra),
                          0 if ra is None else ra.size, cfg_scale, seed, max_new_tokens, split_chars, temperature,
                          top_k, top_p, repetition_penalty)
        r._keep = ra  # the PCM must outlive the request
        return r

    def generate(self, req: BreezeRequest, stop_after_chunks: int = 0, ref_codes: Optional[np.ndarray] = None,
                 max_frames: int = 4096):
        """Runs one request (bzb_generate_codes: breeze_generate plus encoded reference codes);
        returns (pcm, chunk sizes, frames [F][nc], F, timings dict). With stop_after_chunks > 0
        the callback asks to stop after that many chunks."""
        chunks: List[np.ndarray] = []

        def on_audio(ptr, n, user):
            chunks.append(np.ctypeslib.as_array(ptr, shape=(n,)).copy())
            return 1 if stop_after_chunks and len(chunks) >= stop_after_chunks else 0

        cb = AUDIO_CB(on_audio)
        codes = np.zeros((max_frames, self.nc), np.int32)
        nf = ctypes.c_int()
        tm = np.zeros(7, np.float64)
        rc = None if ref_codes is None else np.ascontiguousarray(ref_codes, np.int32)
        res = self.lib.lib.bzb_generate_codes(self.handle, ctypes.byref(req), None if rc is None else _ip(rc),
                                              0 if rc is None else rc.shape[0], ctypes.cast(cb, ctypes.c_void_p), None,
                                              _ip(codes), max_frames, ctypes.byref(nf), tm.ctypes.data_as(_c_double_p))
        if res != 0:
            raise RuntimeError(f"breeze_generate failed: {self.lib.last_error()}")
        pcm = np.concatenate(chunks) if chunks else np.zeros(0, np.float32)
        timings = dict(zip(["prefill_ms", "steps_ms", "vocoder_ms", "first_audio_ms", "frames", "flushes", "pieces"],
                           tm.tolist()))
        n = int(nf.value)
        return pcm, [c.size for c in chunks], codes[:min(n, max_frames)], n, timings

    def generate_wav(self, req: BreezeRequest, path: str) -> None:
        if self.lib.lib.breeze_generate_wav(self.handle, ctypes.byref(req), path.encode()) != 0:
            raise RuntimeError(f"breeze_generate_wav failed: {self.lib.last_error()}")

    def close(self):
        if getattr(self, "handle", None):
            self.lib.lib.breeze_free(self.handle)
            self.handle = None

    def __del__(self):
        self.close()


def mbar_timeout_probe(polls: int, device: int = 0) -> int:
    """Error code recorded by the tcgen05 pipelines' bounded mbarrier wait when it runs out on a
    barrier nothing arrives on (bzb_debug_mbar_timeout)."""
    code = lib().lib.bzb_debug_mbar_timeout(device, int(polls))
    if code < 0:
        raise RuntimeError(lib().last_error())
    return code


def split_text(text: str, budget: int, first_budget: int = 0) -> List[str]:
    """The library's long-text splitter (bzb_split_text)."""
    need = lib().lib.bzb_split_text(text.encode("utf-8"), budget, first_budget, None, 0)
    buf = ctypes.create_string_buffer(-need)
    n = lib().lib.bzb_split_text(text.encode("utf-8"), budget, first_budget, buf, len(buf))
    if n < 0:
        raise RuntimeError("split_text: buffer sizing failed")
    parts = buf.raw.split(b"\0")[:n]
    return [p.decode("utf-8") for p in parts]


def write_wav(path: str, samples: np.ndarray, sample_rate: int) -> None:
    """The library's 16-bit WAV writer (bzb_write_wav)."""
    x = np.ascontiguousarray(samples, np.float32)
    if lib().lib.bzb_write_wav(path.encode(), _fp(x), x.size, sample_rate) != 0:
        raise RuntimeError(lib().last_error())


def gguf_inspect(path: str):
    h, nc, nt = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    if lib().lib.bzb_gguf_inspect(path.encode(), ctypes.byref(h), ctypes.byref(nc), ctypes.byref(nt)) != 0:
        raise RuntimeError(lib().last_error())
    return h.value, nc.value, nt.value


def tokenize(path: str, text: str, add_bos: bool = True) -> List[int]:
    buf = np.zeros(1 << 16, np.int32)
    n = lib().lib.bzb_tokenize(path.encode(), text.encode("utf-8"), 1 if add_bos else 0, _ip(buf), buf.size)
    if n < 0:
        raise RuntimeError(lib().last_error())
    return buf[:n].tolist()


def synth_model(out_path: str, preset: str = "full", nc: int = 0, quant: str = "q8_0", seed: int = 0,
                eos_off: bool = False, max_new_tokens: int = 0, depth_top_k: int = -1) -> str:
    """Write a seeded random-init Breeze-TTS-2 GGUF (the stand-in for real weights)."""
    if not os.path.exists(SYNTH_BIN):
        raise FileNotFoundError(f"{SYNTH_BIN} missing; run `make -C {HERE}`")
    cmd = [SYNTH_BIN, "--out", out_path, "--preset", preset, "--quant", quant, "--seed", str(seed)]
    if nc:
        cmd += ["--nc", str(nc)]
    if eos_off:
        cmd += ["--eos-off"]
    if max_new_tokens:
        cmd += ["--max-new-tokens", str(max_new_tokens)]
    if depth_top_k >= 0:
        cmd += ["--depth-top-k", str(depth_top_k)]
    subprocess.run(cmd, check=True)
    return out_path


def ids_to_text(ids: Sequence[int]) -> str:
    """Text whose synthetic-vocabulary tokenisation is exactly `ids` (ids >= 264)."""
    return "".join(f"<|t{int(i)}|>" for i in ids)
