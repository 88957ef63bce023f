"""CPU oracle for the Breeze-TTS-2 generation path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, what the reference computes on its ggml CPU path for the
batched decode step and the session prefill that feeds it. Only `tests/`, the package's
`smoke()` entry and `bench.py`'s CPU-baseline leg may import it, and only as the checker:
no product code path calls into it.

Parity anchoring: the reference's arithmetic lives in ggml (un-vendored, unpinned: a
`master` FetchContent in CMakeLists.txt:26-35), and the reference's own tests hold no
golden logits, tokens or PCM. The dequantisers below are pinned bit-exactly against
gguf-py 0.19.0 (`gguf.quants`); everything downstream of them is a restatement of the
reference call sites cited on each function ("parity unpinned" beyond dequantisation).

Two numeric modes for quantised linears (`linear`):
  * "exact": f32 activations times the dequantised f32 weights (the engine computes this to
    within f16 activation rounding);
  * "ggml": activations quantised per 32-block to Q8_0 before an integer dot, the way ggml's
    CPU backend evaluates a Q8_0 weight (vec_dot_type Q8_0).
"""
from __future__ import annotations

import ctypes
import math
import os
from dataclasses import dataclass, field

import numpy as np

try:  # gguf-py is the third-party reader used to walk the file; dequantisation is ours
    import gguf  # type: ignore
except Exception:  # pragma: no cover
    gguf = None

_LIBM = ctypes.CDLL("libm.so.6")
_LIBM.powf.restype = ctypes.c_float
_LIBM.powf.argtypes = [ctypes.c_float, ctypes.c_float]

F32, F16, Q8_0, Q4_K = 0, 1, 8, 12


# ----------------------------------------------------------------------------- dequantisation
def dequant_q8_0(raw: np.ndarray, n: int) -> np.ndarray:
    """Q8_0 blocks (f16 d + 32 x int8) -> f32; ggml-quants.c dequantize_row_q8_0 semantics."""
    b = raw.reshape(-1, 34)
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    q = b[:, 2:].copy().view(np.int8).astype(np.float32)
    return (q * d).reshape(-1)[:n]


def q4k_scale_min(scales: np.ndarray):
    """6-bit scale/min unpacking of a Q4_K block (ggml get_scale_min_k4)."""
    s = scales.astype(np.int32)
    sc = np.empty((s.shape[0], 8), np.int32)
    mn = np.empty((s.shape[0], 8), np.int32)
    for j in range(4):
        sc[:, j] = s[:, j] & 63
        mn[:, j] = s[:, j + 4] & 63
    for j in range(4, 8):
        sc[:, j] = (s[:, j + 4] & 0xF) | ((s[:, j - 4] >> 6) << 4)
        mn[:, j] = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
    return sc, mn


def dequant_q4_k(raw: np.ndarray, n: int) -> np.ndarray:
    """Q4_K super-blocks of 256 (d, dmin, 12 packed scale bytes, 128 nibble bytes) -> f32."""
    b = raw.reshape(-1, 144)
    d = b[:, 0:2].copy().view(np.float16).astype(np.float32)
    dmin = b[:, 2:4].copy().view(np.float16).astype(np.float32)
    sc, mn = q4k_scale_min(b[:, 4:16])
    qs = b[:, 16:]
    out = np.empty((b.shape[0], 256), np.float32)
    for c in range(4):
        q = qs[:, c * 32:(c + 1) * 32]
        lo = (q & 0xF).astype(np.float32)
        hi = (q >> 4).astype(np.float32)
        d1 = d * sc[:, 2 * c:2 * c + 1].astype(np.float32)
        m1 = dmin * mn[:, 2 * c:2 * c + 1].astype(np.float32)
        d2 = d * sc[:, 2 * c + 1:2 * c + 2].astype(np.float32)
        m2 = dmin * mn[:, 2 * c + 1:2 * c + 2].astype(np.float32)
        out[:, c * 64:c * 64 + 32] = d1 * lo - m1
        out[:, c * 64 + 32:c * 64 + 64] = d2 * hi - m2
    return out.reshape(-1)[:n]


def quant_q8_0_rows(x: np.ndarray):
    """Activation Q8_0 quantisation per 32-block (ggml quantize_row_q8_0 rule): returns int8
    values and the f16-rounded block scales as f32."""
    xb = x.astype(np.float32).reshape(x.shape[0], -1, 32)
    amax = np.abs(xb).max(axis=2, keepdims=True)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d == 0, np.float32(0), np.float32(1.0) / d).astype(np.float32)
    v = (xb * idv).astype(np.float32)
    a = np.abs(v)
    fl = np.floor(a)
    q = (np.sign(v) * (fl + np.floor(2 * (a - fl)))).astype(np.int8)
    return q, d.astype(np.float16).astype(np.float32)


# ----------------------------------------------------------------------------- model file
@dataclass
class TensorRec:
    name: str
    ne: tuple
    type: int
    raw: np.ndarray


class GGUFFile:
    """Reads tensors and KV fields of a GGUF through gguf-py's reader (test infrastructure)."""

    def __init__(self, path: str):
        if gguf is None:
            raise RuntimeError("gguf-py is required by the oracle")
        self.path = path
        r = gguf.GGUFReader(path)
        self.fields = {}
        for k, f in r.fields.items():
            self.fields[k] = f
        self.tensors = {}
        for t in r.tensors:
            ne = tuple(int(x) for x in t.shape)
            self.tensors[t.name] = TensorRec(t.name, ne, int(t.tensor_type), np.asarray(t.data).view(np.uint8).reshape(-1))
        self._cache = {}

    def kv(self, key, default=None):
        f = self.fields.get(key)
        if f is None:
            return default
        types = [int(x) for x in f.types]
        if types[0] == 8:  # string
            return bytes(f.parts[f.data[0]]).decode("utf-8")
        if types[0] == 9:  # array
            if len(types) > 1 and types[1] == 8:
                return [bytes(f.parts[i]).decode("utf-8") for i in f.data]
            return [int(f.parts[i][0]) for i in f.data]
        v = f.parts[f.data[0]][0]
        return float(v) if types[0] in (6, 12) else int(v)

    def has(self, name):
        return name in self.tensors

    def weight(self, name) -> np.ndarray:
        """Dequantised f32 tensor shaped [ne_{n-1}, ..., ne_0] (row-major rows of ne0)."""
        if name in self._cache:
            return self._cache[name]
        t = self.tensors[name]
        n = int(np.prod(t.ne))
        if t.type == F32:
            w = t.raw[: n * 4].view(np.float32).copy()
        elif t.type == F16:
            w = t.raw[: n * 2].view(np.float16).astype(np.float32)
        elif t.type == Q8_0:
            w = dequant_q8_0(t.raw, n)
        elif t.type == Q4_K:
            w = dequant_q4_k(t.raw, n)
        else:
            raise ValueError(f"unsupported tensor type {t.type} for {name}")
        w = w.reshape(tuple(reversed(t.ne)))
        self._cache[name] = w
        return w


# ----------------------------------------------------------------------------- config
@dataclass
class Config:
    """Keys and defaults of src/config.cpp:6-102 (only what the generation path reads)."""
    hidden: int = 2048
    nc: int = 16
    vs: int = 2051
    cb_size: int = 2048
    bb_eos: int = 2051
    cb_eos: int = 0
    max_new_tokens: int = 750
    temperature: float = 0.9
    top_k: int = 50
    top_p: float = 1.0
    rep: float = 1.1
    depth_temperature: float = 0.9
    depth_top_k: int = 50
    depth_top_p: float = 1.0
    te: dict = field(default_factory=dict)
    bb: dict = field(default_factory=dict)
    dd: dict = field(default_factory=dict)
    voc: dict = field(default_factory=dict)
    codec: dict = field(default_factory=dict)


def parse_config(g: GGUFFile) -> Config:
    c = Config()
    c.hidden = g.kv("breeze.hidden_size", 2048)
    c.nc = g.kv("breeze.num_codebooks", 16)
    c.vs = g.kv("breeze.audio_vocab_size", 2051)
    c.cb_size = g.kv("breeze.codec_codebook_size", 2048)
    c.bb_eos = g.kv("breeze.backbone_eos_token_id", 2051)
    c.cb_eos = g.kv("breeze.codebook_eos_token_id", 0)
    c.max_new_tokens = g.kv("breeze.max_new_tokens", 750)
    c.temperature = g.kv("breeze.temperature", 0.9)
    c.top_k = g.kv("breeze.top_k", 50)
    c.top_p = g.kv("breeze.top_p", 1.0)
    c.rep = g.kv("breeze.repetition_penalty", 1.1)
    c.depth_temperature = g.kv("breeze.depth_temperature", 0.9)
    c.depth_top_k = g.kv("breeze.depth_top_k", 50)
    c.depth_top_p = g.kv("breeze.depth_top_p", 1.0)
    c.te = dict(hidden=g.kv("breeze.te.hidden_size", 1152), n_layer=g.kv("breeze.te.block_count", 26),
                n_head=g.kv("breeze.te.head_count", 4), n_kv=g.kv("breeze.te.head_count_kv", 1),
                hd=g.kv("breeze.te.head_dim", 256), ffn=g.kv("breeze.te.feed_forward_length", 6912),
                eps=g.kv("breeze.te.rms_eps", 1e-6), theta_full=g.kv("breeze.te.rope_theta_full", 1e6),
                fscale_full=g.kv("breeze.te.rope_freq_scale_full", 0.125),
                theta_sliding=g.kv("breeze.te.rope_theta_sliding", 10000.0),
                window=g.kv("breeze.te.sliding_window", 512),
                qpas=g.kv("breeze.te.query_pre_attn_scalar", 256.0),
                embed_scale=g.kv("breeze.te.embed_scale", 1.0),
                is_full=g.kv("breeze.te.layer_is_full", []) or [])
    c.bb = dict(hidden=g.kv("breeze.bb.hidden_size", 2048), n_layer=g.kv("breeze.bb.block_count", 28),
                n_head=g.kv("breeze.bb.head_count", 16), n_kv=g.kv("breeze.bb.head_count_kv", 8),
                hd=g.kv("breeze.bb.head_dim", 128), ffn=g.kv("breeze.bb.feed_forward_length", 6144),
                eps=g.kv("breeze.bb.rms_eps", 1e-6), theta=g.kv("breeze.bb.rope_theta", 1e6))
    c.dd = dict(hidden=g.kv("breeze.dd.hidden_size", 1024), n_layer=g.kv("breeze.dd.block_count", 12),
                n_head=g.kv("breeze.dd.head_count", 8), n_kv=g.kv("breeze.dd.head_count_kv", 2),
                hd=g.kv("breeze.dd.head_dim", 128), ffn=g.kv("breeze.dd.feed_forward_length", 8192),
                eps=g.kv("breeze.dd.rms_eps", 1e-5), theta=g.kv("breeze.dd.rope_theta", 500000.0),
                factor=g.kv("breeze.dd.rope_factor", 32.0),
                high=g.kv("breeze.dd.rope_high_freq_factor", 0.0078125),
                low=g.kv("breeze.dd.rope_low_freq_factor", 0.001953125),
                orig=g.kv("breeze.dd.rope_orig_ctx", 16))
    # src/config.cpp:84-99
    c.voc = dict(hidden=g.kv("breeze.codec.dec.hidden_size", 512), n_layer=g.kv("breeze.codec.dec.block_count", 8),
                 n_head=g.kv("breeze.codec.dec.head_count", 16), n_kv=g.kv("breeze.codec.dec.head_count_kv", 16),
                 hd=g.kv("breeze.codec.dec.head_dim", 64), ffn=g.kv("breeze.codec.dec.feed_forward_length", 1024),
                 eps=g.kv("breeze.codec.dec.rms_eps", 1e-5), theta=g.kv("breeze.codec.dec.rope_theta", 10000.0),
                 window=g.kv("breeze.codec.dec.sliding_window", 72),
                 rates=list(g.kv("breeze.codec.dec.upsample_rates", []) or [8, 5, 4, 3]),
                 ratios=list(g.kv("breeze.codec.dec.upsampling_ratios", []) or [2, 2]))
    # src/config.cpp:68-81 (the codec encoder)
    c.codec = dict(hidden=g.kv("breeze.codec.hidden_size", 512), n_layer=g.kv("breeze.codec.block_count", 8),
                   n_head=g.kv("breeze.codec.head_count", 8), hd=g.kv("breeze.codec.head_dim", 64),
                   ffn=g.kv("breeze.codec.feed_forward_length", 2048), theta=g.kv("breeze.codec.rope_theta", 10000.0),
                   window=g.kv("breeze.codec.sliding_window", 250), nf=g.kv("breeze.codec.num_filters", 64),
                   dim=g.kv("breeze.codec.codebook_dim", 256), n_sem=g.kv("breeze.codec.num_semantic", 1),
                   eps=g.kv("breeze.codec.layer_norm_eps", 1e-5),
                   ratios=list(g.kv("breeze.codec.upsampling_ratios", []) or [8, 6, 5, 4]))
    return c


# ----------------------------------------------------------------------------- tokenizer
_META = "▁"


class Tokenizer:
    """SentencePiece-style BPE of src/tokenizer.cpp:19-124 (longest special first, byte
    fallback, rank-ordered merges)."""

    def __init__(self, g: GGUFFile):
        self.id_to_token = g.kv("tokenizer.ggml.tokens")
        types = g.kv("tokenizer.ggml.token_type", []) or []
        self.token_to_id = {}
        self.byte_to_id = {}
        self.specials = {}
        for i, t in enumerate(self.id_to_token):
            self.token_to_id[t] = i
            if len(t) == 6 and t.startswith("<0x") and t.endswith(">"):
                self.byte_to_id[int(t[3:5], 16)] = i
            if i < len(types) and types[i] in (3, 4):
                self.specials[t] = i
        self.special_lens = sorted({len(s) for s in self.specials}, reverse=True)
        merges = g.kv("tokenizer.ggml.merges", []) or []
        self.merge_rank = {m: i for i, m in enumerate(merges)}
        self.bos = g.kv("tokenizer.ggml.bos_token_id", 2)
        self.unk = g.kv("tokenizer.ggml.unknown_token_id", 3)

    def _bpe(self, word: str, out: list):
        syms = []
        for ch in word:
            if ch in self.token_to_id:
                syms.append(ch)
            else:
                for b in ch.encode("utf-8"):
                    syms.append(self.id_to_token[self.byte_to_id[b]] if b in self.byte_to_id else chr(b))
        while len(syms) > 1:
            best, best_i = None, -1
            for i in range(len(syms) - 1):
                r = self.merge_rank.get(syms[i] + " " + syms[i + 1])
                if r is not None and (best is None or r < best):
                    best, best_i = r, i
            if best_i < 0:
                break
            syms[best_i] += syms[best_i + 1]
            del syms[best_i + 1]
        for s in syms:
            if s in self.token_to_id:
                out.append(self.token_to_id[s])
            else:
                for b in s.encode("utf-8"):
                    out.append(self.byte_to_id.get(b, self.unk))

    def encode(self, text: str, add_bos=True) -> list:
        out = [self.bos] if add_bos else []
        normal = []
        i = 0
        while i < len(text):
            hit = None
            for L in self.special_lens:
                s = text[i:i + L]
                if len(s) == L and s in self.specials:
                    hit = s
                    break
            if hit is not None:
                if normal:
                    self._bpe("".join(normal).replace(" ", _META), out)
                    normal = []
                out.append(self.specials[hit])
                i += len(hit)
            else:
                normal.append(text[i])
                i += 1
        if normal:
            self._bpe("".join(normal).replace(" ", _META), out)
        return out


# ----------------------------------------------------------------------------- primitives
def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """ggml_rms_norm (mean of squares in double) followed by ggml_mul with the weight
    (src/common.cpp:127-129)."""
    x = x.astype(np.float32)
    ms = (x.astype(np.float64) ** 2).mean(axis=-1, keepdims=True)
    scale = (np.float32(1.0) / np.sqrt((ms + eps).astype(np.float32))).astype(np.float32)
    return ((x * scale).astype(np.float32) * w.astype(np.float32)).astype(np.float32)


def linear(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """ggml_mul_mat(w, x) evaluated exactly: f32 activations times the dequantised weight
    w [out, in] (src/common.cpp:136-138)."""
    return (x.astype(np.float32) @ w.T).astype(np.float32)


def linear_q8(x: np.ndarray, raw: np.ndarray, out_dim: int, in_dim: int, row0: int = 0) -> np.ndarray:
    """ggml-mode linear on raw Q8_0 weight bytes: activations quantised to Q8_0 per block,
    integer block dots, f32 accumulation of sumi * (dw * dx) (ggml vec_dot_q8_0_q8_0)."""
    q, d = quant_q8_0_rows(x.astype(np.float32))
    nb = in_dim // 32
    b = raw[row0 * nb * 34:(row0 + out_dim) * nb * 34].reshape(out_dim, nb, 34)
    wd = b[:, :, :2].copy().view(np.float16).astype(np.float32)[:, :, 0]   # [out, nb]
    wq = b[:, :, 2:].copy().view(np.int8).astype(np.int32)                  # [out, nb, 32]
    qi = q.astype(np.int32)
    out = np.zeros((x.shape[0], out_dim), np.float32)
    for blk in range(nb):
        sumi = qi[:, blk, :] @ wq[:, blk, :].T                              # [n, out] exact ints
        out += sumi.astype(np.float32) * (wd[None, :, blk] * d[:, blk, 0][:, None]).astype(np.float32)
    return out


def silu(x):
    x = x.astype(np.float32)
    return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def gelu_tanh(x):
    x = x.astype(np.float32)
    c = np.float32(math.sqrt(2.0 / math.pi))
    return (np.float32(0.5) * x * (np.float32(1.0) + np.tanh(c * x * (np.float32(1.0) + np.float32(0.044715) * x * x)))).astype(np.float32)


def rope_cos_sin(pos: np.ndarray, n_dims: int, base: float, freq_scale: float = 1.0, ff=None):
    """ggml rope cache for NEOX mode: theta_i = pos * theta_scale^i built by repeated f32
    multiplication, theta_scale = powf(base, -2/n_dims), divided by the optional frequency
    factor and multiplied by freq_scale (ext_factor 0)."""
    ts = np.float32(_LIBM.powf(ctypes.c_float(base), ctypes.c_float(-2.0 / n_dims)))
    half = n_dims // 2
    theta = pos.astype(np.float32).copy()
    cos = np.empty((pos.shape[0], half), np.float32)
    sin = np.empty((pos.shape[0], half), np.float32)
    for i in range(half):
        t = theta if ff is None else (theta / np.float32(ff[i])).astype(np.float32)
        t = (np.float32(freq_scale) * t).astype(np.float32)
        cos[:, i] = np.cos(t)
        sin[:, i] = np.sin(t)
        theta = (theta * ts).astype(np.float32)
    return cos, sin


def rope_neox(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """x [T, H, hd]; rotate pairs (i, i + hd/2) with the per-token cos/sin [T, hd/2]."""
    half = x.shape[-1] // 2
    x0, x1 = x[..., :half], x[..., half:]
    c, s = cos[:, None, :], sin[:, None, :]
    return np.concatenate([x0 * c - x1 * s, x0 * s + x1 * c], axis=-1).astype(np.float32)


def llama3_freq_factors(dd: dict) -> np.ndarray:
    """src/depth_decoder.cpp:10-29."""
    hd = dd["hd"]
    half = hd // 2
    ff = np.ones(half, np.float32)
    pi = np.float32(3.14159265358979323846)
    low_wl = np.float32(dd["orig"]) / np.float32(dd["low"])
    high_wl = np.float32(dd["orig"]) / np.float32(dd["high"])
    for i in range(half):
        freq = np.float32(_LIBM.powf(ctypes.c_float(dd["theta"]), ctypes.c_float(np.float32(-2.0 * i) / np.float32(hd))))
        wavelen = np.float32(2.0) * pi / freq
        if wavelen > low_wl:
            ff[i] = dd["factor"]
        elif wavelen < high_wl:
            ff[i] = 1.0
        else:
            smooth = (np.float32(dd["orig"]) / wavelen - np.float32(dd["low"])) / (np.float32(dd["high"]) - np.float32(dd["low"]))
            ff[i] = np.float32(1.0) / ((np.float32(1.0) - smooth) / np.float32(dd["factor"]) + smooth)
    return ff


def attention(q, k, v, scale, mask=None):
    """softmax(K.q * scale + mask) . V with GQA broadcast (src/common.cpp:147-160).
    q [Tq, H, hd], k/v [Tk, Hkv, hd] -> [Tq, H*hd]."""
    Tq, H, hd = q.shape
    Hkv = k.shape[1]
    g = H // Hkv
    out = np.empty((Tq, H, hd), np.float32)
    for h in range(H):
        kh = k[:, h // g, :]
        vh = v[:, h // g, :]
        s = (q[:, h, :] @ kh.T).astype(np.float32) * np.float32(scale)
        if mask is not None:
            s = s + mask
        m = s.max(axis=1, keepdims=True)
        e = np.exp((s - m).astype(np.float32))
        p = (e / e.sum(axis=1, keepdims=True, dtype=np.float64)).astype(np.float32)
        out[:, h, :] = p @ vh
    return out.reshape(Tq, H * hd)


# ----------------------------------------------------------------------------- model
class Model:
    def __init__(self, path: str, mode: str = "exact"):
        self.g = GGUFFile(path)
        self.cfg = parse_config(self.g)
        self.tok = Tokenizer(self.g)
        self.mode = mode
        self.dd_ff = llama3_freq_factors(self.cfg.dd)

    def _file(self, name) -> "GGUFFile":
        dd = getattr(self, "dd_file", None)
        return dd if dd is not None and name.startswith("dd.") else self.g

    def w(self, name):
        return self._file(name).weight(name)

    def with_depth_override(self, path: str) -> "Model":
        """This model with its dd.* tensors read from another GGUF: the Q4_K depth override of
        src/c_api.cpp:532-566 (BreezeModel::w routes dd.* to dd_override, src/model.h:26-43)."""
        import copy
        m = copy.copy(self)
        m.dd_file = GGUFFile(path)
        return m

    def lin(self, x, name, sub: int = -1):
        """Quantised linear; `sub` selects one [rows, in] slice of a 3-D weight."""
        w = self.w(name)
        if sub >= 0:
            w = w[sub]
        w = w.reshape(-1, w.shape[-1])
        t = self._file(name).tensors[name]
        if self.mode == "ggml" and t.type == Q8_0:
            return linear_q8(x, t.raw, w.shape[0], w.shape[1], max(sub, 0) * w.shape[0])
        return linear(x, w)

    def embed_rows(self, name, idx) -> np.ndarray:
        w = self.w(name)
        return w.reshape(-1, w.shape[-1])[np.asarray(idx, np.int64)].astype(np.float32)

    # ------------------------------------------------------------------ text encoder
    def text_encoder(self, tokens) -> np.ndarray:
        """src/text_encoder.cpp:8-72 (Gemma-style bidirectional encoder + projection)."""
        c = self.cfg.te
        T = len(tokens)
        x = self.embed_rows("te.token_embd.weight", tokens) * np.float32(c["embed_scale"])
        pos = np.arange(T)
        mfull = np.zeros((T, T), np.float32)
        mwin = np.zeros((T, T), np.float32)
        if c["window"] > 0:
            left, right = (c["window"] + 1) // 2, c["window"] // 2 + 1
            qi = np.arange(T)[:, None]
            ki = np.arange(T)[None, :]
            dist = qi - ki
            ok = ((dist >= 0) & (dist < left)) | ((dist < 0) & (-dist < right))
            mwin = np.where(ok, 0.0, -np.inf).astype(np.float32)
        scale = 1.0 / math.sqrt(c["qpas"])
        for il in range(c["n_layer"]):
            p = f"te.blk.{il}"
            full = il < len(c["is_full"]) and c["is_full"][il] != 0
            theta = c["theta_full"] if full else c["theta_sliding"]
            fs = c["fscale_full"] if full else 1.0
            cos, sin = rope_cos_sin(pos, c["hd"], theta, fs)
            res = x
            h = rms_norm(x, self.w(p + ".attn_norm.weight"), c["eps"])
            q = self.lin(h, p + ".attn_q.weight").reshape(T, c["n_head"], c["hd"])
            k = self.lin(h, p + ".attn_k.weight").reshape(T, c["n_kv"], c["hd"])
            v = self.lin(h, p + ".attn_v.weight").reshape(T, c["n_kv"], c["hd"])
            q = rms_norm(q, self.w(p + ".attn_q_norm.weight"), c["eps"])
            k = rms_norm(k, self.w(p + ".attn_k_norm.weight"), c["eps"])
            q = rope_neox(q, cos, sin)
            k = rope_neox(k, cos, sin)
            a = attention(q, k, v, scale, mfull if full else mwin)
            a = self.lin(a, p + ".attn_output.weight")
            a = rms_norm(a, self.w(p + ".post_attn_norm.weight"), c["eps"])
            x = (res + a).astype(np.float32)
            res = x
            h = rms_norm(x, self.w(p + ".ffn_norm.weight"), c["eps"])
            gt = gelu_tanh(self.lin(h, p + ".ffn_gate.weight"))
            up = self.lin(h, p + ".ffn_up.weight")
            h = self.lin((gt * up).astype(np.float32), p + ".ffn_down.weight")
            h = rms_norm(h, self.w(p + ".post_ffn_norm.weight"), c["eps"])
            x = (res + h).astype(np.float32)
        x = rms_norm(x, self.w("te.output_norm.weight"), c["eps"])
        return self.lin(x, "te.proj.weight")

    # ------------------------------------------------------------------ audio embedding
    def audio_embed(self, frames: np.ndarray) -> np.ndarray:
        """Sum over codebooks of audio_embd rows code + cb*vs (src/backbone.cpp:223-246).
        frames [F, nc] int -> [F, hidden]."""
        frames = np.asarray(frames, np.int64)
        nc, vs = frames.shape[1], self.cfg.vs
        idx = frames + (np.arange(nc) * vs)[None, :]
        rows = self.embed_rows("audio_embd.weight", idx.reshape(-1)).reshape(frames.shape[0], nc, -1)
        acc = np.zeros((frames.shape[0], rows.shape[2]), np.float32)
        for cb in range(nc):   # ggml_sum_rows accumulates in order
            acc = (acc + rows[:, cb, :]).astype(np.float32)
        return acc

    # ------------------------------------------------------------------ backbone
    def bb_layer_tokens(self, st: "BBState", x: np.ndarray, il: int, pos: np.ndarray):
        """One pre-norm block over tokens appended at `pos` (src/backbone.cpp:248-276)."""
        c = self.cfg.bb
        p = f"bb.blk.{il}"
        T = x.shape[0]
        res = x
        h = rms_norm(x, self.w(p + ".attn_norm.weight"), c["eps"])
        q = self.lin(h, p + ".attn_q.weight").reshape(T, c["n_head"], c["hd"])
        k = self.lin(h, p + ".attn_k.weight").reshape(T, c["n_kv"], c["hd"])
        v = self.lin(h, p + ".attn_v.weight").reshape(T, c["n_kv"], c["hd"])
        q = rms_norm(q, self.w(p + ".attn_q_norm.weight"), c["eps"])
        k = rms_norm(k, self.w(p + ".attn_k_norm.weight"), c["eps"])
        cos, sin = rope_cos_sin(pos, c["hd"], c["theta"])
        q = rope_neox(q, cos, sin)
        k = rope_neox(k, cos, sin)
        st.k[il][pos[0]:pos[0] + T] = k
        st.v[il][pos[0]:pos[0] + T] = v
        L = pos[0] + T
        qi = pos[:, None]
        ki = np.arange(L)[None, :]
        mask = np.where(ki <= qi, 0.0, -np.inf).astype(np.float32)
        a = attention(q, st.k[il][:L], st.v[il][:L], 1.0 / math.sqrt(c["hd"]), mask)
        x = (res + self.lin(a, p + ".attn_output.weight")).astype(np.float32)
        res = x
        h = rms_norm(x, self.w(p + ".ffn_norm.weight"), c["eps"])
        g = silu(self.lin(h, p + ".ffn_gate.weight"))
        u = self.lin(h, p + ".ffn_up.weight")
        return (res + self.lin((g * u).astype(np.float32), p + ".ffn_down.weight")).astype(np.float32)

    def backbone_run(self, st: "BBState", embeds: np.ndarray):
        """Prefill or single-token run; returns (last normed hidden, logits)
        (src/backbone.cpp:68-96)."""
        c = self.cfg.bb
        T = embeds.shape[0]
        pos = np.arange(st.pos, st.pos + T)
        x = embeds.astype(np.float32)
        for il in range(c["n_layer"]):
            x = self.bb_layer_tokens(st, x, il, pos)
        x = rms_norm(x, self.w("bb.output_norm.weight"), c["eps"])
        last = x[-1:]
        logits = self.lin(last, "bb.lm_head.weight")
        st.pos += T
        return last[0], logits[0]

    def backbone_step_batched(self, states: list, embeds: np.ndarray):
        """One token per session, each attending to its own cache (src/backbone.cpp:98-179):
        linears batched over sessions, attention per session over its cache."""
        c = self.cfg.bb
        N = embeds.shape[0]
        x = embeds.astype(np.float32)
        scale = 1.0 / math.sqrt(c["hd"])
        pos = np.array([st.pos for st in states])
        for il in range(c["n_layer"]):
            p = f"bb.blk.{il}"
            res = x
            h = rms_norm(x, self.w(p + ".attn_norm.weight"), c["eps"])
            q = self.lin(h, p + ".attn_q.weight").reshape(N, c["n_head"], c["hd"])
            k = self.lin(h, p + ".attn_k.weight").reshape(N, c["n_kv"], c["hd"])
            v = self.lin(h, p + ".attn_v.weight").reshape(N, c["n_kv"], c["hd"])
            q = rms_norm(q, self.w(p + ".attn_q_norm.weight"), c["eps"])
            k = rms_norm(k, self.w(p + ".attn_k_norm.weight"), c["eps"])
            a = np.empty((N, c["n_head"] * c["hd"]), np.float32)
            for i, st in enumerate(states):
                cos, sin = rope_cos_sin(pos[i:i + 1], c["hd"], c["theta"])
                qi = rope_neox(q[i:i + 1], cos, sin)
                ki = rope_neox(k[i:i + 1], cos, sin)
                st.k[il][pos[i]] = ki[0]
                st.v[il][pos[i]] = v[i]
                L = pos[i] + 1
                a[i] = attention(qi, st.k[il][:L], st.v[il][:L], scale)[0]
            x = (res + self.lin(a, p + ".attn_output.weight")).astype(np.float32)
            res = x
            h = rms_norm(x, self.w(p + ".ffn_norm.weight"), c["eps"])
            g = silu(self.lin(h, p + ".ffn_gate.weight"))
            u = self.lin(h, p + ".ffn_up.weight")
            x = (res + self.lin((g * u).astype(np.float32), p + ".ffn_down.weight")).astype(np.float32)
        x = rms_norm(x, self.w("bb.output_norm.weight"), c["eps"])
        logits = self.lin(x, "bb.lm_head.weight")
        for st in states:
            st.pos += 1
        return x, logits

    # ------------------------------------------------------------------ depth decoder
    def depth_logits_chain(self, hiddens: np.ndarray, cb0: np.ndarray, forced=None):
        """Unified batched depth decode (src/depth_decoder.cpp:249-365): position 0 is the
        backbone hidden, position 1 the cb0 embedding, then one position per codebook; each
        sub-step's logits come from head j-1 and its argmax feeds the next embedding.
        `forced` [N, nc-1] replaces the argmax as the next input (teacher forcing).
        Returns (codes [N, nc-1], logits [N, nc-1, vs])."""
        N = hiddens.shape[0]
        codes = np.zeros((N, self.cfg.nc - 1), np.int64)

        def choose(j, lg):
            codes[:, j - 1] = np.argmax(lg, axis=1)
            return codes[:, j - 1] if forced is None else np.asarray(forced)[:, j - 1]

        logits_all = self.depth_chain(hiddens, cb0, choose)
        return codes, logits_all

    def depth_chain(self, hiddens: np.ndarray, cb0: np.ndarray, choose):
        """The depth decode of src/depth_decoder.cpp:89-128 over N rows (branches), with the code
        of each sub-step j = 1..nc-1 chosen by choose(j, logits [N, vs]) -> codes [N] (fed to
        the next sub-step). Returns the logits [N, nc-1, vs]."""
        c = self.cfg.dd
        nc, vs = self.cfg.nc, self.cfg.vs
        N = hiddens.shape[0]
        kc = np.zeros((c["n_layer"], N, nc + 1, c["n_kv"], c["hd"]), np.float32)
        vc = np.zeros_like(kc)
        logits_all = np.zeros((N, nc - 1, vs), np.float32)
        scale = 1.0 / math.sqrt(c["hd"])

        def run_layers(x, start, n_pos):
            # x [N, n_pos, dd_hidden] for positions start..start+n_pos-1
            pos = np.arange(start, start + n_pos)
            cos, sin = rope_cos_sin(pos, c["hd"], c["theta"], 1.0, self.dd_ff)
            for il in range(c["n_layer"]):
                p = f"dd.blk.{il}"
                res = x
                flat = x.reshape(N * n_pos, -1)
                h = rms_norm(flat, self.w(p + ".attn_norm.weight"), c["eps"])
                q = self.lin(h, p + ".attn_q.weight").reshape(N, n_pos, c["n_head"], c["hd"])
                k = self.lin(h, p + ".attn_k.weight").reshape(N, n_pos, c["n_kv"], c["hd"])
                v = self.lin(h, p + ".attn_v.weight").reshape(N, n_pos, c["n_kv"], c["hd"])
                a = np.empty((N, n_pos, c["n_head"] * c["hd"]), np.float32)
                for s in range(N):
                    qs_ = rope_neox(q[s], cos, sin)
                    ks_ = rope_neox(k[s], cos, sin)
                    kc[il, s, start:start + n_pos] = ks_
                    vc[il, s, start:start + n_pos] = v[s]
                    L = start + n_pos
                    mask = np.where(np.arange(L)[None, :] <= pos[:, None], 0.0, -np.inf).astype(np.float32)
                    a[s] = attention(qs_, kc[il, s, :L], vc[il, s, :L], scale, mask)
                o = self.lin(a.reshape(N * n_pos, -1), p + ".attn_output.weight").reshape(x.shape)
                x = (res + o).astype(np.float32)
                res = x
                flat = x.reshape(N * n_pos, -1)
                h = rms_norm(flat, self.w(p + ".ffn_norm.weight"), c["eps"])
                gt = silu(self.lin(h, p + ".ffn_gate.weight"))
                up = self.lin(h, p + ".ffn_up.weight")
                d = self.lin((gt * up).astype(np.float32), p + ".ffn_down.weight").reshape(x.shape)
                x = (res + d).astype(np.float32)
            return x

        e0 = self.embed_rows("audio_embd.weight", cb0)
        inp = np.stack([hiddens.astype(np.float32), e0], axis=1)       # [N, 2, hidden]
        x = self.lin(inp.reshape(2 * N, -1), "dd.in_proj.weight").reshape(N, 2, -1)
        x = run_layers(x, 0, 2)
        last = rms_norm(x[:, 1], self.w("dd.output_norm.weight"), c["eps"])
        lg = self.lin(last, "dd.codebooks_head.weight", 0)
        logits_all[:, 0] = lg
        prev = np.asarray(choose(1, lg), np.int64)
        for j in range(2, nc):
            e = self.embed_rows("audio_embd.weight", (j - 1) * vs + prev)
            x = self.lin(e, "dd.in_proj.weight").reshape(N, 1, -1)
            x = run_layers(x, j, 1)
            last = rms_norm(x[:, 0], self.w("dd.output_norm.weight"), c["eps"])
            lg = self.lin(last, "dd.codebooks_head.weight", j - 1)
            logits_all[:, j - 1] = lg
            prev = np.asarray(choose(j, lg), np.int64)
        return logits_all


@dataclass
class BBState:
    """Per-session backbone KV (f32 like the reference KVCache, common.cpp:48-63)."""
    k: list
    v: list
    pos: int = 0

    @staticmethod
    def new(m: Model, max_seq: int) -> "BBState":
        c = m.cfg.bb
        return BBState([np.zeros((max_seq, c["n_kv"], c["hd"]), np.float32) for _ in range(c["n_layer"])],
                       [np.zeros((max_seq, c["n_kv"], c["hd"]), np.float32) for _ in range(c["n_layer"])])


# ----------------------------------------------------------------------------- sampling
_PH_M0, _PH_M1 = 0xD2511F53, 0xCD9E8D57
_PH_W0, _PH_W1 = 0x9E3779B9, 0xBB67AE85
PHILOX_KEY_HI = 0x42524545


def philox4x32_10(ctr, key):
    """Philox4x32-10 (Salmon et al., SC'11): 10 rounds of the published round function."""
    c0, c1, c2, c3 = [x & 0xFFFFFFFF for x in ctr]
    k0, k1 = [x & 0xFFFFFFFF for x in key]
    for _ in range(10):
        p0 = _PH_M0 * c0
        p1 = _PH_M1 * c2
        hi0, lo0 = p0 >> 32, p0 & 0xFFFFFFFF
        hi1, lo1 = p1 >> 32, p1 & 0xFFFFFFFF
        c0, c1, c2, c3 = (hi1 ^ c1 ^ k0) & 0xFFFFFFFF, lo1, (hi0 ^ c3 ^ k1) & 0xFFFFFFFF, lo0
        k0 = (k0 + _PH_W0) & 0xFFFFFFFF
        k1 = (k1 + _PH_W1) & 0xFFFFFFFF
    return c0, c1, c2, c3


def philox_uniform(seed: int, draw: int) -> np.float32:
    """u in [0, 1) from the top 24 bits of the first Philox word for (seed, draw index)."""
    w = philox4x32_10((draw & 0xFFFFFFFF, (draw >> 32) & 0xFFFFFFFF, 0, 0), (seed & 0xFFFFFFFF, PHILOX_KEY_HI))
    return np.float32((w[0] >> 8) * (1.0 / 16777216.0))


def apply_penalties(logits: np.ndarray, rep: float, hist_counts, suppress_lo: int, suppress_hi: int) -> np.ndarray:
    """Suppression then repetition penalty, applied once per history occurrence
    (src/sampling.cpp:13-23)."""
    l = logits.astype(np.float32).copy()
    n = l.shape[0]
    l[max(0, suppress_lo):min(n, suppress_hi)] = -np.inf
    if hist_counts is not None and rep != 1.0:
        r = np.float32(rep)
        for t, cnt in hist_counts.items():
            if t < 0 or t >= n:
                continue
            for _ in range(cnt):
                l[t] = l[t] / r if l[t] > 0 else l[t] * r
    return l


def sample_philox(logits, temp, top_k, top_p, u: np.float32) -> int:
    """The engine's sampler: top-k by (logit desc, index asc), softmax at temperature in f32,
    optional top-p cut (src/sampling.cpp:25-56), then inverse-CDF with a Philox uniform in
    place of std::discrete_distribution."""
    n = logits.shape[0]
    t = np.float32(temp if temp > 0 else 1.0)
    keep = top_k if 0 < top_k < n else n
    order = np.lexsort((np.arange(n), -logits.astype(np.float64)))[:keep]
    maxl = logits[order[0]]
    p = np.exp(((logits[order] - maxl) / t).astype(np.float32)).astype(np.float32)
    s = np.float32(0)
    for v in p:
        s = np.float32(s + v)
    probs = (p / s).astype(np.float32)
    if top_p < 1.0:
        cum = np.float32(0)
        cut = keep
        for i, v in enumerate(probs):
            cum = np.float32(cum + v)
            if cum >= np.float32(top_p):
                cut = i + 1
                break
        probs = probs[:cut]
        order = order[:cut]
        s2 = np.float32(0)
        for v in probs:
            s2 = np.float32(s2 + v)
        probs = (probs / s2).astype(np.float32)
    cdf = np.empty_like(probs)
    acc = np.float32(0)
    for i, v in enumerate(probs):
        acc = np.float32(acc + v)
        cdf[i] = acc
    r = np.float32(u * cdf[-1])
    for i in range(len(cdf)):
        if r < cdf[i]:
            return int(order[i])
    return int(order[-1])


def sample_margin(logits, temp, top_k, u: np.float32) -> float:
    """Distance of the sampler's inverse-CDF target from the nearest CDF boundary, as a
    fraction of the total mass: how far a logit perturbation must move the CDF to change
    the draw (used to recognise numerical ties in parity tests)."""
    n = logits.shape[0]
    keep = top_k if 0 < top_k < n else n
    order = np.lexsort((np.arange(n), -logits.astype(np.float64)))[:keep]
    t = np.float64(temp if temp > 0 else 1.0)
    p = np.exp((logits[order].astype(np.float64) - logits[order[0]]) / t)
    cdf = np.cumsum(p) / p.sum()
    return float(np.min(np.abs(cdf - float(u))))


def sample_reachable(logits, temp, top_k, u: np.float32, token: int, eps: float) -> bool:
    """Whether the sampler (same top-k, temperature and uniform u) can return `token` for some
    logits within +-eps of `logits`. A perturbation of at most eps scales every unnormalised
    weight exp(l/T) by a factor in [e^(-eps/T), e^(eps/T)], so each CDF boundary moves by at most
    e^(2 eps/T) - 1; the token must also be able to enter the top-k set."""
    n = logits.shape[0]
    keep = top_k if 0 < top_k < n else n
    order = np.lexsort((np.arange(n), -logits.astype(np.float64)))
    t = np.float64(temp if temp > 0 else 1.0)
    delta = float(np.expm1(2.0 * eps / t))
    rank = int(np.nonzero(order == token)[0][0])
    if rank >= keep:
        # outside the top-k: it can only displace the k-th entry, at the top of the CDF
        if logits[token] < logits[order[keep - 1]] - 2 * eps:
            return False
        return float(u) >= 1.0 - delta - float(np.exp((logits[token] - logits[order[0]]) / t))
    top = order[:keep]
    p = np.exp((logits[top].astype(np.float64) - logits[top[0]]) / t)
    cdf = np.cumsum(p) / p.sum()
    lo = 0.0 if rank == 0 else cdf[rank - 1]
    hi = cdf[rank]
    return lo - delta <= float(u) <= hi + delta


class PhiloxStream:
    """Per-session sampler state: seed (key) and draw counter; reseeding resets the counter,
    mirroring std::mt19937::seed in src/c_api.cpp:343, 631, 816."""

    def __init__(self, seed: int):
        self.seed(seed)

    def seed(self, s: int):
        self.key = s & 0xFFFFFFFF
        self.draw = 0

    def next_uniform(self) -> np.float32:
        u = philox_uniform(self.key, self.draw)
        self.draw += 1
        return u


# ----------------------------------------------------------------------------- sessions
@dataclass
class SamplerParams:
    """src/sampling.h SampleParams for cb0 plus the depth sampler (src/depth_decoder.cpp:134-140);
    the generator ABI fixes the cb0 part (src/c_api.cpp:343-347)."""
    temp: float = 0.9
    top_k: int = 50
    top_p: float = 1.0
    rep: float = 1.1
    dtemp: float = 0.9
    dtop_k: int = 50
    dtop_p: float = 1.0


@dataclass
class Session:
    sid: int
    st: BBState
    hist: dict
    last_hidden: np.ndarray
    last_cb0: int
    rng: PhiloxStream
    max_tokens: int
    steps_taken: int = 0
    active: bool = True
    cfg: float = 1.0               # guidance scale; != 1 adds the unconditional branch below
    st_u: BBState = None
    last_hidden_u: np.ndarray = None
    sp: SamplerParams = field(default_factory=SamplerParams)
    use_q4: bool = False           # depth codes from the Q4_K override (src/c_api.cpp:570-578)


def combine_logits(lc, lu, scale):
    """src/c_api.cpp:148-155: uncond + scale * (cond - uncond)."""
    if lu is None:
        return lc
    return (lu + np.float32(scale) * (lc - lu).astype(np.float32)).astype(np.float32)


def depth_uniform(key: int, draw: int, j: int) -> np.float32:
    """The engine's depth draw for codebook j: Philox counter (draw, j) under the key, so depth
    draws never collide with the cb0 draws (counter (draw, 0))."""
    return philox_uniform(key, (draw & 0xFFFFFFFF) | (j << 32))


class Generator:
    """Session semantics of the generator C ABI (src/c_api.cpp:325-451, 459-519, 601-949) with
    the engine's Philox sampler, including the two-branch (classifier-free guidance) sessions and
    the sampled depth decode (src/depth_decoder.cpp:130-247)."""

    def __init__(self, model: Model):
        self.m = model
        self.sessions = {}
        self.q4 = None
        # per session: (penalised logits, Philox key, draw index) of its latest cb0 draw
        self.last_cb0_logits = {}

    def load_q4_depth(self, path: str):
        self.q4 = self.m.with_depth_override(path)

    def session_set_q4(self, sid, on: bool) -> int:
        if sid not in self.sessions:
            return -1
        self.sessions[sid].use_q4 = bool(on) and self.q4 is not None
        return 0

    def abi_params(self) -> SamplerParams:
        c = self.m.cfg
        return SamplerParams(0.9, 50, 1.0, 1.1, c.depth_temperature, c.depth_top_k, c.depth_top_p)

    def _sample_cb0(self, sess: Session, logits) -> int:
        c = self.m.cfg
        sp = sess.sp
        l = apply_penalties(logits, sp.rep, sess.hist, c.cb_size, c.vs)
        return sample_philox(l, sp.temp, sp.top_k, sp.top_p, sess.rng.next_uniform())

    def prompt_embeds(self, text, instruction=None, ref_text=None, ref_codes=None, cond=True):
        """src/c_api.cpp:366-396 (cond) and 411-423 (the unconditional branch: no instruction)."""
        m = self.m
        ins = instruction if instruction is not None else "Speak clearly and naturally."
        has_ref = ref_codes is not None and len(ref_codes) > 0 and ref_text
        embs = []
        if has_ref:
            embs.append(m.text_encoder(m.tok.encode("[S0]" + ref_text, True)))
            embs.append(m.audio_embed(np.asarray(ref_codes).reshape(-1, m.cfg.nc)))
            embs.append(m.audio_embed(np.full((1, m.cfg.nc), m.cfg.cb_eos)))
        tail = "[S0]<ins_bos>" + ins + "<ins_eos>" + text if cond else "[S0]" + text
        embs.append(m.text_encoder(m.tok.encode(tail, True)))
        return np.concatenate(embs, axis=0)

    def session_create(self, sid, text, instruction=None, ref_text=None, ref_codes=None,
                       seed=0, max_new_tokens=0, embeds=None, cfg_scale=1.0, params=None,
                       embeds_u=None, clamp_total=True):
        cfg = cfg_scale if cfg_scale > 0 else 1.0
        if embeds is None:
            embeds = self.prompt_embeds(text, instruction, ref_text, ref_codes)
        if cfg != 1.0 and embeds_u is None:
            embeds_u = self.prompt_embeds(text, instruction, ref_text, ref_codes, cond=False)
        est = max_new_tokens
        if est <= 0:
            words = len(text.split())
            est = min(1000, int(math.ceil(words * 1.5)) + 30)
        total = embeds.shape[0]
        if clamp_total:
            avail = 2040 - total
            if est > avail:
                est = max(64, avail)
        st = BBState.new(self.m, total + est + 8)
        h, lg = self.m.backbone_run(st, embeds)
        sess = Session(sid, st, {}, h, -1, PhiloxStream(seed), est, sp=params or self.abi_params())
        alloc = total + est + 8
        lu = None
        if cfg != 1.0:
            sess.cfg = cfg
            sess.st_u = BBState.new(self.m, embeds_u.shape[0] + est + 8)
            sess.last_hidden_u, lu = self.m.backbone_run(sess.st_u, embeds_u)
            alloc += embeds_u.shape[0] + est + 8
        first = combine_logits(lg, lu, sess.cfg)
        self.last_cb0_logits[sid] = (apply_penalties(first, sess.sp.rep, sess.hist, self.m.cfg.cb_size, self.m.cfg.vs),
                                     sess.rng.key, sess.rng.draw)
        cb0 = self._sample_cb0(sess, first)
        sess.hist[cb0] = sess.hist.get(cb0, 0) + 1
        sess.last_cb0 = cb0
        self.sessions[sid] = sess
        return cb0, alloc

    def convert_create(self, sid, text, ref_codes=None, ref_frames=0, ref_text="", cfg_scale=1.5, seed=42, src_T=1):
        """Voice-conversion session (src/generation.cpp:315-345): the conditional prompt carries the
        reference (its text, frames and EOS frame) and no instruction, the unconditional one the
        text alone; depth codes from the top-1 of temperature 0.3 (ConvertOptions)."""
        m = self.m
        embs = [m.text_encoder(m.tok.encode("[S0]" + (ref_text or ""), True))]
        if ref_frames > 0:
            embs.append(m.audio_embed(np.asarray(ref_codes).reshape(-1, m.cfg.nc)[:ref_frames]))
        embs.append(m.audio_embed(np.full((1, m.cfg.nc), m.cfg.cb_eos)))
        embs.append(m.text_encoder(m.tok.encode("[S0]" + text, True)))
        eu = m.text_encoder(m.tok.encode("[S0]" + text, True)) if cfg_scale != 1.0 else None
        return self.session_create(sid, text, embeds=np.concatenate(embs), embeds_u=eu, cfg_scale=cfg_scale,
                                   seed=seed, max_new_tokens=src_T, clamp_total=False,
                                   params=SamplerParams(0.9, 50, 1.0, 1.1, 0.3, 1, 1.0))

    def step_batched(self, sids, seeds=None, forced_depth=None, depth_logits_out=None, sampled_depth=False,
                     depth_seeds=None, force_frames=None, feed_frames=None):
        """One frame for each active session; returns (frames [N, nc], next_cb0 [N]).
        Depth codes are the argmax, or each session's depth sampler when a listed session has two
        branches (src/depth_decoder.cpp:252-257) or `sampled_depth` is set (the single-session
        steps, src/c_api.cpp:468-479) unless every session's depth top-k is 1. `depth_seeds` [N]
        reseed the depth draws per call. `forced_depth` [N, nc-1] (rows of `sids`) teacher-forces
        the depth codes: they become the frame and the next inputs; the oracle's own (combined)
        logits go to `depth_logits_out` (a dict filled per session id) and the uniforms it would
        have drawn to `self.last_depth_uniforms`. `force_frames` [N, nc] teacher-forces a voice
        conversion step (src/generation.cpp:347-368): cb0 and the depth codes >= 0 come from it,
        no cb0 is drawn, and `feed_frames` [N, nc], when given, is what the backbone consumes."""
        m = self.m
        nc = m.cfg.nc
        act = [i for i, s in enumerate(sids) if s in self.sessions and self.sessions[s].active]
        frames = np.full((len(sids), nc), -1, np.int64)
        nxt = np.full(len(sids), -1, np.int64)
        if not act:
            return frames, nxt
        ss = [self.sessions[sids[i]] for i in act]
        if seeds is not None:
            for i, s in zip(act, ss):
                s.rng.seed(int(seeds[i]))
        pairs = [k for k, s in enumerate(ss) if s.cfg != 1.0]
        sampled = bool(pairs) or (sampled_depth and any(s.sp.dtop_k != 1 for s in ss)) or force_frames is not None
        ff = None if force_frames is None else np.asarray(force_frames)[act]
        n = len(ss)
        hid = np.stack([s.last_hidden for s in ss] + [ss[k].last_hidden_u for k in pairs])
        cb0 = np.array([s.last_cb0 for s in ss] + [ss[k].last_cb0 for k in pairs])
        if ff is not None:
            cb0 = np.array([int(ff[k, 0]) for k in range(len(ss))] + [int(ff[k, 0]) for k in pairs])
        urow = {k: n + q for q, k in enumerate(pairs)}
        forced = None if forced_depth is None else np.asarray(forced_depth)[act]
        comb_logits = np.zeros((n, nc - 1, m.cfg.vs), np.float32)
        self.last_depth_uniforms = {}
        chosen = np.zeros((n, nc - 1), np.int64)

        def choose(j, lg, ks):
            out = np.zeros(lg.shape[0], np.int64)
            for k in ks:
                s = ss[k]
                l = combine_logits(lg[k], lg[urow[k]] if k in urow else None, s.cfg)
                comb_logits[k, j - 1] = l
                if ff is not None and ff[k, j] >= 0:
                    code = int(ff[k, j])
                elif not sampled or s.sp.dtop_k == 1:
                    code = int(np.argmax(l))
                else:
                    if seeds is not None:
                        key, draw = s.rng.key, 0
                    elif depth_seeds is not None:
                        key, draw = int(depth_seeds[act[k]]) & 0xFFFFFFFF, 0
                    else:
                        key, draw = s.rng.key, s.rng.draw
                    u = depth_uniform(key, draw, j)
                    self.last_depth_uniforms.setdefault(s.sid, {})[j - 1] = u
                    code = sample_philox(l, s.sp.dtemp, s.sp.dtop_k, s.sp.dtop_p, u)
                if forced is not None:
                    code = int(forced[k, j - 1])
                chosen[k, j - 1] = code
                out[k] = code
                if k in urow:
                    out[urow[k]] = code
            return out

        # each depth weight set decodes its own sessions' rows (src/c_api.cpp:622-650)
        for use_q4 in (False, True):
            ks = [k for k in range(n) if ss[k].use_q4 == use_q4]
            if not ks:
                continue
            model = self.q4 if use_q4 else m
            rows = ks + [urow[k] for k in ks if k in urow]

            def choose_set(j, lg_local, ks=ks, rows=rows):
                lg = np.zeros((hid.shape[0], lg_local.shape[1]), np.float32)
                lg[rows] = lg_local
                return choose(j, lg, ks)[rows]

            model.depth_chain(hid[rows], cb0[rows], choose_set)
        if depth_logits_out is not None:
            for k, i in enumerate(act):
                depth_logits_out[sids[i]] = comb_logits[k]
        fr = np.concatenate([cb0[:n, None], chosen], axis=1)
        fed = fr if feed_frames is None else np.asarray(feed_frames)[act].astype(np.int64)
        ae = m.audio_embed(np.concatenate([fed, fed[pairs]], axis=0) if pairs else fed)
        hs, ls = m.backbone_step_batched([s.st for s in ss] + [ss[k].st_u for k in pairs], ae)
        self.last_cb0_logits = {}
        for k, (i, s) in enumerate(zip(act, ss)):
            frames[i] = fr[k]
            if ff is not None:
                s.steps_taken += 1
                s.last_hidden = hs[k]
                if k in urow:
                    s.last_hidden_u = hs[urow[k]]
                nxt[i] = 0
                continue
            lk = combine_logits(ls[k], ls[urow[k]] if k in urow else None, s.cfg)
            self.last_cb0_logits[s.sid] = (apply_penalties(lk, s.sp.rep, s.hist, m.cfg.cb_size, m.cfg.vs),
                                           s.rng.key, s.rng.draw)
            nx = self._sample_cb0(s, lk)
            s.steps_taken += 1
            if nx == m.cfg.bb_eos or s.steps_taken >= s.max_tokens:
                s.active = False
            else:
                s.hist[nx] = s.hist.get(nx, 0) + 1
                s.last_cb0 = nx
                s.last_hidden = hs[k]
                if k in urow:
                    s.last_hidden_u = hs[urow[k]]
                nxt[i] = nx
        return frames, nxt


# ----------------------------------------------------------------------------- vocoder
# Codec decoder (src/codec_decoder.cpp:11-98, src/codec_conv.cpp:9-59,
# src/codec_transformer.cpp:48-83). Activations are [channels, time] as in the reference's ggml
# [L, C] tensors (time contiguous); the transformer works on [time, channels].

def conv1d_causal(x, w, b, stride=1, dilation=1):
    """src/codec_conv.cpp:9-23: ggml_conv_1d with pad = (K-1)*dilation - (stride-1) on both sides,
    keeping the first n_out outputs, plus bias. x [Cin, L], w [Cout, Cin, K] -> [Cout, n_out]."""
    cout, cin, K = w.shape
    L = x.shape[1]
    pad = max(0, (K - 1) * dilation - (stride - 1))
    n_out = (L + pad - dilation * (K - 1) - 1) // stride + 1
    xp = np.concatenate([np.zeros((cin, pad), np.float32), x.astype(np.float32),
                         np.zeros((cin, pad), np.float32)], axis=1)
    y = np.zeros((cout, n_out), np.float64)
    for k in range(K):
        cols = xp[:, k * dilation: k * dilation + (n_out - 1) * stride + 1: stride]
        y += w[:, :, k].astype(np.float64) @ cols.astype(np.float64)
    if b is not None:
        y += b.astype(np.float64)[:, None]
    return y.astype(np.float32)


def convtr1d_causal(x, w, b, stride):
    """src/codec_conv.cpp:25-32: ggml_conv_transpose_1d (padding 0), the first L*stride outputs
    kept, plus bias. x [Cin, L], w [Cin, Cout, K] -> [Cout, L*stride]."""
    cin, cout, K = w.shape
    L = x.shape[1]
    full = np.zeros((cout, (L - 1) * stride + K), np.float64)
    for k in range(K):
        contrib = w[:, :, k].astype(np.float64).T @ x.astype(np.float64)     # [Cout, L]
        full[:, k: k + (L - 1) * stride + 1: stride] += contrib
    y = full[:, : L * stride]
    if b is not None:
        y = y + b.astype(np.float64)[:, None]
    return y.astype(np.float32)


def depthwise1d_causal(x, w, b):
    """src/codec_conv.cpp:42-59: y[c, t] = sum_k w[k, c] x[c, t - (K-1) + k] + b[c]; w [K, C]."""
    K = w.shape[0]
    C, L = x.shape
    xp = np.concatenate([np.zeros((C, K - 1), np.float32), x.astype(np.float32)], axis=1)
    y = np.zeros((C, L), np.float64)
    for k in range(K):
        y += w[k].astype(np.float64)[:, None] * xp[:, k: k + L]
    if b is not None:
        y += b.astype(np.float64)[:, None]
    return y.astype(np.float32)


def snake_beta(x, la, lb):
    """src/codec_decoder.cpp:10-16: x + sin(x * exp(la))^2 / exp(lb), per channel."""
    a = np.exp(la.astype(np.float32))[:, None]
    bb = np.exp(lb.astype(np.float32))[:, None]
    s = np.sin((x * a).astype(np.float32)).astype(np.float32)
    return (x + (s * s) / bb).astype(np.float32)


def layer_norm_rows(x, w, b, eps):
    """ggml_norm over each row (mean and variance accumulated in double) times w plus b
    (src/common.cpp:131-134). x [rows, C]."""
    x = x.astype(np.float32)
    mean = x.astype(np.float64).mean(axis=-1, keepdims=True)
    xc = (x - mean.astype(np.float32)).astype(np.float32)
    var = (xc.astype(np.float64) ** 2).mean(axis=-1, keepdims=True)
    scale = (np.float32(1.0) / np.sqrt((var + eps).astype(np.float32))).astype(np.float32)
    return ((xc * scale).astype(np.float32) * w.astype(np.float32) + b.astype(np.float32)).astype(np.float32)


def gelu_erf(x):
    x = x.astype(np.float64)
    from math import sqrt
    from scipy.special import erf
    return (0.5 * x * (1.0 + erf(x / sqrt(2.0)))).astype(np.float32)


def sliding_causal_mask(T, window):
    """src/common.cpp:162-173: key k visible to query q when k <= q and q - k < window."""
    q = np.arange(T)[:, None]
    k = np.arange(T)[None, :]
    ok = (k <= q) & ((window <= 0) | (q - k < window))
    return np.where(ok, 0.0, -np.inf).astype(np.float32)


class Vocoder:
    """Batch-free restatement of MimiCodec::decode (src/codec.cpp:15-24) on the model's
    `codec.*` tensors, and of the vocoder sessions' windowed decoding (src/c_api.cpp:1004-1064)."""

    SAMPLES_PER_FRAME = 1920   # src/c_api.cpp:1025 (a constant of the C API)
    MAX_HISTORY = 32           # src/c_api.cpp:1051

    def __init__(self, model: "Model"):
        self.m = model
        self.c = model.cfg.voc
        self.history = {}

    def w(self, name):
        return self.m.w(name)

    def _conv_w(self, name):
        return self.w(name)           # ggml [K, Cin, Cout] -> numpy [Cout, Cin, K]

    def quantizer_decode(self, codes, n_cb):
        """src/codec_decoder.cpp:40-63 -> [codebook_dim, T]."""
        codes = np.asarray(codes, np.int64).reshape(-1, self.m.cfg.nc)
        first = self.w("codec.dq.first.0.embed")[codes[:, 0]]
        first = linear(first, self.w("codec.dq.first.out_proj.weight"))
        if n_cb > 1:
            rest = None
            for cb in range(1, n_cb):
                e = self.w(f"codec.dq.rest.{cb - 1}.embed")[codes[:, cb]]
                rest = e if rest is None else (rest + e).astype(np.float32)
            rest = linear(rest, self.w("codec.dq.rest.out_proj.weight"))
            first = (first + rest).astype(np.float32)
        return first.T.copy()

    def transformer(self, x):
        """src/codec_transformer.cpp:48-83. x [T, latent] -> [T, latent]."""
        c = self.c
        T = x.shape[0]
        h = (linear(x, self.w("codec.dtf.in_proj.weight")) + self.w("codec.dtf.in_proj.bias")).astype(np.float32)
        cos, sin = rope_cos_sin(np.arange(T), c["hd"], c["theta"])
        mask = sliding_causal_mask(T, c["window"])
        scale = 1.0 / math.sqrt(c["hd"])
        for il in range(c["n_layer"]):
            p = f"codec.dtf.blk.{il}"
            res = h
            cur = rms_norm(h, self.w(p + ".attn_norm.weight"), c["eps"])
            q = linear(cur, self.w(p + ".attn_q.weight")).reshape(T, c["n_head"], c["hd"])
            k = linear(cur, self.w(p + ".attn_k.weight")).reshape(T, c["n_kv"], c["hd"])
            v = linear(cur, self.w(p + ".attn_v.weight")).reshape(T, c["n_kv"], c["hd"])
            q = rope_neox(q, cos, sin)
            k = rope_neox(k, cos, sin)
            a = attention(q, k, v, scale, mask)
            a = linear(a, self.w(p + ".attn_output.weight")) * self.w(p + ".attn_scale")
            h = (res + a).astype(np.float32)
            res = h
            cur = rms_norm(h, self.w(p + ".ffn_norm.weight"), c["eps"])
            g = silu(linear(cur, self.w(p + ".ffn_gate.weight")))
            u = linear(cur, self.w(p + ".ffn_up.weight"))
            cur = linear((g * u).astype(np.float32), self.w(p + ".ffn_down.weight")) * self.w(p + ".ffn_scale")
            h = (res + cur).astype(np.float32)
        h = rms_norm(h, self.w("codec.dtf.norm.weight"), c["eps"])
        return (linear(h, self.w("codec.dtf.out_proj.weight")) + self.w("codec.dtf.out_proj.bias")).astype(np.float32)

    def convnext(self, p, x):
        """src/codec_decoder.cpp:18-29 over x [C, L]."""
        h = depthwise1d_causal(x, self.w(p + ".dw.weight"), self.w(p + ".dw.bias"))
        h = layer_norm_rows(h.T, self.w(p + ".norm.weight"), self.w(p + ".norm.bias"), 1e-6)
        h = (linear(h, self.w(p + ".pw1.weight")) + self.w(p + ".pw1.bias")).astype(np.float32)
        h = gelu_erf(h)
        h = (linear(h, self.w(p + ".pw2.weight")) + self.w(p + ".pw2.bias")).astype(np.float32)
        h = (h * self.w(p + ".gamma")).astype(np.float32)
        return (x + h.T).astype(np.float32)

    def residual_unit(self, p, x, dilation):
        """src/codec_decoder.cpp:31-38."""
        h = snake_beta(x, self.w(p + ".a1"), self.w(p + ".b1"))
        h = conv1d_causal(h, self._conv_w(p + ".conv1.conv.weight"), self.w(p + ".conv1.conv.bias"), 1, dilation)
        h = snake_beta(h, self.w(p + ".a2"), self.w(p + ".b2"))
        h = conv1d_causal(h, self._conv_w(p + ".conv2.conv.weight"), self.w(p + ".conv2.conv.bias"), 1, 1)
        return (x + h).astype(np.float32)

    def decode(self, codes, T, n_cb=0):
        """src/codec_decoder.cpp:65-98: codes frame-major [T * nc] -> PCM [T * 1920] in [-1, 1]."""
        c = self.c
        n_cb = n_cb or self.m.cfg.nc
        h = self.quantizer_decode(codes, n_cb)
        h = conv1d_causal(h, self._conv_w("codec.dpre.conv.weight"), self.w("codec.dpre.conv.bias"))
        h = self.transformer(h.T).T.copy()
        for i, r in enumerate(c["ratios"]):
            p = f"codec.dup.{i}"
            h = convtr1d_causal(h, self.w(p + ".up.conv.weight"), self.w(p + ".up.conv.bias"), r)
            h = self.convnext(p, h)
        h = conv1d_causal(h, self._conv_w("codec.dhead.conv.weight"), self.w("codec.dhead.conv.bias"))
        for i, r in enumerate(c["rates"]):
            p = f"codec.dblk.{i}"
            h = snake_beta(h, self.w(p + ".alpha"), self.w(p + ".beta"))
            h = convtr1d_causal(h, self.w(p + ".up.conv.weight"), self.w(p + ".up.conv.bias"), r)
            for j, d in enumerate((1, 3, 9)):
                h = self.residual_unit(p + f".res.{j}", h, d)
        h = snake_beta(h, self.w("codec.dfin.alpha"), self.w("codec.dfin.beta"))
        h = conv1d_causal(h, self._conv_w("codec.dfin.conv.weight"), self.w("codec.dfin.conv.bias"))
        return np.clip(h.reshape(-1), -1.0, 1.0).astype(np.float32)

    def session_decode(self, sid, frames, n_frames):
        """src/c_api.cpp:1004-1064: decode the kept history plus the new frames, return the new
        frames' samples, keep the last 32 frames."""
        nc = self.m.cfg.nc
        new = np.asarray(frames, np.int64).reshape(-1)[: n_frames * nc]
        hist = self.history.get(sid, np.zeros(0, np.int64))
        past = hist.size // nc
        audio = self.decode(np.concatenate([hist, new]), past + n_frames)
        out = audio[past * self.SAMPLES_PER_FRAME: (past + n_frames) * self.SAMPLES_PER_FRAME]
        hist = np.concatenate([hist, new])
        if hist.size // nc > self.MAX_HISTORY:
            hist = hist[(hist.size // nc - self.MAX_HISTORY) * nc:]
        self.history[sid] = hist
        return out


# ----------------------------------------------------------------------------- generate
# breeze_generate's host logic: the long-text splitter (src/text_split.cpp:6-111) and the
# streaming flush schedule of src/generation.cpp:137-168.

def _utf8_chars(text: str):
    """(character, UTF-8 byte length) pairs."""
    return [(ch, len(ch.encode("utf-8"))) for ch in text]


def text_weight(text: str) -> int:
    """One per single-byte character, three per multi-byte one (src/text_split.cpp:16-24)."""
    return sum(1 if n == 1 else 3 for _, n in _utf8_chars(text))


_CJK_STOPS = {"。", "！", "？", "；", "…", "．"}


def split_sentences(t: str):
    """src/text_split.cpp:32-62: a newline, or . ! ? ; followed (after closing quotes/brackets)
    by a space, newline or the end, or a full-width stop ends a sentence."""
    out, cur, i = [], "", 0
    while i < len(t):
        ch = t[i]
        cur += ch
        i += 1
        brk = False
        if len(ch.encode("utf-8")) > 1:
            brk = ch in _CJK_STOPS
        elif ch == "\n":
            brk = True
        elif ch in ".!?;":
            j = i
            while j < len(t) and t[j] in "\"')]":
                j += 1
            brk = j >= len(t) or t[j] in " \n"
            if brk:
                cur += t[i:j]
                i = j
        if brk:
            out.append(cur)
            cur = ""
    if cur:
        out.append(cur)
    return out


def split_clauses(s: str, budget: int):
    """src/text_split.cpp:64-87."""
    if text_weight(s) <= budget:
        return [s]
    out, cur, cw, since = [], "", 0, 0
    for ch, n in _utf8_chars(s):
        cur += ch
        w = 1 if n == 1 else 3
        cw += w
        since += w
        comma = ch in (",", "，", "、", ":")
        space = ch == " "
        if cw >= budget and (comma or (space and since > budget // 4)):
            out.append(cur)
            cur, cw, since = "", 0, 0
        elif comma or space:
            since = 0
    if cur:
        out.append(cur)
    return out


def split_text(text: str, budget: int, first_budget: int = 0):
    """src/text_split.cpp:89-111."""
    if budget <= 0 or text_weight(text) <= budget:
        return [text]
    out, cur, cw = [], "", 0
    limit = first_budget if first_budget > 0 else budget
    for s in split_sentences(text):
        for p in split_clauses(s, budget):
            w = text_weight(p)
            if cw > 0 and cw + w > limit:
                out.append(cur)
                cur, cw = "", 0
                limit = budget
            cur += p
            cw += w
    if cur:
        out.append(cur)
    return out or [text]


def stream_chunks(voc: "Vocoder", frames: np.ndarray, chunk_first: int = 4, chunk_max: int = 25, stop_after: int = 0):
    """PCM chunks that one piece's frames [F, nc] stream through the callback, frames arriving
    one at a time (src/generation.cpp:137-168): each window decodes up to window + 16 frames of
    left context and emits only the new frames' samples; chunk sizes ramp c -> c + c//3 + 1."""
    frames = np.asarray(frames).reshape(-1, voc.m.cfg.nc)
    spf = Vocoder.SAMPLES_PER_FRAME
    ctx = voc.c["window"] + 16
    chunk_max = max(1, chunk_max)
    chunk = min(max(1, chunk_first), chunk_max)
    emitted = 0
    out = []

    def flush(have, final):
        nonlocal emitted, chunk
        while have - emitted >= chunk or (final and have > emitted):
            start = emitted
            count = have - emitted if final else chunk
            cs = start - ctx if start > ctx else 0
            audio = voc.decode(frames[cs:start + count].reshape(-1), start + count - cs)
            out.append(audio[(start - cs) * spf:(start - cs + count) * spf])
            if stop_after and len(out) >= stop_after:
                return False
            emitted += count
            chunk = min(chunk + chunk // 3 + 1, chunk_max)
            if not final and have - emitted < chunk:
                break
        return True

    for have in range(1, frames.shape[0] + 1):
        if not flush(have, False):
            return out
    flush(frames.shape[0], True)
    return out


def wav_bytes(samples, sample_rate: int) -> bytes:
    """16-bit mono PCM WAV (src/audio.cpp:80-107): clamp to [-1, 1], scale by 32767, truncate
    toward zero, little-endian, 44-byte RIFF header."""
    import struct
    x = np.clip(np.asarray(samples, np.float32), -1.0, 1.0)
    pcm = (x * np.float32(32767.0)).astype(np.float32).astype(np.int16).astype("<i2").tobytes()
    hdr = b"RIFF" + struct.pack("<I", 36 + len(pcm)) + b"WAVE" + b"fmt " + struct.pack(
        "<IHHIIHH", 16, 1, 1, sample_rate, sample_rate * 2, 2, 16) + b"data" + struct.pack("<I", len(pcm))
    return hdr + pcm


# ----------------------------------------------------------------------------- codec encoder
def elu(x):
    """ggml_elu: x for x > 0, exp(x) - 1 otherwise."""
    x = x.astype(np.float32)
    return np.where(x > 0, x, np.expm1(np.minimum(x, 0).astype(np.float64)).astype(np.float32)).astype(np.float32)


class CodecEncoder:
    """MimiCodec::encode (src/codec.cpp:80-123): SEANet encoder (src/codec_conv.cpp:33-78), the
    Mimi encoder transformer (src/codec_transformer.cpp:9-45), the stride-2 downsample and the
    semantic + residual acoustic nearest-codebook search. PCM [L] at 24 kHz -> codes [T][nc]."""

    def __init__(self, model: "Model"):
        self.m = model
        self.c = model.cfg.codec

    def w(self, name):
        return self.m.w(name)

    def seanet(self, x):
        """src/codec_conv.cpp:60-77 over [1, L] -> [hidden, T]."""
        ratios = self.c["ratios"]
        rev = [ratios[3], ratios[2], ratios[1], ratios[0]]

        def conv(i, h, stride):
            p = f"codec.enc.{i}.conv"
            return conv1d_causal(h, self.w(p + ".weight"), self.w(p + ".bias"), stride, 1)

        h = conv(0, x, 1)
        for st, (ri, ci) in enumerate(zip((1, 4, 7, 10), (3, 6, 9, 12))):
            p = f"codec.enc.{ri}"
            r = elu(h)
            r = conv1d_causal(r, self.w(p + ".block.1.conv.weight"), self.w(p + ".block.1.conv.bias"), 1, 1)
            r = elu(r)
            r = conv1d_causal(r, self.w(p + ".block.3.conv.weight"), self.w(p + ".block.3.conv.bias"), 1, 1)
            h = (h + r).astype(np.float32)
            h = conv(ci, elu(h), rev[st])
        return conv(14, elu(h), 1)

    def transformer(self, x):
        """src/codec_transformer.cpp:9-45 over [T, hidden]."""
        c = self.c
        T = x.shape[0]
        cos, sin = rope_cos_sin(np.arange(T), c["hd"], c["theta"])
        mask = sliding_causal_mask(T, c["window"])
        scale = 1.0 / math.sqrt(c["hd"])
        h = x.astype(np.float32)
        for il in range(c["n_layer"]):
            p = f"codec.enct.blk.{il}"
            cur = layer_norm_rows(h, self.w(p + ".attn_norm.weight"), self.w(p + ".attn_norm.bias"), c["eps"])
            q = linear(cur, self.w(p + ".attn_q.weight")).reshape(T, c["n_head"], c["hd"])
            k = linear(cur, self.w(p + ".attn_k.weight")).reshape(T, c["n_head"], c["hd"])
            v = linear(cur, self.w(p + ".attn_v.weight")).reshape(T, c["n_head"], c["hd"])
            a = attention(rope_neox(q, cos, sin), rope_neox(k, cos, sin), v, scale, mask)
            a = (linear(a, self.w(p + ".attn_output.weight")) * self.w(p + ".attn_scale")).astype(np.float32)
            h = (h + a).astype(np.float32)
            cur = layer_norm_rows(h, self.w(p + ".ffn_norm.weight"), self.w(p + ".ffn_norm.bias"), c["eps"])
            cur = gelu_erf(linear(cur, self.w(p + ".ffn_up.weight")))
            cur = (linear(cur, self.w(p + ".ffn_down.weight")) * self.w(p + ".ffn_scale")).astype(np.float32)
            h = (h + cur).astype(np.float32)
        return h

    def embeddings(self, audio):
        """The projected quantiser inputs: (semantic [T2, dim], acoustic [T2, dim])."""
        x = np.asarray(audio, np.float32).reshape(1, -1)
        h = self.seanet(x)                                   # [hidden, T]
        h = self.transformer(h.T).T                          # [hidden, T]
        h = conv1d_causal(h, self.w("codec.downsample.conv.weight"), None, 2, 1)   # [hidden, T2]
        emb = h.T.astype(np.float32)
        return linear(emb, self.w("codec.sq.in_proj.weight")), linear(emb, self.w("codec.aq.in_proj.weight"))

    @staticmethod
    def nearest(book, v):
        """src/codec.cpp:61-74: the first entry with the least squared distance (f32, summed
        over the dimension in order). book [n, dim], v [dim]."""
        d = ((v[None, :].astype(np.float32) - book.astype(np.float32)) ** 2).astype(np.float32)
        dist = np.zeros(book.shape[0], np.float32)
        for k in range(book.shape[1]):
            dist = (dist + d[:, k]).astype(np.float32)
        return int(np.argmin(dist)), dist

    def encode(self, audio, want_dists=False):
        c = self.c
        nc = self.m.cfg.nc
        rs, ra = self.embeddings(audio)
        T = rs.shape[0]
        sbook = self.w("codec.sq.0.embed")                   # [book, dim]
        abooks = [self.w(f"codec.aq.{i}.embed") for i in range(nc - c["n_sem"])]
        codes = np.zeros((T, nc), np.int64)
        dists = []
        for f in range(T):
            codes[f, 0], d0 = self.nearest(sbook, rs[f])
            res = ra[f].astype(np.float32).copy()
            fd = [d0]
            for i, book in enumerate(abooks):
                ci, di = self.nearest(book, res)
                codes[f, c["n_sem"] + i] = ci
                res = (res - book[ci]).astype(np.float32)
                fd.append(di)
            dists.append(fd)
        return (codes, dists) if want_dists else codes

    def follow(self, audio, codes):
        """Walks the quantiser chain with the given codes [T][nc] in place of the nearest
        choices (teacher forcing) and returns, per frame and codebook, the squared distances of
        the given code and of the nearest entry at that stage."""
        c = self.c
        nc = self.m.cfg.nc
        rs, ra = self.embeddings(audio)
        sbook = self.w("codec.sq.0.embed")
        abooks = [self.w(f"codec.aq.{i}.embed") for i in range(nc - c["n_sem"])]
        out = np.zeros((rs.shape[0], nc, 2), np.float64)
        for f in range(min(rs.shape[0], len(codes))):
            _, d = self.nearest(sbook, rs[f])
            out[f, 0] = (d[int(codes[f][0])], d.min())
            res = ra[f].astype(np.float32).copy()
            for i, book in enumerate(abooks):
                _, d = self.nearest(book, res)
                ci = int(codes[f][c["n_sem"] + i])
                out[f, c["n_sem"] + i] = (d[ci], d.min())
                res = (res - book[ci]).astype(np.float32)
        return out
