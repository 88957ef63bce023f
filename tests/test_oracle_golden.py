"""Pins the oracle (and the model writer) against independent references: gguf-py 0.19.0's
Q8_0 / Q4_K codecs and the published Philox4x32-10 known-answer vectors. CPU only."""
import os
import subprocess

import numpy as np
import pytest

import breeze_oracle as bo

gguf = pytest.importorskip("gguf")


def test_q8_0_dequant_bit_exact_vs_gguf_py(tiny_oracle):
    for name in ["bb.blk.0.attn_q.weight", "dd.codebooks_head.weight", "te.token_embd.weight", "audio_embd.weight"]:
        t = tiny_oracle.g.tensors[name]
        ref = gguf.dequantize(t.raw.reshape(-1), t.type).reshape(-1)
        assert np.array_equal(tiny_oracle.w(name).reshape(-1), ref), name


def test_writer_q8_0_quantiser_bit_exact_vs_gguf_py(pkg, tmp_path):
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(32 * 2000) * 0.02).astype(np.float32)
    x[:32] = 0.0                                # all-zero block: d = 0, q = 0
    x[32:64] = 1.0                              # constant block
    x[64:96] = np.linspace(-1, 1, 32)           # exact half-way values
    x[96:128] = np.float32(127 / 2) * np.arange(-16, 16) / np.float32(63.5)
    f_in, f_out = tmp_path / "x.f32", tmp_path / "x.q8"
    x.tofile(f_in)
    subprocess.run([pkg.SYNTH_BIN, "--quantize-f32", str(f_in), str(f_out)], check=True)
    ours = np.fromfile(f_out, np.uint8)
    ref = gguf.quants.quantize(x.reshape(-1, 320), gguf.GGMLQuantizationType.Q8_0).reshape(-1)
    assert np.array_equal(ours, ref)


def test_q4_k_dequant_bit_exact_vs_gguf_py(pkg, tmp_path):
    rng = np.random.default_rng(1)
    x = (rng.standard_normal(256 * 64) * 0.02).astype(np.float32)
    f_in, f_out = tmp_path / "x.f32", tmp_path / "x.q4k"
    x.tofile(f_in)
    subprocess.run([pkg.SYNTH_BIN, "--quantize-f32", str(f_in), str(f_out), "--quant", "q4_k"], check=True)
    raw = np.fromfile(f_out, np.uint8)
    ours = bo.dequant_q4_k(raw, x.size)
    ref = gguf.dequantize(raw, gguf.GGMLQuantizationType.Q4_K).reshape(-1)
    assert np.array_equal(ours, ref)
    # and the writer's min/max quantiser represents the floats closely (valid blocks)
    assert np.abs(ours - x).max() < 0.02


def test_philox_known_answers():
    # Random123 philox4x32_10 known-answer vectors
    assert bo.philox4x32_10((0, 0, 0, 0), (0, 0)) == (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)
    assert bo.philox4x32_10((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF)) == (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)
    assert bo.philox4x32_10((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0)) == \
        (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)


def test_philox_uniform_range_and_reseed():
    u = [bo.philox_uniform(7, d) for d in range(2000)]
    assert min(u) >= 0.0 and max(u) < 1.0
    assert abs(np.mean(u) - 0.5) < 0.03
    s = bo.PhiloxStream(9)
    a = [s.next_uniform() for _ in range(3)]
    s.seed(9)
    assert [s.next_uniform() for _ in range(3)] == a


def test_oracle_modes_agree_within_tolerance(tiny_model):
    """ggml's CPU path quantises activations to Q8_0 before each quantised linear; the exact
    mode does not. Both stay inside the parity tolerance of each other."""
    ex = bo.Model(tiny_model, mode="exact")
    gg = bo.Model(tiny_model, mode="ggml")
    rng = np.random.default_rng(2)
    h = rng.standard_normal((3, ex.cfg.hidden)).astype(np.float32)
    cb0 = rng.integers(0, 2048, 3)
    codes, lx = ex.depth_logits_chain(h, cb0)
    _, lg = gg.depth_logits_chain(h, cb0, forced=codes)
    assert np.abs(lx - lg).max() < 2e-2
    for i in range(3):
        for j in range(ex.cfg.nc - 1):
            a, b = lx[i, j].astype(np.float64), lg[i, j].astype(np.float64)
            assert a @ b / np.linalg.norm(a) / np.linalg.norm(b) > 0.9995


def test_ggml_mode_linear_matches_integer_definition(tiny_oracle):
    t = tiny_oracle.g.tensors["bb.blk.0.attn_k.weight"]
    w = tiny_oracle.w("bb.blk.0.attn_k.weight")
    x = np.random.default_rng(3).standard_normal((2, w.shape[1])).astype(np.float32)
    y = bo.linear_q8(x, t.raw, w.shape[0], w.shape[1])
    q, d = bo.quant_q8_0_rows(x)
    # the per-block definition: sum_b sumi_b * dw_b * dx_b
    xq = (q.astype(np.float64) * d.astype(np.float64)).reshape(2, -1)
    assert np.abs(y - xq @ w.T.astype(np.float64)).max() < 1e-4
