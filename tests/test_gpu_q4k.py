"""Q4_K weights on the GPU (needs a B200).

Two uses are covered:
- A fully Q4_K model file: every linear and embedding table, as in the reference's Q4_K
  serving configuration.
- The Q4_K depth override: breeze_generator_load_q4_depth / session_set_q4
  (src/c_api.cpp:532-578). It routes the depth codes of flagged sessions through the dd.*
  tensors of a second file.

The kernel dequantises each 32-value sub-block as f16(a q - b), with a = d * scale and
b = dmin * min exact f32 products and a q - b one f32 fused multiply-add. The GEMM check
restates exactly that; the model checks use the oracle's f32 dequantisation and its logit
tolerance.
"""
import numpy as np
import pytest

import breeze_oracle as bo
from parity_helpers import LOGIT_ATOL, TIE_GAP, check_depth, flip_budget, kernel_weights_q4k, reconcile_cb0, snr_db

pytestmark = pytest.mark.gpu

COS_MIN = 0.9995


def cosine(a, b):
    a = a.reshape(-1).astype(np.float64)
    b = b.reshape(-1).astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))


@pytest.fixture(scope="module")
def q4_model(pkg, model_dir):
    return pkg.synth_model(str(model_dir / "tiny_q4k.gguf"), preset="tiny", quant="q4_k", seed=3)


@pytest.fixture(scope="module")
def q4_oracle(q4_model):
    return bo.Model(q4_model)


@pytest.fixture(scope="module")
def q4_gen(pkg, q4_model):
    g = pkg.GeneratorHandle(q4_model, 0)
    yield g
    g.close()


@pytest.mark.parametrize("tensor,sub", [("bb.blk.0.attn_q.weight", -1), ("bb.blk.1.ffn_down.weight", -1),
                                        ("dd.codebooks_head.weight", 3), ("te.blk.0.ffn_gate.weight", -1),
                                        ("bb.lm_head.weight", -1)])
@pytest.mark.parametrize("rows,prefill", [(1, "auto"), (16, "auto"), (100, "auto"), (300, "1")])
def test_q4k_gemm_matches_oracle(q4_gen, q4_oracle, tensor, sub, rows, prefill, monkeypatch):
    """Decode-shaped and (forced from 256 rows by BZB_PREFILL_GEMM=1) prefill-shaped GEMM."""
    if prefill != "auto":
        monkeypatch.setenv("BZB_PREFILL_GEMM", prefill)
    t = q4_oracle.g.tensors[tensor]
    assert t.type == bo.Q4_K
    w = q4_oracle.w(tensor)
    K = w.shape[-1]
    n_rows = w.shape[-2]
    raw = t.raw
    if sub >= 0:
        w = w[sub]
        raw = raw[sub * n_rows * K // 256 * 144:]
    rng = np.random.default_rng(rows + 7)
    x = rng.standard_normal((rows, K)).astype(np.float32)
    y = q4_gen.debug_gemv(tensor, x, n_rows, sub)
    x16 = x.astype(np.float16).astype(np.float64)
    wk = kernel_weights_q4k(raw, n_rows, K)
    ref16 = x16 @ wk.T
    scale = np.abs(x16) @ np.abs(wk).T + 1e-6
    assert np.max(np.abs(y - ref16) / scale) < 1e-5
    ref = bo.linear(x, w)
    assert np.abs(y - ref).max() < LOGIT_ATOL
    assert cosine(y, ref) > COS_MIN


def test_q4k_model_decode_matches_oracle(pkg, q4_gen, q4_oracle):
    cfg = q4_oracle.cfg
    ref = bo.Generator(q4_oracle)
    ids = [81, 82, 83]
    rng = np.random.default_rng(5)
    try:
        for sid in ids:
            text = pkg.ids_to_text([sid * 11, 900 + sid, 30000 + sid]) + " four bit"
            ref_codes = rng.integers(0, 2048, (2, cfg.nc)).astype(np.int32) if sid == 83 else None
            kw = dict(ref_text=pkg.ids_to_text([7, 8]) if sid == 83 else None, ref_codes=ref_codes, seed=sid,
                      max_new_tokens=6)
            cb0, alloc = q4_gen.session_create_ext(sid, text, ref_frames=2 if sid == 83 else 0, **kw)
            rcb0, ralloc = ref.session_create(sid, text, **kw)
            assert (cb0, alloc) == (rcb0, ralloc)
            h = q4_gen.debug_hidden(sid, cfg.hidden)
            rh = ref.sessions[sid].last_hidden
            assert np.abs(h - rh).max() < LOGIT_ATOL and cosine(h, rh) > COS_MIN
        flips = 0
        for step in range(3):
            seeds = [7 * step + s for s in ids]
            n_exec, frames, nxt = q4_gen.step_frames(ids, 1, seeds)
            dl = {}
            rf, rn = ref.step_batched(ids, seeds=seeds, forced_depth=frames[0][:, 1:], depth_logits_out=dl)
            assert np.array_equal(frames[0][:, 0], rf[:, 0])
            for i, sid in enumerate(ids):
                flips += check_depth(ref, cfg.nc, sid, frames[0][i, 1:], dl, 1.0, step)
                flips += reconcile_cb0(ref, sid, int(nxt[i]), int(rn[i]), 1.0, step)
        assert flips <= flip_budget(3 * len(ids) * cfg.nc)
    finally:
        for sid in ids:
            q4_gen.session_free(sid)


def test_q4_depth_override_routes_flagged_sessions(pkg, tiny_model, tiny_oracle, q4_model):
    cfg = tiny_oracle.cfg
    gen = pkg.GeneratorHandle(tiny_model, 0)
    try:
        with pytest.raises(RuntimeError):
            gen.load_q4_depth(tiny_model + ".missing")
        assert gen.load_q4_depth(q4_model)
        ref = bo.Generator(tiny_oracle)
        ref.load_q4_depth(q4_model)
        # argmax depth (persistent schedule, two masked passes), then with a guided session
        # in the batch (sampled depth for all, src/depth_decoder.cpp:252-257)
        for case, scales in (("argmax", {91: 1.0, 92: 1.0, 93: 1.0}), ("guided", {94: 1.0, 95: 2.0, 96: 1.0})):
            ids = sorted(scales)
            for sid in ids:
                text = pkg.ids_to_text([sid, sid + 1000, sid + 20000]) + " route"
                gen.session_create_ext(sid, text, seed=sid, max_new_tokens=5, cfg_scale=scales[sid])
                ref.session_create(sid, text, seed=sid, max_new_tokens=5, cfg_scale=scales[sid])
            for sid in ids[1:]:
                assert gen.session_set_q4(sid, True)
                assert ref.session_set_q4(sid, True) == 0
            flips = 0
            for step in range(3):
                seeds = [11 * step + s for s in ids]
                nxt, frames = gen.sessions_step_batched(ids, seeds=seeds)
                frames = np.asarray(frames)
                dl = {}
                rf, rn = ref.step_batched(ids, seeds=seeds, forced_depth=frames[:, 1:cfg.nc], depth_logits_out=dl)
                for i, sid in enumerate(ids):
                    assert frames[i][0] == rf[i][0], (case, step, sid)
                    flips += check_depth(ref, cfg.nc, sid, frames[i][1:cfg.nc], dl, scales[sid], (case, step))
                    flips += reconcile_cb0(ref, sid, int(nxt[i]), int(rn[i]), scales[sid], (case, step))
            assert flips <= flip_budget(3 * len(ids) * cfg.nc), (case, flips)
            for sid in ids:
                gen.session_free(sid)
        assert not gen.session_set_q4(12345, True)  # unknown session
    finally:
        gen.close()


def test_q4_override_flag_needs_a_loaded_override(pkg, tiny_model, tiny_oracle):
    """Without a loaded override the flag resolves to off (src/c_api.cpp:576): the session's
    codes come from the model's own depth weights."""
    gen = pkg.GeneratorHandle(tiny_model, 0)
    try:
        text = pkg.ids_to_text([5, 6, 7])
        gen.session_create_ext(1, text, seed=3, max_new_tokens=4)
        gen.session_create_ext(2, text, seed=3, max_new_tokens=4)
        assert gen.session_set_q4(2, True)
        a = gen.sessions_step_batched([1], seeds=[9])
        b = gen.sessions_step_batched([2], seeds=[9])
        assert a == b
    finally:
        gen.close()


def test_q4k_vocoder_full_shapes(pkg, model_dir):
    """The codec decoder's Q4_K linears (tcgen05 4-bit tiles) at the full decoder's shapes."""
    path = pkg.synth_model(str(model_dir / "depth_q4k.gguf"), preset="depth", quant="q4_k", seed=4)
    m = bo.Model(path)
    assert m.g.tensors["codec.dtf.blk.0.attn_q.weight"].type == bo.Q4_K
    voc = pkg.VocoderHandle(path, 0)
    ovoc = bo.Vocoder(m)
    try:
        codes = np.random.default_rng(8).integers(0, 2048, (3, m.cfg.nc)).astype(np.int32)
        pcm = voc.stream_decode(codes)
        ref = ovoc.decode(codes.reshape(-1), 3)
        assert snr_db(ref, pcm) > 40.0, snr_db(ref, pcm)
    finally:
        voc.close()


def test_vocoder_load_independent_of_stale_device_memory(pkg, model_dir):
    """Weights uploaded at load must be complete before the repacking kernels read them: two
    vocoders built on device memory last filled with different values decode bit-identical PCM.
    (A pageable cudaMemcpy may still be in flight when it returns, and the load's own stream does
    not wait for it; the repack then read part of the previous contents.)"""
    import torch
    path = pkg.synth_model(str(model_dir / "depth_q4k.gguf"), preset="depth", quant="q4_k", seed=4)
    codes = np.random.default_rng(8).integers(0, 2048, (3, bo.Model(path).cfg.nc)).astype(np.int32)
    outs = []
    for fill in (1e30, -3.0, float("nan")):
        junk = torch.full((1 << 30,), fill, device="cuda")  # 4 GB, freed back to the driver below
        del junk
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        voc = pkg.VocoderHandle(path, 0)
        try:
            outs.append(voc.stream_decode(codes))
        finally:
            voc.close()
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])
