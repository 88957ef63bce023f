"""Batched session creation on the GPU (bzb_generator_sessions_create_batch), through the C ABI,
against the oracle's one-at-a-time restatement of breeze_generator_session_create_ext
(src/c_api.cpp:326-445) (needs a B200).

Every session of the batch must get what its own session_create_ext call gives: the prompt (with
the reference segment and the unconditional branch of a guided session), the budget clamp and
allocation, the first cb0 from the combined prefill logits, and the KV cache that the following
decode steps read. The prompts of all sessions and branches are prefilled as packed rows, so the
text encoder's sliding window, the backbone's causal attention and the rotary positions must stay
inside each prompt; the decode steps after the batch check the cached keys and values.
"""
import numpy as np
import pytest

import breeze_oracle as bo
from parity_helpers import LOGIT_ATOL, check_depth, flip_budget, reconcile_cb0

pytestmark = pytest.mark.gpu

COS_MIN = 0.9995


def cosine(a, b):
    a = a.reshape(-1).astype(np.float64)
    b = b.reshape(-1).astype(np.float64)
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30))


@pytest.fixture(scope="module")
def gen(pkg, tiny_model):
    g = pkg.GeneratorHandle(tiny_model, 0)
    yield g
    g.close()


def _specs(pkg, cfg, rng):
    """Plain, guided, referenced and guided+referenced sessions, prompts from 2 to ~60 tokens (the
    tiny text encoder's window is 8 positions, the packed query blocks 8 rows)."""
    words = lambda ids: pkg.ids_to_text(ids)
    long_ids = list(range(3000, 3050))
    return [
        dict(session_id=81, text=words([311, 312, 313]) + " plain", seed=1, max_new_tokens=6),
        dict(session_id=82, text=words(long_ids) + " long guided", seed=2, max_new_tokens=5, cfg_scale=2.0),
        dict(session_id=83, text=words([321, 322]), seed=3, max_new_tokens=4, cfg_scale=1.5,
             ref_text=words([305, 306, 307]), ref_codes=rng.integers(0, 2048, (3, cfg.nc)).astype(np.int32), ref_frames=3),
        dict(session_id=84, text=words([331]), seed=4, max_new_tokens=7, instruction="Whisper.",
             ref_text=words(list(range(400, 420))), ref_codes=rng.integers(0, 2048, (9, cfg.nc)).astype(np.int32),
             ref_frames=9),
        dict(session_id=85, text=words(list(range(5000, 5013))), seed=5, max_new_tokens=0),
        dict(session_id=86, text=words(list(range(7000, 7190))) + " long", seed=6, max_new_tokens=5),
    ]


def _oracle_create(ref, sp):
    kw = {k: sp[k] for k in ("ref_text", "ref_codes", "seed", "max_new_tokens", "cfg_scale", "instruction") if k in sp}
    return ref.session_create(sp["session_id"], sp["text"], **kw)


def _create(gen, specs, mode):
    if mode == "batch":
        return gen.sessions_create_batch(specs)
    out = [gen.session_create_ext(sp["session_id"], sp["text"],
                                  **{k: v for k, v in sp.items() if k not in ("session_id", "text")}) for sp in specs]
    return [o[0] for o in out], [o[1] for o in out]


_FLIPS = {}


@pytest.mark.parametrize("mode", ["sequential", "batch", "batch-prefill-gemm"])
def test_batch_create_then_steps_match_oracle(pkg, gen, tiny_oracle, mode, monkeypatch):
    """The same checks for one session_create_ext call per session and for the batched call. The
    draws that land across a CDF boundary are counted per session and step in both modes; the
    batch must flip exactly where the one-at-a-time creation does. The tiny random-init model's
    depth logits are near flat (a boundary every ~2% of the mass), so about one draw in ten of
    these prompts flips in either mode. The third mode forces the 256-row prefill GEMM
    (BZB_PREFILL_GEMM=1) for every linear of the packed passes (over 300 rows here), so its four
    epilogues (store, residual add, SwiGLU, GeGLU) run on the same checks."""
    if mode == "batch-prefill-gemm":
        monkeypatch.setenv("BZB_PREFILL_GEMM", "1")
    cfg = tiny_oracle.cfg
    ref = bo.Generator(tiny_oracle)
    specs = _specs(pkg, cfg, np.random.default_rng(8))
    # a live session whose id the batch reuses: the batch replaces it (src/c_api.cpp:333-337)
    gen.session_create_ext(81, pkg.ids_to_text([301, 302]), seed=9, max_new_tokens=3)
    try:
        cb0s, allocs = _create(gen, specs, "sequential" if mode == "sequential" else "batch")
        scales = {}
        for sp, cb0, alloc in zip(specs, cb0s, allocs):
            sid = sp["session_id"]
            rcb0, ralloc = _oracle_create(ref, sp)
            assert alloc == ralloc, (sid, alloc, ralloc)
            assert cb0 == rcb0, (sid, cb0, rcb0)
            h = gen.debug_hidden(sid, cfg.hidden)
            rh = ref.sessions[sid].last_hidden
            assert np.abs(h - rh).max() < LOGIT_ATOL and cosine(h, rh) > COS_MIN, sid
            scales[sid] = sp.get("cfg_scale", 1.0)
        assert gen.active_session_count() == len(specs)
        ids = sorted(scales)
        flips, per = 0, {}
        for step in range(4):
            seeds = [100 * step + i for i in range(len(ids))]
            nxt, frames = gen.sessions_step_batched(ids, seeds=seeds)
            frames = np.asarray(frames)
            forced = np.where(frames[:, 1:cfg.nc] < 0, 0, frames[:, 1:cfg.nc])
            dl = {}
            rf, rn = ref.step_batched(ids, seeds=seeds, forced_depth=forced, depth_logits_out=dl)
            for i, sid in enumerate(ids):
                if sid not in dl:
                    assert nxt[i] == -1
                    continue
                assert frames[i][0] == rf[i][0], (step, sid)
                f = check_depth(ref, cfg.nc, sid, frames[i][1:cfg.nc], dl, scales[sid], step)
                f += reconcile_cb0(ref, sid, int(nxt[i]), int(rn[i]), scales[sid], step)
                per[(sid, step)] = f
                flips += f
        _FLIPS[mode] = per
        assert flips <= flip_budget(4 * len(ids) * cfg.nc), (flips, sorted(per.items()))
        if mode == "batch" and "sequential" in _FLIPS:
            assert per == _FLIPS["sequential"]
    finally:
        for sp in specs:
            gen.session_free(sp["session_id"])
    assert gen.active_session_count() == 0


def test_batch_create_equals_sequential_create(pkg, gen, tiny_oracle):
    """The packed prefill leaves each session where its own session_create_ext call leaves it:
    same first cb0 and allocation, and the same last hidden within the parity tolerance."""
    cfg = tiny_oracle.cfg
    specs = _specs(pkg, cfg, np.random.default_rng(9))
    ids = [sp["session_id"] for sp in specs]
    seq = {}
    for sp in specs:
        kw = {k: v for k, v in sp.items() if k not in ("session_id", "text")}
        cb0, alloc = gen.session_create_ext(sp["session_id"], sp["text"], **kw)
        seq[sp["session_id"]] = (cb0, alloc, gen.debug_hidden(sp["session_id"], cfg.hidden))
    for sid in ids:
        gen.session_free(sid)
    cb0s, allocs = gen.sessions_create_batch(specs)
    try:
        for sid, cb0, alloc in zip(ids, cb0s, allocs):
            scb0, salloc, sh = seq[sid]
            assert (cb0, alloc) == (scb0, salloc), sid
            h = gen.debug_hidden(sid, cfg.hidden)
            assert np.abs(h - sh).max() < LOGIT_ATOL and cosine(h, sh) > COS_MIN, sid
    finally:
        for sid in ids:
            gen.session_free(sid)


def test_batch_create_errors_and_empty(pkg, gen):
    text = pkg.ids_to_text([340, 341])
    assert gen.sessions_create_batch([]) == ([], [])
    with pytest.raises(RuntimeError, match="twice"):
        gen.sessions_create_batch([dict(session_id=91, text=text), dict(session_id=91, text=text)])
    assert gen.active_session_count() == 0
    # a burst over batch-created sessions retires each at its budget and frees every page
    for rep in range(3):
        cb0s, _ = gen.sessions_create_batch([dict(session_id=92, text=text, seed=rep, max_new_tokens=3, cfg_scale=2.5),
                                             dict(session_id=93, text=text, seed=rep, max_new_tokens=5)])
        assert all(c >= 0 for c in cb0s)
        nxt, frames = gen.sessions_step_burst([92, 93], 8, seeds=[1, 2])
        frames = np.asarray(frames).transpose(1, 0, 2)
        for i, budget in enumerate([3, 5]):
            live = frames[:, i, 0] >= 0
            n_live = int(live.sum())
            assert 0 < n_live <= budget and live[:n_live].all()
        assert list(nxt) == [-1, -1]
        assert gen.session_free(92) == 0 and gen.session_free(93) == 0
    assert gen.active_session_count() == 0
