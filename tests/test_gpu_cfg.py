"""Two-branch (classifier-free guidance) sessions and the sampled depth decode on the GPU, through
the generator C ABI, against the oracle's restatement (needs a B200).

Reference behaviour:
- A session created with cfg_scale != 1 prefills a second, unconditional prompt, the one without
  the instruction (src/c_api.cpp:411-434). Its allocation adds to out_allocated_tokens. Every cb0
  is drawn from uncond + s * (cond - uncond) (src/c_api.cpp:148-155, 720-745).
- While such a session is in the batch, every session's depth codes come from its depth sampler
  (src/depth_decoder.cpp:163-257), on combined logits for two-branch sessions.
- breeze_generator_session_step samples its depth codes with the call's seed (src/c_api.cpp:468-479).

The draws are Philox, so parity holds draw by draw. The oracle takes the engine's codes (teacher
forcing) and checks that each one is what the same uniform picks from logits within the logit
tolerance of its own, scaled by the guidance combination's gain (|1 - s| + |s|).
"""
import numpy as np
import pytest

import breeze_oracle as bo
from parity_helpers import check_depth as _check, flip_budget, reconcile_cb0

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gen(pkg, tiny_model):
    g = pkg.GeneratorHandle(tiny_model, 0)
    yield g
    g.close()


def test_cfg_sessions_batched_match_oracle(pkg, gen, tiny_oracle):
    cfg = tiny_oracle.cfg
    ref = bo.Generator(tiny_oracle)
    rng = np.random.default_rng(4)
    scales = {41: 2.0, 42: 1.0, 43: 1.5}
    made = {}
    try:
        for sid, s in scales.items():
            text = pkg.ids_to_text([sid * 7 + 3, 1000 + sid, 20000 + sid]) + " guided"
            ref_codes = rng.integers(0, 2048, (2, cfg.nc)).astype(np.int32) if sid == 43 else None
            kw = dict(ref_text=pkg.ids_to_text([5, 6]) if sid == 43 else None, ref_codes=ref_codes,
                      seed=sid, max_new_tokens=5)
            cb0, alloc = gen.session_create_ext(sid, text, ref_frames=2 if sid == 43 else 0, cfg_scale=s, **kw)
            rcb0, ralloc = ref.session_create(sid, text, cfg_scale=s, **kw)
            assert alloc == ralloc, (sid, alloc, ralloc)
            assert cb0 == rcb0, (sid, cb0, rcb0)
            made[sid] = s
        # three listed sessions plus two unconditional branches; one id never created
        ids = sorted(made) + [4999]
        flips = 0
        for step in range(4):
            seeds = [100 * step + i for i in range(len(ids))]
            nxt, frames = gen.sessions_step_batched(ids, seeds=seeds)
            frames = np.asarray(frames)
            dl = {}
            forced = np.where(frames[:, 1:cfg.nc] < 0, 0, frames[:, 1:cfg.nc])
            rf, rn = ref.step_batched(ids, seeds=seeds, forced_depth=forced, depth_logits_out=dl)
            for i, sid in enumerate(ids):
                if sid not in dl:
                    assert nxt[i] == -1
                    continue
                assert frames[i][0] == rf[i][0], (step, sid)
                # the batch holds two-branch sessions: every session draws its depth codes
                assert len(ref.last_depth_uniforms.get(sid, {})) == cfg.nc - 1
                flips += _check(ref, cfg.nc, sid, frames[i][1:cfg.nc], dl, made[sid], step)
                flips += reconcile_cb0(ref, sid, int(nxt[i]), int(rn[i]), made[sid], step)
        assert flips <= flip_budget(4 * len(made) * cfg.nc), flips
    finally:
        for sid in made:
            gen.session_free(sid)
    assert gen.active_session_count() == 0


def test_session_step_samples_depth_with_call_seed(pkg, gen, tiny_oracle):
    cfg = tiny_oracle.cfg
    ref = bo.Generator(tiny_oracle)
    sid = 51
    text = pkg.ids_to_text([71, 72, 73, 74]) + " single"
    cb0, _ = gen.session_create_ext(sid, text, seed=9, max_new_tokens=6)
    rcb0, _ = ref.session_create(sid, text, seed=9, max_new_tokens=6)
    assert cb0 == rcb0
    flips = 0
    try:
        for step in range(4):
            seed = 1000 + 17 * step
            nxt, frame = gen.session_step(sid, seed)
            frame = np.asarray(frame)
            dl = {}
            rf, rn = ref.step_batched([sid], forced_depth=frame[None, 1:cfg.nc], depth_logits_out=dl,
                                      sampled_depth=True, depth_seeds=[seed])
            assert frame[0] == rf[0][0]
            assert len(ref.last_depth_uniforms[sid]) == cfg.nc - 1
            flips += _check(ref, cfg.nc, sid, frame[1:cfg.nc], dl, 1.0, step)
            flips += reconcile_cb0(ref, sid, int(nxt), int(rn[0]), 1.0, step)
        assert flips <= flip_budget(4 * cfg.nc), flips
        # the same call seed gives the same depth codes from the same state: replay on a twin
        twin = 52
        gen.session_create_ext(twin, text, seed=9, max_new_tokens=6)
        a = gen.session_step(twin, 77)
        gen.session_create_ext(twin, text, seed=9, max_new_tokens=6)
        b = gen.session_step(twin, 77)
        assert a == b
        c_ = gen.session_step(twin, 78)
        assert c_[1][0] == b[0]   # the next frame starts with the cb0 the previous step returned
    finally:
        gen.session_free(sid)
        gen.session_free(52)


def test_cfg_burst_retires_both_branches(pkg, gen, tiny_oracle):
    """A guided session in a burst retires at max_new_tokens with its unconditional branch; its
    pages return to the pool (a new session of the same size fits again and again)."""
    text = pkg.ids_to_text([900, 901, 902])
    for rep in range(3):
        gen.session_create_ext(61, text, seed=rep, max_new_tokens=3, cfg_scale=3.0)
        gen.session_create_ext(62, text, seed=rep, max_new_tokens=5)
        nxt, frames = gen.sessions_step_burst([61, 62], 8, seeds=[1, 2])
        frames = np.asarray(frames).transpose(1, 0, 2)
        for i, budget in enumerate([3, 5]):
            live = frames[:, i, 0] >= 0
            n_live = int(live.sum())
            # frames are contiguous from step 0 and stop at the budget (earlier only at EOS)
            assert 0 < n_live <= budget and live[:n_live].all() and (frames[n_live:, i] == -1).all()
        assert list(nxt) == [-1, -1]
        assert gen.session_free(61) == 0 and gen.session_free(62) == 0
    assert gen.active_session_count() == 0


def test_sessions_step_round_matches_oracle(pkg, gen, tiny_oracle):
    """breeze_generator_sessions_step_round (src/c_api.cpp:584-599): session_step for each listed
    session in order with seed + i; the return value counts the sessions still going; an unknown
    or finished session gets -1 and its frame row is not written."""
    cfg = tiny_oracle.cfg
    ref = bo.Generator(tiny_oracle)
    scales = {71: 1.0, 72: 2.0, 73: 1.0}
    budgets = {71: 6, 72: 6, 73: 2}
    flips = 0
    try:
        for sid, s in scales.items():
            text = pkg.ids_to_text([sid * 5, 3000 + sid, 40000 + sid]) + " round"
            cb0, alloc = gen.session_create_ext(sid, text, seed=sid, max_new_tokens=budgets[sid], cfg_scale=s)
            rcb0, ralloc = ref.session_create(sid, text, seed=sid, max_new_tokens=budgets[sid], cfg_scale=s)
            assert alloc == ralloc
            flips += reconcile_cb0(ref, sid, cb0, rcb0, s, "create")
        ids = [71, 4242, 72, 73]
        for rnd in range(3):
            seed = 500 + 10 * rnd
            live = {sid: ref.sessions[sid].active for sid in scales}
            nxt, frames = gen.sessions_step_round(ids, seed)
            frames = np.asarray(frames)
            going = 0
            for i, sid in enumerate(ids):
                if sid not in scales or not live[sid]:
                    assert nxt[i] == -1 and (frames[i] == 0).all(), (rnd, sid)
                    continue
                dl = {}
                rf, rn = ref.step_batched([sid], forced_depth=frames[i][None, 1:cfg.nc], depth_logits_out=dl,
                                          sampled_depth=True, depth_seeds=[seed + i])
                assert frames[i][0] == rf[0][0], (rnd, sid)
                flips += _check(ref, cfg.nc, sid, frames[i][1:cfg.nc], dl, scales[sid], (rnd, sid))
                if rn[0] >= 0 and nxt[i] >= 0:
                    flips += reconcile_cb0(ref, sid, int(nxt[i]), int(rn[0]), scales[sid], (rnd, sid))
                else:
                    assert nxt[i] == rn[0] == -1, (rnd, sid, nxt[i], rn[0])
                going += int(nxt[i] >= 0)
            assert gen.last_round_completed == going
        # session 73's budget of 2 ran out in the second round
        assert not ref.sessions[73].active
        assert flips <= flip_budget(3 * 3 * cfg.nc), flips
    finally:
        for sid in scales:
            gen.session_free(sid)
