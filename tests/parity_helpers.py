"""Shared checks of the engine's sampled tokens against the oracle (test infrastructure).

The engine and the oracle draw the same Philox uniforms. Their logits agree within LOGIT_ATOL,
so a draw may land on different sides of a CDF boundary only when the uniform is within reach of
one. A differing token is accepted when the sampler, given logits within the tolerance of the
oracle's, can return it with that uniform. The oracle then follows the engine's token.
"""
import numpy as np

import breeze_oracle as bo

LOGIT_ATOL = 2e-2
TIE_GAP = 1e-3


def gain(scale):
    """How much a guidance combination lu + s (lc - lu) amplifies a logit error."""
    return abs(1.0 - scale) + abs(scale)


def check_depth(ref, nc, sid, engine_codes, dl, scale, tag):
    """Each engine depth code against the oracle's (combined) logits: a sampled code must be
    reachable with the same uniform; an argmax code may differ only at a numerical tie. Returns
    how many codes differ from the oracle's own pick."""
    sp = ref.sessions[sid].sp
    us = ref.last_depth_uniforms.get(sid, {})
    eps = LOGIT_ATOL * gain(scale)
    flips = 0
    for j in range(nc - 1):
        lg = dl[sid][j]
        code = int(engine_codes[j])
        if j in us:
            ok = bo.sample_reachable(lg, sp.dtemp, sp.dtop_k, us[j], code, eps)
            assert ok, (tag, sid, j, code, bo.sample_margin(lg, sp.dtemp, sp.dtop_k, us[j]))
            flips += int(code != bo.sample_philox(lg, sp.dtemp, sp.dtop_k, sp.dtop_p, us[j]))
        elif code != int(np.argmax(lg)):
            s = np.sort(lg)
            assert s[-1] - s[-2] < TIE_GAP * gain(scale), (tag, sid, j)
            flips += 1
    return flips


def reconcile_cb0(ref, sid, engine_next, oracle_next, scale, tag):
    """Accepts a differing cb0 only within reach of a CDF boundary (or a top-1 tie), then makes
    the oracle follow the engine's token. Returns 1 for a tolerated difference, 0 for agreement."""
    if engine_next == oracle_next:
        return 0
    pl, key, draw = ref.last_cb0_logits[sid]
    sp = ref.sessions[sid].sp
    u = bo.philox_uniform(key, draw)
    eps = LOGIT_ATOL * gain(scale)
    ok = engine_next >= 0 and oracle_next >= 0 and bo.sample_reachable(pl, sp.temp, sp.top_k, u, engine_next, eps)
    assert ok, (tag, sid, engine_next, oracle_next)
    rs = ref.sessions[sid]
    rs.hist[int(oracle_next)] -= 1
    rs.hist[int(engine_next)] = rs.hist.get(int(engine_next), 0) + 1
    rs.last_cb0 = int(engine_next)
    rs.active = True
    return 1


def flip_budget(draws):
    """Tolerated draws that land on the other side of a CDF boundary. Near-flat top-k 50 logits put
    a boundary every ~2% of the mass, and a 1e-3 logit difference (f16 operands in the GEMMs and
    the attention against the oracle's f32) moves each by a few 1e-4, so about one draw in ten
    flips. The budget is that rate plus two binomial standard deviations, so a small sample is
    not failed by chance; every flipped draw is still checked to be reachable within the logit
    tolerance, which is what catches a wrong result."""
    rate = 0.1
    return max(3, int(rate * draws + 2.0 * (rate * (1.0 - rate) * draws) ** 0.5 + 1.0))


def snr_db(ref, got):
    ref = np.asarray(ref, np.float64)
    err = np.asarray(got, np.float64) - ref
    return 10.0 * np.log10((ref @ ref + 1e-30) / (err @ err + 1e-30))


def kernel_weights_q4k(raw: np.ndarray, rows: int, K: int) -> np.ndarray:
    """The f16 weights the kernel feeds the tensor cores: per sub-block a = d * scale and
    b = dmin * min (exact), w = a q - b by one f32 fused multiply-add, then rounded to f16."""
    blocks = raw[: rows * K // 256 * 144].reshape(-1, 144)
    d = blocks[:, 0:2].copy().view(np.float16).astype(np.float32)[:, 0]
    dmin = blocks[:, 2:4].copy().view(np.float16).astype(np.float32)[:, 0]
    sc, mn = bo.q4k_scale_min(blocks[:, 4:16])
    a = d[:, None].astype(np.float64) * sc.astype(np.float64)
    b = dmin[:, None].astype(np.float64) * mn.astype(np.float64)
    qs = blocks[:, 16:]
    q = np.empty((blocks.shape[0], 8, 32), np.float64)
    for s in range(8):
        byte = qs[:, 32 * (s // 2): 32 * (s // 2) + 32]
        q[:, s] = (byte >> (4 * (s % 2))) & 0xF
    w = (a[:, :, None] * q - b[:, :, None]).astype(np.float32).astype(np.float16)
    return w.reshape(rows, K).astype(np.float64)
