"""The cb0 sampler's two top-k paths give the same picks (needs a B200).

For top-k <= 64 (the reference's 50, src/sampling.cpp:25-40) the sampler kernel selects the k
largest (logit, index) keys with a radix select instead of sorting all V keys; any other top-k
takes the full bitonic sort. Both must hand the same ordered top-k list to the same inverse-CDF
draw, so for every logits row, top-k, temperature, top-p and Philox draw the picks are identical.
The cases cover ragged vocabularies (2051, the model's cb0 vocabulary, and sizes at and below
64), runs of -inf (suppressed or masked entries, fewer finite entries than k), and tied logits,
where the order between equal logits is by index. The draws are also checked against the
oracle's sampler wherever the uniform sits clear of a CDF boundary.
"""
import numpy as np
import pytest

from oracle import breeze_oracle as bo

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def gen(pkg, tiny_model):
    g = pkg.GeneratorHandle(tiny_model, 0)
    yield g
    g.close()


def _both(gen, logits, k, temp, top_p, seed, draws):
    fast = gen.debug_sample(logits, k, temp, top_p, seed=seed, draws=draws, force_sort=False)
    full = gen.debug_sample(logits, k, temp, top_p, seed=seed, draws=draws, force_sort=True)
    assert fast.shape == (draws, logits.shape[0])
    assert np.array_equal(fast, full), (k, top_p, np.argwhere(fast != full)[:8])
    return fast


def _check_oracle(logits, picks, k, temp, top_p, seed):
    """Draws equal to the oracle's where the uniform is clear of the CDF's boundaries (the GPU's
    exp may move a boundary by a few ulps); returns how many draws were compared."""
    checked = 0
    for d in range(picks.shape[0]):
        for r in range(logits.shape[0]):
            u = bo.philox_uniform(seed + r, d)
            if bo.sample_margin(logits[r], temp, k, u) < 1e-4:
                continue
            want = bo.sample_philox(logits[r], temp, k, top_p, u)
            assert picks[d, r] == want, (d, r, int(picks[d, r]), want)
            checked += 1
    return checked


@pytest.mark.parametrize("k", [1, 5, 50, 64])
@pytest.mark.parametrize("top_p", [1.0, 0.8])
def test_select_and_sort_agree_on_random_logits(gen, k, top_p):
    rng = np.random.default_rng(100 + k)
    logits = (3.0 * rng.standard_normal((8, 2051))).astype(np.float32)
    picks = _both(gen, logits, k, 0.9, top_p, seed=1234 + k, draws=6)
    assert _check_oracle(logits, picks, k, 0.9, top_p, 1234 + k) >= 40


def test_select_and_sort_agree_with_few_finite_logits(gen):
    rng = np.random.default_rng(7)
    logits = np.full((6, 2051), -np.inf, np.float32)
    for r, n_finite in enumerate([1, 3, 20, 49, 51, 70]):
        idx = rng.choice(2051, n_finite, replace=False)
        logits[r, idx] = rng.standard_normal(n_finite).astype(np.float32)
    rows = np.arange(6)[None, :]
    for k in (5, 50, 64):
        picks = _both(gen, logits, k, 0.9, 1.0, seed=55, draws=8)
        assert np.isfinite(logits[rows, picks]).all()


def test_select_and_sort_agree_on_tied_logits(gen):
    rng = np.random.default_rng(11)
    # values on a 0.5 grid: dozens of exact ties inside and at the edge of the top-k
    logits = (np.round(2.0 * rng.standard_normal((8, 2051))) / 2.0).astype(np.float32)
    for k in (5, 50, 64):
        picks = _both(gen, logits, k, 0.9, 1.0, seed=77, draws=6)
        _check_oracle(logits, picks, k, 0.9, 1.0, 77)
    flat = np.zeros((4, 2051), np.float32)  # every logit tied: the top-k is indices 0..k-1
    picks = _both(gen, flat, 50, 0.9, 1.0, seed=3, draws=16)
    assert (picks < 50).all()


@pytest.mark.parametrize("V,k", [(40, 50), (40, 5), (64, 64), (64, 63), (65, 64)])
def test_select_and_sort_agree_on_small_vocabularies(gen, V, k):
    rng = np.random.default_rng(V * 100 + k)
    logits = (2.0 * rng.standard_normal((8, V))).astype(np.float32)
    picks = _both(gen, logits, k, 0.9, 1.0, seed=V + k, draws=8)
    assert (picks >= 0).all() and (picks < V).all()
    _check_oracle(logits, picks, k, 0.9, 1.0, V + k)
