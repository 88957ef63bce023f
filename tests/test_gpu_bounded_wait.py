"""Bounded device waits give up cleanly (needs a B200).

Every spin-wait in the kernels has a poll limit. When it runs out, the kernel records an error
code, lets the copies and tensor-core operations it issued land, frees its tensor memory and
returns; the host reports the code through the C ABI (-1 and breeze_last_error()) and clears it,
so the generator stays usable. These tests make waits run out without any fault: a barrier that
nothing arrives on, and the persistent depth decoder's grid barriers given a limit of a few
polls, so that CTAs stop waiting for the others before the others arrive.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_mbarrier_wait_gives_up_and_records_its_code(pkg):
    assert pkg.mbar_timeout_probe(1000) == 1
    assert pkg.mbar_timeout_probe(1) == 1


def test_depth_grid_barrier_timeout_is_reported_and_recovered(pkg, tiny_model, tiny_oracle):
    cfg = tiny_oracle.cfg
    gen = pkg.GeneratorHandle(tiny_model, 0)
    try:
        rng = np.random.default_rng(9)
        hidden = rng.standard_normal((6, cfg.hidden)).astype(np.float32)
        cb0 = rng.integers(0, 2048, 6)
        codes, logits = gen.debug_depth(hidden, cb0, cfg.vs)
        gen.set_debug_grid_spin(2)
        with pytest.raises(RuntimeError, match="bounded wait timed out"):
            gen.debug_depth(hidden, cb0, cfg.vs)
        err = gen.lib.last_error()
        assert "device error code" in err, err
        gen.set_debug_grid_spin(0)
        # the error word was cleared: the same launch gives the same codes and logits again
        codes2, logits2 = gen.debug_depth(hidden, cb0, cfg.vs)
        assert np.array_equal(codes2, codes) and np.array_equal(logits2, logits)
        # and the frame step still runs
        gen.session_create_ext(5, pkg.ids_to_text([300, 301, 302]), seed=1, max_new_tokens=4)
        n_exec, frames, nxt = gen.step_frames([5], 2, [1])
        assert n_exec == 2 and (frames[:, 0, 0] >= 0).all()
    finally:
        gen.close()
