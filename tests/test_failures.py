"""Failure paths, made on the host and reported by the kernels as status words (never a trap): a contact table too
small for the scene (overflow, reference goi_jax/box2d/pairs.py:176-178) and a non-finite body state. The GPU tests
compare with the oracle; nothing here faults or hangs a GPU."""
import numpy as np
import pytest

import goldens
import oracle_lib
from test_oracle import assert_states_equal

ST_OVERFLOW, ST_NONFINITE, ST_CAP, ST_LIMIT = 1, 2, 4, 8


def with_capacity(state, C):
    """The State with its contact table cut to C slots (every slot from C on must be free)."""
    from goib2d import native
    from goib2d.world import leaf_names, state_from_leaves, state_leaves
    B = state.bodies.type.shape[1]
    rows, J, C0 = state.fixtures.friction.shape[1], state.joints.motor_speed.shape[1], state.contacts.pair.shape[1]
    assert (np.asarray(state.contacts.pair)[:, C:] < 0).all()
    out = []
    for name, leaf, (_, shape, _) in zip(leaf_names(), state_leaves(state), native.leaf_spec(B, rows, J, C0)):
        c_dim = (name.startswith("contacts.") or (name.startswith("toi.") and name not in ("toi.alpha0", "toi.events")))
        out.append(np.ascontiguousarray(np.asarray(leaf)[:, :C]) if c_dim else np.asarray(leaf).copy())
    return state_from_leaves(out)


def test_overflow_on_the_oracle_matches_the_reference_rule():
    """CPU: with 2 slots the stack's new contacts overflow; State.overflow counts the pairs that found no free slot
    and every slot is taken (pairs.py:160-178)."""
    g = goldens.Golden("stock_box_stack")
    st = with_capacity(g.state(0, batch=2), 2)
    out = oracle_lib.step(g.model, st, g.settings, g.dt, 3)
    assert (out.overflow > 0).all()
    assert (out.contacts.pair >= 0).all()


@pytest.mark.gpu
def test_gpu_overflow_status_and_counts_match_oracle():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from goib2d import api
    g = goldens.Golden("stock_box_stack")
    host = with_capacity(g.state(0, batch=8), 2)
    steps = 10
    for mode in (1, 2):
        eng = api.Engine(g.model, host.bodies.type.shape[1])
        try:
            eng.set_step_mode(mode)
            dev = api.to_device(host)
            eng.step_(dev, g.settings, g.dt, steps)
            status = eng.status()
        finally:
            eng.close()
        want = oracle_lib.step(g.model, host, g.settings, g.dt, steps)
        got = api.to_host(dev)
        assert_states_equal(got, want, f"overflow mode {mode}")
        assert (got.overflow > 0).all()
        assert ((status & ST_OVERFLOW) != 0).all()
        assert ((status & (ST_NONFINITE | ST_LIMIT)) == 0).all()


@pytest.mark.gpu
def test_gpu_nonfinite_state_is_flagged_on_its_world_only():
    """A NaN written into one world's body velocity on the host: that world reports ST_NONFINITE after the call,
    every other world equals the oracle and reports nothing."""
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from goib2d import api, configs
    from goib2d.world import map_state
    n, bad, steps = 64, 13, 6
    sc, model, host = configs.batch("c1", n)
    host.bodies.v[bad, 1, 0] = np.float32(np.nan)
    for mode in (1, 2):
        eng = api.Engine(model, host.bodies.type.shape[1])
        try:
            eng.set_step_mode(mode)
            dev = api.to_device(host)
            eng.step_(dev, sc.settings, configs.DT, steps)
            status = eng.status()
        finally:
            eng.close()
        assert status[bad] & ST_NONFINITE
        others = np.r_[0:bad, bad + 1:n]
        assert ((status[others] & (ST_NONFINITE | ST_OVERFLOW | ST_LIMIT)) == 0).all()
        got = map_state(lambda x: np.asarray(x)[others], api.to_host(dev))
        want = oracle_lib.step(model, map_state(lambda x: np.ascontiguousarray(np.asarray(x)[others]), host),
                               sc.settings, configs.DT, steps, threads=8)
        assert_states_equal(got, want, f"nan mode {mode}")
