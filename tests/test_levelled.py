"""The island sweeps levelled over a world's lanes (constraints that share no dynamic body solved at once, level after
level in pass order) against the parity oracle's one-after-another sweeps, bit for bit, on scenes whose islands are
large: piles that merge into one island (c2, sleeping off), many bullets resting on targets (c3), and the reference's
pile scene under the game's 300 velocity iterations. Needs a B200."""
import numpy as np
import pytest

import goldens
import oracle_lib
from test_oracle import assert_states_equal

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def api():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from goib2d import api
    return api


@pytest.mark.parametrize("mode", [1, 2])
@pytest.mark.parametrize("cfg,n,steps", [("c2", 5, 120), ("c3", 48, 60), ("c0", 32, 200)])
def test_levelled_sweeps_match_oracle(api, mode, cfg, n, steps):
    from goib2d import configs
    sc, model, host = configs.batch(cfg, n)
    eng = api.Engine(model, host.bodies.type.shape[1])
    try:
        eng.set_step_mode(mode)
        dev = api.to_device(host)
        eng.step_(dev, sc.settings, configs.DT, n_steps=steps)
        status = eng.status()
    finally:
        eng.close()
    want = oracle_lib.step(model, host, sc.settings, configs.DT, steps, threads=8)
    got = api.to_host(dev)
    assert_states_equal(got, want, f"{cfg} mode {mode}")
    assert ((status & 0b1011) == 0).all()
    if cfg == "c2":  # the pile has formed: islands far above the levelled path's threshold
        assert (got.contacts.touching.sum(1) > 100).all()


def test_levelled_sweeps_on_game_pile(api):
    """The reference's pile (game settings: 300 velocity and 30 position iterations), perturbed, 16 worlds."""
    g = goldens.Golden("game_pile")
    host = g.state(0, batch=16)
    rng = np.random.default_rng(21)
    dyn = (host.bodies.type == 2)[..., None]
    host.bodies.v[...] = np.where(dyn, host.bodies.v + rng.normal(0, 0.2, host.bodies.v.shape),
                                  host.bodies.v).astype(np.float32)
    dev = api.to_device(host)
    api.step_(g.model, dev, g.settings, g.dt, n_steps=40)
    want = oracle_lib.step(g.model, host, g.settings, g.dt, 40, threads=8)
    assert_states_equal(api.to_host(dev), want, "game_pile")
