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


def joints_scene():
    """One world of 24 independent jointed bodies (revolute with motor and limits, prismatic with limits, weld, motor
    joint) hanging from the static ground, with loose boxes falling among them: a large constraint set with many
    constraints per level, so the levelled sweeps solve every joint type."""
    from goib2d import DYNAMIC, STATIC, Settings, WorldDef
    d = WorldDef(Settings.stock(gravity=(0.0, -10.0)))
    g = d.add_body(STATIC)
    d.add_box(g, (30.0, 0.5), center=(0.0, -6.0))
    for i in range(24):
        x = -23.0 + 2.0 * i
        b = d.add_body(DYNAMIC, (x + 0.6, 2.0), 0.1 * i, mass=1.0, inertia=0.2, allow_sleep=False)
        d.add_box(b, (0.5, 0.15), friction=0.4)
        k = i % 4
        if k == 0:
            d.add_revolute(g, b, (x, 2.0), (-0.6, 0.0), limits=(-0.8, 0.8), motor_speed=1.5, max_motor_torque=3.0,
                           enable_motor=True)
        elif k == 1:
            d.add_prismatic(g, b, (x, 2.0), (0.0, 0.0), axis=(0.3, 1.0), limits=(-1.0, 0.5), motor_speed=-0.5,
                            max_motor_force=4.0, enable_motor=True)
        elif k == 2:
            d.add_weld(g, b, (x, 2.0), (-0.6, 0.0), frequency=4.0, damping=0.5)
        else:
            d.add_motor(g, b, (x + 0.5, 1.0), 0.4, max_force=20.0, max_torque=5.0)
        c = d.add_body(DYNAMIC, (x + 0.6, 4.0 + 0.3 * k), 0.0, mass=0.5, inertia=0.05, allow_sleep=False)
        d.add_box(c, (0.2, 0.2), friction=0.5)
    return d


@pytest.mark.parametrize("mode", [1, 2])
def test_levelled_sweeps_with_every_joint_type(api, mode):
    from goib2d.world import map_state
    d = joints_scene()
    model, st = d.build(96)
    n = 8
    host = map_state(lambda x: np.ascontiguousarray(np.repeat(np.asarray(x)[None], n, 0)), st)
    rng = np.random.default_rng(23)
    dyn = (host.bodies.type == 2)[..., None]
    host.bodies.v[...] = np.where(dyn, rng.normal(0, 0.5, host.bodies.v.shape), host.bodies.v).astype(np.float32)
    dt = np.float32(1.0 / 60.0)
    eng = api.Engine(model, host.bodies.type.shape[1])
    try:
        eng.set_step_mode(mode)
        dev = api.to_device(host)
        eng.step_(dev, d.settings, dt, n_steps=90)
        got = api.to_host(dev)
    finally:
        eng.close()
    want = oracle_lib.step(model, host, d.settings, dt, 90, threads=8)
    assert_states_equal(got, want, f"joints mode {mode}")
    assert (got.contacts.touching.sum(1) > 4).all()  # the loose boxes landed on the jointed ones or the ground


def wide_level_scene():
    """One world of 40 boxes resting on the static ground, every fourth with a second box on top: the first level of
    each pass holds at least 40 contacts, more than a world's lanes, the second the stacked ones."""
    from goib2d import DYNAMIC, STATIC, Settings, WorldDef
    d = WorldDef(Settings.stock(gravity=(0.0, -10.0), allow_sleep=False))
    g = d.add_body(STATIC)
    d.add_box(g, (60.0, 0.5), center=(0.0, -0.5))
    for i in range(40):
        x = -48.0 + 2.4 * i
        b = d.add_body(DYNAMIC, (x, 0.49), 0.0, mass=1.0, inertia=0.2)
        d.add_box(b, (0.5, 0.5), friction=0.6)
        if i % 4 == 0:
            c = d.add_body(DYNAMIC, (x + 0.1, 1.48), 0.0, mass=0.5, inertia=0.1)
            d.add_box(c, (0.4, 0.5), friction=0.6)
    return d


@pytest.mark.parametrize("mode", [1, 2])
def test_levelled_sweeps_with_levels_wider_than_the_lanes(api, mode):
    from goib2d.world import map_state
    d = wide_level_scene()
    model, st = d.build(128)
    n = 6
    host = map_state(lambda x: np.ascontiguousarray(np.repeat(np.asarray(x)[None], n, 0)), st)
    rng = np.random.default_rng(29)
    dyn = (host.bodies.type == 2)[..., None]
    host.bodies.v[...] = np.where(dyn, rng.normal(0, 0.3, host.bodies.v.shape), host.bodies.v).astype(np.float32)
    dt = np.float32(1.0 / 60.0)
    eng = api.Engine(model, host.bodies.type.shape[1])
    try:
        eng.set_step_mode(mode)
        dev = api.to_device(host)
        eng.step_(dev, d.settings, dt, n_steps=60)
        got = api.to_host(dev)
    finally:
        eng.close()
    want = oracle_lib.step(model, host, d.settings, dt, 60, threads=8)
    assert_states_equal(got, want, f"wide levels mode {mode}")
    assert (got.contacts.touching.sum(1) >= 50).all()
