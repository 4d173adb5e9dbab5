"""The CUDA engine (libgoib2d.so through the C ABI) against the reference engine's states (tests/golden) and the
parity oracle, bit for bit: every leaf of every world after every checkpoint. Needs a B200."""
import numpy as np
import pytest

import goldens
import oracle_lib
from test_oracle import assert_states_equal

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

NAMES = goldens.names()


@pytest.fixture(scope="module")
def api():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from goib2d import api
    return api


def world(state, i):
    from goib2d.world import map_state
    return map_state(lambda x: np.asarray(x)[i], state)


@pytest.mark.parametrize("name", NAMES)
def test_gpu_matches_reference(api, name):
    """Three copies of the scene stepped on the GPU equal the reference's own states at every checkpoint."""
    g = goldens.Golden(name)
    dev = api.to_device(g.state(0, batch=3))
    prev = 0
    for k in g.checkpoints[1:]:
        api.step_(g.model, dev, g.settings, g.dt, n_steps=k - prev)
        prev = k
        host = api.to_host(dev)
        for i in range(3):
            assert_states_equal(world(host, i), g.state(k), f"{name} world {i} step {k}")


def _perturbed(g, n, seed, scale):
    host = g.state(0, batch=n)
    rng = np.random.default_rng(seed)
    dyn = (host.bodies.type == 2)[..., None]
    host.bodies.v[...] = np.where(dyn, host.bodies.v + rng.normal(0, scale, host.bodies.v.shape),
                                  host.bodies.v).astype(np.float32)
    host.bodies.w[...] = np.where(dyn[..., 0], host.bodies.w + rng.normal(0, scale, host.bodies.w.shape),
                                  host.bodies.w).astype(np.float32)
    return host


@pytest.mark.parametrize("name,n,steps", [("stock_pile", 64, 40), ("game_pile", 16, 20), ("game_revolute", 32, 20),
                                          ("game_prismatic", 32, 20), ("game_weld", 32, 20), ("game_misc", 32, 20),
                                          ("game_limits_mid_run", 32, 30), ("game_polygons_at_angles", 32, 20),
                                          ("game_polygon_circle", 32, 20), ("game_box_on_ground", 32, 20),
                                          ("toi_island_walk", 32, 15), ("toi_multi_event", 32, 15),
                                          ("toi_poly_angles", 32, 15), ("toi_hammer_chain", 32, 15)])
def test_gpu_matches_oracle_on_perturbed_batches(api, name, n, steps):
    """Every world of a batch with per-world perturbed velocities equals the oracle (the batch is independent)."""
    g = goldens.Golden(name)
    host = _perturbed(g, n, 11, 0.3)
    dev = api.to_device(host)
    api.step_(g.model, dev, g.settings, g.dt, n_steps=steps)
    want = oracle_lib.step(g.model, host, g.settings, g.dt, steps, threads=8)
    assert_states_equal(api.to_host(dev), want, name)


@pytest.mark.parametrize("cfg,n,steps", [("c0", 64, 60), ("c1", 256, 40), ("c2", 8, 10), ("c3", 128, 20),
                                         ("c4", 64, 20)])
def test_gpu_matches_oracle_on_workloads(api, cfg, n, steps):
    """The benchmark workloads (batched, seeded worlds) on the GPU equal the oracle world for world."""
    from goib2d import configs
    sc, model, host = configs.batch(cfg, n)
    dev = api.to_device(host)
    eng = api.engine_for(model, host.bodies.type.shape[1])
    eng.step_(dev, sc.settings, configs.DT, n_steps=steps)
    want = oracle_lib.step(model, host, sc.settings, configs.DT, steps, threads=8)
    assert_states_equal(api.to_host(dev), want, cfg)
    assert ((eng.status() & 0b1011) == 0).all()  # no overflow, no non-finite state, no table limit


@pytest.mark.parametrize("name,n,steps", [("circle_on_edge", 8, 120), ("box_on_chain", 16, 120),
                                          ("box_on_edges", 16, 120), ("slope_chain", 32, 200),
                                          ("bullet_at_edge", 8, 30)])
def test_gpu_matches_oracle_on_edge_scenes(api, name, n, steps):
    """Edge and chain shapes (this engine's own; no reference states exist): perturbed batches on the GPU equal
    the oracle's restatement of the same method, bit for bit."""
    import edge_scenes
    from goib2d.world import map_state
    model, st = edge_scenes.build(name, 64)
    settings = edge_scenes.SCENES[name]().settings
    host = map_state(lambda x: np.ascontiguousarray(np.repeat(np.asarray(x)[None], n, 0)), st)
    rng = np.random.default_rng(7)
    dyn = (host.bodies.type == 2)[..., None]
    host.bodies.v[...] = np.where(dyn, host.bodies.v + rng.normal(0, 0.4, host.bodies.v.shape), host.bodies.v)
    dev = api.to_device(host)
    api.step_(model, dev, settings, edge_scenes.DT, n_steps=steps)
    want = oracle_lib.step(model, host, settings, edge_scenes.DT, steps, threads=8)
    assert_states_equal(api.to_host(dev), want, name)


@pytest.mark.parametrize("cfg,n,steps", [("c0e", 64, 60), ("c1e", 256, 40), ("c3e", 128, 20)])
def test_gpu_matches_oracle_on_edge_workloads(api, cfg, n, steps):
    """BASELINE's own levels with edge shapes (chain terrain, lone edge targets) equal the oracle world for world."""
    from goib2d import configs
    sc, model, host = configs.batch(cfg, n)
    dev = api.to_device(host)
    eng = api.engine_for(model, host.bodies.type.shape[1])
    eng.step_(dev, sc.settings, configs.DT, n_steps=steps)
    want = oracle_lib.step(model, host, sc.settings, configs.DT, steps, threads=8)
    assert_states_equal(api.to_host(dev), want, cfg)
    assert ((eng.status() & 0b1011) == 0).all()


@pytest.mark.parametrize("mode", [1, 2])
@pytest.mark.parametrize("cfg,n,steps", [("c0", 63, 40), ("c1", 255, 30), ("c2", 7, 8), ("c3", 127, 20),
                                         ("c4", 63, 20), ("c1e", 129, 20)])
def test_step_modes_match_oracle(api, mode, cfg, n, steps):
    """The one-launch step with one world per warp (mode 1) and with two worlds per warp, one per half-warp (mode 2),
    equals the oracle world for world; odd batches leave a half-warp without a world."""
    from goib2d import configs
    sc, model, host = configs.batch(cfg, n)
    dev = api.to_device(host)
    eng = api.Engine(model, host.bodies.type.shape[1])
    try:
        eng.set_step_mode(mode)
        eng.step_(dev, sc.settings, configs.DT, n_steps=steps)
        status = eng.status()
    finally:
        eng.close()
    want = oracle_lib.step(model, host, sc.settings, configs.DT, steps, threads=8)
    assert_states_equal(api.to_host(dev), want, f"{cfg} mode {mode}")
    assert ((status & 0b1011) == 0).all()


def test_kernels_per_step(api):
    """One launch per step, except large batches of models with many joints (six part kernels)."""
    from goib2d import configs
    for cfg, n, want in (("c1", 4096, 1), ("c1", 1 << 16, 1), ("c4", 8192, 1), ("c4", 1 << 16, 6)):
        sc, model, host = configs.batch(cfg, 2)
        eng = api.Engine(model, host.bodies.type.shape[1])
        try:
            assert eng.kernels_per_step(n) == want, (cfg, n)
        finally:
            eng.close()


def test_bench_batch_matches_oracle(api):
    """The benchmark's batch (c1, 4096 worlds: two worlds per warp by the per-batch choice) equals the oracle on
    worlds from both ends of the batch."""
    from goib2d import configs
    from goib2d.world import map_state
    n, steps = 4096, 12
    sc, model, host = configs.batch("c1", n)
    dev = api.to_device(host)
    eng = api.engine_for(model, host.bodies.type.shape[1])
    eng.step_(dev, sc.settings, configs.DT, n_steps=steps)
    got = api.to_host(dev)
    pick = np.r_[0:64, 2048:2080, n - 64:n]
    want = oracle_lib.step(model, map_state(lambda x: np.ascontiguousarray(np.asarray(x)[pick]), host), sc.settings,
                           configs.DT, steps, threads=8)
    assert_states_equal(map_state(lambda x: np.asarray(x)[pick], got), want, f"c1 n={n}")
    assert ((eng.status() & 0b1011) == 0).all()


@pytest.mark.parametrize("cfg,steps", [("c1", 12), ("c4", 6)])
def test_large_batches_match_oracle(api, cfg, steps):
    """Large batches (16384 worlds) equal the oracle on worlds taken from both ends of the batch: c1 as one launch
    per step (two worlds per warp), c4 (22 joints) as part kernels with the constraint sweeps one world per thread."""
    from goib2d import configs
    from goib2d.world import map_state
    n = 16384
    sc, model, host = configs.batch(cfg, n)
    dev = api.to_device(host)
    eng = api.engine_for(model, host.bodies.type.shape[1])
    eng.step_(dev, sc.settings, configs.DT, n_steps=steps)
    got = api.to_host(dev)
    pick = np.r_[0:96, n - 96:n]
    want = oracle_lib.step(model, map_state(lambda x: np.ascontiguousarray(np.asarray(x)[pick]), host), sc.settings,
                           configs.DT, steps, threads=8)
    assert_states_equal(map_state(lambda x: np.asarray(x)[pick], got), want, f"{cfg} n={n}")
    assert ((eng.status() & 0b1011) == 0).all()


def test_actions_drive_joint_motors(api):
    """The action channels set joints.motor_speed before each step, as the oracle does."""
    from goib2d import configs
    sc, model, host = configs.batch("c1", 64)
    rng = np.random.default_rng(3)
    r, th = 2 * np.sqrt(rng.uniform(0, 1, 64)), rng.uniform(0, 2 * np.pi, 64)
    act = np.stack([r * np.cos(th), r * np.sin(th)], 1).astype(np.float32)
    eng = api.Engine(model, host.bodies.type.shape[1], sc.action_joints, sc.action_scale)
    dev = api.to_device(host)
    eng.step_(dev, sc.settings, configs.DT, n_steps=5, actions=torch.from_numpy(act).cuda())
    want = oracle_lib.step(model, host, sc.settings, configs.DT, 5, threads=8, actions=act,
                           action_joints=sc.action_joints, action_scale=sc.action_scale)
    assert_states_equal(api.to_host(dev), want, "c1 actions")
    assert np.allclose(api.to_host(dev).joints.motor_speed[:, 0], act[:, 0] * np.float32(4.0))


def test_pure_step_and_single_world(api):
    """step() is pure and accepts a single-world State (the reference's unbatched call)."""
    g = goldens.Golden("stock_box_stack")
    one = api.to_device(g.state(0))
    out = api.step(g.model, one, g.settings, g.dt)
    assert_states_equal(api.to_host(one), g.state(0), "input unchanged")
    assert_states_equal(api.to_host(out), g.state(1), "one step")


def test_errors_are_reported_not_trapped(api):
    """Bad layouts come back as error codes with a message; an empty batch is a no-op."""
    from goib2d import native
    g = goldens.Golden("stock_box_stack")
    dev = api.to_device(g.state(0, batch=2))
    bad = dev._replace(fixtures=dev.fixtures._replace(friction=dev.fixtures.friction[:, :1].contiguous()))
    with pytest.raises(RuntimeError, match="fixture rows"):
        api.step_(g.model, bad, g.settings, g.dt)
    empty = api.to_device(g.state(0, batch=0))
    api.step_(g.model, empty, g.settings, g.dt)
    assert native.load().goib2d_version() == 2
