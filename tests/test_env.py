"""The env helpers around the step (resets, observations, ray casts; no counterpart in the reference engine). CPU:
the oracle's ray casts give the distances geometry says. GPU: the device kernels equal the oracle and plain numpy."""
import numpy as np
import pytest

import edge_scenes
import oracle_lib
from goib2d.settings import Settings
from goib2d.world import DYNAMIC, STATIC, WorldDef, map_state

torch = pytest.importorskip("torch")


def _ray_scene():
    d = WorldDef(Settings.stock())
    g = d.add_body(STATIC)
    d.add_box(g, (5.0, 0.5), (0.0, -0.5))          # floor, top at y = 0
    d.add_edge(g, (3.0, -1.0), (3.0, 5.0))         # wall at x = 3
    d.add_circle(g, 1.0, (-4.0, 2.0))              # a disc left of the origin
    b = d.add_body(DYNAMIC, (0.0, 2.0), mass=1.0, inertia=0.1)
    d.add_circle(b, 0.2)
    return d.build(16)


def test_oracle_ray_distances_match_the_geometry():
    model, st = _ray_scene()
    f = oracle_lib.raycast(model, st, 1, 4, 10.0)[0]  # rays at 0, 90, 180, 270 degrees from (0, 2)
    assert abs(f[0] - 0.3) < 1e-6      # right: the wall at x = 3
    assert f[1] == 1.0                 # up: nothing within 10 m
    assert abs(f[2] - 0.3) < 1e-6      # left: the disc's near side at x = -3
    assert abs(f[3] - 0.2) < 2e-6      # down: the floor at y = 0 (the polygon cast ignores the skin)


@pytest.mark.gpu
def test_gpu_raycast_observe_equal_the_oracle_and_numpy():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from goib2d import api, configs
    for cfg, n in (("c1", 128), ("c1e", 128), ("c3e", 64)):
        sc, model, host = configs.batch(cfg, n)
        eng = api.Engine(model, host.bodies.type.shape[1], sc.action_joints, sc.action_scale)
        dev = api.to_device(host)
        eng.step_(dev, sc.settings, configs.DT, n_steps=10)
        now = api.to_host(dev)
        got = eng.raycast(dev, 1, 32, 8.0).cpu().numpy()
        want = oracle_lib.raycast(model, now, 1, 32, 8.0)
        assert np.array_equal(got, want), cfg
        assert (got < 1.0).any() and (got == 1.0).any()  # some rays hit the level, some do not
        obs = eng.observe(dev, [1, 2]).cpu().numpy()
        ref = np.concatenate([now.bodies.c[:, [1, 2]], now.bodies.a[:, [1, 2], None], now.bodies.v[:, [1, 2]],
                              now.bodies.w[:, [1, 2], None]], -1)
        assert np.array_equal(obs, ref), cfg


@pytest.mark.gpu
def test_gpu_resets_restore_the_initial_rows():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from goib2d import api, configs
    from goib2d.world import state_leaves
    sc, model, host = configs.batch("c4", 64)
    eng = api.Engine(model, host.bodies.type.shape[1], sc.action_joints, sc.action_scale)
    init = api.to_device(host)
    dev = api.to_device(host)
    eng.step_(dev, sc.settings, configs.DT, n_steps=20)
    before = api.to_host(dev)
    mask = torch.zeros(64, dtype=torch.bool, device="cuda")
    mask[::3] = True
    eng.reset_masked(dev, init, mask)
    after = api.to_host(dev)
    m = mask.cpu().numpy()
    for a, b, h in zip(state_leaves(after), state_leaves(before), state_leaves(host)):
        assert np.array_equal(np.asarray(a)[m], np.asarray(h)[m])
        assert np.array_equal(np.asarray(a)[~m], np.asarray(b)[~m])
    # reset on fall: push every other world's pot below y = -5 and reset those
    dev2 = api.to_device(before)
    c = dev2.bodies.c
    c[1::2, 1, 1] = -6.0
    counts = torch.zeros(64, dtype=torch.int32, device="cuda")
    eng.reset_below(dev2, init, 1, -5.0, counts)
    got = api.to_host(dev2)
    fell = (np.arange(64) % 2 == 1) | (before.bodies.c[:, 1, 1] < -5.0)
    assert np.array_equal(counts.cpu().numpy(), fell.astype(np.int32))
    for a, b, h in zip(state_leaves(got), state_leaves(before), state_leaves(host)):
        assert np.array_equal(np.asarray(a)[fell], np.asarray(h)[fell])
        assert np.array_equal(np.asarray(a)[~fell], np.asarray(b)[~fell])


@pytest.mark.gpu
def test_gpu_pinned_host_buffers_equal_device_buffers():
    """Actions read from pinned host memory and observations written into it by the kernels (no separate copy) give
    the same results as device buffers."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from goib2d import api, configs
    from goib2d.world import state_leaves
    sc, model, host = configs.batch("c1", 128)
    eng = api.Engine(model, host.bodies.type.shape[1], sc.action_joints, sc.action_scale)
    a = torch.from_numpy(np.random.default_rng(4).uniform(-2, 2, (5, 128, 2)).astype(np.float32))
    d1, d2 = api.to_device(host), api.to_device(host)
    a_pin = a.pin_memory()
    for k in range(5):
        eng.step_(d1, sc.settings, 0.02, 1, a[k].cuda())
        eng.step_(d2, sc.settings, 0.02, 1, a_pin[k])
    for x, y in zip(state_leaves(api.to_host(d1)), state_leaves(api.to_host(d2))):
        assert np.array_equal(np.asarray(x), np.asarray(y))
    out = torch.empty((128, 2, 6), dtype=torch.float32).pin_memory()
    eng.observe(d2, [1, 3], out=out)
    torch.cuda.synchronize()
    assert np.array_equal(out.numpy(), eng.observe(d2, [1, 3]).cpu().numpy())
    with pytest.raises(RuntimeError):  # pageable host memory cannot be read by a kernel
        eng.observe(d2, [1], out=torch.empty((128, 1, 6), dtype=torch.float32))
