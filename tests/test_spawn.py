"""Scene spawn on the device (goib2d_spawn, goib2d_seed_placements): per-world initial States built on the GPU.

The reference builds every world on the host through WorldDef and stacks them (world.py:186-386); this repo's
host builder is pinned to it bit for bit (test_host.py). goib2d_spawn must give the State that builder gives for the
same poses, leaf for leaf, bit for bit; goib2d_seed_placements must equal the oracle's restatement of its generator
(Philox4x32-10, pinned to the published known-answer vectors), and its draws must depend only on (seed, world)."""
import ctypes as C

import numpy as np
import pytest

import oracle_lib
from goib2d import configs, native
from goib2d.world import state_leaves

CONFIGS = ("c0", "c1", "c2", "c3", "c4")
SMALL = {"c0": 64, "c1": 64, "c2": 8, "c3": 64, "c4": 32}


def _equal(a, b):
    for name, x, y in zip(_names(), state_leaves(a), state_leaves(b)):
        x, y = np.asarray(x), np.asarray(y)
        assert x.shape == y.shape and x.dtype == y.dtype, name
        assert np.array_equal(x.view(np.uint8), y.view(np.uint8)), name  # bit for bit (-0, NaN payloads)


def _names():
    from goib2d.world import leaf_names
    return leaf_names()


# ---- CPU: the generator's oracle, the host mapping, argument checks


def test_philox_known_answers():
    """Random123's known-answer vectors for Philox4x32-10."""
    kat = [((0, 0, 0, 0), 0, 0, (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
           ((0xFFFFFFFF,) * 4, 0xFFFFFFFF, 0xFFFFFFFF, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
           ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), 0xA4093822, 0x299F31D0,
            (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1))]
    for ctr, k0, k1, want in kat:
        assert tuple(int(x) for x in oracle_lib.philox4x32_10(ctr, k0, k1)) == want


@pytest.mark.parametrize("name", CONFIGS)
def test_placements_rebuild_the_same_worlds(name):
    """placements(scene) -> seeded_dyn -> the builder gives the scene's own worlds back (the mapping goib2d_spawn
    and the seeded path rely on)."""
    n = 3
    sc = configs.scene(name, 0, n)
    _, pl, joints, sp = configs.placements(sc)
    assert pl.shape == (n, {"c0": 8, "c2": 256, "c3": 32}.get(name, 3), 6) and pl.dtype == np.float32
    _, _, a = configs.batch(name, n, device_pairs=False)
    _, _, b = configs.batch(name, n, device_pairs=False,
                            dyn=configs.seeded_dyn(sc, pl, None if sp is None else sp[:, 0]))
    _equal(a, b)


@pytest.mark.parametrize("name", CONFIGS)
def test_seeded_draws_depend_only_on_seed_and_world(name):
    sc = configs.scene(name, 0, 1)
    rule, keep = configs.spawn_rule(sc, host=True)
    a, sa = oracle_lib.seed_placements(rule, 7, 0, 12)
    b, sb = oracle_lib.seed_placements(rule, 7, 5, 3)  # worlds 5..7 of the same scene
    assert np.array_equal(a[5:8], b)
    if sa is not None:
        assert np.array_equal(sa[5:8], sb)
    c, _ = oracle_lib.seed_placements(rule, 8, 0, 12)
    assert not np.array_equal(a, c)  # another seed, other worlds
    assert np.isfinite(a).all()
    if name in ("c0", "c3"):
        assert (a[..., 0] >= rule.x_lo).all() and (a[..., 0] < rule.x_hi).all()
        assert (a[..., 1] >= rule.y_lo).all() and (a[..., 1] < rule.y_hi).all()
    if name == "c3":
        speed = np.hypot(a[..., 3].astype(np.float64), a[..., 4].astype(np.float64))
        assert (speed > 49.99).all() and (speed < 200.01).all()
    if name == "c2":
        assert (np.abs(a[..., 0]) < 9.2).all() and (np.abs(a[..., 1]) < 9.2).all()
    if name in ("c1", "c4"):
        h, x0, dx = sc.level
        for w in range(len(a)):
            x, y = float(a[w, 0, 0]), float(a[w, 0, 1])
            i0, i1 = int((x - 0.8 - x0) / dx), int((x + 0.8 - x0) / dx) + 1
            assert abs(y - (float(np.max(h[i0:i1 + 1])) + 0.62)) < 1e-4  # resting on the ground under it
            assert all((x - px) ** 2 + (y - py) ** 2 > (r + 2.8) ** 2 - 1e-3 for px, py, r in sc.rocks)
            if name == "c4":
                assert float(np.min(h[i0:i1 + 1])) >= -3.0
            assert -2.0 <= sa[w] < 2.0 and 0.2 * np.pi - 1e-6 <= a[w, 1, 2] < 0.8 * np.pi + 1e-6
            hx, hy = a[w, 2, 0], a[w, 2, 1]
            assert abs(np.hypot(hx - a[w, 0, 0], hy - a[w, 0, 1]) - 1.0) < 1e-5  # the hammer one arm away


def test_seed_placements_rejects_bad_rules_without_a_gpu():
    lib = native.load()
    assert lib.goib2d_seed_placements(None, 0, 0, 1, None, None, None) == -1
    r = native.SpawnRule()
    r.kind = 7
    assert lib.goib2d_seed_placements(C.byref(r), 0, 0, 1, None, None, None) == -1
    r.kind, r.n_bodies, r.max_tries = native.SPAWN_RIG, 3, 0
    assert lib.goib2d_seed_placements(C.byref(r), 0, 0, 1, None, None, None) < 0
    assert b"max_tries" in lib.goib2d_last_error()
    r.kind, r.n_bodies = native.SPAWN_GRID, 4
    r.grid_side = 0
    assert lib.goib2d_seed_placements(C.byref(r), 0, 0, 1, None, None, None) == -1
    r.kind, r.grid_side = native.SPAWN_UNIFORM, 1
    assert lib.goib2d_seed_placements(C.byref(r), 0, -1, 1, None, None, None) == -1
    assert lib.goib2d_seed_placements(C.byref(r), 0, 0, 1, None, None, None) == -1  # null placements


# ---- GPU: the device spawn against the host builder, the device generator against the oracle


@pytest.mark.gpu
@pytest.mark.parametrize("name", CONFIGS)
def test_spawn_equals_the_host_builder(name):
    from goib2d import api
    n = SMALL[name]
    for first in (0, 37):
        _, model, dev, _, _ = configs.spawn_batch(name, n, first=first)
        _, model_h, host = configs.batch(name, n, first=first)
        _equal(api.to_host(dev), host)


@pytest.mark.gpu
@pytest.mark.parametrize("name", CONFIGS)
def test_seeded_placements_equal_the_oracle(name):
    import torch

    from goib2d import api
    sc = configs.scene(name, 0, 1)
    n = 64 if name == "c2" else 1024
    rule_d, keep_d = configs.spawn_rule(sc)
    rule_h, keep_h = configs.spawn_rule(sc, host=True)
    for seed, first in ((0, 0), (123456789012345, 1 << 33)):
        pl, sp = api.seed_placements(rule_d, seed, first, n)
        torch.cuda.synchronize()
        want, want_sp = oracle_lib.seed_placements(rule_h, seed, first, n)
        assert np.array_equal(pl.cpu().numpy().view(np.uint32), want.view(np.uint32))
        if want_sp is not None:
            assert np.array_equal(sp.cpu().numpy().view(np.uint32), want_sp.view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("name", CONFIGS)
def test_seeded_spawn_equals_the_host_builder(name):
    from goib2d import api
    n = SMALL[name]
    sc, model, dev, pl, sp = configs.spawn_batch(name, n, seed=3, first=11, seeded=True)
    dyn = configs.seeded_dyn(sc, pl.cpu().numpy(), None if sp is None else sp.cpu().numpy())
    _, model_h, host = configs.batch(name, n, seed=3, first=11, dyn=dyn)
    _equal(api.to_host(dev), host)
    assert np.array_equal(model.reference_angle, model_h.reference_angle)


@pytest.mark.gpu
@pytest.mark.parametrize("name", ("c1", "c3"))
def test_spawned_worlds_step_like_the_oracle(name):
    """A device-seeded batch steps on the GPU exactly as the oracle steps the same worlds built on the host."""
    from goib2d import api
    n, steps = 48, 6
    sc, model, dev, pl, sp = configs.spawn_batch(name, n, seed=5, seeded=True)
    host = api.to_host(dev)
    want = oracle_lib.step(model, host, sc.settings, configs.DT, steps)
    eng = api.Engine(model, host.bodies.type.shape[1])
    try:
        eng.step_(dev, sc.settings, configs.DT, n_steps=steps)
        _equal(api.to_host(dev), want)
    finally:
        eng.close()


@pytest.mark.gpu
def test_spawn_rejects_bad_arguments():
    import torch

    from goib2d import api
    sc, model, host = configs.batch("c1", 1)
    eng = api.Engine(model, host.bodies.type.shape[1])
    try:
        tmpl = api.to_device(host)
        with pytest.raises(RuntimeError, match="placed bodies"):
            eng.spawn(tmpl, 4, 2, torch.zeros(4, 3, 6, device="cuda"))  # bodies 2..4 of 4
        with pytest.raises(RuntimeError, match="16 at most"):
            eng.spawn(tmpl, 4, 1, torch.zeros(4, 3, 6, device="cuda"), [0] * 17,
                      torch.zeros(4, 17, device="cuda"))
        with pytest.raises(RuntimeError, match="out of range"):
            eng.spawn(tmpl, 4, 1, torch.zeros(4, 3, 6, device="cuda"), (5,), torch.zeros(4, 1, device="cuda"))
        out = eng.spawn(tmpl, 0, 1, torch.zeros(0, 3, 6, device="cuda"))  # an empty batch launches nothing
        assert out.bodies.type.shape == (0, 4)
    finally:
        eng.close()
