"""Checkpoint / resume of a batched State (goib2d.checkpoint): saved leaves load back bit for bit, a malformed file
is refused, and stepping a resumed State continues exactly where the saved run stopped (on the oracle, and on the
GPU against an unbroken run)."""
import numpy as np
import pytest

import goldens
import oracle_lib
from goib2d import checkpoint, configs
from goib2d.world import leaf_names, state_leaves


def _same(a, b):
    for name, x, y in zip(leaf_names(), state_leaves(a), state_leaves(b)):
        x, y = np.asarray(x), np.asarray(y)
        assert x.dtype == y.dtype and x.shape == y.shape, name
        assert np.array_equal(x.view(np.uint8), y.view(np.uint8)), name


def test_round_trip_and_meta(tmp_path):
    _, _, st = configs.batch("c1", 5, device_pairs=False)
    p = tmp_path / "c1.npz"
    checkpoint.save_state(p, st, step=130, scene="c1_rig")
    back, meta = checkpoint.load_state(p)
    _same(st, back)
    assert int(meta["step"]) == 130 and str(meta["scene"]) == "c1_rig"


def test_resume_continues_the_run_on_the_oracle(tmp_path):
    """3 steps, save, load, 4 steps == 7 steps without a break (game-settings scene with TOI)."""
    g = goldens.Golden("game_late_wake")
    st = g.state(0, batch=3)
    mid = oracle_lib.step(g.model, st, g.settings, g.dt, 3)
    checkpoint.save_state(tmp_path / "mid.npz", mid)
    resumed, _ = checkpoint.load_state(tmp_path / "mid.npz")
    _same(oracle_lib.step(g.model, resumed, g.settings, g.dt, 4), oracle_lib.step(g.model, st, g.settings, g.dt, 7))


def test_malformed_files_are_refused(tmp_path):
    _, _, st = configs.batch("c0", 2, device_pairs=False)
    p = tmp_path / "ok.npz"
    checkpoint.save_state(p, st)
    with np.load(p) as f:
        good = {k: f[k] for k in f.files}
    bad = dict(good)
    del bad["contacts.key"]
    np.savez(tmp_path / "missing.npz", **bad)
    with pytest.raises(ValueError, match="missing leaves"):
        checkpoint.load_state(tmp_path / "missing.npz")
    bad = dict(good)
    bad["bodies.v"] = bad["bodies.v"].astype(np.float64)
    np.savez(tmp_path / "dtype.npz", **bad)
    with pytest.raises(ValueError, match="bodies.v"):
        checkpoint.load_state(tmp_path / "dtype.npz")
    bad = dict(good)
    bad["__format__"] = np.asarray("something-else")
    np.savez(tmp_path / "fmt.npz", **bad)
    with pytest.raises(ValueError, match="not a goib2d-state-v1"):
        checkpoint.load_state(tmp_path / "fmt.npz")
    with pytest.raises(ValueError, match="reserved"):
        checkpoint.save_state(tmp_path / "x.npz", st, **{"__format__": 1})


@pytest.mark.gpu
def test_resume_on_the_gpu_equals_an_unbroken_run(tmp_path):
    """A device State saved mid-run and loaded into a new engine steps on exactly as the unbroken run does."""
    from goib2d import api
    sc, model, host = configs.batch("c3", 64)
    eng = api.Engine(model, host.bodies.type.shape[1])
    try:
        a = api.to_device(host)
        eng.step_(a, sc.settings, configs.DT, n_steps=12)
        b = api.to_device(host)
        eng.step_(b, sc.settings, configs.DT, n_steps=5)
        checkpoint.save_state(tmp_path / "b.npz", b)
    finally:
        eng.close()
    c, _ = checkpoint.load_state(tmp_path / "b.npz", device="cuda")
    eng2 = api.Engine(model, host.bodies.type.shape[1])
    try:
        eng2.step_(c, sc.settings, configs.DT, n_steps=7)
        _same(api.to_host(c), api.to_host(a))
    finally:
        eng2.close()
