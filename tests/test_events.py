"""The contact event log (the reference C API's Begin / End / PostSolve listener, goi_jax/reference/capi.cpp:45-78,
838-847; the reference JAX engine has none). CPU: the oracle's log follows Box2D's listener semantics on simple
scenes and changes no result. GPU: the device log equals the oracle's, event for event."""
import numpy as np
import pytest

import edge_scenes
import goldens
import oracle_lib
from goib2d import native
from goib2d.world import map_state, state_leaves

BEGIN, END, POST = 0, 1, 2


def _run(model, st, settings, dt, steps, cap=32):
    out, logs = st, []
    for _ in range(steps):
        out, ev, cnt = oracle_lib.step_events(model, out, settings, dt, 1, cap)
        logs.append([ev[w, :min(int(cnt[w]), cap)] for w in range(len(cnt))])
    return out, logs


def test_a_landing_circle_begins_touching_then_reports_impulses():
    model, st = edge_scenes.build("circle_on_edge")
    s = edge_scenes.circle_on_edge().settings
    _, logs = _run(model, oracle_lib.batched(st), s, edge_scenes.DT, 90)
    kinds = [[int(e["kind"]) for e in step[0]] for step in logs]
    first = next(i for i, k in enumerate(kinds) if k)
    assert kinds[first][0] == BEGIN and all(k == [] for k in kinds[:first])
    assert POST in kinds[first]  # the touching contact is solved in the same step
    later = [step[0] for step in logs[first + 1:]]
    # resting: one PostSolve per step and no Begin / End, until the body sleeps (a sleeping island is not solved)
    assert all(len(e) <= 1 and all(x["kind"] == POST for x in e) for e in later)
    awake = [i for i, e in enumerate(later) if len(e)]
    assert len(awake) > 10 and all(later[i][0]["normal_impulse"][0] > 0 and later[i][0]["count"] == 1 for i in awake)
    assert awake == list(range(len(awake)))  # reported every step until it sleeps, then silent
    assert int(logs[first][0][0]["fixture_a"]) == 0 and int(logs[first][0][0]["fixture_b"]) == 1  # edge, circle


def test_the_log_changes_no_result():
    g = goldens.Golden("toi_multi_event")
    st = g.state(0, batch=4)
    with_log, _ = _run(g.model, st, g.settings, g.dt, 20)
    plain = oracle_lib.step(g.model, st, g.settings, g.dt, 20)
    for a, b in zip(state_leaves(with_log), state_leaves(plain)):
        assert np.array_equal(np.asarray(a), np.asarray(b))


def test_end_events_follow_separation():
    """A stack knocked over: every contact that ends touching raises an End, each after its Begin."""
    g = goldens.Golden("game_pile")
    st = oracle_lib.batched(g.state(0))
    _, logs = _run(g.model, st, g.settings, g.dt, 120, cap=256)
    open_ = set()
    n_end = 0
    for step in logs:
        for e in step[0]:
            key = (int(e["fixture_a"]), int(e["fixture_b"]))
            if e["kind"] == BEGIN:
                assert key not in open_
                open_.add(key)
            elif e["kind"] == END:
                assert key in open_
                open_.discard(key)
                n_end += 1
            else:
                assert key in open_  # PostSolve only for touching contacts
    assert n_end > 0


@pytest.mark.gpu
@pytest.mark.parametrize("name,n,steps", [("game_pile", 8, 60), ("toi_multi_event", 16, 30),
                                          ("toi_hammer_chain", 16, 30), ("c1", 64, 40), ("c1e", 64, 40)])
def test_gpu_event_log_equals_the_oracle(name, n, steps):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from goib2d import api, configs
    if name.startswith("c"):
        sc, model, host = configs.batch(name, n)
        settings, dt = sc.settings, configs.DT
    else:
        g = goldens.Golden(name)
        model, settings, dt = g.model, g.settings, g.dt
        host = g.state(0, batch=n)
        rng = np.random.default_rng(3)
        dyn = (host.bodies.type == 2)[..., None]
        host.bodies.v[...] = np.where(dyn, host.bodies.v + rng.normal(0, 0.3, host.bodies.v.shape),
                                      host.bodies.v).astype(np.float32)
    cap = 64
    eng = api.Engine(model, host.bodies.type.shape[1])
    eng.set_event_log(cap)
    dev = api.to_device(host)
    want_state = host
    for k in range(steps):
        eng.step_(dev, settings, dt, 1)
        want_state, want_ev, want_cnt = oracle_lib.step_events(model, want_state, settings, dt, 1, cap, threads=8)
        got_ev, got_cnt = eng.events()
        assert np.array_equal(got_cnt, want_cnt), (name, k)
        for w in range(n):
            m = min(int(want_cnt[w]), cap)
            assert got_ev[w, :m].tobytes() == want_ev[w, :m].tobytes(), (name, k, w)
    for a, b in zip(state_leaves(api.to_host(dev)), state_leaves(want_state)):
        assert np.array_equal(np.asarray(a), np.asarray(b))
