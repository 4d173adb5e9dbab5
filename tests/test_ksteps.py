"""The persistent K-step launch (goib2d_step_seq / goib2d_step with n_steps > 1: one kernel runs every step of the
call) against K separate one-step calls and the parity oracle, bit for bit. Needs a B200."""
import numpy as np
import pytest

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


def disc_actions(k, n, seed):
    rng = np.random.default_rng(seed)
    r, th = 2 * np.sqrt(rng.uniform(0, 1, (k, n))), rng.uniform(0, 2 * np.pi, (k, n))
    return np.stack([r * np.cos(th), r * np.sin(th)], -1).astype(np.float32)


def oracle_per_step(model, host, sc, dt, acts):
    st = host
    for a in acts:
        st = oracle_lib.step(model, st, sc.settings, dt, 1, threads=8, actions=a, action_joints=sc.action_joints,
                             action_scale=sc.action_scale)
    return st


@pytest.mark.parametrize("mode", [1, 2])
@pytest.mark.parametrize("where", ["device", "pinned"])
def test_per_step_actions_in_one_launch(api, mode, where):
    """K = 12 steps in one call, each step reading its own (N, 2) row of a (K, N, 2) action buffer, equal the oracle
    stepped one step at a time with the same rows."""
    from goib2d import configs
    n, K = 200, 12
    sc, model, host = configs.batch("c1", n)
    acts = disc_actions(K, n, 4)
    eng = api.Engine(model, host.bodies.type.shape[1], sc.action_joints, sc.action_scale)
    try:
        eng.set_step_mode(mode)
        assert eng.launches(n, K) == 1
        t = torch.from_numpy(acts)
        t = t.cuda() if where == "device" else t.pin_memory()
        dev = api.to_device(host)
        eng.step_(dev, sc.settings, configs.DT, n_steps=K, actions=t)
        torch.cuda.synchronize()
        got = api.to_host(dev)
    finally:
        eng.close()
    assert_states_equal(got, oracle_per_step(model, host, sc, configs.DT, acts), f"c1 K={K} mode {mode} {where}")
    assert np.array_equal(got.joints.motor_speed[:, 0], acts[-1, :, 0] * np.float32(4.0))


@pytest.mark.parametrize("mode", [1, 2])
@pytest.mark.parametrize("cfg,n,K", [("c0", 100, 30), ("c1", 300, 25), ("c3", 96, 15), ("c4", 40, 10),
                                     ("c1e", 64, 20)])
def test_k_step_launch_equals_single_steps(api, mode, cfg, n, K):
    """One call of K steps (one launch) and K calls of one step give the same State, status words and last-step
    event log, bit for bit."""
    from goib2d import configs
    sc, model, host = configs.batch(cfg, n)
    na = len(sc.action_joints)
    acts = torch.from_numpy(disc_actions(K, n, 8)).cuda() if na else None
    results = []
    for split in (False, True):
        eng = api.Engine(model, host.bodies.type.shape[1], sc.action_joints, sc.action_scale)
        try:
            eng.set_step_mode(mode)
            eng.set_event_log(64)
            dev = api.to_device(host)
            if split:
                status = np.zeros(n, np.int32)
                for k in range(K):
                    eng.step_(dev, sc.settings, configs.DT, 1, acts[k] if na else None)
                    status |= eng.status()
            else:
                eng.step_(dev, sc.settings, configs.DT, K, acts)
                status = eng.status()
            ev, cnt = eng.events()
            results.append((api.to_host(dev), status, ev, cnt))
        finally:
            eng.close()
    (a, sa, ea, ca), (b, sb, eb, cb) = results
    assert_states_equal(a, b, f"{cfg} K={K} mode {mode}")
    assert np.array_equal(ca, cb)
    for w in range(n):
        assert ea[w, :min(ca[w], 64)].tobytes() == eb[w, :min(cb[w], 64)].tobytes(), (cfg, w)
    # status: bit 0 (overflow) and bit 2 (cap) are sticky over the call; bit 1 (non-finite) is the end state's
    assert np.array_equal(sa & ~2, sb & ~2)


def test_launch_counts(api):
    """One launch per call for the one-kernel step, six per step for the part-kernel batches."""
    from goib2d import configs
    for cfg, n, K, want in (("c1", 4096, 10, 1), ("c1", 1 << 16, 10, 1), ("c4", 8192, 7, 1),
                            ("c4", 1 << 16, 7, 42), ("c1", 0, 10, 0), ("c1", 4096, 0, 0)):
        sc, model, host = configs.batch(cfg, 2)
        eng = api.Engine(model, host.bodies.type.shape[1])
        try:
            assert eng.launches(n, K) == want, (cfg, n, K)
        finally:
            eng.close()
