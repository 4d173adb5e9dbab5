"""State rows staged in shared memory across a one-launch call (goib2d_set_state_staging): with every row that fits
staged, with a few hundred bytes (the world scalars and some body rows only) and with none, the CUDA engine equals the
parity oracle bit for bit, in both world-to-warp mappings, including the rows written back at the end of the call.
Needs a B200."""
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


@pytest.mark.parametrize("stage", [16384, 320])
@pytest.mark.parametrize("mode", [1, 2])
@pytest.mark.parametrize("cfg,n,K", [("c1", 200, 30), ("c0", 64, 40), ("c3", 48, 30), ("c4", 24, 12)])
def test_staged_rows_match_oracle(api, stage, mode, cfg, n, K):
    from goib2d import configs
    sc, model, host = configs.batch(cfg, n)
    na = len(sc.action_joints)
    rng = np.random.default_rng(31)
    acts = rng.uniform(-1, 1, (K, n, 2)).astype(np.float32) if na else None
    eng = api.Engine(model, host.bodies.type.shape[1], sc.action_joints, sc.action_scale)
    try:
        eng.set_step_mode(mode)
        eng.set_state_staging(stage)
        dev = api.to_device(host)
        eng.step_(dev, sc.settings, configs.DT, n_steps=K, actions=torch.from_numpy(acts).cuda() if na else None)
        status = eng.status()
        got = api.to_host(dev)
    finally:
        eng.close()
    st = host
    for k in range(K):
        st = oracle_lib.step(model, st, sc.settings, configs.DT, 1, threads=8,
                             **(dict(actions=acts[k], action_joints=sc.action_joints, action_scale=sc.action_scale)
                                if na else {}))
    assert_states_equal(got, st, f"{cfg} staged {stage} mode {mode}")
    assert ((status & 0b1011) == 0).all()


def test_staging_setting_is_checked(api):
    from goib2d import configs
    sc, model, host = configs.batch("c1", 2)
    eng = api.Engine(model, host.bodies.type.shape[1])
    try:
        with pytest.raises(RuntimeError, match="negative staging size"):
            eng.set_state_staging(-1)
    finally:
        eng.close()
