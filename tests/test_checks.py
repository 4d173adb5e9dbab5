"""Checked stepping and State validation (goib2d_set_checks, goib2d_validate): a State whose index fields are out of
range is refused before any step kernel runs, naming the world and the field; a valid State steps exactly as without
checks. The bad values are written into the State on the host; only the validation kernel, which compares them with
their ranges and reads the Model at no unchecked index, ever sees them."""
import ctypes

import numpy as np
import pytest

from goib2d import configs, native
from goib2d.world import leaf_names, map_state, state_leaves


def test_checks_entry_points_reject_a_null_model():
    lib = native.load()
    assert lib.goib2d_set_checks(None, 1) < 0 and b"null" in lib.goib2d_last_error()
    bw, bl = ctypes.c_int64(), ctypes.c_int32()
    assert lib.goib2d_validate(None, 8, 1, 1, None, ctypes.byref(bw), ctypes.byref(bl), None) < 0


def _stepped_c1(n=8, steps=30):
    from goib2d import api
    sc, model, host = configs.batch("c1", n)
    eng = api.Engine(model, host.bodies.type.shape[1])
    dev = api.to_device(host)
    eng.step_(dev, sc.settings, configs.DT, n_steps=steps)
    return sc, model, eng, api.to_host(dev)


@pytest.mark.gpu
def test_checked_step_equals_the_unchecked_step():
    from goib2d import api
    sc, model, eng, host = _stepped_c1()
    try:
        a, b = api.to_device(host), api.to_device(host)
        assert eng.validate(a) is None
        eng.step_(a, sc.settings, configs.DT, n_steps=10)
        eng.set_checks(True)
        eng.step_(b, sc.settings, configs.DT, n_steps=10)
        for name, x, y in zip(leaf_names(), state_leaves(api.to_host(a)), state_leaves(api.to_host(b))):
            assert np.array_equal(np.asarray(x).view(np.uint8), np.asarray(y).view(np.uint8)), name
    finally:
        eng.close()


@pytest.mark.gpu
def test_bad_index_fields_are_refused_before_the_step():
    from goib2d import api
    sc, model, eng, host = _stepped_c1()
    P = len(model.pair_a)
    live = np.argwhere(np.asarray(host.contacts.pair) >= 0)
    assert len(live), "the stepped rigs touch the level"
    w, s = (int(v) for v in live[0])

    def corrupt(fn):
        st = map_state(lambda x: np.array(x, copy=True), host)
        fn(st)
        return st

    cases = [
        ("contacts.pair", 3, lambda st: st.contacts.pair.__setitem__((3, 0), P + 5)),
        ("bodies.type", 5, lambda st: st.bodies.type.__setitem__((5, 1), 7)),
        ("joints.limit_state", 2, lambda st: st.joints.limit_state.__setitem__((2, 1), 4)),
        ("contacts.fa", w, lambda st: st.contacts.fa.__setitem__((w, s), st.contacts.fa[w, s] + 1)),
        ("contacts.count", w, lambda st: st.contacts.count.__setitem__((w, s), 3)),
        ("contacts.mtype", w, lambda st: st.contacts.mtype.__setitem__((w, s), 9)),
    ]
    try:
        eng.set_checks(True)
        for leaf, world, fn in cases:
            bad = corrupt(fn)
            dev = api.to_device(bad)
            assert eng.validate(dev) == (world, leaf), leaf
            with pytest.raises(RuntimeError, match=f"world {world} has an out-of-range {leaf}"):
                eng.step_(dev, sc.settings, configs.DT, n_steps=2)
            for name, x, y in zip(leaf_names(), state_leaves(api.to_host(dev)), state_leaves(bad)):
                assert np.array_equal(np.asarray(x).view(np.uint8), np.asarray(y).view(np.uint8)), name  # untouched
        two = corrupt(lambda st: (st.contacts.pair.__setitem__((6, 1), -3), st.bodies.type.__setitem__((4, 0), -1)))
        assert eng.validate(api.to_device(two)) == (4, "bodies.type")  # the first failing world is reported
    finally:
        eng.close()
