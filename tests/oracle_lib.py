"""The parity oracle (oracle/liboracle_goib2d.so, a C++ restatement of the reference engine) through ctypes.

Test and CPU-baseline infrastructure only: it steps numpy States (leading world axis) in place on the host."""
import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

from goib2d import native
from goib2d.settings import settings_struct
from goib2d.world import state_from_leaves, state_leaves

ORACLE_DIR = Path(__file__).resolve().parents[1] / "oracle"
LIB = ORACLE_DIR / "liboracle_goib2d.so"
_lib = None


def load(build=True):
    global _lib
    if _lib is not None:
        return _lib
    if build:
        subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)
    lib = C.CDLL(str(LIB))
    vp = C.c_void_p
    lib.oracle_step_batch.restype = C.c_int
    lib.oracle_step_batch.argtypes = [C.POINTER(native.ModelDesc), vp, C.c_float, C.c_int32, C.c_int32, C.c_int64,
                                      C.c_int32, C.POINTER(vp), vp, C.c_int32, vp, vp, C.c_int32]
    lib.oracle_sin_cos.argtypes = [vp, C.c_int64, vp, vp]
    lib.oracle_max_threads.restype = C.c_int
    lib.oracle_leaf_elems.restype = C.c_int64
    lib.oracle_leaf_elems.argtypes = [C.c_int, C.c_int32, C.c_int32, C.c_int32, C.c_int32]
    lib.oracle_leaf_dtype.argtypes = [C.c_int]
    _lib = lib
    return lib


def batched(state):
    """A State with a leading world axis (a single-world State gets one)."""
    if np.asarray(state.bodies.type).ndim == 1:
        return state_from_leaves([np.ascontiguousarray(np.asarray(x)[None]) for x in state_leaves(state)])
    return state_from_leaves([np.ascontiguousarray(np.asarray(x)) for x in state_leaves(state)])


def step(model, state, settings, dt, n_steps=1, threads=0, actions=None, action_joints=(), action_scale=()):
    """Step a copy of `state` (numpy, batched or single world) n_steps times; returns the new State."""
    lib = load()
    single = np.asarray(state.bodies.type).ndim == 1
    st = batched(state)
    leaves = [np.ascontiguousarray(x).copy() for x in state_leaves(st)]
    N, B = leaves[0].shape[0], leaves[0].shape[1]
    rows = st.fixtures.friction.shape[1]
    J = st.joints.motor_speed.shape[1]
    Cc = st.contacts.pair.shape[1]
    pm = native.model_desc(model, B)
    ss = settings_struct(settings)
    ptrs = (C.c_void_p * len(leaves))(*[x.ctypes.data for x in leaves])
    act = aj = asc = None
    na = 0
    if actions is not None:
        actions = np.ascontiguousarray(actions, np.float32)
        na = actions.shape[1]
        aj = np.ascontiguousarray(action_joints, np.int32)
        asc = np.ascontiguousarray(action_scale, np.float32)
        if actions.shape[0] != N or aj.shape != (na,) or asc.shape != (na,):
            raise ValueError(f"actions {actions.shape} for {N} worlds need {na} action joints and scales, got "
                             f"{aj.shape[0]} and {asc.shape[0]}")
        act, aj_p, asc_p = actions.ctypes.data, aj.ctypes.data, asc.ctypes.data
    else:
        aj_p = asc_p = None
    rc = lib.oracle_step_batch(C.byref(pm.desc), C.addressof(ss), C.c_float(dt), Cc, rows, N, n_steps, ptrs, act,
                               na, aj_p, asc_p, threads)
    assert rc == 0
    out = state_from_leaves(leaves)
    if single:
        out = state_from_leaves([x[0] for x in leaves])
    return out


def step_events(model, state, settings, dt, n_steps, capacity, threads=0):
    """Step a copy of `state` with the contact event log on: (new State, events (N, capacity), counts (N,)); the log
    holds the last step's events (goib2d_event layout)."""
    lib = load()
    st = batched(state)
    leaves = [np.ascontiguousarray(x).copy() for x in state_leaves(st)]
    N, B = leaves[0].shape[0], leaves[0].shape[1]
    pm = native.model_desc(model, B)
    ss = settings_struct(settings)
    ptrs = (C.c_void_p * len(leaves))(*[x.ctypes.data for x in leaves])
    ev = np.zeros((N, capacity), native.EVENT_DTYPE)
    cnt = np.zeros(N, np.int32)
    lib.oracle_step_batch_events.argtypes = [C.POINTER(native.ModelDesc), C.c_void_p, C.c_float, C.c_int32, C.c_int32,
                                             C.c_int64, C.c_int32, C.POINTER(C.c_void_p), C.c_void_p, C.c_void_p,
                                             C.c_int32, C.c_int32]
    assert lib.oracle_step_batch_events(C.byref(pm.desc), C.addressof(ss), C.c_float(dt), st.contacts.pair.shape[1],
                                        st.fixtures.friction.shape[1], N, n_steps, ptrs, ev.ctypes.data,
                                        cnt.ctypes.data, capacity, threads) == 0
    return state_from_leaves(leaves), ev, cnt


def raycast(model, state, body, n_rays, max_length):
    """The oracle's ray casts (see goib2d_raycast) for a batched numpy State: (N, n_rays) float32."""
    lib = load()
    st = batched(state)
    leaves = [np.ascontiguousarray(x) for x in state_leaves(st)]
    N, B = leaves[0].shape[0], leaves[0].shape[1]
    pm = native.model_desc(model, B)
    out = np.zeros((N, n_rays), np.float32)
    ptrs = (C.c_void_p * len(leaves))(*[x.ctypes.data for x in leaves])
    lib.oracle_raycast.argtypes = [C.POINTER(native.ModelDesc), C.c_int32, C.c_int64, C.POINTER(C.c_void_p),
                                   C.c_int32, C.c_int32, C.c_float, C.c_void_p]
    assert lib.oracle_raycast(C.byref(pm.desc), st.fixtures.friction.shape[1], N, ptrs, body, n_rays,
                              C.c_float(max_length), out.ctypes.data) == 0
    return out


def sin_cos(x):
    lib = load()
    x = np.ascontiguousarray(x, np.float32)
    s, c = np.empty_like(x), np.empty_like(x)
    lib.oracle_sin_cos(x.ctypes.data, x.size, s.ctypes.data, c.ctypes.data)
    return s, c


def seed_placements(rule, seed, first_world, n_worlds):
    """The oracle's restatement of goib2d_seed_placements: (placements (n, k, 6), speeds (n,) or None). rule:
    native.SpawnRule whose heights / discs point at host float32 arrays."""
    lib = load()
    k = 3 if rule.kind == native.SPAWN_RIG else int(rule.n_bodies)
    pl = np.zeros((n_worlds, k, 6), np.float32)
    sp = np.zeros(n_worlds, np.float32)
    lib.oracle_seed_placements.argtypes = [C.POINTER(native.SpawnRule), C.c_uint64, C.c_int64, C.c_int64,
                                           C.c_void_p, C.c_void_p]
    assert lib.oracle_seed_placements(C.byref(rule), seed, first_world, n_worlds, pl.ctypes.data,
                                      sp.ctypes.data) == 0
    return pl, (sp if rule.kind == native.SPAWN_RIG else None)


def philox4x32_10(ctr, k0, k1):
    lib = load()
    c = np.ascontiguousarray(ctr, np.uint32)
    out = np.zeros(4, np.uint32)
    lib.oracle_philox4x32_10.argtypes = [C.c_void_p, C.c_uint32, C.c_uint32, C.c_void_p]
    lib.oracle_philox4x32_10(c.ctypes.data, k0, k1, out.ctypes.data)
    return out
