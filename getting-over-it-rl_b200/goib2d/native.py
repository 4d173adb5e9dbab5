"""ctypes view of the C ABI in include/goib2d.h: the model descriptor, the State leaf table, and the library.

`model_desc(model)` packs a Model (numpy arrays) into `goib2d_model_desc`; the returned object keeps the arrays
alive. `leaf_spec(B, rows, J, C)` gives each State leaf's per-world shape and dtype in C-ABI order.
"""
import ctypes as C
import os
from pathlib import Path

import numpy as np

from .world import leaf_names

HERE = Path(__file__).resolve().parent
LIB_NAME = "libgoib2d.so"

_f = C.POINTER(C.c_float)
_i = C.POINTER(C.c_int32)
_u = C.POINTER(C.c_uint8)


class PairDesc(C.Structure):
    _fields_ = [("n_bodies", C.c_int32), ("n_fixtures", C.c_int32), ("n_joints", C.c_int32), ("body_type", _i),
                ("fixture_body", _i), ("shape_type", _i), ("sensor", _u), ("category", _i), ("mask", _i),
                ("group", _i), ("layer", _i), ("layer_masks", C.POINTER(C.c_uint32)), ("joint_a", _i),
                ("joint_b", _i), ("joint_collide", _u)]



SPAWN_UNIFORM, SPAWN_GRID, SPAWN_RIG = 0, 1, 2  # goib2d_spawn_rule.kind


class SpawnRule(C.Structure):
    """goib2d_spawn_rule: how goib2d_seed_placements draws a world's placements from (seed, world)."""
    _fields_ = [("kind", C.c_int32), ("n_bodies", C.c_int32)] + \
        [(k, C.c_float) for k in ("x_lo", "x_hi", "y_lo", "y_hi", "angle_lo", "angle_hi", "speed_lo", "speed_hi")] + \
        [("grid_side", C.c_int32)] + [(k, C.c_float) for k in ("grid_x0", "grid_y0", "grid_pitch", "jitter")] + \
        [("heights", C.c_void_p), ("n_heights", C.c_int32)] + \
        [(k, C.c_float) for k in ("h_x0", "h_dx", "half_width", "lift", "min_ground", "arm")] + \
        [("discs", C.c_void_p), ("n_discs", C.c_int32), ("clearance", C.c_float), ("max_tries", C.c_int32)]

def candidate_pairs_device(body_type, fixtures, joints, layer_masks=None):
    """goib2d_candidate_pairs on the current CUDA device: fixtures / joints as the WorldDef dicts; returns the
    (P, 2) int32 pair list."""
    lib = load()
    F, J = len(fixtures), len(joints)
    keep = []

    def arr(x, dt):
        a = np.ascontiguousarray(np.asarray(x, dt).reshape(-1))
        if a.size == 0:
            a = np.zeros(1, dt)
        keep.append(a)
        return a
    d = PairDesc()
    d.n_bodies, d.n_fixtures, d.n_joints = len(body_type), F, J
    d.body_type = arr(body_type, np.int32).ctypes.data_as(_i)
    d.fixture_body = arr([f["body"] for f in fixtures], np.int32).ctypes.data_as(_i)
    d.shape_type = arr([f["shape_type"] for f in fixtures], np.int32).ctypes.data_as(_i)
    d.sensor = arr([f["sensor"] for f in fixtures], np.uint8).ctypes.data_as(_u)
    d.category = arr([f["category"] for f in fixtures], np.int32).ctypes.data_as(_i)
    d.mask = arr([f["mask"] for f in fixtures], np.int32).ctypes.data_as(_i)
    d.group = arr([f["group"] for f in fixtures], np.int32).ctypes.data_as(_i)
    d.layer = arr([f["layer"] for f in fixtures], np.int32).ctypes.data_as(_i)
    d.layer_masks = None if layer_masks is None else \
        arr(np.asarray(layer_masks, np.int64) & 0xFFFFFFFF, np.uint32).ctypes.data_as(C.POINTER(C.c_uint32))
    d.joint_a = arr([j["a"] for j in joints], np.int32).ctypes.data_as(_i)
    d.joint_b = arr([j["b"] for j in joints], np.int32).ctypes.data_as(_i)
    d.joint_collide = arr([j["collide"] for j in joints], np.uint8).ctypes.data_as(_u)
    n = C.c_int64()
    rc = lib.goib2d_candidate_pairs(C.byref(d), None, None, 0, C.byref(n))
    if rc not in (0, -4):
        check(rc)
    out = np.zeros((max(n.value, 1), 2), np.int32)
    pa, pb = np.zeros(max(n.value, 1), np.int32), np.zeros(max(n.value, 1), np.int32)
    check(lib.goib2d_candidate_pairs(C.byref(d), pa.ctypes.data_as(_i), pb.ctypes.data_as(_i), n.value, C.byref(n)))
    out[:, 0], out[:, 1] = pa, pb
    return out[:n.value]


# goib2d_event: kind, fixture_a, fixture_b, child_a, child_b, count, normal_impulse[2], tangent_impulse[2]
EVENT_DTYPE = np.dtype([("kind", np.int32), ("fixture_a", np.int32), ("fixture_b", np.int32), ("child_a", np.int32),
                        ("child_b", np.int32), ("count", np.int32), ("normal_impulse", np.float32, 2),
                        ("tangent_impulse", np.float32, 2)])
assert EVENT_DTYPE.itemsize == 40


class ModelDesc(C.Structure):
    _fields_ = [("n_bodies", C.c_int32), ("n_fixtures", C.c_int32), ("n_joints", C.c_int32), ("n_pairs", C.c_int32),
                ("fixture_body", _i), ("shape_type", _i), ("count", _i), ("radius", _f), ("verts", _f),
                ("normals", _f), ("joint_type", _i), ("joint_a", _i), ("joint_b", _i), ("local_anchor_a", _f),
                ("local_anchor_b", _f), ("local_axis_a", _f), ("local_yaxis_a", _f), ("reference_angle", _f),
                ("pair_a", _i), ("pair_b", _i), ("toi_bodies", _u), ("fixture_slot", _i), ("static_fat", _f),
                ("static_friction", _f), ("static_restitution", _f), ("edge_ghost", _i)]


_MODEL_FIELDS = (("fixture_body", np.int32, _i), ("shape_type", np.int32, _i), ("count", np.int32, _i),
                 ("radius", np.float32, _f), ("verts", np.float32, _f), ("normals", np.float32, _f),
                 ("joint_type", np.int32, _i), ("joint_a", np.int32, _i), ("joint_b", np.int32, _i),
                 ("local_anchor_a", np.float32, _f), ("local_anchor_b", np.float32, _f),
                 ("local_axis_a", np.float32, _f), ("local_yaxis_a", np.float32, _f),
                 ("reference_angle", np.float32, _f), ("pair_a", np.int32, _i), ("pair_b", np.int32, _i),
                 ("toi_bodies", np.uint8, _u), ("fixture_slot", np.int32, _i), ("static_fat", np.float32, _f),
                 ("static_friction", np.float32, _f), ("static_restitution", np.float32, _f),
                 ("edge_ghost", np.int32, _i))


class PackedModel:
    """A goib2d_model_desc plus the host arrays it points into."""

    def __init__(self, model, n_bodies):
        self.keep = {}
        d = ModelDesc()
        d.n_bodies = int(n_bodies)
        d.n_fixtures = int(np.asarray(model.fixture_body).shape[0])
        d.n_joints = int(np.asarray(model.joint_type).shape[0])
        d.n_pairs = int(np.asarray(model.pair_a).shape[0])
        for name, dt, ptr in _MODEL_FIELDS:
            v = getattr(model, name)
            if v is None:
                setattr(d, name, None)
                continue
            a = np.ascontiguousarray(np.asarray(v).astype(dt))
            if a.size == 0:  # keep a valid pointer for empty tables
                a = np.zeros(1, dt)
            self.keep[name] = a
            setattr(d, name, a.ctypes.data_as(ptr))
        self.desc = d
        self.compact = model.fixture_slot is not None


def model_desc(model, n_bodies):
    return PackedModel(model, n_bodies)


# State leaf table: (dtype, entity, width) with entity one of "B", "rows", "J", "C", "1"
_LEAF_SPEC = (
    [(np.int32, "B", 1)] + [(np.bool_, "B", 1)] * 5 + [(np.float32, "B", 1)] + [(np.float32, "B", 2)] * 5 +
    [(np.float32, "B", 1)] * 2 + [(np.float32, "B", 2), (np.float32, "B", 1), (np.float32, "B", 2),
                                  (np.float32, "B", 1)] + [(np.float32, "B", 1)] * 7 +
    [(np.float32, "rows", 1), (np.float32, "rows", 1), (np.float32, "rows", 4)] +
    [(np.bool_, "J", 1), (np.float32, "J", 1), (np.float32, "J", 1), (np.bool_, "J", 1)] + [(np.float32, "J", 1)] * 4 +
    [(np.float32, "J", 3), (np.float32, "J", 1), (np.int32, "J", 1), (np.float32, "J", 1), (np.float32, "J", 1)] +
    [(np.int32, "C", 1)] * 4 + [(np.bool_, "C", 1), (np.int32, "C", 1), (np.int32, "C", 1)] +
    [(np.float32, "C", 2), (np.float32, "C", 2), (np.float32, "C", 4), (np.int32, "C", 2), (np.float32, "C", 2),
     (np.float32, "C", 2)] + [(np.float32, "C", 1)] * 3 +
    [(np.float32, "1", 2), (np.float32, "1", 1), (np.int32, "1", 1), (np.bool_, "1", 1), (np.int32, "1", 1)] +
    [(np.float32, "B", 1), (np.int32, "C", 1), (np.float32, "C", 1), (np.bool_, "C", 1), (np.bool_, "C", 1),
     (np.bool_, "C", 1), (np.float32, "C", 2), (np.float32, "C", 2), (np.int32, "1", 1)])
assert len(_LEAF_SPEC) == len(leaf_names()) == 71

# leaves whose per-world shape is (n, width) rather than (n,) / (2, 2) for point_local
_SHAPES = {"bodies.xf_p": 2, "bodies.xf_q": 2, "bodies.local_center": 2, "bodies.c0": 2, "bodies.c": 2,
           "bodies.v": 2, "bodies.force": 2, "fixtures.fat": 4, "joints.impulse": 3, "contacts.local_normal": 2,
           "contacts.local_point": 2, "contacts.point_local": (2, 2), "contacts.point_id": 2,
           "contacts.normal_impulse": 2, "contacts.tangent_impulse": 2, "toi.normal_impulse": 2,
           "toi.tangent_impulse": 2}


def leaf_spec(B, rows, J, C_):
    """[(name, per-world shape, numpy dtype)] in C-ABI order."""
    n = {"B": B, "rows": rows, "J": J, "C": C_}
    out = []
    for name, (dt, ent, width) in zip(leaf_names(), _LEAF_SPEC):
        if ent == "1":
            shape = () if width == 1 else (width,)
        else:
            w = _SHAPES.get(name)
            shape = (n[ent],) if w is None else ((n[ent], w) if isinstance(w, int) else (n[ent],) + w)
        out.append((name, shape, np.dtype(dt)))
    return out


def state_bytes_per_world(B, rows, J, C_):
    return sum(int(np.prod(s)) * dt.itemsize for _, s, dt in leaf_spec(B, rows, J, C_))


# ---- the CUDA library


_LIB = None


class NativeMissing(RuntimeError):
    pass


def lib_path():
    return Path(os.environ.get("GOIB2D_LIB", HERE / LIB_NAME))


def load():
    """libgoib2d.so (built in-tree by __graft_entry__.build / goib2d.build). No fallback: a missing library is an
    error."""
    global _LIB
    if _LIB is not None:
        return _LIB
    p = lib_path()
    if not p.exists():
        raise NativeMissing(f"{p} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'`")
    lib = C.CDLL(str(p))
    vp = C.c_void_p
    sig = {
        "goib2d_version": (C.c_int, []),
        "goib2d_last_error": (C.c_char_p, []),
        "goib2d_leaf_dtype": (C.c_int, [C.c_int]),
        "goib2d_leaf_elems": (C.c_int64, [C.c_int, C.c_int32, C.c_int32, C.c_int32, C.c_int32]),
        "goib2d_model_create": (C.c_int, [C.POINTER(ModelDesc), C.POINTER(vp)]),
        "goib2d_model_destroy": (C.c_int, [vp]),
        "goib2d_model_set_action_map": (C.c_int, [vp, C.c_int32, _i, _f]),
        "goib2d_step": (C.c_int, [vp, vp, C.c_float, C.c_int32, C.c_int32, C.c_int64, C.c_int32,
                                  C.POINTER(vp), vp, vp]),
        "goib2d_step_seq": (C.c_int, [vp, vp, C.c_float, C.c_int32, C.c_int32, C.c_int64, C.c_int32,
                                      C.POINTER(vp), vp, C.c_int64, vp]),
        "goib2d_launches": (C.c_int64, [vp, C.c_int64, C.c_int32]),
        "goib2d_status": (C.c_int, [vp, C.POINTER(vp), C.POINTER(C.c_int64)]),
        "goib2d_status_copy": (C.c_int, [vp, _i, C.c_int64]),
        "goib2d_step_noalloc": (C.c_int, [vp, vp, C.c_float, C.c_int32, C.c_int32, C.c_int64, C.c_int32,
                                          C.POINTER(vp), vp, vp]),
        "goib2d_kernels_per_step": (C.c_int, [vp, C.c_int64]),
        "goib2d_candidate_pairs": (C.c_int, [C.POINTER(PairDesc), _i, _i, C.c_int64, C.POINTER(C.c_int64)]),
        "goib2d_set_event_log": (C.c_int, [vp, C.c_int32]),
        "goib2d_set_step_mode": (C.c_int, [vp, C.c_int32]),
        "goib2d_set_state_staging": (C.c_int, [vp, C.c_int32]),
        "goib2d_events": (C.c_int, [vp, C.POINTER(vp), C.POINTER(vp), C.POINTER(C.c_int64), C.POINTER(C.c_int32)]),
        "goib2d_events_copy": (C.c_int, [vp, vp, _i, C.c_int64]),
        "goib2d_reset_masked": (C.c_int, [vp, C.c_int32, C.c_int32, C.c_int64, C.POINTER(vp), C.POINTER(vp), vp, vp]),
        "goib2d_reset_below": (C.c_int, [vp, C.c_int32, C.c_int32, C.c_int64, C.POINTER(vp), C.POINTER(vp),
                                         C.c_int32, C.c_float, vp, vp]),
        "goib2d_observe": (C.c_int, [vp, C.c_int32, C.c_int32, C.c_int64, C.POINTER(vp), C.c_int32, _i, vp, vp]),
        "goib2d_raycast": (C.c_int, [vp, C.c_int32, C.c_int32, C.c_int64, C.POINTER(vp), C.c_int32, C.c_int32,
                                     C.c_float, vp, vp]),
        "goib2d_set_checks": (C.c_int, [vp, C.c_int32]),
        "goib2d_validate": (C.c_int, [vp, C.c_int32, C.c_int32, C.c_int64, C.POINTER(vp), C.POINTER(C.c_int64),
                                      C.POINTER(C.c_int32), vp]),
        "goib2d_spawn": (C.c_int, [vp, C.c_int32, C.c_int32, C.c_int64, C.POINTER(vp), C.POINTER(vp), C.c_int32,
                                   C.c_int32, vp, C.c_int32, _i, vp, vp]),
        "goib2d_seed_placements": (C.c_int, [C.POINTER(SpawnRule), C.c_uint64, C.c_int64, C.c_int64, vp, vp, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    _LIB = lib
    return lib


def check(rc):
    if rc != 0:
        msg = load().goib2d_last_error().decode()
        raise RuntimeError(f"goib2d error {rc}: {msg}")
    return rc
