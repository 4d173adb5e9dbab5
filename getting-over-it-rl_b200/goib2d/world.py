"""World layout and the host-side scene builder.

Mirrors goi_jax/box2d/world.py (reference world.py:30-386): a `Model` shared by every world (fixture geometry,
joint frames, the candidate pair list in b2BroadPhase::UpdatePairs order) and a per-world `State`, both NamedTuples
of fixed-shape arrays, plus `WorldDef` whose builder methods and defaults are the reference's. Capacities are fixed
at build: B bodies, F fixtures, J joints, C contact slots, P candidate pairs.

Batched states carry a leading world axis N on every leaf: leaf `(N, ...)` row-major is exactly the layout the CUDA
engine reads and writes in place (one world = one contiguous row per leaf), and the layout jax.vmap gives the
reference's batched pytree. `state_leaves()` fixes the leaf order the C-ABI takes (include/goib2d.h).

Indices follow creation order, which Box2D's orderings depend on: body i is the i-th created (Box2D's body list is
newest first); fixture i gets broad-phase proxy id i; joint i is the i-th created.
"""
from typing import NamedTuple

import numpy as np

from . import shapes
from .settings import MAX_POLYGON_VERTICES, Settings

F32, I32 = np.float32, np.int32
STATIC, KINEMATIC, DYNAMIC = 0, 1, 2  # b2BodyType
REVOLUTE, PRISMATIC, WELD = 1, 2, 8  # b2JointType
MOTOR = 11  # b2JointType e_motorJoint: this package's addition (the reference engine has no motor joint)
INACTIVE_LIMIT, AT_LOWER, AT_UPPER, EQUAL_LIMITS = 0, 1, 2, 3  # b2LimitState
CIRCLES, FACE_A, FACE_B = 0, 1, 2  # b2Manifold::Type


class Model(NamedTuple):
    """Scene constants shared by every world (reference world.py:30-67)."""
    fixture_body: np.ndarray  # i32[F]
    shape_type: np.ndarray  # i32[F]
    radius: np.ndarray  # f32[F]
    count: np.ndarray  # i32[F]
    verts: np.ndarray  # f32[F, 8, 2]
    normals: np.ndarray  # f32[F, 8, 2]
    joint_type: np.ndarray  # i32[J]
    joint_a: np.ndarray  # i32[J]
    joint_b: np.ndarray  # i32[J]
    local_anchor_a: np.ndarray  # f32[J, 2]
    local_anchor_b: np.ndarray  # f32[J, 2]
    local_axis_a: np.ndarray  # f32[J, 2]
    local_yaxis_a: np.ndarray  # f32[J, 2]
    reference_angle: np.ndarray  # f32[J]
    pair_a: np.ndarray  # i32[P]
    pair_b: np.ndarray  # i32[P]
    toi_bodies: np.ndarray = None  # bool[B] bullet or continuous at build
    fixture_slot: np.ndarray = None  # i32[F] row in State.fixtures, -1 for a static body's fixture (compact layout)
    slot_fixture: np.ndarray = None  # i32[Fd]
    static_fat: np.ndarray = None  # f32[F, 4]
    static_friction: np.ndarray = None  # f32[F]
    static_restitution: np.ndarray = None  # f32[F]
    # The reference's culled-scan tables for its Pallas kernel; this engine has its own broadphase (model.py) and
    # leaves them unset.
    scan_cand: np.ndarray = None
    scan_row: np.ndarray = None
    scan_box: np.ndarray = None
    # Edge fixtures (this engine's addition): bit 0 / bit 1 set when verts[f, 2] / verts[f, 3] is a ghost vertex
    edge_ghost: np.ndarray = None  # i32[F]


class Bodies(NamedTuple):
    type: np.ndarray  # i32[B]
    active: np.ndarray  # bool[B]
    awake: np.ndarray  # bool[B]
    allow_sleep: np.ndarray  # bool[B]
    bullet: np.ndarray  # bool[B]
    continuous: np.ndarray  # bool[B]
    sleep_time: np.ndarray  # f32[B]
    xf_p: np.ndarray  # f32[B, 2]
    xf_q: np.ndarray  # f32[B, 2] (cos, sin)
    local_center: np.ndarray  # f32[B, 2]
    c0: np.ndarray  # f32[B, 2]
    c: np.ndarray  # f32[B, 2]
    a0: np.ndarray  # f32[B]
    a: np.ndarray  # f32[B]
    v: np.ndarray  # f32[B, 2]
    w: np.ndarray  # f32[B]
    force: np.ndarray  # f32[B, 2]
    torque: np.ndarray  # f32[B]
    mass: np.ndarray
    inv_mass: np.ndarray
    inertia: np.ndarray
    inv_inertia: np.ndarray
    linear_damping: np.ndarray
    angular_damping: np.ndarray
    gravity_scale: np.ndarray


class Fixtures(NamedTuple):
    friction: np.ndarray  # f32[F or Fd]
    restitution: np.ndarray  # f32[F or Fd]
    fat: np.ndarray  # f32[F or Fd, 4]


class Joints(NamedTuple):
    enable_motor: np.ndarray  # bool[J]
    motor_speed: np.ndarray  # f32[J]
    max_motor: np.ndarray  # f32[J]
    enable_limit: np.ndarray  # bool[J]
    lower: np.ndarray  # f32[J]
    upper: np.ndarray  # f32[J]
    frequency: np.ndarray  # f32[J]
    damping: np.ndarray  # f32[J]
    impulse: np.ndarray  # f32[J, 3]
    motor_impulse: np.ndarray  # f32[J]
    limit_state: np.ndarray  # i32[J]
    lower_impulse: np.ndarray  # f32[J]
    upper_impulse: np.ndarray  # f32[J]


class Contacts(NamedTuple):
    pair: np.ndarray  # i32[C] candidate index, -1 empty
    fa: np.ndarray  # i32[C]
    fb: np.ndarray  # i32[C]
    key: np.ndarray  # i32[C] creation order (larger = newer)
    touching: np.ndarray  # bool[C]
    mtype: np.ndarray  # i32[C]
    count: np.ndarray  # i32[C]
    local_normal: np.ndarray  # f32[C, 2]
    local_point: np.ndarray  # f32[C, 2]
    point_local: np.ndarray  # f32[C, 2, 2]
    point_id: np.ndarray  # i32[C, 2]
    normal_impulse: np.ndarray  # f32[C, 2]
    tangent_impulse: np.ndarray  # f32[C, 2]
    friction: np.ndarray  # f32[C]
    restitution: np.ndarray  # f32[C]
    tangent_speed: np.ndarray  # f32[C]


class ContactTOI(NamedTuple):
    alpha0: np.ndarray  # f32[B]
    count: np.ndarray  # i32[C]
    toi: np.ndarray  # f32[C]
    flag: np.ndarray  # bool[C]
    enabled: np.ndarray  # bool[C]
    solved: np.ndarray  # bool[C]
    normal_impulse: np.ndarray  # f32[C, 2]
    tangent_impulse: np.ndarray  # f32[C, 2]
    events: np.ndarray  # i32


class State(NamedTuple):
    bodies: Bodies
    fixtures: Fixtures
    joints: Joints
    contacts: Contacts
    gravity: np.ndarray  # f32[2]
    inv_dt0: np.ndarray  # f32
    next_key: np.ndarray  # i32
    new_fixture: np.ndarray  # bool
    overflow: np.ndarray  # i32
    toi: ContactTOI = None


def empty_toi(B, C):
    return ContactTOI(alpha0=np.zeros(B, F32), count=np.zeros(C, I32), toi=np.ones(C, F32),
                      flag=np.zeros(C, bool), enabled=np.ones(C, bool), solved=np.zeros(C, bool),
                      normal_impulse=np.zeros((C, 2), F32), tangent_impulse=np.zeros((C, 2), F32),
                      events=np.asarray(I32(0)))


def empty_contacts(C):
    f = lambda *s: np.zeros((C,) + s, F32)  # noqa: E731
    i = lambda *s: np.zeros((C,) + s, I32)  # noqa: E731
    return Contacts(pair=np.full(C, -1, I32), fa=i(), fb=i(), key=i(), touching=np.zeros(C, bool), mtype=i(),
                    count=i(), local_normal=f(2), local_point=f(2), point_local=f(2, 2), point_id=i(2),
                    normal_impulse=f(2), tangent_impulse=f(2), friction=f(), restitution=f(), tangent_speed=f())


# ---- leaf order of the C-ABI (include/goib2d.h GOIB2D_LEAF_*)

STATE_LEAVES = (
    ("bodies", Bodies._fields), ("fixtures", Fixtures._fields), ("joints", Joints._fields),
    ("contacts", Contacts._fields), ("gravity", None), ("inv_dt0", None), ("next_key", None), ("new_fixture", None),
    ("overflow", None), ("toi", ContactTOI._fields))


def leaf_names():
    out = []
    for grp, fl in STATE_LEAVES:
        if fl is None:
            out.append(grp)
        else:
            out.extend(f"{grp}.{f}" for f in fl)
    return out


def state_leaves(state):
    """The State's leaves in C-ABI order (every one present; a State without `toi` gets none here)."""
    out = []
    for grp, fl in STATE_LEAVES:
        v = getattr(state, grp)
        if fl is None:
            out.append(v)
        else:
            out.extend(getattr(v, f) for f in fl)
    return out


def state_from_leaves(leaves):
    it = iter(leaves)
    parts = {}
    for grp, fl in STATE_LEAVES:
        if fl is None:
            parts[grp] = next(it)
        else:
            cls = {"bodies": Bodies, "fixtures": Fixtures, "joints": Joints, "contacts": Contacts,
                   "toi": ContactTOI}[grp]
            parts[grp] = cls(*(next(it) for _ in fl))
    return State(**parts)


def map_state(fn, *states):
    """Apply fn leafwise over States of the same structure."""
    return state_from_leaves([fn(*xs) for xs in zip(*(state_leaves(s) for s in states))])


# ---- builder


def _filter_ok(fa, fb, masks):
    """Filter::ShouldCollide of the reference C API: the Unity layer matrix when given, else Box2D's groups."""
    if masks is not None:
        return bool(((int(masks[fa["layer"]]) & 0xFFFFFFFF) >> fb["layer"]) & 1)
    if fa["group"] == fb["group"] and fa["group"] != 0:
        return fa["group"] > 0
    return (fa["mask"] & fb["category"]) != 0 and (fa["category"] & fb["mask"]) != 0


class WorldDef:
    """Host-side builder with the reference's method names and defaults (reference world.py:186-304)."""

    def __init__(self, settings=None, layer_masks=None):
        self.settings = settings or Settings()
        self.layer_masks = layer_masks
        self.bodies, self.fixtures, self.joints = [], [], []

    def add_body(self, type=DYNAMIC, position=(0, 0), angle=0.0, velocity=(0, 0), angular_velocity=0.0, *,
                 mass=None, center=(0, 0), inertia=0.0, exact_inertia=True, linear_damping=0.0,
                 angular_damping=0.0, gravity_scale=1.0, fixed_rotation=False, bullet=False, continuous=False,
                 awake=True, allow_sleep=True, active=True):
        ang = F32(angle)
        s, c = shapes.host_sin_cos(ang)
        dyn = type == DYNAMIC
        body = dict(type=type, active=active, awake=awake, allow_sleep=allow_sleep, bullet=bullet,
                    continuous=continuous, fixed_rotation=fixed_rotation, p=np.array(position, F32), q=(c, s),
                    local_center=np.zeros(2, F32), c=np.array(position, F32), a=ang, v=np.zeros(2, F32), w=F32(0),
                    mass=F32(1 if dyn else 0), inv_mass=F32(1 if dyn else 0), inertia=F32(0),
                    inv_inertia=F32(0), linear_damping=F32(linear_damping), angular_damping=F32(angular_damping),
                    gravity_scale=F32(gravity_scale), sleep_time=F32(0))
        self.bodies.append(body)
        bid = len(self.bodies) - 1
        if mass is not None:
            self.set_mass(bid, mass, center, inertia, exact_inertia)
        moving = velocity[0] or velocity[1] or angular_velocity
        if type != STATIC and moving:
            body["v"], body["w"], body["awake"] = np.array(velocity, F32), F32(angular_velocity), True
            if not awake:  # SetAwake(false) after setting a velocity zeroes it again
                body["awake"], body["v"], body["w"] = False, np.zeros(2, F32), F32(0)
        return bid

    def set_mass(self, body, mass, center=(0, 0), inertia=0.0, exact=True):
        """b2MassData (I about the origin = I_com + m |c|^2) through b2Body::SetMassData, then, with `exact`, the
        given I_com verbatim (reference world.py:220-244)."""
        b = self.bodies[body]
        if b["type"] != DYNAMIC:
            return
        m, cx, cy, icom = F32(mass), F32(center[0]), F32(center[1]), F32(inertia)
        cc = F32(F32(cx * cx) + F32(cy * cy))
        i_origin = F32(icom + F32(m * cc))
        m_eff = m if m > 0 else F32(1)
        b["mass"], b["inv_mass"] = m_eff, F32(F32(1) / m_eff)
        b["inertia"], b["inv_inertia"] = F32(0), F32(0)
        if i_origin > 0 and not b["fixed_rotation"]:
            b["inertia"] = F32(i_origin - F32(m_eff * cc))
            b["inv_inertia"] = F32(F32(1) / b["inertia"])
        if exact and b["inertia"] > 0:
            b["inertia"], b["inv_inertia"] = icom, F32(F32(1) / icom)
        old = b["c"].copy()
        qc, qs = b["q"]
        px, py = b["p"]
        b["local_center"] = np.array([cx, cy], F32)
        b["c"] = np.array([F32(F32(F32(qc * cx) - F32(qs * cy)) + px), F32(F32(F32(qs * cx) + F32(qc * cy)) + py)], F32)
        dx, dy = F32(b["c"][0] - old[0]), F32(b["c"][1] - old[1])
        w = b["w"]
        b["v"] = np.array([F32(b["v"][0] + F32(-w * dy)), F32(b["v"][1] + F32(w * dx))], F32)

    def _add_fixture(self, body, shape_type, verts, normals, radius, friction, restitution, sensor, layer,
                     category, mask, group, count=None, ghost=0):
        vv, nn = shapes.pad(verts, normals)
        self.fixtures.append(dict(body=body, shape_type=shape_type, verts=vv, normals=nn,
                                  count=len(verts) if count is None else count, ghost=int(ghost),
                                  radius=F32(radius), friction=F32(friction), restitution=F32(restitution),
                                  sensor=bool(sensor), layer=int(layer) & 31, category=category, mask=mask,
                                  group=group))
        return len(self.fixtures) - 1

    def add_edge(self, body, v1, v2, v0=None, v3=None, *, friction=0.2, restitution=0.0, sensor=False, layer=0,
                 category=1, mask=0xFFFF, group=0):
        """b2EdgeShape: the segment v1-v2 with the optional ghost vertices v0 (before v1) and v3 (after v2), skin
        radius b2_polygonRadius. Massless; collides with circles and polygons, not with other edges. No counterpart in
        the reference engine."""
        p1, p2 = (F32(v1[0]), F32(v1[1])), (F32(v2[0]), F32(v2[1]))
        g0 = (F32(0), F32(0)) if v0 is None else (F32(v0[0]), F32(v0[1]))
        g3 = (F32(0), F32(0)) if v3 is None else (F32(v3[0]), F32(v3[1]))
        nx, ny = shapes.normalize(F32(p2[1] - p1[1]), F32(-(p2[0] - p1[0])))
        verts = np.array([p1, p2, g0, g3], F32)
        normals = np.array([(nx, ny), (-nx, -ny), (0, 0), (0, 0)], F32)
        ghost = (0 if v0 is None else 1) | (0 if v3 is None else 2)
        return self._add_fixture(body, shapes.EDGE, verts, normals, self.settings.polygon_radius, friction,
                                 restitution, sensor, layer, category, mask, group, count=2, ghost=ghost)

    def add_chain(self, body, vertices, loop=False, prev_vertex=None, next_vertex=None, **kw):
        """b2ChainShape as its child edges, one edge fixture per segment in order, each with its neighbours' ends
        as ghost vertices (b2ChainShape::GetChildEdge). loop=True closes the chain (b2ChainShape::CreateLoop); an open
        chain takes prev_vertex / next_vertex as its end ghosts when given. Returns the fixture indices."""
        v = [(float(p[0]), float(p[1])) for p in np.asarray(vertices, np.float64).reshape(-1, 2)]
        if loop:
            if len(v) < 3:
                raise ValueError("a chain loop needs 3 vertices or more")
            prev_vertex, next_vertex = v[-1], v[1]
            v = v + [v[0]]
        elif len(v) < 2:
            raise ValueError("a chain needs 2 vertices or more")
        out = []
        for i in range(len(v) - 1):
            v0 = v[i - 1] if i > 0 else prev_vertex
            v3 = v[i + 2] if i + 2 < len(v) else next_vertex
            out.append(self.add_edge(body, v[i], v[i + 1], v0, v3, **kw))
        return out

    def add_polygon(self, body, vertices, radius=None, raw=False, *, friction=0.2, restitution=0.0, density=0.0,
                    sensor=False, layer=0, category=1, mask=0xFFFF, group=0):
        v, n = shapes.polygon_raw(vertices) if raw else shapes.polygon_set(vertices, self.settings.linear_slop)
        r = self.settings.polygon_radius if radius is None else radius
        return self._add_fixture(body, shapes.POLYGON, v, n, r, friction, restitution, sensor, layer, category,
                                 mask, group)

    def add_box(self, body, half_extents, center=(0, 0), angle=0.0, radius=None, *, friction=0.2, restitution=0.0,
                density=0.0, sensor=False, layer=0, category=1, mask=0xFFFF, group=0):
        v, n = shapes.box(half_extents[0], half_extents[1], center, angle)
        r = self.settings.polygon_radius if radius is None else radius
        return self._add_fixture(body, shapes.POLYGON, v, n, r, friction, restitution, sensor, layer, category,
                                 mask, group)

    def add_circle(self, body, radius, center=(0, 0), *, friction=0.2, restitution=0.0, density=0.0, sensor=False,
                   layer=0, category=1, mask=0xFFFF, group=0):
        return self._add_fixture(body, shapes.CIRCLE, np.array([center], F32), np.zeros((1, 2), F32), radius,
                                 friction, restitution, sensor, layer, category, mask, group)

    def _add_joint(self, **j):
        self.joints.append(j)
        return len(self.joints) - 1

    def add_revolute(self, body_a, body_b, anchor_a=(0, 0), anchor_b=(0, 0), reference_angle=0.0, *,
                     limits=None, motor_speed=0.0, max_motor_torque=0.0, enable_motor=False, collide=False):
        lo, hi = limits if limits is not None else (0.0, 0.0)
        return self._add_joint(type=REVOLUTE, a=body_a, b=body_b, la=anchor_a, lb=anchor_b, ref=reference_angle,
                               axis=(1, 0), enable_limit=limits is not None, lower=lo, upper=hi,
                               motor_speed=motor_speed, max_motor=max_motor_torque, enable_motor=enable_motor,
                               frequency=0.0, damping=0.0, collide=collide)

    def add_prismatic(self, body_a, body_b, anchor_a=(0, 0), anchor_b=(0, 0), axis=(1, 0), reference_angle=0.0, *,
                      limits=None, motor_speed=0.0, max_motor_force=0.0, enable_motor=False, collide=False):
        lo, hi = limits if limits is not None else (0.0, 0.0)
        return self._add_joint(type=PRISMATIC, a=body_a, b=body_b, la=anchor_a, lb=anchor_b, ref=reference_angle,
                               axis=axis, enable_limit=limits is not None, lower=lo, upper=hi,
                               motor_speed=motor_speed, max_motor=max_motor_force, enable_motor=enable_motor,
                               frequency=0.0, damping=0.0, collide=collide)

    def add_weld(self, body_a, body_b, anchor_a=(0, 0), anchor_b=(0, 0), reference_angle=0.0, *, frequency=0.0,
                 damping=0.0, collide=False):
        return self._add_joint(type=WELD, a=body_a, b=body_b, la=anchor_a, lb=anchor_b, ref=reference_angle,
                               axis=(1, 0), enable_limit=False, lower=0.0, upper=0.0, motor_speed=0.0,
                               max_motor=0.0, enable_motor=False, frequency=frequency, damping=damping,
                               collide=collide)

    def add_motor(self, body_a, body_b, linear_offset=(0, 0), angular_offset=0.0, *, max_force=1.0, max_torque=1.0,
                  correction_factor=0.3, collide=False):
        """Box2D 2.3.1's b2MotorJoint (not in the reference engine; parity with it cannot be pinned): drives body B
        toward linear_offset (in body A's frame, from A's origin to B's origin) and angular_offset (B's angle minus
        A's) with impulses limited to max_force and max_torque per second, correcting correction_factor of the error
        per step. The joint row of the State carries its parameters, so that each world (and the action channels,
        which write motor_speed) can set its own targets: lower / upper = the linear offset's x / y, motor_speed =
        the angular offset, max_motor = max torque, frequency = max force, damping = the correction factor;
        impulse = (linear x, linear y, angular)."""
        return self._add_joint(type=MOTOR, a=body_a, b=body_b, la=(0, 0), lb=(0, 0), ref=0.0, axis=(1, 0),
                               enable_limit=False, lower=float(linear_offset[0]), upper=float(linear_offset[1]),
                               motor_speed=float(angular_offset), max_motor=max_torque, enable_motor=False,
                               frequency=max_force, damping=correction_factor, collide=collide)

    # ---- build

    def candidate_pairs(self, device=False):
        """Fixture pairs that can ever touch, in b2BroadPhase::UpdatePairs order (ascending (lower, higher) proxy
        id), polygon first in a polygon-circle pair as b2Contact::Create orders them. Dropped for good: same body,
        both static, joined by a joint without collideConnected, filtered out, or a sensor (reference
        world.py:308-329). device=True builds the same list on the GPU (goib2d_candidate_pairs)."""
        if device:
            from . import native
            pairs = native.candidate_pairs_device([b["type"] for b in self.bodies], self.fixtures, self.joints,
                                                  self.layer_masks)
            return [(int(a), int(b)) for a, b in pairs]
        no_collide = {frozenset((j["a"], j["b"])) for j in self.joints if not j["collide"]}
        fx, out = self.fixtures, []
        E = shapes.EDGE
        for i in range(len(fx)):
            fi = fx[i]
            ti = self.bodies[fi["body"]]["type"]
            for k in range(i + 1, len(fx)):
                fk = fx[k]
                if fi["body"] == fk["body"] or fi["sensor"] or fk["sensor"]:
                    continue
                if fi["shape_type"] == E and fk["shape_type"] == E:  # no edge-edge collider
                    continue
                if ti == STATIC and self.bodies[fk["body"]]["type"] == STATIC:
                    continue
                if frozenset((fi["body"], fk["body"])) in no_collide:
                    continue
                if not _filter_ok(fi, fk, self.layer_masks):
                    continue
                first_k = ((fi["shape_type"] == shapes.CIRCLE and fk["shape_type"] == shapes.POLYGON) or
                           fk["shape_type"] == E)  # b2Contact::Create's primary order: polygon > circle, edge first
                out.append((k, i) if first_k else (i, k))
        return out

    def body_arrays(self):
        bs = self.bodies
        B = len(bs)

        def col(key, dt, shape=()):
            return np.array([x[key] for x in bs], dt).reshape((B,) + shape)
        return Bodies(
            type=col("type", I32), active=col("active", bool), awake=col("awake", bool),
            allow_sleep=col("allow_sleep", bool), bullet=col("bullet", bool), continuous=col("continuous", bool),
            sleep_time=col("sleep_time", F32), xf_p=col("p", F32, (2,)),
            xf_q=np.array([b["q"] for b in bs], F32).reshape(B, 2), local_center=col("local_center", F32, (2,)),
            c0=col("c", F32, (2,)), c=col("c", F32, (2,)), a0=col("a", F32), a=col("a", F32), v=col("v", F32, (2,)),
            w=col("w", F32), force=np.zeros((B, 2), F32), torque=np.zeros(B, F32), mass=col("mass", F32),
            inv_mass=col("inv_mass", F32), inertia=col("inertia", F32), inv_inertia=col("inv_inertia", F32),
            linear_damping=col("linear_damping", F32), angular_damping=col("angular_damping", F32),
            gravity_scale=col("gravity_scale", F32))

    def fixture_geometry(self):
        fs = self.fixtures
        F = len(fs)

        def col(key, dt, shape=()):
            return np.array([x[key] for x in fs], dt).reshape((F,) + shape)
        geom = dict(fixture_body=col("body", I32), shape_type=col("shape_type", I32), radius=col("radius", F32),
                    count=col("count", I32), verts=col("verts", F32, (MAX_POLYGON_VERTICES, 2)),
                    normals=col("normals", F32, (MAX_POLYGON_VERTICES, 2)))
        if any(f["shape_type"] == shapes.EDGE for f in fs):
            geom["edge_ghost"] = col("ghost", I32)
        return geom

    def fixture_arrays(self, bodies, geom=None):
        """Fixtures (friction, restitution, fat AABB at the bodies' transforms) for the given Bodies."""
        g = geom or self.fixture_geometry()
        fs = self.fixtures
        F = len(fs)
        fb = g["fixture_body"]
        lx, ly, ux, uy = shapes.fixture_aabbs(g["shape_type"], g["count"], g["radius"], g["verts"],
                                              bodies.xf_p[fb, 0], bodies.xf_p[fb, 1], bodies.xf_q[fb, 0],
                                              bodies.xf_q[fb, 1])
        fat = np.stack(shapes.fatten(lx, ly, ux, uy), axis=-1).astype(F32).reshape(F, 4)
        return Fixtures(friction=np.array([f["friction"] for f in fs], F32).reshape(F),
                        restitution=np.array([f["restitution"] for f in fs], F32).reshape(F), fat=fat)

    def joint_arrays(self):
        js = self.joints
        J = len(js)

        def col(key, dt, shape=()):
            return np.array([x[key] for x in js], dt).reshape((J,) + shape)
        return Joints(
            enable_motor=col("enable_motor", bool), motor_speed=col("motor_speed", F32),
            max_motor=col("max_motor", F32), enable_limit=col("enable_limit", bool), lower=col("lower", F32),
            upper=col("upper", F32), frequency=col("frequency", F32), damping=col("damping", F32),
            impulse=np.zeros((J, 3), F32), motor_impulse=np.zeros(J, F32), limit_state=np.zeros(J, I32),
            lower_impulse=np.zeros(J, F32), upper_impulse=np.zeros(J, F32))

    def build(self, contact_capacity=16, device_pairs=False):
        """(Model, State) as numpy arrays: fat AABBs from b2BroadPhase::CreateProxy (shape AABB at the body
        transform, extended), contacts empty, new_fixture set (reference world.py:331-386)."""
        B, F, J, C = len(self.bodies), len(self.fixtures), len(self.joints), contact_capacity
        js = self.joints
        pairs = self.candidate_pairs(device_pairs)
        bodies = self.body_arrays()
        geom = self.fixture_geometry()
        xaxes, yaxes = [], []
        for j in js:
            # prismatic m_localXAxisA: normalized twice (the C API normalizes, then b2PrismaticJoint's constructor
            # again; the second pass changes the last bit of some axes); m_localYAxisA = b2Cross(1.0f, x axis)
            x, y = shapes.normalize(*shapes.normalize(F32(j["axis"][0]), F32(j["axis"][1])))
            xaxes.append((x, y))
            yaxes.append((F32(-F32(1) * y), F32(F32(1) * x)))

        def jcol(key, dt, shape=()):
            return np.array([x[key] for x in js], dt).reshape((J,) + shape)
        model = Model(
            **geom, joint_type=jcol("type", I32), joint_a=jcol("a", I32), joint_b=jcol("b", I32),
            local_anchor_a=jcol("la", F32, (2,)), local_anchor_b=jcol("lb", F32, (2,)),
            local_axis_a=np.array(xaxes, F32).reshape(J, 2), local_yaxis_a=np.array(yaxes, F32).reshape(J, 2),
            reference_angle=jcol("ref", F32),
            pair_a=np.array([p[0] for p in pairs], I32).reshape(-1),
            pair_b=np.array([p[1] for p in pairs], I32).reshape(-1),
            toi_bodies=bodies.bullet | bodies.continuous)
        state = State(bodies=bodies, fixtures=self.fixture_arrays(bodies, geom), joints=self.joint_arrays(),
                      contacts=empty_contacts(C), gravity=np.array(self.settings.gravity, F32),
                      inv_dt0=np.asarray(F32(0)), next_key=np.asarray(I32(0)), new_fixture=np.asarray(F > 0),
                      overflow=np.asarray(I32(0)), toi=empty_toi(B, C))
        return model, state


# ---- compact fixture layout (reference world.py:400-562)


def is_compact(model, fixtures):
    return model.fixture_slot is not None and fixtures.fat.shape[-2] != model.fixture_body.shape[-1]


def compact_model(model, state):
    """The Model with the static-body fixtures' fat AABB, friction and restitution moved into it (shared by every
    world), from a full-layout State (any leading batch axes) whose static rows agree across worlds."""
    if model.fixture_slot is not None:
        return model
    btype = np.asarray(state.bodies.type)
    btype = btype.reshape(-1, btype.shape[-1])
    if not (btype == btype[0]).all():
        raise ValueError("compact_model: body types differ between worlds")
    fb = np.asarray(model.fixture_body)
    static = btype[0][fb] == STATIC
    if not static.any():
        return model
    F = fb.shape[0]
    fat = np.asarray(state.fixtures.fat).reshape(-1, F, 4)
    fr = np.asarray(state.fixtures.friction).reshape(-1, F)
    rs = np.asarray(state.fixtures.restitution).reshape(-1, F)
    for name, a in (("fat", fat), ("friction", fr), ("restitution", rs)):
        if not (a[:, static] == a[:1, static]).all():
            raise ValueError(f"compact_model: static fixtures' {name} differs between worlds")
    rows = np.nonzero(~static)[0].astype(I32)
    slot = np.full(F, -1, I32)
    slot[rows] = np.arange(len(rows), dtype=I32)

    def keep(a):
        mask = static.reshape((F,) + (1,) * (a.ndim - 1))
        return np.where(mask, a, 0).astype(a.dtype)
    return model._replace(fixture_slot=slot, slot_fixture=rows, static_fat=keep(fat[0]),
                          static_friction=keep(fr[0]), static_restitution=keep(rs[0]))


def compact_state(model, state, check=True):
    """A full-layout State (any leading batch axes) in the compact layout of `model`; idempotent."""
    fx = state.fixtures
    if model.fixture_slot is None or is_compact(model, fx):
        return state
    rows = np.asarray(model.slot_fixture)
    F = model.fixture_body.shape[-1]
    if check:
        static = np.asarray(model.fixture_slot) < 0
        for name, a, shared in (("fat", fx.fat, model.static_fat), ("friction", fx.friction, model.static_friction),
                                ("restitution", fx.restitution, model.static_restitution)):
            a = np.asarray(a)
            tail = a.shape[a.ndim - (2 if name == "fat" else 1) + 1:]
            a = a.reshape((-1, F) + tail)
            if not (a[:, static] == np.asarray(shared)[static][None]).all():
                raise ValueError(f"compact_state: static fixtures' {name} differs from the model's")
    fx = Fixtures(friction=np.take(np.asarray(fx.friction), rows, axis=-1),
                  restitution=np.take(np.asarray(fx.restitution), rows, axis=-1),
                  fat=np.take(np.asarray(fx.fat), rows, axis=-2))
    return state._replace(fixtures=fx)


def expand_state(model, state):
    """The full-layout State of a compact one (static rows from the Model); any leading batch axes."""
    fx = state.fixtures
    if not is_compact(model, fx):
        return state
    rows = np.asarray(model.slot_fixture)
    lead = np.asarray(fx.fat).shape[:-2]

    def put(shared, mine, ax):
        out = np.array(np.broadcast_to(np.asarray(shared), lead + np.asarray(shared).shape))
        idx = (Ellipsis, rows) + (slice(None),) * (-1 - ax)
        out[idx] = np.asarray(mine)
        return out
    return state._replace(fixtures=Fixtures(friction=put(model.static_friction, fx.friction, -1),
                                            restitution=put(model.static_restitution, fx.restitution, -1),
                                            fat=put(model.static_fat, fx.fat, -2)))
