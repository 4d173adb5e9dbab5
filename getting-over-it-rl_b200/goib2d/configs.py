"""The five benchmark workloads, as seeded synthetic scenes built through the `WorldDef` builder API.

Every world of a workload shares one static level (the reference's Model is shared by all worlds of a batch);
worlds differ in their dynamic bodies' initial state, drawn from the seed per world index. Edge and chain shapes are
not in the reference engine, so the chain terrain and zero-thickness edges are built as their polygon-terrain
variants: each chain segment becomes the static convex quad (x_i, floor), (x_i+1, floor), (x_i+1, h_i+1), (x_i, h_i),
and each zero-thickness edge a 0.02 m thick box.

Contact capacities are sized so that no world of the benchmark horizon overflows its contact table (a full table
drops new contacts, as the reference does): c0 64, c1 48, c2 1536, c3 256, c4 64. c2's pile holds up to ~1.1k live
contacts (overlapping fat AABBs, ~500 of them touching) once it has formed; 1024 slots overflow from about step 75.

`scene(name, seed)` gives a `Scene`: the level arrays plus, per world index, the dynamic bodies' parameters.
`scene.build_world(defn, i)` issues the builder calls of world i on any WorldDef-like object (this package's, or the
reference's when generating golden vectors); `batch(name, n, seed)` builds the Model once and the n world States
vectorised, bit-identical to building each world through WorldDef (tests/test_host.py checks that).
"""
import math
from dataclasses import dataclass, field

import numpy as np

from . import shapes
from .settings import Settings
from .world import DYNAMIC, STATIC, WorldDef

F32 = np.float32
DT = F32(0.02)
GRAVITY = (F32(0.0), F32(-9.81))


def _per_world(seed, n, draw, first=0):
    """Stack draw(rng) over worlds first..first+n-1, each world with its own generator seeded (seed, 1, i): world
    i's values do not depend on the batch size or on which shard holds it."""
    first = first or _FIRST[0]
    rows = [draw(np.random.default_rng([seed, 1, i])) for i in range(first, first + n)]
    return {k: np.stack([r[k] for r in rows], 0) for k in rows[0]}


def _settings(continuous, allow_sleep=True):
    return Settings.stock(gravity=GRAVITY, velocity_iterations=8, position_iterations=3,
                          continuous_physics=continuous, allow_sleep=allow_sleep)


def _convex(rng, k, r):
    """A convex polygon: k points on a circle of radius r, evenly spaced angles jittered by under a third of the
    spacing (strictly convex, counter-clockwise, never closer than Set's weld distance)."""
    step = 2 * np.pi / k
    ang = rng.uniform(0, 2 * np.pi) + step * np.arange(k) + rng.uniform(-0.3, 0.3, k) * step
    return np.stack([r * np.cos(ang), r * np.sin(ang)], 1).astype(F32)


def polygon_mass(verts, density):
    """Mass, centroid and rotational inertia about the centroid of a convex polygon (b2PolygonShape::ComputeMass's
    triangle-fan formula, evaluated in float64 on the host; the scene only needs plausible values)."""
    v = np.asarray(verts, np.float64)
    ref = v.mean(0)
    area, cx, cy, inertia = 0.0, 0.0, 0.0, 0.0
    for i in range(len(v)):
        e1, e2 = v[i] - ref, v[(i + 1) % len(v)] - ref
        d = e1[0] * e2[1] - e1[1] * e2[0]
        a = 0.5 * d
        area += a
        cx += a * (e1[0] + e2[0]) / 3.0
        cy += a * (e1[1] + e2[1]) / 3.0
        intx2 = e1[0] * e1[0] + e2[0] * e1[0] + e2[0] * e2[0]
        inty2 = e1[1] * e1[1] + e2[1] * e1[1] + e2[1] * e2[1]
        inertia += (0.25 / 3.0 * d) * (intx2 + inty2)
    m = density * area
    c = np.array([cx / area, cy / area])
    i_ref = density * inertia
    i_com = i_ref - m * float(c @ c)
    return float(m), (c + ref), float(i_com)


@dataclass
class Scene:
    name: str
    settings: Settings
    capacity: int
    steps: int
    n_worlds: int
    static_polys: list = field(default_factory=list)  # (verts (k,2), friction)
    static_boxes: list = field(default_factory=list)  # (half (2,), centre (2,), angle, friction)
    static_chains: list = field(default_factory=list)  # (vertices (k,2), friction): open chains of edges
    static_edges: list = field(default_factory=list)  # ((v1, v2), friction): lone edges, no ghost vertices
    level_calls: list = field(default_factory=list)  # extra builder calls for the level (anchors)
    dyn: dict = field(default_factory=dict)  # per-world arrays, first axis = world
    builder: object = None  # fn(defn, scene, i) adding the dynamic part of world i
    action_joints: tuple = ()  # joints whose motor speed follows an action channel
    action_scale: tuple = ()
    level: tuple = ()
    rocks: list = field(default_factory=list)  # (x, y, r) of the c1 / c4 rocks
    anchor: tuple = ()

    def build_world(self, defn, i):
        g = defn.add_body(STATIC)
        for verts, fr in self.static_polys:
            defn.add_polygon(g, verts, friction=fr)
        for half, ctr, ang, fr in self.static_boxes:
            defn.add_box(g, tuple(half), tuple(ctr), ang, friction=fr)
        for verts, fr in self.static_chains:
            defn.add_chain(g, verts, friction=fr)
        for (v1, v2), fr in self.static_edges:
            defn.add_edge(g, v1, v2, friction=fr)
        self.builder(defn, self, i)
        return defn

    def world_def(self, i, cls=WorldDef):
        return self.build_world(cls(self.settings), i)


# ---- c0: box drop on a terrain chain (polygon-terrain variant)


def _terrain_quads(heights, x0, dx, floor, friction):
    out = []
    for i in range(len(heights) - 1):
        xa, xb = x0 + i * dx, x0 + (i + 1) * dx
        quad = np.array([(xa, floor), (xb, floor), (xb, heights[i + 1]), (xa, heights[i])], F32)
        out.append((quad, friction))
    return out


def _c0_bodies(defn, sc, i):
    d = sc.dyn
    for k in range(8):
        b = defn.add_body(DYNAMIC, (float(d["x"][i, k]), float(d["y"][i, k])), float(d["angle"][i, k]),
                          mass=0.25, inertia=F32(0.25) * F32(0.5) / F32(12.0))
        defn.add_box(b, (0.25, 0.25), friction=0.6)


def _terrain_chain(heights, x0, dx):
    return np.array([(x0 + i * dx, heights[i]) for i in range(len(heights))], F32)


def c0(seed=0, n=256, terrain="quads"):
    """terrain "quads": the polygon-terrain variant (static quads down to a floor, parity pinned to the reference);
    "chain": BASELINE's own level, one chain of edges (this engine's edge shapes; no reference to pin)."""
    rng = np.random.default_rng(seed)
    h = rng.uniform(-0.5, 0.5, 128).astype(F32)
    x0, dx = -32.0, 0.5
    sc = Scene("c0_box_drop" if terrain == "quads" else "c0_box_drop_chain", _settings(False), 64, 600, n)
    if terrain == "quads":
        sc.static_polys = _terrain_quads(h, x0, dx, -2.0, 0.6)
    else:
        sc.static_chains = [(_terrain_chain(h, x0, dx), 0.6)]
    sc.dyn = _per_world(seed, n, lambda r: dict(x=r.uniform(x0 + 1, x0 + 127 * dx - 1, 8).astype(F32),
                                               y=r.uniform(2, 6, 8).astype(F32),
                                               angle=r.uniform(0, 2 * np.pi, 8).astype(F32)))
    sc.builder = _c0_bodies
    return sc


# ---- c1: character rig (pot, hub, hammer; revolute motor + prismatic slide) on a chain level with rocks


def _rig(defn, sc, i, x, y, ang):
    d = sc.dyn
    pot = defn.add_body(DYNAMIC, (x, y), 0.0, mass=30.0, inertia=5.4)
    defn.add_circle(pot, 0.6, friction=0.8, group=-1)  # group -1: the pot and the hammer never collide
    hub = defn.add_body(DYNAMIC, (x, y), ang, mass=1.0, inertia=0.05)
    hx, hy = (float(d["hx"][i]), float(d["hy"][i])) if "hx" in d else _hammer_at(x, y, ang)
    ham = defn.add_body(DYNAMIC, (hx, hy), ang, mass=2.0, inertia=0.43, bullet=True)
    defn.add_box(ham, (0.7, 0.04), (-0.1, 0.0), friction=0.6, group=-1)
    defn.add_polygon(ham, _HEAD, friction=0.6, group=-1)
    defn.add_revolute(pot, hub, (0, 0), (0, 0), ang, motor_speed=float(d["w0"][i]), max_motor_torque=1000.0,
                      enable_motor=True)
    defn.add_prismatic(hub, ham, (0, 0), (0, 0), (1, 0), 0.0, limits=(0.3, 1.9), motor_speed=0.0,
                       max_motor_force=1000.0, enable_motor=True)
    return pot, hub, ham


_HEAD = [(0.55, -0.08), (0.8, -0.08), (0.85, 0.0), (0.8, 0.08), (0.55, 0.08)]


def _hammer_at(x, y, ang):
    """The hammer's position one arm length along its angle from the pot (host double trig; the device-seeded
    scenes give it explicitly, as dyn["hx"], dyn["hy"])."""
    return x + 1.0 * math.cos(ang), y + 1.0 * math.sin(ang)


def _c1_bodies(defn, sc, i):
    d = sc.dyn
    _rig(defn, sc, i, float(d["x"][i]), float(d["y"][i]), float(d["angle"][i]))


def _level_c1(rng, friction=0.7, terrain="quads"):
    steps = rng.normal(0, 0.15, 2000)
    h = np.concatenate([[0.0], np.cumsum(steps)]).astype(F32)
    x0, dx = -250.0, 0.25
    floor = float(h.min()) - 1.0
    polys = _terrain_quads(h, x0, dx, floor, friction) if terrain == "quads" else []
    rocks = []
    for _ in range(60):
        k = int(rng.integers(3, 9))
        r = float(rng.uniform(0.3, 2.0))
        px = float(rng.uniform(x0 + 5, x0 + 2000 * dx - 5))
        ix = int((px - x0) / dx)
        py = float(h[ix]) + float(rng.uniform(0.0, 3.0))
        polys.append(((_convex(rng, k, r) + np.array([px, py], F32)).astype(F32), friction))
        rocks.append((px, py, r))
    return h, x0, dx, polys, rocks


def _rig_start(h, x0, dx, rocks, r, min_ground=None):
    """The pot resting just above the terrain under it, away from every rock; the hammer above the pot (pointing
    up and to either side), as the character starts in the game. min_ground: only where the ground under the pot is
    above it (c4, whose reset-on-fall rule is pot y < -5)."""
    while True:
        x = r.uniform(x0 + 10, x0 + 2000 * dx - 10)
        i0, i1 = int((x - 0.8 - x0) / dx), int((x + 0.8 - x0) / dx) + 1
        y = float(h[i0:i1 + 1].max()) + 0.62
        if min_ground is not None and float(h[i0:i1 + 1].min()) < min_ground:
            continue
        if all((x - px) ** 2 + (y - py) ** 2 > (rr + 2.8) ** 2 for px, py, rr in rocks):
            break
    ang = r.uniform(0.2 * np.pi, 0.8 * np.pi)
    return dict(x=F32(x), y=F32(y), angle=F32(ang), w0=F32(r.uniform(-2, 2)))


def c1(seed=0, n=4096, terrain="quads"):
    """terrain "quads": the polygon-terrain variant; "chain": BASELINE's 2000-segment edge chain (own edge shapes,
    no reference to pin). The same level, rocks and rig starts either way."""
    rng = np.random.default_rng(seed)
    h, x0, dx, polys, rocks = _level_c1(rng, terrain=terrain)
    sc = Scene("c1_rig" if terrain == "quads" else "c1_rig_chain", _settings(True), 48, 1000, n)
    sc.static_polys = polys
    if terrain != "quads":
        sc.static_chains = [(_terrain_chain(h, x0, dx), 0.7)]
    sc.dyn = _per_world(seed, n, lambda r: _rig_start(h, x0, dx, rocks, r))
    sc.builder = _c1_bodies
    sc.level = (h, x0, dx)
    sc.rocks = rocks
    sc.action_joints, sc.action_scale = (0, 1), (4.0, 2.0)
    return sc


# ---- c2: 256 mixed bodies in a 20 x 20 m box, sleeping off


def _c2_bodies(defn, sc, i):
    d = sc.dyn
    for k in range(256):
        kind = int(d["kind"][k])
        x, y, a = float(d["x"][i, k]), float(d["y"][i, k]), float(d["angle"][i, k])
        m, ctr, inertia = d["mass"][k], d["center"][k], d["inertia"][k]
        b = defn.add_body(DYNAMIC, (x, y), a, mass=float(m), center=tuple(float(c) for c in ctr),
                          inertia=float(inertia))
        e = float(d["restitution"][k])
        if kind == 0:
            defn.add_circle(b, float(d["size"][k, 0]), friction=0.4, restitution=e)
        elif kind == 1:
            defn.add_box(b, (float(d["size"][k, 0]), float(d["size"][k, 1])), friction=0.4, restitution=e)
        else:
            defn.add_polygon(b, d["poly"][k][: int(d["nv"][k])], friction=0.4, restitution=e)


def c2(seed=0, n=1024, bodies=256):
    rng = np.random.default_rng(seed)
    sc = Scene("c2_stress", _settings(False, allow_sleep=False), 6 * bodies, 500, n)
    sc.static_boxes = [((10.0, 0.25), (0.0, -10.25), 0.0, 0.4), ((10.0, 0.25), (0.0, 10.25), 0.0, 0.4),
                       ((0.25, 10.0), (-10.25, 0.0), 0.0, 0.4), ((0.25, 10.0), (10.25, 0.0), 0.0, 0.4)]
    kind = rng.integers(0, 3, bodies)
    size = rng.uniform(0.1, 0.4, (bodies, 2)).astype(F32)
    dens = rng.uniform(0.5, 2.0, bodies)
    nv = rng.integers(5, 9, bodies)
    poly = np.zeros((bodies, 8, 2), F32)
    mass, center, inertia = np.zeros(bodies, F32), np.zeros((bodies, 2), F32), np.zeros(bodies, F32)
    for k in range(bodies):
        if kind[k] == 0:
            r = float(size[k, 0])
            m = dens[k] * np.pi * r * r
            mass[k], inertia[k] = m, 0.5 * m * r * r
        elif kind[k] == 1:
            hx, hy = float(size[k, 0]), float(size[k, 1])
            m = dens[k] * 4 * hx * hy
            mass[k], inertia[k] = m, m * (hx * hx + hy * hy) / 3.0
        else:
            pv = _convex(rng, int(nv[k]), float(size[k, 0]) + 0.05)
            poly[k, : nv[k]] = pv
            m, c, icom = polygon_mass(pv, dens[k])
            mass[k], center[k], inertia[k] = m, c, icom
    side = int(math.ceil(math.sqrt(bodies)))
    gx, gy = np.meshgrid(np.arange(side), np.arange(side))
    gx, gy = gx.ravel()[:bodies], gy.ravel()[:bodies]
    pitch = 18.0 / side
    def draw(r):
        jit = r.uniform(-0.1, 0.1, (bodies, 2))
        return dict(x=(-9.0 + pitch * (gx + 0.5) + jit[:, 0]).astype(F32),
                    y=(-9.0 + pitch * (gy + 0.5) + jit[:, 1]).astype(F32),
                    angle=r.uniform(0, 2 * np.pi, bodies).astype(F32))
    sc.dyn = dict(kind=kind, size=size, nv=nv, poly=poly, mass=mass, center=center, inertia=inertia,
                  restitution=rng.uniform(0, 0.3, bodies).astype(F32), **_per_world(seed, n, draw))
    sc.builder = _c2_bodies
    return sc


# ---- c3: 32 bullet circles among thin static targets


def _c3_bodies(defn, sc, i):
    d = sc.dyn
    for k in range(32):
        b = defn.add_body(DYNAMIC, (float(d["x"][i, k]), float(d["y"][i, k])), 0.0,
                          (float(d["vx"][i, k]), float(d["vy"][i, k])), 0.0, mass=F32(0.0785), inertia=F32(0.0001),
                          bullet=True)
        defn.add_circle(b, 0.05, friction=0.2)


def c3(seed=0, n=8192, terrain="quads"):
    """terrain "quads": the 64 zero-thickness targets as 0.02 m boxes; "chain": as edge shapes (own, unpinned)."""
    rng = np.random.default_rng(seed)
    sc = Scene("c3_toi" if terrain == "quads" else "c3_toi_edges", _settings(True), 256, 300, n)
    boxes = [((10.0, 0.01), (0.0, -10.0), 0.0, 0.3), ((10.0, 0.01), (0.0, 10.0), 0.0, 0.3),
             ((0.01, 10.0), (-10.0, 0.0), 0.0, 0.3), ((0.01, 10.0), (10.0, 0.0), 0.0, 0.3)]
    for _ in range(12):
        boxes.append(((float(rng.uniform(0.5, 2.0)), 0.01), (float(rng.uniform(-8, 8)), float(rng.uniform(-8, 8))),
                      float(rng.uniform(0, np.pi)), 0.3))
    for _ in range(64):  # zero-thickness edges: 0.02 m thick boxes, or edge shapes
        half, cx, cy = float(rng.uniform(0.25, 1.5)), float(rng.uniform(-9, 9)), float(rng.uniform(-9, 9))
        ang = float(rng.uniform(0, np.pi))
        if terrain == "quads":
            boxes.append(((half, 0.01), (cx, cy), ang, 0.3))
        else:
            ca, sa = math.cos(ang) * half, math.sin(ang) * half
            sc.static_edges.append((((cx - ca, cy - sa), (cx + ca, cy + sa)), 0.3))
    sc.static_boxes = boxes
    def draw(r):
        speed, th = r.uniform(50, 200, 32), r.uniform(0, 2 * np.pi, 32)
        return dict(x=r.uniform(-9.5, 9.5, 32).astype(F32), y=r.uniform(-9.5, 9.5, 32).astype(F32),
                    vx=(speed * np.cos(th)).astype(F32), vy=(speed * np.sin(th)).astype(F32))
    sc.dyn = _per_world(seed, n, draw)
    sc.builder = _c3_bodies
    return sc


# ---- c4: the c1 rig plus a 20-link revolute chain hanging from a static anchor


def _c4_bodies(defn, sc, i):
    d = sc.dyn
    x, y = float(d["x"][i]), float(d["y"][i])
    _rig(defn, sc, i, x, y, float(d["angle"][i]))
    ax, ay = sc.anchor  # one anchor for every world: static bodies are shared by the batch
    anchor = defn.add_body(STATIC, (ax, ay))
    defn.add_box(anchor, (0.1, 0.1))
    prev, px = anchor, ax
    for k in range(20):
        ly = ay - 0.5 * (k + 1)
        link = defn.add_body(DYNAMIC, (px, ly), 0.0, mass=0.5, inertia=F32(0.5) * F32(0.26) / F32(12.0))
        defn.add_box(link, (0.05, 0.25), friction=0.5)
        defn.add_revolute(prev, link, (0, -0.1 if k == 0 else -0.25), (0, 0.25), 0.0)
        prev = link


def c4(seed=0, n=65536, terrain="quads"):
    sc = c1(seed, n, terrain)
    h, x0, dx = sc.level
    rocks = _level_c1(np.random.default_rng(seed), terrain=terrain)[4]
    sc.dyn = _per_world(seed, n, lambda r: _rig_start(h, x0, dx, rocks, r, min_ground=-3.0))
    sc.name, sc.capacity, sc.steps = "c4_scale" if terrain == "quads" else "c4_scale_chain", 64, 10000
    sc.builder = _c4_bodies
    h, x0, dx = sc.level
    ix = int((20.0 - x0) / dx)
    sc.anchor = (20.0, float(h[ix]) + 12.0)
    return sc


_FIRST = [0]

DEFAULT_N = {"c0": 256, "c1": 4096, "c2": 1024, "c3": 8192, "c4": 65536}
CONFIGS = {"c0": c0, "c1": c1, "c2": c2, "c3": c3, "c4": c4}
# BASELINE's own levels with edge shapes (chains, lone edges): this engine's edge colliders, parity unpinned


def _edge_variant(base):
    def fn(seed=0, n=None):
        return CONFIGS[base](seed, DEFAULT_N[base] if n is None else n, "chain")
    return fn


for _k in ("c0", "c1", "c3", "c4"):
    CONFIGS[_k + "e"] = _edge_variant(_k)
    DEFAULT_N[_k + "e"] = DEFAULT_N[_k]
del _k


def scene(name, seed=0, n=None, first=0):
    """The workload's Scene; its per-world arrays hold worlds first..first+n-1 (row 0 = world `first`)."""
    fn = CONFIGS[name]
    _FIRST[0] = first
    try:
        return fn(seed) if n is None else fn(seed, n)
    finally:
        _FIRST[0] = 0


# ---- batches


def _cuda():
    try:
        import torch
        return torch.cuda.is_available()
    except ImportError:
        return False


def batch(name, n, seed=0, compact=True, first=0, device_pairs=None, dyn=None):
    """(scene, Model, batched State (leaves (n, ...))) for n worlds of a workload. The Model comes from world 0's
    full build; each world's bodies, joints and dynamic-fixture AABBs come from replaying that world's dynamic
    builder calls on a WorldDef holding only the ground body, so every world equals its full WorldDef build (the
    static level is identical in all of them). compact: the compact fixture layout (static fixtures in the Model).
    device_pairs: build the candidate list on the GPU (default: when CUDA is available). dyn: per-world arrays that
    replace the scene's own draws (seeded_dyn: the placements drawn on the device)."""
    from .world import Fixtures, State, compact_model, compact_state, empty_contacts, empty_toi

    sc = scene(name, seed, n, first)
    if dyn is not None:
        sc.dyn = {**sc.dyn, **dyn}
    full = sc.world_def(0)
    # the candidate list on the GPU when there is one (goib2d_candidate_pairs: the host scan's list, checked equal)
    model, st0 = full.build(sc.capacity, device_pairs=_cuda() if device_pairs is None else device_pairs)
    n_static = sum(1 for f in full.fixtures if f["body"] == 0)  # the level: fixtures of the ground body
    geom = full.fixture_geometry()
    per = []
    for i in range(n):
        d = WorldDef(sc.settings)
        d.add_body(STATIC)
        sc.builder(d, sc, i)
        bodies = d.body_arrays()
        fx = d.fixture_arrays(bodies)
        per.append((bodies, fx, d.joint_arrays()))
    stack = lambda xs: np.stack(xs, 0)  # noqa: E731
    bodies = type(st0.bodies)(*(stack([p[0][k] for p in per]) for k in range(len(st0.bodies))))
    joints = type(st0.joints)(*(stack([p[2][k] for p in per]) for k in range(len(st0.joints))))
    fat = np.broadcast_to(st0.fixtures.fat, (n,) + st0.fixtures.fat.shape).copy()
    fat[:, n_static:] = stack([p[1].fat for p in per])
    fixtures = Fixtures(friction=np.broadcast_to(st0.fixtures.friction, (n,) + st0.fixtures.friction.shape).copy(),
                        restitution=np.broadcast_to(st0.fixtures.restitution,
                                                    (n,) + st0.fixtures.restitution.shape).copy(), fat=fat)
    del geom
    rep = lambda x: np.broadcast_to(x, (n,) + np.shape(x)).copy()  # noqa: E731
    C, B = sc.capacity, bodies.type.shape[1]
    contacts = type(st0.contacts)(*(rep(x) for x in empty_contacts(C)))
    toi = type(st0.toi)(*(rep(x) for x in empty_toi(B, C)))
    state = State(bodies=bodies, fixtures=fixtures, joints=joints, contacts=contacts, gravity=rep(st0.gravity),
                  inv_dt0=rep(st0.inv_dt0), next_key=rep(st0.next_key), new_fixture=rep(st0.new_fixture),
                  overflow=rep(st0.overflow), toi=toi)
    if compact:
        model = compact_model(model, state)
        state = compact_state(model, state, check=False)
    return sc, model, state


# ---- scene spawn on the device (goib2d_spawn, goib2d_seed_placements)

def placements(sc):
    """(first_body, placements float32 (n, k, 6), speed_joints, speeds float32 (n, len) or None) of a Scene's worlds:
    the poses its builder gives bodies 1 .. k (x, y, angle, v.x, v.y, w), as goib2d_spawn takes them."""
    d, n = sc.dyn, sc.n_worlds
    base = sc.name.split("_")[0]
    if base in ("c1", "c4"):
        x, y, a = (np.asarray(d[k], F32) for k in ("x", "y", "angle"))
        if "hx" in d:
            hx, hy = np.asarray(d["hx"], F32), np.asarray(d["hy"], F32)
        else:
            hx, hy = (np.array(v, F32) for v in zip(*[_hammer_at(float(x[i]), float(y[i]), float(a[i]))
                                                    for i in range(n)]))
        z = np.zeros(n, F32)
        pl = np.stack([np.stack([x, y, z, z, z, z], -1), np.stack([x, y, a, z, z, z], -1),
                       np.stack([hx, hy, a, z, z, z], -1)], 1)
        return 1, pl, (0,), np.asarray(d["w0"], F32).reshape(n, 1)
    if base == "c3":
        x, y, vx, vy = (np.asarray(d[k], F32) for k in ("x", "y", "vx", "vy"))
        z = np.zeros_like(x)
        return 1, np.stack([x, y, z, vx, vy, z], -1), (), None
    x, y, a = (np.asarray(d[k], F32) for k in ("x", "y", "angle"))  # c0, c2
    z = np.zeros_like(x)
    return 1, np.stack([x, y, a, z, z, z], -1), (), None


def spawn_rule(sc, host=False):
    """The goib2d_spawn_rule of a workload's device-seeded variant (the same spawn pattern as its numpy draws, from
    Philox streams per (seed, world) instead), and the arrays it points at (keep them alive while it is used):
    device tensors, or host numpy arrays with host=True (for the parity oracle)."""
    from . import native
    r = native.SpawnRule()
    base = sc.name.split("_")[0]
    keep = ()
    if base == "c0":
        x0, dx = -32.0, 0.5
        r.kind, r.n_bodies = native.SPAWN_UNIFORM, 8
        r.x_lo, r.x_hi, r.y_lo, r.y_hi = x0 + 1, x0 + 127 * dx - 1, 2.0, 6.0
        r.angle_lo, r.angle_hi = 0.0, 2 * np.pi
    elif base == "c2":
        k = len(sc.dyn["kind"])
        side = int(math.ceil(math.sqrt(k)))
        r.kind, r.n_bodies, r.grid_side = native.SPAWN_GRID, k, side
        r.grid_x0 = r.grid_y0 = -9.0
        r.grid_pitch, r.jitter, r.angle_lo, r.angle_hi = 18.0 / side, 0.1, 0.0, 2 * np.pi
    elif base == "c3":
        r.kind, r.n_bodies = native.SPAWN_UNIFORM, 32
        r.x_lo, r.x_hi, r.y_lo, r.y_hi, r.speed_lo, r.speed_hi = -9.5, 9.5, -9.5, 9.5, 50.0, 200.0
    elif base in ("c1", "c4"):
        h, x0, dx = sc.level
        heights = np.ascontiguousarray(h, F32)
        discs = np.ascontiguousarray(np.asarray(sc.rocks, F32).reshape(-1, 3))
        if host:
            keep, ph, pd = (heights, discs), heights.ctypes.data, discs.ctypes.data
        else:
            import torch
            keep = (torch.from_numpy(heights).cuda(), torch.from_numpy(discs).cuda())
            ph, pd = keep[0].data_ptr(), keep[1].data_ptr()
        r.kind, r.n_bodies = native.SPAWN_RIG, 3
        r.x_lo, r.x_hi = x0 + 10, x0 + 2000 * dx - 10
        r.heights, r.n_heights, r.h_x0, r.h_dx = ph, len(heights), x0, dx
        r.half_width, r.lift, r.arm = 0.8, 0.62, 1.0
        r.min_ground = -3.0 if base == "c4" else -np.inf
        r.discs, r.n_discs, r.clearance, r.max_tries = pd, len(discs), 2.8, 64
        r.angle_lo, r.angle_hi, r.speed_lo, r.speed_hi = 0.2 * np.pi, 0.8 * np.pi, -2.0, 2.0
    else:
        raise ValueError(f"no spawn rule for {sc.name}")
    return r, keep


def seeded_dyn(sc, pl, speeds):
    """The per-world Scene arrays equal to device-drawn placements (host numpy), for building the same worlds through
    WorldDef (batch(..., dyn=...))."""
    pl = np.asarray(pl, F32)
    base = sc.name.split("_")[0]
    if base in ("c1", "c4"):
        return dict(x=pl[:, 0, 0], y=pl[:, 0, 1], angle=pl[:, 1, 2], hx=pl[:, 2, 0], hy=pl[:, 2, 1],
                    w0=np.asarray(speeds, F32))
    if base == "c3":
        return dict(x=pl[..., 0], y=pl[..., 1], vx=pl[..., 3], vy=pl[..., 4])
    return dict(x=pl[..., 0], y=pl[..., 1], angle=pl[..., 2])


def spawn_batch(name, n, seed=0, first=0, seeded=False, device_pairs=None):
    """(scene, Model, device State, placements, speeds) of n worlds built on the device: the template world (the
    first) from the host builder, every world placed by goib2d_spawn. seeded=False: the scene's own numpy draws (the
    State equals batch(name, n, seed, first=first)); True: placements drawn on the device by goib2d_seed_placements
    (the workload's device-seeded variant, equal to batch(..., dyn=seeded_dyn(...)) of the same draws), with no
    per-world host work."""
    import torch

    from . import api
    sc = scene(name, seed, 1 if seeded else n, first)
    dyn = None
    if seeded:
        rule, keep = spawn_rule(sc)
        pl, sp = api.seed_placements(rule, seed, first, n)
        torch.cuda.current_stream().synchronize()
        del keep
        dyn = seeded_dyn(sc, pl[:1].cpu().numpy(), None if sp is None else sp[:1].cpu().numpy())
    else:
        _, pl_np, _, sp_np = placements(sc)
        pl = torch.from_numpy(pl_np).cuda()
        sp = torch.from_numpy(sp_np).cuda() if sp_np is not None else None
    sc1, model, tmpl_host = batch(name, 1, seed, first=first, device_pairs=device_pairs, dyn=dyn)
    eng = api.Engine(model, tmpl_host.bodies.type.shape[1])
    try:
        state = eng.spawn(api.to_device(tmpl_host), n, 1, pl, (0,) if sp is not None else (), sp)
        torch.cuda.current_stream().synchronize()
    finally:
        eng.close()
    return sc1, model, state, pl, sp
