"""Edge and chain shapes (this engine's addition: the reference engine has none, so parity with it is unpinned).
On the CPU: the oracle's restatement of Box2D's edge method behaves as the method promises, and the host builder
and the C ABI handle edges; the CUDA engine is held to the oracle bit for bit in test_gpu_parity.py."""
import ctypes

import numpy as np
import pytest

import edge_scenes
import oracle_lib
from goib2d import native, shapes
from goib2d.world import map_state


def run(name, steps, capacity=32):
    model, state = edge_scenes.build(name, capacity)
    out, traj = state, []
    for _ in range(steps):
        out = oracle_lib.step(model, out, edge_scenes.SCENES[name]().settings, edge_scenes.DT, 1)
        traj.append(out)
    return model, traj


def test_circle_comes_to_rest_on_an_edge():
    _, traj = run("circle_on_edge", 180)
    c, v = traj[-1].bodies.c[1], traj[-1].bodies.v[1]
    # rests on the two skins (circle 0.5 + edge polygon radius 0.01) less the solver's allowed penetration
    assert 0.5 < c[1] < 0.5 + 0.01 + 1e-4, c
    assert abs(float(v[1])) < 1e-3 and abs(float(c[0]) - 0.3) < 1e-3


def test_box_slides_over_a_chain_without_catching():
    """Frictionless box across 40 collinear segments: the ghost vertices keep every contact normal straight up, so
    the box keeps its speed and does not rotate at the inner vertices."""
    _, traj = run("box_on_chain", 150)
    vx = np.array([float(s.bodies.v[1][0]) for s in traj])
    w = np.array([float(s.bodies.w[1]) for s in traj])
    y = np.array([float(s.bodies.c[1][1]) for s in traj])
    assert vx.min() > 4.99 and np.abs(w).max() < 1e-3, (vx.min(), np.abs(w).max())
    assert 0.25 < y.min() and y.max() < 0.27
    assert float(traj[-1].bodies.c[1][0]) > 3.0  # it crossed many inner vertices


def test_lone_edges_can_catch_where_a_chain_does_not():
    """The same ground as separate edges (no ghost vertices) admits normals off vertical at the joints."""
    _, chain = run("box_on_chain", 150)
    _, lone = run("box_on_edges", 150)
    dev = lambda tr: max(abs(float(s.bodies.v[1][1])) + abs(float(s.bodies.w[1])) for s in tr)  # noqa: E731
    assert dev(chain) <= dev(lone)


def test_bullet_stops_at_an_edge():
    _, traj = run("bullet_at_edge", 30)
    x = max(float(s.bodies.c[1][0]) for s in traj)
    assert x < 1.0 - 0.05 + 0.02, x  # never passes the edge at x = 1 (radius 0.05, skins)


def test_chain_children_carry_their_neighbours_as_ghost_vertices():
    d = edge_scenes.box_on_chain()
    model, _ = d.build(16)
    edges = np.flatnonzero(model.shape_type == shapes.EDGE)
    assert len(edges) == 40
    g = model.edge_ghost[edges]
    assert g[0] == 2 and g[-1] == 1 and (g[1:-1] == 3).all()
    for i in edges[1:-1]:  # v0 = previous edge's v1, v3 = next edge's v2
        assert np.array_equal(model.verts[i, 2], model.verts[i - 1, 0])
        assert np.array_equal(model.verts[i, 3], model.verts[i + 1, 1])


def test_candidate_pairs_put_the_edge_first_and_skip_edge_pairs():
    model, _ = edge_scenes.build("slope_chain")
    st = model.shape_type
    assert (st[model.pair_b] != shapes.EDGE).all()
    assert not ((st[model.pair_a] == shapes.EDGE) & (st[model.pair_b] == shapes.EDGE)).any()
    assert (st[model.pair_a] == shapes.EDGE).sum() > 0


def test_chain_loop_closes():
    d = edge_scenes.slope_chain()
    model, _ = d.build(16)
    loop = [i for i, f in enumerate(d.fixtures) if f["shape_type"] == shapes.EDGE][36:40]
    assert np.array_equal(model.verts[loop[0], 2], model.verts[loop[-1], 0])  # first's v0 = last's v1
    assert np.array_equal(model.verts[loop[-1], 3], model.verts[loop[0], 1])  # last's v3 = first's v2


def test_model_create_rejects_an_edge_listed_second_without_a_gpu():
    if not native.lib_path().exists():
        pytest.skip("libgoib2d.so not built")
    model, _ = edge_scenes.build("circle_on_edge")
    bad = model._replace(pair_a=model.pair_b.copy(), pair_b=model.pair_a.copy())
    lib = native.load()
    pm = native.model_desc(bad, 2)
    h = ctypes.c_void_p()
    assert lib.goib2d_model_create(ctypes.byref(pm.desc), ctypes.byref(h)) == -1
    assert b"edge" in lib.goib2d_last_error()


def test_edge_worlds_are_independent_in_a_batch():
    """A batch of perturbed copies equals stepping each world alone (the oracle's batch path)."""
    model, st = edge_scenes.build("slope_chain")
    n = 4
    batch = map_state(lambda x: np.repeat(np.asarray(x)[None], n, 0), st)
    batch.bodies.v[:, 1:] += np.random.default_rng(2).normal(0, 0.5, batch.bodies.v[:, 1:].shape).astype(np.float32)
    s = edge_scenes.slope_chain().settings
    out = oracle_lib.step(model, batch, s, edge_scenes.DT, 40)
    for i in range(n):
        one = oracle_lib.step(model, map_state(lambda x: np.asarray(x)[i], batch), s, edge_scenes.DT, 40)
        for a, b in zip(oracle_lib.state_leaves(map_state(lambda x: np.asarray(x)[i], out)),
                        oracle_lib.state_leaves(one)):
            assert np.array_equal(np.asarray(a), np.asarray(b))


def _world_normals(st, box):
    """The world-frame normals (from the static edge to the box) of the box's touching contacts."""
    from goib2d.world import FACE_A
    out = []
    for s in range(st.contacts.pair.shape[0]):
        if st.contacts.pair[s] < 0 or not st.contacts.touching[s] or st.contacts.count[s] == 0:
            continue
        n = np.asarray(st.contacts.local_normal[s], np.float64)
        if int(st.contacts.mtype[s]) == FACE_A:  # the edge (body 0, identity transform) holds the reference face
            out.append(n)
        else:  # the box's face: rotate into the world and flip (the normal points from the edge to the box)
            c, sn = float(st.bodies.xf_q[box][0]), float(st.bodies.xf_q[box][1])
            out.append(-np.array([c * n[0] - sn * n[1], sn * n[0] + c * n[1]]))
    return out


def _settle(verts, pos, angle=0.0, steps=300, friction=0.8):
    from goib2d.settings import Settings
    from goib2d.world import DYNAMIC, STATIC, WorldDef
    d = WorldDef(Settings.stock())
    g = d.add_body(STATIC)
    d.add_chain(g, verts, friction=friction)
    b = d.add_body(DYNAMIC, pos, angle, mass=1.0, inertia=1.0 / 24.0)
    d.add_box(b, (0.25, 0.25), friction=friction)
    model, st = d.build(16)
    for _ in range(steps):
        st = oracle_lib.step(model, st, d.settings, edge_scenes.DT, 1)
    return st


def test_box_in_a_concave_chain_vertex_takes_both_face_normals():
    """Known answer: a box at rest in a 90-degree V of a chain touches both walls, and every contact normal is a wall's
    face normal (perpendicular to its segment, pointing into the V) - the concave vertex admits no other normal."""
    st = _settle([(-3.0, 3.0), (0.0, 0.0), (3.0, 3.0)], (0.05, 1.5), angle=0.7853982)
    assert np.abs(st.bodies.v[1]).max() < 1e-3 and abs(float(st.bodies.w[1])) < 1e-3
    ns = _world_normals(st, 1)
    r = 1.0 / np.sqrt(2.0)
    walls = [np.array([r, r]), np.array([-r, r])]  # left wall's normal (into the V) and the right wall's
    hit = [min(range(2), key=lambda k: np.abs(n - walls[k]).max()) for n in ns]
    assert set(hit) == {0, 1}, ns
    for n, k in zip(ns, hit):
        assert np.abs(n - walls[k]).max() < 1e-6, (n, walls[k])


def test_box_over_a_convex_chain_vertex_keeps_the_flat_normal():
    """Known answer: a box resting on the flat part of a chain with a corner past a convex vertex (the ground falls
    away beyond it) keeps the flat segment's normal (0, 1) at every contact and does not tip: the ghost vertex
    excludes the vertex normals a lone edge would produce."""
    st = _settle([(-3.0, 0.0), (0.0, 0.0), (2.0, -2.0)], (-0.1, 0.27))
    assert abs(float(st.bodies.a[1])) < 1e-4 and np.abs(st.bodies.v[1]).max() < 1e-3
    ns = _world_normals(st, 1)
    # (0, 1) up to the box's own resting tilt (a few 1e-6 rad) where its face is the reference; a vertex normal at
    # this corner would lean towards the slope's normal (0.71, 0.71)
    assert ns and all(np.abs(n - np.array([0.0, 1.0])).max() < 1e-4 for n in ns), ns
