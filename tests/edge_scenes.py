"""Scenes with edge shapes (single edges, chains with ghost vertices) for the edge tests. The reference engine has
no edge shapes, so these scenes pin the CUDA engine to the oracle's restatement of the same method and to expected
behaviour (resting heights, no catching on a chain's inner vertices, no tunnelling), not to reference states."""
import numpy as np

from goib2d.settings import Settings
from goib2d.world import DYNAMIC, STATIC, WorldDef

F32 = np.float32
DT = F32(1.0 / 60.0)


def circle_on_edge():
    d = WorldDef(Settings.stock())
    g = d.add_body(STATIC)
    d.add_edge(g, (-5.0, 0.0), (5.0, 0.0))
    b = d.add_body(DYNAMIC, (0.3, 1.0), mass=0.785, inertia=0.098)
    d.add_circle(b, 0.5, friction=0.6)
    return d


def box_on_chain(ghosts=True, vx=5.0, friction=0.0):
    """A box moving along a flat ground of 40 collinear 0.5 m segments (a chain, or lone edges without ghosts)."""
    d = WorldDef(Settings.stock())
    g = d.add_body(STATIC)
    xs = np.linspace(-10.0, 10.0, 41)
    verts = [(float(x), 0.0) for x in xs]
    if ghosts:
        d.add_chain(g, verts, friction=friction)
    else:
        for a, b in zip(verts[:-1], verts[1:]):
            d.add_edge(g, a, b, friction=friction)
    b = d.add_body(DYNAMIC, (-8.0, 0.26), velocity=(vx, 0.0), mass=0.5, inertia=F32(0.5) * F32(1.25) / F32(12.0))
    d.add_box(b, (0.5, 0.25), friction=friction)
    return d


def slope_chain():
    """Circles and polygons tumbling down a bumpy chain with a loop at the bottom: every edge collider path, with
    continuous collision on (edge proxies in b2TimeOfImpact)."""
    d = WorldDef(Settings.stock(continuous_physics=True))
    g = d.add_body(STATIC)
    rng = np.random.default_rng(5)
    xs = np.linspace(-12.0, 6.0, 37)
    ys = -0.4 * xs + rng.uniform(-0.15, 0.15, xs.shape)
    d.add_chain(g, np.stack([xs, ys], 1), friction=0.5)
    d.add_chain(g, [(7.0, -4.0), (11.0, -4.0), (11.0, -1.0), (7.0, -1.0)], loop=True, friction=0.5)
    d.add_edge(g, (6.0, -2.6), (7.0, -4.5), friction=0.3)
    for k in range(4):
        b = d.add_body(DYNAMIC, (-10.0 + 1.3 * k, 6.5 + 0.7 * k), 0.3 * k, mass=1.0, inertia=0.1)
        if k % 2:
            d.add_circle(b, 0.3, friction=0.5)
        else:
            d.add_polygon(b, [(-0.3, -0.2), (0.35, -0.25), (0.4, 0.2), (0.0, 0.35), (-0.35, 0.15)], friction=0.5)
    return d


def bullet_at_edge():
    """A 0.05 m bullet circle at 120 m/s towards a lone edge 1 m away: continuous collision stops it."""
    d = WorldDef(Settings.stock(continuous_physics=True))
    g = d.add_body(STATIC)
    d.add_edge(g, (1.0, -2.0), (1.0, 2.0))
    b = d.add_body(DYNAMIC, (0.0, 0.0), velocity=(120.0, 0.0), mass=0.0785, inertia=0.0001, bullet=True)
    d.add_circle(b, 0.05, friction=0.2)
    return d


SCENES = {"circle_on_edge": circle_on_edge, "box_on_chain": box_on_chain,
          "box_on_edges": lambda: box_on_chain(ghosts=False), "slope_chain": slope_chain,
          "bullet_at_edge": bullet_at_edge}


def build(name, capacity=32):
    return SCENES[name]().build(capacity)
