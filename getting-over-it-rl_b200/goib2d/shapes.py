"""Host-side shape construction in float32: b2PolygonShape::Set / SetAsBox and b2CircleShape, v2.3.1.

Mirrors goi_jax/box2d/shapes.py (reference shapes.py:36-146): the same vertex, normal and AABB floats, because the
CUDA engine and the reference must start from bit-identical geometry. Every product and sum below is a separate
float32 rounding in Box2D's C evaluation order (no fused multiply-add).
"""
import math

import numpy as np

from .settings import AABB_EXTENSION, AABB_MULTIPLIER, EPSILON, MAX_POLYGON_VERTICES

F32 = np.float32
CIRCLE, EDGE, POLYGON = 0, 1, 2  # b2Shape::Type. Edges are this engine's own addition (the reference engine has
# neither edges nor chains); a chain is built as a run of edge fixtures with ghost vertices (WorldDef.add_chain).


def host_sin_cos(a):
    """(float)sin((double)a), (float)cos((double)a): the C library's double trig rounded once (reference
    math2d.py:321-325). Used only while building scenes on the host."""
    x = float(F32(a))
    return F32(math.sin(x)), F32(math.cos(x))


def normalize(x, y):
    """b2Vec2::Normalize in float32: unchanged below b2_epsilon, else times 1/length."""
    x, y = F32(x), F32(y)
    n = F32(np.sqrt(F32(F32(x * x) + F32(y * y))))
    if n < EPSILON:
        return x, y
    inv = F32(F32(1.0) / n)
    return F32(x * inv), F32(y * inv)


def edge_normals(v):
    """b2PolygonShape::Set's edge normals: Normalize(b2Cross(v[i+1] - v[i], 1.0f)), i.e. (1*e.y, -1*e.x)."""
    k = len(v)
    out = np.zeros((k, 2), F32)
    for i in range(k):
        a, b = v[i], v[(i + 1) % k]
        ex, ey = F32(b[0] - a[0]), F32(b[1] - a[1])
        out[i] = normalize(F32(F32(1.0) * ey), F32(F32(-1.0) * ex))
    return out


def polygon_raw(vertices):
    """Vertices verbatim (must be strictly convex and counter-clockwise), normals derived as Set derives them."""
    v = np.asarray(vertices, F32).reshape(-1, 2)
    k = len(v)
    if k < 3 or k > MAX_POLYGON_VERTICES:
        raise ValueError("polygon needs 3..8 vertices")
    for i in range(k):
        ex, ey = v[(i + 1) % k] - v[i]
        for j in range(2, k):
            dx, dy = v[(i + j) % k] - v[i]
            if F32(F32(ex * dy) - F32(ey * dx)) <= 0:
                raise ValueError("polygon not strictly convex CCW")
    return v, edge_normals(v)


def _dist2(p, q):
    dx, dy = F32(p[0] - q[0]), F32(p[1] - q[1])
    return F32(F32(dx * dx) + F32(dy * dy))


def polygon_set(vertices, linear_slop):
    """b2PolygonShape::Set v2.3.1: weld points whose squared distance is below 0.5*linearSlop, then gift-wrap the
    hull counter-clockwise from the rightmost (lowest on ties) point. Raises where Box2D would fall back to a box."""
    pts = [(F32(p[0]), F32(p[1])) for p in np.asarray(vertices, F32).reshape(-1, 2)[:MAX_POLYGON_VERTICES]]
    weld = F32(F32(0.5) * F32(linear_slop))
    kept = []
    for p in pts:
        if all(_dist2(p, q) >= weld for q in kept):
            kept.append(p)
    n = len(kept)
    if n < 3:
        raise ValueError("degenerate polygon (Box2D would use SetAsBox(1, 1))")
    start = 0
    for i in range(1, n):
        if kept[i][0] > kept[start][0] or (kept[i][0] == kept[start][0] and kept[i][1] < kept[start][1]):
            start = i
    hull = []
    cur = start
    while True:
        hull.append(cur)
        nxt = 0
        for j in range(1, n):
            if nxt == cur:
                nxt = j
                continue
            o = kept[hull[-1]]
            rx, ry = F32(kept[nxt][0] - o[0]), F32(kept[nxt][1] - o[1])
            vx, vy = F32(kept[j][0] - o[0]), F32(kept[j][1] - o[1])
            c = F32(F32(rx * vy) - F32(ry * vx))
            if c < 0:
                nxt = j
            if c == 0 and F32(F32(vx * vx) + F32(vy * vy)) > F32(F32(rx * rx) + F32(ry * ry)):
                nxt = j
        cur = nxt
        if nxt == start:
            break
    if len(hull) < 3:
        raise ValueError("degenerate hull")
    v = np.array([kept[i] for i in hull], F32)
    return v, edge_normals(v)


def box(hx, hy, center=(0.0, 0.0), angle=0.0):
    """b2PolygonShape::SetAsBox(hx, hy, center, angle): the axis box, rotated by b2Rot(angle), then shifted."""
    hx, hy = F32(hx), F32(hy)
    corners = [(-hx, -hy), (hx, -hy), (hx, hy), (-hx, hy)]
    norms = [(F32(0), F32(-1)), (F32(1), F32(0)), (F32(0), F32(1)), (F32(-1), F32(0))]
    s, c = host_sin_cos(angle)
    px, py = F32(center[0]), F32(center[1])
    v = np.zeros((4, 2), F32)
    n = np.zeros((4, 2), F32)
    for i in range(4):
        x, y = corners[i]
        v[i, 0] = F32(F32(F32(c * x) - F32(s * y)) + px)
        v[i, 1] = F32(F32(F32(s * x) + F32(c * y)) + py)
        x, y = norms[i]
        n[i, 0] = F32(F32(c * x) - F32(s * y))
        n[i, 1] = F32(F32(s * x) + F32(c * y))
    return v, n


def pad(v, n):
    """(8, 2) vertex / normal tables padded with entry 0 (pads are masked by the vertex count)."""
    k = len(v)
    vv = np.repeat(np.asarray(v, F32)[:1], MAX_POLYGON_VERTICES, axis=0)
    nn = np.repeat(np.asarray(n, F32)[:1], MAX_POLYGON_VERTICES, axis=0)
    vv[:k], nn[:k] = v, n
    return vv, nn


def fixture_aabbs(shape_type, count, radius, verts, px, py, c, s):
    """b2Shape::ComputeAABB for fixtures given their bodies' transforms ((F,) float32 arrays each): polygon vertices
    through b2Mul(xf, v), min/max, minus/plus the skin radius; circles at xf.p + b2Mul(xf.q, centre) +- radius."""
    vx, vy = verts[..., 0], verts[..., 1]
    with np.errstate(all="ignore"):
        wx = (c[:, None] * vx - s[:, None] * vy).astype(F32) + px[:, None]
        wy = (s[:, None] * vx + c[:, None] * vy).astype(F32) + py[:, None]
    # the products above are float32 x float32 -> float32 (numpy does not fuse); sums are float32
    valid = np.arange(MAX_POLYGON_VERTICES)[None, :] < count[:, None]
    lx = np.where(valid, wx, np.inf).min(1).astype(F32)
    ly = np.where(valid, wy, np.inf).min(1).astype(F32)
    ux = np.where(valid, wx, -np.inf).max(1).astype(F32)
    uy = np.where(valid, wy, -np.inf).max(1).astype(F32)
    rx = (c * vx[:, 0] - s * vy[:, 0]).astype(F32)
    ry = (s * vx[:, 0] + c * vy[:, 0]).astype(F32)
    cx, cy = (px + rx).astype(F32), (py + ry).astype(F32)
    circ = shape_type == CIRCLE
    r = radius
    return (np.where(circ, cx - r, lx - r).astype(F32), np.where(circ, cy - r, ly - r).astype(F32),
            np.where(circ, cx + r, ux + r).astype(F32), np.where(circ, cy + r, uy + r).astype(F32))


def fatten(lx, ly, ux, uy):
    """b2DynamicTree::CreateProxy's fat AABB: the shape AABB extended by b2_aabbExtension on every side."""
    e = AABB_EXTENSION
    return (lx - e).astype(F32), (ly - e).astype(F32), (ux + e).astype(F32), (uy + e).astype(F32)


__all__ = ["CIRCLE", "EDGE", "POLYGON", "AABB_MULTIPLIER", "box", "polygon_set", "polygon_raw", "pad", "fixture_aabbs",
           "fatten", "host_sin_cos", "normalize", "edge_normals"]
