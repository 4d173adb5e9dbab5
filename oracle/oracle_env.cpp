// Parity oracle (test infrastructure, see oracle.h): the env helpers' ray casts restated on the host, one world and
// one ray at a time, testing every fixture of every static body (the device walks its static-fixture grid; the
// nearest hit is the same). Shape ray casts follow Box2D 2.3.1's b2CircleShape / b2PolygonShape / b2EdgeShape
// ::RayCast with maxFraction 1; the ray is taken into the fixture body's frame first.
#include "oracle.h"

namespace orc {
namespace {
float cast_circle(V2 p1, V2 d, V2 centre, float r) {
    const V2 s = sub(p1, centre);
    const float b = dot(s, s) - r * r;
    const float c = dot(s, d), rr = dot(d, d);
    const float sigma = c * c - rr * b;
    if (sigma < 0.0f || rr < EPS) return 1.0f;
    const float a = -(c + std::sqrt(sigma));
    return (0.0f <= a && a <= rr) ? a / rr : 1.0f;
}
float cast_polygon(V2 p1, V2 d, const float *v, const float *n, int count) {
    float lo = 0.0f, hi = 1.0f;
    bool entered = false;
    for (int i = 0; i < count; ++i) {
        const V2 ni{n[2 * i], n[2 * i + 1]}, vi{v[2 * i], v[2 * i + 1]};
        const float num = dot(ni, sub(vi, p1)), den = dot(ni, d);
        if (den == 0.0f) {
            if (num < 0.0f) return 1.0f;  // parallel to this face and outside it
        } else if (den < 0.0f && num < lo * den) {
            lo = num / den, entered = true;  // entering through this face, later than so far
        } else if (den > 0.0f && num < hi * den) {
            hi = num / den;  // leaving through this face, earlier than so far
        }
        if (hi < lo) return 1.0f;
    }
    return entered ? lo : 1.0f;
}
float cast_edge(V2 p1, V2 d, V2 a, V2 b) {
    const V2 e = sub(b, a);
    const V2 nrm = normalize(V2{e.y, -e.x});
    const float num = dot(nrm, sub(a, p1)), den = dot(nrm, d);
    if (den == 0.0f) return 1.0f;
    const float t = num / den;
    if (t < 0.0f || 1.0f < t) return 1.0f;
    const V2 q{p1.x + t * d.x, p1.y + t * d.y};
    const float ee = dot(e, e);
    if (ee == 0.0f) return 1.0f;
    const float along = dot(sub(q, a), e) / ee;
    return (along < 0.0f || 1.0f < along) ? 1.0f : t;
}
}  // namespace
}  // namespace orc

using namespace orc;

// out[w * n_rays + k] = nearest hit fraction of ray k of world w (see goib2d_raycast in include/goib2d.h)
extern "C" int oracle_raycast(const goib2d_model_desc *desc, int32_t rows, int64_t n_worlds, void *const *leaves,
                              int32_t body, int32_t n_rays, float max_length, float *out) {
    const int B = desc->n_bodies, F = desc->n_fixtures;
    (void)rows;
    for (int64_t w = 0; w < n_worlds; ++w) {
        const float *c = (const float *)leaves[GOIB2D_B_C] + w * 2 * B;
        const float *xp = (const float *)leaves[GOIB2D_B_XF_P] + w * 2 * B;
        const float *xq = (const float *)leaves[GOIB2D_B_XF_Q] + w * 2 * B;
        const int32_t *type = (const int32_t *)leaves[GOIB2D_B_TYPE] + w * B;
        for (int k = 0; k < n_rays; ++k) {
            const Rot dir = rot_of((float)k * (2.0f * PI_F / (float)n_rays));
            const V2 p1{c[2 * body], c[2 * body + 1]};
            const V2 d{max_length * dir.c, max_length * dir.s};
            float best = 1.0f;
            for (int f = 0; f < F; ++f) {
                const int b = desc->fixture_body[f];
                if (type[b] != STATIC) continue;
                const Xf xf{{xp[2 * b], xp[2 * b + 1]}, {xq[2 * b], xq[2 * b + 1]}};
                const V2 lp = xf_mul_t(xf, p1), ld = rot_t(xf.q, d);
                const float *v = desc->verts + 16 * f;
                float t;
                if (desc->shape_type[f] == CIRCLE)
                    t = cast_circle(lp, ld, V2{v[0], v[1]}, desc->radius[f]);
                else if (desc->shape_type[f] == EDGE)
                    t = cast_edge(lp, ld, V2{v[0], v[1]}, V2{v[2], v[3]});
                else
                    t = cast_polygon(lp, ld, v, desc->normals + 16 * f, desc->count[f]);
                best = std::fmin(best, t);
            }
            out[w * n_rays + k] = best;
        }
    }
    return 0;
}
