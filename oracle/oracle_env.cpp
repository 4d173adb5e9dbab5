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

// ---------------------------------------------------------------- seeded per-world placements (goib2d_seed_placements)
// The device generator restated one world at a time: Philox4x32-10 (Salmon et al., SC'11) keyed by the seed, counter
// (world low, world high, block, 0), draw d = word d % 4 of block d / 4; uniform on [lo, hi) = lo + (hi - lo) * u with
// u = (word >> 8) * 2^-24, float32; the rules as include/goib2d.h states them.
namespace orc {
namespace {
void philox4x32_10(uint32_t ctr[4], uint32_t k0, uint32_t k1) {
    for (int r = 0; r < 10; ++r) {
        if (r) k0 += 0x9E3779B9u, k1 += 0xBB67AE85u;
        const uint64_t p0 = (uint64_t)0xD2511F53u * ctr[0], p1 = (uint64_t)0xCD9E8D57u * ctr[2];
        const uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0, hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        const uint32_t n0 = hi1 ^ ctr[1] ^ k0, n2 = hi0 ^ ctr[3] ^ k1;
        ctr[0] = n0, ctr[1] = lo1, ctr[2] = n2, ctr[3] = lo0;
    }
}
struct Draws {
    uint32_t k0, k1;
    uint64_t world;
    float uniform(uint32_t d, float lo, float hi) const {
        uint32_t c[4] = {(uint32_t)world, (uint32_t)(world >> 32), d >> 2, 0u};
        philox4x32_10(c, k0, k1);
        const float u = (float)(c[d & 3] >> 8) * 0x1p-24f;
        return lo + (hi - lo) * u;
    }
};
constexpr float TWO_PI = 6.28318548202514648f;
}  // namespace
}  // namespace orc

extern "C" {
// One Philox4x32-10 block (known-answer tests): ctr[4] in, out[4] = the block.
void oracle_philox4x32_10(const uint32_t *ctr, uint32_t k0, uint32_t k1, uint32_t *out) {
    uint32_t c[4] = {ctr[0], ctr[1], ctr[2], ctr[3]};
    orc::philox4x32_10(c, k0, k1);
    for (int i = 0; i < 4; ++i) out[i] = c[i];
}

int oracle_seed_placements(const goib2d_spawn_rule *r, uint64_t seed, int64_t first_world, int64_t n_worlds,
                           float *placements, float *speeds) {
    using namespace orc;
    const int nb = r->kind == GOIB2D_SPAWN_RIG ? 3 : r->n_bodies;
    for (int64_t i = 0; i < n_worlds; ++i) {
        const Draws g{(uint32_t)seed, (uint32_t)(seed >> 32), (uint64_t)(first_world + i)};
        float *out = placements + i * nb * 6;
        if (r->kind == GOIB2D_SPAWN_UNIFORM) {
            for (int k = 0; k < nb; ++k) {
                const uint32_t d = 5u * (uint32_t)k;
                const float x = g.uniform(d, r->x_lo, r->x_hi), y = g.uniform(d + 1, r->y_lo, r->y_hi);
                const float ang = g.uniform(d + 2, r->angle_lo, r->angle_hi);
                const float speed = g.uniform(d + 3, r->speed_lo, r->speed_hi);
                const Rot h = rot_of(g.uniform(d + 4, 0.0f, TWO_PI));
                float *o = out + 6 * k;
                o[0] = x, o[1] = y, o[2] = ang, o[3] = speed * h.c, o[4] = speed * h.s, o[5] = 0.0f;
            }
        } else if (r->kind == GOIB2D_SPAWN_GRID) {
            for (int k = 0; k < nb; ++k) {
                const uint32_t d = 3u * (uint32_t)k;
                const float gx = (float)(k % r->grid_side) + 0.5f, gy = (float)(k / r->grid_side) + 0.5f;
                float *o = out + 6 * k;
                o[0] = (r->grid_x0 + r->grid_pitch * gx) + g.uniform(d, -r->jitter, r->jitter);
                o[1] = (r->grid_y0 + r->grid_pitch * gy) + g.uniform(d + 1, -r->jitter, r->jitter);
                o[2] = g.uniform(d + 2, r->angle_lo, r->angle_hi), o[3] = o[4] = o[5] = 0.0f;
            }
        } else {
            const int last = r->n_heights - 1;
            float x = 0.0f, y = 0.0f;
            for (int t = 0; t < r->max_tries; ++t) {
                x = g.uniform((uint32_t)t, r->x_lo, r->x_hi);
                int i0 = (int)((x - r->half_width - r->h_x0) / r->h_dx);
                int i1 = (int)((x + r->half_width - r->h_x0) / r->h_dx) + 1;
                i0 = i0 < 0 ? 0 : i0 > last ? last : i0;
                i1 = i1 < 0 ? 0 : i1 > last ? last : i1;
                float hi = r->heights[i0], lo = r->heights[i0];
                for (int s = i0 + 1; s <= i1; ++s) hi = bmax(hi, r->heights[s]), lo = bmin(lo, r->heights[s]);
                y = hi + r->lift;
                bool ok = lo >= r->min_ground;
                for (int q = 0; q < r->n_discs && ok; ++q) {
                    const float dx = x - r->discs[3 * q], dy = y - r->discs[3 * q + 1];
                    const float rr = r->discs[3 * q + 2] + r->clearance;
                    ok = dx * dx + dy * dy > rr * rr;
                }
                if (ok) break;
            }
            const float ang = g.uniform((uint32_t)r->max_tries, r->angle_lo, r->angle_hi);
            const float speed = g.uniform((uint32_t)r->max_tries + 1, r->speed_lo, r->speed_hi);
            const Rot q = rot_of(ang);
            const float rows[3][3] = {{x, y, 0.0f}, {x, y, ang}, {x + r->arm * q.c, y + r->arm * q.s, ang}};
            for (int k = 0; k < 3; ++k) {
                float *o = out + 6 * k;
                o[0] = rows[k][0], o[1] = rows[k][1], o[2] = rows[k][2], o[3] = o[4] = o[5] = 0.0f;
            }
            speeds[i] = speed;
        }
    }
    return 0;
}
}  // extern "C"
