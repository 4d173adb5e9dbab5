// Parity oracle (test infrastructure, see oracle.h): math, layout, shapes and the narrow phase.
#include <cstdlib>

#include "oracle.h"

namespace orc {

// ---------------------------------------------------------------- sin / cos (math2d.py:218-316)
// float-float arithmetic: Dekker/Knuth exact products and sums on float32 pairs (hi, lo).
namespace {
struct FF {
    float h, l;
};
inline float bits_hi(float a) {
    uint32_t u;
    std::memcpy(&u, &a, 4);
    u &= 0xFFFFF000u;
    float r;
    std::memcpy(&r, &u, 4);
    return r;
}
inline FF two_prod(float a, float b) {  // math2d.py:230-234
    float p = a * b;
    float ah = bits_hi(a), al = a - ah, bh = bits_hi(b), bl = b - bh;
    return {p, (((ah * bh - p) + ah * bl) + al * bh) + al * bl};
}
inline FF two_sum(float a, float b) {  // math2d.py:237-240
    float s = a + b;
    float bb = s - a;
    return {s, (a - (s - bb)) + (b - bb)};
}
inline FF fast_two_sum(float a, float b) {  // math2d.py:243-245
    float s = a + b;
    return {s, b - (s - a)};
}
inline FF ff_add(FF a, FF b) {  // math2d.py:248-252
    FF s = two_sum(a.h, b.h), t = two_sum(a.l, b.l);
    FF u = fast_two_sum(s.h, s.l + t.h);
    return fast_two_sum(u.h, u.l + t.l);
}
inline FF ff_mul(FF a, FF b) {  // math2d.py:255-257
    FF p = two_prod(a.h, b.h);
    return fast_two_sum(p.h, p.l + (a.h * b.l + a.l * b.h));
}
// Taylor coefficients (-1)^k/(2k+1)! and (-1)^k/(2k)!, k = 0..9, each as the float pair (f32(c), f32(c - f32(c)))
// of the double value (math2d.py:260-278)
const float SIN_C[10][2] = {{0x1p+0f, 0x0p+0f}, {-0x1.555556p-3f, 0x1.555556p-28f}, {0x1.111112p-7f, -0x1.dddddep-32f},
                            {-0x1.a01a02p-13f, 0x1.7f97fap-39f}, {0x1.71de3ap-19f, 0x1.55b1ccp-45f},
                            {-0x1.ae6456p-26f, -0x1.fd5138p-52f}, {0x1.612462p-33f, -0x1.8af25ep-58f},
                            {-0x1.ae7f3ep-41f, -0x1.ccee08p-67f}, {0x1.952c78p-49f, -0x1.f9ea56p-74f},
                            {-0x1.2f49b4p-57f, -0x1.a05056p-83f}};
const float COS_C[10][2] = {{0x1p+0f, 0x0p+0f}, {-0x1p-1f, 0x0p+0f}, {0x1.555556p-5f, -0x1.555556p-30f},
                            {-0x1.6c16c2p-10f, 0x1.27d27ep-35f}, {0x1.a01a02p-16f, -0x1.7f97fap-42f},
                            {-0x1.27e4fcp-22f, 0x1.10ec14p-47f}, {0x1.1eed8ep-29f, 0x1.ff1b14p-54f},
                            {-0x1.93974ap-37f, -0x1.180f94p-62f}, {0x1.ae7f3ep-45f, 0x1.ccee08p-71f},
                            {-0x1.682786p-53f, -0x1.dcbeccp-80f}};
// pi/2 in three float32 parts, and float32(2/pi)
const float PIO2_0 = 0x1.921fb6p+0f, PIO2_1 = -0x1.777a5cp-25f, PIO2_2 = -0x1.ee59dap-50f;
const float TWO_OVER_PI = 0x1.45f306p-1f;

inline FF poly(FF x, const float (*c)[2]) {  // math2d.py:281-288, Horner from the highest term
    FF s = {c[9][0], c[9][1]};
    for (int k = 8; k >= 0; --k) s = ff_add(ff_mul(s, x), FF{c[k][0], c[k][1]});
    return s;
}
}  // namespace

float sin_of(float x, float *cos_out) {
    float k = std::nearbyint(x * TWO_OVER_PI);  // round half to even
    FF p1 = two_prod(k, PIO2_0);
    FF r = ff_add(FF{x, 0.0f}, FF{-p1.h, -p1.l});
    FF p2 = two_prod(k, PIO2_1);
    r = ff_add(r, FF{-p2.h, -p2.l});
    r = ff_add(r, FF{-(k * PIO2_2), 0.0f});
    FF r2 = ff_mul(r, r);
    FF sp = ff_mul(r, poly(r2, SIN_C));
    FF cp = poly(r2, COS_C);
    float s = sp.h + sp.l, c = cp.h + cp.l;
    int q = ((int)k % 4 + 4) % 4;
    float sn = q == 0 ? s : q == 1 ? c : q == 2 ? -s : -c;
    float cs = q == 0 ? c : q == 1 ? -s : q == 2 ? -c : s;
    *cos_out = cs;
    return x == 0 ? x : sn;
}

// ---------------------------------------------------------------- State leaves
namespace {
struct LeafSpec {
    int dtype;  // 0 f32, 1 i32, 2 bool
    int dim;    // 0 B, 1 rows, 2 J, 3 C, 4 scalar
    int width;  // elements per entity
};
const LeafSpec LEAVES[GOIB2D_NUM_LEAVES] = {
    // bodies
    {1, 0, 1}, {2, 0, 1}, {2, 0, 1}, {2, 0, 1}, {2, 0, 1}, {2, 0, 1}, {0, 0, 1}, {0, 0, 2}, {0, 0, 2}, {0, 0, 2},
    {0, 0, 2}, {0, 0, 2}, {0, 0, 1}, {0, 0, 1}, {0, 0, 2}, {0, 0, 1}, {0, 0, 2}, {0, 0, 1}, {0, 0, 1}, {0, 0, 1},
    {0, 0, 1}, {0, 0, 1}, {0, 0, 1}, {0, 0, 1}, {0, 0, 1},
    // fixtures
    {0, 1, 1}, {0, 1, 1}, {0, 1, 4},
    // joints
    {2, 2, 1}, {0, 2, 1}, {0, 2, 1}, {2, 2, 1}, {0, 2, 1}, {0, 2, 1}, {0, 2, 1}, {0, 2, 1}, {0, 2, 3}, {0, 2, 1},
    {1, 2, 1}, {0, 2, 1}, {0, 2, 1},
    // contacts
    {1, 3, 1}, {1, 3, 1}, {1, 3, 1}, {1, 3, 1}, {2, 3, 1}, {1, 3, 1}, {1, 3, 1}, {0, 3, 2}, {0, 3, 2}, {0, 3, 4},
    {1, 3, 2}, {0, 3, 2}, {0, 3, 2}, {0, 3, 1}, {0, 3, 1}, {0, 3, 1},
    // scalars: gravity [2], inv_dt0, next_key, new_fixture, overflow
    {0, 4, 2}, {0, 4, 1}, {1, 4, 1}, {2, 4, 1}, {1, 4, 1},
    // toi
    {0, 0, 1}, {1, 3, 1}, {0, 3, 1}, {2, 3, 1}, {2, 3, 1}, {2, 3, 1}, {0, 3, 2}, {0, 3, 2}, {1, 4, 1}};
}  // namespace

int leaf_dtype(int leaf) { return LEAVES[leaf].dtype; }

int64_t leaf_elems(int leaf, int32_t B, int32_t rows, int32_t J, int32_t C) {
    const LeafSpec &s = LEAVES[leaf];
    int64_t n = s.dim == 0 ? B : s.dim == 1 ? rows : s.dim == 2 ? J : s.dim == 3 ? C : 1;
    return n * s.width;
}

void bind_world(World &w, void *const *L, int64_t wi, int B, int rows, int J, int C) {
    w.B = B, w.rows = rows, w.J = J, w.C = C;
    auto P = [&](int leaf) -> char * {
        int64_t e = leaf_elems(leaf, B, rows, J, C);
        int64_t sz = LEAVES[leaf].dtype == 2 ? 1 : 4;
        return (char *)L[leaf] + wi * e * sz;
    };
#define F_(leaf) ((float *)P(leaf))
#define I_(leaf) ((int32_t *)P(leaf))
#define U_(leaf) ((uint8_t *)P(leaf))
    w.type = I_(GOIB2D_B_TYPE);
    w.active = U_(GOIB2D_B_ACTIVE);
    w.awake = U_(GOIB2D_B_AWAKE);
    w.allow_sleep = U_(GOIB2D_B_ALLOW_SLEEP);
    w.bullet = U_(GOIB2D_B_BULLET);
    w.continuous = U_(GOIB2D_B_CONTINUOUS);
    w.sleep_time = F_(GOIB2D_B_SLEEP_TIME);
    w.xf_p = F_(GOIB2D_B_XF_P);
    w.xf_q = F_(GOIB2D_B_XF_Q);
    w.local_center = F_(GOIB2D_B_LOCAL_CENTER);
    w.c0 = F_(GOIB2D_B_C0);
    w.c = F_(GOIB2D_B_C);
    w.a0 = F_(GOIB2D_B_A0);
    w.a = F_(GOIB2D_B_A);
    w.v = F_(GOIB2D_B_V);
    w.w = F_(GOIB2D_B_W);
    w.force = F_(GOIB2D_B_FORCE);
    w.torque = F_(GOIB2D_B_TORQUE);
    w.mass = F_(GOIB2D_B_MASS);
    w.inv_mass = F_(GOIB2D_B_INV_MASS);
    w.inertia = F_(GOIB2D_B_INERTIA);
    w.inv_inertia = F_(GOIB2D_B_INV_INERTIA);
    w.linear_damping = F_(GOIB2D_B_LINEAR_DAMPING);
    w.angular_damping = F_(GOIB2D_B_ANGULAR_DAMPING);
    w.gravity_scale = F_(GOIB2D_B_GRAVITY_SCALE);
    w.fx_friction = F_(GOIB2D_F_FRICTION);
    w.fx_restitution = F_(GOIB2D_F_RESTITUTION);
    w.fx_fat = F_(GOIB2D_F_FAT);
    w.enable_motor = U_(GOIB2D_J_ENABLE_MOTOR);
    w.motor_speed = F_(GOIB2D_J_MOTOR_SPEED);
    w.max_motor = F_(GOIB2D_J_MAX_MOTOR);
    w.enable_limit = U_(GOIB2D_J_ENABLE_LIMIT);
    w.lower = F_(GOIB2D_J_LOWER);
    w.upper = F_(GOIB2D_J_UPPER);
    w.frequency = F_(GOIB2D_J_FREQUENCY);
    w.damping = F_(GOIB2D_J_DAMPING);
    w.impulse = F_(GOIB2D_J_IMPULSE);
    w.motor_impulse = F_(GOIB2D_J_MOTOR_IMPULSE);
    w.limit_state = I_(GOIB2D_J_LIMIT_STATE);
    w.lower_impulse = F_(GOIB2D_J_LOWER_IMPULSE);
    w.upper_impulse = F_(GOIB2D_J_UPPER_IMPULSE);
    w.pair = I_(GOIB2D_C_PAIR);
    w.fa = I_(GOIB2D_C_FA);
    w.fb = I_(GOIB2D_C_FB);
    w.key = I_(GOIB2D_C_KEY);
    w.touching = U_(GOIB2D_C_TOUCHING);
    w.mtype = I_(GOIB2D_C_MTYPE);
    w.count = I_(GOIB2D_C_COUNT);
    w.local_normal = F_(GOIB2D_C_LOCAL_NORMAL);
    w.local_point = F_(GOIB2D_C_LOCAL_POINT);
    w.point_local = F_(GOIB2D_C_POINT_LOCAL);
    w.point_id = I_(GOIB2D_C_POINT_ID);
    w.normal_impulse = F_(GOIB2D_C_NORMAL_IMPULSE);
    w.tangent_impulse = F_(GOIB2D_C_TANGENT_IMPULSE);
    w.friction = F_(GOIB2D_C_FRICTION);
    w.restitution = F_(GOIB2D_C_RESTITUTION);
    w.tangent_speed = F_(GOIB2D_C_TANGENT_SPEED);
    w.gravity = F_(GOIB2D_GRAVITY);
    w.inv_dt0 = F_(GOIB2D_INV_DT0);
    w.next_key = I_(GOIB2D_NEXT_KEY);
    w.new_fixture = U_(GOIB2D_NEW_FIXTURE);
    w.overflow = I_(GOIB2D_OVERFLOW);
    w.t_alpha0 = F_(GOIB2D_T_ALPHA0);
    w.t_count = I_(GOIB2D_T_COUNT);
    w.t_toi = F_(GOIB2D_T_TOI);
    w.t_flag = U_(GOIB2D_T_FLAG);
    w.t_enabled = U_(GOIB2D_T_ENABLED);
    w.t_solved = U_(GOIB2D_T_SOLVED);
    w.t_ni = F_(GOIB2D_T_NORMAL_IMPULSE);
    w.t_ti = F_(GOIB2D_T_TANGENT_IMPULSE);
    w.t_events = I_(GOIB2D_T_EVENTS);
#undef F_
#undef I_
#undef U_
}

// ---------------------------------------------------------------- fixtures (world.py:413-434, shapes.py:118-146)
AABB fixture_fat(const Model &m, const World &w, int f) {
    int r = fixture_row(m, f);
    const float *p = r >= 0 ? w.fx_fat + 4 * r : m.d->static_fat + 4 * f;
    return {p[0], p[1], p[2], p[3]};
}
float fixture_friction(const Model &m, const World &w, int f) {
    int r = fixture_row(m, f);
    return r >= 0 ? w.fx_friction[r] : m.d->static_friction[f];
}
float fixture_restitution(const Model &m, const World &w, int f) {
    int r = fixture_row(m, f);
    return r >= 0 ? w.fx_restitution[r] : m.d->static_restitution[f];
}

// b2Shape::ComputeAABB (shapes.py:118-133)
AABB fixture_aabb(const Model &m, int f, Xf xf) {
    const float *vv = m.d->verts + 16 * f;
    float r = m.d->radius[f];
    if (m.d->shape_type[f] == CIRCLE) {
        V2 p = rot(xf.q, v2(vv[0], vv[1]));
        float cx = xf.p.x + p.x, cy = xf.p.y + p.y;
        return {cx - r, cy - r, cx + r, cy + r};
    }
    int n = m.d->count[f];
    float lx = INFINITY, ly = INFINITY, ux = -INFINITY, uy = -INFINITY;
    for (int i = 0; i < n; ++i) {
        V2 p = xf_mul(xf, v2(vv[2 * i], vv[2 * i + 1]));
        lx = std::fmin(lx, p.x), ly = std::fmin(ly, p.y), ux = std::fmax(ux, p.x), uy = std::fmax(uy, p.y);
    }
    return {lx - r, ly - r, ux + r, uy + r};
}

// ---------------------------------------------------------------- narrow phase (collide.py)
namespace {
enum { E_VERTEX = 0, E_FACE = 1 };
inline int32_t feature_key(int ia, int ib, int ta, int tb) { return ia | (ib << 8) | (ta << 16) | (tb << 24); }
struct Poly {
    const float *v, *n;
    int count;
    float radius;
    V2 vert(int i) const { return {v[2 * i], v[2 * i + 1]}; }
    V2 norm(int i) const { return {n[2 * i], n[2 * i + 1]}; }
};
inline Poly poly_of(const Model &m, int f) {
    return {m.d->verts + 16 * f, m.d->normals + 16 * f, m.d->count[f], m.d->radius[f]};
}

// b2FindMaxSeparation (collide.py:32-42)
float find_max_separation(const Poly &p1, Xf xf1, const Poly &p2, Xf xf2, int *edge) {
    // xf = b2MulT(xf2, xf1)
    Rot q{xf2.q.c * xf1.q.c + xf2.q.s * xf1.q.s, xf2.q.c * xf1.q.s - xf2.q.s * xf1.q.c};
    V2 p = rot_t(xf2.q, sub(xf1.p, xf2.p));
    Xf xf{p, q};
    int best = 0;
    float maxsep = -MAXF;
    bool first = true;
    for (int i = 0; i < p1.count; ++i) {
        V2 n = rot(q, p1.norm(i));
        V2 v1 = xf_mul(xf, p1.vert(i));
        float si = MAXF;
        for (int j = 0; j < p2.count; ++j) {
            float sij = dot(n, sub(p2.vert(j), v1));
            si = std::fmin(si, sij);
        }
        if (first || si > maxsep) {  // argmax, first occurrence
            maxsep = si, best = i, first = false;
        }
    }
    *edge = best;
    return maxsep;
}

struct ClipV {
    V2 v;
    int ia, ib, ta, tb;
};
// b2ClipSegmentToLine for two inputs (collide.py:45-62)
int clip(const ClipV in[2], V2 n, float offset, int vertex_index_a, ClipV out[2]) {
    float d0 = dot(n, in[0].v) - offset, d1 = dot(n, in[1].v) - offset;
    bool in0 = d0 <= 0, in1 = d1 <= 0, crs = d0 * d1 < 0;
    float interp = d0 / (d0 - d1);
    V2 ip{in[0].v.x + interp * (in[1].v.x - in[0].v.x), in[0].v.y + interp * (in[1].v.y - in[0].v.y)};
    ClipV iv{ip, vertex_index_a, in[0].ib, E_VERTEX, E_FACE};
    out[0] = in0 ? in[0] : in[1];
    out[1] = (in0 && in1) ? in[1] : iv;
    return (int)in0 + (int)in1 + (int)crs;
}

void collide_polygons(const Poly &pa, Xf xfa, const Poly &pb, Xf xfb, float linear_slop, Manifold *out) {
    // collide.py:65-127
    float total_radius = pa.radius + pb.radius;
    int edge_a, edge_b;
    float sep_a = find_max_separation(pa, xfa, pb, xfb, &edge_a);
    float sep_b = find_max_separation(pb, xfb, pa, xfa, &edge_b);
    float k_tol = K_TOL * linear_slop;
    bool flip = sep_b > sep_a + k_tol;
    const Poly &p1 = flip ? pb : pa, &p2 = flip ? pa : pb;
    Xf xf1 = flip ? xfb : xfa, xf2 = flip ? xfa : xfb;
    int edge1 = flip ? edge_b : edge_a;
    // b2FindIncidentEdge
    V2 rn = rot_t(xf2.q, rot(xf1.q, p1.norm(edge1)));
    int i1 = 0;
    float mind = MAXF;
    bool first = true;
    for (int i = 0; i < p2.count; ++i) {
        float d = dot(rn, p2.norm(i));
        if (first || d < mind) mind = d, i1 = i, first = false;  // argmin, first occurrence
    }
    int i2 = i1 + 1 < p2.count ? i1 + 1 : 0;
    ClipV inc[2] = {{xf_mul(xf2, p2.vert(i1)), edge1, i1, E_FACE, E_VERTEX},
                    {xf_mul(xf2, p2.vert(i2)), edge1, i2, E_FACE, E_VERTEX}};
    int iv1 = edge1, iv2 = edge1 + 1 < p1.count ? edge1 + 1 : 0;
    V2 v11 = p1.vert(iv1), v12 = p1.vert(iv2);
    V2 tangent = normalize(sub(v12, v11));
    V2 local_normal = cross_vs(tangent, 1.0f);
    V2 plane_point{0.5f * (v11.x + v12.x), 0.5f * (v11.y + v12.y)};
    V2 tg = rot(xf1.q, tangent);
    V2 nrm = cross_vs(tg, 1.0f);
    V2 w11 = xf_mul(xf1, v11), w12 = xf_mul(xf1, v12);
    float front = dot(nrm, w11);
    float side1 = -dot(tg, w11) + total_radius;
    float side2 = dot(tg, w12) + total_radius;
    ClipV c1[2], c2[2];
    int np1 = clip(inc, neg(tg), side1, iv1, c1);
    int np2 = clip(c1, tg, side2, iv2, c2);
    bool ok = np1 >= 2 && np2 >= 2;
    V2 pts[2];
    int32_t ids[2];
    bool keep[2];
    for (int k = 0; k < 2; ++k) {
        float sep = dot(nrm, c2[k].v) - front;
        keep[k] = sep <= total_radius;
        pts[k] = xf_mul_t(xf2, c2[k].v);
        const ClipV &c = c2[k];
        ids[k] = flip ? feature_key(c.ib, c.ia, c.tb, c.ta) : feature_key(c.ia, c.ib, c.ta, c.tb);
    }
    int count = ok ? (int)keep[0] + (int)keep[1] : 0;
    if (sep_a > total_radius || sep_b > total_radius) count = 0;
    out->mtype = flip ? FACE_B : FACE_A;
    out->count = count;
    out->local_normal = local_normal;
    out->local_point = plane_point;
    out->point[0] = keep[0] ? pts[0] : pts[1];
    out->id[0] = keep[0] ? ids[0] : ids[1];
    out->point[1] = pts[1];
    out->id[1] = ids[1];
}

void collide_polygon_circle(const Poly &pa, Xf xfa, const Poly &pb, Xf xfb, Manifold *out) {
    // collide.py:130-170
    V2 cw = xf_mul(xfb, pb.vert(0));
    V2 cl = xf_mul_t(xfa, cw);
    float radius = pa.radius + pb.radius;
    bool early = false;
    int ni = 0;
    float separation = -MAXF;
    bool first = true;
    for (int i = 0; i < pa.count; ++i) {
        float s = dot(pa.norm(i), sub(cl, pa.vert(i)));
        if (s > radius) early = true;
        if (first || s > separation) separation = s, ni = i, first = false;
    }
    int i2 = ni + 1 < pa.count ? ni + 1 : 0;
    V2 v1 = pa.vert(ni), vv2 = pa.vert(i2), nf = pa.norm(ni);
    float rr = radius * radius;
    V2 face_c{0.5f * (v1.x + vv2.x), 0.5f * (v1.y + vv2.y)};
    bool inside = separation < EPS;
    float u1 = dot(sub(cl, v1), sub(vv2, v1));
    float u2 = dot(sub(cl, vv2), sub(v1, vv2));
    V2 d1 = sub(cl, v1), d2 = sub(cl, vv2);
    bool far1 = dot(d1, d1) > rr, far2 = dot(d2, d2) > rr;
    V2 n1 = normalize(d1), n2 = normalize(d2);
    float sep_face = dot(sub(cl, face_c), nf);
    bool c1 = u1 <= 0, c2 = !(u1 <= 0) && u2 <= 0, c3 = !(u1 <= 0) && !(u2 <= 0);
    bool none = early || (!inside && ((c1 && far1) || (c2 && far2) || (c3 && sep_face > radius)));
    out->mtype = FACE_A;
    out->count = none ? 0 : 1;
    out->local_normal = inside ? nf : c1 ? n1 : c2 ? n2 : nf;
    out->local_point = inside ? face_c : c1 ? v1 : c2 ? vv2 : face_c;
    out->point[0] = out->point[1] = pb.vert(0);
    out->id[0] = out->id[1] = 0;
}

void collide_circles(const Poly &pa, Xf xfa, const Poly &pb, Xf xfb, Manifold *out) {
    // collide.py:173-186
    V2 p1 = xf_mul(xfa, pa.vert(0)), p2 = xf_mul(xfb, pb.vert(0));
    V2 d = sub(p2, p1);
    float r = pa.radius + pb.radius;
    bool hit = !(dot(d, d) > r * r);
    out->mtype = CIRCLES;
    out->count = hit ? 1 : 0;
    out->local_normal = {0.0f, 0.0f};
    out->local_point = pa.vert(0);
    out->point[0] = out->point[1] = pb.vert(0);
    out->id[0] = out->id[1] = 0;
}

// ---- edges (no counterpart in the reference engine). An edge fixture: count 2, the segment in verts[0..1], the
// ghost vertices of its chain in verts[2] (before) and verts[3] (after), flagged by edge_ghost bits 0 and 1.
struct EdgeShape {
    V2 g0, a, b, g3;
    bool has_g0, has_g3;
    float radius;
};
EdgeShape edge_shape(const Model &m, int f) {
    const float *v = m.d->verts + 16 * f;
    int flags = m.d->edge_ghost ? m.d->edge_ghost[f] : 0;
    return {{v[4], v[5]}, {v[0], v[1]}, {v[2], v[3]}, {v[6], v[7]}, (flags & 1) != 0, (flags & 2) != 0,
            m.d->radius[f]};
}
inline float lesser(float a, float b) { return a < b ? a : b; }
void no_points(Manifold *out, int mtype) {
    out->mtype = mtype, out->count = 0;
    out->local_normal = out->local_point = out->point[0] = out->point[1] = V2{0.0f, 0.0f};
    out->id[0] = out->id[1] = 0;
}

// edge against circle: the circle centre's region of the segment (end a, end b or the face between); an end whose
// region belongs to the neighbouring edge of the chain yields nothing here
void collide_edge_circle(const EdgeShape &e, Xf xfa, const Poly &c, Xf xfb, Manifold *out) {
    const V2 centre = xf_mul_t(xfa, xf_mul(xfb, c.vert(0)));
    const V2 seg = sub(e.b, e.a);
    const float to_b = dot(seg, sub(e.b, centre)), from_a = dot(seg, sub(centre, e.a));
    const float r = e.radius + c.radius;
    no_points(out, CIRCLES);
    out->point[0] = out->point[1] = c.vert(0);
    if (from_a <= 0.0f) {
        V2 d = sub(centre, e.a);
        if (dot(d, d) > r * r) return;
        if (e.has_g0 && dot(sub(e.a, e.g0), sub(e.a, centre)) > 0.0f) return;  // the previous edge's region
        out->count = 1, out->local_point = e.a, out->id[0] = feature_key(0, 0, E_VERTEX, E_VERTEX);
        return;
    }
    if (to_b <= 0.0f) {
        V2 d = sub(centre, e.b);
        if (dot(d, d) > r * r) return;
        if (e.has_g3 && dot(sub(e.g3, e.b), sub(centre, e.b)) > 0.0f) return;  // the next edge's region
        out->count = 1, out->local_point = e.b, out->id[0] = feature_key(1, 0, E_VERTEX, E_VERTEX);
        return;
    }
    const float inv_len2 = 1.0f / dot(seg, seg);
    const V2 foot{inv_len2 * (to_b * e.a.x + from_a * e.b.x), inv_len2 * (to_b * e.a.y + from_a * e.b.y)};
    const V2 d = sub(centre, foot);
    if (dot(d, d) > r * r) return;
    V2 n{-seg.y, seg.x};
    if (dot(n, sub(centre, e.a)) < 0.0f) n = neg(n);
    out->mtype = FACE_A, out->count = 1, out->local_normal = normalize(n), out->local_point = e.a;
    out->id[0] = feature_key(0, 0, E_FACE, E_VERTEX);
}

V2 area_centroid(const Poly &p) {  // triangles fanned from the origin
    float area = 0.0f, sx = 0.0f, sy = 0.0f;
    const float third = 1.0f / 3.0f;
    for (int i = 0; i < p.count; ++i) {
        const V2 u = p.vert(i), w = p.vert((i + 1) % p.count);
        const float t = 0.5f * cross(u, w);
        area = area + t;
        sx = sx + t * third * (u.x + w.x);
        sy = sy + t * third * (u.y + w.y);
    }
    const float inv = 1.0f / area;
    return {sx * inv, sy * inv};
}

// the side of the edge the polygon's centroid c is on, and the admissible contact normals [lo, hi] there
struct NormalRange {
    bool front;
    V2 normal, lo, hi;
};
NormalRange normal_range(const EdgeShape &e, V2 c) {
    const V2 d1 = normalize(sub(e.b, e.a));
    const V2 n1{d1.y, -d1.x}, m1 = neg(n1);
    const float off1 = dot(n1, sub(c, e.a));
    V2 n0{0.0f, 0.0f}, n2{0.0f, 0.0f};
    float off0 = 0.0f, off2 = 0.0f;
    bool convex_a = false, convex_b = false;
    if (e.has_g0) {
        const V2 d0 = normalize(sub(e.a, e.g0));
        n0 = V2{d0.y, -d0.x};
        convex_a = cross(d0, d1) >= 0.0f;
        off0 = dot(n0, sub(c, e.g0));
    }
    if (e.has_g3) {
        const V2 d2 = normalize(sub(e.g3, e.b));
        n2 = V2{d2.y, -d2.x};
        convex_b = cross(d1, d2) > 0.0f;
        off2 = dot(n2, sub(c, e.b));
    }
    const bool f0 = off0 >= 0.0f, f1 = off1 >= 0.0f, f2 = off2 >= 0.0f;
    NormalRange r{};
    if (e.has_g0 && e.has_g3) {
        if (convex_a && convex_b) {
            r.front = f0 || f1 || f2;
            r.lo = r.front ? n0 : m1;
            r.hi = r.front ? n2 : m1;
        } else if (convex_a) {
            r.front = f0 || (f1 && f2);
            r.lo = r.front ? n0 : neg(n2);
            r.hi = r.front ? n1 : m1;
        } else if (convex_b) {
            r.front = f2 || (f0 && f1);
            r.lo = r.front ? n1 : m1;
            r.hi = r.front ? n2 : neg(n0);
        } else {
            r.front = f0 && f1 && f2;
            r.lo = r.front ? n1 : neg(n2);
            r.hi = r.front ? n1 : neg(n0);
        }
    } else if (e.has_g0) {
        if (convex_a) {
            r.front = f0 || f1;
            r.lo = r.front ? n0 : n1;
            r.hi = m1;
        } else {
            r.front = f0 && f1;
            r.lo = n1;
            r.hi = r.front ? m1 : neg(n0);
        }
    } else if (e.has_g3) {
        if (convex_b) {
            r.front = f1 || f2;
            r.lo = m1;
            r.hi = r.front ? n2 : n1;
        } else {
            r.front = f1 && f2;
            r.lo = r.front ? m1 : neg(n2);
            r.hi = n1;
        }
    } else {
        r.front = f1;
        r.lo = r.front ? m1 : n1;
        r.hi = r.front ? m1 : n1;
    }
    r.normal = r.front ? n1 : m1;
    return r;
}

// edge against polygon: separating axes (the edge's normal; the polygon's face normals inside the admissible range),
// the reference face (the polygon's only if clearly deeper: 0.98 x + 0.001), the incident feature clipped to it
void collide_edge_polygon(const EdgeShape &e, Xf xfa, const Poly &p, Xf xfb, float angular_slop, Manifold *out) {
    const Rot q{xfa.q.c * xfb.q.c + xfa.q.s * xfb.q.s, xfa.q.c * xfb.q.s - xfa.q.s * xfb.q.c};
    const Xf rel{rot_t(xfa.q, sub(xfb.p, xfa.p)), q};  // the polygon's frame seen from the edge's
    const int k = p.count;
    no_points(out, FACE_A);
    const NormalRange nr = normal_range(e, xf_mul(rel, area_centroid(p)));
    const float r = e.radius + p.radius;
    float edge_sep = MAXF;
    for (int i = 0; i < k; ++i) edge_sep = lesser(edge_sep, dot(nr.normal, sub(xf_mul(rel, p.vert(i)), e.a)));
    if (edge_sep > r) return;
    int face = -1;
    float face_sep = -MAXF;
    const V2 perp{-nr.normal.y, nr.normal.x};
    for (int i = 0; i < k; ++i) {
        const V2 nn = neg(rot(rel.q, p.norm(i)));
        const V2 vi = xf_mul(rel, p.vert(i));
        const float sep = lesser(dot(nn, sub(vi, e.a)), dot(nn, sub(vi, e.b)));
        if (sep > r) {
            face = i, face_sep = sep;
            break;
        }
        const V2 limit = dot(nn, perp) >= 0.0f ? nr.hi : nr.lo;
        if (dot(sub(nn, limit), nr.normal) < -angular_slop) continue;
        if (sep > face_sep) face = i, face_sep = sep;
    }
    if (face >= 0 && face_sep > r) return;
    const bool poly_ref = face >= 0 && face_sep > 0.98f * edge_sep + 0.001f;
    ClipV inc[2];
    int ia, ib;
    V2 ref_a, ref_b, ref_n;
    if (poly_ref) {
        inc[0] = ClipV{e.a, 0, face, E_VERTEX, E_FACE};
        inc[1] = ClipV{e.b, 0, face, E_VERTEX, E_FACE};
        ia = face, ib = (face + 1) % k;
        ref_a = xf_mul(rel, p.vert(ia)), ref_b = xf_mul(rel, p.vert(ib)), ref_n = rot(rel.q, p.norm(ia));
    } else {
        int low = 0;
        float low_dot = dot(nr.normal, rot(rel.q, p.norm(0)));
        for (int i = 1; i < k; ++i) {
            const float dv = dot(nr.normal, rot(rel.q, p.norm(i)));
            if (dv < low_dot) low_dot = dv, low = i;
        }
        const int nxt = (low + 1) % k;
        inc[0] = ClipV{xf_mul(rel, p.vert(low)), 0, low, E_FACE, E_VERTEX};
        inc[1] = ClipV{xf_mul(rel, p.vert(nxt)), 0, nxt, E_FACE, E_VERTEX};
        ia = nr.front ? 0 : 1, ib = nr.front ? 1 : 0;
        ref_a = nr.front ? e.a : e.b, ref_b = nr.front ? e.b : e.a, ref_n = nr.normal;
    }
    const V2 side1{ref_n.y, -ref_n.x}, side2 = neg(side1);
    ClipV once[2], twice[2];
    if (clip(inc, side1, dot(side1, ref_a), ia, once) < 2) return;
    if (clip(once, side2, dot(side2, ref_b), ib, twice) < 2) return;
    out->mtype = poly_ref ? FACE_B : FACE_A;
    out->local_normal = poly_ref ? p.norm(ia) : ref_n;
    out->local_point = poly_ref ? p.vert(ia) : ref_a;
    int n = 0;
    for (int j = 0; j < 2; ++j) {
        const ClipV &cv = twice[j];
        if (dot(ref_n, sub(cv.v, ref_a)) > r) continue;
        out->point[n] = poly_ref ? cv.v : xf_mul_t(rel, cv.v);
        out->id[n] = poly_ref ? feature_key(cv.ib, cv.ia, cv.tb, cv.ta) : feature_key(cv.ia, cv.ib, cv.ta, cv.tb);
        ++n;
    }
    out->count = n;
}
}  // namespace

void evaluate(const Model &m, int fa, int fb, Xf xfa, Xf xfb, float linear_slop, float angular_slop, Manifold *out) {
    // collide.py:189-207, plus the edge pairs (edge first, as b2Contact::Create orders them)
    Poly pa = poly_of(m, fa), pb = poly_of(m, fb);
    int ta = m.d->shape_type[fa], tb = m.d->shape_type[fb];
    if (ta == POLYGON && tb == POLYGON)
        collide_polygons(pa, xfa, pb, xfb, linear_slop, out);
    else if (ta == POLYGON && tb == CIRCLE)
        collide_polygon_circle(pa, xfa, pb, xfb, out);
    else if (ta == EDGE && tb == CIRCLE)
        collide_edge_circle(edge_shape(m, fa), xfa, pb, xfb, out);
    else if (ta == EDGE && tb == POLYGON)
        collide_edge_polygon(edge_shape(m, fa), xfa, pb, xfb, angular_slop, out);
    else
        collide_circles(pa, xfa, pb, xfb, out);
}

}  // namespace orc
