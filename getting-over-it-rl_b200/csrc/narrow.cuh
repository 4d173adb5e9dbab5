// goib2d device code: State binding, fixture access, AABBs and the narrow phase (one contact per lane).
#pragma once
#include "engine.cuh"

namespace gb {

__device__ __forceinline__ void bind_world(W &w, const Leaves &L, int64_t wi, int B, int rows, int J, int C) {
    w.B = B, w.rows = rows, w.J = J, w.C = C;
#define GBF(leaf, per) ((float *)L.p[leaf] + wi * (int64_t)(per))
#define GBI(leaf, per) ((int32_t *)L.p[leaf] + wi * (int64_t)(per))
#define GBU(leaf, per) ((uint8_t *)L.p[leaf] + wi * (int64_t)(per))
    w.type = GBI(GOIB2D_B_TYPE, B);
    w.active = GBU(GOIB2D_B_ACTIVE, B);
    w.awake = GBU(GOIB2D_B_AWAKE, B);
    w.allow_sleep = GBU(GOIB2D_B_ALLOW_SLEEP, B);
    w.bullet = GBU(GOIB2D_B_BULLET, B);
    w.continuous = GBU(GOIB2D_B_CONTINUOUS, B);
    w.sleep_time = GBF(GOIB2D_B_SLEEP_TIME, B);
    w.xf_p = GBF(GOIB2D_B_XF_P, 2 * B);
    w.xf_q = GBF(GOIB2D_B_XF_Q, 2 * B);
    w.local_center = GBF(GOIB2D_B_LOCAL_CENTER, 2 * B);
    w.c0 = GBF(GOIB2D_B_C0, 2 * B);
    w.c = GBF(GOIB2D_B_C, 2 * B);
    w.a0 = GBF(GOIB2D_B_A0, B);
    w.a = GBF(GOIB2D_B_A, B);
    w.v = GBF(GOIB2D_B_V, 2 * B);
    w.w = GBF(GOIB2D_B_W, B);
    w.force = GBF(GOIB2D_B_FORCE, 2 * B);
    w.torque = GBF(GOIB2D_B_TORQUE, B);
    w.mass = GBF(GOIB2D_B_MASS, B);
    w.inv_mass = GBF(GOIB2D_B_INV_MASS, B);
    w.inertia = GBF(GOIB2D_B_INERTIA, B);
    w.inv_inertia = GBF(GOIB2D_B_INV_INERTIA, B);
    w.linear_damping = GBF(GOIB2D_B_LINEAR_DAMPING, B);
    w.angular_damping = GBF(GOIB2D_B_ANGULAR_DAMPING, B);
    w.gravity_scale = GBF(GOIB2D_B_GRAVITY_SCALE, B);
    w.fx_friction = GBF(GOIB2D_F_FRICTION, rows);
    w.fx_restitution = GBF(GOIB2D_F_RESTITUTION, rows);
    w.fx_fat = GBF(GOIB2D_F_FAT, 4 * rows);
    w.enable_motor = GBU(GOIB2D_J_ENABLE_MOTOR, J);
    w.motor_speed = GBF(GOIB2D_J_MOTOR_SPEED, J);
    w.max_motor = GBF(GOIB2D_J_MAX_MOTOR, J);
    w.enable_limit = GBU(GOIB2D_J_ENABLE_LIMIT, J);
    w.lower = GBF(GOIB2D_J_LOWER, J);
    w.upper = GBF(GOIB2D_J_UPPER, J);
    w.frequency = GBF(GOIB2D_J_FREQUENCY, J);
    w.damping = GBF(GOIB2D_J_DAMPING, J);
    w.impulse = GBF(GOIB2D_J_IMPULSE, 3 * J);
    w.motor_impulse = GBF(GOIB2D_J_MOTOR_IMPULSE, J);
    w.limit_state = GBI(GOIB2D_J_LIMIT_STATE, J);
    w.lower_impulse = GBF(GOIB2D_J_LOWER_IMPULSE, J);
    w.upper_impulse = GBF(GOIB2D_J_UPPER_IMPULSE, J);
    w.pair = GBI(GOIB2D_C_PAIR, C);
    w.fa = GBI(GOIB2D_C_FA, C);
    w.fb = GBI(GOIB2D_C_FB, C);
    w.key = GBI(GOIB2D_C_KEY, C);
    w.touching = GBU(GOIB2D_C_TOUCHING, C);
    w.mtype = GBI(GOIB2D_C_MTYPE, C);
    w.count = GBI(GOIB2D_C_COUNT, C);
    w.local_normal = GBF(GOIB2D_C_LOCAL_NORMAL, 2 * C);
    w.local_point = GBF(GOIB2D_C_LOCAL_POINT, 2 * C);
    w.point_local = GBF(GOIB2D_C_POINT_LOCAL, 4 * C);
    w.point_id = GBI(GOIB2D_C_POINT_ID, 2 * C);
    w.normal_impulse = GBF(GOIB2D_C_NORMAL_IMPULSE, 2 * C);
    w.tangent_impulse = GBF(GOIB2D_C_TANGENT_IMPULSE, 2 * C);
    w.friction = GBF(GOIB2D_C_FRICTION, C);
    w.restitution = GBF(GOIB2D_C_RESTITUTION, C);
    w.tangent_speed = GBF(GOIB2D_C_TANGENT_SPEED, C);
    w.gravity = GBF(GOIB2D_GRAVITY, 2);
    w.inv_dt0 = GBF(GOIB2D_INV_DT0, 1);
    w.next_key = GBI(GOIB2D_NEXT_KEY, 1);
    w.new_fixture = GBU(GOIB2D_NEW_FIXTURE, 1);
    w.overflow = GBI(GOIB2D_OVERFLOW, 1);
    w.t_alpha0 = GBF(GOIB2D_T_ALPHA0, B);
    w.t_count = GBI(GOIB2D_T_COUNT, C);
    w.t_toi = GBF(GOIB2D_T_TOI, C);
    w.t_flag = GBU(GOIB2D_T_FLAG, C);
    w.t_enabled = GBU(GOIB2D_T_ENABLED, C);
    w.t_solved = GBU(GOIB2D_T_SOLVED, C);
    w.t_ni = GBF(GOIB2D_T_NORMAL_IMPULSE, 2 * C);
    w.t_ti = GBF(GOIB2D_T_TANGENT_IMPULSE, 2 * C);
    w.t_events = GBI(GOIB2D_T_EVENTS, 1);
#undef GBF
#undef GBI
#undef GBU
}

// Point the binding's row of one leaf elsewhere (a copy of the row in shared memory, see stage_rows in step.cu).
__device__ __forceinline__ void set_leaf(W &w, int leaf, char *row) {
#define GBS(name, field, T) \
    case name: w.field = reinterpret_cast<T *>(row); break
    switch (leaf) {
        GBS(GOIB2D_B_TYPE, type, int32_t); GBS(GOIB2D_B_ACTIVE, active, uint8_t); GBS(GOIB2D_B_AWAKE, awake, uint8_t);
        GBS(GOIB2D_B_ALLOW_SLEEP, allow_sleep, uint8_t); GBS(GOIB2D_B_BULLET, bullet, uint8_t);
        GBS(GOIB2D_B_CONTINUOUS, continuous, uint8_t); GBS(GOIB2D_B_SLEEP_TIME, sleep_time, float);
        GBS(GOIB2D_B_XF_P, xf_p, float); GBS(GOIB2D_B_XF_Q, xf_q, float); GBS(GOIB2D_B_LOCAL_CENTER, local_center, float);
        GBS(GOIB2D_B_C0, c0, float); GBS(GOIB2D_B_C, c, float); GBS(GOIB2D_B_A0, a0, float); GBS(GOIB2D_B_A, a, float);
        GBS(GOIB2D_B_V, v, float); GBS(GOIB2D_B_W, w, float); GBS(GOIB2D_B_FORCE, force, float);
        GBS(GOIB2D_B_TORQUE, torque, float); GBS(GOIB2D_B_MASS, mass, float); GBS(GOIB2D_B_INV_MASS, inv_mass, float);
        GBS(GOIB2D_B_INERTIA, inertia, float); GBS(GOIB2D_B_INV_INERTIA, inv_inertia, float);
        GBS(GOIB2D_B_LINEAR_DAMPING, linear_damping, float); GBS(GOIB2D_B_ANGULAR_DAMPING, angular_damping, float);
        GBS(GOIB2D_B_GRAVITY_SCALE, gravity_scale, float);
        GBS(GOIB2D_F_FRICTION, fx_friction, float); GBS(GOIB2D_F_RESTITUTION, fx_restitution, float);
        GBS(GOIB2D_F_FAT, fx_fat, float);
        GBS(GOIB2D_J_ENABLE_MOTOR, enable_motor, uint8_t); GBS(GOIB2D_J_MOTOR_SPEED, motor_speed, float);
        GBS(GOIB2D_J_MAX_MOTOR, max_motor, float); GBS(GOIB2D_J_ENABLE_LIMIT, enable_limit, uint8_t);
        GBS(GOIB2D_J_LOWER, lower, float); GBS(GOIB2D_J_UPPER, upper, float); GBS(GOIB2D_J_FREQUENCY, frequency, float);
        GBS(GOIB2D_J_DAMPING, damping, float); GBS(GOIB2D_J_IMPULSE, impulse, float);
        GBS(GOIB2D_J_MOTOR_IMPULSE, motor_impulse, float); GBS(GOIB2D_J_LIMIT_STATE, limit_state, int32_t);
        GBS(GOIB2D_J_LOWER_IMPULSE, lower_impulse, float); GBS(GOIB2D_J_UPPER_IMPULSE, upper_impulse, float);
        GBS(GOIB2D_C_PAIR, pair, int32_t); GBS(GOIB2D_C_FA, fa, int32_t); GBS(GOIB2D_C_FB, fb, int32_t);
        GBS(GOIB2D_C_KEY, key, int32_t); GBS(GOIB2D_C_TOUCHING, touching, uint8_t); GBS(GOIB2D_C_MTYPE, mtype, int32_t);
        GBS(GOIB2D_C_COUNT, count, int32_t); GBS(GOIB2D_C_LOCAL_NORMAL, local_normal, float);
        GBS(GOIB2D_C_LOCAL_POINT, local_point, float); GBS(GOIB2D_C_POINT_LOCAL, point_local, float);
        GBS(GOIB2D_C_POINT_ID, point_id, int32_t); GBS(GOIB2D_C_NORMAL_IMPULSE, normal_impulse, float);
        GBS(GOIB2D_C_TANGENT_IMPULSE, tangent_impulse, float); GBS(GOIB2D_C_FRICTION, friction, float);
        GBS(GOIB2D_C_RESTITUTION, restitution, float); GBS(GOIB2D_C_TANGENT_SPEED, tangent_speed, float);
        GBS(GOIB2D_GRAVITY, gravity, float); GBS(GOIB2D_INV_DT0, inv_dt0, float); GBS(GOIB2D_NEXT_KEY, next_key, int32_t);
        GBS(GOIB2D_NEW_FIXTURE, new_fixture, uint8_t); GBS(GOIB2D_OVERFLOW, overflow, int32_t);
        GBS(GOIB2D_T_ALPHA0, t_alpha0, float); GBS(GOIB2D_T_COUNT, t_count, int32_t); GBS(GOIB2D_T_TOI, t_toi, float);
        GBS(GOIB2D_T_FLAG, t_flag, uint8_t); GBS(GOIB2D_T_ENABLED, t_enabled, uint8_t);
        GBS(GOIB2D_T_SOLVED, t_solved, uint8_t); GBS(GOIB2D_T_NORMAL_IMPULSE, t_ni, float);
        GBS(GOIB2D_T_TANGENT_IMPULSE, t_ti, float); GBS(GOIB2D_T_EVENTS, t_events, int32_t);
        default: break;
    }
#undef GBS
}

// ---- fixtures in either layout (world.py:413-434)
__device__ __forceinline__ AABB fixture_fat(const DevModel &m, const W &w, int f) {
    int r = m.fixture_slot[f];
    const float *p = r >= 0 ? w.fx_fat + 4 * r : m.static_fat + 4 * f;
    return {p[0], p[1], p[2], p[3]};
}
__device__ __forceinline__ float fixture_friction(const DevModel &m, const W &w, int f) {
    int r = m.fixture_slot[f];
    return r >= 0 ? w.fx_friction[r] : m.static_friction[f];
}
__device__ __forceinline__ float fixture_restitution(const DevModel &m, const W &w, int f) {
    int r = m.fixture_slot[f];
    return r >= 0 ? w.fx_restitution[r] : m.static_restitution[f];
}

// b2Shape::ComputeAABB (shapes.py:118-133)
__device__ AABB fixture_aabb(const DevModel &m, int f, Xf xf) {
    const float *vv = m.verts + 16 * f;
    float r = m.radius[f];
    if (m.shape_type[f] == CIRCLE) {
        V2 p = rot(xf.q, V2{vv[0], vv[1]});
        float cx = xf.p.x + p.x, cy = xf.p.y + p.y;
        return {cx - r, cy - r, cx + r, cy + r};
    }
    int n = m.count[f];
    float lx = __int_as_float(0x7f800000), ly = lx, ux = -lx, uy = -lx;
    for (int i = 0; i < n; ++i) {
        V2 p = xf_mul(xf, V2{vv[2 * i], vv[2 * i + 1]});
        lx = fminf(lx, p.x), ly = fminf(ly, p.y), ux = fmaxf(ux, p.x), uy = fmaxf(uy, p.y);
    }
    return {lx - r, ly - r, ux + r, uy + r};
}

// ---------------------------------------------------------------- narrow phase (collide.py)
enum { E_VERTEX = 0, E_FACE = 1 };
__device__ __forceinline__ int feature_key(int ia, int ib, int ta, int tb) {
    return ia | (ib << 8) | (ta << 16) | (tb << 24);
}
struct Poly {
    const float *v, *n;
    int count;
    float radius;
    __device__ V2 vert(int i) const { return {v[2 * i], v[2 * i + 1]}; }
    __device__ V2 norm(int i) const { return {n[2 * i], n[2 * i + 1]}; }
};
__device__ __forceinline__ Poly poly_of(const DevModel &m, int f) {
    return {m.verts + 16 * f, m.normals + 16 * f, m.count[f], m.radius[f]};
}

// b2FindMaxSeparation (collide.py:32-42)
__device__ float find_max_separation(const Poly &p1, Xf xf1, const Poly &p2, Xf xf2, int *edge) {
    Rot q{xf2.q.c * xf1.q.c + xf2.q.s * xf1.q.s, xf2.q.c * xf1.q.s - xf2.q.s * xf1.q.c};
    V2 p = rot_t(xf2.q, sub(xf1.p, xf2.p));
    Xf xf{p, q};
    // p2's vertices load once, as the four 16-byte words of its 64-byte-aligned slot, for every edge of p1
    const float4 *q2 = reinterpret_cast<const float4 *>(p2.v);
    float4 w[MAXV / 2];
#pragma unroll
    for (int k = 0; k < MAXV / 2; ++k) w[k] = __ldg(q2 + k);
    int best = 0;
    float maxsep = -MAXF;
    for (int i = 0; i < p1.count; ++i) {
        V2 n = rot(q, p1.norm(i));
        V2 v1 = xf_mul(xf, p1.vert(i));
        float si = MAXF;
#pragma unroll
        for (int j = 0; j < MAXV; ++j) {
            V2 pj = (j & 1) ? V2{w[j >> 1].z, w[j >> 1].w} : V2{w[j >> 1].x, w[j >> 1].y};
            float dj = dot(n, sub(pj, v1));
            if (j < p2.count) si = fminf(si, dj);
        }
        if (i == 0 || si > maxsep) maxsep = si, best = i;
    }
    *edge = best;
    return maxsep;
}

struct ClipV {
    V2 v;
    int ia, ib, ta, tb;
};
// b2ClipSegmentToLine for two inputs (collide.py:45-62)
__device__ __forceinline__ int clip2(const ClipV in[2], V2 n, float offset, int vertex_index_a, ClipV out[2]) {
    float d0 = dot(n, in[0].v) - offset, d1 = dot(n, in[1].v) - offset;
    bool in0 = d0 <= 0, in1 = d1 <= 0, crs = d0 * d1 < 0;
    float interp = d0 / (d0 - d1);
    V2 ip{in[0].v.x + interp * (in[1].v.x - in[0].v.x), in[0].v.y + interp * (in[1].v.y - in[0].v.y)};
    ClipV iv{ip, vertex_index_a, in[0].ib, E_VERTEX, E_FACE};
    out[0] = in0 ? in[0] : in[1];
    out[1] = (in0 && in1) ? in[1] : iv;
    return (int)in0 + (int)in1 + (int)crs;
}

__device__ void collide_polygons(const Poly &pa, Xf xfa, const Poly &pb, Xf xfb, float linear_slop, Man &out) {
    // b2CollidePolygons (collide.py:65-127)
    float total_radius = pa.radius + pb.radius;
    int edge_a, edge_b;
    float sep_a = find_max_separation(pa, xfa, pb, xfb, &edge_a);
    float sep_b = find_max_separation(pb, xfb, pa, xfa, &edge_b);
    float k_tol = K_TOL * linear_slop;
    bool flip = sep_b > sep_a + k_tol;
    const Poly &p1 = flip ? pb : pa, &p2 = flip ? pa : pb;
    Xf xf1 = flip ? xfb : xfa, xf2 = flip ? xfa : xfb;
    int edge1 = flip ? edge_b : edge_a;
    V2 rn = rot_t(xf2.q, rot(xf1.q, p1.norm(edge1)));
    int i1 = 0;
    float mind = MAXF;
    for (int i = 0; i < p2.count; ++i) {
        float d = dot(rn, p2.norm(i));
        if (i == 0 || d < mind) mind = d, i1 = i;
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
    int np1 = clip2(inc, neg(tg), side1, iv1, c1);
    int np2 = clip2(c1, tg, side2, iv2, c2);
    bool ok = np1 >= 2 && np2 >= 2;
    V2 pts[2];
    int ids[2];
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
    out.mtype = flip ? FACE_B : FACE_A;
    out.count = count;
    out.ln = local_normal;
    out.lp = plane_point;
    out.pt[0] = keep[0] ? pts[0] : pts[1];
    out.id[0] = keep[0] ? ids[0] : ids[1];
    out.pt[1] = pts[1];
    out.id[1] = ids[1];
}

__device__ void collide_polygon_circle(const Poly &pa, Xf xfa, const Poly &pb, Xf xfb, Man &out) {
    // b2CollidePolygonAndCircle (collide.py:130-170)
    V2 cl = xf_mul_t(xfa, xf_mul(xfb, pb.vert(0)));
    float radius = pa.radius + pb.radius;
    bool early = false;
    int ni = 0;
    float separation = -MAXF;
    for (int i = 0; i < pa.count; ++i) {
        float s = dot(pa.norm(i), sub(cl, pa.vert(i)));
        if (s > radius) early = true;
        if (i == 0 || s > separation) separation = s, ni = i;
    }
    int i2 = ni + 1 < pa.count ? ni + 1 : 0;
    V2 v1 = pa.vert(ni), v2 = pa.vert(i2), nf = pa.norm(ni);
    float rr = radius * radius;
    V2 face_c{0.5f * (v1.x + v2.x), 0.5f * (v1.y + v2.y)};
    bool inside = separation < EPS;
    float u1 = dot(sub(cl, v1), sub(v2, v1));
    float u2 = dot(sub(cl, v2), sub(v1, v2));
    V2 d1 = sub(cl, v1), d2 = sub(cl, v2);
    bool far1 = dot(d1, d1) > rr, far2 = dot(d2, d2) > rr;
    V2 n1 = normalize(d1), n2 = normalize(d2);
    float sep_face = dot(sub(cl, face_c), nf);
    bool c1 = u1 <= 0, c2 = !(u1 <= 0) && u2 <= 0, c3 = !(u1 <= 0) && !(u2 <= 0);
    bool none = early || (!inside && ((c1 && far1) || (c2 && far2) || (c3 && sep_face > radius)));
    out.mtype = FACE_A;
    out.count = none ? 0 : 1;
    out.ln = inside ? nf : c1 ? n1 : c2 ? n2 : nf;
    out.lp = inside ? face_c : c1 ? v1 : c2 ? v2 : face_c;
    out.pt[0] = out.pt[1] = pb.vert(0);
    out.id[0] = out.id[1] = 0;
}

__device__ void collide_circles(const Poly &pa, Xf xfa, const Poly &pb, Xf xfb, Man &out) {
    // b2CollideCircles (collide.py:173-186)
    V2 p1 = xf_mul(xfa, pa.vert(0)), p2 = xf_mul(xfb, pb.vert(0));
    V2 d = sub(p2, p1);
    float r = pa.radius + pb.radius;
    out.mtype = CIRCLES;
    out.count = !(dot(d, d) > r * r) ? 1 : 0;
    out.ln = {0.0f, 0.0f};
    out.lp = pa.vert(0);
    out.pt[0] = out.pt[1] = pb.vert(0);
    out.id[0] = out.id[1] = 0;
}

// ---------------------------------------------------------------- edges (no counterpart in the reference engine)
// Box2D 2.3.1's method for edge shapes, in this engine's own code: a segment v1-v2 of an edge fixture, with the
// optional ghost vertices v0 (before v1) and v3 (after v2) of a chain. The ghost vertices decide which side of a
// shared chain vertex owns a contact, so that a shape sliding along a chain is not caught by its inner vertices.
struct Edge {
    V2 v0, v1, v2, v3;
    bool has0, has3;
    float radius;
};
__device__ __forceinline__ Edge edge_of(const DevModel &m, int f) {
    const float *v = m.verts + 16 * f;
    int g = m.edge_ghost[f];
    return {{v[4], v[5]}, {v[0], v[1]}, {v[2], v[3]}, {v[6], v[7]}, (g & 1) != 0, (g & 2) != 0, m.radius[f]};
}

__device__ __forceinline__ void man_empty(Man &out, int mtype) {
    out.mtype = mtype, out.count = 0;
    out.ln = out.lp = out.pt[0] = out.pt[1] = V2{0.0f, 0.0f};
    out.id[0] = out.id[1] = 0;
}

// b2CollideEdgeAndCircle: the circle centre's Voronoi region of the segment (vertex v1, vertex v2 or the face); a
// vertex region owned by the neighbouring edge (the centre lies beyond the shared vertex along that edge) gives no
// contact here.
__device__ void collide_edge_circle(const Edge &e, Xf xfa, const Poly &cb, Xf xfb, Man &out) {
    V2 q = xf_mul_t(xfa, xf_mul(xfb, cb.vert(0)));  // the centre in the edge's frame
    V2 a = e.v1, b = e.v2, ab = sub(b, a);
    float u = dot(ab, sub(b, q)), v = dot(ab, sub(q, a));
    float radius = e.radius + cb.radius;
    man_empty(out, CIRCLES);
    out.pt[0] = out.pt[1] = cb.vert(0);
    if (v <= 0.0f) {  // vertex v1
        V2 d = sub(q, a);
        if (dot(d, d) > radius * radius) return;
        if (e.has0 && dot(sub(a, e.v0), sub(a, q)) > 0.0f) return;
        out.count = 1, out.lp = a, out.id[0] = feature_key(0, 0, E_VERTEX, E_VERTEX);
        return;
    }
    if (u <= 0.0f) {  // vertex v2
        V2 d = sub(q, b);
        if (dot(d, d) > radius * radius) return;
        if (e.has3 && dot(sub(e.v3, b), sub(q, b)) > 0.0f) return;
        out.count = 1, out.lp = b, out.id[0] = feature_key(1, 0, E_VERTEX, E_VERTEX);
        return;
    }
    float inv = 1.0f / dot(ab, ab);
    V2 p{inv * (u * a.x + v * b.x), inv * (u * a.y + v * b.y)};  // the closest point of the face
    V2 d = sub(q, p);
    if (dot(d, d) > radius * radius) return;
    V2 n{-ab.y, ab.x};
    if (dot(n, sub(q, a)) < 0.0f) n = neg(n);
    out.mtype = FACE_A, out.count = 1, out.ln = normalize(n), out.lp = a;
    out.id[0] = feature_key(0, 0, E_FACE, E_VERTEX);
}

// The polygon's area centroid (b2PolygonShape::m_centroid), fan of triangles from the origin.
__device__ __forceinline__ V2 poly_centroid(const Poly &p) {
    float area = 0.0f, cx = 0.0f, cy = 0.0f;
    const float third = 1.0f / 3.0f;
    for (int i = 0; i < p.count; ++i) {
        V2 p2 = p.vert(i), p3 = p.vert(i + 1 < p.count ? i + 1 : 0);
        float tri = 0.5f * cross(p2, p3);
        area = area + tri;
        cx = cx + tri * third * (p2.x + p3.x);
        cy = cy + tri * third * (p2.y + p3.y);
    }
    float inv = 1.0f / area;
    return {cx * inv, cy * inv};
}

// Which side of the edge the polygon is on (front) and the range of contact normals the edge admits there: a
// normal must lie between `lower` and `upper`. With a ghost vertex, the range reaches the neighbouring edge's
// normal across a convex vertex and stops at this edge's across a concave one; without, the free end turns the
// range all the way round to the opposite side.
struct EdgeRange {
    bool front;
    V2 normal, lower, upper;
};
__device__ EdgeRange edge_range(const Edge &e, V2 c) {
    V2 e1 = normalize(sub(e.v2, e.v1));
    V2 n1{e1.y, -e1.x};
    float o1 = dot(n1, sub(c, e.v1));
    V2 n0{0.0f, 0.0f}, n2{0.0f, 0.0f};
    float o0 = 0.0f, o2 = 0.0f;
    bool cv1 = false, cv2 = false;
    if (e.has0) {
        V2 e0 = normalize(sub(e.v1, e.v0));
        n0 = {e0.y, -e0.x}, cv1 = cross(e0, e1) >= 0.0f, o0 = dot(n0, sub(c, e.v0));
    }
    if (e.has3) {
        V2 e2 = normalize(sub(e.v3, e.v2));
        n2 = {e2.y, -e2.x}, cv2 = cross(e1, e2) > 0.0f, o2 = dot(n2, sub(c, e.v2));
    }
    const V2 m1 = neg(n1);
    EdgeRange r;
    if (e.has0 && e.has3) {
        if (cv1 && cv2) {
            r.front = o0 >= 0.0f || o1 >= 0.0f || o2 >= 0.0f;
            r.lower = r.front ? n0 : m1, r.upper = r.front ? n2 : m1;
        } else if (cv1) {
            r.front = o0 >= 0.0f || (o1 >= 0.0f && o2 >= 0.0f);
            r.lower = r.front ? n0 : neg(n2), r.upper = r.front ? n1 : m1;
        } else if (cv2) {
            r.front = o2 >= 0.0f || (o0 >= 0.0f && o1 >= 0.0f);
            r.lower = r.front ? n1 : m1, r.upper = r.front ? n2 : neg(n0);
        } else {
            r.front = o0 >= 0.0f && o1 >= 0.0f && o2 >= 0.0f;
            r.lower = r.front ? n1 : neg(n2), r.upper = r.front ? n1 : neg(n0);
        }
    } else if (e.has0) {
        if (cv1) {
            r.front = o0 >= 0.0f || o1 >= 0.0f;
            r.lower = r.front ? n0 : n1, r.upper = m1;
        } else {
            r.front = o0 >= 0.0f && o1 >= 0.0f;
            r.lower = n1, r.upper = r.front ? m1 : neg(n0);
        }
    } else if (e.has3) {
        if (cv2) {
            r.front = o1 >= 0.0f || o2 >= 0.0f;
            r.lower = m1, r.upper = r.front ? n2 : n1;
        } else {
            r.front = o1 >= 0.0f && o2 >= 0.0f;
            r.lower = r.front ? m1 : neg(n2), r.upper = n1;
        }
    } else {
        r.front = o1 >= 0.0f;
        r.lower = r.front ? m1 : n1, r.upper = r.front ? m1 : n1;
    }
    r.normal = r.front ? n1 : m1;
    return r;
}

// b2CollideEdgeAndPolygon: the polygon in the edge's frame; the edge's own axis against the polygon's face axes
// restricted to the admissible normal range (angular_slop of slack), the polygon axis preferred only when clearly
// deeper (0.98 x the edge separation + 0.001); the incident feature clipped to the reference face's side planes.
__device__ void collide_edge_polygon(const Edge &e, Xf xfa, const Poly &pb, Xf xfb, float angular_slop, Man &out) {
    const Rot q{xfa.q.c * xfb.q.c + xfa.q.s * xfb.q.s, xfa.q.c * xfb.q.s - xfa.q.s * xfb.q.c};
    const Xf xf{rot_t(xfa.q, sub(xfb.p, xfa.p)), q};  // polygon frame -> edge frame
    const int n = pb.count;
    auto PV = [&](int i) { return xf_mul(xf, pb.vert(i)); };
    auto PN = [&](int i) { return rot(xf.q, pb.norm(i)); };
    man_empty(out, FACE_A);
    const EdgeRange rg = edge_range(e, xf_mul(xf, poly_centroid(pb)));
    const float radius = e.radius + pb.radius;
    float sep_e = MAXF;  // the edge's axis
    for (int i = 0; i < n; ++i) sep_e = bmin(sep_e, dot(rg.normal, sub(PV(i), e.v1)));
    if (sep_e > radius) return;
    int pidx = -1;  // the polygon's axes
    float psep = -MAXF;
    const V2 perp{-rg.normal.y, rg.normal.x};
    for (int i = 0; i < n; ++i) {
        V2 nn = neg(PN(i)), v = PV(i);
        float s = bmin(dot(nn, sub(v, e.v1)), dot(nn, sub(v, e.v2)));
        if (s > radius) {  // a separating axis
            pidx = i, psep = s;
            break;
        }
        V2 lim = dot(nn, perp) >= 0.0f ? rg.upper : rg.lower;
        if (dot(sub(nn, lim), rg.normal) < -angular_slop) continue;
        if (s > psep) pidx = i, psep = s;
    }
    if (pidx >= 0 && psep > radius) return;
    const bool on_b = pidx >= 0 && psep > 0.98f * sep_e + 0.001f;
    ClipV ie[2];
    int r1, r2;
    V2 rv1, rv2, rn;
    if (!on_b) {  // the edge is the reference face; the polygon edge most anti-parallel to it is incident
        int best = 0;
        float bv = dot(rg.normal, PN(0));
        for (int i = 1; i < n; ++i) {
            float val = dot(rg.normal, PN(i));
            if (val < bv) bv = val, best = i;
        }
        int i2 = best + 1 < n ? best + 1 : 0;
        ie[0] = {PV(best), 0, best, E_FACE, E_VERTEX};
        ie[1] = {PV(i2), 0, i2, E_FACE, E_VERTEX};
        r1 = rg.front ? 0 : 1, r2 = rg.front ? 1 : 0;
        rv1 = rg.front ? e.v1 : e.v2, rv2 = rg.front ? e.v2 : e.v1;
        rn = rg.normal;  // n1 in front, -n1 behind
    } else {  // a polygon face is the reference; the segment is incident
        ie[0] = {e.v1, 0, pidx, E_VERTEX, E_FACE};
        ie[1] = {e.v2, 0, pidx, E_VERTEX, E_FACE};
        r1 = pidx, r2 = pidx + 1 < n ? pidx + 1 : 0;
        rv1 = PV(r1), rv2 = PV(r2), rn = PN(r1);
    }
    const V2 sn1{rn.y, -rn.x}, sn2 = neg(sn1);
    ClipV c1[2], c2[2];
    if (clip2(ie, sn1, dot(sn1, rv1), r1, c1) < 2) return;
    if (clip2(c1, sn2, dot(sn2, rv2), r2, c2) < 2) return;
    out.mtype = on_b ? FACE_B : FACE_A;
    out.ln = on_b ? pb.norm(r1) : rn;
    out.lp = on_b ? pb.vert(r1) : rv1;
    int count = 0;
    for (int k = 0; k < 2; ++k) {
        const ClipV &c = c2[k];
        if (dot(rn, sub(c.v, rv1)) > radius) continue;
        out.pt[count] = on_b ? c.v : xf_mul_t(xf, c.v);
        out.id[count] = on_b ? feature_key(c.ib, c.ia, c.tb, c.ta) : feature_key(c.ia, c.ib, c.ta, c.tb);
        ++count;
    }
    out.count = count;
}

// b2Contact::Evaluate dispatch (collide.py:189-207; edge pairs put the edge first, as b2Contact::Create does)
__device__ __noinline__ void evaluate(const DevModel &m, int fa, int fb, Xf xfa, Xf xfb, float slop, float angular_slop,
                                      Man &out) {
    Poly pa = poly_of(m, fa), pb = poly_of(m, fb);
    int ta = m.shape_type[fa], tb = m.shape_type[fb];
    if (ta == POLYGON && tb == POLYGON)
        collide_polygons(pa, xfa, pb, xfb, slop, out);
    else if (ta == POLYGON && tb == CIRCLE)
        collide_polygon_circle(pa, xfa, pb, xfb, out);
    else if (ta == EDGE && tb == CIRCLE)
        collide_edge_circle(edge_of(m, fa), xfa, pb, xfb, out);
    else if (ta == EDGE && tb == POLYGON)
        collide_edge_polygon(edge_of(m, fa), xfa, pb, xfb, angular_slop, out);
    else
        collide_circles(pa, xfa, pb, xfb, out);
}

// b2Contact::Update's manifold write: impulses carried over by feature key, touching flag (pairs.py:55-83)
__device__ __forceinline__ bool apply_manifold(W &w, int s, const Man &mn_) {
    const Man mn = mn_;  // every load first (the manifold, then the slot's old state), the stores last
    const int old_n = w.count[s], pid0 = w.point_id[2 * s], pid1 = w.point_id[2 * s + 1];
    const float on0 = w.normal_impulse[2 * s], on1 = w.normal_impulse[2 * s + 1];
    const float ot0 = w.tangent_impulse[2 * s], ot1 = w.tangent_impulse[2 * s + 1];
    const bool was_touching = w.touching[s];
    float ni[2], ti[2];
    for (int i = 0; i < 2; ++i) {
        int nid = mn.id[i];
        bool m0 = old_n > 0 && pid0 == nid;
        bool m1 = old_n > 1 && pid1 == nid && !m0;
        ni[i] = m0 ? on0 : m1 ? on1 : 0.0f;
        ti[i] = m0 ? ot0 : m1 ? ot1 : 0.0f;
        if (!(i < mn.count)) ni[i] = ti[i] = 0.0f;
    }
    bool touching = mn.count > 0;
    bool flip = touching != was_touching;
    w.touching[s] = touching;
    w.count[s] = mn.count;
    if (mn.count > 0) {
        w.mtype[s] = mn.mtype;
        w.local_normal[2 * s] = mn.ln.x, w.local_normal[2 * s + 1] = mn.ln.y;
        w.local_point[2 * s] = mn.lp.x, w.local_point[2 * s + 1] = mn.lp.y;
        for (int k = 0; k < 2; ++k) {
            w.point_local[4 * s + 2 * k] = mn.pt[k].x, w.point_local[4 * s + 2 * k + 1] = mn.pt[k].y;
            w.point_id[2 * s + k] = mn.id[k];
        }
    }
    for (int k = 0; k < 2; ++k) w.normal_impulse[2 * s + k] = ni[k], w.tangent_impulse[2 * s + k] = ti[k];
    return flip;
}

}  // namespace gb
