// goib2d device code: the sequential-impulse contact solver (contact_solver.py) and the revolute, prismatic and
// weld joints (joints.py). Row set-up runs one constraint per lane; the Gauss-Seidel sweeps run in solve order.
#pragma once
#include "narrow.cuh"

namespace gb {

// Body working arrays of the island solve (velocities and positions, B entries each). qc / qs hold rot_of(qa[b]):
// a memo of each body's last rotation, keyed on the angle's bits, so a body whose angle did not change (a static
// body in the position passes) reuses it; the same angle gives the same floats, so the memo is exact.
struct Bodies {
    float *vx, *vy, *vw, *cx, *cy, *ca, *qc, *qs, *qa;
};

__device__ __forceinline__ Rot body_rot(const Bodies &bd, int b, float angle) {
    if (__float_as_uint(bd.qa[b]) == __float_as_uint(angle)) return {bd.qc[b], bd.qs[b]};
    Rot q = rot_of(angle);
    bd.qa[b] = angle, bd.qc[b] = q.c, bd.qs[b] = q.s;
    return q;
}

// b2ContactSolver constructor + InitializeVelocityConstraints for one ordered contact (contact_solver.py:32-147).
// Every load comes first (three dependent levels: the slot's fields, its fixtures, their bodies), then the
// arithmetic, then the row's stores: to the compiler a store to the row may alias the State's float arrays, so a
// load placed after one could not be hoisted above it and would wait for all the arithmetic before it.
__device__ __noinline__ void prepare_contact(const DevModel &m, const W &w, int slot, const Bodies &bd, bool warm,
                                             float dt_ratio, float velocity_threshold, VCRow &c) {
    const int fa = w.fa[slot], fb = w.fb[slot];
    const int mtype = w.mtype[slot], count = w.count[slot];
    const V2 ln{w.local_normal[2 * slot], w.local_normal[2 * slot + 1]};
    const V2 lp{w.local_point[2 * slot], w.local_point[2 * slot + 1]};
    V2 pl[2];
    float ni[2], ti[2];
    for (int j = 0; j < 2; ++j) {
        pl[j] = {w.point_local[4 * slot + 2 * j], w.point_local[4 * slot + 2 * j + 1]};
        ni[j] = warm ? dt_ratio * w.normal_impulse[2 * slot + j] : 0.0f;
        ti[j] = warm ? dt_ratio * w.tangent_impulse[2 * slot + j] : 0.0f;
    }
    const float friction = w.friction[slot], tangent_speed = w.tangent_speed[slot];
    const float restitution = w.restitution[slot];
    const int ia = m.fixture_body[fa], ib = m.fixture_body[fb];
    const float rA_ = m.radius[fa], rB_ = m.radius[fb];
    const float mA = w.inv_mass[ia], mB = w.inv_mass[ib], iA = w.inv_inertia[ia], iB = w.inv_inertia[ib];
    const V2 lcA = w.blc(ia), lcB = w.blc(ib);
    const V2 cA{bd.cx[ia], bd.cy[ia]}, cB{bd.cx[ib], bd.cy[ib]};
    const Rot qA{bd.qc[ia], bd.qs[ia]}, qB{bd.qc[ib], bd.qs[ib]};
    const V2 vA{bd.vx[ia], bd.vy[ia]}, vB{bd.vx[ib], bd.vy[ib]};
    const float wA = bd.vw[ia], wB = bd.vw[ib];

    const Xf xfA = xf_from_q(cA, qA, lcA);
    const Xf xfB = xf_from_q(cB, qB, lcB);
    V2 nrm, pts[2];
    if (mtype == CIRCLES) {  // b2WorldManifold::Initialize
        V2 pA = xf_mul(xfA, lp), pB = xf_mul(xfB, pl[0]);
        V2 d = sub(pB, pA);
        bool far = dot(d, d) > EPS * EPS;
        V2 nn = normalize(d);
        V2 cn = far ? nn : V2{1.0f, 0.0f};
        V2 ccA{pA.x + rA_ * cn.x, pA.y + rA_ * cn.y}, ccB{pB.x - rB_ * cn.x, pB.y - rB_ * cn.y};
        V2 cp{0.5f * (ccA.x + ccB.x), 0.5f * (ccA.y + ccB.y)};
        nrm = cn, pts[0] = pts[1] = cp;
    } else if (mtype == FACE_A) {
        V2 fn = rot(xfA.q, ln), fpl = xf_mul(xfA, lp);
        for (int j = 0; j < 2; ++j) {
            V2 qp = xf_mul(xfB, pl[j]);
            float d = dot(sub(qp, fpl), fn);
            float s_ = rA_ - d;
            V2 aA{qp.x + s_ * fn.x, qp.y + s_ * fn.y}, aB{qp.x - rB_ * fn.x, qp.y - rB_ * fn.y};
            pts[j] = {0.5f * (aA.x + aB.x), 0.5f * (aA.y + aB.y)};
        }
        nrm = fn;
    } else {
        V2 fn = rot(xfB.q, ln), fpl = xf_mul(xfB, lp);
        for (int j = 0; j < 2; ++j) {
            V2 qp = xf_mul(xfA, pl[j]);
            float d = dot(sub(qp, fpl), fn);
            float s_ = rB_ - d;
            V2 bB{qp.x + s_ * fn.x, qp.y + s_ * fn.y}, bA{qp.x - rA_ * fn.x, qp.y - rA_ * fn.y};
            pts[j] = {0.5f * (bA.x + bB.x), 0.5f * (bA.y + bB.y)};
        }
        nrm = neg(fn);
    }
    const V2 t = cross_vs(nrm, 1.0f);
    V2 ra[2], rb[2];
    float nmass[2], tmass[2], bias[2];
    for (int j = 0; j < 2; ++j) {
        ra[j] = sub(pts[j], cA), rb[j] = sub(pts[j], cB);
        float rnA = cross(ra[j], nrm), rnB = cross(rb[j], nrm);
        float kn = ((mA + mB) + (iA * rnA) * rnA) + (iB * rnB) * rnB;
        float rtA = cross(ra[j], t), rtB = cross(rb[j], t);
        float kt = ((mA + mB) + (iA * rtA) * rtA) + (iB * rtB) * rtB;
        V2 wBr = cross_sv(wB, rb[j]), wAr = cross_sv(wA, ra[j]);
        float vrel = dot(nrm, V2{((vB.x + wBr.x) - vA.x) - wAr.x, ((vB.y + wBr.y) - vA.y) - wAr.y});
        nmass[j] = inv_if_pos(kn);
        tmass[j] = inv_if_pos(kt);
        bias[j] = vrel < -velocity_threshold ? -restitution * vrel : 0.0f;
    }
    float rn1A = cross(ra[0], nrm), rn1B = cross(rb[0], nrm);
    float rn2A = cross(ra[1], nrm), rn2B = cross(rb[1], nrm);
    float k11 = ((mA + mB) + (iA * rn1A) * rn1A) + (iB * rn1B) * rn1B;
    float k22 = ((mA + mB) + (iA * rn2A) * rn2A) + (iB * rn2B) * rn2B;
    float k12 = ((mA + mB) + (iA * rn1A) * rn2A) + (iB * rn1B) * rn2B;
    bool safe = k11 * k11 < MAX_COND * (k11 * k22 - k12 * k12);
    bool two = count == 2;
    float det = inv_or_zero(k11 * k22 - k12 * k12);
    bool use_k = two && safe;

    c.slot = slot, c.ia = ia, c.ib = ib;
    c.count = (two && !safe) ? 1 : count;
    c.pc_count = count;
    c.mtype = mtype;
    c.mA = mA, c.mB = mB, c.iA = iA, c.iB = iB;
    c.n = nrm;
    c.friction = friction, c.tangent_speed = tangent_speed;
    for (int j = 0; j < 2; ++j) {
        c.rA[j] = ra[j], c.rB[j] = rb[j];
        c.nmass[j] = nmass[j], c.tmass[j] = tmass[j], c.bias[j] = bias[j];
        c.ni[j] = ni[j], c.ti[j] = ti[j];
        c.pl[j] = pl[j];
    }
    c.K[0] = use_k ? k11 : 0.0f, c.K[1] = use_k ? k12 : 0.0f, c.K[2] = use_k ? k12 : 0.0f;
    c.K[3] = use_k ? k22 : 0.0f;
    c.NM[0] = use_k ? det * k22 : 0.0f, c.NM[1] = use_k ? -det * k12 : 0.0f;
    c.NM[2] = use_k ? -det * k12 : 0.0f, c.NM[3] = use_k ? det * k11 : 0.0f;
    c.ln = ln, c.lp = lp, c.lcA = lcA, c.lcB = lcB;
    c.radA = rA_, c.radB = rB_;
}

__device__ __forceinline__ void contact_warm_start(const VCRow &c, const Bodies &bd) {  // contact_solver.py:165-184
    V2 vA{bd.vx[c.ia], bd.vy[c.ia]}, vB{bd.vx[c.ib], bd.vy[c.ib]};
    float wA = bd.vw[c.ia], wB = bd.vw[c.ib];
    V2 t = cross_vs(c.n, 1.0f);
    for (int j = 0; j < c.count; ++j) {
        V2 P{c.ni[j] * c.n.x + c.ti[j] * t.x, c.ni[j] * c.n.y + c.ti[j] * t.y};
        wA = wA - c.iA * cross(c.rA[j], P);
        vA = {vA.x - c.mA * P.x, vA.y - c.mA * P.y};
        wB = wB + c.iB * cross(c.rB[j], P);
        vB = {vB.x + c.mB * P.x, vB.y + c.mB * P.y};
    }
    bd.vx[c.ia] = vA.x, bd.vy[c.ia] = vA.y, bd.vw[c.ia] = wA;
    bd.vx[c.ib] = vB.x, bd.vy[c.ib] = vB.y, bd.vw[c.ib] = wB;
}

__device__ __forceinline__ V2 dvel(V2 vB, float wB, V2 rb, V2 vA, float wA, V2 ra) {
    V2 b = cross_sv(wB, rb), a = cross_sv(wA, ra);
    return {((vB.x + b.x) - vA.x) - a.x, ((vB.y + b.y) - vA.y) - a.y};
}

// b2ContactSolver::SolveVelocityConstraints for one contact (contact_solver.py:194-279)
__device__ __forceinline__ void contact_solve_velocity(VCRow &c, const Bodies &bd) {
    V2 vA{bd.vx[c.ia], bd.vy[c.ia]}, vB{bd.vx[c.ib], bd.vy[c.ib]};
    float wA = bd.vw[c.ia], wB = bd.vw[c.ib];
    const float mA = c.mA, mB = c.mB, iA = c.iA, iB = c.iB;
    V2 n = c.n, t = cross_vs(n, 1.0f);
    for (int j = 0; j < c.count; ++j) {
        V2 d = dvel(vB, wB, c.rB[j], vA, wA, c.rA[j]);
        float vt = dot(d, t) - c.tangent_speed;
        float lam = c.tmass[j] * -vt;
        float maxf = c.friction * c.ni[j];
        float nw = clampf(c.ti[j] + lam, -maxf, maxf);
        lam = nw - c.ti[j];
        V2 P{lam * t.x, lam * t.y};
        vA = {vA.x - mA * P.x, vA.y - mA * P.y};
        wA = wA - iA * cross(c.rA[j], P);
        vB = {vB.x + mB * P.x, vB.y + mB * P.y};
        wB = wB + iB * cross(c.rB[j], P);
        c.ti[j] = nw;
    }
    if (c.count == 1) {
        V2 d = dvel(vB, wB, c.rB[0], vA, wA, c.rA[0]);
        float vn = dot(d, n);
        float lam = -c.nmass[0] * (vn - c.bias[0]);
        float nw = bmax(c.ni[0] + lam, 0.0f);
        lam = nw - c.ni[0];
        V2 P{lam * n.x, lam * n.y};
        vA = {vA.x - mA * P.x, vA.y - mA * P.y};
        wA = wA - iA * cross(c.rA[0], P);
        vB = {vB.x + mB * P.x, vB.y + mB * P.y};
        wB = wB + iB * cross(c.rB[0], P);
        c.ni[0] = nw;
    } else if (c.count == 2) {
        float ax = c.ni[0], ay = c.ni[1];
        V2 d1 = dvel(vB, wB, c.rB[0], vA, wA, c.rA[0]);
        V2 d2 = dvel(vB, wB, c.rB[1], vA, wA, c.rA[1]);
        float vn1 = dot(d1, n), vn2 = dot(d2, n);
        float bx = vn1 - c.bias[0], by = vn2 - c.bias[1];
        bx = bx - (c.K[0] * ax + c.K[2] * ay);
        by = by - (c.K[1] * ax + c.K[3] * ay);
        float x1x = -(c.NM[0] * bx + c.NM[2] * by), x1y = -(c.NM[1] * bx + c.NM[3] * by);
        bool ok1 = x1x >= 0 && x1y >= 0;
        float x2x = -c.nmass[0] * bx;
        bool ok2 = x2x >= 0 && (c.K[1] * x2x + by) >= 0;
        float x3y = -c.nmass[1] * by;
        bool ok3 = x3y >= 0 && (c.K[2] * x3y + bx) >= 0;
        bool ok4 = bx >= 0 && by >= 0;
        bool c1 = ok1, c2 = !ok1 && ok2, c3 = !ok1 && !ok2 && ok3, c4 = !ok1 && !ok2 && !ok3 && ok4;
        if (c1 || c2 || c3 || c4) {
            float xx = c1 ? x1x : c2 ? x2x : 0.0f;
            float xy = c1 ? x1y : c3 ? x3y : 0.0f;
            float dx = xx - ax, dy = xy - ay;
            V2 P1{dx * n.x, dx * n.y}, P2{dy * n.x, dy * n.y};
            vA = {vA.x - mA * (P1.x + P2.x), vA.y - mA * (P1.y + P2.y)};
            wA = wA - iA * (cross(c.rA[0], P1) + cross(c.rA[1], P2));
            vB = {vB.x + mB * (P1.x + P2.x), vB.y + mB * (P1.y + P2.y)};
            wB = wB + iB * (cross(c.rB[0], P1) + cross(c.rB[1], P2));
            c.ni[0] = xx, c.ni[1] = xy;
        }
    }
    bd.vx[c.ia] = vA.x, bd.vy[c.ia] = vA.y, bd.vw[c.ia] = wA;
    bd.vx[c.ib] = vB.x, bd.vy[c.ib] = vB.y, bd.vw[c.ib] = wB;
}

// b2ContactSolver::SolvePositionConstraints for one contact (contact_solver.py:307-354); masses passed so that
// SolveTOI can zero those of the bodies that are not the TOI pair.
__device__ __forceinline__ float contact_solve_position(const VCRow &c, const Bodies &bd, float baumgarte, float slop,
                                                     float max_lin, float mA, float mB, float iA, float iB) {
    V2 cA{bd.cx[c.ia], bd.cy[c.ia]}, cB{bd.cx[c.ib], bd.cy[c.ib]};
    float aA = bd.ca[c.ia], aB = bd.ca[c.ib];
    float min_sep = 0.0f;
    for (int j = 0; j < c.pc_count; ++j) {
        Xf xfA = xf_from_q(cA, body_rot(bd, c.ia, aA), c.lcA), xfB = xf_from_q(cB, body_rot(bd, c.ib, aB), c.lcB);
        V2 nrm, p;
        float sep;
        if (c.mtype == CIRCLES) {
            V2 pA = xf_mul(xfA, c.lp), pB = xf_mul(xfB, c.pl[0]);
            V2 cn = normalize(sub(pB, pA));
            p = {0.5f * (pA.x + pB.x), 0.5f * (pA.y + pB.y)};
            sep = (dot(sub(pB, pA), cn) - c.radA) - c.radB;
            nrm = cn;
        } else if (c.mtype == FACE_A) {
            V2 an = rot(xfA.q, c.ln), apl = xf_mul(xfA, c.lp), aq = xf_mul(xfB, c.pl[j]);
            sep = (dot(sub(aq, apl), an) - c.radA) - c.radB;
            nrm = an, p = aq;
        } else {
            V2 bn = rot(xfB.q, c.ln), bpl = xf_mul(xfB, c.lp), bq = xf_mul(xfA, c.pl[j]);
            sep = (dot(sub(bq, bpl), bn) - c.radA) - c.radB;
            nrm = neg(bn), p = bq;
        }
        V2 ra = sub(p, cA), rb = sub(p, cB);
        min_sep = bmin(min_sep, sep);
        float C_ = clampf(baumgarte * (sep + slop), -max_lin, 0.0f);
        float rnA = cross(ra, nrm), rnB = cross(rb, nrm);
        float K = ((mA + mB) + (iA * rnA) * rnA) + (iB * rnB) * rnB;
        float imp = K > 0 ? -C_ / K : 0.0f;
        V2 P{imp * nrm.x, imp * nrm.y};
        cA = {cA.x - mA * P.x, cA.y - mA * P.y};
        aA = aA - iA * cross(ra, P);
        cB = {cB.x + mB * P.x, cB.y + mB * P.y};
        aB = aB + iB * cross(rb, P);
    }
    bd.cx[c.ia] = cA.x, bd.cy[c.ia] = cA.y, bd.ca[c.ia] = aA;
    bd.cx[c.ib] = cB.x, bd.cy[c.ib] = cB.y, bd.ca[c.ib] = aB;
    return min_sep;
}

// ---------------------------------------------------------------- joints (joints.py)
__device__ __forceinline__ void k_rev(float mA, float mB, float iA, float iB, V2 rA, V2 rB, V3 &ex, V3 &ey, V3 &ez) {
    float exx = ((mA + mB) + (rA.y * rA.y) * iA) + (rB.y * rB.y) * iB;
    float eyx = (-rA.y * rA.x) * iA - (rB.y * rB.x) * iB;
    float ezx = -rA.y * iA - rB.y * iB;
    float eyy = ((mA + mB) + (rA.x * rA.x) * iA) + (rB.x * rB.x) * iB;
    float ezy = rA.x * iA + rB.x * iB;
    float ezz = iA + iB;
    ex = {exx, eyx, ezx}, ey = {eyx, eyy, ezy}, ez = {ezx, ezy, ezz};
}
__device__ __forceinline__ void k_prism(float mA, float mB, float iA, float iB, float s1, float s2, float a1,
                                        float a2, V3 &ex, V3 &ey, V3 &ez) {
    float k11 = ((mA + mB) + (iA * s1) * s1) + (iB * s2) * s2;
    float k12 = iA * s1 + iB * s2;
    float k13 = (iA * s1) * a1 + (iB * s2) * a2;
    float k22 = iA + iB;
    if (k22 == 0) k22 = 1.0f;
    float k23 = iA * a1 + iB * a2;
    float k33 = ((mA + mB) + (iA * a1) * a1) + (iB * a2) * a2;
    ex = {k11, k12, k13}, ey = {k12, k22, k23}, ez = {k13, k23, k33};
}

// InitVelocityConstraints for one ordered joint, without the velocity writes (joints.py:61-174)
__device__ __noinline__ void prepare_joint(const DevModel &m, const W &w, int jid, const Bodies &bd,
                                           const goib2d_settings &s, float dt, float dt_ratio, bool warm, JRow &r) {
    // every load first (the joint's fields, then its bodies), then the arithmetic, then the row's stores (see
    // prepare_contact)
    const bool v24 = s.revolute_v24;
    const int type = m.joint_type[jid];
    const int ia = m.joint_a[jid], ib = m.joint_b[jid];
    const V2 laa{m.local_anchor_a[2 * jid], m.local_anchor_a[2 * jid + 1]};
    const V2 lab{m.local_anchor_b[2 * jid], m.local_anchor_b[2 * jid + 1]};
    const float ref = m.reference_angle[jid];
    const V2 lxa{m.local_axis_a[2 * jid], m.local_axis_a[2 * jid + 1]};
    const V2 lya{m.local_yaxis_a[2 * jid], m.local_yaxis_a[2 * jid + 1]};
    const bool en_motor = w.enable_motor[jid], en_limit = w.enable_limit[jid];
    const float lower = w.lower[jid], upper = w.upper[jid];
    const int state_in = w.limit_state[jid];
    float ix = w.impulse[3 * jid], iy = w.impulse[3 * jid + 1], iz = w.impulse[3 * jid + 2];
    float mimp = w.motor_impulse[jid];
    const float frequency = w.frequency[jid], damping = w.damping[jid];
    const float motor_speed = w.motor_speed[jid], max_motor = w.max_motor[jid];
    const float lower_imp = w.lower_impulse[jid], upper_imp = w.upper_impulse[jid];
    const float mA = w.inv_mass[ia], mB = w.inv_mass[ib], iA = w.inv_inertia[ia], iB = w.inv_inertia[ib];
    const V2 lcA = w.blc(ia), lcB = w.blc(ib);
    const V2 cA{bd.cx[ia], bd.cy[ia]}, cB{bd.cx[ib], bd.cy[ib]};
    const float aA = bd.ca[ia], aB = bd.ca[ib];
    const Rot qA{bd.qc[ia], bd.qs[ia]}, qB{bd.qc[ib], bd.qs[ib]};

    const V2 la{laa.x - lcA.x, laa.y - lcA.y};
    const V2 lb{lab.x - lcB.x, lab.y - lcB.y};
    const V2 rA = rot(qA, la), rB = rot(qB, lb);
    const bool is_rev = type == REVOLUTE, is_pri = type == PRISMATIC;
    V3 revx, revy, revz;
    k_rev(mA, mB, iA, iB, rA, rB, revx, revy, revz);
    bool fixed = (iA + iB) == 0;
    float rev_mm = inv_if_pos(iA + iB);
    float rev_mimp = (!en_motor || fixed) ? 0.0f : mimp;
    float angle = (aB - aA) - ref;
    bool equal = babs(upper - lower) < 2.0f * s.angular_slop;
    bool lim_on = en_limit && !fixed;
    int rev_state = !lim_on ? INACTIVE_LIMIT
                    : equal ? EQUAL_LIMITS
                    : angle <= lower ? AT_LOWER
                    : angle >= upper ? AT_UPPER
                                     : INACTIVE_LIMIT;
    bool rev_zero_z = lim_on && !equal && (rev_state == INACTIVE_LIMIT || rev_state != state_in);
    float dx = ((cB.x - cA.x) + rB.x) - rA.x, dy = ((cB.y - cA.y) + rB.y) - rA.y;
    V2 ax = rot(qA, lxa);
    float a1 = cross(V2{dx + rA.x, dy + rA.y}, ax), a2 = cross(rB, ax);
    float pri_mm = ((mA + mB) + (iA * a1) * a1) + (iB * a2) * a2;
    pri_mm = pri_mm > 0 ? 1.0f / pri_mm : pri_mm;
    V2 pe = rot(qA, lya);
    float s1 = cross(V2{dx + rA.x, dy + rA.y}, pe), s2 = cross(rB, pe);
    V3 prx, pry, prz;
    k_prism(mA, mB, iA, iB, s1, s2, a1, a2, prx, pry, prz);
    float trans = dot(ax, V2{dx, dy});
    bool pequal = babs(upper - lower) < 2.0f * s.linear_slop;
    int pri_state = !en_limit ? INACTIVE_LIMIT
                    : pequal ? EQUAL_LIMITS
                    : trans <= lower ? AT_LOWER
                    : trans >= upper ? AT_UPPER
                                     : INACTIVE_LIMIT;
    bool pri_zero_z = !en_limit || (!pequal && (pri_state == INACTIVE_LIMIT || pri_state != state_in));
    float pri_mimp = en_motor ? mimp : 0.0f;
    bool soft = frequency > 0;
    V3 i22x, i22y, i22z, symx, symy, symz;
    inverse22_of33(revx, revy, i22x, i22y, i22z);
    sym_inverse33(revx, revy, revz, symx, symy, symz);
    float invM = iA + iB;
    float wm = inv_if_pos(invM);
    float C = (aB - aA) - ref;
    const float two_pi = 2.0f * PI_F;
    float omega = two_pi * frequency;
    float d = ((2.0f * wm) * damping) * omega;
    float kk = (wm * omega) * omega;
    float h = dt;
    float gamma = inv_or_zero(h * (d + h * kk));
    float bias = ((C * h) * kk) * gamma;
    float ezz_soft = inv_or_zero(invM + gamma);
    bool use22 = soft || revz.z == 0;
    V3 wmx = use22 ? i22x : symx, wmy = use22 ? i22y : symy, wmz = use22 ? i22z : symz;
    if (soft) wmz.z = ezz_soft;
    const bool is_mot = type == MOTOR;
    const V3 Kx = is_rev || is_mot ? revx : is_pri ? prx : wmx;
    const V3 Ky = is_rev || is_mot ? revy : is_pri ? pry : wmy;
    const V3 Kz = is_rev || is_mot ? revz : is_pri ? prz : wmz;
    // the motor joint's position errors (b2MotorJoint::InitVelocityConstraints): linear offset = (lower, upper),
    // angular offset = motor_speed in the joint row (see motor_velocity)
    const V2 mro = rot(qA, V2{lower, upper});
    const V2 mot_err{(((cB.x + rB.x) - cA.x) - rA.x) - mro.x, (((cB.y + rB.y) - cA.y) - rA.y) - mro.y};
    const float mot_ang = (aB - aA) - motor_speed;
    const int limit_state = is_rev ? rev_state : is_pri ? pri_state : INACTIVE_LIMIT;
    bool zero_z = is_rev ? (v24 ? false : rev_zero_z) : is_pri ? pri_zero_z : false;
    if (zero_z) iz = 0.0f;
    mimp = is_rev ? rev_mimp : is_pri ? pri_mimp : 0.0f;
    float imp[5];
#define SC(x) (warm ? (x) * dt_ratio : 0.0f)
    if (v24) {
        float lo = (is_rev && lim_on) ? lower_imp : 0.0f;
        float up = (is_rev && lim_on) ? upper_imp : 0.0f;
        imp[0] = SC(ix), imp[1] = SC(iy), imp[2] = is_rev ? iz : SC(iz), imp[3] = SC(lo), imp[4] = SC(up);
    } else {
        imp[0] = SC(ix), imp[1] = SC(iy), imp[2] = SC(iz), imp[3] = 0.0f, imp[4] = 0.0f;
    }
    const float mimp_row = SC(mimp);
#undef SC
    const float d33 = det33_inv(Kx, Ky, Kz);
    const float d22 = det22_inv(Kx.x, Ky.x, Kx.y, Ky.y);

    r.jid = jid, r.type = type, r.ia = ia, r.ib = ib;
    r.mA = mA, r.mB = mB, r.iA = iA, r.iB = iB;
    r.rA = rA, r.rB = rB, r.la = la, r.lb = lb;
    r.ref = ref;
    r.lx = lxa, r.ly = lya;
    r.Kx = Kx, r.Ky = Ky, r.Kz = Kz;
    r.limit_state = limit_state;
    for (int k = 0; k < 5; ++k) r.imp[k] = imp[k];
    r.d33 = d33, r.d22 = d22;
    r.mimp = mimp_row;
    r.inv_dt = dt > 0 ? 1.0f / dt : 0.0f;
    r.motor_mass = is_rev ? rev_mm : is_pri ? pri_mm : 0.0f;
    r.enable_motor = en_motor, r.enable_limit = en_limit;
    r.motor_speed = motor_speed;
    r.max_impulse = dt * max_motor;
    r.ax = ax, r.pe = pe, r.a1 = a1, r.a2 = a2, r.s1 = s1, r.s2 = s2;
    r.soft = soft, r.gamma = soft ? gamma : 0.0f, r.bias = soft ? bias : 0.0f, r.angle = angle;
    r.lower = lower, r.upper = upper;
    if (is_mot) {
        r.ax = mot_err, r.angle = mot_ang, r.motor_mass = rev_mm;
        r.gamma = dt * frequency;  // the linear impulse's limit, h * max force
        r.bias = damping;          // the correction factor
        r.soft = false;
    }
}

__device__ __forceinline__ void joint_warm_start(const JRow &r, const Bodies &bd, bool v24) {  // joints.py:202-248
    V2 vA{bd.vx[r.ia], bd.vy[r.ia]}, vB{bd.vx[r.ib], bd.vy[r.ib]};
    float wA = bd.vw[r.ia], wB = bd.vw[r.ib];
    float ix = r.imp[0], iy = r.imp[1], iz = r.imp[2], mi = r.mimp;
    const float mA = r.mA, mB = r.mB, iA = r.iA, iB = r.iB;
    if (r.type == REVOLUTE) {
        V2 P{ix, iy};
        if (v24) {
            float axial = (mi + r.imp[3]) - r.imp[4];
            vA = {vA.x - mA * P.x, vA.y - mA * P.y};
            wA = wA - iA * (cross(r.rA, P) + axial);
            vB = {vB.x + mB * P.x, vB.y + mB * P.y};
            wB = wB + iB * (cross(r.rB, P) + axial);
        } else {
            vA = {vA.x - mA * P.x, vA.y - mA * P.y};
            wA = wA - iA * ((cross(r.rA, P) + mi) + iz);
            vB = {vB.x + mB * P.x, vB.y + mB * P.y};
            wB = wB + iB * ((cross(r.rB, P) + mi) + iz);
        }
    } else if (r.type == PRISMATIC) {
        float mz = mi + iz;
        V2 P{ix * r.pe.x + mz * r.ax.x, ix * r.pe.y + mz * r.ax.y};
        float LA = (ix * r.s1 + iy) + mz * r.a1;
        float LB = (ix * r.s2 + iy) + mz * r.a2;
        vA = {vA.x - mA * P.x, vA.y - mA * P.y};
        wA = wA - iA * LA;
        vB = {vB.x + mB * P.x, vB.y + mB * P.y};
        wB = wB + iB * LB;
    } else {
        V2 P{ix, iy};
        vA = {vA.x - mA * P.x, vA.y - mA * P.y};
        wA = wA - iA * (cross(r.rA, P) + iz);
        vB = {vB.x + mB * P.x, vB.y + mB * P.y};
        wB = wB + iB * (cross(r.rB, P) + iz);
    }
    bd.vx[r.ia] = vA.x, bd.vy[r.ia] = vA.y, bd.vw[r.ia] = wA;
    bd.vx[r.ib] = vB.x, bd.vy[r.ib] = vB.y, bd.vw[r.ib] = wB;
}

__device__ __forceinline__ void rev_velocity(JRow &r, V2 &vA, float &wA, V2 &vB, float &wB) {  // joints.py:257-299
    const float mA = r.mA, mB = r.mB, iA = r.iA, iB = r.iB;
    V3 ex = r.Kx, ey = r.Ky, ez = r.Kz;
    bool fixed = (iA + iB) == 0;
    int st = r.limit_state;
    bool on = r.enable_motor && st != EQUAL_LIMITS && !fixed;
    {
        float cdot = (wB - wA) - r.motor_speed;
        float impulse = -r.motor_mass * cdot;
        float nmi = clampf(r.mimp + impulse, -r.max_impulse, r.max_impulse);
        impulse = nmi - r.mimp;
        if (on) wA = wA - iA * impulse, wB = wB + iB * impulse, r.mimp = nmi;
    }
    float ix = r.imp[0], iy = r.imp[1], iz = r.imp[2];
    V2 c1 = dvel(vB, wB, r.rB, vA, wA, r.rA);
    bool lim = r.enable_limit && st != INACTIVE_LIMIT && !fixed;
    if (lim) {
        float c2 = wB - wA;
        V3 sv = solve33d(ex, ey, ez, V3{c1.x, c1.y, c2}, r.d33);
        float jx = -sv.x, jy = -sv.y, jz = -sv.z;
        float new_z = iz + jz;
        bool redo = (st == AT_LOWER && new_z < 0) || (st == AT_UPPER && new_z > 0);
        V2 rr{0.0f, 0.0f};
        if (redo) rr = solve22d(ex.x, ey.x, ex.y, ey.y, -c1.x + iz * ez.x, -c1.y + iz * ez.y, r.d22);
        float lx = redo ? rr.x : jx, ly = redo ? rr.y : jy, lz = redo ? -iz : jz;
        float nix = redo ? ix + rr.x : ix + jx, niy = redo ? iy + rr.y : iy + jy, niz = redo ? 0.0f : iz + jz;
        vA = {vA.x - mA * lx, vA.y - mA * ly};
        wA = wA - iA * (cross(r.rA, V2{lx, ly}) + lz);
        vB = {vB.x + mB * lx, vB.y + mB * ly};
        wB = wB + iB * (cross(r.rB, V2{lx, ly}) + lz);
        r.imp[0] = nix, r.imp[1] = niy, r.imp[2] = niz;
    } else {
        V2 p = solve22d(ex.x, ey.x, ex.y, ey.y, -c1.x, -c1.y, r.d22);
        vA = {vA.x - mA * p.x, vA.y - mA * p.y};
        wA = wA - iA * cross(r.rA, p);
        vB = {vB.x + mB * p.x, vB.y + mB * p.y};
        wB = wB + iB * cross(r.rB, p);
        r.imp[0] = ix + p.x, r.imp[1] = iy + p.y;
    }
}

__device__ __forceinline__ void rev24_velocity(JRow &r, V2 &vA, float &wA, V2 &vB, float &wB) {  // joints.py:302-343
    const float mA = r.mA, mB = r.mB, iA = r.iA, iB = r.iB;
    V3 ex = r.Kx, ey = r.Ky;
    bool fixed = (iA + iB) == 0;
    float am = r.motor_mass;
    bool on = r.enable_motor && !fixed;
    {
        float cdot = (wB - wA) - r.motor_speed;
        float impulse = -am * cdot;
        float nmi = clampf(r.mimp + impulse, -r.max_impulse, r.max_impulse);
        impulse = nmi - r.mimp;
        if (on) wA = wA - iA * impulse, wB = wB + iB * impulse, r.mimp = nmi;
    }
    bool lim = r.enable_limit && !fixed;
    {
        float C = r.angle - r.lower;
        float impulse = -am * ((wB - wA) + bmax(C, 0.0f) * r.inv_dt);
        float nlo = bmax(r.imp[3] + impulse, 0.0f);
        impulse = nlo - r.imp[3];
        if (lim) wA = wA - iA * impulse, wB = wB + iB * impulse, r.imp[3] = nlo;
    }
    {
        float C = r.upper - r.angle;
        float impulse = -am * ((wA - wB) + bmax(C, 0.0f) * r.inv_dt);
        float nup = bmax(r.imp[4] + impulse, 0.0f);
        impulse = nup - r.imp[4];
        if (lim) wA = wA + iA * impulse, wB = wB - iB * impulse, r.imp[4] = nup;
    }
    V2 c1 = dvel(vB, wB, r.rB, vA, wA, r.rA);
    V2 p = solve22d(ex.x, ey.x, ex.y, ey.y, -c1.x, -c1.y, r.d22);
    vA = {vA.x - mA * p.x, vA.y - mA * p.y};
    wA = wA - iA * cross(r.rA, p);
    vB = {vB.x + mB * p.x, vB.y + mB * p.y};
    wB = wB + iB * cross(r.rB, p);
    r.imp[0] = r.imp[0] + p.x, r.imp[1] = r.imp[1] + p.y;
}

__device__ __forceinline__ void pri_velocity(JRow &r, V2 &vA, float &wA, V2 &vB, float &wB) {  // joints.py:354-404
    const float mA = r.mA, mB = r.mB, iA = r.iA, iB = r.iB;
    V3 ex = r.Kx, ey = r.Ky, ez = r.Kz;
    int st = r.limit_state;
    V2 ax = r.ax, pe = r.pe;
    float a1 = r.a1, a2 = r.a2, s1 = r.s1, s2 = r.s2;
    bool on = r.enable_motor && st != EQUAL_LIMITS;
    {
        float cdot = (dot(ax, sub(vB, vA)) + a2 * wB) - a1 * wA;
        float impulse = r.motor_mass * (r.motor_speed - cdot);
        float nmi = clampf(r.mimp + impulse, -r.max_impulse, r.max_impulse);
        impulse = nmi - r.mimp;
        V2 P{impulse * ax.x, impulse * ax.y};
        float LA = impulse * a1, LB = impulse * a2;
        if (on) {
            vA = {vA.x - mA * P.x, vA.y - mA * P.y};
            wA = wA - iA * LA;
            vB = {vB.x + mB * P.x, vB.y + mB * P.y};
            wB = wB + iB * LB;
            r.mimp = nmi;
        }
    }
    float c1x = (dot(pe, sub(vB, vA)) + s2 * wB) - s1 * wA;
    float c1y = wB - wA;
    float ix = r.imp[0], iy = r.imp[1], iz = r.imp[2];
    bool lim = r.enable_limit && st != INACTIVE_LIMIT;
    float Px, Py, LA, LB;
    if (lim) {
        float c2 = (dot(ax, sub(vB, vA)) + a2 * wB) - a1 * wA;
        V3 df = solve33d(ex, ey, ez, V3{-c1x, -c1y, -c2}, r.d33);
        float nz_ = iz + df.z;
        nz_ = st == AT_LOWER ? bmax(nz_, 0.0f) : st == AT_UPPER ? bmin(nz_, 0.0f) : nz_;
        float bx = -c1x - (nz_ - iz) * ez.x;
        float by = -c1y - (nz_ - iz) * ez.y;
        V2 f = solve22d(ex.x, ey.x, ex.y, ey.y, bx, by, r.d22);
        float fx = f.x + ix, fy = f.y + iy;
        float dfx = fx - ix, dfy = fy - iy, dfz = nz_ - iz;
        Px = dfx * pe.x + dfz * ax.x;
        Py = dfx * pe.y + dfz * ax.y;
        LA = (dfx * s1 + dfy) + dfz * a1;
        LB = (dfx * s2 + dfy) + dfz * a2;
        r.imp[0] = fx, r.imp[1] = fy, r.imp[2] = nz_;
    } else {
        V2 g = solve22d(ex.x, ey.x, ex.y, ey.y, -c1x, -c1y, r.d22);
        Px = g.x * pe.x, Py = g.x * pe.y;
        LA = g.x * s1 + g.y;
        LB = g.x * s2 + g.y;
        r.imp[0] = ix + g.x, r.imp[1] = iy + g.y;
    }
    vA = {vA.x - mA * Px, vA.y - mA * Py};
    wA = wA - iA * LA;
    vB = {vB.x + mB * Px, vB.y + mB * Py};
    wB = wB + iB * LB;
}

__device__ __forceinline__ void weld_velocity(JRow &r, V2 &vA, float &wA, V2 &vB, float &wB) {  // joints.py:407-437
    const float mA = r.mA, mB = r.mB, iA = r.iA, iB = r.iB;
    V3 ex = r.Kx, ey = r.Ky, ez = r.Kz;
    float ix = r.imp[0], iy = r.imp[1], iz = r.imp[2];
    if (r.soft) {
        float c2 = wB - wA;
        float i2 = -ez.z * ((c2 + r.bias) + r.gamma * iz);
        float s_iz = iz + i2;
        float swA = wA - iA * i2, swB = wB + iB * i2;
        V2 c1 = dvel(vB, swB, r.rB, vA, swA, r.rA);
        V2 qv = mat33_mul22(ex, ey, c1);
        float i1x = -qv.x, i1y = -qv.y;
        vA = {vA.x - mA * i1x, vA.y - mA * i1y};
        wA = swA - iA * cross(r.rA, V2{i1x, i1y});
        vB = {vB.x + mB * i1x, vB.y + mB * i1y};
        wB = swB + iB * cross(r.rB, V2{i1x, i1y});
        r.imp[0] = ix + i1x, r.imp[1] = iy + i1y, r.imp[2] = s_iz;
    } else {
        V2 d1 = dvel(vB, wB, r.rB, vA, wA, r.rA);
        V3 q3 = mat33_mul(ex, ey, ez, V3{d1.x, d1.y, wB - wA});
        float jx = -q3.x, jy = -q3.y, jz = -q3.z;
        vA = {vA.x - mA * jx, vA.y - mA * jy};
        wA = wA - iA * (cross(r.rA, V2{jx, jy}) + jz);
        vB = {vB.x + mB * jx, vB.y + mB * jy};
        wB = wB + iB * (cross(r.rB, V2{jx, jy}) + jz);
        r.imp[0] = ix + jx, r.imp[1] = iy + jy, r.imp[2] = iz + jz;
    }
}

// b2MotorJoint::SolveVelocityConstraints, Box2D 2.3.1's motor joint (the reference engine has none; this follows the
// published method): the angular impulse toward the angular offset, clamped to h * max torque, then the linear
// impulse toward the linear offset through the 2x2 point mass, its length clamped to h * max force; both drive the
// position errors of the step's start, scaled by correction factor / h. Row fields: ax = linear error, angle =
// angular error, bias = correction factor, max_impulse = h * max torque, gamma = h * max force, imp = (linear x,
// linear y, angular). The same operations as the oracle's motor_velocity.
__device__ __forceinline__ void motor_velocity(JRow &r, V2 &vA, float &wA, V2 &vB, float &wB) {
    const float mA = r.mA, mB = r.mB, iA = r.iA, iB = r.iB;
    const float k = r.inv_dt * r.bias;
    {
        const float cdot = (wB - wA) + k * r.angle;
        float impulse = -r.motor_mass * cdot;
        const float old = r.imp[2];
        const float ni = clampf(old + impulse, -r.max_impulse, r.max_impulse);
        impulse = ni - old;
        wA = wA - iA * impulse, wB = wB + iB * impulse;
        r.imp[2] = ni;
    }
    const V2 d = dvel(vB, wB, r.rB, vA, wA, r.rA);
    const float cx = d.x + k * r.ax.x, cy = d.y + k * r.ax.y;
    const V2 sv = solve22d(r.Kx.x, r.Ky.x, r.Kx.y, r.Ky.y, cx, cy, r.d22);
    const float ox = r.imp[0], oy = r.imp[1];
    float nx = ox - sv.x, ny = oy - sv.y;
    const float max_f = r.gamma;
    if (nx * nx + ny * ny > max_f * max_f) {
        const V2 u = normalize(V2{nx, ny});
        nx = u.x * max_f, ny = u.y * max_f;
    }
    const float jx = nx - ox, jy = ny - oy;
    vA = {vA.x - mA * jx, vA.y - mA * jy};
    wA = wA - iA * cross(r.rA, V2{jx, jy});
    vB = {vB.x + mB * jx, vB.y + mB * jy};
    wB = wB + iB * cross(r.rB, V2{jx, jy});
    r.imp[0] = nx, r.imp[1] = ny;
}

__device__ __forceinline__ void joint_solve_velocity(JRow &r, const Bodies &bd, bool v24) {  // joints.py:440-459
    V2 vA{bd.vx[r.ia], bd.vy[r.ia]}, vB{bd.vx[r.ib], bd.vy[r.ib]};
    float wA = bd.vw[r.ia], wB = bd.vw[r.ib];
    if (r.type == REVOLUTE) {
        if (v24)
            rev24_velocity(r, vA, wA, vB, wB);
        else
            rev_velocity(r, vA, wA, vB, wB);
    } else if (r.type == PRISMATIC) {
        pri_velocity(r, vA, wA, vB, wB);
    } else if (r.type == MOTOR) {
        motor_velocity(r, vA, wA, vB, wB);
    } else {
        weld_velocity(r, vA, wA, vB, wB);
    }
    bd.vx[r.ia] = vA.x, bd.vy[r.ia] = vA.y, bd.vw[r.ia] = wA;
    bd.vx[r.ib] = vB.x, bd.vy[r.ib] = vB.y, bd.vw[r.ib] = wB;
}

__device__ __forceinline__ bool rev_point_position(const JRow &r, const Bodies &bd, V2 &cA, float &aA, V2 &cB,
                                                   float &aB, const goib2d_settings &s,
                                                   float ang_err) {  // joints.py:501-520
    const float mA = r.mA, mB = r.mB, iA = r.iA, iB = r.iB;
    Rot qA = body_rot(bd, r.ia, aA), qB = body_rot(bd, r.ib, aB);
    V2 ra = rot(qA, r.la), rb = rot(qB, r.lb);
    float Cx = ((cB.x + rb.x) - cA.x) - ra.x;
    float Cy = ((cB.y + rb.y) - cA.y) - ra.y;
    float pos_err = length(V2{Cx, Cy});
    float kxx = ((mA + mB) + (iA * ra.y) * ra.y) + (iB * rb.y) * rb.y;
    float kxy = (-iA * ra.x) * ra.y - (iB * rb.x) * rb.y;
    float kyy = ((mA + mB) + (iA * ra.x) * ra.x) + (iB * rb.x) * rb.x;
    V2 jj = solve22(kxx, kxy, kxy, kyy, Cx, Cy);
    float jx = -jj.x, jy = -jj.y;
    cA = {cA.x - mA * jx, cA.y - mA * jy};
    aA = aA - iA * cross(ra, V2{jx, jy});
    cB = {cB.x + mB * jx, cB.y + mB * jy};
    aB = aB + iB * cross(rb, V2{jx, jy});
    return pos_err <= s.linear_slop && ang_err <= s.angular_slop;
}

__device__ __forceinline__ bool joint_solve_position(const JRow &r, const Bodies &bd, const goib2d_settings &s) {
    if (r.type == MOTOR) return true;  // b2MotorJoint::SolvePositionConstraints corrects nothing
    V2 cA{bd.cx[r.ia], bd.cy[r.ia]}, cB{bd.cx[r.ib], bd.cy[r.ib]};
    float aA = bd.ca[r.ia], aB = bd.ca[r.ib];
    const float mA = r.mA, mB = r.mB, iA = r.iA, iB = r.iB;
    bool ok;
    if (r.type == REVOLUTE) {
        bool fixed = (iA + iB) == 0;
        float angle = (aB - aA) - r.ref;
        float mac = s.max_angular_correction;
        float C, ang_err;
        bool lim;
        if (s.revolute_v24) {  // joints.py:482-498
            lim = r.enable_limit && !fixed;
            bool equal = babs(r.upper - r.lower) < 2.0f * s.angular_slop;
            C = equal              ? clampf(angle - r.lower, -mac, mac)
                : angle <= r.lower ? clampf((angle - r.lower) + s.angular_slop, -mac, 0.0f)
                : angle >= r.upper ? clampf((angle - r.upper) - s.angular_slop, 0.0f, mac)
                                   : 0.0f;
            ang_err = lim ? babs(C) : 0.0f;
        } else {  // joints.py:462-479
            int st = r.limit_state;
            lim = r.enable_limit && st != INACTIVE_LIMIT && !fixed;
            float ce = clampf(angle - r.lower, -mac, mac);
            float cl = angle - r.lower, cu = angle - r.upper;
            C = st == EQUAL_LIMITS ? ce
                : st == AT_LOWER   ? clampf(cl + s.angular_slop, -mac, 0.0f)
                                   : clampf(cu - s.angular_slop, 0.0f, mac);
            ang_err = st == EQUAL_LIMITS ? babs(ce) : st == AT_LOWER ? -cl : cu;
            if (!lim) ang_err = 0.0f;
        }
        float limit_impulse = -r.motor_mass * C;
        if (lim) aA = aA - iA * limit_impulse, aB = aB + iB * limit_impulse;
        ok = rev_point_position(r, bd, cA, aA, cB, aB, s, ang_err);
    } else if (r.type == PRISMATIC) {  // joints.py:523-566
        Rot qA = body_rot(bd, r.ia, aA), qB = body_rot(bd, r.ib, aB);
        V2 ra = rot(qA, r.la), rb = rot(qB, r.lb);
        float dx = ((cB.x + rb.x) - cA.x) - ra.x, dy = ((cB.y + rb.y) - cA.y) - ra.y;
        V2 ax = rot(qA, r.lx);
        float a1 = cross(V2{dx + ra.x, dy + ra.y}, ax), a2 = cross(rb, ax);
        V2 pe = rot(qA, r.ly);
        float s1 = cross(V2{dx + ra.x, dy + ra.y}, pe), s2 = cross(rb, pe);
        float c1x = dot(pe, V2{dx, dy});
        float c1y = (aB - aA) - r.ref;
        float lin_err = babs(c1x), ang_err = babs(c1y);
        float lo = r.lower, hi = r.upper;
        float t = dot(ax, V2{dx, dy});
        float mlc = s.max_linear_correction;
        bool eq = babs(hi - lo) < 2.0f * s.linear_slop;
        bool at_lo = t <= lo, at_hi = t >= hi;
        bool active = r.enable_limit && (eq || at_lo || at_hi);
        float c2 = eq      ? clampf(t, -mlc, mlc)
                   : at_lo ? clampf((t - lo) + s.linear_slop, -mlc, 0.0f)
                           : clampf((t - hi) - s.linear_slop, 0.0f, mlc);
        float e2 = eq ? babs(t) : at_lo ? lo - t : t - hi;
        if (active) lin_err = bmax(lin_err, e2);
        V3 ex, ey, ez;
        k_prism(mA, mB, iA, iB, s1, s2, a1, a2, ex, ey, ez);
        float ix, iy, iz;
        if (active) {
            V3 i3 = solve33(ex, ey, ez, V3{-c1x, -c1y, -c2});
            ix = i3.x, iy = i3.y, iz = i3.z;
        } else {
            V2 g = solve22(ex.x, ex.y, ex.y, ey.y, -c1x, -c1y);
            ix = g.x, iy = g.y, iz = 0.0f;
        }
        float Px = ix * pe.x + iz * ax.x, Py = ix * pe.y + iz * ax.y;
        float LA = (ix * s1 + iy) + iz * a1, LB = (ix * s2 + iy) + iz * a2;
        cA = {cA.x - mA * Px, cA.y - mA * Py};
        aA = aA - iA * LA;
        cB = {cB.x + mB * Px, cB.y + mB * Py};
        aB = aB + iB * LB;
        ok = lin_err <= s.linear_slop && ang_err <= s.angular_slop;
    } else {  // joints.py:569-595
        Rot qA = body_rot(bd, r.ia, aA), qB = body_rot(bd, r.ib, aB);
        V2 ra = rot(qA, r.la), rb = rot(qB, r.lb);
        V3 ex, ey, ez;
        k_rev(mA, mB, iA, iB, ra, rb, ex, ey, ez);
        float c1x = ((cB.x + rb.x) - cA.x) - ra.x, c1y = ((cB.y + rb.y) - cA.y) - ra.y;
        float pos_err = length(V2{c1x, c1y});
        float c2 = (aB - aA) - r.ref;
        bool use33 = !r.soft && ez.z > 0;
        float ix, iy, iz;
        if (use33) {
            V3 p = solve33(ex, ey, ez, V3{c1x, c1y, c2});
            ix = -p.x, iy = -p.y, iz = -p.z;
        } else {
            V2 p = solve22(ex.x, ey.x, ex.y, ey.y, c1x, c1y);
            ix = -p.x, iy = -p.y, iz = 0.0f;
        }
        float ang_err = r.soft ? 0.0f : babs(c2);
        float tA = r.soft ? cross(ra, V2{ix, iy}) : cross(ra, V2{ix, iy}) + iz;
        float tB = r.soft ? cross(rb, V2{ix, iy}) : cross(rb, V2{ix, iy}) + iz;
        cA = {cA.x - mA * ix, cA.y - mA * iy};
        aA = aA - iA * tA;
        cB = {cB.x + mB * ix, cB.y + mB * iy};
        aB = aB + iB * tB;
        ok = pos_err <= s.linear_slop && ang_err <= s.angular_slop;
    }
    bd.cx[r.ia] = cA.x, bd.cy[r.ia] = cA.y, bd.ca[r.ia] = aA;
    bd.cx[r.ib] = cB.x, bd.cy[r.ib] = cB.y, bd.ca[r.ib] = aB;
    return ok;
}

}  // namespace gb
