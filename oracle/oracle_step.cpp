// Parity oracle (test infrastructure, see oracle.h): b2World::Step without SolveTOI, one world.
#include <algorithm>
#include <vector>

#include "oracle.h"

namespace orc {

// ---------------------------------------------------------------- pairs.py
static void wake(World &w, int b) {  // b2Body::SetAwake(true)
    if (!w.awake[b]) {
        w.awake[b] = 1;
        w.sleep_time[b] = 0.0f;
    }
}

// b2ContactManager::FindNewContacts (pairs.py:134-178)
void find_new_contacts(const Model &m, World &w) {
    const int P = m.P, C = w.C;
    if (P == 0) return;
    const int32_t *pa = m.d->pair_a, *pb = m.d->pair_b, *fbody = m.d->fixture_body;
    std::vector<uint8_t> exists(P, 0);
    for (int s = 0; s < C; ++s)
        if (w.pair[s] >= 0 && w.pair[s] < P) exists[w.pair[s]] = 1;
    std::vector<int> free_slots;
    for (int s = 0; s < C; ++s)
        if (w.pair[s] < 0) free_slots.push_back(s);
    const int n_free = (int)free_slots.size();
    int n_new = 0;
    std::vector<int> placed_b;
    for (int p = 0; p < P; ++p) {
        int ba = fbody[pa[p]], bb = fbody[pb[p]];
        if (!overlap(fixture_fat(m, w, pa[p]), fixture_fat(m, w, pb[p]))) continue;
        bool can = (w.type[ba] == DYNAMIC || w.type[bb] == DYNAMIC) && w.active[ba] && w.active[bb];
        if (!can || exists[p]) continue;
        int rank = n_new++;
        if (rank >= n_free) continue;
        int s = free_slots[rank];
        w.pair[s] = p;
        w.fa[s] = pa[p];
        w.fb[s] = pb[p];
        w.key[s] = *w.next_key + rank;
        w.touching[s] = 0;
        w.count[s] = 0;
        w.normal_impulse[2 * s] = w.normal_impulse[2 * s + 1] = 0.0f;
        w.tangent_impulse[2 * s] = w.tangent_impulse[2 * s + 1] = 0.0f;
        w.point_id[2 * s] = w.point_id[2 * s + 1] = 0;
        w.friction[s] = std::sqrt(fixture_friction(m, w, pa[p]) * fixture_friction(m, w, pb[p]));
        float ra = fixture_restitution(m, w, pa[p]), rb = fixture_restitution(m, w, pb[p]);
        w.restitution[s] = ra > rb ? ra : rb;
        w.tangent_speed[s] = 0.0f;
        placed_b.push_back(ba);
        placed_b.push_back(bb);
    }
    for (int b : placed_b) wake(w, b);  // AddPair wakes both bodies
    int n_placed = std::min(n_new, n_free);
    *w.next_key += n_new;
    *w.overflow += n_new - n_placed;
}

// Slots in contact-list order: live slots by descending key (Box2D's list is newest first)
static std::vector<int> list_order(const World &w) {
    std::vector<int> live;
    for (int s = 0; s < w.C; ++s)
        if (w.pair[s] >= 0) live.push_back(s);
    std::stable_sort(live.begin(), live.end(), [&](int x, int y) { return w.key[x] > w.key[y]; });
    return live;
}

// b2ContactManager::Collide (pairs.py:38-117); the fixed point of _active_in_list_order is the sequential walk
static void collide(const Model &m, World &w, const goib2d_settings &s) {
    const int C = w.C;
    const int32_t *fbody = m.d->fixture_body;
    std::vector<int> order = list_order(w);
    std::vector<uint8_t> aw(w.awake, w.awake + w.B);
    std::vector<uint8_t> active(C, 0), over(C, 0);
    std::vector<Manifold> man(C);
    for (int s_ : order) {
        int ba = fbody[w.fa[s_]], bb = fbody[w.fb[s_]];
        over[s_] = overlap(fixture_fat(m, w, w.fa[s_]), fixture_fat(m, w, w.fb[s_]));
        evaluate(m, w.fa[s_], w.fb[s_], w.bxf(ba), w.bxf(bb), s.linear_slop, s.angular_slop, &man[s_]);
    }
    for (int s_ : order) {
        int ba = fbody[w.fa[s_]], bb = fbody[w.fb[s_]];
        bool movA = w.type[ba] != STATIC, movB = w.type[bb] != STATIC;
        bool visit = (aw[ba] && movA) || (aw[bb] && movB);
        active[s_] = visit;
        bool touching_new = man[s_].count > 0;
        bool wakes = over[s_] ? (touching_new != (bool)w.touching[s_]) : (w.count[s_] > 0);
        if (visit && wakes) aw[ba] = aw[bb] = 1;
    }
    if (w.events) *w.event_count = 0;  // a new step's log
    for (int s_ : order) {
        if (!active[s_]) continue;
        if (!over[s_]) {  // destroy (EndContact when it was touching)
            if (w.touching[s_]) emit_event(w, EV_END, s_);
            w.pair[s_] = -1;
            w.touching[s_] = 0;
            w.count[s_] = 0;
            continue;
        }
        if ((man[s_].count > 0) != (bool)w.touching[s_]) emit_event(w, man[s_].count > 0 ? EV_BEGIN : EV_END, s_);
        const Manifold &mn = man[s_];
        int old_n = w.count[s_];
        float ni[2], ti[2];
        for (int i = 0; i < 2; ++i) {
            int32_t nid = mn.id[i];
            bool m0 = old_n > 0 && w.point_id[2 * s_] == nid;
            bool m1 = old_n > 1 && w.point_id[2 * s_ + 1] == nid && !m0;
            ni[i] = m0 ? w.normal_impulse[2 * s_] : m1 ? w.normal_impulse[2 * s_ + 1] : 0.0f;
            ti[i] = m0 ? w.tangent_impulse[2 * s_] : m1 ? w.tangent_impulse[2 * s_ + 1] : 0.0f;
            if (!(i < mn.count)) ni[i] = ti[i] = 0.0f;
        }
        w.touching[s_] = mn.count > 0;
        w.count[s_] = mn.count;
        if (mn.count > 0) {
            w.mtype[s_] = mn.mtype;
            w.local_normal[2 * s_] = mn.local_normal.x, w.local_normal[2 * s_ + 1] = mn.local_normal.y;
            w.local_point[2 * s_] = mn.local_point.x, w.local_point[2 * s_ + 1] = mn.local_point.y;
            for (int k = 0; k < 2; ++k) {
                w.point_local[4 * s_ + 2 * k] = mn.point[k].x;
                w.point_local[4 * s_ + 2 * k + 1] = mn.point[k].y;
                w.point_id[2 * s_ + k] = mn.id[k];
            }
        }
        for (int k = 0; k < 2; ++k) w.normal_impulse[2 * s_ + k] = ni[k], w.tangent_impulse[2 * s_ + k] = ti[k];
    }
    for (int b = 0; b < w.B; ++b) {
        if (aw[b] && !w.awake[b]) w.sleep_time[b] = 0.0f;
        w.awake[b] = aw[b];
    }
}

// ---------------------------------------------------------------- island.py
struct Islands {
    std::vector<int> corder, jorder;  // solve order
    std::vector<int> body_island, contact_island, joint_island;
    int n_islands = 0;
};

static void find_islands(const Model &m, World &w, Islands &isl) {
    const int B = w.B, C = w.C, J = w.J;
    const int32_t *fbody = m.d->fixture_body;
    isl.body_island.assign(B, -1);
    isl.contact_island.assign(C, -1);
    isl.joint_island.assign(J, -1);
    isl.corder.clear();
    isl.jorder.clear();
    // contact edges: live & touching slots, descending key
    std::vector<int> edges;
    for (int s = 0; s < C; ++s)
        if (w.pair[s] >= 0 && w.touching[s]) edges.push_back(s);
    std::stable_sort(edges.begin(), edges.end(), [&](int x, int y) { return w.key[x] > w.key[y]; });
    std::vector<uint8_t> flag(B, 0), cflag(C, 0), jflag(J, 0);
    std::vector<int> stack;
    for (;;) {
        if (stack.empty()) {
            int seed = -1;
            for (int b = B - 1; b >= 0; --b)
                if (w.active[b] && w.type[b] != STATIC && w.awake[b] && !flag[b]) {
                    seed = b;
                    break;
                }
            if (seed < 0) break;
            isl.n_islands++;
            stack.push_back(seed);
            flag[seed] = 1;
            continue;
        }
        int b = stack.back();
        stack.pop_back();
        int id = isl.n_islands - 1;
        for (int s : edges) {
            int ca = fbody[w.fa[s]], cb = fbody[w.fb[s]];
            if ((ca != b && cb != b) || cflag[s]) continue;
            isl.corder.push_back(s);
            isl.contact_island[s] = id;
            cflag[s] = 1;
            int other = ca == b ? cb : ca;
            if (!flag[other] && w.type[other] != STATIC) {
                stack.push_back(other);
                flag[other] = 1;
            }
        }
        for (int j = J - 1; j >= 0; --j) {
            int ja = m.d->joint_a[j], jb = m.d->joint_b[j];
            if ((ja != b && jb != b) || jflag[j]) continue;
            int other = ja == b ? jb : ja;
            if (!w.active[other]) continue;
            isl.jorder.push_back(j);
            isl.joint_island[j] = id;
            jflag[j] = 1;
            if (!flag[other] && w.type[other] != STATIC) {
                stack.push_back(other);
                flag[other] = 1;
            }
        }
        isl.body_island[b] = id;
        wake(w, b);
    }
}

// ---------------------------------------------------------------- contact_solver.py
struct VC {  // one velocity + position constraint (contact_solver.py:103-146)
    int slot, ia, ib;
    float mA, mB, iA, iB;
    V2 n;
    float friction, tangent_speed;
    int count, pc_count;
    V2 rA[2], rB[2];
    float nmass[2], tmass[2], bias[2];
    float ni[2], ti[2];
    float K[4], NM[4];
    int mtype;
    V2 ln, lp, pl[2], lcA, lcB;
    float radA, radB;
};

struct Pos {
    std::vector<float> cx, cy, a;
};
struct Vel {
    std::vector<float> vx, vy, w;
};

static inline Xf xf_of(float cx, float cy, Rot q, V2 lc) {  // contact_solver.py:20-29
    V2 r = rot(q, lc);
    return {{cx - r.x, cy - r.y}, q};
}

static void prepare_contacts(const Model &m, const World &w, const std::vector<int> &order, const Pos &pos,
                             const Vel &vel, const std::vector<Rot> &q, bool warm, float dt_ratio,
                             float velocity_threshold, std::vector<VC> &out) {
    // contact_solver.py:32-147
    const int32_t *fbody = m.d->fixture_body;
    out.resize(order.size());
    for (size_t k = 0; k < order.size(); ++k) {
        VC &c = out[k];
        int s = order[k];
        c.slot = s;
        int fa = w.fa[s], fb = w.fb[s];
        int ia = fbody[fa], ib = fbody[fb];
        c.ia = ia, c.ib = ib;
        c.mA = w.inv_mass[ia], c.mB = w.inv_mass[ib], c.iA = w.inv_inertia[ia], c.iB = w.inv_inertia[ib];
        c.lcA = {w.local_center[2 * ia], w.local_center[2 * ia + 1]};
        c.lcB = {w.local_center[2 * ib], w.local_center[2 * ib + 1]};
        float rA_ = m.d->radius[fa], rB_ = m.d->radius[fb];
        c.radA = rA_, c.radB = rB_;
        c.mtype = w.mtype[s];
        int count = w.count[s];
        c.ln = {w.local_normal[2 * s], w.local_normal[2 * s + 1]};
        c.lp = {w.local_point[2 * s], w.local_point[2 * s + 1]};
        for (int j = 0; j < 2; ++j) c.pl[j] = {w.point_local[4 * s + 2 * j], w.point_local[4 * s + 2 * j + 1]};
        for (int j = 0; j < 2; ++j) {
            c.ni[j] = warm ? dt_ratio * w.normal_impulse[2 * s + j] : 0.0f;
            c.ti[j] = warm ? dt_ratio * w.tangent_impulse[2 * s + j] : 0.0f;
        }
        V2 cA{pos.cx[ia], pos.cy[ia]}, cB{pos.cx[ib], pos.cy[ib]};
        Xf xfA = xf_of(cA.x, cA.y, q[ia], c.lcA), xfB = xf_of(cB.x, cB.y, q[ib], c.lcB);
        // b2WorldManifold::Initialize
        V2 nrm, pts[2];
        if (c.mtype == CIRCLES) {
            V2 pA = xf_mul(xfA, c.lp), pB = xf_mul(xfB, c.pl[0]);
            V2 d = sub(pB, pA);
            bool far = dot(d, d) > EPS * EPS;
            V2 nn = normalize(d);
            V2 cn = far ? nn : V2{1.0f, 0.0f};
            V2 ccA{pA.x + rA_ * cn.x, pA.y + rA_ * cn.y}, ccB{pB.x - rB_ * cn.x, pB.y - rB_ * cn.y};
            V2 cp{0.5f * (ccA.x + ccB.x), 0.5f * (ccA.y + ccB.y)};
            nrm = cn, pts[0] = pts[1] = cp;
        } else if (c.mtype == FACE_A) {
            V2 fn = rot(xfA.q, c.ln), fpl = xf_mul(xfA, c.lp);
            for (int j = 0; j < 2; ++j) {
                V2 qp = xf_mul(xfB, c.pl[j]);
                float d = dot(sub(qp, fpl), fn);
                float s_ = rA_ - d;
                V2 aA{qp.x + s_ * fn.x, qp.y + s_ * fn.y}, aB{qp.x - rB_ * fn.x, qp.y - rB_ * fn.y};
                pts[j] = {0.5f * (aA.x + aB.x), 0.5f * (aA.y + aB.y)};
            }
            nrm = fn;
        } else {
            V2 fn = rot(xfB.q, c.ln), fpl = xf_mul(xfB, c.lp);
            for (int j = 0; j < 2; ++j) {
                V2 qp = xf_mul(xfA, c.pl[j]);
                float d = dot(sub(qp, fpl), fn);
                float s_ = rB_ - d;
                V2 bB{qp.x + s_ * fn.x, qp.y + s_ * fn.y}, bA{qp.x - rA_ * fn.x, qp.y - rA_ * fn.y};
                pts[j] = {0.5f * (bA.x + bB.x), 0.5f * (bA.y + bB.y)};
            }
            nrm = neg(fn);
        }
        c.n = nrm;
        V2 t = cross_vs(nrm, 1.0f);
        V2 vA{vel.vx[ia], vel.vy[ia]}, vB{vel.vx[ib], vel.vy[ib]};
        float wA = vel.w[ia], wB = vel.w[ib];
        c.friction = w.friction[s], c.tangent_speed = w.tangent_speed[s];
        float restitution = w.restitution[s];
        for (int j = 0; j < 2; ++j) {
            V2 ra = sub(pts[j], cA), rb = sub(pts[j], cB);
            float rnA = cross(ra, nrm), rnB = cross(rb, nrm);
            float kn = ((c.mA + c.mB) + (c.iA * rnA) * rnA) + (c.iB * rnB) * rnB;
            float rtA = cross(ra, t), rtB = cross(rb, t);
            float kt = ((c.mA + c.mB) + (c.iA * rtA) * rtA) + (c.iB * rtB) * rtB;
            V2 wBr = cross_sv(wB, rb), wAr = cross_sv(wA, ra);
            float vrel = dot(nrm, V2{((vB.x + wBr.x) - vA.x) - wAr.x, ((vB.y + wBr.y) - vA.y) - wAr.y});
            c.rA[j] = ra, c.rB[j] = rb;
            c.nmass[j] = inv_if_pos(kn);
            c.tmass[j] = inv_if_pos(kt);
            c.bias[j] = vrel < -velocity_threshold ? -restitution * vrel : 0.0f;
        }
        float rn1A = cross(c.rA[0], nrm), rn1B = cross(c.rB[0], nrm);
        float rn2A = cross(c.rA[1], nrm), rn2B = cross(c.rB[1], nrm);
        float k11 = ((c.mA + c.mB) + (c.iA * rn1A) * rn1A) + (c.iB * rn1B) * rn1B;
        float k22 = ((c.mA + c.mB) + (c.iA * rn2A) * rn2A) + (c.iB * rn2B) * rn2B;
        float k12 = ((c.mA + c.mB) + (c.iA * rn1A) * rn2A) + (c.iB * rn1B) * rn2B;
        bool safe = k11 * k11 < MAX_COND * (k11 * k22 - k12 * k12);
        bool two = count == 2;
        c.count = (two && !safe) ? 1 : count;
        c.pc_count = count;
        float det = inv_or_zero(k11 * k22 - k12 * k12);
        bool use_k = two && safe;
        c.K[0] = use_k ? k11 : 0.0f, c.K[1] = use_k ? k12 : 0.0f, c.K[2] = use_k ? k12 : 0.0f,
        c.K[3] = use_k ? k22 : 0.0f;
        c.NM[0] = use_k ? det * k22 : 0.0f, c.NM[1] = use_k ? -det * k12 : 0.0f;
        c.NM[2] = use_k ? -det * k12 : 0.0f, c.NM[3] = use_k ? det * k11 : 0.0f;
    }
}

static void contact_warm_start(const std::vector<VC> &vc, Vel &vel) {  // contact_solver.py:165-184
    for (const VC &c : vc) {
        V2 vA{vel.vx[c.ia], vel.vy[c.ia]}, vB{vel.vx[c.ib], vel.vy[c.ib]};
        float wA = vel.w[c.ia], wB = vel.w[c.ib];
        V2 t = cross_vs(c.n, 1.0f);
        for (int j = 0; j < c.count; ++j) {
            V2 P{c.ni[j] * c.n.x + c.ti[j] * t.x, c.ni[j] * c.n.y + c.ti[j] * t.y};
            wA = wA - c.iA * cross(c.rA[j], P);
            vA = {vA.x - c.mA * P.x, vA.y - c.mA * P.y};
            wB = wB + c.iB * cross(c.rB[j], P);
            vB = {vB.x + c.mB * P.x, vB.y + c.mB * P.y};
        }
        vel.vx[c.ia] = vA.x, vel.vy[c.ia] = vA.y, vel.w[c.ia] = wA;
        vel.vx[c.ib] = vB.x, vel.vy[c.ib] = vB.y, vel.w[c.ib] = wB;
    }
}

static inline V2 dv(V2 vB, float wB, V2 rb, V2 vA, float wA, V2 ra) {  // vB + wB x rB - vA - wA x rA
    V2 b = cross_sv(wB, rb), a = cross_sv(wA, ra);
    return {((vB.x + b.x) - vA.x) - a.x, ((vB.y + b.y) - vA.y) - a.y};
}

static void contact_solve_velocity(std::vector<VC> &vcs, Vel &vel) {  // contact_solver.py:194-290
    for (VC &c : vcs) {
        V2 vA{vel.vx[c.ia], vel.vy[c.ia]}, vB{vel.vx[c.ib], vel.vy[c.ib]};
        float wA = vel.w[c.ia], wB = vel.w[c.ib];
        const float mA = c.mA, mB = c.mB, iA = c.iA, iB = c.iB;
        V2 n = c.n, t = cross_vs(n, 1.0f);
        for (int j = 0; j < c.count; ++j) {  // tangent constraints first
            V2 d = dv(vB, wB, c.rB[j], vA, wA, c.rA[j]);
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
            V2 d = dv(vB, wB, c.rB[0], vA, wA, c.rA[0]);
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
            V2 d1 = dv(vB, wB, c.rB[0], vA, wA, c.rA[0]);
            V2 d2 = dv(vB, wB, c.rB[1], vA, wA, c.rA[1]);
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
        vel.vx[c.ia] = vA.x, vel.vy[c.ia] = vA.y, vel.w[c.ia] = wA;
        vel.vx[c.ib] = vB.x, vel.vy[c.ib] = vB.y, vel.w[c.ib] = wB;
    }
}

// b2ContactSolver::SolvePositionConstraints for one contact (contact_solver.py:307-354)
static float contact_solve_position(const VC &c, Pos &pos, const goib2d_settings &s, float baumgarte, float mA,
                                    float mB, float iA, float iB) {
    V2 cA{pos.cx[c.ia], pos.cy[c.ia]}, cB{pos.cx[c.ib], pos.cy[c.ib]};
    float aA = pos.a[c.ia], aB = pos.a[c.ib];
    float min_sep = 0.0f;
    for (int j = 0; j < c.pc_count; ++j) {
        Xf xfA = xf_of(cA.x, cA.y, rot_of(aA), c.lcA), xfB = xf_of(cB.x, cB.y, rot_of(aB), c.lcB);
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
        float C_ = clampf(baumgarte * (sep + s.linear_slop), -s.max_linear_correction, 0.0f);
        float rnA = cross(ra, nrm), rnB = cross(rb, nrm);
        float K = ((mA + mB) + (iA * rnA) * rnA) + (iB * rnB) * rnB;
        float imp = K > 0 ? -C_ / K : 0.0f;
        V2 P{imp * nrm.x, imp * nrm.y};
        cA = {cA.x - mA * P.x, cA.y - mA * P.y};
        aA = aA - iA * cross(ra, P);
        cB = {cB.x + mB * P.x, cB.y + mB * P.y};
        aB = aB + iB * cross(rb, P);
    }
    pos.cx[c.ia] = cA.x, pos.cy[c.ia] = cA.y, pos.a[c.ia] = aA;
    pos.cx[c.ib] = cB.x, pos.cy[c.ib] = cB.y, pos.a[c.ib] = aB;
    return min_sep;
}

// ---------------------------------------------------------------- joints.py
struct JR {  // one joint row (joints.py:163-173)
    int jid, type, ia, ib;
    float mA, mB, iA, iB;
    V2 rA, rB;
    V3 Kx, Ky, Kz;
    float motor_mass;
    int limit_state;
    bool enable_motor, enable_limit;
    float motor_speed, max_impulse;
    V2 ax, pe;
    float a1, a2, s1, s2;
    bool soft;
    float gamma, bias, angle, inv_dt;
    V2 la, lb;
    float ref, lower, upper;
    V2 lx, ly;
    float imp[5];  // x, y, z, lower, upper
    float mimp;
};

static void k_rev(float mA, float mB, float iA, float iB, V2 rA, V2 rB, V3 *ex, V3 *ey, V3 *ez) {  // joints.py:39-47
    float exx = ((mA + mB) + (rA.y * rA.y) * iA) + (rB.y * rB.y) * iB;
    float eyx = (-rA.y * rA.x) * iA - (rB.y * rB.x) * iB;
    float ezx = -rA.y * iA - rB.y * iB;
    float eyy = ((mA + mB) + (rA.x * rA.x) * iA) + (rB.x * rB.x) * iB;
    float ezy = rA.x * iA + rB.x * iB;
    float ezz = iA + iB;
    *ex = {exx, eyx, ezx}, *ey = {eyx, eyy, ezy}, *ez = {ezx, ezy, ezz};
}

static void k_prism(float mA, float mB, float iA, float iB, float s1, float s2, float a1, float a2, V3 *ex, V3 *ey,
                    V3 *ez) {  // joints.py:50-58
    float k11 = ((mA + mB) + (iA * s1) * s1) + (iB * s2) * s2;
    float k12 = iA * s1 + iB * s2;
    float k13 = (iA * s1) * a1 + (iB * s2) * a2;
    float k22 = iA + iB;
    if (k22 == 0) k22 = 1.0f;
    float k23 = iA * a1 + iB * a2;
    float k33 = ((mA + mB) + (iA * a1) * a1) + (iB * a2) * a2;
    *ex = {k11, k12, k13}, *ey = {k12, k22, k23}, *ez = {k13, k23, k33};
}

static const float TWO_PI = 2.0f * PI_F;

static void prepare_joints(const Model &m, const World &w, const std::vector<int> &order, const Pos &pos,
                           const std::vector<Rot> &q, const goib2d_settings &s, float dt, float dt_ratio, bool warm,
                           std::vector<JR> &out) {
    // joints.py:61-174
    const bool v24 = s.revolute_v24;
    out.resize(order.size());
    for (size_t k = 0; k < order.size(); ++k) {
        JR &r = out[k];
        int jid = order[k];
        r.jid = jid;
        r.type = m.d->joint_type[jid];
        int ia = m.d->joint_a[jid], ib = m.d->joint_b[jid];
        r.ia = ia, r.ib = ib;
        float mA = w.inv_mass[ia], mB = w.inv_mass[ib], iA = w.inv_inertia[ia], iB = w.inv_inertia[ib];
        r.mA = mA, r.mB = mB, r.iA = iA, r.iB = iB;
        float lcAx = w.local_center[2 * ia], lcAy = w.local_center[2 * ia + 1];
        float lcBx = w.local_center[2 * ib], lcBy = w.local_center[2 * ib + 1];
        V2 cA{pos.cx[ia], pos.cy[ia]}, cB{pos.cx[ib], pos.cy[ib]};
        float aA = pos.a[ia], aB = pos.a[ib];
        Rot qA = q[ia], qB = q[ib];
        V2 la{m.d->local_anchor_a[2 * jid] - lcAx, m.d->local_anchor_a[2 * jid + 1] - lcAy};
        V2 lb{m.d->local_anchor_b[2 * jid] - lcBx, m.d->local_anchor_b[2 * jid + 1] - lcBy};
        V2 rA = rot(qA, la), rB = rot(qB, lb);
        r.rA = rA, r.rB = rB, r.la = la, r.lb = lb;
        float ref = m.d->reference_angle[jid];
        r.ref = ref;
        bool en_motor = w.enable_motor[jid], en_limit = w.enable_limit[jid];
        float lower = w.lower[jid], upper = w.upper[jid];
        int state_in = w.limit_state[jid];
        float ix = w.impulse[3 * jid], iy = w.impulse[3 * jid + 1], iz = w.impulse[3 * jid + 2];
        float mimp = w.motor_impulse[jid];
        bool is_rev = r.type == REVOLUTE, is_pri = r.type == PRISMATIC;
        // revolute
        V3 revx, revy, revz;
        k_rev(mA, mB, iA, iB, rA, rB, &revx, &revy, &revz);
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
        // prismatic
        float dx = ((cB.x - cA.x) + rB.x) - rA.x, dy = ((cB.y - cA.y) + rB.y) - rA.y;
        V2 lxa{m.d->local_axis_a[2 * jid], m.d->local_axis_a[2 * jid + 1]};
        V2 lya{m.d->local_yaxis_a[2 * jid], m.d->local_yaxis_a[2 * jid + 1]};
        r.lx = lxa, r.ly = lya;
        V2 ax = rot(qA, lxa);
        float a1 = cross(V2{dx + rA.x, dy + rA.y}, ax), a2 = cross(rB, ax);
        float pri_mm = ((mA + mB) + (iA * a1) * a1) + (iB * a2) * a2;
        pri_mm = pri_mm > 0 ? 1.0f / pri_mm : pri_mm;
        V2 pe = rot(qA, lya);
        float s1 = cross(V2{dx + rA.x, dy + rA.y}, pe), s2 = cross(rB, pe);
        V3 prx, pry, prz;
        k_prism(mA, mB, iA, iB, s1, s2, a1, a2, &prx, &pry, &prz);
        float trans = dot(ax, V2{dx, dy});
        bool pequal = babs(upper - lower) < 2.0f * s.linear_slop;
        int pri_state = !en_limit ? INACTIVE_LIMIT
                        : pequal ? EQUAL_LIMITS
                        : trans <= lower ? AT_LOWER
                        : trans >= upper ? AT_UPPER
                                         : INACTIVE_LIMIT;
        bool pri_zero_z = !en_limit || (!pequal && (pri_state == INACTIVE_LIMIT || pri_state != state_in));
        float pri_mimp = en_motor ? mimp : 0.0f;
        // weld
        bool soft = w.frequency[jid] > 0;
        V3 i22x, i22y, i22z, symx, symy, symz;
        inverse22_of33(revx, revy, &i22x, &i22y, &i22z);
        sym_inverse33(revx, revy, revz, &symx, &symy, &symz);
        float invM = iA + iB;
        float wm = inv_if_pos(invM);
        float C = (aB - aA) - ref;
        float omega = TWO_PI * w.frequency[jid];
        float d = ((2.0f * wm) * w.damping[jid]) * omega;
        float kk = (wm * omega) * omega;
        float h = dt;
        float gamma = inv_or_zero(h * (d + h * kk));
        float bias = ((C * h) * kk) * gamma;
        float ezz_soft = inv_or_zero(invM + gamma);
        bool use22 = soft || revz.z == 0;
        V3 wmx = use22 ? i22x : symx, wmy = use22 ? i22y : symy, wmz = use22 ? i22z : symz;
        if (soft) wmz.z = ezz_soft;
        float w_gamma = soft ? gamma : 0.0f, w_bias = soft ? bias : 0.0f;
        const bool is_mot = r.type == MOTOR;
        if (is_rev || is_mot)
            r.Kx = revx, r.Ky = revy, r.Kz = revz;
        else if (is_pri)
            r.Kx = prx, r.Ky = pry, r.Kz = prz;
        else
            r.Kx = wmx, r.Ky = wmy, r.Kz = wmz;
        r.limit_state = is_rev ? rev_state : is_pri ? pri_state : INACTIVE_LIMIT;
        bool zero_z = is_rev ? (v24 ? false : rev_zero_z) : is_pri ? pri_zero_z : false;
        if (zero_z) iz = 0.0f;
        mimp = is_rev ? rev_mimp : is_pri ? pri_mimp : 0.0f;
        auto sc = [&](float x) { return warm ? x * dt_ratio : 0.0f; };
        if (v24) {
            float lo = (is_rev && lim_on) ? w.lower_impulse[jid] : 0.0f;
            float up = (is_rev && lim_on) ? w.upper_impulse[jid] : 0.0f;
            r.imp[0] = sc(ix), r.imp[1] = sc(iy), r.imp[2] = is_rev ? iz : sc(iz), r.imp[3] = sc(lo), r.imp[4] = sc(up);
        } else {
            r.imp[0] = sc(ix), r.imp[1] = sc(iy), r.imp[2] = sc(iz), r.imp[3] = 0.0f, r.imp[4] = 0.0f;
        }
        r.mimp = sc(mimp);
        r.inv_dt = dt > 0 ? 1.0f / dt : 0.0f;
        r.motor_mass = is_rev ? rev_mm : is_pri ? pri_mm : 0.0f;
        r.enable_motor = en_motor, r.enable_limit = en_limit;
        r.motor_speed = w.motor_speed[jid];
        r.max_impulse = dt * w.max_motor[jid];
        r.ax = ax, r.pe = pe, r.a1 = a1, r.a2 = a2, r.s1 = s1, r.s2 = s2;
        r.soft = soft, r.gamma = w_gamma, r.bias = w_bias, r.angle = angle;
        r.lower = lower, r.upper = upper;
        if (is_mot) {  // b2MotorJoint::InitVelocityConstraints; the joint row holds its parameters (see motor_velocity)
            const float lin_x = lower, lin_y = upper, ang_off = w.motor_speed[jid];
            const V2 ro = rot(qA, V2{lin_x, lin_y});
            r.ax = {(((cB.x + rB.x) - cA.x) - rA.x) - ro.x, (((cB.y + rB.y) - cA.y) - rA.y) - ro.y};
            r.angle = (aB - aA) - ang_off;
            r.motor_mass = rev_mm;
            r.gamma = dt * w.frequency[jid];  // the linear impulse's limit, h * max force
            r.bias = w.damping[jid];          // the correction factor
            r.soft = false;
        }
    }
}

static void joint_warm_start(const std::vector<JR> &rows, Vel &vel, bool v24) {  // joints.py:202-248
    for (const JR &r : rows) {
        V2 vA{vel.vx[r.ia], vel.vy[r.ia]}, vB{vel.vx[r.ib], vel.vy[r.ib]};
        float wA = vel.w[r.ia], wB = vel.w[r.ib];
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
        vel.vx[r.ia] = vA.x, vel.vy[r.ia] = vA.y, vel.w[r.ia] = wA;
        vel.vx[r.ib] = vB.x, vel.vy[r.ib] = vB.y, vel.w[r.ib] = wB;
    }
}

static void rev_velocity(JR &r, V2 &vA, float &wA, V2 &vB, float &wB) {  // joints.py:257-299 (2.3.1)
    const float mA = r.mA, mB = r.mB, iA = r.iA, iB = r.iB;
    V3 ex = r.Kx, ey = r.Ky, ez = r.Kz;
    bool fixed = (iA + iB) == 0;
    int st = r.limit_state;
    bool on = r.enable_motor && st != EQUAL_LIMITS && !fixed;
    float mi = r.mimp;
    {
        float cdot = (wB - wA) - r.motor_speed;
        float impulse = -r.motor_mass * cdot;
        float nmi = clampf(mi + impulse, -r.max_impulse, r.max_impulse);
        impulse = nmi - mi;
        if (on) {
            wA = wA - iA * impulse;
            wB = wB + iB * impulse;
            r.mimp = nmi;
        }
    }
    float ix = r.imp[0], iy = r.imp[1], iz = r.imp[2];
    V2 c1 = dv(vB, wB, r.rB, vA, wA, r.rA);
    bool lim = r.enable_limit && st != INACTIVE_LIMIT && !fixed;
    if (lim) {
        float c2 = wB - wA;
        V3 sv = solve33(ex, ey, ez, V3{c1.x, c1.y, c2});
        float jx = -sv.x, jy = -sv.y, jz = -sv.z;
        float new_z = iz + jz;
        bool redo = (st == AT_LOWER && new_z < 0) || (st == AT_UPPER && new_z > 0);
        V2 rr = solve22(ex.x, ey.x, ex.y, ey.y, -c1.x + iz * ez.x, -c1.y + iz * ez.y);
        float lx = redo ? rr.x : jx, ly = redo ? rr.y : jy, lz = redo ? -iz : jz;
        float nix = redo ? ix + rr.x : ix + jx, niy = redo ? iy + rr.y : iy + jy, niz = redo ? 0.0f : iz + jz;
        vA = {vA.x - mA * lx, vA.y - mA * ly};
        wA = wA - iA * (cross(r.rA, V2{lx, ly}) + lz);
        vB = {vB.x + mB * lx, vB.y + mB * ly};
        wB = wB + iB * (cross(r.rB, V2{lx, ly}) + lz);
        r.imp[0] = nix, r.imp[1] = niy, r.imp[2] = niz;
    } else {
        V2 p = solve22(ex.x, ey.x, ex.y, ey.y, -c1.x, -c1.y);
        vA = {vA.x - mA * p.x, vA.y - mA * p.y};
        wA = wA - iA * cross(r.rA, p);
        vB = {vB.x + mB * p.x, vB.y + mB * p.y};
        wB = wB + iB * cross(r.rB, p);
        r.imp[0] = ix + p.x, r.imp[1] = iy + p.y;
    }
}

static void rev24_velocity(JR &r, V2 &vA, float &wA, V2 &vB, float &wB) {  // joints.py:302-343
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
        if (on) {
            wA = wA - iA * impulse;
            wB = wB + iB * impulse;
            r.mimp = nmi;
        }
    }
    bool lim = r.enable_limit && !fixed;
    {
        float C = r.angle - r.lower;
        float impulse = -am * ((wB - wA) + bmax(C, 0.0f) * r.inv_dt);
        float nlo = bmax(r.imp[3] + impulse, 0.0f);
        impulse = nlo - r.imp[3];
        if (lim) {
            wA = wA - iA * impulse;
            wB = wB + iB * impulse;
            r.imp[3] = nlo;
        }
    }
    {
        float C = r.upper - r.angle;
        float impulse = -am * ((wA - wB) + bmax(C, 0.0f) * r.inv_dt);
        float nup = bmax(r.imp[4] + impulse, 0.0f);
        impulse = nup - r.imp[4];
        if (lim) {
            wA = wA + iA * impulse;
            wB = wB - iB * impulse;
            r.imp[4] = nup;
        }
    }
    V2 c1 = dv(vB, wB, r.rB, vA, wA, r.rA);
    V2 p = solve22(ex.x, ey.x, ex.y, ey.y, -c1.x, -c1.y);
    vA = {vA.x - mA * p.x, vA.y - mA * p.y};
    wA = wA - iA * cross(r.rA, p);
    vB = {vB.x + mB * p.x, vB.y + mB * p.y};
    wB = wB + iB * cross(r.rB, p);
    r.imp[0] = r.imp[0] + p.x, r.imp[1] = r.imp[1] + p.y;
}

static void pri_velocity(JR &r, V2 &vA, float &wA, V2 &vB, float &wB) {  // joints.py:354-404
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
        V3 df = solve33(ex, ey, ez, V3{-c1x, -c1y, -c2});
        float nx_ = ix + df.x, ny_ = iy + df.y, nz_ = iz + df.z;
        (void)nx_, (void)ny_;
        nz_ = st == AT_LOWER ? bmax(nz_, 0.0f) : st == AT_UPPER ? bmin(nz_, 0.0f) : nz_;
        float bx = -c1x - (nz_ - iz) * ez.x;
        float by = -c1y - (nz_ - iz) * ez.y;
        V2 f = solve22(ex.x, ey.x, ex.y, ey.y, bx, by);
        float fx = f.x + ix, fy = f.y + iy;
        float dfx = fx - ix, dfy = fy - iy, dfz = nz_ - iz;
        Px = dfx * pe.x + dfz * ax.x;
        Py = dfx * pe.y + dfz * ax.y;
        LA = (dfx * s1 + dfy) + dfz * a1;
        LB = (dfx * s2 + dfy) + dfz * a2;
        r.imp[0] = fx, r.imp[1] = fy, r.imp[2] = nz_;
    } else {
        V2 g = solve22(ex.x, ey.x, ex.y, ey.y, -c1x, -c1y);
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

static void weld_velocity(JR &r, V2 &vA, float &wA, V2 &vB, float &wB) {  // joints.py:407-437
    const float mA = r.mA, mB = r.mB, iA = r.iA, iB = r.iB;
    V3 ex = r.Kx, ey = r.Ky, ez = r.Kz;
    float ix = r.imp[0], iy = r.imp[1], iz = r.imp[2];
    if (r.soft) {
        float c2 = wB - wA;
        float i2 = -ez.z * ((c2 + r.bias) + r.gamma * iz);
        float s_iz = iz + i2;
        float swA = wA - iA * i2, swB = wB + iB * i2;
        V2 c1 = dv(vB, swB, r.rB, vA, swA, r.rA);
        V2 qv = mat33_mul22(ex, ey, c1);
        float i1x = -qv.x, i1y = -qv.y;
        vA = {vA.x - mA * i1x, vA.y - mA * i1y};
        wA = swA - iA * cross(r.rA, V2{i1x, i1y});
        vB = {vB.x + mB * i1x, vB.y + mB * i1y};
        wB = swB + iB * cross(r.rB, V2{i1x, i1y});
        r.imp[0] = ix + i1x, r.imp[1] = iy + i1y, r.imp[2] = s_iz;
    } else {
        V2 d1 = dv(vB, wB, r.rB, vA, wA, r.rA);
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
// linear y, angular).
static void motor_velocity(JR &r, V2 &vA, float &wA, V2 &vB, float &wB) {
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
    const V2 b = cross_sv(wB, r.rB), a = cross_sv(wA, r.rA);
    const float dx = ((vB.x + b.x) - vA.x) - a.x, dy = ((vB.y + b.y) - vA.y) - a.y;
    const float cx = dx + k * r.ax.x, cy = dy + k * r.ax.y;
    const V2 sv = solve22(r.Kx.x, r.Ky.x, r.Kx.y, r.Ky.y, cx, cy);
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

static void joint_solve_velocity(std::vector<JR> &rows, Vel &vel, bool v24) {  // joints.py:440-459
    for (JR &r : rows) {
        V2 vA{vel.vx[r.ia], vel.vy[r.ia]}, vB{vel.vx[r.ib], vel.vy[r.ib]};
        float wA = vel.w[r.ia], wB = vel.w[r.ib];
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
        vel.vx[r.ia] = vA.x, vel.vy[r.ia] = vA.y, vel.w[r.ia] = wA;
        vel.vx[r.ib] = vB.x, vel.vy[r.ib] = vB.y, vel.w[r.ib] = wB;
    }
}

// the point-to-point part of the revolute position solve (joints.py:501-520)
static bool rev_point_position(const JR &r, V2 &cA, float &aA, V2 &cB, float &aB, const goib2d_settings &s,
                               float ang_err) {
    const float mA = r.mA, mB = r.mB, iA = r.iA, iB = r.iB;
    Rot qA = rot_of(aA), qB = rot_of(aB);
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

static bool rev_position(const JR &r, V2 &cA, float &aA, V2 &cB, float &aB, const goib2d_settings &s) {
    // joints.py:462-479 (2.3.1)
    const float iA = r.iA, iB = r.iB;
    bool fixed = (iA + iB) == 0;
    int st = r.limit_state;
    bool lim = r.enable_limit && st != INACTIVE_LIMIT && !fixed;
    float angle = (aB - aA) - r.ref;
    float mac = s.max_angular_correction;
    float ce = clampf(angle - r.lower, -mac, mac);
    float cl = angle - r.lower, cu = angle - r.upper;
    float C = st == EQUAL_LIMITS ? ce
              : st == AT_LOWER   ? clampf(cl + s.angular_slop, -mac, 0.0f)
                                 : clampf(cu - s.angular_slop, 0.0f, mac);
    float ang_err = st == EQUAL_LIMITS ? babs(ce) : st == AT_LOWER ? -cl : cu;
    float limit_impulse = -r.motor_mass * C;
    if (lim) {
        aA = aA - iA * limit_impulse;
        aB = aB + iB * limit_impulse;
    }
    if (!lim) ang_err = 0.0f;
    return rev_point_position(r, cA, aA, cB, aB, s, ang_err);
}

static bool rev24_position(const JR &r, V2 &cA, float &aA, V2 &cB, float &aB, const goib2d_settings &s) {
    // joints.py:482-498
    const float iA = r.iA, iB = r.iB;
    bool fixed = (iA + iB) == 0;
    bool lim = r.enable_limit && !fixed;
    float angle = (aB - aA) - r.ref;
    float lower = r.lower, upper = r.upper;
    float mac = s.max_angular_correction;
    bool equal = babs(upper - lower) < 2.0f * s.angular_slop;
    float C = equal             ? clampf(angle - lower, -mac, mac)
              : angle <= lower ? clampf((angle - lower) + s.angular_slop, -mac, 0.0f)
              : angle >= upper ? clampf((angle - upper) - s.angular_slop, 0.0f, mac)
                               : 0.0f;
    float limit_impulse = -r.motor_mass * C;
    if (lim) {
        aA = aA - iA * limit_impulse;
        aB = aB + iB * limit_impulse;
    }
    float ang_err = lim ? babs(C) : 0.0f;
    return rev_point_position(r, cA, aA, cB, aB, s, ang_err);
}

static bool pri_position(const JR &r, V2 &cA, float &aA, V2 &cB, float &aB, const goib2d_settings &s) {
    // joints.py:523-566
    const float mA = r.mA, mB = r.mB, iA = r.iA, iB = r.iB;
    Rot qA = rot_of(aA), qB = rot_of(aB);
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
    float c2 = eq ? clampf(t, -mlc, mlc)
               : at_lo ? clampf((t - lo) + s.linear_slop, -mlc, 0.0f)
                       : clampf((t - hi) - s.linear_slop, 0.0f, mlc);
    float e2 = eq ? babs(t) : at_lo ? lo - t : t - hi;
    if (active) lin_err = bmax(lin_err, e2);
    V3 ex, ey, ez;
    k_prism(mA, mB, iA, iB, s1, s2, a1, a2, &ex, &ey, &ez);
    float ix, iy, iz;
    if (active) {
        V3 i3 = solve33(ex, ey, ez, V3{-c1x, -c1y, -c2});
        ix = i3.x, iy = i3.y, iz = i3.z;
    } else {
        float k11 = ex.x, k12 = ex.y, k22 = ey.y;
        V2 g = solve22(k11, k12, k12, k22, -c1x, -c1y);
        ix = g.x, iy = g.y, iz = 0.0f;
    }
    float Px = ix * pe.x + iz * ax.x, Py = ix * pe.y + iz * ax.y;
    float LA = (ix * s1 + iy) + iz * a1, LB = (ix * s2 + iy) + iz * a2;
    cA = {cA.x - mA * Px, cA.y - mA * Py};
    aA = aA - iA * LA;
    cB = {cB.x + mB * Px, cB.y + mB * Py};
    aB = aB + iB * LB;
    return lin_err <= s.linear_slop && ang_err <= s.angular_slop;
}

static bool weld_position(const JR &r, V2 &cA, float &aA, V2 &cB, float &aB, const goib2d_settings &s) {
    // joints.py:569-595
    const float mA = r.mA, mB = r.mB, iA = r.iA, iB = r.iB;
    Rot qA = rot_of(aA), qB = rot_of(aB);
    V2 ra = rot(qA, r.la), rb = rot(qB, r.lb);
    V3 ex, ey, ez;
    k_rev(mA, mB, iA, iB, ra, rb, &ex, &ey, &ez);
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
    return pos_err <= s.linear_slop && ang_err <= s.angular_slop;
}

static bool joint_solve_position(const JR &r, Pos &pos, const goib2d_settings &s) {  // joints.py:598-606
    if (r.type == MOTOR) return true;  // b2MotorJoint::SolvePositionConstraints corrects nothing
    V2 cA{pos.cx[r.ia], pos.cy[r.ia]}, cB{pos.cx[r.ib], pos.cy[r.ib]};
    float aA = pos.a[r.ia], aB = pos.a[r.ib];
    bool ok;
    if (r.type == REVOLUTE)
        ok = s.revolute_v24 ? rev24_position(r, cA, aA, cB, aB, s) : rev_position(r, cA, aA, cB, aB, s);
    else if (r.type == PRISMATIC)
        ok = pri_position(r, cA, aA, cB, aB, s);
    else
        ok = weld_position(r, cA, aA, cB, aB, s);
    pos.cx[r.ia] = cA.x, pos.cy[r.ia] = cA.y, pos.a[r.ia] = aA;
    pos.cx[r.ib] = cB.x, pos.cy[r.ib] = cB.y, pos.a[r.ib] = aB;
    return ok;
}

// ---------------------------------------------------------------- pairs.py:181-207
void synchronize_fixtures(const Model &m, World &w, const uint8_t *moved) {
    for (int f = 0; f < m.F; ++f) {
        int row = fixture_row(m, f);
        if (row < 0) continue;
        int b = m.d->fixture_body[f];
        if (!moved[b]) continue;
        Rot q1 = rot_of(w.a0[b]);
        V2 lc{w.local_center[2 * b], w.local_center[2 * b + 1]};
        V2 r = rot(q1, lc);
        V2 p1{w.c0[2 * b] - r.x, w.c0[2 * b + 1] - r.y};
        AABB a1 = fixture_aabb(m, f, Xf{p1, q1});
        AABB a2 = fixture_aabb(m, f, w.bxf(b));
        float lx = bmin(a1.lx, a2.lx), ly = bmin(a1.ly, a2.ly), ux = bmax(a1.ux, a2.ux), uy = bmax(a1.uy, a2.uy);
        float dx = w.xf_p[2 * b] - p1.x, dy = w.xf_p[2 * b + 1] - p1.y;
        float *old = w.fx_fat + 4 * row;
        bool contains = old[0] <= lx && old[1] <= ly && ux <= old[2] && uy <= old[3];
        if (contains) continue;
        lx = lx - AABB_EXT, ly = ly - AABB_EXT, ux = ux + AABB_EXT, uy = uy + AABB_EXT;
        float ddx = AABB_MUL * dx, ddy = AABB_MUL * dy;
        if (ddx < 0)
            lx = lx + ddx;
        else
            ux = ux + ddx;
        if (ddy < 0)
            ly = ly + ddy;
        else
            uy = uy + ddy;
        old[0] = lx, old[1] = ly, old[2] = ux, old[3] = uy;
    }
}

// ---------------------------------------------------------------- step.py:73-251
static void solve(const Model &m, World &w, const goib2d_settings &s, float dt, float inv_dt, float dt_ratio) {
    (void)inv_dt;
    const int B = w.B;
    Islands isl;
    find_islands(m, w, isl);
    const float h = dt;
    std::vector<uint8_t> in_isl(B);
    for (int b = 0; b < B; ++b) in_isl[b] = isl.body_island[b] >= 0;
    Vel vel{std::vector<float>(B), std::vector<float>(B), std::vector<float>(B)};
    Pos pos{std::vector<float>(B), std::vector<float>(B), std::vector<float>(B)};
    const float gx = w.gravity[0], gy = w.gravity[1];
    for (int b = 0; b < B; ++b) {  // integrate velocities (step.py:83-96)
        float gs = w.gravity_scale[b];
        float ax = gs * gx + w.inv_mass[b] * w.force[2 * b];
        float ay = gs * gy + w.inv_mass[b] * w.force[2 * b + 1];
        float vx = w.v[2 * b] + h * ax, vy = w.v[2 * b + 1] + h * ay;
        float ww = w.w[b] + (h * w.inv_inertia[b]) * w.torque[b];
        float ld = 1.0f / (1.0f + h * w.linear_damping[b]);
        float ad = 1.0f / (1.0f + h * w.angular_damping[b]);
        vx = vx * ld, vy = vy * ld, ww = ww * ad;
        bool dyn = in_isl[b] && w.type[b] == DYNAMIC;
        vel.vx[b] = dyn ? vx : w.v[2 * b];
        vel.vy[b] = dyn ? vy : w.v[2 * b + 1];
        vel.w[b] = dyn ? ww : w.w[b];
        pos.cx[b] = w.c[2 * b], pos.cy[b] = w.c[2 * b + 1], pos.a[b] = w.a[b];
        if (in_isl[b]) {
            w.c0[2 * b] = w.c[2 * b], w.c0[2 * b + 1] = w.c[2 * b + 1];
            w.a0[b] = w.a[b];
        }
    }
    std::vector<Rot> q(B);
    for (int b = 0; b < B; ++b) q[b] = rot_of(pos.a[b]);
    const bool warm = s.warm_starting;
    std::vector<VC> vc;
    prepare_contacts(m, w, isl.corder, pos, vel, q, warm, dt_ratio, s.velocity_threshold, vc);
    if (warm) contact_warm_start(vc, vel);
    std::vector<JR> jr;
    prepare_joints(m, w, isl.jorder, pos, q, s, dt, dt_ratio, warm, jr);
    joint_warm_start(jr, vel, s.revolute_v24);
    for (int it = 0; it < s.velocity_iterations; ++it) {
        joint_solve_velocity(jr, vel, s.revolute_v24);
        contact_solve_velocity(vc, vel);
    }
    for (const VC &c : vc)  // store impulses (contact_solver.py:293-304)
        for (int j = 0; j < c.count; ++j) {
            w.normal_impulse[2 * c.slot + j] = c.ni[j];
            w.tangent_impulse[2 * c.slot + j] = c.ti[j];
        }
    for (const VC &c : vc) emit_event(w, EV_POST_SOLVE, c.slot, c.count, c.ni, c.ti);  // b2Island::Report
    for (const JR &r : jr) {  // joints.py:609-622
        if (s.revolute_v24) w.lower_impulse[r.jid] = r.imp[3], w.upper_impulse[r.jid] = r.imp[4];
        for (int k = 0; k < 3; ++k) w.impulse[3 * r.jid + k] = r.imp[k];
        w.motor_impulse[r.jid] = r.mimp;
        w.limit_state[r.jid] = r.limit_state;
    }
    // integrate positions (step.py:120-135)
    float max_t = s.clamps_per_second ? s.max_translation * h : s.max_translation;
    float max_r = s.clamps_per_second ? s.max_rotation * h : s.max_rotation;
    for (int b = 0; b < B; ++b) {
        if (!in_isl[b]) continue;
        float vx = vel.vx[b], vy = vel.vy[b], ww = vel.w[b];
        float tx = h * vx, ty = h * vy;
        if (tx * tx + ty * ty > max_t * max_t) {
            float ratio = max_t / length(V2{tx, ty});
            vx = vx * ratio, vy = vy * ratio;
        }
        float rt = h * ww;
        if (rt * rt > max_r * max_r) {
            float rr = max_r / babs(rt);
            ww = ww * rr;
        }
        pos.cx[b] = pos.cx[b] + h * vx, pos.cy[b] = pos.cy[b] + h * vy, pos.a[b] = pos.a[b] + h * ww;
        vel.vx[b] = vx, vel.vy[b] = vy, vel.w[b] = ww;
    }
    // position iterations with per-island early exit (step.py:197-251)
    const int NI = isl.n_islands;
    std::vector<uint8_t> done(B, 0);
    for (int i = 0; i < B; ++i) done[i] = i >= NI;
    auto all_done = [&]() {
        for (int i = 0; i < B; ++i)
            if (!done[i]) return false;
        return true;
    };
    for (int it = 0; it < s.position_iterations && !all_done(); ++it) {
        std::vector<float> min_sep(B, 0.0f);
        std::vector<uint8_t> jok(B, 1);
        for (const VC &c : vc) {
            int i = isl.contact_island[c.slot];
            if (done[i]) continue;
            float ms = contact_solve_position(c, pos, s, s.baumgarte, c.mA, c.mB, c.iA, c.iB);
            min_sep[i] = bmin(min_sep[i], ms);
        }
        for (const JR &r : jr) {
            int i = isl.joint_island[r.jid];
            if (done[i]) continue;
            bool ok = joint_solve_position(r, pos, s);
            jok[i] = jok[i] && ok;
        }
        for (int i = 0; i < B; ++i)
            if (min_sep[i] >= -3.0f * s.linear_slop && jok[i]) done[i] = 1;
    }
    // write back + SynchronizeTransform (step.py:141-151)
    for (int b = 0; b < B; ++b) {
        if (!in_isl[b]) continue;
        w.c[2 * b] = pos.cx[b], w.c[2 * b + 1] = pos.cy[b], w.a[b] = pos.a[b];
        w.v[2 * b] = vel.vx[b], w.v[2 * b + 1] = vel.vy[b], w.w[b] = vel.w[b];
        Rot qq = rot_of(w.a[b]);
        V2 r = rot(qq, V2{w.local_center[2 * b], w.local_center[2 * b + 1]});
        w.xf_p[2 * b] = w.c[2 * b] - r.x, w.xf_p[2 * b + 1] = w.c[2 * b + 1] - r.y;
        w.xf_q[2 * b] = qq.c, w.xf_q[2 * b + 1] = qq.s;
    }
    // sleep, per island (step.py:153-171)
    std::vector<uint8_t> isl_sleep(B, 0);
    if (s.allow_sleep) {
        float lin_tol = s.linear_sleep_tolerance * s.linear_sleep_tolerance;
        float ang_tol = s.angular_sleep_tolerance * s.angular_sleep_tolerance;
        std::vector<float> min_st(B, MAXF), st(B);
        std::vector<uint8_t> nonstatic(B);
        for (int b = 0; b < B; ++b) {
            nonstatic[b] = in_isl[b] && w.type[b] != STATIC;
            bool moving = !w.allow_sleep[b] || (w.w[b] * w.w[b] > ang_tol) ||
                          (w.v[2 * b] * w.v[2 * b] + w.v[2 * b + 1] * w.v[2 * b + 1] > lin_tol);
            float t = moving ? 0.0f : w.sleep_time[b] + h;
            st[b] = nonstatic[b] ? t : w.sleep_time[b];
            if (nonstatic[b]) {
                int i = isl.body_island[b];
                float v = moving ? 0.0f : st[b];
                min_st[i] = std::fmin(min_st[i], v);
            }
        }
        for (int i = 0; i < B; ++i) isl_sleep[i] = min_st[i] >= s.time_to_sleep && done[i];
        for (int b = 0; b < B; ++b) {
            bool sl = nonstatic[b] && isl_sleep[isl.body_island[b]];
            w.sleep_time[b] = sl ? 0.0f : st[b];
            if (sl) {
                w.awake[b] = 0;
                w.v[2 * b] = w.v[2 * b + 1] = 0.0f, w.w[b] = 0.0f;
                w.force[2 * b] = w.force[2 * b + 1] = 0.0f, w.torque[b] = 0.0f;
            }
        }
    }
    // static bodies' awake flag: the last island that touched them (step.py:173-194)
    std::vector<int> last(B, -1);
    const int32_t *fbody = m.d->fixture_body;
    for (int sl = 0; sl < w.C; ++sl) {
        int i = isl.contact_island[sl];
        if (i < 0) continue;
        int ba = fbody[w.fa[sl]], bb = fbody[w.fb[sl]];
        last[ba] = std::max(last[ba], i), last[bb] = std::max(last[bb], i);
    }
    for (int j = 0; j < w.J; ++j) {
        int i = isl.joint_island[j];
        if (i < 0) continue;
        int ja = m.d->joint_a[j], jb = m.d->joint_b[j];
        last[ja] = std::max(last[ja], i), last[jb] = std::max(last[jb], i);
    }
    for (int b = 0; b < B; ++b)
        if (w.type[b] == STATIC && last[b] >= 0) {
            w.awake[b] = !isl_sleep[last[b]];
            w.sleep_time[b] = 0.0f;
        }
    std::vector<uint8_t> moved(B);
    for (int b = 0; b < B; ++b) moved[b] = in_isl[b] && w.type[b] != STATIC;
    synchronize_fixtures(m, w, moved.data());
    find_new_contacts(m, w);
}

// b2World::Step (step.py:28-47)
static void step(const Model &m, World &w, const goib2d_settings &s, float dt) {
    if (*w.new_fixture) find_new_contacts(m, w);
    *w.new_fixture = 0;
    float inv_dt = dt > 0 ? 1.0f / dt : 0.0f;
    float dt_ratio = *w.inv_dt0 * dt;
    collide(m, w, s);
    solve(m, w, s, dt, inv_dt, dt_ratio);
    if (s.continuous_physics) solve_toi(m, w, s, dt);
    if (dt > 0) *w.inv_dt0 = inv_dt;
    if (s.auto_clear_forces)
        for (int b = 0; b < w.B; ++b) w.force[2 * b] = w.force[2 * b + 1] = 0.0f, w.torque[b] = 0.0f;
}

}  // namespace orc

// ---------------------------------------------------------------- C entry points for the tests and the CPU baseline
extern "C" {

int oracle_leaf_dtype(int leaf) { return orc::leaf_dtype(leaf); }
int64_t oracle_leaf_elems(int leaf, int32_t B, int32_t rows, int32_t J, int32_t C) {
    return orc::leaf_elems(leaf, B, rows, J, C);
}

void oracle_sin_cos(const float *x, int64_t n, float *s, float *c) {
    for (int64_t i = 0; i < n; ++i) s[i] = orc::sin_of(x[i], &c[i]);
}

// Step worlds [w0, w1) of a batch n_steps times on the host (leaves: host pointers, (N, ...) layout).
// actions: NULL or float [N][n_action]; before each step joints.motor_speed[joint[k]] = scale[k] * action[k].
int oracle_step_range_events(const goib2d_model_desc *desc, const goib2d_settings *s, float dt, int32_t C,
                             int32_t rows, int64_t w0, int64_t w1, int32_t n_steps, void *const *leaves,
                             const float *actions, int32_t n_action, const int32_t *action_joint,
                             const float *action_scale, goib2d_event *events, int32_t *event_count,
                             int32_t event_cap) {
    orc::Model m{desc, desc->n_bodies, desc->n_fixtures, desc->n_joints, desc->n_pairs, desc->fixture_slot != nullptr};
    if (m.compact && rows == m.F) m.compact = false;  // a full-layout State also works with a compact Model
    for (int64_t wi = w0; wi < w1; ++wi) {
        orc::World w;
        orc::bind_world(w, leaves, wi, m.B, rows, m.J, C);
        if (events) w.events = events + wi * event_cap, w.event_count = event_count + wi, w.event_cap = event_cap;
        for (int k = 0; k < n_steps; ++k) {
            if (actions)
                for (int a = 0; a < n_action; ++a)
                    w.motor_speed[action_joint[a]] = action_scale[a] * actions[wi * n_action + a];
            orc::step(m, w, *s, dt);
        }
    }
    return 0;
}

int oracle_step_range(const goib2d_model_desc *desc, const goib2d_settings *s, float dt, int32_t C, int32_t rows,
                      int64_t w0, int64_t w1, int32_t n_steps, void *const *leaves, const float *actions,
                      int32_t n_action, const int32_t *action_joint, const float *action_scale) {
    return oracle_step_range_events(desc, s, dt, C, rows, w0, w1, n_steps, leaves, actions, n_action, action_joint,
                                    action_scale, nullptr, nullptr, 0);
}
}
