// Parity oracle (test infrastructure, see oracle.h): b2World::SolveTOI (reference toi.py), one world.
#include <algorithm>
#include <vector>

#include "oracle.h"

namespace orc {

namespace {
enum { E_UNKNOWN = 0, E_FAILED = 1, E_OVERLAPPED = 2, E_TOUCHING = 3, E_SEPARATED = 4 };
enum { E_POINTS = 0, E_FACE_A = 1, E_FACE_B = 2 };
constexpr int GJK_ITERS = 20, TOI_ITERS = 20, ROOT_ITERS = 50;

struct Sweep {  // b2Sweep (toi.py:73-111)
    V2 lc, c0, c;
    float a0, a;
};
struct Proxy {  // b2DistanceProxy over a fixture (toi.py:483-485)
    const float *v;
    int count;
    float radius;
    V2 vert(int i) const {
        i = i < 0 ? 0 : (i > MAXV - 1 ? MAXV - 1 : i);
        return {v[2 * i], v[2 * i + 1]};
    }
    int support(V2 d) const {  // b2DistanceProxy::GetSupport: first index of the largest dot
        int best = 0;
        float bv = 0;
        for (int i = 0; i < count; ++i) {
            float val = v[2 * i] * d.x + v[2 * i + 1] * d.y;
            if (i == 0 || val > bv) best = i, bv = val;
        }
        return best;
    }
};
inline Proxy proxy_of(const Model &m, int f) { return {m.d->verts + 16 * f, m.d->count[f], m.d->radius[f]}; }

inline Xf sweep_xf(const Sweep &sw, float t) {  // b2Sweep::GetTransform (toi.py:73-81)
    float omb = 1.0f - t;
    float px = omb * sw.c0.x + t * sw.c.x, py = omb * sw.c0.y + t * sw.c.y;
    Rot q = rot_of(omb * sw.a0 + t * sw.a);
    V2 r = rot(q, sw.lc);
    return {{px - r.x, py - r.y}, q};
}

inline void normalize_sweep(Sweep &sw) {  // b2Sweep::Normalize (toi.py:92-97)
    const float two_pi = 2.0f * PI_F;
    float d = two_pi * std::floor(sw.a0 / two_pi);
    sw.a0 = sw.a0 - d, sw.a = sw.a - d;
}

struct SV {  // b2SimplexVertex
    V2 wA, wB, w;
    float a;
    int iA, iB;
};
struct Cache {  // b2SimplexCache
    int count = 0;
    int iA[3] = {0, 0, 0}, iB[3] = {0, 0, 0};
    float metric = 0.0f;
};

inline SV make_vertex(const Proxy &pA, Xf xfA, int iA, const Proxy &pB, Xf xfB, int iB) {
    SV v;
    v.wA = xf_mul(xfA, pA.vert(iA));
    v.wB = xf_mul(xfB, pB.vert(iB));
    v.w = sub(v.wB, v.wA);
    v.a = 0.0f, v.iA = iA, v.iB = iB;
    return v;
}

inline float simplex_metric(const SV *s, int count) {  // b2Simplex::GetMetric (toi.py:152-157)
    if (count == 2) return length(sub(s[0].w, s[1].w));
    if (count == 3) return cross(sub(s[1].w, s[0].w), sub(s[2].w, s[0].w));
    return 0.0f;
}

void solve2(SV *s, int &count) {  // b2Simplex::Solve2 (toi.py:160-175)
    V2 w1 = s[0].w, w2 = s[1].w;
    V2 e12 = sub(w2, w1);
    float d12_2 = -dot(w1, e12);
    float d12_1 = dot(w2, e12);
    if (d12_2 <= 0) {
        s[0].a = 1.0f;
        count = 1;
        return;
    }
    if (d12_1 <= 0) {
        s[1].a = 1.0f;
        s[0] = s[1];
        count = 1;
        return;
    }
    float inv = 1.0f / (d12_1 + d12_2);
    s[0].a = d12_1 * inv, s[1].a = d12_2 * inv;
    count = 2;
}

void solve3(SV *s, int &count) {  // b2Simplex::Solve3 (toi.py:178-227)
    V2 w1 = s[0].w, w2 = s[1].w, w3 = s[2].w;
    V2 e12 = sub(w2, w1);
    float d12_1 = dot(w2, e12), d12_2 = -dot(w1, e12);
    V2 e13 = sub(w3, w1);
    float d13_1 = dot(w3, e13), d13_2 = -dot(w1, e13);
    V2 e23 = sub(w3, w2);
    float d23_1 = dot(w3, e23), d23_2 = -dot(w2, e23);
    float n123 = cross(e12, e13);
    float d123_1 = n123 * cross(w2, w3), d123_2 = n123 * cross(w3, w1), d123_3 = n123 * cross(w1, w2);
    if (d12_2 <= 0 && d13_2 <= 0) {
        s[0].a = 1.0f;
        count = 1;
    } else if (d12_1 > 0 && d12_2 > 0 && d123_3 <= 0) {
        float inv = 1.0f / (d12_1 + d12_2);
        s[0].a = d12_1 * inv, s[1].a = d12_2 * inv;
        count = 2;
    } else if (d13_1 > 0 && d13_2 > 0 && d123_2 <= 0) {
        float inv = 1.0f / (d13_1 + d13_2);
        s[0].a = d13_1 * inv, s[2].a = d13_2 * inv;
        s[1] = s[2];
        count = 2;
    } else if (d12_1 <= 0 && d23_2 <= 0) {
        s[1].a = 1.0f;
        s[0] = s[1];
        count = 1;
    } else if (d13_1 <= 0 && d23_1 <= 0) {
        s[2].a = 1.0f;
        s[0] = s[2];
        count = 1;
    } else if (d23_1 > 0 && d23_2 > 0 && d123_1 <= 0) {
        float inv = 1.0f / (d23_1 + d23_2);
        s[1].a = d23_1 * inv, s[2].a = d23_2 * inv;
        s[0] = s[2];
        count = 2;
    } else {
        float inv = 1.0f / ((d123_1 + d123_2) + d123_3);
        s[0].a = d123_1 * inv, s[1].a = d123_2 * inv, s[2].a = d123_3 * inv;
        count = 3;
    }
}

// b2Distance with useRadii = false (toi.py:230-294)
float distance(Cache &cache, const Proxy &pA, Xf xfA, const Proxy &pB, Xf xfB) {
    SV s[3];
    for (int j = 0; j < 3; ++j) s[j] = SV{{0, 0}, {0, 0}, {0, 0}, 0.0f, 0, 0};
    for (int j = 0; j < cache.count; ++j) s[j] = make_vertex(pA, xfA, cache.iA[j], pB, xfB, cache.iB[j]);
    int count = cache.count;
    float metric2 = simplex_metric(s, count);
    if (count > 1 && (metric2 < 0.5f * cache.metric || 2.0f * cache.metric < metric2 || metric2 < EPS)) count = 0;
    if (count == 0) {
        s[0] = make_vertex(pA, xfA, 0, pB, xfB, 0);
        s[0].a = 1.0f;
        count = 1;
    }
    int it = 0;
    while (it < GJK_ITERS) {
        int save_count = count, saveA[3], saveB[3];
        for (int j = 0; j < 3; ++j) saveA[j] = s[j].iA, saveB[j] = s[j].iB;
        if (count == 2) solve2(s, count);
        else if (count == 3) solve3(s, count);
        if (count == 3) break;
        V2 d;
        if (count == 1) {
            d = neg(s[0].w);
        } else {
            V2 e12 = sub(s[1].w, s[0].w);
            float sgn = cross(e12, neg(s[0].w));
            d = sgn > 0 ? cross_sv(1.0f, e12) : cross_vs(e12, 1.0f);
        }
        if (dot(d, d) < EPS * EPS) break;
        int iA = pA.support(rot_t(xfA.q, neg(d)));
        int iB = pB.support(rot_t(xfB.q, d));
        SV v = make_vertex(pA, xfA, iA, pB, xfB, iB);
        v.a = s[count].a;  // the tentative vertex's barycentric weight is not set
        s[count] = v;
        ++it;
        bool dup = false;
        for (int j = 0; j < save_count; ++j)
            if (saveA[j] == iA && saveB[j] == iB) dup = true;
        if (dup) break;
        ++count;
    }
    V2 pa, pb;
    if (count == 1) {
        pa = s[0].wA, pb = s[0].wB;
    } else if (count == 2) {
        pa = {s[0].a * s[0].wA.x + s[1].a * s[1].wA.x, s[0].a * s[0].wA.y + s[1].a * s[1].wA.y};
        pb = {s[0].a * s[0].wB.x + s[1].a * s[1].wB.x, s[0].a * s[0].wB.y + s[1].a * s[1].wB.y};
    } else {
        V2 p2{s[0].a * s[0].wA.x + s[1].a * s[1].wA.x, s[0].a * s[0].wA.y + s[1].a * s[1].wA.y};
        pa = {p2.x + s[2].a * s[2].wA.x, p2.y + s[2].a * s[2].wA.y};
        pb = pa;
    }
    float dist = length(sub(pa, pb));
    cache.count = count;
    for (int j = 0; j < 3; ++j) cache.iA[j] = s[j].iA, cache.iB[j] = s[j].iB;
    cache.metric = simplex_metric(s, count);
    return dist;
}

struct SepFn {  // b2SeparationFunction (toi.py:299-359)
    int type;
    V2 axis, lp;
};

SepFn sep_init(const Cache &cache, const Proxy &pA, Xf xfA, const Proxy &pB, Xf xfB) {
    SepFn f;
    if (cache.count == 1) {
        V2 pa = xf_mul(xfA, pA.vert(cache.iA[0])), pb = xf_mul(xfB, pB.vert(cache.iB[0]));
        f.type = E_POINTS, f.axis = normalize(sub(pb, pa)), f.lp = {0.0f, 0.0f};
    } else if (cache.iA[0] == cache.iA[1]) {
        V2 b1 = pB.vert(cache.iB[0]), b2 = pB.vert(cache.iB[1]);
        V2 ax = normalize(cross_vs(sub(b2, b1), 1.0f));
        V2 n = rot(xfB.q, ax);
        V2 lp{0.5f * (b1.x + b2.x), 0.5f * (b1.y + b2.y)};
        V2 qb = xf_mul(xfB, lp), pa = xf_mul(xfA, pA.vert(cache.iA[0]));
        float s = dot(sub(pa, qb), n);
        f.type = E_FACE_B, f.axis = s < 0 ? neg(ax) : ax, f.lp = lp;
    } else {
        V2 a1 = pA.vert(cache.iA[0]), a2 = pA.vert(cache.iA[1]);
        V2 ax = normalize(cross_vs(sub(a2, a1), 1.0f));
        V2 n = rot(xfA.q, ax);
        V2 lp{0.5f * (a1.x + a2.x), 0.5f * (a1.y + a2.y)};
        V2 qa = xf_mul(xfA, lp), pb = xf_mul(xfB, pB.vert(cache.iB[0]));
        float s = dot(sub(pb, qa), n);
        f.type = E_FACE_A, f.axis = s < 0 ? neg(ax) : ax, f.lp = lp;
    }
    return f;
}

float sep_eval(const SepFn &f, const Proxy &pA, Xf xfA, int iA, const Proxy &pB, Xf xfB, int iB) {
    if (f.type == E_POINTS) {
        V2 pa = xf_mul(xfA, pA.vert(iA)), pb = xf_mul(xfB, pB.vert(iB));
        return dot(sub(pb, pa), f.axis);
    }
    if (f.type == E_FACE_A) {
        V2 n = rot(xfA.q, f.axis), qa = xf_mul(xfA, f.lp), pb = xf_mul(xfB, pB.vert(iB));
        return dot(sub(pb, qa), n);
    }
    V2 n = rot(xfB.q, f.axis), qb = xf_mul(xfB, f.lp), pa = xf_mul(xfA, pA.vert(iA));
    return dot(sub(pa, qb), n);
}

float sep_find_min(const SepFn &f, const Proxy &pA, Xf xfA, const Proxy &pB, Xf xfB, int *iA, int *iB) {
    if (f.type == E_POINTS) {
        *iA = pA.support(rot_t(xfA.q, f.axis));
        *iB = pB.support(rot_t(xfB.q, neg(f.axis)));
    } else if (f.type == E_FACE_A) {
        V2 n = rot(xfA.q, f.axis);
        *iA = -1;
        *iB = pB.support(rot_t(xfB.q, neg(n)));
    } else {
        V2 n = rot(xfB.q, f.axis);
        *iB = -1;
        *iA = pA.support(rot_t(xfA.q, neg(n)));
    }
    return sep_eval(f, pA, xfA, *iA, pB, xfB, *iB);
}

// b2TimeOfImpact with tMax = 1 (toi.py:364-457)
int time_of_impact(const Proxy &pA, Sweep swA, const Proxy &pB, Sweep swB, float linear_slop, float *t_out) {
    normalize_sweep(swA);
    normalize_sweep(swB);
    float total_radius = pA.radius + pB.radius;
    float target = bmax(linear_slop, total_radius - 3.0f * linear_slop);
    float tol = 0.25f * linear_slop;
    float t1 = 0.0f;
    int iter = 0;
    Cache cache;
    for (;;) {
        Xf xfA = sweep_xf(swA, t1), xfB = sweep_xf(swB, t1);
        float dist = distance(cache, pA, xfA, pB, xfB);
        if (dist <= 0.0f) {
            *t_out = 0.0f;
            return E_OVERLAPPED;
        }
        if (dist < target + tol) {
            *t_out = t1;
            return E_TOUCHING;
        }
        SepFn f = sep_init(cache, pA, xfA, pB, xfB);
        float t2 = 1.0f;
        int push = 0;
        for (;;) {
            int iA, iB;
            Xf xA2 = sweep_xf(swA, t2), xB2 = sweep_xf(swB, t2);
            float s2 = sep_find_min(f, pA, xA2, pB, xB2, &iA, &iB);
            if (s2 > target + tol) {
                *t_out = 1.0f;
                return E_SEPARATED;
            }
            if (s2 > target - tol) {
                t1 = t2;
                break;
            }
            Xf xA1 = sweep_xf(swA, t1), xB1 = sweep_xf(swB, t1);
            float s1 = sep_eval(f, pA, xA1, iA, pB, xB1, iB);
            if (s1 < target - tol) {
                *t_out = t1;
                return E_FAILED;
            }
            if (s1 <= target + tol) {
                *t_out = t1;
                return E_TOUCHING;
            }
            int cnt = 0;
            float a1 = t1, a2 = t2;
            for (;;) {
                float t = (cnt & 1) ? a1 + ((target - s1) * (a2 - a1)) / (s2 - s1) : 0.5f * (a1 + a2);
                ++cnt;
                Xf xa = sweep_xf(swA, t), xb = sweep_xf(swB, t);
                float s = sep_eval(f, pA, xa, iA, pB, xb, iB);
                if (babs(s - target) < tol) {
                    t2 = t;
                    break;
                }
                if (s > target)
                    a1 = t, s1 = s;
                else
                    a2 = t, s2 = s;
                if (cnt == ROOT_ITERS) break;
            }
            ++push;
            if (push == MAXV) break;
        }
        ++iter;
        if (iter == TOI_ITERS) {
            *t_out = t1;
            return E_FAILED;
        }
    }
}

inline void advance(float &c0x, float &c0y, float &a0, float &alpha0, float cx, float cy, float a, float alpha) {
    // b2Sweep::Advance (toi.py:100-104)
    float den = 1.0f - alpha0;
    float beta = (alpha - alpha0) / (den != 0 ? den : 1.0f);
    c0x = c0x + beta * (cx - c0x), c0y = c0y + beta * (cy - c0y), a0 = a0 + beta * (a - a0), alpha0 = alpha;
}

inline Xf sync_xf(float cx, float cy, float a, V2 lc) {  // b2Body::SynchronizeTransform
    Rot q = rot_of(a);
    V2 r = rot(q, lc);
    return {{cx - r.x, cy - r.y}, q};
}

inline bool pair_rule(const World &w, int a, int b, bool unity) {  // toi.py:462-470
    bool dyn_a = w.type[a] == DYNAMIC, dyn_b = w.type[b] == DYNAMIC;
    bool stock = w.bullet[a] || !dyn_a || w.bullet[b] || !dyn_b;
    if (!unity) return stock;
    bool rule = (w.bullet[a] || w.bullet[b]) || (!dyn_b ? (bool)w.continuous[a] : (!dyn_a ? (bool)w.continuous[b] : false));
    return stock && rule;
}

std::vector<int> list_order(const World &w) {
    std::vector<int> live;
    for (int s = 0; s < w.C; ++s)
        if (w.pair[s] >= 0) live.push_back(s);
    std::stable_sort(live.begin(), live.end(), [&](int x, int y) { return w.key[x] > w.key[y]; });
    return live;
}

// one pass of the min-TOI search (toi.py:488-558)
bool search(const Model &m, World &w, const goib2d_settings &s, int *min_slot, float *min_alpha) {
    const int C = w.C;
    const int32_t *fbody = m.d->fixture_body;
    std::vector<int> order = list_order(w);
    std::vector<int> pos(C, C);
    for (size_t k = 0; k < order.size(); ++k) pos[order[k]] = (int)k;
    for (int slot : order) {
        bool base = w.t_enabled[slot] && w.t_count[slot] <= MAX_SUB_STEPS;
        if (!base || w.t_flag[slot]) continue;
        int A = fbody[w.fa[slot]], B = fbody[w.fb[slot]];
        bool actA = w.awake[A] && w.type[A] != STATIC, actB = w.awake[B] && w.type[B] != STATIC;
        if (!(actA || actB) || !pair_rule(w, A, B, s.unity_toi)) continue;
        // put both sweeps on the same time interval: advance the body that is behind
        float alA = w.t_alpha0[A], alB = w.t_alpha0[B];
        float common = alA;
        if (alA < alB) {
            advance(w.c0[2 * A], w.c0[2 * A + 1], w.a0[A], w.t_alpha0[A], w.c[2 * A], w.c[2 * A + 1], w.a[A], alB);
            common = alB;
        } else if (alB < alA) {
            advance(w.c0[2 * B], w.c0[2 * B + 1], w.a0[B], w.t_alpha0[B], w.c[2 * B], w.c[2 * B + 1], w.a[B], alA);
        }
        Sweep swA{{w.local_center[2 * A], w.local_center[2 * A + 1]}, {w.c0[2 * A], w.c0[2 * A + 1]},
                  {w.c[2 * A], w.c[2 * A + 1]}, w.a0[A], w.a[A]};
        Sweep swB{{w.local_center[2 * B], w.local_center[2 * B + 1]}, {w.c0[2 * B], w.c0[2 * B + 1]},
                  {w.c[2 * B], w.c[2 * B + 1]}, w.a0[B], w.a[B]};
        float beta;
        int st = time_of_impact(proxy_of(m, w.fa[slot]), swA, proxy_of(m, w.fb[slot]), swB, s.linear_slop, &beta);
        float alpha = st == E_TOUCHING ? bmin(common + (1.0f - common) * beta, 1.0f) : 1.0f;
        w.t_toi[slot] = alpha;
        w.t_flag[slot] = 1;
    }
    float best = 1.0f;
    bool any = false;
    for (int slot : order) {
        bool base = w.t_enabled[slot] && w.t_count[slot] <= MAX_SUB_STEPS;
        if (base && w.t_flag[slot] && w.t_toi[slot] < 1.0f) {
            any = true;
            best = std::fmin(best, w.t_toi[slot]);
        }
    }
    int ms = 0, msp = s.toi_tie_oldest ? -1 : C;
    for (int slot = 0; slot < C; ++slot) {
        if (w.pair[slot] < 0) continue;
        bool base = w.t_enabled[slot] && w.t_count[slot] <= MAX_SUB_STEPS;
        if (!(base && w.t_flag[slot] && w.t_toi[slot] < 1.0f && w.t_toi[slot] == best)) continue;
        if (s.toi_tie_oldest ? pos[slot] > msp : pos[slot] < msp) ms = slot, msp = pos[slot];
    }
    *min_slot = ms;
    *min_alpha = best;
    const float done_alpha = 1.0f - 10.0f * EPS;
    return any && !(done_alpha < best);
}

void update_contact(World &w, int s_, const Manifold &mn, bool *flip) {  // b2Contact::Update (toi.py:567-594)
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
    bool touching = mn.count > 0;
    *flip = touching != (bool)w.touching[s_];
    if (*flip) emit_event(w, touching ? EV_BEGIN : EV_END, s_);
    w.touching[s_] = touching;
    w.count[s_] = mn.count;
    if (mn.count > 0) {
        w.mtype[s_] = mn.mtype;
        w.local_normal[2 * s_] = mn.local_normal.x, w.local_normal[2 * s_ + 1] = mn.local_normal.y;
        w.local_point[2 * s_] = mn.local_point.x, w.local_point[2 * s_ + 1] = mn.local_point.y;
        for (int k = 0; k < 2; ++k) {
            w.point_local[4 * s_ + 2 * k] = mn.point[k].x, w.point_local[4 * s_ + 2 * k + 1] = mn.point[k].y;
            w.point_id[2 * s_ + k] = mn.id[k];
        }
    }
    for (int k = 0; k < 2; ++k) w.normal_impulse[2 * s_ + k] = ni[k], w.tangent_impulse[2 * s_ + k] = ti[k];
}

inline void wake(World &w, int b) {
    if (!w.awake[b]) w.awake[b] = 1, w.sleep_time[b] = 0.0f;
}

// one TOI event (toi.py:604-716) with b2Island::SolveTOI (toi.py:719-799)
void event(const Model &m, World &w, const goib2d_settings &s, float dt, int min_slot, float min_alpha) {
    const int B = w.B, C = w.C;
    const int32_t *fbody = m.d->fixture_body;
    const int A = fbody[w.fa[min_slot]], Bb = fbody[w.fb[min_slot]];
    auto lc_of = [&](int b) { return V2{w.local_center[2 * b], w.local_center[2 * b + 1]}; };
    // every body advanced to min_alpha; the walk keeps that only for island bodies
    std::vector<float> ac0x(B), ac0y(B), aa0(B), aal0(B);
    std::vector<Xf> axf(B);
    for (int b = 0; b < B; ++b) {
        ac0x[b] = w.c0[2 * b], ac0y[b] = w.c0[2 * b + 1], aa0[b] = w.a0[b], aal0[b] = w.t_alpha0[b];
        advance(ac0x[b], ac0y[b], aa0[b], aal0[b], w.c[2 * b], w.c[2 * b + 1], w.a[b], min_alpha);
        axf[b] = sync_xf(ac0x[b], ac0y[b], aa0[b], lc_of(b));
    }
    auto man_of = [&](int slot, Manifold *mn) {
        int ba = fbody[w.fa[slot]], bb = fbody[w.fb[slot]];
        evaluate(m, w.fa[slot], w.fb[slot], axf[ba], axf[bb], s.linear_slop, s.angular_slop, mn);
    };
    std::vector<uint8_t> flip_b(B, 0), in_isl_other(B, 0), touched_other(B, 0), newbody(B, 0);
    Manifold mmin;
    man_of(min_slot, &mmin);
    bool t_min = mmin.count > 0;
    bool fl;
    update_contact(w, min_slot, mmin, &fl);
    if (fl) flip_b[fbody[w.fa[min_slot]]] = flip_b[fbody[w.fb[min_slot]]] = 1;
    w.t_enabled[min_slot] = t_min;
    w.t_count[min_slot] += 1;
    w.t_flag[min_slot] = 0;
    std::vector<int> island_contacts;
    if (t_min) {
        island_contacts.push_back(min_slot);
        std::vector<int> order = list_order(w);
        int n_bodies = 2;
        std::vector<uint8_t> isl_flag_body(B, 0);
        const int owners[2] = {A, Bb};
        bool stop = false;
        for (int oi = 0; oi < 2 && !stop; ++oi) {
            int owner = owners[oi];
            if (w.type[owner] != DYNAMIC) continue;
            for (int slot : order) {
                int ca = fbody[w.fa[slot]], cb = fbody[w.fb[slot]];
                if (ca != owner && cb != owner) continue;
                if (oi == 1 && w.type[A] == DYNAMIC && (ca == A || cb == A)) continue;  // seen in bodyA's list
                if (!((int)island_contacts.size() < MAX_TOI_CONTACTS && n_bodies < 2 * MAX_TOI_CONTACTS)) {
                    stop = true;
                    break;
                }
                if (slot == min_slot) continue;
                int other = ca == owner ? cb : ca;
                if (w.type[other] == DYNAMIC && !w.bullet[owner] && !w.bullet[other]) continue;
                if (s.unity_toi && !pair_rule(w, owner, other, true)) continue;
                Manifold mn;
                man_of(slot, &mn);
                update_contact(w, slot, mn, &fl);
                if (fl) flip_b[ca] = flip_b[cb] = 1;
                w.t_enabled[slot] = 1;
                touched_other[other] = 1;
                if (mn.count <= 0) continue;
                island_contacts.push_back(slot);
                in_isl_other[other] = 1;
                if (other != A && other != Bb && !isl_flag_body[other]) {
                    isl_flag_body[other] = 1;
                    newbody[other] = 1;
                    ++n_bodies;
                }
            }
        }
    }
    // body sweeps after the walk
    for (int b = 0; b < B; ++b) {
        bool pair_b = b == A || b == Bb;
        bool keep_adv = (pair_b && t_min) || in_isl_other[b];
        bool restore = (pair_b && !t_min) || (touched_other[b] && !in_isl_other[b]);
        if (keep_adv) {
            w.c0[2 * b] = ac0x[b], w.c0[2 * b + 1] = ac0y[b], w.a0[b] = aa0[b];
            w.c[2 * b] = ac0x[b], w.c[2 * b + 1] = ac0y[b], w.a[b] = aa0[b];
            w.t_alpha0[b] = aal0[b];
            w.xf_p[2 * b] = axf[b].p.x, w.xf_p[2 * b + 1] = axf[b].p.y;
            w.xf_q[2 * b] = axf[b].q.c, w.xf_q[2 * b + 1] = axf[b].q.s;
        } else if (restore) {
            Xf o = sync_xf(w.c[2 * b], w.c[2 * b + 1], w.a[b], lc_of(b));
            w.xf_p[2 * b] = o.p.x, w.xf_p[2 * b + 1] = o.p.y;
            w.xf_q[2 * b] = o.q.c, w.xf_q[2 * b + 1] = o.q.s;
        }
    }
    for (int b = 0; b < B; ++b) {
        bool pair_b = b == A || b == Bb;
        if (flip_b[b] || (pair_b && t_min) || (newbody[b] && w.type[b] != STATIC)) wake(w, b);
    }
    std::vector<uint8_t> in_isl(B, 0);
    if (t_min)
        for (int b = 0; b < B; ++b) in_isl[b] = b == A || b == Bb || in_isl_other[b];
    // b2Island::SolveTOI
    std::vector<uint8_t> solved(C, 0);
    std::vector<float> ni_r(2 * C, 0.0f), ti_r(2 * C, 0.0f);
    if (t_min) {
        const int n = (int)island_contacts.size();
        // position rows from the updated contacts; masses only for the TOI pair
        std::vector<float> px(B), py(B), pa(B);
        for (int b = 0; b < B; ++b) px[b] = w.c[2 * b], py[b] = w.c[2 * b + 1], pa[b] = w.a[b];
        struct PC {
            int ia, ib, mtype, pc_count;
            float mA, mB, iA, iB, radA, radB;
            V2 ln, lp, pl[2], lcA, lcB;
        };
        std::vector<PC> pcs(n);
        for (int k = 0; k < n; ++k) {
            int slot = island_contacts[k];
            PC &p = pcs[k];
            p.ia = fbody[w.fa[slot]], p.ib = fbody[w.fb[slot]];
            bool ta = p.ia == A || p.ia == Bb, tb = p.ib == A || p.ib == Bb;
            p.mA = ta ? w.inv_mass[p.ia] : 0.0f, p.iA = ta ? w.inv_inertia[p.ia] : 0.0f;
            p.mB = tb ? w.inv_mass[p.ib] : 0.0f, p.iB = tb ? w.inv_inertia[p.ib] : 0.0f;
            p.pc_count = w.count[slot], p.mtype = w.mtype[slot];
            p.ln = {w.local_normal[2 * slot], w.local_normal[2 * slot + 1]};
            p.lp = {w.local_point[2 * slot], w.local_point[2 * slot + 1]};
            for (int j = 0; j < 2; ++j) p.pl[j] = {w.point_local[4 * slot + 2 * j], w.point_local[4 * slot + 2 * j + 1]};
            p.lcA = lc_of(p.ia), p.lcB = lc_of(p.ib);
            p.radA = m.d->radius[w.fa[slot]], p.radB = m.d->radius[w.fb[slot]];
        }
        const float okay_sep = -1.5f * s.linear_slop;
        for (int it = 0; it < 20; ++it) {
            float min_sep = 0.0f;
            for (int k = 0; k < n; ++k) {
                const PC &c = pcs[k];
                V2 cA{px[c.ia], py[c.ia]}, cB{px[c.ib], py[c.ib]};
                float aA = pa[c.ia], aB = pa[c.ib];
                float msep = 0.0f;
                for (int j = 0; j < c.pc_count; ++j) {  // contact_solver.py:307-354 with toi_baumgarte
                    Xf xfA = sync_xf(cA.x, cA.y, aA, c.lcA), xfB = sync_xf(cB.x, cB.y, aB, c.lcB);
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
                    msep = bmin(msep, sep);
                    float C_ = clampf(s.toi_baumgarte * (sep + s.linear_slop), -s.max_linear_correction, 0.0f);
                    float rnA = cross(ra, nrm), rnB = cross(rb, nrm);
                    float K = ((c.mA + c.mB) + (c.iA * rnA) * rnA) + (c.iB * rnB) * rnB;
                    float imp = K > 0 ? -C_ / K : 0.0f;
                    V2 P{imp * nrm.x, imp * nrm.y};
                    cA = {cA.x - c.mA * P.x, cA.y - c.mA * P.y};
                    aA = aA - c.iA * cross(ra, P);
                    cB = {cB.x + c.mB * P.x, cB.y + c.mB * P.y};
                    aB = aB + c.iB * cross(rb, P);
                }
                px[c.ia] = cA.x, py[c.ia] = cA.y, pa[c.ia] = aA;
                px[c.ib] = cB.x, py[c.ib] = cB.y, pa[c.ib] = aB;
                min_sep = bmin(min_sep, msep);
            }
            if (min_sep >= okay_sep) break;
        }
        // leap of faith: the TOI bodies' sweep start is the solved pose
        for (int b : {A, Bb}) w.c0[2 * b] = px[b], w.c0[2 * b + 1] = py[b], w.a0[b] = pa[b];
        // velocity constraints without warm start (contact_solver.prepare with warm = False)
        std::vector<float> vx(B), vy(B), vw(B);
        for (int b = 0; b < B; ++b) vx[b] = w.v[2 * b], vy[b] = w.v[2 * b + 1], vw[b] = w.w[b];
        struct TV {
            int slot, ia, ib, count;
            float mA, mB, iA, iB, friction, tangent_speed;
            V2 n, rA[2], rB[2];
            float nmass[2], tmass[2], bias[2], ni[2], ti[2], K[4], NM[4];
        };
        std::vector<TV> vcs(n);
        for (int k = 0; k < n; ++k) {
            int slot = island_contacts[k];
            TV &c = vcs[k];
            int fa = w.fa[slot], fb = w.fb[slot];
            int ia = fbody[fa], ib = fbody[fb];
            c.slot = slot, c.ia = ia, c.ib = ib;
            c.mA = w.inv_mass[ia], c.mB = w.inv_mass[ib], c.iA = w.inv_inertia[ia], c.iB = w.inv_inertia[ib];
            float rA_ = m.d->radius[fa], rB_ = m.d->radius[fb];
            int mtype = w.mtype[slot], count = w.count[slot];
            V2 ln{w.local_normal[2 * slot], w.local_normal[2 * slot + 1]};
            V2 lp{w.local_point[2 * slot], w.local_point[2 * slot + 1]};
            V2 pl[2] = {{w.point_local[4 * slot], w.point_local[4 * slot + 1]},
                        {w.point_local[4 * slot + 2], w.point_local[4 * slot + 3]}};
            c.ni[0] = c.ni[1] = c.ti[0] = c.ti[1] = 0.0f;
            V2 cA{px[ia], py[ia]}, cB{px[ib], py[ib]};
            Xf xfA = sync_xf(cA.x, cA.y, pa[ia], lc_of(ia)), xfB = sync_xf(cB.x, cB.y, pa[ib], lc_of(ib));
            V2 nrm, pts[2];
            if (mtype == CIRCLES) {
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
            c.n = nrm;
            V2 t = cross_vs(nrm, 1.0f);
            V2 vA{vx[ia], vy[ia]}, vB{vx[ib], vy[ib]};
            float wA = vw[ia], wB = vw[ib];
            c.friction = w.friction[slot], c.tangent_speed = w.tangent_speed[slot];
            float restitution = w.restitution[slot];
            for (int j = 0; j < 2; ++j) {
                V2 ra = sub(pts[j], cA), rb = sub(pts[j], cB);
                float rnA = cross(ra, nrm), rnB = cross(rb, nrm);
                float kn = ((c.mA + c.mB) + (c.iA * rnA) * rnA) + (c.iB * rnB) * rnB;
                float rtA = cross(ra, t), rtB = cross(rb, t);
                float kt = ((c.mA + c.mB) + (c.iA * rtA) * rtA) + (c.iB * rtB) * rtB;
                V2 wBr = cross_sv(wB, rb), wAr = cross_sv(wA, ra);
                float vrel = dot(nrm, V2{((vB.x + wBr.x) - vA.x) - wAr.x, ((vB.y + wBr.y) - vA.y) - wAr.y});
                c.rA[j] = ra, c.rB[j] = rb;
                c.nmass[j] = inv_if_pos(kn), c.tmass[j] = inv_if_pos(kt);
                c.bias[j] = vrel < -s.velocity_threshold ? -restitution * vrel : 0.0f;
            }
            float rn1A = cross(c.rA[0], nrm), rn1B = cross(c.rB[0], nrm);
            float rn2A = cross(c.rA[1], nrm), rn2B = cross(c.rB[1], nrm);
            float k11 = ((c.mA + c.mB) + (c.iA * rn1A) * rn1A) + (c.iB * rn1B) * rn1B;
            float k22 = ((c.mA + c.mB) + (c.iA * rn2A) * rn2A) + (c.iB * rn2B) * rn2B;
            float k12 = ((c.mA + c.mB) + (c.iA * rn1A) * rn2A) + (c.iB * rn1B) * rn2B;
            bool safe = k11 * k11 < MAX_COND * (k11 * k22 - k12 * k12);
            bool two = count == 2;
            c.count = (two && !safe) ? 1 : count;
            float det = inv_or_zero(k11 * k22 - k12 * k12);
            bool use_k = two && safe;
            c.K[0] = use_k ? k11 : 0.0f, c.K[1] = use_k ? k12 : 0.0f, c.K[2] = use_k ? k12 : 0.0f;
            c.K[3] = use_k ? k22 : 0.0f;
            c.NM[0] = use_k ? det * k22 : 0.0f, c.NM[1] = use_k ? -det * k12 : 0.0f;
            c.NM[2] = use_k ? -det * k12 : 0.0f, c.NM[3] = use_k ? det * k11 : 0.0f;
        }
        for (int it = 0; it < s.velocity_iterations; ++it) {
            for (TV &c : vcs) {  // contact_solver.py:194-279
                V2 vA{vx[c.ia], vy[c.ia]}, vB{vx[c.ib], vy[c.ib]};
                float wA = vw[c.ia], wB = vw[c.ib];
                const float mA = c.mA, mB = c.mB, iA = c.iA, iB = c.iB;
                V2 nn = c.n, t = cross_vs(nn, 1.0f);
                auto dvf = [](V2 vb, float wb, V2 rb, V2 va, float wa, V2 ra) {
                    V2 b_ = cross_sv(wb, rb), a_ = cross_sv(wa, ra);
                    return V2{((vb.x + b_.x) - va.x) - a_.x, ((vb.y + b_.y) - va.y) - a_.y};
                };
                for (int j = 0; j < c.count; ++j) {
                    V2 d = dvf(vB, wB, c.rB[j], vA, wA, c.rA[j]);
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
                    V2 d = dvf(vB, wB, c.rB[0], vA, wA, c.rA[0]);
                    float vn = dot(d, nn);
                    float lam = -c.nmass[0] * (vn - c.bias[0]);
                    float nw = bmax(c.ni[0] + lam, 0.0f);
                    lam = nw - c.ni[0];
                    V2 P{lam * nn.x, lam * nn.y};
                    vA = {vA.x - mA * P.x, vA.y - mA * P.y};
                    wA = wA - iA * cross(c.rA[0], P);
                    vB = {vB.x + mB * P.x, vB.y + mB * P.y};
                    wB = wB + iB * cross(c.rB[0], P);
                    c.ni[0] = nw;
                } else if (c.count == 2) {
                    float ax = c.ni[0], ay = c.ni[1];
                    V2 d1 = dvf(vB, wB, c.rB[0], vA, wA, c.rA[0]), d2 = dvf(vB, wB, c.rB[1], vA, wA, c.rA[1]);
                    float vn1 = dot(d1, nn), vn2 = dot(d2, nn);
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
                        V2 P1{dx * nn.x, dx * nn.y}, P2{dy * nn.x, dy * nn.y};
                        vA = {vA.x - mA * (P1.x + P2.x), vA.y - mA * (P1.y + P2.y)};
                        wA = wA - iA * (cross(c.rA[0], P1) + cross(c.rA[1], P2));
                        vB = {vB.x + mB * (P1.x + P2.x), vB.y + mB * (P1.y + P2.y)};
                        wB = wB + iB * (cross(c.rB[0], P1) + cross(c.rB[1], P2));
                        c.ni[0] = xx, c.ni[1] = xy;
                    }
                }
                vx[c.ia] = vA.x, vy[c.ia] = vA.y, vw[c.ia] = wA;
                vx[c.ib] = vB.x, vy[c.ib] = vB.y, vw[c.ib] = wB;
            }
        }
        // integrate the island bodies over the rest of the step (toi.py:769-790)
        float h = (1.0f - min_alpha) * dt;
        float max_t = s.clamps_per_second ? s.max_translation * dt : s.max_translation;
        float max_r = s.clamps_per_second ? s.max_rotation * dt : s.max_rotation;
        for (int b = 0; b < B; ++b) {
            if (!in_isl[b]) continue;
            float bvx = vx[b], bvy = vy[b], bw = vw[b];
            float tx = h * bvx, ty = h * bvy;
            if (tx * tx + ty * ty > max_t * max_t) {
                float ratio = max_t / length(V2{tx, ty});
                bvx = bvx * ratio, bvy = bvy * ratio;
            }
            float rt = h * bw;
            if (rt * rt > max_r * max_r) bw = bw * (max_r / babs(rt));
            float ncx = px[b] + h * bvx, ncy = py[b] + h * bvy, na = pa[b] + h * bw;
            Xf x = sync_xf(ncx, ncy, na, lc_of(b));
            w.c[2 * b] = ncx, w.c[2 * b + 1] = ncy, w.a[b] = na;
            w.v[2 * b] = bvx, w.v[2 * b + 1] = bvy, w.w[b] = bw;
            w.xf_p[2 * b] = x.p.x, w.xf_p[2 * b + 1] = x.p.y, w.xf_q[2 * b] = x.q.c, w.xf_q[2 * b + 1] = x.q.s;
        }
        for (const TV &c : vcs) {  // b2Island::Report
            emit_event(w, EV_POST_SOLVE, c.slot, c.count, c.ni, c.ti);
            solved[c.slot] = 1;
            for (int j = 0; j < 2; ++j) {
                ni_r[2 * c.slot + j] = j < c.count ? c.ni[j] : 0.0f;
                ti_r[2 * c.slot + j] = j < c.count ? c.ti[j] : 0.0f;
            }
        }
        // synchronize the moved bodies' fixtures, invalidate their contacts' TOIs, find new contacts
        std::vector<uint8_t> moved(B);
        for (int b = 0; b < B; ++b) moved[b] = in_isl[b] && w.type[b] == DYNAMIC;
        synchronize_fixtures(m, w, moved.data());
        for (int slot = 0; slot < C; ++slot)
            if (moved[fbody[w.fa[slot]]] || moved[fbody[w.fb[slot]]]) w.t_flag[slot] = 0;
        std::vector<int32_t> old_pair(w.pair, w.pair + C), old_key(w.key, w.key + C);
        find_new_contacts(m, w);
        for (int slot = 0; slot < C; ++slot) {
            bool is_new = w.pair[slot] >= 0 && (old_pair[slot] < 0 || old_key[slot] != w.key[slot]);
            if (is_new) w.t_count[slot] = 0, w.t_flag[slot] = 0, w.t_enabled[slot] = 1;
        }
    }
    for (int slot = 0; slot < C; ++slot)
        if (solved[slot]) {
            w.t_solved[slot] = 1;
            for (int j = 0; j < 2; ++j) w.t_ni[2 * slot + j] = ni_r[2 * slot + j], w.t_ti[2 * slot + j] = ti_r[2 * slot + j];
        }
    *w.t_events += 1;
}
}  // namespace

// b2World::SolveTOI without sub-stepping (toi.py:827-865)
void solve_toi(const Model &m, World &w, const goib2d_settings &s, float dt) {
    if (w.C == 0 || m.P == 0) return;
    if (s.unity_toi && m.d->toi_bodies) {  // the reference skips SolveTOI at trace time for such a Model
        bool any = false;
        for (int b = 0; b < m.B; ++b) any = any || m.d->toi_bodies[b];
        if (!any) return;
    }
    for (int b = 0; b < w.B; ++b) w.t_alpha0[b] = 0.0f;
    for (int c = 0; c < w.C; ++c) {
        w.t_count[c] = 0, w.t_toi[c] = 1.0f, w.t_flag[c] = 0, w.t_enabled[c] = 1, w.t_solved[c] = 0;
        w.t_ni[2 * c] = w.t_ni[2 * c + 1] = w.t_ti[2 * c] = w.t_ti[2 * c + 1] = 0.0f;
    }
    *w.t_events = 0;
    if (!(dt > 0)) return;
    const int max_events = w.C * (MAX_SUB_STEPS + 1) + 8;
    int min_slot;
    float min_alpha;
    bool pending = false;
    for (int it = 0; it <= max_events; ++it) {
        if (pending) event(m, w, s, dt, min_slot, min_alpha);
        bool found = search(m, w, s, &min_slot, &min_alpha);
        if (!found) break;
        pending = true;
    }
}

}  // namespace orc
