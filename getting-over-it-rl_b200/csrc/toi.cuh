// goib2d device code: b2Distance (GJK), b2SeparationFunction and b2TimeOfImpact (toi.py:114-457), one contact per
// lane. Box2D's nested loops; every loop has its fixed iteration cap (GJK 20, separating axes 20, push-backs 8,
// root finder 50), so a lane always finishes.
#pragma once
#include "narrow.cuh"

#ifndef GB_COUNT
#define GB_COUNT(i, v) \
    do {               \
    } while (0)
#define GB_TOI_T0() \
    do {            \
    } while (0)
#define GB_TOI_T1(i) \
    do {             \
    } while (0)
#endif

namespace gb {

enum { E_UNKNOWN = 0, E_FAILED = 1, E_OVERLAPPED = 2, E_TOUCHING = 3, E_SEPARATED = 4 };
enum { E_POINTS = 0, E_FACE_A = 1, E_FACE_B = 2 };

struct Sweep {
    V2 lc, c0, c;
    float a0, a;
};
struct Proxy {
    const float *v;
    int count;
    float radius;
    __device__ V2 vert(int i) const {
        i = i < 0 ? 0 : (i > MAXV - 1 ? MAXV - 1 : i);
        return {v[2 * i], v[2 * i + 1]};
    }
    // b2DistanceProxy::GetSupport: the first vertex of largest projection on d, returned with its coordinates in
    // *pt. A fixture's slot holds MAXV vertices in one 64-byte-aligned run, so the four 16-byte words load together
    // (one memory round trip, not one per vertex); vertices past `count` are loaded but never chosen.
    __device__ __forceinline__ int support(V2 d, V2 *pt = nullptr) const {
        const float4 *q = reinterpret_cast<const float4 *>(v);
        float4 w[MAXV / 2];
#pragma unroll
        for (int k = 0; k < MAXV / 2; ++k) w[k] = __ldg(q + k);
        int best = 0;
        float bv = w[0].x * d.x + w[0].y * d.y;
        V2 bp{w[0].x, w[0].y};
#pragma unroll
        for (int i = 1; i < MAXV; ++i) {
            const float px = (i & 1) ? w[i >> 1].z : w[i >> 1].x, py = (i & 1) ? w[i >> 1].w : w[i >> 1].y;
            float val = px * d.x + py * d.y;
            if (i < count && val > bv) best = i, bv = val, bp = V2{px, py};
        }
        if (pt) *pt = bp;
        return best;
    }
};
__device__ __forceinline__ Proxy proxy_of(const DevModel &m, int f) {
    return {m.verts + 16 * f, m.count[f], m.radius[f]};
}

__device__ __forceinline__ Xf sweep_xf(const Sweep &sw, float t) {  // b2Sweep::GetTransform (toi.py:73-81)
    float omb = 1.0f - t;
    float px = omb * sw.c0.x + t * sw.c.x, py = omb * sw.c0.y + t * sw.c.y;
    Rot q = rot_of(omb * sw.a0 + t * sw.a);
    V2 r = rot(q, sw.lc);
    return {{px - r.x, py - r.y}, q};
}

struct SV {
    V2 wA, wB, w;
    float a;
    int iA, iB;
};
struct Cache {
    int count;
    int iA[3], iB[3];
    float metric;
};

__device__ __forceinline__ SV make_vertex_at(Xf xfA, V2 la, int iA, Xf xfB, V2 lb, int iB) {
    SV v;
    v.wA = xf_mul(xfA, la);
    v.wB = xf_mul(xfB, lb);
    v.w = sub(v.wB, v.wA);
    v.a = 0.0f, v.iA = iA, v.iB = iB;
    return v;
}
__device__ __forceinline__ SV make_vertex(const Proxy &pA, Xf xfA, int iA, const Proxy &pB, Xf xfB, int iB) {
    return make_vertex_at(xfA, pA.vert(iA), iA, xfB, pB.vert(iB), iB);
}
__device__ __forceinline__ float simplex_metric(const SV &s0, const SV &s1, const SV &s2, int count) {
    if (count == 2) return length(sub(s0.w, s1.w));
    if (count == 3) return cross(sub(s1.w, s0.w), sub(s2.w, s0.w));
    return 0.0f;
}

__device__ __forceinline__ void gjk_solve2(SV &s0, SV &s1, int &count) {  // toi.py:160-175
    V2 w1 = s0.w, w2 = s1.w;
    V2 e12 = sub(w2, w1);
    float d12_2 = -dot(w1, e12), d12_1 = dot(w2, e12);
    if (d12_2 <= 0) {
        s0.a = 1.0f, count = 1;
        return;
    }
    if (d12_1 <= 0) {
        s1.a = 1.0f, s0 = s1, count = 1;
        return;
    }
    float inv = 1.0f / (d12_1 + d12_2);
    s0.a = d12_1 * inv, s1.a = d12_2 * inv, count = 2;
}

__device__ __forceinline__ void gjk_solve3(SV &s0, SV &s1, SV &s2, int &count) {  // toi.py:178-227
    V2 w1 = s0.w, w2 = s1.w, w3 = s2.w;
    V2 e12 = sub(w2, w1);
    float d12_1 = dot(w2, e12), d12_2 = -dot(w1, e12);
    V2 e13 = sub(w3, w1);
    float d13_1 = dot(w3, e13), d13_2 = -dot(w1, e13);
    V2 e23 = sub(w3, w2);
    float d23_1 = dot(w3, e23), d23_2 = -dot(w2, e23);
    float n123 = cross(e12, e13);
    float d123_1 = n123 * cross(w2, w3), d123_2 = n123 * cross(w3, w1), d123_3 = n123 * cross(w1, w2);
    if (d12_2 <= 0 && d13_2 <= 0) {
        s0.a = 1.0f, count = 1;
    } else if (d12_1 > 0 && d12_2 > 0 && d123_3 <= 0) {
        float inv = 1.0f / (d12_1 + d12_2);
        s0.a = d12_1 * inv, s1.a = d12_2 * inv, count = 2;
    } else if (d13_1 > 0 && d13_2 > 0 && d123_2 <= 0) {
        float inv = 1.0f / (d13_1 + d13_2);
        s0.a = d13_1 * inv, s2.a = d13_2 * inv, s1 = s2, count = 2;
    } else if (d12_1 <= 0 && d23_2 <= 0) {
        s1.a = 1.0f, s0 = s1, count = 1;
    } else if (d13_1 <= 0 && d23_1 <= 0) {
        s2.a = 1.0f, s0 = s2, count = 1;
    } else if (d23_1 > 0 && d23_2 > 0 && d123_1 <= 0) {
        float inv = 1.0f / (d23_1 + d23_2);
        s1.a = d23_1 * inv, s2.a = d23_2 * inv, s0 = s2, count = 2;
    } else {
        float inv = 1.0f / ((d123_1 + d123_2) + d123_3);
        s0.a = d123_1 * inv, s1.a = d123_2 * inv, s2.a = d123_3 * inv, count = 3;
    }
}

// b2Distance, useRadii = false (toi.py:230-294)
// The simplex lives in three named vertices (s0, s1, s2), not an indexed array, so that it stays in registers.
__device__ __forceinline__ float gjk_distance(Cache &cache, const Proxy &pA, Xf xfA, const Proxy &pB, Xf xfB) {
    const SV zero{{0, 0}, {0, 0}, {0, 0}, 0.0f, 0, 0};
    SV s0 = zero, s1 = zero, s2 = zero;
    const int cc = cache.count;
    if (cc > 0) s0 = make_vertex(pA, xfA, cache.iA[0], pB, xfB, cache.iB[0]);
    if (cc > 1) s1 = make_vertex(pA, xfA, cache.iA[1], pB, xfB, cache.iB[1]);
    if (cc > 2) s2 = make_vertex(pA, xfA, cache.iA[2], pB, xfB, cache.iB[2]);
    int count = cc;
    float metric2 = simplex_metric(s0, s1, s2, count);
    if (count > 1 && (metric2 < 0.5f * cache.metric || 2.0f * cache.metric < metric2 || metric2 < EPS)) count = 0;
    if (count == 0) {
        s0 = make_vertex(pA, xfA, 0, pB, xfB, 0);
        s0.a = 1.0f;
        count = 1;
    }
    for (int it = 0; it < 20;) {
        const int save_count = count;
        const int sa0 = s0.iA, sa1 = s1.iA, sa2 = s2.iA, sb0 = s0.iB, sb1 = s1.iB, sb2 = s2.iB;
        if (count == 2)
            gjk_solve2(s0, s1, count);
        else if (count == 3)
            gjk_solve3(s0, s1, s2, count);
        if (count == 3) break;
        V2 d;
        if (count == 1) {
            d = neg(s0.w);
        } else {
            V2 e12 = sub(s1.w, s0.w);
            float sgn = cross(e12, neg(s0.w));
            d = sgn > 0 ? cross_sv(1.0f, e12) : cross_vs(e12, 1.0f);
        }
        if (dot(d, d) < EPS * EPS) break;
        V2 la, lb;
        int iA = pA.support(rot_t(xfA.q, neg(d)), &la);
        int iB = pB.support(rot_t(xfB.q, d), &lb);
        SV v = make_vertex_at(xfA, la, iA, xfB, lb, iB);
        if (count == 1) {  // the new vertex goes to slot `count`; its weight is left as the slot had it
            v.a = s1.a;
            s1 = v;
        } else {
            v.a = s2.a;
            s2 = v;
        }
        ++it;
        GB_COUNT(9, 1);
        bool dup = (save_count > 0 && sa0 == iA && sb0 == iB) || (save_count > 1 && sa1 == iA && sb1 == iB) ||
                   (save_count > 2 && sa2 == iA && sb2 == iB);
        if (dup) break;
        ++count;
    }
    V2 pa, pb;
    if (count == 1) {
        pa = s0.wA, pb = s0.wB;
    } else if (count == 2) {
        pa = {s0.a * s0.wA.x + s1.a * s1.wA.x, s0.a * s0.wA.y + s1.a * s1.wA.y};
        pb = {s0.a * s0.wB.x + s1.a * s1.wB.x, s0.a * s0.wB.y + s1.a * s1.wB.y};
    } else {
        V2 p2{s0.a * s0.wA.x + s1.a * s1.wA.x, s0.a * s0.wA.y + s1.a * s1.wA.y};
        pa = {p2.x + s2.a * s2.wA.x, p2.y + s2.a * s2.wA.y};
        pb = pa;
    }
    cache.count = count;
    cache.iA[0] = s0.iA, cache.iA[1] = s1.iA, cache.iA[2] = s2.iA;
    cache.iB[0] = s0.iB, cache.iB[1] = s1.iB, cache.iB[2] = s2.iB;
    cache.metric = simplex_metric(s0, s1, s2, count);
    return length(sub(pa, pb));
}

struct SepFn {
    int type;
    V2 axis, lp;
};

__device__ SepFn sep_init(const Cache &cache, const Proxy &pA, Xf xfA, const Proxy &pB, Xf xfB) {  // toi.py:299-326
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

__device__ float sep_eval(const SepFn &f, const Proxy &pA, Xf xfA, int iA, const Proxy &pB, Xf xfB, int iB) {
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

// b2SeparationFunction::FindMinSeparation: the support points, then Evaluate's arithmetic on them (sep_eval)
__device__ float sep_find_min(const SepFn &f, const Proxy &pA, Xf xfA, const Proxy &pB, Xf xfB, int &iA, int &iB) {
    V2 la, lb;
    if (f.type == E_POINTS) {
        iA = pA.support(rot_t(xfA.q, f.axis), &la);
        iB = pB.support(rot_t(xfB.q, neg(f.axis)), &lb);
        V2 pa = xf_mul(xfA, la), pb = xf_mul(xfB, lb);
        return dot(sub(pb, pa), f.axis);
    }
    if (f.type == E_FACE_A) {
        iA = -1;
        V2 n = rot(xfA.q, f.axis);
        iB = pB.support(rot_t(xfB.q, neg(n)), &lb);
        V2 qa = xf_mul(xfA, f.lp), pb = xf_mul(xfB, lb);
        return dot(sub(pb, qa), n);
    }
    iB = -1;
    V2 n = rot(xfB.q, f.axis);
    iA = pA.support(rot_t(xfA.q, neg(n)), &la);
    V2 qb = xf_mul(xfB, f.lp), pa = xf_mul(xfA, la);
    return dot(sub(pa, qb), n);
}

// b2TimeOfImpact with tMax = 1 (toi.py:364-457). Returns the b2TOIOutput state; *t_out its t.
__device__ __forceinline__ int time_of_impact(const Proxy &pA, Sweep swA, const Proxy &pB, Sweep swB, float slop,
                                           float *t_out) {
    const float two_pi = 2.0f * PI_F;
    {  // b2Sweep::Normalize
        float d = two_pi * floorf(swA.a0 / two_pi);
        swA.a0 = swA.a0 - d, swA.a = swA.a - d;
        d = two_pi * floorf(swB.a0 / two_pi);
        swB.a0 = swB.a0 - d, swB.a = swB.a - d;
    }
    float total_radius = pA.radius + pB.radius;
    float target = bmax(slop, total_radius - 3.0f * slop);
    float tol = 0.25f * slop;
    float t1 = 0.0f;
    Cache cache;
    cache.count = 0, cache.metric = 0.0f;
    for (int j = 0; j < 3; ++j) cache.iA[j] = cache.iB[j] = 0;
    for (int iter = 0;;) {
        Xf xfA, xfB;
        float dist;
        {
            GB_TOI_T0();
            xfA = sweep_xf(swA, t1), xfB = sweep_xf(swB, t1);
            GB_TOI_T1(0);
        }
        {
            GB_TOI_T0();
            dist = gjk_distance(cache, pA, xfA, pB, xfB);
            GB_TOI_T1(1);
        }
        GB_COUNT(6, 1);
        if (dist <= 0.0f) {
            *t_out = 0.0f;
            GB_COUNT(13, 1);
            return E_OVERLAPPED;
        }
        if (dist < target + tol) {
            *t_out = t1;
            GB_COUNT(11, 1);
            return E_TOUCHING;
        }
        SepFn f;
        {
            GB_TOI_T0();
            f = sep_init(cache, pA, xfA, pB, xfB);
            GB_TOI_T1(2);
        }
        float t2 = 1.0f;
        for (int push = 0;;) {
            int iA, iB;
            Xf xa2, xb2;
            float s2;
            {
                GB_TOI_T0();
                xa2 = sweep_xf(swA, t2), xb2 = sweep_xf(swB, t2);
                GB_TOI_T1(0);
            }
            {
                GB_TOI_T0();
                s2 = sep_find_min(f, pA, xa2, pB, xb2, iA, iB);
                GB_TOI_T1(3);
            }
            GB_COUNT(7, 1);
            if (s2 > target + tol) {
                *t_out = 1.0f;
                GB_COUNT(10, 1);
                return E_SEPARATED;
            }
            if (s2 > target - tol) {
                t1 = t2;
                break;
            }
            float s1 = sep_eval(f, pA, sweep_xf(swA, t1), iA, pB, sweep_xf(swB, t1), iB);
            if (s1 < target - tol) {
                *t_out = t1;
                GB_COUNT(12, 1);
                return E_FAILED;
            }
            if (s1 <= target + tol) {
                *t_out = t1;
                GB_COUNT(11, 1);
                return E_TOUCHING;
            }
            float a1 = t1, a2 = t2;
            for (int cnt = 0;;) {
                float t = (cnt & 1) ? a1 + ((target - s1) * (a2 - a1)) / (s2 - s1) : 0.5f * (a1 + a2);
                ++cnt;
                GB_COUNT(8, 1);
                float s = sep_eval(f, pA, sweep_xf(swA, t), iA, pB, sweep_xf(swB, t), iB);
                if (babs(s - target) < tol) {
                    t2 = t;
                    break;
                }
                if (s > target)
                    a1 = t, s1 = s;
                else
                    a2 = t, s2 = s;
                if (cnt == 50) break;
            }
            ++push;
            if (push == MAXV) break;
        }
        ++iter;
        if (iter == 20) {
            *t_out = t1;
            GB_COUNT(12, 1);
            return E_FAILED;
        }
    }
}

__device__ __forceinline__ void sweep_advance(float &c0x, float &c0y, float &a0, float &alpha0, float cx, float cy,
                                              float a, float alpha) {  // b2Sweep::Advance (toi.py:100-104)
    float den = 1.0f - alpha0;
    float beta = (alpha - alpha0) / (den != 0 ? den : 1.0f);
    c0x = c0x + beta * (cx - c0x), c0y = c0y + beta * (cy - c0y), a0 = a0 + beta * (a - a0), alpha0 = alpha;
}

__device__ __forceinline__ bool toi_pair_rule(const W &w, int a, int b, bool unity) {  // toi.py:462-470
    bool dyn_a = w.type[a] == DYNAMIC, dyn_b = w.type[b] == DYNAMIC;
    bool stock = w.bullet[a] || !dyn_a || w.bullet[b] || !dyn_b;
    if (!unity) return stock;
    bool rule = (w.bullet[a] || w.bullet[b]) ||
                (!dyn_b ? (bool)w.continuous[a] : (!dyn_a ? (bool)w.continuous[b] : false));
    return stock && rule;
}

}  // namespace gb
