// goib2d env helpers around the step (no counterpart in the reference engine, whose env lives in a module that is
// not part of it): resets of whole worlds to an initial State, observation gathers, and ray casts from a body
// against the world's static level. All are one thread or one warp per world, in the caller's stream. Compiled
// with the step (step.cu includes this file), so the device helpers exist once.
#pragma once
#include "narrow.cuh"

namespace gb {


// One warp per world: copy every leaf's row of world w from the initial State when the world resets.
__global__ void __launch_bounds__(128) goib2d_reset_kernel(const __grid_constant__ EnvParams p) {
    const int64_t w = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= p.n_worlds) return;
    bool reset;
    if (p.mask) {
        reset = p.mask[w] != 0;
    } else {
        const float *c = (const float *)p.L.p[GOIB2D_B_C] + w * 2 * p.B;
        reset = c[2 * p.body + 1] < p.y_min;
    }
    if (!reset) return;
    for (int i = 0; i < GOIB2D_NUM_LEAVES; ++i) {
        const int64_t nb = p.leaf_bytes[i];
        const uint8_t *src = (const uint8_t *)p.I.p[i] + w * nb;
        uint8_t *dst = (uint8_t *)p.L.p[i] + w * nb;
        for (int64_t k = lane; k < nb; k += 32) dst[k] = src[k];
    }
    if (lane == 0 && p.reset_count) p.reset_count[w] += 1;
}

// One thread per (world, observed body): position, angle, linear and angular velocity. A block's rows are gathered
// in shared memory and written out as consecutive floats (each warp store a whole 128-byte line), which matters
// when out is pinned host memory written over the bus.
constexpr int OBS_THREADS = 256;
__global__ void __launch_bounds__(OBS_THREADS) goib2d_observe_kernel(const __grid_constant__ EnvParams p) {
    __shared__ float stage[OBS_THREADS * 6];
    const int64_t total = p.n_worlds * p.n_obs;
    const int64_t t = (int64_t)blockIdx.x * OBS_THREADS + threadIdx.x;
    if (t < total) {
        const int64_t w = t / p.n_obs;
        const int b = p.obs_body[t % p.n_obs];
        const float *c = (const float *)p.L.p[GOIB2D_B_C] + w * 2 * p.B;
        const float *a = (const float *)p.L.p[GOIB2D_B_A] + w * p.B;
        const float *v = (const float *)p.L.p[GOIB2D_B_V] + w * 2 * p.B;
        const float *av = (const float *)p.L.p[GOIB2D_B_W] + w * p.B;
        float *o = stage + threadIdx.x * 6;
        o[0] = c[2 * b], o[1] = c[2 * b + 1], o[2] = a[b], o[3] = v[2 * b], o[4] = v[2 * b + 1], o[5] = av[b];
    }
    __syncthreads();
    const int64_t base = (int64_t)blockIdx.x * OBS_THREADS * 6, end = total * 6;
    for (int i = threadIdx.x; i < OBS_THREADS * 6; i += OBS_THREADS)
        if (base + i < end) p.out[base + i] = stage[i];
}

// ---- ray casts (b2RayCastInput p1 -> p2, maxFraction 1; each shape's hit fraction along p1 -> p2)
__device__ __forceinline__ float ray_circle(V2 p1, V2 d, V2 centre, float r) {  // b2CircleShape::RayCast
    V2 s = sub(p1, centre);
    float b = dot(s, s) - r * r;
    float c = dot(s, d), rr = dot(d, d);
    float sigma = c * c - rr * b;
    if (sigma < 0.0f || rr < EPS) return 1.0f;
    float a = -(c + sqrtf(sigma));
    if (0.0f <= a && a <= rr) return a / rr;
    return 1.0f;
}
__device__ __forceinline__ float ray_polygon(V2 p1, V2 d, const Poly &pg) {  // b2PolygonShape::RayCast (local frame)
    float lower = 0.0f, upper = 1.0f;
    int index = -1;
    for (int i = 0; i < pg.count; ++i) {
        float num = dot(pg.norm(i), sub(pg.vert(i), p1)), den = dot(pg.norm(i), d);
        if (den == 0.0f) {
            if (num < 0.0f) return 1.0f;
        } else if (den < 0.0f && num < lower * den) {
            lower = num / den, index = i;
        } else if (den > 0.0f && num < upper * den) {
            upper = num / den;
        }
        if (upper < lower) return 1.0f;
    }
    return index >= 0 ? lower : 1.0f;
}
__device__ __forceinline__ float ray_edge(V2 p1, V2 d, V2 v1, V2 v2) {  // b2EdgeShape::RayCast (local frame)
    V2 e = sub(v2, v1);
    V2 n = normalize(V2{e.y, -e.x});
    float num = dot(n, sub(v1, p1)), den = dot(n, d);
    if (den == 0.0f) return 1.0f;
    float t = num / den;
    if (t < 0.0f || 1.0f < t) return 1.0f;
    V2 q{p1.x + t * d.x, p1.y + t * d.y};
    float rr = dot(e, e);
    if (rr == 0.0f) return 1.0f;
    float s = dot(sub(q, v1), e) / rr;
    if (s < 0.0f || 1.0f < s) return 1.0f;
    return t;
}
// the hit fraction of fixture f (body transform xf) for the world-frame ray p1 + t d, t in [0, 1]
__device__ float ray_fixture(const DevModel &m, int f, Xf xf, V2 p1, V2 d) {
    V2 lp = xf_mul_t(xf, p1), ld = rot_t(xf.q, d);
    int t = m.shape_type[f];
    const float *v = m.verts + 16 * f;
    if (t == CIRCLE) return ray_circle(lp, ld, V2{v[0], v[1]}, m.radius[f]);
    if (t == EDGE) return ray_edge(lp, ld, V2{v[0], v[1]}, V2{v[2], v[3]});
    return ray_polygon(lp, ld, poly_of(m, f));
}

// One thread per (world, ray): ray k leaves body `body`'s centre of mass in direction 2 pi k / n_rays (world
// frame) for max_length; out = the nearest hit fraction over the static level's fixtures (1 = none). Compact models
// visit the static-fixture grid cells under the ray's box; otherwise every fixture of a static body is tested.
__global__ void goib2d_raycast_kernel(const __grid_constant__ EnvParams p) {
    const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= p.n_worlds * p.n_rays) return;
    const int64_t w = t / p.n_rays;
    const int k = (int)(t % p.n_rays);
    const DevModel &m = p.m;
    const float *c = (const float *)p.L.p[GOIB2D_B_C] + w * 2 * p.B;
    const float *xp = (const float *)p.L.p[GOIB2D_B_XF_P] + w * 2 * p.B;
    const float *xq = (const float *)p.L.p[GOIB2D_B_XF_Q] + w * 2 * p.B;
    const int32_t *type = (const int32_t *)p.L.p[GOIB2D_B_TYPE] + w * p.B;
    const Rot dir = rot_of((float)k * (2.0f * PI_F / (float)p.n_rays));
    const V2 p1{c[2 * p.body], c[2 * p.body + 1]};
    const V2 d{p.max_length * dir.c, p.max_length * dir.s};
    float best = 1.0f;
    auto test = [&](int f) {
        int b = m.fixture_body[f];
        Xf xf{{xp[2 * b], xp[2 * b + 1]}, {xq[2 * b], xq[2 * b + 1]}};
        best = fminf(best, ray_fixture(m, f, xf, p1, d));
    };
    if (m.grid) {
        const V2 p2{p1.x + d.x, p1.y + d.y};
        int cx0 = grid_cell(fminf(p1.x, p2.x), m.gx0, m.inv_cell, m.nx);
        int cx1 = grid_cell(fmaxf(p1.x, p2.x), m.gx0, m.inv_cell, m.nx);
        int cy0 = grid_cell(fminf(p1.y, p2.y), m.gy0, m.inv_cell, m.ny);
        int cy1 = grid_cell(fmaxf(p1.y, p2.y), m.gy0, m.inv_cell, m.ny);
        for (int cy = cy0; cy <= cy1; ++cy)
            for (int cx = cx0; cx <= cx1; ++cx) {
                int cell = cy * m.nx + cx;
                for (int i = m.cell_start[cell]; i < m.cell_start[cell + 1]; ++i) test(m.sfix[m.cell_items[i]]);
            }
    } else {
        for (int f = 0; f < m.F; ++f)
            if (type[m.fixture_body[f]] == STATIC) test(f);
    }
    p.out[t] = best;
}

cudaError_t launch_reset(const EnvParams &p, cudaStream_t s) {
    if (p.n_worlds > 0) goib2d_reset_kernel<<<(unsigned)((p.n_worlds + 3) / 4), 128, 0, s>>>(p);
    return cudaGetLastError();
}
cudaError_t launch_observe(const EnvParams &p, cudaStream_t s) {
    int64_t n = p.n_worlds * p.n_obs;
    if (n > 0) goib2d_observe_kernel<<<(unsigned)((n + OBS_THREADS - 1) / OBS_THREADS), OBS_THREADS, 0, s>>>(p);
    return cudaGetLastError();
}
cudaError_t launch_raycast(const EnvParams &p, cudaStream_t s) {
    int64_t n = p.n_worlds * p.n_rays;
    if (n > 0) goib2d_raycast_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(p);
    return cudaGetLastError();
}

}  // namespace gb
