// goib2d scene spawn on the device: each world's initial State from one template world and per-world body
// placements (goib2d_spawn), and the placements themselves drawn per world from a seed (goib2d_seed_placements).
// The reference builds every world on the host through WorldDef (world.py:186-386) and stacks them; here one kernel
// broadcasts the template's rows to every world (coalesced over each leaf), then a warp per world places its bodies
// with the same float32 operations as the builder's add_body / set_mass (world.py:196-244) and
// b2BroadPhase::CreateProxy's fat AABB (shapes.py:118-153), so the State is the one the builder makes. Compiled with
// the step (step.cu includes this file).
#pragma once
#include "narrow.cuh"

namespace gb {

// Every world's row of every leaf from the template's (row 0): blockIdx.y = the leaf, the threads stride over the
// leaf's words (bytes where a row is not a whole number of words) across all worlds, so consecutive threads store
// consecutive words - coalesced writes of the whole batch instead of a warp per world over 71 short rows.
__global__ void __launch_bounds__(256) goib2d_spawn_copy_kernel(const __grid_constant__ EnvParams p) {
    const int i = blockIdx.y;
    const uint32_t nb = (uint32_t)p.leaf_bytes[i];
    if (nb == 0) return;
    const uint8_t *src = (const uint8_t *)p.I.p[i];
    uint8_t *dst = (uint8_t *)p.L.p[i];
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t t0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if ((nb & 3) == 0 && (((uintptr_t)dst | (uintptr_t)src) & 3) == 0) {
        const uint32_t nw = nb >> 2;
        const uint64_t tw = (uint64_t)nw * (uint64_t)p.n_worlds;
        if (tw + stride <= 0xffffffffull) {  // 32-bit index arithmetic, no wrap of t + stride (the usual case)
            for (uint32_t t = (uint32_t)t0; t < (uint32_t)tw; t += (uint32_t)stride)
                ((uint32_t *)dst)[t] = ((const uint32_t *)src)[t % nw];
        } else {
            for (uint64_t t = t0; t < tw; t += stride) ((uint32_t *)dst)[t] = ((const uint32_t *)src)[t % nw];
        }
    } else {
        const uint64_t tb = (uint64_t)nb * (uint64_t)p.n_worlds;
        for (uint64_t t = t0; t < tb; t += stride) dst[t] = src[t % nb];
    }
}

// One warp per world (4 per block), after goib2d_spawn_copy_kernel: the placed bodies, their fixture rows' fat AABBs
// and the per-world motor speeds. A placed body's transform is recomputed by every lane that needs it (rot_of is the
// engine's correctly rounded float32 sin/cos, the builder's (float)sin((double)angle)).
__global__ void __launch_bounds__(128) goib2d_spawn_kernel(const __grid_constant__ EnvParams p) {
    const int64_t w = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= p.n_worlds) return;
    const int B = p.B;
    const int32_t *type = (const int32_t *)p.I.p[GOIB2D_B_TYPE];
    const uint8_t *awake = (const uint8_t *)p.I.p[GOIB2D_B_AWAKE];
    const float *lc_t = (const float *)p.I.p[GOIB2D_B_LOCAL_CENTER];
    const float *pl = p.placements + w * (int64_t)p.n_placed * 6;
    float *xf_p = (float *)p.L.p[GOIB2D_B_XF_P] + w * 2 * B;
    float *xf_q = (float *)p.L.p[GOIB2D_B_XF_Q] + w * 2 * B;
    float *c0 = (float *)p.L.p[GOIB2D_B_C0] + w * 2 * B;
    float *c = (float *)p.L.p[GOIB2D_B_C] + w * 2 * B;
    float *a0 = (float *)p.L.p[GOIB2D_B_A0] + w * B;
    float *a = (float *)p.L.p[GOIB2D_B_A] + w * B;
    float *v = (float *)p.L.p[GOIB2D_B_V] + w * 2 * B;
    float *av = (float *)p.L.p[GOIB2D_B_W] + w * B;
    for (int k = lane; k < p.n_placed; k += 32) {
        const int b = p.first_body + k;
        if (type[b] == STATIC) continue;
        const float x = pl[6 * k], y = pl[6 * k + 1], ang = pl[6 * k + 2];
        const float vx = pl[6 * k + 3], vy = pl[6 * k + 4], wv = pl[6 * k + 5];
        const Xf xf{{x, y}, rot_of(ang)};
        const V2 cc = xf_mul(xf, V2{lc_t[2 * b], lc_t[2 * b + 1]});  // set_mass: c = xf * local_center
        xf_p[2 * b] = x, xf_p[2 * b + 1] = y;
        xf_q[2 * b] = xf.q.c, xf_q[2 * b + 1] = xf.q.s;
        c0[2 * b] = cc.x, c0[2 * b + 1] = cc.y, c[2 * b] = cc.x, c[2 * b + 1] = cc.y;
        a0[b] = ang, a[b] = ang;
        // add_body: a velocity is kept when some component is non-zero and the body is awake (SetAwake(false)
        // after SetLinearVelocity zeroes it); the awake flag itself is the template's
        const bool keep = (vx != 0.0f || vy != 0.0f || wv != 0.0f) && awake[b];
        v[2 * b] = keep ? vx : 0.0f, v[2 * b + 1] = keep ? vy : 0.0f;
        av[b] = keep ? wv : 0.0f;
    }
    float *fat = (float *)p.L.p[GOIB2D_F_FAT] + w * 4 * (int64_t)p.rows;
    for (int r = lane; r < p.rows; r += 32) {
        const int f = p.m.row_fixture[r];
        const int b = p.m.fixture_body[f];
        const int k = b - p.first_body;
        if (k < 0 || k >= p.n_placed || type[b] == STATIC) continue;
        const Xf xf{{pl[6 * k], pl[6 * k + 1]}, rot_of(pl[6 * k + 2])};
        const AABB bb = fixture_aabb(p.m, f, xf);
        fat[4 * r] = bb.lx - AABB_EXT, fat[4 * r + 1] = bb.ly - AABB_EXT;
        fat[4 * r + 2] = bb.ux + AABB_EXT, fat[4 * r + 3] = bb.uy + AABB_EXT;
    }
    float *ms = (float *)p.L.p[GOIB2D_J_MOTOR_SPEED] + w * (int64_t)p.J;
    for (int k = lane; k < p.n_speeds; k += 32) ms[p.speed_joint[k]] = p.speeds[w * p.n_speeds + k];
}

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC'11): ten rounds of
// two 32x32->64 multiplies with the round keys bumped by the Weyl constants between rounds.
__device__ __forceinline__ uint4 philox4x32_10(uint4 ctr, uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        if (r) k0 += 0x9E3779B9u, k1 += 0xBB67AE85u;
        const uint32_t lo0 = 0xD2511F53u * ctr.x, hi0 = __umulhi(0xD2511F53u, ctr.x);
        const uint32_t lo1 = 0xCD9E8D57u * ctr.z, hi1 = __umulhi(0xCD9E8D57u, ctr.z);
        ctr = make_uint4(hi1 ^ ctr.y ^ k0, lo1, hi0 ^ ctr.w ^ k1, lo0);
    }
    return ctr;
}

// A world's stream of draws: draw d is word d % 4 of the block (world low, world high, d / 4, 0).
struct WorldDraws {
    uint32_t k0, k1, wlo, whi, block;
    uint4 cur;
    __device__ WorldDraws(uint32_t key0, uint32_t key1, uint64_t world)
        : k0(key0), k1(key1), wlo((uint32_t)world), whi((uint32_t)(world >> 32)), block(0xffffffffu) {}
    __device__ uint32_t word(uint32_t d) {
        const uint32_t b = d >> 2;
        if (b != block) cur = philox4x32_10(make_uint4(wlo, whi, b, 0u), k0, k1), block = b;
        const uint32_t i = d & 3;
        return i == 0 ? cur.x : i == 1 ? cur.y : i == 2 ? cur.z : cur.w;
    }
    __device__ float uniform(uint32_t d, float lo, float hi) {
        const float u = (float)(word(d) >> 8) * 0x1p-24f;
        return lo + (hi - lo) * u;
    }
};

constexpr float TWO_PI_F = 6.28318548202514648f;  // float32(2 pi)

// One thread per world.
__global__ void __launch_bounds__(128) goib2d_seed_kernel(const __grid_constant__ SeedParams p) {
    const int64_t i = (int64_t)blockIdx.x * 128 + threadIdx.x;
    if (i >= p.n_worlds) return;
    const goib2d_spawn_rule &r = p.rule;
    WorldDraws g(p.key0, p.key1, (uint64_t)(p.first_world + i));
    const int nb = r.kind == GOIB2D_SPAWN_RIG ? 3 : r.n_bodies;
    float *out = p.placements + i * (int64_t)nb * 6;
    if (r.kind == GOIB2D_SPAWN_UNIFORM) {
        for (int k = 0; k < nb; ++k) {
            const uint32_t d = 5u * (uint32_t)k;
            const float x = g.uniform(d, r.x_lo, r.x_hi), y = g.uniform(d + 1, r.y_lo, r.y_hi);
            const float ang = g.uniform(d + 2, r.angle_lo, r.angle_hi);
            const float speed = g.uniform(d + 3, r.speed_lo, r.speed_hi);
            const Rot h = rot_of(g.uniform(d + 4, 0.0f, TWO_PI_F));
            float *o = out + 6 * k;
            o[0] = x, o[1] = y, o[2] = ang, o[3] = speed * h.c, o[4] = speed * h.s, o[5] = 0.0f;
        }
    } else if (r.kind == GOIB2D_SPAWN_GRID) {
        for (int k = 0; k < nb; ++k) {
            const uint32_t d = 3u * (uint32_t)k;
            const float gx = (float)(k % r.grid_side) + 0.5f, gy = (float)(k / r.grid_side) + 0.5f;
            const float x = (r.grid_x0 + r.grid_pitch * gx) + g.uniform(d, -r.jitter, r.jitter);
            const float y = (r.grid_y0 + r.grid_pitch * gy) + g.uniform(d + 1, -r.jitter, r.jitter);
            float *o = out + 6 * k;
            o[0] = x, o[1] = y, o[2] = g.uniform(d + 2, r.angle_lo, r.angle_hi), o[3] = 0.0f, o[4] = 0.0f,
            o[5] = 0.0f;
        }
    } else {  // GOIB2D_SPAWN_RIG
        const int last = r.n_heights - 1;
        float x = 0.0f, y = 0.0f;
        for (int t = 0; t < r.max_tries; ++t) {
            x = g.uniform((uint32_t)t, r.x_lo, r.x_hi);
            int i0 = (int)((x - r.half_width - r.h_x0) / r.h_dx), i1 = (int)((x + r.half_width - r.h_x0) / r.h_dx) + 1;
            i0 = i0 < 0 ? 0 : i0 > last ? last : i0;
            i1 = i1 < 0 ? 0 : i1 > last ? last : i1;
            float hi = r.heights[i0], lo = r.heights[i0];
            for (int s = i0 + 1; s <= i1; ++s) {
                const float h = r.heights[s];
                hi = h > hi ? h : hi, lo = h < lo ? h : lo;
            }
            y = hi + r.lift;
            bool ok = lo >= r.min_ground;
            for (int q = 0; q < r.n_discs && ok; ++q) {
                const float dx = x - r.discs[3 * q], dy = y - r.discs[3 * q + 1], rr = r.discs[3 * q + 2] + r.clearance;
                ok = dx * dx + dy * dy > rr * rr;
            }
            if (ok) break;
        }
        const float ang = g.uniform((uint32_t)r.max_tries, r.angle_lo, r.angle_hi);
        const float speed = g.uniform((uint32_t)r.max_tries + 1, r.speed_lo, r.speed_hi);
        const Rot q = rot_of(ang);
        const float rows[3][3] = {{x, y, 0.0f}, {x, y, ang}, {x + r.arm * q.c, y + r.arm * q.s, ang}};
        for (int k = 0; k < 3; ++k) {
            float *o = out + 6 * k;
            o[0] = rows[k][0], o[1] = rows[k][1], o[2] = rows[k][2], o[3] = 0.0f, o[4] = 0.0f, o[5] = 0.0f;
        }
        p.speeds[i] = speed;
    }
}

cudaError_t launch_spawn(const EnvParams &p, cudaStream_t s) {
    if (p.n_worlds <= 0) return cudaSuccess;
    int64_t most = 1;  // the largest leaf's words (bytes) over the batch sets the grid's width
    for (int i = 0; i < GOIB2D_NUM_LEAVES; ++i) most = p.leaf_bytes[i] * p.n_worlds > most ? p.leaf_bytes[i] * p.n_worlds : most;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int64_t bx = (most / 4 + 255) / 256;  // up to 4 blocks of 256 threads per SM for each leaf
    bx = bx < 1 ? 1 : bx > 4 * (int64_t)sms ? 4 * (int64_t)sms : bx;
    goib2d_spawn_copy_kernel<<<dim3((unsigned)bx, GOIB2D_NUM_LEAVES), 256, 0, s>>>(p);
    goib2d_spawn_kernel<<<(unsigned)((p.n_worlds + 3) / 4), 128, 0, s>>>(p);
    return cudaGetLastError();
}
cudaError_t launch_seed(const SeedParams &p, cudaStream_t s) {
    if (p.n_worlds > 0) goib2d_seed_kernel<<<(unsigned)((p.n_worlds + 127) / 128), 128, 0, s>>>(p);
    return cudaGetLastError();
}

}  // namespace gb
