// goib2d State validation (goib2d_validate, and every step while goib2d_set_checks is on): the State's integer fields
// that the step kernels use as indices or loop bounds, checked against the Model before a step is launched, so a
// corrupted State is refused with an error instead of reaching the kernels. The reference trusts its State (its
// kernels have no bounds checks either); compute-sanitizer being unavailable, this is the engine's own guard. The
// kernel compares the fields with their ranges and reads the Model only at a pair index it has checked, so it is
// safe on any State.
#pragma once
#include "engine.cuh"

namespace gb {

// One warp per world (4 per block); lanes over bodies, joints and contact slots.
__global__ void __launch_bounds__(128) goib2d_check_kernel(const __grid_constant__ CheckParams p) {
    const int64_t w = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (w >= p.n_worlds) return;
    const DevModel &m = p.m;
    const int B = m.B, J = m.J, C = p.C;
    unsigned long long bad = ~0ull;
    auto flag = [&](int leaf) {
        const unsigned long long v = ((unsigned long long)w << 8) | (unsigned long long)leaf;
        bad = v < bad ? v : bad;
    };
    const int32_t *type = (const int32_t *)p.L.p[GOIB2D_B_TYPE] + w * B;
    for (int b = lane; b < B; b += 32)
        if (type[b] < STATIC || type[b] > DYNAMIC) flag(GOIB2D_B_TYPE);
    const int32_t *ls = (const int32_t *)p.L.p[GOIB2D_J_LIMIT_STATE] + w * J;
    for (int j = lane; j < J; j += 32)
        if (ls[j] < INACTIVE_LIMIT || ls[j] > EQUAL_LIMITS) flag(GOIB2D_J_LIMIT_STATE);
    const int32_t *pair = (const int32_t *)p.L.p[GOIB2D_C_PAIR] + w * C;
    const int32_t *fa = (const int32_t *)p.L.p[GOIB2D_C_FA] + w * C;
    const int32_t *fb = (const int32_t *)p.L.p[GOIB2D_C_FB] + w * C;
    const int32_t *count = (const int32_t *)p.L.p[GOIB2D_C_COUNT] + w * C;
    const int32_t *mtype = (const int32_t *)p.L.p[GOIB2D_C_MTYPE] + w * C;
    for (int s = lane; s < C; s += 32) {
        const int pr = pair[s];
        if (pr < -1 || pr >= m.P) {
            flag(GOIB2D_C_PAIR);
            continue;
        }
        if (pr < 0) continue;  // an empty slot: its other fields are not read
        if (fa[s] != m.pair_a[pr]) flag(GOIB2D_C_FA);
        if (fb[s] != m.pair_b[pr]) flag(GOIB2D_C_FB);
        if (count[s] < 0 || count[s] > 2) flag(GOIB2D_C_COUNT);
        if (mtype[s] < CIRCLES || mtype[s] > FACE_B) flag(GOIB2D_C_MTYPE);
    }
    for (int o = 16; o; o >>= 1) {
        const unsigned long long v = __shfl_xor_sync(0xffffffffu, bad, o);
        bad = v < bad ? v : bad;
    }
    if (lane == 0 && bad != ~0ull) atomicMin(p.first_bad, bad);
}

cudaError_t launch_check(const CheckParams &p, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(p.first_bad, 0xff, sizeof(unsigned long long), s);
    if (e != cudaSuccess) return e;
    if (p.n_worlds > 0) goib2d_check_kernel<<<(unsigned)((p.n_worlds + 3) / 4), 128, 0, s>>>(p);
    return cudaGetLastError();
}

}  // namespace gb
