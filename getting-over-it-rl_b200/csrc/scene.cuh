// goib2d scene build on the device: the candidate-pair list of a Model (the host builder's O(F^2) scan of every
// fixture pair, goib2d/world.py WorldDef.candidate_pairs, after reference world.py:308-329), one thread per fixture
// row: a counting pass, a host-side exclusive sum of the row counts, a filling pass that writes each row's pairs in
// ascending partner order - so the list comes out in b2BroadPhase::UpdatePairs order, as the host builds it.
// Compiled with the step (step.cu includes this file).
#pragma once
#include "b2dev.cuh"

namespace gb {


__device__ __forceinline__ bool pair_ok(const PairScene &s, int i, int k) {
    int bi = s.fixture_body[i], bk = s.fixture_body[k];
    if (bi == bk || s.sensor[i] || s.sensor[k]) return false;
    if (s.shape_type[i] == EDGE && s.shape_type[k] == EDGE) return false;  // no edge-edge collider
    if (s.body_type[bi] == STATIC && s.body_type[bk] == STATIC) return false;
    int64_t key = bi < bk ? ((int64_t)bi << 32) | bk : ((int64_t)bk << 32) | bi;
    int lo = 0, hi = s.n_no_collide;  // joined without collideConnected
    while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if (s.no_collide[mid] < key)
            lo = mid + 1;
        else
            hi = mid;
    }
    if (lo < s.n_no_collide && s.no_collide[lo] == key) return false;
    if (s.layer_masks) return ((s.layer_masks[s.layer[i] & 31] >> (s.layer[k] & 31)) & 1u) != 0;  // Unity layers
    if (s.group[i] == s.group[k] && s.group[i] != 0) return s.group[i] > 0;  // b2Filter groups
    return (s.mask[i] & s.category[k]) != 0 && (s.category[i] & s.mask[k]) != 0;
}

__global__ void goib2d_pair_count_kernel(const __grid_constant__ PairScene s, int64_t *count) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= s.F) return;
    int64_t n = 0;
    for (int k = i + 1; k < s.F; ++k) n += pair_ok(s, i, k);
    count[i] = n;
}

// b2Contact::Create's primary order: the edge first, the polygon before the circle
__global__ void goib2d_pair_fill_kernel(const __grid_constant__ PairScene s, const int64_t *start, int32_t *pa,
                                        int32_t *pb) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= s.F) return;
    int64_t o = start[i];
    for (int k = i + 1; k < s.F; ++k) {
        if (!pair_ok(s, i, k)) continue;
        bool k_first = (s.shape_type[i] == CIRCLE && s.shape_type[k] == POLYGON) || s.shape_type[k] == EDGE;
        pa[o] = k_first ? k : i, pb[o] = k_first ? i : k;
        ++o;
    }
}

cudaError_t launch_pair_count(const PairScene &s, int64_t *count) {
    if (s.F > 0) goib2d_pair_count_kernel<<<(s.F + 127) / 128, 128>>>(s, count);
    return cudaGetLastError();
}
cudaError_t launch_pair_fill(const PairScene &s, const int64_t *start, int32_t *pa, int32_t *pb) {
    if (s.F > 0) goib2d_pair_fill_kernel<<<(s.F + 127) / 128, 128>>>(s, start, pa, pb);
    return cudaGetLastError();
}

}  // namespace gb
