// goib2d rot_of self-check: compares the fast double-precision path of rot_of with the float-float evaluation
// rot_of_ff over float32 bit patterns, bit for bit. Test support only (libgoib2d_rotcheck.so); the engine does not
// link it.
#include <cstdint>
#include <cstdio>

#include "b2dev.cuh"

using namespace gb;

// out[0] arguments checked, out[1] differing results, out[2] arguments sent to rot_of_ff, out[3] lowest differing
// pattern, out[4 + e] differing results per biased exponent e of the argument
__global__ void rot_check_kernel(uint64_t lo, uint64_t hi, uint64_t stride, unsigned long long *out) {
    unsigned long long checked = 0, bad = 0, slow = 0;
    for (uint64_t i = lo + ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) * stride; i < hi;
         i += (uint64_t)gridDim.x * blockDim.x * stride) {
        uint32_t bits = (uint32_t)i;
        float x = __uint_as_float(bits);
        if (!isfinite(x)) continue;
        ++checked;
        Rot f;
        bool fast = rot_fast(x, f);
        if (!fast) {
            ++slow;
            continue;
        }
        Rot r = rot_of_ff(x);
        if (__float_as_uint(f.c) != __float_as_uint(r.c) || __float_as_uint(f.s) != __float_as_uint(r.s)) {
            ++bad;
            atomicMin(&out[3], (unsigned long long)bits);
            atomicAdd(&out[4 + ((bits >> 23) & 0xff)], 1ull);
        }
    }
    atomicAdd(&out[0], checked);
    atomicAdd(&out[1], bad);
    atomicAdd(&out[2], slow);
}

// Checks the patterns lo, lo + stride, ... below hi (hi <= 2^32) in launches of at most 2^26 patterns; host_out
// receives the 260 counters above. Returns 0, or the CUDA error code.
extern "C" int goib2d_rot_check(uint64_t lo, uint64_t hi, uint64_t stride, unsigned long long *host_out) {
    unsigned long long *d = nullptr;
    cudaError_t e = cudaMalloc(&d, 260 * sizeof(unsigned long long));
    if (e != cudaSuccess) return (int)e;
    cudaMemset(d, 0, 260 * sizeof(unsigned long long));
    unsigned long long init = ~0ull;
    cudaMemcpy(d + 3, &init, sizeof(init), cudaMemcpyHostToDevice);
    if (stride == 0) stride = 1;
    const uint64_t chunk = (uint64_t)1 << 26;
    for (uint64_t a = lo; a < hi; a += chunk * stride) {
        uint64_t b = a + chunk * stride < hi ? a + chunk * stride : hi;
        rot_check_kernel<<<148 * 8, 256>>>(a, b, stride, d);
        if ((e = cudaGetLastError()) != cudaSuccess) break;
    }
    if (e == cudaSuccess) e = cudaMemcpy(host_out, d, 260 * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    cudaFree(d);
    return (int)e;
}
