// goib2d device math: Box2D 2.3.1's b2Math in float32 with one rounding per C operation.
//
// Built with -fmad=false (no multiply-add contraction), IEEE division and square root, denormals kept: every
// expression below rounds exactly as Box2D compiled with -ffp-contract=off does, in the evaluation order of the
// reference engine goi_jax/box2d/math2d.py (whose functions are cited per helper).
#pragma once
#include <cstdint>

namespace gb {

constexpr float EPS = 1.1920928955078125e-07f;  // b2_epsilon
constexpr float MAXF = 3.4028234663852886e+38f;  // b2_maxFloat
constexpr float PI_F = 3.14159265359f;           // b2_pi
constexpr int MAXV = 8;                          // b2_maxPolygonVertices
constexpr float AABB_EXT = 0.1f, AABB_MUL = 2.0f;
constexpr int MAX_SUB_STEPS = 8, MAX_TOI_CONTACTS = 32;
constexpr float MAX_COND = 1000.0f, K_TOL = 0.1f;
enum { STATIC = 0, KINEMATIC = 1, DYNAMIC = 2 };
enum { REVOLUTE = 1, PRISMATIC = 2, WELD = 8, MOTOR = 11 };  // b2JointType (MOTOR: no counterpart in the reference engine)
enum { INACTIVE_LIMIT = 0, AT_LOWER = 1, AT_UPPER = 2, EQUAL_LIMITS = 3 };
enum { CIRCLES = 0, FACE_A = 1, FACE_B = 2 };
enum { CIRCLE = 0, EDGE = 1, POLYGON = 2 };

struct V2 {
    float x, y;
};
struct Rot {
    float c, s;
};
struct Xf {
    V2 p;
    Rot q;
};
struct V3 {
    float x, y, z;
};
struct AABB {
    float lx, ly, ux, uy;
};

#define GBD __device__ __forceinline__

GBD V2 add(V2 a, V2 b) { return {a.x + b.x, a.y + b.y}; }
GBD V2 sub(V2 a, V2 b) { return {a.x - b.x, a.y - b.y}; }
GBD V2 neg(V2 a) { return {-a.x, -a.y}; }
GBD float dot(V2 a, V2 b) { return a.x * b.x + a.y * b.y; }          // math2d.py:39-41
GBD float cross(V2 a, V2 b) { return a.x * b.y - a.y * b.x; }        // math2d.py:44-46
GBD V2 cross_vs(V2 a, float s) { return {s * a.y, -s * a.x}; }       // math2d.py:49-51
GBD V2 cross_sv(float s, V2 a) { return {-s * a.y, s * a.x}; }       // math2d.py:54-56
GBD V2 rot(Rot q, V2 v) { return {q.c * v.x - q.s * v.y, q.s * v.x + q.c * v.y}; }    // math2d.py:64-66
GBD V2 rot_t(Rot q, V2 v) { return {q.c * v.x + q.s * v.y, -q.s * v.x + q.c * v.y}; }  // math2d.py:69-71
GBD V2 xf_mul(Xf t, V2 v) {  // math2d.py:74-76
    return {(t.q.c * v.x - t.q.s * v.y) + t.p.x, (t.q.s * v.x + t.q.c * v.y) + t.p.y};
}
GBD V2 xf_mul_t(Xf t, V2 v) {  // math2d.py:79-82
    float dx = v.x - t.p.x, dy = v.y - t.p.y;
    return {t.q.c * dx + t.q.s * dy, -t.q.s * dx + t.q.c * dy};
}
GBD float length(V2 a) { return sqrtf(a.x * a.x + a.y * a.y); }
GBD V2 normalize(V2 a) {  // math2d.py:102-107
    float n = length(a);
    if (n < EPS) return a;
    float inv = 1.0f / n;
    return {a.x * inv, a.y * inv};
}
GBD float bmin(float a, float b) { return a < b ? a : b; }
GBD float bmax(float a, float b) { return a > b ? a : b; }
GBD float babs(float a) { return a > 0 ? a : -a; }
GBD float clampf(float a, float lo, float hi) { return bmax(lo, bmin(a, hi)); }
GBD float inv_or_zero(float x) { return x != 0 ? 1.0f / x : 0.0f; }
GBD float inv_if_pos(float x) { return x > 0 ? 1.0f / x : 0.0f; }

GBD V2 solve22(float a11, float a12, float a21, float a22, float bx, float by) {  // math2d.py:162-165
    float det = inv_or_zero(a11 * a22 - a12 * a21);
    return {det * (a22 * bx - a12 * by), det * (a11 * by - a21 * bx)};
}
// The same solves with the inverse determinant given: a constraint whose K stays fixed over the velocity iterations
// computes it once (same operands, so the same float as the solves above compute on every call).
GBD float det22_inv(float a11, float a12, float a21, float a22) { return inv_or_zero(a11 * a22 - a12 * a21); }
GBD V2 solve22d(float a11, float a12, float a21, float a22, float bx, float by, float det) {
    return {det * (a22 * bx - a12 * by), det * (a11 * by - a21 * bx)};
}
GBD V3 cross3(V3 a, V3 b) { return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x}; }
GBD float dot3(V3 a, V3 b) { return (a.x * b.x + a.y * b.y) + a.z * b.z; }
GBD V3 solve33(V3 ex, V3 ey, V3 ez, V3 b) {  // math2d.py:178-182
    float det = inv_or_zero(dot3(ex, cross3(ey, ez)));
    return {det * dot3(b, cross3(ey, ez)), det * dot3(ex, cross3(b, ez)), det * dot3(ex, cross3(ey, b))};
}
GBD float det33_inv(V3 ex, V3 ey, V3 ez) { return inv_or_zero(dot3(ex, cross3(ey, ez))); }
GBD V3 solve33d(V3 ex, V3 ey, V3 ez, V3 b, float det) {
    return {det * dot3(b, cross3(ey, ez)), det * dot3(ex, cross3(b, ez)), det * dot3(ex, cross3(ey, b))};
}
GBD void inverse22_of33(V3 ex, V3 ey, V3 &ox, V3 &oy, V3 &oz) {  // math2d.py:185-190
    float a = ex.x, b = ey.x, c = ex.y, d = ey.y;
    float det = inv_or_zero(a * d - b * c);
    ox = {det * d, -det * c, 0.0f};
    oy = {-det * b, det * a, 0.0f};
    oz = {0.0f, 0.0f, 0.0f};
}
GBD void sym_inverse33(V3 ex, V3 ey, V3 ez, V3 &ox, V3 &oy, V3 &oz) {  // math2d.py:193-205
    float det = inv_or_zero(dot3(ex, cross3(ey, ez)));
    float a11 = ex.x, a12 = ey.x, a13 = ez.x, a22 = ey.y, a23 = ez.y, a33 = ez.z;
    float exx = det * (a22 * a33 - a23 * a23);
    float exy = det * (a13 * a23 - a12 * a33);
    float exz = det * (a12 * a23 - a13 * a22);
    float eyy = det * (a11 * a33 - a13 * a13);
    float eyz = det * (a13 * a12 - a11 * a23);
    float ezz = det * (a11 * a22 - a12 * a12);
    ox = {exx, exy, exz};
    oy = {exy, eyy, eyz};
    oz = {exz, eyz, ezz};
}
GBD V3 mat33_mul(V3 ex, V3 ey, V3 ez, V3 v) {  // math2d.py:208-210
    return {(v.x * ex.x + v.y * ey.x) + v.z * ez.x, (v.x * ex.y + v.y * ey.y) + v.z * ez.y,
            (v.x * ex.z + v.y * ey.z) + v.z * ez.z};
}
GBD V2 mat33_mul22(V3 ex, V3 ey, V2 v) { return {ex.x * v.x + ey.x * v.y, ex.y * v.x + ey.y * v.y}; }

GBD bool overlap(const AABB &a, const AABB &b) {  // b2TestOverlap (shapes.py:149-153)
    float d1x = b.lx - a.ux, d1y = b.ly - a.uy, d2x = a.lx - b.ux, d2y = a.ly - b.uy;
    return !((d1x > 0) || (d1y > 0) || (d2x > 0) || (d2y > 0));
}

// ---------------------------------------------------------------- correctly rounded sin / cos
// Float-float evaluation (Dekker/Knuth exact products and sums on (hi, lo) float32 pairs): Cody-Waite reduction
// by pi/2 in three float32 parts, then the Taylor series of sin and cos to degree 19/18 in float-float, rounded once.
// The method and its constants are the reference's (math2d.py:218-316); the result equals (float)sin((double)x).
struct FF {
    float h, l;
};
GBD float ff_hi(float a) { return __uint_as_float(__float_as_uint(a) & 0xFFFFF000u); }
GBD FF two_prod(float a, float b) {
    float p = a * b;
    float ah = ff_hi(a), al = a - ah, bh = ff_hi(b), bl = b - bh;
    return {p, (((ah * bh - p) + ah * bl) + al * bh) + al * bl};
}
GBD FF two_sum(float a, float b) {
    float s = a + b;
    float bb = s - a;
    return {s, (a - (s - bb)) + (b - bb)};
}
GBD FF fast_two_sum(float a, float b) {
    float s = a + b;
    return {s, b - (s - a)};
}
GBD FF ff_add(FF a, FF b) {
    FF s = two_sum(a.h, b.h), t = two_sum(a.l, b.l);
    FF u = fast_two_sum(s.h, s.l + t.h);
    return fast_two_sum(u.h, u.l + t.l);
}
GBD FF ff_mul(FF a, FF b) {
    FF p = two_prod(a.h, b.h);
    return fast_two_sum(p.h, p.l + (a.h * b.l + a.l * b.h));
}

static __device__ __constant__ float k_sin_c[10][2] = {
    {0x1p+0f, 0x0p+0f}, {-0x1.555556p-3f, 0x1.555556p-28f}, {0x1.111112p-7f, -0x1.dddddep-32f},
    {-0x1.a01a02p-13f, 0x1.7f97fap-39f}, {0x1.71de3ap-19f, 0x1.55b1ccp-45f}, {-0x1.ae6456p-26f, -0x1.fd5138p-52f},
    {0x1.612462p-33f, -0x1.8af25ep-58f}, {-0x1.ae7f3ep-41f, -0x1.ccee08p-67f}, {0x1.952c78p-49f, -0x1.f9ea56p-74f},
    {-0x1.2f49b4p-57f, -0x1.a05056p-83f}};
static __device__ __constant__ float k_cos_c[10][2] = {
    {0x1p+0f, 0x0p+0f}, {-0x1p-1f, 0x0p+0f}, {0x1.555556p-5f, -0x1.555556p-30f}, {-0x1.6c16c2p-10f, 0x1.27d27ep-35f},
    {0x1.a01a02p-16f, -0x1.7f97fap-42f}, {-0x1.27e4fcp-22f, 0x1.10ec14p-47f}, {0x1.1eed8ep-29f, 0x1.ff1b14p-54f},
    {-0x1.93974ap-37f, -0x1.180f94p-62f}, {0x1.ae7f3ep-45f, 0x1.ccee08p-71f}, {-0x1.682786p-53f, -0x1.dcbeccp-80f}};

static __device__ __noinline__ Rot rot_of_ff(float x) {
    const float pio2_0 = 0x1.921fb6p+0f, pio2_1 = -0x1.777a5cp-25f, pio2_2 = -0x1.ee59dap-50f;
    const float two_over_pi = 0x1.45f306p-1f;
    float k = rintf(x * two_over_pi);
    FF p1 = two_prod(k, pio2_0);
    FF r = ff_add(FF{x, 0.0f}, FF{-p1.h, -p1.l});
    FF p2 = two_prod(k, pio2_1);
    r = ff_add(r, FF{-p2.h, -p2.l});
    r = ff_add(r, FF{-(k * pio2_2), 0.0f});
    FF r2 = ff_mul(r, r);
    FF sp{k_sin_c[9][0], k_sin_c[9][1]}, cp{k_cos_c[9][0], k_cos_c[9][1]};
#pragma unroll
    for (int i = 8; i >= 0; --i) {
        sp = ff_add(ff_mul(sp, r2), FF{k_sin_c[i][0], k_sin_c[i][1]});
        cp = ff_add(ff_mul(cp, r2), FF{k_cos_c[i][0], k_cos_c[i][1]});
    }
    sp = ff_mul(r, sp);
    float s = sp.h + sp.l, c = cp.h + cp.l;
    int q = ((int)k % 4 + 4) % 4;
    float sn = q == 0 ? s : q == 1 ? c : q == 2 ? -s : -c;
    float cs = q == 0 ? c : q == 1 ? -s : q == 2 ? -c : s;
    return {cs, x == 0 ? x : sn};
}

// The same values, fast: sin and cos in double precision (sincos_short, below) rounded once to float, which is the
// correct rounding of sin(x) / cos(x) unless the double lies within 2^-36 (relative) of a midpoint between two
// floats; those arguments, and |x| > ROT_FAST_MAX, take rot_of_ff. Checked equal to rot_of_ff, bit for bit, on every
// float32 argument (rot_check.cu runs the sweep; with CUDA's double sincos in place of sincos_short and no cutoff,
// the first difference is at |x| = 2^24, where the float-float reduction drifts from the true value).
constexpr float ROT_FAST_MAX = 0x1p+16f;
// Rounding a normal double to float looks only at the 29 bits it drops: the double is |low29 - 2^28| of its own
// ulps from the float midpoint that decides the rounding. ROT_CLEAR such ulps is 2^-36 of |d| at least.
constexpr long long ROT_CLEAR = 1LL << 17;
GBD bool rounds_clear(double d) {  // false also for doubles below the normal float range
    long long b = __double_as_longlong(d);
    long long low = b & 0x1FFFFFFFLL, dist = low - 0x10000000LL;
    return ((b >> 52) & 0x7FF) > 1023 - 126 && (dist > ROT_CLEAR || dist < -ROT_CLEAR);
}
// sin and cos in double for |x| <= ROT_FAST_MAX, short latency: Cody-Waite reduction by pi/2 in two parts (PIO2_HI
// has 35 significant bits, so k * PIO2_HI is exact for |k| < 2^17, and x - k * PIO2_HI is exact by Sterbenz), then
// the Taylor series of sin to r^13 and of cos to r^14 on |r| <= pi/4, Horner in r^2 with fused multiply-adds.
// Truncation below 2^-44 relative, reduction error below 2^-70: far inside the rounding test's 2^-36. The constants are pi/2 split
// from a 78-digit Machin-formula value of pi, and 1/n!.
GBD void sincos_short(double x, double &sn, double &cs) {
    const double TWO_OVER_PI = 0x1.45f306dc9c883p-1, PIO2_HI = 0x1.921fb54440000p+0, PIO2_LO = 0x1.68c234c4c6629p-39;
    double k = rint(x * TWO_OVER_PI);
    double r = fma(-k, PIO2_LO, x - k * PIO2_HI);
    double r2 = r * r;
    double ps = fma(r2, 1.0 / 6227020800.0, -1.0 / 39916800.0);
    ps = fma(r2, ps, 1.0 / 362880.0);
    ps = fma(r2, ps, -1.0 / 5040.0);
    ps = fma(r2, ps, 1.0 / 120.0);
    ps = fma(r2, ps, -1.0 / 6.0);
    double pc = fma(r2, -1.0 / 87178291200.0, 1.0 / 479001600.0);
    pc = fma(r2, pc, -1.0 / 3628800.0);
    pc = fma(r2, pc, 1.0 / 40320.0);
    pc = fma(r2, pc, -1.0 / 720.0);
    pc = fma(r2, pc, 1.0 / 24.0);
    pc = fma(r2, pc, -0.5);
    double s = fma(r * r2, ps, r), c = fma(r2, pc, 1.0);
    int q = (int)k & 3;
    sn = q == 0 ? s : q == 1 ? c : q == 2 ? -s : -c;
    cs = q == 0 ? c : q == 1 ? -s : q == 2 ? -c : s;
}
GBD bool rot_fast(float x, Rot &q) {  // false: the argument needs rot_of_ff
    if (!(fabsf(x) <= ROT_FAST_MAX)) return false;
    if (x == 0.0f) {
        q = {1.0f, x};
        return true;
    }
    double sd, cd;
    sincos_short((double)x, sd, cd);
    float s = __double2float_rn(sd), c = __double2float_rn(cd);
    q = {c, s};
    return rounds_clear(sd) && rounds_clear(cd);
}
static __device__ __noinline__ Rot rot_of(float x) {
    Rot q;
    return rot_fast(x, q) ? q : rot_of_ff(x);
}

GBD Xf xf_from(V2 c, float a, V2 lc) {  // b2Body::SynchronizeTransform: q.Set(a); p = c - q lc
    Rot q = rot_of(a);
    V2 r = rot(q, lc);
    return {{c.x - r.x, c.y - r.y}, q};
}
GBD Xf xf_from_q(V2 c, Rot q, V2 lc) {
    V2 r = rot(q, lc);
    return {{c.x - r.x, c.y - r.y}, q};
}

}  // namespace gb
