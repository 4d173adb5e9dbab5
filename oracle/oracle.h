// Parity oracle: a scalar C++ restatement of the reference engine goi_jax/box2d (miwate/getting-over-it-rl), one
// world at a time. TEST INFRASTRUCTURE ONLY - the checker for the CUDA engine, the timed CPU baseline of bench.py,
// never part of the product path (getting-over-it-rl_b200/ links nothing from here).
//
// Parity is pinned: tests/golden/*.npz hold states produced by the reference's own Python engine (stepped through
// tests/golden/jaxshim, a numpy stand-in for jax), and tests/test_oracle.py requires this oracle to reproduce them
// bit for bit. Each function cites the reference file:line it restates.
//
// Floating point: every C operation is one float32 rounding in the reference's order, as Box2D built with
// -ffp-contract=off computes it (reference math2d.py:1-13); build with -O2 -ffp-contract=off -fno-fast-math.
#pragma once
#include <cmath>
#include <cstdint>
#include <cstring>

#include "../include/goib2d.h"

namespace orc {

constexpr float EPS = 1.1920928955078125e-07f;  // b2_epsilon = FLT_EPSILON (settings.py:86)
constexpr float MAXF = 3.4028234663852886e+38f;  // b2_maxFloat = FLT_MAX
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
static inline V2 v2(float x, float y) { return V2{x, y}; }
static inline V2 add(V2 a, V2 b) { return {a.x + b.x, a.y + b.y}; }
static inline V2 sub(V2 a, V2 b) { return {a.x - b.x, a.y - b.y}; }
static inline V2 neg(V2 a) { return {-a.x, -a.y}; }
static inline V2 smul(float s, V2 a) { return {s * a.x, s * a.y}; }
static inline float dot(V2 a, V2 b) { return a.x * b.x + a.y * b.y; }
static inline float cross(V2 a, V2 b) { return a.x * b.y - a.y * b.x; }
static inline V2 cross_vs(V2 a, float s) { return {s * a.y, -s * a.x}; }  // b2Cross(v, s)
static inline V2 cross_sv(float s, V2 a) { return {-s * a.y, s * a.x}; }  // b2Cross(s, v)
struct Rot {
    float c, s;
};
static inline V2 rot(Rot q, V2 v) { return {q.c * v.x - q.s * v.y, q.s * v.x + q.c * v.y}; }
static inline V2 rot_t(Rot q, V2 v) { return {q.c * v.x + q.s * v.y, -q.s * v.x + q.c * v.y}; }
struct Xf {
    V2 p;
    Rot q;
};
// b2Mul(T, v) = (q.c v.x - q.s v.y) + p.x, (q.s v.x + q.c v.y) + p.y  (math2d.py:74-76)
static inline V2 xf_mul(Xf t, V2 v) { return {(t.q.c * v.x - t.q.s * v.y) + t.p.x, (t.q.s * v.x + t.q.c * v.y) + t.p.y}; }
static inline V2 xf_mul_t(Xf t, V2 v) {  // math2d.py:79-82
    float dx = v.x - t.p.x, dy = v.y - t.p.y;
    return {t.q.c * dx + t.q.s * dy, -t.q.s * dx + t.q.c * dy};
}
static inline float length(V2 a) { return std::sqrt(a.x * a.x + a.y * a.y); }
// b2Vec2::Normalize (math2d.py:102-107): unchanged below b2_epsilon
static inline V2 normalize(V2 a, float *len = nullptr) {
    float n = length(a);
    if (n < EPS) {
        if (len) *len = 0.0f;
        return a;
    }
    float inv = 1.0f / n;
    if (len) *len = n;
    return {a.x * inv, a.y * inv};
}
static inline float bmin(float a, float b) { return a < b ? a : b; }
static inline float bmax(float a, float b) { return a > b ? a : b; }
static inline float babs(float a) { return a > 0 ? a : -a; }
static inline float clampf(float a, float lo, float hi) { return bmax(lo, bmin(a, hi)); }
static inline float inv_or_zero(float x) { return x != 0 ? 1.0f / x : 0.0f; }
static inline float inv_if_pos(float x) { return x > 0 ? 1.0f / x : 0.0f; }

// ---- b2Mat22 / b2Mat33 (math2d.py:162-215); columns ex, ey, ez
struct V3 {
    float x, y, z;
};
static inline V2 solve22(float a11, float a12, float a21, float a22, float bx, float by) {
    float det = inv_or_zero(a11 * a22 - a12 * a21);
    return {det * (a22 * bx - a12 * by), det * (a11 * by - a21 * bx)};
}
static inline V3 cross3(V3 a, V3 b) { return {a.y * b.z - a.z * b.y, a.z * b.x - a.x * b.z, a.x * b.y - a.y * b.x}; }
static inline float dot3(V3 a, V3 b) { return (a.x * b.x + a.y * b.y) + a.z * b.z; }
static inline V3 solve33(V3 ex, V3 ey, V3 ez, V3 b) {
    float det = inv_or_zero(dot3(ex, cross3(ey, ez)));
    return {det * dot3(b, cross3(ey, ez)), det * dot3(ex, cross3(b, ez)), det * dot3(ex, cross3(ey, b))};
}
static inline void inverse22_of33(V3 ex, V3 ey, V3 *ox, V3 *oy, V3 *oz) {
    float a = ex.x, b = ey.x, c = ex.y, d = ey.y;
    float det = inv_or_zero(a * d - b * c);
    *ox = {det * d, -det * c, 0.0f};
    *oy = {-det * b, det * a, 0.0f};
    *oz = {0.0f, 0.0f, 0.0f};
}
static inline void sym_inverse33(V3 ex, V3 ey, V3 ez, V3 *ox, V3 *oy, V3 *oz) {
    float det = inv_or_zero(dot3(ex, cross3(ey, ez)));
    float a11 = ex.x, a12 = ey.x, a13 = ez.x, a22 = ey.y, a23 = ez.y, a33 = ez.z;
    float exx = det * (a22 * a33 - a23 * a23);
    float exy = det * (a13 * a23 - a12 * a33);
    float exz = det * (a12 * a23 - a13 * a22);
    float eyy = det * (a11 * a33 - a13 * a13);
    float eyz = det * (a13 * a12 - a11 * a23);
    float ezz = det * (a11 * a22 - a12 * a12);
    *ox = {exx, exy, exz};
    *oy = {exy, eyy, eyz};
    *oz = {exz, eyz, ezz};
}
static inline V3 mat33_mul(V3 ex, V3 ey, V3 ez, V3 v) {
    return {(v.x * ex.x + v.y * ey.x) + v.z * ez.x, (v.x * ex.y + v.y * ey.y) + v.z * ez.y,
            (v.x * ex.z + v.y * ey.z) + v.z * ez.z};
}
static inline V2 mat33_mul22(V3 ex, V3 ey, V2 v) { return {ex.x * v.x + ey.x * v.y, ex.y * v.x + ey.y * v.y}; }

// ---- correctly rounded sin/cos: float-float Cody-Waite reduction by pi/2 and Taylor series (math2d.py:218-316)
float sin_of(float x, float *cos_out);
static inline Rot rot_of(float a) {
    Rot r;
    r.s = sin_of(a, &r.c);
    return r;
}

// ---- AABBs (shapes.py:136-153)
struct AABB {
    float lx, ly, ux, uy;
};
static inline bool overlap(const AABB &a, const AABB &b) {
    float d1x = b.lx - a.ux, d1y = b.ly - a.uy, d2x = a.lx - b.ux, d2y = a.ly - b.uy;
    return !((d1x > 0) || (d1y > 0) || (d2x > 0) || (d2y > 0));
}

// ---- the world view: typed pointers into the State leaves of one world
struct Model {
    const goib2d_model_desc *d;
    int B, F, J, P;
    bool compact;
};

struct World {
    int B, rows, J, C;
    // contact event log of the current step (null: off), see goib2d_event in include/goib2d.h
    goib2d_event *events = nullptr;
    int32_t *event_count = nullptr;
    int event_cap = 0;
    // bodies
    int32_t *type;
    uint8_t *active, *awake, *allow_sleep, *bullet, *continuous;
    float *sleep_time, *xf_p, *xf_q, *local_center, *c0, *c, *a0, *a, *v, *w, *force, *torque, *mass, *inv_mass,
        *inertia, *inv_inertia, *linear_damping, *angular_damping, *gravity_scale;
    // fixtures
    float *fx_friction, *fx_restitution, *fx_fat;
    // joints
    uint8_t *enable_motor, *enable_limit;
    float *motor_speed, *max_motor, *lower, *upper, *frequency, *damping, *impulse, *motor_impulse, *lower_impulse,
        *upper_impulse;
    int32_t *limit_state;
    // contacts
    int32_t *pair, *fa, *fb, *key, *mtype, *count, *point_id;
    uint8_t *touching;
    float *local_normal, *local_point, *point_local, *normal_impulse, *tangent_impulse, *friction, *restitution,
        *tangent_speed;
    // scalars
    float *gravity, *inv_dt0;
    int32_t *next_key, *overflow;
    uint8_t *new_fixture;
    // toi
    float *t_alpha0, *t_toi, *t_ni, *t_ti;
    int32_t *t_count, *t_events;
    uint8_t *t_flag, *t_enabled, *t_solved;

    V2 bxf_p(int b) const { return {xf_p[2 * b], xf_p[2 * b + 1]}; }
    Rot bxf_q(int b) const { return {xf_q[2 * b], xf_q[2 * b + 1]}; }
    Xf bxf(int b) const { return {bxf_p(b), bxf_q(b)}; }
};

int leaf_dtype(int leaf);
int64_t leaf_elems(int leaf, int32_t B, int32_t rows, int32_t J, int32_t C);
void bind_world(World &w, void *const *leaves, int64_t wi, int B, int rows, int J, int C);

// Fixture accessors in either layout (world.py:400-434)
static inline int fixture_row(const Model &m, int f) { return m.compact ? m.d->fixture_slot[f] : f; }
AABB fixture_fat(const Model &m, const World &w, int f);
float fixture_friction(const Model &m, const World &w, int f);
float fixture_restitution(const Model &m, const World &w, int f);
AABB fixture_aabb(const Model &m, int f, Xf xf);

// Contact events (the reference C API's listener): appended in the order they are raised
enum { EV_BEGIN = 0, EV_END = 1, EV_POST_SOLVE = 2 };
static inline void emit_event(World &w, int kind, int slot, int count = 0, const float *ni = nullptr,
                              const float *ti = nullptr) {
    if (!w.events) return;
    int k = (*w.event_count)++;
    if (k >= w.event_cap) return;
    goib2d_event e{};
    e.kind = kind, e.fixture_a = w.fa[slot], e.fixture_b = w.fb[slot], e.count = count;
    for (int j = 0; j < count && j < 2; ++j) e.normal_impulse[j] = ni[j], e.tangent_impulse[j] = ti[j];
    w.events[k] = e;
}

// Narrow phase (collide.py)
struct Manifold {
    int32_t mtype, count;
    V2 local_normal, local_point, point[2];
    int32_t id[2];
};
// Contact manifold of a candidate pair (b2Contact::Evaluate); edges (shape type 1) have no counterpart in the
// reference engine: they follow the same method as the device code, Box2D 2.3.1's ghost-vertex colliders.
void evaluate(const Model &m, int fa, int fb, Xf xfa, Xf xfb, float linear_slop, float angular_slop, Manifold *out);

// Pieces shared by the step and SolveTOI
void find_new_contacts(const Model &m, World &w);
void synchronize_fixtures(const Model &m, World &w, const uint8_t *moved);
void solve_toi(const Model &m, World &w, const goib2d_settings &s, float dt);

}  // namespace orc
