// goib2d device-side data: the Model in HBM, the State leaves of one world, and the per-world scratch arena.
#pragma once
#include <cstdint>

#include "../../include/goib2d.h"
#include "b2dev.cuh"

namespace gb {

// The Model on the device (uploaded once by goib2d_model_create).
struct DevModel {
    int B, F, J, P;
    int compact;  // fixture_slot given (compact fixture layout)
    const int32_t *fixture_body, *shape_type, *count;
    const float *radius, *verts, *normals;
    const int32_t *joint_type, *joint_a, *joint_b;
    const float *local_anchor_a, *local_anchor_b, *local_axis_a, *local_yaxis_a, *reference_angle;
    const int32_t *pair_a, *pair_b;
    const int32_t *fixture_slot;  // [F] row of each fixture (identity for the full layout), -1 static
    const int32_t *edge_ghost;    // [F] ghost-vertex flags of edge fixtures (0 elsewhere)
    const float *static_fat, *static_friction, *static_restitution;
    const int32_t *row_fixture;   // [F] fixture of each State.fixtures row (valid for rows < n_rows)
    int any_toi_body;             // some body is bullet or continuous at build
    const int32_t *jadj_start;    // [B + 1] CSR over bodies of jadj
    const int32_t *jadj;          // (joint, other body) pairs: each body's joints, highest index first
    // Static-fixture grid (compact models; built by goib2d_model_create). FindNewContacts asks it for the static
    // fixtures near each non-static fixture instead of scanning every candidate pair; the hits are sorted back into
    // candidate order, so the created contacts are the same as the full scan's.
    int grid;                     // 1 when the tables below are set
    int n_static, n_rows, nx, ny;
    float gx0, gy0, inv_cell;     // origin and 1 / cell size
    const int32_t *cell_start;    // [nx * ny + 1] CSR over cells
    const int32_t *cell_items;    // static indices, per cell
    const float *sfat;            // [n_static][4] fat AABB of each static fixture
    const int32_t *sfix;          // [n_static] fixture of each static index
    const int32_t *cand_rs;       // [n_rows][n_static] candidate of (row's fixture, static fixture), -1 if none
    int n_dd;                     // candidates whose fixtures are both non-static
    const int32_t *dd;            // [n_dd] those candidates, ascending
    const int32_t *dd_row_start;  // [n_rows + 1] CSR over rows of dd_row_idx
    const int32_t *dd_row_idx;    // each row's entries of dd (its pairs with another non-static fixture), ascending
    const int4 *dd_rb;            // [n_dd] each dd entry's rows (x: fixture a's, y: b's) and bodies (z: a's, w: b's)
    int max_hits;                 // per-world hit buffer; more hits fall back to the full scan
};

// Grid cell of a coordinate (the same float operations on the host, when binning, and on the device)
__host__ __device__ __forceinline__ int grid_cell(float x, float x0, float inv, int n) {
    float f = floorf((x - x0) * inv);
    int c = f < 0.0f ? 0 : (f > (float)(n - 1) ? n - 1 : (int)f);
    return c;
}

struct Leaves {
    void *p[GOIB2D_NUM_LEAVES];
};

// Velocity + position constraint of one ordered contact (contact_solver.py:103-146).
struct alignas(16) VCRow {
    int slot, ia, ib, count, pc_count, mtype, pad0, pad1;
    float mA, mB, iA, iB;
    V2 n;
    float friction, tangent_speed;
    V2 rA[2], rB[2];
    float nmass[2], tmass[2], bias[2], ni[2], ti[2];
    float K[4], NM[4];
    V2 ln, lp, pl[2], lcA, lcB;
    float radA, radB;
};

// One ordered joint (joints.py:163-173). The fields the revolute velocity solves read come first (148 bytes, five
// 32-byte sectors): a row read from memory on every iteration (the one-world-per-thread sweeps of large batches)
// then moves five sectors per joint and iteration instead of all eight. 256 bytes, so that rows in an array whose
// start is 32-byte aligned (the arena's) stay aligned to sectors.
struct alignas(16) JRow {
    int type, ia, ib, limit_state, enable_motor, enable_limit, soft, jid;
    float mA, mB, iA, iB;
    V2 rA, rB;
    V3 Kx, Ky;
    float motor_mass, motor_speed, max_impulse, angle, inv_dt, lower, upper;
    float imp[5];
    float mimp;
    float d22, d33;  // inverse determinants of K's upper-left 2x2 block and of K (fixed over the velocity iterations)
    V3 Kz;
    V2 ax, pe;
    float a1, a2, s1, s2;
    float gamma, bias;
    V2 la, lb;
    float ref;
    V2 lx, ly;
    float pad_[4];
};
static_assert(sizeof(JRow) == 256, "JRow: 8 sectors");

// A narrow-phase result (collide.py:5-7).
struct Man {
    int mtype, count;
    V2 ln, lp, pt[2];
    int id[2];
};

// Byte offsets of the per-world scratch arrays (computed on the host by scratch_layout()).
struct Layout {
    // [B]
    int64_t vx, vy, vw, cx, cy, ca, qc, qs, qa;
    int64_t aw, bisl, stack, bflag, last, moved, done, minsep, jok, islsleep, minst, st;
    int64_t adv;  // [B][8] TOI: advanced c0x, c0y, a0, alpha0, xf (px, py, c, s)
    // [C]
    int64_t order, lpos, corder, cisl, cflag, freeslot, active, over, edges, tneed;
    int64_t man;  // [C] Man
    int64_t vc;   // [C] VCRow
    int64_t rec;  // [C][8] TOI sweep records
    int64_t tisl; // [C] TOI island contacts
    int64_t solved;  // [C]
    // [J]
    int64_t jr, jorder, jisl, jflag;
    int64_t isl;  // [3] island counts: contacts, joints, islands
    // island graph: [B + 1] CSR start and [B] fill cursor over bodies, [2C] (contact slot, other body) pairs
    int64_t adj_start, adj_cur, adj;
    int64_t lkey;    // [C] int64: the live slots' packed list-order keys (list_order)
    int64_t order2;  // [C] list_order's staging copy of the new list
    // [ceil(P/32)]
    // levelled sweeps (solve_constraints_levelled): per pass position its level and the positions sorted by level,
    // the level starts, fill cursors, each body's next free level, and the position passes' per-row results
    int64_t lv_level, lv_items, lv_start, lv_items2, lv_start2, lv_cur, lv_sep, lv_ok;
    int64_t bitmap;
    int64_t hits;  // [max_hits] new-pair candidates of the grid path
    int64_t stride;  // bytes per world (multiple of 256)
    // Shared-memory copies (per warp) used by the per-step kernels: the arena's first hot_end bytes - the small
    // arrays whose writes the sequential phases read back, which through global memory is an L2 round trip each
    // (0: the arena only) - and, in the step kernel after them, rows_bytes of constraint rows: the joint rows
    // at sm_jr and up to sm_vc_cap contact rows at sm_vc (see IslandWork in step.cu)
    int hot_end, rows_bytes, sm_jr, sm_vc, sm_vc_cap;
};

struct StepParams {
    DevModel m;
    Leaves L;
    goib2d_settings s;
    float dt;
    int C, rows;
    int64_t n_worlds;
    int n_steps;
    int step_mode;   // below 16384 worlds: 0 chosen per batch, 1 one world per warp, 2 two worlds per warp
    int step;        // index of the step a per-step launch belongs to (the one-launch step runs all n_steps)
    int64_t world0;  // a launch covers worlds world0 .. world_end - 1
    int64_t world_end;
    const float *actions;   // step k of a launch reads actions + k * action_stride (stride 0: the same every step)
    int64_t action_stride;
    int n_action;
    const int32_t *action_joint;
    const float *action_scale;
    char *scratch;
    Layout lay;
    int32_t *status;
    goib2d_event *events;  // contact event log [n_worlds][event_cap], or null (goib2d_set_event_log)
    int32_t *event_count;  // [n_worlds]
    int event_cap;
    // State rows staged in shared memory for a whole launch (the one-launch step): each world copies the rows of the
    // leaves with stage_off >= 0 into its staging area at stage_off, steps on the copies, and writes them back once
    int32_t stage_off[GOIB2D_NUM_LEAVES];
    int32_t leaf_bytes[GOIB2D_NUM_LEAVES];  // bytes of one world's row of each leaf
    int32_t stage_bytes;                    // the staging area per world (0: nothing staged)
    int32_t stage_max;                      // the model's staging limit per world (goib2d_set_state_staging)
};

// Parameters of the env kernels (env.cu): resets, observations, ray casts.
struct EnvParams {
    DevModel m;
    Leaves L;     // the batch's State
    Leaves I;     // a State of the same shape holding each world's initial state (resets)
    int32_t leaf_bytes[GOIB2D_NUM_LEAVES];  // bytes of one world's row of each leaf
    int64_t n_worlds;
    int B, rows;
    const uint8_t *mask;  // reset where mask[w] != 0 ...
    int body;             // ... or where bodies.c[w][body].y < y_min
    float y_min;
    int32_t *reset_count;  // optional per-world counters
    int n_obs;
    int32_t obs_body[16];
    float *out;
    int n_rays;
    float max_length;
    // goib2d_spawn (spawn.cuh): I holds one template world (row 0 of every leaf)
    int first_body, n_placed;
    const float *placements;  // [n_worlds][n_placed][6]
    int n_speeds;
    int32_t speed_joint[16];
    const float *speeds;      // [n_worlds][n_speeds]
    int J;
};

// goib2d_validate and checked stepping (check.cuh)
struct CheckParams {
    DevModel m;
    Leaves L;
    int64_t n_worlds;
    int C;
    unsigned long long *first_bad;  // min over failures of (world << 8 | leaf); all ones when none
};

// goib2d_seed_placements (spawn.cuh)
struct SeedParams {
    goib2d_spawn_rule rule;
    uint32_t key0, key1;
    int64_t first_world, n_worlds;
    float *placements, *speeds;
};

// The scene given to the candidate-pair build (scene.cuh), device arrays.
struct PairScene {
    int F, J;
    const int32_t *fixture_body, *shape_type, *body_type;
    const uint8_t *sensor;
    const int32_t *category, *mask, *group, *layer;
    const uint32_t *layer_masks;  // [32] or null
    const int64_t *no_collide;    // [J] sorted keys (lower body << 32 | higher body) of joints without collideConnected
    int n_no_collide;
};

// The step kernel's per-world shared-memory region for constraint rows (Layout::rows_bytes at most): the joint rows and
// the first contact rows of the island solve, within a small budget that leaves most of the L1 cache.
constexpr int ROWS_MAX_BYTES = 1536;

// Status bits (include/goib2d.h goib2d_status)
enum { ST_OVERFLOW = 1, ST_NONFINITE = 2, ST_CAP = 4, ST_LIMIT = 8 };

// Typed pointers into the State leaves of one world (the row of every leaf for world `wi`).
struct W {
    int B, rows, J, C;
    int32_t *type;
    uint8_t *active, *awake, *allow_sleep, *bullet, *continuous;
    float *sleep_time, *xf_p, *xf_q, *local_center, *c0, *c, *a0, *a, *v, *w, *force, *torque, *mass, *inv_mass,
        *inertia, *inv_inertia, *linear_damping, *angular_damping, *gravity_scale;
    float *fx_friction, *fx_restitution, *fx_fat;
    uint8_t *enable_motor, *enable_limit;
    float *motor_speed, *max_motor, *lower, *upper, *frequency, *damping, *impulse, *motor_impulse, *lower_impulse,
        *upper_impulse;
    int32_t *limit_state;
    int32_t *pair, *fa, *fb, *key, *mtype, *count, *point_id;
    uint8_t *touching;
    float *local_normal, *local_point, *point_local, *normal_impulse, *tangent_impulse, *friction, *restitution,
        *tangent_speed;
    float *gravity, *inv_dt0;
    int32_t *next_key, *overflow;
    uint8_t *new_fixture;
    float *t_alpha0, *t_toi, *t_ni, *t_ti;
    int32_t *t_count, *t_events;
    uint8_t *t_flag, *t_enabled, *t_solved;

    __device__ V2 bc(int b) const { return {c[2 * b], c[2 * b + 1]}; }
    __device__ V2 blc(int b) const { return {local_center[2 * b], local_center[2 * b + 1]}; }
    __device__ Xf bxf(int b) const { return {{xf_p[2 * b], xf_p[2 * b + 1]}, {xf_q[2 * b], xf_q[2 * b + 1]}}; }
};

}  // namespace gb
