/* goib2d: batched Box2D 2.3.1 world step on NVIDIA B200 (sm_100a) - the C ABI of libgoib2d.so.
 *
 * The library replaces the batched step of the reference engine goi_jax/box2d (miwate/getting-over-it-rl):
 *   - goi_jax/box2d/step.py:28        step(model, state, settings, dt, axis_name)   one b2World::Step per world;
 *   - goi_jax/box2d/gpu/kernel.py:573-599, gpu/pairs.py:242-259, gpu/islands.py:273-286,
 *     gpu/toi_search.py:567-581, gpu/toi_event.py:732-743   the jax.custom_batching.custom_vmap batch rules that
 *     receive the whole batch of worlds and launch one kernel over it. A JAX FFI handler registered for
 *     "goib2d_step" calls goib2d_step() from exactly that seam.
 *
 * Data contract. A batch of N worlds shares one Model (scene constants; uploaded once, goib2d_model_create) and
 * owns one State: GOIB2D_NUM_LEAVES arrays ("leaves"), each laid out (N, ...) row-major - the layout of the
 * reference's State pytree under jax.vmap, leaf order as in goib2d/world.py leaf_names(). Per world the leaf holds
 * the element counts given by goib2d_leaf_elems(). bool leaves are one byte (0/1), int leaves int32, float leaves
 * float32. goib2d_step() reads and writes the leaves in place (device pointers); the library never keeps a caller
 * pointer past a call.
 *
 * Errors: every entry point returns 0 on success and a negative GOIB2D_E* code otherwise, with a message for
 * goib2d_last_error() (thread-local). Per-world conditions (contact table overflow, non-finite state, an iteration
 * cap reached) are reported in the State (State.overflow) and by goib2d_status(), never by trapping the GPU.
 */
#ifndef GOIB2D_H
#define GOIB2D_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GOIB2D_ABI_VERSION 2

#define GOIB2D_OK 0
#define GOIB2D_EINVAL (-1)   /* bad argument (null pointer, size out of range, inconsistent layout) */
#define GOIB2D_ECUDA (-2)    /* a CUDA runtime call failed */
#define GOIB2D_ENOMEM (-3)   /* device allocation failed */
#define GOIB2D_ELIMIT (-4)   /* a capacity the kernels support was exceeded */

/* b2Settings globals + b2World flags; field for field goib2d.settings.SettingsC and the reference's Settings
 * dataclass (goi_jax/box2d/settings.py:109-148). */
typedef struct goib2d_settings {
    float gravity_x, gravity_y;
    float linear_slop, angular_slop, polygon_radius, velocity_threshold;
    float max_linear_correction, max_angular_correction, max_translation, max_rotation;
    float baumgarte, toi_baumgarte, time_to_sleep, linear_sleep_tolerance, angular_sleep_tolerance;
    int32_t velocity_iterations, position_iterations;
    int32_t clamps_per_second, allow_sleep, warm_starting, continuous_physics, unity_toi, toi_tie_oldest;
    int32_t auto_clear_forces, revolute_v24;
} goib2d_settings;

/* The scene constants of goi_jax/box2d/world.py:30-67 (Model), as host arrays. fixture_slot == NULL: full fixture
 * layout (State.fixtures has one row per fixture); otherwise the compact layout (reference world.py:437-472): rows
 * only for fixtures of non-static bodies, static_* hold the static fixtures' values.
 * shape_type: 0 circle (verts[0] the centre), 2 polygon (count vertices and normals), 1 edge (no counterpart in the
 * reference engine): count 2, verts[0] and verts[1] the segment, verts[2] and verts[3] the ghost vertices before and
 * after it (a chain is a run of edges whose ghost vertices are their neighbours' ends), present per edge_ghost. */
typedef struct goib2d_model_desc {
    int32_t n_bodies, n_fixtures, n_joints, n_pairs;
    const int32_t *fixture_body, *shape_type, *count;   /* [F] */
    const float *radius;                                /* [F] */
    const float *verts, *normals;                       /* [F][8][2] */
    const int32_t *joint_type, *joint_a, *joint_b;      /* [J] */
    const float *local_anchor_a, *local_anchor_b;       /* [J][2] */
    const float *local_axis_a, *local_yaxis_a;          /* [J][2] */
    const float *reference_angle;                       /* [J] */
    const int32_t *pair_a, *pair_b;                     /* [P], b2BroadPhase::UpdatePairs order */
    const uint8_t *toi_bodies;                          /* [B] bullet|continuous at build; NULL = unknown */
    const int32_t *fixture_slot;                        /* [F] or NULL */
    const float *static_fat;                            /* [F][4] (compact layout) */
    const float *static_friction, *static_restitution;  /* [F]    (compact layout) */
    const int32_t *edge_ghost;  /* [F] edges: bit 0 verts[2] is a ghost vertex, bit 1 verts[3]; NULL = none */
} goib2d_model_desc;

/* State leaves, in order (goib2d/world.py STATE_LEAVES). */
enum goib2d_leaf {
    /* Bodies [B] */
    GOIB2D_B_TYPE, GOIB2D_B_ACTIVE, GOIB2D_B_AWAKE, GOIB2D_B_ALLOW_SLEEP, GOIB2D_B_BULLET, GOIB2D_B_CONTINUOUS,
    GOIB2D_B_SLEEP_TIME, GOIB2D_B_XF_P, GOIB2D_B_XF_Q, GOIB2D_B_LOCAL_CENTER, GOIB2D_B_C0, GOIB2D_B_C,
    GOIB2D_B_A0, GOIB2D_B_A, GOIB2D_B_V, GOIB2D_B_W, GOIB2D_B_FORCE, GOIB2D_B_TORQUE, GOIB2D_B_MASS,
    GOIB2D_B_INV_MASS, GOIB2D_B_INERTIA, GOIB2D_B_INV_INERTIA, GOIB2D_B_LINEAR_DAMPING, GOIB2D_B_ANGULAR_DAMPING,
    GOIB2D_B_GRAVITY_SCALE,
    /* Fixtures [rows] */
    GOIB2D_F_FRICTION, GOIB2D_F_RESTITUTION, GOIB2D_F_FAT,
    /* Joints [J] */
    GOIB2D_J_ENABLE_MOTOR, GOIB2D_J_MOTOR_SPEED, GOIB2D_J_MAX_MOTOR, GOIB2D_J_ENABLE_LIMIT, GOIB2D_J_LOWER,
    GOIB2D_J_UPPER, GOIB2D_J_FREQUENCY, GOIB2D_J_DAMPING, GOIB2D_J_IMPULSE, GOIB2D_J_MOTOR_IMPULSE,
    GOIB2D_J_LIMIT_STATE, GOIB2D_J_LOWER_IMPULSE, GOIB2D_J_UPPER_IMPULSE,
    /* Contacts [C] */
    GOIB2D_C_PAIR, GOIB2D_C_FA, GOIB2D_C_FB, GOIB2D_C_KEY, GOIB2D_C_TOUCHING, GOIB2D_C_MTYPE, GOIB2D_C_COUNT,
    GOIB2D_C_LOCAL_NORMAL, GOIB2D_C_LOCAL_POINT, GOIB2D_C_POINT_LOCAL, GOIB2D_C_POINT_ID, GOIB2D_C_NORMAL_IMPULSE,
    GOIB2D_C_TANGENT_IMPULSE, GOIB2D_C_FRICTION, GOIB2D_C_RESTITUTION, GOIB2D_C_TANGENT_SPEED,
    /* world scalars */
    GOIB2D_GRAVITY, GOIB2D_INV_DT0, GOIB2D_NEXT_KEY, GOIB2D_NEW_FIXTURE, GOIB2D_OVERFLOW,
    /* ContactTOI */
    GOIB2D_T_ALPHA0, GOIB2D_T_COUNT, GOIB2D_T_TOI, GOIB2D_T_FLAG, GOIB2D_T_ENABLED, GOIB2D_T_SOLVED,
    GOIB2D_T_NORMAL_IMPULSE, GOIB2D_T_TANGENT_IMPULSE, GOIB2D_T_EVENTS,
    GOIB2D_NUM_LEAVES
};

/* Element type of a leaf: 0 float32, 1 int32, 2 bool (uint8). */
int goib2d_leaf_dtype(int leaf);

/* Elements per world of a leaf for a model with B bodies, `rows` fixture rows, J joints and C contact slots. */
int64_t goib2d_leaf_elems(int leaf, int32_t B, int32_t rows, int32_t J, int32_t C);

typedef struct goib2d_model goib2d_model;

/* ABI version (GOIB2D_ABI_VERSION). */
int goib2d_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char *goib2d_last_error(void);

/* Upload a Model to the current CUDA device and build the device-side broadphase tables. Replaces passing the
 * Model as a jit argument (scripts/bench_gpu.py:76-84): one handle per scene, shared by every world. */
int goib2d_model_create(const goib2d_model_desc *desc, goib2d_model **out);
int goib2d_model_destroy(goib2d_model *model);

/* Optional action channels (an RL env's per-step input): before each step, joints.motor_speed[joint[k]] of world w
 * = scale[k] * actions[w * n + k]. n == 0 clears the map. */
int goib2d_model_set_action_map(goib2d_model *model, int32_t n, const int32_t *joint, const float *scale);

/* Step n_worlds worlds n_steps times: b2World::Step (reference step.py:28-47) per world, in place on the State
 * leaves (device pointers, leaves[GOIB2D_NUM_LEAVES]). contact_capacity = C, fixture_rows = F (full layout) or the
 * number of non-static fixtures (compact). actions: NULL, or float32 [n_worlds][n_action] used before every
 * step (goib2d_model_set_action_map), in device memory or in page-locked host memory (read by the kernel over the
 * bus: no separate copy). stream: a cudaStream_t (NULL = the legacy default stream). Asynchronous:
 * returns after enqueueing the launches on `stream`. */
int goib2d_step(goib2d_model *model, const goib2d_settings *settings, float dt, int32_t contact_capacity,
                int32_t fixture_rows, int64_t n_worlds, int32_t n_steps, void *const *leaves, const float *actions,
                void *stream);

/* goib2d_step with its own row of actions for every step: step k of the call reads the float32 [n_worlds][n_action]
 * row at actions + k * action_step_stride (a [n_steps][n_worlds][n_action] buffer has stride n_worlds * n_action;
 * stride 0 reuses one row for every step, which is goib2d_step). Same memory rules for actions as goib2d_step.
 * The K steps of a call run in one persistent launch (goib2d_launches): each block steps its worlds K times with
 * no grid-wide boundary between the steps. Replaces a Python loop of K reference step() calls under jax.jit
 * (goi_jax/box2d/step.py:28-47 per step); the reference has no multi-step entry. */
int goib2d_step_seq(goib2d_model *model, const goib2d_settings *settings, float dt, int32_t contact_capacity,
                    int32_t fixture_rows, int64_t n_worlds, int32_t n_steps, void *const *leaves,
                    const float *actions, int64_t action_step_stride, void *stream);

/* Per-world status words of the last goib2d_step on this model (device int32 [n_worlds]; bit 0 contact table
 * overflow in this step, bit 1 non-finite body state, bit 2 an iteration cap was reached, bit 3 a capacity of the
 * kernels' on-chip tables was exceeded). Valid until the next goib2d_step with this model. */
int goib2d_status(goib2d_model *model, const int32_t **device_status, int64_t *n_worlds);

/* The same status words copied to host memory (n <= the last step's n_worlds); synchronises the device. */
int goib2d_status_copy(goib2d_model *model, int32_t *host_status, int64_t n);

/* Kernels one step runs for a batch of n_worlds worlds of this model: 1 (the whole step in one kernel, which also
 * runs every other step of the call), or 6 for batches of 16384 worlds and more of models with 8 joints or more
 * (collide, the solve in four pieces with the constraint sweeps run one world per thread, TOI; six launches per
 * step). For launch accounting and profilers; no counterpart in the reference engine. */
int goib2d_kernels_per_step(const goib2d_model *model, int64_t n_worlds);

/* Kernel launches one goib2d_step / goib2d_step_seq call of n_steps steps makes: 1 when the kernel runs every step
 * (goib2d_kernels_per_step 1), else 6 * n_steps; 0 for an empty call. No counterpart in the reference engine. */
int64_t goib2d_launches(const goib2d_model *model, int64_t n_worlds, int32_t n_steps);

/* How the one-launch step (goib2d_kernels_per_step 1) maps worlds to warps: 0 (default) chosen per batch - two
 * worlds per warp for batches of more than 16 worlds per SM with at most 128 contact slots, else one; 1 one world
 * per warp; 2 two worlds per warp (one per half-warp). Results are identical in every mode; only the speed differs.
 * No counterpart in the reference engine. */
int goib2d_set_step_mode(goib2d_model *model, int32_t mode);

/* Keep up to max_bytes_per_world bytes of each world's State rows in shared memory for the whole one-launch step
 * call (read from HBM at its start, written back at its end; the most used rows first, as far as the block's shared
 * memory allows). 0 (default) stages nothing. Results are identical either way; only the speed differs. No
 * counterpart in the reference engine. */
int goib2d_set_state_staging(goib2d_model *model, int32_t max_bytes_per_world);

/* Checked stepping: with on != 0, every later goib2d_step / goib2d_step_seq call on this model first validates the
 * State's index fields on the device (goib2d_validate's checks), synchronises the stream, and returns GOIB2D_EINVAL
 * naming the first bad world and field, launching no step, when one fails. Off by default (the check costs a kernel
 * and a synchronisation per call); goib2d_step_noalloc does not run it. No counterpart in the reference engine,
 * which trusts its State. */
int goib2d_set_checks(goib2d_model *model, int32_t on);

/* Validate a batch's State without stepping it: the integer fields the step kernels use as indices or loop bounds,
 * against the Model - bodies.type in STATIC..DYNAMIC, joints.limit_state in 0..3, contacts.pair in -1..P-1 and, for a
 * live slot, contacts.fa / fb equal to the candidate's fixtures, contacts.count in 0..2, contacts.mtype in 0..2. The
 * kernel only compares values, so it is safe on any State. *bad_world = the first failing world (-1: none) and
 * *bad_leaf its failing leaf (GOIB2D_* leaf id). Synchronises the stream. */
int goib2d_validate(goib2d_model *model, int32_t contact_capacity, int32_t fixture_rows, int64_t n_worlds,
                    void *const *leaves, int64_t *bad_world, int32_t *bad_leaf, void *stream);

/* ---- Env helpers around the step (no counterpart in the reference engine, whose RL env is outside it). Same
 * contact_capacity / fixture_rows / leaves conventions as goib2d_step; asynchronous on `stream`. */

/* Reset world w (every leaf's row) to init_leaves' row w where mask[w] != 0 (device uint8 [n_worlds]). init_leaves:
 * a State of the same shape holding each world's initial state. */
int goib2d_reset_masked(goib2d_model *model, int32_t contact_capacity, int32_t fixture_rows, int64_t n_worlds,
                        void *const *leaves, void *const *init_leaves, const uint8_t *mask, void *stream);

/* The same reset for the worlds whose body `body` has its centre of mass below y_min (bodies.c[w][body].y < y_min):
 * BASELINE c4's reset-on-fall. reset_count: NULL, or device int32 [n_worlds] incremented per reset world. */
int goib2d_reset_below(goib2d_model *model, int32_t contact_capacity, int32_t fixture_rows, int64_t n_worlds,
                       void *const *leaves, void *const *init_leaves, int32_t body, float y_min, int32_t *reset_count,
                       void *stream);

/* Observations: out (float32 [n_worlds][n_bodies][6], device or page-locked host memory, written by the kernel)
 * = c.x, c.y, angle, v.x, v.y, w of bodies[k] (host int32 [n_bodies], at most 16). */
int goib2d_observe(goib2d_model *model, int32_t contact_capacity, int32_t fixture_rows, int64_t n_worlds,
                   void *const *leaves, int32_t n_bodies, const int32_t *bodies, float *out, void *stream);

/* Ray casts against the static level: ray k of world w leaves body `body`'s centre of mass in direction
 * 2 pi k / n_rays (world frame) for max_length; out (float32 [n_worlds][n_rays], device or page-locked host
 * memory) = the nearest hit fraction
 * over the fixtures of static bodies (b2RayCastOutput::fraction; 1 = no hit). */
int goib2d_raycast(goib2d_model *model, int32_t contact_capacity, int32_t fixture_rows, int64_t n_worlds,
                   void *const *leaves, int32_t body, int32_t n_rays, float max_length, float *out, void *stream);

/* ---- Scene build on the device. The candidate pairs of a Model (the host builder's O(F^2) scan, goib2d/world.py
 * WorldDef.candidate_pairs; reference world.py:308-329): every fixture pair (i < k) except same body, a sensor, two
 * edges, two static bodies, bodies joined without collideConnected, or filtered out (the Unity layer matrix when
 * layer_masks is given, else Box2D's groups, categories and masks); ordered by i then k, each pair written edge
 * first, else polygon before circle. Host arrays in and out: *n_pairs = the number of pairs (also when capacity is
 * too small, then nothing is written and GOIB2D_ELIMIT is returned). */
typedef struct goib2d_pair_desc {
    int32_t n_bodies, n_fixtures, n_joints;
    const int32_t *body_type;                          /* [B] */
    const int32_t *fixture_body, *shape_type;          /* [F] */
    const uint8_t *sensor;                             /* [F] */
    const int32_t *category, *mask, *group, *layer;    /* [F] */
    const uint32_t *layer_masks;                       /* [32] or NULL */
    const int32_t *joint_a, *joint_b;                  /* [J] */
    const uint8_t *joint_collide;                      /* [J] collideConnected */
} goib2d_pair_desc;
int goib2d_candidate_pairs(const goib2d_pair_desc *desc, int32_t *pair_a, int32_t *pair_b, int64_t capacity,
                           int64_t *n_pairs);

/* Per-world initial States built on the device: every world of the batch (leaves, as goib2d_step's) starts as a copy
 * of one template world (template_leaves: a one-world State of the same shape, e.g. world 0's WorldDef.build),
 * then bodies first_body .. first_body + n_placed - 1 are placed per world as the host builder's
 * WorldDef.add_body(type, position, angle, velocity, angular_velocity) with the template body's mass data would
 * place them (reference world.py:186-244, b2Body::SetMassData / SetTransform): placements (float32
 * [n_worlds][n_placed][6], device or page-locked host memory) = x, y, angle, v.x, v.y, w. Per placed body: xf = (x, y,
 * sin/cos of the angle), sweep c0 = c = xf * local_center, a0 = a = angle; v and w as given when some is non-zero and
 * the template body is awake, else zero; the fat AABBs of its fixture rows from b2BroadPhase::CreateProxy (the shape
 * AABB at xf, extended by b2_aabbExtension). Static bodies keep the template's pose (the level is the batch's). Then
 * joint speed_joints[k] (host int32 [n_speeds], at most 16) gets motor_speed = speeds[w][k] (float32 [n_worlds]
 * [n_speeds], device or page-locked host memory). Replaces the host loop that builds each world through WorldDef
 * (the reference builds each world's State on the host; a batch is a stack of them). Asynchronous on `stream`. */
int goib2d_spawn(goib2d_model *model, int32_t contact_capacity, int32_t fixture_rows, int64_t n_worlds,
                 void *const *leaves, void *const *template_leaves, int32_t first_body, int32_t n_placed,
                 const float *placements, int32_t n_speeds, const int32_t *speed_joints, const float *speeds,
                 void *stream);

/* Seeded per-world placements on the device: world first_world + i of a scene seeded `seed` draws its placements
 * (and motor speeds) from a counter-based generator, Philox4x32-10 (Salmon et al., SC'11) keyed by the seed with
 * counter (world low, world high, block, 0): so a world's draws depend only on (seed, world), not on the batch or
 * the shard. A uniform draw on [lo, hi) is lo + (hi - lo) * u in float32, u = (r >> 8) * 2^-24 of the block's next
 * 32-bit word. Rules (goib2d_spawn_rule.kind), the benchmark scenes' spawn patterns:
 *   GOIB2D_SPAWN_UNIFORM: n_bodies bodies, body k from draws 5k .. 5k + 4: x ~ [x_lo, x_hi), y ~ [y_lo, y_hi),
 *     angle ~ [angle_lo, angle_hi), speed ~ [speed_lo, speed_hi), heading ~ [0, 2 pi): v = speed (cos, sin)
 *     heading, w = 0 (BASELINE c0's box drop, c3's bullets);
 *   GOIB2D_SPAWN_GRID: body k at the grid cell (k mod grid_side, k / grid_side) of pitch grid_pitch from
 *     (grid_x0, grid_y0), cell centre plus a jitter ~ [-jitter, jitter) per axis, angle ~ [angle_lo, angle_hi)
 *     (draws 3k .. 3k + 2; BASELINE c2);
 *   GOIB2D_SPAWN_RIG: the character rig (3 bodies: pot, hub, hammer) over a height field (heights: device float32
 *     [n_heights], x of sample i = h_x0 + i h_dx): try t < max_tries draws x ~ [x_lo, x_hi) (draw t); the ground
 *     under the pot spans samples (int)((x - half_width - h_x0) / h_dx) .. (int)((x + half_width - h_x0) / h_dx) + 1
 *     (clamped); y = its highest sample + lift; a try is kept when the lowest sample is >= min_ground and the pot
 *     clears every disc (discs: device float32 [n_discs][3] = x, y, r; (x - dx)^2 + (y - dy)^2 > (r + clearance)^2),
 *     the last try otherwise; angle ~ [angle_lo, angle_hi) (draw max_tries), the motor speed ~ [speed_lo,
 *     speed_hi) (draw max_tries + 1) into speeds; pot at (x, y, 0), hub at (x, y, angle), hammer at
 *     (x + arm cos angle, y + arm sin angle, angle) (BASELINE c1 and c4).
 * placements: device float32 [n_worlds][n_bodies][6] (n_bodies = 3 for RIG); speeds: device float32 [n_worlds]
 * (RIG only, may be NULL otherwise). No counterpart in the reference, whose worlds come from host numpy seeds. */
enum { GOIB2D_SPAWN_UNIFORM = 0, GOIB2D_SPAWN_GRID = 1, GOIB2D_SPAWN_RIG = 2 };
typedef struct goib2d_spawn_rule {
    int32_t kind, n_bodies;
    float x_lo, x_hi, y_lo, y_hi, angle_lo, angle_hi, speed_lo, speed_hi;
    int32_t grid_side;
    float grid_x0, grid_y0, grid_pitch, jitter;
    const float *heights;
    int32_t n_heights;
    float h_x0, h_dx, half_width, lift, min_ground, arm;
    const float *discs;
    int32_t n_discs;
    float clearance;
    int32_t max_tries;
} goib2d_spawn_rule;
int goib2d_seed_placements(const goib2d_spawn_rule *rule, uint64_t seed, int64_t first_world, int64_t n_worlds,
                           float *placements, float *speeds, void *stream);

/* ---- Contact event log: the reference C API's listener (goi_jax/reference/capi.cpp:45-78, goi_b2_events at
 * :838-847) for a batch. Per world, the Begin (kind 0), End (1) and PostSolve (2) events of the last step, in the
 * order Box2D raises them: Collide's updates in contact-list order (End also for a touching contact that Collide
 * destroys), PostSolve per island contact after the island solve, then each TOI event's updates and its PostSolve.
 * The record has the reference's Event layout; child indices are 0 (a chain's children are fixtures here). */
typedef struct goib2d_event {
    int32_t kind, fixture_a, fixture_b, child_a, child_b, count;
    float normal_impulse[2], tangent_impulse[2];
} goib2d_event;
/* capacity events per world (0: off, the default). Logging changes no result. With n_steps > 1 the log holds the
 * last step's events. */
int goib2d_set_event_log(goib2d_model *model, int32_t capacity);
/* The log of the last step: device goib2d_event [n_worlds][capacity] and device int32 [n_worlds] counts (a count
 * above capacity: the events past capacity were dropped). Valid until the next step on this model. */
int goib2d_events(goib2d_model *model, const goib2d_event **device_events, const int32_t **device_counts,
                  int64_t *n_worlds, int32_t *capacity);
/* The same log copied to host memory: n_worlds x capacity events and n_worlds counts; synchronises the device. */
int goib2d_events_copy(goib2d_model *model, goib2d_event *host_events, int32_t *host_counts, int64_t n_worlds);

/* Bytes of the static scratch arena used by goib2d_step_noalloc (on every device that loads the library). */
#define GOIB2D_NOALLOC_SCRATCH_BYTES (32u << 20)

/* goib2d_step without any device allocation, for callers that cannot allocate while they step (code inside a CUDA
 * graph capture, a host whose pool allocator owns the GPU's memory, a loop that forbids allocation after start-up).
 * No counterpart in the reference engine. Same arguments and results as goib2d_step, but the per-world scratch arena
 * is a GOIB2D_NOALLOC_SCRATCH_BYTES static device array, so n_worlds is limited to that size divided by the arena
 * bytes one world needs (which grow with bodies, contact slots, joints and candidate pairs); larger batches return
 * GOIB2D_ELIMIT with a message and launch nothing. The first call on each device looks the array's address up
 * (cudaGetSymbolAddress): make that call before any stream capture. All calls share the array, so calls that
 * overlap on the GPU race and must be serialised by the caller; earlier contents never affect a call. It sets no
 * status words and records no contact events (even with goib2d_set_event_log on): after it, goib2d_status and
 * goib2d_events report zero worlds until the next goib2d_step. The first call on a device also raises the kernel's
 * shared-memory limit (cudaFuncSetAttribute, no allocation), another reason to make it before any capture. */
int goib2d_step_noalloc(goib2d_model *model, const goib2d_settings *settings, float dt, int32_t contact_capacity,
                        int32_t fixture_rows, int64_t n_worlds, int32_t n_steps, void *const *leaves,
                        const float *actions, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* GOIB2D_H */
