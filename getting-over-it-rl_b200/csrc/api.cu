// goib2d C ABI (include/goib2d.h): model upload, scratch management, kernel launch, errors.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "engine.cuh"

namespace gb {
cudaError_t launch_steps(StepParams p, cudaStream_t stream);  // step.cu
int kernels_per_step(int64_t n_worlds, int n_joints);         // step.cu
int64_t launches_per_call(int64_t n_worlds, int n_joints, int n_steps);  // step.cu
int hot_budget(int64_t n_worlds, int n_joints, int contact_capacity, int step_mode);  // step.cu
cudaError_t launch_reset(const EnvParams &p, cudaStream_t s);    // env.cuh (compiled in step.cu)
cudaError_t launch_observe(const EnvParams &p, cudaStream_t s);  // env.cuh
cudaError_t launch_raycast(const EnvParams &p, cudaStream_t s);  // env.cuh
cudaError_t launch_spawn(const EnvParams &p, cudaStream_t s);    // spawn.cuh (compiled in step.cu)
cudaError_t launch_seed(const SeedParams &p, cudaStream_t s);    // spawn.cuh
cudaError_t launch_check(const CheckParams &p, cudaStream_t s);  // check.cuh (compiled in step.cu)
cudaError_t launch_pair_count(const PairScene &s, int64_t *count);                              // scene.cuh
cudaError_t launch_pair_fill(const PairScene &s, const int64_t *start, int32_t *pa, int32_t *pb);  // scene.cuh
}

namespace {

// An NVTX range over each C entry point (header-only NVTX3: a no-op unless a profiler such as Nsight Systems or
// Nsight Compute is attached), so a profile shows which call issued which kernels.
struct Range {
    explicit Range(const char *name) { nvtxRangePushA(name); }
    ~Range() { nvtxRangePop(); }
    Range(const Range &) = delete;
    Range &operator=(const Range &) = delete;
};

thread_local std::string g_err;

int fail(int code, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

#define CUDA_TRY(expr)                                                                          \
    do {                                                                                        \
        cudaError_t e_ = (expr);                                                                \
        if (e_ != cudaSuccess) return fail(GOIB2D_ECUDA, "%s: %s", #expr, cudaGetErrorString(e_)); \
    } while (0)

struct LeafSpec {
    int dtype, dim, width;  // dtype 0 f32 1 i32 2 bool; dim 0 B 1 rows 2 J 3 C 4 scalar
};
const LeafSpec LEAVES[GOIB2D_NUM_LEAVES] = {
    {1, 0, 1}, {2, 0, 1}, {2, 0, 1}, {2, 0, 1}, {2, 0, 1}, {2, 0, 1}, {0, 0, 1}, {0, 0, 2}, {0, 0, 2}, {0, 0, 2},
    {0, 0, 2}, {0, 0, 2}, {0, 0, 1}, {0, 0, 1}, {0, 0, 2}, {0, 0, 1}, {0, 0, 2}, {0, 0, 1}, {0, 0, 1}, {0, 0, 1},
    {0, 0, 1}, {0, 0, 1}, {0, 0, 1}, {0, 0, 1}, {0, 0, 1},
    {0, 1, 1}, {0, 1, 1}, {0, 1, 4},
    {2, 2, 1}, {0, 2, 1}, {0, 2, 1}, {2, 2, 1}, {0, 2, 1}, {0, 2, 1}, {0, 2, 1}, {0, 2, 1}, {0, 2, 3}, {0, 2, 1},
    {1, 2, 1}, {0, 2, 1}, {0, 2, 1},
    {1, 3, 1}, {1, 3, 1}, {1, 3, 1}, {1, 3, 1}, {2, 3, 1}, {1, 3, 1}, {1, 3, 1}, {0, 3, 2}, {0, 3, 2}, {0, 3, 4},
    {1, 3, 2}, {0, 3, 2}, {0, 3, 2}, {0, 3, 1}, {0, 3, 1}, {0, 3, 1},
    {0, 4, 2}, {0, 4, 1}, {1, 4, 1}, {2, 4, 1}, {1, 4, 1},
    {0, 0, 1}, {1, 3, 1}, {0, 3, 1}, {2, 3, 1}, {2, 3, 1}, {2, 3, 1}, {0, 3, 2}, {0, 3, 2}, {1, 4, 1}};

// Per-world scratch arena: every array of the step's working set, 16-byte aligned, stride a multiple of 256 B.
gb::Layout scratch_layout(int B, int C, int J, int P, int max_hits, int hot_max = 6144) {
    gb::Layout L{};
    int64_t off = 0;
    auto take = [&](int64_t bytes) {
        int64_t o = off;
        off += (bytes + 15) & ~int64_t(15);
        return o;
    };
    const int64_t b4 = 4 * (int64_t)(B > 0 ? B : 1), c4 = 4 * (int64_t)(C > 0 ? C : 1), j4 = 4 * (int64_t)(J > 0 ? J : 1);
    // the hot part first: the small arrays the sequential phases write and read back (see Layout::hot_end), the
    // most used first, so that the prefix a kernel keeps in shared memory (hot_max bytes at most) holds them when the
    // whole part does not fit; the offsets do not depend on hot_max
    int64_t fits = 0;  // the largest array boundary within the shared-memory budget
    auto hot = [&](int64_t bytes) {
        int64_t o = take(bytes);
        if (off <= hot_max) fits = off;
        return o;
    };
    L.vx = hot(b4), L.vy = hot(b4), L.vw = hot(b4), L.cx = hot(b4), L.cy = hot(b4), L.ca = hot(b4);
    L.qc = hot(b4), L.qs = hot(b4), L.qa = hot(b4);
    L.aw = hot(b4), L.bisl = hot(b4), L.stack = hot(b4), L.bflag = hot(b4), L.last = hot(b4);
    L.moved = hot(b4), L.done = hot(b4), L.minsep = hot(b4), L.jok = hot(b4), L.islsleep = hot(b4);
    L.minst = hot(b4), L.st = hot(b4);
    L.isl = hot(16);
    L.order = hot(c4), L.lpos = hot(c4), L.lkey = hot(8 * (int64_t)(C > 0 ? C : 1)), L.order2 = hot(c4);
    L.adv = hot(8 * b4);
    L.corder = hot(c4), L.cisl = hot(c4), L.cflag = hot(c4);
    L.freeslot = hot(c4), L.active = hot(c4), L.over = hot(c4), L.edges = hot(c4), L.tneed = hot(c4);
    L.tisl = hot(c4), L.solved = hot(c4);
    L.jorder = hot(j4), L.jisl = hot(j4), L.jflag = hot(j4);
    L.adj_start = hot(4 * (int64_t)(B + 1)), L.adj_cur = hot(b4), L.adj = hot(2 * 8 * (int64_t)(C > 0 ? C : 1));
    L.hot_end = (int)fits;
    // the cold part: rows, manifolds, records and the broadphase buffers
    L.man = take((int64_t)sizeof(gb::Man) * (C > 0 ? C : 1));
    off = (off + 31) & ~int64_t(31);  // contact rows (7 sectors each) start on a 32-byte sector
    L.vc = take((int64_t)sizeof(gb::VCRow) * (C > 0 ? C : 1));
    L.rec = take(8 * c4);
    off = (off + 31) & ~int64_t(31);  // joint rows start on a 32-byte sector (gb::JRow)
    L.jr = take((int64_t)sizeof(gb::JRow) * (J > 0 ? J : 1));
    const int64_t n_rows4 = 4 * (int64_t)((C > 0 ? C : 0) + (J > 0 ? J : 0) + 2);
    L.lv_level = take(n_rows4), L.lv_items = take(n_rows4), L.lv_start = take(n_rows4), L.lv_cur = take(n_rows4);
    L.lv_items2 = take(n_rows4), L.lv_start2 = take(n_rows4);
    L.lv_sep = take(c4), L.lv_ok = take(j4);
    L.bitmap = take(4 * (int64_t)((P + 31) / 32 + 1));
    L.hits = take(8 * (int64_t)(max_hits > 0 ? max_hits : 1));  // unsorted + sorted halves
    L.stride = (off + 255) & ~int64_t(255);
    // the step kernel's constraint rows in shared memory (after the hot part): the joint rows and the first
    // contact rows, within gb::ROWS_MAX_BYTES
    const int jbytes = (int)sizeof(gb::JRow) * J;
    if (L.hot_end > 0 && jbytes <= gb::ROWS_MAX_BYTES) {
        int cap = (gb::ROWS_MAX_BYTES - jbytes) / (int)sizeof(gb::VCRow);
        cap = cap < C ? cap : C;
        L.sm_jr = 0, L.sm_vc = jbytes, L.sm_vc_cap = cap;
        L.rows_bytes = (jbytes + (int)sizeof(gb::VCRow) * cap + 15) & ~15;
    }
    return L;
}

template <class T>
int upload(std::vector<void *> &allocs, const T *src, size_t n, const T **dst) {
    *dst = nullptr;
    size_t bytes = sizeof(T) * (n > 0 ? n : 1);
    void *p = nullptr;
    CUDA_TRY(cudaMalloc(&p, bytes));
    allocs.push_back(p);
    if (src && n) CUDA_TRY(cudaMemcpy(p, src, sizeof(T) * n, cudaMemcpyHostToDevice));
    else CUDA_TRY(cudaMemset(p, 0, bytes));
    *dst = (const T *)p;
    return 0;
}

// The static-fixture grid of a compact model (see gb::DevModel).
int build_grid(const goib2d_model_desc &d, const std::vector<int32_t> &rows, std::vector<void *> &allocs,
               gb::DevModel &g) {
    const int F = d.n_fixtures, P = d.n_pairs, R = (int)rows.size();
    std::vector<int32_t> sfix, sidx(F, -1);
    for (int f = 0; f < F; ++f)
        if (d.fixture_slot[f] < 0) sidx[f] = (int)sfix.size(), sfix.push_back(f);
    const int S = (int)sfix.size();
    g.grid = 0;
    if (S == 0 || R == 0 || (int64_t)R * S > (int64_t)1 << 26) return 0;  // full scan
    std::vector<float> sfat(4 * (size_t)S);
    float x0 = INFINITY, y0 = INFINITY, x1 = -INFINITY, y1 = -INFINITY;
    std::vector<float> small;
    for (int i = 0; i < S; ++i) {
        const float *a = d.static_fat + 4 * sfix[i];
        for (int k = 0; k < 4; ++k) sfat[4 * i + k] = a[k];
        if (!(a[0] <= a[2] && a[1] <= a[3])) return 0;  // a non-finite or inverted box: keep the full scan
        x0 = fminf(x0, a[0]), y0 = fminf(y0, a[1]), x1 = fmaxf(x1, a[2]), y1 = fmaxf(y1, a[3]);
        small.push_back(fminf(a[2] - a[0], a[3] - a[1]));
    }
    std::nth_element(small.begin(), small.begin() + small.size() / 2, small.end());
    float cell = fmaxf(2.0f * small[small.size() / 2], 1e-3f);
    int nx = 0, ny = 0;
    std::vector<int32_t> start, items;
    for (int attempt = 0; attempt < 24; ++attempt, cell *= 1.5f) {
        double fx = ((double)x1 - x0) / cell + 1, fy = ((double)y1 - y0) / cell + 1;
        if (fx * fy > 4e6) continue;
        nx = (int)fx, ny = (int)fy;
        float inv = 1.0f / cell;
        std::vector<int32_t> cnt((size_t)nx * ny + 1, 0);
        int64_t total = 0;
        for (int i = 0; i < S; ++i) {
            int cx0 = gb::grid_cell(sfat[4 * i], x0, inv, nx), cx1 = gb::grid_cell(sfat[4 * i + 2], x0, inv, nx);
            int cy0 = gb::grid_cell(sfat[4 * i + 1], y0, inv, ny), cy1 = gb::grid_cell(sfat[4 * i + 3], y0, inv, ny);
            total += (int64_t)(cx1 - cx0 + 1) * (cy1 - cy0 + 1);
        }
        if (total > (int64_t)1 << 24) continue;
        start.assign((size_t)nx * ny + 1, 0);
        for (int i = 0; i < S; ++i) {
            int cx0 = gb::grid_cell(sfat[4 * i], x0, inv, nx), cx1 = gb::grid_cell(sfat[4 * i + 2], x0, inv, nx);
            int cy0 = gb::grid_cell(sfat[4 * i + 1], y0, inv, ny), cy1 = gb::grid_cell(sfat[4 * i + 3], y0, inv, ny);
            for (int cy = cy0; cy <= cy1; ++cy)
                for (int cx = cx0; cx <= cx1; ++cx) start[(size_t)cy * nx + cx + 1]++;
        }
        for (size_t k = 1; k < start.size(); ++k) start[k] += start[k - 1];
        items.assign((size_t)total, 0);
        std::vector<int32_t> fill(start.begin(), start.end() - 1);
        for (int i = 0; i < S; ++i) {
            int cx0 = gb::grid_cell(sfat[4 * i], x0, inv, nx), cx1 = gb::grid_cell(sfat[4 * i + 2], x0, inv, nx);
            int cy0 = gb::grid_cell(sfat[4 * i + 1], y0, inv, ny), cy1 = gb::grid_cell(sfat[4 * i + 3], y0, inv, ny);
            for (int cy = cy0; cy <= cy1; ++cy)
                for (int cx = cx0; cx <= cx1; ++cx) items[fill[(size_t)cy * nx + cx]++] = i;
        }
        g.inv_cell = inv;
        break;
    }
    if (start.empty()) return 0;
    std::vector<int32_t> cand((size_t)R * S, -1), dd;
    std::vector<int32_t> row_of(F, -1);
    for (int r = 0; r < R; ++r) row_of[rows[r]] = r;
    for (int p = 0; p < P; ++p) {
        int a = d.pair_a[p], b = d.pair_b[p];
        if (row_of[a] >= 0 && row_of[b] >= 0)
            dd.push_back(p);
        else if (row_of[a] >= 0 && sidx[b] >= 0)
            cand[(size_t)row_of[a] * S + sidx[b]] = p;
        else if (row_of[b] >= 0 && sidx[a] >= 0)
            cand[(size_t)row_of[b] * S + sidx[a]] = p;
    }
    // each row's entries of dd (indices into dd, ascending): a TOI event's FindNewContacts visits only the moved rows'
    std::vector<int32_t> dd_start((size_t)R + 1, 0), dd_idx(2 * dd.size() + 1, 0);
    for (int32_t p : dd) ++dd_start[row_of[d.pair_a[p]] + 1], ++dd_start[row_of[d.pair_b[p]] + 1];
    for (int r = 0; r < R; ++r) dd_start[r + 1] += dd_start[r];
    {
        std::vector<int32_t> fill(dd_start.begin(), dd_start.end() - 1);
        for (size_t k = 0; k < dd.size(); ++k) {
            dd_idx[fill[row_of[d.pair_a[dd[k]]]]++] = (int32_t)k;
            dd_idx[fill[row_of[d.pair_b[dd[k]]]]++] = (int32_t)k;
        }
    }
    // each dd entry's two rows and bodies in one 16-byte record (the full scan's one load per pair)
    std::vector<int32_t> dd4(4 * dd.size() + 4, 0);
    for (size_t k = 0; k < dd.size(); ++k) {
        const int a = d.pair_a[dd[k]], b = d.pair_b[dd[k]];
        dd4[4 * k] = row_of[a], dd4[4 * k + 1] = row_of[b];
        dd4[4 * k + 2] = d.fixture_body[a], dd4[4 * k + 3] = d.fixture_body[b];
    }
    int rc = 0;
    const int32_t *d_start, *d_items, *d_sfix, *d_cand, *d_dd, *d_dd_start, *d_dd_idx, *d_dd4;
    const float *d_sfat;
    rc = rc ? rc : upload(allocs, start.data(), start.size(), &d_start);
    rc = rc ? rc : upload(allocs, items.data(), items.size(), &d_items);
    rc = rc ? rc : upload(allocs, sfix.data(), sfix.size(), &d_sfix);
    rc = rc ? rc : upload(allocs, sfat.data(), sfat.size(), &d_sfat);
    rc = rc ? rc : upload(allocs, cand.data(), cand.size(), &d_cand);
    rc = rc ? rc : upload(allocs, dd.data(), dd.size(), &d_dd);
    rc = rc ? rc : upload(allocs, dd_start.data(), dd_start.size(), &d_dd_start);
    rc = rc ? rc : upload(allocs, dd_idx.data(), dd_idx.size(), &d_dd_idx);
    rc = rc ? rc : upload(allocs, dd4.data(), dd4.size(), &d_dd4);
    if (rc) return rc;
    g.n_static = S, g.n_rows = R, g.nx = nx, g.ny = ny, g.gx0 = x0, g.gy0 = y0;
    g.cell_start = d_start, g.cell_items = d_items, g.sfix = d_sfix, g.sfat = d_sfat, g.cand_rs = d_cand;
    g.n_dd = (int)dd.size(), g.dd = d_dd, g.dd_row_start = d_dd_start, g.dd_row_idx = d_dd_idx;
    g.dd_rb = reinterpret_cast<const int4 *>(d_dd4);
    g.max_hits = 256;
    g.grid = 1;
    return 0;
}

}  // namespace

struct goib2d_model {
    gb::DevModel full{}, compact{};  // the same model read through the full or the compact fixture layout
    int has_compact = 0, n_rows_compact = 0;
    int device = 0;
    std::vector<void *> allocs;
    char *scratch = nullptr;
    size_t scratch_bytes = 0;
    int32_t *status = nullptr;
    int64_t status_cap = 0, status_n = 0;
    int32_t n_action = 0;
    int32_t *action_joint = nullptr;
    float *action_scale = nullptr;
    int32_t step_mode = 0;  // goib2d_set_step_mode
    int32_t stage_max = 0;  // goib2d_set_state_staging
    int32_t event_cap = 0;  // contact event log per world (0: off)
    goib2d_event *events = nullptr;
    int32_t *event_count = nullptr;
    int64_t event_worlds = 0, event_n = 0;
    int32_t checks = 0;                       // goib2d_set_checks
    unsigned long long *check_buf = nullptr;  // the validation kernel's result (allocated once, freed with the model)
    std::mutex mu;
};

extern "C" {

// A kernel-accessible address for a caller's buffer: device memory as is; page-locked (pinned) host memory through
// its mapped device address, so the kernels read or write it over the bus with no separate copy.
static int device_view(const void *ptr, const void **out) {
    *out = ptr;
    if (!ptr) return 0;
    cudaPointerAttributes a{};
    CUDA_TRY(cudaPointerGetAttributes(&a, ptr));
    if (a.type == cudaMemoryTypeHost) {
        void *d = nullptr;
        CUDA_TRY(cudaHostGetDevicePointer(&d, const_cast<void *>(ptr), 0));
        *out = d;
    } else if (a.type == cudaMemoryTypeUnregistered) {
        return fail(GOIB2D_EINVAL, "a host buffer that is not page-locked cannot be read by the kernels");
    }
    return 0;
}

int goib2d_version(void) { return GOIB2D_ABI_VERSION; }

int goib2d_kernels_per_step(const goib2d_model *model, int64_t n_worlds) {
    if (!model) return fail(GOIB2D_EINVAL, "null argument");
    return gb::kernels_per_step(n_worlds, model->full.J);
}

int64_t goib2d_launches(const goib2d_model *model, int64_t n_worlds, int32_t n_steps) {
    if (!model) return fail(GOIB2D_EINVAL, "null argument");
    if (n_worlds < 0 || n_steps < 0) return fail(GOIB2D_EINVAL, "negative size");
    return gb::launches_per_call(n_worlds, model->full.J, n_steps);
}

const char *goib2d_last_error(void) { return g_err.c_str(); }

int goib2d_leaf_dtype(int leaf) {
    if (leaf < 0 || leaf >= GOIB2D_NUM_LEAVES) return fail(GOIB2D_EINVAL, "leaf %d out of range", leaf);
    return LEAVES[leaf].dtype;
}

int64_t goib2d_leaf_elems(int leaf, int32_t B, int32_t rows, int32_t J, int32_t C) {
    if (leaf < 0 || leaf >= GOIB2D_NUM_LEAVES) return fail(GOIB2D_EINVAL, "leaf %d out of range", leaf);
    const LeafSpec &s = LEAVES[leaf];
    int64_t n = s.dim == 0 ? B : s.dim == 1 ? rows : s.dim == 2 ? J : s.dim == 3 ? C : 1;
    return n * s.width;
}

int goib2d_model_create(const goib2d_model_desc *d, goib2d_model **out) {
    Range range("goib2d_model_create");
    if (!d || !out) return fail(GOIB2D_EINVAL, "null argument");
    *out = nullptr;
    const int B = d->n_bodies, F = d->n_fixtures, J = d->n_joints, P = d->n_pairs;
    if (B < 0 || F < 0 || J < 0 || P < 0) return fail(GOIB2D_EINVAL, "negative model size");
    if (F && (!d->fixture_body || !d->shape_type || !d->count || !d->radius || !d->verts || !d->normals))
        return fail(GOIB2D_EINVAL, "fixture arrays missing");
    if (J && (!d->joint_type || !d->joint_a || !d->joint_b || !d->local_anchor_a || !d->local_anchor_b ||
              !d->local_axis_a || !d->local_yaxis_a || !d->reference_angle))
        return fail(GOIB2D_EINVAL, "joint arrays missing");
    if (P && (!d->pair_a || !d->pair_b)) return fail(GOIB2D_EINVAL, "pair arrays missing");
    for (int f = 0; f < F; ++f) {
        if (d->fixture_body[f] < 0 || d->fixture_body[f] >= B) return fail(GOIB2D_EINVAL, "fixture %d body", f);
        if (d->count[f] < 1 || d->count[f] > gb::MAXV) return fail(GOIB2D_EINVAL, "fixture %d vertex count", f);
        if (d->shape_type[f] != gb::CIRCLE && d->shape_type[f] != gb::POLYGON && d->shape_type[f] != gb::EDGE)
            return fail(GOIB2D_EINVAL, "fixture %d shape type %d (circle, edge or polygon)", f, d->shape_type[f]);
        if (d->shape_type[f] == gb::EDGE && d->count[f] != 2)
            return fail(GOIB2D_EINVAL, "edge fixture %d has vertex count %d (2)", f, d->count[f]);
    }
    for (int j = 0; j < J; ++j)
        if (d->joint_a[j] < 0 || d->joint_a[j] >= B || d->joint_b[j] < 0 || d->joint_b[j] >= B)
            return fail(GOIB2D_EINVAL, "joint %d bodies", j);
    for (int p = 0; p < P; ++p) {
        if (d->pair_a[p] < 0 || d->pair_a[p] >= F || d->pair_b[p] < 0 || d->pair_b[p] >= F)
            return fail(GOIB2D_EINVAL, "pair %d fixtures", p);
        if (d->shape_type[d->pair_b[p]] == gb::EDGE ||
            (d->shape_type[d->pair_a[p]] == gb::CIRCLE && d->shape_type[d->pair_b[p]] == gb::POLYGON))
            return fail(GOIB2D_EINVAL, "pair %d: an edge pair lists the edge first, a polygon-circle pair the polygon "
                        "(and two edges never collide)", p);
    }
    auto *m = new goib2d_model();
    int rc = 0;
    cudaGetDevice(&m->device);
    gb::DevModel &g = m->full;
    g.B = B, g.F = F, g.J = J, g.P = P;
    std::vector<int32_t> ident(F > 0 ? F : 1);
    for (int f = 0; f < F; ++f) ident[f] = f;
    int any_toi = 0;
    if (d->toi_bodies) {
        for (int b = 0; b < B; ++b) any_toi |= d->toi_bodies[b] != 0;
    } else {
        any_toi = 1;
    }
    g.any_toi_body = any_toi;
#define UP(field, n) \
    if (!rc) rc = upload(m->allocs, d->field, (size_t)(n), &g.field)
    UP(fixture_body, F);
    UP(shape_type, F);
    UP(count, F);
    UP(radius, F);
    UP(verts, 16 * (size_t)F);
    UP(normals, 16 * (size_t)F);
    UP(joint_type, J);
    UP(joint_a, J);
    UP(joint_b, J);
    UP(local_anchor_a, 2 * (size_t)J);
    UP(local_anchor_b, 2 * (size_t)J);
    UP(local_axis_a, 2 * (size_t)J);
    UP(local_yaxis_a, 2 * (size_t)J);
    UP(reference_angle, J);
    UP(pair_a, P);
    UP(pair_b, P);
    UP(edge_ghost, F);  // zeros when NULL
#undef UP
    if (!rc) {  // each body's joints, highest index first, with the body at the other end (the island walk's order)
        std::vector<int32_t> jstart(B + 1, 0), jadj(2 * (size_t)(2 * J > 0 ? 2 * J : 1));
        for (int j = 0; j < J; ++j) {
            ++jstart[d->joint_a[j] + 1];
            if (d->joint_b[j] != d->joint_a[j]) ++jstart[d->joint_b[j] + 1];
        }
        for (int b = 0; b < B; ++b) jstart[b + 1] += jstart[b];
        std::vector<int32_t> pos(jstart.begin(), jstart.end() - 1);
        for (int j = J - 1; j >= 0; --j) {
            int a = d->joint_a[j], b = d->joint_b[j];
            jadj[2 * pos[a]] = j, jadj[2 * pos[a] + 1] = b, ++pos[a];
            if (b != a) jadj[2 * pos[b]] = j, jadj[2 * pos[b] + 1] = a, ++pos[b];
        }
        rc = upload(m->allocs, jstart.data(), jstart.size(), &g.jadj_start);
        if (!rc) rc = upload(m->allocs, jadj.data(), jadj.size(), &g.jadj);
    }
    const int32_t *d_ident = nullptr;
    if (!rc) rc = upload(m->allocs, ident.data(), (size_t)F, &d_ident);
    g.fixture_slot = d_ident, g.row_fixture = d_ident, g.compact = 0;
    const float *zf = nullptr;
    if (!rc) rc = upload<float>(m->allocs, nullptr, 4 * (size_t)(F > 0 ? F : 1), &zf);
    g.static_fat = zf, g.static_friction = zf, g.static_restitution = zf;
    m->compact = g;
    if (!rc && d->fixture_slot) {
        if (!d->static_fat || !d->static_friction || !d->static_restitution) {
            rc = fail(GOIB2D_EINVAL, "compact model without static fixture tables");
        } else {
            std::vector<int32_t> rows;
            for (int f = 0; f < F; ++f)
                if (d->fixture_slot[f] >= 0) {
                    if (d->fixture_slot[f] != (int)rows.size()) {
                        rc = fail(GOIB2D_EINVAL, "fixture_slot must number the non-static fixtures in order");
                        break;
                    }
                    rows.push_back(f);
                }
            gb::DevModel &c = m->compact;
            const int32_t *slot = nullptr, *rowf = nullptr;
            const float *sf = nullptr, *sfr = nullptr, *srs = nullptr;
            if (!rc) rc = upload(m->allocs, d->fixture_slot, (size_t)F, &slot);
            if (!rc) rc = upload(m->allocs, rows.data(), rows.size(), &rowf);
            if (!rc) rc = upload(m->allocs, d->static_fat, 4 * (size_t)F, &sf);
            if (!rc) rc = upload(m->allocs, d->static_friction, (size_t)F, &sfr);
            if (!rc) rc = upload(m->allocs, d->static_restitution, (size_t)F, &srs);
            c.fixture_slot = slot, c.row_fixture = rowf, c.static_fat = sf, c.static_friction = sfr;
            c.static_restitution = srs, c.compact = 1;
            m->has_compact = 1, m->n_rows_compact = (int)rows.size();
            if (!rc) rc = build_grid(*d, rows, m->allocs, c);
        }
    }
    if (rc) {
        goib2d_model_destroy(m);
        return rc;
    }
    *out = m;
    return 0;
}

int goib2d_model_destroy(goib2d_model *m) {
    if (!m) return 0;
    for (void *p : m->allocs) cudaFree(p);
    if (m->scratch) cudaFree(m->scratch);
    if (m->status) cudaFree(m->status);
    if (m->action_joint) cudaFree(m->action_joint);
    if (m->action_scale) cudaFree(m->action_scale);
    if (m->events) cudaFree(m->events);
    if (m->event_count) cudaFree(m->event_count);
    delete m;
    return 0;
}

int goib2d_model_set_action_map(goib2d_model *m, int32_t n, const int32_t *joint, const float *scale) {
    if (!m) return fail(GOIB2D_EINVAL, "null model");
    if (n < 0 || n > 32) return fail(GOIB2D_EINVAL, "action channels %d outside 0..32", n);
    std::lock_guard<std::mutex> lk(m->mu);
    for (int k = 0; k < n; ++k)
        if (!joint || !scale || joint[k] < 0 || joint[k] >= m->full.J)
            return fail(GOIB2D_EINVAL, "action channel %d joint", k);
    if (m->action_joint) cudaFree(m->action_joint), m->action_joint = nullptr;
    if (m->action_scale) cudaFree(m->action_scale), m->action_scale = nullptr;
    m->n_action = 0;
    if (n == 0) return 0;
    CUDA_TRY(cudaMalloc(&m->action_joint, sizeof(int32_t) * n));
    CUDA_TRY(cudaMalloc(&m->action_scale, sizeof(float) * n));
    CUDA_TRY(cudaMemcpy(m->action_joint, joint, sizeof(int32_t) * n, cudaMemcpyHostToDevice));
    CUDA_TRY(cudaMemcpy(m->action_scale, scale, sizeof(float) * n, cudaMemcpyHostToDevice));
    m->n_action = n;
    return 0;
}

// The validation kernel over a batch (check.cuh) and its result, with the model's mutex held: the first failing
// world (-1 when none) and the leaf that failed. Synchronises the stream.
static const char *leaf_name(int leaf) {
    switch (leaf) {
        case GOIB2D_B_TYPE: return "bodies.type";
        case GOIB2D_J_LIMIT_STATE: return "joints.limit_state";
        case GOIB2D_C_PAIR: return "contacts.pair";
        case GOIB2D_C_FA: return "contacts.fa";
        case GOIB2D_C_FB: return "contacts.fb";
        case GOIB2D_C_COUNT: return "contacts.count";
        case GOIB2D_C_MTYPE: return "contacts.mtype";
        default: return "leaf";
    }
}
static int validate_locked(goib2d_model *m, const gb::DevModel &dm, int32_t C, int64_t n_worlds, void *const *leaves,
                           int64_t *bad_world, int32_t *bad_leaf, cudaStream_t stream) {
    if (!m->check_buf) {
        CUDA_TRY(cudaMalloc(&m->check_buf, sizeof(unsigned long long)));
        m->allocs.push_back(m->check_buf);
    }
    gb::CheckParams p{};
    p.m = dm;
    for (int i = 0; i < GOIB2D_NUM_LEAVES; ++i) p.L.p[i] = leaves[i];
    p.n_worlds = n_worlds, p.C = C, p.first_bad = m->check_buf;
    CUDA_TRY(gb::launch_check(p, stream));
    unsigned long long r = ~0ull;
    CUDA_TRY(cudaMemcpyAsync(&r, m->check_buf, sizeof r, cudaMemcpyDeviceToHost, stream));
    CUDA_TRY(cudaStreamSynchronize(stream));
    *bad_world = r == ~0ull ? -1 : (int64_t)(r >> 8);
    *bad_leaf = r == ~0ull ? -1 : (int32_t)(r & 0xff);
    return 0;
}

int goib2d_set_checks(goib2d_model *m, int32_t on) {
    if (!m) return fail(GOIB2D_EINVAL, "null argument");
    std::lock_guard<std::mutex> lk(m->mu);
    if (on && !m->check_buf) {
        int dev = 0;
        CUDA_TRY(cudaGetDevice(&dev));
        if (dev != m->device) return fail(GOIB2D_EINVAL, "model lives on device %d, current device is %d", m->device,
                                          dev);
        CUDA_TRY(cudaMalloc(&m->check_buf, sizeof(unsigned long long)));
        m->allocs.push_back(m->check_buf);
    }
    m->checks = on ? 1 : 0;
    return 0;
}

int goib2d_validate(goib2d_model *m, int32_t C, int32_t rows, int64_t n_worlds, void *const *leaves,
                    int64_t *bad_world, int32_t *bad_leaf, void *stream) {
    Range range("goib2d_validate");
    if (!m || !leaves || !bad_world || !bad_leaf) return fail(GOIB2D_EINVAL, "null argument");
    if (C < 0 || n_worlds < 0) return fail(GOIB2D_EINVAL, "negative size");
    *bad_world = -1, *bad_leaf = -1;
    std::lock_guard<std::mutex> lk(m->mu);
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev));
    if (dev != m->device) return fail(GOIB2D_EINVAL, "model lives on device %d, current device is %d", m->device, dev);
    const gb::DevModel *dm = nullptr;
    if (rows == m->full.F)
        dm = &m->full;
    else if (m->has_compact && rows == m->n_rows_compact)
        dm = &m->compact;
    else
        return fail(GOIB2D_EINVAL, "fixture rows %d match neither the full (%d) nor the compact (%d) layout", rows,
                    m->full.F, m->has_compact ? m->n_rows_compact : -1);
    for (int i = 0; i < GOIB2D_NUM_LEAVES; ++i)
        if (!leaves[i] && goib2d_leaf_elems(i, dm->B, rows, dm->J, C) > 0 && n_worlds > 0)
            return fail(GOIB2D_EINVAL, "leaf %d is null", i);
    if (n_worlds == 0) return 0;
    return validate_locked(m, *dm, C, n_worlds, leaves, bad_world, bad_leaf, (cudaStream_t)stream);
}

int goib2d_step_seq(goib2d_model *m, const goib2d_settings *s, float dt, int32_t C, int32_t rows, int64_t n_worlds,
                    int32_t n_steps, void *const *leaves, const float *actions, int64_t action_step_stride,
                    void *stream) {
    Range range("goib2d_step_seq");
    if (!m || !s || !leaves) return fail(GOIB2D_EINVAL, "null argument");
    if (C < 0 || n_worlds < 0 || n_steps < 0) return fail(GOIB2D_EINVAL, "negative size");
    if (action_step_stride < 0) return fail(GOIB2D_EINVAL, "negative action step stride");
    if (s->velocity_iterations < 0 || s->position_iterations < 0) return fail(GOIB2D_EINVAL, "negative iterations");
    std::lock_guard<std::mutex> lk(m->mu);
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != m->device) return fail(GOIB2D_EINVAL, "model lives on device %d, current device is %d", m->device, dev);
    const gb::DevModel *dm = nullptr;
    if (rows == m->full.F)
        dm = &m->full;
    else if (m->has_compact && rows == m->n_rows_compact)
        dm = &m->compact;
    else
        return fail(GOIB2D_EINVAL, "fixture rows %d match neither the full (%d) nor the compact (%d) layout", rows,
                    m->full.F, m->has_compact ? m->n_rows_compact : -1);
    for (int i = 0; i < GOIB2D_NUM_LEAVES; ++i)
        if (!leaves[i] && goib2d_leaf_elems(i, dm->B, rows, dm->J, C) > 0 && n_worlds > 0)
            return fail(GOIB2D_EINVAL, "leaf %d is null", i);
    if (n_worlds == 0 || n_steps == 0) return 0;
    if (m->checks) {  // checked stepping: refuse a State whose index fields the kernels cannot use
        int64_t bw = -1;
        int32_t bl = -1;
        int rc = validate_locked(m, *dm, C, n_worlds, leaves, &bw, &bl, (cudaStream_t)stream);
        if (rc) return rc;
        if (bw >= 0) return fail(GOIB2D_EINVAL, "checked step: world %lld has an out-of-range %s; nothing was stepped",
                                 (long long)bw, leaf_name(bl));
    }
    gb::StepParams p{};
    p.m = *dm;
    for (int i = 0; i < GOIB2D_NUM_LEAVES; ++i) p.L.p[i] = leaves[i];
    p.s = *s, p.dt = dt, p.C = C, p.rows = rows, p.n_worlds = n_worlds, p.n_steps = n_steps;
    p.step_mode = m->step_mode;
    p.stage_max = m->stage_max;
    p.lay = scratch_layout(dm->B, C, dm->J, dm->P, dm->grid ? dm->max_hits : 0,
                           gb::hot_budget(n_worlds, dm->J, C, m->step_mode));
    size_t need = (size_t)p.lay.stride * (size_t)n_worlds;
    if (need > m->scratch_bytes) {
        if (m->scratch) cudaFree(m->scratch), m->scratch = nullptr, m->scratch_bytes = 0;
        CUDA_TRY(cudaMalloc(&m->scratch, need));
        m->scratch_bytes = need;
    }
    if (n_worlds > m->status_cap) {
        if (m->status) cudaFree(m->status), m->status = nullptr, m->status_cap = 0;
        CUDA_TRY(cudaMalloc(&m->status, sizeof(int32_t) * n_worlds));
        m->status_cap = n_worlds;
    }
    m->status_n = n_worlds;
    p.scratch = m->scratch, p.status = m->status;
    if (m->event_cap > 0) {  // the contact event log
        if (n_worlds > m->event_worlds) {
            if (m->events) cudaFree(m->events), m->events = nullptr;
            if (m->event_count) cudaFree(m->event_count), m->event_count = nullptr;
            m->event_worlds = 0;
            CUDA_TRY(cudaMalloc(&m->events, sizeof(goib2d_event) * (size_t)m->event_cap * n_worlds));
            CUDA_TRY(cudaMalloc(&m->event_count, sizeof(int32_t) * n_worlds));
            m->event_worlds = n_worlds;
        }
        m->event_n = n_worlds;
        p.events = m->events, p.event_count = m->event_count, p.event_cap = m->event_cap;
    }
    if (actions && m->n_action > 0) {
        const void *a = nullptr;
        int arc = device_view(actions, &a);
        if (arc) return arc;
        p.actions = (const float *)a, p.n_action = m->n_action, p.action_joint = m->action_joint;
        p.action_scale = m->action_scale, p.action_stride = action_step_stride;
    }
    if ((n_worlds + 3) / 4 > 0x7fffffff) return fail(GOIB2D_ELIMIT, "too many worlds");
    CUDA_TRY(gb::launch_steps(p, (cudaStream_t)stream));
    return 0;
}

int goib2d_step(goib2d_model *m, const goib2d_settings *s, float dt, int32_t C, int32_t rows, int64_t n_worlds,
                int32_t n_steps, void *const *leaves, const float *actions, void *stream) {
    return goib2d_step_seq(m, s, dt, C, rows, n_worlds, n_steps, leaves, actions, 0, stream);
}

int goib2d_set_step_mode(goib2d_model *m, int32_t mode) {
    if (!m) return fail(GOIB2D_EINVAL, "null argument");
    if (mode < 0 || mode > 2) return fail(GOIB2D_EINVAL, "step mode %d: 0 (per batch), 1 or 2 worlds per warp", mode);
    std::lock_guard<std::mutex> lk(m->mu);
    m->step_mode = mode;
    return 0;
}

int goib2d_set_state_staging(goib2d_model *m, int32_t max_bytes_per_world) {
    if (!m) return fail(GOIB2D_EINVAL, "null argument");
    if (max_bytes_per_world < 0) return fail(GOIB2D_EINVAL, "negative staging size");
    std::lock_guard<std::mutex> lk(m->mu);
    m->stage_max = max_bytes_per_world;
    return 0;
}

int goib2d_set_event_log(goib2d_model *m, int32_t capacity) {
    if (!m) return fail(GOIB2D_EINVAL, "null argument");
    if (capacity < 0) return fail(GOIB2D_EINVAL, "negative capacity");
    std::lock_guard<std::mutex> lk(m->mu);
    if (capacity != m->event_cap) {  // the buffers follow the next step's batch
        if (m->events) cudaFree(m->events), m->events = nullptr;
        if (m->event_count) cudaFree(m->event_count), m->event_count = nullptr;
        m->event_worlds = m->event_n = 0;
    }
    m->event_cap = capacity;
    return 0;
}

int goib2d_events(goib2d_model *m, const goib2d_event **events, const int32_t **counts, int64_t *n, int32_t *cap) {
    if (!m || !events || !counts || !n || !cap) return fail(GOIB2D_EINVAL, "null argument");
    *events = m->events, *counts = m->event_count, *n = m->event_n, *cap = m->event_cap;
    return 0;
}

int goib2d_events_copy(goib2d_model *m, goib2d_event *host_events, int32_t *host_counts, int64_t n) {
    if (!m || ((!host_events || !host_counts) && n)) return fail(GOIB2D_EINVAL, "null argument");
    if (n > m->event_n) return fail(GOIB2D_EINVAL, "%lld worlds requested, the log holds %lld", (long long)n,
                                    (long long)m->event_n);
    if (n == 0 || m->event_cap == 0) return 0;
    CUDA_TRY(cudaMemcpy(host_events, m->events, sizeof(goib2d_event) * (size_t)m->event_cap * n,
                        cudaMemcpyDeviceToHost));
    CUDA_TRY(cudaMemcpy(host_counts, m->event_count, sizeof(int32_t) * n, cudaMemcpyDeviceToHost));
    return 0;
}

int goib2d_status(goib2d_model *m, const int32_t **device_status, int64_t *n) {
    if (!m || !device_status || !n) return fail(GOIB2D_EINVAL, "null argument");
    *device_status = m->status, *n = m->status_n;
    return 0;
}

int goib2d_status_copy(goib2d_model *m, int32_t *host, int64_t n) {
    if (!m || (!host && n)) return fail(GOIB2D_EINVAL, "null argument");
    if (n < 0 || n > m->status_n) return fail(GOIB2D_EINVAL, "status count %lld outside 0..%lld", (long long)n,
                                              (long long)m->status_n);
    if (n) CUDA_TRY(cudaMemcpy(host, m->status, sizeof(int32_t) * n, cudaMemcpyDeviceToHost));
    return 0;
}

// ---- goib2d_step_noalloc: the step without any device allocation
//
// Some callers cannot allocate device memory at the moment they step: code running while a stream is being
// captured into a CUDA graph, a host that hands every byte of the GPU to its own pool allocator, or a real-time loop
// that forbids allocation after start-up. goib2d_step allocates its per-world scratch arena on first use (and grows
// it); this variant takes the arena from a file-scope device array instead, so it calls no cudaMalloc, cudaFree or
// allocating library routine. The array is GOIB2D_NOALLOC_SCRATCH_BYTES on every device that loads this library, held
// until the process exits. In host code the array's name is only a host-side stand-in, so its device address is
// looked up with cudaGetSymbolAddress once per device (by that device's first call, which should therefore come
// before any stream capture). All calls share the array: calls that overlap on the GPU (other streams, other host
// threads) race on it and must be serialised by the caller. The kernel initialises every scratch word it reads
// within a call, so the contents left by an earlier call never matter and nothing is cleared here.

static __device__ __align__(256) unsigned char g_noalloc_scratch[GOIB2D_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
char *g_noalloc_ptr[kMaxDevices] = {};
}  // namespace

int goib2d_step_noalloc(goib2d_model *m, const goib2d_settings *s, float dt, int32_t C, int32_t rows,
                        int64_t n_worlds, int32_t n_steps, void *const *leaves, const float *actions, void *stream) {
    if (!m || !s || !leaves) return fail(GOIB2D_EINVAL, "null argument");
    if (C < 0 || n_worlds < 0 || n_steps < 0) return fail(GOIB2D_EINVAL, "negative size");
    if (s->velocity_iterations < 0 || s->position_iterations < 0) return fail(GOIB2D_EINVAL, "negative iterations");
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return fail(GOIB2D_ELIMIT, "device %d beyond %d", dev, kMaxDevices);
    if (dev != m->device) return fail(GOIB2D_EINVAL, "model lives on device %d, current device is %d", m->device, dev);
    char *scratch = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        if (!g_noalloc_ptr[dev]) {  // set-up, once per device, with that device current
            void *ptr = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
            if (e != cudaSuccess)
                return fail(GOIB2D_ECUDA, "cudaGetSymbolAddress(no-alloc scratch): %s", cudaGetErrorString(e));
            g_noalloc_ptr[dev] = (char *)ptr;
        }
        scratch = g_noalloc_ptr[dev];
    }
    std::lock_guard<std::mutex> lk(m->mu);
    const gb::DevModel *dm = nullptr;
    if (rows == m->full.F)
        dm = &m->full;
    else if (m->has_compact && rows == m->n_rows_compact)
        dm = &m->compact;
    else
        return fail(GOIB2D_EINVAL, "fixture rows %d match neither the full (%d) nor the compact (%d) layout", rows,
                    m->full.F, m->has_compact ? m->n_rows_compact : -1);
    for (int i = 0; i < GOIB2D_NUM_LEAVES; ++i)
        if (!leaves[i] && goib2d_leaf_elems(i, dm->B, rows, dm->J, C) > 0 && n_worlds > 0)
            return fail(GOIB2D_EINVAL, "leaf %d is null", i);
    gb::StepParams p{};
    p.lay = scratch_layout(dm->B, C, dm->J, dm->P, dm->grid ? dm->max_hits : 0);
    // The arena's size bounds the batch far below the grid-size limit goib2d_step checks ((n_worlds + 3) / 4 blocks
    // < 2^31): a world's arena stride is at least 256 bytes, so at most 131072 worlds fit.
    const int64_t max_worlds = (int64_t)GOIB2D_NOALLOC_SCRATCH_BYTES / p.lay.stride;
    if (n_worlds > max_worlds)
        return fail(GOIB2D_ELIMIT,
                    "goib2d_step_noalloc: %lld worlds need %lld bytes of scratch, the static arena holds %lld bytes "
                    "(%lld worlds of %lld bytes each); use goib2d_step or fewer worlds per call",
                    (long long)n_worlds, (long long)(n_worlds * p.lay.stride),
                    (long long)GOIB2D_NOALLOC_SCRATCH_BYTES, (long long)max_worlds, (long long)p.lay.stride);
    if (n_worlds == 0 || n_steps == 0) return 0;
    p.m = *dm;
    for (int i = 0; i < GOIB2D_NUM_LEAVES; ++i) p.L.p[i] = leaves[i];
    p.s = *s, p.dt = dt, p.C = C, p.rows = rows, p.n_worlds = n_worlds, p.n_steps = n_steps;
    p.step_mode = m->step_mode;
    p.stage_max = m->stage_max;
    p.scratch = scratch;
    p.status = nullptr;  // no per-world status words (their buffer would need an allocation) ...
    p.events = nullptr;  // ... and no event log: neither reports an earlier call's results as this one's
    m->status_n = 0, m->event_n = 0;
    if (actions && m->n_action > 0) {
        const void *a = nullptr;
        int arc = device_view(actions, &a);
        if (arc) return arc;
        p.actions = (const float *)a, p.n_action = m->n_action, p.action_joint = m->action_joint;
        p.action_scale = m->action_scale;
    }
    CUDA_TRY(gb::launch_steps(p, (cudaStream_t)stream));
    return 0;
}

// ---- env helpers (env.cuh)
namespace {
// the Model layout a call's fixture_rows selects (as goib2d_step does)
int pick_layout(goib2d_model *m, int32_t rows, const gb::DevModel **dm) {
    if (rows == m->full.F)
        *dm = &m->full;
    else if (m->has_compact && rows == m->n_rows_compact)
        *dm = &m->compact;
    else
        return fail(GOIB2D_EINVAL, "fixture rows %d match neither the full (%d) nor the compact (%d) layout", rows,
                    m->full.F, m->has_compact ? m->n_rows_compact : -1);
    return 0;
}
int env_params(goib2d_model *m, int32_t C, int32_t rows, int64_t n_worlds, void *const *leaves, gb::EnvParams &p) {
    if (!m || !leaves) return fail(GOIB2D_EINVAL, "null argument");
    if (C < 0 || n_worlds < 0) return fail(GOIB2D_EINVAL, "negative size");
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev));
    if (dev != m->device) return fail(GOIB2D_EINVAL, "model lives on device %d, current device is %d", m->device, dev);
    const gb::DevModel *dm = nullptr;
    int rc = pick_layout(m, rows, &dm);
    if (rc) return rc;
    p = gb::EnvParams{};
    p.m = *dm;
    p.n_worlds = n_worlds, p.B = dm->B, p.rows = rows;
    for (int i = 0; i < GOIB2D_NUM_LEAVES; ++i) {
        if (!leaves[i] && goib2d_leaf_elems(i, dm->B, rows, dm->J, C) > 0 && n_worlds > 0)
            return fail(GOIB2D_EINVAL, "leaf %d is null", i);
        p.L.p[i] = leaves[i];
        p.leaf_bytes[i] = (int32_t)(goib2d_leaf_elems(i, dm->B, rows, dm->J, C) * (LEAVES[i].dtype == 2 ? 1 : 4));
    }
    return 0;
}
}  // namespace

int goib2d_reset_masked(goib2d_model *m, int32_t C, int32_t rows, int64_t n_worlds, void *const *leaves,
                        void *const *init_leaves, const uint8_t *mask, void *stream) {
    Range range("goib2d_reset_masked");
    gb::EnvParams p;
    int rc = env_params(m, C, rows, n_worlds, leaves, p);
    if (rc) return rc;
    if (!init_leaves || (!mask && n_worlds > 0)) return fail(GOIB2D_EINVAL, "null argument");
    for (int i = 0; i < GOIB2D_NUM_LEAVES; ++i) p.I.p[i] = init_leaves[i];
    p.mask = mask;
    CUDA_TRY(gb::launch_reset(p, (cudaStream_t)stream));
    return 0;
}

int goib2d_reset_below(goib2d_model *m, int32_t C, int32_t rows, int64_t n_worlds, void *const *leaves,
                       void *const *init_leaves, int32_t body, float y_min, int32_t *reset_count, void *stream) {
    Range range("goib2d_reset_below");
    gb::EnvParams p;
    int rc = env_params(m, C, rows, n_worlds, leaves, p);
    if (rc) return rc;
    if (!init_leaves) return fail(GOIB2D_EINVAL, "null argument");
    if (body < 0 || body >= p.B) return fail(GOIB2D_EINVAL, "body %d out of range", body);
    for (int i = 0; i < GOIB2D_NUM_LEAVES; ++i) p.I.p[i] = init_leaves[i];
    p.body = body, p.y_min = y_min, p.reset_count = reset_count;
    CUDA_TRY(gb::launch_reset(p, (cudaStream_t)stream));
    return 0;
}

int goib2d_observe(goib2d_model *m, int32_t C, int32_t rows, int64_t n_worlds, void *const *leaves, int32_t n_bodies,
                   const int32_t *bodies, float *out, void *stream) {
    Range range("goib2d_observe");
    gb::EnvParams p;
    int rc = env_params(m, C, rows, n_worlds, leaves, p);
    if (rc) return rc;
    if (n_bodies < 0 || n_bodies > 16) return fail(GOIB2D_ELIMIT, "%d observed bodies (16 at most)", n_bodies);
    if ((n_bodies && !bodies) || (!out && n_worlds && n_bodies)) return fail(GOIB2D_EINVAL, "null argument");
    for (int k = 0; k < n_bodies; ++k) {
        if (bodies[k] < 0 || bodies[k] >= p.B) return fail(GOIB2D_EINVAL, "body %d out of range", bodies[k]);
        p.obs_body[k] = bodies[k];
    }
    const void *o = nullptr;
    if ((rc = device_view(out, &o))) return rc;
    p.n_obs = n_bodies, p.out = (float *)o;
    CUDA_TRY(gb::launch_observe(p, (cudaStream_t)stream));
    return 0;
}

int goib2d_raycast(goib2d_model *m, int32_t C, int32_t rows, int64_t n_worlds, void *const *leaves, int32_t body,
                   int32_t n_rays, float max_length, float *out, void *stream) {
    Range range("goib2d_raycast");
    gb::EnvParams p;
    int rc = env_params(m, C, rows, n_worlds, leaves, p);
    if (rc) return rc;
    if (body < 0 || body >= p.B) return fail(GOIB2D_EINVAL, "body %d out of range", body);
    if (n_rays < 0 || (!out && n_worlds && n_rays)) return fail(GOIB2D_EINVAL, "bad ray arguments");
    const void *o = nullptr;
    if ((rc = device_view(out, &o))) return rc;
    p.body = body, p.n_rays = n_rays, p.max_length = max_length, p.out = (float *)o;
    CUDA_TRY(gb::launch_raycast(p, (cudaStream_t)stream));
    return 0;
}

// ---- scene spawn on the device (spawn.cuh)
int goib2d_spawn(goib2d_model *m, int32_t C, int32_t rows, int64_t n_worlds, void *const *leaves,
                 void *const *template_leaves, int32_t first_body, int32_t n_placed, const float *placements,
                 int32_t n_speeds, const int32_t *speed_joints, const float *speeds, void *stream) {
    Range range("goib2d_spawn");
    gb::EnvParams p;
    int rc = env_params(m, C, rows, n_worlds, leaves, p);
    if (rc) return rc;
    if (!template_leaves) return fail(GOIB2D_EINVAL, "null argument");
    for (int i = 0; i < GOIB2D_NUM_LEAVES; ++i) {
        if (!template_leaves[i] && p.leaf_bytes[i] > 0) return fail(GOIB2D_EINVAL, "template leaf %d is null", i);
        p.I.p[i] = template_leaves[i];
    }
    if (first_body < 0 || n_placed < 0 || (int64_t)first_body + n_placed > p.B)
        return fail(GOIB2D_EINVAL, "placed bodies %d..%d outside 0..%d", first_body, first_body + n_placed - 1, p.B - 1);
    if (n_placed > 0 && n_worlds > 0 && !placements) return fail(GOIB2D_EINVAL, "null placements");
    if (n_speeds < 0 || n_speeds > 16) return fail(GOIB2D_ELIMIT, "%d motor speeds per world (16 at most)", n_speeds);
    if (n_speeds > 0 && (!speed_joints || (!speeds && n_worlds > 0))) return fail(GOIB2D_EINVAL, "null speeds");
    p.J = p.m.J;
    for (int k = 0; k < n_speeds; ++k) {
        if (speed_joints[k] < 0 || speed_joints[k] >= p.J) return fail(GOIB2D_EINVAL, "joint %d out of range",
                                                                         speed_joints[k]);
        p.speed_joint[k] = speed_joints[k];
    }
    const void *pl = nullptr, *sp = nullptr;
    if ((rc = device_view(n_placed > 0 ? placements : nullptr, &pl))) return rc;
    if ((rc = device_view(n_speeds > 0 ? speeds : nullptr, &sp))) return rc;
    p.first_body = first_body, p.n_placed = n_placed, p.placements = (const float *)pl;
    p.n_speeds = n_speeds, p.speeds = (const float *)sp;
    CUDA_TRY(gb::launch_spawn(p, (cudaStream_t)stream));
    return 0;
}

int goib2d_seed_placements(const goib2d_spawn_rule *rule, uint64_t seed, int64_t first_world, int64_t n_worlds,
                           float *placements, float *speeds, void *stream) {
    Range range("goib2d_seed_placements");
    if (!rule) return fail(GOIB2D_EINVAL, "null argument");
    if (first_world < 0 || n_worlds < 0) return fail(GOIB2D_EINVAL, "negative world range");
    const goib2d_spawn_rule &r = *rule;
    if (r.kind < GOIB2D_SPAWN_UNIFORM || r.kind > GOIB2D_SPAWN_RIG) return fail(GOIB2D_EINVAL, "rule kind %d", r.kind);
    const int nb = r.kind == GOIB2D_SPAWN_RIG ? 3 : r.n_bodies;
    if (nb < 0 || nb > 65536) return fail(GOIB2D_ELIMIT, "%d bodies per world (65536 at most)", nb);
    if (r.kind == GOIB2D_SPAWN_RIG && r.n_bodies != 3) return fail(GOIB2D_EINVAL, "the rig rule places 3 bodies");
    if (r.kind == GOIB2D_SPAWN_GRID && r.grid_side < 1) return fail(GOIB2D_EINVAL, "grid_side %d", r.grid_side);
    if (r.kind == GOIB2D_SPAWN_RIG) {
        if (r.max_tries < 1 || r.max_tries > 4096) return fail(GOIB2D_ELIMIT, "max_tries %d (1..4096)", r.max_tries);
        if (r.n_heights < 1 || !r.heights) return fail(GOIB2D_EINVAL, "the rig rule needs a height field");
        if (r.n_discs < 0 || (r.n_discs > 0 && !r.discs)) return fail(GOIB2D_EINVAL, "bad discs");
        if (!(r.h_dx > 0.0f)) return fail(GOIB2D_EINVAL, "h_dx must be positive");
        if (n_worlds > 0 && !speeds) return fail(GOIB2D_EINVAL, "the rig rule writes motor speeds: null speeds");
    }
    if (n_worlds > 0 && nb > 0 && !placements) return fail(GOIB2D_EINVAL, "null placements");
    if ((uint64_t)(first_world + n_worlds) >> 63) return fail(GOIB2D_ELIMIT, "world range overflows");
    gb::SeedParams p{};
    p.rule = r;
    int rc;
    const void *v = nullptr;
    if (r.kind == GOIB2D_SPAWN_RIG) {
        if ((rc = device_view(r.heights, &v))) return rc;
        p.rule.heights = (const float *)v;
        if ((rc = device_view(r.n_discs > 0 ? r.discs : nullptr, &v))) return rc;
        p.rule.discs = (const float *)v;
        if ((rc = device_view(speeds, &v))) return rc;
        p.speeds = (float *)v;
    }
    if ((rc = device_view(placements, &v))) return rc;
    p.placements = (float *)v;
    p.key0 = (uint32_t)seed, p.key1 = (uint32_t)(seed >> 32);
    p.first_world = first_world, p.n_worlds = n_worlds;
    CUDA_TRY(gb::launch_seed(p, (cudaStream_t)stream));
    return 0;
}

int goib2d_candidate_pairs(const goib2d_pair_desc *d, int32_t *pair_a, int32_t *pair_b, int64_t capacity,
                           int64_t *n_pairs) {
    Range range("goib2d_candidate_pairs");
    if (!d || !n_pairs) return fail(GOIB2D_EINVAL, "null argument");
    *n_pairs = 0;
    const int B = d->n_bodies, F = d->n_fixtures, J = d->n_joints;
    if (B < 0 || F < 0 || J < 0 || capacity < 0) return fail(GOIB2D_EINVAL, "negative size");
    if (F && (!d->fixture_body || !d->shape_type || !d->sensor || !d->category || !d->mask || !d->group || !d->layer))
        return fail(GOIB2D_EINVAL, "null fixture array");
    if ((B && !d->body_type) || (J && (!d->joint_a || !d->joint_b || !d->joint_collide)))
        return fail(GOIB2D_EINVAL, "null body or joint array");
    for (int f = 0; f < F; ++f)
        if (d->fixture_body[f] < 0 || d->fixture_body[f] >= B) return fail(GOIB2D_EINVAL, "fixture %d body", f);
    std::vector<int64_t> keys;  // bodies joined without collideConnected
    for (int j = 0; j < J; ++j) {
        int a = d->joint_a[j], b = d->joint_b[j];
        if (a < 0 || a >= B || b < 0 || b >= B) return fail(GOIB2D_EINVAL, "joint %d bodies", j);
        if (!d->joint_collide[j]) keys.push_back(a < b ? ((int64_t)a << 32) | b : ((int64_t)b << 32) | a);
    }
    std::sort(keys.begin(), keys.end());
    keys.erase(std::unique(keys.begin(), keys.end()), keys.end());
    if (F == 0) return 0;
    std::vector<void *> tmp;
    struct Free {
        std::vector<void *> &v;
        ~Free() {
            for (void *p : v) cudaFree(p);
        }
    } release{tmp};
    gb::PairScene s{};
    s.F = F, s.J = J, s.n_no_collide = (int)keys.size();
    int rc = 0;
    rc = rc ? rc : upload(tmp, d->fixture_body, (size_t)F, &s.fixture_body);
    rc = rc ? rc : upload(tmp, d->shape_type, (size_t)F, &s.shape_type);
    rc = rc ? rc : upload(tmp, d->body_type, (size_t)B, &s.body_type);
    rc = rc ? rc : upload(tmp, d->sensor, (size_t)F, &s.sensor);
    rc = rc ? rc : upload(tmp, d->category, (size_t)F, &s.category);
    rc = rc ? rc : upload(tmp, d->mask, (size_t)F, &s.mask);
    rc = rc ? rc : upload(tmp, d->group, (size_t)F, &s.group);
    rc = rc ? rc : upload(tmp, d->layer, (size_t)F, &s.layer);
    rc = rc ? rc : upload(tmp, (const int64_t *)keys.data(), keys.size(), &s.no_collide);
    if (!rc && d->layer_masks) rc = upload(tmp, d->layer_masks, 32, &s.layer_masks);
    if (rc) return rc;
    const int64_t *count_c = nullptr;
    if ((rc = upload<int64_t>(tmp, nullptr, (size_t)F, &count_c))) return rc;
    int64_t *count = const_cast<int64_t *>(count_c);
    CUDA_TRY(gb::launch_pair_count(s, count));
    std::vector<int64_t> start((size_t)F + 1, 0);
    CUDA_TRY(cudaMemcpy(start.data() + 1, count, sizeof(int64_t) * F, cudaMemcpyDeviceToHost));
    for (int f = 0; f < F; ++f) start[f + 1] += start[f];
    *n_pairs = start[F];
    if (start[F] > capacity) return fail(GOIB2D_ELIMIT, "%lld candidate pairs, capacity %lld", (long long)start[F],
                                         (long long)capacity);
    if (start[F] == 0) return 0;
    if (!pair_a || !pair_b) return fail(GOIB2D_EINVAL, "null output");
    const int64_t *d_start = nullptr;
    const int32_t *d_pa = nullptr, *d_pb = nullptr;
    rc = rc ? rc : upload(tmp, start.data(), (size_t)F, &d_start);
    rc = rc ? rc : upload<int32_t>(tmp, nullptr, (size_t)start[F], &d_pa);
    rc = rc ? rc : upload<int32_t>(tmp, nullptr, (size_t)start[F], &d_pb);
    if (rc) return rc;
    CUDA_TRY(gb::launch_pair_fill(s, d_start, const_cast<int32_t *>(d_pa), const_cast<int32_t *>(d_pb)));
    CUDA_TRY(cudaMemcpy(pair_a, d_pa, sizeof(int32_t) * start[F], cudaMemcpyDeviceToHost));
    CUDA_TRY(cudaMemcpy(pair_b, d_pb, sizeof(int32_t) * start[F], cudaMemcpyDeviceToHost));
    return 0;
}

}  // extern "C"
