// goib2d: the batched b2World::Step for sm_100a. One warp (or half-warp) per world; every step of a call runs in one
// persistent launch (goib2d_step_kernel / goib2d_step_pair_kernel), or, for batches of 16384 worlds and more of
// joint-heavy models, as a sequence of part kernels per step.
//
// Mapping. Each world's State is a row of every leaf (contiguous per world), so a warp reads and writes its own
// world with unit-stride lane accesses. Data-parallel phases run one element per lane: the candidate-pair queries
// (ballot-compacted), the narrow phase over contact slots, constraint set-up, integration, fixture synchronisation,
// b2TimeOfImpact over the TOI candidates and the levelled island sweeps. The phases whose order defines the floats -
// Collide's wake walk, the island DFS, the Gauss-Seidel sweeps of small islands and the TOI island walk - run on
// lane 0 in exactly the reference's order (goi_jax/box2d/step.py, island.py, pairs.py, toi.py), or are restructured
// so that every float is computed from the same inputs in the same order, so results are bit-identical to it.
// Per-world working arrays live in a scratch arena (its hot part in shared memory), laid out by scratch_layout().
#include <climits>
#include <cstdio>
#include <mutex>

// Optional per-phase cycle counters for profiling builds (-DGOIB2D_PHASE_TIMERS): lane 0 of every warp adds the
// clock64 cycles spent in each phase; goib2d_debug_phase_cycles() reads them. Compiled out otherwise.
#ifdef GOIB2D_PHASE_TIMERS
namespace gb {
__device__ unsigned long long g_phase_cycles[16];
__device__ unsigned long long g_phase_max[16];  // the longest single warp's time in each phase
#define GB_PHASE(x, i)                                                                             \
    do {                                                                                           \
        long long t1_ = clock64();                                                                 \
        if ((x).lane == 0) {                                                                       \
            atomicAdd(&g_phase_cycles[i], (unsigned long long)(t1_ - (x).t0));                     \
            atomicMax(&g_phase_max[i], (unsigned long long)(t1_ - (x).t0));                        \
        }                                                                                          \
        (x).t0 = t1_;                                                                              \
    } while (0)
// 0 events, 1 TOI position passes, 2 TOI solves, 3 searches, 4 max events, 5 TOI cycles, 6 outer iterations,
// 7 push-backs, 8 root-finder steps, 9 GJK iterations, 10-13 TOI outcomes
__device__ unsigned long long g_counts[16];
// cycles in the TOI parts (0 sweep_xf, 1 GJK, 2 sep_init, 3 sep_find_min), in a TOI event's island solve (4 position
// rows, 5 position passes, 6 velocity rows, 7 velocity passes; 11 its contacts) and in a TOI event (12 the walk,
// 13 the island solve, 14 synchronize and FindNewContacts)
__device__ unsigned long long g_toi_cycles[16];
// per-world cycles in a part (sum, worlds, max): 0-2 TOI without events, 3-5 TOI with events, 9-11 collide
__device__ unsigned long long g_span[16];
// cycles in the parts of the levelled sweeps (lane 0): 0 velocity levelling, 1 contacts-first levelling, 2 warm
// start, 3 velocity iterations, 4 impulses and integration, 5 position levels, 6 position reductions
__device__ unsigned long long g_lv_cycles[16];
}  // namespace gb
#define GB_LV_T0(x) long long gb_lv_ = clock64()
#define GB_LV(x, i)                                                                                \
    do {                                                                                           \
        const long long t_ = clock64();                                                            \
        if ((x).lane == 0) atomicAdd(&g_lv_cycles[i], (unsigned long long)(t_ - gb_lv_));          \
        gb_lv_ = t_;                                                                               \
    } while (0)
#define GB_SPAN(x, k, ev)                                                                   \
    do {                                                                                    \
        if ((x).lane == 0) {                                                                \
            unsigned long long d_ = (unsigned long long)(clock64() - gb_span0_);              \
            const int i_ = (k) + 3 * ((ev) ? 1 : 0);                                        \
            atomicAdd(&g_span[i_], d_), atomicAdd(&g_span[i_ + 1], 1ull), atomicMax(&g_span[i_ + 2], d_); \
        }                                                                                   \
    } while (0)
#define GB_COUNT(i, v) atomicAdd(&g_counts[i], (unsigned long long)(v))
#define GB_TOI_T0() long long gb_t0_ = clock64()
#define GB_TOI_T1(i) atomicAdd(&g_toi_cycles[i], (unsigned long long)(clock64() - gb_t0_))
#else
#define GB_PHASE(x, i) \
    do {               \
    } while (0)
#define GB_COUNT(i, v) \
    do {               \
    } while (0)
#define GB_TOI_T0() \
    do {            \
    } while (0)
#define GB_TOI_T1(i) \
    do {             \
    } while (0)
#define GB_SPAN(x, k, ev) \
    do {                  \
    } while (0)
#define GB_LV_T0(x) \
    do {            \
    } while (0)
#define GB_LV(x, i) \
    do {            \
    } while (0)
#endif

#include "env.cuh"
#include "spawn.cuh"
#include "check.cuh"
#include "scene.cuh"
#include "solver.cuh"
#include "toi.cuh"

namespace gb {

constexpr unsigned FULL = 0xffffffffu;

template <class T>
__device__ __forceinline__ T *sp(char *base, int64_t off) {
    return reinterpret_cast<T *>(base + off);
}

struct Ctx {
    const StepParams &p;
    const DevModel &m;
    const goib2d_settings &s;
    W &w;  // shared memory, one per world: a per-thread copy would cost 32x its size in local memory
    char *scr;   // the world's arena (global memory)
    char *hot;   // this world's shared copy of the arena's hot part (Layout::hot_end), or null
    char *rows;  // this world's shared constraint rows (solve and TOI phases), or null
    int lane;    // the thread's lane in the world's group, 0 .. wl - 1
    int status;
    int step;      // the step of the call being run (0 .. n_steps - 1)
    int fnc_clean; // the world's last FindNewContacts placed every new pair (no overflow); 0 at a kernel's start
    int order_n;   // live contacts of the list order in the arena's order / lpos, if still valid; else -1
    int base_n;    // the arena's order holds the list as of next_key == kref (base_n contacts), or -1 (list_order)
    int kref;
    long long t0;  // phase timer origin (GOIB2D_PHASE_TIMERS builds only)
    int64_t world;
    unsigned gmask;  // the world's lanes in the warp: all 32, or one half (the step kernel: two worlds per warp)
    int gbase, wl;   // the group's first lane in the warp, and its width (32 or 16)
};

// Warp collectives over the world's own group of lanes. Every function below runs all of a world's lanes through
// the same sequence of these calls; the two worlds of a warp may be at different calls at the same time.
__device__ __forceinline__ void gsync(const Ctx &x) { __syncwarp(x.gmask); }
__device__ __forceinline__ unsigned gballot(const Ctx &x, bool pred) {
    return (__ballot_sync(x.gmask, pred) & x.gmask) >> x.gbase;  // bit i: the group's lane i
}
template <class T>
__device__ __forceinline__ T gshfl(const Ctx &x, T v, int src) {  // from the group's lane src
    return __shfl_sync(x.gmask, v, src, x.wl);
}

// ---- contact event log (the reference C API's Begin / End / PostSolve listener, capi.cpp:45-78)
enum { EV_BEGIN = 0, EV_END = 1, EV_POST_SOLVE = 2 };
__device__ __forceinline__ void put_event(const StepParams &p, int64_t world, int idx, int kind, int fa, int fb,
                                          int count = 0, const float *ni = nullptr, const float *ti = nullptr) {
    if (idx >= p.event_cap) return;
    goib2d_event &e = p.events[world * p.event_cap + idx];
    e.kind = kind, e.fixture_a = fa, e.fixture_b = fb, e.child_a = 0, e.child_b = 0, e.count = count;
    for (int j = 0; j < 2; ++j)
        e.normal_impulse[j] = j < count ? ni[j] : 0.0f, e.tangent_impulse[j] = j < count ? ti[j] : 0.0f;
}

// An arena array of the world: in the warp's shared memory when the kernel holds the hot part there, else global.
template <class T>
__device__ __forceinline__ T *ap(const Ctx &x, int64_t off) {
    return reinterpret_cast<T *>((x.hot && off < x.p.lay.hot_end ? x.hot : x.scr) + off);
}


__device__ __forceinline__ void wake_body(W &w, int b) {  // b2Body::SetAwake(true)
    if (!w.awake[b]) {
        w.awake[b] = 1;
        w.sleep_time[b] = 0.0f;
    }
}

// ---------------------------------------------------------------- FindNewContacts (pairs.py:134-178)
// A new contact for every candidate pair whose fat AABBs overlap, whose bodies may collide and that has no contact
// yet, created in candidate (b2BroadPhase::UpdatePairs) order into the lowest free slots. Two exact ways to find the
// pairs: the grid path (compact models) asks the static-fixture grid for each non-static fixture's neighbours and
// scans only the pairs of two non-static fixtures, then sorts its hits into candidate order; the scan path tests
// every candidate in order (full-layout models, or more hits than the grid path's buffer holds).

__device__ __forceinline__ void place_contact(Ctx &x, int s, int p, int key) {
    const DevModel &m = x.m;
    W &w = x.w;
    const int fa = m.pair_a[p], fb = m.pair_b[p];  // every load first, the stores last
    const float fra = fixture_friction(m, w, fa), frb = fixture_friction(m, w, fb);
    const float ra = fixture_restitution(m, w, fa), rb = fixture_restitution(m, w, fb);
    const int ba = m.fixture_body[fa], bb = m.fixture_body[fb];
    w.pair[s] = p, w.fa[s] = fa, w.fb[s] = fb, w.key[s] = key;
    w.touching[s] = 0, w.count[s] = 0;
    w.normal_impulse[2 * s] = w.normal_impulse[2 * s + 1] = 0.0f;
    w.tangent_impulse[2 * s] = w.tangent_impulse[2 * s + 1] = 0.0f;
    w.point_id[2 * s] = w.point_id[2 * s + 1] = 0;
    w.friction[s] = sqrtf(fra * frb);
    w.restitution[s] = ra > rb ? ra : rb;
    w.tangent_speed[s] = 0.0f;
    wake_body(w, ba);
    wake_body(w, bb);
}

// is candidate p a new pair (overlap, ShouldCollide, no contact yet)?
__device__ __forceinline__ bool is_new_pair(Ctx &x, int p, const uint32_t *bitmap) {
    const DevModel &m = x.m;
    const W &w = x.w;
    int fa = m.pair_a[p], fb = m.pair_b[p];
    int ba = m.fixture_body[fa], bb = m.fixture_body[fb];
    if (!overlap(fixture_fat(m, w, fa), fixture_fat(m, w, fb))) return false;
    bool can = (w.type[ba] == DYNAMIC || w.type[bb] == DYNAMIC) && w.active[ba] && w.active[bb];
    return can && !((bitmap[p >> 5] >> (p & 31)) & 1u);
}

// does candidate p join a fixture of a moved body?
__device__ __forceinline__ bool pair_moved(const DevModel &m, int p, const int *moved) {
    return moved[m.fixture_body[m.pair_a[p]]] || moved[m.fixture_body[m.pair_b[p]]];
}

// Exclusive scan of v over the world's lanes; *total = the sum.
__device__ __forceinline__ int gscan(const Ctx &x, int v, int *total) {
    int inc = v;
    for (int o = 1; o < x.wl; o <<= 1) {
        const int t = __shfl_up_sync(x.gmask, inc, o, x.wl);
        if (x.lane >= o) inc += t;
    }
    *total = gshfl(x, inc, x.wl - 1);
    return inc - v;
}
// The lane whose range [off, off + cnt) of an exclusive scan holds position q (q below the total): the last lane
// with a non-empty range starting at or before q. Every lane of the world runs it (its own q).
__device__ __forceinline__ int gowner(const Ctx &x, int off, int cnt, int q) {
    int owner = 0;
    for (int j = 1; j < x.wl; ++j) {
        const int oj = gshfl(x, off, j), cj = gshfl(x, cnt, j);
        if (cj > 0 && oj <= q) owner = j;
    }
    return owner;
}

// the grid path's hits (candidate indices, any order); returns the count, or -1 when the buffer overflowed.
// The query is dealt across the world's lanes in rounds rather than walked cell by cell: per round of WL fixture
// rows, each lane takes a row's cell rectangle; the (row, cell) pairs are then dealt one per lane, each lane reading
// its cell's range of listed static fixtures; and the listed (row, static fixture) items are dealt one per lane for
// the overlap tests. A world's query is thus a few chains of dependent loads instead of one chain per cell.
__device__ int grid_new_pairs(Ctx &x, const uint32_t *bitmap, int *hits, const int *moved) {
    const DevModel &m = x.m;
    const W &w = x.w;
    const int lane = x.lane, cap = m.max_hits, WL = x.wl;
    int n = 0;
    for (int r0 = 0; r0 < m.n_rows; r0 += WL) {
        const int r = r0 + lane;
        int cx0 = 0, cy0 = 0, ncx = 1, nq = 0;
        if (r < m.n_rows && (!moved || moved[m.fixture_body[m.row_fixture[r]]])) {
            const float *dp = w.fx_fat + 4 * r;
            const int ax = grid_cell(dp[0], m.gx0, m.inv_cell, m.nx), bx = grid_cell(dp[2], m.gx0, m.inv_cell, m.nx);
            const int ay = grid_cell(dp[1], m.gy0, m.inv_cell, m.ny), by = grid_cell(dp[3], m.gy0, m.inv_cell, m.ny);
            cx0 = ax, cy0 = ay, ncx = bx - ax + 1, nq = ncx * (by - ay + 1);
        }
        int Q = 0;
        const int qoff = gscan(x, nq, &Q);
        for (int q0 = 0; q0 < Q; q0 += WL) {  // (row, cell) pairs, one per lane
            const int q = q0 + lane;
            const int ro = gowner(x, qoff, nq, q);
            const int o_off = gshfl(x, qoff, ro), o_cx0 = gshfl(x, cx0, ro), o_cy0 = gshfl(x, cy0, ro);
            const int o_ncx = gshfl(x, ncx, ro);
            int row = r0 + ro, cx = 0, cy = 0, b0 = 0, ni = 0;
            if (q < Q) {
                const int l = q - o_off;
                cx = o_cx0 + l % o_ncx, cy = o_cy0 + l / o_ncx;
                const int c = cy * m.nx + cx;
                b0 = m.cell_start[c], ni = m.cell_start[c + 1] - b0;
            }
            int T = 0;
            const int ioff = gscan(x, ni, &T);
            for (int t0 = 0; t0 < T; t0 += WL) {  // listed static fixtures of those cells, one per lane
                const int t = t0 + lane;
                const int co = gowner(x, ioff, ni, t);
                const int c_off = gshfl(x, ioff, co), c_b0 = gshfl(x, b0, co), c_cx = gshfl(x, cx, co);
                const int c_cy = gshfl(x, cy, co), c_row = gshfl(x, row, co);
                int p = -1;
                if (t < T) {
                    const int si = m.cell_items[c_b0 + (t - c_off)];
                    const float *dp = w.fx_fat + 4 * c_row;
                    const AABB D{dp[0], dp[1], dp[2], dp[3]};
                    const float *sf = m.sfat + 4 * si;
                    const AABB S{sf[0], sf[1], sf[2], sf[3]};
                    // report the pair only in the cell holding the lower corner of the two boxes' overlap
                    const bool here = grid_cell(fmaxf(D.lx, S.lx), m.gx0, m.inv_cell, m.nx) == c_cx &&
                                      grid_cell(fmaxf(D.ly, S.ly), m.gy0, m.inv_cell, m.ny) == c_cy;
                    if (here && overlap(D, S)) {
                        const int pc = m.cand_rs[(int64_t)c_row * m.n_static + si];
                        if (pc >= 0 && is_new_pair(x, pc, bitmap)) p = pc;
                    }
                }
                const unsigned mk = gballot(x, p >= 0);
                if (p >= 0) {
                    const int k = n + __popc(mk & ((1u << lane) - 1));
                    if (k < cap) hits[k] = p;
                }
                n += __popc(mk);
            }
        }
    }
    if (!moved) {
        // pairs of two non-static fixtures: every one, DD_UNROLL per lane at a time so that their loads (the pair's
        // rows and bodies in one record, then their boxes, types and the contact bitmap) are in flight together
        constexpr int DD_UNROLL = 4;
        for (int base = 0; base < m.n_dd; base += DD_UNROLL * WL) {
            int p[DD_UNROLL];
            int4 rb[DD_UNROLL];
#pragma unroll
            for (int u = 0; u < DD_UNROLL; ++u) {
                const int i = base + u * WL + lane;
                p[u] = i < m.n_dd ? m.dd[i] : -1;
                rb[u] = i < m.n_dd ? m.dd_rb[i] : make_int4(0, 0, 0, 0);
            }
            bool hit[DD_UNROLL];
#pragma unroll
            for (int u = 0; u < DD_UNROLL; ++u) {  // is_new_pair, from the record
                const float *fa = w.fx_fat + 4 * rb[u].x, *fb = w.fx_fat + 4 * rb[u].y;
                const bool ov = overlap(AABB{fa[0], fa[1], fa[2], fa[3]}, AABB{fb[0], fb[1], fb[2], fb[3]});
                const int ba = rb[u].z, bb = rb[u].w;
                const bool can = (w.type[ba] == DYNAMIC || w.type[bb] == DYNAMIC) && w.active[ba] && w.active[bb];
                hit[u] = p[u] >= 0 && ov && can && !((bitmap[p[u] >> 5] >> (p[u] & 31)) & 1u);
            }
#pragma unroll
            for (int u = 0; u < DD_UNROLL; ++u) {
                const unsigned mk = gballot(x, hit[u]);
                if (hit[u]) {
                    const int k = n + __popc(mk & ((1u << lane) - 1));
                    if (k < cap) hits[k] = p[u];
                }
                n += __popc(mk);
            }
        }
    } else {
        // the pairs of two non-static fixtures that join a moved body's fixture: each moved row's entries of dd, dealt
        // one per lane; a pair whose two rows both moved is taken from its lower row only
        for (int r0 = 0; r0 < m.n_rows; r0 += WL) {
            const int r = r0 + lane;
            const bool mv = r < m.n_rows && moved[m.fixture_body[m.row_fixture[r]]];
            const int e0 = mv ? m.dd_row_start[r] : 0, ne = mv ? m.dd_row_start[r + 1] - e0 : 0;
            int T = 0;
            const int eoff = gscan(x, ne, &T);
            for (int t0 = 0; t0 < T; t0 += WL) {
                const int t = t0 + lane;
                const int co = gowner(x, eoff, ne, t);
                const int c_off = gshfl(x, eoff, co), c_e0 = gshfl(x, e0, co), row = r0 + co;
                int p = -1;
                if (t < T) {
                    const int pc = m.dd[m.dd_row_idx[c_e0 + (t - c_off)]];
                    const int ra = m.fixture_slot[m.pair_a[pc]], rb = m.fixture_slot[m.pair_b[pc]];
                    const int other = ra == row ? rb : ra;
                    const bool twice = other < row && moved[m.fixture_body[m.row_fixture[other]]];
                    if (!twice && is_new_pair(x, pc, bitmap)) p = pc;
                }
                const unsigned mk = gballot(x, p >= 0);
                if (p >= 0) {
                    const int k = n + __popc(mk & ((1u << lane) - 1));
                    if (k < cap) hits[k] = p;
                }
                n += __popc(mk);
            }
        }
    }
    gsync(x);
    return n <= cap ? n : -1;
}

// moved (or null): the call follows a FindNewContacts of this world that placed every new pair, and since then only
// the fixtures of the bodies flagged in moved were re-fattened (a TOI event: b2Island::SolveTOI's bodies) and no
// contact was destroyed. Every other candidate pair then kept its overlap and already has its contact, so only pairs
// joining a moved body's fixture are tested: the same new contacts, slots and keys as testing every pair.
__device__ void find_new_contacts(Ctx &x, const int *moved = nullptr) {
    const DevModel &m = x.m;
    W &w = x.w;
    const int P = m.P, C = w.C, lane = x.lane;
    if (P == 0) return;
#ifdef GOIB2D_PHASE_TIMERS
    const long long fnc_t0 = clock64();
#endif
    uint32_t *bitmap = ap<uint32_t>(x, x.p.lay.bitmap);
    int *freeslot = ap<int>(x, x.p.lay.freeslot);
    const int nw = (P + 31) >> 5;
    for (int i = lane; i < nw; i += x.wl) bitmap[i] = 0u;
    gsync(x);
    for (int s = lane; s < C; s += x.wl) {
        int pr = w.pair[s];
        if (pr >= 0 && pr < P) atomicOr(&bitmap[pr >> 5], 1u << (pr & 31));
    }
    int n_free = 0;
    for (int base = 0; base < C; base += x.wl) {
        int s = base + lane;
        bool f = s < C && w.pair[s] < 0;
        unsigned mk = gballot(x, f);
        if (f) freeslot[n_free + __popc(mk & ((1u << lane) - 1))] = s;
        n_free += __popc(mk);
    }
    const int key0 = *w.next_key;
    gsync(x);
#ifdef GOIB2D_PHASE_TIMERS
    const long long fnc_t1 = clock64();
    if (lane == 0) atomicAdd(&g_toi_cycles[9], (unsigned long long)(fnc_t1 - fnc_t0));
#endif
    int n_new = -1;
    if (m.grid) {
        int *hits = ap<int>(x, x.p.lay.hits), *sorted = hits + m.max_hits;
        n_new = grid_new_pairs(x, bitmap, hits, moved);
        if (n_new > 0) {  // into candidate order (the hits are distinct), then into the lowest free slots
            for (int i = lane; i < n_new; i += x.wl) {
                int h = hits[i], rank = 0;
                for (int j = 0; j < n_new; ++j) rank += hits[j] < h;
                sorted[rank] = h;
            }
            gsync(x);
            for (int k = lane; k < n_new && k < n_free; k += x.wl) place_contact(x, freeslot[k], sorted[k], key0 + k);
        }
    }
    if (n_new < 0) {  // the scan path
        n_new = 0;
        for (int base = 0; base < P; base += x.wl) {
            int p = base + lane;
            bool nw_ = p < P && (!moved || pair_moved(m, p, moved)) && is_new_pair(x, p, bitmap);
            unsigned mk = gballot(x, nw_);
            if (nw_) {
                int rank = n_new + __popc(mk & ((1u << lane) - 1));
                if (rank < n_free) place_contact(x, freeslot[rank], p, key0 + rank);
            }
            n_new += __popc(mk);
        }
    }
    gsync(x);
    if (lane == 0) {
        *w.next_key = key0 + n_new;
        int placed = n_new < n_free ? n_new : n_free;
        *w.overflow += n_new - placed;
        if (n_new > placed) x.status |= ST_OVERFLOW;
    }
#ifdef GOIB2D_PHASE_TIMERS
    if (lane == 0) atomicAdd(&g_toi_cycles[8], (unsigned long long)(clock64() - fnc_t0)), atomicAdd(&g_toi_cycles[10], 1ull);
#endif
    x.fnc_clean = n_new <= n_free;  // both are the same on every lane of the world
    if (n_new > 0 && n_free > 0) x.order_n = -1;  // contacts were placed
    gsync(x);
}

// Live slots in contact-list order (descending key): order[0..n) and each slot's position lpos[slot] (C if dead).
// A list is ranked from the packed keys (key in the high word, the slot's complement in the low word: a larger
// packed key is a larger key, or the same key - never in a valid State - at a lower slot, the order of a stable
// sort): each entry's position is the number of packed keys above its own. The first list of a kernel ranks every
// live slot. Later lists are the earlier one brought up to date: new contacts get keys from next_key upwards, so the
// contacts with a key at or above the earlier list's next_key (kref) are the ones created since - ranked among
// themselves, they come first - and the earlier list's entries that still hold a contact with a key below kref
// follow in their order (a destroyed contact drops out; a slot reused since holds a key at or above kref). A State
// whose live keys reach its next_key (never made by a step) is ranked in full every time.
__device__ __forceinline__ long long list_key(int key, int slot) {
    return (long long)key * 4294967296LL + (long long)(~(unsigned)slot);
}
// rank lk[0 .. n) (packed keys) into out[0 .. n) (slots), descending
__device__ __forceinline__ void rank_desc(const Ctx &x, const long long *lk, int n, int *out) {
    for (int j = x.lane; j < n; j += x.wl) {
        const long long k = lk[j];
        int cnt = 0;
        for (int i = 0; i < n; ++i) cnt += lk[i] > k;
        out[cnt] = (int)~(unsigned)(k & 0xffffffffLL);
    }
}
__device__ int list_order(Ctx &x, int *order, int *lpos) {
    GB_TOI_T0();
    W &w = x.w;
    const int C = w.C, lane = x.lane;
    long long *lk = ap<long long>(x, x.p.lay.lkey);
    int *staged = ap<int>(x, x.p.lay.order2);
    const int kref = x.kref, next_key = *w.next_key;
    const bool incremental = x.base_n >= 0;
    int n_new = 0, max_key = INT_MIN;
    for (int base = 0; base < C; base += x.wl) {  // the live slots (all of them, or those created since kref)
        const int s = base + lane;
        bool pick = false;
        if (s < C && w.pair[s] >= 0) {
            const int k = w.key[s];
            max_key = k > max_key ? k : max_key;
            pick = !incremental || k >= kref;
        }
        const unsigned mk = gballot(x, pick);
        if (pick) lk[n_new + __popc(mk & ((1u << lane) - 1))] = list_key(w.key[s], s);
        n_new += __popc(mk);
    }
    gsync(x);
    rank_desc(x, lk, n_new, staged);
    int n = n_new;
    if (incremental) {  // the earlier list's surviving contacts, in their order, after the new ones
        for (int base = 0; base < x.base_n; base += x.wl) {
            const int j = base + lane;
            int s = -1;
            if (j < x.base_n) {
                s = order[j];
                if (!(w.pair[s] >= 0 && w.key[s] < kref)) s = -1;
            }
            const unsigned mk = gballot(x, s >= 0);
            if (s >= 0) staged[n + __popc(mk & ((1u << lane) - 1))] = s;
            n += __popc(mk);
        }
    }
    gsync(x);
    for (int s = lane; s < C; s += x.wl) lpos[s] = C;
    gsync(x);
    for (int j = lane; j < n; j += x.wl) {
        const int s = staged[j];
        order[j] = s, lpos[s] = j;
    }
    for (int o = x.wl >> 1; o > 0; o >>= 1) {
        const int t = __shfl_xor_sync(x.gmask, max_key, o, x.wl);
        max_key = t > max_key ? t : max_key;
    }
    gsync(x);
    if (x.lane == 0) GB_TOI_T1(15);
    x.order_n = n;
    const bool keys_below = n == 0 || max_key < next_key;  // a State made by steps: every key below next_key
    x.base_n = keys_below ? n : -1, x.kref = next_key;
    return n;
}
// The list order, recomputed only when a contact was created or destroyed since the last list_order: the TOI loop
// (a search, then an event, then a search ...) changes the slots only where an event creates contacts.
__device__ __forceinline__ int list_order_kept(Ctx &x, int *order, int *lpos) {
    return x.order_n >= 0 ? x.order_n : list_order(x, order, lpos);
}

// ---------------------------------------------------------------- b2ContactManager::Collide (pairs.py:38-117)
__device__ void collide(Ctx &x) {
    const DevModel &m = x.m;
    W &w = x.w;
    const int C = w.C, B = w.B, lane = x.lane;
    const Layout &L = x.p.lay;
    int *order = ap<int>(x, L.order), *lpos = ap<int>(x, L.lpos), *active = ap<int>(x, L.active);
    int *over = ap<int>(x, L.over), *aw = ap<int>(x, L.aw);
    Man *man = ap<Man>(x, L.man);
    int n_live = list_order(x, order, lpos);
    for (int s = lane; s < C; s += x.wl) {  // loads first, stores last
        const bool live = w.pair[s] >= 0;
        if (live) {
            const int fa = w.fa[s], fb = w.fb[s];
            const int ba = m.fixture_body[fa], bb = m.fixture_body[fb];
            const Xf xfa = w.bxf(ba), xfb = w.bxf(bb);
            const int ov = overlap(fixture_fat(m, w, fa), fixture_fat(m, w, fb));
            evaluate(m, fa, fb, xfa, xfb, x.s.linear_slop, x.s.angular_slop, man[s]);
            over[s] = ov;
        }
        active[s] = 0;
    }
    for (int b = lane; b < B; b += x.wl) aw[b] = w.awake[b];
    gsync(x);
    // The walk newest first (pairs.py:60-90): a contact is visited when one of its bodies is awake and not static,
    // and a visited contact whose touching state changes wakes both bodies for the contacts after it. Between two
    // wakes of a non-static body nothing changes, so each round settles, in parallel, every contact up to the next
    // such wake, which lane 0 then applies. Wakes of static bodies only reach their awake flag, at the end.
    for (int k0 = 0;;) {
        int first = n_live;
        for (int base = k0; base < n_live; base += x.wl) {
            int k = base + lane, s = -1;
            bool visit = false, wakes = false, change = false;
            if (k < n_live) {
                s = order[k];
                int ba = m.fixture_body[w.fa[s]], bb = m.fixture_body[w.fb[s]];
                bool sa = w.type[ba] == STATIC, sb = w.type[bb] == STATIC;
                visit = (aw[ba] && !sa) || (aw[bb] && !sb);
                wakes = over[s] ? ((man[s].count > 0) != (bool)w.touching[s]) : (w.count[s] > 0);
                change = visit && wakes && ((!sa && !aw[ba]) || (!sb && !aw[bb]));
            }
            unsigned mk = gballot(x, change);
            int f = mk ? base + __ffs(mk) - 1 : n_live;
            if (s >= 0 && k <= f) active[s] = visit && wakes ? 2 : (int)visit;
            if (mk) {
                first = f;
                break;
            }
        }
        gsync(x);
        if (first == n_live) break;
        if (lane == 0) {
            int s = order[first];
            aw[m.fixture_body[w.fa[s]]] = 1, aw[m.fixture_body[w.fb[s]]] = 1;
        }
        gsync(x);
        k0 = first + 1;
    }
    for (int s = lane; s < C; s += x.wl)  // wakes of static bodies (value 2: visited and waking)
        if (active[s] == 2) aw[m.fixture_body[w.fa[s]]] = 1, aw[m.fixture_body[w.fb[s]]] = 1, active[s] = 1;
    gsync(x);
    for (int s = lane; s < C; s += x.wl) {
        if (!active[s]) continue;
        int ev = -1;  // the event this update raises
        if (!over[s]) {
            if (w.touching[s]) ev = EV_END;  // a touching contact destroyed
            w.pair[s] = -1, w.touching[s] = 0, w.count[s] = 0;
        } else if (apply_manifold(w, s, man[s])) {
            ev = w.touching[s] ? EV_BEGIN : EV_END;
        }
        active[s] = ev + 1;  // reused: the event of each visited slot
    }
    x.order_n = -1;  // contacts may have been destroyed
    if (x.p.events) {  // the step's log starts with Collide's events, in contact-list order
        gsync(x);
        int n = 0;
        for (int base = 0; base < n_live; base += x.wl) {
            int k = base + lane, s = k < n_live ? order[k] : -1;
            int ev = s >= 0 ? active[s] - 1 : -1;
            unsigned mk = gballot(x, ev >= 0);
            if (ev >= 0) put_event(x.p, x.world, n + __popc(mk & ((1u << lane) - 1)), ev, w.fa[s], w.fb[s]);
            n += __popc(mk);
        }
        if (lane == 0) x.p.event_count[x.world] = n;
    }
    for (int b = lane; b < B; b += x.wl) {
        if (aw[b] && !w.awake[b]) w.sleep_time[b] = 0.0f;
        w.awake[b] = aw[b];
    }
    gsync(x);
}

// ---------------------------------------------------------------- islands (island.py:41-140), lane 0
struct IslandOut {
    int n_contacts, n_joints, n_islands;
};

__device__ IslandOut find_islands(Ctx &x) {
    const DevModel &m = x.m;
    W &w = x.w;
    const int C = w.C, B = w.B, J = w.J, lane = x.lane;
    const Layout &L = x.p.lay;
    int *order = ap<int>(x, L.order), *lpos = ap<int>(x, L.lpos), *edges = ap<int>(x, L.edges);
    int *corder = ap<int>(x, L.corder), *cisl = ap<int>(x, L.cisl);
    int *jorder = ap<int>(x, L.jorder), *jisl = ap<int>(x, L.jisl), *jflag = ap<int>(x, L.jflag);
    int *bisl = ap<int>(x, L.bisl), *bflag = ap<int>(x, L.bflag), *stack = ap<int>(x, L.stack);
    int *adj_start = ap<int>(x, L.adj_start), *adj_cur = ap<int>(x, L.adj_cur);
    int2 *adj = ap<int2>(x, L.adj);
    int n_live = list_order(x, order, lpos);
    for (int s = lane; s < C; s += x.wl) cisl[s] = -1;
    for (int j = lane; j < J; j += x.wl) jisl[j] = -1, jflag[j] = 0;
    for (int b = lane; b < B; b += x.wl) bisl[b] = -1, bflag[b] = 0, adj_cur[b] = 0;
    gsync(x);
    // The contact graph the walk follows: the touching contacts in list order (edges) and, per non-static body, its
    // edges in that order with the body at the other end (~body when that one is static). Walking a body's list is
    // the reference's scan of every edge for those incident to the body, in the same order.
    int n_edges = 0;
    for (int base = 0; base < n_live; base += x.wl) {
        int k = base + lane;
        int s = k < n_live ? order[k] : -1;
        bool t = s >= 0 && w.touching[s];
        unsigned mk = gballot(x, t);
        if (t) {
            edges[n_edges + __popc(mk & ((1u << lane) - 1))] = s;
            int ba = m.fixture_body[w.fa[s]], bb = m.fixture_body[w.fb[s]];
            if (w.type[ba] != STATIC) atomicAdd(&adj_cur[ba], 1);
            if (w.type[bb] != STATIC) atomicAdd(&adj_cur[bb], 1);
        }
        n_edges += __popc(mk);
    }
    gsync(x);
    int run = 0;  // exclusive scan of the degrees
    for (int base = 0; base < B; base += x.wl) {
        int b = base + lane;
        int d = b < B ? adj_cur[b] : 0, inc = d;
        for (int o = 1; o < x.wl; o <<= 1) {
            int t = __shfl_up_sync(x.gmask, inc, o, x.wl);
            if (lane >= o) inc += t;
        }
        if (b < B) adj_start[b] = run + inc - d, adj_cur[b] = 0;
        run += gshfl(x, inc, x.wl - 1);
    }
    if (lane == 0) adj_start[B] = run;
    const int n_adj = run;
    gsync(x);
    for (int base = 0; base < n_edges; base += x.wl) {  // fill 32 edges at a time, in edge order within each list
        int e = base + lane;
        int s = -1, a = -1, b = -1, oa = 0, ob = 0;
        if (e < n_edges) {
            s = edges[e];
            int ba = m.fixture_body[w.fa[s]], bb = m.fixture_body[w.fb[s]];
            bool sa = w.type[ba] == STATIC, sb = w.type[bb] == STATIC;
            a = sa ? -1 : ba, b = sb || bb == ba ? -1 : bb;  // one entry for a contact within one body
            oa = sb ? ~bb : bb, ob = sa ? ~ba : ba;           // the other end, seen from a and from b
        }
        int ra = 0, rb = 0;  // incidences of a (of b) on earlier lanes of this chunk
        for (int j = 0; j < x.wl; ++j) {
            int aj = gshfl(x, a, j), bj = gshfl(x, b, j);
            if (j < lane) ra += (aj == a) + (bj == a), rb += (aj == b) + (bj == b);
        }
        if (a >= 0) adj[adj_start[a] + adj_cur[a] + ra] = make_int2(s, oa);
        if (b >= 0) adj[adj_start[b] + adj_cur[b] + rb] = make_int2(s, ob);
        gsync(x);
        if (a >= 0) atomicAdd(&adj_cur[a], 1);
        if (b >= 0) atomicAdd(&adj_cur[b], 1);
        gsync(x);
    }
    // The walk (b2World::Solve's island DFS, island.py:41-140). A contact sits in the lists of its non-static bodies
    // only and is taken when the first of them is popped, so it was taken before exactly when its other end is a
    // non-static body already walked (bisl set): no per-contact flag is read. With the lists in shared memory lane 0
    // walks alone; otherwise, per popped body, the lanes read its list (32 / 16 entries at a time) and lane 0 takes
    // the entries in order, and the seed search is a ballot over 32 / 16 bodies at a time, highest index first (the
    // list starts are then kept in jok, free until the sweeps fill it).
    IslandOut out{0, 0, 0};
    if (x.hot && L.adj + 16 * (int64_t)C <= L.hot_end) {
        if (lane == 0) {
            int sp_ = 0, nc = 0, nj = 0, ni = 0;
            int next_seed = B - 1;  // bodies above the last seed never qualify again: flags only get set, and only
                                    // bodies already flagged are woken
            for (;;) {
                if (sp_ == 0) {
                    int seed = -1;
                    for (int b = next_seed; b >= 0; --b)
                        if (w.active[b] && w.type[b] != STATIC && w.awake[b] && !bflag[b]) {
                            seed = b;
                            break;
                        }
                    if (seed < 0) break;
                    next_seed = seed - 1;
                    ++ni;
                    stack[sp_++] = seed;
                    bflag[seed] = 1;
                    continue;
                }
                const int b = stack[--sp_], id = ni - 1;
                for (int q = adj_start[b], qe = adj_start[b + 1]; q < qe; ++q) {
                    const int2 en = adj[q];
                    const int s_ = en.x, other = en.y;
                    if (other >= 0 && other != b && bisl[other] >= 0) continue;
                    corder[nc++] = s_;
                    cisl[s_] = id;
                    if (other >= 0 && !bflag[other]) stack[sp_++] = other, bflag[other] = 1;
                }
                for (int q = m.jadj_start[b], qe = m.jadj_start[b + 1]; q < qe; ++q) {
                    int j = m.jadj[2 * q], other = m.jadj[2 * q + 1];
                    if (jflag[j] || !w.active[other]) continue;
                    jorder[nj++] = j;
                    jisl[j] = id;
                    jflag[j] = 1;
                    if (!bflag[other] && w.type[other] != STATIC) stack[sp_++] = other, bflag[other] = 1;
                }
                bisl[b] = id;
                wake_body(w, b);
            }
            out = {nc, nj, ni};
        }
        out.n_contacts = gshfl(x, out.n_contacts, 0);
        out.n_joints = gshfl(x, out.n_joints, 0);
        out.n_islands = gshfl(x, out.n_islands, 0);
        gsync(x);
        return out;
    }
    int *astart = ap<int>(x, L.jok);
    for (int b = lane; b < B; b += x.wl) astart[b] = adj_start[b];
    gsync(x);
    int sp_ = 0, nc = 0, nj = 0, ni = 0;  // sp_, nc and nj: lane 0's
    int next_seed = B - 1;  // bodies above the last seed never qualify again: flags only get set, and only bodies
                            // already flagged are woken
    for (;;) {
        if (gshfl(x, sp_, 0) == 0) {
            int seed = -1;
            for (int hi = next_seed; hi >= 0 && seed < 0; hi -= x.wl) {
                const int c = hi - lane;
                const bool q = c >= 0 && w.active[c] && w.type[c] != STATIC && w.awake[c] && !bflag[c];
                const unsigned mk = gballot(x, q);
                if (mk) seed = hi - (__ffs(mk) - 1);
            }
            if (seed < 0) break;
            next_seed = seed - 1;
            ++ni;
            if (lane == 0) stack[sp_++] = seed, bflag[seed] = 1;
            gsync(x);
            continue;
        }
        int b = 0;
        if (lane == 0) b = stack[--sp_];
        b = gshfl(x, b, 0);
        const int id = ni - 1;
        const int q0 = astart[b], q1 = b + 1 < B ? astart[b + 1] : n_adj;
        for (int c0 = q0; c0 < q1; c0 += x.wl) {
            const int2 en = c0 + lane < q1 ? adj[c0 + lane] : make_int2(-1, -1);
            const int n_en = q1 - c0 < x.wl ? q1 - c0 : x.wl;
            for (int j = 0; j < n_en; ++j) {
                const int s_ = gshfl(x, en.x, j), other = gshfl(x, en.y, j);
                if (lane == 0 && !(other >= 0 && other != b && bisl[other] >= 0)) {
                    corder[nc++] = s_;
                    cisl[s_] = id;
                    if (other >= 0 && !bflag[other]) stack[sp_++] = other, bflag[other] = 1;
                }
            }
        }
        if (lane == 0) {
            for (int q = m.jadj_start[b], qe = m.jadj_start[b + 1]; q < qe; ++q) {
                int j = m.jadj[2 * q], other = m.jadj[2 * q + 1];
                if (jflag[j] || !w.active[other]) continue;
                jorder[nj++] = j;
                jisl[j] = id;
                jflag[j] = 1;
                if (!bflag[other] && w.type[other] != STATIC) stack[sp_++] = other, bflag[other] = 1;
            }
            bisl[b] = id;
            wake_body(w, b);
        }
        gsync(x);
    }
    if (lane == 0) out = {nc, nj, ni};
    out.n_contacts = gshfl(x, out.n_contacts, 0);
    out.n_joints = gshfl(x, out.n_joints, 0);
    out.n_islands = gshfl(x, out.n_islands, 0);
    gsync(x);
    return out;
}

// ---------------------------------------------------------------- SynchronizeFixtures (pairs.py:181-207)
__device__ void synchronize_fixtures(Ctx &x, const int *moved, int n_rows) {
    const DevModel &m = x.m;
    W &w = x.w;
    for (int r = x.lane; r < n_rows; r += x.wl) {
        int f = m.row_fixture[r];
        int b = m.fixture_body[f];
        if (!moved[b]) continue;
        Rot q1 = rot_of(w.a0[b]);
        V2 rr = rot(q1, w.blc(b));
        V2 p1{w.c0[2 * b] - rr.x, w.c0[2 * b + 1] - rr.y};
        AABB a1 = fixture_aabb(m, f, Xf{p1, q1});
        AABB a2 = fixture_aabb(m, f, w.bxf(b));
        float lx = bmin(a1.lx, a2.lx), ly = bmin(a1.ly, a2.ly), ux = bmax(a1.ux, a2.ux), uy = bmax(a1.uy, a2.uy);
        float dx = w.xf_p[2 * b] - p1.x, dy = w.xf_p[2 * b + 1] - p1.y;
        float *old = w.fx_fat + 4 * r;
        bool contains = old[0] <= lx && old[1] <= ly && ux <= old[2] && uy <= old[3];
        if (contains) continue;
        lx = lx - AABB_EXT, ly = ly - AABB_EXT, ux = ux + AABB_EXT, uy = uy + AABB_EXT;
        float ddx = AABB_MUL * dx, ddy = AABB_MUL * dy;
        if (ddx < 0)
            lx = lx + ddx;
        else
            ux = ux + ddx;
        if (ddy < 0)
            ly = ly + ddy;
        else
            uy = uy + ddy;
        old[0] = lx, old[1] = ly, old[2] = ux, old[3] = uy;
    }
    gsync(x);
}

__device__ __forceinline__ Bodies bodies_of(Ctx &x) {
    const Layout &L = x.p.lay;
    return {ap<float>(x, L.vx), ap<float>(x, L.vy), ap<float>(x, L.vw), ap<float>(x, L.cx),
            ap<float>(x, L.cy), ap<float>(x, L.ca), ap<float>(x, L.qc), ap<float>(x, L.qs),
            ap<float>(x, L.qa)};
}

// Where the island solve keeps its working set: the body arrays, the per-island flags of the position iterations,
// the joint rows and the contact rows. In the world's arena, or (the step kernel) in the warp's region of
// shared memory: the Gauss-Seidel sweeps store a body's velocity and read it back in the next constraint, which
// through global memory is a ~680-cycle round trip on this part (stores do not stay in L1) and through shared
// memory ~30. Islands with more contact rows than the region holds keep those rows in the arena.
struct IslandWork {
    Bodies bd;
    int *done, *jok;
    float *minsep;
    VCRow *vc;
    JRow *jr;
};
__device__ __forceinline__ IslandWork sweep_arena(char *scr, const Layout &L) {  // global memory (any kernel)
    return {{sp<float>(scr, L.vx), sp<float>(scr, L.vy), sp<float>(scr, L.vw), sp<float>(scr, L.cx),
             sp<float>(scr, L.cy), sp<float>(scr, L.ca), sp<float>(scr, L.qc), sp<float>(scr, L.qs),
             sp<float>(scr, L.qa)},
            sp<int>(scr, L.done), sp<int>(scr, L.jok), sp<float>(scr, L.minsep), sp<VCRow>(scr, L.vc),
            sp<JRow>(scr, L.jr)};
}
__device__ __forceinline__ IslandWork sweep_of(const Ctx &x, int n_contacts) {  // the kernel's own placement
    const Layout &L = x.p.lay;
    return {{ap<float>(x, L.vx), ap<float>(x, L.vy), ap<float>(x, L.vw), ap<float>(x, L.cx), ap<float>(x, L.cy),
             ap<float>(x, L.ca), ap<float>(x, L.qc), ap<float>(x, L.qs), ap<float>(x, L.qa)},
            ap<int>(x, L.done), ap<int>(x, L.jok), ap<float>(x, L.minsep),
            x.rows && n_contacts <= L.sm_vc_cap ? reinterpret_cast<VCRow *>(x.rows + L.sm_vc) : ap<VCRow>(x, L.vc),
            x.rows ? reinterpret_cast<JRow *>(x.rows + L.sm_jr) : ap<JRow>(x, L.jr)};
}

// ---------------------------------------------------------------- b2World::Solve (step.py:73-194)
// velocity integration and the constraint rows of the islands find_islands() built
__device__ IslandWork solve_rows(Ctx &x, float dt, float dt_ratio, const IslandOut &isl) {
    const DevModel &m = x.m;
    const goib2d_settings &s = x.s;
    W &w = x.w;
    const int B = w.B, lane = x.lane;
    const Layout &L = x.p.lay;
    int *bisl = ap<int>(x, L.bisl), *corder = ap<int>(x, L.corder), *cisl = ap<int>(x, L.cisl);
    int *jorder = ap<int>(x, L.jorder);
    const IslandWork sw = sweep_of(x, isl.n_contacts);
    const Bodies &bd = sw.bd;
    VCRow *vc = sw.vc;
    JRow *jr = sw.jr;
    const float h = dt;
    const float gx = w.gravity[0], gy = w.gravity[1];
    for (int b = lane; b < B; b += x.wl) {  // integrate velocities (step.py:83-100); loads first, stores last
        const bool in_isl = bisl[b] >= 0;
        const float gs = w.gravity_scale[b], im = w.inv_mass[b], fx = w.force[2 * b], fy = w.force[2 * b + 1];
        const float v0x = w.v[2 * b], v0y = w.v[2 * b + 1], w0 = w.w[b], ii = w.inv_inertia[b], tq = w.torque[b];
        const float lin_d = w.linear_damping[b], ang_d = w.angular_damping[b];
        const bool dyn = in_isl && w.type[b] == DYNAMIC;
        const float cx = w.c[2 * b], cy = w.c[2 * b + 1], ca = w.a[b];
        float ax = gs * gx + im * fx;
        float ay = gs * gy + im * fy;
        float vx = v0x + h * ax, vy = v0y + h * ay;
        float ww = w0 + (h * ii) * tq;
        float ld = 1.0f / (1.0f + h * lin_d);
        float ad = 1.0f / (1.0f + h * ang_d);
        vx = vx * ld, vy = vy * ld, ww = ww * ad;
        const Rot q = rot_of(ca);
        bd.vx[b] = dyn ? vx : v0x;
        bd.vy[b] = dyn ? vy : v0y;
        bd.vw[b] = dyn ? ww : w0;
        bd.cx[b] = cx, bd.cy[b] = cy, bd.ca[b] = ca;
        if (in_isl) w.c0[2 * b] = cx, w.c0[2 * b + 1] = cy, w.a0[b] = ca;
        bd.qc[b] = q.c, bd.qs[b] = q.s, bd.qa[b] = ca;
    }
    gsync(x);
    const bool warm = s.warm_starting;
    for (int k = lane; k < isl.n_contacts; k += x.wl)
        prepare_contact(m, w, corder[k], bd, warm, dt_ratio, s.velocity_threshold, vc[k]);
    for (int k = lane; k < isl.n_joints; k += x.wl) prepare_joint(m, w, jorder[k], bd, s, dt, dt_ratio, warm, jr[k]);
    gsync(x);
    GB_PHASE(x, 3);
    if (lane == 0) {  // the island counts, for the constraint sweeps (solve_constraints)
        int *cnt = ap<int>(x, L.isl);
        cnt[0] = isl.n_contacts, cnt[1] = isl.n_joints, cnt[2] = isl.n_islands;
    }
    gsync(x);
    GB_PHASE(x, 3);
    return sw;
}
__device__ __forceinline__ IslandWork solve(Ctx &x, float dt, float dt_ratio) {
    const IslandOut isl = find_islands(x);
    GB_PHASE(x, 2);
    return solve_rows(x, dt, dt_ratio, isl);
}

// The island constraint sweeps of one world (step.py:101-140, 197-251), run by ONE thread: warm start, the
// velocity iterations, StoreImpulses, position integration and the position iterations with per-island early
// exit. These loops are sequential within a world, so a warp runs 32 worlds' sweeps side by side (one per lane)
// rather than one world's on a single lane. Reads the rows solve() prepared in the world's arena.
// The island's arrays the sweeps read (counts, island ids), wherever the calling kernel keeps them.
struct IslandIds {
    const int *cnt, *bisl, *cisl, *jisl;
};
// The State rows the sweeps write (StoreImpulses) or read (the PostSolve events' fixtures): the world's binding (whose
// rows may be staged in shared memory), or the global leaves (the one-world-per-thread kernel, which binds nothing).
struct StoreTo {
    float *normal_impulse, *tangent_impulse, *lower_impulse, *upper_impulse, *impulse, *motor_impulse;
    int32_t *limit_state;
    const int32_t *fa, *fb;
};
__device__ __forceinline__ StoreTo store_to(const W &w) {
    return {w.normal_impulse, w.tangent_impulse, w.lower_impulse, w.upper_impulse, w.impulse, w.motor_impulse,
            w.limit_state, w.fa, w.fb};
}
__device__ __forceinline__ StoreTo store_to(const StepParams &p, int64_t world) {
    const int C = p.C, J = p.m.J;
    return {(float *)p.L.p[GOIB2D_C_NORMAL_IMPULSE] + world * 2 * C,
            (float *)p.L.p[GOIB2D_C_TANGENT_IMPULSE] + world * 2 * C,
            (float *)p.L.p[GOIB2D_J_LOWER_IMPULSE] + world * J, (float *)p.L.p[GOIB2D_J_UPPER_IMPULSE] + world * J,
            (float *)p.L.p[GOIB2D_J_IMPULSE] + world * 3 * J, (float *)p.L.p[GOIB2D_J_MOTOR_IMPULSE] + world * J,
            (int32_t *)p.L.p[GOIB2D_J_LIMIT_STATE] + world * J, (const int32_t *)p.L.p[GOIB2D_C_FA] + world * C,
            (const int32_t *)p.L.p[GOIB2D_C_FB] + world * C};
}
__device__ __forceinline__ void solve_constraints(const StepParams &p, int64_t world, const IslandWork &sw,
                                                  const IslandIds &ids, const StoreTo &st) {
    const goib2d_settings &s = p.s;
    const int B = p.m.B;
    const int n_contacts = ids.cnt[0], n_joints = ids.cnt[1], n_islands = ids.cnt[2];
    const int *bisl = ids.bisl, *cisl = ids.cisl, *jisl = ids.jisl;
    int *done = sw.done, *jok = sw.jok;
    float *minsep = sw.minsep;
    VCRow *vc = sw.vc;
    JRow *jr = sw.jr;
    const Bodies &bd = sw.bd;
    const bool warm = s.warm_starting, v24 = s.revolute_v24;
    if (warm)
        for (int k = 0; k < n_contacts; ++k) contact_warm_start(vc[k], bd);
    for (int k = 0; k < n_joints; ++k) joint_warm_start(jr[k], bd, v24);
    for (int it = 0; it < s.velocity_iterations; ++it) {
        for (int k = 0; k < n_joints; ++k) joint_solve_velocity(jr[k], bd, v24);
        for (int k = 0; k < n_contacts; ++k) contact_solve_velocity(vc[k], bd);
    }
    for (int k = 0; k < n_contacts; ++k) {  // StoreImpulses (contact_solver.py:293-304)
        const VCRow &c = vc[k];
        for (int j = 0; j < c.count; ++j)
            st.normal_impulse[2 * c.slot + j] = c.ni[j], st.tangent_impulse[2 * c.slot + j] = c.ti[j];
    }
    for (int k = 0; k < n_joints; ++k) {  // joints.py:609-622
        const JRow &r = jr[k];
        if (v24) st.lower_impulse[r.jid] = r.imp[3], st.upper_impulse[r.jid] = r.imp[4];
        for (int i = 0; i < 3; ++i) st.impulse[3 * r.jid + i] = r.imp[i];
        st.motor_impulse[r.jid] = r.mimp;
        st.limit_state[r.jid] = r.limit_state;
    }
    if (p.events) {  // b2Island::Report: PostSolve per island contact, in solve order
        const int base = p.event_count[world];
        for (int k = 0; k < n_contacts; ++k) {
            const VCRow &c = vc[k];
            put_event(p, world, base + k, EV_POST_SOLVE, st.fa[c.slot], st.fb[c.slot], c.count, c.ni, c.ti);
        }
        p.event_count[world] = base + n_contacts;
    }
    const float h = p.dt;
    const float max_t = s.clamps_per_second ? s.max_translation * h : s.max_translation;
    const float max_r = s.clamps_per_second ? s.max_rotation * h : s.max_rotation;
    for (int b = 0; b < B; ++b) {  // integrate positions (step.py:120-135)
        if (bisl[b] < 0) continue;
        float vx = bd.vx[b], vy = bd.vy[b], ww = bd.vw[b];
        float tx = h * vx, ty = h * vy;
        if (tx * tx + ty * ty > max_t * max_t) {
            float ratio = max_t / length(V2{tx, ty});
            vx = vx * ratio, vy = vy * ratio;
        }
        float rt = h * ww;
        if (rt * rt > max_r * max_r) ww = ww * (max_r / babs(rt));
        bd.cx[b] = bd.cx[b] + h * vx, bd.cy[b] = bd.cy[b] + h * vy, bd.ca[b] = bd.ca[b] + h * ww;
        bd.vx[b] = vx, bd.vy[b] = vy, bd.vw[b] = ww;
    }
    for (int i = 0; i < B; ++i) done[i] = i >= n_islands;
    for (int it = 0; it < s.position_iterations; ++it) {  // per-island early exit (step.py:197-251)
        bool all = true;
        for (int i = 0; i < n_islands; ++i) all = all && done[i];
        if (all) break;
        for (int i = 0; i < n_islands; ++i) minsep[i] = 0.0f, jok[i] = 1;
        for (int k = 0; k < n_contacts; ++k) {
            const VCRow &c = vc[k];
            int i = cisl[c.slot];
            if (done[i]) continue;
            float ms = contact_solve_position(c, bd, s.baumgarte, s.linear_slop, s.max_linear_correction, c.mA, c.mB,
                                              c.iA, c.iB);
            minsep[i] = bmin(minsep[i], ms);
        }
        for (int k = 0; k < n_joints; ++k) {
            const JRow &r = jr[k];
            int i = jisl[r.jid];
            if (done[i]) continue;
            bool ok = joint_solve_position(r, bd, s);
            jok[i] = jok[i] && ok;
        }
        for (int i = 0; i < n_islands; ++i)
            if (minsep[i] >= -3.0f * s.linear_slop && jok[i]) done[i] = 1;
    }
}

// ---------------------------------------------------------------- the island sweeps over the world's lanes
// A pass of the sweeps solves the island constraints one after another in a fixed order: the contacts then the
// joints (warm start, each position iteration) or the joints then the contacts (each velocity iteration). A
// constraint reads and writes the velocities (positions) of its two bodies only, so its result depends only on the
// earlier constraints of the pass that share a body with it. Level l of a pass holds the constraints whose earlier
// neighbours all sit on levels below l (greedy levelling in pass order): the constraints of one level share no body,
// and solving the levels one after another, each level's constraints at once on the world's lanes, gives every
// constraint the same inputs as the sequential pass - the same floats. Bodies that are not dynamic (inverse mass and
// inertia 0) are no dependency: a solve adds or subtracts 0 * impulse to their values, which leaves a finite value
// that is not -0 unchanged; a world with a -0 among those values takes the sequential pass.
constexpr int LV_MIN_CONSTRAINTS = 12;  // smaller islands: lane 0, one constraint after another

struct LvPass {  // one pass's order: element e is a contact (row e or e - nj) or a joint (row e - nc or e)
    int nc, nj;  // contacts and joints in the pass
    bool joints_first;
    __device__ __forceinline__ bool is_joint(int e) const { return joints_first ? e < nj : e >= nc; }
    __device__ __forceinline__ int row(int e) const { return joints_first ? (e < nj ? e : e - nj) : (e < nc ? e : e - nc); }
};

// The levels of a pass: items[start[l] .. start[l + 1]) are the pass elements of level l; returns the level count.
__device__ int lv_levels(Ctx &x, const IslandWork &sw, const LvPass &ps, int *level, int *items, int *start,
                         int *cur, int *last) {
    W &w = x.w;
    const int n = ps.nc + ps.nj, lane = x.lane;
    for (int b = lane; b < w.B; b += x.wl) last[b] = 0;
    gsync(x);
    int nl = 0;
    // greedy levelling in pass order (sequential by nature: each level depends on earlier ones): the lanes read the
    // dynamic bodies of 32 (16) elements at a time, lane 0 walks them in order
    for (int e0 = 0; e0 < n; e0 += x.wl) {
        const int e = e0 + lane;
        int a = -1, b = -1;
        if (e < n) {
            const bool jt = ps.is_joint(e);
            const int r = ps.row(e);
            a = jt ? sw.jr[r].ia : sw.vc[r].ia, b = jt ? sw.jr[r].ib : sw.vc[r].ib;
            if (w.type[a] != DYNAMIC) a = -1;
            if (w.type[b] != DYNAMIC) b = -1;
        }
        const int m = n - e0 < x.wl ? n - e0 : x.wl;
        for (int j = 0; j < m; ++j) {
            const int ja = gshfl(x, a, j), jb = gshfl(x, b, j);
            if (lane == 0) {
                const int la = ja >= 0 ? last[ja] : 0, lb = jb >= 0 ? last[jb] : 0;
                const int l = la > lb ? la : lb;
                level[e0 + j] = l;
                if (ja >= 0) last[ja] = l + 1;
                if (jb >= 0) last[jb] = l + 1;
                nl = nl > l + 1 ? nl : l + 1;
            }
        }
    }
    nl = gshfl(x, nl, 0);
    gsync(x);
    for (int l = lane; l <= nl; l += x.wl) start[l] = 0;
    gsync(x);
    for (int e = lane; e < n; e += x.wl) atomicAdd(&start[level[e] + 1], 1);
    gsync(x);
    if (lane == 0)
        for (int l = 0; l < nl; ++l) start[l + 1] += start[l];
    gsync(x);
    for (int l = lane; l < nl; l += x.wl) cur[l] = start[l];
    gsync(x);
    for (int e = lane; e < n; e += x.wl) items[atomicAdd(&cur[level[e]], 1)] = e;
    gsync(x);
    return nl;
}

// Does a body that is not dynamic hold -0 in the values the sweeps read (velocities, or positions)? Then the world
// takes the sequential sweeps (see above).
__device__ __forceinline__ bool lv_minus_zero(const Ctx &x, const Bodies &bd) {
    bool bad = false;
    for (int b = x.lane; b < x.w.B; b += x.wl) {
        if (x.w.type[b] == DYNAMIC) continue;
        const float v[6] = {bd.vx[b], bd.vy[b], bd.vw[b], bd.cx[b], bd.cy[b], bd.ca[b]};
        for (int k = 0; k < 6; ++k) bad = bad || __float_as_uint(v[k]) == 0x80000000u;
    }
    return gballot(x, bad) != 0;
}

// solve_constraints with the passes levelled over the world's lanes: the same results, bit for bit (every lane of
// the world calls it). Islands below LV_MIN_CONSTRAINTS constraints, and those whose velocity pass has fewer than
// 1.5 constraints per level on average, run sequentially on lane 0: c4's 20-link chain with the rig (~1.25 per
// level) runs faster sequentially, c2's piles (~2.1) levelled.
__device__ void solve_constraints_levelled(Ctx &x, const IslandWork &sw, const IslandIds &ids) {
    const StepParams &p = x.p;
    const goib2d_settings &s = x.s;
    const int nc = ids.cnt[0], nj = ids.cnt[1], n_islands = ids.cnt[2], lane = x.lane;
    const Layout &L = p.lay;
    // the levelling's per-body table in the island walk's stack (shared memory when the arena's hot part holds it;
    // the stack is free from the end of find_islands to the TOI events, which clear it before use)
    int *level = sp<int>(x.scr, L.lv_level), *cur = sp<int>(x.scr, L.lv_cur), *last = ap<int>(x, L.stack);
    int *vitems = sp<int>(x.scr, L.lv_items), *vstart = sp<int>(x.scr, L.lv_start);  // velocity pass
    int *citems = sp<int>(x.scr, L.lv_items2), *cstart = sp<int>(x.scr, L.lv_start2);  // contacts-first passes
    const LvPass vps{nc, nj, true}, cps{nc, nj, false};
    int vnl = 0;
    GB_LV_T0(x);
    bool seq = nc + nj < LV_MIN_CONSTRAINTS || lv_minus_zero(x, sw.bd);
    if (!seq) {
        vnl = lv_levels(x, sw, vps, level, vitems, vstart, cur, last);
        GB_LV(x, 0);
        seq = 3 * vnl > 2 * (nc + nj);
    }
    if (seq) {
        if (lane == 0) solve_constraints(p, x.world, sw, ids, store_to(x.w));
        gsync(x);
        return;
    }
    if (lane == 0) {
        GB_COUNT(14, 1);
        GB_COUNT(15, vnl);
    }
    const int cnl = lv_levels(x, sw, cps, level, citems, cstart, cur, last);
    GB_LV(x, 1);
    const int B = p.m.B;
    const int64_t world = x.world;
    float *sep = sp<float>(x.scr, L.lv_sep);
    int *okj = sp<int>(x.scr, L.lv_ok);
    const int *cisl = ids.cisl, *jisl = ids.jisl;
    int *done = sw.done, *jok = sw.jok;
    float *minsep = sw.minsep;
    VCRow *vc = sw.vc;
    JRow *jr = sw.jr;
    const Bodies &bd = sw.bd;
    const bool warm = s.warm_starting, v24 = s.revolute_v24;
    // warm start: the contacts (when warm starting) then the joints, the contacts-first levels (a level's contacts
    // keep their independence when the joints are left out)
    for (int l = 0; l < cnl; ++l) {
        for (int i = cstart[l] + lane; i < cstart[l + 1]; i += x.wl) {
            const int e = citems[i];
            if (cps.is_joint(e)) joint_warm_start(jr[cps.row(e)], bd, v24);
            else if (warm) contact_warm_start(vc[cps.row(e)], bd);
        }
        gsync(x);
    }
    GB_LV(x, 2);
    // velocity iterations: the joints then the contacts, the same levels every iteration
    for (int it = 0; it < s.velocity_iterations; ++it)
        for (int l = 0; l < vnl; ++l) {
            for (int i = vstart[l] + lane; i < vstart[l + 1]; i += x.wl) {
                const int e = vitems[i];
                if (vps.is_joint(e)) joint_solve_velocity(jr[vps.row(e)], bd, v24);
                else contact_solve_velocity(vc[vps.row(e)], bd);
            }
            gsync(x);
        }
    GB_LV(x, 3);
    // StoreImpulses (contact_solver.py:293-304, joints.py:609-622), one row per lane
    const StoreTo st = store_to(x.w);
    for (int k = lane; k < nc; k += x.wl) {
        const VCRow &c = vc[k];
        for (int j = 0; j < c.count; ++j)
            st.normal_impulse[2 * c.slot + j] = c.ni[j], st.tangent_impulse[2 * c.slot + j] = c.ti[j];
    }
    for (int k = lane; k < nj; k += x.wl) {
        const JRow &r = jr[k];
        if (v24) st.lower_impulse[r.jid] = r.imp[3], st.upper_impulse[r.jid] = r.imp[4];
        for (int i = 0; i < 3; ++i) st.impulse[3 * r.jid + i] = r.imp[i];
        st.motor_impulse[r.jid] = r.mimp;
        st.limit_state[r.jid] = r.limit_state;
    }
    if (p.events) {  // b2Island::Report: PostSolve per island contact, in solve order
        const int base = p.event_count[world];
        for (int k = lane; k < nc; k += x.wl) {
            const VCRow &c = vc[k];
            put_event(p, world, base + k, EV_POST_SOLVE, st.fa[c.slot], st.fb[c.slot], c.count, c.ni, c.ti);
        }
        gsync(x);
        if (lane == 0) p.event_count[world] = base + nc;
    }
    const float h = p.dt;
    const float max_t = s.clamps_per_second ? s.max_translation * h : s.max_translation;
    const float max_r = s.clamps_per_second ? s.max_rotation * h : s.max_rotation;
    for (int b = lane; b < B; b += x.wl) {  // integrate positions (step.py:120-135)
        if (ids.bisl[b] < 0) continue;
        float vx = bd.vx[b], vy = bd.vy[b], ww = bd.vw[b];
        float tx = h * vx, ty = h * vy;
        if (tx * tx + ty * ty > max_t * max_t) {
            float ratio = max_t / length(V2{tx, ty});
            vx = vx * ratio, vy = vy * ratio;
        }
        float rt = h * ww;
        if (rt * rt > max_r * max_r) ww = ww * (max_r / babs(rt));
        bd.cx[b] = bd.cx[b] + h * vx, bd.cy[b] = bd.cy[b] + h * vy, bd.ca[b] = bd.ca[b] + h * ww;
        bd.vx[b] = vx, bd.vy[b] = vy, bd.vw[b] = ww;
    }
    for (int i = lane; i < B; i += x.wl) done[i] = i >= n_islands;
    gsync(x);
    GB_LV(x, 4);
    // position iterations with per-island early exit (step.py:197-251): the contacts then the joints, levelled; the
    // islands' minimum separations are taken in pass order afterwards (the float minimum's order rules for -0)
    const LvPass &ps = cps;
    const int nl = cnl;
    const int *items = citems, *start = cstart;
    for (int it = 0; it < s.position_iterations; ++it) {
        bool open = false;
        for (int i = lane; i < n_islands; i += x.wl) open = open || !done[i];
        if (!gballot(x, open)) break;
        for (int l = 0; l < nl; ++l) {
            for (int q = start[l] + lane; q < start[l + 1]; q += x.wl) {
                const int e = items[q];
                if (ps.is_joint(e)) {
                    const int k = ps.row(e);
                    const JRow &r = jr[k];
                    if (!done[jisl[r.jid]]) okj[k] = joint_solve_position(r, bd, s);
                } else {
                    const int k = ps.row(e);
                    const VCRow &c = vc[k];
                    if (!done[cisl[c.slot]])
                        sep[k] = contact_solve_position(c, bd, s.baumgarte, s.linear_slop, s.max_linear_correction,
                                                        c.mA, c.mB, c.iA, c.iB);
                }
            }
            gsync(x);
        }
        GB_LV(x, 5);
        // An island is done when the minimum of 0 and its contacts' separations, taken in row order, is at least
        // -3 linear slop and its joints are within tolerance. Without a NaN separation the minimum is at least the
        // tolerance exactly when 0 and every separation are (any order); a NaN is replaced by the next value of the
        // fold, so then the minimum is taken in order.
        const float tol = -3.0f * s.linear_slop;
        for (int i = lane; i < n_islands; i += x.wl) jok[i] = 1;
        gsync(x);
        bool nan = false;
        for (int k = lane; k < nc; k += x.wl) {
            const int i = cisl[vc[k].slot];
            if (done[i]) continue;
            const float v = sep[k];
            nan = nan || v != v;
            if (v < tol) jok[i] = 0;
        }
        for (int k = lane; k < nj; k += x.wl) {
            const int i = jisl[jr[k].jid];
            if (!done[i] && !okj[k]) jok[i] = 0;
        }
        if (!gballot(x, nan)) {
            gsync(x);
            const bool zero_ok = 0.0f >= tol;
            for (int i = lane; i < n_islands; i += x.wl)
                if (zero_ok && jok[i]) done[i] = 1;
            gsync(x);
            GB_LV(x, 6);
            continue;
        }
        gsync(x);
        for (int i = lane; i < n_islands; i += x.wl) minsep[i] = 0.0f, jok[i] = 1;
        gsync(x);
        // the lanes read 32 (16) rows' islands and separations at a time, lane 0 folds them in order
        for (int k0 = 0; k0 < nc; k0 += x.wl) {
            const int k = k0 + lane;
            int ik = -1;
            float sk = 0.0f;
            if (k < nc) {
                ik = cisl[vc[k].slot], sk = sep[k];
                if (done[ik]) ik = -1;
            }
            const int m = nc - k0 < x.wl ? nc - k0 : x.wl;
            for (int j = 0; j < m; ++j) {
                const int i = gshfl(x, ik, j);
                const float v = gshfl(x, sk, j);
                if (lane == 0 && i >= 0) minsep[i] = bmin(minsep[i], v);
            }
        }
        for (int k = lane; k < nj; k += x.wl) {  // a logical and: any order
            const int i = jisl[jr[k].jid];
            if (!done[i] && !okj[k]) jok[i] = 0;
        }
        gsync(x);
        for (int i = lane; i < n_islands; i += x.wl)
            if (minsep[i] >= tol && jok[i]) done[i] = 1;
        gsync(x);
        GB_LV(x, 6);
    }
}

// A float's order-preserving integer key (NaN excluded): the integer order of keys is the float order, -0 below +0.
__device__ __forceinline__ int fkey(float f) {
    const int i = __float_as_int(f);
    return i ^ ((i >> 31) & 0x7fffffff);
}
__device__ __forceinline__ float fkey_inv(int k) { return __int_as_float(k ^ ((k >> 31) & 0x7fffffff)); }

// b2World::Solve after the sweeps (step.py:141-194): write back, sleep, the moved bodies
__device__ void solve_finish(Ctx &x, float dt, const IslandWork &sw) {
    const DevModel &m = x.m;
    const goib2d_settings &s = x.s;
    W &w = x.w;
    const int B = w.B, C = w.C, J = w.J, lane = x.lane;
    const Layout &L = x.p.lay;
    const float h = dt;
    int *bisl = ap<int>(x, L.bisl), *cisl = ap<int>(x, L.cisl), *jisl = ap<int>(x, L.jisl);
    int *moved = ap<int>(x, L.moved);
    const int *done = sw.done;
    const Bodies &bd = sw.bd;
    for (int b = lane; b < B; b += x.wl) {  // write back + SynchronizeTransform (step.py:141-151); loads first
        if (bisl[b] < 0) continue;
        const float cx = bd.cx[b], cy = bd.cy[b], ca = bd.ca[b], vx = bd.vx[b], vy = bd.vy[b], vw = bd.vw[b];
        const Xf xf = xf_from(V2{cx, cy}, ca, w.blc(b));
        w.c[2 * b] = cx, w.c[2 * b + 1] = cy, w.a[b] = ca;
        w.v[2 * b] = vx, w.v[2 * b + 1] = vy, w.w[b] = vw;
        w.xf_p[2 * b] = xf.p.x, w.xf_p[2 * b + 1] = xf.p.y, w.xf_q[2 * b] = xf.q.c, w.xf_q[2 * b + 1] = xf.q.s;
    }
    gsync(x);
    int *islsleep = ap<int>(x, L.islsleep), *last = ap<int>(x, L.last);
    float *st = ap<float>(x, L.st);
    int *minkey = ap<int>(x, L.minst);
    // Sleep per island (step.py:153-171) and the static bodies' awake flag (step.py:173-194), all lanes. The two
    // reductions have no order: an island's minimum sleep time (a float minimum, as integer atomics on the order-
    // preserving key of the float; a NaN time, which the float minimum skips, is skipped) and a static body's last
    // island (an integer maximum).
    for (int i = lane; i < B; i += x.wl) islsleep[i] = 0, last[i] = -1, minkey[i] = fkey(MAXF);
    gsync(x);
    if (s.allow_sleep) {
        const float lin_tol = s.linear_sleep_tolerance * s.linear_sleep_tolerance;
        const float ang_tol = s.angular_sleep_tolerance * s.angular_sleep_tolerance;
        for (int b = lane; b < B; b += x.wl) {
            const bool nonstatic = bisl[b] >= 0 && w.type[b] != STATIC;
            const float t0 = w.sleep_time[b];
            float stb = t0;
            if (nonstatic) {  // the island's velocities are the ones just written back
                const float vx = bd.vx[b], vy = bd.vy[b], vw = bd.vw[b];
                const bool mov = !w.allow_sleep[b] || (vw * vw > ang_tol) || (vx * vx + vy * vy > lin_tol);
                stb = mov ? 0.0f : t0 + h;
                const float contrib = mov ? 0.0f : stb;
                if (contrib == contrib) atomicMin(minkey + bisl[b], fkey(contrib));
            }
            st[b] = stb;
        }
        gsync(x);
        for (int i = lane; i < B; i += x.wl) islsleep[i] = fkey_inv(minkey[i]) >= s.time_to_sleep && done[i];
        gsync(x);
        for (int b = lane; b < B; b += x.wl) {
            const bool sl = bisl[b] >= 0 && w.type[b] != STATIC && islsleep[bisl[b]];
            w.sleep_time[b] = sl ? 0.0f : st[b];
            if (sl) {
                w.awake[b] = 0;
                w.v[2 * b] = w.v[2 * b + 1] = 0.0f, w.w[b] = 0.0f;
                w.force[2 * b] = w.force[2 * b + 1] = 0.0f, w.torque[b] = 0.0f;
            }
        }
    }
    for (int sl = lane; sl < C; sl += x.wl) {
        const int i = cisl[sl];
        if (i < 0) continue;
        atomicMax(last + m.fixture_body[w.fa[sl]], i), atomicMax(last + m.fixture_body[w.fb[sl]], i);
    }
    for (int j = lane; j < J; j += x.wl) {
        const int i = jisl[j];
        if (i < 0) continue;
        atomicMax(last + m.joint_a[j], i), atomicMax(last + m.joint_b[j], i);
    }
    gsync(x);
    for (int b = lane; b < B; b += x.wl)
        if (w.type[b] == STATIC && last[b] >= 0) w.awake[b] = !islsleep[last[b]], w.sleep_time[b] = 0.0f;
    for (int b = lane; b < B; b += x.wl) moved[b] = bisl[b] >= 0 && w.type[b] != STATIC;
    gsync(x);
    GB_PHASE(x, 6);
}

// the end of b2World::Solve: SynchronizeFixtures of the moved bodies, then FindNewContacts (step.py:185-194)
__device__ void broadphase(Ctx &x) {
    synchronize_fixtures(x, ap<int>(x, x.p.lay.moved), x.w.rows);
    GB_PHASE(x, 7);
    find_new_contacts(x);
    GB_PHASE(x, 8);
}

// ---------------------------------------------------------------- b2World::SolveTOI (toi.py:462-865)
// Is the contact in `slot` a TOI candidate before sweep alignment (toi.py:500-520)? Sets its bodies.
__device__ __forceinline__ bool toi_candidate(Ctx &x, int slot, int &A, int &Bb) {
    const W &w = x.w;
    bool base = w.t_enabled[slot] && w.t_count[slot] <= MAX_SUB_STEPS;
    if (!base || w.t_flag[slot]) return false;
    A = x.m.fixture_body[w.fa[slot]], Bb = x.m.fixture_body[w.fb[slot]];
    bool actA = w.awake[A] && w.type[A] != STATIC, actB = w.awake[Bb] && w.type[Bb] != STATIC;
    return (actA || actB) && toi_pair_rule(w, A, Bb, x.s.unity_toi);
}

// The sweeps a candidate's b2TimeOfImpact starts from: both bodies' (c0, a0) and the common alpha0.
__device__ __forceinline__ void toi_record(const W &w, int A, int Bb, float common, float *r) {
    r[0] = w.c0[2 * A], r[1] = w.c0[2 * A + 1], r[2] = w.a0[A];
    r[3] = w.c0[2 * Bb], r[4] = w.c0[2 * Bb + 1], r[5] = w.a0[Bb], r[6] = common;
}

// one pass of the min-TOI search; returns found, sets *min_slot / *min_alpha (all lanes)
__device__ bool toi_search(Ctx &x, int *min_slot, float *min_alpha) {
    const DevModel &m = x.m;
    W &w = x.w;
    const int lane = x.lane;
    const Layout &L = x.p.lay;
    int *order = ap<int>(x, L.order), *lpos = ap<int>(x, L.lpos), *tneed = ap<int>(x, L.tneed);
    float *rec = ap<float>(x, L.rec);
    int n_live = list_order_kept(x, order, lpos);
    // Sweep alignment in list order (toi.py:500-536): a candidate whose bodies' sweeps sit at different alpha0
    // advances the one behind, which every later candidate of that body sees. Between two advances nothing moves, so
    // each round records, in parallel, every candidate up to the next advance, which lane 0 then performs.
    for (int k0 = 0;;) {
        int first = n_live;
        for (int base = k0; base < n_live; base += x.wl) {
            int k = base + lane, slot = -1, A = 0, Bb = 0;
            bool cand = false;
            float alA = 0.0f, alB = 0.0f;
            if (k < n_live) {
                slot = order[k];
                cand = toi_candidate(x, slot, A, Bb);
                if (cand) alA = w.t_alpha0[A], alB = w.t_alpha0[Bb];
            }
            unsigned mk = gballot(x, cand && alA != alB);
            int f = mk ? base + __ffs(mk) - 1 : n_live;
            if (slot >= 0 && k < f) {
                tneed[slot] = cand;
                if (cand) toi_record(w, A, Bb, alA, rec + 8 * slot);
            }
            if (mk) {
                first = f;
                break;
            }
        }
        gsync(x);
        if (first == n_live) break;
        if (lane == 0) {
            int slot = order[first], A = 0, Bb = 0;
            toi_candidate(x, slot, A, Bb);
            float alA = w.t_alpha0[A], alB = w.t_alpha0[Bb];
            float common = alA;
            if (alA < alB) {
                sweep_advance(w.c0[2 * A], w.c0[2 * A + 1], w.a0[A], w.t_alpha0[A], w.c[2 * A], w.c[2 * A + 1],
                              w.a[A], alB);
                common = alB;
            } else {
                sweep_advance(w.c0[2 * Bb], w.c0[2 * Bb + 1], w.a0[Bb], w.t_alpha0[Bb], w.c[2 * Bb],
                              w.c[2 * Bb + 1], w.a[Bb], alA);
            }
            toi_record(w, A, Bb, common, rec + 8 * slot);
            tneed[slot] = 1;
        }
        gsync(x);
        k0 = first + 1;
    }
    for (int k = lane; k < n_live; k += x.wl) {  // b2TimeOfImpact per queued contact
        int slot = order[k];
        if (!tneed[slot]) continue;
        int A = m.fixture_body[w.fa[slot]], Bb = m.fixture_body[w.fb[slot]];
        const float *r = rec + 8 * slot;
        Sweep swA{w.blc(A), {r[0], r[1]}, {w.c[2 * A], w.c[2 * A + 1]}, r[2], w.a[A]};
        Sweep swB{w.blc(Bb), {r[3], r[4]}, {w.c[2 * Bb], w.c[2 * Bb + 1]}, r[5], w.a[Bb]};
        float beta;
        GB_COUNT(2, 1);
#ifdef GOIB2D_PHASE_TIMERS
        long long tt0 = clock64();
#endif
        int st = time_of_impact(proxy_of(m, w.fa[slot]), swA, proxy_of(m, w.fb[slot]), swB, x.s.linear_slop, &beta);
#ifdef GOIB2D_PHASE_TIMERS
        GB_COUNT(5, clock64() - tt0);
#endif
        float common = r[6];
        w.t_toi[slot] = st == E_TOUCHING ? bmin(common + (1.0f - common) * beta, 1.0f) : 1.0f;
        w.t_flag[slot] = 1;
    }
    gsync(x);
    // The minimum, first (or last) in list order among exact ties (toi.py:550-557), as warp reductions.
    const bool oldest = x.s.toi_tie_oldest;
    float best = 1.0f;
    for (int k = lane; k < n_live; k += x.wl) {
        int slot = order[k];
        bool base = w.t_enabled[slot] && w.t_count[slot] <= MAX_SUB_STEPS;
        if (base && w.t_flag[slot] && w.t_toi[slot] < 1.0f) best = fminf(best, w.t_toi[slot]);
    }
    for (int o = x.wl >> 1; o > 0; o >>= 1) best = fminf(best, __shfl_xor_sync(x.gmask, best, o, x.wl));
    int pos = oldest ? -1 : n_live;
    for (int k = lane; k < n_live; k += x.wl) {
        int slot = order[k];
        bool base = w.t_enabled[slot] && w.t_count[slot] <= MAX_SUB_STEPS;
        if (base && w.t_flag[slot] && w.t_toi[slot] < 1.0f && w.t_toi[slot] == best) pos = oldest ? k : min(pos, k);
    }
    for (int o = x.wl >> 1; o > 0; o >>= 1) {
        int q = __shfl_xor_sync(x.gmask, pos, o, x.wl);
        pos = oldest ? max(pos, q) : min(pos, q);
    }
    const float done_alpha = 1.0f - 10.0f * EPS;
    bool any = pos >= 0 && pos < n_live;
    *min_slot = any ? order[pos] : 0;
    *min_alpha = best;
    return any && !(done_alpha < best);
}

// one TOI event (toi.py:604-716) with b2Island::SolveTOI (toi.py:719-799)
__device__ void toi_event(Ctx &x, float dt, int min_slot, float min_alpha) {
    const DevModel &m = x.m;
    const goib2d_settings &s = x.s;
    W &w = x.w;
    const int B = w.B, C = w.C, lane = x.lane;
    const Layout &L = x.p.lay;
    int *order = ap<int>(x, L.order), *lpos = ap<int>(x, L.lpos), *tisl = ap<int>(x, L.tisl);
    int *flip_b = ap<int>(x, L.aw), *in_other = ap<int>(x, L.bflag), *touched = ap<int>(x, L.stack);
    int *newbody = ap<int>(x, L.last), *moved = ap<int>(x, L.moved), *solved = ap<int>(x, L.solved);
    int *old_pair = ap<int>(x, L.cflag), *old_key = ap<int>(x, L.active);
    float *adv = ap<float>(x, L.adv);
    Man *man = ap<Man>(x, L.man);
    VCRow *vc = ap<VCRow>(x, L.vc);
    Bodies bd = bodies_of(x);
    const int A = m.fixture_body[w.fa[min_slot]], Bb = m.fixture_body[w.fb[min_slot]];
#ifdef GOIB2D_PHASE_TIMERS
    long long ev_t0 = clock64();
#endif
    for (int b = lane; b < B; b += x.wl) {  // every body advanced to min_alpha, and its transform there
        float c0x = w.c0[2 * b], c0y = w.c0[2 * b + 1], a0 = w.a0[b], al0 = w.t_alpha0[b];
        const float cx = w.c[2 * b], cy = w.c[2 * b + 1], ca = w.a[b];
        const V2 lc = w.blc(b);
        sweep_advance(c0x, c0y, a0, al0, cx, cy, ca, min_alpha);
        const Xf xf = xf_from(V2{c0x, c0y}, a0, lc);
        float *d = adv + 8 * b;
        d[0] = c0x, d[1] = c0y, d[2] = a0, d[3] = al0;
        d[4] = xf.p.x, d[5] = xf.p.y, d[6] = xf.q.c, d[7] = xf.q.s;
        flip_b[b] = in_other[b] = touched[b] = newbody[b] = 0;
    }
    int n_live = list_order_kept(x, order, lpos);
    for (int s_ = lane; s_ < C; s_ += x.wl) {  // manifolds at the advanced poses for the pair's contacts
        solved[s_] = 0;
        if (w.pair[s_] < 0) continue;
        int ba = m.fixture_body[w.fa[s_]], bb = m.fixture_body[w.fb[s_]];
        // the minimum contact and the contacts the island walk visits: those of a dynamic TOI body (a static or
        // kinematic one's contacts are not walked, toi.py:633-657)
        const bool of_a = (ba == A || bb == A) && w.type[A] == DYNAMIC;
        const bool of_b = (ba == Bb || bb == Bb) && w.type[Bb] == DYNAMIC;
        if (s_ != min_slot && !of_a && !of_b) continue;
        const float *da = adv + 8 * ba, *db = adv + 8 * bb;
        evaluate(m, w.fa[s_], w.fb[s_], Xf{{da[4], da[5]}, {da[6], da[7]}}, Xf{{db[4], db[5]}, {db[6], db[7]}},
                 s.linear_slop, s.angular_slop, man[s_]);
    }
    gsync(x);
    // The island walk (toi.py:633-657): bodyA's contact list then bodyB's, newest first; each walked contact is
    // updated (b2Contact::Update, Begin / End events) and, when touching, joins the island. Its only order-dependent
    // rule is the cap (32 contacts, 64 bodies): when a side-effect-free count shows the island cannot reach it, the
    // walk runs on all lanes, island and event order kept by ballots; otherwise on lane 0 as listed.
    auto walked = [&](int oi, int slot, int &other) {  // does the walk of owner oi update this contact?
        const int owner = oi ? Bb : A;
        int ca = m.fixture_body[w.fa[slot]], cb = m.fixture_body[w.fb[slot]];
        if (ca != owner && cb != owner) return false;
        if (oi == 1 && w.type[A] == DYNAMIC && (ca == A || cb == A)) return false;
        if (slot == min_slot) return false;
        other = ca == owner ? cb : ca;
        if (w.type[other] == DYNAMIC && !w.bullet[owner] && !w.bullet[other]) return false;
        if (s.unity_toi && !toi_pair_rule(w, owner, other, true)) return false;
        return true;
    };
    int n_isl = 0, ev_n = 0;
    bool t_min = false;
    if (lane == 0) {  // the minimum contact
        ev_n = x.p.events ? x.p.event_count[x.world] : 0;
        t_min = man[min_slot].count > 0;
        if (apply_manifold(w, min_slot, man[min_slot])) {
            flip_b[m.fixture_body[w.fa[min_slot]]] = flip_b[m.fixture_body[w.fb[min_slot]]] = 1;
            if (x.p.events)
                put_event(x.p, x.world, ev_n++, w.touching[min_slot] ? EV_BEGIN : EV_END, w.fa[min_slot],
                          w.fb[min_slot]);
        }
        w.t_enabled[min_slot] = t_min;
        w.t_count[min_slot] += 1;
        w.t_flag[min_slot] = 0;
        if (t_min) tisl[n_isl++] = min_slot;
    }
    t_min = gshfl(x, (int)t_min, 0);
    ev_n = gshfl(x, ev_n, 0);
    n_isl = gshfl(x, n_isl, 0);
    gsync(x);
    if (t_min) {
        int total = 0;  // contacts the walk would add to the island
        for (int oi = 0; oi < 2; ++oi) {
            if (w.type[oi ? Bb : A] != DYNAMIC) continue;
            for (int base = 0; base < n_live; base += x.wl) {
                int k = base + lane, other = 0;
                bool add = k < n_live && walked(oi, order[k], other) && man[order[k]].count > 0;
                total += __popc(gballot(x, add));
            }
        }
        if (total + 1 < MAX_TOI_CONTACTS) {  // the cap cannot be reached: all lanes
            for (int oi = 0; oi < 2; ++oi) {
                if (w.type[oi ? Bb : A] != DYNAMIC) continue;
                for (int base = 0; base < n_live; base += x.wl) {
                    int k = base + lane, other = 0, slot = k < n_live ? order[k] : -1;
                    bool upd = slot >= 0 && walked(oi, slot, other), flip = false, add = false;
                    if (upd) {
                        flip = apply_manifold(w, slot, man[slot]);
                        if (flip) flip_b[m.fixture_body[w.fa[slot]]] = flip_b[m.fixture_body[w.fb[slot]]] = 1;
                        w.t_enabled[slot] = 1;
                        touched[other] = 1;
                        add = man[slot].count > 0;
                        if (add) {
                            in_other[other] = 1;
                            if (other != A && other != Bb) newbody[other] = 1;
                        }
                    }
                    unsigned fm = gballot(x, flip), am = gballot(x, add);
                    const unsigned below = (1u << lane) - 1;
                    if (flip && x.p.events)
                        put_event(x.p, x.world, ev_n + __popc(fm & below), w.touching[slot] ? EV_BEGIN : EV_END,
                                  w.fa[slot], w.fb[slot]);
                    if (add) tisl[n_isl + __popc(am & below)] = slot;
                    ev_n += __popc(fm), n_isl += __popc(am);
                }
            }
            gsync(x);
        } else if (lane == 0) {  // near the cap: as listed
            int n_bodies = 2;
            bool stop = false;
            for (int oi = 0; oi < 2 && !stop; ++oi) {
                int owner = oi ? Bb : A;
                if (w.type[owner] != DYNAMIC) continue;
                for (int k = 0; k < n_live; ++k) {
                    int slot = order[k];
                    int ca = m.fixture_body[w.fa[slot]], cb = m.fixture_body[w.fb[slot]];
                    if (ca != owner && cb != owner) continue;
                    if (oi == 1 && w.type[A] == DYNAMIC && (ca == A || cb == A)) continue;
                    if (!(n_isl < MAX_TOI_CONTACTS && n_bodies < 2 * MAX_TOI_CONTACTS)) {
                        stop = true;
                        break;
                    }
                    int other = 0;
                    if (!walked(oi, slot, other)) continue;
                    if (apply_manifold(w, slot, man[slot])) {
                        flip_b[ca] = flip_b[cb] = 1;
                        if (x.p.events)
                            put_event(x.p, x.world, ev_n++, w.touching[slot] ? EV_BEGIN : EV_END, w.fa[slot],
                                      w.fb[slot]);
                    }
                    w.t_enabled[slot] = 1;
                    touched[other] = 1;
                    if (man[slot].count <= 0) continue;
                    tisl[n_isl++] = slot;
                    in_other[other] = 1;
                    if (other != A && other != Bb && !newbody[other]) newbody[other] = 1, ++n_bodies;
                }
            }
        }
        n_isl = gshfl(x, n_isl, 0);
        ev_n = gshfl(x, ev_n, 0);
    }
    if (lane == 0 && x.p.events) x.p.event_count[x.world] = ev_n;
    gsync(x);
    for (int b = lane; b < B; b += x.wl) {  // body sweeps after the walk (toi.py:667-681)
        bool pair_b = b == A || b == Bb;
        bool keep = (pair_b && t_min) || in_other[b];
        bool restore = (pair_b && !t_min) || (touched[b] && !in_other[b]);
        const float *d = adv + 8 * b;
        if (keep) {
            w.c0[2 * b] = d[0], w.c0[2 * b + 1] = d[1], w.a0[b] = d[2];
            w.c[2 * b] = d[0], w.c[2 * b + 1] = d[1], w.a[b] = d[2];
            w.t_alpha0[b] = d[3];
            w.xf_p[2 * b] = d[4], w.xf_p[2 * b + 1] = d[5], w.xf_q[2 * b] = d[6], w.xf_q[2 * b + 1] = d[7];
        } else if (restore) {
            Xf o = xf_from(w.bc(b), w.a[b], w.blc(b));
            w.xf_p[2 * b] = o.p.x, w.xf_p[2 * b + 1] = o.p.y, w.xf_q[2 * b] = o.q.c, w.xf_q[2 * b + 1] = o.q.s;
        }
        if (flip_b[b] || (pair_b && t_min) || (newbody[b] && w.type[b] != STATIC)) wake_body(w, b);
        moved[b] = t_min && (pair_b || in_other[b]) && w.type[b] == DYNAMIC;
    }
    gsync(x);
    if (!t_min) {
        if (lane == 0) *w.t_events += 1;
        gsync(x);
        return;
    }
#ifdef GOIB2D_PHASE_TIMERS
    if (lane == 0) atomicAdd(&g_toi_cycles[12], (unsigned long long)(clock64() - ev_t0));
    ev_t0 = clock64();
#endif
    // b2Island::SolveTOI: position passes moving only the TOI pair, then velocity passes, then integration; the
    // island's rows in the warp's shared rows region when they fit
    if (x.rows && n_isl <= L.sm_vc_cap) vc = reinterpret_cast<VCRow *>(x.rows + L.sm_vc);
    for (int b = lane; b < B; b += x.wl) {
        const float cx = w.c[2 * b], cy = w.c[2 * b + 1], ca = w.a[b];
        const float vx = w.v[2 * b], vy = w.v[2 * b + 1], vw = w.w[b];
        const Rot q = rot_of(ca);
        bd.cx[b] = cx, bd.cy[b] = cy, bd.ca[b] = ca;
        bd.vx[b] = vx, bd.vy[b] = vy, bd.vw[b] = vw;
        bd.qc[b] = q.c, bd.qs[b] = q.s, bd.qa[b] = ca;
    }
    gsync(x);
#ifdef GOIB2D_PHASE_TIMERS
    long long isl_t0 = clock64();
#endif
    for (int k = lane; k < n_isl; k += x.wl)  // position rows (the position-independent fields)
        prepare_contact(m, w, tisl[k], bd, false, 1.0f, s.velocity_threshold, vc[k]);
    gsync(x);
#ifdef GOIB2D_PHASE_TIMERS
    if (lane == 0) atomicAdd(&g_toi_cycles[4], (unsigned long long)(clock64() - isl_t0)), isl_t0 = clock64();
#endif
    if (lane == 0) {
        const float okay_sep = -1.5f * s.linear_slop;
        for (int it = 0; it < 20; ++it) {
            float min_sep = 0.0f;
            for (int k = 0; k < n_isl; ++k) {
                const VCRow &c = vc[k];
                bool ta = c.ia == A || c.ia == Bb, tb = c.ib == A || c.ib == Bb;
                float ms = contact_solve_position(c, bd, s.toi_baumgarte, s.linear_slop, s.max_linear_correction,
                                                  ta ? c.mA : 0.0f, tb ? c.mB : 0.0f, ta ? c.iA : 0.0f,
                                                  tb ? c.iB : 0.0f);
                min_sep = bmin(min_sep, ms);
            }
            GB_COUNT(1, 1);
            if (min_sep >= okay_sep) break;
        }
        // leap of faith: the TOI bodies' sweep start is the solved pose
        w.c0[2 * A] = bd.cx[A], w.c0[2 * A + 1] = bd.cy[A], w.a0[A] = bd.ca[A];
        w.c0[2 * Bb] = bd.cx[Bb], w.c0[2 * Bb + 1] = bd.cy[Bb], w.a0[Bb] = bd.ca[Bb];
    }
    gsync(x);
    for (int b = lane; b < B; b += x.wl) body_rot(bd, b, bd.ca[b]);
    gsync(x);
#ifdef GOIB2D_PHASE_TIMERS
    if (lane == 0) atomicAdd(&g_toi_cycles[5], (unsigned long long)(clock64() - isl_t0)), isl_t0 = clock64();
#endif
    for (int k = lane; k < n_isl; k += x.wl)  // velocity constraints at the solved poses, no warm start
        prepare_contact(m, w, tisl[k], bd, false, 1.0f, s.velocity_threshold, vc[k]);
    gsync(x);
#ifdef GOIB2D_PHASE_TIMERS
    if (lane == 0) atomicAdd(&g_toi_cycles[6], (unsigned long long)(clock64() - isl_t0)), isl_t0 = clock64();
#endif
    if (lane == 0)
        for (int it = 0; it < s.velocity_iterations; ++it)
            for (int k = 0; k < n_isl; ++k) contact_solve_velocity(vc[k], bd);
    gsync(x);
#ifdef GOIB2D_PHASE_TIMERS
    if (lane == 0) atomicAdd(&g_toi_cycles[7], (unsigned long long)(clock64() - isl_t0)), isl_t0 = clock64();
    if (lane == 0) atomicAdd(&g_toi_cycles[11], (unsigned long long)n_isl);
#endif
    const float h = (1.0f - min_alpha) * dt;
    const float max_t = s.clamps_per_second ? s.max_translation * dt : s.max_translation;
    const float max_r = s.clamps_per_second ? s.max_rotation * dt : s.max_rotation;
    for (int b = lane; b < B; b += x.wl) {  // integrate the island bodies over the rest of the step
        bool pair_b = b == A || b == Bb;
        if (!(pair_b || in_other[b])) continue;
        float vx = bd.vx[b], vy = bd.vy[b], ww = bd.vw[b];
        float tx = h * vx, ty = h * vy;
        if (tx * tx + ty * ty > max_t * max_t) {
            float ratio = max_t / length(V2{tx, ty});
            vx = vx * ratio, vy = vy * ratio;
        }
        float rt = h * ww;
        if (rt * rt > max_r * max_r) ww = ww * (max_r / babs(rt));
        float ncx = bd.cx[b] + h * vx, ncy = bd.cy[b] + h * vy, na = bd.ca[b] + h * ww;
        Xf xf = xf_from(V2{ncx, ncy}, na, w.blc(b));
        w.c[2 * b] = ncx, w.c[2 * b + 1] = ncy, w.a[b] = na;
        w.v[2 * b] = vx, w.v[2 * b + 1] = vy, w.w[b] = ww;
        w.xf_p[2 * b] = xf.p.x, w.xf_p[2 * b + 1] = xf.p.y, w.xf_q[2 * b] = xf.q.c, w.xf_q[2 * b + 1] = xf.q.s;
    }
    const int ev_base = x.p.events ? x.p.event_count[x.world] : 0;
    for (int k = lane; k < n_isl; k += x.wl) {  // b2Island::Report (PostSolve per island contact)
        const VCRow &c = vc[k];
        solved[c.slot] = 1;
        w.t_solved[c.slot] = 1;
        for (int j = 0; j < 2; ++j) {
            w.t_ni[2 * c.slot + j] = j < c.count ? c.ni[j] : 0.0f;
            w.t_ti[2 * c.slot + j] = j < c.count ? c.ti[j] : 0.0f;
        }
        if (x.p.events) put_event(x.p, x.world, ev_base + k, EV_POST_SOLVE, w.fa[c.slot], w.fb[c.slot], c.count, c.ni, c.ti);
    }
    gsync(x);
    if (lane == 0 && x.p.events) x.p.event_count[x.world] = ev_base + n_isl;
    gsync(x);
#ifdef GOIB2D_PHASE_TIMERS
    if (lane == 0) atomicAdd(&g_toi_cycles[13], (unsigned long long)(clock64() - ev_t0));
    ev_t0 = clock64();
#endif
    synchronize_fixtures(x, moved, w.rows);
    for (int s_ = lane; s_ < C; s_ += x.wl) {
        if (moved[m.fixture_body[w.fa[s_]]] || moved[m.fixture_body[w.fb[s_]]]) w.t_flag[s_] = 0;  // every slot
        old_pair[s_] = w.pair[s_], old_key[s_] = w.key[s_];
    }
    gsync(x);
    find_new_contacts(x, x.fnc_clean ? moved : nullptr);
    for (int s_ = lane; s_ < C; s_ += x.wl) {
        bool is_new = w.pair[s_] >= 0 && (old_pair[s_] < 0 || old_key[s_] != w.key[s_]);
        if (is_new) w.t_count[s_] = 0, w.t_flag[s_] = 0, w.t_enabled[s_] = 1;
    }
    if (lane == 0) *w.t_events += 1;
    gsync(x);
#ifdef GOIB2D_PHASE_TIMERS
    if (lane == 0) atomicAdd(&g_toi_cycles[14], (unsigned long long)(clock64() - ev_t0));
#endif
}

__device__ void solve_toi(Ctx &x, float dt) {  // toi.py:827-865
    W &w = x.w;
    const int C = w.C, B = w.B, lane = x.lane;
    if (C == 0 || x.m.P == 0) return;
    if (x.s.unity_toi && !x.m.any_toi_body) return;
    for (int b = lane; b < B; b += x.wl) w.t_alpha0[b] = 0.0f;
    for (int c = lane; c < C; c += x.wl) {
        w.t_count[c] = 0, w.t_toi[c] = 1.0f, w.t_flag[c] = 0, w.t_enabled[c] = 1, w.t_solved[c] = 0;
        w.t_ni[2 * c] = w.t_ni[2 * c + 1] = w.t_ti[2 * c] = w.t_ti[2 * c + 1] = 0.0f;
    }
    if (lane == 0) *w.t_events = 0;
    x.order_n = -1;
    gsync(x);
    if (!(dt > 0)) return;
    const int max_events = C * (MAX_SUB_STEPS + 1) + 8;
    int min_slot = 0;
    float min_alpha = 1.0f;
    bool pending = false;
    int n_ev = 0;
    for (int it = 0; it <= max_events; ++it) {
        if (pending) toi_event(x, dt, min_slot, min_alpha), ++n_ev;
        if (x.lane == 0) GB_COUNT(3, 1);
        GB_PHASE(x, 10);
        bool found = toi_search(x, &min_slot, &min_alpha);
        GB_PHASE(x, 9);
        if (!found) {
            pending = false;
            break;
        }
        pending = true;
    }
    if (pending) x.status |= ST_CAP;  // events capped with one still pending (the reference's limit too)
#ifdef GOIB2D_PHASE_TIMERS
    if (x.lane == 0) GB_COUNT(0, n_ev), atomicMax(&g_counts[4], (unsigned long long)n_ev);
#endif
}

// b2World::Step (step.py:28-47) in parts. A step is one launch (goib2d_step_kernel / goib2d_step_pair_kernel,
// whole_step: the parts' phases with block barriers between them) or, for the batches part_kernels() picks, each part
// a kernel of its own (one warp per world).
//   0  the action channels, FindNewContacts for new fixtures, b2ContactManager::Collide
//   1  b2World::Solve: islands, velocity integration, the constraint rows (solve), the constraint sweeps on lane 0
//      (solve_constraints), write back and sleep (solve_finish), SynchronizeFixtures and FindNewContacts
//   2, 3, 4  part 1 in pieces for large batches: solve; solve_finish; SynchronizeFixtures and FindNewContacts, with
//      the sweeps between the first two run one world per thread (goib2d_constraints_kernel)
//   5  SolveTOI, then the end of the step (inv_dt0, cleared forces; the status word after the last step)
// Every value one part hands the next is in the State or the world's arena.
// One part of one world's step on the world's group of lanes (Ctx x: the bound State and its regions).
template <int PART>
__device__ __forceinline__ void run_part(Ctx &x) {
    const StepParams &p = x.p;
    W &w = x.w;
    const float dt = p.dt;
#ifdef GOIB2D_PHASE_TIMERS
    const long long gb_span0_ = clock64();
#endif
    if (PART == 0) {
        if (p.actions) {  // action channels -> joint motor speeds, from this step's row of the actions
            const float *a = p.actions + x.step * p.action_stride + x.world * p.n_action;
            for (int c = x.lane; c < p.n_action; c += x.wl) w.motor_speed[p.action_joint[c]] = p.action_scale[c] * a[c];
        }
        gsync(x);
        GB_PHASE(x, 11);
        if (*w.new_fixture) find_new_contacts(x);
        gsync(x);
        if (x.lane == 0) *w.new_fixture = 0;
        gsync(x);
        GB_PHASE(x, 0);
        collide(x);
        GB_PHASE(x, 1);
        GB_SPAN(x, 9, false);
    } else if (PART == 2) {
        solve(x, dt, *w.inv_dt0 * dt);
    } else if (PART == 3) {
        solve_finish(x, dt, sweep_of(x, 0));
    } else if (PART == 4) {
        broadphase(x);
    } else {
        if (x.s.continuous_physics) solve_toi(x, dt);
        gsync(x);
        GB_SPAN(x, 0, x.s.continuous_physics && *w.t_events > 0);
        if (x.lane == 0 && dt > 0) *w.inv_dt0 = 1.0f / dt;
        if (x.s.auto_clear_forces)
            for (int b = x.lane; b < w.B; b += x.wl) w.force[2 * b] = w.force[2 * b + 1] = 0.0f, w.torque[b] = 0.0f;
        if (x.step == p.n_steps - 1) {
            bool bad = false;  // non-finite body state
            for (int b = x.lane; b < w.B; b += x.wl)
                bad = bad || !isfinite(w.c[2 * b]) || !isfinite(w.c[2 * b + 1]) || !isfinite(w.a[b]) ||
                      !isfinite(w.v[2 * b]) || !isfinite(w.v[2 * b + 1]) || !isfinite(w.w[b]);
            if (__any_sync(x.gmask, bad)) x.status |= ST_NONFINITE;
        }
        gsync(x);
    }
}

// the status word of the world after a part (part 0 of the first step starts it afresh)
__device__ __forceinline__ void put_status(const Ctx &x, bool first) {
    if (x.lane == 0 && x.p.status) {
        if (first)
            x.p.status[x.world] = x.status;
        else if (x.status)
            x.p.status[x.world] |= x.status;
    }
}

// A part kernel (the batches part_kernels() picks): one warp per world, 4 worlds per block.
template <int PART>
__device__ __forceinline__ void step_part(const StepParams &p) {
    const int warp = threadIdx.x >> 5;
    const int64_t world = p.world0 + (int64_t)blockIdx.x * (blockDim.x >> 5) + warp;
    if (world >= p.world_end) return;
    __shared__ W s_world[4];  // blockDim.x <= 128
    if ((threadIdx.x & 31) == 0) bind_world(s_world[warp], p.L, world, p.m.B, p.rows, p.m.J, p.C);
    __syncwarp();
    // the collide and TOI part kernels keep the arena's hot part in shared memory: every arena array
    // they use is written and read within the kernel; the large-batch split solve passes arrays between kernels
    extern __shared__ __align__(16) char dyn_smem[];
    const bool hot = (PART == 0 || PART == 5) && p.lay.hot_end > 0;
    const bool rows = hot && PART == 5 && p.lay.rows_bytes;  // the TOI island's rows
    const int region = hot ? p.lay.hot_end + (rows ? p.lay.rows_bytes : 0) : 0;
    char *mine = dyn_smem + warp * region;
    Ctx x{p, p.m, p.s, s_world[warp], p.scratch + world * p.lay.stride, hot ? mine : nullptr,
          rows ? mine + p.lay.hot_end : nullptr, (int)(threadIdx.x & 31), 0, p.step, 0, -1, -1, 0, clock64(), world, FULL, 0, 32};
    run_part<PART>(x);
    put_status(x, PART == 0 && p.step == 0);
}

// Every step of a call in one launch (see part_kernels for the batches that run part kernels instead): one block
// per SM where the batch allows, each block running all p.n_steps steps of its worlds before it exits, the block's
// threads meeting between the phases of a step (step_sync: collide | islands and rows | sweeps | write back, sleep
// and broadphase | TOI; two more barriers, between islands and rows and before the broadphase, measured 1 % slower),
// and WPW worlds per warp.
// - Persistent over the steps: worlds are independent, so a block runs its worlds' steps back to back with no
//   grid-wide boundary between them. A step no longer waits for the slowest block of the batch (a TOI event chain in
//   one of its worlds), only the block's own phases do; the per-world binding, shared-memory regions and the State
//   rows and arena lines the block's worlds touch stay on the SM and in L2 across the steps, and per-step launch gaps
//   vanish (c1, 4096 worlds, steps 50-1000: 15.8 M world-steps/s as one launch per step, 18.2 M as calls of 10 steps,
//   19.6 M as calls of 50).
// - Phase barriers: a phase's tail is the slowest of the block's worlds rather than of the whole batch, and every
//   warp of an SM runs the same phase at the same time (the step's code does not fit the SM's instruction cache;
//   warps spread over all phases thrash it).
// - WPW = 2 (goib2d_step_pair_kernel), one world per half-warp: the order-dependent sections run on each world's
//   lane 0, so lanes 0 and 16 run two worlds' sequential work in the same instructions where their control flow
//   agrees - half the issue slots per world, which pays when an SM holds many small worlds - and 16 warps per SM
//   leave 128 registers per thread (28 single-world warps: 72, with spills). Where the two worlds' sequential work
//   diverges (large islands, frequent TOI events) the warp runs both paths one after the other, so WPW = 1
//   (goib2d_step_kernel, 28 warps of 72 registers) serves the other batches (launch_steps chooses).
// Per world in dynamic shared memory: the bound State, the arena's hot part and the rows region. A group of lanes
// without a world (the batch's tail) runs no phase but meets every barrier, so all threads reach every step_sync.
constexpr int STEP_MAX_WARPS = 28;       // one world per warp: 72 registers per thread
constexpr int WIDE_MAX_WARPS = 8;        // one world per warp, few warps: 255 registers per thread
constexpr int PAIR_MAX_WARPS = 16;       // two worlds per warp: 128 registers per thread
constexpr int STEP_MAX_SMEM = 232448;    // dynamic shared memory per block
__host__ __device__ __forceinline__ int step_region(const Layout &L) {
    return (int)((sizeof(W) + 15) & ~size_t(15)) + L.hot_end + (L.hot_end > 0 ? L.rows_bytes : 0);
}
// Copy the world's rows of the staged leaves into its staging area in shared memory and point the binding there
// (in), or copy them back to the State (out). Every leaf row of a world is contiguous; 4-byte leaves' rows start on
// 4-byte boundaries, and one-byte leaves whose rows are a multiple of 4 bytes do too.
__device__ __forceinline__ void stage_rows(const StepParams &p, W &w, int64_t world, int lane, int wl,
                                           unsigned gmask, char *area, bool in) {
    for (int leaf = 0; leaf < GOIB2D_NUM_LEAVES; ++leaf) {
        const int off = p.stage_off[leaf];
        if (off < 0) continue;
        const int nb = p.leaf_bytes[leaf];
        char *g = static_cast<char *>(p.L.p[leaf]) + world * (int64_t)nb;
        char *s = area + off;
        if ((nb & 3) == 0) {
            uint32_t *gw = reinterpret_cast<uint32_t *>(g), *sw = reinterpret_cast<uint32_t *>(s);
            for (int i = lane; i < nb / 4; i += wl) {
                if (in) sw[i] = gw[i];
                else gw[i] = sw[i];
            }
        } else {
            for (int i = lane; i < nb; i += wl) {
                if (in) s[i] = g[i];
                else g[i] = s[i];
            }
        }
    }
    __syncwarp(gmask);
    if (in && lane == 0)
        for (int leaf = 0; leaf < GOIB2D_NUM_LEAVES; ++leaf)
            if (p.stage_off[leaf] >= 0) set_leaf(w, leaf, area + p.stage_off[leaf]);
    __syncwarp(gmask);
}

// the warp reconverges (all its lanes are at this same call), then the block's threads meet
__device__ __forceinline__ void step_sync() {
    __syncwarp();
    __syncthreads();
}
template <int WPW>
__device__ __forceinline__ void whole_step(const StepParams &p) {
    constexpr int WL = 32 / WPW;  // lanes per world
    const int lane32 = threadIdx.x & 31, half = WPW == 2 ? lane32 >> 4 : 0;
    const int slot = WPW * (int)(threadIdx.x >> 5) + half;  // the world's place in the block
    const int64_t world = p.world0 + (int64_t)blockIdx.x * (WPW * (blockDim.x >> 5)) + slot;
    const bool active = world < p.world_end;
    extern __shared__ __align__(16) char dyn_smem[];
    char *mine = dyn_smem + slot * (step_region(p.lay) + p.stage_bytes);
    W &w = *reinterpret_cast<W *>(mine);
    char *hot = p.lay.hot_end > 0 ? mine + ((sizeof(W) + 15) & ~size_t(15)) : nullptr;
    char *rows = hot && p.lay.rows_bytes ? hot + p.lay.hot_end : nullptr;
    char *staged = mine + step_region(p.lay);  // the world's staged State rows (p.stage_bytes)
    if (active && (lane32 & (WL - 1)) == 0) bind_world(w, p.L, world, p.m.B, p.rows, p.m.J, p.C);
    __syncwarp();
    Ctx x{p, p.m, p.s, w, p.scratch + world * p.lay.stride, hot, rows, lane32 & (WL - 1), 0, 0, 0, -1, -1, 0, clock64(), world,
          WPW == 2 ? 0xffffu << (16 * half) : FULL, WL * half, WL};
    const unsigned gmask = WPW == 2 ? 0xffffu << (16 * half) : FULL;
    if (active && p.stage_bytes) stage_rows(p, w, world, lane32 & (WL - 1), WL, gmask, staged, true);
    const float dt = p.dt;
    for (int k = 0; k < p.n_steps; ++k) {
        x.step = k;
        if (active) run_part<0>(x);
        step_sync();
        IslandOut isl{0, 0, 0};
        if (active) {
            isl = find_islands(x);
            GB_PHASE(x, 2);
        }
        IslandWork sw{};
        if (active) sw = solve_rows(x, dt, *w.inv_dt0 * dt, isl);
        step_sync();
        if (active)
            solve_constraints_levelled(x, sw,
                                       {ap<int>(x, p.lay.isl), ap<int>(x, p.lay.bisl), ap<int>(x, p.lay.cisl),
                                        ap<int>(x, p.lay.jisl)});
        step_sync();
        if (active) {
            GB_PHASE(x, 5);
            solve_finish(x, dt, sw);
        }
        if (active) broadphase(x);
        step_sync();
        if (active) {
            run_part<5>(x);
            put_status(x, k == 0);
        }
        // the block's threads also meet between one step and the next: without this barrier a world that finished
        // its TOI phase starts the next step's collide while a TOI event chain runs in another warp, and the two
        // phases' code evicts each other from the instruction cache (c1, steps 50-1000: 18.2 M world-steps/s with
        // it, 17.1 M without)
        step_sync();
    }
    if (active && p.stage_bytes) stage_rows(p, w, world, lane32 & (WL - 1), WL, gmask, staged, false);
}

}  // namespace gb

using namespace gb;

// One warp per world; blockDim.x = 32 * worlds per block. GOIB2D_MIN_BLOCKS bounds the registers per thread so that
// that many 128-thread blocks fit on an SM (65536 / (128 * blocks) registers).
#ifndef GOIB2D_MIN_BLOCKS
#define GOIB2D_MIN_BLOCKS 7
#endif
extern "C" __global__ void __launch_bounds__(128, GOIB2D_MIN_BLOCKS)
    goib2d_collide_kernel(const __grid_constant__ StepParams p) {
    step_part<0>(p);
}
extern "C" __global__ void __launch_bounds__(128, GOIB2D_MIN_BLOCKS)
    goib2d_solve_rows_kernel(const __grid_constant__ StepParams p) {
    step_part<2>(p);
}
// one world per THREAD (solve_constraints)
extern "C" __global__ void __launch_bounds__(32) goib2d_constraints_kernel(const __grid_constant__ StepParams p) {
    const int64_t world = p.world0 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (world >= p.world_end) return;
    char *scr = p.scratch + world * p.lay.stride;
    const Layout &L = p.lay;
    solve_constraints(p, world, sweep_arena(scr, L),
                      {sp<int>(scr, L.isl), sp<int>(scr, L.bisl), sp<int>(scr, L.cisl), sp<int>(scr, L.jisl)},
                      store_to(p, world));
}
extern "C" __global__ void __launch_bounds__(128, GOIB2D_MIN_BLOCKS)
    goib2d_finish_kernel(const __grid_constant__ StepParams p) {
    step_part<3>(p);
}
extern "C" __global__ void __launch_bounds__(128, GOIB2D_MIN_BLOCKS)
    goib2d_broadphase_kernel(const __grid_constant__ StepParams p) {
    step_part<4>(p);
}
extern "C" __global__ void __launch_bounds__(128, GOIB2D_MIN_BLOCKS)
    goib2d_toi_kernel(const __grid_constant__ StepParams p) {
    step_part<5>(p);
}
// the whole step, one world per warp (whole_step)
// the whole step, one world per warp, for blocks of at most WIDE_MAX_WARPS warps (few worlds per SM: c0, c2): the
// same code with up to 255 registers per thread instead of 72, so its sequential sections do not spill
extern "C" __global__ void __launch_bounds__(32 * WIDE_MAX_WARPS, 1)
    goib2d_step_wide_kernel(const __grid_constant__ StepParams p) {
    whole_step<1>(p);
}
extern "C" __global__ void __launch_bounds__(32 * STEP_MAX_WARPS, 1)
    goib2d_step_kernel(const __grid_constant__ StepParams p) {
    whole_step<1>(p);
}
// the whole step, two worlds per warp (whole_step)
extern "C" __global__ void __launch_bounds__(32 * PAIR_MAX_WARPS, 1)
    goib2d_step_pair_kernel(const __grid_constant__ StepParams p) {
    whole_step<2>(p);
}

namespace gb {
// Batches of at least THREAD_SWEEPS_MIN_WORLDS worlds whose model has at least THREAD_SWEEPS_MIN_JOINTS joints run
// a step as six part kernels with the constraint sweeps one world per THREAD (goib2d_constraints_kernel): 32
// worlds' long sequential joint sweeps share one warp instruction. Everything else is the one-launch step. Both run
// the same code in the same order within a world, so results are identical. Measured with calls of 10 steps over
// the first 300 steps of c4's episode: 65536 worlds 12.7 M world-steps/s as part kernels, 9.3 M as one persistent
// launch; 16384 worlds 7.8-17.6 M and 7.1-16.2 M per 50-step window.
constexpr int64_t THREAD_SWEEPS_MIN_WORLDS = 16384;
constexpr int THREAD_SWEEPS_MIN_JOINTS = 8;
bool part_kernels(int64_t n_worlds, int n_joints) {
    return n_worlds >= THREAD_SWEEPS_MIN_WORLDS && n_joints >= THREAD_SWEEPS_MIN_JOINTS;
}
// p.n_steps steps of worlds world0 .. world_end - 1, in order on one stream: one goib2d_step(_pair)_kernel running
// every step, or per step the collide part, the solve part in pieces (rows / thread sweeps / finish / broadphase)
// and the TOI part
int kernels_per_step(int64_t n_worlds, int n_joints) { return part_kernels(n_worlds, n_joints) ? 6 : 1; }
int64_t launches_per_call(int64_t n_worlds, int n_joints, int n_steps) {
    if (n_worlds <= 0 || n_steps <= 0) return 0;
    return part_kernels(n_worlds, n_joints) ? 6 * (int64_t)n_steps : 1;
}
// Two worlds per warp (goib2d_step_pair_kernel) for crowded batches of small worlds: more than PAIR_MIN_PER_SM
// worlds per SM (fewer leave the SM's issue slots free, and a pair only adds the two worlds' divergence) and at most
// PAIR_MAX_CONTACTS contact slots (worlds with more grow islands and TOI event chains that differ between the two
// worlds of a warp). Measured: c1 (4096 worlds, 48 slots) +12 %; c0 (256 worlds) -7 %, c2 (1024 slots) -39 %,
// c3 (256 slots) -21 % had they been paired.
constexpr int PAIR_MIN_PER_SM = 16, PAIR_MAX_CONTACTS = 128;
bool step_pairs(int64_t n_worlds, int sms, int contact_capacity) {
    return n_worlds > (int64_t)PAIR_MIN_PER_SM * sms && contact_capacity <= PAIR_MAX_CONTACTS;
}

// The one-launch step's block for a batch: warps, worlds per warp (2 when paired), before the shared-memory cap - one
// block per SM where the batch allows.
struct BlockShape {
    int warps, wpw;
};
BlockShape block_shape(int64_t n, int sms, int contact_capacity, int step_mode) {
    const int per_sm = (int)((n + sms - 1) / sms);
    const bool pair = step_mode ? step_mode == 2 : step_pairs(n, sms, contact_capacity);
    const int wpw = pair ? 2 : 1, max_warps = pair ? PAIR_MAX_WARPS : STEP_MAX_WARPS;
    int warps = (per_sm + wpw - 1) / wpw;
    warps = warps < 1 ? 1 : (warps > max_warps ? max_warps : warps);
    return {warps, wpw};
}
// Shared memory per world for the arena's hot part (Layout::hot_end): what a block's share per world leaves after the
// bound State and the rows region, at least HOT_MIN_BYTES (the part kernels' fixed budget) and at most HOT_MAX_BYTES.
// A block of few, large worlds (c2: 7 worlds of 257 bodies) keeps their body arrays in shared memory.
constexpr int HOT_MIN_BYTES = 6144, HOT_MAX_BYTES = 65536;
int hot_budget(int64_t n_worlds, int n_joints, int contact_capacity, int step_mode) {
    if (n_worlds <= 0 || part_kernels(n_worlds, n_joints)) return HOT_MIN_BYTES;
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) return HOT_MIN_BYTES;
    const BlockShape b = block_shape(n_worlds, sms, contact_capacity, step_mode);
    const int per_world = STEP_MAX_SMEM / (b.warps * b.wpw) - (int)((sizeof(W) + 15) & ~size_t(15)) - ROWS_MAX_BYTES;
    return per_world < HOT_MIN_BYTES ? HOT_MIN_BYTES : per_world > HOT_MAX_BYTES ? HOT_MAX_BYTES : per_world;
}

// Which State rows the one-launch step keeps in shared memory for the whole launch (goib2d_set_state_staging; off by
// default), within `budget` bytes per world (what the block's shared memory leaves after the binding, the arena's hot
// part and the rows region; at most STAGE_MAX_BYTES and the model's setting): the most used leaves first - the world
// scalars, the bodies, the joints, the fixtures, then the contact slots' fields in order of use - each taken if it
// still fits, on 16-byte boundaries. Measured (10-step calls, steps 50-400): c1 +0.5 % with everything that fits,
// -2.5 % with the non-contact rows only; c0 -7 %, c3 -10 %, c4 at 8192 worlds +2 %. The rows' reads are L1 hits
// already, the interleaved pairs and quadruples of floats (c[2b], point_local[4s + k]) conflict in shared-memory
// banks, and the staging area takes from the L1, so the default stages nothing.
constexpr int STAGE_MAX_BYTES = 16384;
void plan_staging(StepParams &p, int budget, int model_max) {
    static const int order[] = {
        GOIB2D_GRAVITY, GOIB2D_INV_DT0, GOIB2D_NEXT_KEY, GOIB2D_NEW_FIXTURE, GOIB2D_OVERFLOW, GOIB2D_T_EVENTS,
        GOIB2D_B_TYPE, GOIB2D_B_ACTIVE, GOIB2D_B_AWAKE, GOIB2D_B_ALLOW_SLEEP, GOIB2D_B_BULLET, GOIB2D_B_CONTINUOUS,
        GOIB2D_B_SLEEP_TIME, GOIB2D_B_XF_P, GOIB2D_B_XF_Q, GOIB2D_B_LOCAL_CENTER, GOIB2D_B_C0, GOIB2D_B_C,
        GOIB2D_B_A0, GOIB2D_B_A, GOIB2D_B_V, GOIB2D_B_W, GOIB2D_B_FORCE, GOIB2D_B_TORQUE, GOIB2D_B_MASS,
        GOIB2D_B_INV_MASS, GOIB2D_B_INERTIA, GOIB2D_B_INV_INERTIA, GOIB2D_B_LINEAR_DAMPING,
        GOIB2D_B_ANGULAR_DAMPING, GOIB2D_B_GRAVITY_SCALE, GOIB2D_T_ALPHA0,
        GOIB2D_J_ENABLE_MOTOR, GOIB2D_J_MOTOR_SPEED, GOIB2D_J_MAX_MOTOR, GOIB2D_J_ENABLE_LIMIT, GOIB2D_J_LOWER,
        GOIB2D_J_UPPER, GOIB2D_J_FREQUENCY, GOIB2D_J_DAMPING, GOIB2D_J_IMPULSE, GOIB2D_J_MOTOR_IMPULSE,
        GOIB2D_J_LIMIT_STATE, GOIB2D_J_LOWER_IMPULSE, GOIB2D_J_UPPER_IMPULSE,
        GOIB2D_F_FAT, GOIB2D_F_FRICTION, GOIB2D_F_RESTITUTION,
        GOIB2D_C_PAIR, GOIB2D_C_KEY, GOIB2D_C_FA, GOIB2D_C_FB, GOIB2D_C_TOUCHING, GOIB2D_C_COUNT, GOIB2D_T_FLAG,
        GOIB2D_T_ENABLED, GOIB2D_T_COUNT, GOIB2D_T_TOI, GOIB2D_C_MTYPE, GOIB2D_C_LOCAL_NORMAL, GOIB2D_C_LOCAL_POINT,
        GOIB2D_C_POINT_LOCAL, GOIB2D_C_POINT_ID, GOIB2D_C_NORMAL_IMPULSE, GOIB2D_C_TANGENT_IMPULSE,
        GOIB2D_C_FRICTION, GOIB2D_C_RESTITUTION, GOIB2D_C_TANGENT_SPEED, GOIB2D_T_SOLVED, GOIB2D_T_NORMAL_IMPULSE,
        GOIB2D_T_TANGENT_IMPULSE};
    static_assert(sizeof(order) / sizeof(order[0]) == GOIB2D_NUM_LEAVES, "every leaf once");
    budget = budget < STAGE_MAX_BYTES ? budget : STAGE_MAX_BYTES;
    budget = budget < model_max ? budget : model_max;
    int used = 0;
    for (int i = 0; i < GOIB2D_NUM_LEAVES; ++i) {
        const int leaf = order[i];
        const int64_t elems = goib2d_leaf_elems(leaf, p.m.B, p.rows, p.m.J, p.C);
        const int nb = (int)(elems * (goib2d_leaf_dtype(leaf) == 2 ? 1 : 4));
        p.leaf_bytes[leaf] = nb;
        const int padded = (nb + 15) & ~15;
        if (nb > 0 && used + padded <= budget) {
            p.stage_off[leaf] = used;
            used += padded;
        } else {
            p.stage_off[leaf] = -1;
        }
    }
    p.stage_bytes = used;
}

cudaError_t launch_steps(StepParams p, cudaStream_t stream) {
    p.world0 = 0, p.world_end = p.n_worlds;
    const int64_t n = p.n_worlds;
    if (!part_kernels(n, p.m.J)) {  // one launch for every step of the call
        int dev = 0, sms = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const int region = step_region(p.lay);
        const BlockShape shape = block_shape(n, sms, p.C, p.step_mode);
        const bool pair = shape.wpw == 2;
        const int wpw = shape.wpw;
        int warps = shape.warps;
        const int fit = STEP_MAX_SMEM / (wpw * region);
        warps = warps > fit ? fit : warps;
        plan_staging(p, STEP_MAX_SMEM / (wpw * warps) - region, p.stage_max);
        const size_t smem = (size_t)wpw * warps * (region + p.stage_bytes);
        const int which = pair ? 1 : warps <= WIDE_MAX_WARPS ? 2 : 0;
        auto kern = which == 1 ? goib2d_step_pair_kernel : which == 2 ? goib2d_step_wide_kernel : goib2d_step_kernel;
        // the dynamic shared memory limit set per kernel and device (host threads may launch concurrently)
        static std::mutex smem_mu;
        static int smem_set[3][64];
        if (smem > 48 * 1024) {
            std::lock_guard<std::mutex> lk(smem_mu);
            if (dev >= 64 || (size_t)smem_set[which][dev] < smem) {
                cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
                if (e != cudaSuccess) return e;
                if (dev < 64) smem_set[which][dev] = (int)smem;
            }
        }
        const int per_block = wpw * warps;
        const unsigned sblocks = (unsigned)((n + per_block - 1) / per_block);
        p.step = 0;
        kern<<<sblocks, 32 * warps, smem, stream>>>(p);  // every step in this one launch (whole_step)
        return cudaGetLastError();
    }
    const int wpb = 4;  // worlds (warps) per block
    const unsigned blocks = (unsigned)((n + wpb - 1) / wpb);
    const size_t hot = (size_t)wpb * p.lay.hot_end;  // dynamic shared memory of the per-step kernels
    for (int k = 0; k < p.n_steps; ++k) {
        p.step = k;
        goib2d_collide_kernel<<<blocks, 32 * wpb, hot, stream>>>(p);
        goib2d_solve_rows_kernel<<<blocks, 32 * wpb, 0, stream>>>(p);
        goib2d_constraints_kernel<<<(unsigned)((n + 31) / 32), 32, 0, stream>>>(p);
        goib2d_finish_kernel<<<blocks, 32 * wpb, 0, stream>>>(p);
        goib2d_broadphase_kernel<<<blocks, 32 * wpb, 0, stream>>>(p);
        goib2d_toi_kernel<<<blocks, 32 * wpb, hot ? hot + (size_t)wpb * p.lay.rows_bytes : 0, stream>>>(p);
    }
    return cudaGetLastError();
}
}  // namespace gb

#ifdef GOIB2D_PHASE_TIMERS
extern "C" int goib2d_debug_phase_cycles(unsigned long long *out, int reset) {
    if (cudaMemcpyFromSymbol(out, g_phase_cycles, sizeof(g_phase_cycles)) != cudaSuccess) return -2;
    if (cudaMemcpyFromSymbol(out + 16, g_counts, sizeof(g_counts)) != cudaSuccess) return -2;
    if (cudaMemcpyFromSymbol(out + 32, g_toi_cycles, sizeof(g_toi_cycles)) != cudaSuccess) return -2;
    if (cudaMemcpyFromSymbol(out + 48, g_span, sizeof(g_span)) != cudaSuccess) return -2;
    if (cudaMemcpyFromSymbol(out + 64, g_phase_max, sizeof(g_phase_max)) != cudaSuccess) return -2;
    if (cudaMemcpyFromSymbol(out + 80, g_lv_cycles, sizeof(g_lv_cycles)) != cudaSuccess) return -2;
    if (reset) {
        unsigned long long z[16] = {0};
        cudaMemcpyToSymbol(g_phase_cycles, z, sizeof(z));
        cudaMemcpyToSymbol(g_counts, z, sizeof(z));
        cudaMemcpyToSymbol(g_toi_cycles, z, sizeof(g_toi_cycles));
        cudaMemcpyToSymbol(g_span, z, sizeof(g_span));
        cudaMemcpyToSymbol(g_phase_max, z, sizeof(g_phase_max));
        cudaMemcpyToSymbol(g_lv_cycles, z, sizeof(g_lv_cycles));
    }
    return 0;
}
#endif
