// Parity oracle (test infrastructure, see oracle.h): batch driver, worlds spread over host threads (the CPU
// baseline). std::thread, because this toolchain has no OpenMP runtime.
#include <atomic>
#include <thread>
#include <vector>

#include "oracle.h"

extern "C" int oracle_step_range(const goib2d_model_desc *desc, const goib2d_settings *s, float dt, int32_t C,
                                 int32_t rows, int64_t w0, int64_t w1, int32_t n_steps, void *const *leaves,
                                 const float *actions, int32_t n_action, const int32_t *action_joint,
                                 const float *action_scale);

extern "C" int oracle_step_range_events(const goib2d_model_desc *desc, const goib2d_settings *s, float dt,
                                        int32_t C, int32_t rows, int64_t w0, int64_t w1, int32_t n_steps,
                                        void *const *leaves, const float *actions, int32_t n_action,
                                        const int32_t *action_joint, const float *action_scale, goib2d_event *events,
                                        int32_t *event_count, int32_t event_cap);

extern "C" int oracle_max_threads(void) {
    unsigned n = std::thread::hardware_concurrency();
    return n ? (int)n : 1;
}

extern "C" int oracle_step_batch(const goib2d_model_desc *desc, const goib2d_settings *s, float dt, int32_t C,
                                 int32_t rows, int64_t n_worlds, int32_t n_steps, void *const *leaves,
                                 const float *actions, int32_t n_action, const int32_t *action_joint,
                                 const float *action_scale, int32_t n_threads) {
    if (n_threads <= 0) n_threads = oracle_max_threads();
    if (n_threads > n_worlds) n_threads = (int32_t)(n_worlds > 0 ? n_worlds : 1);
    std::atomic<int64_t> next{0};
    auto work = [&]() {
        for (;;) {
            int64_t w = next.fetch_add(1);
            if (w >= n_worlds) break;
            oracle_step_range(desc, s, dt, C, rows, w, w + 1, n_steps, leaves, actions, n_action, action_joint,
                              action_scale);
        }
    };
    std::vector<std::thread> pool;
    for (int t = 1; t < n_threads; ++t) pool.emplace_back(work);
    work();
    for (auto &t : pool) t.join();
    return 0;
}

// oracle_step_batch with the contact event log (goib2d_event, include/goib2d.h): events [n_worlds][event_cap],
// event_count [n_worlds]; the log holds the last step's events.
extern "C" int oracle_step_batch_events(const goib2d_model_desc *desc, const goib2d_settings *s, float dt, int32_t C,
                                        int32_t rows, int64_t n_worlds, int32_t n_steps, void *const *leaves,
                                        goib2d_event *events, int32_t *event_count, int32_t event_cap,
                                        int32_t n_threads) {
    if (n_threads <= 0) n_threads = oracle_max_threads();
    if (n_threads > n_worlds) n_threads = (int32_t)(n_worlds > 0 ? n_worlds : 1);
    std::atomic<int64_t> next{0};
    auto work = [&]() {
        for (;;) {
            int64_t w = next.fetch_add(1);
            if (w >= n_worlds) break;
            oracle_step_range_events(desc, s, dt, C, rows, w, w + 1, n_steps, leaves, nullptr, 0, nullptr, nullptr,
                                     events, event_count, event_cap);
        }
    };
    std::vector<std::thread> pool;
    for (int t = 1; t < n_threads; ++t) pool.emplace_back(work);
    work();
    for (auto &t : pool) t.join();
    return 0;
}
