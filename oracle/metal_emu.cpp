// ORACLE (test infrastructure only): runs one threadgroup of a reference
// Metal kernel on the host.  Every simulated thread is an OS thread, but they
// run one at a time: each runs until its next threadgroup_barrier (or until
// it returns), then hands over to the next lower thread index that is still
// running; after thread 0 (or the lowest live thread) the next phase starts
// again at the highest index.  The order is therefore fixed, and within a
// phase every thread runs before any lower-indexed one.
//
// Why a fixed order: the reference's row softmax (metal_softmax_f32) reads
// the row maximum from partial[0] in the same barrier interval in which
// thread 0 stores its partial sum into partial[0].  Free-running threads give
// a different routing from run to run; with the highest index first every
// thread reads the maximum before thread 0 overwrites it, which is what the
// kernel relies on.  The reductions (rows, L2 norms, RMSNorm) write only
// their own slot in a phase and do not depend on the order.
#include <memory>
#include <semaphore>
#include <thread>
#include <vector>

namespace {

struct Group {
    int n = 0;
    std::vector<std::unique_ptr<std::binary_semaphore>> turn;
    std::vector<char> alive;

    // the live thread after `from` in the order: lower indices first, then
    // wrap to the highest live index (a new phase); -1 when none is left
    int next(int from) const {
        for (int j = from - 1; j >= 0; --j)
            if (alive[j]) return j;
        for (int j = n - 1; j >= 0; --j)
            if (alive[j]) return j;
        return -1;
    }
};

thread_local Group* t_group = nullptr;
thread_local int t_index = 0;

}  // namespace

extern "C" void metal_shim_barrier(void) {
    Group& g = *t_group;
    const int j = g.next(t_index);
    g.turn[j]->release();
    g.turn[t_index]->acquire();
}

extern "C" void metal_shim_run_group(unsigned threads, void (*body)(void*, unsigned), void* ctx) {
    Group g;
    g.n = (int)threads;
    g.alive.assign(threads, 1);
    for (unsigned t = 0; t < threads; ++t) g.turn.emplace_back(std::make_unique<std::binary_semaphore>(0));
    std::vector<std::thread> pool;
    pool.reserve(threads);
    for (unsigned t = 0; t < threads; ++t)
        pool.emplace_back([&g, body, ctx, t] {
            t_group = &g;
            t_index = (int)t;
            g.turn[t]->acquire();
            body(ctx, t);
            g.alive[t] = 0;
            const int j = g.next((int)t);
            if (j >= 0) g.turn[j]->release();
        });
    g.turn[threads - 1]->release();
    for (auto& th : pool) th.join();
}
