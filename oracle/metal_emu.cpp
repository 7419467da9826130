// ORACLE (test infrastructure only): runs one threadgroup of a reference
// Metal kernel on the host.  Every simulated thread is a coroutine
// (ucontext) on the calling thread with its own stack; they run one at a
// time: each runs until its next threadgroup_barrier (or until it returns),
// then the next lower thread index that is still running resumes; after the
// lowest, the next phase starts again at the highest index.  The order is
// therefore fixed, and within a phase every thread runs before any
// lower-indexed one.
//
// Why a fixed order: the reference's row softmax (metal_softmax_f32) reads
// the row maximum from partial[0] in the same barrier interval in which
// thread 0 stores its partial sum into partial[0].  Free-running threads give
// a different routing from run to run; with the highest index first every
// thread reads the maximum before thread 0 overwrites it, which is what the
// kernel relies on.  The reductions (rows, L2 norms, RMSNorm) write only
// their own slot in a phase and do not depend on the order.
#include <ucontext.h>

#include <vector>

namespace {

constexpr size_t kStack = 256 * 1024;

struct Sim {
    ucontext_t main;
    std::vector<ucontext_t> ctx;
    std::vector<char> alive;
    std::vector<std::vector<char>> stacks;  // kept between groups
    void (*body)(void*, unsigned) = nullptr;
    void* arg = nullptr;
    int cur = 0;
};

Sim g_sim;  // one threadgroup at a time, on the thread that runs it

void entry() {
    g_sim.body(g_sim.arg, (unsigned)g_sim.cur);
    g_sim.alive[g_sim.cur] = 0;
}  // returns to uc_link: the scheduler

}  // namespace

extern "C" void metal_shim_barrier(void) { swapcontext(&g_sim.ctx[g_sim.cur], &g_sim.main); }

extern "C" void metal_shim_run_group(unsigned threads, void (*body)(void*, unsigned), void* ctx) {
    Sim& s = g_sim;
    s.body = body;
    s.arg = ctx;
    s.ctx.resize(threads);
    s.alive.assign(threads, 1);
    if (s.stacks.size() < threads) s.stacks.resize(threads);
    for (unsigned t = 0; t < threads; ++t) {
        if (s.stacks[t].empty()) s.stacks[t].resize(kStack);
        getcontext(&s.ctx[t]);
        s.ctx[t].uc_stack.ss_sp = s.stacks[t].data();
        s.ctx[t].uc_stack.ss_size = kStack;
        s.ctx[t].uc_link = &s.main;
        makecontext(&s.ctx[t], entry, 0);
    }
    for (bool any = true; any;) {
        any = false;
        for (int t = (int)threads - 1; t >= 0; --t) {
            if (!s.alive[t]) continue;
            s.cur = t;
            swapcontext(&s.main, &s.ctx[t]);
            any = any || s.alive[t];
        }
    }
}
