// The same calls as profile_check.cpp through the reference's Profiler
// (profiler.h / profiler.cpp, compiled from the reference sources by the
// test): one ForwardScope per call with one Scope named like the reference's
// GPU backends name theirs (metal_llm.mm:3216-3221).
#include "profiler.h"

namespace {
void call(llm::Profiler& p, std::size_t tokens, const char* stage, llm::ProfileMetrics m) {
    llm::Profiler::ForwardScope f(&p, tokens);
    llm::Profiler::Scope s(&p, stage, m);
}
}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    llm::Profiler p(argv[1]);
    llm::ProfileMetrics a, b, c;
    a.flops = 1000000000ull; a.read_bytes = 2000000ull; a.write_bytes = 300000ull;
    b.flops = 500000000ull; b.read_bytes = 1000000ull; b.write_bytes = 100ull;
    c.flops = 600000000ull; c.read_bytes = 1100000ull; c.write_bytes = 100ull; c.temporary_bytes = 7ull;
    c.allocations = 1ull;
    call(p, 16, "prefill.gpu_resident", a);
    call(p, 17, "decode.gpu_resident", b);
    call(p, 18, "decode.gpu_resident", c);
    return 0;
}
