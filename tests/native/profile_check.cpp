// Writes a profile CSV through the product's writer (myllm_b200/csrc/host/
// profile.cpp) for a fixed sequence of calls; tests/test_profile_csv.py
// compares it with the reference Profiler's file for the same calls.
#include "profile.h"

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    cudallm::ProfileCsv p(argv[1]);
    p.forward("prefill.gpu_resident", 16, 2500000, {1000000000ull, 2000000ull, 300000ull, 0, 0});
    p.forward("decode.gpu_resident", 17, 1000000, {500000000ull, 1000000ull, 100ull, 0, 0});
    p.forward("decode.gpu_resident", 18, 1500000, {600000000ull, 1100000ull, 100ull, 7ull, 1ull});
    return 0;
}
