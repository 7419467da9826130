// Profile CSV in the reference's format, so tools that read MyLLM profiles
// read these too: the same 19-column header (profiler.cpp:627-631), one
// `forward_total` row (stage "forward.total") and one `forward_stage` row per
// prefill / decode call (profiler.cpp:660-700), and `global` rows per stage
// when the file is closed (profiler.cpp:843-851).  The derived columns follow
// the reference's definitions (profiler.cpp:783-841): logical bytes = read +
// write, estimated bytes = logical + temporary, GFLOP/s and GB/s over the
// call's wall time, arithmetic intensity = FLOPs / bytes.
//
// The FLOP and byte figures are logical, shape-derived estimates of the call
// (weights at their native GGML block size, KV rows, logits), not hardware
// counters.  Time is host wall time around the call, as in the reference,
// which includes the device work and the token read-back.
#pragma once

#include <cstddef>
#include <cstdint>
#include <fstream>
#include <map>
#include <string>

namespace cudallm {

struct ProfileMetrics {
    std::uint64_t flops = 0;
    std::uint64_t read_bytes = 0;
    std::uint64_t write_bytes = 0;
    std::uint64_t temporary_bytes = 0;
    std::uint64_t allocations = 0;
};

class ProfileCsv {
public:
    // Throws std::invalid_argument for an empty path, std::runtime_error when
    // the file cannot be opened (the reference Profiler's contract).
    explicit ProfileCsv(const std::string& path);
    // Writes the `global` rows.
    ~ProfileCsv();
    ProfileCsv(const ProfileCsv&) = delete;
    ProfileCsv& operator=(const ProfileCsv&) = delete;

    // One prefill / decode call: `stage` (e.g. "decode.gpu_resident"),
    // `sequence_tokens` (prompt length, or position + 1 for a decode step).
    void forward(const std::string& stage, std::size_t sequence_tokens, std::uint64_t elapsed_ns,
                 const ProfileMetrics& metrics);

private:
    struct Aggregate {
        std::uint64_t calls = 0;
        std::uint64_t elapsed_ns = 0;
        ProfileMetrics metrics;
    };
    void add(Aggregate& a, std::uint64_t elapsed_ns, const ProfileMetrics& m);
    void row(const char* record_type, const std::string& forward_index, const std::string& sequence_tokens,
             const std::string& stage, const Aggregate& a);

    std::ofstream out_;
    std::size_t forward_index_ = 0;
    std::map<std::string, Aggregate> global_;
};

}  // namespace cudallm
