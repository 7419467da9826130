#include "profile.h"

#include <iomanip>
#include <limits>
#include <stdexcept>

namespace cudallm {

namespace {

std::uint64_t sat_add(std::uint64_t a, std::uint64_t b) {
    return a > std::numeric_limits<std::uint64_t>::max() - b ? std::numeric_limits<std::uint64_t>::max() : a + b;
}

std::string csv_field(const std::string& v) {
    if (v.find_first_of(",\"\r\n") == std::string::npos) return v;
    std::string q = "\"";
    for (char c : v) {
        if (c == '"') q += '"';
        q += c;
    }
    return q + "\"";
}

}  // namespace

ProfileCsv::ProfileCsv(const std::string& path) {
    if (path.empty()) throw std::invalid_argument("Profile CSV path cannot be empty");
    out_.open(path, std::ios::out | std::ios::trunc);
    if (!out_) throw std::runtime_error("Cannot open profile CSV: " + path);
    out_ << "record_type,forward_index,sequence_tokens,layer_index,stage,calls,time_ms,flops,read_bytes,"
            "write_bytes,temporary_bytes,logical_bytes,estimated_bytes_with_temporaries,allocations,gflops,"
            "logical_gbps,estimated_gbps,arithmetic_intensity,arithmetic_intensity_with_temporaries\n";
    out_.flush();
}

ProfileCsv::~ProfileCsv() {
    if (!out_) return;
    for (const auto& g : global_) row("global", "", "", g.first, g.second);
    out_.flush();
}

void ProfileCsv::add(Aggregate& a, std::uint64_t elapsed_ns, const ProfileMetrics& m) {
    a.calls += 1;
    a.elapsed_ns = sat_add(a.elapsed_ns, elapsed_ns);
    a.metrics.flops = sat_add(a.metrics.flops, m.flops);
    a.metrics.read_bytes = sat_add(a.metrics.read_bytes, m.read_bytes);
    a.metrics.write_bytes = sat_add(a.metrics.write_bytes, m.write_bytes);
    a.metrics.temporary_bytes = sat_add(a.metrics.temporary_bytes, m.temporary_bytes);
    a.metrics.allocations = sat_add(a.metrics.allocations, m.allocations);
}

void ProfileCsv::forward(const std::string& stage, std::size_t sequence_tokens, std::uint64_t elapsed_ns,
                         const ProfileMetrics& metrics) {
    Aggregate one;
    add(one, elapsed_ns, metrics);
    const std::string fi = std::to_string(forward_index_), st = std::to_string(sequence_tokens);
    // the call is the forward's only stage: the forward total equals it
    row("forward_total", fi, st, "forward.total", one);
    row("forward_stage", fi, st, stage, one);
    out_.flush();
    add(global_["forward.total"], elapsed_ns, metrics);
    add(global_[stage], elapsed_ns, metrics);
    ++forward_index_;
}

void ProfileCsv::row(const char* record_type, const std::string& forward_index, const std::string& sequence_tokens,
                     const std::string& stage, const Aggregate& a) {
    const double s = (double)a.elapsed_ns / 1e9;
    const std::uint64_t logical = sat_add(a.metrics.read_bytes, a.metrics.write_bytes);
    const std::uint64_t estimated = sat_add(logical, a.metrics.temporary_bytes);
    const double flops = (double)a.metrics.flops;
    out_ << record_type << ',' << forward_index << ',' << sequence_tokens << ",," << csv_field(stage) << ','
         << a.calls << ',' << std::fixed << std::setprecision(3) << (double)a.elapsed_ns / 1e6 << ','
         << a.metrics.flops << ',' << a.metrics.read_bytes << ',' << a.metrics.write_bytes << ','
         << a.metrics.temporary_bytes << ',' << logical << ',' << estimated << ',' << a.metrics.allocations << ','
         << (s > 0 ? flops / s / 1e9 : 0.0) << ',' << (s > 0 ? (double)logical / s / 1e9 : 0.0) << ','
         << (s > 0 ? (double)estimated / s / 1e9 : 0.0) << ',' << (logical ? flops / (double)logical : 0.0) << ','
         << (estimated ? flops / (double)estimated : 0.0) << '\n';
}

}  // namespace cudallm
