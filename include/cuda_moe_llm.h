// cuda_moe_llm.h — CudaMoeLLM: qwen35moe (Qwen3.5/3.6 A3B) on B200s.
//
// The same backend contract as the reference's MoeLLM (moe_llm.h:26-60):
// reset / prefill / decode, exceptions std::invalid_argument (protocol),
// std::out_of_range (token ids), std::length_error (capacity),
// std::runtime_error (file / device).  reset() zeroes the DeltaNet state and
// convolution history and rewinds the KV position (moe_llm.mm:1537-1547).
// All experts stay resident in HBM, so the reference's expert cache becomes
// "every expert of this rank is cached".
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "cuda_llm.h"

namespace cudallm {

struct ExpertCacheStats {
    std::uint64_t hits = 0;
    std::uint64_t misses = 0;
    std::uint64_t requests() const noexcept { return hits + misses; }
};

// Expert-parallel placement: routed expert e lives on rank e % world, stacked
// in expert order (local index e / world); layer l's shared expert runs on
// rank l % world.  The device kernels (cl_moe_expert_gemv, cl_moe_combine)
// apply the same rule to the expert ids they read.
inline int ep_expert_rank(std::size_t expert, int world) noexcept { return (int)(expert % (std::size_t)world); }
inline std::size_t ep_local_index(std::size_t expert, int world) noexcept { return expert / (std::size_t)world; }
inline int ep_shared_rank(std::size_t layer, int world) noexcept { return (int)(layer % (std::size_t)world); }

class CUDALLM_CXX_API CudaMoeLLM {
public:
    // parallel.world > 1: expert parallel — expert e lives on rank
    // e % world; attention, DeltaNet and the LM head are replicated.
    explicit CudaMoeLLM(const std::string& gguf_path, std::size_t max_sequence = 0, int device = -1,
                        const ParallelConfig& parallel = ParallelConfig{});
    ~CudaMoeLLM();

    CudaMoeLLM(const CudaMoeLLM&) = delete;
    CudaMoeLLM& operator=(const CudaMoeLLM&) = delete;
    CudaMoeLLM(CudaMoeLLM&&) noexcept;
    CudaMoeLLM& operator=(CudaMoeLLM&&) noexcept;

    void reset();
    std::int32_t prefill(const std::vector<std::int32_t>& token_ids);
    std::int32_t decode(std::int32_t token_id);

    void enable_profiling(const std::string& csv_path, bool kernel_timing = false);
    void disable_profiling();

    const ModelConfig& config() const;
    std::size_t position() const noexcept;
    std::size_t max_sequence() const noexcept;
    std::size_t expert_cache_count() const noexcept;  // experts resident per layer on this rank
    ExpertCacheStats expert_cache_stats() const noexcept;  // every routed expert is a hit
    bool uses_gpu() const noexcept;
    MemoryStats memory_stats() const noexcept;
    bool available() const noexcept;
    const std::string& device_name() const;

    void last_logits(float* out, std::size_t n) const;
    float last_call_ms() const noexcept;
    float last_kernel_ms() const noexcept;  // 0: the MoE decode has no one-launch step

private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
};

// "qwen2", "qwen35moe", ...: the general.architecture of a GGUF file.
CUDALLM_CXX_API std::string gguf_architecture(const std::string& gguf_path);

}  // namespace cudallm
