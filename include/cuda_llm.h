// cuda_llm.h — C++17 API of the CudaLLM backend.
//
// CudaLLM is a drop-in sibling of the reference's CPULLM / MetalLLM
// (cpu_llm.h:167-194, metal_llm.h:20-51): same constructor shape, the same
// reset() / prefill(ids) / decode(id) -> greedy token contract, the same
// exception types, and no CPU fallback.  Weights stay native GGML blocks in
// HBM; all arithmetic runs in sm_100a kernels behind cudallm_kernels.h.
//
// Multi-GPU: one process per GPU.  With world > 1 the dense Qwen2 model is
// tensor-parallel (column-split QKV / gate / up, row-split o_proj / down,
// NCCL all-reduce after each row split); every rank calls the same methods
// with the same arguments and receives the same token.  One process may also
// hold models on several devices (each model's calls run with its device
// current): the kernels' shared-memory limits and SM counts are set up per
// device, the first time a launch runs on it.
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <limits>
#include <memory>
#include <string>
#include <vector>

// The C++ API is exported from libcudallm.so (which builds everything else
// with hidden visibility), so C++ hosts can link against it.
#if defined(__GNUC__)
#define CUDALLM_CXX_API __attribute__((visibility("default")))
#else
#define CUDALLM_CXX_API
#endif

namespace cudallm {

// Byte accounting returned by every backend (memory_stats.h:11-36 layout).
struct MemoryStats {
    std::uint64_t weight_bytes = 0;
    std::uint64_t kv_cache_bytes = 0;
    std::uint64_t recurrent_state_bytes = 0;
    std::uint64_t intermediate_bytes = 0;
    bool intermediate_is_estimate = false;

    std::uint64_t total_bytes() const noexcept {
        const std::uint64_t parts[] = {weight_bytes, kv_cache_bytes, recurrent_state_bytes, intermediate_bytes};
        std::uint64_t t = 0;
        for (std::uint64_t p : parts) {
            if (p > std::numeric_limits<std::uint64_t>::max() - t) return std::numeric_limits<std::uint64_t>::max();
            t += p;
        }
        return t;
    }

    // Converts to any stats struct with these five fields, such as the
    // reference's MemoryStats, so that callers written against it (a generic
    // generate<Backend> storing backend.memory_stats()) compile unchanged.
    template <typename Stats>
    operator Stats() const {
        Stats s{};
        s.weight_bytes = weight_bytes;
        s.kv_cache_bytes = kv_cache_bytes;
        s.recurrent_state_bytes = recurrent_state_bytes;
        s.intermediate_bytes = intermediate_bytes;
        s.intermediate_is_estimate = intermediate_is_estimate;
        return s;
    }
};

// Model hyper-parameters read from GGUF metadata (model.h:14-35 fields that
// the compute path uses; tokenizer tables are outside this backend).
struct ModelConfig {
    std::string architecture;
    std::size_t tensor_count = 0;
    std::size_t parameter_count = 0;
    std::size_t stored_weight_bytes = 0;
    std::size_t layer_count = 0;
    std::size_t embedding_size = 0;
    std::size_t feed_forward_size = 0;
    std::size_t attention_head_count = 0;
    std::size_t kv_head_count = 0;
    std::size_t head_size = 0;
    std::size_t rotary_dimension = 0;
    std::size_t vocabulary_size = 0;
    std::size_t context_length = 0;
    std::int32_t eos_token_id = 0;
    float rope_theta = 1000000.0f;
    float norm_epsilon = 1e-6f;
    // qwen35moe (zero for qwen2)
    std::size_t full_attention_interval = 0;
    std::size_t expert_count = 0;
    std::size_t expert_used_count = 0;
    std::size_t expert_feed_forward_size = 0;
    std::size_t shared_expert_feed_forward_size = 0;
    std::size_t ssm_conv_kernel = 0;
    std::size_t ssm_state_size = 0;
    std::size_t ssm_group_count = 0;
    std::size_t ssm_time_step_rank = 0;
    std::size_t ssm_inner_size = 0;
    // tokenizer tables, for callers that build their tokenizer from the
    // backend's config (model.h:30-32): tokenizer.ggml.tokens / .merges /
    // .pre; empty when the file carries only a token count
    std::vector<std::string> vocabulary;
    std::vector<std::string> merges;
    std::string tokenizer_pre;
};

// Rank layout for multi-GPU runs.  nccl_id is the 128-byte ncclUniqueId that
// rank 0 created (cudallm_nccl_unique_id) and every rank received.
struct ParallelConfig {
    int rank = 0;
    int world = 1;
    std::array<char, 128> nccl_id{};
};

// One rank's tensor-parallel share of a qwen2 model: the split CudaLLM loads
// and computes with (world == 1: everything on the one rank).
//  * query and KV heads: an even split (world must divide both counts);
//  * gate / up rows and ffn_down input columns: contiguous shares of the
//    256-column block grid, the lower ranks taking the extra blocks;
//  * o_proj input columns: this rank's heads when their columns start and end
//    on the o_proj block grid (o_block: the widest column block among the
//    layers' attn_output types), otherwise a contiguous share of that grid over
//    the all-gathered attention output (gather_attn);
//  * LM-head rows: contiguous shares of the vocabulary, uneven by one row.
// Rank 0 always holds a non-empty share of every split, so it can add the
// residual; a later rank's share may be empty (fewer blocks than ranks).
struct TensorParallelShard {
    std::size_t q_head0 = 0, q_heads = 0;
    std::size_t kv_head0 = 0, kv_heads = 0;
    std::size_t ffn0 = 0, ffn_rows = 0;
    std::size_t o_col0 = 0, o_cols = 0;
    bool gather_attn = false;
    std::size_t vocab0 = 0, vocab_rows = 0;
};

// Throws std::invalid_argument for a rank / world or a shape the split does
// not take.  Host only: needs no GPU.
CUDALLM_CXX_API TensorParallelShard plan_tensor_parallel(std::size_t feed_forward, std::size_t vocabulary,
                                                         std::size_t heads, std::size_t kv_heads,
                                                         std::size_t head_size, std::size_t o_block, int world,
                                                         int rank);

class CUDALLM_CXX_API CudaLLM {
public:
    // device < 0 uses the current CUDA device.
    explicit CudaLLM(const std::string& gguf_path, std::size_t max_sequence = 0, int device = -1,
                     const ParallelConfig& parallel = ParallelConfig{});
    ~CudaLLM();

    CudaLLM(const CudaLLM&) = delete;
    CudaLLM& operator=(const CudaLLM&) = delete;
    CudaLLM(CudaLLM&&) noexcept;
    CudaLLM& operator=(CudaLLM&&) noexcept;

    void reset();
    std::int32_t prefill(const std::vector<std::int32_t>& token_ids);
    std::int32_t decode(std::int32_t token_id);

    void enable_profiling(const std::string& csv_path, bool kernel_timing = false);
    void disable_profiling();

    const ModelConfig& config() const;
    std::size_t position() const noexcept;
    std::size_t max_sequence() const noexcept;
    bool uses_gpu() const noexcept;
    MemoryStats memory_stats() const noexcept;
    bool available() const noexcept;
    const std::string& device_name() const;

    // Extensions used by parity tests and benchmarks.
    // Logits of the most recent prefill/decode (host copy, FP32, vocab size).
    void last_logits(float* out, std::size_t n) const;
    // Device time of the most recent prefill / decode call, milliseconds.
    float last_call_ms() const noexcept;
    // Device time of the most recent decode's one-launch step kernel alone
    // (without the token copies around it), milliseconds; 0 when the decode
    // ran as the per-operator graph.
    float last_kernel_ms() const noexcept;

private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
};

}  // namespace cudallm
