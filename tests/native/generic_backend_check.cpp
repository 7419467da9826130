// The members a generic host of the reference's backend contract uses
// (a generate<Backend> loop and its helpers: profiling switches, capacity and protocol checks,
// stop tokens from config().eos_token_id, a tokenizer built from
// config().vocabulary / merges / tokenizer_pre, stats kept in the caller's own
// memory-stats struct), instantiated for both CUDA backends.  Compile-only:
// tests/test_abi.py checks that it compiles against include/.
#include <cstdint>
#include <string>
#include <vector>

#include "cuda_llm.h"
#include "cuda_moe_llm.h"

namespace {

// The caller's own stats type, with the fields of the reference's MemoryStats.
struct CallerMemoryStats {
    std::uint64_t weight_bytes = 0;
    std::uint64_t kv_cache_bytes = 0;
    std::uint64_t recurrent_state_bytes = 0;
    std::uint64_t intermediate_bytes = 0;
    bool intermediate_is_estimate = false;
};

template <typename Backend>
std::size_t drive(Backend& backend, std::vector<std::int32_t> ids) {
    const auto& config = backend.config();
    if (config.layer_count == 0 || config.vocabulary_size == 0 || config.context_length == 0) return 0;
    if (backend.max_sequence() == 0 || ids.size() >= backend.max_sequence()) return 0;
    std::size_t tables = config.vocabulary.size() + config.merges.size() + config.tokenizer_pre.size();
    std::vector<std::int32_t> stop{config.eos_token_id};
    const bool gpu = backend.uses_gpu();
    backend.enable_profiling("profile.csv");          // the CLI's call for a non-Metal backend
    backend.enable_profiling("profile.csv", false);   // and the two-argument form
    backend.reset();
    std::int32_t next = backend.prefill(ids);
    next = backend.decode(next);
    CallerMemoryStats memory;
    memory = backend.memory_stats();
    backend.disable_profiling();
    return tables + stop.size() + (std::size_t)next + (std::size_t)memory.weight_bytes + (gpu ? 1 : 0) +
           backend.position() + config.embedding_size;
}

}  // namespace

template std::size_t drive<cudallm::CudaLLM>(cudallm::CudaLLM&, std::vector<std::int32_t>);
template std::size_t drive<cudallm::CudaMoeLLM>(cudallm::CudaMoeLLM&, std::vector<std::int32_t>);
