// cudallm_* C-ABI over cudallm::CudaLLM (qwen2) and cudallm::CudaMoeLLM
// (qwen35moe), chosen by the GGUF's general.architecture (see include/cudallm.h).
#include "cudallm.h"

#include <nccl.h>

#include <cstring>
#include <stdexcept>
#include <string>

#include "cuda_llm.h"
#include "cuda_moe_llm.h"
#include "gguf.h"

#include <memory>

struct cudallm_model {
    std::unique_ptr<cudallm::CudaLLM> dense;
    std::unique_ptr<cudallm::CudaMoeLLM> moe;

    template <typename F>
    auto with(F&& f) -> decltype(f(*dense)) {
        if (moe) return f(*moe);
        return f(*dense);
    }
    template <typename F>
    auto with(F&& f) const -> decltype(f(*dense)) {
        if (moe) return f(static_cast<const cudallm::CudaMoeLLM&>(*moe));
        return f(static_cast<const cudallm::CudaLLM&>(*dense));
    }
};

namespace {

thread_local std::string g_error;

template <typename F>
int guard(F&& f) {
    try {
        f();
        return CUDALLM_OK;
    } catch (const std::invalid_argument& e) {
        g_error = e.what();
        return CUDALLM_EINVAL;
    } catch (const std::out_of_range& e) {
        g_error = e.what();
        return CUDALLM_ERANGE;
    } catch (const std::length_error& e) {
        g_error = e.what();
        return CUDALLM_ELENGTH;
    } catch (const std::exception& e) {
        g_error = e.what();
        return CUDALLM_ERUNTIME;
    } catch (...) {
        g_error = "unknown error";
        return CUDALLM_ERUNTIME;
    }
}

void need(const void* p) {
    if (p == nullptr) throw std::invalid_argument("null handle or pointer");
}

}  // namespace

extern "C" {

CUDALLM_API const char* cudallm_last_error(void) { return g_error.c_str(); }

CUDALLM_API int cudallm_nccl_unique_id(char out[128]) {
    return guard([&] {
        need(out);
        ncclUniqueId id;
        if (ncclGetUniqueId(&id) != ncclSuccess) throw std::runtime_error("ncclGetUniqueId failed");
        static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
        std::memcpy(out, &id, 128);
    });
}

CUDALLM_API int cudallm_create(const char* gguf_path, size_t max_sequence, int device, int rank, int world,
                               const char* nccl_id, cudallm_model** out) {
    return guard([&] {
        need(gguf_path);
        need(out);
        cudallm::ParallelConfig par;
        par.rank = rank;
        par.world = world;
        if (world > 1) {
            need(nccl_id);
            std::memcpy(par.nccl_id.data(), nccl_id, 128);
        }
        auto* m = new cudallm_model{};
        try {
            if (cudallm::gguf_architecture(gguf_path) == "qwen35moe")
                m->moe = std::make_unique<cudallm::CudaMoeLLM>(gguf_path, max_sequence, device, par);
            else
                m->dense = std::make_unique<cudallm::CudaLLM>(gguf_path, max_sequence, device, par);
        } catch (...) {
            delete m;
            throw;
        }
        *out = m;
    });
}

CUDALLM_API void cudallm_destroy(cudallm_model* m) { delete m; }

CUDALLM_API int cudallm_reset(cudallm_model* m) {
    return guard([&] {
        need(m);
        m->with([](auto& b) { b.reset(); });
    });
}

CUDALLM_API int cudallm_prefill(cudallm_model* m, const int32_t* ids, size_t n, int32_t* token) {
    return guard([&] {
        need(m);
        need(token);
        if (n > 0) need(ids);
        *token = m->with([&](auto& b) { return b.prefill(std::vector<int32_t>(ids, ids + n)); });
    });
}

CUDALLM_API int cudallm_decode(cudallm_model* m, int32_t id, int32_t* token) {
    return guard([&] {
        need(m);
        need(token);
        *token = m->with([&](auto& b) { return b.decode(id); });
    });
}

CUDALLM_API int cudallm_last_logits(cudallm_model* m, float* out, size_t n) {
    return guard([&] {
        need(m);
        need(out);
        m->with([&](auto& b) { b.last_logits(out, n); });
    });
}

CUDALLM_API float cudallm_last_call_ms(const cudallm_model* m) {
    return m ? m->with([](const auto& b) { return b.last_call_ms(); }) : 0.0f;
}
CUDALLM_API float cudallm_last_kernel_ms(const cudallm_model* m) {
    return m ? m->with([](const auto& b) { return b.last_kernel_ms(); }) : 0.0f;
}
CUDALLM_API size_t cudallm_position(const cudallm_model* m) {
    return m ? m->with([](const auto& b) { return b.position(); }) : 0;
}
CUDALLM_API size_t cudallm_max_sequence(const cudallm_model* m) {
    return m ? m->with([](const auto& b) { return b.max_sequence(); }) : 0;
}

CUDALLM_API int cudallm_config(const cudallm_model* m, long long* out, int n) {
    return guard([&] {
        need(m);
        need(out);
        const cudallm::ModelConfig& c = m->with([](const auto& b) -> const cudallm::ModelConfig& { return b.config(); });
        const long long v[] = {(long long)c.layer_count,          (long long)c.embedding_size,
                               (long long)c.feed_forward_size,    (long long)c.attention_head_count,
                               (long long)c.kv_head_count,        (long long)c.head_size,
                               (long long)c.vocabulary_size,      (long long)c.context_length};
        for (int i = 0; i < n && i < 8; ++i) out[i] = v[i];
    });
}

CUDALLM_API int cudallm_memory_stats(const cudallm_model* m, uint64_t out[4]) {
    return guard([&] {
        need(m);
        need(out);
        const cudallm::MemoryStats s = m->with([](const auto& b) { return b.memory_stats(); });
        out[0] = s.weight_bytes;
        out[1] = s.kv_cache_bytes;
        out[2] = s.recurrent_state_bytes;
        out[3] = s.intermediate_bytes;
    });
}

CUDALLM_API int cudallm_enable_profiling(cudallm_model* m, const char* csv_path) {
    return guard([&] {
        need(m);
        need(csv_path);
        m->with([&](auto& b) { b.enable_profiling(csv_path); });
    });
}

CUDALLM_API int cudallm_disable_profiling(cudallm_model* m) {
    return guard([&] {
        need(m);
        m->with([](auto& b) { b.disable_profiling(); });
    });
}

CUDALLM_API int cudallm_device_name(const cudallm_model* m, char* buf, size_t n) {
    return guard([&] {
        need(m);
        need(buf);
        const std::string& s = m->with([](const auto& b) -> const std::string& { return b.device_name(); });
        if (n == 0) throw std::invalid_argument("empty name buffer");
        std::strncpy(buf, s.c_str(), n - 1);
        buf[n - 1] = 0;
    });
}

CUDALLM_API int cudallm_available(const cudallm_model* m) {
    return m && m->with([](const auto& b) { return b.available(); }) ? 1 : 0;
}

CUDALLM_API int cudallm_expert_cache(const cudallm_model* m, uint64_t out[3]) {
    return guard([&] {
        need(m);
        need(out);
        out[0] = out[1] = out[2] = 0;
        if (m->moe) {
            const cudallm::ExpertCacheStats st = m->moe->expert_cache_stats();
            out[0] = m->moe->expert_cache_count();
            out[1] = st.hits;
            out[2] = st.misses;
        }
    });
}

CUDALLM_API int cudallm_gguf_inspect(const char* gguf_path, char* arch, size_t n, uint64_t* tensor_count) {
    return guard([&] {
        need(gguf_path);
        const cudallm::GgufFile f(gguf_path);
        if (arch) {
            if (n == 0) throw std::invalid_argument("empty architecture buffer");
            const std::string a = f.text("general.architecture");
            std::strncpy(arch, a.c_str(), n - 1);
            arch[n - 1] = 0;
        }
        if (tensor_count) *tensor_count = f.tensors().size();
    });
}

CUDALLM_API int cudallm_tp_plan(uint64_t feed_forward, uint64_t vocabulary, uint64_t heads, uint64_t kv_heads,
                                uint64_t head_size, uint64_t o_block, int world, int rank, cudallm_tp_shard* out) {
    return guard([&] {
        need(out);
        const cudallm::TensorParallelShard s =
            cudallm::plan_tensor_parallel(feed_forward, vocabulary, heads, kv_heads, head_size, o_block, world, rank);
        *out = cudallm_tp_shard{s.q_head0, s.q_heads, s.kv_head0, s.kv_heads, s.ffn0,   s.ffn_rows,
                                s.o_col0,  s.o_cols,  s.vocab0,   s.vocab_rows, s.gather_attn ? 1 : 0};
    });
}

CUDALLM_API int cudallm_ep_plan(uint64_t experts, uint64_t layers, int world, int32_t* expert_rank,
                                int32_t* expert_local, int32_t* shared_rank) {
    return guard([&] {
        if (world < 1) throw std::invalid_argument("invalid parallel world");
        for (uint64_t e = 0; e < experts; ++e) {
            if (expert_rank) expert_rank[e] = cudallm::ep_expert_rank(e, world);
            if (expert_local) expert_local[e] = (int32_t)cudallm::ep_local_index(e, world);
        }
        for (uint64_t l = 0; l < layers && shared_rank; ++l) shared_rank[l] = cudallm::ep_shared_rank(l, world);
    });
}

}  // extern "C"
