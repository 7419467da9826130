// Test infrastructure only: a C-ABI harness around the reference's own CPU
// path, compiled from the reference sources where they lie (see Makefile).
//
// CPULLM (cpu_llm.cpp:916-1073) returns only the greedy token.  Parity needs
// the logits too, so this harness links the same object files and re-drives
// the reference's public functions in exactly the order CPULLM::prefill and
// CPULLM::decode use them (cpu_llm.cpp:1003-1020, 1051-1070):
//   embedding -> cpu_prefill_layer / cpu_decode_layer per layer
//   -> rmsnorm(output_norm) -> gevmt(output.weight, last row).
// It also wraps CPULLM itself, for the timed CPU baseline and to confirm the
// harness's argmax equals CPULLM's token.
#include "cpu_llm.h"
#include "model.h"

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace {

thread_local std::string g_error;

int fail(const std::exception& e, int code) {
    g_error = e.what();
    return code;
}

template <typename F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::invalid_argument& e) {
        return fail(e, 1);
    } catch (const std::length_error& e) {
        return fail(e, 3);
    } catch (const std::out_of_range& e) {
        return fail(e, 2);
    } catch (const std::exception& e) {
        return fail(e, 4);
    }
}

struct Harness {
    std::unique_ptr<llm::ModelFile> file;
    llm::ModelConfig config;
    llm::Matrix embed;
    llm::Vector out_norm;
    llm::Matrix out_weight;
    std::vector<llm::Layer> layers;
    std::vector<llm::CPUKVCache> caches;
    std::size_t position = 0;
};

int32_t argmax_first(const llm::Vector& v) {
    return static_cast<int32_t>(std::distance(
        v.values.begin(), std::max_element(v.values.begin(), v.values.end())));
}

void emit(const llm::Vector& logits, float* out, int32_t* token) {
    if (out != nullptr) {
        std::memcpy(out, logits.values.data(), logits.values.size() * sizeof(float));
    }
    if (token != nullptr) {
        *token = argmax_first(logits);
    }
}

}  // namespace

extern "C" {

const char* ref_last_error() { return g_error.c_str(); }

int ref_open(const char* path, void** handle) {
    return guarded([&] {
        auto h = std::make_unique<Harness>();
        h->file = std::make_unique<llm::ModelFile>(path);
        h->config = h->file->config();
        h->embed = h->file->load_token_embedding();
        h->out_norm = h->file->load_output_norm();
        h->out_weight = h->file->load_output_weight();
        h->layers.reserve(h->config.layer_count);
        for (std::size_t l = 0; l < h->config.layer_count; ++l) {
            h->layers.emplace_back(*h->file, l);
        }
        h->file->validate_all_tensors_loaded();
        h->caches.resize(h->layers.size());
        *handle = h.release();
    });
}

void ref_close(void* handle) { delete static_cast<Harness*>(handle); }

int ref_config(void* handle, long long* out, int n) {
    return guarded([&] {
        const auto& c = static_cast<Harness*>(handle)->config;
        const long long v[] = {
            (long long)c.layer_count, (long long)c.embedding_size,
            (long long)c.feed_forward_size, (long long)c.attention_head_count,
            (long long)c.kv_head_count, (long long)c.head_size,
            (long long)c.vocabulary_size, (long long)c.context_length};
        for (int i = 0; i < n && i < 8; ++i) out[i] = v[i];
    });
}

void ref_reset(void* handle) {
    auto* h = static_cast<Harness*>(handle);
    h->position = 0;
    for (auto& c : h->caches) c = llm::CPUKVCache{};
}

int ref_prefill(void* handle, const int32_t* ids, size_t n, float* logits, int32_t* token) {
    return guarded([&] {
        auto* h = static_cast<Harness*>(handle);
        if (h->position != 0) throw std::invalid_argument("harness prefill requires reset");
        std::vector<int32_t> tokens(ids, ids + n);
        llm::Matrix hidden = llm::embedding(tokens, h->embed);
        for (std::size_t l = 0; l < h->layers.size(); ++l) {
            hidden = llm::cpu_prefill_layer(hidden, h->layers[l], h->config.norm_epsilon,
                                            h->config.rotary_dimension, h->config.rope_theta,
                                            h->config.head_size, h->caches[l]);
        }
        hidden.rmsnorm(h->out_norm, h->config.norm_epsilon);
        emit(llm::gevmt(h->out_weight, hidden.values.back()), logits, token);
        h->position = n;
    });
}

int ref_decode(void* handle, int32_t id, float* logits, int32_t* token) {
    return guarded([&] {
        auto* h = static_cast<Harness*>(handle);
        if (h->position == 0) throw std::invalid_argument("harness decode requires prefill");
        const llm::Matrix embedded = llm::embedding(std::vector<int32_t>{id}, h->embed);
        llm::Vector hidden = embedded.values.front();
        for (std::size_t l = 0; l < h->layers.size(); ++l) {
            hidden = llm::cpu_decode_layer(hidden, h->layers[l], h->config.norm_epsilon,
                                           h->config.rotary_dimension, h->config.rope_theta,
                                           h->config.head_size, h->caches[l]);
        }
        hidden.rmsnorm(h->out_norm, h->config.norm_epsilon);
        emit(llm::gevmt(h->out_weight, hidden), logits, token);
        h->position += 1;
    });
}

// Copy one dequantized tensor (as the reference's GgufDequantizer produced
// it) into `out`.  `which` names a Layer member or a global tensor.
int ref_tensor(void* handle, int layer, const char* which, float* out, size_t capacity,
               size_t* rows, size_t* cols) {
    return guarded([&] {
        auto* h = static_cast<Harness*>(handle);
        const std::string w(which);
        const llm::Matrix* m = nullptr;
        const llm::Vector* v = nullptr;
        if (layer < 0) {
            if (w == "token_embd") m = &h->embed;
            else if (w == "output") m = &h->out_weight;
            else if (w == "output_norm") v = &h->out_norm;
        } else {
            const llm::Layer& L = h->layers.at(static_cast<size_t>(layer));
            if (w == "attn_norm") v = &L.attn_norm_weight;
            else if (w == "attn_q") m = &L.attn_q_weight;
            else if (w == "attn_q_bias") v = &L.attn_q_bias;
            else if (w == "attn_k") m = &L.attn_k_weight;
            else if (w == "attn_k_bias") v = &L.attn_k_bias;
            else if (w == "attn_v") m = &L.attn_v_weight;
            else if (w == "attn_v_bias") v = &L.attn_v_bias;
            else if (w == "attn_output") m = &L.attn_output_weight;
            else if (w == "ffn_norm") v = &L.ffn_norm_weight;
            else if (w == "ffn_gate") m = &L.ffn_gate_weight;
            else if (w == "ffn_up") m = &L.ffn_up_weight;
            else if (w == "ffn_down") m = &L.ffn_down_weight;
        }
        if (m != nullptr) {
            *rows = m->rows;
            *cols = m->cols;
            if (out != nullptr) {
                if (capacity < m->rows * m->cols) throw std::length_error("capacity");
                for (size_t r = 0; r < m->rows; ++r) {
                    std::memcpy(out + r * m->cols, m->values[r].values.data(),
                                m->cols * sizeof(float));
                }
            }
        } else if (v != nullptr) {
            *rows = 1;
            *cols = v->lens;
            if (out != nullptr) {
                if (capacity < v->lens) throw std::length_error("capacity");
                std::memcpy(out, v->values.data(), v->lens * sizeof(float));
            }
        } else {
            throw std::invalid_argument("unknown tensor " + w);
        }
    });
}

// ---- CPULLM itself (timed CPU baseline, token cross-check) ----
int ref_cpullm_open(const char* path, size_t max_sequence, void** handle) {
    return guarded([&] { *handle = new llm::CPULLM(path, max_sequence); });
}

void ref_cpullm_close(void* handle) { delete static_cast<llm::CPULLM*>(handle); }

int ref_cpullm_reset(void* handle) {
    return guarded([&] { static_cast<llm::CPULLM*>(handle)->reset(); });
}

int ref_cpullm_prefill(void* handle, const int32_t* ids, size_t n, int32_t* token) {
    return guarded([&] {
        *token = static_cast<llm::CPULLM*>(handle)->prefill(std::vector<int32_t>(ids, ids + n));
    });
}

int ref_cpullm_decode(void* handle, int32_t id, int32_t* token) {
    return guarded([&] { *token = static_cast<llm::CPULLM*>(handle)->decode(id); });
}

}  // extern "C"
