/*
 * cudallm.h — backend C-ABI of CudaLLM (qwen2) for harnesses in other
 * languages (Python ctypes, cgo, ...).
 *
 * Each call maps one-to-one onto the reference backend contract used by
 * chat::generate (chat.cpp:832-878) and declared by CPULLM / MetalLLM
 * (cpu_llm.h:167-194, metal_llm.h:20-51):
 *   cudallm_create   <- CPULLM(const std::string&, std::size_t max_sequence)
 *   cudallm_reset    <- void reset()
 *   cudallm_prefill  <- std::int32_t prefill(const std::vector<std::int32_t>&)
 *   cudallm_decode   <- std::int32_t decode(std::int32_t)
 *   cudallm_position / cudallm_max_sequence / cudallm_memory_stats /
 *   cudallm_enable_profiling / cudallm_disable_profiling <- same-named members
 * The C++ exceptions of that contract become status codes:
 *   std::invalid_argument -> CUDALLM_EINVAL, std::out_of_range -> CUDALLM_ERANGE,
 *   std::length_error -> CUDALLM_ELENGTH, std::runtime_error -> CUDALLM_ERUNTIME;
 * cudallm_last_error() returns the message of the last failure on the
 * calling thread.
 */
#ifndef CUDALLM_H
#define CUDALLM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CUDALLM_API __attribute__((visibility("default")))

enum {
    CUDALLM_OK = 0,
    CUDALLM_EINVAL = 1,
    CUDALLM_ERANGE = 2,
    CUDALLM_ELENGTH = 3,
    CUDALLM_ERUNTIME = 4
};

typedef struct cudallm_model cudallm_model;

CUDALLM_API const char* cudallm_last_error(void);
/* 128-byte NCCL unique id for a multi-GPU job (rank 0 creates, all receive). */
CUDALLM_API int cudallm_nccl_unique_id(char out[128]);

/* device < 0: current device.  world == 1: single GPU (nccl_id ignored). */
CUDALLM_API int cudallm_create(const char* gguf_path, size_t max_sequence, int device, int rank, int world,
                               const char* nccl_id, cudallm_model** out);
CUDALLM_API void cudallm_destroy(cudallm_model* m);
CUDALLM_API int cudallm_reset(cudallm_model* m);
CUDALLM_API int cudallm_prefill(cudallm_model* m, const int32_t* ids, size_t n, int32_t* token);
CUDALLM_API int cudallm_decode(cudallm_model* m, int32_t id, int32_t* token);
/* Logits of the last prefill/decode, n >= vocabulary size (collective when world > 1). */
CUDALLM_API int cudallm_last_logits(cudallm_model* m, float* out, size_t n);
CUDALLM_API float cudallm_last_call_ms(const cudallm_model* m);
/* Device time of the last decode's one-launch step kernel alone (qwen2 on one
 * GPU), milliseconds; 0 when the decode ran as a graph of per-operator kernels. */
CUDALLM_API float cudallm_last_kernel_ms(const cudallm_model* m);
CUDALLM_API size_t cudallm_position(const cudallm_model* m);
CUDALLM_API size_t cudallm_max_sequence(const cudallm_model* m);
/* layer_count, embedding_size, feed_forward_size, attention_head_count,
 * kv_head_count, head_size, vocabulary_size, context_length (up to n). */
CUDALLM_API int cudallm_config(const cudallm_model* m, long long* out, int n);
/* weight, kv_cache, recurrent_state, intermediate bytes. */
CUDALLM_API int cudallm_memory_stats(const cudallm_model* m, uint64_t out[4]);
CUDALLM_API int cudallm_enable_profiling(cudallm_model* m, const char* csv_path);
CUDALLM_API int cudallm_disable_profiling(cudallm_model* m);
CUDALLM_API int cudallm_device_name(const cudallm_model* m, char* buf, size_t n);
/* available() of the reference GPU backends (metal_llm.h:46, moe_llm.h:55):
 * 1 for a created model, 0 for NULL. */
CUDALLM_API int cudallm_available(const cudallm_model* m);
/* The qwen35moe expert cache (moe_llm.h:9-17, 49-50): out[0] = experts
 * resident per layer on this rank (all of them: every expert stays in HBM),
 * out[1] = hits (routed expert uses so far), out[2] = misses (always 0).
 * A qwen2 model reports zeros. */
CUDALLM_API int cudallm_expert_cache(const cudallm_model* m, uint64_t out[3]);

/* Host only (no GPU needed): parse a GGUF file's header, metadata and tensor
 * table without reading tensor data, the first step of cudallm_create.
 * Writes general.architecture (NUL-terminated, cut to n - 1 bytes) and the
 * tensor count (either may be NULL).  A malformed or truncated file returns
 * CUDALLM_ERUNTIME with the reader's message, as the reference's readers
 * throw std::runtime_error (model.cpp:376-448, metal_model.cpp:450-562). */
CUDALLM_API int cudallm_gguf_inspect(const char* gguf_path, char* arch, size_t n, uint64_t* tensor_count);

/* Multi-GPU placement, host only (no GPU needed): the shards cudallm_create
 * loads on each rank.  No counterpart in the reference, which runs on one GPU;
 * these make the split inspectable by harnesses and CPU tests.
 *
 * Tensor parallel (qwen2): rank `rank` of `world` holds query heads
 * [q_head0, q_head0 + q_heads) and KV heads [kv_head0, kv_head0 + kv_heads)
 * (Q/K/V rows of those heads), gate/up rows and ffn_down input columns
 * [ffn0, ffn0 + ffn_rows), o_proj input columns [o_col0, o_col0 + o_cols) (of
 * the all-gathered attention output when gather_attn), and LM-head rows
 * [vocab0, vocab0 + vocab_rows).  o_block: the widest column block of the
 * layers' attn_output types (256 for K-quants, 32 for Q5_0 / Q8_0, 1 for F32). */
typedef struct cudallm_tp_shard {
    uint64_t q_head0, q_heads, kv_head0, kv_heads;
    uint64_t ffn0, ffn_rows, o_col0, o_cols, vocab0, vocab_rows;
    int32_t gather_attn;
} cudallm_tp_shard;
CUDALLM_API int cudallm_tp_plan(uint64_t feed_forward, uint64_t vocabulary, uint64_t heads, uint64_t kv_heads,
                                uint64_t head_size, uint64_t o_block, int world, int rank, cudallm_tp_shard* out);
/* Expert parallel (qwen35moe): expert_rank[e] / expert_local[e] = the rank
 * holding routed expert e and its index in that rank's stacked expert
 * tensors, for e < experts; shared_rank[l] = the rank running layer l's
 * shared expert, for l < layers.  Any output may be NULL. */
CUDALLM_API int cudallm_ep_plan(uint64_t experts, uint64_t layers, int world, int32_t* expert_rank,
                                int32_t* expert_local, int32_t* shared_rank);

#ifdef __cplusplus
}
#endif

#endif /* CUDALLM_H */
