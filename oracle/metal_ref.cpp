// ORACLE (test infrastructure only): the reference's own Metal compute
// kernels (metal_llm.metal, compiled where they lie through metal_shim.h) run
// on the host, one C entry per kernel the qwen35moe checks use.  Each entry
// fills the kernel's own parameter struct and dispatches it the way the
// reference's MoE host does (moe_llm.mm):
//   * dispatch_flat (moe_llm.mm:1829-1842): ceil(count / 256) groups of 256
//     threads, thread_position_in_grid = the flat index; these kernels never
//     share data between threads, so the threads run one after another;
//   * dispatch_rows (moe_llm.mm:1844-1857): one group of 256 threads per row,
//     run with their threadgroup barriers (metal_emu.cpp);
//   * the DeltaNet recurrence (moe_llm.mm:2603-2612): one group per value
//     head, head_dim threads, each owning one state column (no barriers).
#include MYLLM_METAL_SOURCE

extern "C" void metal_shim_run_group(unsigned threads, void (*body)(void*, unsigned), void* ctx);

namespace {

constexpr uint kGroup = 256;  // kReductionThreads (moe_llm.mm:40)

template <class F>
void flat(unsigned long long count, F&& f) {
    const unsigned long long groups = (count + kGroup - 1) / kGroup;
    for (unsigned long long i = 0; i < groups * kGroup; ++i) f((uint)i);
}

template <class F>
void rows(unsigned long long n, F f) {
    struct Ctx {
        F* f;
        uint row;
    };
    for (unsigned long long r = 0; r < n; ++r) {
        Ctx ctx{&f, (uint)r};
        metal_shim_run_group(kGroup, [](void* c, unsigned local) {
            Ctx* x = static_cast<Ctx*>(c);
            (*x->f)((uint)local, uint3(x->row, 0, 0));
        }, &ctx);
    }
}

}  // namespace

extern "C" {

// encode_rmsnorm: rows of `cols`, gamma per column
void mref_rmsnorm(const float* in, const float* gamma, float* out, uint n_rows, uint cols, float eps) {
    MetalRmsNormParams p{};
    p.rows = n_rows;
    p.cols = cols;
    p.epsilon = eps;
    rows(n_rows, [&](uint local, uint3 g) { metal_rmsnorm_f32(in, gamma, out, p, local, g); });
}

// encode_softmax: row-wise, in place allowed
void mref_softmax(const float* in, float* out, uint n_rows, uint cols) {
    MetalElementwiseParams p{};
    p.rows = n_rows;
    p.cols = cols;
    rows(n_rows, [&](uint local, uint3 g) { metal_softmax_f32(in, out, p, local, g); });
}

// encode_unary: 0 sigmoid, 1 silu, 2 softplus, 3 exp
void mref_unary(int op, const float* in, float* out, uint n) {
    MetalElementwiseParams p{};
    p.rows = 1;
    p.cols = n;
    flat(n, [&](uint i) {
        switch (op) {
            case 0: metal_sigmoid_f32(in, out, p, i); break;
            case 1: metal_silu_only_f32(in, out, p, i); break;
            case 2: metal_softplus_f32(in, out, p, i); break;
            default: metal_exp_f32(in, out, p, i); break;
        }
    });
}

// encode_binary: 0 multiply, 1 SwiGLU (silu(a) * b)
void mref_binary(int op, const float* a, const float* b, float* out, uint n) {
    MetalElementwiseParams p{};
    p.rows = 1;
    p.cols = n;
    flat(n, [&](uint i) {
        if (op == 0)
            metal_mul_f32(a, b, out, p, i);
        else
            metal_swiglu_f32(a, b, out, p, i);
    });
}

// encode_channel: 0 add a per-column vector, 1 multiply by it
void mref_channel(int op, const float* in, const float* channel, float* out, uint n_rows, uint cols) {
    MetalBroadcastParams p{};
    p.rows = n_rows;
    p.cols = cols;
    flat((unsigned long long)n_rows * cols, [&](uint i) {
        if (op == 0)
            metal_add_channel_bias_f32(in, channel, out, p, i);
        else
            metal_mul_channel_f32(in, channel, out, p, i);
    });
}

// the DeltaNet causal convolution and its history commit (moe_llm.mm:2501-2531)
void mref_conv1d(const float* in, const float* history, const float* weight, float* out, uint tokens, uint channels,
                 uint kernel_size) {
    MetalDepthwiseConvParams p{};
    p.tokens = tokens;
    p.channels = channels;
    p.kernel_size = kernel_size;
    flat((unsigned long long)tokens * channels,
         [&](uint i) { metal_depthwise_conv1d_causal_f32(in, history, weight, out, p, i); });
}

void mref_conv_commit(const float* in, float* history, uint tokens, uint channels, uint kernel_size) {
    MetalDepthwiseConvParams p{};
    p.tokens = tokens;
    p.channels = channels;
    p.kernel_size = kernel_size;
    flat(channels, [&](uint i) { metal_conv_history_commit_f32(in, history, p, i); });
}

// per-head L2 norm of [tokens][heads * head_dim] views (moe_llm.mm:2545-2568)
void mref_l2norm_heads(const float* in, float* out, uint tokens, uint heads, uint head_dim, uint in_stride,
                       float eps) {
    MetalHeadNormParams p{};
    p.tokens = tokens;
    p.head_count = heads;
    p.head_dim = head_dim;
    p.input_token_stride = in_stride;
    p.epsilon = eps;
    rows((unsigned long long)tokens * heads,
         [&](uint local, uint3 g) { metal_l2norm_heads_f32(in, out, p, local, g); });
}

void mref_gdn(const float* q, const float* k, const float* v, const float* decay, const float* beta, float* state,
              float* out, uint tokens, uint key_heads, uint value_heads, uint head_dim, uint q_stride,
              uint k_stride, uint v_stride, uint out_stride) {
    MetalGdnParams p{};
    p.tokens = tokens;
    p.key_head_count = key_heads;
    p.value_head_count = value_heads;
    p.head_dim = head_dim;
    p.q_stride = q_stride;
    p.k_stride = k_stride;
    p.v_stride = v_stride;
    p.output_stride = out_stride;
    for (uint g = 0; g < value_heads; ++g)
        for (uint t = 0; t < head_dim; ++t)
            metal_gdn_recurrence_f32(q, k, v, decay, beta, state, out, p, t, uint3(g, 0, 0));
}

// routing (moe_llm.mm:2642-2690): top-k per row, then the renormalisation
void mref_topk(const float* in, uint* indices, float* values, uint n_rows, uint cols, uint k) {
    MetalTopKParams p{};
    p.rows = n_rows;
    p.cols = cols;
    p.k = k;
    flat(n_rows, [&](uint i) { metal_topk_f32(in, indices, values, p, i); });
}

void mref_topk_renorm(float* values, uint n_rows, uint k) {
    MetalTopKParams p{};
    p.rows = n_rows;
    p.k = k;
    flat(n_rows, [&](uint i) { metal_topk_renorm_f32(values, p, i); });
}

// routed expert product (moe_llm.mm:2703-2760); type 12 = Q4_K, 14 = Q6_K
int mref_expert(int type, const float* act, const uchar* w, const uint* ids, float* out, uint tokens, uint routes,
                uint out_size, uint in_size, uint act_stride, uint row_bytes, uint expert_stride, uint routed) {
    if (type != 12 && type != 14) return 1;
    MetalExpertProductParams p{};
    p.tokens = tokens;
    p.routes = routes;
    p.output_size = out_size;
    p.input_size = in_size;
    p.activation_stride = act_stride;
    p.weight_row_bytes = row_bytes;
    p.expert_stride_bytes = expert_stride;
    p.activation_is_routed = routed;
    flat((unsigned long long)tokens * routes * out_size, [&](uint i) {
        if (type == 12)
            metal_expert_gemm_q4_k_f32(act, w, ids, out, p, i);
        else
            metal_expert_gemm_q6_k_f32(act, w, ids, out, p, i);
    });
    return 0;
}

void mref_weighted_reduce(const float* in, const float* weights, float* out, uint tokens, uint routes, uint cols) {
    MetalExpertWeightedReduceParams p{};
    p.tokens = tokens;
    p.routes = routes;
    p.cols = cols;
    flat((unsigned long long)tokens * cols, [&](uint i) { metal_expert_weighted_reduce_f32(in, weights, out, p, i); });
}

// gated attention (moe_llm.mm:2238-2434)
void mref_split_q_gate(const float* in, float* q, float* gate, uint n_rows, uint heads, uint head_dim) {
    MetalSplitQGateParams p{};
    p.rows = n_rows;
    p.head_count = heads;
    p.head_dim = head_dim;
    flat((unsigned long long)n_rows * heads * head_dim,
         [&](uint i) { metal_split_interleaved_q_gate_f32(in, q, gate, p, i); });
}

void mref_rope_heads(const float* in, float* out, uint n_rows, uint cols, uint head_dim, uint rot, uint position,
                     float theta) {
    MetalRopeHeadsParams p{};
    p.rows = n_rows;
    p.cols = cols;
    p.head_dim = head_dim;
    p.rotary_dimension = rot;
    p.position = position;
    p.theta = theta;
    flat((unsigned long long)n_rows * cols, [&](uint i) { metal_rope_heads_f32(in, out, p, i); });
}

void mref_kv_write(const float* k, const float* v, float* kc, float* vc, uint n_rows, uint cols, uint stride,
                   uint position) {
    MetalKVCacheWriteParams p{};
    p.source_rows = n_rows;
    p.source_cols = cols;
    p.cache_stride = stride;
    p.position = position;
    flat((unsigned long long)n_rows * cols, [&](uint i) { metal_kv_cache_write_f32(k, v, kc, vc, p, i); });
}

void mref_qk(const float* q, const float* kc, float* out, uint q_rows, uint key_length, uint q_heads, uint kv_heads,
             uint cache_stride, uint q_stride, uint head_dim, uint q_position, float scale) {
    MetalKVCacheQKParams p{};
    p.query_rows = q_rows;
    p.key_length = key_length;
    p.query_heads = q_heads;
    p.kv_heads = kv_heads;
    p.cache_stride = cache_stride;
    p.query_stride = q_stride;
    p.head_dim = head_dim;
    p.query_position = q_position;
    p.scale = scale;
    flat((unsigned long long)q_rows * q_heads * key_length, [&](uint i) { metal_kv_cache_qk_f32(q, kc, out, p, i); });
}

void mref_av(const float* scores, const float* vc, float* out, uint q_rows, uint key_length, uint q_heads,
             uint kv_heads, uint cache_stride, uint score_stride, uint head_dim, uint out_stride) {
    MetalKVCacheAVParams p{};
    p.query_rows = q_rows;
    p.key_length = key_length;
    p.query_heads = q_heads;
    p.kv_heads = kv_heads;
    p.cache_stride = cache_stride;
    p.score_stride = score_stride;
    p.head_dim = head_dim;
    p.output_stride = out_stride;
    flat((unsigned long long)q_rows * q_heads * head_dim, [&](uint i) { metal_kv_cache_av_f32(scores, vc, out, p, i); });
}

// encode_product for one row (moe_llm.mm:1978-2030): one thread per output;
// type 0 = F32 (metal_gevm_f32, row-major weight), else a GGML block type
int mref_gevm(int type, const void* w, const float* x, float* out, uint n, uint k, uint row_bytes) {
    if (type == 0) {
        MetalGemvParams p{};
        p.output_size = n;
        p.input_size = k;
        p.matrix_stride = row_bytes / 4;
        p.matrix_transposed = 1;
        p.has_bias = 0;
        p.scale = 1.0f;
        flat(n, [&](uint i) { metal_gevm_f32(static_cast<const float*>(w), x, nullptr, out, p, i); });
        return 0;
    }
    MetalQuantizedProductParams p{};
    p.m = 1;
    p.n = n;
    p.k = k;
    p.activation_stride = k;
    p.weight_row_bytes = row_bytes;
    p.has_bias = 0;
    p.scale = 1.0f;
    const uchar* q = static_cast<const uchar*>(w);
    switch (type) {
        case 6: flat(n, [&](uint i) { metal_gevm_q5_0_f32(q, x, nullptr, out, p, i); }); return 0;
        case 8: flat(n, [&](uint i) { metal_gevm_q8_0_f32(q, x, nullptr, out, p, i); }); return 0;
        case 12: flat(n, [&](uint i) { metal_gevm_q4_k_f32(q, x, nullptr, out, p, i); }); return 0;
        case 13: flat(n, [&](uint i) { metal_gevm_q5_k_f32(q, x, nullptr, out, p, i); }); return 0;
        case 14: flat(n, [&](uint i) { metal_gevm_q6_k_f32(q, x, nullptr, out, p, i); }); return 0;
        default: return 1;
    }
}

// encode_embedding (moe_llm.mm:1951-1976)
int mref_embedding(int type, const int* ids, const void* w, float* out, uint n_rows, uint size, uint vocab,
                   uint row_bytes) {
    MetalEmbeddingParams p{};
    p.sequence_length = n_rows;
    p.embedding_size = size;
    p.vocabulary_size = vocab;
    p.weight_row_bytes = row_bytes;
    const uchar* q = static_cast<const uchar*>(w);
    const unsigned long long count = (unsigned long long)n_rows * size;
    switch (type) {
        case 0: flat(count, [&](uint i) { metal_embedding_f32(ids, static_cast<const float*>(w), out, p, i); }); return 0;
        case 6: flat(count, [&](uint i) { metal_embedding_q5_0_f32(ids, q, out, p, i); }); return 0;
        case 8: flat(count, [&](uint i) { metal_embedding_q8_0_f32(ids, q, out, p, i); }); return 0;
        case 12: flat(count, [&](uint i) { metal_embedding_q4_k_f32(ids, q, out, p, i); }); return 0;
        case 14: flat(count, [&](uint i) { metal_embedding_q6_k_f32(ids, q, out, p, i); }); return 0;
        default: return 1;
    }
}

// encode_row_scale (moe_llm.mm:2204-2236): row r times row_weights[r * stride + column]
void mref_row_scale(const float* in, const float* row_weights, float* out, uint n_rows, uint cols, uint stride,
                    uint column) {
    MetalRowScaleParams p{};
    p.rows = n_rows;
    p.cols = cols;
    p.weight_stride = stride;
    p.weight_column = column;
    flat((unsigned long long)n_rows * cols, [&](uint i) { metal_row_scale_selected_f32(in, row_weights, out, p, i); });
}

// encode_binary with the residual kernel: a + b
void mref_residual(const float* a, const float* b, float* out, uint n) {
    MetalElementwiseParams p{};
    p.rows = 1;
    p.cols = n;
    flat(n, [&](uint i) { metal_residual_f32(a, b, out, p, i); });
}

}  // extern "C"
