// CudaLLM: the qwen2 decode/prefill graph on one or more B200s.
//
// Graph order follows cpu_prefill_layer / cpu_decode_layer (cpu_llm.cpp:
// 774-914) and encode_{prefill,decode}_layer (metal_llm.mm:2619-2904):
//   h = embed(ids)
//   per layer: a = rmsnorm(h); q,k,v = a W^T + b; rope(q,k); cache k,v;
//              o = attention; h += o Wo^T; f = rmsnorm(h);
//              h += (silu(f Wg^T) * f Wu^T) Wd^T
//   logits = rmsnorm(h_last) Wout^T; token = argmax (lowest index on ties).
// Decode is one CUDA graph per step (captured once, replayed); the only host
// synchronisation is the 4-byte token read-back.
#include "cuda_llm.h"

#include <nccl.h>

#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <stdexcept>

#include "device.h"
#include "gguf.h"
#include "profile.h"

namespace cudallm {

namespace {

#define CUDALLM_NCCL(expr)                                                                    \
    do {                                                                                      \
        ncclResult_t r_ = (expr);                                                             \
        if (r_ != ncclSuccess)                                                                \
            throw std::runtime_error(std::string("NCCL error ") + ncclGetErrorString(r_) +    \
                                     " in " #expr);                                           \
    } while (0)

ModelConfig read_qwen2_config(const GgufFile& f) {
    ModelConfig c;
    c.architecture = f.text("general.architecture");
    if (c.architecture != "qwen2") {
        throw std::runtime_error("CudaLLM supports qwen2 GGUF models, got " + c.architecture);
    }
    c.tensor_count = f.tensors().size();
    c.layer_count = f.size("qwen2.block_count");
    c.embedding_size = f.size("qwen2.embedding_length");
    c.feed_forward_size = f.size("qwen2.feed_forward_length");
    c.attention_head_count = f.size("qwen2.attention.head_count");
    c.kv_head_count = f.size("qwen2.attention.head_count_kv");
    c.context_length = f.size("qwen2.context_length");
    c.vocabulary_size = f.array_length("tokenizer.ggml.tokens");
    if (c.vocabulary_size == 0) c.vocabulary_size = f.size("tokenizer.ggml.tokens_count");
    c.vocabulary = f.strings("tokenizer.ggml.tokens");
    c.merges = f.strings("tokenizer.ggml.merges");
    c.tokenizer_pre = f.text("tokenizer.ggml.pre");
    if (c.embedding_size % c.attention_head_count != 0)
        throw std::runtime_error("embedding size must be divisible by attention head count");
    if (c.attention_head_count % c.kv_head_count != 0)
        throw std::runtime_error("attention head count must be divisible by KV head count");
    c.head_size = c.embedding_size / c.attention_head_count;
    c.rotary_dimension = c.head_size;
    c.rope_theta = (float)f.real("qwen2.rope.freq_base", 1000000.0);
    c.norm_epsilon = (float)f.real("qwen2.attention.layer_norm_rms_epsilon", 1e-6);
    if (!std::isfinite(c.rope_theta) || c.rope_theta <= 0.0f)
        throw std::runtime_error("RoPE theta must be finite and positive");
    if (!std::isfinite(c.norm_epsilon) || c.norm_epsilon <= 0.0f)
        throw std::runtime_error("RMSNorm epsilon must be finite and positive");
    const uint64_t eos = f.integer("tokenizer.ggml.eos_token_id", 151645);
    if (eos > (uint64_t)INT32_MAX) throw std::runtime_error("EOS token id does not fit in int32_t");
    c.eos_token_id = (int32_t)eos;
    for (const TensorInfo& t : f.tensors()) {
        c.parameter_count += t.rows * t.cols;
        c.stored_weight_bytes += t.bytes;
    }
    return c;
}

// cos/sin of NeoX RoPE for every position, computed on the host with the
// CPU path's float expressions (cpu_llm.cpp:220-227) so that the rotation
// inputs match it exactly.
std::vector<float> rope_table(std::size_t positions, std::size_t rot, float theta) {
    const std::size_t half = rot / 2;
    std::vector<float> freq(half);
    for (std::size_t p = 0; p < half; ++p)
        freq[p] = std::pow(theta, -2.0f * static_cast<float>(p) / static_cast<float>(rot));
    std::vector<float> t(positions * half * 2);
    for (std::size_t pos = 0; pos < positions; ++pos) {
        for (std::size_t p = 0; p < half; ++p) {
            const float angle = static_cast<float>(pos) * freq[p];
            t[(pos * half + p) * 2] = std::cos(angle);
            t[(pos * half + p) * 2 + 1] = std::sin(angle);
        }
    }
    return t;
}

struct Layer {
    const float* attn_norm = nullptr;
    DevMat q, k, v, o;
    const float *q_b = nullptr, *k_b = nullptr, *v_b = nullptr;
    const float* ffn_norm = nullptr;
    DevMat gate, up, down;
    float* k_cache = nullptr;
    float* v_cache = nullptr;
    // 16-bit prefill copies (row-major [rows][cols]): Q|K|V rows, o, gate|up rows, down
    void *qkv16 = nullptr, *o16 = nullptr, *gu16 = nullptr, *down16 = nullptr;
    // split form: device maxima of q, k, v, o, gate, up, down (the scales of their 16-bit copies)
    float* wmax = nullptr;
};

// Contiguous, block-aligned share [begin, end) of `n` units for one rank.
std::pair<std::size_t, std::size_t> split_range(std::size_t n, int world, int rank) {
    const std::size_t base = n / world, extra = n % world;
    const std::size_t begin = rank * base + std::min<std::size_t>(rank, extra);
    return {begin, begin + base + ((std::size_t)rank < extra ? 1 : 0)};
}

std::size_t block_cols(int type) {
    return (type == kQ4_K || type == kQ5_K || type == kQ6_K) ? 256 : (type == kQ5_0 || type == kQ8_0) ? 32 : 1;
}

}  // namespace

TensorParallelShard plan_tensor_parallel(std::size_t F, std::size_t V, std::size_t hq, std::size_t hkv, std::size_t d,
                                         std::size_t o_block, int W, int R) {
    if (W < 1 || R < 0 || R >= W) throw std::invalid_argument("invalid parallel rank/world");
    if (hq == 0 || hkv == 0 || hkv % W != 0 || hq % W != 0)
        throw std::invalid_argument("tensor-parallel world must divide the query and KV head counts");
    if (o_block == 0 || (hq * d) % o_block != 0)
        throw std::invalid_argument("attention output width is not a multiple of the o_proj block");
    TensorParallelShard s;
    s.q_heads = hq / W;
    s.q_head0 = R * s.q_heads;
    s.kv_heads = hkv / W;
    s.kv_head0 = R * s.kv_heads;
    s.ffn_rows = F;
    s.o_cols = hq * d;
    s.vocab_rows = V;
    if (W == 1) return s;
    // FFN rows split on the widest block grid both formats share.
    const std::size_t blk = 256;
    if (F % blk) throw std::invalid_argument("FFN width must be a multiple of 256 for tensor parallelism");
    auto fr = split_range(F / blk, W, R);
    s.ffn0 = fr.first * blk;
    s.ffn_rows = (fr.second - fr.first) * blk;
    // o_proj input columns: the local heads when they are block aligned,
    // otherwise a block-aligned share of the all-gathered output.
    const std::size_t heads_cols = s.q_heads * d;
    if (heads_cols % o_block == 0) {
        s.o_col0 = R * heads_cols;
        s.o_cols = heads_cols;
    } else {
        s.gather_attn = true;
        auto orng = split_range(hq * d / o_block, W, R);
        s.o_col0 = orng.first * o_block;
        s.o_cols = (orng.second - orng.first) * o_block;
    }
    auto vr = split_range(V, W, R);
    s.vocab0 = vr.first;
    s.vocab_rows = vr.second - vr.first;
    return s;
}

struct CudaLLM::Impl {
    ModelConfig config;
    ParallelConfig par;
    int device = 0;
    std::string device_name;
    cudaStream_t stream = nullptr;
    ncclComm_t comm = nullptr;

    // shard geometry (world == 1: everything full)
    std::size_t H = 0, F = 0, V = 0, d = 0, hq = 0, hkv = 0;
    std::size_t hq_l = 0, hkv_l = 0;      // local heads
    std::size_t ffn0 = 0, F_l = 0;        // local FFN rows [ffn0, ffn0 + F_l)
    std::size_t vocab0 = 0, V_l = 0;      // local LM-head rows
    std::size_t o_k0 = 0, o_kl = 0;       // local o_proj input columns
    bool gather_attn = false;             // o_proj K shard is not the local heads

    std::size_t max_seq = 0;
    std::size_t prefill_chunk = 0;
    std::size_t position = 0;

    DeviceBuffer weight_mem, state_mem, act_mem;
    std::uint64_t weight_payload = 0, kv_bytes = 0, act_bytes = 0;

    DevMat tok_embd, out_w;
    const float* out_norm = nullptr;
    std::vector<Layer> layers;
    const float* rope = nullptr;

    // decode activations
    float *h = nullptr, *part = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *att = nullptr,
          *att_full = nullptr, *act = nullptr, *logits = nullptr;
    void *attn_ws = nullptr, *arg_ws = nullptr;
    std::size_t attn_ws_bytes = 0, arg_ws_bytes = 0;
    int32_t* ints = nullptr;  // [0] token in, [1] pos, [2] len, [3] token out, [4..] scratch
    float* best = nullptr;    // TP argmax records [world][2]
    // prefill activations
    float *X = nullptr, *Xn = nullptr, *Q = nullptr, *K = nullptr, *Vv = nullptr, *A = nullptr,
          *A_full = nullptr, *G = nullptr, *U = nullptr, *P = nullptr;
    int32_t* ids_dev = nullptr;

    PinnedBuffer host_io;  // [0] token in, [1] token out, [2] exchange status, [4..] ids staging

    // Decode all-reduce through peer memory (CUDALLM_ALLREDUCE=p2p): this
    // rank's exchange buffer and every rank's buffer as mapped here.
    DeviceBuffer peer_buf;
    std::vector<void*> peer_bufs;
    bool peer_allreduce = false;
    cudaGraphExec_t decode_exec = nullptr;
    // One-GPU decode as one persistent launch (cl_qwen2_decode_step) where
    // the model's shapes and types allow it; CUDALLM_DECODE=graph selects the
    // per-operator graph instead.
    bool fused = false;
    cl_qwen2_decode fused_desc{};
    std::vector<cl_qwen2_layer> fused_layers;
    cl_qwen2_layer* fused_layers_dev = nullptr;
    void* fused_ws = nullptr;
    std::size_t fused_ws_bytes = 0;
    // CUDALLM_DECODE_TRACE=<file>: every fused step's per-CTA, per-phase
    // timestamps (int64 [grid][phases][3]) overwrite <file> after the step
    DeviceBuffer trace_mem;
    std::string trace_path;
    DeviceBuffer pack_mem;  // every layer matrix and the LM head in the tiled decode layout
    // Decode GEMVs over fragment-packed copies (cl_gemv_packed), which stream
    // a large matrix faster than the shared-memory ring kernels but carry a
    // larger fixed cost per launch (measured on B200: the 7B LM head 87 vs
    // 111 us; a 7B layer's QKV, o_proj, gate/up and down all slower).  So by
    // default only the LM head is packed; CUDALLM_DECODE_GEMV=packed packs
    // every decode matrix, =ring none.  Q4_K / Q6_K on the 256-column grid.
    struct PackedLayer {
        const void *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr, *gate = nullptr, *down = nullptr;
    };
    bool packed_layers = false;
    std::vector<PackedLayer> pk_layers;
    const void* pk_head = nullptr;
    DeviceBuffer pk_mem, pk_ws;  // packed matrices, GEMV workspace
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    cudaEvent_t kev0 = nullptr, kev1 = nullptr;  // around the fused step kernel
    float last_ms = 0.0f, last_kernel_ms = 0.0f;
    std::unique_ptr<ProfileCsv> profile;
    std::chrono::steady_clock::time_point call_start;
    bool have_logits = false;

    ~Impl() {
        // the mappings belong to this model's device, which another model of
        // the same process may not have left current
        if (!peer_bufs.empty()) cudaSetDevice(device);
        for (std::size_t r = 0; r < peer_bufs.size(); ++r)
            if ((int)r != par.rank && peer_bufs[r]) cudaIpcCloseMemHandle(peer_bufs[r]);
        if (decode_exec) cudaGraphExecDestroy(decode_exec);
        if (comm) ncclCommDestroy(comm);
        if (ev0) cudaEventDestroy(ev0);
        if (ev1) cudaEventDestroy(ev1);
        if (kev0) cudaEventDestroy(kev0);
        if (kev1) cudaEventDestroy(kev1);
        if (stream) cudaStreamDestroy(stream);
    }

    // o_block: the widest column block among the layers' attn_output types.
    void plan_shards(std::size_t o_block) {
        H = config.embedding_size;
        F = config.feed_forward_size;
        V = config.vocabulary_size;
        d = config.head_size;
        hq = config.attention_head_count;
        hkv = config.kv_head_count;
        const TensorParallelShard sh = plan_tensor_parallel(F, V, hq, hkv, d, o_block, par.world, par.rank);
        hq_l = sh.q_heads;
        hkv_l = sh.kv_heads;
        ffn0 = sh.ffn0;
        F_l = sh.ffn_rows;
        o_k0 = sh.o_col0;
        o_kl = sh.o_cols;
        gather_attn = sh.gather_attn;
        vocab0 = sh.vocab0;
        V_l = sh.vocab_rows;
    }

    // Planning pass (arena base null) then the real pass with the same calls.
    void load_weights(GgufFile& file, Arena& arena, bool real) {
        WeightLoader wl(file, arena, stream);
        const std::size_t kvd = hkv * d;
        tok_embd = wl.matrix("token_embd.weight", V, H);
        out_norm = wl.vector("output_norm.weight", H);
        out_w = wl.matrix("output.weight", V, H, vocab0, vocab0 + V_l);
        layers.assign(config.layer_count, Layer{});
        for (std::size_t l = 0; l < config.layer_count; ++l) {
            const std::string p = "blk." + std::to_string(l) + ".";
            Layer& L = layers[l];
            const std::size_t q0 = par.rank * hq_l * d, qn = hq_l * d;
            const std::size_t k0 = par.rank * hkv_l * d, kn = hkv_l * d;
            L.attn_norm = wl.vector(p + "attn_norm.weight", H);
            L.q = wl.matrix(p + "attn_q.weight", H, H, q0, q0 + qn);
            L.q_b = wl.vector(p + "attn_q.bias", H, q0, q0 + qn);
            L.k = wl.matrix(p + "attn_k.weight", kvd, H, k0, k0 + kn);
            L.k_b = wl.vector(p + "attn_k.bias", kvd, k0, k0 + kn);
            L.v = wl.matrix(p + "attn_v.weight", kvd, H, k0, k0 + kn);
            L.v_b = wl.vector(p + "attn_v.bias", kvd, k0, k0 + kn);
            // a rank whose share of a row-split matrix is empty (fewer blocks
            // than ranks) loads nothing and contributes zeros to the all-reduce
            if (o_kl > 0)
                L.o = wl.matrix(p + "attn_output.weight", H, H, 0, H, o_k0, o_k0 + o_kl);
            else
                file.mark_loaded(p + "attn_output.weight");
            L.ffn_norm = wl.vector(p + "ffn_norm.weight", H);
            if (F_l > 0) {
                L.gate = wl.matrix(p + "ffn_gate.weight", F, H, ffn0, ffn0 + F_l);
                L.up = wl.matrix(p + "ffn_up.weight", F, H, ffn0, ffn0 + F_l);
                L.down = wl.matrix(p + "ffn_down.weight", H, F, 0, H, ffn0, ffn0 + F_l);
            } else {
                file.mark_loaded(p + "ffn_gate.weight");
                file.mark_loaded(p + "ffn_up.weight");
                file.mark_loaded(p + "ffn_down.weight");
            }
            if (L.gate.type != L.up.type) throw std::runtime_error("ffn_gate and ffn_up must share a type");
        }
        file.validate_all_loaded();
        if (real) wl.finish();
        weight_payload = wl.payload_bytes();
    }

    void allocate_state(Arena& a) {
        const std::size_t kvd_l = hkv_l * d;
        for (Layer& L : layers) {
            L.k_cache = a.take_n<float>(max_seq * kvd_l);
            L.v_cache = a.take_n<float>(max_seq * kvd_l);
        }
        rope = a.take_n<float>(max_seq * (config.rotary_dimension / 2) * 2);
    }

    void allocate_activations(Arena& a) {
        const std::size_t qd_l = hq_l * d, kvd_l = hkv_l * d, chunk = prefill_chunk;
        h = a.take_n<float>(H);
        part = a.take_n<float>(H);
        q = a.take_n<float>(qd_l);
        k = a.take_n<float>(kvd_l);
        v = a.take_n<float>(kvd_l);
        att = a.take_n<float>(qd_l);
        att_full = a.take_n<float>(hq * d);
        act = a.take_n<float>(F_l);
        logits = a.take_n<float>(V_l);
        attn_ws_bytes = cl_attn_decode_workspace_bytes((int)hq_l, (int)d, (int)max_seq);
        attn_ws = a.take(attn_ws_bytes);
        arg_ws_bytes = cl_argmax_workspace_bytes((int)V_l);
        arg_ws = a.take(arg_ws_bytes);
        ints = a.take_n<int32_t>(16);
        best = a.take_n<float>(2 * (std::size_t)par.world + 2);
        X = a.take_n<float>(chunk * H);
        Xn = a.take_n<float>(chunk * H);
        Q = a.take_n<float>(chunk * qd_l);
        K = a.take_n<float>(chunk * kvd_l);
        Vv = a.take_n<float>(chunk * kvd_l);
        A = a.take_n<float>(chunk * qd_l);
        A_full = a.take_n<float>(gather_attn ? chunk * hq * d : 1);
        G = a.take_n<float>(chunk * F_l);
        U = a.take_n<float>(chunk * F_l);
        P = a.take_n<float>(chunk * H);
        ids_dev = a.take_n<int32_t>(chunk);
        if (par.world == 1) {
            fill_fused_desc();
            fused_layers_dev = a.take_n<cl_qwen2_layer>(layers.size());
            fused_ws_bytes = cl_qwen2_decode_workspace_bytes(&fused_desc);
            fused_ws = fused_ws_bytes ? a.take(fused_ws_bytes) : nullptr;
        }
    }

    // The fused step's description of this model (pointers valid once the
    // arenas are bound).
    void fill_fused_desc() {
        cl_qwen2_decode& m = fused_desc;
        m = cl_qwen2_decode{};
        m.layers = fused_layers_dev;
        m.n_layers = (int)layers.size();
        m.hidden = (int)H;
        m.ffn = (int)F;
        m.vocab = (int)V;
        m.q_heads = (int)hq;
        m.kv_heads = (int)hkv;
        m.head_dim = (int)d;
        m.capacity = (int)max_seq;
        m.eps = eps();
        m.scale = 1.0f / std::sqrt(static_cast<float>(d));
        m.embd = tok_embd.ptr;
        m.embd_stride = tok_embd.stride;
        m.embd_type = tok_embd.type;
        m.out_w = out_w.ptr;
        m.out_type = out_w.type;
        m.out_norm = out_norm;
        m.rope = rope;
        m.ints = ints;
        m.h = h;
        m.q = q;
        m.k = k;
        m.v = v;
        m.att = att;
        m.act = act;
        m.logits = logits;
        fused_layers.assign(layers.size(), cl_qwen2_layer{});
        for (std::size_t l = 0; l < layers.size(); ++l) {
            const Layer& L = layers[l];
            cl_qwen2_layer& f = fused_layers[l];
            f.q = L.q.ptr;
            f.k = L.k.ptr;
            f.v = L.v.ptr;
            f.o = L.o.ptr;
            f.gate = L.gate.ptr;
            f.up = L.up.ptr;
            f.down = L.down.ptr;
            f.q_bias = L.q_b;
            f.k_bias = L.k_b;
            f.v_bias = L.v_b;
            f.attn_norm = L.attn_norm;
            f.ffn_norm = L.ffn_norm;
            f.k_cache = L.k_cache;
            f.v_cache = L.v_cache;
            f.q_type = L.q.type;
            f.k_type = L.k.type;
            f.v_type = L.v.type;
            f.o_type = L.o.type;
            f.gate_type = L.gate.type;
            f.down_type = L.down.type;
        }
    }

    // Resident 16-bit copies of every layer matrix for the prefill GEMMs, each
    // element the CPU decoder's FP32 value rounded once (cl_dequant16); the
    // activations are rounded into x16 per product.  Matrices whose inner
    // size the 16-bit GEMM does not take keep the native-block path.
    static bool gemm16_ok(std::size_t kdim) { return kdim > 0 && kdim % 64 == 0; }

    void setup_wide16() {
        const std::size_t kmax = std::max<std::size_t>(std::max<std::size_t>(H, F_l), std::max<std::size_t>(o_kl, 1));
        const std::size_t eb = split16() ? 4 : 2;  // bytes per element: the split form keeps hi and lo
        std::size_t bytes = 0;
        auto plan = [&](std::size_t rows, std::size_t cols) {
            const std::size_t b = (rows * cols * eb + 255) / 256 * 256;
            bytes += b;
            return b;
        };
        for (Layer& L : layers) {
            if (gemm16_ok(H)) plan((std::size_t)L.q.rows + L.k.rows + L.v.rows, H);
            if (o_kl > 0 && gemm16_ok(o_kl)) plan(H, o_kl);
            if (F_l > 0 && gemm16_ok(H)) plan(2 * F_l, H);
            if (F_l > 0 && gemm16_ok(F_l)) plan(H, F_l);
        }
        w16_mem = DeviceBuffer(bytes + (prefill_chunk * kmax * eb + 255) / 256 * 256 + 256);
        amax_mem = DeviceBuffer((layers.size() * 7 + 1) * sizeof(float));
        xmax = static_cast<float*>(amax_mem.get()) + layers.size() * 7;
        char* base = static_cast<char*>(w16_mem.get());
        const int fmt = fmt16();
        float* wm = nullptr;
        auto dq = [&](const DevMat& m, char* dst) {
            if (split16()) {
                CUDALLM_CL(cl_amax_dequant(m.type, m.ptr, m.stride, m.rows, m.cols, wm, stream));
                CUDALLM_CL(cl_dequant16_split(m.type, m.ptr, m.stride, m.rows, m.cols, wm, dst, stream));
            } else {
                CUDALLM_CL(cl_dequant16(m.type, m.ptr, m.stride, m.rows, m.cols, dst, fmt, stream));
            }
            ++wm;
        };
        for (std::size_t l = 0; l < layers.size(); ++l) {
            Layer& L = layers[l];
            L.wmax = static_cast<float*>(amax_mem.get()) + 7 * l;
            wm = L.wmax;
            if (gemm16_ok(H)) {
                L.qkv16 = base;
                dq(L.q, base);
                dq(L.k, base + (std::size_t)L.q.rows * H * eb);
                dq(L.v, base + ((std::size_t)L.q.rows + L.k.rows) * H * eb);
                base += (((std::size_t)L.q.rows + L.k.rows + L.v.rows) * H * eb + 255) / 256 * 256;
            }
            wm = L.wmax + 3;
            if (o_kl > 0 && gemm16_ok(o_kl)) {
                L.o16 = base;
                dq(L.o, base);
                base += (H * o_kl * eb + 255) / 256 * 256;
            }
            wm = L.wmax + 4;
            if (F_l > 0 && gemm16_ok(H)) {
                L.gu16 = base;
                dq(L.gate, base);
                dq(L.up, base + F_l * H * eb);
                base += (2 * F_l * H * eb + 255) / 256 * 256;
            }
            wm = L.wmax + 6;
            if (F_l > 0 && gemm16_ok(F_l)) {
                L.down16 = base;
                dq(L.down, base);
                base += (H * F_l * eb + 255) / 256 * 256;
            }
        }
        x16 = base;
        // K-split partials of the 16-bit GEMM (a product runs unsplit when they do not fit)
        g16_ws_mem = DeviceBuffer((std::size_t)64 << 20);
    }

    // One output column range of a 16-bit product (the split form names the scales).
    cl_gemm_out out16(float* y, const float* bias, const float* res, int col0, int cols, int ld,
                      const float* wm) const {
        cl_gemm_out o{};
        o.y = y;
        o.bias = bias;
        o.residual = res;
        o.col0 = col0;
        o.cols = cols;
        o.ld = ld;
        if (split16()) {
            o.xmax = xmax;
            o.wmax = wm;
        }
        return o;
    }

    // Y column ranges = X[m, kdim] W16^T on the 16-bit path.
    void gemm16(const void* w16, int n, int kdim, const float* x, int m, const cl_gemm_out* outs, int nout) {
        if (split16()) {
            CUDALLM_CL(cl_amax(x, (long long)m * kdim, xmax, stream));
            CUDALLM_CL(cl_split16(x, m, kdim, xmax, x16, stream));
        } else {
            CUDALLM_CL(cl_convert16(x, (long long)m * kdim, x16, fmt16(), stream));
        }
        CUDALLM_CL(cl_gemm16_run(w16, n, kdim, x16, m, outs, nout, fmt16(), g16_ws_mem.get(), g16_ws_mem.size(),
                                 stream));
    }

    // Pack the decode matrices for cl_gemv_packed (see `packed_layers`).
    void setup_packed() {
        std::string mode = "head";
        if (const char* e = std::getenv("CUDALLM_DECODE_GEMV")) mode = e;
        if (mode != "head" && mode != "packed" && mode != "ring")
            throw std::invalid_argument("CUDALLM_DECODE_GEMV must be head, packed or ring");
        if (mode == "ring" || fused) return;
        auto ok = [](const DevMat& m, std::size_t kdim) {
            return (m.type == kQ4_K || m.type == kQ6_K) && kdim % 256 == 0 && kdim <= 21504 && m.ptr != nullptr;
        };
        const bool layers_too = mode == "packed";
        bool all = ok(out_w, H);
        if (layers_too) {
            all = all && o_kl > 0 && F_l > 0;
            for (const Layer& L : layers)
                all = all && ok(L.q, H) && ok(L.k, H) && ok(L.v, H) && ok(L.o, o_kl) && ok(L.gate, H) &&
                      L.up.type == L.gate.type && ok(L.down, F_l);
        }
        if (!all) {
            if (layers_too)
                throw std::runtime_error("CUDALLM_DECODE_GEMV=packed: a decode matrix is not Q4_K / Q6_K on the "
                                         "256-column grid");
            return;  // the head stays on the ring kernels
        }
        auto bytes = [](const DevMat& m, std::size_t kdim, bool pair) {
            return (cl_gemv_pack_bytes(m.type, m.rows, (int)kdim, pair ? 1 : 0) + 255) / 256 * 256;
        };
        std::size_t total = bytes(out_w, H, false);
        if (layers_too)
            for (const Layer& L : layers)
                total += bytes(L.q, H, false) + bytes(L.k, H, false) + bytes(L.v, H, false) +
                         bytes(L.o, o_kl, false) + bytes(L.gate, H, true) + bytes(L.down, F_l, false);
        pk_mem = DeviceBuffer(total + 256);
        char* base = static_cast<char*>(pk_mem.get());
        auto pack = [&](const DevMat& m, std::size_t kdim, const DevMat* up) -> const void* {
            char* dst = base;
            CUDALLM_CL(cl_gemv_pack(m.type, m.ptr, m.stride, m.rows, (int)kdim, up ? up->ptr : nullptr, dst, stream));
            base += bytes(m, kdim, up != nullptr);
            return dst;
        };
        pk_head = pack(out_w, H, nullptr);
        std::size_t tiles = (V_l + 15) / 16;
        if (layers_too) {
            pk_layers.resize(layers.size());
            for (std::size_t l = 0; l < layers.size(); ++l) {
                const Layer& L = layers[l];
                PackedLayer& P = pk_layers[l];
                P.q = pack(L.q, H, nullptr);
                P.k = pack(L.k, H, nullptr);
                P.v = pack(L.v, H, nullptr);
                P.o = pack(L.o, o_kl, nullptr);
                P.gate = pack(L.gate, H, &L.up);
                P.down = pack(L.down, F_l, nullptr);
            }
            // the widest launch: the LM head, QKV, gate/up pairs or o / down
            tiles = std::max<std::size_t>(tiles, (F_l + 7) / 8);
            tiles = std::max<std::size_t>(tiles, (hq_l * d + 15) / 16 + 2 * ((hkv_l * d + 15) / 16));
            tiles = std::max<std::size_t>(tiles, (H + 15) / 16);
            packed_layers = true;
        }
        const std::size_t wsb = cl_gemv_packed_workspace_bytes((int)tiles);
        if (wsb == 0) throw std::runtime_error("cl_gemv_packed_workspace_bytes failed");
        pk_ws = DeviceBuffer(wsb);
        CUDALLM_CUDA(cudaMemsetAsync(pk_ws.get(), 0, pk_ws.size(), stream));
    }

    // Decode path: "graph" (default: the per-operator kernels in one CUDA
    // graph per step, measured faster on the 7B) or "fused" (the one-launch
    // step, cl_qwen2_decode_step; construction fails if the model does not
    // qualify).
    void setup_fused() {
        if (par.world != 1 || fused_ws == nullptr) return;
        std::string mode;
        if (const char* e = std::getenv("CUDALLM_DECODE")) mode = e;
        if (mode != "" && mode != "fused" && mode != "graph")
            throw std::invalid_argument("CUDALLM_DECODE must be fused or graph");
        if (mode != "fused") return;
        fill_fused_desc();
        const int rc = cl_qwen2_decode_supported(&fused_desc, fused_layers.data());
        if (rc != CL_OK) {
            if (mode == "fused") throw std::runtime_error(std::string("fused decode: ") + cl_status_string(rc));
            return;
        }
        // the step streams each matrix from its tiled copy (cl_decode_pack)
        {
            auto bytes = [](const DevMat& m, bool pair) {
                return (cl_decode_pack_bytes(m.type, m.rows, m.cols, pair ? 1 : 0) + 255) / 256 * 256;
            };
            std::size_t total = bytes(out_w, false);
            for (const Layer& L : layers)
                total += bytes(L.q, false) + bytes(L.k, false) + bytes(L.v, false) + bytes(L.o, false) +
                         bytes(L.gate, true) + bytes(L.down, false);
            pack_mem = DeviceBuffer(total + 256);
            char* base = static_cast<char*>(pack_mem.get());
            auto pack = [&](const DevMat& m, const DevMat* up) -> const void* {
                char* dst = base;
                CUDALLM_CL(cl_decode_pack(m.type, m.ptr, m.stride, m.rows, m.cols, up ? up->ptr : nullptr, dst, stream));
                base += bytes(m, up != nullptr);
                return dst;
            };
            fused_desc.out_w = pack(out_w, nullptr);
            for (std::size_t l = 0; l < layers.size(); ++l) {
                const Layer& L = layers[l];
                cl_qwen2_layer& f = fused_layers[l];
                f.q = pack(L.q, nullptr);
                f.k = pack(L.k, nullptr);
                f.v = pack(L.v, nullptr);
                f.o = pack(L.o, nullptr);
                f.gate = pack(L.gate, &L.up);
                f.up = nullptr;
                f.down = pack(L.down, nullptr);
            }
            CUDALLM_CL(cl_qwen2_decode_supported(&fused_desc, fused_layers.data()));
        }
        if (const char* e = std::getenv("CUDALLM_DECODE_SPLITS")) {
            // attention key splits per KV head (tests use few, to cover multi-tile splits)
            fused_desc.attn_splits = std::atoi(e);
            CUDALLM_CL(cl_qwen2_decode_supported(&fused_desc, fused_layers.data()));
        }
        if (const char* e = std::getenv("CUDALLM_DECODE_TRACE")) {
            int sms = 0;
            CUDALLM_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
            trace_path = e;
            trace_mem = DeviceBuffer((std::size_t)sms * (5 * layers.size() + 1) * 16 * sizeof(long long));
            CUDALLM_CUDA(cudaMemsetAsync(trace_mem.get(), 0, trace_mem.size(), stream));
            fused_desc.trace = static_cast<long long*>(trace_mem.get());
        }
        CUDALLM_CUDA(cudaMemcpyAsync(fused_layers_dev, fused_layers.data(),
                                     fused_layers.size() * sizeof(cl_qwen2_layer), cudaMemcpyHostToDevice, stream));
        CUDALLM_CL(cl_qwen2_decode_init(fused_ws, fused_ws_bytes, stream));
        fused = true;
    }

    void init(const std::string& path, std::size_t max_sequence, int dev, const ParallelConfig& parallel) {
        par = parallel;
        if (dev < 0) CUDALLM_CUDA(cudaGetDevice(&dev));
        device = dev;
        CUDALLM_CUDA(cudaSetDevice(device));
        cudaDeviceProp prop{};
        CUDALLM_CUDA(cudaGetDeviceProperties(&prop, device));
        device_name = prop.name;
        CUDALLM_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
        CUDALLM_CUDA(cudaEventCreate(&ev0));
        CUDALLM_CUDA(cudaEventCreate(&ev1));
        CUDALLM_CUDA(cudaEventCreate(&kev0));
        CUDALLM_CUDA(cudaEventCreate(&kev1));

        GgufFile file(path);
        config = read_qwen2_config(file);
        if (max_sequence == 0) max_sequence = config.context_length;
        if (max_sequence == 0 || max_sequence > config.context_length)
            throw std::invalid_argument("CUDA maximum sequence must be within the model context length");
        max_seq = max_sequence;
        prefill_chunk = std::min<std::size_t>(max_seq, 1024);
        // Diagnostics: a smaller prefill chunk exercises the cross-chunk KV path.
        if (const char* e = std::getenv("CUDALLM_PREFILL_CHUNK")) {
            const long val = std::strtol(e, nullptr, 10);
            if (val > 0) prefill_chunk = std::min<std::size_t>(max_seq, (std::size_t)val);
        }
        // Prefill GEMM: "fp16x3" (default: resident split FP16 copies, three
        // tcgen05 MMAs per step, FP32-grade like the reference's FP32 GEMM),
        // "fp16" / "bf16" (one 16-bit pass), "tf32x3" (split TF32 over the
        // native blocks, FP32-grade), "f16" (one FP16 pass over the native
        // blocks) or "simt" (FP32 CUDA cores).
        if (const char* e = std::getenv("CUDALLM_PREFILL_ATTN")) {
            const std::string v(e);
            if (v == "fp32") prefill_attn = PrefillAttn::Fp32;
            else if (v == "fp16") prefill_attn = PrefillAttn::Tc;
            else if (v == "fp16x3") prefill_attn = PrefillAttn::Tc3;
            else if (!v.empty()) throw std::invalid_argument("CUDALLM_PREFILL_ATTN must be fp32, fp16 or fp16x3");
        }
        if (const char* e = std::getenv("CUDALLM_PREFILL_GEMM")) {
            const std::string val(e);
            if (val == "fp16")
                gemm_path = GemmPath::Fp16;
            else if (val == "f16")
                gemm_path = GemmPath::F16;
            else if (val == "simt")
                gemm_path = GemmPath::Simt;
            else if (val == "tf32x3")
                gemm_path = GemmPath::Auto;
            else if (val == "bf16")
                gemm_path = GemmPath::Bf16;
            else if (val != "fp16x3" && !val.empty())
                throw std::invalid_argument("CUDALLM_PREFILL_GEMM must be fp16x3, fp16, bf16, tf32x3, f16 or simt");
        }
        std::size_t o_block = 1;
        for (std::size_t l = 0; l < config.layer_count; ++l) {
            const std::string name = "blk." + std::to_string(l) + ".attn_output.weight";
            if (file.has_tensor(name)) o_block = std::max(o_block, block_cols((int)file.require(name).type));
        }
        plan_shards(o_block);

        if (par.world > 1) {
            ncclUniqueId id;
            std::memcpy(&id, par.nccl_id.data(), sizeof(id));
            CUDALLM_NCCL(ncclCommInitRank(&comm, par.world, id, par.rank));
            // decode all-reduce: "nccl" (default) or "p2p" (cl_peer_allreduce)
            if (const char* e = std::getenv("CUDALLM_ALLREDUCE")) {
                const std::string val(e);
                if (val == "p2p")
                    setup_peer_exchange();
                else if (val != "nccl" && !val.empty())
                    throw std::invalid_argument("CUDALLM_ALLREDUCE must be nccl or p2p");
            }
        }

        Arena plan;
        load_weights(file, plan, false);
        weight_mem = DeviceBuffer(plan.used() + 256);
        Arena wa;
        wa.bind(weight_mem.get(), weight_mem.size());
        GgufFile file2(path);
        load_weights(file2, wa, true);

        Arena sp;
        allocate_state(sp);
        state_mem = DeviceBuffer(sp.used() + 256);
        Arena sa;
        sa.bind(state_mem.get(), state_mem.size());
        allocate_state(sa);
        kv_bytes = (std::uint64_t)layers.size() * 2 * max_seq * hkv_l * d * sizeof(float);

        Arena ap;
        allocate_activations(ap);
        act_mem = DeviceBuffer(ap.used() + 256);
        Arena aa;
        aa.bind(act_mem.get(), act_mem.size());
        allocate_activations(aa);
        act_bytes = ap.used();
        CUDALLM_CUDA(cudaMemsetAsync(act_mem.get(), 0, act_mem.size(), stream));

        const std::vector<float> table = rope_table(max_seq, config.rotary_dimension, config.rope_theta);
        CUDALLM_CUDA(cudaMemcpyAsync(const_cast<float*>(rope), table.data(), table.size() * sizeof(float),
                                     cudaMemcpyHostToDevice, stream));
        host_io = PinnedBuffer(sizeof(int32_t) * (4 + prefill_chunk));
        if (wide16()) setup_wide16();
        setup_fused();
        setup_packed();
        CUDALLM_CUDA(cudaStreamSynchronize(stream));
    }

    float eps() const { return config.norm_epsilon; }
    int32_t* host_in() const { return static_cast<int32_t*>(host_io.get()); }

    void all_reduce(float* send, float* recv, std::size_t n) {
        CUDALLM_NCCL(ncclAllReduce(send, recv, n, ncclFloat32, ncclSum, comm, stream));
    }

    // The [hidden] all-reduces of a decode step.
    void decode_all_reduce(float* send, float* recv) {
        if (peer_allreduce)
            CUDALLM_CL(cl_peer_allreduce(send, recv, (int)H, (int)H, par.rank, par.world, peer_bufs.data(), stream));
        else
            all_reduce(send, recv, H);
    }

    // Exchange buffers for decode_all_reduce: allocate and zero this rank's,
    // all-gather the IPC handles over NCCL, map the others.  The all-gather
    // also orders every rank's zeroing before any rank's first call.
    void setup_peer_exchange() {
        const int W = par.world, R = par.rank;
        if (H % 4 != 0) throw std::invalid_argument("peer all-reduce needs a hidden size that is a multiple of 4");
        peer_buf = DeviceBuffer(cl_peer_exchange_bytes((int)H));
        CUDALLM_CL(cl_peer_exchange_init(peer_buf.get(), (int)H, stream));
        cudaIpcMemHandle_t mine;
        CUDALLM_CUDA(cudaIpcGetMemHandle(&mine, peer_buf.get()));
        const std::size_t hb = sizeof(cudaIpcMemHandle_t);
        DeviceBuffer handles(hb * W);
        char* hd = static_cast<char*>(handles.get());
        CUDALLM_CUDA(cudaMemcpyAsync(hd + R * hb, &mine, hb, cudaMemcpyHostToDevice, stream));
        CUDALLM_NCCL(ncclAllGather(hd + R * hb, hd, hb, ncclChar, comm, stream));
        std::vector<cudaIpcMemHandle_t> all(W);
        CUDALLM_CUDA(cudaMemcpyAsync(all.data(), hd, hb * W, cudaMemcpyDeviceToHost, stream));
        CUDALLM_CUDA(cudaStreamSynchronize(stream));
        peer_bufs.assign(W, nullptr);
        peer_bufs[R] = peer_buf.get();
        for (int r = 0; r < W; ++r) {
            if (r == R) continue;
            void* p = nullptr;
            CUDALLM_CUDA(cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess));
            peer_bufs[r] = p;
        }
        peer_allreduce = true;
    }

    // A packed decode GEMV (x RMS-normalised by gamma when given).
    void gemv_packed(const cl_gemv_packed_segment* segs, int nseg, std::size_t kdim, const float* x,
                     const float* gamma, int swiglu) {
        CUDALLM_CL(cl_gemv_packed(segs, nseg, (int)kdim, x, gamma, eps(), swiglu, pk_ws.get(), pk_ws.size(), stream));
    }

    // Final RMSNorm + LM head + greedy token for the hidden row `hrow`.
    void record_head(const float* hrow, int32_t* token_out) {
        cudaStream_t s = stream;
        if (pk_head) {
            const cl_gemv_packed_segment seg{out_w.type, pk_head, (int)V_l, nullptr, nullptr, logits};
            gemv_packed(&seg, 1, H, hrow, out_norm, 0);
        } else {
            const cl_gemv_segment seg{out_w.type, out_w.ptr, out_w.stride, (int)V_l, nullptr, nullptr, logits};
            CUDALLM_CL(cl_gemv_multi(&seg, 1, (int)H, hrow, out_norm, eps(), s));
        }
        if (par.world == 1) {
            CUDALLM_CL(cl_argmax(logits, (int)V_l, token_out, arg_ws, arg_ws_bytes, s));
        } else {
            float* rec = best + 2 * par.rank;
            CUDALLM_CL(cl_argmax_ex(logits, (int)V_l, (int)vocab0, reinterpret_cast<int32_t*>(rec + 1), rec, arg_ws,
                                    arg_ws_bytes, s));
            CUDALLM_NCCL(ncclAllGather(rec, best, 2, ncclFloat32, comm, s));
            CUDALLM_CL(cl_argmax_merge(best, par.world, token_out, s));
        }
    }

    // One decode step: host_in[0] -> token; host_in[1] <- greedy token.
    void record_decode() {
        cudaStream_t s = stream;
        if (fused) {
            CUDALLM_CUDA(cudaMemcpyAsync(ints, host_in(), sizeof(int32_t), cudaMemcpyHostToDevice, s));
            CUDALLM_CUDA(cudaEventRecord(kev0, s));
            CUDALLM_CL(cl_qwen2_decode_step(&fused_desc, fused_layers.data(), fused_ws, fused_ws_bytes, s));
            CUDALLM_CUDA(cudaEventRecord(kev1, s));
            CUDALLM_CUDA(cudaMemcpyAsync(host_in() + 1, ints + 3, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
            CUDALLM_CUDA(cudaMemcpyAsync(host_in() + 2, cl_qwen2_decode_status(fused_ws), sizeof(int32_t),
                                         cudaMemcpyDeviceToHost, s));
            return;
        }
        const int W = par.world;
        const float scale = 1.0f / std::sqrt(static_cast<float>(d));
        int32_t* tok_in = ints + 0;
        int* pos = ints + 1;
        CUDALLM_CUDA(cudaMemcpyAsync(tok_in, host_in(), sizeof(int32_t), cudaMemcpyHostToDevice, s));
        CUDALLM_CL(cl_embed(tok_embd.type, tok_embd.ptr, tok_embd.stride, (int)V, (int)H, tok_in, 1, h, ints + 4, s));
        float* out = W > 1 ? part : h;
        const float* res = par.rank == 0 ? h : nullptr;
        for (std::size_t l = 0; l < layers.size(); ++l) {
            Layer& L = layers[l];
            const PackedLayer* PL = packed_layers ? &pk_layers[l] : nullptr;
            if (PL) {
                const cl_gemv_packed_segment segs[3] = {
                    {L.q.type, PL->q, L.q.rows, L.q_b, nullptr, q},
                    {L.k.type, PL->k, L.k.rows, L.k_b, nullptr, k},
                    {L.v.type, PL->v, L.v.rows, L.v_b, nullptr, v},
                };
                gemv_packed(segs, 3, H, h, L.attn_norm, 0);
            } else {
                const cl_gemv_segment segs[3] = {
                    {L.q.type, L.q.ptr, L.q.stride, L.q.rows, L.q_b, nullptr, q},
                    {L.k.type, L.k.ptr, L.k.stride, L.k.rows, L.k_b, nullptr, k},
                    {L.v.type, L.v.ptr, L.v.stride, L.v.rows, L.v_b, nullptr, v},
                };
                CUDALLM_CL(cl_gemv_multi(segs, 3, (int)H, h, L.attn_norm, eps(), s));
            }
            // RoPE of q/k at *pos, the KV append and attention over keys 0..*pos in one launch pair
            CUDALLM_CL(cl_attn_decode_rope(q, k, v, rope, pos, (int)config.rotary_dimension, L.k_cache, L.v_cache,
                                           (int)max_seq, (int)hq_l, (int)hkv_l, (int)d, scale, att, nullptr, attn_ws,
                                           attn_ws_bytes, s));
            const float* o_in = att;
            if (gather_attn) {
                CUDALLM_NCCL(ncclAllGather(att, att_full, hq_l * d, ncclFloat32, comm, s));
                o_in = att_full + o_k0;
            }
            if (PL) {
                const cl_gemv_packed_segment seg{L.o.type, PL->o, (int)H, nullptr, res, out};
                gemv_packed(&seg, 1, o_kl, o_in, nullptr, 0);
            } else if (o_kl > 0)
                CUDALLM_CL(cl_gemv(L.o.type, L.o.ptr, L.o.stride, (int)H, (int)o_kl, o_in, nullptr, res, out, s));
            else
                CUDALLM_CUDA(cudaMemsetAsync(out, 0, H * sizeof(float), s));
            if (W > 1) decode_all_reduce(part, h);
            if (F_l == 0) {
                CUDALLM_CUDA(cudaMemsetAsync(out, 0, H * sizeof(float), s));
                if (W > 1) decode_all_reduce(part, h);
                continue;
            }
            if (PL) {
                const cl_gemv_packed_segment gu{L.gate.type, PL->gate, (int)F_l, nullptr, nullptr, act};
                gemv_packed(&gu, 1, H, h, L.ffn_norm, 1);
                const cl_gemv_packed_segment dn{L.down.type, PL->down, (int)H, nullptr, res, out};
                gemv_packed(&dn, 1, F_l, act, nullptr, 0);
            } else {
                CUDALLM_CL(cl_gemv_swiglu(L.gate.type, L.gate.ptr, L.up.ptr, L.gate.stride, (int)F_l, (int)H, h,
                                          L.ffn_norm, eps(), act, s));
                CUDALLM_CL(cl_gemv(L.down.type, L.down.ptr, L.down.stride, (int)H, (int)F_l, act, nullptr, res, out,
                                   s));
            }
            if (W > 1) decode_all_reduce(part, h);
        }
        record_head(h, ints + 3);
        CUDALLM_CL(cl_counter_add(pos, 2, 1, s));
        CUDALLM_CUDA(cudaMemcpyAsync(host_in() + 1, ints + 3, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
        if (peer_allreduce)
            CUDALLM_CUDA(cudaMemcpyAsync(host_in() + 2, cl_peer_exchange_status(peer_buf.get()), sizeof(int32_t),
                                         cudaMemcpyDeviceToHost, s));
    }

    void build_decode_graph() {
        cudaGraph_t graph = nullptr;
        CUDALLM_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
        try {
            record_decode();
        } catch (...) {
            cudaStreamEndCapture(stream, &graph);
            if (graph) cudaGraphDestroy(graph);
            throw;
        }
        CUDALLM_CUDA(cudaStreamEndCapture(stream, &graph));
        const cudaError_t e = cudaGraphInstantiate(&decode_exec, graph, 0);
        cudaGraphDestroy(graph);
        CUDALLM_CUDA(e);
    }

    // Prefill GEMM: the 16-bit tensor-core path over resident 16-bit weight
    // copies (Fp16x3, the default: split hi + lo, FP32-grade; Fp16; Bf16),
    // the split-TF32 tcgen05 path over the native blocks (Auto: FP32-grade),
    // its one-pass FP16 form, or the FP32 CUDA-core kernel.
    enum class GemmPath { Auto, F16, Simt, Fp16, Bf16, Fp16x3 };
    // Prefill attention: Auto (by the GEMM path's grade), or forced with
    // CUDALLM_PREFILL_ATTN=fp32 | fp16 | fp16x3.
    enum class PrefillAttn { Auto, Fp32, Tc, Tc3 };
    PrefillAttn prefill_attn = PrefillAttn::Auto;
    GemmPath gemm_path = GemmPath::Fp16x3;
    DeviceBuffer w16_mem, g16_ws_mem, amax_mem;
    float* xmax = nullptr;  // split form: the device maximum of the current product's X
    void* x16 = nullptr;  // [prefill_chunk][max(H, F_l, o_kl)] 16-bit activations
    bool wide16() const {
        return gemm_path == GemmPath::Fp16 || gemm_path == GemmPath::Bf16 || gemm_path == GemmPath::Fp16x3;
    }
    bool split16() const { return gemm_path == GemmPath::Fp16x3; }
    int fmt16() const {
        return gemm_path == GemmPath::Bf16 ? CL_GEMM_BF16 : split16() ? CL_GEMM_F16X3 : CL_GEMM_F16;
    }

    // Y[m, W.rows] = X[m, kdim] W^T (+ bias) (+ residual) on the selected path.
    void gemm(const DevMat& Wm, int n, int kdim, const float* x, int m, const float* bias, const float* res, float* y) {
        switch (gemm_path) {
        case GemmPath::F16: {
            const int rc = cl_gemm_tc(Wm.type, Wm.ptr, Wm.stride, n, kdim, x, m, bias, res, y, CL_GEMM_F16, stream);
            if (rc != CL_ERR_UNSUPPORTED) {
                CUDALLM_CL(rc);
                return;
            }
            break;  // shapes the FP16 path does not take use the default path
        }
        case GemmPath::Simt:
            CUDALLM_CL(cl_gemm_simt(Wm.type, Wm.ptr, Wm.stride, n, kdim, x, m, bias, res, y, stream));
            return;
        case GemmPath::Auto:
        case GemmPath::Fp16:  // matrices the 16-bit GEMM does not take
        case GemmPath::Bf16:
        case GemmPath::Fp16x3: break;
        }
        CUDALLM_CL(cl_gemm(Wm.type, Wm.ptr, Wm.stride, n, kdim, x, m, bias, res, y, stream));
    }

    // Rows [0, m) of X hold the chunk at positions pos0..pos0+m-1.
    void prefill_chunk_layers(int m, int pos0) {
        cudaStream_t s = stream;
        const int W = par.world;
        float* out = W > 1 ? P : X;
        const float* res = par.rank == 0 ? X : nullptr;
        const std::size_t qd_l = hq_l * d;
        for (Layer& L : layers) {
            CUDALLM_CL(cl_rmsnorm(X, L.attn_norm, m, (int)H, eps(), Xn, nullptr, s));
            if (L.qkv16) {
                const cl_gemm_out outs[3] = {out16(Q, L.q_b, nullptr, 0, L.q.rows, L.q.rows, L.wmax),
                                             out16(K, L.k_b, nullptr, L.q.rows, L.k.rows, L.k.rows, L.wmax + 1),
                                             out16(Vv, L.v_b, nullptr, L.q.rows + L.k.rows, L.v.rows, L.v.rows,
                                                   L.wmax + 2)};
                gemm16(L.qkv16, L.q.rows + L.k.rows + L.v.rows, (int)H, Xn, m, outs, 3);
            } else {
                gemm(L.q, L.q.rows, (int)H, Xn, m, L.q_b, nullptr, Q);
                gemm(L.k, L.k.rows, (int)H, Xn, m, L.k_b, nullptr, K);
                gemm(L.v, L.v.rows, (int)H, Xn, m, L.v_b, nullptr, Vv);
            }
            CUDALLM_CL(cl_rope_kv(Q, K, Vv, m, (int)hq_l, (int)hkv_l, (int)d, (int)config.rotary_dimension, rope, nullptr,
                                  pos0, L.k_cache, L.v_cache, s));
            // the one-pass 16-bit prefill paths take the FP16 tensor-core attention, the
            // FP32-grade paths its split-FP16 form (head_dim 128); else the FP32 kernel
            const PrefillAttn pa = prefill_attn == PrefillAttn::Auto
                                       ? (wide16() && !split16() ? PrefillAttn::Tc : PrefillAttn::Tc3)
                                       : prefill_attn;
            if (!(d == 128 && pa != PrefillAttn::Fp32 &&
                  (pa == PrefillAttn::Tc ? cl_attn_prefill_tc : cl_attn_prefill_tc3)(
                      Q, L.k_cache, L.v_cache, pos0, m, (int)hq_l, (int)hkv_l, (int)d, A, s) == CL_OK))
                CUDALLM_CL(cl_attn_prefill(Q, L.k_cache, L.v_cache, pos0, m, (int)hq_l, (int)hkv_l, (int)d, A, s));
            const float* o_in = A;
            if (gather_attn) {
                // rank-major gather [W][m][qd_l] -> rows [m][hq*d], then the
                // contiguous o_proj column share into A.
                CUDALLM_NCCL(ncclAllGather(A, A_full, (std::size_t)m * qd_l, ncclFloat32, comm, s));
                for (int r = 0; r < W; ++r) {
                    const std::size_t c0 = std::max(o_k0, r * qd_l);
                    const std::size_t c1 = std::min(o_k0 + o_kl, (r + 1) * qd_l);
                    if (c0 >= c1) continue;
                    CUDALLM_CUDA(cudaMemcpy2DAsync(Xn + (c0 - o_k0), o_kl * sizeof(float),
                                                   A_full + (std::size_t)r * m * qd_l + (c0 - r * qd_l),
                                                   qd_l * sizeof(float), (c1 - c0) * sizeof(float), m,
                                                   cudaMemcpyDeviceToDevice, s));
                }
                o_in = Xn;
            }
            if (o_kl > 0 && L.o16) {
                const cl_gemm_out o = out16(out, nullptr, res, 0, (int)H, (int)H, L.wmax + 3);
                gemm16(L.o16, (int)H, (int)o_kl, o_in, m, &o, 1);
            } else if (o_kl > 0) {
                gemm(L.o, (int)H, (int)o_kl, o_in, m, nullptr, res, out);
            } else {
                CUDALLM_CUDA(cudaMemsetAsync(out, 0, (std::size_t)m * H * sizeof(float), s));
            }
            if (W > 1) all_reduce(P, X, (std::size_t)m * H);
            CUDALLM_CL(cl_rmsnorm(X, L.ffn_norm, m, (int)H, eps(), Xn, nullptr, s));
            if (F_l == 0) {
                CUDALLM_CUDA(cudaMemsetAsync(out, 0, (std::size_t)m * H * sizeof(float), s));
                if (W > 1) all_reduce(P, X, (std::size_t)m * H);
                continue;
            }
            if (L.gu16) {
                const cl_gemm_out gu[2] = {out16(G, nullptr, nullptr, 0, (int)F_l, (int)F_l, L.wmax + 4),
                                           out16(U, nullptr, nullptr, (int)F_l, (int)F_l, (int)F_l, L.wmax + 5)};
                gemm16(L.gu16, 2 * (int)F_l, (int)H, Xn, m, gu, 2);
            } else {
                gemm(L.gate, (int)F_l, (int)H, Xn, m, nullptr, nullptr, G);
                gemm(L.up, (int)F_l, (int)H, Xn, m, nullptr, nullptr, U);
            }
            CUDALLM_CL(cl_swiglu(G, U, G, (long long)m * F_l, s));
            if (L.down16) {
                const cl_gemm_out dn = out16(out, nullptr, res, 0, (int)H, (int)H, L.wmax + 6);
                gemm16(L.down16, (int)H, (int)F_l, G, m, &dn, 1);
            } else {
                gemm(L.down, (int)H, (int)F_l, G, m, nullptr, res, out);
            }
            if (W > 1) all_reduce(P, X, (std::size_t)m * H);
        }
    }

    void begin_timing() {
        call_start = std::chrono::steady_clock::now();
        CUDALLM_CUDA(cudaEventRecord(ev0, stream));
    }

    // Logical, shape-derived FLOPs and bytes of a call on this rank: prefill
    // of n tokens (n > 0) or one decode step (n == 0) at the current position.
    ProfileMetrics call_metrics(std::size_t n) const {
        std::uint64_t elems = 0;
        for (const Layer& L : layers)
            for (const DevMat* m : {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down})
                elems += (std::uint64_t)m->rows * (std::uint64_t)m->cols;
        const std::uint64_t head = (std::uint64_t)out_w.rows * (std::uint64_t)out_w.cols;
        const std::uint64_t kv_row = 2 * hkv_l * d * sizeof(float) * layers.size();  // K and V, all layers
        const std::uint64_t embed_row = V ? tok_embd.payload / V : 0;
        const std::uint64_t weights = weight_payload - tok_embd.payload;
        const std::uint64_t attn = 4 * d * hq_l * layers.size();  // QK and AV per (query, key)
        ProfileMetrics m;
        if (n > 0) {  // causal: query i reads keys 0..i
            const std::uint64_t pairs = (std::uint64_t)n * (n + 1) / 2;
            m.flops = 2 * n * elems + 2 * head + attn * pairs;
            m.read_bytes = weights + n * embed_row + kv_row * pairs;
            m.write_bytes = kv_row * n + 4 * (std::uint64_t)V_l;
        } else {  // the new key at `position` and keys 0..position
            const std::uint64_t keys = position + 1;
            m.flops = 2 * (elems + head) + attn * keys;
            m.read_bytes = weights + embed_row + kv_row * keys;
            m.write_bytes = kv_row + 4 * (std::uint64_t)V_l;
        }
        return m;
    }

    void end_timing(const char* phase, std::size_t tokens) {
        CUDALLM_CUDA(cudaEventRecord(ev1, stream));
        CUDALLM_CUDA(cudaEventSynchronize(ev1));
        CUDALLM_CUDA(cudaEventElapsedTime(&last_ms, ev0, ev1));
        if (profile) {
            const bool pre = std::strcmp(phase, "prefill") == 0;
            const auto ns = std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() -
                                                                                 call_start);
            // stage names of the reference's resident GPU path (metal_llm.mm:3219-3221, 3319-3321)
            profile->forward(pre ? "prefill.gpu_resident" : "decode.gpu_resident", pre ? tokens : position + 1,
                             (std::uint64_t)ns.count(), call_metrics(pre ? tokens : 0));
        }
    }

    int32_t prefill(const std::vector<int32_t>& ids) {
        if (ids.empty()) throw std::invalid_argument("CUDA prefill requires at least one token");
        if (position != 0) throw std::invalid_argument("CUDA prefill requires an empty conversation; call reset first");
        if (ids.size() > max_seq) throw std::length_error("CUDA prefill exceeds sequence capacity");
        for (int32_t id : ids) {
            if (id < 0 || (std::size_t)id >= config.vocabulary_size)
                throw std::out_of_range("CUDA prefill token id is outside the vocabulary");
        }
        CUDALLM_CUDA(cudaSetDevice(device));
        const TraceRange trace("prefill.gpu_resident");
        begin_timing();
        const std::size_t n = ids.size();
        int32_t* staging = host_in() + 4;
        std::size_t last_m = 0;
        for (std::size_t c0 = 0; c0 < n; c0 += prefill_chunk) {
            const std::size_t m = std::min(prefill_chunk, n - c0);
            // the previous chunk's copy must be done before the staging is reused
            CUDALLM_CUDA(cudaStreamSynchronize(stream));
            std::memcpy(staging, ids.data() + c0, m * sizeof(int32_t));
            CUDALLM_CUDA(cudaMemcpyAsync(ids_dev, staging, m * sizeof(int32_t), cudaMemcpyHostToDevice, stream));
            CUDALLM_CL(cl_embed(tok_embd.type, tok_embd.ptr, tok_embd.stride, (int)V, (int)H, ids_dev, (int)m, X,
                                ints + 4, stream));
            prefill_chunk_layers((int)m, (int)c0);
            last_m = m;
        }
        record_head(X + (last_m - 1) * H, ints + 3);
        int32_t* hi = host_in();
        hi[2] = (int32_t)n;
        hi[3] = (int32_t)(n + 1);
        CUDALLM_CUDA(cudaMemcpyAsync(ints + 1, hi + 2, 2 * sizeof(int32_t), cudaMemcpyHostToDevice, stream));
        CUDALLM_CUDA(cudaMemcpyAsync(hi + 1, ints + 3, sizeof(int32_t), cudaMemcpyDeviceToHost, stream));
        end_timing("prefill", n);
        position = n;
        have_logits = true;
        return hi[1];
    }

    int32_t decode(int32_t token) {
        if (position == 0) throw std::invalid_argument("CUDA decode requires a completed prefill");
        if (token < 0 || (std::size_t)token >= config.vocabulary_size)
            throw std::out_of_range("CUDA decode token id is outside the vocabulary");
        if (position >= max_seq) throw std::length_error("CUDA decode exceeds sequence capacity");
        CUDALLM_CUDA(cudaSetDevice(device));
        // The fused step is three stream operations (token copy, the step
        // kernel between two timing events, token copy back), launched
        // directly; the per-operator path is one captured graph.
        if (decode_exec == nullptr && !fused) build_decode_graph();
        host_in()[0] = token;
        const TraceRange trace("decode.gpu_resident");
        begin_timing();
        if (fused)
            record_decode();
        else
            CUDALLM_CUDA(cudaGraphLaunch(decode_exec, stream));
        end_timing("decode", 1);
        last_kernel_ms = 0.0f;
        if (fused) CUDALLM_CUDA(cudaEventElapsedTime(&last_kernel_ms, kev0, kev1));
        if (fused && !trace_path.empty()) {
            std::vector<long long> t(trace_mem.size() / sizeof(long long));
            CUDALLM_CUDA(cudaMemcpy(t.data(), trace_mem.get(), trace_mem.size(), cudaMemcpyDeviceToHost));
            std::ofstream f(trace_path, std::ios::binary | std::ios::trunc);
            f.write(reinterpret_cast<const char*>(t.data()), (std::streamsize)(t.size() * sizeof(long long)));
        }
        if (peer_allreduce && host_in()[2] != 0)
            throw std::runtime_error("peer all-reduce: a rank did not reach the decode step within the wait limit");
        if (fused && host_in()[2] != 0) {
            const int phase = host_in()[2];
            CUDALLM_CL(cl_qwen2_decode_init(fused_ws, fused_ws_bytes, stream));
            CUDALLM_CUDA(cudaStreamSynchronize(stream));
            throw std::runtime_error("fused decode: a grid barrier wait ran out in phase " + std::to_string(phase - 1));
        }
        position += 1;
        have_logits = true;
        return host_in()[1];
    }
};

CudaLLM::CudaLLM(const std::string& gguf_path, std::size_t max_sequence, int device, const ParallelConfig& parallel)
    : impl_(std::make_unique<Impl>()) {
    impl_->init(gguf_path, max_sequence, device, parallel);
}

CudaLLM::~CudaLLM() = default;
CudaLLM::CudaLLM(CudaLLM&&) noexcept = default;
CudaLLM& CudaLLM::operator=(CudaLLM&&) noexcept = default;

void CudaLLM::reset() {
    if (!impl_) throw std::runtime_error("CUDA model is not initialized");
    // Logical reset only (metal_llm.mm:3185-3187): KV rows are overwritten.
    impl_->position = 0;
    impl_->have_logits = false;
}

std::int32_t CudaLLM::prefill(const std::vector<std::int32_t>& token_ids) {
    if (!impl_) throw std::runtime_error("CUDA model is not initialized");
    return impl_->prefill(token_ids);
}

std::int32_t CudaLLM::decode(std::int32_t token_id) {
    if (!impl_) throw std::runtime_error("CUDA model is not initialized");
    return impl_->decode(token_id);
}

void CudaLLM::enable_profiling(const std::string& csv_path, bool) {
    if (!impl_) throw std::runtime_error("CUDA model is not initialized");
    impl_->profile.reset();  // a previous file gets its summary rows first
    impl_->profile = std::make_unique<ProfileCsv>(csv_path);
}

void CudaLLM::disable_profiling() {
    if (impl_) impl_->profile.reset();
}

const ModelConfig& CudaLLM::config() const {
    if (!impl_) throw std::runtime_error("CUDA model is not initialized");
    return impl_->config;
}

std::size_t CudaLLM::position() const noexcept { return impl_ ? impl_->position : 0; }
std::size_t CudaLLM::max_sequence() const noexcept { return impl_ ? impl_->max_seq : 0; }
bool CudaLLM::uses_gpu() const noexcept { return true; }
bool CudaLLM::available() const noexcept { return impl_ != nullptr; }

const std::string& CudaLLM::device_name() const {
    if (!impl_) throw std::runtime_error("CUDA model is not initialized");
    return impl_->device_name;
}

MemoryStats CudaLLM::memory_stats() const noexcept {
    if (!impl_) return {};
    MemoryStats m;
    m.weight_bytes = impl_->weight_mem.size() + impl_->w16_mem.size() + impl_->pack_mem.size();
    m.kv_cache_bytes = impl_->kv_bytes;
    m.recurrent_state_bytes = 0;
    m.intermediate_bytes = impl_->act_bytes;
    m.intermediate_is_estimate = false;
    return m;
}

void CudaLLM::last_logits(float* out, std::size_t n) const {
    if (!impl_ || !impl_->have_logits) throw std::invalid_argument("no logits: call prefill or decode first");
    Impl& I = *impl_;
    if (n < I.V) throw std::invalid_argument("logits buffer is smaller than the vocabulary");
    CUDALLM_CUDA(cudaSetDevice(I.device));
    if (I.par.world == 1) {
        CUDALLM_CUDA(cudaMemcpy(out, I.logits, I.V * sizeof(float), cudaMemcpyDeviceToHost));
        return;
    }
    // Collective: every rank gathers the vocabulary shards (uneven shares
    // are padded to the largest one).
    const std::size_t chunk = (I.V + I.par.world - 1) / I.par.world;
    DeviceBuffer send(chunk * sizeof(float)), recv(chunk * I.par.world * sizeof(float));
    CUDALLM_CUDA(cudaMemsetAsync(send.get(), 0, send.size(), I.stream));
    CUDALLM_CUDA(cudaMemcpyAsync(send.get(), I.logits, I.V_l * sizeof(float), cudaMemcpyDeviceToDevice, I.stream));
    CUDALLM_NCCL(ncclAllGather(send.get(), recv.get(), chunk, ncclFloat32, I.comm, I.stream));
    std::vector<float> all(chunk * I.par.world);
    CUDALLM_CUDA(cudaMemcpyAsync(all.data(), recv.get(), recv.size(), cudaMemcpyDeviceToHost, I.stream));
    CUDALLM_CUDA(cudaStreamSynchronize(I.stream));
    for (int r = 0; r < I.par.world; ++r) {
        auto rg = split_range(I.V, I.par.world, r);
        std::memcpy(out + rg.first, all.data() + (std::size_t)r * chunk, (rg.second - rg.first) * sizeof(float));
    }
}

float CudaLLM::last_call_ms() const noexcept { return impl_ ? impl_->last_ms : 0.0f; }
float CudaLLM::last_kernel_ms() const noexcept { return impl_ ? impl_->last_kernel_ms : 0.0f; }

}  // namespace cudallm
