// CudaMoeLLM: the qwen35moe graph (Qwen3.5/3.6 A3B) on one or more B200s.
//
// Layer order follows encode_layer_route / encode_layer_experts
// (moe_llm.mm:2845-2885):
//   h = embed(id)
//   per layer: a = rmsnorm(h); h += (full attention if (l + 1) % interval == 0
//              else Gated DeltaNet)(a); f = rmsnorm(h); route(f);
//              h += sum_r w_r expert_r(f) + sigmoid(w_sh . f) shared(f)
//   logits = rmsnorm(h) Wout^T; token = argmax (lowest index on ties).
// Unlike the reference, which reads the route ids back to the host every
// layer (moe_llm.mm:2918-2930), the ids stay on the device: one decode step
// is one CUDA graph with a single 4-byte token read-back.  Prefill replays a
// second graph once per prompt token (token-serial, like the reference's
// DeltaNet scan) and runs the LM head for the last token only.
//
// Expert parallel (world > 1): expert e lives on rank e % world; attention,
// DeltaNet, norms and the LM head are replicated, every rank computes the
// same route on device, evaluates only its local experts (the shared
// expert on rank l % world) and one all-reduce of the [hidden] partial per
// layer sums them; no all-to-all is needed at batch 1.
#include "cuda_moe_llm.h"

#include <nccl.h>

#include <cmath>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <stdexcept>

#include "device.h"
#include "gguf.h"
#include "profile.h"

namespace cudallm {

namespace {

#define MOE_NCCL(expr)                                                                         \
    do {                                                                                       \
        ncclResult_t r_ = (expr);                                                              \
        if (r_ != ncclSuccess)                                                                 \
            throw std::runtime_error(std::string("NCCL error ") + ncclGetErrorString(r_) +     \
                                     " in " #expr);                                            \
    } while (0)

ModelConfig read_moe_config(const GgufFile& f) {
    ModelConfig c;
    c.architecture = f.text("general.architecture");
    if (c.architecture != "qwen35moe")
        throw std::runtime_error("CudaMoeLLM requires qwen35moe, got " + c.architecture);
    const std::string a = "qwen35moe.";
    c.tensor_count = f.tensors().size();
    const std::size_t total = f.size(a + "block_count");
    const std::size_t nextn = (std::size_t)f.integer(a + "nextn_predict_layers", 0);
    if (nextn >= total) throw std::runtime_error("invalid optional NextN/MTP layer count");
    c.layer_count = total - nextn;
    c.embedding_size = f.size(a + "embedding_length");
    c.attention_head_count = f.size(a + "attention.head_count");
    c.kv_head_count = f.size(a + "attention.head_count_kv");
    c.context_length = f.size(a + "context_length");
    c.expert_count = f.size(a + "expert_count");
    c.expert_used_count = f.size(a + "expert_used_count");
    c.expert_feed_forward_size = f.size(a + "expert_feed_forward_length");
    c.shared_expert_feed_forward_size = f.size(a + "expert_shared_feed_forward_length");
    c.feed_forward_size = c.expert_feed_forward_size;
    c.full_attention_interval = f.size(a + "full_attention_interval");
    c.ssm_conv_kernel = f.size(a + "ssm.conv_kernel");
    c.ssm_state_size = f.size(a + "ssm.state_size");
    c.ssm_group_count = f.size(a + "ssm.group_count");
    c.ssm_time_step_rank = f.size(a + "ssm.time_step_rank");
    c.ssm_inner_size = f.size(a + "ssm.inner_size");
    c.vocabulary_size = f.array_length("tokenizer.ggml.tokens");
    if (c.vocabulary_size == 0) c.vocabulary_size = f.size("tokenizer.ggml.tokens_count");
    c.vocabulary = f.strings("tokenizer.ggml.tokens");
    c.merges = f.strings("tokenizer.ggml.merges");
    c.tokenizer_pre = f.text("tokenizer.ggml.pre");
    c.head_size = f.size(a + "attention.key_length");
    if (f.size(a + "attention.value_length") != c.head_size)
        throw std::runtime_error("qwen35moe key/value head dimensions differ");
    c.rotary_dimension = f.size(a + "rope.dimension_count");
    c.rope_theta = (float)f.real(a + "rope.freq_base", 1000000.0);
    c.norm_epsilon = (float)f.real(a + "attention.layer_norm_rms_epsilon", 1e-6);
    const uint64_t eos = f.integer("tokenizer.ggml.eos_token_id", 151645);
    if (eos > (uint64_t)INT32_MAX) throw std::runtime_error("EOS token id does not fit in int32_t");
    c.eos_token_id = (int32_t)eos;
    // the checks of require_qwen35_config (moe_model.cpp:39-80)
    if (c.layer_count == 0 || c.full_attention_interval == 0 || c.embedding_size == 0 ||
        c.attention_head_count == 0 || c.kv_head_count == 0 || c.head_size == 0 || c.rotary_dimension == 0 ||
        c.expert_count == 0 || c.expert_used_count == 0 || c.expert_used_count > c.expert_count ||
        c.expert_feed_forward_size == 0 || c.shared_expert_feed_forward_size == 0 || c.ssm_conv_kernel == 0 ||
        c.ssm_state_size == 0 || c.ssm_group_count == 0 || c.ssm_time_step_rank == 0 || c.ssm_inner_size == 0)
        throw std::runtime_error("incomplete qwen35moe GGUF metadata");
    if (c.rotary_dimension > c.head_size || c.rotary_dimension % 2 != 0)
        throw std::runtime_error("qwen35moe rotary dimension must be even and fit one head");
    if (c.expert_used_count > 8) throw std::runtime_error("qwen35moe supports at most eight selected experts");
    if (c.ssm_conv_kernel > 9) throw std::runtime_error("qwen35moe convolution kernel exceeds 9 taps");
    if (c.ssm_inner_size % c.ssm_time_step_rank != 0 || c.ssm_inner_size / c.ssm_time_step_rank != c.ssm_state_size)
        throw std::runtime_error("qwen35moe DeltaNet value-head dimensions are inconsistent");
    if (c.ssm_time_step_rank % c.ssm_group_count != 0)
        throw std::runtime_error("qwen35moe DeltaNet value heads must group key heads evenly");
    if (c.attention_head_count % c.kv_head_count != 0)
        throw std::runtime_error("attention head count must be divisible by KV head count");
    if (!std::isfinite(c.rope_theta) || c.rope_theta <= 0.0f || !std::isfinite(c.norm_epsilon) ||
        c.norm_epsilon <= 0.0f)
        throw std::runtime_error("invalid RoPE or RMSNorm metadata");
    for (const TensorInfo& t : f.tensors()) {
        c.parameter_count += t.rows * t.cols;
        c.stored_weight_bytes += t.bytes;
    }
    return c;
}

// cos / sin of partial NeoX RoPE (metal_llm.metal:928-967) for every
// position, in double precision, stored as float.
std::vector<float> rope_table_f64(std::size_t positions, std::size_t rot, double theta) {
    const std::size_t half = rot / 2;
    std::vector<float> t(positions * half * 2);
    for (std::size_t pos = 0; pos < positions; ++pos)
        for (std::size_t p = 0; p < half; ++p) {
            const double ang = (double)pos * std::pow(theta, -2.0 * (double)p / (double)rot);
            t[(pos * half + p) * 2] = (float)std::cos(ang);
            t[(pos * half + p) * 2 + 1] = (float)std::sin(ang);
        }
    return t;
}

struct MoeLayer {
    bool attention = false;
    const float* attn_norm = nullptr;
    const float* post_norm = nullptr;
    // gated full attention
    DevMat q_gate, k, v, o;
    const float *q_norm = nullptr, *k_norm = nullptr;
    float *k_cache = nullptr, *v_cache = nullptr;
    // Gated DeltaNet
    DevMat qkv, z, out;
    const float *alpha_w = nullptr, *beta_w = nullptr, *conv_w = nullptr, *dt_bias = nullptr, *a = nullptr,
                *ssm_norm = nullptr;
    float *state = nullptr, *hist = nullptr;
    // experts (this rank's, stacked in expert order) and the shared expert
    const float* router = nullptr;
    DevMat gate_e, up_e, down_e;
    const float* shared_router = nullptr;
    DevMat sh_gate, sh_up, sh_down;
};

}  // namespace

std::string gguf_architecture(const std::string& gguf_path) {
    GgufFile f(gguf_path);
    return f.text("general.architecture");
}

struct CudaMoeLLM::Impl {
    // F32 GEMVs of a decode step that share their input, stacked so that each
    // pair is one launch: per DeltaNet layer the alpha and beta rows, per layer
    // the router and the shared expert's gate row.
    DeviceBuffer stack_mem;
    std::vector<const float*> stack_ab, stack_rs;
    // The LM head on the fragment-packed GEMV (cl_gemv_packed) where it is
    // Q4_K / Q6_K on the 256-column grid: it streams the 248k-row head faster
    // than the ring GEMV; CUDALLM_DECODE_GEMV=ring keeps the ring kernel.
    DeviceBuffer head_pk, head_ws;
    ModelConfig config;
    ParallelConfig par;
    int device = 0;
    std::string device_name;
    cudaStream_t stream = nullptr;
    ncclComm_t comm = nullptr;

    std::size_t H = 0, V = 0, E = 0, Kr = 0, FF = 0, SFF = 0;  // hidden, vocab, experts, routes, expert / shared FFN
    std::size_t hq = 0, hkv = 0, d = 0, rot = 0;             // attention
    std::size_t sg = 0, sr = 0, sd = 0, kc = 0, qkvw = 0;    // DeltaNet heads, state size, conv taps, qkv width
    std::size_t E_l = 0;                                     // experts on this rank
    std::size_t max_seq = 0, position = 0;

    DeviceBuffer weight_mem, state_mem, act_mem;
    std::uint64_t kv_bytes = 0, recurrent_bytes = 0, act_bytes = 0;

    DevMat tok_embd, out_w;
    const float* out_norm = nullptr;
    std::vector<MoeLayer> layers;
    const float* rope = nullptr;

    // step activations
    float *h = nullptr, *xn = nullptr, *big = nullptr, *zb = nullptr, *alpha = nullptr, *beta_raw = nullptr,
          *act = nullptr, *decay = nullptr, *beta = nullptr, *gdn_out = nullptr, *q = nullptr, *gate = nullptr,
          *kb = nullptr, *vb = nullptr, *att = nullptr, *gated = nullptr, *rlog = nullptr, *wts = nullptr,
          *ea = nullptr, *ey = nullptr, *sh_logit = nullptr, *sh_act = nullptr, *sh_y = nullptr, *moe_part = nullptr,
          *logits = nullptr;
    int32_t* ids = nullptr;
    int32_t* ints = nullptr;     // [0] token in, [1] pos, [2] len, [3] token out, [4..] scratch
    int32_t* prompt = nullptr;   // prefill ids on the device
    void *attn_ws = nullptr, *arg_ws = nullptr;
    std::size_t attn_ws_bytes = 0, arg_ws_bytes = 0;

    // token-batched prefill: rows [pre_rows][...] of the chunk's activations
    DeviceBuffer pre_mem;
    std::size_t pre_rows = 0;
    float *px = nullptr, *pxn = nullptr, *pbig = nullptr, *pkb = nullptr, *pvb = nullptr, *pq = nullptr,
          *pgate = nullptr, *patt = nullptr, *pgated = nullptr, *pzb = nullptr, *palpha = nullptr, *pbetar = nullptr,
          *pact = nullptr, *pdecay = nullptr, *pbeta = nullptr, *pgdn = nullptr, *prlog = nullptr, *pwts = nullptr,
          *pea = nullptr, *pey = nullptr, *pshl = nullptr, *psg = nullptr, *psu = nullptr, *pshy = nullptr,
          *ppart = nullptr;
    int32_t* pids = nullptr;
    int32_t *pgoff = nullptr, *plist = nullptr;  // routes bucketed by local expert (grouped expert GEMV)
    void* pplanes = nullptr;                     // XQ encodings of the expert GEMVs' input rows
    std::size_t pplanes_bytes = 0;
    bool serial_prefill = false;
    bool grouped_experts = true;  // CUDALLM_MOE_EXPERTS=grouped|routes: prefill expert GEMV form  // CUDALLM_MOE_PREFILL=serial: one token-step graph per prompt token

    PinnedBuffer host_io;  // [0] token in, [1] token out, [2..3] pos/len, [4..] prompt staging
    cudaGraphExec_t decode_exec = nullptr, prefill_exec = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    float last_ms = 0.0f;
    std::unique_ptr<ProfileCsv> profile;
    std::chrono::steady_clock::time_point call_start;
    bool have_logits = false;
    std::uint64_t routed = 0;

    ~Impl() {
        if (decode_exec) cudaGraphExecDestroy(decode_exec);
        if (prefill_exec) cudaGraphExecDestroy(prefill_exec);
        if (comm) ncclCommDestroy(comm);
        if (ev0) cudaEventDestroy(ev0);
        if (ev1) cudaEventDestroy(ev1);
        if (stream) cudaStreamDestroy(stream);
    }

    float eps() const { return config.norm_epsilon; }
    int32_t* host_in() const { return static_cast<int32_t*>(host_io.get()); }
    bool is_attention(std::size_t l) const { return (l + 1) % config.full_attention_interval == 0; }

    void load_weights(GgufFile& file, Arena& arena, bool real) {
        WeightLoader wl(file, arena, stream);
        const int W = par.world, R = par.rank;
        tok_embd = wl.matrix("token_embd.weight", V, H);
        out_norm = wl.vector("output_norm.weight", H);
        out_w = wl.matrix("output.weight", V, H);
        layers.assign(config.layer_count, MoeLayer{});
        for (std::size_t l = 0; l < config.layer_count; ++l) {
            const std::string p = "blk." + std::to_string(l) + ".";
            MoeLayer& L = layers[l];
            L.attention = is_attention(l);
            L.attn_norm = wl.vector(p + "attn_norm.weight", H);
            L.post_norm = wl.vector(p + "post_attention_norm.weight", H);
            if (L.attention) {
                L.q_gate = wl.matrix(p + "attn_q.weight", 2 * hq * d, H);
                L.k = wl.matrix(p + "attn_k.weight", hkv * d, H);
                L.v = wl.matrix(p + "attn_v.weight", hkv * d, H);
                L.q_norm = wl.vector(p + "attn_q_norm.weight", d);
                L.k_norm = wl.vector(p + "attn_k_norm.weight", d);
                L.o = wl.matrix(p + "attn_output.weight", H, hq * d);
            } else {
                L.qkv = wl.matrix(p + "attn_qkv.weight", qkvw, H);
                L.z = wl.matrix(p + "attn_gate.weight", sr * sd, H);
                L.alpha_w = wl.matrix_f32(p + "ssm_alpha.weight", sr, H);
                L.beta_w = wl.matrix_f32(p + "ssm_beta.weight", sr, H);
                L.conv_w = wl.matrix_f32(p + "ssm_conv1d.weight", qkvw, kc);
                L.dt_bias = wl.vector(p + "ssm_dt.bias", sr);
                L.a = wl.vector(p + "ssm_a", sr);
                L.ssm_norm = wl.vector(p + "ssm_norm.weight", sd);
                L.out = wl.matrix(p + "ssm_out.weight", H, sr * sd);
            }
            L.router = wl.matrix_f32(p + "ffn_gate_inp.weight", E, H);
            std::vector<WeightLoader::Part> g, u, dn;
            for (std::size_t e = 0; e < E; ++e) {
                if (ep_expert_rank(e, W) != R) continue;
                g.push_back({p + "ffn_gate_exps.weight", E * FF, H, e * FF, (e + 1) * FF});
                u.push_back({p + "ffn_up_exps.weight", E * FF, H, e * FF, (e + 1) * FF});
                dn.push_back({p + "ffn_down_exps.weight", E * H, FF, e * H, (e + 1) * H});
            }
            if (g.empty()) {
                // a rank without experts (world > experts) still consumes the tensors
                file.mark_loaded(p + "ffn_gate_exps.weight");
                file.mark_loaded(p + "ffn_up_exps.weight");
                file.mark_loaded(p + "ffn_down_exps.weight");
            } else {
                L.gate_e = wl.stacked(g);
                L.up_e = wl.stacked(u);
                L.down_e = wl.stacked(dn);
                if (L.gate_e.type != L.up_e.type || L.gate_e.stride != L.up_e.stride)
                    throw std::runtime_error("expert gate and up tensors must share a type");
            }
            L.shared_router = wl.vector(p + "ffn_gate_inp_shexp.weight", H);
            L.sh_gate = wl.matrix(p + "ffn_gate_shexp.weight", SFF, H);
            L.sh_up = wl.matrix(p + "ffn_up_shexp.weight", SFF, H);
            L.sh_down = wl.matrix(p + "ffn_down_shexp.weight", H, SFF);
            if (L.sh_gate.type != L.sh_up.type) throw std::runtime_error("shared gate and up must share a type");
        }
        file.validate_all_loaded();
        if (real) wl.finish();
    }

    void allocate_state(Arena& a) {
        for (MoeLayer& L : layers) {
            if (L.attention) {
                L.k_cache = a.take_n<float>(max_seq * hkv * d);
                L.v_cache = a.take_n<float>(max_seq * hkv * d);
            } else {
                L.state = a.take_n<float>(sr * sd * sd);
                L.hist = a.take_n<float>(std::max<std::size_t>(1, (kc - 1) * qkvw));
            }
        }
        rope = a.take_n<float>(max_seq * (rot / 2) * 2);
    }

    void stack_f32() {
        std::size_t total = 0;
        for (const MoeLayer& L : layers) total += (L.attention ? 0 : 2 * sr * H) + (E + 1) * H;
        stack_mem = DeviceBuffer(total * sizeof(float) + 256);
        float* p = static_cast<float*>(stack_mem.get());
        stack_ab.assign(layers.size(), nullptr);
        stack_rs.assign(layers.size(), nullptr);
        auto put = [&](const float* src, std::size_t n) {
            CUDALLM_CUDA(cudaMemcpyAsync(p, src, n * sizeof(float), cudaMemcpyDeviceToDevice, stream));
            p += n;
        };
        for (std::size_t l = 0; l < layers.size(); ++l) {
            const MoeLayer& L = layers[l];
            if (!L.attention) {
                stack_ab[l] = p;
                put(L.alpha_w, sr * H);
                put(L.beta_w, sr * H);
            }
            stack_rs[l] = p;
            put(L.router, E * H);
            put(L.shared_router, H);
        }
    }

    void pack_head() {
        std::string mode = "head";
        if (const char* e = std::getenv("CUDALLM_DECODE_GEMV")) mode = e;
        if (mode == "ring") return;
        if ((out_w.type != CL_TYPE_Q4_K && out_w.type != CL_TYPE_Q6_K) || H % 256 != 0 || H > 21504) return;
        head_pk = DeviceBuffer(cl_gemv_pack_bytes(out_w.type, (int)V, (int)H, 0));
        CUDALLM_CL(cl_gemv_pack(out_w.type, out_w.ptr, out_w.stride, (int)V, (int)H, nullptr, head_pk.get(), stream));
        const std::size_t wsb = cl_gemv_packed_workspace_bytes((int)((V + 15) / 16));
        if (wsb == 0) throw std::runtime_error("cl_gemv_packed_workspace_bytes failed");
        head_ws = DeviceBuffer(wsb);
        CUDALLM_CUDA(cudaMemsetAsync(head_ws.get(), 0, head_ws.size(), stream));
    }

    void allocate_activations(Arena& a) {
        h = a.take_n<float>(H);
        xn = a.take_n<float>(H);
        big = a.take_n<float>(std::max(qkvw, 2 * hq * d));
        zb = a.take_n<float>(sr * sd);
        alpha = a.take_n<float>(2 * sr);  // alpha | beta_raw: one stacked GEMV writes both
        beta_raw = alpha + sr;
        act = a.take_n<float>(qkvw);
        decay = a.take_n<float>(sr);
        beta = a.take_n<float>(sr);
        gdn_out = a.take_n<float>(sr * sd);
        q = a.take_n<float>(hq * d);
        gate = a.take_n<float>(hq * d);
        kb = a.take_n<float>(hkv * d);
        vb = a.take_n<float>(hkv * d);
        att = a.take_n<float>(hq * d);
        gated = a.take_n<float>(hq * d);
        rlog = a.take_n<float>(E + 4);  // router logits | the shared expert's gate logit
        sh_logit = rlog + E;
        wts = a.take_n<float>(Kr);
        ids = a.take_n<int32_t>(Kr);
        ea = a.take_n<float>(Kr * FF);
        ey = a.take_n<float>(Kr * H);
        sh_act = a.take_n<float>(SFF);
        sh_y = a.take_n<float>(H);
        moe_part = a.take_n<float>(H);
        logits = a.take_n<float>(V);
        attn_ws_bytes = cl_attn_decode_workspace_bytes((int)hq, (int)d, (int)max_seq);
        attn_ws = a.take(attn_ws_bytes);
        arg_ws_bytes = cl_argmax_workspace_bytes((int)V);
        arg_ws = a.take(arg_ws_bytes);
        ints = a.take_n<int32_t>(16);
        prompt = a.take_n<int32_t>(max_seq);
    }

    void allocate_prefill(Arena& a, std::size_t C) {
        px = a.take_n<float>(C * H);
        pxn = a.take_n<float>(C * H);
        pbig = a.take_n<float>(C * std::max(qkvw, 2 * hq * d));
        pkb = a.take_n<float>(C * hkv * d);
        pvb = a.take_n<float>(C * hkv * d);
        pq = a.take_n<float>(C * hq * d);
        pgate = a.take_n<float>(C * hq * d);
        patt = a.take_n<float>(C * hq * d);
        pgated = a.take_n<float>(C * hq * d);
        pzb = a.take_n<float>(C * sr * sd);
        palpha = a.take_n<float>(C * sr);
        pbetar = a.take_n<float>(C * sr);
        pact = a.take_n<float>(C * qkvw);
        pdecay = a.take_n<float>(C * sr);
        pbeta = a.take_n<float>(C * sr);
        pgdn = a.take_n<float>(C * sr * sd);
        prlog = a.take_n<float>(C * E);
        pwts = a.take_n<float>(C * Kr);
        pids = a.take_n<int32_t>(C * Kr);
        pea = a.take_n<float>(C * Kr * FF);
        pey = a.take_n<float>(C * Kr * H);
        pshl = a.take_n<float>(C + 4);
        psg = a.take_n<float>(C * SFF);
        psu = a.take_n<float>(C * SFF);
        pshy = a.take_n<float>(C * H);
        ppart = a.take_n<float>(C * H);
        pgoff = a.take_n<int32_t>(E_l + 1);
        plist = a.take_n<int32_t>(C * Kr);
        pplanes_bytes = std::max(cl_moe_xq_planes_bytes((int)C, (int)H), cl_moe_xq_planes_bytes((int)(C * Kr), (int)FF));
        pplanes = a.take(pplanes_bytes);
    }

    void ensure_prefill_buffers() {
        if (pre_rows) return;
        std::size_t C = std::min<std::size_t>(max_seq, 512);
        // Diagnostics: smaller chunks exercise the cross-chunk state (conv history, recurrence, KV)
        if (const char* e = std::getenv("CUDALLM_MOE_PREFILL_CHUNK")) {
            const long v = std::strtol(e, nullptr, 10);
            if (v > 0) C = std::min<std::size_t>(C, (std::size_t)v);
        }
        Arena plan;
        allocate_prefill(plan, C);
        pre_mem = DeviceBuffer(plan.used() + 256);
        Arena a;
        a.bind(pre_mem.get(), pre_mem.size());
        allocate_prefill(a, C);
        pre_rows = C;
    }

    // Y[m][n] = X[m][k] W^T (+ residual) on the prefill GEMM (FP32-grade tensor cores)
    void pgemm(const DevMat& w, int n, int k, const float* x, int m, const float* res, float* y) {
        CUDALLM_CL(cl_gemm(w.type, w.ptr, w.stride, n, k, x, m, nullptr, res, y, stream));
    }
    void pgemm_f32(const float* w, int n, int k, const float* x, int m, float* y) {
        CUDALLM_CL(cl_gemm(CL_TYPE_F32, w, (long long)k * 4, n, k, x, m, nullptr, nullptr, y, stream));
    }

    // m prompt tokens (device ids) at positions pos0 .. pos0 + m - 1 through every
    // layer at once: the projections as GEMMs, the DeltaNet conv and recurrence
    // over the chunk in token order within one launch each, the routed experts
    // over all (token, route) pairs in one launch per matrix.  Leaves the
    // chunk's hidden rows in px.
    void prefill_chunk(const int32_t* toks, int m, int pos0) {
        cudaStream_t s = stream;
        const int W = par.world, R = par.rank;
        const int Hi = (int)H;
        CUDALLM_CL(cl_embed(tok_embd.type, tok_embd.ptr, tok_embd.stride, (int)V, Hi, toks, m, px, ints + 4, s));
        for (std::size_t l = 0; l < layers.size(); ++l) {
            MoeLayer& L = layers[l];
            CUDALLM_CL(cl_rmsnorm(px, L.attn_norm, m, Hi, eps(), pxn, nullptr, s));
            if (L.attention) {
                pgemm(L.q_gate, (int)(2 * hq * d), Hi, pxn, m, nullptr, pbig);
                pgemm(L.k, (int)(hkv * d), Hi, pxn, m, nullptr, pkb);
                pgemm(L.v, (int)(hkv * d), Hi, pxn, m, nullptr, pvb);
                CUDALLM_CL(cl_attn_gate_prep_rows(pbig, pkb, pvb, L.q_norm, L.k_norm, (int)hq, (int)hkv, (int)d,
                                                  (int)rot, rope, pos0, m, eps(), pq, pgate, L.k_cache, L.v_cache, s));
                CUDALLM_CL(cl_attn_prefill(pq, L.k_cache, L.v_cache, pos0, m, (int)hq, (int)hkv, (int)d, patt, s));
                CUDALLM_CL(cl_mul_sigmoid(patt, pgate, pgated, (int)(m * hq * d), s));
                pgemm(L.o, Hi, (int)(hq * d), pgated, m, px, px);
            } else {
                pgemm(L.qkv, (int)qkvw, Hi, pxn, m, nullptr, pbig);
                pgemm(L.z, (int)(sr * sd), Hi, pxn, m, nullptr, pzb);
                pgemm_f32(L.alpha_w, (int)sr, Hi, pxn, m, palpha);
                pgemm_f32(L.beta_w, (int)sr, Hi, pxn, m, pbetar);
                CUDALLM_CL(cl_gdn_prep_rows(pbig, palpha, pbetar, L.conv_w, L.hist, L.dt_bias, L.a, (int)sg, (int)sr,
                                            (int)sd, (int)kc, eps(), m, pact, pdecay, pbeta, s));
                CUDALLM_CL(cl_gdn_step_rows(pact, pdecay, pbeta, pzb, L.ssm_norm, L.state, (int)sg, (int)sr, (int)sd,
                                            eps(), m, pgdn, s));
                pgemm(L.out, Hi, (int)(sr * sd), pgdn, m, px, px);
            }
            CUDALLM_CL(cl_rmsnorm(px, L.post_norm, m, Hi, eps(), pxn, nullptr, s));
            pgemm_f32(L.router, (int)E, Hi, pxn, m, prlog);
            CUDALLM_CL(cl_moe_route_rows(prlog, m, (int)E, (int)Kr, pids, pwts, s));
            if (E_l > 0 && grouped_experts) {
                const int routes = (int)(m * Kr), nl = (int)E_l;
                CUDALLM_CL(cl_moe_group_routes(pids, routes, nl, R, W, pgoff, plist, s));
                CUDALLM_CL(cl_moe_expert_gemv_grouped(L.gate_e.type, L.gate_e.ptr, L.up_e.ptr, L.gate_e.stride,
                                                      (int)FF, Hi, pxn, Hi, (int)Kr, pids, routes, R, W, pgoff, plist,
                                                      nl, pplanes, pplanes_bytes, pea, s));
                CUDALLM_CL(cl_moe_expert_gemv_grouped(L.down_e.type, L.down_e.ptr, nullptr, L.down_e.stride, Hi,
                                                      (int)FF, pea, (int)FF, 1, pids, routes, R, W, pgoff, plist, nl,
                                                      pplanes, pplanes_bytes, pey, s));
            } else if (E_l > 0) {
                CUDALLM_CL(cl_moe_expert_gemv_rows(L.gate_e.type, L.gate_e.ptr, L.up_e.ptr, L.gate_e.stride, (int)FF,
                                                   Hi, pxn, Hi, (int)Kr, pids, (int)(m * Kr), R, W, pea, s));
                CUDALLM_CL(cl_moe_expert_gemv_rows(L.down_e.type, L.down_e.ptr, nullptr, L.down_e.stride, Hi, (int)FF,
                                                   pea, (int)FF, 1, pids, (int)(m * Kr), R, W, pey, s));
            }
            const bool shared_here = ep_shared_rank(l, W) == R;
            if (shared_here) {
                pgemm_f32(L.shared_router, 1, Hi, pxn, m, pshl);
                pgemm(L.sh_gate, (int)SFF, Hi, pxn, m, nullptr, psg);
                pgemm(L.sh_up, (int)SFF, Hi, pxn, m, nullptr, psu);
                CUDALLM_CL(cl_swiglu(psg, psu, psg, (long long)m * SFF, s));
                pgemm(L.sh_down, Hi, (int)SFF, psg, m, nullptr, pshy);
            }
            if (W == 1) {
                CUDALLM_CL(cl_moe_combine_rows(pey, pids, pwts, (int)Kr, Hi, 0, 1, pshy, pshl, px, px, m, s));
            } else {
                CUDALLM_CL(cl_moe_combine_rows(pey, pids, pwts, (int)Kr, Hi, R, W, shared_here ? pshy : nullptr,
                                               shared_here ? pshl : nullptr, nullptr, ppart, m, s));
                MOE_NCCL(ncclAllReduce(ppart, ppart, (std::size_t)m * H, ncclFloat32, ncclSum, comm, s));
                CUDALLM_CL(cl_add(px, ppart, px, (long long)m * H, s));
            }
        }
    }

    void init(const std::string& path, std::size_t max_sequence, int dev, const ParallelConfig& parallel) {
        par = parallel;
        if (par.world < 1 || par.rank < 0 || par.rank >= par.world)
            throw std::invalid_argument("invalid parallel rank/world");
        if (dev < 0) CUDALLM_CUDA(cudaGetDevice(&dev));
        device = dev;
        CUDALLM_CUDA(cudaSetDevice(device));
        cudaDeviceProp prop{};
        CUDALLM_CUDA(cudaGetDeviceProperties(&prop, device));
        device_name = prop.name;
        CUDALLM_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
        CUDALLM_CUDA(cudaEventCreate(&ev0));
        CUDALLM_CUDA(cudaEventCreate(&ev1));

        GgufFile file(path);
        config = read_moe_config(file);
        for (std::size_t l = config.layer_count; l < config.layer_count + (std::size_t)file.integer(
                                                                              "qwen35moe.nextn_predict_layers", 0);
             ++l)
            file.ignore_prefix("blk." + std::to_string(l) + ".");
        if (max_sequence == 0) max_sequence = config.context_length;
        if (max_sequence == 0 || max_sequence > config.context_length)
            throw std::invalid_argument("CUDA maximum sequence must be within the model context length");
        max_seq = max_sequence;
        H = config.embedding_size;
        V = config.vocabulary_size;
        E = config.expert_count;
        Kr = config.expert_used_count;
        FF = config.expert_feed_forward_size;
        SFF = config.shared_expert_feed_forward_size;
        hq = config.attention_head_count;
        hkv = config.kv_head_count;
        d = config.head_size;
        rot = config.rotary_dimension;
        sg = config.ssm_group_count;
        sr = config.ssm_time_step_rank;
        sd = config.ssm_state_size;
        kc = config.ssm_conv_kernel;
        qkvw = 2 * sg * sd + config.ssm_inner_size;
        E_l = 0;
        for (std::size_t e = 0; e < E; ++e) E_l += ep_expert_rank(e, par.world) == par.rank;
        if (sd > 128) throw std::runtime_error("DeltaNet state size above 128 is not supported");
        if (d > 256 || d % 32) throw std::runtime_error("attention head size must be a multiple of 32 up to 256");

        if (par.world > 1) {
            ncclUniqueId id;
            std::memcpy(&id, par.nccl_id.data(), sizeof(id));
            MOE_NCCL(ncclCommInitRank(&comm, par.world, id, par.rank));
        }

        Arena plan;
        load_weights(file, plan, false);
        weight_mem = DeviceBuffer(plan.used() + 256);
        {
            GgufFile real_file(path);
            for (std::size_t l = config.layer_count;
                 l < config.layer_count + (std::size_t)real_file.integer("qwen35moe.nextn_predict_layers", 0); ++l)
                real_file.ignore_prefix("blk." + std::to_string(l) + ".");
            Arena wa;
            wa.bind(weight_mem.get(), weight_mem.size());
            load_weights(real_file, wa, true);
        }

        Arena sp;
        allocate_state(sp);
        state_mem = DeviceBuffer(sp.used() + 256);
        Arena sa;
        sa.bind(state_mem.get(), state_mem.size());
        allocate_state(sa);
        for (const MoeLayer& L : layers) {
            if (L.attention)
                kv_bytes += 2 * max_seq * hkv * d * sizeof(float);
            else
                recurrent_bytes += (sr * sd * sd + (kc - 1) * qkvw) * sizeof(float);
        }
        CUDALLM_CUDA(cudaMemsetAsync(state_mem.get(), 0, state_mem.size(), stream));

        Arena ap;
        allocate_activations(ap);
        act_mem = DeviceBuffer(ap.used() + 256);
        Arena aa;
        aa.bind(act_mem.get(), act_mem.size());
        allocate_activations(aa);
        act_bytes = ap.used();
        CUDALLM_CUDA(cudaMemsetAsync(act_mem.get(), 0, act_mem.size(), stream));

        stack_f32();
        pack_head();

        const std::vector<float> table = rope_table_f64(max_seq, rot, (double)config.rope_theta);
        CUDALLM_CUDA(cudaMemcpyAsync(const_cast<float*>(rope), table.data(), table.size() * sizeof(float),
                                     cudaMemcpyHostToDevice, stream));
        host_io = PinnedBuffer(sizeof(int32_t) * (4 + max_seq));
        // Prefill: "batched" (default; chunks of up to 512 tokens through each layer
        // at once) or "serial" (the one-token step replayed per prompt token)
        if (const char* e = std::getenv("CUDALLM_MOE_PREFILL")) {
            const std::string v(e);
            if (v == "serial")
                serial_prefill = true;
            else if (v != "batched" && !v.empty())
                throw std::invalid_argument("CUDALLM_MOE_PREFILL must be batched or serial");
        }
        // Batched prefill's routed experts: "grouped" (default; routes bucketed by
        // expert, each expert's rows read once per layer) or "routes" (one pass
        // of the expert's rows per route); both give the same rows
        if (const char* e = std::getenv("CUDALLM_MOE_EXPERTS")) {
            const std::string v(e);
            if (v == "routes")
                grouped_experts = false;
            else if (v != "grouped" && !v.empty())
                throw std::invalid_argument("CUDALLM_MOE_EXPERTS must be grouped or routes");
        }
        if (E_l >= 4096) grouped_experts = false;  // beyond cl_moe_group_routes' bucket table
        CUDALLM_CUDA(cudaStreamSynchronize(stream));
    }

    // One token through every layer; the token is read from `tok` (device).
    void record_layers(const int32_t* tok) {
        cudaStream_t s = stream;
        const int W = par.world, R = par.rank;
        int* pos = ints + 1;
        int* len = ints + 2;
        const float scale = 1.0f / std::sqrt(static_cast<float>(d));
        CUDALLM_CL(cl_embed(tok_embd.type, tok_embd.ptr, tok_embd.stride, (int)V, (int)H, tok, 1, h, ints + 4, s));
        for (std::size_t l = 0; l < layers.size(); ++l) {
            MoeLayer& L = layers[l];
            if (L.attention) {
                // the input RMSNorm fused into the projections (x is read by them alone)
                const cl_gemv_segment segs[3] = {
                    {L.q_gate.type, L.q_gate.ptr, L.q_gate.stride, L.q_gate.rows, nullptr, nullptr, big},
                    {L.k.type, L.k.ptr, L.k.stride, L.k.rows, nullptr, nullptr, kb},
                    {L.v.type, L.v.ptr, L.v.stride, L.v.rows, nullptr, nullptr, vb},
                };
                CUDALLM_CL(cl_gemv_multi(segs, 3, (int)H, h, L.attn_norm, eps(), s));
                CUDALLM_CL(cl_attn_gate_prep(big, kb, vb, L.q_norm, L.k_norm, (int)hq, (int)hkv, (int)d, (int)rot, rope,
                                             pos, eps(), q, gate, L.k_cache, L.v_cache, s));
                CUDALLM_CL(cl_attn_decode(q, L.k_cache, L.v_cache, len, (int)max_seq, (int)hq, (int)hkv, (int)d, scale,
                                          att, nullptr, attn_ws, attn_ws_bytes, s));
                CUDALLM_CL(cl_mul_sigmoid(att, gate, gated, (int)(hq * d), s));
                CUDALLM_CL(cl_gemv(L.o.type, L.o.ptr, L.o.stride, (int)H, (int)(hq * d), gated, nullptr, h, h, s));
            } else {
                CUDALLM_CL(cl_rmsnorm(h, L.attn_norm, 1, (int)H, eps(), xn, nullptr, s));
                const cl_gemv_segment segs[2] = {
                    {L.qkv.type, L.qkv.ptr, L.qkv.stride, L.qkv.rows, nullptr, nullptr, big},
                    {L.z.type, L.z.ptr, L.z.stride, L.z.rows, nullptr, nullptr, zb},
                };
                CUDALLM_CL(cl_gemv_multi(segs, 2, (int)H, xn, nullptr, 0.0f, s));
                CUDALLM_CL(cl_gemv_f32(stack_ab[l], (int)(2 * sr), (int)H, xn, alpha, s));  // alpha | beta_raw
                CUDALLM_CL(cl_gdn_prep(big, alpha, beta_raw, L.conv_w, L.hist, L.dt_bias, L.a, (int)sg, (int)sr, (int)sd,
                                       (int)kc, eps(), act, decay, beta, s));
                CUDALLM_CL(cl_gdn_step(act, decay, beta, zb, L.ssm_norm, L.state, (int)sg, (int)sr, (int)sd, eps(),
                                       gdn_out, s));
                CUDALLM_CL(cl_gemv(L.out.type, L.out.ptr, L.out.stride, (int)H, (int)(sr * sd), gdn_out, nullptr, h, h, s));
            }
            // MoE: route on device, local experts, shared expert, combine
            CUDALLM_CL(cl_rmsnorm(h, L.post_norm, 1, (int)H, eps(), xn, nullptr, s));
            CUDALLM_CL(cl_gemv_f32(stack_rs[l], (int)(E + 1), (int)H, xn, rlog, s));  // router | shared gate
            CUDALLM_CL(cl_moe_route(rlog, (int)E, (int)Kr, ids, wts, s));
            if (E_l > 0) {
                CUDALLM_CL(cl_moe_expert_gemv(L.gate_e.type, L.gate_e.ptr, L.up_e.ptr, L.gate_e.stride, (int)FF, (int)H,
                                              xn, 0, ids, (int)Kr, R, W, ea, s));
                CUDALLM_CL(cl_moe_expert_gemv(L.down_e.type, L.down_e.ptr, nullptr, L.down_e.stride, (int)H, (int)FF,
                                              ea, (int)FF, ids, (int)Kr, R, W, ey, s));
            }
            const bool shared_here = ep_shared_rank(l, W) == R;
            if (shared_here) {
                CUDALLM_CL(cl_gemv_swiglu(L.sh_gate.type, L.sh_gate.ptr, L.sh_up.ptr, L.sh_gate.stride, (int)SFF,
                                          (int)H, xn, nullptr, 0.0f, sh_act, s));
                CUDALLM_CL(cl_gemv(L.sh_down.type, L.sh_down.ptr, L.sh_down.stride, (int)H, (int)SFF, sh_act, nullptr,
                                   nullptr, sh_y, s));
            }
            if (W == 1) {
                CUDALLM_CL(cl_moe_combine(ey, ids, wts, (int)Kr, (int)H, 0, 1, sh_y, sh_logit, h, h, s));
            } else {
                CUDALLM_CL(cl_moe_combine(ey, ids, wts, (int)Kr, (int)H, R, W, shared_here ? sh_y : nullptr,
                                          shared_here ? sh_logit : nullptr, nullptr, moe_part, s));
                MOE_NCCL(ncclAllReduce(moe_part, moe_part, H, ncclFloat32, ncclSum, comm, s));
                CUDALLM_CL(cl_add(h, moe_part, h, (long long)H, s));
            }
        }
    }

    void record_head() {
        if (head_pk.get()) {
            const cl_gemv_packed_segment seg{out_w.type, head_pk.get(), (int)V, nullptr, nullptr, logits};
            CUDALLM_CL(cl_gemv_packed(&seg, 1, (int)H, h, out_norm, eps(), 0, head_ws.get(), head_ws.size(), stream));
        } else {
            const cl_gemv_segment seg{out_w.type, out_w.ptr, out_w.stride, (int)V, nullptr, nullptr, logits};
            CUDALLM_CL(cl_gemv_multi(&seg, 1, (int)H, h, out_norm, eps(), stream));
        }
        CUDALLM_CL(cl_argmax(logits, (int)V, ints + 3, arg_ws, arg_ws_bytes, stream));
    }

    // decode: token from the host; the greedy token back to the host
    void record_decode() {
        CUDALLM_CUDA(cudaMemcpyAsync(ints, host_in(), sizeof(int32_t), cudaMemcpyHostToDevice, stream));
        record_layers(ints);
        record_head();
        CUDALLM_CL(cl_counter_add(ints + 1, 2, 1, stream));
        CUDALLM_CUDA(cudaMemcpyAsync(host_in() + 1, ints + 3, sizeof(int32_t), cudaMemcpyDeviceToHost, stream));
    }

    // prefill step: token prompt[pos] (device), no LM head
    void record_prefill_step() {
        CUDALLM_CL(cl_select_token(prompt, ints + 1, ints, stream));
        record_layers(ints);
        CUDALLM_CL(cl_counter_add(ints + 1, 2, 1, stream));
    }

    template <typename F>
    cudaGraphExec_t capture(F&& body) {
        cudaGraph_t graph = nullptr;
        CUDALLM_CUDA(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
        try {
            body();
        } catch (...) {
            cudaStreamEndCapture(stream, &graph);
            if (graph) cudaGraphDestroy(graph);
            throw;
        }
        CUDALLM_CUDA(cudaStreamEndCapture(stream, &graph));
        cudaGraphExec_t exec = nullptr;
        const cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        CUDALLM_CUDA(e);
        return exec;
    }

    void begin_timing() {
        call_start = std::chrono::steady_clock::now();
        CUDALLM_CUDA(cudaEventRecord(ev0, stream));
    }

    // Logical, shape-derived FLOPs and bytes of one token through every layer
    // on this rank with `keys` attention keys (routed experts: the expected
    // share Kr * E_l / E of the routes; the shared expert where it runs).
    ProfileMetrics token_metrics(std::size_t keys) const {
        auto el = [](const DevMat& m) { return (std::uint64_t)m.rows * (std::uint64_t)m.cols; };
        ProfileMetrics t;
        const double routes = E ? (double)Kr * (double)E_l / (double)E : 0.0;
        for (std::size_t l = 0; l < layers.size(); ++l) {
            const MoeLayer& L = layers[l];
            std::uint64_t e = 0, b = 0;
            if (L.attention) {
                for (const DevMat* m : {&L.q_gate, &L.k, &L.v, &L.o}) e += el(*m), b += m->payload;
                t.flops += 4 * d * hq * keys;
                b += 2 * keys * hkv * d * sizeof(float);
                t.write_bytes += 2 * hkv * d * sizeof(float);
            } else {
                for (const DevMat* m : {&L.qkv, &L.z, &L.out}) e += el(*m), b += m->payload;
                e += 2 * sr * H;                             // alpha, beta (F32)
                b += (2 * sr * H + qkvw * kc) * sizeof(float);
                const std::uint64_t state = sr * sd * sd * sizeof(float), hist = (kc - 1) * qkvw * sizeof(float);
                t.flops += 8 * sr * sd * sd;                 // decay, prediction, update, output
                b += state + hist;
                t.write_bytes += state + hist;
            }
            e += E * H;  // router (F32)
            b += E * H * sizeof(float);
            if (E_l > 0) {
                e += (std::uint64_t)(routes * (double)(el(L.gate_e) + el(L.up_e) + el(L.down_e)) / (double)E_l);
                b += (std::uint64_t)(routes * (double)(L.gate_e.payload + L.up_e.payload + L.down_e.payload) /
                                     (double)E_l);
            }
            if (ep_shared_rank(l, par.world) == par.rank)
                for (const DevMat* m : {&L.sh_gate, &L.sh_up, &L.sh_down}) e += el(*m), b += m->payload;
            t.flops += 2 * e;
            t.read_bytes += b;
        }
        t.read_bytes += V ? tok_embd.payload / V : 0;  // one embedding row
        return t;
    }

    // prefill of n tokens (n > 0; positions 0..n-1, then the LM head once) or
    // one decode step at the current position (n == 0)
    ProfileMetrics call_metrics(std::size_t n) const {
        ProfileMetrics m;
        const std::size_t first = n > 0 ? 0 : position, count = n > 0 ? n : 1;
        for (std::size_t i = first; i < first + count; ++i) {
            const ProfileMetrics t = token_metrics(i + 1);
            m.flops += t.flops;
            m.read_bytes += t.read_bytes;
            m.write_bytes += t.write_bytes;
        }
        m.flops += 2 * (std::uint64_t)out_w.rows * (std::uint64_t)out_w.cols;
        m.read_bytes += out_w.payload;
        m.write_bytes += 4 * (std::uint64_t)V;
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
            // stage names of the reference's MoE GPU path (moe_llm.mm:3086, 3136)
            profile->forward(pre ? "prefill.gpu_moe" : "decode.gpu_moe", pre ? tokens : position + 1,
                             (std::uint64_t)ns.count(), call_metrics(pre ? tokens : 0));
        }
    }

    void reset_state() {
        // reset() zeroes the DeltaNet state and convolution history
        // (moe_llm.mm:1537-1547); KV rows are overwritten as positions refill.
        CUDALLM_CUDA(cudaSetDevice(device));
        for (const MoeLayer& L : layers) {
            if (L.attention) continue;
            CUDALLM_CUDA(cudaMemsetAsync(L.state, 0, sr * sd * sd * sizeof(float), stream));
            if (kc > 1) CUDALLM_CUDA(cudaMemsetAsync(L.hist, 0, (kc - 1) * qkvw * sizeof(float), stream));
        }
        CUDALLM_CUDA(cudaStreamSynchronize(stream));
        position = 0;
        have_logits = false;
    }

    int32_t prefill(const std::vector<int32_t>& tokens) {
        if (tokens.empty()) throw std::invalid_argument("CUDA prefill requires at least one token");
        if (position != 0) throw std::invalid_argument("CUDA prefill requires an empty conversation; call reset first");
        if (tokens.size() > max_seq) throw std::length_error("CUDA prefill exceeds sequence capacity");
        for (int32_t id : tokens)
            if (id < 0 || (std::size_t)id >= V) throw std::out_of_range("CUDA prefill token id is outside the vocabulary");
        CUDALLM_CUDA(cudaSetDevice(device));
        if (serial_prefill && prefill_exec == nullptr) prefill_exec = capture([&] { record_prefill_step(); });
        if (!serial_prefill) ensure_prefill_buffers();
        const TraceRange trace("prefill.gpu_moe");
        begin_timing();
        int32_t* hi = host_in();
        const std::size_t n = tokens.size();
        std::memcpy(hi + 4, tokens.data(), n * sizeof(int32_t));
        CUDALLM_CUDA(cudaMemcpyAsync(prompt, hi + 4, n * sizeof(int32_t), cudaMemcpyHostToDevice, stream));
        if (serial_prefill) {
            hi[2] = 0;  // position
            hi[3] = 1;  // attention length
            CUDALLM_CUDA(cudaMemcpyAsync(ints + 1, hi + 2, 2 * sizeof(int32_t), cudaMemcpyHostToDevice, stream));
            for (std::size_t i = 0; i < n; ++i) CUDALLM_CUDA(cudaGraphLaunch(prefill_exec, stream));
        } else {
            std::size_t last = 0;
            for (std::size_t c0 = 0; c0 < n; c0 += pre_rows) {
                const int m = (int)std::min(pre_rows, n - c0);
                prefill_chunk(prompt + c0, m, (int)c0);
                last = (std::size_t)m - 1;
            }
            // the last token's hidden state feeds the head; decode continues at position n
            CUDALLM_CUDA(cudaMemcpyAsync(h, px + last * H, H * sizeof(float), cudaMemcpyDeviceToDevice, stream));
            hi[2] = (int32_t)n;
            hi[3] = (int32_t)n + 1;
            CUDALLM_CUDA(cudaMemcpyAsync(ints + 1, hi + 2, 2 * sizeof(int32_t), cudaMemcpyHostToDevice, stream));
        }
        record_head();
        CUDALLM_CUDA(cudaMemcpyAsync(hi + 1, ints + 3, sizeof(int32_t), cudaMemcpyDeviceToHost, stream));
        end_timing("prefill", tokens.size());
        position = tokens.size();
        routed += tokens.size() * layers.size() * Kr;
        have_logits = true;
        return hi[1];
    }

    int32_t decode(int32_t token) {
        if (position == 0) throw std::invalid_argument("CUDA decode requires a completed prefill");
        if (token < 0 || (std::size_t)token >= V) throw std::out_of_range("CUDA decode token id is outside the vocabulary");
        if (position >= max_seq) throw std::length_error("CUDA decode exceeds sequence capacity");
        CUDALLM_CUDA(cudaSetDevice(device));
        if (decode_exec == nullptr) decode_exec = capture([&] { record_decode(); });
        host_in()[0] = token;
        const TraceRange trace("decode.gpu_moe");
        begin_timing();
        CUDALLM_CUDA(cudaGraphLaunch(decode_exec, stream));
        end_timing("decode", 1);
        position += 1;
        routed += layers.size() * Kr;
        have_logits = true;
        return host_in()[1];
    }
};

CudaMoeLLM::CudaMoeLLM(const std::string& gguf_path, std::size_t max_sequence, int device,
                       const ParallelConfig& parallel)
    : impl_(std::make_unique<Impl>()) {
    impl_->init(gguf_path, max_sequence, device, parallel);
}

CudaMoeLLM::~CudaMoeLLM() = default;
CudaMoeLLM::CudaMoeLLM(CudaMoeLLM&&) noexcept = default;
CudaMoeLLM& CudaMoeLLM::operator=(CudaMoeLLM&&) noexcept = default;

void CudaMoeLLM::reset() {
    if (!impl_) throw std::runtime_error("CUDA model is not initialized");
    impl_->reset_state();
}

std::int32_t CudaMoeLLM::prefill(const std::vector<std::int32_t>& token_ids) {
    if (!impl_) throw std::runtime_error("CUDA model is not initialized");
    return impl_->prefill(token_ids);
}

std::int32_t CudaMoeLLM::decode(std::int32_t token_id) {
    if (!impl_) throw std::runtime_error("CUDA model is not initialized");
    return impl_->decode(token_id);
}

void CudaMoeLLM::enable_profiling(const std::string& csv_path, bool) {
    if (!impl_) throw std::runtime_error("CUDA model is not initialized");
    impl_->profile.reset();  // a previous file gets its summary rows first
    impl_->profile = std::make_unique<ProfileCsv>(csv_path);
}

void CudaMoeLLM::disable_profiling() {
    if (impl_) impl_->profile.reset();
}

const ModelConfig& CudaMoeLLM::config() const {
    if (!impl_) throw std::runtime_error("CUDA model is not initialized");
    return impl_->config;
}

std::size_t CudaMoeLLM::position() const noexcept { return impl_ ? impl_->position : 0; }
std::size_t CudaMoeLLM::max_sequence() const noexcept { return impl_ ? impl_->max_seq : 0; }
std::size_t CudaMoeLLM::expert_cache_count() const noexcept { return impl_ ? impl_->E_l : 0; }
ExpertCacheStats CudaMoeLLM::expert_cache_stats() const noexcept {
    ExpertCacheStats s;
    if (impl_) s.hits = impl_->routed;
    return s;
}
bool CudaMoeLLM::uses_gpu() const noexcept { return true; }
bool CudaMoeLLM::available() const noexcept { return impl_ != nullptr; }

const std::string& CudaMoeLLM::device_name() const {
    if (!impl_) throw std::runtime_error("CUDA model is not initialized");
    return impl_->device_name;
}

MemoryStats CudaMoeLLM::memory_stats() const noexcept {
    if (!impl_) return {};
    MemoryStats m;
    m.weight_bytes = impl_->weight_mem.size();
    m.kv_cache_bytes = impl_->kv_bytes;
    m.recurrent_state_bytes = impl_->recurrent_bytes;
    m.intermediate_bytes = impl_->act_bytes;
    m.intermediate_is_estimate = false;
    return m;
}

void CudaMoeLLM::last_logits(float* out, std::size_t n) const {
    if (!impl_ || !impl_->have_logits) throw std::invalid_argument("no logits: call prefill or decode first");
    if (n < impl_->V) throw std::invalid_argument("logits buffer is smaller than the vocabulary");
    CUDALLM_CUDA(cudaSetDevice(impl_->device));
    CUDALLM_CUDA(cudaMemcpy(out, impl_->logits, impl_->V * sizeof(float), cudaMemcpyDeviceToHost));
}

float CudaMoeLLM::last_call_ms() const noexcept { return impl_ ? impl_->last_ms : 0.0f; }
float CudaMoeLLM::last_kernel_ms() const noexcept { return 0.0f; }

}  // namespace cudallm
