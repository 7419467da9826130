/*
 * cudallm_kernels.h — the kernel C-ABI of the CudaLLM backend (sm_100a).
 *
 * Plain C: device pointers, sizes, a cudaStream_t.  Every entry point returns
 * CL_OK (0) or a CL_ERR_* code, never throws, never allocates device memory
 * and never synchronizes; work is enqueued on `stream`.  Kernels needing
 * scratch take a caller-owned workspace whose size a *_workspace_bytes()
 * query reports.
 *
 * Each entry replaces one operator of the reference's Metal shader library
 * (metal_llm.metal) or CPU operator library (cpu_llm.cpp); the reference
 * interface is cited beside each declaration.
 */
#ifndef CUDALLM_KERNELS_H
#define CUDALLM_KERNELS_H

#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CL_API __attribute__((visibility("default")))

/* GGML tensor types (GGUF on-disk ids; metal_model.h:14-29). */
enum {
    CL_TYPE_F32 = 0,
    CL_TYPE_F16 = 1,
    CL_TYPE_Q5_0 = 6,
    CL_TYPE_Q8_0 = 8,
    CL_TYPE_Q4_K = 12,
    CL_TYPE_Q5_K = 13,
    CL_TYPE_Q6_K = 14
};

enum {
    CL_OK = 0,
    CL_ERR_INVALID = 1,     /* bad argument, shape or alignment */
    CL_ERR_UNSUPPORTED = 2, /* type/shape combination not implemented */
    CL_ERR_CUDA = 3,        /* a CUDA launch failed */
    CL_ERR_WORKSPACE = 4,   /* workspace missing or too small */
    CL_ERR_LIMIT = 5        /* request exceeds a fixed built-in scratch size */
};

CL_API const char* cl_status_string(int status);
/* 1 (default): launch with programmatic dependent launch; 0: plain launches. */
CL_API void cl_set_pdl(int enabled);

/* ---- weight layout ---------------------------------------------------- */
/* Native GGUF bytes per row (metal_model.cpp:437-448); -1 if k is not
 * block aligned for `type`. */
CL_API long long cl_native_row_bytes(int type, int k);
/* Row stride of the device layout (native bytes rounded up to 16). */
CL_API long long cl_row_stride(int type, int k);
/* Native rows -> device layout (per-row structure-of-arrays for Q6_K, Q8_0,
 * Q5_0; K-quants Q4_K/Q5_K unchanged).  Replaces upload_matrix
 * (metal_llm.mm:834-862), which kept native bytes. */
CL_API int cl_repack_rows(int type, const void* native, void* packed, int rows, int k,
                          cudaStream_t stream);

/* ---- activation vectors (XQ) ----------------------------------------- */
/* Bytes of the XQ encoding of a k-vector (k % 32 == 0): per 32-block scale
 * and three int8 limbs per element, |error| < max|x_block| * 2^-22. */
CL_API size_t cl_xq_bytes(int k);
CL_API int cl_quantize_xq(const float* x, int k, void* xq, cudaStream_t stream);

/* ---- decode GEMV (metal_gevm_*_f32, metal_llm.metal:708-781; CPU gevmtb
 * cpu_llm.cpp:528-547) ----------------------------------------------------
 * y[n] = W[n,k] . x (+ bias[n]) (+ residual[n]); W in the device layout,
 * x FP32 (16-byte aligned), k % 32 == 0 and k <= 20480.  The kernel encodes
 * x as XQ on the fly (each CTA in registers), so no workspace is needed.
 * y may alias residual (in-place residual add). */
CL_API int cl_gemv(int type, const void* w, long long stride, int n, int k, const float* x,
                   const float* bias, const float* residual, float* y, cudaStream_t stream);

typedef struct {
    int type;
    const void* w;
    long long stride;
    int n;
    const float* bias;
    const float* residual;
    float* y;
} cl_gemv_segment;

/* Up to 4 matrices (any mix of formats) sharing one input vector, e.g. Q, K
 * and V, in one launch.  With norm_gamma != NULL the input is first RMS-
 * normalised (cpu_llm.cpp:143-166: double sum of squares, x*(inv*gamma)). */
CL_API int cl_gemv_multi(const cl_gemv_segment* segs, int nseg, int k, const float* x,
                         const float* norm_gamma, float eps, cudaStream_t stream);
/* y[i] = SiLU(gate_i . x') * (up_i . x'), x' = optional RMSNorm of x: the
 * gate/up GEMV with SwiGLU (cpu_llm.cpp:188-202, metal_swiglu_f32
 * metal_llm.metal:895) fused.  gate and up share type and stride. */
CL_API int cl_gemv_swiglu(int type, const void* w_gate, const void* w_up, long long stride, int n, int k,
                          const float* x, const float* norm_gamma, float eps, float* y, cudaStream_t stream);

/* ---- decode GEMV over fragment-packed K-quant weights (the same products
 * as metal_gevm_q4_k_f32 / metal_gevm_q6_k_f32, metal_llm.metal:708-781,
 * and the CPU gevmt, cpu_llm.cpp:512-547) ------------------------------
 * cl_gemv_pack regroups a Q4_K or Q6_K matrix in the device layout
 * (cl_repack_rows) into units of 16 rows x one super-block, each lane's
 * tensor-core operand bytes contiguous (k % 256 == 0; rows past the last
 * 16-row tile are zero).  With w_up (pair != 0 in the size query) a unit
 * holds 8 gate rows then the same 8 up rows. */
CL_API size_t cl_gemv_pack_bytes(int type, int rows, int k, int pair);
CL_API int cl_gemv_pack(int type, const void* w, long long stride, int rows, int k, const void* w_up, void* out,
                        cudaStream_t stream);
typedef struct cl_gemv_packed_segment {
    int type;     /* CL_TYPE_Q4_K or CL_TYPE_Q6_K */
    const void* w; /* cl_gemv_pack output (16-byte aligned) */
    int n;        /* output rows (SwiGLU: gate rows) */
    const float* bias;
    const float* residual;
    float* y;
} cl_gemv_packed_segment;
/* Workspace of cl_gemv_packed for launches of at most max_tiles 16-row
 * tiles (SwiGLU: 8-row pairs) on the current device.  Zero it once before
 * first use; every launch leaves it re-armed. */
CL_API size_t cl_gemv_packed_workspace_bytes(int max_tiles);
/* y = W x (+ bias) (+ residual) for 1-4 packed matrices sharing x, with x
 * RMS-normalised first when norm_gamma != NULL (cpu_llm.cpp:143-166); with
 * swiglu != 0 one pair-packed matrix and y = SiLU(gate.x') * (up.x')
 * (cpu_llm.cpp:188-202).  k <= 20480.  Deterministic (partial sums are
 * added in a fixed order).  Launches that share a workspace must not
 * overlap on the GPU. */
CL_API int cl_gemv_packed(const cl_gemv_packed_segment* segs, int nseg, int k, const float* x,
                          const float* norm_gamma, float eps, int swiglu, void* workspace, size_t workspace_bytes,
                          cudaStream_t stream);
/* Device error word of the pipelined kernels: non-zero when a bounded wait
 * gave up (never expected): 1-3 from the GEMV, 16 + 1..3 from the
 * tensor-core GEMM, 32 + 1..3 from the 16-bit GEMM.  Synchronous;
 * clear != 0 resets it. */
CL_API int cl_device_error(int* code, int clear);

/* ---- prefill GEMM (metal_gemm_*_f32, metal_llm.metal:621-704; CPU gemmtb
 * cpu_llm.cpp:631-653) ----------------------------------------------------
 * Y[m,n] = X[m,k] W[n,k]^T (+ bias[n]) (+ R[m,n]); X, Y, R row-major FP32.
 * R may alias Y.  The reference computes in FP32; cl_gemm keeps FP32-grade
 * results: tensor cores with split-TF32 operands (CL_GEMM_TF32X3) when
 * k % 32 == 0 and X, W, stride are 16-byte aligned, else the FP32 CUDA-core
 * kernel. */
CL_API int cl_gemm(int type, const void* w, long long stride, int n, int k, const float* x, int m,
                   const float* bias, const float* residual, float* y, cudaStream_t stream);
enum {
    CL_GEMM_TF32X3 = 0, /* operands split hi + lo TF32, 3 MMAs: FP32-grade (k % 32 == 0) */
    CL_GEMM_F16 = 1,    /* operands rounded to FP16, 1 MMA: 11-bit significands (k % 64 == 0) */
    CL_GEMM_BF16 = 2,   /* operands rounded to BF16 (cl_gemm16 path only): 8-bit significands */
    CL_GEMM_F16X3 = 3   /* operands split hi + lo FP16, 3 MMAs: FP32-grade (cl_gemm16 path only) */
};
/* The tcgen05 path with an explicit precision; CL_ERR_UNSUPPORTED for shapes
 * it does not take. */
CL_API int cl_gemm_tc(int type, const void* w, long long stride, int n, int k, const float* x, int m,
                      const float* bias, const float* residual, float* y, int precision, cudaStream_t stream);
/* The FP32 CUDA-core path (exact reference weights, FMA accumulation). */
CL_API int cl_gemm_simt(int type, const void* w, long long stride, int n, int k, const float* x, int m,
                        const float* bias, const float* residual, float* y, cudaStream_t stream);

/* The 16-bit tensor-core prefill path (same product as metal_gemm_*_f32 /
 * gemmtb, operands rounded once to FP16 or BF16, or split into FP16 hi + lo
 * parts; FP32 accumulation):
 *   cl_dequant16  W rows (device layout) -> row-major [n][k] 16-bit, each
 *                 element the CPU decoder's FP32 value rounded once
 *                 (format CL_GEMM_F16 or CL_GEMM_BF16; k % 32 == 0);
 *   cl_convert16  count FP32 values -> 16-bit (count % 4 == 0);
 * and for the split form (CL_GEMM_F16X3), each operand scaled by the power
 * of two that puts its largest magnitude in [2^13, 2^14):
 *   cl_amax_dequant  *amax = max |element| of the dequantized W rows;
 *   cl_amax          *amax = max |x[i]| (count % 4 == 0);
 *   cl_dequant16_split  W rows -> [n][2k] FP16 rows [hi(k) | lo(k)] of the
 *                 scaled values (hi = FP16(v), lo = FP16(v - hi));
 *   cl_split16    X[rows][k] FP32 -> rows [hi(k) | lo(k)] likewise;
 * the outputs of a split product name both maxima (xmax, wmax) and are
 * multiplied by the exact inverse powers of two;
 *   cl_gemm16_run Y = X16[m][k] W16[n][k]^T on tcgen05 (k % 64 == 0; TMA
 *                 tensor loads, 128 x 256 or 128 x 128 tiles, optional K
 *                 split summed in split order).  The n output columns are
 *                 split into nout (1-3) consecutive ranges, each written to
 *                 its own row-major buffer with its own bias / residual (a
 *                 fused Q/K/V or gate/up product).  A K split needs
 *                 cl_gemm16_workspace_bytes(m, n, k) of workspace; with less
 *                 (or none) the product runs unsplit. */
typedef struct cl_gemm_out {
    float* y;              /* [m][ld], columns col0 .. col0 + cols - 1 of the product */
    const float* bias;     /* [cols] or NULL */
    const float* residual; /* [m][ld] or NULL (may alias y) */
    const float *xmax, *wmax; /* split form: device maxima X and these W rows were scaled by; else NULL */
    int col0, cols, ld;
} cl_gemm_out;
CL_API int cl_dequant16(int type, const void* w, long long stride, int n, int k, void* out, int format,
                        cudaStream_t stream);
CL_API int cl_convert16(const float* x, long long count, void* out, int format, cudaStream_t stream);
CL_API int cl_amax_dequant(int type, const void* w, long long stride, int n, int k, float* amax,
                           cudaStream_t stream);
CL_API int cl_amax(const float* x, long long count, float* amax, cudaStream_t stream);
CL_API int cl_dequant16_split(int type, const void* w, long long stride, int n, int k, const float* amax, void* out,
                              cudaStream_t stream);
CL_API int cl_split16(const float* x, int rows, int k, const float* amax, void* out, cudaStream_t stream);
CL_API size_t cl_gemm16_workspace_bytes(int m, int n, int k);
CL_API int cl_gemm16_run(const void* w16, int n, int k, const void* x16, int m, const cl_gemm_out* outs, int nout,
                         int format, void* workspace, size_t workspace_bytes, cudaStream_t stream);

/* ---- activations ------------------------------------------------------ */
/* Row RMSNorm (cpu_llm.cpp:143-166, metal_rmsnorm_f32 metal_llm.metal:785):
 * sum of squares in double, y = x * (1/sqrt(mean+eps) * gamma).  Either
 * output may be NULL; xq gets one XQ vector per row (stride cl_xq_bytes(k)). */
CL_API int cl_rmsnorm(const float* x, const float* gamma, int rows, int k, float eps, float* y,
                      void* xq, cudaStream_t stream);
/* Embedding gather with dequantization (metal_embedding_*, metal_llm.metal:
 * 1066-1162; CPU embedding cpu_llm.cpp:101-123).  Out-of-range ids produce
 * zero rows and set *error_flag = 1 (error_flag may be NULL). */
CL_API int cl_embed(int type, const void* table, long long stride, int vocab, int k, const int32_t* ids,
                    int count, float* out, int* error_flag, cudaStream_t stream);
/* NeoX RoPE from a precomputed [positions][rot/2] cos/sin table plus K/V
 * cache append (metal_rope_heads_f32 + metal_kv_cache_write_f32,
 * metal_llm.metal:928-990; CPU Vector::rope cpu_llm.cpp:204-235).
 * Rows r = 0..rows-1 sit at position pos0 + r, where pos0 = *pos_dev when
 * pos_dev != NULL, else pos_host.  q is rotated in place; k is rotated and,
 * with v, written to cache rows.  Caches are [capacity][kv_heads*head_dim]. */
CL_API int cl_rope_kv(float* q, const float* k, const float* v, int rows, int q_heads, int kv_heads,
                      int head_dim, int rot_dim, const float* cos_sin, const int* pos_dev, int pos_host,
                      float* k_cache, float* v_cache, cudaStream_t stream);
CL_API int cl_swiglu(const float* gate, const float* up, float* out, long long n, cudaStream_t stream);
CL_API int cl_add(const float* a, const float* b, float* out, long long n, cudaStream_t stream);

/* ---- attention --------------------------------------------------------- */
/* Decode GQA attention over the cache (metal_kv_cache_qk/softmax/av,
 * metal_llm.metal:995-1061; CPU gevmts/softmax/gevm cpu_llm.cpp:888-903).
 * Keys 0..len-1 with len = *len_dev (device int) so the call can be captured
 * once in a CUDA graph; max_len bounds len.  out is [q_heads*head_dim];
 * xq (optional) receives its XQ encoding.  Two launches: key splits per KV
 * head (the split length derived from *len_dev on the device), then a merge
 * per query head; concurrent calls must not share a workspace. */
CL_API size_t cl_attn_decode_workspace_bytes(int q_heads, int head_dim, int max_len);
CL_API int cl_attn_decode(const float* q, const float* k_cache, const float* v_cache, const int* len_dev,
                          int max_len, int q_heads, int kv_heads, int head_dim, float scale, float* out,
                          void* xq, void* workspace, size_t workspace_bytes, cudaStream_t stream);
/* cl_attn_decode with the NeoX RoPE of the current position and the KV
 * append fused in (replaces cl_rope_kv + cl_attn_decode for one decode row;
 * cpu_llm.cpp:204-235 rotation, cpu_llm.cpp:885-886 append): q holds the
 * unrotated query [q_heads*head_dim] (left unchanged), k_new / v_new the new
 * key / value [kv_heads*head_dim]; the position is *pos_dev (device int) and
 * the live length *pos_dev + 1; cos_sin is the [capacity][rot_dim/2][2]
 * table.  Writes the rotated key and the value to cache row *pos_dev.
 * Results equal the two separate calls exactly. */
CL_API int cl_attn_decode_rope(const float* q, const float* k_new, const float* v_new, const float* cos_sin,
                               const int* pos_dev, int rot_dim, float* k_cache, float* v_cache, int max_len,
                               int q_heads, int kv_heads, int head_dim, float scale, float* out, void* xq,
                               void* workspace, size_t workspace_bytes, cudaStream_t stream);
/* cl_attn_decode without a workspace argument, for callers that cannot
 * allocate device memory (no counterpart in the reference: MetalLLM and
 * CPULLM allocate their scratch themselves).  The split partials live in a
 * fixed 2 MiB array compiled into the library (held by every GPU that loads
 * it until exit); requests needing more than
 * cl_attn_decode_noalloc_limit_bytes() return CL_ERR_LIMIT.  A request needs
 * cl_attn_decode_workspace_bytes(q_heads, head_dim, max_len) =
 * q_heads * min(32, ceil(max_len / 16)) * (head_dim + 2) * 4 bytes.  The first call on a device
 * looks up the array's device address with that device current; make that
 * first call before any stream capture.  All calls on a device share the
 * array, so calls that overlap on the GPU (e.g. on concurrent streams) race;
 * serialise them.  Allocates nothing (no cudaMalloc/cudaFree). */
CL_API size_t cl_attn_decode_noalloc_limit_bytes(void);
CL_API int cl_attn_decode_noalloc(const float* q, const float* k_cache, const float* v_cache, const int* len_dev,
                                  int max_len, int q_heads, int kv_heads, int head_dim, float scale, float* out,
                                  cudaStream_t stream);
/* Causal prefill attention for rows at positions pos0..pos0+rows-1 against
 * cache rows 0..pos0+rows-1 (CPU gemmts/causal_mask/softmax/gemm,
 * cpu_llm.cpp:816-827).  q, out: [rows][q_heads*head_dim]. */
CL_API int cl_attn_prefill(const float* q, const float* k_cache, const float* v_cache, int pos0, int rows,
                           int q_heads, int kv_heads, int head_dim, float* out, cudaStream_t stream);
/* The same causal prefill attention on the tensor cores: q, k, v and the
 * probabilities rounded to FP16 for mma.sync, FP32 accumulation and
 * softmax (the fast prefill path).  head_dim 128 (else CL_ERR_UNSUPPORTED);
 * q, caches and out 16-byte aligned. */
CL_API int cl_attn_prefill_tc(const float* q, const float* k_cache, const float* v_cache, int pos0, int rows,
                              int q_heads, int kv_heads, int head_dim, float* out, cudaStream_t stream);
/* The same attention FP32-grade on the tensor cores: q, k, v and the
 * probabilities each carried as an FP16 pair (hi + lo, 22 significant
 * bits; probabilities scaled by 2^12 first), every product as three
 * FP16 MMAs (hi.hi + hi.lo + lo.hi) with FP32 accumulation and softmax.
 * head_dim 128 (else CL_ERR_UNSUPPORTED); q, caches and out 16-byte
 * aligned.  The FP32-grade prefill paths use it. */
CL_API int cl_attn_prefill_tc3(const float* q, const float* k_cache, const float* v_cache, int pos0, int rows,
                               int q_heads, int kv_heads, int head_dim, float* out, cudaStream_t stream);

/* ---- greedy token (metal_argmax_partial/finalize_f32, metal_llm.metal:
 * 1544-1644; CPU greedy_token cpu_llm.cpp:34-48) -------------------------
 * *token = argmax(logits[0..n)), lowest index on ties.  Single pass: the
 * last CTA to finish reduces the per-CTA partials and re-arms the workspace
 * (zeroed once by the caller before first use). */
CL_API size_t cl_argmax_workspace_bytes(int n);
CL_API int cl_argmax(const float* logits, int n, int32_t* token, void* workspace, size_t workspace_bytes,
                     cudaStream_t stream);
/* Shard form for a vocabulary split across ranks: *token = local argmax +
 * index_offset and *value = its logit (value may be NULL). */
CL_API int cl_argmax_ex(const float* logits, int n, int index_offset, int32_t* token, float* value,
                        void* workspace, size_t workspace_bytes, cudaStream_t stream);
/* Merge n (value, index-bits) records gathered from the shards: highest
 * value, lowest index on ties. */
CL_API int cl_argmax_merge(const float* records, int n, int32_t* token, cudaStream_t stream);

/* counters[0..n) += delta on the device (position bookkeeping inside a
 * captured decode graph). */
CL_API int cl_counter_add(int* counters, int n, int delta, cudaStream_t stream);

/* ---- one decode step of a qwen2 model in one launch ------------------------
 * The whole batch-1 decode step of cpu_decode_layer x n_layers + the head
 * (cpu_llm.cpp:843-914, 1051-1070; Metal encode_decode_layer,
 * metal_llm.mm:2758-2904): embedding row of ints[0], per layer RMSNorm ->
 * Q/K/V (+bias) -> NeoX RoPE -> KV append at ints[1] -> GQA attention over
 * keys 0..ints[1] -> o_proj + residual -> RMSNorm -> gate/up -> SwiGLU ->
 * down + residual, then RMSNorm -> LM head -> greedy token (lowest index on
 * ties) into ints[3]; ints[1] advances by one.  The same products and
 * expressions as the per-operator entry points (the GEMVs' exact integer
 * dots, the RMSNorm sum in double), in one persistent cooperative launch
 * with one CTA per SM: every warp streams its share of each weight matrix
 * through its own shared-memory ring and keeps loading the next matrix while
 * the grid waits at the barrier between two products.
 *
 * Supported: every layer matrix Q4_K or Q6_K (gate and up one type), hidden,
 * ffn % 256 == 0, output rows % 16 == 0, head_dim 128 with RoPE over the
 * whole head, q_heads / kv_heads <= 8, kv_heads <= 32, hidden <= 6144,
 * ffn <= 20480; else CL_ERR_UNSUPPORTED (use the per-operator path).
 * `layers` is a device array of n_layers entries; `host_layers` the same
 * table in host memory (checked here).  Every layer matrix and out_w is in
 * the tiled decode layout of cl_decode_pack (gate: the pack of gate and up
 * together; `up` is not read); embd stays in the device layout
 * (cl_repack_rows).  The workspace (cl_qwen2_decode_workspace_bytes, for
 * the current device) must be zeroed once by cl_qwen2_decode_init; every
 * step leaves it re-armed.  If a grid barrier wait runs out (2 s) the step
 * stops, and cl_qwen2_decode_status reports it (a device int: 0 = ok,
 * else 1 + the phase); re-run cl_qwen2_decode_init before the next step. */
typedef struct cl_qwen2_layer {
    const void *q, *k, *v, *o, *gate, *up, *down;
    const float *q_bias, *k_bias, *v_bias, *attn_norm, *ffn_norm;
    float *k_cache, *v_cache; /* [capacity][kv_heads * head_dim], K after RoPE */
    int q_type, k_type, v_type, o_type, gate_type, down_type;
    int reserved[2];
} cl_qwen2_layer;

typedef struct cl_qwen2_decode {
    const cl_qwen2_layer* layers; /* device array [n_layers] */
    int n_layers, hidden, ffn, vocab, q_heads, kv_heads, head_dim, capacity;
    float eps, scale;             /* RMSNorm epsilon; attention scale 1/sqrt(head_dim) */
    const void* embd;             /* token_embd rows (device layout) */
    long long embd_stride;
    int embd_type, out_type;
    const void* out_w;            /* output.weight rows */
    const float* out_norm;
    const float* rope;            /* [capacity][head_dim / 2][cos, sin] */
    int* ints;                    /* [0] token in, [1] position, [3] token out */
    float *h, *q, *k, *v, *att, *act, *logits; /* [hidden], [q_heads*d], [kv*d] x2, [q_heads*d], [ffn], [vocab] */
    long long* trace;             /* optional (NULL): [grid][5 n_layers + 1][16] %globaltimer stamps per CTA
                                     and phase: start, input ready, work done, then points inside the phase
                                     (projection phases: warp 0's cycles waiting, computing, issuing,
                                     flushing, and its unit count) */
    int attn_splits;              /* key splits per KV head in attention, 0..32; 0 = automatic (one per 16
                                     keys, at most 32 and at most SMs / kv_heads) */
} cl_qwen2_decode;

/* The tiled decode layout of one matrix: its device-layout rows
 * (cl_repack_rows) regrouped so that each unit the step streams is one
 * contiguous block: Q4_K 16 rows x two super-blocks (2 x 144 bytes; an odd
 * last one padded with a zero super-block), Q6_K 16 rows x one super-block
 * as two 112-byte halves (ql, qh, sc of the half, f16 d, zero pad).  With
 * w_up (pair != 0 for the size query) the gate and up rows are interleaved
 * 8 by 8.  rows % 16 == 0 (pair: % 8), k % 256 == 0. */
CL_API size_t cl_decode_pack_bytes(int type, int rows, int k, int pair);
CL_API int cl_decode_pack(int type, const void* w, long long stride, int rows, int k, const void* w_up, void* out,
                          cudaStream_t stream);
CL_API int cl_qwen2_decode_supported(const cl_qwen2_decode* m, const cl_qwen2_layer* host_layers);
CL_API size_t cl_qwen2_decode_workspace_bytes(const cl_qwen2_decode* m);
CL_API int cl_qwen2_decode_init(void* workspace, size_t workspace_bytes, cudaStream_t stream);
CL_API int cl_qwen2_decode_step(const cl_qwen2_decode* m, const cl_qwen2_layer* host_layers, void* workspace,
                                size_t workspace_bytes, cudaStream_t stream);
CL_API const int* cl_qwen2_decode_status(const void* workspace);

/* ---- tensor-parallel exchange over peer memory --------------------------- */
/* One-shot all-reduce (sum) of a decode-size FP32 vector across up to 8 ranks
 * of one node, through exchange buffers that every rank maps from every
 * other (CUDA IPC over NVLink / NVSwitch).  It replaces the NCCL all-reduce
 * after the row-split o_proj and ffn_down products of a tensor-parallel
 * decode token; the reference has no multi-GPU path (its layer computes the
 * unsplit products, cpu_llm.cpp:774-914).
 *
 * Each rank allocates one buffer of cl_peer_exchange_bytes(max_n) bytes with
 * cudaMalloc (256-byte aligned), zeroes its header once with
 * cl_peer_exchange_init before any rank's first call, and shares it by IPC
 * handle.  buffers[r] = rank r's buffer as mapped in this process
 * (buffers[rank] = its own).  Every rank makes the same calls in the same
 * order.  n % 4 == 0, n <= max_n (the max_n the buffers were sized for), in
 * and out 16-byte aligned and not overlapping.  out receives the sum in rank
 * order 0..world-1, bit-identical on every rank.  A rank that waits longer
 * than the wait limit (20 s unless cl_peer_set_wait_limit_ns changed it) for
 * the others sets the buffer's status word (cl_peer_exchange_status: a
 * device address; 0 = ok), skips the sum and returns; re-initialise every
 * rank's buffer (cl_peer_exchange_init) before the ranks exchange again.
 * cl_peer_set_wait_limit_ns sets the limit for later launches of this
 * process (1 ms .. 120 s, else CL_ERR_INVALID); it has no counterpart in
 * the reference. */
CL_API size_t cl_peer_exchange_bytes(int max_n);
CL_API int cl_peer_exchange_init(void* buffer, int max_n, cudaStream_t stream);
CL_API const int* cl_peer_exchange_status(const void* buffer);
CL_API int cl_peer_allreduce(const float* in, float* out, int n, int max_n, int rank, int world,
                             void* const* buffers, cudaStream_t stream);
CL_API int cl_peer_set_wait_limit_ns(unsigned long long ns);

/* ---- qwen35moe ---------------------------------------------------------- */
/* y[n] = W[n,k] x for an FP32 row-major W (the router, DeltaNet alpha/beta
 * and shared-expert gate products, encode_product on F32 tensors,
 * moe_llm.mm:2642-2690, 2476-2490, 2820-2824); k % 4 == 0. */
CL_API int cl_gemv_f32(const float* w, int n, int k, const float* x, float* y, cudaStream_t stream);
/* Router: softmax over n_experts logits, top-k by strict '>' (lower expert
 * id first on ties), the k probabilities renormalised to sum 1
 * (metal_softmax_f32 + metal_topk_f32 + metal_topk_renorm_f32,
 * metal_llm.metal:826-890, 1424-1474).  ids / weights: device [k], k <= 8. */
CL_API int cl_moe_route(const float* logits, int n_experts, int k, int32_t* ids, float* weights,
                        cudaStream_t stream);
/* Routed expert product (metal_expert_gemm_{q4_k,q6_k}_f32, metal_llm.metal:
 * 1476-1524): for route r < routes, expert e = ids[r] (device),
 * y[r][i] = W_e[i] . x_r with x_r = x + r * x_stride (x_stride 0: one shared
 * input).  w holds this rank's experts e % world == rank as consecutive
 * [n, k] blocks (local index e / world); routes of other ranks are skipped.
 * With w_up != NULL the SwiGLU silu(W_e[i] . x) * (U_e[i] . x) is stored.
 * Precondition: every ids[r] lies in [0, experts) for the expert count the
 * stacked w was built for, as cl_moe_route produces them.  The ids are read
 * on the device, where the kernel has no expert count to check them
 * against, so another value would index outside w. */
CL_API int cl_moe_expert_gemv(int type, const void* w, const void* w_up, long long stride, int n, int k,
                              const float* x, int x_stride, const int32_t* ids, int routes, int rank, int world,
                              float* y, cudaStream_t stream);
/* out = residual + (sum_r weights[r] y[r] + sigmoid(*shared_logit) shared_y)
 * over this rank's routes (metal_expert_weighted_reduce_f32 + row scale +
 * residual, moe_llm.mm:2786-2843); residual and the shared pair may be NULL.
 * out may alias residual. */
CL_API int cl_moe_combine(const float* y, const int32_t* ids, const float* weights, int routes, int n, int rank,
                          int world, const float* shared_y, const float* shared_logit, const float* residual,
                          float* out, cudaStream_t stream);
/* Gated DeltaNet, one token (moe_llm.mm:2436-2640): causal depthwise conv of
 * qkv [(2 key_heads + value_heads) * head_dim] over the conv_kernel - 1
 * history rows (hist, updated) with conv_w [channels][conv_kernel], SiLU,
 * L2 norm of each q / k head (metal_llm.metal:1288-1420) -> act; and
 * decay = exp(softplus(alpha + dt_bias) * a), beta = sigmoid(beta_raw). */
CL_API int cl_gdn_prep(const float* qkv, const float* alpha, const float* beta_raw, const float* conv_w, float* hist,
                       const float* dt_bias, const float* a, int key_heads, int value_heads, int head_dim,
                       int conv_kernel, float eps, float* act, float* decay, float* beta, cudaStream_t stream);
/* The delta-rule step per value head h (key head h % key_heads) on
 * state [value_heads][head_dim][head_dim] (metal_gdn_recurrence_f32,
 * metal_llm.metal:1366-1420), then RMSNorm(o; gamma) * silu(z); head_dim <= 128. */
CL_API int cl_gdn_step(const float* act, const float* decay, const float* beta, const float* z, const float* gamma,
                       float* state, int key_heads, int value_heads, int head_dim, float eps, float* out,
                       cudaStream_t stream);
/* Gated attention prologue (moe_llm.mm:2238-2363): split the packed
 * [query, gate] heads of mixed, RMSNorm q and k per head, NeoX RoPE on the
 * first rot_dim dims from cos_sin [positions][rot_dim/2][2] at *pos_dev, and
 * append k / v to the caches at *pos_dev. */
CL_API int cl_attn_gate_prep(const float* mixed, const float* k_raw, const float* v_raw, const float* q_norm,
                             const float* k_norm, int q_heads, int kv_heads, int head_dim, int rot_dim,
                             const float* cos_sin, const int* pos_dev, float eps, float* q_out, float* gate_out,
                             float* k_cache, float* v_cache, cudaStream_t stream);
/* Token-batched forms for prefill, `rows` consecutive tokens at once (the
 * per-token arithmetic and its order unchanged):
 *   cl_moe_route_rows       logits [rows][n_experts] -> ids / weights [rows][k];
 *   cl_moe_expert_gemv_rows routes r < routes with x_r = x + (r / x_group) *
 *                           x_stride (x_group routes per token share its row);
 *   cl_moe_combine_rows     token t: y rows [t routes, (t + 1) routes), ids /
 *                           weights [t][routes], shared_y / residual / out
 *                           row t, shared_logit[t];
 *   cl_gdn_prep_rows        qkv [rows][channels], alpha / beta_raw
 *                           [rows][value_heads]: the conv over the history and
 *                           the chunk in token order (hist left holding the
 *                           chunk's last conv_kernel - 1 rows), act / decay /
 *                           beta per token;
 *   cl_gdn_step_rows        the recurrence over the rows in order, the state
 *                           held on chip between tokens (z / out
 *                           [rows][value_heads * head_dim]; head_dim % 32 == 0,
 *                           head_dim <= 128);
 *   cl_attn_gate_prep_rows  token t at position pos0 + t. */
CL_API int cl_moe_route_rows(const float* logits, int rows, int n_experts, int k, int32_t* ids, float* weights,
                             cudaStream_t stream);
CL_API int cl_moe_expert_gemv_rows(int type, const void* w, const void* w_up, long long stride, int n, int k,
                                   const float* x, int x_stride, int x_group, const int32_t* ids, int routes,
                                   int rank, int world, float* y, cudaStream_t stream);
/* Grouped form of cl_moe_expert_gemv_rows for prefill: the routes of a
 * prompt chunk evaluated expert by expert (the reference's per-expert
 * evaluation of a prompt's (token, expert) pairs, moe_llm.mm:2692-2843 and
 * 3087-3108), so an expert's rows are read from HBM once per launch rather
 * than once per route, and each input row is encoded once.
 *   cl_moe_group_routes      buckets this rank's routes (ids[r] % world ==
 *                            rank) by local expert ids[r] / world:
 *                            offsets [n_local + 1] (offsets[e] .. offsets[e+1]
 *                            index `list`), list [routes] (route indices; the
 *                            order within an expert is unspecified).
 *                            1 <= n_local <= 4095.  Once per layer: the gate/up
 *                            and the down product share it;
 *   cl_moe_expert_gemv_grouped  y rows of this rank's routes, each equal to
 *                            what cl_moe_expert_gemv_rows writes for the same
 *                            arguments (same unit dots in the same order);
 *                            offsets / list / n_local from cl_moe_group_routes
 *                            over the same ids; planes = scratch of
 *                            cl_moe_xq_planes_bytes(ceil(routes / x_group), k)
 *                            bytes (the XQ encoding of each input row). */
CL_API size_t cl_moe_xq_planes_bytes(int inputs, int k);
CL_API int cl_moe_group_routes(const int32_t* ids, int routes, int n_local, int rank, int world, int32_t* offsets,
                               int32_t* list, cudaStream_t stream);
CL_API int cl_moe_expert_gemv_grouped(int type, const void* w, const void* w_up, long long stride, int n, int k,
                                      const float* x, int x_stride, int x_group, const int32_t* ids, int routes,
                                      int rank, int world, const int32_t* offsets, const int32_t* list, int n_local,
                                      void* planes, size_t planes_bytes, float* y, cudaStream_t stream);
CL_API int cl_moe_combine_rows(const float* y, const int32_t* ids, const float* weights, int routes, int n, int rank,
                               int world, const float* shared_y, const float* shared_logit, const float* residual,
                               float* out, int rows, cudaStream_t stream);
CL_API int cl_gdn_prep_rows(const float* qkv, const float* alpha, const float* beta_raw, const float* conv_w,
                            float* hist, const float* dt_bias, const float* a, int key_heads, int value_heads,
                            int head_dim, int conv_kernel, float eps, int rows, float* act, float* decay, float* beta,
                            cudaStream_t stream);
CL_API int cl_gdn_step_rows(const float* act, const float* decay, const float* beta, const float* z,
                            const float* gamma, float* state, int key_heads, int value_heads, int head_dim, float eps,
                            int rows, float* out, cudaStream_t stream);
CL_API int cl_attn_gate_prep_rows(const float* mixed, const float* k_raw, const float* v_raw, const float* q_norm,
                                  const float* k_norm, int q_heads, int kv_heads, int head_dim, int rot_dim,
                                  const float* cos_sin, int pos0, int rows, float eps, float* q_out, float* gate_out,
                                  float* k_cache, float* v_cache, cudaStream_t stream);
/* *out = ids[*index_dev] (the next prompt token inside a captured prefill step). */
CL_API int cl_select_token(const int32_t* ids, const int* index_dev, int32_t* out, cudaStream_t stream);
/* out = a * sigmoid(g) (the attention output gate, moe_llm.mm:2420-2429). */
CL_API int cl_mul_sigmoid(const float* a, const float* g, float* out, int n, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* CUDALLM_KERNELS_H */
