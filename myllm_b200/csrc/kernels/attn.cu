// GQA attention over the FP32 KV cache.
//
// Decode: flash-decoding.  CTA (kv head, key split) scores the group's query
// heads against <= kKeysPerSplit keys, keeps an unnormalised softmax partial
// (max, sum, sum p*V) in the workspace; a combine kernel merges the splits,
// normalises and emits the head outputs (and their XQ encoding for the
// o_proj GEMV).  Reference: metal_kv_cache_qk/softmax/av (metal_llm.metal:
// 995-1061, 826-890) and cpu_decode_layer's gevmts/softmax/gevm
// (cpu_llm.cpp:888-903): score = (q.k) * (1/sqrt(d)), head h uses KV head
// h / (q_heads / kv_heads).
//
// Prefill: causal flash attention in FP32, one CTA per (query head, 32-row
// query tile), online softmax over 32-key tiles; no [N, N] score matrix.
// Reference: cpu_prefill_layer (cpu_llm.cpp:816-827): score = (q.k)/sqrt(d),
// keys after the query position masked.
#include "common.cuh"
#include "launch.cuh"

#include <mutex>

namespace cl {

constexpr int kKeysPerSplit = 64;   // decode split size (keys)
constexpr int kDecThreads = 128;
constexpr int kMaxGroup = 16;
constexpr int kMaxHeadDim = 256;

__host__ __device__ inline int attn_splits(int max_len) { return (max_len + kKeysPerSplit - 1) / kKeysPerSplit; }

// Dynamic smem: q [group][d] | tile [64][d + 4] (K, then V) | p [group][64] | stats [group][2]
__host__ __device__ inline size_t attn_decode_smem(int group, int d) {
    return sizeof(float) * ((size_t)group * d + (size_t)kKeysPerSplit * (d + 4) + (size_t)group * kKeysPerSplit +
                            2 * group);
}

// partial record per (q head, split): [m, l, o[d]] with o unnormalised
__global__ void __launch_bounds__(kDecThreads)
attn_decode_split(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
                  const int* __restrict__ len_dev, int hq, int hkv, int d, float scale,
                  float* __restrict__ part) {
    grid_launch_dependents();
    grid_wait();
    const int g = blockIdx.x, split = blockIdx.y, splits = gridDim.y;
    const int group = hq / hkv;
    const int L = *len_dev;
    const int k0 = split * kKeysPerSplit;
    const int nk = min(kKeysPerSplit, L - k0);
    const int rec = d + 2;
    if (nk <= 0) return;  // the combine kernel only reads splits below ceil(L / 64)
    extern __shared__ __align__(16) float sm[];
    float* qs = sm;                                    // [group][d]
    float* tile = qs + group * d;                      // [64][d + 4]
    float* ps = tile + kKeysPerSplit * (d + 4);        // [group][64]
    float* st = ps + group * kKeysPerSplit;            // [group][2]
    const int kvd = hkv * d, d4 = d / 4, ld = d + 4;
    for (int i = threadIdx.x; i < group * d4; i += kDecThreads)
        reinterpret_cast<float4*>(qs)[i] = reinterpret_cast<const float4*>(q + (size_t)g * group * d)[i];
    // K tile, coalesced float4 rows into padded smem rows
    for (int i = threadIdx.x; i < nk * d4; i += kDecThreads) {
        const int t = i / d4, c = i % d4;
        *reinterpret_cast<float4*>(tile + t * ld + 4 * c) =
            reinterpret_cast<const float4*>(kc + (size_t)(k0 + t) * kvd + (size_t)g * d)[c];
    }
    __syncthreads();
    // scores: thread t -> key t, all heads of the group (q reads broadcast)
    if (threadIdx.x < nk) {
        const int t = threadIdx.x;
        float acc[kMaxGroup];
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) acc[h] = 0.0f;
        for (int c = 0; c < d4; ++c) {
            const float4 kv = *reinterpret_cast<const float4*>(tile + t * ld + 4 * c);
#pragma unroll
            for (int h = 0; h < kMaxGroup; ++h) {
                if (h < group) {
                    const float4 qv = reinterpret_cast<const float4*>(qs + h * d)[c];
                    acc[h] += kv.x * qv.x;
                    acc[h] += kv.y * qv.y;
                    acc[h] += kv.z * qv.z;
                    acc[h] += kv.w * qv.w;
                }
            }
        }
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h)
            if (h < group) ps[h * kKeysPerSplit + t] = acc[h] * scale;
    }
    __syncthreads();
    // V tile into the same buffer; per-head max/exp-sum meanwhile
    for (int i = threadIdx.x; i < nk * d4; i += kDecThreads) {
        const int t = i / d4, c = i % d4;
        *reinterpret_cast<float4*>(tile + t * ld + 4 * c) =
            reinterpret_cast<const float4*>(vc + (size_t)(k0 + t) * kvd + (size_t)g * d)[c];
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int h = warp; h < group; h += kDecThreads / 32) {
        float m = -INFINITY;
        for (int t = lane; t < nk; t += 32) m = fmaxf(m, ps[h * kKeysPerSplit + t]);
        m = warp_max(m);
        float l = 0.0f;
        for (int t = lane; t < nk; t += 32) {
            const float e = expf(ps[h * kKeysPerSplit + t] - m);
            ps[h * kKeysPerSplit + t] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) {
            st[2 * h] = m;
            st[2 * h + 1] = l;
        }
    }
    __syncthreads();
    // p . V: thread -> output dims
    for (int dim = threadIdx.x; dim < d; dim += kDecThreads) {
        float acc[kMaxGroup];
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) acc[h] = 0.0f;
        for (int t = 0; t < nk; ++t) {
            const float vv = tile[t * ld + dim];
#pragma unroll
            for (int h = 0; h < kMaxGroup; ++h)
                if (h < group) acc[h] += ps[h * kKeysPerSplit + t] * vv;
        }
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) {
            if (h < group) {
                float* pr = part + ((size_t)(g * group + h) * splits + split) * rec;
                pr[2 + dim] = acc[h];
                if (dim == 0) {
                    pr[0] = st[2 * h];
                    pr[1] = st[2 * h + 1];
                }
            }
        }
    }
}

__global__ void attn_decode_combine(const float* __restrict__ part, const int* __restrict__ len_dev, int splits,
                                    int d, float* __restrict__ out, void* xq, int xq_k) {
    grid_launch_dependents();
    grid_wait();
    const int h = blockIdx.x;
    const int L = *len_dev;
    const int used = min(splits, attn_splits(L));
    const int rec = d + 2;
    const float* pr = part + (size_t)h * splits * rec;
    float m = -INFINITY;
    for (int s = 0; s < used; ++s) m = fmaxf(m, pr[(size_t)s * rec]);
    float l = 0.0f;
    for (int s = 0; s < used; ++s) l += pr[(size_t)s * rec + 1] * expf(pr[(size_t)s * rec] - m);
    const float inv = 1.0f / l;
    XQMut q{};
    if (xq) q = xq_mut(xq, xq_k);
    for (int dim = threadIdx.x; dim < d; dim += blockDim.x) {
        float o = 0.0f;
        for (int s = 0; s < used; ++s) o += pr[(size_t)s * rec + 2 + dim] * expf(pr[(size_t)s * rec] - m);
        o *= inv;
        out[(size_t)h * d + dim] = o;
        if (xq) xq_store_block_warp(q, (h * d + dim) / 32, o);
    }
}

// ---- prefill -------------------------------------------------------------------
constexpr int kQT = 32;   // query rows per CTA
constexpr int kKT = 32;   // keys per tile
constexpr int kPreThreads = 256;

__global__ void __launch_bounds__(kPreThreads)
attn_prefill_kernel(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
                    int pos0, int rows, int hq, int hkv, int d, float* __restrict__ out) {
    grid_launch_dependents();
    grid_wait();
    extern __shared__ __align__(16) float sm[];
    float* Qs = sm;                      // [kQT][d]
    float* Ks = Qs + kQT * d;            // [kKT][d + 1]
    float* Vs = Ks + kKT * (d + 1);      // [kKT][d]
    float* Ps = Vs + kKT * d;            // [kQT][kKT + 1]
    float* Ms = Ps + kQT * (kKT + 1);    // [kQT] running max
    float* Ls = Ms + kQT;                // [kQT] running sum
    float* As = Ls + kQT;                // [kQT] rescale factor
    const int h = blockIdx.x, qt = blockIdx.y;
    const int g = h / (hq / hkv);
    const int r0 = qt * kQT;
    const int nq = min(kQT, rows - r0);
    const int qd = hq * d, kvd = hkv * d;
    const float sqrt_d = sqrtf((float)d);
    for (int i = threadIdx.x; i < kQT * d; i += kPreThreads) {
        const int r = i / d, c = i % d;
        Qs[i] = r < nq ? q[(size_t)(r0 + r) * qd + (size_t)h * d + c] : 0.0f;
    }
    if (threadIdx.x < kQT) {
        Ms[threadIdx.x] = -INFINITY;
        Ls[threadIdx.x] = 0.0f;
    }
    const int orow = threadIdx.x / 8, olane = threadIdx.x % 8;
    const int per = d / 8;  // dims per thread
    float o[kMaxHeadDim / 8];
#pragma unroll
    for (int j = 0; j < kMaxHeadDim / 8; ++j) o[j] = 0.0f;
    const int last_key = pos0 + r0 + nq - 1;  // inclusive
    const int tiles = last_key / kKT + 1;
    for (int kt = 0; kt < tiles; ++kt) {
        const int kb = kt * kKT;
        __syncthreads();
        for (int i = threadIdx.x; i < kKT * d; i += kPreThreads) {
            const int r = i / d, c = i % d;
            const int key = kb + r;
            const bool ok = key <= last_key;
            Ks[r * (d + 1) + c] = ok ? kc[(size_t)key * kvd + (size_t)g * d + c] : 0.0f;
            Vs[r * d + c] = ok ? vc[(size_t)key * kvd + (size_t)g * d + c] : 0.0f;
        }
        __syncthreads();
        // scores: thread -> row orow, keys olane*4 .. +3
        for (int jj = 0; jj < 4; ++jj) {
            const int j = olane * 4 + jj;
            float acc = 0.0f;
            const float* qr = Qs + orow * d;
            const float* kr = Ks + j * (d + 1);
            for (int c = 0; c < d; ++c) acc += qr[c] * kr[c];
            const int qpos = pos0 + r0 + orow;
            Ps[orow * (kKT + 1) + j] = (kb + j <= qpos && orow < nq) ? acc / sqrt_d : -INFINITY;
        }
        __syncthreads();
        // online softmax: warp w -> rows 4w..4w+3, lane -> key
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int rr = 0; rr < 4; ++rr) {
            const int r = warp * 4 + rr;
            const float s = Ps[r * (kKT + 1) + lane];
            const float mold = Ms[r];
            const float mnew = fmaxf(mold, warp_max(s));
            const float p = mnew == -INFINITY ? 0.0f : expf(s - mnew);
            const float psum = warp_sum(p);
            Ps[r * (kKT + 1) + lane] = p;
            if (lane == 0) {
                const float a = mold == -INFINITY ? 0.0f : expf(mold - mnew);
                As[r] = a;
                Ls[r] = Ls[r] * a + psum;
                Ms[r] = mnew;
            }
        }
        __syncthreads();
        const float a = As[orow];
#pragma unroll
        for (int j = 0; j < kMaxHeadDim / 8; ++j) {
            if (j < per) {
                const int dim = olane + 8 * j;
                float acc = o[j] * a;
                for (int kk = 0; kk < kKT; ++kk) acc += Ps[orow * (kKT + 1) + kk] * Vs[kk * d + dim];
                o[j] = acc;
            }
        }
    }
    if (orow < nq) {
        const float inv = 1.0f / Ls[orow];
#pragma unroll
        for (int j = 0; j < kMaxHeadDim / 8; ++j) {
            if (j < per) out[(size_t)(r0 + orow) * qd + (size_t)h * d + olane + 8 * j] = o[j] * inv;
        }
    }
}

}  // namespace cl

using namespace cl;

extern "C" {

CL_API size_t cl_attn_decode_workspace_bytes(int q_heads, int head_dim, int max_len) {
    if (q_heads <= 0 || head_dim <= 0 || max_len <= 0) return 0;
    return (size_t)q_heads * attn_splits(max_len) * (head_dim + 2) * sizeof(float);
}

CL_API int cl_attn_decode(const float* q, const float* k_cache, const float* v_cache, const int* len_dev,
                          int max_len, int q_heads, int kv_heads, int head_dim, float scale, float* out, void* xq,
                          void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (q == nullptr || k_cache == nullptr || v_cache == nullptr || len_dev == nullptr || out == nullptr ||
        max_len <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads || q_heads / kv_heads > kMaxGroup ||
        head_dim <= 0 || head_dim % 32 || head_dim > kMaxHeadDim)
        return CL_ERR_INVALID;
    if (workspace == nullptr || workspace_bytes < cl_attn_decode_workspace_bytes(q_heads, head_dim, max_len))
        return CL_ERR_WORKSPACE;
    const int splits = attn_splits(max_len);
    float* part = static_cast<float*>(workspace);
    const size_t smem = attn_decode_smem(q_heads / kv_heads, head_dim);
    static int configured_for = 0;
    if ((int)smem > configured_for) {
        if (cudaFuncSetAttribute(attn_decode_split, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return CL_ERR_CUDA;
        configured_for = (int)smem;
    }
    if (launch_pdl(attn_decode_split, dim3(kv_heads, splits), dim3(kDecThreads), smem, stream, q, k_cache, v_cache,
                   len_dev, q_heads, kv_heads, head_dim, scale, part) != cudaSuccess)
        return CL_ERR_CUDA;
    const int threads = head_dim < 1024 ? head_dim : 1024;
    return launch_pdl(attn_decode_combine, dim3(q_heads), dim3(threads), 0, stream, part, len_dev, splits, head_dim,
                      out, xq, q_heads * head_dim) == cudaSuccess
               ? CL_OK
               : CL_ERR_CUDA;
}

static size_t prefill_smem(int d) {
    return sizeof(float) * ((size_t)kQT * d + (size_t)kKT * (d + 1) + (size_t)kKT * d + kQT * (kKT + 1) + 3 * kQT);
}

CL_API int cl_attn_prefill(const float* q, const float* k_cache, const float* v_cache, int pos0, int rows,
                           int q_heads, int kv_heads, int head_dim, float* out, cudaStream_t stream) {
    if (q == nullptr || k_cache == nullptr || v_cache == nullptr || out == nullptr || rows <= 0 || pos0 < 0 ||
        q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads || head_dim <= 0 || head_dim % 8 ||
        head_dim > kMaxHeadDim)
        return CL_ERR_INVALID;
    const size_t smem = prefill_smem(head_dim);
    static int configured_for = 0;
    if ((int)smem > configured_for) {
        if (cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return CL_ERR_CUDA;
        configured_for = (int)smem;
    }
    return launch_pdl(attn_prefill_kernel, dim3(q_heads, (rows + kQT - 1) / kQT), dim3(kPreThreads), smem, stream,
                      q, k_cache, v_cache, pos0, rows, q_heads, kv_heads, head_dim, out) == cudaSuccess
               ? CL_OK
               : CL_ERR_CUDA;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decode attention without a caller workspace.
//
// Some callers cannot allocate device memory at the moment they run decode
// attention: host code inside a CUDA stream capture in a mode where
// cudaMalloc is refused, runtimes that hand out a fixed device-memory budget
// at start-up and forbid later allocations, latency-critical loops where the
// implicit device synchronisation of cudaMalloc/cudaFree is unacceptable, and
// foreign-language bindings that have no way to own or free CUDA buffers.
// This variant keeps the per-split softmax partials in a fixed array that
// is part of the library image instead: every GPU that loads the library
// holds kAttnNoAllocScratchBytes for it until the process exits.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kAttnNoAllocScratchBytes = 2u << 20;  // 2 MiB per GPU
constexpr int kMaxDevicesTracked = 64;

static __device__ __align__(256) unsigned char g_attn_noalloc_scratch[kAttnNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kMaxDevicesTracked] = {};

// Device address of the array on the current device.  The symbol name is a
// host-side stand-in, so the address is looked up once per device (with
// that device current) and cached; the lookup itself allocates nothing.
int noalloc_scratch(void** ptr) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return CL_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevicesTracked) return CL_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_attn_noalloc_scratch) != cudaSuccess || p == nullptr) return CL_ERR_CUDA;
        g_noalloc_ptr[dev] = p;
    }
    *ptr = g_noalloc_ptr[dev];
    return CL_OK;
}

}  // namespace

extern "C" CL_API size_t cl_attn_decode_noalloc_limit_bytes(void) { return kAttnNoAllocScratchBytes; }

extern "C" CL_API int cl_attn_decode_noalloc(const float* q, const float* k_cache, const float* v_cache,
                                             const int* len_dev, int max_len, int q_heads, int kv_heads,
                                             int head_dim, float scale, float* out, cudaStream_t stream) {
    const size_t need = cl_attn_decode_workspace_bytes(q_heads, head_dim, max_len);
    if (need == 0) return CL_ERR_INVALID;
    if (need > kAttnNoAllocScratchBytes) return CL_ERR_LIMIT;
    void* scratch = nullptr;
    const int rc = noalloc_scratch(&scratch);
    if (rc != CL_OK) return rc;
    // Nothing in the array has to start at zero: the split kernel writes
    // every partial that the combine kernel reads in the same call.
    return cl_attn_decode(q, k_cache, v_cache, len_dev, max_len, q_heads, kv_heads, head_dim, scale, out, nullptr,
                          scratch, kAttnNoAllocScratchBytes, stream);
}
