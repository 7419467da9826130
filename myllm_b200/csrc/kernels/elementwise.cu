// RoPE + KV append, SwiGLU, residual add and the greedy-token argmax.
#include "common.cuh"
#include "launch.cuh"

namespace cl {

// One thread per element pair.  Head slot s < q_heads: query head (rotated in
// place); next kv_heads slots: key heads (rotated into the cache); last
// kv_heads slots: value heads (copied into the cache).
__global__ void rope_kv_kernel(float* q, const float* k, const float* v,
                               int rows, int hq, int hkv, int d, int rot, const float* __restrict__ cs,
                               const int* pos_dev, int pos_host, float* kc,
                               float* vc) {
    grid_launch_dependents();
    grid_wait();
    const int half = rot / 2, pairs = d / 2, slots = hq + 2 * hkv;
    const long long total = (long long)rows * slots * pairs;
    const int pos0 = pos_dev ? *pos_dev : pos_host;
    const int kvd = hkv * d;
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const int p = (int)(t % pairs);
        const int s = (int)((t / pairs) % slots);
        const int r = (int)(t / ((long long)pairs * slots));
        const int pos = pos0 + r;
        int i0, i1;
        bool rotary = p < half;
        if (rotary) {
            i0 = p;
            i1 = p + half;
        } else {
            i0 = rot + 2 * (p - half);
            i1 = i0 + 1;
        }
        if (s < hq) {
            if (!rotary) continue;
            float* h = q + (size_t)r * hq * d + (size_t)s * d;
            const float c = cs[((size_t)pos * half + p) * 2], sn = cs[((size_t)pos * half + p) * 2 + 1];
            const float a = h[i0], b = h[i1];
            h[i0] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
            h[i1] = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, c));
        } else if (s < hq + hkv) {
            const int hh = s - hq;
            const float* src = k + (size_t)r * kvd + (size_t)hh * d;
            float* dst = kc + (size_t)pos * kvd + (size_t)hh * d;
            const float a = src[i0], b = src[i1];
            if (rotary) {
                const float c = cs[((size_t)pos * half + p) * 2], sn = cs[((size_t)pos * half + p) * 2 + 1];
                dst[i0] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
                dst[i1] = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, c));
            } else {
                dst[i0] = a;
                dst[i1] = b;
            }
        } else {
            const int hh = s - hq - hkv;
            const float* src = v + (size_t)r * kvd + (size_t)hh * d;
            float* dst = vc + (size_t)pos * kvd + (size_t)hh * d;
            dst[i0] = src[i0];
            dst[i1] = src[i1];
        }
    }
}

__global__ void swiglu_kernel(const float* g, const float* u, float* o,
                              long long n) {
    grid_launch_dependents();
    grid_wait();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const float gate = g[i];
        const float sig = gate >= 0.0f ? 1.0f / (1.0f + expf(-gate)) : expf(gate) / (1.0f + expf(gate));
        o[i] = __fmul_rn(__fmul_rn(gate, sig), u[i]);
    }
}

__global__ void add_kernel(const float* a, const float* b, float* o,
                           long long n) {
    grid_launch_dependents();
    grid_wait();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x)
        o[i] = a[i] + b[i];
}

// ---- argmax -------------------------------------------------------------------
constexpr int kArgThreads = 256;

CL_DEVINL bool better(float v, int i, float bv, int bi) { return v > bv || (v == bv && i < bi); }

CL_DEVINL void block_best(float& v, int& i) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (better(ov, oi, v, i)) {
            v = ov;
            i = oi;
        }
    }
    __shared__ float sv[kArgThreads / 32];
    __shared__ int si[kArgThreads / 32];
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        sv[w] = v;
        si[w] = i;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        v = threadIdx.x < kArgThreads / 32 ? sv[threadIdx.x] : -INFINITY;
        i = threadIdx.x < kArgThreads / 32 ? si[threadIdx.x] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, i, o);
            if (better(ov, oi, v, i)) {
                v = ov;
                i = oi;
            }
        }
    }
}

struct ArgmaxWS {
    unsigned int* counter;
    float2* partial;  // (value, index bits)
};

__host__ __device__ inline int argmax_ctas(int n) {
    const int c = (n + 4095) / 4096;
    return c < 1 ? 1 : (c > 512 ? 512 : c);
}

__global__ void __launch_bounds__(kArgThreads)
argmax_kernel(const float* x, int n, int index_offset, int32_t* token, float* value,
              unsigned int* counter, float2* partial) {
    grid_launch_dependents();
    grid_wait();
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = blockIdx.x * kArgThreads + threadIdx.x; i < n; i += gridDim.x * kArgThreads) {
        const float v = x[i];
        if (better(v, i, bv, bi)) {
            bv = v;
            bi = i;
        }
    }
    block_best(bv, bi);
    __shared__ bool last;
    if (threadIdx.x == 0) {
        partial[blockIdx.x] = make_float2(bv, __int_as_float(bi));
        __threadfence();
        last = atomicAdd(counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    bv = -INFINITY;
    bi = 0x7fffffff;
    for (int c = threadIdx.x; c < (int)gridDim.x; c += kArgThreads) {
        const float2 p = __ldcg(partial + c);
        const int pi = __float_as_int(p.y);
        if (better(p.x, pi, bv, bi)) {
            bv = p.x;
            bi = pi;
        }
    }
    block_best(bv, bi);
    if (threadIdx.x == 0) {
        *token = (bi == 0x7fffffff ? 0 : bi) + index_offset;
        if (value) *value = bv;
        *counter = 0u;
    }
}

// records[i] = (value, index bits); lowest index wins ties.
__global__ void argmax_merge_kernel(const float2* rec, int n, int32_t* token) {
    grid_launch_dependents();
    grid_wait();
    if (threadIdx.x != 0) return;
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = 0; i < n; ++i) {
        const int ri = __float_as_int(rec[i].y);
        if (better(rec[i].x, ri, bv, bi)) {
            bv = rec[i].x;
            bi = ri;
        }
    }
    *token = bi == 0x7fffffff ? 0 : bi;
}

__global__ void counter_add_kernel(int* c, int n, int delta) {
    grid_launch_dependents();
    grid_wait();
    if ((int)threadIdx.x < n) c[threadIdx.x] += delta;
}

}  // namespace cl

using namespace cl;

extern "C" {

CL_API int cl_rope_kv(float* q, const float* k, const float* v, int rows, int q_heads, int kv_heads, int head_dim,
                      int rot_dim, const float* cos_sin, const int* pos_dev, int pos_host, float* k_cache,
                      float* v_cache, cudaStream_t stream) {
    if (q == nullptr || k == nullptr || v == nullptr || cos_sin == nullptr || k_cache == nullptr ||
        v_cache == nullptr || rows <= 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || head_dim % 2 ||
        rot_dim <= 0 || rot_dim % 2 || rot_dim > head_dim || (pos_dev == nullptr && pos_host < 0))
        return CL_ERR_INVALID;
    const long long total = (long long)rows * (q_heads + 2 * kv_heads) * (head_dim / 2);
    const int grid = (int)min((total + 255) / 256, 8192LL);
    return launch_pdl(rope_kv_kernel, dim3(grid), dim3(256), 0, stream, q, k, v, rows, q_heads, kv_heads, head_dim,
                      rot_dim, cos_sin, pos_dev, pos_host, k_cache, v_cache) == cudaSuccess
               ? CL_OK
               : CL_ERR_CUDA;
}

CL_API int cl_swiglu(const float* gate, const float* up, float* out, long long n, cudaStream_t stream) {
    if (gate == nullptr || up == nullptr || out == nullptr || n <= 0) return CL_ERR_INVALID;
    const int grid = (int)min((n + 255) / 256, 8192LL);
    return launch_pdl(swiglu_kernel, dim3(grid), dim3(256), 0, stream, gate, up, out, n) == cudaSuccess
               ? CL_OK
               : CL_ERR_CUDA;
}

CL_API int cl_add(const float* a, const float* b, float* out, long long n, cudaStream_t stream) {
    if (a == nullptr || b == nullptr || out == nullptr || n <= 0) return CL_ERR_INVALID;
    const int grid = (int)min((n + 255) / 256, 8192LL);
    return launch_pdl(add_kernel, dim3(grid), dim3(256), 0, stream, a, b, out, n) == cudaSuccess ? CL_OK
                                                                                              : CL_ERR_CUDA;
}

CL_API size_t cl_argmax_workspace_bytes(int n) {
    return n > 0 ? 16 + sizeof(float2) * (size_t)argmax_ctas(n) : 0;
}

CL_API int cl_argmax_ex(const float* logits, int n, int index_offset, int32_t* token, float* value,
                        void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (logits == nullptr || token == nullptr || n <= 0) return CL_ERR_INVALID;
    if (workspace == nullptr || workspace_bytes < cl_argmax_workspace_bytes(n) ||
        reinterpret_cast<uintptr_t>(workspace) % 16)
        return CL_ERR_WORKSPACE;
    unsigned int* counter = static_cast<unsigned int*>(workspace);
    float2* partial = reinterpret_cast<float2*>(static_cast<char*>(workspace) + 16);
    return launch_pdl(argmax_kernel, dim3(argmax_ctas(n)), dim3(kArgThreads), 0, stream, logits, n, index_offset,
                      token, value, counter, partial) == cudaSuccess
               ? CL_OK
               : CL_ERR_CUDA;
}

CL_API int cl_argmax(const float* logits, int n, int32_t* token, void* workspace, size_t workspace_bytes,
                     cudaStream_t stream) {
    return cl_argmax_ex(logits, n, 0, token, nullptr, workspace, workspace_bytes, stream);
}

CL_API int cl_argmax_merge(const float* records, int n, int32_t* token, cudaStream_t stream) {
    if (records == nullptr || token == nullptr || n <= 0) return CL_ERR_INVALID;
    return launch_pdl(argmax_merge_kernel, dim3(1), dim3(32), 0, stream, reinterpret_cast<const float2*>(records), n,
                      token) == cudaSuccess
               ? CL_OK
               : CL_ERR_CUDA;
}

CL_API int cl_counter_add(int* counters, int n, int delta, cudaStream_t stream) {
    if (counters == nullptr || n <= 0 || n > 32) return CL_ERR_INVALID;
    return launch_pdl(counter_add_kernel, dim3(1), dim3(32), 0, stream, counters, n, delta) == cudaSuccess
               ? CL_OK
               : CL_ERR_CUDA;
}

}  // extern "C"
