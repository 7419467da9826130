// Layout, activation-vector and element-wise kernels of the decode/prefill graph.
#include "common.cuh"
#include "dequant.cuh"
#include "launch.cuh"

namespace cl {

int g_pdl_enabled = 1;

// ---- weight repack ----------------------------------------------------------
// One thread per GGML block: native row bytes -> device layout (gemv.cu header).
__global__ void repack_kernel(int type, const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                              int rows, int k, long long src_rb, long long dst_rb) {
    grid_wait();  // launched with programmatic dependent launch: the previous kernel's writes first
    const int bsize = (type == CL_TYPE_Q8_0 || type == CL_TYPE_Q5_0) ? 32 : 256;
    const int nb = k / bsize;
    const long long total = (long long)rows * nb;
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const long long r = t / nb;
        const int b = (int)(t % nb);
        const uint8_t* s = src + r * src_rb;
        uint8_t* d = dst + r * dst_rb;
        switch (type) {
        case CL_TYPE_Q4_K:
        case CL_TYPE_Q5_K: {
            const int bs = type == CL_TYPE_Q4_K ? 144 : 176;
            const uint8_t* sb = s + b * bs;
            uint8_t* db = d + b * bs;
            for (int i = 0; i < 4; ++i) db[i] = sb[i];
            for (int i = 16; i < bs; ++i) db[i] = sb[i];
            uint8_t slots[12] = {0};
            for (int i = 0; i < 8; ++i) {
                int sc, m;
                kscale_native(sb + 4, i, sc, m);
                const uint32_t v = (uint32_t)sc | ((uint32_t)m << 6);
                const int bit = 12 * i;
                slots[bit >> 3] |= (uint8_t)((v << (bit & 7)) & 0xffu);
                slots[(bit >> 3) + 1] |= (uint8_t)((v << (bit & 7)) >> 8);
            }
            for (int i = 0; i < 12; ++i) db[4 + i] = slots[i];
            break;
        }
        case CL_TYPE_Q6_K:
            for (int i = 0; i < 208; ++i) d[b * 208 + i] = s[b * 210 + i];
            d[nb * 208 + 2 * b] = s[b * 210 + 208];
            d[nb * 208 + 2 * b + 1] = s[b * 210 + 209];
            break;
        case CL_TYPE_Q8_0:
            for (int i = 0; i < 32; ++i) d[b * 32 + i] = s[b * 34 + 2 + i];
            d[nb * 32 + 2 * b] = s[b * 34];
            d[nb * 32 + 2 * b + 1] = s[b * 34 + 1];
            break;
        case CL_TYPE_Q5_0:
            for (int i = 0; i < 16; ++i) d[b * 16 + i] = s[b * 22 + 6 + i];
            for (int i = 0; i < 4; ++i) d[nb * 16 + 4 * b + i] = s[b * 22 + 2 + i];
            d[nb * 20 + 2 * b] = s[b * 22];
            d[nb * 20 + 2 * b + 1] = s[b * 22 + 1];
            break;
        default: break;
        }
        // zero the row pad once per row
        if (b == 0) {
            for (long long i = src_rb; i < dst_rb; ++i) d[i] = 0;
        }
    }
}

__global__ void copy_rows_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int rows,
                                 long long src_rb, long long dst_rb) {
    grid_wait();
    const long long total = (long long)rows * dst_rb;
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const long long r = t / dst_rb, i = t % dst_rb;
        dst[t] = i < src_rb ? src[r * src_rb + i] : 0;
    }
}

// ---- XQ quantization --------------------------------------------------------
__global__ void quantize_xq_kernel(const float* x, int k, void* xq) {
    grid_launch_dependents();
    grid_wait();
    const int blk = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (blk >= k / 32) return;
    xq_store_block_warp(xq_mut(xq, k), blk, x[blk * 32 + (threadIdx.x & 31)]);
}

// ---- RMSNorm ----------------------------------------------------------------
constexpr int kNormThreads = 512;

__global__ void __launch_bounds__(kNormThreads)
rmsnorm_kernel(const float* x, const float* __restrict__ gamma, int k, float eps,
               float* y, void* xq, long long xq_stride) {
    grid_launch_dependents();
    grid_wait();
    const int row = blockIdx.x;
    const float* xr = x + (size_t)row * k;
    double ss = 0.0;
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        const double v = (double)xr[i];
        ss += v * v;
    }
    __shared__ double red[kNormThreads / 32];
    ss = warp_sum_d(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
        t = warp_sum_d(t);
        if (threadIdx.x == 0) red[0] = t;
    }
    __syncthreads();
    // cpu_llm.cpp:160-165: mean in double -> float, 1/sqrt in float, x*(inv*g)
    const float mean_square = (float)(red[0] / (double)k);
    const float inv = 1.0f / sqrtf(mean_square + eps);
    XQMut q{};
    if (xq) q = xq_mut(static_cast<char*>(xq) + (size_t)row * xq_stride, k);
    // Whole warps walk 32-blocks so each can emit its XQ block.
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, warps = blockDim.x >> 5;
    for (int b = warp; b < k / 32; b += warps) {
        const int i = b * 32 + lane;
        const float v = __fmul_rn(xr[i], __fmul_rn(inv, gamma[i]));
        if (y) y[(size_t)row * k + i] = v;
        if (xq) xq_store_block_warp(q, b, v);
    }
    // tail (k not a multiple of 32: fp32 output only)
    for (int i = (k / 32) * 32 + threadIdx.x; i < k; i += blockDim.x) {
        if (y) y[(size_t)row * k + i] = __fmul_rn(xr[i], __fmul_rn(inv, gamma[i]));
    }
}

// ---- embedding ---------------------------------------------------------------
__global__ void embed_kernel(int type, const uint8_t* __restrict__ table, long long stride, int vocab, int k,
                             const int32_t* ids, int count, float* out,
                             int* error_flag) {
    grid_launch_dependents();
    grid_wait();
    const long long total = (long long)count * k;
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(t / k), c = (int)(t % k);
        const int id = ids[r];
        float v = 0.0f;
        if (id >= 0 && id < vocab) {
            v = dequant_at(type, table + (size_t)id * stride, k, c);
        } else if (c == 0 && error_flag) {
            *error_flag = 1;
        }
        out[t] = v;
    }
}

}  // namespace cl

using namespace cl;

extern "C" {

CL_API const char* cl_status_string(int status) {
    switch (status) {
    case CL_OK: return "ok";
    case CL_ERR_INVALID: return "invalid argument";
    case CL_ERR_UNSUPPORTED: return "unsupported type or shape";
    case CL_ERR_CUDA: return "CUDA launch failed";
    case CL_ERR_WORKSPACE: return "workspace missing or too small";
    case CL_ERR_LIMIT: return "request exceeds the fixed no-allocation scratch size";
    default: return "unknown status";
    }
}

CL_API void cl_set_pdl(int enabled) { g_pdl_enabled = enabled ? 1 : 0; }

CL_API long long cl_native_row_bytes(int type, int k) {
    if (k <= 0) return -1;
    switch (type) {
    case CL_TYPE_F32: return 4LL * k;
    case CL_TYPE_F16: return 2LL * k;
    case CL_TYPE_Q5_0: return k % 32 ? -1 : k / 32 * 22LL;
    case CL_TYPE_Q8_0: return k % 32 ? -1 : k / 32 * 34LL;
    case CL_TYPE_Q4_K: return k % 256 ? -1 : k / 256 * 144LL;
    case CL_TYPE_Q5_K: return k % 256 ? -1 : k / 256 * 176LL;
    case CL_TYPE_Q6_K: return k % 256 ? -1 : k / 256 * 210LL;
    default: return -1;
    }
}

CL_API long long cl_row_stride(int type, int k) {
    const long long rb = cl_native_row_bytes(type, k);
    return rb < 0 ? -1 : (rb + 15) / 16 * 16;
}

CL_API int cl_repack_rows(int type, const void* native, void* packed, int rows, int k, cudaStream_t stream) {
    const long long srb = cl_native_row_bytes(type, k), drb = cl_row_stride(type, k);
    if (srb < 0 || rows < 0 || native == nullptr || packed == nullptr) return CL_ERR_INVALID;
    if (rows == 0) return CL_OK;
    // the launch's own status (a stale error of an earlier runtime call must
    // not be reported as this launch's)
    cudaError_t e;
    if (type == CL_TYPE_F32 || type == CL_TYPE_F16)
        e = launch_pdl(copy_rows_kernel, dim3(1184), dim3(256), 0, stream, static_cast<const uint8_t*>(native),
                       static_cast<uint8_t*>(packed), rows, srb, drb);
    else
        e = launch_pdl(repack_kernel, dim3(1184), dim3(256), 0, stream, type, static_cast<const uint8_t*>(native),
                       static_cast<uint8_t*>(packed), rows, k, srb, drb);
    return e == cudaSuccess ? CL_OK : CL_ERR_CUDA;
}

CL_API size_t cl_xq_bytes(int k) { return k > 0 && k % 32 == 0 ? xq_total_bytes(k) : 0; }

CL_API int cl_quantize_xq(const float* x, int k, void* xq, cudaStream_t stream) {
    if (x == nullptr || xq == nullptr || k <= 0 || k % 32) return CL_ERR_INVALID;
    const int blocks = k / 32;
    return launch_pdl(quantize_xq_kernel, dim3((blocks + 7) / 8), dim3(256), 0, stream, x, k, xq) ==
                   cudaSuccess
               ? CL_OK
               : CL_ERR_CUDA;
}

CL_API int cl_rmsnorm(const float* x, const float* gamma, int rows, int k, float eps, float* y, void* xq,
                      cudaStream_t stream) {
    if (x == nullptr || gamma == nullptr || rows <= 0 || k <= 0 || !(eps > 0.0f)) return CL_ERR_INVALID;
    if (xq && k % 32) return CL_ERR_INVALID;
    const long long xs = xq ? (long long)xq_total_bytes(k) : 0;
    return launch_pdl(rmsnorm_kernel, dim3(rows), dim3(kNormThreads), 0, stream, x, gamma, k, eps, y, xq, xs) ==
                   cudaSuccess
               ? CL_OK
               : CL_ERR_CUDA;
}

CL_API int cl_embed(int type, const void* table, long long stride, int vocab, int k, const int32_t* ids,
                    int count, float* out, int* error_flag, cudaStream_t stream) {
    if (table == nullptr || ids == nullptr || out == nullptr || count <= 0 || k <= 0 || vocab <= 0 ||
        cl_native_row_bytes(type, k) < 0 || stride < cl_row_stride(type, k))
        return CL_ERR_INVALID;
    // quantized rows are read byte by byte; F32 rows as floats
    if (type == CL_TYPE_F32 && (reinterpret_cast<uintptr_t>(table) % 4 || stride % 4)) return CL_ERR_INVALID;
    const long long total = (long long)count * k;
    const int grid = (int)min((total + 255) / 256, 4096LL);
    return launch_pdl(embed_kernel, dim3(grid), dim3(256), 0, stream, type,
                      static_cast<const uint8_t*>(table), stride, vocab, k, ids, count, out, error_flag) ==
                   cudaSuccess
               ? CL_OK
               : CL_ERR_CUDA;
}

}  // extern "C"
