// Prefill GEMM, FP32 CUDA-core path: Y[m,n] = X[m,k] W[n,k]^T (+bias) (+R).
//
// Reference: metal_gemm_{q5_0,q8_0,q4_k,q5_k,q6_k}_f32 (metal_llm.metal:
// 621-704) and the CPU gemmtb/gemmt loops (cpu_llm.cpp:591-653).  Weight
// tiles are dequantized into shared memory with the CPU decoder's exact FP32
// element values, then multiplied in FP32 in k order, so the result differs
// from the CPU only by FMA rounding.  cl_gemm uses it for shapes the
// tensor-core path (gemm_tc.cu) does not take; cl_gemm_simt calls it directly.
#include "common.cuh"
#include "dequant.cuh"
#include "launch.cuh"

namespace cl {

constexpr int kBM = 64, kBN = 64, kBK = 32, kSimtThreads = 256;

__global__ void __launch_bounds__(kSimtThreads)
gemm_simt_kernel(int type, const uint8_t* __restrict__ w, long long stride, int n, int k,
                 const float* x, int m, const float* __restrict__ bias,
                 const float* res, float* y) {
    grid_launch_dependents();
    grid_wait();
    __shared__ float Xs[kBK][kBM + 4];
    __shared__ float Ws[kBK][kBN + 4];
    const int n0 = blockIdx.x * kBN, m0 = blockIdx.y * kBM;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;  // 16 x 16 threads, 4 x 4 outputs each
    float acc[4][4] = {};
    for (int k0 = 0; k0 < k; k0 += kBK) {
        for (int i = threadIdx.x; i < kBM * kBK; i += kSimtThreads) {
            const int r = i / kBK, c = i % kBK;
            const int gm = m0 + r, gk = k0 + c;
            Xs[c][r] = (gm < m && gk < k) ? x[(size_t)gm * k + gk] : 0.0f;
        }
        for (int i = threadIdx.x; i < kBN * kBK; i += kSimtThreads) {
            const int r = i / kBK, c = i % kBK;
            const int gn = n0 + r, gk = k0 + c;
            Ws[c][r] = (gn < n && gk < k) ? dequant_at(type, w + (size_t)gn * stride, k, gk) : 0.0f;
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < kBK; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                a[i] = Xs[kk][ty * 4 + i];
                b[i] = Ws[kk][tx * 4 + i];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] += a[i] * b[j];
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int gm = m0 + ty * 4 + i;
        if (gm >= m) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gn = n0 + tx * 4 + j;
            if (gn >= n) continue;
            float v = acc[i][j];
            if (bias) v += bias[gn];
            if (res) v = res[(size_t)gm * n + gn] + v;
            y[(size_t)gm * n + gn] = v;
        }
    }
}

int launch_gemm_simt(int type, const void* w, long long stride, int n, int k, const float* x, int m,
                     const float* bias, const float* residual, float* y, cudaStream_t stream) {
    dim3 grid((n + kBN - 1) / kBN, (m + kBM - 1) / kBM);
    return launch_pdl(gemm_simt_kernel, grid, dim3(kSimtThreads), 0, stream, type,
                      static_cast<const uint8_t*>(w), stride, n, k, x, m, bias, residual, y) == cudaSuccess
               ? CL_OK
               : CL_ERR_CUDA;
}

}  // namespace cl

namespace cl {
bool gemm_tc_supported(int type, int n, int k, int m, int precision);
int launch_gemm_tc(int type, const void* w, long long stride, int n, int k, const float* x, int m, const float* bias,
                   const float* residual, float* y, int precision, cudaStream_t stream);
}  // namespace cl

namespace {
bool gemm_args_ok(int type, const void* w, long long stride, int n, int k, const float* x, int m, float* y) {
    // quantized rows are read byte by byte; F32 rows as floats
    return w != nullptr && x != nullptr && y != nullptr && n > 0 && k > 0 && m > 0 &&
           cl_native_row_bytes(type, k) >= 0 && stride >= cl_row_stride(type, k) &&
           (type != CL_TYPE_F32 || (reinterpret_cast<uintptr_t>(w) % 4 == 0 && stride % 4 == 0));
}
}  // namespace

extern "C" CL_API int cl_gemm_simt(int type, const void* w, long long stride, int n, int k, const float* x, int m,
                                   const float* bias, const float* residual, float* y, cudaStream_t stream) {
    if (!gemm_args_ok(type, w, stride, n, k, x, m, y)) return CL_ERR_INVALID;
    return cl::launch_gemm_simt(type, w, stride, n, k, x, m, bias, residual, y, stream);
}

extern "C" CL_API int cl_gemm(int type, const void* w, long long stride, int n, int k, const float* x, int m,
                              const float* bias, const float* residual, float* y, cudaStream_t stream) {
    if (!gemm_args_ok(type, w, stride, n, k, x, m, y)) return CL_ERR_INVALID;
    const bool aligned = reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0 &&
                         stride % 16 == 0;
    if (aligned && cl::gemm_tc_supported(type, n, k, m, CL_GEMM_TF32X3))
        return cl::launch_gemm_tc(type, w, stride, n, k, x, m, bias, residual, y, CL_GEMM_TF32X3, stream);
    return cl::launch_gemm_simt(type, w, stride, n, k, x, m, bias, residual, y, stream);
}
