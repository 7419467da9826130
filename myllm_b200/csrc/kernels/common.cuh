// Shared device helpers for the sm_100a kernels.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "cudallm_kernels.h"

#define CL_DEVINL __device__ __forceinline__

namespace cl {

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  Every kernel launched by this library
// carries the programmatic-stream-serialization attribute, so the next kernel
// in the stream may start while this one drains.  Rules kept by every kernel:
// * before grid_wait() a kernel reads only immutable data (weights, tables)
//   and writes nothing;
// * data an earlier kernel wrote (activations, caches, maxima, ids) is never
//   read on the non-coherent path (ld.global.nc, __ldg, or a const
//   __restrict__ pointer the compiler may read that way): the kernel may
//   have started before that data was written, and a line of a buffer that
//   every layer reuses can still sit in the SM's read-only cache from an
//   earlier kernel.  Measured on B200: the split tensor-core prefill
//   attention read Q and the KV cache through const __restrict__ pointers
//   and gave a wrong prefill, different each run, with programmatic
//   dependent launch on; coherent loads made it exact.  Weights keep
//   __restrict__ and the non-coherent loads.
// ---------------------------------------------------------------------------
CL_DEVINL void grid_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
CL_DEVINL void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Bulk L2 prefetch of [ptr, ptr + bytes): one TMA-engine request per call.
// ptr must be 16-byte aligned and bytes a multiple of 16.
CL_DEVINL void prefetch_l2(const void* ptr, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(ptr), "r"(bytes) : "memory");
}

CL_DEVINL uint4 ldg_nc_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

CL_DEVINL uint2 ldg_nc_v2(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

CL_DEVINL uint32_t ldg_nc_u32(const void* p) {
    uint32_t v;
    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

CL_DEVINL uint32_t ldg_nc_u16(const void* p) {
    unsigned short v;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

// 4-way byte dot products with 32-bit accumulation.
CL_DEVINL int dp4a_us(uint32_t a_unsigned, int b_signed, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a_unsigned), "r"(b_signed), "r"(c));
    return d;
}

CL_DEVINL int dp4a_ss(int a, int b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

CL_DEVINL float half_bits_to_float(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xffffu)));
}

CL_DEVINL float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

CL_DEVINL float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

CL_DEVINL double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------------------
// XQ: the activation-vector format every decode GEMV consumes.
//
// A vector x of K floats (K % 32 == 0) is stored per 32-element block b as a
// scale s_b = max|x| / 127 and, per element, three signed 8-bit limbs with
//     x ~= s_b * (l0 + l1 / 2^7 + l2 / 2^14),   |l0| <= 127, |l1|,|l2| <= 64,
// an absolute error below max|x_b| * 2^-22 (FP32-grade).  The integer dot
// product with quantized weights is then exact with dp4a, and only the
// per-block sums are scaled in FP32.
//
// Planes (all offsets 16-byte aligned):
//   limbs[K/16][3][16] int8   chunk c = elements 16c..16c+15, limb-major
//   lsum [K/16]        int2   (sum of l0, sum of l1*2^7 + l2) over the chunk
//   scale[K/32]        float  s_b * 2^-14, so x = scale * (l0*2^14 + l1*2^7 + l2)
// ---------------------------------------------------------------------------
struct XQView {
    const int4* limbs;   // 3 int4 per chunk
    const int2* lsum;    // 1 per chunk
    const float* scale;  // 1 per 32-block
};

struct XQMut {
    int4* limbs;
    int2* lsum;
    float* scale;
};

__host__ __device__ inline size_t xq_limb_bytes(int k) { return (size_t)k / 16 * 48; }
__host__ __device__ inline size_t xq_lsum_offset(int k) { return xq_limb_bytes(k); }
__host__ __device__ inline size_t xq_scale_offset(int k) {
    return xq_lsum_offset(k) + (((size_t)k / 16 * 8 + 15) & ~(size_t)15);
}
__host__ __device__ inline size_t xq_total_bytes(int k) {
    return xq_scale_offset(k) + (((size_t)k / 32 * 4 + 15) & ~(size_t)15);
}

__host__ __device__ inline XQView xq_view(const void* base, int k) {
    const char* p = static_cast<const char*>(base);
    return XQView{reinterpret_cast<const int4*>(p), reinterpret_cast<const int2*>(p + xq_lsum_offset(k)),
                  reinterpret_cast<const float*>(p + xq_scale_offset(k))};
}

__host__ __device__ inline XQMut xq_mut(void* base, int k) {
    char* p = static_cast<char*>(base);
    return XQMut{reinterpret_cast<int4*>(p), reinterpret_cast<int2*>(p + xq_lsum_offset(k)),
                 reinterpret_cast<float*>(p + xq_scale_offset(k))};
}

// Quantize one 32-element block held as one value per lane of a full warp.
// Lane i holds element i of the block; chunk 2*blk + (i >= 16).
CL_DEVINL void xq_store_block_warp(XQMut q, int blk, float v) {
    const int lane = threadIdx.x & 31;
    const float amax = warp_max(fabsf(v));
    const float s = amax / 127.0f;
    const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
    float r0 = v * inv;
    float l0 = fminf(fmaxf(rintf(r0), -127.0f), 127.0f);
    float r1 = (r0 - l0) * 128.0f;
    float l1 = fminf(fmaxf(rintf(r1), -64.0f), 64.0f);
    float r2 = (r1 - l1) * 128.0f;
    float l2 = fminf(fmaxf(rintf(r2), -64.0f), 64.0f);
    const int i0 = (int)l0, i1 = (int)l1, i2 = (int)l2;
    // byte store into the chunk's limb planes
    const int chunk = 2 * blk + (lane >> 4);
    int8_t* base = reinterpret_cast<int8_t*>(q.limbs + 3 * chunk);
    const int e = lane & 15;
    base[e] = (int8_t)i0;
    base[16 + e] = (int8_t)i1;
    base[32 + e] = (int8_t)i2;
    // chunk sums over 16 lanes
    int t0 = i0, t12 = i1 * 128 + i2;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
        t0 += __shfl_xor_sync(0xffffffffu, t0, o);
        t12 += __shfl_xor_sync(0xffffffffu, t12, o);
    }
    if (e == 0) q.lsum[chunk] = make_int2(t0, t12);
    if (lane == 0) q.scale[blk] = s * (1.0f / 16384.0f);
}

}  // namespace cl

// ---------------------------------------------------------------------------
// mbarrier + bulk-copy (TMA engine) helpers.  Every wait is bounded: after
// kSpinLimit failed polls the caller records an error and gives up instead
// of spinning forever.
// ---------------------------------------------------------------------------
namespace cl {

constexpr uint32_t kSpinLimit = 1u << 22;

CL_DEVINL uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

CL_DEVINL void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

CL_DEVINL void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

CL_DEVINL void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

CL_DEVINL void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

CL_DEVINL bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// true once the phase with `parity` has completed; false after kSpinLimit polls.
CL_DEVINL bool mbar_wait(uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
    }
    return false;
}

// Global -> shared bulk copy completing on `bar` (16-byte aligned, size % 16 == 0).
CL_DEVINL void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

CL_DEVINL void named_barrier(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace cl
