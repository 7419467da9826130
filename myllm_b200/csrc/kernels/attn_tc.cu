// Causal prefill attention on the tensor cores (FP16 operands, FP32
// accumulation and softmax).
//
// Reference: cpu_prefill_layer (cpu_llm.cpp:816-827): score = (q . k) /
// sqrt(d), keys after the query position masked, softmax, weighted sum of V;
// head h reads KV head h / (q_heads / kv_heads).  Same result as
// attn_prefill_kernel (attn.cu, FP32 CUDA cores) up to the FP16 rounding of
// q, k, v and p (11-bit significands): the fast prefill path's attention.
//
// Flash-attention form: CTA = (query head, 64 query rows), 4 warps of 16
// rows.  Per 64-key tile, K (row-major) and V (transposed) are staged in
// shared memory as FP16; S = Q K^T is 8 x 8 mma.sync.m16n8k16 per warp, the
// online softmax runs on the accumulator fragments (a row lives in the 4
// lanes of a quad), and the probabilities feed P V directly as A fragments
// (the accumulator layout of one MMA is the operand layout of the next).
//
// Split form (SPLIT, the FP32-grade prefill's attention): every operand is
// carried as an FP16 pair x = hi + lo (hi = fp16(x), lo = fp16(x - hi): 22
// significant bits), and each product is hi.hi + hi.lo + lo.hi on the tensor
// cores (the lo.lo term is below FP32 rounding).  The probabilities are
// scaled by 2^12 before they are split (p <= 1, so the scaled values stay in
// FP16 range while the small ones stay clear of FP16 subnormals) and the
// output by 2^-12 after: both exact.  Softmax statistics stay FP32.
#include "common.cuh"
#include "launch.cuh"

#include <cuda_fp16.h>

namespace cl {
namespace {

constexpr int kQR = 64;               // query rows per CTA
constexpr int kKR = 64;               // keys per tile
constexpr int kTcThreads = 128;
constexpr int kHD = 128;              // head dim
constexpr int kKLd = kHD + 8;         // K tile row (halves): +16 B keeps the fragment loads conflict-free
constexpr int kVLd = kKR + 8;         // transposed V row (halves)

CL_DEVINL uint32_t pack_half2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

CL_DEVINL void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                        uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// x as an FP16 pair: hi = fp16(x), lo = fp16(x - hi) (packed two per word).
CL_DEVINL void split_half2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

constexpr float kPScale = 4096.0f;  // 2^12: probabilities scaled before the split

template <bool SPLIT>
__global__ void __launch_bounds__(kTcThreads)
attn_prefill_tc_kernel(const float* q, const float* kc, const float* vc,
                       int pos0, int rows, int hq, int hkv, float* out) {
    grid_launch_dependents();
    grid_wait();
    // [hi][K tile], then [hi][V^T tile]; SPLIT adds the lo copies after each
    extern __shared__ __align__(16) uint8_t tc_smem[];
    __half* ks = reinterpret_cast<__half*>(tc_smem);
    __half* ks_lo = ks + kKR * kKLd;
    __half* vt = ks + (SPLIT ? 2 : 1) * kKR * kKLd;
    __half* vt_lo = vt + kHD * kVLd;
    const int h = blockIdx.x, g = h / (hq / hkv);
    const int r0 = blockIdx.y * kQR;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq = lane >> 2, tq = lane & 3;
    const int qd = hq * kHD, kvd = hkv * kHD;
    const float scale = 1.0f / sqrtf((float)kHD);

    // this warp's 16 query rows as A fragments: 8 k-steps of 16 dims
    const int rw = r0 + 16 * warp;  // first row of the warp
    uint32_t qa[8][4], ql[SPLIT ? 8 : 1][4];
#pragma unroll
    for (int ks16 = 0; ks16 < 8; ++ks16) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int row = rw + gq + ((i & 1) ? 8 : 0);
            const int col = 16 * ks16 + 2 * tq + ((i & 2) ? 8 : 0);
            float2 v = make_float2(0.0f, 0.0f);
            // q and the caches come from the previous kernel: read from L2 (see grid_wait's rules)
            if (row < rows) v = __ldcg(reinterpret_cast<const float2*>(q + (size_t)row * qd + (size_t)h * kHD + col));
            if (SPLIT) split_half2(v.x, v.y, qa[ks16][i], ql[SPLIT ? ks16 : 0][i]);
            else qa[ks16][i] = pack_half2(v.x, v.y);
        }
    }
    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;  // rows gq and gq + 8
    const int qp0 = pos0 + rw + gq, qp1 = qp0 + 8;              // their positions

    const int last_key = pos0 + min(rows, r0 + kQR) - 1;
    for (int kb = 0; kb <= last_key; kb += kKR) {
        __syncthreads();  // the previous tile's fragments are read
        // stage K (row-major) and V (transposed) as FP16
        for (int i = tid; i < kKR * (kHD / 4); i += kTcThreads) {
            const int r = i / (kHD / 4), c4 = i - r * (kHD / 4);
            const int key = kb + r;
            float4 kv = make_float4(0.0f, 0.0f, 0.0f, 0.0f), vv = kv;
            if (key <= last_key) {
                kv = __ldcg(reinterpret_cast<const float4*>(kc + (size_t)key * kvd + (size_t)g * kHD + 4 * c4));
                vv = __ldcg(reinterpret_cast<const float4*>(vc + (size_t)key * kvd + (size_t)g * kHD + 4 * c4));
            }
            if (SPLIT) {
                uint32_t h0, l0, h1, l1;
                split_half2(kv.x, kv.y, h0, l0);
                split_half2(kv.z, kv.w, h1, l1);
                *reinterpret_cast<uint2*>(ks + r * kKLd + 4 * c4) = make_uint2(h0, h1);
                *reinterpret_cast<uint2*>(ks_lo + r * kKLd + 4 * c4) = make_uint2(l0, l1);
                const float vv4[4] = {vv.x, vv.y, vv.z, vv.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const __half hi = __float2half_rn(vv4[e]);
                    vt[(4 * c4 + e) * kVLd + r] = hi;
                    vt_lo[(4 * c4 + e) * kVLd + r] = __float2half_rn(vv4[e] - __half2float(hi));
                }
            } else {
                *reinterpret_cast<uint2*>(ks + r * kKLd + 4 * c4) =
                    make_uint2(pack_half2(kv.x, kv.y), pack_half2(kv.z, kv.w));
                vt[(4 * c4 + 0) * kVLd + r] = __float2half_rn(vv.x);
                vt[(4 * c4 + 1) * kVLd + r] = __float2half_rn(vv.y);
                vt[(4 * c4 + 2) * kVLd + r] = __float2half_rn(vv.z);
                vt[(4 * c4 + 3) * kVLd + r] = __float2half_rn(vv.w);
            }
        }
        __syncthreads();
        if (rw >= rows || kb > pos0 + rw + 15) continue;  // no live row, or every key after the warp's rows

        // S = Q K^T: 8 n-tiles of 8 keys
        float s[8][4];
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
            s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.0f;
            const __half* kr = ks + (8 * nt + gq) * kKLd + 2 * tq;
#pragma unroll
            for (int ks16 = 0; ks16 < 8; ++ks16) {
                const uint32_t b0 = *reinterpret_cast<const uint32_t*>(kr + 16 * ks16);
                const uint32_t b1 = *reinterpret_cast<const uint32_t*>(kr + 16 * ks16 + 8);
                if (SPLIT) {
                    const __half* krl = ks_lo + (8 * nt + gq) * kKLd + 2 * tq;
                    const uint32_t c0 = *reinterpret_cast<const uint32_t*>(krl + 16 * ks16);
                    const uint32_t c1 = *reinterpret_cast<const uint32_t*>(krl + 16 * ks16 + 8);
                    const int li = SPLIT ? ks16 : 0;
                    mma16816(s[nt], ql[li][0], ql[li][1], ql[li][2], ql[li][3], b0, b1);
                    mma16816(s[nt], qa[ks16][0], qa[ks16][1], qa[ks16][2], qa[ks16][3], c0, c1);
                }
                mma16816(s[nt], qa[ks16][0], qa[ks16][1], qa[ks16][2], qa[ks16][3], b0, b1);
            }
        }
        // scale, causal mask, tile row max
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = kb + 8 * nt + 2 * tq + (e & 1);
                const int qp = (e & 2) ? qp1 : qp0;
                const float v = key <= qp ? s[nt][e] * scale : -INFINITY;
                s[nt][e] = v;
                if (e & 2) mx1 = fmaxf(mx1, v);
                else mx0 = fmaxf(mx0, v);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float a0 = mn0 == -INFINITY ? 1.0f : expf(m0 - mn0);
        const float a1 = mn1 == -INFINITY ? 1.0f : expf(m1 - mn1);
        float ps0 = 0.0f, ps1 = 0.0f;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float mref = (e & 2) ? mn1 : mn0;
                const float p = mref == -INFINITY ? 0.0f : expf(s[nt][e] - mref);
                s[nt][e] = p;
                if (e & 2) ps1 += p;
                else ps0 += p;
            }
        }
        ps0 += __shfl_xor_sync(0xffffffffu, ps0, 1);
        ps0 += __shfl_xor_sync(0xffffffffu, ps0, 2);
        ps1 += __shfl_xor_sync(0xffffffffu, ps1, 1);
        ps1 += __shfl_xor_sync(0xffffffffu, ps1, 2);
        l0 = l0 * a0 + ps0;
        l1 = l1 * a1 + ps1;
        m0 = mn0;
        m1 = mn1;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            o[j][0] *= a0;
            o[j][1] *= a0;
            o[j][2] *= a1;
            o[j][3] *= a1;
        }
        // O += P V: k-steps of 16 keys (n-tiles 2 kk, 2 kk + 1 of S), 16 n-tiles of 8 dims
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            uint32_t pa0, pa1, pa2, pa3, pl0 = 0u, pl1 = 0u, pl2 = 0u, pl3 = 0u;
            if (SPLIT) {
                split_half2(s[2 * kk][0] * kPScale, s[2 * kk][1] * kPScale, pa0, pl0);
                split_half2(s[2 * kk][2] * kPScale, s[2 * kk][3] * kPScale, pa1, pl1);
                split_half2(s[2 * kk + 1][0] * kPScale, s[2 * kk + 1][1] * kPScale, pa2, pl2);
                split_half2(s[2 * kk + 1][2] * kPScale, s[2 * kk + 1][3] * kPScale, pa3, pl3);
            } else {
                pa0 = pack_half2(s[2 * kk][0], s[2 * kk][1]);
                pa1 = pack_half2(s[2 * kk][2], s[2 * kk][3]);
                pa2 = pack_half2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
                pa3 = pack_half2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const __half* vr = vt + (8 * j + gq) * kVLd + 16 * kk + 2 * tq;
                const uint32_t b0 = *reinterpret_cast<const uint32_t*>(vr);
                const uint32_t b1 = *reinterpret_cast<const uint32_t*>(vr + 8);
                if (SPLIT) {
                    const __half* vrl = vt_lo + (8 * j + gq) * kVLd + 16 * kk + 2 * tq;
                    const uint32_t c0 = *reinterpret_cast<const uint32_t*>(vrl);
                    const uint32_t c1 = *reinterpret_cast<const uint32_t*>(vrl + 8);
                    mma16816(o[j], pl0, pl1, pl2, pl3, b0, b1);
                    mma16816(o[j], pa0, pa1, pa2, pa3, c0, c1);
                }
                mma16816(o[j], pa0, pa1, pa2, pa3, b0, b1);
            }
        }
    }
    // normalise and store rows gq, gq + 8 of the warp
    const int ra = rw + gq, rb = ra + 8;
    const float ps = SPLIT ? 1.0f / kPScale : 1.0f;  // exact (a power of two)
    const float i0 = l0 > 0.0f ? ps / l0 : 0.0f, i1 = l1 > 0.0f ? ps / l1 : 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const int col = 8 * j + 2 * tq;
        if (ra < rows)
            *reinterpret_cast<float2*>(out + (size_t)ra * qd + (size_t)h * kHD + col) = make_float2(o[j][0] * i0, o[j][1] * i0);
        if (rb < rows)
            *reinterpret_cast<float2*>(out + (size_t)rb * qd + (size_t)h * kHD + col) = make_float2(o[j][2] * i1, o[j][3] * i1);
    }
}

}  // namespace
}  // namespace cl

using namespace cl;

namespace {

int prefill_tc(bool split, const float* q, const float* k_cache, const float* v_cache, int pos0, int rows,
               int q_heads, int kv_heads, int head_dim, float* out, cudaStream_t stream) {
    if (q == nullptr || k_cache == nullptr || v_cache == nullptr || out == nullptr || rows <= 0 || pos0 < 0 ||
        q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads)
        return CL_ERR_INVALID;
    if (head_dim != kHD) return CL_ERR_UNSUPPORTED;
    // float4 / float2 loads and stores
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
         reinterpret_cast<uintptr_t>(out)) & 15u)
        return CL_ERR_INVALID;
    const int smem = (split ? 2 : 1) * (kKR * kKLd + kHD * kVLd) * (int)sizeof(__half);
    cudaError_t e;
    if (split) {
        static SmemLimit limit;
        e = limit.ensure(attn_prefill_tc_kernel<true>, smem);
        if (e == cudaSuccess)
            e = launch_pdl(attn_prefill_tc_kernel<true>, dim3(q_heads, (rows + kQR - 1) / kQR), dim3(kTcThreads),
                           (size_t)smem, stream, q, k_cache, v_cache, pos0, rows, q_heads, kv_heads, out);
    } else {
        e = launch_pdl(attn_prefill_tc_kernel<false>, dim3(q_heads, (rows + kQR - 1) / kQR), dim3(kTcThreads),
                       (size_t)smem, stream, q, k_cache, v_cache, pos0, rows, q_heads, kv_heads, out);
    }
    return e == cudaSuccess ? CL_OK : CL_ERR_CUDA;
}

}  // namespace

extern "C" CL_API int cl_attn_prefill_tc(const float* q, const float* k_cache, const float* v_cache, int pos0,
                                         int rows, int q_heads, int kv_heads, int head_dim, float* out,
                                         cudaStream_t stream) {
    return prefill_tc(false, q, k_cache, v_cache, pos0, rows, q_heads, kv_heads, head_dim, out, stream);
}

extern "C" CL_API int cl_attn_prefill_tc3(const float* q, const float* k_cache, const float* v_cache, int pos0,
                                          int rows, int q_heads, int kv_heads, int head_dim, float* out,
                                          cudaStream_t stream) {
    return prefill_tc(true, q, k_cache, v_cache, pos0, rows, q_heads, kv_heads, head_dim, out, stream);
}
