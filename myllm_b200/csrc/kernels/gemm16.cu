// Prefill GEMM on the 5th-generation tensor cores with 16-bit operands:
// Y[m, n] = X[m, k] W[n, k]^T (+ bias) (+ residual).
//
// Reference: metal_gemm_{q4_k,q6_k,q5_0,q8_0,q5_k}_f32 (metal_llm.metal:
// 621-704) and gemmtb / gemmt (cpu_llm.cpp:591-653), FP32 products of the
// dequantized weights.  Here the work is split in two passes:
//   1. cl_dequant16: every weight element dequantized once, with the CPU
//      decoder's FP32 expressions (dequant32<T>), then rounded once to FP16
//      (or BF16) into a row-major [n, k] scratch in HBM; the activations are
//      rounded the same way (cl_convert16).  For a 7B projection this is one
//      read of the native blocks and one write of 2 bytes per weight, against
//      2 m n k FLOPs of the product.
//   2. cl_gemm16_run: a persistent warp-specialised GEMM.  Warp 0 streams
//      128 x 64 (X) and BN x 64 (W) tiles with TMA tensor loads
//      (cp.async.bulk.tensor, 128-byte swizzle, no multicast) into a ring of
//      shared-memory stages; one thread of warp 1 issues tcgen05.mma
//      (kind::f16, M = 128, N = BN, K = 16) into an FP32 accumulator in TMEM;
//      warps 2-5 read the accumulator back with tcgen05.ld, add bias /
//      residual, and store rows through shared memory.  Two TMEM accumulators
//      alternate, so the epilogue of one tile overlaps the next tile's MMAs.
//      Work units (128-row x BN-column tile, K split) are ordered with the
//      row tiles fastest, so CTAs that run together share the weight tile
//      in L2.  With a K split, units store FP32 partials and
//      cl_gemm16 adds them (in split order) with the bias / residual.
// Split form (CL_GEMM_F16X3): each operand is first multiplied by a power
// of two that puts its largest magnitude in [2^13, 2^14) (from a device-side
// absolute maximum, so that the low parts stay clear of FP16's subnormal
// range); each row then holds the FP16 rounding of its k scaled values (hi)
// followed by the FP16 rounding of what hi leaves (lo), so hi + lo carries
// ~22 significant bits.  Every K step issues three MMAs, Xhi Whi + Xhi Wlo +
// Xlo Whi, into the same FP32 accumulator (the Xlo Wlo term is below FP32
// rounding), and the epilogue multiplies by the exact inverse powers of two:
// an FP32-grade product on the 16-bit tensor cores, as CL_GEMM_TF32X3 is on
// the TF32 ones.
// Outputs may be split by column ranges into up to three destinations (a
// fused Q/K/V or gate/up product writes each matrix to its own buffer).
// Every mbarrier wait is bounded; TMEM is always released.
#include "common.cuh"
#include "dequant.cuh"
#include "launch.cuh"

#include <cuda.h>
#include <cuda_bf16.h>

#include <algorithm>
#include <mutex>

namespace cl {
namespace g16 {

constexpr int BM = 128;
constexpr int BK = 64;                 // 16-bit elements per 128-byte row
constexpr int kThreads = 192;          // warp 0 TMA, warp 1 MMA + TMEM, warps 2-5 epilogue
constexpr int kATile = BM * 128;       // 16 KB
constexpr int kStageLd = 33;           // epilogue staging row stride (floats)

__device__ int g_g16_error = 0;

struct OutSeg {
    float* y;
    const float* bias;
    const float* res;
    const float *xmax, *wmax;  // split form: the absolute maxima the operands were scaled by
    int n0, n1, ld;
};

// The power of two that puts |a| <= amax into [2^13, 2^14) at amax (1 for 0).
__host__ __device__ inline int split_exp(float amax) {
    if (!(amax > 0.0f) || !(amax < 3.0e38f)) return 0;
    int e = 0;
    frexpf(amax, &e);  // amax = f 2^e, f in [0.5, 1)
    return max(-100, min(100, 14 - e));
}

// Output multiplier of a segment: 2^-(x exponent + w exponent), exact.
CL_DEVINL float seg_unscale(const OutSeg& sg) {
    if (sg.xmax == nullptr || sg.wmax == nullptr) return 1.0f;
    return ldexpf(1.0f, -(split_exp(__ldcg(sg.xmax)) + split_exp(__ldg(sg.wmax))));  // xmax: the previous kernel's
}

struct Args {
    int m, n, k, splits, kb_per_split, mt, nt, units;
    OutSeg seg[3];
    int nseg;
    float* partial;  // splits > 1: [splits][m][n] FP32
};

template <int BN, bool SPLIT>
struct Cfg {
    static constexpr int kBTile = BN * 128;
    // stage: X hi, W hi (then X lo, W lo in the split form)
    static constexpr int kStage = (SPLIT ? 2 : 1) * (kATile + kBTile);
    static constexpr int NS = SPLIT ? (BN == 256 ? 2 : 3) : (BN == 256 ? 4 : 6);
    static constexpr int kTmemCols = 2 * BN;
    static constexpr size_t kSmem = 1024 + (size_t)NS * kStage + 4 * 32 * kStageLd * 4 + 256;
};

template <int BN>
CL_DEVINL uint32_t instr_desc(int bf16) {
    // D = F32 (bits 4-5), A / B format (bits 7-9 / 10-12: 0 F16, 1 BF16),
    // both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
    return (1u << 4) | ((uint32_t)bf16 << 7) | ((uint32_t)bf16 << 10) | ((uint32_t)(BN >> 3) << 17) |
           ((uint32_t)(BM >> 4) << 24);
}

CL_DEVINL uint64_t smem_desc(uint32_t addr) {
    // K-major, 128-byte swizzle: rows of 128 B, 8-row groups 1024 B apart.
    uint64_t d = (uint64_t)((addr >> 4) & 0x3fffu);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

CL_DEVINL void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

CL_DEVINL void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
CL_DEVINL void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

CL_DEVINL void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}

CL_DEVINL void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

CL_DEVINL void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Unit u -> (row tile, column tile, K split); row tiles fastest.
CL_DEVINL void unit_of(const Args& a, int u, int& mt, int& nt, int& s) {
    mt = u % a.mt;
    const int r = u / a.mt;
    nt = r % a.nt;
    s = r / a.nt;
}

template <int BN, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1)
gemm16_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w,
              const __grid_constant__ CUtensorMap map_xl, const __grid_constant__ CUtensorMap map_wl,
              const __grid_constant__ Args a, int bf16) {
    using C = Cfg<BN, SPLIT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* stage_out = reinterpret_cast<float*>(ring + C::NS * C::kStage);  // [4][32][33]
    uint64_t* full = reinterpret_cast<uint64_t*>(stage_out + 4 * 32 * kStageLd);
    uint64_t* empty = full + C::NS;
    uint64_t* acc_full = empty + C::NS;   // [2] tcgen05.commit: the tile's MMAs finished
    uint64_t* acc_empty = acc_full + 2;   // [2] the epilogue warps drained the accumulator
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < C::NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(C::kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        fence_before_sync();
    }
    __syncthreads();
    fence_after_sync();
    grid_launch_dependents();
    // X comes from the previous kernel and the epilogue reads the residual:
    // every warp waits for the previous grid before touching either
    grid_wait();
    const uint32_t tmem = *tmem_slot;
    const int nkb = a.kb_per_split;

    if (warp == 0) {
        // ---- TMA producer ----
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_x)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_w)) : "memory");
            if (SPLIT) {
                asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_xl)) : "memory");
                asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map_wl)) : "memory");
            }
        }
        int it = 0;
        for (int u = blockIdx.x; u < a.units; u += gridDim.x) {
            if (__shfl_sync(0xffffffffu, *abort_flag, 0)) break;
            int mt, nt, sp;
            unit_of(a, u, mt, nt, sp);
            const int kb0 = sp * nkb, kb1 = min(kb0 + nkb, a.k / BK);
            for (int kb = kb0; kb < kb1; ++kb, ++it) {
                const int s = it % C::NS;
                const uint32_t ph = (uint32_t)(it / C::NS) & 1u;
                int ok = 1;
                if (lane == 0) {
                    ok = mbar_wait(&empty[s], ph ^ 1u);
                    if (ok) {
                        mbar_arrive_expect_tx(&full[s], (uint32_t)C::kStage);
                        uint8_t* st = ring + (size_t)s * C::kStage;
                        tma_load_2d(st, &map_x, kb * BK, mt * BM, &full[s]);
                        tma_load_2d(st + kATile, &map_w, kb * BK, nt * BN, &full[s]);
                        if (SPLIT) {
                            tma_load_2d(st + kATile + C::kBTile, &map_xl, kb * BK, mt * BM, &full[s]);
                            tma_load_2d(st + 2 * kATile + C::kBTile, &map_wl, kb * BK, nt * BN, &full[s]);
                        }
                    } else {
                        atomicExch(&g_g16_error, 1);
                        *abort_flag = 1;
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer ----
        const uint32_t idesc = instr_desc<BN>(bf16);
        int it = 0, t = 0;
        for (int u = blockIdx.x; u < a.units; u += gridDim.x, ++t) {
            if (__shfl_sync(0xffffffffu, *abort_flag, 0)) break;
            int mt, nt, sp;
            unit_of(a, u, mt, nt, sp);
            const int kb0 = sp * nkb, kb1 = min(kb0 + nkb, a.k / BK);
            const int b = t & 1;
            int ok = 1;
            if (lane == 0) {
                ok = t < 2 || mbar_wait(&acc_empty[b], (uint32_t)((t - 2) >> 1) & 1u);
                fence_after_sync();
                const uint32_t td = tmem + (uint32_t)(b * BN);
                for (int kb = kb0; ok && kb < kb1; ++kb, ++it) {
                    const int s = it % C::NS;
                    if (!mbar_wait(&full[s], (uint32_t)(it / C::NS) & 1u)) {
                        ok = 0;
                        break;
                    }
                    fence_after_sync();
                    const uint32_t st = smem_u32(ring + (size_t)s * C::kStage);
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {  // 4 k-steps of 16 elements (32 bytes) per 128-byte row
                        const uint64_t ah = smem_desc(st + 32u * kk), wh = smem_desc(st + kATile + 32u * kk);
                        mma_f16(td, ah, wh, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
                        if (SPLIT) {
                            const uint32_t lo = st + (uint32_t)(kATile + C::kBTile);
                            mma_f16(td, ah, smem_desc(lo + kATile + 32u * kk), idesc, 1u);  // Xhi Wlo
                            mma_f16(td, smem_desc(lo + 32u * kk), wh, idesc, 1u);           // Xlo Whi
                        }
                    }
                    mma_commit(&empty[s]);
                }
                if (ok) mma_commit(&acc_full[b]);
                if (!ok) {
                    atomicExch(&g_g16_error, 2);
                    *abort_flag = 1;
                }
            }
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) break;
        }
    } else {
        // ---- epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31 (output rows) ----
        const int q = warp & 3;
        float* st = stage_out + (size_t)(warp - 2) * 32 * kStageLd;
        int t = 0;
        for (int u = blockIdx.x; u < a.units; u += gridDim.x, ++t) {
            int mt, nt, sp;
            unit_of(a, u, mt, nt, sp);
            const int b = t & 1;
            const int ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[b], (uint32_t)(t >> 1) & 1u));
            if (!ok || __any_sync(0xffffffffu, *abort_flag != 0)) {
                if (lane == 0) {
                    if (!ok) atomicExch(&g_g16_error, 3);
                    *abort_flag = 1;
                }
                break;
            }
            fence_after_sync();
            const int r0 = mt * BM + 32 * q;
            const uint32_t base = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * BN);
#pragma unroll 1
            for (int j = 0; j < BN / 32; ++j) {
                uint32_t v[32];
                tmem_ld32(base + (uint32_t)(32 * j), v);
#pragma unroll
                for (int c = 0; c < 32; ++c) st[lane * kStageLd + c] = __uint_as_float(v[c]);
                __syncwarp();
                const int nn = nt * BN + 32 * j + lane;
                if (nn < a.n) {
                    if (a.splits > 1) {
                        float* pp = a.partial + (size_t)sp * a.m * a.n;
#pragma unroll 4
                        for (int rr = 0; rr < 32; ++rr) {
                            const int mm = r0 + rr;
                            if (mm < a.m) pp[(size_t)mm * a.n + nn] = st[rr * kStageLd + lane];
                        }
                    } else {
                        int si = 0;
                        if (a.nseg > 1 && nn >= a.seg[1].n0) si = 1;
                        if (a.nseg > 2 && nn >= a.seg[2].n0) si = 2;
                        const OutSeg& sg = a.seg[si];
                        const int col = nn - sg.n0;
                        const float bv = sg.bias ? sg.bias[col] : 0.0f;
                        const float us = SPLIT ? seg_unscale(sg) : 1.0f;
#pragma unroll 4
                        for (int rr = 0; rr < 32; ++rr) {
                            const int mm = r0 + rr;
                            if (mm < a.m) {
                                float o = st[rr * kStageLd + lane];
                                if (SPLIT) o *= us;
                                if (sg.bias) o += bv;
                                if (sg.res) o = sg.res[(size_t)mm * sg.ld + col] + o;
                                sg.y[(size_t)mm * sg.ld + col] = o;
                            }
                        }
                    }
                }
                __syncwarp();
            }
            fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols)
                     : "memory");
    }
}

// ---- weight / activation rounding ------------------------------------------------
// Split form: row r of `out` is [hi(k) | lo(k)] (FP16), else [16-bit(k)].
CL_DEVINL uint32_t pack16(float x0, float x1, int bf16) {
    if (bf16) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
        return *reinterpret_cast<const uint32_t*>(&h);
    }
    const __half2 h = __floats2half2_rn(x0, x1);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// x - fp16(x) (exact in FP32), rounded to FP16
CL_DEVINL uint32_t pack16_lo(float x0, float x1) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 b = __half22float2(h);
    const __half2 l = __floats2half2_rn(x0 - b.x, x1 - b.y);
    return *reinterpret_cast<const uint32_t*>(&l);
}

template <int T>
__global__ void dequant16_kernel(const uint8_t* __restrict__ w, long long stride, int n, int k, uint16_t* out,
                                 int bf16, const float* amax) {
    const int split = amax != nullptr;
    grid_launch_dependents();
    grid_wait();  // `out` may still be read by the previous kernel
    const int nc = k / 32;
    const long long total = (long long)n * nc;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / nc), c = (int)(i - (long long)r * nc);
        float v[32];
        dequant32<T>(w + (size_t)r * stride, k, c, v);
        if (split) {
            // the maximum comes from the previous kernel (amax_dequant_kernel): read it from L2
            const float sc = ldexpf(1.0f, split_exp(__ldcg(amax)));
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] *= sc;
        }
        uint16_t* row = out + (size_t)r * k * (split ? 2 : 1);
        uint4* o = reinterpret_cast<uint4*>(row + 32 * c);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t p[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) p[e] = pack16(v[8 * j + 2 * e], v[8 * j + 2 * e + 1], bf16);
            o[j] = make_uint4(p[0], p[1], p[2], p[3]);
        }
        if (split) {
            uint4* ol = reinterpret_cast<uint4*>(row + k + 32 * c);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint32_t p[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) p[e] = pack16_lo(v[8 * j + 2 * e], v[8 * j + 2 * e + 1]);
                ol[j] = make_uint4(p[0], p[1], p[2], p[3]);
            }
        }
    }
}

__global__ void convert16_kernel(const float* x, long long count, uint16_t* out, int bf16) {
    grid_launch_dependents();
    grid_wait();
    const long long n4 = count / 4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
         i += (long long)gridDim.x * blockDim.x) {
        const float4 f = reinterpret_cast<const float4*>(x)[i];
        uint32_t p0, p1;
        if (bf16) {
            const __nv_bfloat162 a = __floats2bfloat162_rn(f.x, f.y), b = __floats2bfloat162_rn(f.z, f.w);
            p0 = *reinterpret_cast<const uint32_t*>(&a);
            p1 = *reinterpret_cast<const uint32_t*>(&b);
        } else {
            const __half2 a = __floats2half2_rn(f.x, f.y), b = __floats2half2_rn(f.z, f.w);
            p0 = *reinterpret_cast<const uint32_t*>(&a);
            p1 = *reinterpret_cast<const uint32_t*>(&b);
        }
        reinterpret_cast<uint2*>(out)[i] = make_uint2(p0, p1);
    }
}

// Largest |value| (dequantized weight rows, or FP32 values) into *amax: a
// block maximum, then one atomic max on the float's bits (non-negative
// floats order as their bit patterns).
CL_DEVINL void amax_commit(float m, float* amax) {
    m = warp_max(m);
    __shared__ float red[8];
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
        atomicMax(reinterpret_cast<unsigned int*>(amax), __float_as_uint(m));
    }
}

template <int T>
__global__ void amax_dequant_kernel(const uint8_t* __restrict__ w, long long stride, int n, int k, float* amax) {
    grid_launch_dependents();
    grid_wait();
    const int nc = k / 32;
    const long long total = (long long)n * nc;
    float m = 0.0f;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / nc), c = (int)(i - (long long)r * nc);
        float v[32];
        dequant32<T>(w + (size_t)r * stride, k, c, v);
#pragma unroll
        for (int e = 0; e < 32; ++e) m = fmaxf(m, fabsf(v[e]));
    }
    amax_commit(m, amax);
}

__global__ void amax_kernel(const float* x, long long count, float* amax) {
    grid_launch_dependents();
    grid_wait();
    float m = 0.0f;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < count / 4;
         i += (long long)gridDim.x * blockDim.x) {
        const float4 f = reinterpret_cast<const float4*>(x)[i];
        m = fmaxf(fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y))), fmaxf(fabsf(f.z), fabsf(f.w)));
    }
    amax_commit(m, amax);
}

// X [rows][k] FP32 -> rows of [hi(k) | lo(k)] FP16 of X scaled by split_exp(*amax) (the split form).
__global__ void split16_kernel(const float* x, int rows, int k, const float* amax, uint16_t* out) {
    grid_launch_dependents();
    grid_wait();
    const float sc = ldexpf(1.0f, split_exp(__ldcg(amax)));  // written by the previous kernel: read from L2
    const int k4 = k / 4;
    const long long n4 = (long long)rows * k4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4;
         i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / k4), c = (int)(i - (long long)r * k4);
        float4 f = reinterpret_cast<const float4*>(x)[i];
        f.x *= sc;
        f.y *= sc;
        f.z *= sc;
        f.w *= sc;
        uint16_t* row = out + (size_t)r * 2 * k;
        reinterpret_cast<uint2*>(row)[c] = make_uint2(pack16(f.x, f.y, 0), pack16(f.z, f.w, 0));
        reinterpret_cast<uint2*>(row + k)[c] = make_uint2(pack16_lo(f.x, f.y), pack16_lo(f.z, f.w));
    }
}

// Sum of the K splits in split order, then bias / residual, per segment.
__global__ void splitk_reduce_kernel(const __grid_constant__ Args a) {
    grid_launch_dependents();
    grid_wait();
    const long long total = (long long)a.m * a.n;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int mm = (int)(i / a.n), nn = (int)(i - (long long)mm * a.n);
        float o = a.partial[i];
        for (int s = 1; s < a.splits; ++s) o += a.partial[(size_t)s * total + i];
        int si = 0;
        if (a.nseg > 1 && nn >= a.seg[1].n0) si = 1;
        if (a.nseg > 2 && nn >= a.seg[2].n0) si = 2;
        const OutSeg& sg = a.seg[si];
        const int col = nn - sg.n0;
        o *= seg_unscale(sg);
        if (sg.bias) o += sg.bias[col];
        if (sg.res) o = sg.res[(size_t)mm * sg.ld + col] + o;
        sg.y[(size_t)mm * sg.ld + col] = o;
    }
}

// ---- host -------------------------------------------------------------------------
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
    static std::once_flag once;
    static EncodeTiled fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

// Row-major [rows, k] 16-bit matrix with rows ld elements apart, box = 64
// columns x box_rows rows, 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* base, int rows, int k, long long ld, int box_rows, int bf16) {
    EncodeTiled fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
              const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// (BN, splits) with the fewest waves of equal-work units over the SMs; ties
// to the larger tile, then to fewer splits.
void plan(int m, int n, int k, int sms, int mmas, int& bn, int& splits) {
    const int mt = (m + BM - 1) / BM, nkb = k / BK;
    double best = 1e300;
    bn = 256;
    splits = 1;
    for (int b : {256, 128}) {
        const int nt = (n + b - 1) / b;
        for (int s = 1; s <= 8; ++s) {
            if (s > 1 && nkb / s < 8) break;  // keep at least 8 k-blocks per unit
            const int per = (nkb + s - 1) / s;
            const long long units = (long long)mt * nt * s;
            const long long waves = (units + sms - 1) / sms;
            // unit time ~ k-blocks x (BN / 256 + a fixed share for the X tile
            // and the epilogue), one 256-wide k-block ~ 0.26 us; a split adds
            // the FP32 partials' write and re-read at ~6.5 TB/s
            // (mmas products per k-block in the split form)
            const double penalty = s > 1 ? (double)m * n * s * 8.0 / 6.5e12 / 0.26e-6 : 0.0;
            const double cost = (double)waves * per * (mmas * b / 256.0 + 0.25) + penalty;
            if (cost < best * 0.999) {
                best = cost;
                bn = b;
                splits = s;
            }
        }
    }
}

template <int BN, bool SPLIT>
cudaError_t launch_gemm(const CUtensorMap& mx, const CUtensorMap& mw, const CUtensorMap& mxl,
                        const CUtensorMap& mwl, const Args& a, int bf16, int sms, cudaStream_t stream) {
    static SmemLimit limit;
    cudaError_t e = limit.ensure(gemm16_kernel<BN, SPLIT>, (int)Cfg<BN, SPLIT>::kSmem);
    if (e != cudaSuccess) return e;
    const int grid = std::min(a.units, sms);
    return launch_pdl(gemm16_kernel<BN, SPLIT>, dim3(grid), dim3(kThreads), Cfg<BN, SPLIT>::kSmem, stream, mx, mw,
                      mxl, mwl, a, bf16);
}

int dequant16_launch(int type, const void* w, long long stride, int n, int k, void* out, int bf, const float* amax,
                     cudaStream_t stream) {
    const uint8_t* wp = static_cast<const uint8_t*>(w);
    uint16_t* o = static_cast<uint16_t*>(out);
    const long long chunks = (long long)n * (k / 32);
    const int grid = (int)std::min<long long>((chunks + 255) / 256, 148LL * 16);
    cudaError_t e;
    switch (type) {
    case CL_TYPE_Q4_K: e = launch_pdl(dequant16_kernel<CL_TYPE_Q4_K>, dim3(grid), dim3(256), 0, stream, wp, stride, n, k, o, bf, amax); break;
    case CL_TYPE_Q5_K: e = launch_pdl(dequant16_kernel<CL_TYPE_Q5_K>, dim3(grid), dim3(256), 0, stream, wp, stride, n, k, o, bf, amax); break;
    case CL_TYPE_Q6_K: e = launch_pdl(dequant16_kernel<CL_TYPE_Q6_K>, dim3(grid), dim3(256), 0, stream, wp, stride, n, k, o, bf, amax); break;
    case CL_TYPE_Q8_0: e = launch_pdl(dequant16_kernel<CL_TYPE_Q8_0>, dim3(grid), dim3(256), 0, stream, wp, stride, n, k, o, bf, amax); break;
    case CL_TYPE_Q5_0: e = launch_pdl(dequant16_kernel<CL_TYPE_Q5_0>, dim3(grid), dim3(256), 0, stream, wp, stride, n, k, o, bf, amax); break;
    case CL_TYPE_F32: e = launch_pdl(dequant16_kernel<CL_TYPE_F32>, dim3(grid), dim3(256), 0, stream, wp, stride, n, k, o, bf, amax); break;
    case CL_TYPE_F16: e = launch_pdl(dequant16_kernel<CL_TYPE_F16>, dim3(grid), dim3(256), 0, stream, wp, stride, n, k, o, bf, amax); break;
    default: return CL_ERR_UNSUPPORTED;
    }
    return e == cudaSuccess ? CL_OK : CL_ERR_CUDA;
}

}  // namespace g16

int gemm16_device_error(int* code, bool clear) {
    if (cudaMemcpyFromSymbol(code, g16::g_g16_error, sizeof(int)) != cudaSuccess) return CL_ERR_CUDA;
    if (clear) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g16::g_g16_error, &zero, sizeof(int)) != cudaSuccess) return CL_ERR_CUDA;
    }
    return CL_OK;
}

}  // namespace cl

using namespace cl;
using namespace cl::g16;

extern "C" {

CL_API int cl_dequant16(int type, const void* w, long long stride, int n, int k, void* out, int format,
                        cudaStream_t stream) {
    if (w == nullptr || out == nullptr || n <= 0 || k <= 0 || k % 32 || cl_native_row_bytes(type, k) < 0 ||
        stride < cl_row_stride(type, k) || (format != CL_GEMM_F16 && format != CL_GEMM_BF16))
        return CL_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(out)) % 16 || stride % 16)
        return CL_ERR_INVALID;
    return g16::dequant16_launch(type, w, stride, n, k, out, format == CL_GEMM_BF16, nullptr, stream);
}

CL_API int cl_amax_dequant(int type, const void* w, long long stride, int n, int k, float* amax,
                           cudaStream_t stream) {
    if (w == nullptr || amax == nullptr || n <= 0 || k <= 0 || k % 32 || cl_native_row_bytes(type, k) < 0 ||
        stride < cl_row_stride(type, k) || (reinterpret_cast<uintptr_t>(amax) & 3u))
        return CL_ERR_INVALID;
    if (cudaMemsetAsync(amax, 0, sizeof(float), stream) != cudaSuccess) return CL_ERR_CUDA;
    const uint8_t* wp = static_cast<const uint8_t*>(w);
    const long long chunks = (long long)n * (k / 32);
    const int grid = (int)std::min<long long>((chunks + 255) / 256, 148LL * 16);
    cudaError_t e;
    switch (type) {
    case CL_TYPE_Q4_K: e = launch_pdl(amax_dequant_kernel<CL_TYPE_Q4_K>, dim3(grid), dim3(256), 0, stream, wp, stride, n, k, amax); break;
    case CL_TYPE_Q5_K: e = launch_pdl(amax_dequant_kernel<CL_TYPE_Q5_K>, dim3(grid), dim3(256), 0, stream, wp, stride, n, k, amax); break;
    case CL_TYPE_Q6_K: e = launch_pdl(amax_dequant_kernel<CL_TYPE_Q6_K>, dim3(grid), dim3(256), 0, stream, wp, stride, n, k, amax); break;
    case CL_TYPE_Q8_0: e = launch_pdl(amax_dequant_kernel<CL_TYPE_Q8_0>, dim3(grid), dim3(256), 0, stream, wp, stride, n, k, amax); break;
    case CL_TYPE_Q5_0: e = launch_pdl(amax_dequant_kernel<CL_TYPE_Q5_0>, dim3(grid), dim3(256), 0, stream, wp, stride, n, k, amax); break;
    case CL_TYPE_F32: e = launch_pdl(amax_dequant_kernel<CL_TYPE_F32>, dim3(grid), dim3(256), 0, stream, wp, stride, n, k, amax); break;
    case CL_TYPE_F16: e = launch_pdl(amax_dequant_kernel<CL_TYPE_F16>, dim3(grid), dim3(256), 0, stream, wp, stride, n, k, amax); break;
    default: return CL_ERR_UNSUPPORTED;
    }
    return e == cudaSuccess ? CL_OK : CL_ERR_CUDA;
}

CL_API int cl_dequant16_split(int type, const void* w, long long stride, int n, int k, const float* amax, void* out,
                              cudaStream_t stream) {
    if (w == nullptr || out == nullptr || amax == nullptr || n <= 0 || k <= 0 || k % 32 ||
        cl_native_row_bytes(type, k) < 0 || stride < cl_row_stride(type, k))
        return CL_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(out)) % 16 || stride % 16 ||
        (reinterpret_cast<uintptr_t>(amax) & 3u))
        return CL_ERR_INVALID;
    return g16::dequant16_launch(type, w, stride, n, k, out, 0, amax, stream);
}

CL_API int cl_amax(const float* x, long long count, float* amax, cudaStream_t stream) {
    if (x == nullptr || amax == nullptr || count <= 0 || count % 4 || (reinterpret_cast<uintptr_t>(x) % 16) ||
        (reinterpret_cast<uintptr_t>(amax) & 3u))
        return CL_ERR_INVALID;
    if (cudaMemsetAsync(amax, 0, sizeof(float), stream) != cudaSuccess) return CL_ERR_CUDA;
    const int grid = (int)std::min<long long>((count / 4 + 255) / 256, 148LL * 4);
    return launch_pdl(amax_kernel, dim3(grid), dim3(256), 0, stream, x, count, amax) == cudaSuccess ? CL_OK
                                                                                                  : CL_ERR_CUDA;
}

CL_API int cl_convert16(const float* x, long long count, void* out, int format, cudaStream_t stream) {
    if (x == nullptr || out == nullptr || count <= 0 || count % 4 || (format != CL_GEMM_F16 && format != CL_GEMM_BF16))
        return CL_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) % 16) return CL_ERR_INVALID;
    const int grid = (int)std::min<long long>((count / 4 + 255) / 256, 148LL * 8);
    return launch_pdl(convert16_kernel, dim3(grid), dim3(256), 0, stream, x, count, static_cast<uint16_t*>(out),
                      format == CL_GEMM_BF16 ? 1 : 0) == cudaSuccess
               ? CL_OK
               : CL_ERR_CUDA;
}

CL_API int cl_split16(const float* x, int rows, int k, const float* amax, void* out, cudaStream_t stream) {
    if (x == nullptr || out == nullptr || amax == nullptr || rows <= 0 || k <= 0 || k % 4) return CL_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out)) % 16 ||
        (reinterpret_cast<uintptr_t>(amax) & 3u))
        return CL_ERR_INVALID;
    const long long n4 = (long long)rows * (k / 4);
    const int grid = (int)std::min<long long>((n4 + 255) / 256, 148LL * 8);
    return launch_pdl(split16_kernel, dim3(grid), dim3(256), 0, stream, x, rows, k, amax,
                      static_cast<uint16_t*>(out)) == cudaSuccess
               ? CL_OK
               : CL_ERR_CUDA;
}

CL_API size_t cl_gemm16_workspace_bytes(int m, int n, int k) {
    if (m <= 0 || n <= 0 || k <= 0) return 0;
    return (size_t)8 * m * n * 4;  // up to 8 K splits of FP32 partials
}

CL_API int cl_gemm16_run(const void* w16, int n, int k, const void* x16, int m, const cl_gemm_out* outs, int nout,
                         int format, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (w16 == nullptr || x16 == nullptr || outs == nullptr || nout < 1 || nout > 3 || m <= 0 || n <= 0 ||
        k <= 0 || k % BK || (format != CL_GEMM_F16 && format != CL_GEMM_BF16 && format != CL_GEMM_F16X3))
        return CL_ERR_INVALID;
    // TMA: 16-byte aligned bases (the tensor maps also want row strides that are multiples of 16 bytes)
    if ((reinterpret_cast<uintptr_t>(w16) | reinterpret_cast<uintptr_t>(x16)) % 16) return CL_ERR_INVALID;
    const bool sp = format == CL_GEMM_F16X3;
    Args a{};
    a.m = m;
    a.n = n;
    a.k = k;
    a.nseg = nout;
    int prev = 0;
    for (int i = 0; i < nout; ++i) {
        const cl_gemm_out& o = outs[i];
        if (o.y == nullptr || o.col0 != prev || o.cols <= 0 || o.ld < o.cols) return CL_ERR_INVALID;
        if (sp != (o.xmax != nullptr && o.wmax != nullptr)) return CL_ERR_INVALID;  // the split form's scales
        a.seg[i] = OutSeg{o.y, o.bias, o.residual, o.xmax, o.wmax, o.col0, o.col0 + o.cols, o.ld};
        prev = o.col0 + o.cols;
    }
    if (prev != n) return CL_ERR_INVALID;
    int sms = 0;
    if (device_sm_count(&sms) != cudaSuccess) return CL_ERR_CUDA;
    int bn = 256, splits = 1;
    plan(m, n, k, sms, sp ? 3 : 1, bn, splits);
    if (splits > 1 && (workspace == nullptr || workspace_bytes < (size_t)splits * m * n * 4)) splits = 1;
    const int nkb = k / BK;
    a.splits = splits;
    a.kb_per_split = (nkb + splits - 1) / splits;
    a.mt = (m + BM - 1) / BM;
    a.nt = (n + bn - 1) / bn;
    a.units = a.mt * a.nt * splits;
    a.partial = static_cast<float*>(workspace);
    const int bf = format == CL_GEMM_BF16;
    const long long ld = sp ? 2LL * k : k;  // split form: [hi | lo] rows
    CUtensorMap mx, mw, mxl, mwl;
    if (!make_map(&mx, x16, m, k, ld, BM, bf) || !make_map(&mw, w16, n, k, ld, bn, bf)) return CL_ERR_UNSUPPORTED;
    if (sp) {
        if (!make_map(&mxl, static_cast<const uint16_t*>(x16) + k, m, k, ld, BM, 0) ||
            !make_map(&mwl, static_cast<const uint16_t*>(w16) + k, n, k, ld, bn, 0))
            return CL_ERR_UNSUPPORTED;
    } else {
        mxl = mx;
        mwl = mw;
    }
    cudaError_t e;
    if (sp)
        e = bn == 256 ? launch_gemm<256, true>(mx, mw, mxl, mwl, a, bf, sms, stream)
                      : launch_gemm<128, true>(mx, mw, mxl, mwl, a, bf, sms, stream);
    else
        e = bn == 256 ? launch_gemm<256, false>(mx, mw, mxl, mwl, a, bf, sms, stream)
                      : launch_gemm<128, false>(mx, mw, mxl, mwl, a, bf, sms, stream);
    if (e != cudaSuccess) return CL_ERR_CUDA;
    if (splits > 1) {
        const long long total = (long long)m * n;
        const int grid = (int)std::min<long long>((total + 255) / 256, (long long)sms * 8);
        if (launch_pdl(splitk_reduce_kernel, dim3(grid), dim3(256), 0, stream, a) != cudaSuccess) return CL_ERR_CUDA;
    }
    return CL_OK;
}

}  // extern "C"
