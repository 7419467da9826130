// Prefill GEMM on the 5th-generation tensor cores: Y[m,n] = X[m,k] W[n,k]^T
// (+ bias) (+ residual), X FP32 row-major, W native GGML blocks in the device
// layout.
//
// Reference: metal_gemm_{q5_0,q8_0,q4_k,q5_k,q6_k}_f32 (metal_llm.metal:621-704)
// and gemmtb/gemmt (cpu_llm.cpp:591-653), both FP32.  Here a CTA owns a
// 128 x 128 output tile and walks K through a shared-memory ring whose
// stages are 128-byte rows (canonical K-major, 128-byte swizzle):
//   * warps 0-3 load the X rows (FP32 from HBM),
//   * warps 4-7 dequantize the W rows with the CPU decoder's FP32
//     expressions (the reference's exact FP32 weights),
//   * one elected thread of warp 8 issues tcgen05.mma with the FP32
//     accumulator in TMEM; tcgen05.commit frees a stage when its MMAs finish,
//   * warps 0-3 read the accumulator back with tcgen05.ld (one TMEM lane per
//     output row), stage it through shared memory and store rows with
//     bias / residual applied.
// Two precisions:
//   CL_GEMM_TF32X3 (default) — each FP32 operand is split into a TF32 head and
//     a TF32 tail (x = hi + lo to within 2^-22 |x|); three MMAs per k-step,
//     hi*hi + hi*lo + lo*hi, give FP32-grade products (the dropped lo*lo term
//     is below 2^-22 relative).  32 K columns per stage.
//   CL_GEMM_F16 — operands rounded once to FP16, one MMA per k-step (11-bit
//     significands; faster, lower precision).  64 K columns per stage.
// Every mbarrier wait is bounded; TMEM is always released.
#include "common.cuh"
#include "dequant.cuh"
#include "launch.cuh"

namespace cl {

namespace tc {

constexpr int BM = 128, BN = 128;
constexpr int kThreads = 288;          // warps 0-7 producers (0-3 also epilogue), warp 8 TMEM + MMA
constexpr int kTile = BM * 128;        // one 128-row x 128-byte operand tile: 16 KB


__device__ int g_tc_error = 0;

template <bool X3>
struct Mode {
    static constexpr int BK = X3 ? 32 : 64;           // K elements per 128-byte row
    static constexpr int NS = X3 ? 3 : 4;             // ring stages
    static constexpr int kTiles = X3 ? 4 : 2;         // X3: A hi, A lo, B hi, B lo; F16: A, B
    static constexpr int kStageBytes = kTiles * kTile;
    static constexpr int kBTile = X3 ? 2 : 1;         // index of the first B tile in a stage
    // Instruction descriptor: D = F32 (bits 4-5), A/B format (bits 7-9 /
    // 10-12: F16 = 0 for kind::f16, TF32 = 2 for kind::tf32), both K-major,
    // N >> 3 at bit 17, M >> 4 at bit 24.
    static constexpr uint32_t kInstr = (1u << 4) | (X3 ? (2u << 7) | (2u << 10) : 0u) |
                                       ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
    static constexpr size_t kSmem = (size_t)NS * kStageBytes + 1024 + 256;
    // TMEM: FP32 accumulators of 128 lanes x 128 columns.  F16: one.  X3: two
    // for the hi*hi products, used in turn per chunk of CH k-blocks, plus one
    // (columns 256-383) for the small hi*lo + lo*hi terms over all of K.  The
    // tensor core's FP32 accumulation does not round to nearest, so its error
    // grows with the number of additions into a large sum; folding each
    // chunk into registers with round-to-nearest adds keeps the result at
    // FP32-sequential accuracy for every K.
    static constexpr int CH = 32;
    static constexpr int kTmemCols = X3 ? 512 : 128;
};

CL_DEVINL uint64_t smem_desc(uint32_t addr) {
    // K-major, 128-byte swizzle: rows of 128 B, 8-row groups 1024 B apart.
    uint64_t d = (uint64_t)((addr >> 4) & 0x3fffu);
    d |= (uint64_t)1 << 16;             // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset
    d |= (uint64_t)1 << 46;             // descriptor version (sm100)
    d |= (uint64_t)2 << 61;             // SWIZZLE_128B
    return d;
}

template <bool X3>
CL_DEVINL void mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    if constexpr (X3) {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(adesc), "l"(bdesc), "r"(Mode<true>::kInstr), "r"(accumulate)
            : "memory");
    } else {
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
            "l"(adesc), "l"(bdesc), "r"(Mode<false>::kInstr), "r"(accumulate)
            : "memory");
    }
}

CL_DEVINL void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

CL_DEVINL void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
CL_DEVINL void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
CL_DEVINL void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

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

// Byte offset of 16-byte chunk j of row r in a 128-byte-swizzled tile whose
// base is 1024-byte aligned (address bits 4-6 XOR bits 7-9).
CL_DEVINL int swz(int r, int j) { return r * 128 + ((j ^ (r & 7)) << 4); }

// 32 values as FP16 into chunks [4 q, 4 q + 4) of row r.
CL_DEVINL void store_f16(uint8_t* tile, int r, int q, const float (&v)[32]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint4 u;
        uint32_t* up = &u.x;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __half2 h = __floats2half2_rn(v[8 * j + 2 * i], v[8 * j + 2 * i + 1]);
            up[i] = *reinterpret_cast<const uint32_t*>(&h);
        }
        *reinterpret_cast<uint4*>(tile + swz(r, 4 * q + j)) = u;
    }
}

CL_DEVINL uint32_t to_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

// 32 values split into a TF32 head (hi tile) and the TF32 rounding of the
// remainder (lo tile), row r.
CL_DEVINL void store_tf32x2(uint8_t* hi, uint8_t* lo, int r, const float (&v)[32]) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        uint4 h, l;
        uint32_t* hp = &h.x;
        uint32_t* lp = &l.x;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float x = v[4 * j + i];
            const uint32_t t = to_tf32(x);
            hp[i] = t;
            lp[i] = to_tf32(__fsub_rn(x, __uint_as_float(t)));
        }
        *reinterpret_cast<uint4*>(hi + swz(r, j)) = h;
        *reinterpret_cast<uint4*>(lo + swz(r, j)) = l;
    }
}

CL_DEVINL void zero_row(uint8_t* tile, int r) {
#pragma unroll
    for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(tile + r * 128 + (j << 4)) = make_uint4(0, 0, 0, 0);
}

// 32 FP32 activations of row mm, columns [32 c, 32 c + 32).
CL_DEVINL void load_x32(const float* x, int k, int mm, int c, float (&v)[32]) {
    const float4* p = reinterpret_cast<const float4*>(x + (size_t)mm * k) + 8 * c;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 f = p[i];
        v[4 * i] = f.x, v[4 * i + 1] = f.y, v[4 * i + 2] = f.z, v[4 * i + 3] = f.w;
    }
}

// ---------------------------------------------------------------------------
// The kernel.  Shared memory: NS stages x kTiles tiles (1024-byte aligned),
// then full[NS], empty[NS], done, the TMEM address and an abort word.
// ---------------------------------------------------------------------------
template <int T, bool X3>
__global__ void __launch_bounds__(kThreads, 1)
gemm_tc_kernel(const uint8_t* __restrict__ w, long long stride, int n, int k, const float* x, int m,
               const float* __restrict__ bias, const float* res, float* y) {
    using P = Mode<X3>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(ring + P::NS * P::kStageBytes);
    uint64_t* empty = full + P::NS;
    uint64_t* done = empty + P::NS;
    uint64_t* chunk_full = done + 1;       // [2] X3: the MMAs of a chunk finished
    uint64_t* chunk_empty = chunk_full + 2;  // [2] X3: the chunk's accumulator was folded
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(chunk_empty + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // blockIdx.x walks M so the CTAs sharing one weight tile run together (L2 reuse)
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    const int nkb = k / P::BK;
    const int nchunks = (nkb + P::CH - 1) / P::CH;
    if (tid == 0) {
        for (int s = 0; s < P::NS; ++s) {
            mbar_init(&full[s], 8);   // one arrival per producer warp
            mbar_init(&empty[s], 1);  // tcgen05.commit
        }
        mbar_init(done, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&chunk_full[b], 1);   // tcgen05.commit
            mbar_init(&chunk_empty[b], 8);  // one arrival per folding warp
        }
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 8) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(P::kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
        fence_before_sync();
    }
    __syncthreads();
    fence_after_sync();
    grid_launch_dependents();
    const uint32_t tmem = *tmem_slot;
    // Warps 0-7 share the accumulator readback: warp w owns TMEM lanes
    // (rows) 32 (w & 3) .. + 31 and columns 64 (w >> 2) .. + 63.
    constexpr int kHalf = BN / 2;
    const uint32_t lane_base = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(kHalf * (warp >> 2));

    // X3: each producer warp folds every finished chunk accumulator into FP32
    // sums (its row, its 64 columns) with round-to-nearest adds.
    float sums[X3 ? kHalf : 1];
#pragma unroll
    for (int i = 0; i < (X3 ? kHalf : 1); ++i) sums[i] = 0.0f;
    int folded = 0;  // chunks folded so far
    bool ok = true;  // warp-uniform

    auto fold = [&](int c) {
        // chunk c's accumulator -> sums; then release it to the MMA issuer
        const int b = c & 1;
        ok = ok && __all_sync(0xffffffffu, mbar_wait(&chunk_full[b], (uint32_t)(c >> 1) & 1u));
        fence_after_sync();
        if (ok) {
#pragma unroll
            for (int j = 0; j < kHalf / 32; ++j) {
                uint32_t a[32];
                tmem_ld32(lane_base + (uint32_t)(b * BN + 32 * j), a);
#pragma unroll
                for (int i = 0; i < 32; ++i) sums[32 * j + i] = __fadd_rn(sums[32 * j + i], __uint_as_float(a[i]));
            }
        }
        fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&chunk_empty[b]);
    };

    if (warp < 8) {
        // ---- producers: X rows (warps 0-3), dequantized W rows (warps 4-7) ----
        grid_wait();
        const bool is_a = warp < 4;
        const int r = is_a ? tid : tid - 128;
        const int g = is_a ? m0 + r : n0 + r;
        const bool live = g < (is_a ? m : n);
        const uint8_t* wrow = w + (size_t)(live && !is_a ? g : 0) * stride;
        for (int kb = 0; kb < nkb; ++kb) {
            if constexpr (X3) {
                // fold chunk c once NS - 1 stages of chunk c + 1 are queued:
                // its MMAs are then finished or nearly so, and the issuer
                // needs the accumulator back only at chunk c + 2.
                const int t = kb - (P::NS - 1);
                if (t > 0 && t % P::CH == 0) {
                    fold(t / P::CH - 1);
                    ++folded;
                    if (!ok) {
                        if (lane == 0) atomicExch(&g_tc_error, 4);
                        *abort_flag = 1;
                        break;
                    }
                }
            }
            const int s = kb % P::NS;
            const uint32_t ph = (uint32_t)(kb / P::NS) & 1u;
            // warp-uniform exits keep the later __syncwarp / .aligned ops convergent
            if (!__all_sync(0xffffffffu, mbar_wait(&empty[s], ph ^ 1u))) {
                if (lane == 0) atomicExch(&g_tc_error, 1);
                *abort_flag = 1;
                ok = false;
                break;
            }
            if (__any_sync(0xffffffffu, *abort_flag != 0)) {
                ok = false;
                break;
            }
            uint8_t* t0 = ring + s * P::kStageBytes + (is_a ? 0 : P::kBTile * kTile);
#pragma unroll 1
            for (int q = 0; q < P::BK / 32; ++q) {
                const int c = kb * (P::BK / 32) + q;
                if (!live) {
                    if (q == 0) {
                        zero_row(t0, r);
                        if constexpr (X3) zero_row(t0 + kTile, r);
                    }
                    continue;
                }
                float v[32];
                if (is_a)
                    load_x32(x, k, g, c, v);
                else
                    dequant32<T>(wrow, k, c, v);
                if constexpr (X3)
                    store_tf32x2(t0, t0 + kTile, r, v);
                else
                    store_f16(t0, r, q, v);
            }
            fence_proxy_async();  // generic-proxy smem writes -> visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[s]);
        }
    } else if (lane == 0) {
        // ---- MMA issuer ----
        for (int kb = 0; kb < nkb; ++kb) {
            const int s = kb % P::NS;
            const uint32_t ph = (uint32_t)(kb / P::NS) & 1u;
            const int c = kb / P::CH, kc = kb % P::CH;
            if (X3 && kc == 0 && c >= 2) {
                // accumulator c & 1 is reused: chunk c - 2 must be folded
                if (!mbar_wait(&chunk_empty[c & 1], (uint32_t)((c - 2) >> 1) & 1u)) {
                    atomicExch(&g_tc_error, 5);
                    *abort_flag = 1;
                    break;
                }
            }
            if (!mbar_wait(&full[s], ph)) {
                atomicExch(&g_tc_error, 2);
                *abort_flag = 1;
                break;
            }
            fence_after_sync();
            const uint32_t st = smem_u32(ring + s * P::kStageBytes);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {  // 4 k-steps of 32 bytes per 128-byte row
                const uint32_t off = 32u * kk;
                if constexpr (X3) {
                    const uint64_t ahi = smem_desc(st + off), alo = smem_desc(st + kTile + off);
                    const uint64_t bhi = smem_desc(st + 2 * kTile + off), blo = smem_desc(st + 3 * kTile + off);
                    const uint32_t tsmall = tmem + 2 * BN, tbig = tmem + (uint32_t)((c & 1) * BN);
                    mma<true>(tsmall, alo, bhi, (kb | kk) != 0 ? 1u : 0u);
                    mma<true>(tsmall, ahi, blo, 1u);
                    mma<true>(tbig, ahi, bhi, (kc | kk) != 0 ? 1u : 0u);
                } else {
                    mma<false>(tmem, smem_desc(st + off), smem_desc(st + kTile + off), (kb | kk) != 0 ? 1u : 0u);
                }
            }
            mma_commit(&empty[s]);  // stage s is free once these MMAs have read it
            if (X3 && (kc == P::CH - 1 || kb == nkb - 1)) mma_commit(&chunk_full[c & 1]);
        }
        mma_commit(done);  // also after an error: done then means "no MMA of this CTA in flight"
    }

    if (warp < 8) {
        // ---- epilogue: TMEM lane = output row; warp w: rows 32 (w & 3) ..,
        // columns 64 (w >> 2) .. ----
        ok = ok && __all_sync(0xffffffffu, mbar_wait(done, 0));
        fence_after_sync();
        if (!ok && lane == 0) atomicExch(&g_tc_error, 3);
        ok = ok && !__any_sync(0xffffffffu, *abort_flag != 0);
        if constexpr (X3) {
            // the last one or two chunks were not folded in the loop
            if (ok) {
                for (int c = folded; c < nchunks; ++c) {
                    const int b = c & 1;
#pragma unroll
                    for (int j = 0; j < kHalf / 32; ++j) {
                        uint32_t a[32];
                        tmem_ld32(lane_base + (uint32_t)(b * BN + 32 * j), a);
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            sums[32 * j + i] = __fadd_rn(sums[32 * j + i], __uint_as_float(a[i]));
                    }
                }
            }
        }
        if (ok) {
            // Each 32 x 32 block goes through shared memory (the drained ring)
            // so the global stores are row-contiguous.
            float* st = reinterpret_cast<float*>(ring) + warp * 32 * 33;
            const int rbase = m0 + 32 * (warp & 3);
#pragma unroll
            for (int j = 0; j < kHalf / 32; ++j) {
                uint32_t a[32];
                tmem_ld32(lane_base + (uint32_t)((X3 ? 2 * BN : 0) + 32 * j), a);
#pragma unroll
                for (int c = 0; c < 32; ++c) {
                    const float v = __uint_as_float(a[c]);
                    st[lane * 33 + c] = X3 ? __fadd_rn(sums[(X3 ? 32 * j + c : 0)], v) : v;
                }
                __syncwarp();
                const int nn = n0 + kHalf * (warp >> 2) + 32 * j + lane;
                if (nn < n) {
                    const float bv = bias ? bias[nn] : 0.0f;
#pragma unroll 4
                    for (int rr = 0; rr < 32; ++rr) {
                        const int mm = rbase + rr;
                        if (mm < m) {
                            float o = st[rr * 33 + lane];
                            if (bias) o += bv;
                            if (res) o = res[(size_t)mm * n + nn] + o;
                            y[(size_t)mm * n + nn] = o;
                        }
                    }
                }
                __syncwarp();
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 8) {
        fence_after_sync();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(P::kTmemCols)
                     : "memory");
    }
}

}  // namespace tc

int gemm_tc_device_error(int* code, bool clear) {
    if (cudaMemcpyFromSymbol(code, tc::g_tc_error, sizeof(int)) != cudaSuccess) return CL_ERR_CUDA;
    if (clear) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(tc::g_tc_error, &zero, sizeof(int)) != cudaSuccess) return CL_ERR_CUDA;
    }
    return CL_OK;
}

bool gemm_tc_supported(int type, int n, int k, int m, int precision) {
    const int bk = precision == CL_GEMM_F16 ? 64 : 32;
    return (precision == CL_GEMM_TF32X3 || precision == CL_GEMM_F16) && k % bk == 0 && n > 0 && m > 0 &&
           (n + tc::BN - 1) / tc::BN <= 65535 &&
           (type == CL_TYPE_Q4_K || type == CL_TYPE_Q5_K || type == CL_TYPE_Q6_K || type == CL_TYPE_Q8_0 ||
            type == CL_TYPE_Q5_0 || type == CL_TYPE_F32 || type == CL_TYPE_F16);
}

namespace {

template <int T, bool X3>
int launch_tc_fmt(const void* w, long long stride, int n, int k, const float* x, int m, const float* bias,
                  const float* residual, float* y, cudaStream_t stream) {
    using P = tc::Mode<X3>;
    static SmemLimit limit;
    if (limit.ensure(tc::gemm_tc_kernel<T, X3>, (int)P::kSmem) != cudaSuccess) return CL_ERR_CUDA;
    const dim3 grid((m + tc::BM - 1) / tc::BM, (n + tc::BN - 1) / tc::BN);
    return launch_pdl(tc::gemm_tc_kernel<T, X3>, grid, dim3(tc::kThreads), P::kSmem, stream,
                      static_cast<const uint8_t*>(w), stride, n, k, x, m, bias, residual, y) == cudaSuccess
               ? CL_OK
               : CL_ERR_CUDA;
}

template <bool X3>
int launch_tc_mode(int type, const void* w, long long stride, int n, int k, const float* x, int m,
                   const float* bias, const float* residual, float* y, cudaStream_t stream) {
    switch (type) {
    case CL_TYPE_Q4_K: return launch_tc_fmt<CL_TYPE_Q4_K, X3>(w, stride, n, k, x, m, bias, residual, y, stream);
    case CL_TYPE_Q5_K: return launch_tc_fmt<CL_TYPE_Q5_K, X3>(w, stride, n, k, x, m, bias, residual, y, stream);
    case CL_TYPE_Q6_K: return launch_tc_fmt<CL_TYPE_Q6_K, X3>(w, stride, n, k, x, m, bias, residual, y, stream);
    case CL_TYPE_Q8_0: return launch_tc_fmt<CL_TYPE_Q8_0, X3>(w, stride, n, k, x, m, bias, residual, y, stream);
    case CL_TYPE_Q5_0: return launch_tc_fmt<CL_TYPE_Q5_0, X3>(w, stride, n, k, x, m, bias, residual, y, stream);
    case CL_TYPE_F32: return launch_tc_fmt<CL_TYPE_F32, X3>(w, stride, n, k, x, m, bias, residual, y, stream);
    case CL_TYPE_F16: return launch_tc_fmt<CL_TYPE_F16, X3>(w, stride, n, k, x, m, bias, residual, y, stream);
    default: return CL_ERR_UNSUPPORTED;
    }
}

}  // namespace

int launch_gemm_tc(int type, const void* w, long long stride, int n, int k, const float* x, int m, const float* bias,
                   const float* residual, float* y, int precision, cudaStream_t stream) {
    if (reinterpret_cast<uintptr_t>(x) % 16 != 0 || reinterpret_cast<uintptr_t>(w) % 16 != 0 || stride % 16 != 0)
        return CL_ERR_INVALID;
    return precision == CL_GEMM_F16 ? launch_tc_mode<false>(type, w, stride, n, k, x, m, bias, residual, y, stream)
                                    : launch_tc_mode<true>(type, w, stride, n, k, x, m, bias, residual, y, stream);
}

}  // namespace cl

extern "C" CL_API int cl_gemm_tc(int type, const void* w, long long stride, int n, int k, const float* x, int m,
                                 const float* bias, const float* residual, float* y, int precision,
                                 cudaStream_t stream) {
    if (w == nullptr || x == nullptr || y == nullptr || n <= 0 || k <= 0 || m <= 0 ||
        cl_native_row_bytes(type, k) < 0 || stride < cl_row_stride(type, k))
        return CL_ERR_INVALID;
    // weight rows and activation rows are read with 16-byte vector loads
    if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x)) % 16 || stride % 16) return CL_ERR_INVALID;
    if (!cl::gemm_tc_supported(type, n, k, m, precision)) return CL_ERR_UNSUPPORTED;
    return cl::launch_gemm_tc(type, w, stride, n, k, x, m, bias, residual, y, precision, stream);
}
