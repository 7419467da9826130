// Decode GEMV over native GGML blocks: y[n] = W[n, k] . x (+ bias) (+ residual).
//
// Reference: metal_gevm_{q4_k,q6_k,q5_0,q8_0,q5_k}_f32 (metal_llm.metal:708-781)
// and the CPU oracle gevmt/gevmtb over GgufDequantizer rows
// (cpu_llm.cpp:512-547, model.cpp:581-683).  Same products, different order:
// the quantized integers are dotted with the XQ limbs of x by dp4a (exact)
// and the per-sub-block scales are applied in FP32 afterwards (the factored
// form d*sc*sum(x*q) - dmin*m*sum(x) that the Metal kernels also use,
// metal_llm.metal:392-393).
//
// Kernel shape (B200): persistent CTAs, one producer warp + NC consumer
// warps.  The producer streams tiles of RT consecutive weight rows (one
// contiguous byte range) into an NS-stage shared-memory ring with
// cp.async.bulk, completion tracked by mbarriers, so ~100-200 KB per SM is
// in flight without tying up registers.  Consumer thread t owns the 32-column
// "unit" t of x for the CTA's lifetime (its XQ limbs stay in registers), dots
// it with unit t of every staged row, and the per-row partials are reduced
// across the CTA.  Weights are immutable, so the producer starts streaming
// before the programmatic-dependent-launch wait; consumers wait before
// reading x.
//
// Device weight layout (cl_repack_rows): each row padded to a multiple of 16
// bytes; Q4_K and Q5_K keep their native blocks, Q6_K/Q8_0/Q5_0 rows are
// re-ordered structure-of-arrays inside the row so vector loads are aligned:
//   Q6_K row: [nb x (ql128 qh64 sc16)] [nb x f16 d]
//   Q8_0 row: [nb x qs32] [nb x f16 d]
//   Q5_0 row: [nb x qs16] [nb x u32 qh] [nb x f16 d]
#include "common.cuh"
#include "gemv_common.cuh"
#include "launch.cuh"

#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>
#include <utility>

namespace cl {

// Device-side error word: set when a bounded wait gives up (never expected).
__device__ int g_gemv_error = 0;

// ---- kernel -------------------------------------------------------------------
constexpr int kMaxSegs = 4;
constexpr int kMaxConsumerWarps = 23;  // k <= 23552
constexpr int kMaxThreads = (kMaxConsumerWarps + 1) * 32;
constexpr int kMaxGroups = 15;         // named barriers 1..15

struct GemvSeg {
    const uint8_t* w;
    const uint8_t* w_up;  // SwiGLU: up rows (same type/stride as w)
    long long stride;
    const float* bias;
    const float* residual;
    float* y;
    int type;
    int n;           // output rows
    int tile_begin;  // first tile index of this segment
};

struct GemvParams {
    GemvSeg seg[kMaxSegs];
    const float* x;
    const float* gamma;  // RMSNorm weight applied to x first (cpu_llm.cpp:143-166), or null
    float eps;
    int nseg;
    int k;
    int units;        // k / 32
    int tiles;        // total tiles (RPG rows each) over all segments
    int stages;       // ring depth per group
    int stage_bytes;  // bytes of one stage (RPG rows x stride x matrices)
    int groups;       // consumer groups; each holds all of x and runs its own ring
    int group_warps;  // warps per group (ceil(units / 32))
};

struct TileInfo {
    int seg, row0, rows;
};

CL_DEVINL TileInfo tile_info(const GemvParams& p, int t, int rt) {
    int s = 0;
#pragma unroll
    for (int i = 1; i < kMaxSegs; ++i)
        if (i < p.nseg && t >= p.seg[i].tile_begin) s = i;
    const int row0 = (t - p.seg[s].tile_begin) * rt;
    return TileInfo{s, row0, min(rt, p.seg[s].n - row0)};
}

// Dynamic shared memory:
//   [full|empty mbarriers: groups x stages x 2 x 8 B][abort flag 16 B]
//   [double norm partials: 32 x 8 B][float row partials: 32 warps x 2 x VPW]
//   [stages: groups x stages x stage_bytes, 128-byte aligned]
// tickets: groups x stages ints after the norm partials; partial sums:
// [group][stage][warp in group][VPW] floats.
__host__ __device__ inline int smem_ticket_offset(int groups, int stages) { return 16 * groups * stages + 16 + 32 * 8; }
__host__ __device__ inline int smem_red_offset(int groups, int stages) {
    return (smem_ticket_offset(groups, stages) + 4 * groups * stages + 15) & ~15;
}
__host__ __device__ inline int smem_xq_offset(int groups, int stages, int vpw, int gwarps) {
    return (smem_red_offset(groups, stages) + 4 * groups * stages * gwarps * vpw + 127) & ~127;
}
__host__ __device__ inline int xpub_bytes(int groups, int k) { return groups > 1 ? (k / 32) * 128 : 0; }
__host__ __device__ inline int smem_stage_offset(int groups, int stages, int vpw, int gwarps, int k) {
    return (smem_xq_offset(groups, stages, vpw, gwarps) + xpub_bytes(groups, k) + 127) & ~127;
}

// Group g of CTA c processes tiles c*G + g, c*G + g + gridDim.x*G, ...; a
// tile is RPG consecutive rows (and the same rows of `up` for SwiGLU).
__host__ __device__ constexpr int nb_of(int type, int units) {
    return (type == CL_TYPE_Q8_0 || type == CL_TYPE_Q5_0) ? units : units / 8;
}

// F2 != F: a fused pair of formats (chosen per tile), e.g. Q4_K q/k with
// Q6_K v in one launch.
template <int F, int RPG, bool SWIGLU, int F2 = F>
__global__ void __launch_bounds__(kMaxThreads) gemv_tma_kernel(const GemvParams p) {
    constexpr int NMAT = SWIGLU ? 2 : 1;
    constexpr int VPW = NMAT * RPG;  // partial sums per warp per tile
    extern __shared__ __align__(128) uint8_t smem[];
    const int G = p.groups, NS = p.stages;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);  // [G][NS][2]
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 16 * G * NS);
    double* dred = reinterpret_cast<double*>(smem + 16 * G * NS + 16);
    int* tickets = reinterpret_cast<int*>(smem + smem_ticket_offset(G, NS));
    float* red = reinterpret_cast<float*>(smem + smem_red_offset(G, NS));
    void* xq_smem = smem + smem_xq_offset(G, NS, VPW, p.group_warps);
    uint8_t* stage_base = smem + smem_stage_offset(G, NS, VPW, p.group_warps, p.k);

    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int gthreads = p.group_warps * 32;
    const int nconsumer = G * gthreads;
    const int tile_stride = gridDim.x * G;
    if (tid == 0) {
        // full: one producer arrival (+ tx bytes); empty: one per warp of the group
        for (int g = 0; g < G; ++g) {
            for (int s = 0; s < NS; ++s) {
                mbar_init(&bars[2 * g * NS + s], 1);
                mbar_init(&bars[2 * g * NS + NS + s], p.group_warps);
            }
        }
        for (int i = 0; i < G * NS; ++i) tickets[i] = 0;
        *abort_flag = 0;
        mbar_fence_init();
    }
    __syncthreads();
    grid_launch_dependents();

    if (tid >= nconsumer) {
        // ---- producer warp: lane g feeds group g (weights are immutable, so
        // streaming starts before the dependency wait) ----
        const int g = tid - nconsumer;
        if (g < G) {
            uint64_t* full = bars + 2 * g * NS;
            uint64_t* empty = full + NS;
            uint8_t* ring = stage_base + (size_t)g * NS * p.stage_bytes;
            int s = 0;
            uint32_t ph = 0;
            for (int t = blockIdx.x * G + g; t < p.tiles; t += tile_stride) {
                if (!mbar_wait(&empty[s], ph ^ 1u)) {
                    atomicExch(&g_gemv_error, 1);
                    *abort_flag = 1;
                    break;
                }
                const TileInfo ti = tile_info(p, t, RPG);
                const GemvSeg& sg = p.seg[ti.seg];
                const uint32_t bytes = (uint32_t)(ti.rows * sg.stride);
                uint8_t* dst = ring + (size_t)s * p.stage_bytes;
                mbar_arrive_expect_tx(&full[s], bytes * NMAT);
                bulk_g2s(dst, sg.w + (size_t)ti.row0 * sg.stride, bytes, &full[s]);
                if (SWIGLU)
                    bulk_g2s(dst + (size_t)RPG * sg.stride, sg.w_up + (size_t)ti.row0 * sg.stride, bytes, &full[s]);
                if (++s == NS) {
                    s = 0;
                    ph ^= 1u;
                }
            }
        }
        return;
    }

    // ---- consumers: group 0 turns x into XQ units (one 32-column unit per
    // thread, in registers) and, when there are more groups, publishes them
    // in shared memory for the others ----
    grid_wait();
    const int grp = tid / gthreads;
    const int gt = tid - grp * gthreads;  // thread within the group = unit index
    const int u = gt;
    const bool active = u < p.units;
    XUnit xu{};
    uint4* xpub = reinterpret_cast<uint4*>(xq_smem);  // [units][8] uint4
    if (grp == 0) {
        float v[32];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 f =
                active ? reinterpret_cast<const float4*>(p.x + 32 * u)[q] : make_float4(0.f, 0.f, 0.f, 0.f);
            v[4 * q] = f.x;
            v[4 * q + 1] = f.y;
            v[4 * q + 2] = f.z;
            v[4 * q + 3] = f.w;
        }
        if (p.gamma) {
            // cpu_llm.cpp:156-165: sum of squares in double, mean -> float,
            // inv = 1/sqrt(mean + eps) in float, x * (inv * gamma).  Every
            // CTA reduces in the same order, so all CTAs see the same inv.
            double ss = 0.0;
#pragma unroll
            for (int e = 0; e < 32; ++e) ss += (double)v[e] * (double)v[e];
            ss = warp_sum_d(ss);
            if (lane == 0) dred[warp] = ss;
            named_barrier(2, gthreads);  // group 0 only (barrier 1 is the all-consumer one)
            double tot = 0.0;
            for (int w = 0; w < p.group_warps; ++w) tot += dred[w];
            const float inv = 1.0f / sqrtf((float)(tot / (double)p.k) + p.eps);
            if (active) {
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    const float4 gm = reinterpret_cast<const float4*>(p.gamma + 32 * u)[q];
                    v[4 * q] = __fmul_rn(v[4 * q], __fmul_rn(inv, gm.x));
                    v[4 * q + 1] = __fmul_rn(v[4 * q + 1], __fmul_rn(inv, gm.y));
                    v[4 * q + 2] = __fmul_rn(v[4 * q + 2], __fmul_rn(inv, gm.z));
                    v[4 * q + 3] = __fmul_rn(v[4 * q + 3], __fmul_rn(inv, gm.w));
                }
            }
        }
        encode_unit(v, xu);
        if (G > 1 && active) {
            uint4* o = xpub + 8 * u;
            o[0] = make_uint4(xu.l[0][0].x, xu.l[0][0].y, xu.l[0][0].z, xu.l[0][0].w);
            o[1] = make_uint4(xu.l[0][1].x, xu.l[0][1].y, xu.l[0][1].z, xu.l[0][1].w);
            o[2] = make_uint4(xu.l[0][2].x, xu.l[0][2].y, xu.l[0][2].z, xu.l[0][2].w);
            o[3] = make_uint4(xu.l[1][0].x, xu.l[1][0].y, xu.l[1][0].z, xu.l[1][0].w);
            o[4] = make_uint4(xu.l[1][1].x, xu.l[1][1].y, xu.l[1][1].z, xu.l[1][1].w);
            o[5] = make_uint4(xu.l[1][2].x, xu.l[1][2].y, xu.l[1][2].z, xu.l[1][2].w);
            o[6] = make_uint4(xu.s[0].x, xu.s[0].y, xu.s[1].x, xu.s[1].y);
            o[7] = make_uint4(__float_as_uint(xu.xs), __float_as_uint(xu.xsum), 0u, 0u);
        }
    }
    if (G > 1) {
        named_barrier(1, nconsumer);
        if (grp > 0 && active) {
            const uint4* o = xpub + 8 * u;
            uint4 t;
            t = o[0]; xu.l[0][0] = make_int4(t.x, t.y, t.z, t.w);
            t = o[1]; xu.l[0][1] = make_int4(t.x, t.y, t.z, t.w);
            t = o[2]; xu.l[0][2] = make_int4(t.x, t.y, t.z, t.w);
            t = o[3]; xu.l[1][0] = make_int4(t.x, t.y, t.z, t.w);
            t = o[4]; xu.l[1][1] = make_int4(t.x, t.y, t.z, t.w);
            t = o[5]; xu.l[1][2] = make_int4(t.x, t.y, t.z, t.w);
            t = o[6]; xu.s[0] = make_int2(t.x, t.y); xu.s[1] = make_int2(t.z, t.w);
            t = o[7]; xu.xs = __uint_as_float(t.x); xu.xsum = __uint_as_float(t.y);
        }
    }
    uint64_t* full = bars + 2 * grp * NS;
    uint64_t* empty = full + NS;
    const uint8_t* ring = stage_base + (size_t)grp * NS * p.stage_bytes;
    int s = 0, it = 0;
    uint32_t ph = 0;
    for (int t = blockIdx.x * G + grp; t < p.tiles; t += tile_stride, ++it) {
        const TileInfo ti = tile_info(p, t, RPG);
        const GemvSeg& sg = p.seg[ti.seg];
        const bool ok = mbar_wait(&full[s], ph);
        if (!ok) {
            atomicExch(&g_gemv_error, 2);
            *abort_flag = 1;
        }
        const uint8_t* st = ring + (size_t)s * p.stage_bytes;
        float acc[VPW];
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
#pragma unroll
            for (int j = 0; j < RPG; ++j) {
                float a = 0.0f;
                if (ok && active && j < ti.rows)
                {
                    const uint8_t* rw = st + (size_t)(m * RPG + j) * sg.stride;
                    a = (F == F2 || sg.type == F) ? Fmt<F>::template dot<SmemLd>(rw, u, nb_of(F, p.units), xu)
                                                  : Fmt<F2>::template dot<SmemLd>(rw, u, nb_of(F2, p.units), xu);
                }
                acc[m * RPG + j] = a;
            }
        }
        // publish this warp's partials; the last warp of the group to finish
        // the tile reduces them and writes the outputs (no group barrier)
        const int gw = warp - grp * p.group_warps;
        float* rb = red + ((size_t)(grp * NS + s) * p.group_warps) * VPW;
        {
            const float w = warp_sum_many<VPW>(acc, lane);
            if ((lane & (32 / VPW - 1)) == 0) rb[gw * VPW + red_index<VPW>(lane)] = w;
        }
        __syncwarp();
        int last = 0;
        if (lane == 0) {
            __threadfence_block();
            last = atomicAdd(&tickets[grp * NS + s], 1) == p.group_warps - 1;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence_block();
            if (lane < ti.rows && !*abort_flag) {
                float y = 0.0f, up = 0.0f;
                for (int w = 0; w < p.group_warps; ++w) {
                    y += rb[w * VPW + lane];
                    if (SWIGLU) up += rb[w * VPW + RPG + lane];
                }
                const int o = ti.row0 + lane;
                if (SWIGLU) {
                    // Branch-stable SiLU(g) * u (cpu_llm.cpp:188-202).
                    const float sig = y >= 0.0f ? 1.0f / (1.0f + expf(-y)) : expf(y) / (1.0f + expf(y));
                    y = __fmul_rn(__fmul_rn(y, sig), up);
                } else {
                    if (sg.bias) y += sg.bias[o];
                    if (sg.residual) y = sg.residual[o] + y;
                }
                sg.y[o] = y;
            }
            if (lane == 0) tickets[grp * NS + s] = 0;
            __syncwarp();
        }
        if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with stage s
        if (*abort_flag) break;
        if (++s == NS) {
            s = 0;
            ph ^= 1u;
        }
    }
}

// ---- host launcher -----------------------------------------------------------
bool gemv_type_ok(int t) {
    return t == CL_TYPE_Q4_K || t == CL_TYPE_Q5_K || t == CL_TYPE_Q6_K || t == CL_TYPE_Q8_0 || t == CL_TYPE_Q5_0;
}

constexpr int kSmemBudget = 190 * 1024;
constexpr int kTargetWarps = 16;  // consumer warps per CTA to aim for

template <int F, int RPG, bool SW, int F2 = F>
cudaError_t launch_cfg(const GemvParams& p, cudaStream_t stream) {
    constexpr int NMAT = SW ? 2 : 1;
    auto kern = gemv_tma_kernel<F, RPG, SW, F2>;
    const int threads = p.groups * p.group_warps * 32 + 32;
    const int smem = smem_stage_offset(p.groups, p.stages, NMAT * RPG, p.group_warps, p.k) +
                     p.groups * p.stages * p.stage_bytes;
    static SmemLimit limit;
    static std::mutex mu;
    static std::map<std::tuple<int, int, int>, int> occ_cache;  // (device, threads, smem) -> CTAs per SM
    cudaError_t e = limit.ensure(kern, 227 * 1024);
    if (e != cudaSuccess) return e;
    int sm_count = 0, dev = 0;
    if ((e = device_sm_count(&sm_count)) != cudaSuccess || (e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    int occ = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = occ_cache.find({dev, threads, smem});
        if (it == occ_cache.end()) {
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, smem);
            if (e != cudaSuccess) return e;
            occ_cache[{dev, threads, smem}] = occ;
        } else {
            occ = it->second;
        }
    }
    if (occ < 1) return cudaErrorInvalidConfiguration;
    const int grid = std::min((p.tiles + p.groups - 1) / p.groups, occ * sm_count);
    return launch_pdl(kern, dim3(grid), dim3(threads), smem, stream, p);
}

template <int F, bool SW, int F2 = F>
cudaError_t launch_fmt(const GemvParams& p, int rpg, cudaStream_t stream) {
    switch (rpg) {
    case 1: return launch_cfg<F, 1, SW, F2>(p, stream);
    case 2: return launch_cfg<F, 2, SW, F2>(p, stream);
    default: return launch_cfg<F, 4, SW, F2>(p, stream);
    }
}

// Format pairs with a fused instance (the Q4_K_M attention projections: Q4_K
// q/k with Q6_K v; small models' Q5_0 with Q8_0).
bool pair_supported(int a, int b) {
    return (a == CL_TYPE_Q4_K && b == CL_TYPE_Q6_K) || (a == CL_TYPE_Q5_0 && b == CL_TYPE_Q8_0);
}

cudaError_t launch_pair(int a, int b, const GemvParams& p, int rpg, cudaStream_t stream) {
    if (a == CL_TYPE_Q4_K && b == CL_TYPE_Q6_K) return launch_fmt<CL_TYPE_Q4_K, false, CL_TYPE_Q6_K>(p, rpg, stream);
    if (a == CL_TYPE_Q5_0 && b == CL_TYPE_Q8_0) return launch_fmt<CL_TYPE_Q5_0, false, CL_TYPE_Q8_0>(p, rpg, stream);
    return cudaErrorInvalidValue;
}

template <bool SW>
cudaError_t launch_type(int type, const GemvParams& p, int rpg, cudaStream_t stream) {
    switch (type) {
    case CL_TYPE_Q4_K: return launch_fmt<CL_TYPE_Q4_K, SW>(p, rpg, stream);
    case CL_TYPE_Q5_K: return launch_fmt<CL_TYPE_Q5_K, SW>(p, rpg, stream);
    case CL_TYPE_Q6_K: return launch_fmt<CL_TYPE_Q6_K, SW>(p, rpg, stream);
    case CL_TYPE_Q8_0: return launch_fmt<CL_TYPE_Q8_0, SW>(p, rpg, stream);
    case CL_TYPE_Q5_0: return launch_fmt<CL_TYPE_Q5_0, SW>(p, rpg, stream);
    default: return cudaErrorInvalidValue;
    }
}

// One launch over segments that share a type.
int launch_gemv_mma(const cl_gemv_segment* segs, int nseg, int k, const float* x, const float* gamma, float eps,
                    const void* w_up, cudaStream_t stream);  // gemv_mma.cu
int gemv_mma_device_error(int* code, bool clear);            // gemv_mma.cu

int launch_same_type(const cl_gemv_segment* segs, int nseg, int k, const float* x, const float* gamma, float eps,
                     const void* w_up, cudaStream_t stream) {
    // Q4_K / Q6_K segments (one type, or the Q4_K + Q6_K pair) go to the
    // tensor-core GEMV (gemv_mma.cu) when it takes the shape; the other types
    // and shapes run here.
    {
        const int rc = launch_gemv_mma(segs, nseg, k, x, gamma, eps, w_up, stream);
        if (rc != CL_ERR_UNSUPPORTED) return rc;
    }
    if (k / 32 > kMaxConsumerWarps * 32) return CL_ERR_UNSUPPORTED;
    const bool sw = w_up != nullptr;
    const int nmat = sw ? 2 : 1;
    GemvParams p{};
    p.units = k / 32;
    p.group_warps = (p.units + 31) / 32;
    long long smax = 0;
    for (int i = 0; i < nseg; ++i) smax = std::max(smax, segs[i].stride);
    // Measured on B200: the kernel is bound by per-tile consumer latency, so
    // prefer 4-row tiles and ~16 consumer warps; 2-4 stages per group suffice.
    int groups = std::max(1, std::min(kMaxGroups, kTargetWarps / p.group_warps));
    while (groups > 1 && groups * p.group_warps > kMaxConsumerWarps) --groups;
    const int budget = kSmemBudget - xpub_bytes(groups, k);
    int rpg = 4;
    while (rpg > 1 && (long long)rpg * smax * nmat > 40 * 1024) rpg /= 2;
    while (groups > 1 && (long long)groups * 2 * rpg * smax * nmat > budget) --groups;
    if ((long long)groups * 2 * rpg * smax * nmat > budget) return CL_ERR_UNSUPPORTED;
    p.groups = groups;
    p.stage_bytes = (int)((long long)rpg * smax * nmat);
    p.stages = std::max(2, std::min(4, budget / (groups * p.stage_bytes)));
    const int rt = rpg;
    int tiles = 0;
    for (int i = 0; i < nseg; ++i) {
        GemvSeg& g = p.seg[i];
        g.w = static_cast<const uint8_t*>(segs[i].w);
        g.w_up = static_cast<const uint8_t*>(w_up);
        g.stride = segs[i].stride;
        g.bias = segs[i].bias;
        g.residual = segs[i].residual;
        g.y = segs[i].y;
        g.type = segs[i].type;
        g.n = segs[i].n;
        g.tile_begin = tiles;
        tiles += (segs[i].n + rt - 1) / rt;
    }
    p.x = x;
    p.gamma = gamma;
    p.eps = eps;
    p.nseg = nseg;
    p.k = k;
    p.tiles = tiles;
    int ta = segs[0].type, tb = segs[0].type;
    for (int i = 1; i < nseg; ++i)
        if (segs[i].type != ta) tb = segs[i].type;
    if (ta > tb) std::swap(ta, tb);
    const cudaError_t e = sw ? launch_type<true>(segs[0].type, p, rpg, stream)
                             : (ta == tb ? launch_type<false>(ta, p, rpg, stream) : launch_pair(ta, tb, p, rpg, stream));
    return e == cudaSuccess ? CL_OK : CL_ERR_CUDA;
}

int launch_gemv(const cl_gemv_segment* segs, int nseg, int k, const float* x, const float* gamma, float eps,
                const void* w_up, cudaStream_t stream) {
    const bool sw = w_up != nullptr;
    if (nseg < 1 || nseg > kMaxSegs || (sw && nseg != 1) || k <= 0 || k % 32 != 0 || x == nullptr ||
        reinterpret_cast<uintptr_t>(x) % 16 != 0 ||
        (gamma && (reinterpret_cast<uintptr_t>(gamma) % 16 != 0 || !(eps > 0.0f))))
        return CL_ERR_INVALID;
    for (int i = 0; i < nseg; ++i) {
        const cl_gemv_segment& s = segs[i];
        if (!gemv_type_ok(s.type) || s.w == nullptr || s.y == nullptr || s.n <= 0) return CL_ERR_INVALID;
        if (cl_native_row_bytes(s.type, k) < 0) return CL_ERR_INVALID;
        if (s.stride < cl_row_stride(s.type, k) || s.stride % 16 != 0 || reinterpret_cast<uintptr_t>(s.w) % 16 != 0)
            return CL_ERR_INVALID;
    }
    if (sw && reinterpret_cast<uintptr_t>(w_up) % 16 != 0) return CL_ERR_INVALID;
    // Consecutive segments of one type, or of a fused pair of types, share a launch.
    for (int i = 0; i < nseg;) {
        int j = i + 1, other = -1;
        while (j < nseg) {
            const int t = segs[j].type;
            if (t == segs[i].type || t == other) {
                ++j;
                continue;
            }
            if (other < 0 && !sw && pair_supported(std::min(t, segs[i].type), std::max(t, segs[i].type))) {
                other = t;
                ++j;
                continue;
            }
            break;
        }
        const int rc = launch_same_type(segs + i, j - i, k, x, gamma, eps, w_up, stream);
        if (rc != CL_OK) return rc;
        i = j;
    }
    return CL_OK;
}

}  // namespace cl

namespace cl {
int gemm_tc_device_error(int* code, bool clear);  // gemm_tc.cu
int gemm16_device_error(int* code, bool clear);   // gemm16.cu
}  // namespace cl

extern "C" {

CL_API int cl_gemv(int type, const void* w, long long stride, int n, int k, const float* x, const float* bias,
                   const float* residual, float* y, cudaStream_t stream) {
    cl_gemv_segment s{type, w, stride, n, bias, residual, y};
    return cl::launch_gemv(&s, 1, k, x, nullptr, 0.0f, nullptr, stream);
}

CL_API int cl_gemv_multi(const cl_gemv_segment* segs, int nseg, int k, const float* x, const float* norm_gamma,
                         float eps, cudaStream_t stream) {
    if (segs == nullptr) return CL_ERR_INVALID;
    return cl::launch_gemv(segs, nseg, k, x, norm_gamma, eps, nullptr, stream);
}

CL_API int cl_gemv_swiglu(int type, const void* w_gate, const void* w_up, long long stride, int n, int k,
                          const float* x, const float* norm_gamma, float eps, float* y, cudaStream_t stream) {
    if (w_up == nullptr) return CL_ERR_INVALID;
    cl_gemv_segment s{type, w_gate, stride, n, nullptr, nullptr, y};
    return cl::launch_gemv(&s, 1, k, x, norm_gamma, eps, w_up, stream);
}

CL_API int cl_device_error(int* code, int clear) {
    if (code == nullptr) return CL_ERR_INVALID;
    int gemv = 0, gemm = 0, mma = 0, g16 = 0;
    if (cudaMemcpyFromSymbol(&gemv, cl::g_gemv_error, sizeof(int)) != cudaSuccess) return CL_ERR_CUDA;
    if (cl::gemv_mma_device_error(&mma, clear != 0) != CL_OK) return CL_ERR_CUDA;
    if (cl::gemm_tc_device_error(&gemm, clear != 0) != CL_OK) return CL_ERR_CUDA;
    if (cl::gemm16_device_error(&g16, clear != 0) != CL_OK) return CL_ERR_CUDA;
    // GEMV codes are 1-5 (4-5: tensor-core GEMV); tensor-core GEMM codes are
    // reported as 16 + code, the 16-bit GEMM's as 32 + code.
    *code = gemv != 0 ? gemv : (mma != 0 ? mma : (gemm != 0 ? 16 + gemm : (g16 != 0 ? 32 + g16 : 0)));
    if (clear) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(cl::g_gemv_error, &zero, sizeof(int)) != cudaSuccess) return CL_ERR_CUDA;
    }
    return CL_OK;
}

}  // extern "C"
