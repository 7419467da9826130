// GQA attention over the FP32 KV cache.
//
// Decode: flash-decoding.  CTA (kv head, key split) scores the group's query
// heads against its share of the live keys, keeps an unnormalised softmax
// partial (max, sum, sum p*V) in the workspace; a combine kernel (CTA per
// query head) merges the splits, normalises and emits the head outputs (and
// optionally their XQ encoding).  Reference: metal_kv_cache_qk/softmax/av (metal_llm.metal:
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

constexpr int kDecThreads = 256;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kMaxGroup = 16;
constexpr int kMaxHeadDim = 256;
constexpr int kTileKeys = 64;         // keys staged per tile
constexpr int kMaxSplits = 32;        // key splits per KV head

// Splits for a KV capacity: 32 (to cover the GPU) unless fewer than 16 keys
// each would remain.  The keys of a split are walked in 64-key tiles.
__host__ __device__ inline int attn_splits(int max_len) {
    return max(1, min(kMaxSplits, (max_len + 15) / 16));
}

CL_DEVINL void cp_async16(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
CL_DEVINL void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
CL_DEVINL void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Butterfly sum of 8 values per lane: afterwards lane l holds the full sum
// of value (l >> 2) & 7.
CL_DEVINL float warp_sum8(float (&v)[8], int lane) {
#pragma unroll
    for (int step = 0, n = 8, bit = 16; step < 3; ++step, n >>= 1, bit >>= 1) {
        const bool upper = (lane & bit) != 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            if (j < n / 2) {
                const float keep = upper ? v[j + n / 2] : v[j];
                const float send = upper ? v[j] : v[j + n / 2];
                v[j] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
            }
        }
    }
    float r = v[0];
    r += __shfl_xor_sync(0xffffffffu, r, 2);
    r += __shfl_xor_sync(0xffffffffu, r, 1);
    return r;
}

// Dynamic smem: q [G][d + 4] | K tile [64][d + 4] | V tile [64][d] | p [G][64] |
//               PV partials [parts - 1][G][d] | running (m, l) [G][2] | rescale [G]
__host__ __device__ inline size_t attn_decode_smem(int group, int d) {
    const int parts = max(1, kDecThreads / d);
    return sizeof(float) * ((size_t)group * (d + 4) + (size_t)kTileKeys * (d + 4) + (size_t)kTileKeys * d +
                            (size_t)group * kTileKeys + (size_t)(parts - 1) * group * d + 3 * group);
}

// One CTA per (KV head, key split).  The split length comes from the live
// length (*len_dev), so a graph captured once spreads every step's keys over
// all CTAs.  K and V tiles are staged with asynchronous copies (a tile's
// loads all in flight at once; K rows padded by 16 bytes so that threads on
// different keys hit different banks).  Scores: one thread per (key, head)
// dot product; the per-head softmax statistics by one warp per head; an
// online softmax carries (m, l, o) across tiles.  Each CTA leaves an
// unnormalised partial [m, l, o[d]] per query head in the workspace.
// Optional fused RoPE + KV append (Rope.cs != null): q holds the unrotated
// query; the CTA rotates its heads in shared memory.  The key and value of
// the current position (Rope.pos_dev; live length = pos + 1) come from
// Rope.k / Rope.v: the CTA whose keys include that position rotates the key,
// writes both rows to the caches and uses them in place of the tile rows it
// loaded.  Same expressions as rope_kv_kernel, so the results are identical
// to RoPE + KV append + attention as separate launches.
struct AttnRope {
    const float* cs;  // [capacity][rot/2][cos, sin], or null
    const float* k;   // [kv_heads * d] new key (unrotated)
    const float* v;   // [kv_heads * d] new value
    const int* pos_dev;
    float* kc;        // caches, written at row pos
    float* vc;
    int rot;
};

__global__ void __launch_bounds__(kDecThreads)
attn_decode_split(const float* q, const float* kc, const float* vc,
                  const int* len_dev, int cap, int hq, int hkv, int d, float scale,
                  float* part, const AttnRope rope) {
    grid_launch_dependents();
    grid_wait();
    const int g = blockIdx.x, split = blockIdx.y, nsplit = gridDim.y;
    const int G = hq / hkv;
    // The live length comes from device memory: clamp it to the cache
    // capacity so that a bad value can never read (or, with the fused
    // append, write) outside the caches; a position beyond them is skipped.
    const int pos_raw = rope.cs ? *rope.pos_dev : -1;
    const int pos = pos_raw < cap ? pos_raw : -1;
    const int L = max(0, min(cap, rope.cs ? pos_raw + 1 : *len_dev));
    const int S = (L + nsplit - 1) / nsplit;
    const int k0 = split * S;
    const int nk_all = max(0, min(S, L - k0));
    const int rec = d + 2, kvd = hkv * d, d4 = d / 4, kld = d + 4;
    const int tid = threadIdx.x;
    extern __shared__ __align__(16) float sm[];
    const int parts = max(1, kDecThreads / d);
    float* qs = sm;                        // [G][d + 4]: rows padded like K (query heads on
                                           // different banks in the score loop)
    float* ks = qs + G * kld;              // [64][d + 4]
    float* vs = ks + kTileKeys * kld;      // [64][d]
    float* ps = vs + kTileKeys * d;        // [G][64]
    float* pv = ps + G * kTileKeys;        // [parts - 1][G][d]
    float* run = pv + (parts - 1) * G * d; // [G][2] running max / sum
    float* fac = run + 2 * G;              // [G] rescale of the running (l, o)

    const int dim = tid % d, pt = tid / d;
    const bool active = pt < parts;  // d not dividing the CTA leaves a few threads idle
    float acc[kMaxGroup];
#pragma unroll
    for (int h = 0; h < kMaxGroup; ++h) acc[h] = 0.0f;
    if (tid < G) {
        run[2 * tid] = -INFINITY;
        run[2 * tid + 1] = 0.0f;
    }
    for (int i = tid; i < G * d4; i += kDecThreads) {
        const int h = i / d4, c = i - h * d4;
        cp_async16(qs + h * kld + 4 * c, q + (size_t)g * G * d + 4 * i);
    }
    cp_async_commit();
    for (int t0 = 0; t0 < nk_all; t0 += kTileKeys) {
        const int nk = min(kTileKeys, nk_all - t0);
        const size_t base = (size_t)(k0 + t0) * kvd + (size_t)g * d;
        for (int i = tid; i < nk * d4; i += kDecThreads) {
            const int t = i / d4, c = i - t * d4;
            cp_async16(ks + t * kld + 4 * c, kc + base + (size_t)t * kvd + 4 * c);
        }
        cp_async_commit();
        for (int i = tid; i < nk * d4; i += kDecThreads) {
            const int t = i / d4, c = i - t * d4;
            cp_async16(vs + t * d + 4 * c, vc + base + (size_t)t * kvd + 4 * c);
        }
        cp_async_commit();
        cp_async_wait<1>();  // q and K
        __syncthreads();
        if (rope.cs) {
            const int half = rope.rot / 2;
            const float* csp = rope.cs + (size_t)max(pos_raw < cap ? pos_raw : 0, 0) * half * 2;
            if (t0 == 0 && pos_raw >= 0 && pos_raw < cap) {
                // rotate this CTA's query heads (NeoX split halves)
                for (int i = tid; i < G * half; i += kDecThreads) {
                    const int h = i / half, pp = i - h * half;
                    float* qh = qs + h * kld;
                    const float c = csp[2 * pp], sn = csp[2 * pp + 1];
                    const float a = qh[pp], b = qh[pp + half];
                    qh[pp] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
                    qh[pp + half] = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, c));
                }
            }
            const int r = pos - (k0 + t0);
            if (pos >= 0 && r >= 0 && r < nk) {
                // the current position's key: rotate, cache it, use it in the tile
                const float* kn = rope.k + (size_t)g * d;
                float* kw = rope.kc + (size_t)pos * kvd + (size_t)g * d;
                for (int pp = tid; pp < d / 2; pp += kDecThreads) {
                    int i0, i1;
                    if (pp < half) {
                        i0 = pp;
                        i1 = pp + half;
                    } else {
                        i0 = rope.rot + 2 * (pp - half);
                        i1 = i0 + 1;
                    }
                    float a = kn[i0], b = kn[i1];
                    if (pp < half) {
                        const float c = csp[2 * pp], sn = csp[2 * pp + 1];
                        const float ra = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
                        const float rb = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, c));
                        a = ra;
                        b = rb;
                    }
                    kw[i0] = a;
                    kw[i1] = b;
                    ks[r * kld + i0] = a;
                    ks[r * kld + i1] = b;
                }
            }
            __syncthreads();
        }
        // scores: thread per (key, head)
        for (int pidx = tid; pidx < nk * G; pidx += kDecThreads) {
            const int t = pidx / G, h = pidx - t * G;
            const float4* kr = reinterpret_cast<const float4*>(ks + t * kld);
            const float4* qr = reinterpret_cast<const float4*>(qs + h * kld);
            float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll 8
            for (int c = 0; c < d4; ++c) {
                const float4 kv = kr[c], qv = qr[c];
                a0 += kv.x * qv.x;
                a1 += kv.y * qv.y;
                a2 += kv.z * qv.z;
                a3 += kv.w * qv.w;
            }
            ps[h * kTileKeys + t] = ((a0 + a1) + (a2 + a3)) * scale;
        }
        __syncthreads();
        // online softmax statistics: one warp per head, lanes over the keys
        {
            const int warp = tid >> 5, lane = tid & 31;
            for (int h = warp; h < G; h += kDecWarps) {
                float* ph = ps + h * kTileKeys;
                const float s0 = lane < nk ? ph[lane] : -INFINITY;
                const float s1 = lane + 32 < nk ? ph[lane + 32] : -INFINITY;
                const float mo = run[2 * h], mn = fmaxf(mo, warp_max(fmaxf(s0, s1)));
                const float e0 = lane < nk ? expf(s0 - mn) : 0.0f;
                const float e1 = lane + 32 < nk ? expf(s1 - mn) : 0.0f;
                if (lane < nk) ph[lane] = e0;
                if (lane + 32 < nk) ph[lane + 32] = e1;
                const float l = warp_sum(e0 + e1);
                if (lane == 0) {
                    const float f = mo == -INFINITY ? 0.0f : expf(mo - mn);
                    fac[h] = f;
                    run[2 * h] = mn;
                    run[2 * h + 1] = run[2 * h + 1] * f + l;
                }
            }
        }
        cp_async_wait<0>();  // V
        if (rope.cs) {
            const int r = pos - (k0 + t0);
            if (pos >= 0 && r >= 0 && r < nk) {
                const float* vn = rope.v + (size_t)g * d;
                float* vw = rope.vc + (size_t)pos * kvd + (size_t)g * d;
                for (int c = tid; c < d; c += kDecThreads) {
                    vw[c] = vn[c];
                    vs[r * d + c] = vn[c];
                }
            }
        }
        __syncthreads();
        if (active) {
#pragma unroll
            for (int h = 0; h < kMaxGroup; ++h)
                if (h < G) acc[h] *= fac[h];
            for (int t = pt; t < nk; t += parts) {
                const float vv = vs[t * d + dim];
#pragma unroll
                for (int h = 0; h < kMaxGroup; ++h)
                    if (h < G) acc[h] += ps[h * kTileKeys + t] * vv;
            }
        }
        __syncthreads();  // the tile buffers are refilled next
    }
    cp_async_wait<0>();
    __syncthreads();
    // this split's partials: [m, l, o[d]] per head (m = -inf, l = 0, o = 0 when empty)
    if (active && pt > 0) {
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h)
            if (h < G) pv[((pt - 1) * G + h) * d + dim] = acc[h];
    }
    __syncthreads();
    if (active && pt == 0) {
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) {
            if (h < G) {
                float o = acc[h];
                for (int r = 1; r < parts; ++r) o += pv[((r - 1) * G + h) * d + dim];
                float* pr = part + ((size_t)(g * G + h) * nsplit + split) * rec;
                pr[2 + dim] = o;
                if (dim == 0) {
                    pr[0] = run[2 * h];
                    pr[1] = run[2 * h + 1];
                }
            }
        }
    }
}

// Merge the splits of one query head: CTA per head, thread per dimension.
// The split weights exp(m_s - m) / l come from one warp; the partial loads
// are independent and unrolled, so they are all in flight together.
__global__ void __launch_bounds__(kMaxHeadDim)
attn_decode_combine(const float* part, int nsplit, int d, float* out, void* xq,
                    int xq_k) {
    grid_launch_dependents();
    grid_wait();
    __shared__ float wsm[kMaxSplits];
    const int h = blockIdx.x, tid = threadIdx.x, rec = d + 2;
    const float* pr = part + (size_t)h * nsplit * rec;
    if (tid < 32) {
        const float ms = tid < nsplit ? pr[(size_t)tid * rec] : -INFINITY;
        const float ls = tid < nsplit ? pr[(size_t)tid * rec + 1] : 0.0f;
        const float m = warp_max(ms);
        const float e = ls > 0.0f ? expf(ms - m) : 0.0f;
        const float l = warp_sum(ls * e);
        wsm[tid] = e / l;
    }
    __syncthreads();
    float o4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int s2 = 0; s2 < kMaxSplits; ++s2)
        if (s2 < nsplit) o4[s2 & 3] += pr[(size_t)s2 * rec + 2 + tid] * wsm[s2];
    const float o = (o4[0] + o4[1]) + (o4[2] + o4[3]);
    out[(size_t)h * d + tid] = o;
    if (xq) xq_store_block_warp(xq_mut(xq, xq_k), (h * d + tid) / 32, o);
}

// ---- prefill -------------------------------------------------------------------
constexpr int kQT = 32;   // query rows per CTA
constexpr int kKT = 32;   // keys per tile
constexpr int kPreThreads = 256;

__global__ void __launch_bounds__(kPreThreads)
attn_prefill_kernel(const float* q, const float* kc, const float* vc,
                    int pos0, int rows, int hq, int hkv, int d, float* out) {
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

static int attn_decode_launch(const float* q, const float* k_cache, const float* v_cache, const int* len_dev,
                              int max_len, int q_heads, int kv_heads, int head_dim, float scale, float* out, void* xq,
                              void* workspace, size_t workspace_bytes, const AttnRope& rope, cudaStream_t stream) {
    if (q == nullptr || k_cache == nullptr || v_cache == nullptr || (len_dev == nullptr && !rope.cs) || out == nullptr ||
        max_len <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads || q_heads / kv_heads > kMaxGroup ||
        head_dim <= 0 || head_dim % 32 || head_dim > kMaxHeadDim)
        return CL_ERR_INVALID;
    // q and the K / V rows are staged with 16-byte cp.async copies, and xq is
    // a set of 16-byte-aligned planes: other alignments would fault
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
         reinterpret_cast<uintptr_t>(xq)) & 15u)
        return CL_ERR_INVALID;
    if (workspace == nullptr || workspace_bytes < cl_attn_decode_workspace_bytes(q_heads, head_dim, max_len))
        return CL_ERR_WORKSPACE;
    const int splits = attn_splits(max_len);
    float* part = static_cast<float*>(workspace);
    const size_t smem = attn_decode_smem(q_heads / kv_heads, head_dim);
    static SmemLimit limit;
    if (smem > 48 * 1024 && limit.ensure(attn_decode_split, (int)smem) != cudaSuccess) return CL_ERR_CUDA;
    if (launch_pdl(attn_decode_split, dim3(kv_heads, splits), dim3(kDecThreads), smem, stream, q, k_cache, v_cache,
                   len_dev, max_len, q_heads, kv_heads, head_dim, scale, part, rope) != cudaSuccess)
        return CL_ERR_CUDA;
    return launch_pdl(attn_decode_combine, dim3(q_heads), dim3(head_dim), 0, stream, part, splits, head_dim, out, xq,
                      q_heads * head_dim) == cudaSuccess
               ? CL_OK
               : CL_ERR_CUDA;
}

CL_API int cl_attn_decode(const float* q, const float* k_cache, const float* v_cache, const int* len_dev,
                          int max_len, int q_heads, int kv_heads, int head_dim, float scale, float* out, void* xq,
                          void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    const AttnRope none{};
    return attn_decode_launch(q, k_cache, v_cache, len_dev, max_len, q_heads, kv_heads, head_dim, scale, out, xq,
                              workspace, workspace_bytes, none, stream);
}

CL_API int cl_attn_decode_rope(const float* q, const float* k_new, const float* v_new, const float* cos_sin,
                               const int* pos_dev, int rot_dim, float* k_cache, float* v_cache, int max_len,
                               int q_heads, int kv_heads, int head_dim, float scale, float* out, void* xq,
                               void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (k_new == nullptr || v_new == nullptr || cos_sin == nullptr || pos_dev == nullptr || rot_dim <= 0 ||
        rot_dim > head_dim || rot_dim % 2)
        return CL_ERR_INVALID;
    const AttnRope rope{cos_sin, k_new, v_new, pos_dev, k_cache, v_cache, rot_dim};
    return attn_decode_launch(q, k_cache, v_cache, nullptr, max_len, q_heads, kv_heads, head_dim, scale, out, xq,
                              workspace, workspace_bytes, rope, stream);
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
    static SmemLimit limit;
    if (limit.ensure(attn_prefill_kernel, (int)smem) != cudaSuccess) return CL_ERR_CUDA;
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
