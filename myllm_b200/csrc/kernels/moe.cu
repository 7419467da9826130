// qwen35moe kernels: router, routed experts, DeltaNet, gated attention.
//
// Reference formulas (moe_llm.mm / metal_llm.metal):
//   * router: FP32 product, softmax, top-k by strict '>' (lower id first on
//     ties), renormalisation (moe_llm.mm:2642-2690; metal_llm.metal:826-890,
//     1424-1474);
//   * routed experts: per route the expert's gate/up/down products, SwiGLU,
//     then the weighted reduce plus the sigmoid-gated shared expert
//     (moe_llm.mm:2692-2843; metal_llm.metal:1476-1542);
//   * Gated DeltaNet: causal depthwise conv over [history, qkv] + SiLU,
//     per-head L2 norm, decay = exp(softplus(alpha + dt_bias) * a),
//     beta = sigmoid, the delta-rule recurrence, per-head RMSNorm and the
//     silu(z) gate (moe_llm.mm:2436-2640; metal_llm.metal:1186-1420);
//   * gated attention: [query, gate] split per head, per-head RMSNorm of q
//     and k, partial NeoX RoPE, KV append (moe_llm.mm:2238-2434;
//     metal_llm.metal:785-823, 928-990, 1164-1183).
// Decode runs with everything on the device: expert ids never leave the GPU
// (the reference reads them back each layer, moe_llm.mm:2918-2930).
#include "common.cuh"
#include "gemv_common.cuh"
#include "launch.cuh"

#include <cooperative_groups.h>

namespace cl {
namespace moe {

CL_DEVINL float sigmoid_stable(float v) {
    return v >= 0.0f ? 1.0f / (1.0f + expf(-v)) : expf(v) / (1.0f + expf(v));
}

// Block-wide sum (blockDim.x a multiple of 32, <= 1024); every thread gets it.
CL_DEVINL float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.0f;
    for (int w = 0; w < nw; ++w) t += red[w];
    return t;
}

// ---- FP32 GEMV (router, DeltaNet alpha/beta, shared-expert gate) -------------
__global__ void gemv_f32_kernel(const float* __restrict__ w, int n, int k, const float* x,
                                float* y) {
    grid_launch_dependents();
    grid_wait();
    const int row = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (row >= n) return;
    const float4* w4 = reinterpret_cast<const float4*>(w + (size_t)row * k);
    const float4* x4 = reinterpret_cast<const float4*>(x);
    float acc = 0.0f;
    for (int i = lane; i < k / 4; i += 32) {
        const float4 a = __ldg(w4 + i), b = x4[i];
        acc += a.x * b.x;
        acc += a.y * b.y;
        acc += a.z * b.z;
        acc += a.w * b.w;
    }
    acc = warp_sum(acc);
    if (lane == 0) y[row] = acc;
}

// ---- router: softmax over the logits, top-k, renormalisation -----------------
constexpr int kRouteThreads = 256;

__global__ void __launch_bounds__(kRouteThreads) route_kernel(const float* logits, int ne, int k,
                                                              int* ids, float* wts) {
    grid_launch_dependents();
    grid_wait();
    extern __shared__ float prob[];  // [ne]
    __shared__ float red[32];
    __shared__ float rv[32];
    __shared__ int ri[32];
    __shared__ float sel_v[8];
    __shared__ int sel_i[8];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // block b: token b of a batch (logits [tokens][ne], ids / wts [tokens][k])
    logits += (size_t)blockIdx.x * ne;
    ids += (size_t)blockIdx.x * k;
    wts += (size_t)blockIdx.x * k;
    // softmax (metal_softmax_f32: max, exp(v - max), sum, numerator / sum)
    float m = -INFINITY;
    for (int i = tid; i < ne; i += kRouteThreads) m = fmaxf(m, logits[i]);
    m = warp_max(m);
    if (lane == 0) red[warp] = m;
    __syncthreads();
    m = red[0];
    for (int w = 1; w < kRouteThreads / 32; ++w) m = fmaxf(m, red[w]);
    __syncthreads();
    float s = 0.0f;
    for (int i = tid; i < ne; i += kRouteThreads) {
        const float e = expf(logits[i] - m);
        prob[i] = e;
        s += e;
    }
    s = block_sum(s, red);
    for (int i = tid; i < ne; i += kRouteThreads) prob[i] = s > 0.0f ? prob[i] / s : 0.0f;
    __syncthreads();
    // top-k: k rounds of argmax (largest value, lowest id on ties), which is
    // the order of the reference's strict-'>' insertion scan
    for (int r = 0; r < k; ++r) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int i = tid; i < ne; i += kRouteThreads) {
            const float v = prob[i];
            if (v > bv || (v == bv && i < bi)) {
                bv = v;
                bi = i;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) {
            rv[warp] = bv;
            ri[warp] = bi;
        }
        __syncthreads();
        if (tid == 0) {
            float v = rv[0];
            int i = ri[0];
            for (int w = 1; w < kRouteThreads / 32; ++w)
                if (rv[w] > v || (rv[w] == v && ri[w] < i)) {
                    v = rv[w];
                    i = ri[w];
                }
            sel_v[r] = v;
            sel_i[r] = i;
            prob[i] = -INFINITY;  // out of the next rounds
        }
        __syncthreads();
    }
    if (tid == 0) {
        // metal_topk_renorm_f32: sum in rank order, multiply by 1 / sum
        float sum = 0.0f;
        for (int r = 0; r < k; ++r) sum += sel_v[r];
        const float inv = sum > 0.0f ? 1.0f / sum : 0.0f;
        for (int r = 0; r < k; ++r) {
            ids[r] = sel_i[r];
            wts[r] = sel_v[r] * inv;
        }
    }
}

// ---- routed expert GEMV -------------------------------------------------------
// y[r][row] = W_e[row] . x_r for route r (e = ids[r]), or with w_up the
// SwiGLU silu(W_e[row] . x) * (U_e[row] . x).  Expert e lives on rank
// e % world as local expert e / world; routes of other ranks are skipped
// (their outputs are neither written nor read).  x_r = x + (r / x_group) *
// x_stride: one input per route (x_group 1), or one per token of a batch
// whose x_group routes share it.
constexpr int kExpWarps = 8, kExpThreads = 32 * kExpWarps, kExpRows = 2;
constexpr int kMaxExpUnits = 256;  // k <= 8192

template <int F, bool SW>
__global__ void __launch_bounds__(kExpThreads)
    expert_gemv_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ w_up, long long stride, int n,
                       int k, const float* x, int x_stride, int x_group, const int* ids,
                       int rank, int world, float* y) {
    constexpr int NV = SW ? 2 * kExpRows : kExpRows;
    __shared__ uint4 planes[8][kMaxExpUnits];  // XQ unit u: 6 limb chunks, lsum, (xs, xsum)
    grid_launch_dependents();
    grid_wait();
    const int r = blockIdx.y;
    const int e = ids[r];
    if (e % world != rank) return;
    const int local = e / world;
    const int units = k / 32;
    const float* xr = x + (size_t)(r / x_group) * x_stride;
    for (int u = threadIdx.x; u < units; u += kExpThreads) {
        float v[32];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float4 f = reinterpret_cast<const float4*>(xr + 32 * u)[q];
            v[4 * q] = f.x;
            v[4 * q + 1] = f.y;
            v[4 * q + 2] = f.z;
            v[4 * q + 3] = f.w;
        }
        XUnit xu;
        encode_unit(v, xu);
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int l = 0; l < 3; ++l) {
                const int4 t = xu.l[c][l];
                planes[3 * c + l][u] = make_uint4((uint32_t)t.x, (uint32_t)t.y, (uint32_t)t.z, (uint32_t)t.w);
            }
        planes[6][u] = make_uint4((uint32_t)xu.s[0].x, (uint32_t)xu.s[0].y, (uint32_t)xu.s[1].x, (uint32_t)xu.s[1].y);
        planes[7][u] = make_uint4(__float_as_uint(xu.xs), __float_as_uint(xu.xsum), 0u, 0u);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * kExpWarps + warp) * kExpRows;
    if (row0 >= n) return;
    const int rows = min(kExpRows, n - row0);
    const int nb = (F == CL_TYPE_Q8_0 || F == CL_TYPE_Q5_0) ? units : units / 8;
    const uint8_t* rp[NV];
#pragma unroll
    for (int j = 0; j < kExpRows; ++j) {
        const size_t off = ((size_t)local * n + row0 + min(j, rows - 1)) * (size_t)stride;
        rp[j] = w + off;
        if (SW) rp[kExpRows + j] = w_up + off;
    }
    float acc[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) acc[j] = 0.0f;
    for (int u = lane; u < units; u += 32) {
        XUnit xu;
#pragma unroll
        for (int c = 0; c < 2; ++c)
#pragma unroll
            for (int l = 0; l < 3; ++l) {
                const uint4 t = planes[3 * c + l][u];
                xu.l[c][l] = make_int4((int)t.x, (int)t.y, (int)t.z, (int)t.w);
            }
        const uint4 s4 = planes[6][u], f4 = planes[7][u];
        xu.s[0] = make_int2((int)s4.x, (int)s4.y);
        xu.s[1] = make_int2((int)s4.z, (int)s4.w);
        xu.xs = __uint_as_float(f4.x);
        xu.xsum = __uint_as_float(f4.y);
#pragma unroll
        for (int j = 0; j < NV; ++j) acc[j] += Fmt<F>::template dot<GlobalLd>(rp[j], u, nb, xu);
    }
    float v = warp_sum_many<NV>(acc, lane);
    constexpr int G = 32 / NV;
    const int idx = red_index<NV>(lane);
    if (SW) {
        const float up = __shfl_down_sync(0xffffffffu, v, (kExpRows * G) & 31);
        // SwiGLU (metal_swiglu_f32, metal_llm.metal:895-910)
        v = v * sigmoid_stable(v) * up;
    }
    if ((lane & (G - 1)) == 0 && idx < kExpRows && idx < rows) y[(size_t)r * n + row0 + idx] = v;
}

// ---- grouped expert GEMV (prefill) --------------------------------------------
// The per-route kernel above encodes a route's input in every CTA of the
// route and reads an expert's rows once per route that picked it.  A prompt
// chunk of m tokens makes m * top_k routes over at most n_experts experts, so
// prefill groups them by expert (the reference evaluates a prompt's
// (token, expert) pairs expert by expert: moe_llm.mm:2692-2843, 3087-3108):
//   1. route_group_kernel buckets this rank's routes by local expert
//      (offsets [n_local + 1], route list; once per layer, shared by the
//      gate/up and the down product);
//   2. xq_planes_kernel encodes every input row once into the XQ unit planes
//      that expert_gemv_kernel builds in shared memory ([input][unit][8]);
//   3. expert_grouped_kernel: CTA (row block, local expert) walks the
//      expert's routes kGroupChunk at a time.  Per route and row it forms the
//      same unit dots in the same order as expert_gemv_kernel, so each output
//      equals that kernel's, while the expert's rows are read from HBM once
//      and come from L1 for the routes after the first.
constexpr int kGroupThreads = 1024, kMaxGroupExperts = 4096, kGroupChunk = 4;

__global__ void __launch_bounds__(kGroupThreads)
    route_group_kernel(const int* ids, int routes, int n_local, int rank, int world, int* offsets, int* list) {
    __shared__ int cnt[kMaxGroupExperts];
    __shared__ int warp_tot[kGroupThreads / 32];
    grid_launch_dependents();
    grid_wait();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int e = tid; e < kMaxGroupExperts; e += kGroupThreads) cnt[e] = 0;
    __syncthreads();
    for (int r = tid; r < routes; r += kGroupThreads) {
        const int e = ids[r];
        if (e >= 0 && e % world == rank && e / world < n_local) atomicAdd(&cnt[e / world], 1);
    }
    __syncthreads();
    // exclusive scan: thread t owns experts [4t, 4t + 4)
    constexpr int kPer = kMaxGroupExperts / kGroupThreads;
    int own[kPer], run = 0;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        own[i] = run;
        run += cnt[kPer * tid + i];
    }
    int incl = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int base = 0;
    for (int w = 0; w < warp; ++w) base += warp_tot[w];
    base += incl - run;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int e = kPer * tid + i;
        cnt[e] = base + own[i];  // from here on: the next free slot of expert e
        if (e <= n_local) offsets[e] = base + own[i];
    }
    __syncthreads();
    for (int r = tid; r < routes; r += kGroupThreads) {
        const int e = ids[r];
        if (e >= 0 && e % world == rank && e / world < n_local) list[atomicAdd(&cnt[e / world], 1)] = r;
    }
}

// Plane p of unit u of input row i at planes[(i * units + u) * 8 + p]: limbs
// (chunk c, limb l) at 3c + l, the chunk sums at 6, (xs, xsum) at 7.
// skip_remote (one input per route): rows of other ranks' routes are skipped.
__global__ void xq_planes_kernel(const float* x, int x_stride, int inputs, int units, const int* ids, int rank,
                                 int world, int skip_remote, uint4* planes) {
    grid_launch_dependents();
    grid_wait();
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (long long)inputs * units) return;
    const int i = (int)(t / units), u = (int)(t - (long long)i * units);
    if (skip_remote && ids[i] % world != rank) return;
    const float* xr = x + (size_t)i * x_stride + 32 * u;
    float v[32];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const float4 f = reinterpret_cast<const float4*>(xr)[q];
        v[4 * q] = f.x;
        v[4 * q + 1] = f.y;
        v[4 * q + 2] = f.z;
        v[4 * q + 3] = f.w;
    }
    XUnit xu;
    encode_unit(v, xu);
    uint4* p = planes + (size_t)t * 8;
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int l = 0; l < 3; ++l) {
            const int4 q = xu.l[c][l];
            p[3 * c + l] = make_uint4((uint32_t)q.x, (uint32_t)q.y, (uint32_t)q.z, (uint32_t)q.w);
        }
    p[6] = make_uint4((uint32_t)xu.s[0].x, (uint32_t)xu.s[0].y, (uint32_t)xu.s[1].x, (uint32_t)xu.s[1].y);
    p[7] = make_uint4(__float_as_uint(xu.xs), __float_as_uint(xu.xsum), 0u, 0u);
}

template <int F, bool SW>
__global__ void __launch_bounds__(kExpThreads)
    expert_grouped_kernel(const uint8_t* __restrict__ w, const uint8_t* __restrict__ w_up, long long stride, int n,
                          int k, const uint4* planes, int x_group, const int* offsets, const int* list, float* y) {
    constexpr int NV = SW ? 2 * kExpRows : kExpRows;
    grid_launch_dependents();
    grid_wait();
    const int local = blockIdx.y;
    const int beg = offsets[local], end = offsets[local + 1];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = (blockIdx.x * kExpWarps + warp) * kExpRows;
    if (beg >= end || row0 >= n) return;
    const int rows = min(kExpRows, n - row0);
    const int units = k / 32;
    const int nb = (F == CL_TYPE_Q8_0 || F == CL_TYPE_Q5_0) ? units : units / 8;
    const uint8_t* rp[NV];
#pragma unroll
    for (int j = 0; j < kExpRows; ++j) {
        const size_t off = ((size_t)local * n + row0 + min(j, rows - 1)) * (size_t)stride;
        rp[j] = w + off;
        if (SW) rp[kExpRows + j] = w_up + off;
    }
    constexpr int G = 32 / NV;
    const int idx = red_index<NV>(lane);
    for (int c0 = beg; c0 < end; c0 += kGroupChunk) {
        const int nr = min(kGroupChunk, end - c0);
        int r[kGroupChunk];
        const uint4* xp[kGroupChunk];
#pragma unroll
        for (int q = 0; q < kGroupChunk; ++q) {
            r[q] = list[c0 + min(q, nr - 1)];
            xp[q] = planes + (size_t)(r[q] / x_group) * units * 8;
        }
        float acc[kGroupChunk][NV];
#pragma unroll
        for (int q = 0; q < kGroupChunk; ++q)
#pragma unroll
            for (int j = 0; j < NV; ++j) acc[q][j] = 0.0f;
        for (int u = lane; u < units; u += 32) {
#pragma unroll
            for (int q = 0; q < kGroupChunk; ++q) {
                if (q >= nr) break;
                const uint4* p = xp[q] + (size_t)u * 8;
                XUnit xu;
#pragma unroll
                for (int c = 0; c < 2; ++c)
#pragma unroll
                    for (int l = 0; l < 3; ++l) {
                        const uint4 t = p[3 * c + l];
                        xu.l[c][l] = make_int4((int)t.x, (int)t.y, (int)t.z, (int)t.w);
                    }
                const uint4 s4 = p[6], f4 = p[7];
                xu.s[0] = make_int2((int)s4.x, (int)s4.y);
                xu.s[1] = make_int2((int)s4.z, (int)s4.w);
                xu.xs = __uint_as_float(f4.x);
                xu.xsum = __uint_as_float(f4.y);
#pragma unroll
                for (int j = 0; j < NV; ++j) acc[q][j] += Fmt<F>::template dot<GlobalLd>(rp[j], u, nb, xu);
            }
        }
#pragma unroll
        for (int q = 0; q < kGroupChunk; ++q) {
            if (q >= nr) break;
            float v = warp_sum_many<NV>(acc[q], lane);
            if (SW) {
                const float up = __shfl_down_sync(0xffffffffu, v, (kExpRows * G) & 31);
                v = v * sigmoid_stable(v) * up;
            }
            if ((lane & (G - 1)) == 0 && idx < kExpRows && idx < rows) y[(size_t)r[q] * n + row0 + idx] = v;
        }
    }
}

// ---- expert combine: out = residual + (sum_r w_r y_r + sigmoid(g) * shared) ----
__global__ void combine_kernel(const float* y, const int* ids, const float* wts,
                               int routes, int n, int rank, int world, const float* shared_y,
                               const float* shared_logit, const float* residual, float* out) {
    grid_launch_dependents();
    grid_wait();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= n) return;
    // blockIdx.y: token of a batch ([tokens][routes] ids / weights, [tokens * routes][n] y, rows of n)
    const size_t tk = blockIdx.y;
    ids += tk * routes;
    wts += tk * routes;
    y += tk * routes * n;
    if (shared_y) {
        shared_y += tk * n;
        shared_logit += tk;
    }
    if (residual) residual += tk * n;
    out += tk * n;
    float acc = 0.0f;
    for (int r = 0; r < routes; ++r)
        if (ids[r] % world == rank) acc += wts[r] * y[(size_t)r * n + c];
    if (shared_y) acc = acc + shared_y[c] * sigmoid_stable(*shared_logit);
    out[c] = residual ? residual[c] + acc : acc;
}

// ---- Gated DeltaNet -------------------------------------------------------------
// Block b of D threads owns qkv channels [b D, b D + D): blocks < 2 G are the
// q and k heads (L2-normalised), the rest the value heads.  Block 0 also
// turns alpha / beta into decay / beta.
__global__ void gdn_prep_kernel(const float* qkv, const float* alpha,
                                const float* beta_raw, const float* __restrict__ conv_w, float* hist,
                                const float* __restrict__ dt_bias, const float* __restrict__ a, int key_heads,
                                int value_heads, int d, int kc, float eps, float* act,
                                float* decay, float* beta) {
    grid_launch_dependents();
    grid_wait();
    __shared__ float red[32];
    const int b = blockIdx.x, t = threadIdx.x;
    const int width = (2 * key_heads + value_heads) * d;
    const int c = b * d + t;
    // causal depthwise conv over [history (kc - 1 rows), this token], then SiLU
    float acc = 0.0f;
    for (int tap = 0; tap < kc - 1; ++tap) acc += hist[(size_t)tap * width + c] * conv_w[(size_t)c * kc + tap];
    const float cur = qkv[c];
    acc += cur * conv_w[(size_t)c * kc + kc - 1];
    // commit the history: row r <- row r + 1, last row <- this token (one
    // thread per channel reads before it writes)
    for (int tap = 0; tap + 1 < kc - 1; ++tap) hist[(size_t)tap * width + c] = hist[(size_t)(tap + 1) * width + c];
    if (kc >= 2) hist[(size_t)(kc - 2) * width + c] = cur;
    float v = acc * sigmoid_stable(acc);
    if (b < 2 * key_heads) {
        const float ss = block_sum(v * v, red);
        v = v * rsqrtf(ss + eps);  // metal_l2norm_heads_f32
    }
    act[c] = v;
    if (b == 0) {
        for (int h = t; h < value_heads; h += blockDim.x) {
            const float ab = alpha[h] + dt_bias[h];
            const float sp = ab > 20.0f ? ab : (ab < -20.0f ? expf(ab) : logf(1.0f + expf(ab)));
            decay[h] = expf(sp * a[h]);
            beta[h] = sigmoid_stable(beta_raw[h]);
        }
    }
}

// The same for `rows` consecutive tokens (a prefill chunk): block b walks
// the tokens in order with the conv window of its channel in registers,
// then leaves the last conv_kernel - 1 inputs as the history.  Per token the
// expressions and their order are those of gdn_prep_kernel.
constexpr int kMaxConv = 9;

__global__ void gdn_prep_rows_kernel(const float* qkv, const float* alpha,
                                     const float* beta_raw, const float* __restrict__ conv_w, float* hist,
                                     const float* __restrict__ dt_bias, const float* __restrict__ a, int key_heads,
                                     int value_heads, int d, int kc, float eps, int rows, float* act,
                                     float* decay, float* beta) {
    grid_launch_dependents();
    grid_wait();
    __shared__ float red[32];
    const int b = blockIdx.x, t = threadIdx.x;
    const int width = (2 * key_heads + value_heads) * d;
    const int c = b * d + t;
    float win[kMaxConv - 1], wk[kMaxConv - 1];
#pragma unroll
    for (int tap = 0; tap < kMaxConv - 1; ++tap) {
        win[tap] = tap < kc - 1 ? hist[(size_t)tap * width + c] : 0.0f;
        wk[tap] = tap < kc - 1 ? conv_w[(size_t)c * kc + tap] : 0.0f;
    }
    const float wlast = conv_w[(size_t)c * kc + kc - 1];
    for (int i = 0; i < rows; ++i) {
        const float cur = qkv[(size_t)i * width + c];
        float acc = 0.0f;
#pragma unroll
        for (int tap = 0; tap < kMaxConv - 1; ++tap)
            if (tap < kc - 1) acc += win[tap] * wk[tap];
        acc += cur * wlast;
#pragma unroll
        for (int tap = 0; tap < kMaxConv - 1; ++tap) {
            if (tap + 1 < kc - 1) win[tap] = win[tap + 1];
            else if (tap == kc - 2) win[tap] = cur;
        }
        float v = acc * sigmoid_stable(acc);
        if (b < 2 * key_heads) {
            const float ss = block_sum(v * v, red);
            v = v * rsqrtf(ss + eps);
        }
        act[(size_t)i * width + c] = v;
    }
#pragma unroll
    for (int tap = 0; tap < kMaxConv - 1; ++tap)
        if (tap < kc - 1) hist[(size_t)tap * width + c] = win[tap];
    if (b == 0) {
        for (int i = 0; i < rows; ++i)
            for (int h = t; h < value_heads; h += blockDim.x) {
                const float ab = alpha[(size_t)i * value_heads + h] + dt_bias[h];
                const float sp = ab > 20.0f ? ab : (ab < -20.0f ? expf(ab) : logf(1.0f + expf(ab)));
                decay[(size_t)i * value_heads + h] = expf(sp * a[h]);
                beta[(size_t)i * value_heads + h] = sigmoid_stable(beta_raw[(size_t)i * value_heads + h]);
            }
    }
}

// One block per value head h (key head h % key_heads), 2 D threads: thread
// (col, half) keeps rows [half D/2, half D/2 + D/2) of state column col in
// registers.  S <- decay S; pred = S^T k; S += k (beta (v - pred))^T;
// o = S^T q / sqrt(D); then RMSNorm(o) * silu(z).
constexpr int kMaxGdnDim = 128;

__global__ void __launch_bounds__(2 * kMaxGdnDim) gdn_step_kernel(
    const float* act, const float* decay, const float* beta,
    const float* z, const float* __restrict__ gamma, float* state, int key_heads,
    int value_heads, int d, float eps, float* out) {
    grid_launch_dependents();
    grid_wait();
    __shared__ float qs[kMaxGdnDim], ks[kMaxGdnDim], part[2][kMaxGdnDim];
    __shared__ float red[32];
    const int h = blockIdx.x, kh = h % key_heads;
    const int t = threadIdx.x, col = t % d, half = t / d, hd = d / 2;
    if (t < d) {
        qs[t] = act[kh * d + t];
        ks[t] = act[key_heads * d + kh * d + t];
    }
    __syncthreads();
    float* S = state + (size_t)h * d * d;
    const float dec = decay[h], bt = beta[h];
    float s[kMaxGdnDim / 2];
    float pred = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxGdnDim / 2; ++i) {
        if (i < hd) {
            const int row = half * hd + i;
            s[i] = S[(size_t)row * d + col] * dec;
            pred += s[i] * ks[row];
        }
    }
    part[half][col] = pred;
    __syncthreads();
    pred = part[0][col] + part[1][col];
    const float delta = bt * (act[2 * key_heads * d + h * d + col] - pred);
    const float qscale = rsqrtf((float)d);
    float o = 0.0f;
#pragma unroll
    for (int i = 0; i < kMaxGdnDim / 2; ++i) {
        if (i < hd) {
            const int row = half * hd + i;
            s[i] += ks[row] * delta;
            S[(size_t)row * d + col] = s[i];
            o += s[i] * qs[row] * qscale;
        }
    }
    __syncthreads();
    part[half][col] = o;
    __syncthreads();
    o = part[0][col] + part[1][col];
    // per-head RMSNorm (metal_rmsnorm_f32) over the d outputs, then the gate
    const float ss = block_sum(half == 0 ? o * o : 0.0f, red);
    const float inv = rsqrtf(ss / (float)d + eps);
    if (half == 0) {
        const float zz = z[h * d + col];
        out[h * d + col] = o * inv * gamma[col] * (zz * sigmoid_stable(zz));
    }
}

// The same step with each head's columns split across a thread-block
// cluster: CTA r of the cluster owns columns 32 r .. 32 r + 31 (the delta
// rule is independent per column: pred, delta, the state update and o all
// read one column of S), 8 warps split the rows.  It runs `rows`
// consecutive tokens (one in decode, a prefill chunk in prefill) with the
// state in registers between them, read once and written once.  The per-head RMSNorm
// needs the sum of o^2 over all columns: each CTA leaves its 32-column sum
// in shared memory and every CTA adds the cluster's sums in rank order
// through distributed shared memory.  d / 32 CTAs per head (4 at d = 128),
// so a 32-head layer runs on 128 SMs instead of 32.
constexpr int kGdnCols = 32, kGdnRowGroups = 8;

__global__ void __launch_bounds__(kGdnCols * kGdnRowGroups) gdn_step_cluster_kernel(
    const float* act, const float* decay, const float* beta,
    const float* z, const float* __restrict__ gamma, float* state, int key_heads,
    int value_heads, int d, float eps, float* out, int rows) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    grid_launch_dependents();
    grid_wait();
    __shared__ float qs[kMaxGdnDim], ks[kMaxGdnDim], part[kGdnRowGroups][kGdnCols];
    __shared__ float ssq;
    const int nparts = d / kGdnCols;
    const int h = blockIdx.x / nparts, cpart = (int)cluster.block_rank(), kh = h % key_heads;
    const int t = threadIdx.x, cl = t % kGdnCols, rg = t / kGdnCols;
    const int col = cpart * kGdnCols + cl, rows_per = d / kGdnRowGroups;
    const int width = (2 * key_heads + value_heads) * d;
    float* S = state + (size_t)h * d * d;
    // the thread's part of state column col stays in registers across the tokens
    float s[kMaxGdnDim / kGdnRowGroups];
#pragma unroll
    for (int i = 0; i < kMaxGdnDim / kGdnRowGroups; ++i)
        if (i < rows_per) s[i] = S[(size_t)(rg * rows_per + i) * d + col];
    const float qscale = rsqrtf((float)d);
    for (int tok = 0; tok < rows; ++tok) {
        const float* at = act + (size_t)tok * width;
        if (tok > 0) __syncthreads();  // the previous token's q / k reads are done
        for (int i = t; i < d; i += blockDim.x) {
            qs[i] = at[kh * d + i];
            ks[i] = at[key_heads * d + kh * d + i];
        }
        __syncthreads();
        const float dec = decay[(size_t)tok * value_heads + h], bt = beta[(size_t)tok * value_heads + h];
        float pred = 0.0f;
#pragma unroll
        for (int i = 0; i < kMaxGdnDim / kGdnRowGroups; ++i) {
            if (i < rows_per) {
                const int row = rg * rows_per + i;
                s[i] = s[i] * dec;
                pred += s[i] * ks[row];
            }
        }
        part[rg][cl] = pred;
        __syncthreads();
        pred = 0.0f;
#pragma unroll
        for (int r = 0; r < kGdnRowGroups; ++r) pred += part[r][cl];
        const float delta = bt * (at[2 * key_heads * d + h * d + col] - pred);
        float o = 0.0f;
#pragma unroll
        for (int i = 0; i < kMaxGdnDim / kGdnRowGroups; ++i) {
            if (i < rows_per) {
                const int row = rg * rows_per + i;
                s[i] += ks[row] * delta;
                o += s[i] * qs[row] * qscale;
            }
        }
        __syncthreads();
        part[rg][cl] = o;
        __syncthreads();
        o = 0.0f;
#pragma unroll
        for (int r = 0; r < kGdnRowGroups; ++r) o += part[r][cl];
        if (t < kGdnCols) {
            const float w = warp_sum(o * o);
            if (t == 0) ssq = w;
        }
        cluster.sync();  // every CTA's ssq is written
        float ss = 0.0f;
        for (int r = 0; r < nparts; ++r) ss += *cluster.map_shared_rank(&ssq, r);
        cluster.sync();  // no CTA rewrites its ssq while another still reads it
        // per-head RMSNorm (metal_rmsnorm_f32) over the d outputs, then the gate
        const float inv = rsqrtf(ss / (float)d + eps);
        if (rg == 0) {
            const size_t oi = (size_t)tok * value_heads * d + (size_t)h * d + col;
            const float zz = z[oi];
            out[oi] = o * inv * gamma[col] * (zz * sigmoid_stable(zz));
        }
    }
#pragma unroll
    for (int i = 0; i < kMaxGdnDim / kGdnRowGroups; ++i)
        if (i < rows_per) S[(size_t)(rg * rows_per + i) * d + col] = s[i];
}

// ---- gated attention: split, per-head norms, partial RoPE, KV append -------
// Blocks [0, hq): query heads (query and gate halves of the packed head);
// blocks [hq, hq + hkv): KV heads.  blockDim = head_dim.
__global__ void attn_gate_prep_kernel(const float* mixed, const float* k_raw,
                                      const float* v_raw, const float* __restrict__ q_norm,
                                      const float* __restrict__ k_norm, int hq, int hkv, int d, int rot,
                                      const float* __restrict__ cos_sin, const int* pos_dev, int pos0,
                                      float eps, float* __restrict__ q_out, float* __restrict__ gate_out,
                                      float* k_cache, float* v_cache) {
    grid_launch_dependents();
    grid_wait();
    extern __shared__ float hs[];  // [d] normalised head
    __shared__ float red[32];
    const int b = blockIdx.x, t = threadIdx.x;
    // blockIdx.y: token of a batch at position (pos_dev ? *pos_dev : pos0) + blockIdx.y
    const int row = blockIdx.y;
    const int pos = (pos_dev ? *pos_dev : pos0) + row;
    mixed += (size_t)row * hq * 2 * d;
    k_raw += (size_t)row * hkv * d;
    v_raw += (size_t)row * hkv * d;
    q_out += (size_t)row * hq * d;
    gate_out += (size_t)row * hq * d;
    const bool is_q = b < hq;
    const int head = is_q ? b : b - hq;
    const float raw = is_q ? mixed[(size_t)head * 2 * d + t] : k_raw[(size_t)head * d + t];
    if (is_q) gate_out[(size_t)head * d + t] = mixed[(size_t)head * 2 * d + d + t];
    const float ss = block_sum(raw * raw, red);
    const float nv = raw * rsqrtf(ss / (float)d + eps) * (is_q ? q_norm[t] : k_norm[t]);
    hs[t] = nv;
    __syncthreads();
    float o = nv;
    if (t < rot) {
        const int half = rot / 2, p = t < half ? t : t - half;
        const float c = cos_sin[((size_t)pos * half + p) * 2], s = cos_sin[((size_t)pos * half + p) * 2 + 1];
        const float x0 = hs[p], x1 = hs[p + half];
        o = t < half ? x0 * c - x1 * s : x0 * s + x1 * c;
    }
    if (is_q) {
        q_out[(size_t)head * d + t] = o;
    } else {
        const size_t kvd = (size_t)hkv * d;
        k_cache[(size_t)pos * kvd + (size_t)head * d + t] = o;
        v_cache[(size_t)pos * kvd + (size_t)head * d + t] = v_raw[(size_t)head * d + t];
    }
}

__global__ void mul_sigmoid_kernel(const float* a, const float* g, float* out,
                                   int n) {
    grid_launch_dependents();
    grid_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = a[i] * sigmoid_stable(g[i]);
}

template <int F, bool SW>
cudaError_t launch_expert(const void* w, const void* w_up, long long stride, int n, int k, const float* x,
                          int x_stride, int x_group, const int* ids, int routes, int rank, int world, float* y,
                          cudaStream_t stream) {
    const dim3 grid((n + kExpWarps * kExpRows - 1) / (kExpWarps * kExpRows), routes);
    return launch_pdl(expert_gemv_kernel<F, SW>, grid, dim3(kExpThreads), 0, stream,
                      static_cast<const uint8_t*>(w), static_cast<const uint8_t*>(w_up), stride, n, k, x, x_stride,
                      x_group, ids, rank, world, y);
}

template <bool SW>
cudaError_t launch_expert_type(int type, const void* w, const void* w_up, long long stride, int n, int k,
                               const float* x, int x_stride, int xg, const int* ids, int routes, int rank, int world,
                               float* y, cudaStream_t stream) {
    switch (type) {
    case CL_TYPE_Q4_K: return launch_expert<CL_TYPE_Q4_K, SW>(w, w_up, stride, n, k, x, x_stride, xg, ids, routes, rank, world, y, stream);
    case CL_TYPE_Q5_K: return launch_expert<CL_TYPE_Q5_K, SW>(w, w_up, stride, n, k, x, x_stride, xg, ids, routes, rank, world, y, stream);
    case CL_TYPE_Q6_K: return launch_expert<CL_TYPE_Q6_K, SW>(w, w_up, stride, n, k, x, x_stride, xg, ids, routes, rank, world, y, stream);
    case CL_TYPE_Q8_0: return launch_expert<CL_TYPE_Q8_0, SW>(w, w_up, stride, n, k, x, x_stride, xg, ids, routes, rank, world, y, stream);
    case CL_TYPE_Q5_0: return launch_expert<CL_TYPE_Q5_0, SW>(w, w_up, stride, n, k, x, x_stride, xg, ids, routes, rank, world, y, stream);
    default: return cudaErrorInvalidValue;
    }
}

template <int F, bool SW>
cudaError_t launch_grouped(const void* w, const void* w_up, long long stride, int n, int k, const uint4* planes,
                           int x_group, const int* offsets, const int* list, int n_local, float* y,
                           cudaStream_t stream) {
    const dim3 grid((n + kExpWarps * kExpRows - 1) / (kExpWarps * kExpRows), n_local);
    return launch_pdl(expert_grouped_kernel<F, SW>, grid, dim3(kExpThreads), 0, stream,
                      static_cast<const uint8_t*>(w), static_cast<const uint8_t*>(w_up), stride, n, k, planes,
                      x_group, offsets, list, y);
}

template <bool SW>
cudaError_t launch_grouped_type(int type, const void* w, const void* w_up, long long stride, int n, int k,
                                const uint4* planes, int xg, const int* offsets, const int* list, int n_local,
                                float* y, cudaStream_t stream) {
    switch (type) {
    case CL_TYPE_Q4_K: return launch_grouped<CL_TYPE_Q4_K, SW>(w, w_up, stride, n, k, planes, xg, offsets, list, n_local, y, stream);
    case CL_TYPE_Q5_K: return launch_grouped<CL_TYPE_Q5_K, SW>(w, w_up, stride, n, k, planes, xg, offsets, list, n_local, y, stream);
    case CL_TYPE_Q6_K: return launch_grouped<CL_TYPE_Q6_K, SW>(w, w_up, stride, n, k, planes, xg, offsets, list, n_local, y, stream);
    case CL_TYPE_Q8_0: return launch_grouped<CL_TYPE_Q8_0, SW>(w, w_up, stride, n, k, planes, xg, offsets, list, n_local, y, stream);
    case CL_TYPE_Q5_0: return launch_grouped<CL_TYPE_Q5_0, SW>(w, w_up, stride, n, k, planes, xg, offsets, list, n_local, y, stream);
    default: return cudaErrorInvalidValue;
    }
}

int status(cudaError_t e) { return e == cudaSuccess ? CL_OK : CL_ERR_CUDA; }
bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace moe
}  // namespace cl

using namespace cl::moe;
using cl::launch_pdl;

extern "C" {

CL_API int cl_gemv_f32(const float* w, int n, int k, const float* x, float* y, cudaStream_t stream) {
    if (w == nullptr || x == nullptr || y == nullptr || n <= 0 || k <= 0 || k % 4 || !aligned16(w) ||
        !aligned16(x))
        return CL_ERR_INVALID;
    const int threads = 256, rows_per_block = threads / 32;
    return status(launch_pdl(gemv_f32_kernel, dim3((n + rows_per_block - 1) / rows_per_block), dim3(threads), 0,
                             stream, w, n, k, x, y));
}

CL_API int cl_moe_route(const float* logits, int n_experts, int k, int* ids, float* weights, cudaStream_t stream) {
    if (logits == nullptr || ids == nullptr || weights == nullptr || n_experts <= 0 || n_experts > 16384 || k <= 0 ||
        k > 8 || k > n_experts)
        return CL_ERR_INVALID;
    return status(launch_pdl(route_kernel, dim3(1), dim3(kRouteThreads), (size_t)n_experts * sizeof(float), stream,
                             logits, n_experts, k, ids, weights));
}

CL_API int cl_moe_expert_gemv(int type, const void* w, const void* w_up, long long stride, int n, int k,
                              const float* x, int x_stride, const int* ids, int routes, int rank, int world,
                              float* y, cudaStream_t stream) {
    if (w == nullptr || x == nullptr || ids == nullptr || y == nullptr || n <= 0 || k <= 0 || k % 32 ||
        k / 32 > kMaxExpUnits || routes <= 0 || routes > 65535 || world <= 0 || rank < 0 || rank >= world ||
        x_stride < 0 || x_stride % 4 || !aligned16(w) || !aligned16(x) || stride % 16 ||
        cl_native_row_bytes(type, k) < 0 || stride < cl_row_stride(type, k) || (w_up && !aligned16(w_up)))
        return CL_ERR_INVALID;
    if (type != CL_TYPE_Q4_K && type != CL_TYPE_Q5_K && type != CL_TYPE_Q6_K && type != CL_TYPE_Q8_0 &&
        type != CL_TYPE_Q5_0)
        return CL_ERR_UNSUPPORTED;
    return status(w_up ? launch_expert_type<true>(type, w, w_up, stride, n, k, x, x_stride, 1, ids, routes, rank,
                                                  world, y, stream)
                       : launch_expert_type<false>(type, w, nullptr, stride, n, k, x, x_stride, 1, ids, routes, rank,
                                                   world, y, stream));
}

CL_API int cl_moe_expert_gemv_rows(int type, const void* w, const void* w_up, long long stride, int n, int k,
                                   const float* x, int x_stride, int x_group, const int* ids, int routes, int rank,
                                   int world, float* y, cudaStream_t stream) {
    if (x_group <= 0) return CL_ERR_INVALID;
    if (w == nullptr || x == nullptr || ids == nullptr || y == nullptr || n <= 0 || k <= 0 || k % 32 ||
        k / 32 > kMaxExpUnits || routes <= 0 || routes > 65535 || world <= 0 || rank < 0 || rank >= world ||
        x_stride < 0 || x_stride % 4 || !aligned16(w) || !aligned16(x) || stride % 16 ||
        cl_native_row_bytes(type, k) < 0 || stride < cl_row_stride(type, k) || (w_up && !aligned16(w_up)))
        return CL_ERR_INVALID;
    if (type != CL_TYPE_Q4_K && type != CL_TYPE_Q5_K && type != CL_TYPE_Q6_K && type != CL_TYPE_Q8_0 &&
        type != CL_TYPE_Q5_0)
        return CL_ERR_UNSUPPORTED;
    return status(w_up ? launch_expert_type<true>(type, w, w_up, stride, n, k, x, x_stride, x_group, ids, routes,
                                                  rank, world, y, stream)
                       : launch_expert_type<false>(type, w, nullptr, stride, n, k, x, x_stride, x_group, ids,
                                                   routes, rank, world, y, stream));
}

CL_API size_t cl_moe_xq_planes_bytes(int inputs, int k) {
    if (inputs <= 0 || k <= 0 || k % 32) return 0;
    return (size_t)inputs * (size_t)(k / 32) * 8 * sizeof(uint4);
}

CL_API int cl_moe_group_routes(const int* ids, int routes, int n_local, int rank, int world, int* offsets, int* list,
                               cudaStream_t stream) {
    if (ids == nullptr || offsets == nullptr || list == nullptr || routes <= 0 || routes > (1 << 24) ||
        n_local <= 0 || n_local >= kMaxGroupExperts || world <= 0 || rank < 0 || rank >= world)
        return CL_ERR_INVALID;
    return status(launch_pdl(route_group_kernel, dim3(1), dim3(kGroupThreads), 0, stream, ids, routes, n_local, rank,
                             world, offsets, list));
}

CL_API int cl_moe_expert_gemv_grouped(int type, const void* w, const void* w_up, long long stride, int n, int k,
                                      const float* x, int x_stride, int x_group, const int* ids, int routes,
                                      int rank, int world, const int* offsets, const int* list, int n_local,
                                      void* planes, size_t planes_bytes, float* y, cudaStream_t stream) {
    if (w == nullptr || x == nullptr || ids == nullptr || offsets == nullptr || list == nullptr ||
        planes == nullptr || y == nullptr || n <= 0 || k <= 0 || k % 32 || x_group <= 0 || routes <= 0 ||
        routes > (1 << 24) || n_local <= 0 || n_local >= kMaxGroupExperts || world <= 0 || rank < 0 ||
        rank >= world || x_stride < 0 || x_stride % 4 || !aligned16(w) || !aligned16(x) || !aligned16(planes) ||
        stride % 16 || cl_native_row_bytes(type, k) < 0 || stride < cl_row_stride(type, k) ||
        (w_up && !aligned16(w_up)))
        return CL_ERR_INVALID;
    if (type != CL_TYPE_Q4_K && type != CL_TYPE_Q5_K && type != CL_TYPE_Q6_K && type != CL_TYPE_Q8_0 &&
        type != CL_TYPE_Q5_0)
        return CL_ERR_UNSUPPORTED;
    const int inputs = (routes + x_group - 1) / x_group, units = k / 32;
    if (planes_bytes < cl_moe_xq_planes_bytes(inputs, k)) return CL_ERR_INVALID;
    uint4* pl = static_cast<uint4*>(planes);
    const long long work = (long long)inputs * units;
    const int threads = 256;
    cudaError_t e = launch_pdl(xq_planes_kernel, dim3((unsigned)((work + threads - 1) / threads)), dim3(threads), 0,
                               stream, x, x_stride, inputs, units, ids, rank, world,
                               (x_group == 1 && world > 1) ? 1 : 0, pl);
    if (e != cudaSuccess) return status(e);
    return status(w_up ? launch_grouped_type<true>(type, w, w_up, stride, n, k, pl, x_group, offsets, list, n_local,
                                                   y, stream)
                       : launch_grouped_type<false>(type, w, nullptr, stride, n, k, pl, x_group, offsets, list,
                                                    n_local, y, stream));
}

CL_API int cl_moe_combine_rows(const float* y, const int* ids, const float* weights, int routes, int n, int rank,
                               int world, const float* shared_y, const float* shared_logit, const float* residual,
                               float* out, int rows, cudaStream_t stream) {
    if (y == nullptr || ids == nullptr || weights == nullptr || out == nullptr || routes <= 0 || n <= 0 ||
        world <= 0 || rank < 0 || rank >= world || ((shared_y == nullptr) != (shared_logit == nullptr)) ||
        rows <= 0 || rows > 65535)
        return CL_ERR_INVALID;
    return status(launch_pdl(combine_kernel, dim3((n + 255) / 256, rows), dim3(256), 0, stream, y, ids, weights,
                             routes, n, rank, world, shared_y, shared_logit, residual, out));
}

CL_API int cl_moe_route_rows(const float* logits, int rows, int n_experts, int k, int* ids, float* weights,
                             cudaStream_t stream) {
    if (logits == nullptr || ids == nullptr || weights == nullptr || n_experts <= 0 || n_experts > 16384 || k <= 0 ||
        k > 8 || k > n_experts || rows <= 0)
        return CL_ERR_INVALID;
    return status(launch_pdl(route_kernel, dim3(rows), dim3(kRouteThreads), (size_t)n_experts * sizeof(float),
                             stream, logits, n_experts, k, ids, weights));
}

CL_API int cl_moe_combine(const float* y, const int* ids, const float* weights, int routes, int n, int rank, int world,
                          const float* shared_y, const float* shared_logit, const float* residual, float* out,
                          cudaStream_t stream) {
    if (y == nullptr || ids == nullptr || weights == nullptr || out == nullptr || routes <= 0 || n <= 0 ||
        world <= 0 || rank < 0 || rank >= world || ((shared_y == nullptr) != (shared_logit == nullptr)))
        return CL_ERR_INVALID;
    return status(launch_pdl(combine_kernel, dim3((n + 255) / 256), dim3(256), 0, stream, y, ids, weights, routes, n,
                             rank, world, shared_y, shared_logit, residual, out));
}

CL_API int cl_gdn_prep(const float* qkv, const float* alpha, const float* beta_raw, const float* conv_w, float* hist,
                       const float* dt_bias, const float* a, int key_heads, int value_heads, int head_dim,
                       int conv_kernel, float eps, float* act, float* decay, float* beta, cudaStream_t stream) {
    if (qkv == nullptr || alpha == nullptr || beta_raw == nullptr || conv_w == nullptr || hist == nullptr ||
        dt_bias == nullptr || a == nullptr || act == nullptr || decay == nullptr || beta == nullptr ||
        key_heads <= 0 || value_heads <= 0 || value_heads % key_heads || head_dim <= 0 || head_dim % 32 ||
        head_dim > 1024 || conv_kernel < 1 || conv_kernel > 9)
        return CL_ERR_INVALID;
    return status(launch_pdl(gdn_prep_kernel, dim3(2 * key_heads + value_heads), dim3(head_dim), 0, stream, qkv,
                             alpha, beta_raw, conv_w, hist, dt_bias, a, key_heads, value_heads, head_dim,
                             conv_kernel, eps, act, decay, beta));
}

CL_API int cl_gdn_step(const float* act, const float* decay, const float* beta, const float* z, const float* gamma,
                       float* state, int key_heads, int value_heads, int head_dim, float eps, float* out,
                       cudaStream_t stream) {
    if (act == nullptr || decay == nullptr || beta == nullptr || z == nullptr || gamma == nullptr ||
        state == nullptr || out == nullptr || key_heads <= 0 || value_heads <= 0 || value_heads % key_heads ||
        head_dim <= 0 || head_dim % 32 || head_dim > kMaxGdnDim)
        return CL_ERR_INVALID;
    const int nparts = head_dim / kGdnCols;
    if (nparts >= 1 && nparts <= 8) {
        // cluster of nparts CTAs per head (programmatic dependent launch as elsewhere)
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(value_heads * nparts);
        cfg.blockDim = dim3(kGdnCols * kGdnRowGroups);
        cfg.stream = stream;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = nparts;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = cl::g_pdl_enabled ? 2 : 1;
        return status(cudaLaunchKernelEx(&cfg, gdn_step_cluster_kernel, act, decay, beta, z, gamma, state, key_heads,
                                         value_heads, head_dim, eps, out, 1));
    }
    return status(launch_pdl(gdn_step_kernel, dim3(value_heads), dim3(2 * head_dim), 0, stream, act, decay, beta, z,
                             gamma, state, key_heads, value_heads, head_dim, eps, out));
}

CL_API int cl_gdn_prep_rows(const float* qkv, const float* alpha, const float* beta_raw, const float* conv_w,
                            float* hist, const float* dt_bias, const float* a, int key_heads, int value_heads,
                            int head_dim, int conv_kernel, float eps, int rows, float* act, float* decay, float* beta,
                            cudaStream_t stream) {
    if (qkv == nullptr || alpha == nullptr || beta_raw == nullptr || conv_w == nullptr || hist == nullptr ||
        dt_bias == nullptr || a == nullptr || act == nullptr || decay == nullptr || beta == nullptr ||
        key_heads <= 0 || value_heads <= 0 || value_heads % key_heads || head_dim <= 0 || head_dim % 32 ||
        head_dim > 1024 || conv_kernel < 1 || conv_kernel > kMaxConv || rows <= 0)
        return CL_ERR_INVALID;
    return status(launch_pdl(gdn_prep_rows_kernel, dim3(2 * key_heads + value_heads), dim3(head_dim), 0, stream, qkv,
                             alpha, beta_raw, conv_w, hist, dt_bias, a, key_heads, value_heads, head_dim, conv_kernel,
                             eps, rows, act, decay, beta));
}

CL_API int cl_gdn_step_rows(const float* act, const float* decay, const float* beta, const float* z,
                            const float* gamma, float* state, int key_heads, int value_heads, int head_dim, float eps,
                            int rows, float* out, cudaStream_t stream) {
    if (act == nullptr || decay == nullptr || beta == nullptr || z == nullptr || gamma == nullptr ||
        state == nullptr || out == nullptr || key_heads <= 0 || value_heads <= 0 || value_heads % key_heads ||
        head_dim <= 0 || head_dim % 32 || head_dim > kMaxGdnDim || rows <= 0)
        return CL_ERR_INVALID;
    const int nparts = head_dim / kGdnCols;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(value_heads * nparts);
    cfg.blockDim = dim3(kGdnCols * kGdnRowGroups);
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = nparts;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = cl::g_pdl_enabled ? 2 : 1;
    return status(cudaLaunchKernelEx(&cfg, gdn_step_cluster_kernel, act, decay, beta, z, gamma, state, key_heads,
                                     value_heads, head_dim, eps, out, rows));
}

CL_API int cl_attn_gate_prep(const float* mixed, const float* k_raw, const float* v_raw, const float* q_norm,
                             const float* k_norm, int q_heads, int kv_heads, int head_dim, int rot_dim,
                             const float* cos_sin, const int* pos_dev, float eps, float* q_out, float* gate_out,
                             float* k_cache, float* v_cache, cudaStream_t stream) {
    if (mixed == nullptr || k_raw == nullptr || v_raw == nullptr || q_norm == nullptr || k_norm == nullptr ||
        cos_sin == nullptr || pos_dev == nullptr || q_out == nullptr || gate_out == nullptr || k_cache == nullptr ||
        v_cache == nullptr || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || head_dim % 32 || head_dim > 1024 ||
        rot_dim < 0 || rot_dim > head_dim || rot_dim % 2)
        return CL_ERR_INVALID;
    return status(launch_pdl(attn_gate_prep_kernel, dim3(q_heads + kv_heads), dim3(head_dim),
                             (size_t)head_dim * sizeof(float), stream, mixed, k_raw, v_raw, q_norm, k_norm, q_heads,
                             kv_heads, head_dim, rot_dim, cos_sin, pos_dev, 0, eps, q_out, gate_out, k_cache,
                             v_cache));
}

CL_API int cl_attn_gate_prep_rows(const float* mixed, const float* k_raw, const float* v_raw, const float* q_norm,
                                  const float* k_norm, int q_heads, int kv_heads, int head_dim, int rot_dim,
                                  const float* cos_sin, int pos0, int rows, float eps, float* q_out, float* gate_out,
                                  float* k_cache, float* v_cache, cudaStream_t stream) {
    if (mixed == nullptr || k_raw == nullptr || v_raw == nullptr || q_norm == nullptr || k_norm == nullptr ||
        cos_sin == nullptr || q_out == nullptr || gate_out == nullptr || k_cache == nullptr || v_cache == nullptr ||
        q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || head_dim % 32 || head_dim > 1024 || rot_dim < 0 ||
        rot_dim > head_dim || rot_dim % 2 || pos0 < 0 || rows <= 0 || rows > 65535)
        return CL_ERR_INVALID;
    return status(launch_pdl(attn_gate_prep_kernel, dim3(q_heads + kv_heads, rows), dim3(head_dim),
                             (size_t)head_dim * sizeof(float), stream, mixed, k_raw, v_raw, q_norm, k_norm, q_heads,
                             kv_heads, head_dim, rot_dim, cos_sin, nullptr, pos0, eps, q_out, gate_out, k_cache,
                             v_cache));
}

CL_API int cl_mul_sigmoid(const float* a, const float* g, float* out, int n, cudaStream_t stream) {
    if (a == nullptr || g == nullptr || out == nullptr || n <= 0) return CL_ERR_INVALID;
    return status(launch_pdl(mul_sigmoid_kernel, dim3((n + 255) / 256), dim3(256), 0, stream, a, g, out, n));
}

}  // extern "C"

namespace cl {
namespace moe {
__global__ void select_token_kernel(const int32_t* ids, const int* index,
                                    int32_t* out) {
    grid_launch_dependents();
    grid_wait();
    out[0] = ids[*index];
}
}  // namespace moe
}  // namespace cl

extern "C" CL_API int cl_select_token(const int32_t* ids, const int* index_dev, int32_t* out, cudaStream_t stream) {
    if (ids == nullptr || index_dev == nullptr || out == nullptr) return CL_ERR_INVALID;
    return cl::moe::status(cl::launch_pdl(cl::moe::select_token_kernel, dim3(1), dim3(1), 0, stream, ids, index_dev, out));
}
