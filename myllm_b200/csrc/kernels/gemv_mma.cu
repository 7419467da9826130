// Decode GEMV over native K-quant blocks with the integer dot products on the
// tensor cores: y[n] = W[n, k] . x (+ bias) (+ residual), optionally with the
// input RMS-normalised first and a fused SwiGLU over (gate, up) row pairs.
//
// Reference: metal_gevm_q4_k_f32 / metal_gevm_q6_k_f32 (metal_llm.metal:708-781)
// and the CPU oracle gevmt over GgufDequantizer rows (cpu_llm.cpp:512-547,
// model.cpp:581-683).  Same products, different order: the factored form
// d*sc*sum(q*x) - dmin*m*sum(x) (metal_llm.metal:392-393), with sum(q*x)
// exact in integers and only the per-super-block sums scaled in FP32.
//
// Why the tensor cores at batch 1 (measured on B200): the per-row dp4a form
// needs ~24 dp4a + masks + scale decode per row and 32 columns, close to the
// issue slots a B200 SM has per HBM byte at 6.5 TB/s (it measured 0.38 of the
// HBM roofline).  Here one mma.sync.m16n8k32 (u8 weights x s8 activations,
// s32 accumulate) replaces 16 rows x 32 columns x 4 limbs of dp4a work: a
// 16-row Q4_K super-block costs 133 warp instructions.
//
// Activation encoding (XQ4, built in shared memory by every CTA): per
// 256-element block b a scale s_b = max|x| / 127 and four signed 8-bit limbs
//     x = s_b * (l0 + l1 / 2^7 + l2 / 2^14 + l3 / 2^21),
// absolute error below max|x_b| * 2^-29.  Limbs are the MMA's N columns.
//
// Q4_K MMA layout.  A 64-element group of a super-block is 32 bytes whose low
// nibbles are unit 2gi (32 elements) and high nibbles unit 2gi + 1.  One MMA
// takes 16 bytes of the group for 16 rows: K slots 0-15 = the bytes' low
// nibbles, K slots 16-31 = their high nibbles, kept in place (16 q) so one
// AND extracts each.  B columns 0-3 = limbs of the low unit (zero on slots
// 16-31), columns 4-7 = limbs of the high unit (zero on slots 0-15).  Two
// MMAs (bytes 8t..8t+3 and 8t+4..8t+7 of lane quad t) chain into one
// accumulator, so lane (g, t) ends a group holding, for rows g and g+8, the
// sums of one unit (low if t < 2) for limbs 2(t&1), 2(t&1)+1; it scales them
// by that unit's 6-bit sc with integer multiply-adds over the super-block
// (|acc| < 2^28) and converts to FP32 once per super-block.
//
// Q6_K MMA layout.  A super-block half (128 elements) holds ql[64] (low 4
// bits), qh[32] (2 high bits) and 8 int8 scales, one per 16 elements; the
// low nibble of ql byte l + 32j is element l + 32j and the high nibble element
// l + 32j + 64 (j = 0, 1).  One MMA takes 16 such bytes (l = 16s .. 16s+15)
// for 16 rows: K slots 0-15 = q of element l + 32j (B columns 0-3, limbs of
// that 16-element sub-block), slots 16-31 = q of element l + 32j + 64
// (columns 4-7), each q = nibble | 2 bits << 4 in [0, 63] as u8; the -32
// offset is folded in as -32 * sum(limb) per sub-block, precomputed with x.
// Every lane then holds one sub-block and scales by its int8 sc.
//
// Kernel shape: persistent CTAs, one producer warp + 16 consumer warps.  The
// producer streams 16-row tiles (whole rows per stage where they fit, else an
// equal K-chunk of each row) into a shared-memory ring with cp.async.bulk
// (mbarrier completion, bounded waits, every wait taken by the whole warp);
// consumer warps take the stage's super-blocks round-robin, and the last warp
// to finish a tile (a shared-memory ticket) sums the warps' partial rows in
// warp order.  Weights are immutable, so the producer starts before the
// programmatic-dependent-launch wait; consumers wait before reading x.
#include "common.cuh"
#include "gemv_mma.cuh"
#include "launch.cuh"

#include <algorithm>

namespace cl {

// Device-side error word: 4 = producer wait gave up, 5 = consumer wait gave up
// (never expected; reported through cl_device_error).
__device__ int g_gemv_mma_error = 0;

namespace gmma {

constexpr int kRows = 16;   // rows per tile (M of the MMA)
constexpr int kWarps = 16;  // consumer warps per CTA
constexpr int kThreads = (kWarps + 1) * 32;
constexpr int kMaxSegs = 4;
constexpr int kZeroBytes = 1024;
constexpr int kMaxBlocksPerWarp = 6;  // x blocks a consumer warp holds: k <= 16 * 6 * 256

struct Seg {
    const uint8_t* w;
    const uint8_t* w_up;  // SwiGLU: up rows (same type/stride as w)
    long long stride;
    const float* bias;
    const float* residual;
    float* y;
    int type;
    int n;
    int tile_begin;
};

// Stage geometry of one weight format in this launch.
struct Geo {
    int bb;      // bytes of one super-block in the device layout
    int c;       // super-blocks per chunk (one stage holds one chunk of 16 rows)
    int chunks;  // chunks per row
    int rs;      // shared-memory row stride of a stage
    int db;      // Q6_K: bytes of the row's scale array copied with every chunk
};

struct Params {
    Seg seg[kMaxSegs];
    Geo geo[2];  // [0]: format F, [1]: format F2
    const float* x;
    const float* gamma;  // RMSNorm weight applied to x first (cpu_llm.cpp:143-166), or null
    float eps;
    int nseg, k, nb, tiles, stages, stage_bytes;
    int off_xs, off_xsum, off_xn, off_xq, off_stage;  // shared-memory offsets
};

// Fixed part of the shared-memory layout: barriers (16 B per stage), abort
// flag, RMSNorm partials, tile tickets and partial rows for R = NS + 1 tiles
// in flight (a warp runs at most NS stages, hence NS tiles, ahead of the
// slowest), and a zero block.
__host__ __device__ constexpr int off_abort(int ns) { return 16 * ns; }
__host__ __device__ constexpr int off_segs(int ns) { return 16 * ns + 16; }
__host__ __device__ constexpr int off_dred(int ns) { return 16 * ns + 16 + kMaxSegs * (int)sizeof(Seg); }
__host__ __device__ constexpr int off_ticket(int ns) { return off_dred(ns) + 256; }
__host__ __device__ constexpr int off_red(int ns) { return (off_ticket(ns) + 4 * (ns + 1) + 15) & ~15; }
__host__ __device__ constexpr int red_floats(int nmat) { return kWarps * kRows * nmat; }
__host__ __device__ constexpr int off_zero(int ns, int nmat) { return off_red(ns) + 4 * (ns + 1) * red_floats(nmat); }
__host__ __device__ constexpr int fixed_bytes(int ns, int nmat) { return off_zero(ns, nmat) + kZeroBytes; }

struct TileInfo {
    int seg, row0, rows;
};

// The segment table is copied to shared memory once per CTA: reading the
// kernel-parameter copy with a runtime index costs an indexed constant-cache
// load per field, which showed up as long-latency stalls in the stage loops.
CL_DEVINL TileInfo tile_of(const Seg* segs, int nseg, int t) {
    int s = 0;
#pragma unroll
    for (int i = 1; i < kMaxSegs; ++i)
        if (i < nseg && t >= segs[i].tile_begin) s = i;
    const int row0 = (t - segs[s].tile_begin) * kRows;
    return TileInfo{s, row0, min(kRows, segs[s].n - row0)};
}

// One Q6_K super-block of 16 rows (device layout: [ql 128][qh 64][sc 16] per
// block, the row's f16 d array copied after the chunk).  bx0/bx1: the lane's
// B words for the 8 MMAs (m = 4 hh + 2 j + s); xn: -32 * sum of the lane's two
// limbs over each of its sub-blocks; dg/d8: the rows' d.
CL_DEVINL void q6k_sb(const uint8_t* bg, const uint8_t* b8, const uint32_t (&bx0)[8], const uint32_t (&bx1)[8],
                      const int2 (&xn)[8], float xs, int t, float dg, float d8, const Q4Lane& L, float& yg,
                      float& y8) {
    const int h = t >> 1;
    int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            const uint32_t qg = *reinterpret_cast<const uint32_t*>(bg + 128 + 32 * hh + 16 * s + 4 * t);
            const uint32_t q8 = *reinterpret_cast<const uint32_t*>(b8 + 128 + 32 * hh + 16 * s + 4 * t);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int m = 4 * hh + 2 * j + s;
                const uint32_t lg = *reinterpret_cast<const uint32_t*>(bg + 64 * hh + 32 * j + 16 * s + 4 * t);
                const uint32_t l8 = *reinterpret_cast<const uint32_t*>(b8 + 64 * hh + 32 * j + 16 * s + 4 * t);
                // high bits of quarter j at bits 4-5 (low-nibble elements) and of quarter j+2
                const uint32_t hag = (j ? (qg << 2) : (qg << 4)) & 0x30303030u;
                const uint32_t ha8 = (j ? (q8 << 2) : (q8 << 4)) & 0x30303030u;
                const uint32_t hbg = (j ? (qg >> 2) : qg) & 0x30303030u;
                const uint32_t hb8 = (j ? (q8 >> 2) : q8) & 0x30303030u;
                int c[4];
                mma_u8s8_z(c, (lg & 0x0f0f0f0fu) | hag, (l8 & 0x0f0f0f0fu) | ha8, ((lg >> 4) & 0x0f0f0f0fu) | hbg,
                           ((l8 >> 4) & 0x0f0f0f0fu) | hb8, bx0[m], bx1[m]);
                // the lane's sub-block: quarter j (t < 2) or j + 2, elements 16 s ..
                const int sci = 192 + 8 * hh + s + 2 * j + 4 * h;
                const int sg = (int)*reinterpret_cast<const int8_t*>(bg + sci);
                const int s8 = (int)*reinterpret_cast<const int8_t*>(b8 + sci);
                a0 += (c[0] + xn[m].x) * sg;
                a1 += (c[1] + xn[m].y) * sg;
                a2 += (c[2] + xn[m].x) * s8;
                a3 += (c[3] + xn[m].y) * s8;
            }
        }
    }
    const float vg = fmaf((float)a0, L.lw0, (float)a1 * L.lw1) * xs;
    const float v8 = fmaf((float)a2, L.lw0, (float)a3 * L.lw1) * xs;
    yg = fmaf(dg, vg, yg);
    y8 = fmaf(d8, v8, y8);
}

template <int F, bool SW, int F2>
__global__ void __launch_bounds__(kThreads) gemv_mma_kernel(const Params p) {
    constexpr int NMAT = SW ? 2 : 1;
    constexpr bool HAS_Q4 = F == CL_TYPE_Q4_K || F2 == CL_TYPE_Q4_K;
    constexpr bool HAS_Q6 = F == CL_TYPE_Q6_K || F2 == CL_TYPE_Q6_K;
    extern __shared__ __align__(128) uint8_t smem[];
    const int NS = p.stages;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + NS;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + off_abort(NS));
    Seg* segs = reinterpret_cast<Seg*>(smem + off_segs(NS));
    double* dred = reinterpret_cast<double*>(smem + off_dred(NS));
    int* tickets = reinterpret_cast<int*>(smem + off_ticket(NS));  // [NS + 1]
    float* red = reinterpret_cast<float*>(smem + off_red(NS));      // [NS + 1][kWarps][NMAT * 16]
    uint8_t* zero = smem + off_zero(NS, NMAT);
    float* xs = reinterpret_cast<float*>(smem + p.off_xs);
    float* xsum = reinterpret_cast<float*>(smem + p.off_xsum);  // Q4_K: [nb][2][4]
    int* xn = reinterpret_cast<int*>(smem + p.off_xn);             // Q6_K: [nb][16][4]
    uint8_t* xq = smem + p.off_xq;                              // [nb][8 units][4 limbs][32]
    uint8_t* stages = smem + p.off_stage;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kWarps);
        }
        for (int r = 0; r <= NS; ++r) tickets[r] = 0;
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (tid < kZeroBytes / 16) reinterpret_cast<uint4*>(zero)[tid] = make_uint4(0u, 0u, 0u, 0u);
    if (tid < p.nseg) segs[tid] = p.seg[tid];
    __syncthreads();
    grid_launch_dependents();

    if (warp == kWarps) {
        // ---- producer: lane r (< 16 NMAT) copies row r of the tile's chunk.
        // Each stage's sources, sizes and byte count are computed before the
        // wait for its slot, so the copies issue as soon as the slot frees. ----
        int s = 0;
        uint32_t ph = 0;
        int tile = blockIdx.x, ch = 0;
        while (tile < p.tiles) {
            const TileInfo ti = tile_of(segs, p.nseg, tile);
            const Seg& sg = segs[ti.seg];
            const Geo& ge = p.geo[(F == F2 || sg.type == F) ? 0 : 1];
            const int sb0 = ch * ge.c, nsb = min(ge.c, p.nb - sb0);
            const uint32_t rb = (uint32_t)(nsb * ge.bb);
            const uint32_t tx = (uint32_t)(NMAT * ti.rows) * (rb + ge.db);
            const int m = lane / kRows, r = lane % kRows;
            const bool copies = lane < NMAT * kRows && r < ti.rows;
            const uint8_t* src = (m ? sg.w_up : sg.w) + (size_t)(ti.row0 + r) * sg.stride;
            const int dst_off = (m * kRows + r) * ge.rs;
            const int db = ge.db, dpos = ge.c * ge.bb;
            const uint8_t* dsrc = src + (size_t)p.nb * ge.bb;
            src += (size_t)sb0 * ge.bb;
            if (++ch == ge.chunks) {
                ch = 0;
                tile += gridDim.x;
            }
            // the whole warp waits: a wait by one elected lane while the
            // others sit in __syncwarp() measured 2.5x slower hand-offs
            int ok = !*abort_flag && mbar_wait(&empty[s], ph ^ 1u);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok && lane == 0) {
                if (!*abort_flag) {
                    atomicExch(&g_gemv_mma_error, 4);
                    *abort_flag = 1;
                }
            }
            if (ok) {
                if (lane == 0) mbar_arrive_expect_tx(&full[s], tx);
                __syncwarp();
                if (copies) {
                    uint8_t* dst = stages + (size_t)s * p.stage_bytes + dst_off;
                    bulk_g2s(dst, src, rb, &full[s]);
                    if (db) bulk_g2s(dst + dpos, dsrc, db, &full[s]);
                }
            }
            __syncwarp();
            if (++s == NS) {
                s = 0;
                ph ^= 1u;
            }
        }
        return;
    }

    // ---- consumers: x -> XQ4 in shared memory (RMS-normalised first if asked).
    // Warp w takes blocks w, w + 16, ...; all of its x loads are issued at
    // once and held in registers for both passes (one dependent load per
    // block measured ~1 us each at K = 18944). ----
    grid_wait();
    const int nb = p.nb;
    float xv[kMaxBlocksPerWarp][8];
#pragma unroll
    for (int i = 0; i < kMaxBlocksPerWarp; ++i) {
        const int b = warp + i * kWarps;
        if (b < nb) {
            const float4* px = reinterpret_cast<const float4*>(p.x + b * 256 + lane * 8);
            const float4 u0 = px[0], u1 = px[1];
            xv[i][0] = u0.x; xv[i][1] = u0.y; xv[i][2] = u0.z; xv[i][3] = u0.w;
            xv[i][4] = u1.x; xv[i][5] = u1.y; xv[i][6] = u1.z; xv[i][7] = u1.w;
        }
    }
    float inv = 1.0f;
    if (p.gamma) {
        // cpu_llm.cpp:156-165: sum of squares in double, mean -> float,
        // inv = 1/sqrt(mean + eps) in float, x * (inv * gamma).  Every CTA
        // reduces in the same order, so all CTAs see the same inv.
        double ss = 0.0;
#pragma unroll
        for (int i = 0; i < kMaxBlocksPerWarp; ++i)
            if (warp + i * kWarps < nb) {
#pragma unroll
                for (int e = 0; e < 8; ++e) ss += (double)xv[i][e] * (double)xv[i][e];
            }
        ss = warp_sum_d(ss);
        if (lane == 0) dred[warp] = ss;
        named_barrier(1, kWarps * 32);
        double tot = 0.0;
        for (int w = 0; w < kWarps; ++w) tot += dred[w];
        inv = 1.0f / sqrtf((float)(tot / (double)p.k) + p.eps);
    }
#pragma unroll
    for (int i = 0; i < kMaxBlocksPerWarp; ++i) {
        const int b = warp + i * kWarps;
        if (b < nb) {
            if (p.gamma) {
                const float4* pg = reinterpret_cast<const float4*>(p.gamma + b * 256 + lane * 8);
                const float4 q0 = pg[0], q1 = pg[1];
                const float gm[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) xv[i][e] = __fmul_rn(xv[i][e], __fmul_rn(inv, gm[e]));
            }
            encode_block<HAS_Q4, HAS_Q6>(xv[i], lane, xq + (size_t)b * 1024, xs + b, xsum + b * 8, xn + b * 64);
        }
    }
    named_barrier(1, kWarps * 32);

    // ---- main loop ----
    const int g = lane >> 2, t = lane & 3, h = t >> 1;
    Q4Lane L;
    L.sh = 12u * (uint32_t)h;
    L.lw0 = ((t & 1) ? (1.0f / 16384.0f) : 1.0f) * (h ? (1.0f / 16.0f) : 1.0f);
    L.lw1 = L.lw0 * (1.0f / 128.0f);
    L.pp = t & 1;
    // B words: columns 0-3 (g < 4) read the low unit, columns 4-7 the high
    // unit; the other half reads the zero block.
    const uint8_t* xb0 = g < 4 ? xq + g * 32 + 8 * t : zero;
    const uint8_t* xb1 = g >= 4 ? xq + 128 + (g - 4) * 32 + 8 * t : zero;
    const int xinc0 = g < 4 ? 1024 : 0, xinc1 = g >= 4 ? 1024 : 0;
    // Q6_K: columns 0-3 read unit 4 hh + j, columns 4-7 unit 4 hh + j + 2
    const uint8_t* xb0q6 = g < 4 ? xq + g * 32 + 4 * t : zero;
    const uint8_t* xb1q6 = g >= 4 ? xq + 256 + (g - 4) * 32 + 4 * t : zero;
    Q4Lane L6 = L;  // Q6_K: no 1/16 factor on the high half
    L6.lw0 = (t & 1) ? (1.0f / 16384.0f) : 1.0f;
    L6.lw1 = L6.lw0 * (1.0f / 128.0f);

    int s = 0, base = 0, slot = 0;
    uint32_t ph = 0;
    for (int tile = blockIdx.x; tile < p.tiles; tile += gridDim.x) {
        const TileInfo ti = tile_of(segs, p.nseg, tile);
        const Seg& sg = segs[ti.seg];
        const Geo& ge = p.geo[(F == F2 || sg.type == F) ? 0 : 1];
        float yg = 0.f, y8 = 0.f, ym = 0.f, ug = 0.f, u8 = 0.f, um = 0.f;
        for (int ch = 0; ch < ge.chunks; ++ch) {
            const int sb0 = ch * ge.c, nsb = min(ge.c, nb - sb0);
            int ok = !*abort_flag && mbar_wait(&full[s], ph);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok && lane == 0) {
                if (!*abort_flag) {
                    atomicExch(&g_gemv_mma_error, 5);
                    *abort_flag = 1;
                }
            }
            if (ok) {
                const uint8_t* st = stages + (size_t)s * p.stage_bytes;
                int j = warp - base;
                if (j < 0) j += kWarps;
                const bool q4 = F == F2 ? F == CL_TYPE_Q4_K : sg.type == CL_TYPE_Q4_K;
                for (; j < nsb; j += kWarps) {
                    const int sb = sb0 + j;
                    const float xsb = xs[sb];
                    const uint8_t* rg = st + (size_t)g * ge.rs + j * ge.bb;
                    const uint8_t* r8 = rg + 8 * ge.rs;
                    if (HAS_Q4 && q4) {
                        uint2 bx0[4], bx1[4];
                        const uint8_t* p0 = xb0 + sb * xinc0;
                        const uint8_t* p1 = xb1 + sb * xinc1;
#pragma unroll
                        for (int gi = 0; gi < 4; ++gi) {
                            bx0[gi] = *reinterpret_cast<const uint2*>(p0 + 256 * gi);
                            bx1[gi] = *reinterpret_cast<const uint2*>(p1 + 256 * gi);
                        }
                        const float4 xsum4 = *reinterpret_cast<const float4*>(xsum + sb * 8 + h * 4);
                        q4k_sb(rg, r8, bx0, bx1, xsum4, xsb, t, L, yg, y8, ym);
                        if (SW)
                            q4k_sb(rg + kRows * ge.rs, r8 + kRows * ge.rs, bx0, bx1, xsum4, xsb, t, L, ug, u8, um);
                    } else if (HAS_Q6) {
                        // B words: MMA m = 4 hh + 2 j + s reads 4 bytes at 16 s + 4 t of unit
                        // 4 hh + j (columns 0-3) or 4 hh + j + 2 (columns 4-7), limb g & 3
                        uint32_t bx0[8], bx1[8];
                        int2 xnl[8];
                        const uint8_t* p0 = xb0q6 + sb * xinc0;
                        const uint8_t* p1 = xb1q6 + sb * xinc1;
#pragma unroll
                        for (int m = 0; m < 8; ++m) {
                            const int hh = m >> 2, jj = (m >> 1) & 1, ss = m & 1;
                            bx0[m] = *reinterpret_cast<const uint32_t*>(p0 + 512 * hh + 128 * jj + 16 * ss);
                            bx1[m] = *reinterpret_cast<const uint32_t*>(p1 + 512 * hh + 128 * jj + 16 * ss);
                            // the lane's sub-block (quarter jj + 2h, half ss) and limb pair
                            const int sbi = 8 * hh + 2 * (jj + 2 * h) + ss;
                            xnl[m] = *reinterpret_cast<const int2*>(xn + sb * 64 + sbi * 4 + 2 * (t & 1));
                        }
                        const uint8_t* dcol = st + (size_t)ge.c * ge.bb + 2 * sb;
                        const float dg = half_bits_to_float(*reinterpret_cast<const unsigned short*>(dcol + (size_t)g * ge.rs));
                        const float d8 = half_bits_to_float(*reinterpret_cast<const unsigned short*>(dcol + (size_t)(g + 8) * ge.rs));
                        q6k_sb(rg, r8, bx0, bx1, xnl, xsb, t, dg, d8, L6, yg, y8);
                        if (SW) {
                            const float ug0 = half_bits_to_float(*reinterpret_cast<const unsigned short*>(dcol + (size_t)(kRows + g) * ge.rs));
                            const float u80 = half_bits_to_float(*reinterpret_cast<const unsigned short*>(dcol + (size_t)(kRows + g + 8) * ge.rs));
                            q6k_sb(rg + kRows * ge.rs, r8 + kRows * ge.rs, bx0, bx1, xnl, xsb, t, ug0, u80, L6, ug, u8);
                        }
                    }
                }
            }
            base += nsb;
            base %= kWarps;
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (++s == NS) {
                s = 0;
                ph ^= 1u;
            }
        }
        // ---- end of tile: quad sums, then warp 0 adds the warps' rows ----
        if (L.pp) y8 += ym; else yg += ym;
        yg += __shfl_xor_sync(0xffffffffu, yg, 1);
        yg += __shfl_xor_sync(0xffffffffu, yg, 2);
        y8 += __shfl_xor_sync(0xffffffffu, y8, 1);
        y8 += __shfl_xor_sync(0xffffffffu, y8, 2);
        if (SW) {
            if (L.pp) u8 += um; else ug += um;
            ug += __shfl_xor_sync(0xffffffffu, ug, 1);
            ug += __shfl_xor_sync(0xffffffffu, ug, 2);
            u8 += __shfl_xor_sync(0xffffffffu, u8, 1);
            u8 += __shfl_xor_sync(0xffffffffu, u8, 2);
        }
        // publish this warp's rows; the last warp to finish the tile sums
        // all warps' rows in warp order and writes the outputs
        float* rb = red + (size_t)slot * red_floats(NMAT);
        if (t == 0) {
            rb[warp * kRows * NMAT + g] = yg;
            rb[warp * kRows * NMAT + g + 8] = y8;
            if (SW) {
                rb[warp * kRows * NMAT + kRows + g] = ug;
                rb[warp * kRows * NMAT + kRows + g + 8] = u8;
            }
        }
        __syncwarp();
        int last = 0;
        if (lane == 0) {
            __threadfence_block();
            last = atomicAdd(&tickets[slot], 1) == kWarps - 1;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
            __threadfence_block();
            if (lane < ti.rows && !*abort_flag) {
                float y = 0.0f, up = 0.0f;
#pragma unroll
                for (int w = 0; w < kWarps; ++w) {
                    y += rb[w * kRows * NMAT + lane];
                    if (SW) up += rb[w * kRows * NMAT + kRows + lane];
                }
                const int o = ti.row0 + lane;
                if (SW) {
                    // Branch-stable SiLU(g) * u (cpu_llm.cpp:188-202).
                    const float sig = y >= 0.0f ? 1.0f / (1.0f + expf(-y)) : expf(y) / (1.0f + expf(y));
                    y = __fmul_rn(__fmul_rn(y, sig), up);
                } else {
                    if (sg.bias) y += sg.bias[o];
                    if (sg.residual) y = sg.residual[o] + y;
                }
                sg.y[o] = y;
            }
            if (lane == 0) tickets[slot] = 0;
            __syncwarp();
        }
        if (++slot > NS) slot = 0;
    }
}

// ---- host side ------------------------------------------------------------------

constexpr int kSmemMax = 227 * 1024;
// Measured on B200: large stages (whole 16-row tiles where they fit) stream
// far better than chunked rows; per-stage hand-off costs dominate below ~32 KB.
constexpr int kStageTarget = 72 * 1024;

bool type_ok(int t) { return t == CL_TYPE_Q4_K || t == CL_TYPE_Q6_K; }

int block_bytes(int type) { return type == CL_TYPE_Q4_K ? 144 : 208; }

// Row stride in a stage for conflict-free fragment reads: Q4_K reads 8 bytes
// per lane (4 lanes per row, 4 rows per half-warp phase) -> stride / 32 odd;
// Q6_K reads 4 bytes per lane (4 lanes per row, 8 rows per access) ->
// stride / 16 odd.
int stage_row_stride(int type, int bytes) {
    int rs = (bytes + 15) & ~15;
    if (type == CL_TYPE_Q4_K)
        while (rs % 64 != 32) rs += 16;
    else
        while (rs % 32 != 16) rs += 16;
    return rs;
}

// Stage geometry: whole rows per stage when 16 of them fit the target, else
// the fewest equal chunks that do.  `limit` caps the stage bytes.
Geo make_geo(int type, int nb, int nmat, int limit) {
    Geo g{};
    g.bb = block_bytes(type);
    g.db = type == CL_TYPE_Q6_K ? ((2 * nb + 15) & ~15) : 0;
    g.chunks = 1;
    for (;;) {
        g.c = (nb + g.chunks - 1) / g.chunks;
        g.rs = stage_row_stride(type, g.c * g.bb + g.db);
        if (nmat * kRows * g.rs <= limit || g.c == 1) break;
        ++g.chunks;
    }
    return g;
}

template <int F, bool SW, int F2>
cudaError_t launch_cfg(const Params& p, int smem, cudaStream_t stream) {
    auto kern = gemv_mma_kernel<F, SW, F2>;
    static SmemLimit limit;
    cudaError_t e = limit.ensure(kern, kSmemMax);
    if (e != cudaSuccess) return e;
    int sm_count = 0;
    if ((e = device_sm_count(&sm_count)) != cudaSuccess) return e;
    const int grid = std::min(p.tiles, sm_count);
    return launch_pdl(kern, dim3(grid), dim3(kThreads), (size_t)smem, stream, p);
}

}  // namespace gmma

// Launch over 1-4 segments of one K-quant type sharing x (optionally
// RMS-normalised by gamma; SwiGLU over (w, w_up) when w_up is given).
// Returns CL_ERR_UNSUPPORTED for shapes this kernel does not take.
int launch_gemv_mma(const cl_gemv_segment* segs, int nseg, int k, const float* x, const float* gamma, float eps,
                    const void* w_up, cudaStream_t stream) {
    using namespace gmma;
    const bool sw = w_up != nullptr;
    const int nmat = sw ? 2 : 1;
    if (nseg < 1 || nseg > kMaxSegs || k <= 0 || k % 256 != 0 || k / 256 > kWarps * kMaxBlocksPerWarp)
        return CL_ERR_UNSUPPORTED;
    // one type, or the fused pair Q4_K + Q6_K (the Q4_K_M attention projections)
    int ta = segs[0].type, tb = segs[0].type;
    for (int i = 0; i < nseg; ++i) {
        if (!type_ok(segs[i].type)) return CL_ERR_UNSUPPORTED;
        if (segs[i].type != ta) tb = segs[i].type;
    }
    if (sw && ta != tb) return CL_ERR_UNSUPPORTED;
    const bool has4 = ta == CL_TYPE_Q4_K || tb == CL_TYPE_Q4_K;
    const bool has6 = ta == CL_TYPE_Q6_K || tb == CL_TYPE_Q6_K;
    Params p{};
    p.nb = k / 256;
    p.k = k;
    int tiles = 0;
    for (int i = 0; i < nseg; ++i) {
        Seg& s = p.seg[i];
        s.w = static_cast<const uint8_t*>(segs[i].w);
        s.w_up = static_cast<const uint8_t*>(w_up);
        s.stride = segs[i].stride;
        s.bias = segs[i].bias;
        s.residual = segs[i].residual;
        s.y = segs[i].y;
        s.type = segs[i].type;
        s.n = segs[i].n;
        s.tile_begin = tiles;
        tiles += (segs[i].n + kRows - 1) / kRows;
    }
    p.nseg = nseg;
    p.tiles = tiles;
    p.x = x;
    p.gamma = gamma;
    p.eps = eps;
    // layout: fixed | xs | xsum (Q4_K) | xn (Q6_K) | xq | stages
    auto layout = [&](int ns) {
        int off = fixed_bytes(ns, nmat);
        p.off_xs = off;
        off += (4 * p.nb + 15) & ~15;
        p.off_xsum = off;
        off += has4 ? 32 * p.nb : 0;
        p.off_xn = off;
        off += has6 ? 256 * p.nb : 0;
        p.off_xq = (off + 127) & ~127;
        off = p.off_xq + 1024 * p.nb;
        p.off_stage = (off + 127) & ~127;
        return p.off_stage + ns * p.stage_bytes;
    };
    // Stages as large as possible (whole tiles), at least two of them.
    const int room = kSmemMax - layout(0);
    const int limit = std::min(kStageTarget, room / 2);
    p.geo[0] = make_geo(has4 ? CL_TYPE_Q4_K : CL_TYPE_Q6_K, p.nb, nmat, limit);
    p.geo[1] = make_geo(has6 ? CL_TYPE_Q6_K : CL_TYPE_Q4_K, p.nb, nmat, limit);
    p.stage_bytes = nmat * kRows * std::max(p.geo[0].rs, p.geo[1].rs);
    int ns = 8;
    while (ns > 2 && layout(ns) > kSmemMax) --ns;
    const int smem = layout(ns);
    if (smem > kSmemMax) return CL_ERR_UNSUPPORTED;
    p.stages = ns;
    cudaError_t e;
    if (has4 && has6)
        e = launch_cfg<CL_TYPE_Q4_K, false, CL_TYPE_Q6_K>(p, smem, stream);
    else if (has4)
        e = sw ? launch_cfg<CL_TYPE_Q4_K, true, CL_TYPE_Q4_K>(p, smem, stream)
               : launch_cfg<CL_TYPE_Q4_K, false, CL_TYPE_Q4_K>(p, smem, stream);
    else
        e = sw ? launch_cfg<CL_TYPE_Q6_K, true, CL_TYPE_Q6_K>(p, smem, stream)
               : launch_cfg<CL_TYPE_Q6_K, false, CL_TYPE_Q6_K>(p, smem, stream);
    return e == cudaSuccess ? CL_OK : CL_ERR_CUDA;
}

int gemv_mma_device_error(int* code, bool clear) {
    if (cudaMemcpyFromSymbol(code, g_gemv_mma_error, sizeof(int)) != cudaSuccess) return CL_ERR_CUDA;
    if (clear) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_gemv_mma_error, &zero, sizeof(int)) != cudaSuccess) return CL_ERR_CUDA;
    }
    return CL_OK;
}

}  // namespace cl
