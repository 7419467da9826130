// Decode GEMV over K-quant weights in the fragment-packed layout, loaded
// straight into the tensor-core operand registers (no shared-memory ring).
//
// Reference: metal_gevm_q4_k_f32 / metal_gevm_q6_k_f32 (metal_llm.metal:708-781)
// and the CPU oracle gevmt over GgufDequantizer rows (cpu_llm.cpp:512-547,
// model.cpp:581-683).  Same products as gemv_mma.cu: the weight integers are
// dotted exactly with the XQ4 limbs of x on mma.sync (u8 x s8 for Q4_K, s8 x
// s8 with q - 32 for Q6_K), and only per-super-block sums are scaled in FP32.
//
// Why this kernel (measured on B200): the shared-memory ring kernels (bulk
// copies, or per-warp cp.async rings in the one-launch step) never waited on
// their rings; they were bound by the consumer warps' issue and latency, with
// 8-17 warps per SM, and streamed the 7B gate/up matrix at ~3.8-4.0 TB/s.
// Here every lane loads its own MMA fragments with 16-byte non-caching loads:
//
// * Packed layout (cl_gemv_pack): a unit is 16 rows x one super-block,
//   contiguous.  Its first 4 (Q4_K) or 6 (Q6_K) 512-byte chunks hold, at
//   16 * lane, exactly the 16 bytes lane (g = lane / 4, t = lane % 4) feeds
//   to the MMAs of row g or g + 8; then the rows' headers (Q4_K: 16 x 16 B)
//   or scales and d (Q6_K).  One unit = 6 (Q4_K) or 8 (Q6_K) loads per lane,
//   each a whole 512-byte (or 128-byte) segment across the warp.
// * Each CTA owns a contiguous range of whole tiles (stream-K over units,
//   with shared tiles finished through a workspace, only when a launch has
//   fewer tiles than CTAs); its 12 warps split the range into equal
//   contiguous unit ranges and keep three units in registers each: the one
//   computed and the next two in flight.  Tiles split between warps are
//   summed in shared memory in warp order (deterministic).
// * Weights are immutable, so the first two units are requested before the
//   programmatic-dependent-launch wait; x is read and encoded (every CTA, in
//   shared memory, RMS-normalised first where asked) after it.
// * SwiGLU: a pair unit holds 8 gate rows (g) and the same 8 up rows (g + 8),
//   so gate and up of one output row meet in one lane.
//
// Measured (B200, CUDA-graph launches, weights rotating beyond L2): the 7B
// LM head (447 MB Q6_K) in 84-88 us (5.1-5.3 TB/s) against 111 us for the
// ring kernel; the in-loop stream reaches 4.9-5.7 TB/s.  But every launch
// pays ~2 us waiting for the previous grid, 2.4 us (k = 3584) to 8 us
// (k = 18944) encoding x in every CTA, and the tail of its CTAs, so a 7B
// layer's QKV, o_proj, gate/up and down are all slower than on the ring
// kernels, whose producers prefetch ~190 KB of weights per SM across the
// wait.  The decode graph therefore uses this kernel for the LM head only.
#include "common.cuh"
#include "gemv_mma.cuh"
#include "launch.cuh"

namespace cl {

namespace gpk {

using gmma::Q4Lane;

constexpr int kW = 12;  // warps per CTA
constexpr int kThreads = kW * 32;
constexpr int kMaxSegs = 4;
constexpr int kMaxBlocksPerWarp = 7;  // x blocks a warp encodes: k <= 12 * 7 * 256
constexpr int kZeroBytes = 1024;
constexpr int kQ4Unit = 2304;         // 16 x 144
constexpr int kQ6Unit = 3360;         // 16 x 210

struct Seg {
    const uint8_t* w;  // packed units, tile by tile
    const float* bias;
    const float* residual;
    float* y;
    long long u0;  // first unit of the segment in the launch
    int tile0;     // first tile of the segment in the launch
    int tiles;
    int type;
    int n;  // output rows
};

struct Params {
    Seg seg[kMaxSegs];
    const float* x;
    const float* gamma;  // RMSNorm weight applied to x first (cpu_llm.cpp:143-166), or null
    float* partials;     // [grid][2][16]
    unsigned int* tickets;  // [tiles], zero between launches
    long long U;         // units in the launch
    float eps;
    int nseg, k, nb, swiglu;
    int whole_tiles;     // 1: each CTA owns whole tiles (no tile is shared between CTAs)
};

// One unit's operand registers: Q4_K a[0..3] = qs chunks (rows g / g + 8,
// groups 0-1 / 2-3), a[4] / a[5] = headers of rows g / g + 8; Q6_K a[0..5] =
// ql (hh 0, 1) and qh of row g, then of row g + 8, s = the lane's 8 scale
// bytes of rows g and g + 8, d = f16 d of rows g (low) and g + 8 (high).
struct Buf {
    uint4 a[6];
    uint4 s;
    uint32_t d;
};

CL_DEVINL uint4 ldg_stream(const void* p, uint64_t policy) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p), "l"(policy));
    return v;
}
CL_DEVINL uint64_t evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

CL_DEVINL int unit_bytes(int type) { return type == CL_TYPE_Q4_K ? kQ4Unit : kQ6Unit; }

// XQ4 vector of nb 256-element blocks as the kernel keeps it in shared
// memory: limbs [nb][8 units][4 limbs][32 B],
// scales xs[nb] (padded to a multiple of 4), unit sums xsum[nb][2][4].
__host__ __device__ inline size_t xq4_bytes(int nb) {
    return (size_t)nb * 1024 + 4 * (size_t)((nb + 3) & ~3) + 32 * (size_t)nb;
}


CL_DEVINL void load_unit(Buf& b, const uint8_t* base, bool q4, int lane, int g, int h, uint64_t pol) {
    const uint8_t* p = base + 16 * lane;
    if (q4) {
        b.a[0] = ldg_stream(p, pol);
        b.a[1] = ldg_stream(p + 512, pol);
        b.a[2] = ldg_stream(p + 1024, pol);
        b.a[3] = ldg_stream(p + 1536, pol);
        b.a[4] = ldg_stream(base + 2048 + 16 * g, pol);
        b.a[5] = ldg_stream(base + 2048 + 16 * (g + 8), pol);
    } else {
#pragma unroll
        for (int c = 0; c < 6; ++c) b.a[c] = ldg_stream(p + 512 * c, pol);
        b.s = ldg_stream(base + 3072 + 16 * (2 * g + h), pol);
        b.d = ldg_nc_u32(base + 3328 + 4 * g);
    }
}

CL_DEVINL uint32_t word(const uint4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// One Q4_K unit (16 rows x 1 super-block) from registers; bx0/bx1, xsum4, xs
// as in gmma::q4k_sb.
CL_DEVINL void q4_unit(const Buf& b, const uint2 (&bx0)[4], const uint2 (&bx1)[4], const float4& xsum4, float xs,
                       const Q4Lane& L, float& yg, float& y8, float& ym) {
    using namespace gmma;
    const uint4 hg = b.a[4], h8 = b.a[5];
    const uint32_t g1 = __funnelshift_r(hg.y, hg.z, L.sh), g2 = __funnelshift_r(hg.z, hg.w, L.sh), g3 = hg.w >> L.sh;
    const uint32_t e1 = __funnelshift_r(h8.y, h8.z, L.sh), e2 = __funnelshift_r(h8.z, h8.w, L.sh), e3 = h8.w >> L.sh;
    int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
    for (int gi = 0; gi < 4; ++gi) {
        const uint4& cg = b.a[gi >> 1];
        const uint4& c8 = b.a[2 + (gi >> 1)];
        const uint32_t wgx = (gi & 1) ? cg.z : cg.x, wgy = (gi & 1) ? cg.w : cg.y;
        const uint32_t w8x = (gi & 1) ? c8.z : c8.x, w8y = (gi & 1) ? c8.w : c8.y;
        int c[4];
        mma_u8s8_z(c, wgx & 0x0f0f0f0fu, w8x & 0x0f0f0f0fu, wgx & 0xf0f0f0f0u, w8x & 0xf0f0f0f0u, bx0[gi].x,
                   bx1[gi].x);
        mma_u8s8(c, wgy & 0x0f0f0f0fu, w8y & 0x0f0f0f0fu, wgy & 0xf0f0f0f0u, w8y & 0xf0f0f0f0u, bx0[gi].y, bx1[gi].y);
        int sg, s8;
        switch (gi) {
            case 0: sg = q4_sc<0>(g1, g2, g3); s8 = q4_sc<0>(e1, e2, e3); break;
            case 1: sg = q4_sc<1>(g1, g2, g3); s8 = q4_sc<1>(e1, e2, e3); break;
            case 2: sg = q4_sc<2>(g1, g2, g3); s8 = q4_sc<2>(e1, e2, e3); break;
            default: sg = q4_sc<3>(g1, g2, g3); s8 = q4_sc<3>(e1, e2, e3); break;
        }
        a0 += c[0] * sg;
        a1 += c[1] * sg;
        a2 += c[2] * s8;
        a3 += c[3] * s8;
    }
    const uint32_t m1 = L.pp ? e1 : g1, m2 = L.pp ? e2 : g2, m3 = L.pp ? e3 : g3;
    const float msum = fmaf(q4_m<0>(m1, m2, m3), xsum4.x,
                            fmaf(q4_m<1>(m1, m2, m3), xsum4.y,
                                 fmaf(q4_m<2>(m1, m2, m3), xsum4.z, q4_m<3>(m1, m2, m3) * xsum4.w)));
    const float dmin = half_bits_to_float((L.pp ? h8.x : hg.x) >> 16);
    ym = fmaf(-dmin, msum, ym);
    const float vg = fmaf((float)a0, L.lw0, (float)a1 * L.lw1) * xs;
    const float v8 = fmaf((float)a2, L.lw0, (float)a3 * L.lw1) * xs;
    yg = fmaf(half_bits_to_float(hg.x), vg, yg);
    y8 = fmaf(half_bits_to_float(h8.x), v8, y8);
}

// Q6_K value bytes v in [0, 63] -> v - 32 as signed bytes, four at a time.
CL_DEVINL uint32_t q6_signed(uint32_t v) { return ((v | 0x80808080u) - 0x20202020u) ^ 0x80808080u; }

// One Q6_K unit (16 rows x 1 super-block) from registers.  MMA (hh, j, s):
// K slots 0-15 = element 16 s + l of quarter j of half hh (B columns 0-3,
// limbs of unit 4 hh + j), slots 16-31 = the same position in quarter j + 2
// (columns 4-7, unit 4 hh + j + 2); p0 / p1: the lane's B bases in the XQ4
// block (the zero block for the other column half).
CL_DEVINL void q6_unit(const Buf& b, const uint8_t* p0, const uint8_t* p1, float xs, const Q4Lane& L6, float& yg,
                       float& y8) {
    int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
    const uint32_t sgl = b.s.x, sgh = b.s.y, s8l = b.s.z, s8h = b.s.w;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
        for (int s = 0; s < 2; ++s) {
            const uint32_t qg = word(b.a[2], 2 * hh + s), q8 = word(b.a[5], 2 * hh + s);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const uint32_t lg = word(b.a[hh], 2 * j + s), l8 = word(b.a[3 + hh], 2 * j + s);
                const uint32_t hag = (j ? (qg << 2) : (qg << 4)) & 0x30303030u;
                const uint32_t ha8 = (j ? (q8 << 2) : (q8 << 4)) & 0x30303030u;
                const uint32_t hbg = (j ? (qg >> 2) : qg) & 0x30303030u;
                const uint32_t hb8 = (j ? (q8 >> 2) : q8) & 0x30303030u;
                const int boff = 512 * hh + 128 * j + 16 * s;
                const uint32_t b0 = *reinterpret_cast<const uint32_t*>(p0 + boff);
                const uint32_t b1 = *reinterpret_cast<const uint32_t*>(p1 + boff);
                int c[4];
                gmma::mma_s8s8_z(c, q6_signed((lg & 0x0f0f0f0fu) | hag), q6_signed((l8 & 0x0f0f0f0fu) | ha8),
                                 q6_signed(((lg >> 4) & 0x0f0f0f0fu) | hbg),
                                 q6_signed(((l8 >> 4) & 0x0f0f0f0fu) | hb8), b0, b1);
                // scale byte mi = 4 hh + 2 j + s of the lane's eight
                const int mi = 4 * hh + 2 * j + s;
                const uint32_t wg = mi < 4 ? sgl : sgh, w8 = mi < 4 ? s8l : s8h;
                const int sg = (int)(int8_t)(uint8_t)(wg >> (8 * (mi & 3)));
                const int s8 = (int)(int8_t)(uint8_t)(w8 >> (8 * (mi & 3)));
                a0 += c[0] * sg;
                a1 += c[1] * sg;
                a2 += c[2] * s8;
                a3 += c[3] * s8;
            }
        }
    }
    const float vg = fmaf((float)a0, L6.lw0, (float)a1 * L6.lw1) * xs;
    const float v8 = fmaf((float)a2, L6.lw0, (float)a3 * L6.lw1) * xs;
    yg = fmaf(half_bits_to_float(b.d), vg, yg);
    y8 = fmaf(half_bits_to_float(b.d >> 16), v8, y8);
}

// Range [begin(w), begin(w + 1)) of the grid's warp w over U units, and the
// warp whose range holds unit u.
CL_DEVINL long long range_begin(long long U, int w, int GW) { return U * w / GW; }
CL_DEVINL int warp_of(long long U, long long u, int GW) { return (int)(((u + 1) * GW - 1) / U); }

// Unit cursor: segment, tile in the segment, super-block.
struct Cursor {
    int s, tile, j;
};

CL_DEVINL Cursor cursor_at(const Seg* segs, int nseg, int nb, int u) {
    int s = 0;
#pragma unroll
    for (int i = 1; i < kMaxSegs; ++i)
        if (i < nseg && u >= segs[i].u0) s = i;
    const int r = u - (int)segs[s].u0;
    return Cursor{s, r / nb, r % nb};
}

CL_DEVINL void cursor_next(const Seg* segs, int nb, Cursor& c) {
    if (++c.j == nb) {
        c.j = 0;
        if (++c.tile == segs[c.s].tiles) {
            c.tile = 0;
            ++c.s;
        }
    }
}

// Output rows of a finished tile: lanes 0-7 (SwiGLU: one output row each,
// gate in yv, up in uv) or lanes 0-15 (one row each, in yv).
CL_DEVINL void write_rows(const Seg& sg, int tile, int swiglu, int r, float yv, float uv) {
    if (swiglu) {
        const int o = 8 * tile + r;
        if (r < 8 && o < sg.n) {
            // Branch-stable SiLU(g) * u (cpu_llm.cpp:188-202).
            const float sig = yv >= 0.0f ? 1.0f / (1.0f + expf(-yv)) : expf(yv) / (1.0f + expf(yv));
            sg.y[o] = __fmul_rn(__fmul_rn(yv, sig), uv);
        }
    } else {
        const int o = 16 * tile + r;
        if (r < 16 && o < sg.n) {
            float y = yv;
            if (sg.bias) y += sg.bias[o];
            if (sg.residual) y = sg.residual[o] + y;
            sg.y[o] = y;
        }
    }
}

// Sum of a lane quad's partial rows (lanes t = 0 end with rows g and g + 8).
CL_DEVINL void quad_rows(float& yg, float& y8, float ym, int t) {
    if (t & 1) y8 += ym;
    else yg += ym;
    yg += __shfl_xor_sync(0xffffffffu, yg, 1);
    yg += __shfl_xor_sync(0xffffffffu, yg, 2);
    y8 += __shfl_xor_sync(0xffffffffu, y8, 1);
    y8 += __shfl_xor_sync(0xffffffffu, y8, 2);
}

// A warp's units: up to three contiguous intervals of the launch's unit
// space (its share of the CTA's first shared tile, of its last shared tile,
// and of the tiles the CTA owns), walked in order with the unit's cursor.
// The intervals are read by index through selects, so that they stay in
// registers.
struct Span {
    int b0, e0, b1, e1, b2, e2;
    CL_DEVINL int b(int k) const { return k == 0 ? b0 : k == 1 ? b1 : b2; }
    CL_DEVINL int e(int k) const { return k == 0 ? e0 : k == 1 ? e1 : e2; }
};

struct Walk {
    int k, u;
    Cursor c;
};

CL_DEVINL void walk_seek(Walk& w, const Span& sp, const Seg* segs, int nseg, int nb) {
    while (w.k < 3 && sp.b(w.k) >= sp.e(w.k)) ++w.k;
    if (w.k < 3) {
        w.u = sp.b(w.k);
        w.c = cursor_at(segs, nseg, nb, w.u);
    }
}

CL_DEVINL void walk_next(Walk& w, const Span& sp, const Seg* segs, int nseg, int nb) {
    if (++w.u < sp.e(w.k)) {
        cursor_next(segs, nb, w.c);
    } else {
        ++w.k;
        walk_seek(w, sp, segs, nseg, nb);
    }
}

// The CTA's partial rows of a tile it shares with other CTAs are in `gpart`
// slot (cta, slot) and visible; take the tile's ticket, and the last of the
// sharing CTAs adds all their partials in CTA order and writes the rows.
// One warp; rows in lanes 0-15.
CL_DEVINL void finish_cta_tile(const Params& p, const Seg* segs, long long gt, int G, int lane) {
    const int nb = p.nb;
    const long long ub = gt * nb, ue = ub + nb;
    const int c0 = warp_of(p.U, ub, G), c1 = warp_of(p.U, ue - 1, G);
    int last = 0;
    if (lane == 0) {
        last = atomicAdd(&p.tickets[gt], 1u) == (unsigned int)(c1 - c0);
        if (last) __threadfence();
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    float acc = 0.0f;
    if (lane < 16) {
        // CTA c0's range may begin before the tile (then the tile is its slot 1)
        const int s0 = range_begin(p.U, c0, G) < ub ? 1 : 0;
        acc = __ldcg(p.partials + ((size_t)c0 * 2 + s0) * 16 + lane);
        for (int c = c0 + 1; c <= c1; ++c) acc += __ldcg(p.partials + (size_t)c * 32 + lane);
    }
    const float up = __shfl_down_sync(0xffffffffu, acc, 8);
    int s = 0;
#pragma unroll
    for (int i = 1; i < kMaxSegs; ++i)
        if (i < p.nseg && gt >= segs[i].tile0) s = i;
    write_rows(segs[s], (int)(gt - segs[s].tile0), p.swiglu, lane, acc, up);
    if (lane == 0) p.tickets[gt] = 0u;
}

// Work split.  With at least as many tiles as CTAs, each CTA owns a
// contiguous range of whole tiles.  Otherwise (stream-K) the launch's units
// (16-row tile x super-block, tile by tile) are cut into equal contiguous
// ranges, one per CTA; a CTA's first and last tile may then be shared with
// neighbouring CTAs (measured: the cross-CTA finish below costs ~4 us of
// tail latency per launch, more than the imbalance of whole tiles); their units are
// computed first, by all warps, summed in shared memory and published as one
// partial per CTA with a ticket (the last sharing CTA writes the rows) while
// the warps go on to the tiles the CTA owns.  Those are cut into equal
// contiguous ranges per warp; a tile inside one warp's range is written by
// it, a tile split between warps is summed in shared memory at the end.
template <bool HAS4, bool HAS6>
__global__ void __launch_bounds__(kThreads, 1) gemv_pk_kernel(const __grid_constant__ Params p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int nb = p.nb;
    uint8_t* xq = smem;                                                     // [nb][8 units][4 limbs][32]
    float* xs = reinterpret_cast<float*>(smem + (size_t)nb * 1024);       // [nb]
    float* xsum = xs + ((nb + 3) & ~3);                                     // [nb][2][4]
    uint8_t* zero = reinterpret_cast<uint8_t*>(xsum + nb * 8);              // kZeroBytes
    float* red_a = reinterpret_cast<float*>(zero + kZeroBytes);            // [kW][2][16] shared-tile partials
    float* red_b = red_a + kW * 32;                                         // [kW][2][16] owned-tile partials
    double* dred = reinterpret_cast<double*>(red_b + kW * 32);             // [kW]
    Seg* segs = reinterpret_cast<Seg*>(dred + kW);                          // [kMaxSegs]

    // CTAs with work (every range non-empty) and this CTA's unit range
    const long long T = p.U / nb;
    const int G = (int)min((long long)gridDim.x, p.whole_tiles ? T : p.U);
    if ((int)blockIdx.x >= G) return;
    const long long cb = p.whole_tiles ? T * blockIdx.x / G * nb : range_begin(p.U, blockIdx.x, G);
    const long long ce = p.whole_tiles ? T * (blockIdx.x + 1) / G * nb : range_begin(p.U, blockIdx.x + 1, G);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3, h = t >> 1;
    if (tid < kZeroBytes / 16) reinterpret_cast<uint4*>(zero)[tid] = make_uint4(0u, 0u, 0u, 0u);
    for (int i = tid; i < 2 * kW * 32; i += kThreads) red_a[i] = 0.0f;
    if (tid < p.nseg) segs[tid] = p.seg[tid];
    __syncthreads();

    // ---- the CTA's range, its shared tiles and this warp's intervals ----
    const long long tf = cb / nb, tl = (ce - 1) / nb;
    const bool f_shared = cb % nb != 0 || ce < tf * nb + nb;
    const bool l_shared = tl != tf && ce % nb != 0;
    const long long a0b = cb, a0e = f_shared ? min(ce, tf * nb + nb) : cb;  // first tile's units
    const long long a1b = l_shared ? tl * nb : ce, a1e = ce;                 // last tile's units
    const long long ob = a0e, oe = a1b;                                      // owned tiles' units
    const long long nA = (a0e - a0b) + (a1e - a1b), nB = oe - ob;
    Span sp;
    {
        const long long i0 = nA * warp / kW, i1 = nA * (warp + 1) / kW, la = a0e - a0b;
        sp.b0 = (int)(a0b + min(i0, la));
        sp.e0 = (int)(a0b + min(i1, la));
        sp.b1 = (int)(a1b + max(i0 - la, 0ll));
        sp.e1 = (int)(a1b + max(i1 - la, 0ll));
        sp.b2 = (int)(ob + nB * warp / kW);
        sp.e2 = (int)(ob + nB * (warp + 1) / kW);
    }
    Walk wk{0, 0, Cursor{0, 0, 0}};
    walk_seek(wk, sp, segs, p.nseg, nb);
    const long long wb = sp.b2, we = sp.e2;  // this warp's owned range

    // ---- the first two units, before the wait (weights are immutable) ----
    const uint64_t pol = evict_first_policy();
    Walk wi = wk;  // the loader runs ahead of the compute walk
    auto unit_ptr = [&](const Cursor& c) {
        const Seg& sg = segs[c.s];
        return sg.w + ((long long)c.tile * nb + c.j) * unit_bytes(sg.type);
    };
    auto is_q4 = [&](const Cursor& c) { return HAS4 && (!HAS6 || segs[c.s].type == CL_TYPE_Q4_K); };
    Buf B0, B1, B2;
    auto request = [&](Buf& buf) {
        if (wi.k < 3) {
            load_unit(buf, unit_ptr(wi.c), is_q4(wi.c), lane, g, h, pol);
            walk_next(wi, sp, segs, p.nseg, nb);
        }
    };
    request(B0);
    request(B1);
    grid_launch_dependents();

    // ---- x -> XQ4 in shared memory (RMS-normalised first if asked) ----
    grid_wait();
    {
        float xv[kMaxBlocksPerWarp][8];
#pragma unroll
        for (int i = 0; i < kMaxBlocksPerWarp; ++i) {
            const int blk = warp + i * kW;
            if (blk < nb) {
                const float4* px = reinterpret_cast<const float4*>(p.x + blk * 256 + lane * 8);
                const float4 u0 = px[0], u1 = px[1];
                xv[i][0] = u0.x; xv[i][1] = u0.y; xv[i][2] = u0.z; xv[i][3] = u0.w;
                xv[i][4] = u1.x; xv[i][5] = u1.y; xv[i][6] = u1.z; xv[i][7] = u1.w;
            }
        }
        float inv = 1.0f;
        if (p.gamma) {
            // cpu_llm.cpp:156-165: sum of squares in double, mean -> float,
            // inv = 1/sqrt(mean + eps) in float, x * (inv * gamma); every CTA
            // reduces in the same order.
            double ss = 0.0;
#pragma unroll
            for (int i = 0; i < kMaxBlocksPerWarp; ++i)
                if (warp + i * kW < nb) {
#pragma unroll
                    for (int q = 0; q < 8; ++q) ss += (double)xv[i][q] * (double)xv[i][q];
                }
            ss = warp_sum_d(ss);
            if (lane == 0) dred[warp] = ss;
            __syncthreads();
            double tot = 0.0;
            for (int w = 0; w < kW; ++w) tot += dred[w];
            inv = 1.0f / sqrtf((float)(tot / (double)p.k) + p.eps);
        }
#pragma unroll
        for (int i = 0; i < kMaxBlocksPerWarp; ++i) {
            const int blk = warp + i * kW;
            if (blk < nb) {
                if (p.gamma) {
                    const float4* pg = reinterpret_cast<const float4*>(p.gamma + blk * 256 + lane * 8);
                    const float4 q0 = pg[0], q1 = pg[1];
                    const float gm[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                    for (int q = 0; q < 8; ++q) xv[i][q] = __fmul_rn(xv[i][q], __fmul_rn(inv, gm[q]));
                }
                gmma::encode_block<HAS4, false>(xv[i], lane, xq + (size_t)blk * 1024, xs + blk, xsum + blk * 8,
                                                nullptr);
            }
        }
    }
    __syncthreads();
    request(B2);

    Q4Lane L;
    L.sh = 12u * (uint32_t)h;
    L.lw0 = ((t & 1) ? (1.0f / 16384.0f) : 1.0f) * (h ? (1.0f / 16.0f) : 1.0f);
    L.lw1 = L.lw0 * (1.0f / 128.0f);
    L.pp = t & 1;
    Q4Lane L6 = L;
    L6.lw0 = (t & 1) ? (1.0f / 16384.0f) : 1.0f;
    L6.lw1 = L6.lw0 * (1.0f / 128.0f);
    // B bases: Q4_K columns 0-3 (g < 4) read the low unit of a group, 4-7
    // the high unit; Q6_K columns 0-3 unit 4 hh + j, 4-7 unit 4 hh + j + 2
    const uint8_t* xb4_0 = g < 4 ? xq + g * 32 + 8 * t : zero;
    const uint8_t* xb4_1 = g >= 4 ? xq + 128 + (g - 4) * 32 + 8 * t : zero;
    const uint8_t* xb6_0 = g < 4 ? xq + g * 32 + 4 * t : zero;
    const uint8_t* xb6_1 = g >= 4 ? xq + 256 + (g - 4) * 32 + 4 * t : zero;
    const int xinc0 = g < 4 ? 1024 : 0, xinc1 = g >= 4 ? 1024 : 0;

    float yg = 0.0f, y8 = 0.0f, ym = 0.0f;
    bool a_done = false;
    // End of the shared-tile units: their sums meet in shared memory, and
    // warp 0 (first tile) / warp kW - 1 (last tile) publish the CTA's
    // partial and take the ticket while the other warps stream on.
    auto shared_tiles_done = [&]() {
        a_done = true;
        if (!f_shared && !l_shared) return;
        named_barrier(1, kThreads);
        const int which = warp == 0 && f_shared ? 0 : warp == kW - 1 && l_shared ? 1 : -1;
        if (which >= 0) {
            float v = 0.0f;
            if (lane < 16)
                for (int w = 0; w < kW; ++w) v += red_a[(w * 2 + which) * 16 + lane];
            if (lane < 16) __stcg(p.partials + ((size_t)blockIdx.x * 2 + which) * 16 + lane, v);
            __threadfence();
            __syncwarp();
            finish_cta_tile(p, segs, which ? tl : tf, G, lane);
        }
    };
    // End of a run of one tile's units in this warp: its rows (quad sums) go
    // to the shared-tile slot, out directly, or to the owned-tile slot.
    auto end_run = [&](const Cursor& c, int k) {
        quad_rows(yg, y8, ym, t);
        if (k < 2) {
            if (t == 0) {
                red_a[(warp * 2 + k) * 16 + g] = yg;
                red_a[(warp * 2 + k) * 16 + g + 8] = y8;
            }
        } else {
            const long long ub = ((long long)segs[c.s].tile0 + c.tile) * nb;
            if (ub >= wb && ub + nb <= we) {
                if (t == 0) {
                    if (p.swiglu) {
                        write_rows(segs[c.s], c.tile, 1, g, yg, y8);
                    } else {
                        write_rows(segs[c.s], c.tile, 0, g, yg, 0.0f);
                        write_rows(segs[c.s], c.tile, 0, g + 8, y8, 0.0f);
                    }
                }
            } else if (t == 0) {
                const int slot = wb < ub ? 1 : 0;  // 1: the tile begins inside the range and runs past its end
                red_b[(warp * 2 + slot) * 16 + g] = yg;
                red_b[(warp * 2 + slot) * 16 + g + 8] = y8;
            }
        }
        yg = y8 = ym = 0.0f;
    };
    auto compute = [&](const Buf& buf) {
        if (!a_done && wk.k == 2) shared_tiles_done();
        const Cursor c = wk.c;
        const int k = wk.k, j = c.j;
        if (is_q4(c)) {
            uint2 bx0[4], bx1[4];
            const uint8_t* p0 = xb4_0 + j * xinc0;
            const uint8_t* p1 = xb4_1 + j * xinc1;
#pragma unroll
            for (int gi = 0; gi < 4; ++gi) {
                bx0[gi] = *reinterpret_cast<const uint2*>(p0 + 256 * gi);
                bx1[gi] = *reinterpret_cast<const uint2*>(p1 + 256 * gi);
            }
            const float4 xsum4 = *reinterpret_cast<const float4*>(xsum + j * 8 + h * 4);
            q4_unit(buf, bx0, bx1, xsum4, xs[j], L, yg, y8, ym);
        } else {
            q6_unit(buf, xb6_0 + j * xinc0, xb6_1 + j * xinc1, xs[j], L6, yg, y8);
        }
        walk_next(wk, sp, segs, p.nseg, nb);
        if (wk.k != k || j == nb - 1) end_run(c, k);
    };
    while (wk.k < 3) {
        compute(B0);
        request(B0);
        if (wk.k >= 3) break;
        compute(B1);
        request(B1);
        if (wk.k >= 3) break;
        compute(B2);
        request(B2);
    }
    if (!a_done) shared_tiles_done();

    // ---- owned tiles split between warps: summed in warp order ----
    __syncthreads();
    // this warp combines the split tiles whose first unit is in its range:
    // slot 0, the tile its range begins with (at the tile's start) and ends
    // inside; slot 1, the tile that begins inside its range and runs past it
    for (int slot = 0; slot < 2; ++slot) {
        if (wb >= we) break;
        long long ub;
        if (slot == 0) {
            if (wb % nb != 0 || wb + nb <= we) continue;
            ub = wb;
        } else {
            ub = (we - 1) / nb * nb;
            if (ub <= wb || ub + nb <= we) continue;
        }
        float acc = 0.0f;
        if (lane < 16) {
            acc = red_b[(warp * 2 + slot) * 16 + lane];
            for (int w = warp + 1; w < kW; ++w) {
                const long long b2 = ob + nB * w / kW, e2 = ob + nB * (w + 1) / kW;
                if (b2 >= ub + nb) break;
                if (b2 < e2) acc += red_b[(w * 2) * 16 + lane];
            }
        }
        const float up = __shfl_down_sync(0xffffffffu, acc, 8);
        const long long gt = ub / nb;
        int s = 0;
#pragma unroll
        for (int i = 1; i < kMaxSegs; ++i)
            if (i < p.nseg && gt >= segs[i].tile0) s = i;
        write_rows(segs[s], (int)(gt - segs[s].tile0), p.swiglu, lane, acc, up);
    }
}

size_t smem_bytes(int nb) { return xq4_bytes(nb) + kZeroBytes + 2 * kW * 32 * 4 + 8 * kW + sizeof(Seg) * kMaxSegs; }

template <bool H4, bool H6>
cudaError_t launch(const Params& p, int grid, cudaStream_t stream) {
    auto kern = gemv_pk_kernel<H4, H6>;
    static SmemLimit limit;
    const size_t smem = smem_bytes(p.nb);
    cudaError_t e = limit.ensure(kern, (int)smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, dim3(grid), dim3(kThreads), smem, stream, p);
}

// Partial rows of shared tiles, one per CTA and slot: [grid][2][16] floats,
// then the tickets.
size_t partial_bytes(int sms) { return ((size_t)sms * 2 * 16 * sizeof(float) + 255) & ~(size_t)255; }

}  // namespace gpk
}  // namespace cl

// ---- fragment packing ---------------------------------------------------------
// Unit (tile T, super-block j) of a matrix in the device layout
// (cl_repack_rows), rows 16T .. 16T + 15 (pair: gate rows 8T .. 8T + 7, then
// up rows 8T .. 8T + 7; rows past the matrix are zero).  One thread per
// 16-byte piece: Q4_K pieces 0-127 = chunk c = piece / 32, lane = piece % 32
// (row g or g + 8 for c < 2 / c >= 2; qs bytes 32 gi + 8 t of groups
// gi = 2 (c & 1), 2 (c & 1) + 1), pieces 128-143 = the 16 headers; Q6_K
// pieces 0-191 = chunk c (row g for c < 3, else g + 8; c % 3 = 0, 1: ql
// words of half c % 3 in (j, s) order; 2: qh words in (hh, s) order), pieces
// 192-207 = scale bytes 4 hh + 2 j + s (of sub-block half h) of rows g and
// g + 8 for (g, h) = piece - 192, pieces 208-209 = f16 d of (g, g + 8).
namespace cl {
namespace gpk {

__device__ const uint8_t* pack_row(const uint8_t* w, const uint8_t* w_up, long long stride, int rows, int T, int r) {
    if (w_up) {
        const int row = 8 * T + (r & 7);
        if (row >= rows) return nullptr;
        return (r < 8 ? w : w_up) + (long long)row * stride;
    }
    const int row = 16 * T + r;
    return row < rows ? w + (long long)row * stride : nullptr;
}

__global__ void gemv_pack_kernel(int type, const uint8_t* __restrict__ w, const uint8_t* __restrict__ w_up,
                                 long long stride, int rows, int k, int tiles, uint8_t* __restrict__ out) {
    grid_wait();
    const int nb = k / 256;
    const bool q4 = type == CL_TYPE_Q4_K;
    const int pieces = q4 ? 144 : 210;
    const long long total = (long long)tiles * nb * pieces;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int pc = (int)(i % pieces);
        const long long tu = i / pieces;
        const int j = (int)(tu % nb);
        const int T = (int)(tu / nb);
        uint32_t v[4] = {0u, 0u, 0u, 0u};
        if (q4) {
            if (pc < 128) {
                const int c = pc >> 5, ln = pc & 31, g = ln >> 2, t = ln & 3;
                const uint8_t* row = pack_row(w, w_up, stride, rows, T, c < 2 ? g : g + 8);
                if (row) {
                    const uint8_t* blk = row + 144LL * j + 16;
                    const int gi = 2 * (c & 1);
                    const uint2 lo = *reinterpret_cast<const uint2*>(blk + 32 * gi + 8 * t);
                    const uint2 hi = *reinterpret_cast<const uint2*>(blk + 32 * (gi + 1) + 8 * t);
                    v[0] = lo.x; v[1] = lo.y; v[2] = hi.x; v[3] = hi.y;
                }
            } else {
                const uint8_t* row = pack_row(w, w_up, stride, rows, T, pc - 128);
                if (row) {
                    const uint4 hd = *reinterpret_cast<const uint4*>(row + 144LL * j);
                    v[0] = hd.x; v[1] = hd.y; v[2] = hd.z; v[3] = hd.w;
                }
            }
        } else if (pc < 192) {
            const int c = pc >> 5, ln = pc & 31, g = ln >> 2, t = ln & 3;
            const uint8_t* row = pack_row(w, w_up, stride, rows, T, c < 3 ? g : g + 8);
            if (row) {
                const uint8_t* blk = row + 208LL * j;
                const int cc = c % 3;
                for (int q = 0; q < 4; ++q) {
                    const int a = q >> 1, s = q & 1;  // (j, s) for ql, (hh, s) for qh
                    const int off = cc < 2 ? 64 * cc + 32 * a + 16 * s + 4 * t : 128 + 32 * a + 16 * s + 4 * t;
                    v[q] = *reinterpret_cast<const uint32_t*>(blk + off);
                }
            }
        } else if (pc < 208) {
            const int g = (pc - 192) >> 1, hf = (pc - 192) & 1;
            for (int half = 0; half < 2; ++half) {
                const uint8_t* row = pack_row(w, w_up, stride, rows, T, half ? g + 8 : g);
                if (!row) continue;
                const uint8_t* sc = row + 208LL * j + 192;
                for (int mi = 0; mi < 8; ++mi) {
                    const int hh = mi >> 2, jj = (mi >> 1) & 1, s = mi & 1;
                    const uint32_t byte = sc[8 * hh + 4 * hf + 2 * jj + s];
                    v[2 * half + (mi >> 2)] |= byte << (8 * (mi & 3));
                }
            }
        } else {
            for (int q = 0; q < 4; ++q) {
                const int g = 4 * (pc - 208) + q;
                uint32_t dd = 0;
                for (int half = 0; half < 2; ++half) {
                    const uint8_t* row = pack_row(w, w_up, stride, rows, T, half ? g + 8 : g);
                    if (!row) continue;
                    const uint8_t* dp = row + 208LL * nb + 2 * j;
                    dd |= ((uint32_t)dp[0] | ((uint32_t)dp[1] << 8)) << (16 * half);
                }
                v[q] = dd;
            }
        }
        reinterpret_cast<uint4*>(out)[i] = make_uint4(v[0], v[1], v[2], v[3]);
    }
}

int pack_tiles(int rows, int pair) { return pair ? (rows + 7) / 8 : (rows + 15) / 16; }

}  // namespace gpk
}  // namespace cl

using namespace cl;
using namespace cl::gpk;

extern "C" {

CL_API size_t cl_gemv_pack_bytes(int type, int rows, int k, int pair) {
    if ((type != CL_TYPE_Q4_K && type != CL_TYPE_Q6_K) || rows <= 0 || k <= 0 || k % 256) return 0;
    return (size_t)pack_tiles(rows, pair) * (size_t)(k / 256) * (type == CL_TYPE_Q4_K ? kQ4Unit : kQ6Unit);
}

CL_API int cl_gemv_pack(int type, const void* w, long long stride, int rows, int k, const void* w_up, void* out,
                        cudaStream_t stream) {
    if (cl_gemv_pack_bytes(type, rows, k, w_up != nullptr) == 0 || w == nullptr || out == nullptr ||
        stride < cl_row_stride(type, k))
        return CL_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(w_up) | reinterpret_cast<uintptr_t>(out)) % 16 ||
        stride % 16)
        return CL_ERR_INVALID;
    int sms = 0;
    if (device_sm_count(&sms) != cudaSuccess) return CL_ERR_CUDA;
    return launch_pdl(gemv_pack_kernel, dim3(sms * 8), dim3(256), 0, stream, type, static_cast<const uint8_t*>(w),
                      static_cast<const uint8_t*>(w_up), stride, rows, k, pack_tiles(rows, w_up != nullptr),
                      static_cast<uint8_t*>(out)) == cudaSuccess
               ? CL_OK
               : CL_ERR_CUDA;
}

CL_API size_t cl_gemv_packed_workspace_bytes(int max_tiles) {
    int sms = 0;
    if (max_tiles <= 0 || device_sm_count(&sms) != cudaSuccess) return 0;
    return partial_bytes(sms) + (((size_t)max_tiles * 4 + 255) & ~(size_t)255);
}

CL_API int cl_gemv_packed(const cl_gemv_packed_segment* segs, int nseg, int k, const float* x, const float* gamma,
                          float eps, int swiglu, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (segs == nullptr || nseg < 1 || nseg > kMaxSegs || k <= 0 || k % 256 || x == nullptr || workspace == nullptr)
        return CL_ERR_INVALID;
    if (k / 256 > kW * kMaxBlocksPerWarp) return CL_ERR_UNSUPPORTED;
    if (swiglu && nseg != 1) return CL_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(gamma) |
         reinterpret_cast<uintptr_t>(workspace)) % 16)
        return CL_ERR_INVALID;
    Params p{};
    p.nb = k / 256;
    p.k = k;
    p.x = x;
    p.gamma = gamma;
    p.eps = eps;
    p.nseg = nseg;
    p.swiglu = swiglu ? 1 : 0;
    bool h4 = false, h6 = false;
    long long U = 0;
    int tiles = 0;
    for (int i = 0; i < nseg; ++i) {
        const cl_gemv_packed_segment& s = segs[i];
        if ((s.type != CL_TYPE_Q4_K && s.type != CL_TYPE_Q6_K) || s.w == nullptr || s.y == nullptr || s.n <= 0)
            return CL_ERR_INVALID;
        if (reinterpret_cast<uintptr_t>(s.w) % 16) return CL_ERR_INVALID;
        if (swiglu && (s.bias || s.residual)) return CL_ERR_INVALID;
        h4 |= s.type == CL_TYPE_Q4_K;
        h6 |= s.type == CL_TYPE_Q6_K;
        Seg& d = p.seg[i];
        d.w = static_cast<const uint8_t*>(s.w);
        d.bias = s.bias;
        d.residual = s.residual;
        d.y = s.y;
        d.type = s.type;
        d.n = s.n;
        d.tiles = pack_tiles(s.n, swiglu);
        d.tile0 = tiles;
        d.u0 = U;
        tiles += d.tiles;
        U += (long long)d.tiles * p.nb;
    }
    if (U >= (1LL << 30)) return CL_ERR_UNSUPPORTED;  // unit indices are 32-bit in the kernel
    p.U = U;
    int sms = 0;
    if (device_sm_count(&sms) != cudaSuccess) return CL_ERR_CUDA;
    p.whole_tiles = tiles >= sms ? 1 : 0;
    const size_t pb = partial_bytes(sms);
    if (workspace_bytes < pb + (size_t)tiles * 4) return CL_ERR_INVALID;
    p.partials = static_cast<float*>(workspace);
    p.tickets = reinterpret_cast<unsigned int*>(static_cast<uint8_t*>(workspace) + pb);
    cudaError_t e;
    if (h4 && h6) e = launch<true, true>(p, sms, stream);
    else if (h4) e = launch<true, false>(p, sms, stream);
    else e = launch<false, true>(p, sms, stream);
    return e == cudaSuccess ? CL_OK : CL_ERR_CUDA;
}

}  // extern "C"
