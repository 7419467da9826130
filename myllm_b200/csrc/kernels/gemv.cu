// Decode GEMV over native GGML blocks: y[n] = W[n, k] . x (+ bias) (+ residual).
//
// Reference: metal_gevm_{q4_k,q6_k,q5_0,q8_0,q5_k}_f32 (metal_llm.metal:708-781)
// and the CPU oracle gevmt/gevmtb over GgufDequantizer rows
// (cpu_llm.cpp:512-547, model.cpp:581-683).  Same products, different order:
// a lane owns a 32-element "unit" of a row, the block bytes are read with
// coalesced 128-bit loads, the quantized integers are dotted with the XQ
// limbs of x by dp4a (exact), and the per-sub-block scales are applied in
// FP32 afterwards (the factored form d*sc*sum(x*q) - dmin*m*sum(x) that the
// Metal kernels also use, metal_llm.metal:392-393).
//
// Device weight layout (cl_repack_rows): each row padded to a multiple of 16
// bytes; Q4_K and Q5_K keep their native blocks (already 16-byte aligned),
// Q6_K/Q8_0/Q5_0 rows are re-ordered structure-of-arrays inside the row so
// that every vector load is aligned.  The byte count per row is unchanged
// apart from the <16-byte pad.
//   Q6_K row: [nb x (ql128 qh64 sc16)] [nb x f16 d]
//   Q8_0 row: [nb x qs32] [nb x f16 d]
//   Q5_0 row: [nb x qs16] [nb x u32 qh] [nb x f16 d]
#include "common.cuh"
#include "launch.cuh"

namespace cl {

// x data of one lane unit: two 16-element chunks.
struct XUnit {
    int4 l[2][3];
    int2 s[2];
    float sc[2];
    float xsum[2];
};

CL_DEVINL void load_xunit(const XQView& x, int c0, int c1, XUnit& u) {
    const int cs[2] = {c0, c1};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int c = cs[h];
        u.l[h][0] = __ldg(x.limbs + 3 * c + 0);
        u.l[h][1] = __ldg(x.limbs + 3 * c + 1);
        u.l[h][2] = __ldg(x.limbs + 3 * c + 2);
        u.s[h] = __ldg(x.lsum + c);
        u.sc[h] = __ldg(x.scale + (c >> 1));
        u.xsum[h] = fmaf((float)u.s[h].x, 16384.0f, (float)u.s[h].y) * u.sc[h];
    }
}

// Integer dot of 16 unsigned weight bytes with one chunk's limbs; `offset`
// is subtracted from every weight (q - offset) exactly via the limb sums.
CL_DEVINL float chunk_dot_u(const uint32_t w[4], const int4 (&l)[3], int2 s, float sc, int offset) {
    int s0 = dp4a_us(w[0], l[0].x, 0);
    s0 = dp4a_us(w[1], l[0].y, s0);
    s0 = dp4a_us(w[2], l[0].z, s0);
    s0 = dp4a_us(w[3], l[0].w, s0);
    int s1 = dp4a_us(w[0], l[1].x, 0);
    s1 = dp4a_us(w[1], l[1].y, s1);
    s1 = dp4a_us(w[2], l[1].z, s1);
    s1 = dp4a_us(w[3], l[1].w, s1);
    int s2 = dp4a_us(w[0], l[2].x, 0);
    s2 = dp4a_us(w[1], l[2].y, s2);
    s2 = dp4a_us(w[2], l[2].z, s2);
    s2 = dp4a_us(w[3], l[2].w, s2);
    int s12 = s1 * 128 + s2;
    if (offset) {
        s0 -= offset * s.x;
        s12 -= offset * s.y;
    }
    return fmaf((float)s0, 16384.0f, (float)s12) * sc;
}

CL_DEVINL float chunk_dot_s(const uint32_t w[4], const int4 (&l)[3], float sc) {
    int s0 = dp4a_ss((int)w[0], l[0].x, 0);
    s0 = dp4a_ss((int)w[1], l[0].y, s0);
    s0 = dp4a_ss((int)w[2], l[0].z, s0);
    s0 = dp4a_ss((int)w[3], l[0].w, s0);
    int s1 = dp4a_ss((int)w[0], l[1].x, 0);
    s1 = dp4a_ss((int)w[1], l[1].y, s1);
    s1 = dp4a_ss((int)w[2], l[1].z, s1);
    s1 = dp4a_ss((int)w[3], l[1].w, s1);
    int s2 = dp4a_ss((int)w[0], l[2].x, 0);
    s2 = dp4a_ss((int)w[1], l[2].y, s2);
    s2 = dp4a_ss((int)w[2], l[2].z, s2);
    s2 = dp4a_ss((int)w[3], l[2].w, s2);
    return fmaf((float)s0, 16384.0f, (float)(s1 * 128 + s2)) * sc;
}

CL_DEVINL uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xffu; }

// 6-bit scale/min of K-quant sub-block i from the 12 scale bytes
// (get_scale_min_k4, model.cpp:524-537), with s0..s2 = bytes 0-3, 4-7, 8-11.
CL_DEVINL void kscale(uint32_t s0, uint32_t s1, uint32_t s2, int i, float& sc, float& m) {
    const int lo = i & 3;
    const uint32_t a = byte_of(s0, lo), b = byte_of(s1, lo), c = byte_of(s2, lo);
    uint32_t vs, vm;
    if (i < 4) {
        vs = a & 63u;
        vm = b & 63u;
    } else {
        vs = (c & 0x0fu) | ((a >> 6) << 4);
        vm = (c >> 4) | ((b >> 6) << 4);
    }
    sc = (float)vs;
    m = (float)vm;
}

// ---- per-format lane-unit kernels --------------------------------------
// chunks(): the two XQ chunk indices a unit reads; dot(): the unit's
// contribution for one row (row points at the row start, nb = blocks/row).
struct FQ4K {
    static constexpr int kType = CL_TYPE_Q4_K;
    CL_DEVINL static void chunks(int u, int& c0, int& c1) {
        const int b = u >> 3, j = u & 7;
        c0 = 16 * b + 4 * (j >> 1) + (j & 1);
        c1 = c0 + 2;
    }
    CL_DEVINL static float dot(const uint8_t* row, int u, int nb, const XUnit& x) {
        const int b = u >> 3, j = u & 7, g = j >> 1;
        const uint8_t* blk = row + b * 144;
        const uint4 hdr = ldg_nc_v4(blk);
        const uint4 q = ldg_nc_v4(blk + 16 + 16 * j);
        const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
        float sc0, m0, sc1, m1;
        kscale(hdr.y, hdr.z, hdr.w, 2 * g, sc0, m0);
        kscale(hdr.y, hdr.z, hdr.w, 2 * g + 1, sc1, m1);
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            lo[i] = qw[i] & 0x0f0f0f0fu;
            hi[i] = (qw[i] >> 4) & 0x0f0f0f0fu;
        }
        const float dl = chunk_dot_u(lo, x.l[0], x.s[0], x.sc[0], 0);
        const float dh = chunk_dot_u(hi, x.l[1], x.s[1], x.sc[1], 0);
        return (d * sc0) * dl - (dmin * m0) * x.xsum[0] + (d * sc1) * dh - (dmin * m1) * x.xsum[1];
    }
};

struct FQ5K {
    static constexpr int kType = CL_TYPE_Q5_K;
    CL_DEVINL static void chunks(int u, int& c0, int& c1) { FQ4K::chunks(u, c0, c1); }
    CL_DEVINL static float dot(const uint8_t* row, int u, int nb, const XUnit& x) {
        const int b = u >> 3, j = u & 7, g = j >> 1;
        const uint8_t* blk = row + b * 176;
        const uint4 hdr = ldg_nc_v4(blk);
        const uint4 h = ldg_nc_v4(blk + 16 + 16 * (j & 1));
        const uint4 q = ldg_nc_v4(blk + 48 + 16 * j);
        const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
        float sc0, m0, sc1, m1;
        kscale(hdr.y, hdr.z, hdr.w, 2 * g, sc0, m0);
        kscale(hdr.y, hdr.z, hdr.w, 2 * g + 1, sc1, m1);
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
        const uint32_t hw[4] = {h.x, h.y, h.z, h.w};
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            lo[i] = (qw[i] & 0x0f0f0f0fu) | (((hw[i] >> (2 * g)) & 0x01010101u) << 4);
            hi[i] = ((qw[i] >> 4) & 0x0f0f0f0fu) | (((hw[i] >> (2 * g + 1)) & 0x01010101u) << 4);
        }
        const float dl = chunk_dot_u(lo, x.l[0], x.s[0], x.sc[0], 0);
        const float dh = chunk_dot_u(hi, x.l[1], x.s[1], x.sc[1], 0);
        return (d * sc0) * dl - (dmin * m0) * x.xsum[0] + (d * sc1) * dh - (dmin * m1) * x.xsum[1];
    }
};

struct FQ6K {
    static constexpr int kType = CL_TYPE_Q6_K;
    CL_DEVINL static void chunks(int u, int& c0, int& c1) {
        const int b = u >> 3, j = u & 7, h = j >> 2, a = j & 3;
        c0 = 16 * b + 8 * h + 2 * (a >> 1) + (a & 1);
        c1 = c0 + 4;
    }
    CL_DEVINL static float dot(const uint8_t* row, int u, int nb, const XUnit& x) {
        const int b = u >> 3, j = u & 7, h = j >> 2, a = j & 3;
        const uint8_t* blk = row + b * 208;
        const uint4 ql = ldg_nc_v4(blk + 64 * h + 16 * a);
        const uint4 qh = ldg_nc_v4(blk + 128 + 32 * h + 16 * (a & 1));
        const uint4 sv = ldg_nc_v4(blk + 192);
        const float d = half_bits_to_float(ldg_nc_u16(row + (size_t)nb * 208 + 2 * b));
        const int sl = 2 * (a >> 1), sh = 4 + sl;
        const uint32_t lw[4] = {ql.x, ql.y, ql.z, ql.w};
        const uint32_t hw[4] = {qh.x, qh.y, qh.z, qh.w};
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            lo[i] = (lw[i] & 0x0f0f0f0fu) | (((hw[i] >> sl) & 0x03030303u) << 4);
            hi[i] = ((lw[i] >> 4) & 0x0f0f0f0fu) | (((hw[i] >> sh) & 0x03030303u) << 4);
        }
        const int il = 8 * h + 2 * (a >> 1) + (a & 1);
        const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
        const float scl = (float)(int8_t)byte_of(sw[il >> 2], il & 3);
        const float sch = (float)(int8_t)byte_of(sw[(il + 4) >> 2], (il + 4) & 3);
        const float dl = chunk_dot_u(lo, x.l[0], x.s[0], x.sc[0], 32);
        const float dh = chunk_dot_u(hi, x.l[1], x.s[1], x.sc[1], 32);
        return d * (scl * dl + sch * dh);
    }
};

struct FQ8_0 {
    static constexpr int kType = CL_TYPE_Q8_0;
    CL_DEVINL static void chunks(int u, int& c0, int& c1) {
        c0 = 2 * u;
        c1 = 2 * u + 1;
    }
    CL_DEVINL static float dot(const uint8_t* row, int u, int nb, const XUnit& x) {
        const uint4 q0 = ldg_nc_v4(row + 32 * u);
        const uint4 q1 = ldg_nc_v4(row + 32 * u + 16);
        const float d = half_bits_to_float(ldg_nc_u16(row + (size_t)nb * 32 + 2 * u));
        const uint32_t a[4] = {q0.x, q0.y, q0.z, q0.w};
        const uint32_t c[4] = {q1.x, q1.y, q1.z, q1.w};
        return d * (chunk_dot_s(a, x.l[0], x.sc[0]) + chunk_dot_s(c, x.l[1], x.sc[1]));
    }
};

struct FQ5_0 {
    static constexpr int kType = CL_TYPE_Q5_0;
    CL_DEVINL static void chunks(int u, int& c0, int& c1) {
        c0 = 2 * u;
        c1 = 2 * u + 1;
    }
    CL_DEVINL static float dot(const uint8_t* row, int u, int nb, const XUnit& x) {
        const uint4 q = ldg_nc_v4(row + 16 * u);
        const uint32_t qh = ldg_nc_u32(row + (size_t)nb * 16 + 4 * u);
        const float d = half_bits_to_float(ldg_nc_u16(row + (size_t)nb * 20 + 2 * u));
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            lo[i] = (qw[i] & 0x0f0f0f0fu) | ((((qh >> (4 * i)) & 0xfu) * 0x02040810u) & 0x10101010u);
            hi[i] = ((qw[i] >> 4) & 0x0f0f0f0fu) |
                    ((((qh >> (16 + 4 * i)) & 0xfu) * 0x02040810u) & 0x10101010u);
        }
        return d * (chunk_dot_u(lo, x.l[0], x.s[0], x.sc[0], 16) +
                    chunk_dot_u(hi, x.l[1], x.s[1], x.sc[1], 16));
    }
};

// ---- kernel ---------------------------------------------------------------
constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kMaxSegs = 4;

struct GemvSeg {
    const uint8_t* w;
    long long stride;
    const float* bias;
    const float* residual;
    float* y;
    int type;
    int n;
    int cta_begin;  // first CTA of this segment
};

struct GemvParams {
    GemvSeg seg[kMaxSegs];
    const void* xq;
    int nseg;
    int k;
    int wpr;      // warps per row group (K split), divides kGemvWarps
    int swiglu;   // 1: seg[0] = gate, seg[1] = up, out = silu(g) * u into seg[0].y
    const uint8_t* w_up;
};

template <int R, class F, bool SWIGLU>
CL_DEVINL void gemv_body(const GemvParams& p, const GemvSeg& s, int cta_in_seg) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wpr = p.wpr;
    const int groups = kGemvWarps / wpr;
    const int rg = warp / wpr, wk = warp % wpr;
    constexpr int OUT = SWIGLU ? R / 2 : R;  // output rows per warp group
    const int out_per_cta = OUT * groups;
    const int out0 = cta_in_seg * out_per_cta + rg * OUT;
    const int k = p.k;
    const int units = k / 32;
    const int nb = F::kType == CL_TYPE_Q8_0 || F::kType == CL_TYPE_Q5_0 ? k / 32 : k / 256;

    const uint8_t* rows[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
        int o = SWIGLU ? out0 + r / 2 : out0 + r;
        o = o < s.n ? o : s.n - 1;
        const uint8_t* base = SWIGLU && (r & 1) ? p.w_up : s.w;
        rows[r] = base + (size_t)o * s.stride;
    }

    // Warm L2 with this CTA's weight rows while the previous kernel drains.
    if (threadIdx.x == 0) {
        const int first = cta_in_seg * out_per_cta;
        const int last = min(first + out_per_cta, s.n);
        if (last > first) {
            const size_t bytes = (size_t)(last - first) * s.stride;
            for (int m = 0; m < (SWIGLU ? 2 : 1); ++m) {
                const uint8_t* b = (m ? p.w_up : s.w) + (size_t)first * s.stride;
                for (size_t off = 0; off < bytes; off += 65536) {
                    prefetch_l2(b + off, (uint32_t)min((size_t)65536, bytes - off));
                }
            }
        }
    }
    grid_launch_dependents();
    grid_wait();

    const XQView xv = xq_view(p.xq, k);
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.0f;

#pragma unroll 2
    for (int u = lane + 32 * wk; u < units; u += 32 * wpr) {
        int c0, c1;
        F::chunks(u, c0, c1);
        XUnit xu;
        load_xunit(xv, c0, c1, xu);
#pragma unroll
        for (int r = 0; r < R; ++r) acc[r] += F::dot(rows[r], u, nb, xu);
    }
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = warp_sum(acc[r]);

    __shared__ float red[kGemvWarps][R];
    if (wpr > 1) {
        if (lane == 0) {
#pragma unroll
            for (int r = 0; r < R; ++r) red[warp][r] = acc[r];
        }
        __syncthreads();
        if (wk != 0) return;
#pragma unroll
        for (int r = 0; r < R; ++r) {
            float t = 0.0f;
            for (int w = 0; w < wpr; ++w) t += red[rg * wpr + w][r];
            acc[r] = t;
        }
    }
    if (lane != 0) return;
#pragma unroll
    for (int r = 0; r < OUT; ++r) {
        const int o = out0 + r;
        if (o >= s.n) break;
        float v;
        if (SWIGLU) {
            // Branch-stable SiLU(g) * u (cpu_llm.cpp:188-202).
            const float g = acc[2 * r], up = acc[2 * r + 1];
            const float sig = g >= 0.0f ? 1.0f / (1.0f + expf(-g)) : expf(g) / (1.0f + expf(g));
            v = g * sig * up;
        } else {
            v = acc[r];
            if (s.bias) v += s.bias[o];
            if (s.residual) v = s.residual[o] + v;
        }
        s.y[o] = v;
    }
}

template <int R, bool SWIGLU>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const GemvParams p) {
    int si = 0;
#pragma unroll
    for (int i = 1; i < kMaxSegs; ++i) {
        if (i < p.nseg && (int)blockIdx.x >= p.seg[i].cta_begin) si = i;
    }
    const GemvSeg& s = p.seg[si];
    const int cta = blockIdx.x - s.cta_begin;
    switch (s.type) {
    case CL_TYPE_Q4_K: gemv_body<R, FQ4K, SWIGLU>(p, s, cta); break;
    case CL_TYPE_Q5_K: gemv_body<R, FQ5K, SWIGLU>(p, s, cta); break;
    case CL_TYPE_Q6_K: gemv_body<R, FQ6K, SWIGLU>(p, s, cta); break;
    case CL_TYPE_Q8_0: gemv_body<R, FQ8_0, SWIGLU>(p, s, cta); break;
    case CL_TYPE_Q5_0: gemv_body<R, FQ5_0, SWIGLU>(p, s, cta); break;
    default: break;
    }
}

constexpr int kRows = 4;

bool gemv_type_ok(int t) {
    return t == CL_TYPE_Q4_K || t == CL_TYPE_Q5_K || t == CL_TYPE_Q6_K || t == CL_TYPE_Q8_0 ||
           t == CL_TYPE_Q5_0;
}

// K-split heuristic: enough CTAs to fill 148 SMs a few times over, but every
// warp keeps at least ~one unit per lane.
int choose_wpr(long long total_out, int out_per_warp, int k) {
    const int units = k / 32;
    int wpr = 1;
    while (wpr < kGemvWarps) {
        const long long ctas = (total_out + (long long)out_per_warp * (kGemvWarps / wpr) - 1) /
                               ((long long)out_per_warp * (kGemvWarps / wpr));
        if (ctas >= 4 * 148) break;
        if (units / (2 * wpr) < 32) break;
        wpr *= 2;
    }
    return wpr;
}

int launch_gemv(const cl_gemv_segment* segs, int nseg, int k, const void* xq, int swiglu,
                const void* w_up, cudaStream_t stream) {
    if (nseg < 1 || nseg > kMaxSegs || k <= 0 || k % 32 != 0 || xq == nullptr) return CL_ERR_INVALID;
    GemvParams p{};
    long long total = 0;
    for (int i = 0; i < nseg; ++i) {
        if (!gemv_type_ok(segs[i].type) || segs[i].w == nullptr || segs[i].y == nullptr ||
            segs[i].n <= 0)
            return CL_ERR_INVALID;
        if ((segs[i].type == CL_TYPE_Q4_K || segs[i].type == CL_TYPE_Q5_K ||
             segs[i].type == CL_TYPE_Q6_K) && k % 256 != 0)
            return CL_ERR_INVALID;
        if (segs[i].stride < cl_row_stride(segs[i].type, k) || segs[i].stride % 16 != 0 ||
            reinterpret_cast<uintptr_t>(segs[i].w) % 16 != 0)
            return CL_ERR_INVALID;
        total += segs[i].n;
    }
    const int out_per_warp = swiglu ? kRows / 2 : kRows;
    p.wpr = choose_wpr(total, out_per_warp, k);
    const int out_per_cta = out_per_warp * (kGemvWarps / p.wpr);
    int ctas = 0;
    for (int i = 0; i < nseg; ++i) {
        GemvSeg& s = p.seg[i];
        s.w = static_cast<const uint8_t*>(segs[i].w);
        s.stride = segs[i].stride;
        s.bias = segs[i].bias;
        s.residual = segs[i].residual;
        s.y = segs[i].y;
        s.type = segs[i].type;
        s.n = segs[i].n;
        s.cta_begin = ctas;
        ctas += (segs[i].n + out_per_cta - 1) / out_per_cta;
    }
    p.nseg = nseg;
    p.k = k;
    p.xq = xq;
    p.swiglu = swiglu;
    p.w_up = static_cast<const uint8_t*>(w_up);
    cudaError_t e = swiglu ? launch_pdl(gemv_kernel<kRows, true>, dim3(ctas), dim3(kGemvThreads), 0, stream, p)
                           : launch_pdl(gemv_kernel<kRows, false>, dim3(ctas), dim3(kGemvThreads), 0, stream, p);
    return e == cudaSuccess ? CL_OK : CL_ERR_CUDA;
}

}  // namespace cl

extern "C" {

CL_API int cl_gemv_xq_multi(const cl_gemv_segment* segs, int nseg, int k, const void* xq,
                            cudaStream_t stream) {
    return cl::launch_gemv(segs, nseg, k, xq, 0, nullptr, stream);
}

CL_API int cl_gemv_xq(int type, const void* w, long long stride, int n, int k, const void* xq,
                      const float* bias, const float* residual, float* y, cudaStream_t stream) {
    cl_gemv_segment s{type, w, stride, n, bias, residual, y};
    return cl::launch_gemv(&s, 1, k, xq, 0, nullptr, stream);
}

CL_API int cl_gemv_xq_swiglu(int type, const void* w_gate, const void* w_up, long long stride, int n,
                             int k, const void* xq, float* y, cudaStream_t stream) {
    if (w_up == nullptr || reinterpret_cast<uintptr_t>(w_up) % 16 != 0) return CL_ERR_INVALID;
    cl_gemv_segment s{type, w_gate, stride, n, nullptr, nullptr, y};
    return cl::launch_gemv(&s, 1, k, xq, 1, w_up, stream);
}

}  // extern "C"
