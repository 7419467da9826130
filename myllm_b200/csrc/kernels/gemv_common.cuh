// Shared pieces of the decode GEMV kernels (gemv.cu, moe.cu): the per-thread
// XQ unit of x, exact integer dots of quantized weights with the XQ limbs
// (dp4a), per-format unit dots, warp reductions and the XQ encoder.
//
// Reference: metal_gevm_{q4_k,q6_k,q5_0,q8_0,q5_k}_f32 (metal_llm.metal:708-781)
// and the CPU oracle gevmt/gevmtb over GgufDequantizer rows
// (cpu_llm.cpp:512-547, model.cpp:581-683).
#pragma once

#include "common.cuh"

namespace cl {

// x data of one consumer thread: the unit's two 16-element chunks.
struct XUnit {
    int4 l[2][3];
    int2 s[2];
    float xs;    // scale * 2^-14 of the unit's 32-block
    float xsum;  // sum of the unit's (encoded) x values
};

CL_DEVINL void load_xunit(const XQView& x, int u, XUnit& r) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const int ch = 2 * u + c;
        r.l[c][0] = x.limbs[3 * ch + 0];
        r.l[c][1] = x.limbs[3 * ch + 1];
        r.l[c][2] = x.limbs[3 * ch + 2];
        r.s[c] = x.lsum[ch];
    }
    r.xs = x.scale[u];
    r.xsum = fmaf((float)(r.s[0].x + r.s[1].x), 16384.0f, (float)(r.s[0].y + r.s[1].y)) * r.xs;
}

struct Sums {
    int s0, s1, s2;
};

CL_DEVINL void acc_u(Sums& a, uint32_t w, int4 const (&l)[3], int i) {
    const int l0 = i == 0 ? l[0].x : i == 1 ? l[0].y : i == 2 ? l[0].z : l[0].w;
    const int l1 = i == 0 ? l[1].x : i == 1 ? l[1].y : i == 2 ? l[1].z : l[1].w;
    const int l2 = i == 0 ? l[2].x : i == 1 ? l[2].y : i == 2 ? l[2].z : l[2].w;
    a.s0 = dp4a_us(w, l0, a.s0);
    a.s1 = dp4a_us(w, l1, a.s1);
    a.s2 = dp4a_us(w, l2, a.s2);
}

CL_DEVINL void acc_s(Sums& a, uint32_t w, int4 const (&l)[3], int i) {
    const int l0 = i == 0 ? l[0].x : i == 1 ? l[0].y : i == 2 ? l[0].z : l[0].w;
    const int l1 = i == 0 ? l[1].x : i == 1 ? l[1].y : i == 2 ? l[1].z : l[1].w;
    const int l2 = i == 0 ? l[2].x : i == 1 ? l[2].y : i == 2 ? l[2].z : l[2].w;
    a.s0 = dp4a_ss((int)w, l0, a.s0);
    a.s1 = dp4a_ss((int)w, l1, a.s1);
    a.s2 = dp4a_ss((int)w, l2, a.s2);
}

// (sum of q * x) / scale; `off` subtracted from every q exactly.
CL_DEVINL float sums_value(const Sums& a, int l0sum, int l12sum, int off) {
    const int s0 = a.s0 - off * l0sum;
    const int s12 = a.s1 * 128 + a.s2 - off * l12sum;
    return fmaf((float)s0, 16384.0f, (float)s12);
}

CL_DEVINL uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xffu; }

// Weight-byte loaders: SmemLd reads a shared-memory copy of the rows, GlobalLd
// reads rows in HBM through the read-only (non-coherent) path.
struct SmemLd {
    CL_DEVINL static uint4 v4(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
    CL_DEVINL static uint32_t u16(const uint8_t* p) { return *reinterpret_cast<const unsigned short*>(p); }
    CL_DEVINL static uint32_t u32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
};
struct GlobalLd {
    CL_DEVINL static uint4 v4(const uint8_t* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
    CL_DEVINL static uint32_t u16(const uint8_t* p) { return __ldg(reinterpret_cast<const unsigned short*>(p)); }
    CL_DEVINL static uint32_t u32(const uint8_t* p) { return __ldg(reinterpret_cast<const unsigned int*>(p)); }
};

// ---- per-format unit dots.  Unit u = elements [32u, 32u + 32) of a row in
// the device layout (through loader L); nb = blocks per row.
template <int T>
struct Fmt;

// Scale/min slot i of a device-layout K-quant header (see dequant.cuh):
// eight 12-bit slots sc | m << 6 in header words 1..3.
CL_DEVINL void kslot(const uint4& hdr, int i, float& sc, float& m) {
    const int bit = 12 * i, wi = bit >> 5, off = bit & 31;
    const uint32_t lo = wi == 0 ? hdr.y : (wi == 1 ? hdr.z : hdr.w);
    const uint32_t hw = wi == 0 ? hdr.z : hdr.w;
    const uint32_t v = __funnelshift_r(lo, hw, off);
    sc = (float)(v & 63u);
    m = (float)((v >> 6) & 63u);
}

template <>
struct Fmt<CL_TYPE_Q4_K> {
    template <class L>
    CL_DEVINL static float dot(const uint8_t* row, int u, int nb, const XUnit& x) {
        const int b = u >> 3, i = u & 7, g = i >> 1;
        const bool hi = (i & 1) != 0;
        const uint8_t* blk = row + b * 144;
        const uint4 hdr = L::v4(blk);
        const uint4 q0 = L::v4(blk + 16 + 32 * g), q1 = L::v4(blk + 32 + 32 * g);
        // high nibbles stay in place (16 q): one AND per word, 1/16 folded below
        const uint32_t mk = hi ? 0xf0f0f0f0u : 0x0f0f0f0fu;
        Sums a{0, 0, 0};
        acc_u(a, q0.x & mk, x.l[0], 0);
        acc_u(a, q0.y & mk, x.l[0], 1);
        acc_u(a, q0.z & mk, x.l[0], 2);
        acc_u(a, q0.w & mk, x.l[0], 3);
        acc_u(a, q1.x & mk, x.l[1], 0);
        acc_u(a, q1.y & mk, x.l[1], 1);
        acc_u(a, q1.z & mk, x.l[1], 2);
        acc_u(a, q1.w & mk, x.l[1], 3);
        float sc, m;
        kslot(hdr, i, sc, m);
        const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
        const float xs = hi ? x.xs * 0.0625f : x.xs;
        return (d * sc) * (sums_value(a, 0, 0, 0) * xs) - (dmin * m) * x.xsum;
    }
};

template <>
struct Fmt<CL_TYPE_Q5_K> {
    template <class L>
    CL_DEVINL static float dot(const uint8_t* row, int u, int nb, const XUnit& x) {
        const int b = u >> 3, i = u & 7, g = i >> 1, sh = 4 * (i & 1);
        const uint8_t* blk = row + b * 176;
        const uint4 hdr = L::v4(blk);
        const uint4 h0 = L::v4(blk + 16), h1 = L::v4(blk + 32);
        const uint4 q0 = L::v4(blk + 48 + 32 * g), q1 = L::v4(blk + 64 + 32 * g);
#define Q5K_W(q, h) ((((q) >> sh) & 0x0f0f0f0fu) | ((((h) >> i) & 0x01010101u) << 4))
        Sums a{0, 0, 0};
        acc_u(a, Q5K_W(q0.x, h0.x), x.l[0], 0);
        acc_u(a, Q5K_W(q0.y, h0.y), x.l[0], 1);
        acc_u(a, Q5K_W(q0.z, h0.z), x.l[0], 2);
        acc_u(a, Q5K_W(q0.w, h0.w), x.l[0], 3);
        acc_u(a, Q5K_W(q1.x, h1.x), x.l[1], 0);
        acc_u(a, Q5K_W(q1.y, h1.y), x.l[1], 1);
        acc_u(a, Q5K_W(q1.z, h1.z), x.l[1], 2);
        acc_u(a, Q5K_W(q1.w, h1.w), x.l[1], 3);
#undef Q5K_W
        float sc, m;
        kslot(hdr, i, sc, m);
        const float d = half_bits_to_float(hdr.x), dmin = half_bits_to_float(hdr.x >> 16);
        return (d * sc) * (sums_value(a, 0, 0, 0) * x.xs) - (dmin * m) * x.xsum;
    }
};

template <>
struct Fmt<CL_TYPE_Q6_K> {
    template <class L>
    CL_DEVINL static float dot(const uint8_t* row, int u, int nb, const XUnit& x) {
        const int b = u >> 3, j = u & 7, h = j >> 2, q = j & 3;
        const uint8_t* blk = row + b * 208;
        const uint4 l0 = L::v4(blk + 64 * h + 32 * (q & 1)), l1 = L::v4(blk + 64 * h + 32 * (q & 1) + 16);
        const uint4 h0 = L::v4(blk + 128 + 32 * h), h1 = L::v4(blk + 144 + 32 * h);
        const int nsh = 4 * (q >> 1), qsh = 2 * q;
#define Q6K_W(l, hh) ((((l) >> nsh) & 0x0f0f0f0fu) | ((((hh) >> qsh) & 0x03030303u) << 4))
        Sums a0{0, 0, 0}, a1{0, 0, 0};
        acc_u(a0, Q6K_W(l0.x, h0.x), x.l[0], 0);
        acc_u(a0, Q6K_W(l0.y, h0.y), x.l[0], 1);
        acc_u(a0, Q6K_W(l0.z, h0.z), x.l[0], 2);
        acc_u(a0, Q6K_W(l0.w, h0.w), x.l[0], 3);
        acc_u(a1, Q6K_W(l1.x, h1.x), x.l[1], 0);
        acc_u(a1, Q6K_W(l1.y, h1.y), x.l[1], 1);
        acc_u(a1, Q6K_W(l1.z, h1.z), x.l[1], 2);
        acc_u(a1, Q6K_W(l1.w, h1.w), x.l[1], 3);
#undef Q6K_W
        const uint32_t s16 = L::u16(blk + 192 + 2 * j);
        const float sc0 = (float)(int8_t)(s16 & 0xffu), sc1 = (float)(int8_t)(s16 >> 8);
        const float d = half_bits_to_float(L::u16(row + (size_t)nb * 208 + 2 * b));
        const float v0 = sums_value(a0, x.s[0].x, x.s[0].y, 32);
        const float v1 = sums_value(a1, x.s[1].x, x.s[1].y, 32);
        return d * (sc0 * v0 + sc1 * v1) * x.xs;
    }
};

template <>
struct Fmt<CL_TYPE_Q8_0> {
    template <class L>
    CL_DEVINL static float dot(const uint8_t* row, int u, int nb, const XUnit& x) {
        const uint4 q0 = L::v4(row + 32 * u), q1 = L::v4(row + 32 * u + 16);
        Sums a{0, 0, 0};
        acc_s(a, q0.x, x.l[0], 0);
        acc_s(a, q0.y, x.l[0], 1);
        acc_s(a, q0.z, x.l[0], 2);
        acc_s(a, q0.w, x.l[0], 3);
        acc_s(a, q1.x, x.l[1], 0);
        acc_s(a, q1.y, x.l[1], 1);
        acc_s(a, q1.z, x.l[1], 2);
        acc_s(a, q1.w, x.l[1], 3);
        const float d = half_bits_to_float(L::u16(row + (size_t)nb * 32 + 2 * u));
        return d * (sums_value(a, 0, 0, 0) * x.xs);
    }
};

template <>
struct Fmt<CL_TYPE_Q5_0> {
    template <class L>
    CL_DEVINL static float dot(const uint8_t* row, int u, int nb, const XUnit& x) {
        const uint4 q = L::v4(row + 16 * u);
        const uint32_t qh = L::u32(row + (size_t)nb * 16 + 4 * u);
        const float d = half_bits_to_float(L::u16(row + (size_t)nb * 20 + 2 * u));
#define Q50_LO(w, i) (((w) & 0x0f0f0f0fu) | ((((qh >> (4 * (i))) & 0xfu) * 0x02040810u) & 0x10101010u))
#define Q50_HI(w, i) ((((w) >> 4) & 0x0f0f0f0fu) | ((((qh >> (16 + 4 * (i))) & 0xfu) * 0x02040810u) & 0x10101010u))
        Sums a{0, 0, 0};
        acc_u(a, Q50_LO(q.x, 0), x.l[0], 0);
        acc_u(a, Q50_LO(q.y, 1), x.l[0], 1);
        acc_u(a, Q50_LO(q.z, 2), x.l[0], 2);
        acc_u(a, Q50_LO(q.w, 3), x.l[0], 3);
        acc_u(a, Q50_HI(q.x, 0), x.l[1], 0);
        acc_u(a, Q50_HI(q.y, 1), x.l[1], 1);
        acc_u(a, Q50_HI(q.z, 2), x.l[1], 2);
        acc_u(a, Q50_HI(q.w, 3), x.l[1], 3);
#undef Q50_LO
#undef Q50_HI
        return d * (sums_value(a, x.s[0].x + x.s[1].x, x.s[0].y + x.s[1].y, 16) * x.xs);
    }
};

// ---- warp reduction of N partial sums at once -------------------------------
// Butterfly that halves the vector each step: N values cost ~N + 5 shuffles
// instead of 5 N.  Afterwards every lane holds the full sum of value
// index red_index<N>(lane).
template <int N>
CL_DEVINL float warp_sum_many(float (&v)[N], int lane) {
    static_assert(N == 1 || N == 2 || N == 4 || N == 8, "N must be 1, 2, 4 or 8");
    float w[N];
#pragma unroll
    for (int j = 0; j < N; ++j) w[j] = v[j];
    int n = N, bit = 16;
#pragma unroll
    for (int step = 0; step < 3; ++step) {
        if (n > 1) {
            const bool upper = (lane & bit) != 0;
#pragma unroll
            for (int j = 0; j < N / 2; ++j) {
                if (j < n / 2) {
                    const float keep = upper ? w[j + n / 2] : w[j];
                    const float send = upper ? w[j] : w[j + n / 2];
                    w[j] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
                }
            }
            n /= 2;
            bit >>= 1;
        }
    }
    float r = w[0];
    for (; bit > 0; bit >>= 1) r += __shfl_xor_sync(0xffffffffu, r, bit);
    return r;
}

template <int N>
CL_DEVINL int red_index(int lane) {
    return N == 1 ? 0 : N == 2 ? (lane >> 4) & 1 : N == 4 ? (lane >> 3) & 3 : (lane >> 2) & 7;
}

// ---- input preparation ---------------------------------------------------------
// Each consumer thread turns x[32u, 32u + 32) (optionally RMS-normalised) into
// its XQ unit in registers, with the expressions of xq_store_block_warp.
CL_DEVINL void encode_unit(const float (&v)[32], XUnit& r) {
    float amax = 0.0f;
#pragma unroll
    for (int e = 0; e < 32; ++e) amax = fmaxf(amax, fabsf(v[e]));
    const float sc = amax / 127.0f;
    const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
    uint32_t w0[8], w1[8], w2[8];
    int t0[2] = {0, 0}, t12[2] = {0, 0};
#pragma unroll
    for (int e = 0; e < 32; ++e) {
        const float r0 = v[e] * inv;
        const float l0 = fminf(fmaxf(rintf(r0), -127.0f), 127.0f);
        const float r1 = (r0 - l0) * 128.0f;
        const float l1 = fminf(fmaxf(rintf(r1), -64.0f), 64.0f);
        const float r2 = (r1 - l1) * 128.0f;
        const float l2 = fminf(fmaxf(rintf(r2), -64.0f), 64.0f);
        const int i0 = (int)l0, i1 = (int)l1, i2 = (int)l2;
        const int sh = 8 * (e & 3);
        if ((e & 3) == 0) {
            w0[e >> 2] = 0u;
            w1[e >> 2] = 0u;
            w2[e >> 2] = 0u;
        }
        w0[e >> 2] |= ((uint32_t)i0 & 0xffu) << sh;
        w1[e >> 2] |= ((uint32_t)i1 & 0xffu) << sh;
        w2[e >> 2] |= ((uint32_t)i2 & 0xffu) << sh;
        t0[e >> 4] += i0;
        t12[e >> 4] += i1 * 128 + i2;
    }
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        r.l[c][0] = make_int4((int)w0[4 * c], (int)w0[4 * c + 1], (int)w0[4 * c + 2], (int)w0[4 * c + 3]);
        r.l[c][1] = make_int4((int)w1[4 * c], (int)w1[4 * c + 1], (int)w1[4 * c + 2], (int)w1[4 * c + 3]);
        r.l[c][2] = make_int4((int)w2[4 * c], (int)w2[4 * c + 1], (int)w2[4 * c + 2], (int)w2[4 * c + 3]);
        r.s[c] = make_int2(t0[c], t12[c]);
    }
    r.xs = sc * (1.0f / 16384.0f);
    r.xsum = fmaf((float)(t0[0] + t0[1]), 16384.0f, (float)(t12[0] + t12[1])) * r.xs;
}

}  // namespace cl
