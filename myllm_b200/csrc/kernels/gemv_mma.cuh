// Device helpers shared by the decode GEMV kernels that dot K-quant weights
// with the XQ4 activation encoding on the tensor cores (gemv_mma.cu, the
// per-layer GEMV launches; decode_fused.cu, the persistent decode step).
// The formats and the fragment layouts are described in gemv_mma.cu.
#pragma once

#include "common.cuh"

namespace cl {
namespace gmma {

// m16n8k32 u8 x s8 -> s32: D = A B + C.
CL_DEVINL void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                        uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
CL_DEVINL void mma_u8s8_z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                          uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// m16n8k32 s8 x s8 -> s32, accumulator starting at zero.
CL_DEVINL void mma_s8s8_z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                          uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// Per-lane constants of a consumer lane (Q4_K; the Q6_K copy has no 1/16
// factor in lw0/lw1).
struct Q4Lane {
    uint32_t sh;     // 12 * h: header shift that puts unit (2gi + h)'s slot at a fixed bit
    float lw0, lw1;  // weights of the lane's two limb columns (1/16 for high-nibble units)
    int pp;          // row of the min term: g (0) or g + 8 (1)
};

// Slot field of unit 2gi + h after the per-lane shift: sc at bit 32 + 24 gi,
// m at bit 38 + 24 gi of the 128-bit header (w1..w3 = header words 1..3).
template <int GI>
CL_DEVINL int q4_sc(uint32_t w1, uint32_t w2, uint32_t w3) {
    if (GI == 0) return (int)(w1 & 63u);
    if (GI == 1) return (int)(__funnelshift_r(w1, w2, 24) & 63u);
    if (GI == 2) return (int)((w2 >> 16) & 63u);
    return (int)((w3 >> 8) & 63u);
}
template <int GI>
CL_DEVINL float q4_m(uint32_t w1, uint32_t w2, uint32_t w3) {
    if (GI == 0) return (float)((w1 >> 6) & 63u);
    if (GI == 1) return (float)(__funnelshift_r(w1, w2, 30) & 63u);
    if (GI == 2) return (float)((w2 >> 22) & 63u);
    return (float)((w3 >> 14) & 63u);
}

// One Q4_K super-block of 16 rows.  bg/b8: the rows' block in shared memory;
// bx0/bx1: the lane's B words for the four groups (low-unit and high-unit
// columns, zero where the lane's column is the other unit); xsum4: sums of x
// over the lane's four units; xs: the block's x scale.
CL_DEVINL void q4k_sb(const uint8_t* bg, const uint8_t* b8, const uint2 (&bx0)[4], const uint2 (&bx1)[4],
                      const float4& xsum4, float xs, int t, const Q4Lane& L, float& yg, float& y8, float& ym) {
    const uint4 hg = *reinterpret_cast<const uint4*>(bg);
    const uint4 h8 = *reinterpret_cast<const uint4*>(b8);
    const uint32_t g1 = __funnelshift_r(hg.y, hg.z, L.sh), g2 = __funnelshift_r(hg.z, hg.w, L.sh), g3 = hg.w >> L.sh;
    const uint32_t e1 = __funnelshift_r(h8.y, h8.z, L.sh), e2 = __funnelshift_r(h8.z, h8.w, L.sh), e3 = h8.w >> L.sh;
    int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
    for (int gi = 0; gi < 4; ++gi) {
        const uint2 wg = *reinterpret_cast<const uint2*>(bg + 16 + 32 * gi + 8 * t);
        const uint2 w8 = *reinterpret_cast<const uint2*>(b8 + 16 + 32 * gi + 8 * t);
        int c[4];
        mma_u8s8_z(c, wg.x & 0x0f0f0f0fu, w8.x & 0x0f0f0f0fu, wg.x & 0xf0f0f0f0u, w8.x & 0xf0f0f0f0u, bx0[gi].x,
                   bx1[gi].x);
        mma_u8s8(c, wg.y & 0x0f0f0f0fu, w8.y & 0x0f0f0f0fu, wg.y & 0xf0f0f0f0u, w8.y & 0xf0f0f0f0u, bx0[gi].y,
                 bx1[gi].y);
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
    // min term of the lane's (row, unit kind): dmin * sum_u m_u * sum(x_u)
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

// Encode one 256-element block (lane holds elements 8 lane .. 8 lane + 7)
// into XQ4: xq[unit][limb][32] bytes, xs = s; for Q4_K xsum[h][gi] = sum of
// the encoded x over unit 2 gi + h; for Q6_K xn[sub-block][limb] =
// -32 * sum of the limb over the 16-element sub-block (sub-block = lane / 2).
template <bool XSUM, bool XN>
CL_DEVINL void encode_block(const float (&v)[8], int lane, uint8_t* xq, float* xs, float* xsum, int* xn) {
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = warp_max(amax);
    const float s = amax / 127.0f;
    const float inv = amax > 0.0f ? 127.0f / amax : 0.0f;
    uint32_t w[4][2] = {};
    int t0 = 0, t123 = 0;
    int ls[4] = {0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float r0 = v[i] * inv;
        const float l0 = fminf(fmaxf(rintf(r0), -127.0f), 127.0f);
        const float r1 = (r0 - l0) * 128.0f;
        const float l1 = fminf(fmaxf(rintf(r1), -64.0f), 64.0f);
        const float r2 = (r1 - l1) * 128.0f;
        const float l2 = fminf(fmaxf(rintf(r2), -64.0f), 64.0f);
        const float r3 = (r2 - l2) * 128.0f;
        const float l3 = fminf(fmaxf(rintf(r3), -64.0f), 64.0f);
        const int i0 = (int)l0, i1 = (int)l1, i2 = (int)l2, i3 = (int)l3;
        const int sh = 8 * (i & 3);
        w[0][i >> 2] |= ((uint32_t)i0 & 0xffu) << sh;
        w[1][i >> 2] |= ((uint32_t)i1 & 0xffu) << sh;
        w[2][i >> 2] |= ((uint32_t)i2 & 0xffu) << sh;
        w[3][i >> 2] |= ((uint32_t)i3 & 0xffu) << sh;
        t0 += i0;
        t123 += i1 * 16384 + i2 * 128 + i3;
        ls[0] += i0;
        ls[1] += i1;
        ls[2] += i2;
        ls[3] += i3;
    }
    if (XN) {
#pragma unroll
        for (int l = 0; l < 4; ++l) ls[l] += __shfl_xor_sync(0xffffffffu, ls[l], 1);
        if ((lane & 1) == 0)
            *reinterpret_cast<int4*>(xn + (lane >> 1) * 4) = make_int4(-32 * ls[0], -32 * ls[1], -32 * ls[2], -32 * ls[3]);
    }
    const int unit = lane >> 2, e0 = (lane & 3) * 8;
#pragma unroll
    for (int l = 0; l < 4; ++l)
        *reinterpret_cast<uint2*>(xq + unit * 128 + l * 32 + e0) = make_uint2(w[l][0], w[l][1]);
    if (XSUM) {
        t0 += __shfl_xor_sync(0xffffffffu, t0, 1);
        t123 += __shfl_xor_sync(0xffffffffu, t123, 1);
        t0 += __shfl_xor_sync(0xffffffffu, t0, 2);
        t123 += __shfl_xor_sync(0xffffffffu, t123, 2);
    }
    if (XSUM && (lane & 3) == 0) {
        // sum of x over the unit = s * 2^-21 * (2^21 sum l0 + sum(l1 2^14 + l2 2^7 + l3))
        const int gi = unit >> 1, h = unit & 1;
        xsum[h * 4 + gi] = fmaf((float)t0, 2097152.0f, (float)t123) * (s * (1.0f / 2097152.0f));
    }
    if (lane == 0) *xs = s;
}

}  // namespace gmma
}  // namespace cl
