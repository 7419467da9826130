// Element dequantization from the device weight layout, with the exact FP32
// expressions of the reference CPU decoder (model.cpp:581-683; Q5_K from
// metal_llm.metal:447-496).  Explicit _rn intrinsics keep nvcc from fusing
// a*b - c into one FMA, so the values match the CPU's two roundings.
#pragma once

#include "common.cuh"

namespace cl {

// Native 6-bit scale/min of sub-block i (get_scale_min_k4, model.cpp:524-537).
__host__ __device__ inline void kscale_native(const uint8_t* s, int i, int& sc, int& m) {
    if (i < 4) {
        sc = s[i] & 63;
        m = s[i + 4] & 63;
    } else {
        sc = (s[i + 4] & 0x0f) | ((s[i - 4] >> 6) << 4);
        m = (s[i + 4] >> 4) | ((s[i] >> 6) << 4);
    }
}

// Device-layout K-quant header (cl_repack_rows): bytes 4..15 hold eight
// 12-bit slots, slot i = sc_i | m_i << 6 at bit 12 i (little endian).  Same
// 16 bytes as the native header, re-arranged so one funnel shift finds a slot.
CL_DEVINL void kscale_slot(const uint8_t* s, int i, int& sc, int& m) {
    const int bit = 12 * i, byte = bit >> 3, sh = bit & 7;
    const uint32_t v = ((uint32_t)s[byte] | ((uint32_t)s[byte + 1] << 8)) >> sh;
    sc = (int)(v & 63u);
    m = (int)((v >> 6) & 63u);
}

CL_DEVINL float load_half(const uint8_t* p) {
    return half_bits_to_float((uint32_t)p[0] | ((uint32_t)p[1] << 8));
}

// Value of column `c` of one packed row of `k` columns.
CL_DEVINL float dequant_at(int type, const uint8_t* row, int k, int c) {
    switch (type) {
    case CL_TYPE_F32: return reinterpret_cast<const float*>(row)[c];
    case CL_TYPE_F16: return load_half(row + 2 * c);
    case CL_TYPE_Q8_0: {
        const int nb = k / 32, b = c / 32;
        const float d = load_half(row + nb * 32 + 2 * b);
        return __fmul_rn((float)(int8_t)row[32 * b + (c & 31)], d);
    }
    case CL_TYPE_Q5_0: {
        const int nb = k / 32, b = c / 32, j = c & 31;
        const float d = load_half(row + nb * 20 + 2 * b);
        const uint8_t* qh8 = row + nb * 16 + 4 * b;
        const uint32_t qh = (uint32_t)qh8[0] | ((uint32_t)qh8[1] << 8) | ((uint32_t)qh8[2] << 16) |
                            ((uint32_t)qh8[3] << 24);
        const uint8_t byte = row[16 * b + (j & 15)];
        const int q = (j < 16 ? (byte & 0x0f) : (byte >> 4)) | (int)(((qh >> j) & 1u) << 4);
        return __fsub_rn(__fmul_rn((float)q, d), __fmul_rn(16.0f, d));
    }
    case CL_TYPE_Q4_K:
    case CL_TYPE_Q5_K: {
        const bool k5 = type == CL_TYPE_Q5_K;
        const uint8_t* blk = row + (c / 256) * (k5 ? 176 : 144);
        const int e = c & 255, g = e >> 6, hi = (e >> 5) & 1, l = e & 31;
        const float d = load_half(blk), dmin = load_half(blk + 2);
        int sc, m;
        kscale_slot(blk + 4, 2 * g + hi, sc, m);
        const uint8_t byte = blk[(k5 ? 48 : 16) + g * 32 + l];
        int q = hi ? (byte >> 4) : (byte & 0x0f);
        if (k5 && (blk[16 + l] & (1u << (2 * g + hi)))) q += 16;
        return __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)m));
    }
    case CL_TYPE_Q6_K: {
        const int nb = k / 256, b = c / 256;
        const uint8_t* blk = row + b * 208;
        const float d = load_half(row + nb * 208 + 2 * b);
        const int e = c & 255, h = e >> 7, r = e & 127, quad = r >> 5, l = r & 31;
        const uint8_t lb = blk[64 * h + (quad & 1) * 32 + l];
        const int low = quad < 2 ? (lb & 0x0f) : (lb >> 4);
        const int high = (blk[128 + 32 * h + l] >> (2 * quad)) & 3;
        const int q = (low | (high << 4)) - 32;
        const int sc = (int8_t)blk[192 + 8 * h + (l >> 4) + 2 * quad];
        return __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
    }
    default: return 0.0f;
    }
}

// ---------------------------------------------------------------------------
// 32 consecutive columns [32 c, 32 c + 32) of one device-layout row, with the
// CPU decoder's FP32 expressions (model.cpp:581-683; Q5_K from
// metal_llm.metal:447-496).  One specialisation per format, fully unrolled.
// ---------------------------------------------------------------------------
CL_DEVINL uint32_t byte_of(const uint32_t (&w)[8], int l) { return (w[l >> 2] >> (8 * (l & 3))) & 0xffu; }

CL_DEVINL void load32(const uint8_t* p, uint32_t (&w)[8]) {
    const uint4 a = *reinterpret_cast<const uint4*>(p), b = *reinterpret_cast<const uint4*>(p + 16);
    w[0] = a.x, w[1] = a.y, w[2] = a.z, w[3] = a.w, w[4] = b.x, w[5] = b.y, w[6] = b.z, w[7] = b.w;
}

template <int T>
CL_DEVINL void dequant32(const uint8_t* row, int k, int c, float (&v)[32]);

template <>
CL_DEVINL void dequant32<CL_TYPE_Q4_K>(const uint8_t* row, int, int c, float (&v)[32]) {
    // sub-block j = c & 7 of super-block c >> 3: nibble (j & 1) of bytes [32 (j >> 1), +32)
    const uint8_t* blk = row + (c >> 3) * 144;
    const int j = c & 7;
    const uint32_t h = *reinterpret_cast<const uint32_t*>(blk);
    const float d = half_bits_to_float(h), dmin = half_bits_to_float(h >> 16);
    int sc, m;
    kscale_slot(blk + 4, j, sc, m);
    const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
    uint32_t q[8];
    load32(blk + 16 + 32 * (j >> 1), q);
    const int sh = 4 * (j & 1);
#pragma unroll
    for (int l = 0; l < 32; ++l) v[l] = __fsub_rn(__fmul_rn(d1, (float)((byte_of(q, l) >> sh) & 15u)), m1);
}

template <>
CL_DEVINL void dequant32<CL_TYPE_Q5_K>(const uint8_t* row, int, int c, float (&v)[32]) {
    const uint8_t* blk = row + (c >> 3) * 176;
    const int j = c & 7;
    const uint32_t h = *reinterpret_cast<const uint32_t*>(blk);
    const float d = half_bits_to_float(h), dmin = half_bits_to_float(h >> 16);
    int sc, m;
    kscale_slot(blk + 4, j, sc, m);
    const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(dmin, (float)m);
    uint32_t q[8], qh[8];
    load32(blk + 48 + 32 * (j >> 1), q);
    load32(blk + 16, qh);
    const int sh = 4 * (j & 1);
#pragma unroll
    for (int l = 0; l < 32; ++l) {
        const uint32_t qv = ((byte_of(q, l) >> sh) & 15u) + (((byte_of(qh, l) >> j) & 1u) << 4);
        v[l] = __fsub_rn(__fmul_rn(d1, (float)qv), m1);
    }
}

template <>
CL_DEVINL void dequant32<CL_TYPE_Q6_K>(const uint8_t* row, int k, int c, float (&v)[32]) {
    // Columns 32 (c & 7) .. of super-block c >> 3: half hh = (c & 7) >> 2,
    // quad = c & 3 (model.cpp:659-683).
    const int nb = k >> 8, b = c >> 3, hh = (c >> 2) & 1, quad = c & 3;
    const uint8_t* blk = row + b * 208;
    const float d = load_half(row + nb * 208 + 2 * b);
    uint32_t ql[8], qh[8];
    load32(blk + 64 * hh + 32 * (quad & 1), ql);
    load32(blk + 128 + 32 * hh, qh);
    const int lsh = quad < 2 ? 0 : 4;
    const uint16_t scw = *reinterpret_cast<const uint16_t*>(blk + 192 + 8 * hh + 2 * quad);
    const float ds0 = __fmul_rn(d, (float)(int8_t)(scw & 0xff)), ds1 = __fmul_rn(d, (float)(int8_t)(scw >> 8));
#pragma unroll
    for (int l = 0; l < 32; ++l) {
        const int qv = ((int)((byte_of(ql, l) >> lsh) & 15u) | (int)(((byte_of(qh, l) >> (2 * quad)) & 3u) << 4)) - 32;
        v[l] = __fmul_rn(l < 16 ? ds0 : ds1, (float)qv);
    }
}

template <>
CL_DEVINL void dequant32<CL_TYPE_Q8_0>(const uint8_t* row, int k, int c, float (&v)[32]) {
    const float d = load_half(row + (k >> 5) * 32 + 2 * c);
    uint32_t q[8];
    load32(row + 32 * c, q);
#pragma unroll
    for (int l = 0; l < 32; ++l) v[l] = __fmul_rn((float)(int8_t)byte_of(q, l), d);
}

template <>
CL_DEVINL void dequant32<CL_TYPE_Q5_0>(const uint8_t* row, int k, int c, float (&v)[32]) {
    const int nb = k >> 5;
    const float d = load_half(row + nb * 20 + 2 * c);
    const float off = __fmul_rn(16.0f, d);
    const uint32_t qh = *reinterpret_cast<const uint32_t*>(row + nb * 16 + 4 * c);
    const uint4 qv = *reinterpret_cast<const uint4*>(row + 16 * c);
    const uint32_t q[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        const uint32_t byte = (q[j >> 2] >> (8 * (j & 3))) & 0xffu;
        const int lo = (int)(byte & 15u) | (int)(((qh >> j) & 1u) << 4);
        const int hi = (int)(byte >> 4) | (int)(((qh >> (j + 16)) & 1u) << 4);
        v[j] = __fsub_rn(__fmul_rn((float)lo, d), off);
        v[16 + j] = __fsub_rn(__fmul_rn((float)hi, d), off);
    }
}

template <>
CL_DEVINL void dequant32<CL_TYPE_F32>(const uint8_t* row, int, int c, float (&v)[32]) {
    const float4* p = reinterpret_cast<const float4*>(row) + 8 * c;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 f = p[i];
        v[4 * i] = f.x, v[4 * i + 1] = f.y, v[4 * i + 2] = f.z, v[4 * i + 3] = f.w;
    }
}

template <>
CL_DEVINL void dequant32<CL_TYPE_F16>(const uint8_t* row, int, int c, float (&v)[32]) {
    const uint4* p = reinterpret_cast<const uint4*>(row + 64 * c);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 u = p[i];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            v[8 * i + 2 * j] = half_bits_to_float(w[j]);
            v[8 * i + 2 * j + 1] = half_bits_to_float(w[j] >> 16);
        }
    }
}

}  // namespace cl
