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

}  // namespace cl
