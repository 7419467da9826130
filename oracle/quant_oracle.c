/*
 * ORACLE — test infrastructure only.  Nothing in the product links this file;
 * it is loaded by tests/ and by bench.py's CPU-baseline leg as the checker.
 *
 * A plain-C restatement of the reference's CPU arithmetic for the quantized
 * projections:
 *   - block decoders with the reference's exact FP32 expressions
 *       Q5_0  model.cpp:581-601   (q|h) * d - 16 * d
 *       Q8_0  model.cpp:603-614   q * d
 *       Q4_K  model.cpp:616-644   (d * sc) * q - (dmin * m)   [get_scale_min_k4 524-537]
 *       Q6_K  model.cpp:646-683   (d * sc) * (q - 32)
 *       F16   model.cpp:500-522   half_to_float
 *       Q5_K  metal_llm.metal:447-496 (no CPU decoder in the reference; the
 *             element value d*sc*q - dmin*m with the fifth bit from qh)
 *   - FP32 dequantize-then-matmul with the loop order of gevmtb / gemmtb
 *     (cpu_llm.cpp:528-547, 631-653): one row dequantized, then a sequential
 *     FP32 accumulation over the columns in index order, bias added last.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { OR_F32 = 0, OR_F16 = 1, OR_Q5_0 = 6, OR_Q8_0 = 8, OR_Q4_K = 12, OR_Q5_K = 13, OR_Q6_K = 14 };

static uint16_t u16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

static float half_value(uint16_t v) {
    const uint32_t sign = v >> 15, exponent = (v >> 10) & 0x1f, mantissa = v & 0x3ff;
    float r;
    if (exponent == 0) {
        r = mantissa == 0 ? 0.0f : ldexpf((float)mantissa / 1024.0f, -14);
    } else if (exponent == 31) {
        r = mantissa == 0 ? INFINITY : NAN;
    } else {
        r = ldexpf(1.0f + (float)mantissa / 1024.0f, (int)exponent - 15);
    }
    return sign ? -r : r;
}

static void scale_min_k4(int i, const uint8_t* s, uint8_t* sc, uint8_t* m) {
    if (i < 4) {
        *sc = s[i] & 63;
        *m = s[i + 4] & 63;
    } else {
        *sc = (uint8_t)((s[i + 4] & 0x0f) | ((s[i - 4] >> 6) << 4));
        *m = (uint8_t)((s[i + 4] >> 4) | ((s[i] >> 6) << 4));
    }
}

long long oracle_row_bytes(int type, long long cols) {
    switch (type) {
    case OR_F32: return cols * 4;
    case OR_F16: return cols * 2;
    case OR_Q5_0: return cols % 32 ? -1 : cols / 32 * 22;
    case OR_Q8_0: return cols % 32 ? -1 : cols / 32 * 34;
    case OR_Q4_K: return cols % 256 ? -1 : cols / 256 * 144;
    case OR_Q5_K: return cols % 256 ? -1 : cols / 256 * 176;
    case OR_Q6_K: return cols % 256 ? -1 : cols / 256 * 210;
    default: return -1;
    }
}

int oracle_dequant_row(int type, const uint8_t* data, long long cols, float* out) {
    if (oracle_row_bytes(type, cols) < 0) return -1;
    switch (type) {
    case OR_F32:
        memcpy(out, data, (size_t)cols * 4);
        return 0;
    case OR_F16:
        for (long long i = 0; i < cols; ++i) out[i] = half_value(u16(data + 2 * i));
        return 0;
    case OR_Q5_0:
        for (long long b = 0; b < cols / 32; ++b) {
            const uint8_t* p = data + b * 22;
            const float d = half_value(u16(p));
            const uint32_t qh = (uint32_t)p[2] | ((uint32_t)p[3] << 8) |
                                ((uint32_t)p[4] << 16) | ((uint32_t)p[5] << 24);
            for (int j = 0; j < 16; ++j) {
                const int h0 = (int)(((qh >> j) << 4) & 0x10);
                const int h1 = (int)((qh >> (j + 12)) & 0x10);
                out[b * 32 + j] = (float)((p[6 + j] & 0x0f) | h0) * d - 16.0f * d;
                out[b * 32 + j + 16] = (float)((p[6 + j] >> 4) | h1) * d - 16.0f * d;
            }
        }
        return 0;
    case OR_Q8_0:
        for (long long b = 0; b < cols / 32; ++b) {
            const uint8_t* p = data + b * 34;
            const float d = half_value(u16(p));
            for (int j = 0; j < 32; ++j) out[b * 32 + j] = (float)(int8_t)p[2 + j] * d;
        }
        return 0;
    case OR_Q4_K:
    case OR_Q5_K: {
        const int bs = type == OR_Q4_K ? 144 : 176;
        for (long long b = 0; b < cols / 256; ++b) {
            const uint8_t* p = data + b * bs;
            const float d = half_value(u16(p));
            const float dmin = half_value(u16(p + 2));
            const uint8_t* s = p + 4;
            const uint8_t* qh = type == OR_Q5_K ? p + 16 : NULL;
            const uint8_t* qs = p + (type == OR_Q5_K ? 48 : 16);
            for (int g = 0; g < 4; ++g) {
                uint8_t sc0, m0, sc1, m1;
                scale_min_k4(2 * g, s, &sc0, &m0);
                scale_min_k4(2 * g + 1, s, &sc1, &m1);
                const float d1 = d * sc0, mm1 = dmin * m0;
                const float d2 = d * sc1, mm2 = dmin * m1;
                for (int l = 0; l < 32; ++l) {
                    int lo = qs[g * 32 + l] & 0x0f, hi = qs[g * 32 + l] >> 4;
                    if (qh) {
                        lo += (qh[l] & (1u << (2 * g))) ? 16 : 0;
                        hi += (qh[l] & (2u << (2 * g))) ? 16 : 0;
                    }
                    out[b * 256 + g * 64 + l] = d1 * (float)lo - mm1;
                    out[b * 256 + g * 64 + 32 + l] = d2 * (float)hi - mm2;
                }
            }
        }
        return 0;
    }
    case OR_Q6_K:
        for (long long b = 0; b < cols / 256; ++b) {
            const uint8_t* p = data + b * 210;
            const uint8_t* ql = p;
            const uint8_t* qh = p + 128;
            const int8_t* sc = (const int8_t*)(p + 192);
            const float d = half_value(u16(p + 208));
            float* o = out + b * 256;
            for (int n = 0; n < 256; n += 128) {
                for (int l = 0; l < 32; ++l) {
                    const int is = l / 16;
                    const int q1 = ((ql[l] & 0x0f) | ((qh[l] & 3) << 4)) - 32;
                    const int q2 = ((ql[l + 32] & 0x0f) | (((qh[l] >> 2) & 3) << 4)) - 32;
                    const int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                    const int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                    o[n + l] = d * sc[is + 0] * q1;
                    o[n + l + 32] = d * sc[is + 2] * q2;
                    o[n + l + 64] = d * sc[is + 4] * q3;
                    o[n + l + 96] = d * sc[is + 6] * q4;
                }
                ql += 64;
                qh += 32;
                sc += 8;
            }
        }
        return 0;
    }
    return -1;
}

int oracle_dequant(int type, const uint8_t* data, long long rows, long long cols, float* out) {
    const long long rb = oracle_row_bytes(type, cols);
    if (rb < 0) return -1;
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
    for (long long r = 0; r < rows; ++r) {
        bad |= oracle_dequant_row(type, data + r * rb, cols, out + r * cols) != 0;
    }
    return bad ? -1 : 0;
}

/* Y[m, n] = sum_k X[m, k] * W[n, k] (+ bias[n]), W dequantized per row. */
int oracle_gemm(int type, const uint8_t* w, long long n, long long k, const float* x,
                long long m, const float* bias, float* y) {
    const long long rb = oracle_row_bytes(type, k);
    if (rb < 0) return -1;
    int bad = 0;
#pragma omp parallel reduction(| : bad)
    {
        float* row = (float*)malloc((size_t)k * sizeof(float));
        if (!row) bad = 1;
#pragma omp for schedule(dynamic, 8)
        for (long long r = 0; r < n; ++r) {
            if (!row) continue;
            oracle_dequant_row(type, w + r * rb, k, row);
            for (long long i = 0; i < m; ++i) {
                float acc = 0.0f;
                const float* xi = x + i * k;
                for (long long c = 0; c < k; ++c) acc += xi[c] * row[c];
                if (bias) acc += bias[r];
                y[i * n + r] = acc;
            }
        }
        free(row);
    }
    return bad ? -1 : 0;
}
