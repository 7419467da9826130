/*
 * Seeded synthetic weights for GGUF test and benchmark models.
 *
 * Every value is a pure function of (tensor key, element index): a
 * splitmix64 hash feeds a Box-Muller transform, so the bytes written do not
 * depend on the thread count or on the order rows are produced in.  Rows are
 * then packed into native GGML blocks by simple quantizers written for this
 * project.  Any valid block encoding is acceptable here because the readers
 * (the reference CPU dequantizer and the CUDA kernels) decode whatever bytes
 * they are given; the quantizers only need to be deterministic and to keep
 * the dequantized values close to the sampled ones.
 *
 * Block layouts (the on-disk GGML formats, as the reference decodes them in
 * model.cpp:581-683 and metal_llm.metal:447-496):
 *   Q8_0  34 B / 32 : f16 d, int8 q[32]                      x = d*q
 *   Q5_0  22 B / 32 : f16 d, u32 qh, u8 qs[16]               x = d*(q-16)
 *   Q4_K 144 B /256 : f16 d, f16 dmin, u8 sc[12], u8 qs[128] x = d*s*q - dmin*m
 *   Q5_K 176 B /256 : f16 d, f16 dmin, u8 sc[12], u8 qh[32], u8 qs[128]
 *   Q6_K 210 B /256 : u8 ql[128], u8 qh[64], i8 sc[16], f16 d   x = d*sc*(q-32)
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

enum {
    SY_F32 = 0,
    SY_F16 = 1,
    SY_Q5_0 = 6,
    SY_Q8_0 = 8,
    SY_Q4_K = 12,
    SY_Q5_K = 13,
    SY_Q6_K = 14,
};

static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

static inline double unit_open(uint64_t h) {
    /* (0, 1): never 0 so log() stays finite. */
    return ((double)(h >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

/* Standard normal sample for element `index` of the stream `key`. */
static inline double normal_at(uint64_t key, uint64_t index) {
    const uint64_t pair = index >> 1;
    const double u1 = unit_open(mix64(key ^ mix64(2 * pair)));
    const double u2 = unit_open(mix64(key ^ mix64(2 * pair + 1)));
    const double r = sqrt(-2.0 * log(u1));
    const double angle = 6.283185307179586 * u2;
    return (index & 1) ? r * sin(angle) : r * cos(angle);
}

static inline uint16_t f16_bits(float v) {
    _Float16 h = (_Float16)v;
    uint16_t bits;
    memcpy(&bits, &h, 2);
    return bits;
}

static inline float f16_value(float v) {
    return (float)(_Float16)v;
}

static inline void put_u16(uint8_t* p, uint16_t v) {
    p[0] = (uint8_t)(v & 0xff);
    p[1] = (uint8_t)(v >> 8);
}

static inline int clampi(int v, int lo, int hi) {
    return v < lo ? lo : (v > hi ? hi : v);
}

static inline int round_nearest(float v) {
    return (int)lrintf(v);
}

long long synth_row_bytes(int type, long long cols) {
    switch (type) {
    case SY_F32: return cols * 4;
    case SY_F16: return cols * 2;
    case SY_Q5_0: return cols % 32 ? -1 : cols / 32 * 22;
    case SY_Q8_0: return cols % 32 ? -1 : cols / 32 * 34;
    case SY_Q4_K: return cols % 256 ? -1 : cols / 256 * 144;
    case SY_Q5_K: return cols % 256 ? -1 : cols / 256 * 176;
    case SY_Q6_K: return cols % 256 ? -1 : cols / 256 * 210;
    default: return -1;
    }
}

static void quant_q8_0(const float* x, long long cols, uint8_t* out) {
    for (long long b = 0; b < cols / 32; ++b) {
        const float* v = x + b * 32;
        uint8_t* o = out + b * 34;
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
        const float d = f16_value(amax / 127.0f);
        put_u16(o, f16_bits(amax / 127.0f));
        for (int i = 0; i < 32; ++i) {
            const int q = d > 0.0f ? clampi(round_nearest(v[i] / d), -127, 127) : 0;
            o[2 + i] = (uint8_t)(int8_t)q;
        }
    }
}

static void quant_q5_0(const float* x, long long cols, uint8_t* out) {
    for (long long b = 0; b < cols / 32; ++b) {
        const float* v = x + b * 32;
        uint8_t* o = out + b * 22;
        float vmax = 0.0f;
        for (int i = 0; i < 32; ++i) {
            if (fabsf(v[i]) > fabsf(vmax)) vmax = v[i];
        }
        /* q in [0, 31], value = d * (q - 16); the signed extreme maps to 0. */
        const float d = f16_value(vmax / -16.0f);
        put_u16(o, f16_bits(vmax / -16.0f));
        uint32_t qh = 0;
        uint8_t q[32];
        for (int i = 0; i < 32; ++i) {
            q[i] = (uint8_t)(d != 0.0f ? clampi((int)floorf(v[i] / d + 16.5f), 0, 31) : 16);
            if (q[i] & 0x10) qh |= 1u << i;
        }
        o[2] = (uint8_t)(qh & 0xff);
        o[3] = (uint8_t)((qh >> 8) & 0xff);
        o[4] = (uint8_t)((qh >> 16) & 0xff);
        o[5] = (uint8_t)(qh >> 24);
        for (int j = 0; j < 16; ++j) {
            o[6 + j] = (uint8_t)((q[j] & 0x0f) | ((q[j + 16] & 0x0f) << 4));
        }
    }
}

/* Shared 6-bit scale/min packing of Q4_K and Q5_K (the inverse of the
 * reference's get_scale_min_k4, model.cpp:524-537). */
static void pack_scale_min_k4(const int sc[8], const int mn[8], uint8_t s[12]) {
    for (int j = 0; j < 4; ++j) {
        s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        s[j + 4] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
        s[j + 8] = (uint8_t)((sc[j + 4] & 0x0f) | ((mn[j + 4] & 0x0f) << 4));
    }
}

/* Q4_K (levels = 15) and Q5_K (levels = 31): asymmetric sub-blocks of 32. */
static void quant_kmin(const float* v, int levels, uint8_t hdr[16], int q[256]) {
    float scale[8], minv[8];
    float max_scale = 0.0f, max_min = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float lo = 0.0f, hi = -INFINITY;
        for (int i = 0; i < 32; ++i) {
            lo = fminf(lo, v[j * 32 + i]);
            hi = fmaxf(hi, v[j * 32 + i]);
        }
        if (hi < lo) hi = lo;
        scale[j] = (hi - lo) / (float)levels;
        minv[j] = -lo;
        max_scale = fmaxf(max_scale, scale[j]);
        max_min = fmaxf(max_min, minv[j]);
    }
    const float d = f16_value(max_scale / 63.0f);
    const float dmin = f16_value(max_min / 63.0f);
    put_u16(hdr, f16_bits(max_scale / 63.0f));
    put_u16(hdr + 2, f16_bits(max_min / 63.0f));
    int sc[8], mn[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = d > 0.0f ? clampi(round_nearest(scale[j] / d), 0, 63) : 0;
        mn[j] = dmin > 0.0f ? clampi(round_nearest(minv[j] / dmin), 0, 63) : 0;
        /* Keep the sub-block representable when its scale rounds to 0. */
        if (sc[j] == 0 && scale[j] > 0.0f && d > 0.0f) sc[j] = 1;
    }
    pack_scale_min_k4(sc, mn, hdr + 4);
    for (int j = 0; j < 8; ++j) {
        const float ds = d * (float)sc[j];
        const float dm = dmin * (float)mn[j];
        for (int i = 0; i < 32; ++i) {
            q[j * 32 + i] = ds > 0.0f
                ? clampi(round_nearest((v[j * 32 + i] + dm) / ds), 0, levels)
                : 0;
        }
    }
}

static void quant_q4_k(const float* x, long long cols, uint8_t* out) {
    int q[256];
    for (long long b = 0; b < cols / 256; ++b) {
        uint8_t* o = out + b * 144;
        quant_kmin(x + b * 256, 15, o, q);
        uint8_t* qs = o + 16;
        for (int g = 0; g < 4; ++g) {
            for (int l = 0; l < 32; ++l) {
                qs[g * 32 + l] = (uint8_t)(q[g * 64 + l] | (q[g * 64 + 32 + l] << 4));
            }
        }
    }
}

static void quant_q5_k(const float* x, long long cols, uint8_t* out) {
    int q[256];
    for (long long b = 0; b < cols / 256; ++b) {
        uint8_t* o = out + b * 176;
        quant_kmin(x + b * 256, 31, o, q);
        uint8_t* qh = o + 16;
        uint8_t* qs = o + 48;
        memset(qh, 0, 32);
        for (int g = 0; g < 4; ++g) {
            for (int l = 0; l < 32; ++l) {
                const int lo = q[g * 64 + l];
                const int hi = q[g * 64 + 32 + l];
                qs[g * 32 + l] = (uint8_t)((lo & 15) | ((hi & 15) << 4));
                if (lo & 16) qh[l] |= (uint8_t)(1u << (2 * g));
                if (hi & 16) qh[l] |= (uint8_t)(2u << (2 * g));
            }
        }
    }
}

static void quant_q6_k(const float* x, long long cols, uint8_t* out) {
    for (long long b = 0; b < cols / 256; ++b) {
        const float* v = x + b * 256;
        uint8_t* o = out + b * 210;
        float scale[16];
        float max_scale = 0.0f;
        for (int j = 0; j < 16; ++j) {
            float amax = 0.0f;
            for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(v[j * 16 + i]));
            scale[j] = amax / 31.0f;
            max_scale = fmaxf(max_scale, scale[j]);
        }
        const float d = f16_value(max_scale / 127.0f);
        put_u16(o + 208, f16_bits(max_scale / 127.0f));
        int8_t* sc = (int8_t*)(o + 192);
        int q[256];
        for (int j = 0; j < 16; ++j) {
            int s = d > 0.0f ? clampi(round_nearest(scale[j] / d), 0, 127) : 0;
            if (s == 0 && scale[j] > 0.0f && d > 0.0f) s = 1;
            sc[j] = (int8_t)s;
            const float ds = d * (float)s;
            for (int i = 0; i < 16; ++i) {
                q[j * 16 + i] = ds > 0.0f
                    ? clampi(round_nearest(v[j * 16 + i] / ds), -32, 31) + 32
                    : 32;
            }
        }
        uint8_t* ql = o;
        uint8_t* qh = o + 128;
        for (int h = 0; h < 2; ++h) {
            for (int l = 0; l < 32; ++l) {
                const int q1 = q[128 * h + l];
                const int q2 = q[128 * h + 32 + l];
                const int q3 = q[128 * h + 64 + l];
                const int q4 = q[128 * h + 96 + l];
                ql[64 * h + l] = (uint8_t)((q1 & 15) | ((q3 & 15) << 4));
                ql[64 * h + 32 + l] = (uint8_t)((q2 & 15) | ((q4 & 15) << 4));
                qh[32 * h + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) |
                                           ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
            }
        }
    }
}

static int quant_row(int type, const float* x, long long cols, uint8_t* out) {
    switch (type) {
    case SY_F32: memcpy(out, x, (size_t)cols * 4); return 0;
    case SY_F16:
        for (long long i = 0; i < cols; ++i) put_u16(out + 2 * i, f16_bits(x[i]));
        return 0;
    case SY_Q5_0: quant_q5_0(x, cols, out); return 0;
    case SY_Q8_0: quant_q8_0(x, cols, out); return 0;
    case SY_Q4_K: quant_q4_k(x, cols, out); return 0;
    case SY_Q5_K: quant_q5_k(x, cols, out); return 0;
    case SY_Q6_K: quant_q6_k(x, cols, out); return 0;
    default: return -1;
    }
}

/* Fill `rows` x `cols` values mean + std * N(0,1) for stream `key` and pack
 * them as `type`.  Returns 0, or -1 on an unsupported type/shape. */
int synth_fill(uint8_t* dst, int type, long long rows, long long cols,
               unsigned long long key, double mean, double stddev, int threads) {
    const long long rb = synth_row_bytes(type, cols);
    if (rb < 0 || rows < 0 || (cols & 1)) return -1;
    int failed = 0;
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads) reduction(| : failed)
#endif
    {
        float* row = (float*)malloc((size_t)cols * sizeof(float));
        if (!row) {
            failed = 1;
        } else {
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 16)
#endif
            for (long long r = 0; r < rows; ++r) {
                const uint64_t base = (uint64_t)r * (uint64_t)cols;
                for (long long c = 0; c < cols; ++c) {
                    row[c] = (float)(mean + stddev * normal_at(key, base + (uint64_t)c));
                }
                if (quant_row(type, row, cols, dst + r * rb) != 0) failed = 1;
            }
            free(row);
        }
    }
    (void)threads;
    return failed ? -1 : 0;
}

/* Threads of the parallel loops below for the calling thread (a launcher
 * such as torch.distributed.run sets OMP_NUM_THREADS=1 for its ranks; the
 * values written do not depend on the thread count). */
void synth_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#endif
    (void)n;
}

/* Pack caller-provided FP32 rows as `type`. */
int synth_quantize(const float* src, uint8_t* dst, int type, long long rows, long long cols) {
    const long long rb = synth_row_bytes(type, cols);
    if (rb < 0) return -1;
    int failed = 0;
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 16) reduction(| : failed)
#endif
    for (long long r = 0; r < rows; ++r) {
        if (quant_row(type, src + r * cols, cols, dst + r * rb) != 0) failed = 1;
    }
    return failed ? -1 : 0;
}

/* FP32 samples mean + std * N(0,1) for stream `key`. */
void synth_normal_f32(float* dst, long long n, unsigned long long key, double mean, double stddev) {
#ifdef _OPENMP
#pragma omp parallel for schedule(static)
#endif
    for (long long i = 0; i < n; ++i) {
        dst[i] = (float)(mean + stddev * normal_at(key, (uint64_t)i));
    }
}

/* -exp(N(mu, sigma)): strictly negative values (DeltaNet ssm_a). */
void synth_negexp_f32(float* dst, long long n, unsigned long long key, double mu, double sigma) {
    for (long long i = 0; i < n; ++i) {
        dst[i] = (float)(-exp(mu + sigma * normal_at(key, (uint64_t)i)));
    }
}

/* Uniform integers in [0, bound) for stream `key` (token ids). */
void synth_uniform_ids(int* dst, long long n, unsigned long long key, long long bound) {
    for (long long i = 0; i < n; ++i) {
        dst[i] = (int)(mix64(key ^ mix64((uint64_t)i)) % (uint64_t)bound);
    }
}

unsigned long long synth_mix64(unsigned long long v) {
    return mix64(v);
}
