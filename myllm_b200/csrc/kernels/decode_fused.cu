// One batch-1 decode step of a qwen2 model in one persistent launch.
//
// Reference: the decode graph of cpu_decode_layer x n_layers + final norm +
// LM head + greedy token (cpu_llm.cpp:843-914, 1051-1070) and Metal
// encode_decode_layer (metal_llm.mm:2758-2904).  Same products and the same
// expressions as the per-operator kernels of this library (the K-quant GEMV
// of gemv_mma.cu with its exact integer dots, RMSNorm summed in double,
// attention as in attn.cu), arranged for the B200 instead of as one launch
// per operator:
//
// * One CTA per SM (cooperative launch, so all CTAs are resident), 12 warps.
//   The step is a fixed sequence of phases: per layer QKV, attention, o_proj,
//   gate/up, down; then the LM head.  Phases are separated by grid barriers
//   (an arrival counter; every wait bounded by a 2 s clock and an abort flag).
// * A GEMV phase is a list of units: 16 output rows x one super-block
//   (Q4_K) or one half super-block (Q6_K); for gate/up, 8 gate + 8 up rows
//   (one m16 MMA computes both, so the SwiGLU pair meets in one lane).  The
//   units of a phase are split into equal contiguous ranges, one per warp of
//   the grid (stream-K), so every SM streams the same bytes of every matrix.
// * Each warp owns a 4-slot shared-memory ring that it fills itself with
//   cp.async (no hand-off between warps).  The ring runs ahead through the
//   warp's units of the following phases: weights never depend on the
//   activations, so while the grid waits at a barrier, or encodes the next
//   input vector, the next matrix is already in flight.
// * At a phase start every CTA reads the input vector (RMS-normalised where
//   the layer says so) and encodes it into the XQ4 limbs in shared memory,
//   exactly as gemv_mma.cu does.
// * A tile (16 rows) whose units span several warps is summed through a
//   global partial buffer: each warp stores its partial and takes a ticket;
//   the last one adds the partials in warp order (deterministic) and writes
//   the rows (bias, residual, SwiGLU, argmax candidates).
// * Attention: CTA (KV head, key split) rotates its query heads, appends the
//   new key / value at the current position, runs an online softmax over its
//   keys in 64-key tiles and leaves (m, l, o) partials; the last split of a
//   KV head (ticket) merges them.  During attention the other warps' rings
//   keep prefetching o_proj.
// * Head: logits for every row, and per row a (value, index) candidate; the
//   last CTA to finish merges the CTAs' candidates (lowest index on ties),
//   writes the token, advances the position and re-arms the control block.
#include "common.cuh"
#include "dequant.cuh"
#include "gemv_mma.cuh"
#include "launch.cuh"

#include <algorithm>

namespace cl {
namespace dfz {

using gmma::Q4Lane;

constexpr int kW = 8;                   // warps per CTA
constexpr int kThreads = kW * 32;
constexpr int kSlots = 3;               // ring depth per warp
// Shared row strides of a unit in a ring slot, each chosen so the MMA
// fragment reads are bank-conflict free: Q4_K 2 x 144 B rows read as 8-byte
// words (stride % 64 == 32), Q6_K 2 x 112 B rows read as 4-byte words
// (stride / 4 = 60: rows 0-7 start 4 banks apart).
constexpr int kRS4 = 288;
constexpr int kRS6 = 240;
constexpr int kSlotBytes = 16 * kRS4;
constexpr int kRingBytes = kW * kSlots * kSlotBytes;
constexpr int kXBlocksPerWarp = 10;     // x blocks one warp encodes: k <= 8 * 10 * 256
constexpr int kMaxK = kW * kXBlocksPerWarp * 256;
constexpr int kNormBlocks = 3;          // RMS-normalised inputs: k <= 8 * 3 * 256
constexpr int kSplitsMax = 32;          // key splits per KV head (one warp merges their weights)
constexpr int kSplitKeys = 16;          // automatic splits: at least this many keys each
constexpr int kGMax = 8;                // query heads per KV head
constexpr int kD = 128;                 // head dim
constexpr int kKT = 64;                 // keys per attention tile
constexpr int kQLD = kD + 4;            // padded q / K rows (bank-conflict-free score loop)
constexpr int kRec = kD + 4;            // a split's record per query head: m, l, 2 pad, o[kD]
constexpr int kRedUnits = 64;           // tile mode: a CTA's units (16 partial rows each in shared memory)
constexpr int kMaxKvHeads = 32;
constexpr unsigned long long kWaitNs = 2000ull * 1000 * 1000;
// Optional trace, per CTA and phase: [0] start, [1] input ready, [2] work
// done, [3 .. 3 + kW) each warp's last unit computed; in attention phases
// [11 .. 15) points inside attention (K/V landed, scores and PV done,
// partials published, combined); in projection phases [11 .. 15) warp 0's
// SM cycles waiting for its ring, computing, issuing loads and flushing
// tiles in its unit loop, and [15] its unit count.
constexpr int kTraceSlots = 16;

// Control block at the head of the workspace; zero between steps.
struct Ctl {
    unsigned int bar;    // grid-barrier arrivals of this step
    unsigned int done;   // CTAs that finished the head phase
    int error;           // 0, or 1 + the phase whose barrier wait ran out
    int abort;
    unsigned int attn_ticket[kMaxKvHeads];
    unsigned int pad[28];
};
static_assert(sizeof(Ctl) == 256, "control block is 256 bytes");

struct Seg {
    const uint8_t* w;     // the matrix in the tiled decode layout (cl_decode_pack)
    const float* bias;
    float* y;
    long long u0;         // first unit of the segment in its phase
    int type, nsub, tile0, tiles, sw;
};

struct Phase {
    Seg seg[3];
    long long U;          // units in the phase
    const float* x;       // input vector; null in layer 0's QKV (the embedding row)
    const float* gamma;   // RMSNorm weight, or null
    const float* gamma_out;  // the next GEMV's RMSNorm weight over this phase's output, or null
    int nseg, nb, K, sw, head, residual, attn;
    int ctile;            // whole tiles per CTA (tile c, c + grid, ...; the CTA's warps take its
                          // units in turn and add them up in shared memory), else warp ranges
    int ntiles;
    int in_buf;           // encoded input buffer (0 / 1), or -1: encode here (layer 0's embedding)
    int out_buf;          // buffer this phase's output is encoded into, or -1
    int out_target;       // tile (or head) completions per 256-row output block
};

struct Params {
    const cl_qwen2_layer* layers;
    int n_layers, H, F, V, hq, hkv, cap, max_tiles;
    float eps, scale;
    const uint8_t* embd;
    long long embd_stride;
    int embd_type, out_type;
    const uint8_t* out_w;
    const float* out_norm;
    const float* rope;
    int* ints;
    float *h, *q, *k, *v, *att, *act, *logits;
    Ctl* ctl;
    unsigned int* tickets;  // [max_tiles]
    float2* records;        // [grid] head candidates (value, index as float bits)
    float* partials;        // [grid * kW][2][16]
    float* attn_part;       // [hkv][kSplitsMax][G][kRec]
    long long* trace;       // optional [grid][phases][3] timestamps
    uint8_t* enc[2];        // encoded vectors: [nb_max] limbs (1 KB) | xs | xsum [8] | ssq (double)
    unsigned int* enc_cnt;  // [2][nb_max] block completions
    int nb_max;
    int region_bytes;
    int attn_off;           // attention's part of the region: after the QKV input, so that the
                            // first key tile can land while the QKV phase still reads its input
    int splits;             // key splits per KV head requested (0: automatic)
};

// Planes of an encoded-vector buffer of nb_max blocks.
struct EncView {
    uint8_t* xq;
    float* xs;
    float* xsum;
    double* ssq;
};

__host__ __device__ inline size_t enc_bytes(int nb_max) {
    return (size_t)nb_max * 1024 + (((size_t)nb_max * 4 + 15) & ~(size_t)15) + (size_t)nb_max * 32 +
           (size_t)nb_max * 8;
}

CL_DEVINL EncView enc_view(const Params& P, int buf) {
    uint8_t* b = P.enc[buf];
    EncView v;
    v.xq = b;
    v.xs = reinterpret_cast<float*>(b + (size_t)P.nb_max * 1024);
    v.xsum = reinterpret_cast<float*>(b + (size_t)P.nb_max * 1024 + (((size_t)P.nb_max * 4 + 15) & ~(size_t)15));
    v.ssq = reinterpret_cast<double*>(reinterpret_cast<uint8_t*>(v.xsum) + (size_t)P.nb_max * 32);
    return v;
}

// Bytes of one unit (16 rows) in the tiled decode layout: Q4_K two
// super-blocks (2 x 144 B per row), Q6_K one super-block as two 112-byte
// halves per row.
__host__ __device__ constexpr int unit_bytes(int type) { return type == CL_TYPE_Q4_K ? 16 * 288 : 16 * 224; }

CL_DEVINL void set_seg(Seg& s, const void* w, bool sw, int type, int rows, int nb, const float* bias, float* y,
                       long long& u, int& tile) {
    s.w = static_cast<const uint8_t*>(w);
    s.sw = sw;
    s.bias = bias;
    s.y = y;
    s.type = type;
    s.nsub = type == CL_TYPE_Q4_K ? (nb + 1) / 2 : nb;
    s.tiles = sw ? rows / 8 : rows / 16;
    s.u0 = u;
    s.tile0 = tile;
    u += (long long)s.tiles * s.nsub;
    tile += s.tiles;
}

// Phase p: 5 per layer (QKV, attention, o_proj, gate/up, down), then the head.
CL_DEVINL void make_phase(const Params& P, int p, Phase& ph) {
    long long u = 0;
    int tile = 0;
    ph.x = nullptr;
    ph.gamma = nullptr;
    ph.gamma_out = nullptr;
    ph.nseg = 1;
    ph.sw = ph.head = ph.residual = ph.attn = ph.ctile = 0;
    ph.U = 0;
    // The encoded input of every GEMV phase but the first was written by the
    // phase before it (buffers alternate by phase parity).
    ph.in_buf = p == 0 ? -1 : (p - 1) & 1;
    ph.out_buf = -1;
    ph.out_target = 0;
    const int d = kD;
    if (p >= 5 * P.n_layers) {
        ph.nb = P.H / 256;
        ph.K = P.H;
        ph.x = P.h;
        ph.gamma = P.out_norm;
        ph.head = 1;
        set_seg(ph.seg[0], P.out_w, false, P.out_type, P.V, ph.nb, nullptr, P.logits, u, tile);
        ph.U = u;
        return;
    }
    const cl_qwen2_layer& L = P.layers[p / 5];
    switch (p % 5) {
    case 0:
        ph.nb = P.H / 256;
        ph.K = P.H;
        ph.x = p == 0 ? nullptr : P.h;
        ph.gamma = L.attn_norm;
        ph.nseg = 3;
        set_seg(ph.seg[0], L.q, false, L.q_type, P.hq * d, ph.nb, L.q_bias, P.q, u, tile);
        set_seg(ph.seg[1], L.k, false, L.k_type, P.hkv * d, ph.nb, L.k_bias, P.k, u, tile);
        set_seg(ph.seg[2], L.v, false, L.v_type, P.hkv * d, ph.nb, L.v_bias, P.v, u, tile);
        ph.ctile = 1;
        break;
    case 1:  // attention output, encoded per block of two 128-wide heads
        ph.attn = 1;
        ph.nb = 0;
        ph.K = 0;
        ph.out_buf = p & 1;
        ph.out_target = 256 / kD;
        break;
    case 2:  // o_proj: h, encoded with ffn_norm for gate / up
        ph.nb = P.H / 256;
        ph.K = P.H;
        ph.x = P.att;
        ph.residual = 1;
        ph.gamma_out = L.ffn_norm;
        ph.out_buf = p & 1;
        ph.out_target = 256 / 16;
        set_seg(ph.seg[0], L.o, false, L.o_type, P.H, ph.nb, nullptr, P.h, u, tile);
        ph.ctile = 1;
        break;
    case 3:  // gate / up: act, 8-row tiles
        ph.nb = P.H / 256;
        ph.K = P.H;
        ph.x = P.h;
        ph.gamma = L.ffn_norm;
        ph.sw = 1;
        ph.out_buf = p & 1;
        ph.out_target = 256 / 8;
        set_seg(ph.seg[0], L.gate, true, L.gate_type, P.F, ph.nb, nullptr, P.act, u, tile);
        break;
    default:  // down: h, encoded with the next layer's attn_norm (or output_norm)
        ph.nb = P.F / 256;
        ph.K = P.F;
        ph.x = P.act;
        ph.residual = 1;
        ph.gamma_out = p / 5 + 1 < P.n_layers ? P.layers[p / 5 + 1].attn_norm : P.out_norm;
        ph.out_buf = p & 1;
        ph.out_target = 256 / 16;
        set_seg(ph.seg[0], L.down, false, L.down_type, P.H, ph.nb, nullptr, P.h, u, tile);
        break;
    }
    ph.U = u;
    ph.ntiles = tile;
    if (ph.ctile) {
        // tile mode while a CTA's units fit the shared partial sums
        int nsub_max = 0;
        for (int i = 0; i < ph.nseg; ++i) nsub_max = max(nsub_max, ph.seg[i].nsub);
        const int per_cta = (tile + (int)gridDim.x - 1) / (int)gridDim.x;
        ph.ctile = per_cta * nsub_max <= kRedUnits;
    }
}

// A warp's position in its range of a phase: unit j of tile `tile` of
// segment s, `left` units to go.  Advanced without divisions.
struct Cursor {
    int s, tile, j, left;
};

CL_DEVINL Cursor cursor_at(const Phase& ph, long long u, long long e) {
    int s = 0;
    if (ph.nseg > 1 && u >= ph.seg[1].u0) s = 1;
    if (ph.nseg > 2 && u >= ph.seg[2].u0) s = 2;
    const int local = (int)(u - ph.seg[s].u0);
    const int ns = ph.seg[s].nsub;
    return Cursor{s, local / ns, local % ns, (int)(e - u)};
}

CL_DEVINL void cursor_next(const Phase& ph, Cursor& c) {
    --c.left;
    if (++c.j == ph.seg[c.s].nsub) {
        c.j = 0;
        if (++c.tile == ph.seg[c.s].tiles) {
            c.tile = 0;
            ++c.s;
        }
    }
}

// Tile mode: global tile index -> (segment, tile in segment); false past the end.
CL_DEVINL bool tile_locate(const Phase& ph, int tg, int& s, int& tile) {
    if (tg >= ph.ntiles) return false;
    s = 0;
    if (ph.nseg > 1 && tg >= ph.seg[1].tile0) s = 1;
    if (ph.nseg > 2 && tg >= ph.seg[2].tile0) s = 2;
    tile = tg - ph.seg[s].tile0;
    return true;
}

// Tile mode: the CTA's units in order (its tiles c, c + grid, ..., each
// tile's units in turn), position `pos` onward in steps of kW; `left` the
// positions of this warp still to go.
CL_DEVINL Cursor cursor_ctile(const Phase& ph, int pos) {
    int s = 0, tile = 0, total = 0;
    for (int tg = blockIdx.x; tile_locate(ph, tg, s, tile); tg += gridDim.x) total += ph.seg[s].nsub;
    Cursor c{0, 0, 0, pos < total ? (total - pos + kW - 1) / kW : 0};
    if (c.left == 0) return c;
    int tg = blockIdx.x;
    tile_locate(ph, tg, c.s, c.tile);
    c.j = pos;
    while (c.j >= ph.seg[c.s].nsub) {
        c.j -= ph.seg[c.s].nsub;
        tg += gridDim.x;
        tile_locate(ph, tg, c.s, c.tile);
    }
    return c;
}

CL_DEVINL void cursor_ctile_next(const Phase& ph, Cursor& c) {
    if (--c.left == 0) return;
    c.j += kW;
    int tg = ph.seg[c.s].tile0 + c.tile;
    while (c.j >= ph.seg[c.s].nsub) {
        c.j -= ph.seg[c.s].nsub;
        tg += gridDim.x;
        tile_locate(ph, tg, c.s, c.tile);
    }
}

// Range [begin(w), begin(w + 1)) of the grid's warp w over U units.
CL_DEVINL long long range_begin(long long U, int w, int GW) { return U * w / GW; }
// The warp whose range holds unit u.
CL_DEVINL int warp_of(long long U, long long u, int GW) { return (int)(((u + 1) * GW - 1) / U); }

// First byte of a unit: units are stored tile by tile, each 16 rows x the
// unit's bytes per row, contiguous.
CL_DEVINL const uint8_t* unit_src(const Seg& sg, int tile, int j) {
    return sg.w + ((long long)tile * sg.nsub + j) * unit_bytes(sg.type);
}

CL_DEVINL void cp16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
CL_DEVINL void cp8(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
CL_DEVINL void cp4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
// Weights are read once per step: evict-first keeps the KV cache, the
// activations and the partials resident in L2 meanwhile.
CL_DEVINL void cp16_stream(void* dst, const void* src, uint64_t policy) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "l"(policy)
                 : "memory");
}
CL_DEVINL uint64_t evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
CL_DEVINL void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
CL_DEVINL void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
CL_DEVINL void cp_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

CL_DEVINL void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// The lane's share of a unit's 16-byte pieces: a unit is 16 rows of 18
// (Q4_K: 288 B) or 14 (Q6_K: 224 B) pieces, contiguous in global memory;
// piece c goes to row c / P, offset 16 (c % P) of the slot's padded rows.
// Pieces lane + 32 i, fixed per lane (Q4_K: 9 each, Q6_K: 7 each).  (Per
// lane cp.async measured faster here than one bulk copy per unit, and much
// faster than one per 224-byte Q6_K row.)
struct LanePlan {
    int dst4[9];
    int dst6[7];
};

CL_DEVINL LanePlan lane_plan(int lane) {
    LanePlan pl;
#pragma unroll
    for (int i = 0; i < 9; ++i) {
        const int c = lane + 32 * i;
        pl.dst4[i] = (c / 18) * kRS4 + 16 * (c % 18);
    }
#pragma unroll
    for (int i = 0; i < 7; ++i) {
        const int c = lane + 32 * i;
        pl.dst6[i] = (c / 14) * kRS6 + 16 * (c % 14);
    }
    return pl;
}

// The lane's copies of the cursor's unit into a ring slot.  Row layout in
// the slot: Q4_K (stride kRS4) super-blocks 2j and 2j + 1, 144 bytes each;
// Q6_K (stride kRS6) the two halves of super-block j, 112 bytes each: ql of
// the half at 0, qh at 64, sc at 96, the block's f16 d at 104.
CL_DEVINL void issue_unit(const Phase& ph, const Cursor& cu, uint8_t* slot, int lane, const LanePlan& pl,
                          uint64_t policy) {
    const Seg& sg = ph.seg[cu.s];
    const uint8_t* src = unit_src(sg, cu.tile, cu.j) + 16 * lane;
    if (sg.type == CL_TYPE_Q4_K) {
#pragma unroll
        for (int i = 0; i < 9; ++i) cp16_stream(slot + pl.dst4[i], src + 512 * i, policy);
    } else {
#pragma unroll
        for (int i = 0; i < 7; ++i) cp16_stream(slot + pl.dst6[i], src + 512 * i, policy);
    }
}

// Q6_K value bytes v in [0, 63] -> v - 32 as signed bytes, four at a time
// (v | 0x80 never borrows when 0x20 is taken away; xor 0x80 restores).
CL_DEVINL uint32_t q6_signed(uint32_t v) { return ((v | 0x80808080u) - 0x20202020u) ^ 0x80808080u; }

// Half hh of one Q6_K super-block for 16 rows (the layout of issue_unit),
// on s8 x s8 MMAs (q - 32 in the weights).  p0 / p1: the lane's B bases in
// the XQ4 block (the zero block for the other column half).
CL_DEVINL void q6k_half(const uint8_t* bg, const uint8_t* b8, const uint8_t* p0, const uint8_t* p1, int hh,
                        int sb, float xs, int t, int h, const Q4Lane& L6, float& yg, float& y8) {
    int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
    for (int s = 0; s < 2; ++s) {
        const uint32_t qg = *reinterpret_cast<const uint32_t*>(bg + 64 + 16 * s + 4 * t);
        const uint32_t q8 = *reinterpret_cast<const uint32_t*>(b8 + 64 + 16 * s + 4 * t);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint32_t lg = *reinterpret_cast<const uint32_t*>(bg + 32 * j + 16 * s + 4 * t);
            const uint32_t l8 = *reinterpret_cast<const uint32_t*>(b8 + 32 * j + 16 * s + 4 * t);
            const uint32_t hag = (j ? (qg << 2) : (qg << 4)) & 0x30303030u;
            const uint32_t ha8 = (j ? (q8 << 2) : (q8 << 4)) & 0x30303030u;
            const uint32_t hbg = (j ? (qg >> 2) : qg) & 0x30303030u;
            const uint32_t hb8 = (j ? (q8 >> 2) : q8) & 0x30303030u;
            const int boff = 512 * hh + 128 * j + 16 * s;
            const uint32_t b0 = *reinterpret_cast<const uint32_t*>(p0 + boff);
            const uint32_t b1 = *reinterpret_cast<const uint32_t*>(p1 + boff);
            int c[4];
            gmma::mma_s8s8_z(c, q6_signed((lg & 0x0f0f0f0fu) | hag), q6_signed((l8 & 0x0f0f0f0fu) | ha8),
                             q6_signed(((lg >> 4) & 0x0f0f0f0fu) | hbg), q6_signed(((l8 >> 4) & 0x0f0f0f0fu) | hb8),
                             b0, b1);
            const int sci = 96 + s + 2 * j + 4 * h;
            const int sg = (int)*reinterpret_cast<const int8_t*>(bg + sci);
            const int s8 = (int)*reinterpret_cast<const int8_t*>(b8 + sci);
            a0 += c[0] * sg;
            a1 += c[1] * sg;
            a2 += c[2] * s8;
            a3 += c[3] * s8;
        }
    }
    const float dg = half_bits_to_float(*reinterpret_cast<const uint16_t*>(bg + 104));
    const float d8 = half_bits_to_float(*reinterpret_cast<const uint16_t*>(b8 + 104));
    const float vg = fmaf((float)a0, L6.lw0, (float)a1 * L6.lw1) * xs;
    const float v8 = fmaf((float)a2, L6.lw0, (float)a3 * L6.lw1) * xs;
    yg = fmaf(dg, vg, yg);
    y8 = fmaf(d8, v8, y8);
}

CL_DEVINL unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// One-step publication: the add is a release of this thread's earlier
// writes (and, through the preceding warp / CTA barrier, of the other
// threads'), the returned count an acquire of the other adders' writes.
CL_DEVINL unsigned int atom_add_acq_rel(unsigned int* p, unsigned int v) {
    unsigned int old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
CL_DEVINL void red_add_release(unsigned int* p, unsigned int v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

CL_DEVINL unsigned int ld_acquire(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct Best {
    float v;
    int i;
    CL_DEVINL void consider(float y, int o) {
        if (y > v || (y == v && o < i)) {
            v = y;
            i = o;
        }
    }
};

CL_DEVINL bool better(float v1, int i1, float v2, int i2) { return v1 > v2 || (v1 == v2 && i1 < i2); }

// Rows of a finished tile: lanes with t == 0 hold rows g (vg) and g + 8 (v8).
// Bias and residual of the lane's two rows of a tile, loaded when the warp
// starts the tile so that no load waits at its end.
struct RowPre {
    float b[2], r[2];
};

CL_DEVINL RowPre row_pre(const Phase& ph, const Seg& sg, int tile_l, int g, int t) {
    RowPre pr{{0.0f, 0.0f}, {0.0f, 0.0f}};
    if (t == 0 && !ph.sw) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int o = tile_l * 16 + g + 8 * i;
            if (sg.bias) pr.b[i] = sg.bias[o];
            if (ph.residual) pr.r[i] = __ldcg(sg.y + o);
        }
    }
    return pr;
}

CL_DEVINL void tile_out(const Phase& ph, const Seg& sg, int tile_l, int g, float vg, float v8, Best& best,
                        const RowPre& pr) {
    if (ph.sw) {
        // Branch-stable SiLU(gate) * up (cpu_llm.cpp:188-202), as gemv_mma.cu.
        const int o = tile_l * 8 + g;
        const float sig = vg >= 0.0f ? 1.0f / (1.0f + expf(-vg)) : expf(vg) / (1.0f + expf(vg));
        sg.y[o] = __fmul_rn(__fmul_rn(vg, sig), v8);
        return;
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int o = tile_l * 16 + g + 8 * i;
        float y = i ? v8 : vg;
        if (sg.bias) y += pr.b[i];
        if (ph.residual) y = pr.r[i] + y;
        sg.y[o] = y;
        if (ph.head) best.consider(y, o);
    }
}

struct Smem {
    uint8_t* ring;
    uint8_t* region;
    const uint8_t* zero;
    float* red;    // [kRedUnits][16] tile mode: each unit's 16 row sums
    Phase* pc;     // [kPhaseCache] descriptors of the coming phases: phase q in slot q % kPhaseCache
    Phase* wph;    // [kW] the phase each warp is issuing from
    double* dred;  // [kW]
    float2* bests; // [kW]
    int* flags;    // [0] barrier ok, [1] last-of-split / last CTA, [4 ..) the phase in each cache slot
    uint64_t* xbar;  // completion of the encoded-input bulk copies
};

// Phase descriptors are built from the layer table in global memory (a few
// dependent loads); thread 0 builds them kPhaseCache - 1 phases ahead, while
// the grid waits at a barrier, so that no warp builds one in its unit loop.
constexpr int kPhaseCache = 4;
constexpr int kPhaseWords = (int)(sizeof(Phase) / 8);
static_assert(sizeof(Phase) % 8 == 0 && kPhaseWords <= 32, "a phase descriptor is copied by one warp, 8 B a lane");

// ---- encode the phase's input into XQ4 limbs (all warps) -------------------
CL_DEVINL void encode_input(const Params& P, const Phase& ph, const Smem& S, int tok, int warp, int lane) {
    const int nb = ph.nb;
    uint8_t* xq = S.region;
    float* xs = reinterpret_cast<float*>(S.region + nb * 1024);
    float* xsum = reinterpret_cast<float*>(S.region + nb * 1024 + ((nb * 4 + 15) & ~15));
    if (ph.gamma) {
        // RMS-normalised input (k = hidden <= kW * kNormBlocks * 256): x and
        // gamma loads all in flight together, then cpu_llm.cpp:156-165's
        // arithmetic: sum of squares in double, the same order in every CTA,
        // inv = 1/sqrt(mean + eps) in float, x * (inv * gamma).
        float xv[kNormBlocks][8], gv[kNormBlocks][8];
        const bool embed = ph.x == nullptr;
        const uint8_t* erow = P.embd + (long long)tok * P.embd_stride;
#pragma unroll
        for (int i = 0; i < kNormBlocks; ++i) {
            const int b = warp + i * kW;
            if (b < nb) {
                const int c0 = b * 256 + lane * 8;
                const float4 q0 = *reinterpret_cast<const float4*>(ph.gamma + c0);
                const float4 q1 = *reinterpret_cast<const float4*>(ph.gamma + c0 + 4);
                gv[i][0] = q0.x; gv[i][1] = q0.y; gv[i][2] = q0.z; gv[i][3] = q0.w;
                gv[i][4] = q1.x; gv[i][5] = q1.y; gv[i][6] = q1.z; gv[i][7] = q1.w;
                if (embed) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) xv[i][e] = dequant_at(P.embd_type, erow, P.H, c0 + e);
                    if (blockIdx.x == 0) {
#pragma unroll
                        for (int e = 0; e < 8; ++e) P.h[c0 + e] = xv[i][e];
                    }
                } else {
                    const float4 u0 = __ldcg(reinterpret_cast<const float4*>(ph.x + c0));
                    const float4 u1 = __ldcg(reinterpret_cast<const float4*>(ph.x + c0 + 4));
                    xv[i][0] = u0.x; xv[i][1] = u0.y; xv[i][2] = u0.z; xv[i][3] = u0.w;
                    xv[i][4] = u1.x; xv[i][5] = u1.y; xv[i][6] = u1.z; xv[i][7] = u1.w;
                }
            }
        }
        double ss = 0.0;
#pragma unroll
        for (int i = 0; i < kNormBlocks; ++i)
            if (warp + i * kW < nb) {
#pragma unroll
                for (int e = 0; e < 8; ++e) ss += (double)xv[i][e] * (double)xv[i][e];
            }
        ss = warp_sum_d(ss);
        if (lane == 0) S.dred[warp] = ss;
        __syncthreads();
        double tot = 0.0;
        for (int w = 0; w < kW; ++w) tot += S.dred[w];
        const float inv = 1.0f / sqrtf((float)(tot / (double)ph.K) + P.eps);
#pragma unroll
        for (int i = 0; i < kNormBlocks; ++i) {
            const int b = warp + i * kW;
            if (b < nb) {
#pragma unroll
                for (int e = 0; e < 8; ++e) xv[i][e] = __fmul_rn(xv[i][e], __fmul_rn(inv, gv[i][e]));
                gmma::encode_block<true, false>(xv[i], lane, xq + (size_t)b * 1024, xs + b, xsum + b * 8, nullptr);
            }
        }
    } else {
        float xv[kXBlocksPerWarp][8];
#pragma unroll
        for (int i = 0; i < kXBlocksPerWarp; ++i) {
            const int b = warp + i * kW;
            if (b < nb) {
                const int c0 = b * 256 + lane * 8;
                const float4 u0 = __ldcg(reinterpret_cast<const float4*>(ph.x + c0));
                const float4 u1 = __ldcg(reinterpret_cast<const float4*>(ph.x + c0 + 4));
                xv[i][0] = u0.x; xv[i][1] = u0.y; xv[i][2] = u0.z; xv[i][3] = u0.w;
                xv[i][4] = u1.x; xv[i][5] = u1.y; xv[i][6] = u1.z; xv[i][7] = u1.w;
            }
        }
#pragma unroll
        for (int i = 0; i < kXBlocksPerWarp; ++i) {
            const int b = warp + i * kW;
            if (b < nb)
                gmma::encode_block<true, false>(xv[i], lane, xq + (size_t)b * 1024, xs + b, xsum + b * 8, nullptr);
        }
    }
    __syncthreads();
}

// ---- inputs encoded by the phase that produces them -------------------------
// Block b (256 elements) of the finished vector y, by one warp, into buffer
// `buf`: the XQ4 limbs of y (or, for the next RMSNorm, of y * gamma; the
// consumer multiplies the block scales by 1/rms) and the block's sum of y^2
// in double.
CL_DEVINL void encode_out_block(const Params& P, const float* y, const float* gamma, int buf, int b, int lane) {
    const EncView ev = enc_view(P, buf);
    const int c0 = b * 256 + lane * 8;
    const float4 u0 = __ldcg(reinterpret_cast<const float4*>(y + c0));
    const float4 u1 = __ldcg(reinterpret_cast<const float4*>(y + c0 + 4));
    float v[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
    if (gamma) {
        double ss = 0.0;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += (double)v[e] * (double)v[e];
        ss = warp_sum_d(ss);
        if (lane == 0) ev.ssq[b] = ss;
        const float4 g0 = *reinterpret_cast<const float4*>(gamma + c0);
        const float4 g1 = *reinterpret_cast<const float4*>(gamma + c0 + 4);
        const float gm[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(v[e], gm[e]);
    }
    gmma::encode_block<true, false>(v, lane, ev.xq + (size_t)b * 1024, ev.xs + b, ev.xsum + b * 8, nullptr);
}

// `add` completions of output block b (full warp, after its rows are
// written): the completion that finishes the block encodes it.
CL_DEVINL void block_done(const Params& P, const Phase& ph, const float* y, int b, int add, int lane) {
    __syncwarp();  // the warp's rows, published by lane 0's release add
    int last = 0;
    if (lane == 0) {
        unsigned int* c = P.enc_cnt + (size_t)ph.out_buf * P.nb_max + b;
        last = atom_add_acq_rel(c, (unsigned int)add) + (unsigned int)add == (unsigned int)ph.out_target;
        if (last) *c = 0u;  // re-armed: the buffer's next use is two phases later
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    encode_out_block(P, y, ph.gamma_out, ph.out_buf, b, lane);
}

// The phase's encoded input into shared memory: the limbs, scales and unit
// sums by bulk copies completing on the CTA's input barrier; for a
// normalised input the scales and sums are multiplied by 1/rms, summed from
// the blocks' sums of squares in block order (the same in every CTA;
// cpu_llm.cpp:156-165: the mean in double, inv = 1/sqrt(mean + eps) in float).
CL_DEVINL bool load_input(const Params& P, const Phase& ph, const Smem& S, uint32_t parity) {
    const int nb = ph.nb, tid = threadIdx.x;
    const EncView ev = enc_view(P, ph.in_buf);
    uint8_t* xq = S.region;
    const int xs_bytes = (nb * 4 + 15) & ~15;
    float* xs = reinterpret_cast<float*>(S.region + nb * 1024);
    float* xsum = reinterpret_cast<float*>(S.region + nb * 1024 + xs_bytes);
    if (tid == 0) {
        fence_proxy_async_smem();  // the region's last readers passed the CTA barrier before this phase
        mbar_arrive_expect_tx(S.xbar, (uint32_t)(nb * 1024 + xs_bytes + nb * 32));
        bulk_g2s(xq, ev.xq, (uint32_t)(nb * 1024), S.xbar);
        bulk_g2s(xs, ev.xs, (uint32_t)xs_bytes, S.xbar);
        bulk_g2s(xsum, ev.xsum, (uint32_t)(nb * 32), S.xbar);
    }
    float inv = 1.0f;
    if (ph.gamma) {
        // every warp: lane b holds block b's sum (nb <= 32), one butterfly:
        // the same order, hence the same bits, in every warp of every CTA
        const int lane = tid & 31;
        double tot = lane < nb ? __ldcg(ev.ssq + lane) : 0.0;
        tot = warp_sum_d(tot);
        inv = 1.0f / sqrtf((float)(tot / (double)ph.K) + P.eps);
    }
    const bool ok = __syncthreads_and(mbar_wait(S.xbar, parity));
    if (ok && ph.gamma) {
        for (int i = tid; i < nb; i += kThreads) xs[i] *= inv;
        for (int i = tid; i < nb * 8; i += kThreads) xsum[i] *= inv;
    }
    __syncthreads();
    return ok;
}

// ---- attention of one layer (CTA = KV head x key split) -------------------
// Splits per KV head: as requested, else one per kSplitKeys keys, at most
// kSplitsMax and at most the CTAs per KV head; split sp of KV head g holds
// keys k0 .. k0 + nk - 1 (nk may be 0 for a requested count).
struct AttnSplit {
    int g, sp, ns, k0, nk;
};

CL_DEVINL bool attn_split(const Params& P, int len, AttnSplit& a) {
    int ns = P.splits > 0 ? P.splits : (len + kSplitKeys - 1) / kSplitKeys;
    ns = max(1, min(min(ns, kSplitsMax), (int)gridDim.x / P.hkv));
    if ((int)blockIdx.x >= P.hkv * ns) return false;
    a.ns = ns;
    a.g = blockIdx.x / ns;
    a.sp = blockIdx.x - a.g * ns;
    const int per = (len + ns - 1) / ns;
    a.k0 = a.sp * per;
    a.nk = max(0, min(per, len - a.k0));
    return true;
}

// Attention's shared memory: after the QKV phase's input in the region.
struct AttnSmem {
    float *qs, *ks, *vs, *ps, *run, *fac, *csm;
};

CL_DEVINL AttnSmem attn_smem(const Params& P, const Smem& S) {
    AttnSmem a;
    a.qs = reinterpret_cast<float*>(S.region + P.attn_off);  // [G][kQLD]
    a.ks = a.qs + kGMax * kQLD;                              // [kKT][kQLD]
    a.vs = a.ks + kKT * kQLD;                                // [kKT][kD]
    a.ps = a.vs + kKT * kD;                                  // [G][kKT]
    a.run = a.ps + kGMax * kKT;                              // [G][2]
    a.fac = a.run + 2 * kGMax;                               // [G]
    a.csm = a.fac + kGMax;                                   // [d/2][cos, sin] of the position
    return a;
}

// Rows r0, r0 + step, ... of the key tile at t0 of a split into shared
// memory (K rows padded to kQLD), one 16-byte piece per lane and row.  The
// row of the current position holds a stale key until attention writes it.
CL_DEVINL void attn_load_rows(const Params& P, const cl_qwen2_layer& L, const AttnSplit& a, const AttnSmem& A,
                              int t0, int r0, int step, int lane) {
    const int kvd = P.hkv * kD, nk = min(kKT, a.nk - t0);
    const size_t base = (size_t)(a.k0 + t0) * kvd + (size_t)a.g * kD;
    for (int r = r0; r < nk; r += step) {
        cp16(A.ks + r * kQLD + 4 * lane, L.k_cache + base + (size_t)r * kvd + 4 * lane);
        cp16(A.vs + r * kD + 4 * lane, L.v_cache + base + (size_t)r * kvd + 4 * lane);
    }
}

CL_DEVINL void attention(const Params& P, const Phase& aph, int layer, int pos, const Smem& S, long long* tr) {
    const cl_qwen2_layer& L = P.layers[layer];
    auto stamp = [&](int slot) {
        if (tr && threadIdx.x == 0) tr[slot] = (long long)global_ns();
    };
    const int G = P.hq / P.hkv, kvd = P.hkv * kD, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    AttnSplit sa;
    if (!attn_split(P, pos + 1, sa)) return;
    const int g = sa.g, sp = sa.sp, ns = sa.ns, k0 = sa.k0, nk_all = sa.nk;
    const AttnSmem A = attn_smem(P, S);
    float *qs = A.qs, *ks = A.ks, *vs = A.vs, *ps = A.ps, *run = A.run, *fac = A.fac, *csm = A.csm;
    const float* cs = P.rope + (size_t)pos * kD;
    const int half = kD / 2;
    // The first key tile is in flight since the QKV phase (attn_prefetch);
    // the query heads, the position's rotation row and, in the split holding
    // the position, the new key and value are loaded now, all at once.
    constexpr int kQv = (kGMax * kD / 4 + kThreads - 1) / kThreads;
    float4 qv[kQv];
#pragma unroll
    for (int j = 0; j < kQv; ++j) {
        const int i = tid + j * kThreads;
        if (i < G * (kD / 4)) {
            const int hh = i / (kD / 4), c = i - hh * (kD / 4);
            qv[j] = __ldcg(reinterpret_cast<const float4*>(P.q + (size_t)(g * G + hh) * kD + 4 * c));
        }
    }
    const float4 csv = tid < kD / 4 ? *reinterpret_cast<const float4*>(cs + 4 * tid) : make_float4(0.f, 0.f, 0.f, 0.f);
    const int rpos = pos - k0;  // the new key's row in this split, if 0 <= rpos < nk_all
    const bool holds = rpos >= 0 && rpos < nk_all;
    float ka = 0.0f, kb = 0.0f, vn = 0.0f;
    if (holds) {
        if (tid < half) {
            ka = __ldcg(P.k + (size_t)g * kD + tid);
            kb = __ldcg(P.k + (size_t)g * kD + tid + half);
        }
        if (tid < kD) vn = __ldcg(P.v + (size_t)g * kD + tid);
    }
#pragma unroll
    for (int j = 0; j < kQv; ++j) {
        const int i = tid + j * kThreads;
        if (i < G * (kD / 4)) {
            const int hh = i / (kD / 4), c = i - hh * (kD / 4);
            *reinterpret_cast<float4*>(qs + hh * kQLD + 4 * c) = qv[j];
        }
    }
    if (tid < kD / 4) *reinterpret_cast<float4*>(csm + 4 * tid) = csv;
    if (tid < G) {
        run[2 * tid] = -INFINITY;
        run[2 * tid + 1] = 0.0f;
    }
    __syncthreads();
    // NeoX RoPE of the query heads (the expressions of attn.cu / rope_kv_kernel)
    for (int i = tid; i < G * half; i += kThreads) {
        const int hh = i / half, pp = i - hh * half;
        float* qh = qs + hh * kQLD;
        const float c = csm[2 * pp], sn = csm[2 * pp + 1];
        const float a = qh[pp], b = qh[pp + half];
        qh[pp] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, sn));
        qh[pp + half] = __fadd_rn(__fmul_rn(a, sn), __fmul_rn(b, c));
    }
    const int dim = tid & (kD - 1), pt = tid / kD;  // parts of the PV sums
    float acc[kGMax];
#pragma unroll
    for (int hh = 0; hh < kGMax; ++hh) acc[hh] = 0.0f;
    for (int t0 = 0; t0 < nk_all; t0 += kKT) {
        const int nk = min(kKT, nk_all - t0);
        if (t0 > 0) {
            attn_load_rows(P, L, sa, A, t0, warp, kW, lane);
            cp_commit();
        }
        cp_wait<0>();
        __syncthreads();
        if (t0 == 0) stamp(11);
        const int r = rpos - t0;
        if (holds && r >= 0 && r < nk) {
            // the current position: rotate the new key, append K and V, use them here
            float* kw = L.k_cache + (size_t)pos * kvd + (size_t)g * kD;
            float* vw = L.v_cache + (size_t)pos * kvd + (size_t)g * kD;
            if (tid < half) {
                const float c = csm[2 * tid], sn = csm[2 * tid + 1];
                const float ra = __fsub_rn(__fmul_rn(ka, c), __fmul_rn(kb, sn));
                const float rb = __fadd_rn(__fmul_rn(ka, sn), __fmul_rn(kb, c));
                kw[tid] = ra;
                kw[tid + half] = rb;
                ks[r * kQLD + tid] = ra;
                ks[r * kQLD + tid + half] = rb;
            }
            if (tid < kD) {
                vw[tid] = vn;
                vs[r * kD + tid] = vn;
            }
        }
        __syncthreads();
        // scores: thread per (key, head)
        for (int pidx = tid; pidx < nk * G; pidx += kThreads) {
            const int tk = pidx / G, hh = pidx - tk * G;
            const float4* kr = reinterpret_cast<const float4*>(ks + tk * kQLD);
            const float4* qr = reinterpret_cast<const float4*>(qs + hh * kQLD);
            float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll 8
            for (int c = 0; c < kD / 4; ++c) {
                const float4 kv = kr[c], qv = qr[c];
                a0 += kv.x * qv.x;
                a1 += kv.y * qv.y;
                a2 += kv.z * qv.z;
                a3 += kv.w * qv.w;
            }
            ps[hh * kKT + tk] = ((a0 + a1) + (a2 + a3)) * P.scale;
        }
        __syncthreads();
        if (warp < G) {
            float* ph = ps + warp * kKT;
            const float s0 = lane < nk ? ph[lane] : -INFINITY;
            const float s1 = lane + 32 < nk ? ph[lane + 32] : -INFINITY;
            const float mo = run[2 * warp], mn = fmaxf(mo, warp_max(fmaxf(s0, s1)));
            const float e0 = lane < nk ? expf(s0 - mn) : 0.0f;
            const float e1 = lane + 32 < nk ? expf(s1 - mn) : 0.0f;
            if (lane < nk) ph[lane] = e0;
            if (lane + 32 < nk) ph[lane + 32] = e1;
            const float l = warp_sum(e0 + e1);
            if (lane == 0) {
                const float f = mo == -INFINITY ? 0.0f : expf(mo - mn);
                fac[warp] = f;
                run[2 * warp] = mn;
                run[2 * warp + 1] = run[2 * warp + 1] * f + l;
            }
        }
        __syncthreads();
#pragma unroll
        for (int hh = 0; hh < kGMax; ++hh)
            if (hh < G) acc[hh] *= fac[hh];
        for (int tk = pt; tk < nk; tk += kThreads / kD) {
            const float vv = vs[tk * kD + dim];
#pragma unroll
            for (int hh = 0; hh < kGMax; ++hh)
                if (hh < G) acc[hh] += ps[hh * kKT + tk] * vv;
        }
        __syncthreads();  // tile buffers are refilled next
    }
    if (nk_all == 0) cp_wait<0>();  // an empty split: its (empty) prefetch group
    stamp(12);
    // this split's (m, l, o) per head; the K tile buffer holds the PV parts
    float* pv = ks;
    if (pt > 0) {
#pragma unroll
        for (int hh = 0; hh < kGMax; ++hh)
            if (hh < G) pv[((pt - 1) * G + hh) * kD + dim] = acc[hh];
    }
    __syncthreads();
    float* part = P.attn_part + (size_t)g * kSplitsMax * G * kRec;
    if (pt == 0) {
#pragma unroll
        for (int hh = 0; hh < kGMax; ++hh) {
            if (hh < G) {
                float o = acc[hh];
                for (int q2 = 1; q2 < kThreads / kD; ++q2) o += pv[((q2 - 1) * G + hh) * kD + dim];
                float* pr = part + ((size_t)sp * G + hh) * kRec;
                __stcg(pr + 4 + dim, o);
                if (dim == 0) {
                    __stcg(pr, run[2 * hh]);
                    __stcg(pr + 1, run[2 * hh + 1]);
                }
            }
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        atomicAdd(&P.ctl->attn_ticket[g], 1u);
    }
    stamp(13);
    // Splits 0 .. G - 1 merge one query head each (split sp: heads sp, sp + ns,
    // ... when there are fewer splits than heads) once every split of the KV
    // head has published; the tickets count on through the step's layers.
    if (sp >= G) return;
    if (tid == 0) {
        const unsigned int target = (unsigned int)((layer + 1) * ns);
        const unsigned long long t0 = global_ns();
        int ok = 1;
        while (ld_acquire(&P.ctl->attn_ticket[g]) < target) {
            if (*reinterpret_cast<volatile int*>(&P.ctl->abort) || global_ns() - t0 > kWaitNs) {
                atomicCAS(&P.ctl->error, 0, 5 * layer + 2);
                atomicExch(&P.ctl->abort, 1);
                ok = 0;
                break;
            }
        }
        S.flags[1] = ok;
    }
    __syncthreads();
    if (!S.flags[1]) return;  // the grid barrier ends the step
    // (attn_decode_combine's weights: exp(m_s - m) / l); thread: one dim, half the splits
    constexpr int kHalf = kSplitsMax / 2;
    float* wsm = ps;                                   // [kSplitsMax]
    float* osm = ps + kSplitsMax;                      // [kD] the second half's sums
    const int dd = tid & (kD - 1), part2 = tid / kD;   // part2 in {0, 1}
    for (int hh = sp; hh < G; hh += ns) {
        float ov[kHalf];
#pragma unroll
        for (int i = 0; i < kHalf; ++i) {
            const int s2 = part2 * kHalf + i;
            ov[i] = s2 < ns ? __ldcg(part + ((size_t)s2 * G + hh) * kRec + 4 + dd) : 0.0f;
        }
        if (warp == 0) {
            const float ms = lane < ns ? __ldcg(part + ((size_t)lane * G + hh) * kRec) : -INFINITY;
            const float ls = lane < ns ? __ldcg(part + ((size_t)lane * G + hh) * kRec + 1) : 0.0f;
            const float m = warp_max(ms);
            const float e = ls > 0.0f ? expf(ms - m) : 0.0f;
            const float l = warp_sum(ls * e);
            wsm[lane] = lane < ns ? e / l : 0.0f;
        }
        __syncthreads();
        float o = 0.0f;
#pragma unroll
        for (int i = 0; i < kHalf; ++i) o += ov[i] * wsm[part2 * kHalf + i];
        if (part2 == 1) osm[dd] = o;
        __syncthreads();
        if (part2 == 0) P.att[(size_t)(g * G + hh) * kD + dd] = o + osm[dd];
        __syncthreads();
        // the o_proj input block of the head (two 128-wide heads per block)
        if (aph.out_buf >= 0 && warp == 0) block_done(P, aph, P.att, (g * G + hh) / 2, 1, lane);
    }
    stamp(14);
}

// The first key tile of the CTA's split of layer l's attention, issued by
// each warp as it finishes its QKV units (rows warp, warp + kW, ...): the
// cached keys do not depend on the QKV products, and the region past the
// QKV input is free.  One commit group per warp, waited for by attention.
CL_DEVINL void attn_prefetch(const Params& P, const cl_qwen2_layer& L, int pos, const Smem& S, int warp,
                             int lane) {
    AttnSplit sa;
    if (attn_split(P, pos + 1, sa) && sa.nk > 0) attn_load_rows(P, L, sa, attn_smem(P, S), 0, warp, kW, lane);
    cp_commit();
}

// Tile completions of output blocks a warp has not yet counted: its tiles
// are consecutive, so it counts them per block and adds them to the block's
// counter when it moves to another block or ends its range (one atomic per
// block touched instead of one per tile).
struct Pending {
    int block, count;
};

CL_DEVINL void pending_flush(const Params& P, const Phase& ph, const float* y, Pending& pd, int lane) {
    if (pd.count > 0) block_done(P, ph, y, pd.block, pd.count, lane);
    pd.count = 0;
}

CL_DEVINL void pending_add(const Params& P, const Phase& ph, const float* y, int block, Pending& pd, int lane) {
    if (ph.out_buf < 0) return;
    if (pd.count > 0 && pd.block != block) pending_flush(P, ph, y, pd, lane);
    pd.block = block;
    ++pd.count;
}

// A warp's sums over a unit or tile -> lanes with t == 0: rows g (yg) and g + 8 (y8).
CL_DEVINL void quad_rows(float& yg, float& y8, float ym, int t) {
    if (t & 1) y8 += ym;
    else yg += ym;
    yg += __shfl_xor_sync(0xffffffffu, yg, 1);
    yg += __shfl_xor_sync(0xffffffffu, yg, 2);
    y8 += __shfl_xor_sync(0xffffffffu, y8, 1);
    y8 += __shfl_xor_sync(0xffffffffu, y8, 2);
}

// Tile mode, after the CTA's units: warp w finishes the CTA's tiles w, w +
// kW, ...: each row the sum of its units in order, then bias and residual
// (as tile_out), then the output block's completion.
CL_DEVINL void finish_ctile(const Params& P, const Phase& ph, const Smem& S, int warp, int lane) {
    // the warp's first tile: bias and residual loads in flight across the CTA barrier
    int s0 = 0, tl0 = 0;
    const bool has0 = tile_locate(ph, blockIdx.x + warp * gridDim.x, s0, tl0);
    float cb = 0.0f, cr = 0.0f;
    if (has0 && lane < 16) {
        const Seg& sg = ph.seg[s0];
        if (sg.bias) cb = sg.bias[tl0 * 16 + lane];
        if (ph.residual) cr = __ldcg(sg.y + tl0 * 16 + lane);
    }
    __syncthreads();
    int pos0 = 0, k = 0, s = 0, tl = 0;
    for (int tg = blockIdx.x; tile_locate(ph, tg, s, tl); tg += gridDim.x, ++k) {
        const Seg& sg = ph.seg[s];
        if (k % kW == warp) {
            if (lane < 16) {
                float v = 0.0f;
                for (int j = 0; j < sg.nsub; ++j) v += S.red[(pos0 + j) * 16 + lane];
                const int o = tl * 16 + lane;
                const bool first = k == warp;
                if (sg.bias) v += first ? cb : sg.bias[o];
                if (ph.residual) v = (first ? cr : __ldcg(sg.y + o)) + v;
                sg.y[o] = v;
            }
            if (ph.out_buf >= 0) block_done(P, ph, sg.y, (tl * 16) / 256, 1, lane);
        }
        pos0 += sg.nsub;
    }
}

// A finished tile's rows, direct or through the partial buffer.
CL_DEVINL void flush_tile(const Params& P, const Phase& ph, int s, int tile_l, long long b, long long e, int gw,
                          int GW, float yg, float y8, float ym, int lane, Best& best, Pending& pd,
                          const RowPre& pre) {
    const int g = lane >> 2, t = lane & 3;
    quad_rows(yg, y8, ym, t);
    const Seg& sg = ph.seg[s];
    const long long uf = sg.u0 + (long long)tile_l * sg.nsub, ul = uf + sg.nsub - 1;
    const int out_block = (tile_l * (sg.sw ? 8 : 16)) / 256;
    if (uf >= b && ul < e) {
        if (t == 0) tile_out(ph, sg, tile_l, g, yg, y8, best, pre);
        pending_add(P, ph, sg.y, out_block, pd, lane);
        return;
    }
    float* mine = P.partials + ((size_t)gw * 2 + (b >= uf ? 0 : 1)) * 16;
    if (t == 0) {
        __stcg(mine + g, yg);
        __stcg(mine + 8 + g, y8);
    }
    __syncwarp();
    // The warps covering the tile, in order.  With at least one unit per
    // warp (U >= GW) they are wf .. wl, each with a non-empty range; the
    // first one's partial is in its slot 1 unless its range starts exactly
    // at the tile, every later one's in slot 0.  With fewer units than warps
    // every warp holds at most one unit: the tile's units lie in distinct
    // warps, each partial in slot 0.
    const bool sparse = ph.U < GW;
    const int wf = warp_of(ph.U, uf, GW), wl = warp_of(ph.U, ul, GW);
    const int count = sparse ? sg.nsub : wl - wf + 1;
    int last = 0;
    if (lane == 0) {
        const unsigned int old = atom_add_acq_rel(&P.tickets[sg.tile0 + tile_l], 1u);
        last = old == (unsigned int)(count - 1);
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    if (t == 0) {
        float vg = 0.0f, v8 = 0.0f;
        const int first_slot = (!sparse && range_begin(ph.U, wf, GW) < uf) ? 1 : 0;
        // 16 partials in flight at a time, added in warp order
        for (int i0 = 0; i0 < count; i0 += 16) {
            float pg[16], p8[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                pg[i] = p8[i] = 0.0f;
                if (i0 + i < count) {
                    const int k = sparse ? warp_of(ph.U, uf + i0 + i, GW) : wf + i0 + i;
                    const float* pk = P.partials + ((size_t)k * 2 + (i0 + i == 0 ? first_slot : 0)) * 16;
                    pg[i] = __ldcg(pk + g);
                    p8[i] = __ldcg(pk + 8 + g);
                }
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (i0 + i < count) {
                    vg += pg[i];
                    v8 += p8[i];
                }
            }
        }
        tile_out(ph, sg, tile_l, g, vg, v8, best, pre);
    }
    if (lane == 0) P.tickets[sg.tile0 + tile_l] = 0u;
    pending_add(P, ph, sg.y, out_block, pd, lane);
}

__global__ void __launch_bounds__(kThreads, 1) decode_fused_kernel(const __grid_constant__ Params P) {
    extern __shared__ __align__(128) uint8_t smem[];
    Smem S;
    S.ring = smem;
    S.region = smem + kRingBytes;
    uint8_t* zero = S.region + P.region_bytes;
    S.zero = zero;
    S.red = reinterpret_cast<float*>(zero + 1024);
    S.pc = reinterpret_cast<Phase*>(S.red + kRedUnits * 16);
    S.wph = S.pc + kPhaseCache;
    S.dred = reinterpret_cast<double*>(S.wph + kW);
    S.bests = reinterpret_cast<float2*>(S.dred + kW);
    S.flags = reinterpret_cast<int*>(S.bests + kW);
    S.xbar = reinterpret_cast<uint64_t*>(S.flags + 4 + kPhaseCache);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3, h = t >> 1;
    const int GW = gridDim.x * kW, gw = blockIdx.x * kW + warp;
    if (tid < 64) reinterpret_cast<uint4*>(zero)[tid] = make_uint4(0u, 0u, 0u, 0u);
    if (tid == 0) {
        mbar_init(S.xbar, 1);
        mbar_fence_init();
    }
    uint32_t xloads = 0;  // uses of the input barrier (its phase parity)
    const int tok = __ldcg(P.ints);
    const int pos = __ldcg(P.ints + 1);
    const int nph = 5 * P.n_layers + 1;
    if (lane == 0 && warp < kPhaseCache) {  // phases 0 .. kPhaseCache - 1, one per warp
        S.flags[4 + warp] = -1;
        if (warp < nph) {
            make_phase(P, warp, S.pc[warp]);
            S.flags[4 + warp] = warp;
        }
    }
    __syncthreads();

    // ---- the warp's ring: issue iterator (lane-uniform) ----
    uint8_t* ring = S.ring + (size_t)warp * kSlots * kSlotBytes;
    Phase& wph = S.wph[warp];
    const LanePlan plan = lane_plan(lane);
    const uint64_t policy = evict_first_policy();
    int ip = -1;
    Cursor ic{0, 0, 0, 0};
    int n_issued = 0;  // commit groups: one per unit, empty once the step's units are all issued
    auto issue_next = [&]() {
        while (ic.left == 0) {
            ++ip;
            if (ip >= nph) {
                ip = nph;
                return;
            }
            if (ip < 5 * P.n_layers && ip % 5 == 1) continue;  // attention: no weight units
            const int slot = ip % kPhaseCache;
            if (S.flags[4 + slot] == ip) {
                if (lane < kPhaseWords)
                    reinterpret_cast<long long*>(&wph)[lane] = reinterpret_cast<const long long*>(S.pc + slot)[lane];
            } else if (lane == 0) {
                make_phase(P, ip, wph);  // further ahead than the cache (few units per warp)
            }
            __syncwarp();
            if (wph.ctile) {
                ic = cursor_ctile(wph, warp);
            } else {
                const long long b0 = range_begin(wph.U, gw, GW), e0 = range_begin(wph.U, gw + 1, GW);
                ic = b0 < e0 ? cursor_at(wph, b0, e0) : Cursor{0, 0, 0, 0};
            }
            __syncwarp();
        }
        issue_unit(wph, ic, ring + (size_t)(n_issued % kSlots) * kSlotBytes, lane, plan, policy);
        if (wph.ctile) cursor_ctile_next(wph, ic);
        else cursor_next(wph, ic);
    };
    for (int i = 0; i < kSlots; ++i) {
        if (ip < nph) issue_next();
        cp_commit();
        ++n_issued;
    }
    int n_done = 0;

    Q4Lane L;
    L.sh = 12u * (uint32_t)h;
    L.lw0 = ((t & 1) ? (1.0f / 16384.0f) : 1.0f) * (h ? (1.0f / 16.0f) : 1.0f);
    L.lw1 = L.lw0 * (1.0f / 128.0f);
    L.pp = t & 1;
    Q4Lane L6 = L;
    L6.lw0 = (t & 1) ? (1.0f / 16384.0f) : 1.0f;
    L6.lw1 = L6.lw0 * (1.0f / 128.0f);

    Best best{-INFINITY, 0x7fffffff};
    __syncthreads();

    long long* trace = P.trace ? P.trace + (size_t)blockIdx.x * nph * kTraceSlots : nullptr;
    // (the cache is filled before the warps' first issues read it)
    for (int p = 0; p < nph; ++p) {
        if (trace && tid == 0) trace[kTraceSlots * p] = (long long)global_ns();
        __syncthreads();
        const Phase& ph = S.pc[p % kPhaseCache];
        if (ph.attn) {
            attention(P, ph, p / 5, pos, S, trace ? trace + kTraceSlots * p : nullptr);
            if (trace && tid == 0) trace[kTraceSlots * p + 1] = (long long)global_ns();
        } else {
            if (ph.in_buf >= 0) {
                if (!load_input(P, ph, S, xloads++ & 1u)) {
                    if (tid == 0) {
                        atomicCAS(&P.ctl->error, 0, p + 1);
                        atomicExch(&P.ctl->abort, 1);
                    }
                    cp_wait_all();
                    return;
                }
            } else {
                encode_input(P, ph, S, tok, warp, lane);
            }
            if (trace && tid == 0) trace[kTraceSlots * p + 1] = (long long)global_ns();
            const uint8_t* xq = S.region;
            const int nb = ph.nb;
            const float* xs = reinterpret_cast<const float*>(S.region + nb * 1024);
            const float* xsum = reinterpret_cast<const float*>(S.region + nb * 1024 + ((nb * 4 + 15) & ~15));
            const long long b = range_begin(ph.U, gw, GW), e = range_begin(ph.U, gw + 1, GW);
            int cur_s = -1, cur_tl = -1;
            Pending pend{0, 0};
            RowPre pre{{0.0f, 0.0f}, {0.0f, 0.0f}};
            float yg = 0.0f, y8 = 0.0f, ym = 0.0f;
            Cursor cc = ph.ctile ? cursor_ctile(ph, warp) : b < e ? cursor_at(ph, b, e) : Cursor{0, 0, 0, 0};
            int upos = warp;  // tile mode: the unit's position in the CTA's list
            // traced: SM cycles spent waiting for the ring, computing units,
            // issuing loads and flushing tiles, and the units computed
            unsigned int cyc[4] = {0u, 0u, 0u, 0u};
            int n_units = 0;
            for (; cc.left > 0; ph.ctile ? cursor_ctile_next(ph, cc) : cursor_next(ph, cc)) {
                const Cursor un = cc;
                if (!ph.ctile && (un.s != cur_s || un.tile != cur_tl)) {
                    const unsigned int cf = trace ? (unsigned int)clock() : 0u;
                    if (cur_s >= 0) flush_tile(P, ph, cur_s, cur_tl, b, e, gw, GW, yg, y8, ym, lane, best, pend, pre);
                    if (trace) cyc[3] += (unsigned int)clock() - cf;
                    cur_s = un.s;
                    cur_tl = un.tile;
                    pre = row_pre(ph, ph.seg[cur_s], cur_tl, g, t);
                    yg = y8 = ym = 0.0f;
                }
                const unsigned int c0 = trace ? (unsigned int)clock() : 0u;
                cp_wait<kSlots - 1>();
                __syncwarp();
                const unsigned int c1 = trace ? (unsigned int)clock() : 0u;
                if (trace) {
                    cyc[0] += c1 - c0;
                    ++n_units;
                }
                const uint8_t* slot = ring + (size_t)(n_done % kSlots) * kSlotBytes;
                if (ph.seg[un.s].type == CL_TYPE_Q4_K) {
                    // super-blocks 2j and 2j + 1: two independent dot chains
                    const uint8_t* bg = slot + g * kRS4;
                    const uint8_t* b8 = bg + 8 * kRS4;
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        // the zero super-block padding an odd count: all its bytes
                        // (d, dmin included) are zero, read against zeros
                        const int sb = 2 * un.j + q;
                        const bool live = sb < nb;
                        const uint8_t* p0 = live && g < 4 ? xq + (size_t)sb * 1024 + g * 32 + 8 * t : S.zero;
                        const uint8_t* p1 = live && g >= 4 ? xq + (size_t)sb * 1024 + 128 + (g - 4) * 32 + 8 * t
                                                           : S.zero;
                        uint2 bx0[4], bx1[4];
#pragma unroll
                        for (int gi = 0; gi < 4; ++gi) {
                            bx0[gi] = *reinterpret_cast<const uint2*>(p0 + 256 * gi);
                            bx1[gi] = *reinterpret_cast<const uint2*>(p1 + 256 * gi);
                        }
                        const float4 xsum4 = live ? *reinterpret_cast<const float4*>(xsum + sb * 8 + h * 4)
                                                  : make_float4(0.f, 0.f, 0.f, 0.f);
                        gmma::q4k_sb(bg + 144 * q, b8 + 144 * q, bx0, bx1, xsum4, live ? xs[sb] : 0.0f, t, L, yg,
                                     y8, ym);
                    }
                } else {
                    const int sb = un.j;
                    const uint8_t* bg = slot + g * kRS6;
                    const uint8_t* b8 = bg + 8 * kRS6;
                    const uint8_t* p0 = g < 4 ? xq + (size_t)sb * 1024 + g * 32 + 4 * t : S.zero;
                    const uint8_t* p1 = g >= 4 ? xq + (size_t)sb * 1024 + 256 + (g - 4) * 32 + 4 * t : S.zero;
#pragma unroll
                    for (int hh = 0; hh < 2; ++hh)
                        q6k_half(bg + 112 * hh, b8 + 112 * hh, p0, p1, hh, sb, xs[sb], t, h, L6, yg, y8);
                }
                if (ph.ctile) {
                    // the unit's 16 row sums into the CTA's list
                    quad_rows(yg, y8, ym, t);
                    if (t == 0) {
                        S.red[upos * 16 + g] = yg;
                        S.red[upos * 16 + 8 + g] = y8;
                    }
                    upos += kW;
                    yg = y8 = ym = 0.0f;
                }
                __syncwarp();
                const unsigned int c2 = trace ? (unsigned int)clock() : 0u;
                ++n_done;
                if (ip < nph) issue_next();
                cp_commit();
                ++n_issued;
                if (trace) {
                    cyc[1] += c2 - c1;
                    cyc[2] += (unsigned int)clock() - c2;
                }
            }
            if (trace && lane == 0) {
                trace[kTraceSlots * p + 3 + warp] = (long long)global_ns();
                if (warp == 0) {
                    for (int i = 0; i < 4; ++i) trace[kTraceSlots * p + 11 + i] = cyc[i];  // (attention: 11-14)
                    trace[kTraceSlots * p + 15] = n_units;
                }
            }
            if (p % 5 == 0 && p < 5 * P.n_layers) attn_prefetch(P, P.layers[p / 5], pos, S, warp, lane);
            if (ph.ctile) {
                finish_ctile(P, ph, S, warp, lane);
            } else {
                if (cur_s >= 0) flush_tile(P, ph, cur_s, cur_tl, b, e, gw, GW, yg, y8, ym, lane, best, pend, pre);
                pending_flush(P, ph, ph.seg[0].y, pend, lane);
            }
        }
        if (p + 1 < nph) {
            // ---- grid barrier ----
            __syncthreads();
            if (trace && tid == 0) trace[kTraceSlots * p + 2] = (long long)global_ns();
            if (tid == 0) {
                red_add_release(&P.ctl->bar, 1u);
                // phase p's slot: the descriptor of phase p + kPhaseCache, built while the
                // grid arrives (every warp of the CTA is past phase p)
                if (p + kPhaseCache < nph) {
                    make_phase(P, p + kPhaseCache, S.pc[p % kPhaseCache]);
                    S.flags[4 + p % kPhaseCache] = p + kPhaseCache;
                }
                const unsigned int target = (unsigned int)(p + 1) * gridDim.x;
                const unsigned long long t0 = global_ns();
                int ok = 1;
                while (ld_acquire(&P.ctl->bar) < target) {
                    if (*reinterpret_cast<volatile int*>(&P.ctl->abort)) {
                        ok = 0;
                        break;
                    }
                    if (global_ns() - t0 > kWaitNs) {
                        atomicCAS(&P.ctl->error, 0, p + 1);
                        atomicExch(&P.ctl->abort, 1);
                        ok = 0;
                        break;
                    }
                }
                S.flags[0] = ok;
            }
            __syncthreads();
            if (!S.flags[0]) {
                cp_wait_all();
                return;
            }
        }
    }

    if (trace && tid == 0) trace[kTraceSlots * (nph - 1) + 2] = (long long)global_ns();
    // ---- head: the CTAs' candidates, merged by the last CTA ----
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best.v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, best.i, o);
        if (better(ov, oi, best.v, best.i)) {
            best.v = ov;
            best.i = oi;
        }
    }
    if (lane == 0) S.bests[warp] = make_float2(best.v, __int_as_float(best.i));
    cp_wait_all();
    __syncthreads();
    if (tid == 0) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int w = 0; w < kW; ++w) {
            const float v = S.bests[w].x;
            const int i = __float_as_int(S.bests[w].y);
            if (better(v, i, bv, bi)) {
                bv = v;
                bi = i;
            }
        }
        __stcg(&P.records[blockIdx.x], make_float2(bv, __int_as_float(bi)));
        __threadfence();
        const unsigned int old = atomicAdd(&P.ctl->done, 1u);
        if (old == gridDim.x - 1) {
            __threadfence();
            bv = -INFINITY;
            bi = 0x7fffffff;
            for (int c = 0; c < (int)gridDim.x; ++c) {
                const float2 r = __ldcg(&P.records[c]);
                const int i = __float_as_int(r.y);
                if (better(r.x, i, bv, bi)) {
                    bv = r.x;
                    bi = i;
                }
            }
            P.ints[3] = bi;
            P.ints[1] = pos + 1;  // position and live length advance together (as cl_counter_add)
            P.ints[2] = pos + 2;
            P.ctl->bar = 0u;
            P.ctl->done = 0u;
            for (int i = 0; i < kMaxKvHeads; ++i) P.ctl->attn_ticket[i] = 0u;
            __threadfence();
        }
    }
}

// ---- the tiled decode layout -------------------------------------------------
// Matrix [rows][k] (device layout, cl_repack_rows) -> units stored tile by
// tile: tile t = rows 16t .. 16t + 15 (with w_up: gate rows 8t .. 8t + 7, then
// up rows 8t .. 8t + 7), unit j of the tile = 16 rows x (Q4_K: super-blocks
// 2j and 2j + 1, 2 x 144 B, the second zero when the row has an odd count;
// Q6_K: super-block j as two 112-byte halves, each ql 64, qh 32, sc 8, f16 d,
// 6 zero bytes).  One thread per 16-byte piece.
__global__ void decode_pack_kernel(int type, const uint8_t* __restrict__ w, const uint8_t* __restrict__ w_up,
                                   long long stride, int rows, int k, uint8_t* __restrict__ out) {
    grid_wait();
    const int nb = k / 256;
    const bool q4 = type == CL_TYPE_Q4_K;
    const int nsub = q4 ? (nb + 1) / 2 : nb, pieces = q4 ? 18 : 14;
    const int tiles = w_up ? rows / 8 : rows / 16;
    const long long total = (long long)tiles * nsub * 16 * pieces;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        int pc = (int)(i % pieces);
        const long long ur = i / pieces;  // (tile, unit, row)
        const int r = (int)(ur % 16);
        const long long tu = ur / 16;
        const int j = (int)(tu % nsub);
        const int t = (int)(tu / nsub);
        const uint8_t* row = w_up ? (r < 8 ? w + (long long)(8 * t + r) * stride : w_up + (long long)(8 * t + r - 8) * stride)
                                  : w + (long long)(16 * t + r) * stride;
        uint4 v;
        if (q4) {
            v = 2 * j + pc / 9 < nb ? *reinterpret_cast<const uint4*>(row + 288LL * j + 16 * pc)
                                    : make_uint4(0u, 0u, 0u, 0u);
        } else {
            const int sb = j, hh = pc / 7;
            pc -= 7 * hh;
            const uint8_t* blk = row + 208LL * sb;
            if (pc < 4) {
                v = *reinterpret_cast<const uint4*>(blk + 64 * hh + 16 * pc);
            } else if (pc < 6) {
                v = *reinterpret_cast<const uint4*>(blk + 128 + 32 * hh + 16 * (pc - 4));
            } else {
                const uint2 sc = *reinterpret_cast<const uint2*>(blk + 192 + 8 * hh);
                const uint8_t* dp = row + 208LL * nb + 2 * sb;
                v = make_uint4(sc.x, sc.y, (uint32_t)dp[0] | ((uint32_t)dp[1] << 8), 0u);
            }
        }
        reinterpret_cast<uint4*>(out)[i] = v;
    }
}

size_t xq_bytes(int nb) { return (size_t)nb * 1024 + (((size_t)nb * 4 + 15) & ~(size_t)15) + (size_t)nb * 32; }

size_t attn_off(int hidden) { return (xq_bytes(hidden / 256) + 127) & ~(size_t)127; }

size_t region_bytes(int hidden, int ffn) {
    const size_t xq = xq_bytes(std::max(hidden, ffn) / 256);
    const size_t attn = sizeof(float) * ((size_t)kGMax * kQLD + (size_t)kKT * kQLD + (size_t)kKT * kD +
                                         (size_t)kGMax * kKT + 3 * kGMax + kD);
    return (std::max(xq, attn_off(hidden) + attn) + 127) & ~(size_t)127;
}

size_t smem_bytes(int hidden, int ffn) {
    return kRingBytes + region_bytes(hidden, ffn) + 1024 + kRedUnits * 16 * sizeof(float) +
           (2 + kW) * sizeof(Phase) + kW * sizeof(double) +
           kW * sizeof(float2) + 16 + 4 * kPhaseCache + 16 + 3 * sizeof(Phase);
}

int max_tiles(const cl_qwen2_decode* m) {
    const int d = m->head_dim;
    return std::max({m->vocab / 16, m->ffn / 8, (m->q_heads + 2 * m->kv_heads) * d / 16, m->hidden / 16});
}

struct Layout {
    size_t tickets, records, partials, attn, enc0, enc1, enc_cnt, total;
};

Layout layout(const cl_qwen2_decode* m, int grid) {
    Layout l{};
    size_t off = sizeof(Ctl);
    l.tickets = off;
    off += ((size_t)max_tiles(m) * 4 + 255) & ~(size_t)255;
    l.records = off;
    off += ((size_t)grid * 8 + 255) & ~(size_t)255;
    l.partials = off;
    off += (size_t)grid * kW * 2 * 16 * 4;
    l.attn = off;
    off += (size_t)m->kv_heads * kSplitsMax * (m->q_heads / m->kv_heads) * kRec * 4;
    const int nbm = std::max(m->hidden, m->ffn) / 256;
    off = (off + 255) & ~(size_t)255;
    l.enc0 = off;
    off += (enc_bytes(nbm) + 255) & ~(size_t)255;
    l.enc1 = off;
    off += (enc_bytes(nbm) + 255) & ~(size_t)255;
    l.enc_cnt = off;
    off += (size_t)2 * nbm * 4;
    l.total = (off + 255) & ~(size_t)255;
    return l;
}

bool k_type_ok(int t) { return t == CL_TYPE_Q4_K || t == CL_TYPE_Q6_K; }

}  // namespace dfz
}  // namespace cl

using namespace cl;
using namespace cl::dfz;

extern "C" {

CL_API size_t cl_decode_pack_bytes(int type, int rows, int k, int pair) {
    if ((type != CL_TYPE_Q4_K && type != CL_TYPE_Q6_K) || rows <= 0 || k <= 0 || k % 256 || rows % (pair ? 8 : 16))
        return 0;
    const size_t nsub = type == CL_TYPE_Q4_K ? ((size_t)k / 256 + 1) / 2 : (size_t)k / 256;
    const size_t tiles = pair ? (size_t)rows / 8 : (size_t)rows / 16;
    return tiles * nsub * (size_t)unit_bytes(type);
}

CL_API int cl_decode_pack(int type, const void* w, long long stride, int rows, int k, const void* w_up, void* out,
                          cudaStream_t stream) {
    if (cl_decode_pack_bytes(type, rows, k, w_up != nullptr) == 0 || w == nullptr || out == nullptr ||
        stride < cl_row_stride(type, k))
        return CL_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(w_up) | reinterpret_cast<uintptr_t>(out)) % 16 ||
        stride % 16)
        return CL_ERR_INVALID;
    return launch_pdl(decode_pack_kernel, dim3(148 * 8), dim3(256), 0, stream, type, static_cast<const uint8_t*>(w),
                      static_cast<const uint8_t*>(w_up), stride, rows, k, static_cast<uint8_t*>(out)) == cudaSuccess
               ? CL_OK
               : CL_ERR_CUDA;
}

CL_API int cl_qwen2_decode_supported(const cl_qwen2_decode* m, const cl_qwen2_layer* hl) {
    if (m == nullptr || hl == nullptr || m->layers == nullptr || m->n_layers <= 0) return CL_ERR_INVALID;
    if (m->hidden <= 0 || m->ffn <= 0 || m->hidden % 256 || m->ffn % 256 || m->hidden > kW * kNormBlocks * 256 ||
        m->ffn > kMaxK ||
        m->head_dim != kD || m->q_heads <= 0 || m->kv_heads <= 0 || m->kv_heads > kMaxKvHeads ||
        m->q_heads % m->kv_heads || m->q_heads / m->kv_heads > kGMax || m->q_heads * kD != m->hidden ||
        m->vocab <= 0 || m->vocab % 16 || m->ffn % 8 || m->capacity <= 0 || m->attn_splits < 0 ||
        m->attn_splits > kSplitsMax)
        return CL_ERR_UNSUPPORTED;
    if (!k_type_ok(m->out_type) || m->embd == nullptr || m->out_w == nullptr || m->out_norm == nullptr ||
        m->rope == nullptr || m->ints == nullptr || !m->h || !m->q || !m->k || !m->v || !m->att || !m->act ||
        !m->logits)
        return CL_ERR_UNSUPPORTED;
    if (m->embd_type != CL_TYPE_F32 && m->embd_type != CL_TYPE_F16 && m->embd_type != CL_TYPE_Q4_K &&
        m->embd_type != CL_TYPE_Q5_K && m->embd_type != CL_TYPE_Q6_K && m->embd_type != CL_TYPE_Q8_0 &&
        m->embd_type != CL_TYPE_Q5_0)
        return CL_ERR_UNSUPPORTED;
    // 16-byte alignment of every vector read with float4 / cp.async
    const uintptr_t vec = reinterpret_cast<uintptr_t>(m->h) | reinterpret_cast<uintptr_t>(m->q) |
                          reinterpret_cast<uintptr_t>(m->k) | reinterpret_cast<uintptr_t>(m->v) |
                          reinterpret_cast<uintptr_t>(m->att) | reinterpret_cast<uintptr_t>(m->act) |
                          reinterpret_cast<uintptr_t>(m->out_norm) | reinterpret_cast<uintptr_t>(m->out_w);
    if (vec & 15u) return CL_ERR_INVALID;
    for (int l = 0; l < m->n_layers; ++l) {
        const cl_qwen2_layer& L = hl[l];
        if (!k_type_ok(L.q_type) || !k_type_ok(L.k_type) || !k_type_ok(L.v_type) || !k_type_ok(L.o_type) ||
            !k_type_ok(L.gate_type) || !k_type_ok(L.down_type))
            return CL_ERR_UNSUPPORTED;
        if (!L.q || !L.k || !L.v || !L.o || !L.gate || !L.down || !L.attn_norm || !L.ffn_norm || !L.k_cache ||
            !L.v_cache)
            return CL_ERR_INVALID;
        const uintptr_t a = reinterpret_cast<uintptr_t>(L.q) | reinterpret_cast<uintptr_t>(L.k) |
                            reinterpret_cast<uintptr_t>(L.v) | reinterpret_cast<uintptr_t>(L.o) |
                            reinterpret_cast<uintptr_t>(L.gate) |
                            reinterpret_cast<uintptr_t>(L.down) | reinterpret_cast<uintptr_t>(L.attn_norm) |
                            reinterpret_cast<uintptr_t>(L.ffn_norm) | reinterpret_cast<uintptr_t>(L.k_cache) |
                            reinterpret_cast<uintptr_t>(L.v_cache);
        if (a & 15u) return CL_ERR_INVALID;
    }
    return CL_OK;
}

CL_API size_t cl_qwen2_decode_workspace_bytes(const cl_qwen2_decode* m) {
    if (m == nullptr || m->kv_heads <= 0 || m->q_heads <= 0 || m->q_heads % m->kv_heads) return 0;
    int grid = 0;
    if (device_sm_count(&grid) != cudaSuccess || grid <= 0) return 0;
    return layout(m, grid).total;
}

CL_API int cl_qwen2_decode_init(void* workspace, size_t workspace_bytes, cudaStream_t stream) {
    if (workspace == nullptr || workspace_bytes < sizeof(Ctl) || (reinterpret_cast<uintptr_t>(workspace) & 255u))
        return CL_ERR_INVALID;
    // the control block and the tile tickets must start at zero; the rest is
    // written before it is read in every step
    return cudaMemsetAsync(workspace, 0, workspace_bytes, stream) == cudaSuccess ? CL_OK : CL_ERR_CUDA;
}

CL_API const int* cl_qwen2_decode_status(const void* workspace) {
    if (workspace == nullptr) return nullptr;
    return &static_cast<const Ctl*>(workspace)->error;
}

CL_API int cl_qwen2_decode_step(const cl_qwen2_decode* m, const cl_qwen2_layer* host_layers, void* workspace,
                                size_t workspace_bytes, cudaStream_t stream) {
    const int rc = cl_qwen2_decode_supported(m, host_layers);
    if (rc != CL_OK) return rc;
    if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255u)) return CL_ERR_INVALID;
    int grid = 0;
    if (device_sm_count(&grid) != cudaSuccess) return CL_ERR_CUDA;
    const Layout lay = layout(m, grid);
    if (workspace_bytes < lay.total) return CL_ERR_WORKSPACE;
    const size_t smem = smem_bytes(m->hidden, m->ffn);
    static SmemLimit limit;
    if (limit.ensure(decode_fused_kernel, (int)smem) != cudaSuccess) return CL_ERR_UNSUPPORTED;
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_fused_kernel, kThreads, smem) != cudaSuccess ||
        occ < 1)
        return CL_ERR_UNSUPPORTED;
    char* ws = static_cast<char*>(workspace);
    Params p{};
    p.layers = m->layers;
    p.n_layers = m->n_layers;
    p.H = m->hidden;
    p.F = m->ffn;
    p.V = m->vocab;
    p.hq = m->q_heads;
    p.hkv = m->kv_heads;
    p.cap = m->capacity;
    p.max_tiles = max_tiles(m);
    p.eps = m->eps;
    p.scale = m->scale;
    p.embd = static_cast<const uint8_t*>(m->embd);
    p.embd_stride = m->embd_stride;
    p.embd_type = m->embd_type;
    p.out_type = m->out_type;
    p.out_w = static_cast<const uint8_t*>(m->out_w);
    p.out_norm = m->out_norm;
    p.rope = m->rope;
    p.ints = m->ints;
    p.h = m->h;
    p.q = m->q;
    p.k = m->k;
    p.v = m->v;
    p.att = m->att;
    p.act = m->act;
    p.logits = m->logits;
    p.ctl = reinterpret_cast<Ctl*>(ws);
    p.tickets = reinterpret_cast<unsigned int*>(ws + lay.tickets);
    p.records = reinterpret_cast<float2*>(ws + lay.records);
    p.partials = reinterpret_cast<float*>(ws + lay.partials);
    p.attn_part = reinterpret_cast<float*>(ws + lay.attn);
    p.trace = m->trace;
    p.enc[0] = reinterpret_cast<uint8_t*>(ws + lay.enc0);
    p.enc[1] = reinterpret_cast<uint8_t*>(ws + lay.enc1);
    p.enc_cnt = reinterpret_cast<unsigned int*>(ws + lay.enc_cnt);
    p.nb_max = std::max(m->hidden, m->ffn) / 256;
    p.region_bytes = (int)region_bytes(m->hidden, m->ffn);
    p.attn_off = (int)attn_off(m->hidden);
    p.splits = m->attn_splits;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_fused_kernel, p) == cudaSuccess ? CL_OK : CL_ERR_CUDA;
}

}  // extern "C"
