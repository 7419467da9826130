// One-shot all-reduce over peer memory for tensor-parallel decode.
//
// A decode token of a tensor-parallel qwen2 model sums two [hidden] FP32
// partials across the ranks in every layer (after o_proj and after ffn_down,
// cpu_llm.cpp:774-914 computes the unsplit products).  At 20 KB a call is
// pure latency, so instead of a ring this kernel exchanges through buffers
// every rank maps from every other (CUDA IPC over NVLink / NVSwitch):
//
//   block b of rank r   1. stores r's vector into rank b's slot [parity][r]
//                          (remote stores over NVLink, one pass);
//                       2. release-stores the call's epoch into rank b's
//                          flag [parity][r];
//                       3. waits (acquire loads, bounded by a wall-clock
//                          limit) until all `world` flags of its own buffer
//                          carry the epoch;
//                       4. sums slice b of the vector over the slots in rank
//                          order 0..world-1 (so every rank gets the same bits)
//                          into `out`.
//
// Two parities alternate so a rank one call ahead writes the other set; it
// cannot be two calls ahead, because finishing a call needs every rank's flag
// of that call.  Each block keeps its own call counter in its own header
// (read after griddepcontrol.wait), so no block waits on another block of the
// same launch.  A wait that runs out sets the buffer's status word and the
// kernel returns; the host reads the word after the step.
//
// The exchange buffer of one rank (cl_peer_exchange_bytes):
//   header (256 B): u32 epoch[8], u32 flag[2][8], u32 status, padding
//   data: f32 [2][8][slot], slot = max_n rounded up to 64 floats
#include "common.cuh"
#include "launch.cuh"

namespace cl {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kThreads = 512;
// A peer may start the same decode step seconds later (host jitter, a
// profiler); only a rank that never arrives should trip this.  Process-wide,
// read at each launch; cl_peer_set_wait_limit_ns changes it (tests shorten it
// to make the wait run out quickly).
constexpr unsigned long long kDefaultWaitLimitNs = 20ull * 1000 * 1000 * 1000;
constexpr unsigned long long kMinWaitLimitNs = 1000ull * 1000;                // 1 ms
constexpr unsigned long long kMaxWaitLimitNs = 120ull * 1000 * 1000 * 1000;  // 2 min
unsigned long long g_wait_limit_ns = kDefaultWaitLimitNs;

struct PeerHeader {
    uint32_t epoch[kMaxRanks];
    uint32_t flag[2][kMaxRanks];
    uint32_t status;
    uint32_t pad[64 - 3 * kMaxRanks - 1];
};
static_assert(sizeof(PeerHeader) == 256, "exchange header is 256 bytes");

struct PeerBuffers {
    char* buf[kMaxRanks];
};

size_t slot_floats(int max_n) { return ((size_t)max_n + 63) / 64 * 64; }

CL_DEVINL uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

CL_DEVINL void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

CL_DEVINL unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__global__ void __launch_bounds__(kThreads)
    peer_allreduce_kernel(const float* in, float* out, int n, int rank, int world,
                          size_t slot, unsigned long long wait_limit_ns, const __grid_constant__ PeerBuffers peers) {
    const int b = blockIdx.x;
    PeerHeader* mine = reinterpret_cast<PeerHeader*>(peers.buf[rank]);
    __shared__ uint32_t s_epoch;
    __shared__ int s_fail;
    grid_wait();  // `in` comes from the previous kernel; the counter from the previous call
    if (threadIdx.x == 0) {
        s_epoch = mine->epoch[b] + 1u;
        s_fail = 0;
    }
    __syncthreads();
    const uint32_t e = s_epoch;
    const int par = (int)(e & 1u);
    const int n4 = n >> 2;

    // 1-2. this rank's vector into rank b's slot, then rank b's flag
    PeerHeader* dst_hdr = reinterpret_cast<PeerHeader*>(peers.buf[b]);
    float4* dst = reinterpret_cast<float4*>(peers.buf[b] + sizeof(PeerHeader)) +
                  ((size_t)par * kMaxRanks + (size_t)rank) * (slot / 4);
    const float4* src = reinterpret_cast<const float4*>(in);
    for (int i = threadIdx.x; i < n4; i += blockDim.x) __stcg(dst + i, __ldcg(src + i));
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        st_release_sys(&dst_hdr->flag[par][rank], e);
    }

    // 3. every rank's vector has arrived in this rank's slots
    if (threadIdx.x < world) {
        const uint32_t* f = &mine->flag[par][threadIdx.x];
        const unsigned long long t0 = global_ns();
        while ((int)(ld_acquire_sys(f) - e) < 0) {
            if (global_ns() - t0 > wait_limit_ns) {
                atomicOr(&mine->status, 1u);
                s_fail = 1;
                break;
            }
            __nanosleep(32);
        }
    }
    __syncthreads();

    // 4. slice b, summed in rank order
    if (!s_fail) {
        const int per = (n4 + world - 1) / world;
        const int i0 = b * per;
        const int i1 = min(n4, i0 + per);
        const float4* base = reinterpret_cast<const float4*>(peers.buf[rank] + sizeof(PeerHeader)) +
                             (size_t)par * kMaxRanks * (slot / 4);
        float4* o = reinterpret_cast<float4*>(out);
        for (int i = i0 + (int)threadIdx.x; i < i1; i += blockDim.x) {
            float4 acc = __ldcg(base + i);
            for (int r = 1; r < world; ++r) {
                const float4 v = __ldcg(base + (size_t)r * (slot / 4) + i);
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
            o[i] = acc;
        }
    }
    if (threadIdx.x == 0) mine->epoch[b] = e;
}

}  // namespace
}  // namespace cl

using namespace cl;

extern "C" {

CL_API size_t cl_peer_exchange_bytes(int max_n) {
    if (max_n <= 0) return 0;
    return sizeof(PeerHeader) + 2 * kMaxRanks * slot_floats(max_n) * sizeof(float);
}

CL_API int cl_peer_exchange_init(void* buffer, int max_n, cudaStream_t stream) {
    if (buffer == nullptr || max_n <= 0 || (reinterpret_cast<uintptr_t>(buffer) & 255u) != 0) return CL_ERR_INVALID;
    return cudaMemsetAsync(buffer, 0, sizeof(PeerHeader), stream) == cudaSuccess ? CL_OK : CL_ERR_CUDA;
}

CL_API const int* cl_peer_exchange_status(const void* buffer) {
    if (buffer == nullptr) return nullptr;
    return reinterpret_cast<const int*>(&static_cast<const PeerHeader*>(buffer)->status);
}

CL_API int cl_peer_allreduce(const float* in, float* out, int n, int max_n, int rank, int world,
                             void* const* buffers, cudaStream_t stream) {
    if (in == nullptr || out == nullptr || buffers == nullptr || n <= 0 || n % 4 != 0 || n > max_n ||
        world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
        return CL_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15u) return CL_ERR_INVALID;
    // out must not overlap in: a block writes its slice of out while other
    // blocks may still be sending in
    if (out < in + n && in < out + n) return CL_ERR_INVALID;
    PeerBuffers peers{};
    for (int r = 0; r < world; ++r) {
        if (buffers[r] == nullptr || (reinterpret_cast<uintptr_t>(buffers[r]) & 255u) != 0) return CL_ERR_INVALID;
        peers.buf[r] = static_cast<char*>(buffers[r]);
    }
    return launch_pdl(peer_allreduce_kernel, dim3(world), dim3(kThreads), 0, stream, in, out, n, rank, world,
                      slot_floats(max_n), g_wait_limit_ns, peers) == cudaSuccess
               ? CL_OK
               : CL_ERR_CUDA;
}

CL_API int cl_peer_set_wait_limit_ns(unsigned long long ns) {
    if (ns < kMinWaitLimitNs || ns > kMaxWaitLimitNs) return CL_ERR_INVALID;
    g_wait_limit_ns = ns;
    return CL_OK;
}

}  // extern "C"
