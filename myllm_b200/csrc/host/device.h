// Host-side CUDA plumbing shared by the backends: error checks, RAII device
// and pinned buffers, a 256-byte-aligned bump arena, and the weight loader
// that streams GGUF tensors into HBM in the kernels' device layout.
#pragma once

#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "cudallm_kernels.h"
#include "gguf.h"

namespace cudallm {

[[noreturn]] void throw_cuda(cudaError_t e, const char* what, const char* file, int line);
[[noreturn]] void throw_cl(int status, const char* what, const char* file, int line);

#define CUDALLM_CUDA(expr)                                                       \
    do {                                                                         \
        cudaError_t e_ = (expr);                                                 \
        if (e_ != cudaSuccess) ::cudallm::throw_cuda(e_, #expr, __FILE__, __LINE__); \
    } while (0)

#define CUDALLM_CL(expr)                                                         \
    do {                                                                         \
        int s_ = (expr);                                                         \
        if (s_ != CL_OK) ::cudallm::throw_cl(s_, #expr, __FILE__, __LINE__);     \
    } while (0)

class DeviceBuffer {
public:
    DeviceBuffer() = default;
    explicit DeviceBuffer(std::size_t bytes);
    ~DeviceBuffer();
    DeviceBuffer(DeviceBuffer&& o) noexcept;
    DeviceBuffer& operator=(DeviceBuffer&& o) noexcept;
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    void* get() const noexcept { return ptr_; }
    std::size_t size() const noexcept { return bytes_; }

private:
    void* ptr_ = nullptr;
    std::size_t bytes_ = 0;
};

// An NVTX range around one backend call (closed on every exit path), named
// like the reference profiler's stage for it, so that timelines taken with
// NVIDIA's tools show each prefill / decode.  Without a tool attached the
// calls return at once.
class TraceRange {
public:
    explicit TraceRange(const char* name) { nvtxRangePushA(name); }
    ~TraceRange() { nvtxRangePop(); }
    TraceRange(const TraceRange&) = delete;
    TraceRange& operator=(const TraceRange&) = delete;
};

class PinnedBuffer {
public:
    PinnedBuffer() = default;
    explicit PinnedBuffer(std::size_t bytes);
    ~PinnedBuffer();
    PinnedBuffer(PinnedBuffer&& o) noexcept;
    PinnedBuffer& operator=(PinnedBuffer&& o) noexcept;
    PinnedBuffer(const PinnedBuffer&) = delete;
    PinnedBuffer& operator=(const PinnedBuffer&) = delete;
    void* get() const noexcept { return ptr_; }
    std::size_t size() const noexcept { return bytes_; }

private:
    void* ptr_ = nullptr;
    std::size_t bytes_ = 0;
};

// Bump allocator: plan() with a null base counts bytes, then bind() a real
// buffer and replay the same sequence of take() calls.
class Arena {
public:
    void bind(void* base, std::size_t bytes) {
        base_ = static_cast<char*>(base);
        cap_ = bytes;
        used_ = 0;
    }
    void* take(std::size_t bytes) {
        const std::size_t at = (used_ + 255) / 256 * 256;
        used_ = at + bytes;
        if (base_ == nullptr) return nullptr;
        if (used_ > cap_) throw std::runtime_error("device arena overflow");
        return base_ + at;
    }
    template <typename T>
    T* take_n(std::size_t n) {
        return static_cast<T*>(take(n * sizeof(T)));
    }
    std::size_t used() const noexcept { return used_; }

private:
    char* base_ = nullptr;
    std::size_t cap_ = 0;
    std::size_t used_ = 0;
};

// A weight matrix [rows, cols] in the device layout of cl_repack_rows.
struct DevMat {
    const void* ptr = nullptr;
    int type = 0;
    int rows = 0;
    int cols = 0;
    long long stride = 0;
    std::size_t payload = 0;  // native GGUF bytes represented
};

// Streams tensors from a GGUF file into an Arena.  With a null arena base
// (planning pass) it only accounts bytes.  Row/column ranges select a shard:
// column ranges must be block aligned for the tensor's type.
class WeightLoader {
public:
    WeightLoader(GgufFile& file, Arena& arena, cudaStream_t stream);
    ~WeightLoader();

    DevMat matrix(const std::string& name, std::size_t rows, std::size_t cols, std::size_t row_begin = 0,
                  std::size_t row_end = SIZE_MAX, std::size_t col_begin = 0, std::size_t col_end = SIZE_MAX);
    // Several native tensors stacked as one matrix (rows concatenated),
    // each tensor given as (name, rows, cols, row_begin, row_end).
    struct Part {
        std::string name;
        std::size_t rows, cols, row_begin, row_end;
    };
    DevMat stacked(const std::vector<Part>& parts);
    // F32/F16 vector (or [1, n] tensor) as FP32 on the device; ranges as above.
    float* vector(const std::string& name, std::size_t n, std::size_t begin = 0, std::size_t end = SIZE_MAX);
    // Rows [row_begin, row_end) of an F32/F16 matrix as FP32 on the device.
    float* matrix_f32(const std::string& name, std::size_t rows, std::size_t cols, std::size_t row_begin = 0,
                      std::size_t row_end = SIZE_MAX);
    std::size_t payload_bytes() const noexcept { return payload_; }
    void finish();  // wait for outstanding copies

private:
    void upload(const void* host, std::size_t bytes, void* dst);
    GgufFile& file_;
    Arena& arena_;
    cudaStream_t stream_;
    PinnedBuffer pinned_;
    DeviceBuffer staging_;
    std::vector<uint8_t> host_;
    std::size_t payload_ = 0;
};

}  // namespace cudallm
