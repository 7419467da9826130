#include "device.h"

#include <set>

#include <algorithm>
#include <cstring>

namespace cudallm {

void throw_cuda(cudaError_t e, const char* what, const char* file, int line) {
    throw std::runtime_error(std::string("CUDA error ") + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) +
                             ") in " + what + " at " + file + ":" + std::to_string(line));
}

void throw_cl(int status, const char* what, const char* file, int line) {
    throw std::runtime_error(std::string("kernel call failed: ") + cl_status_string(status) + " in " + what +
                             " at " + file + ":" + std::to_string(line));
}

DeviceBuffer::DeviceBuffer(std::size_t bytes) : bytes_(bytes) {
    if (bytes) CUDALLM_CUDA(cudaMalloc(&ptr_, bytes));
}
DeviceBuffer::~DeviceBuffer() {
    if (ptr_) cudaFree(ptr_);
}
DeviceBuffer::DeviceBuffer(DeviceBuffer&& o) noexcept : ptr_(o.ptr_), bytes_(o.bytes_) {
    o.ptr_ = nullptr;
    o.bytes_ = 0;
}
DeviceBuffer& DeviceBuffer::operator=(DeviceBuffer&& o) noexcept {
    if (this != &o) {
        if (ptr_) cudaFree(ptr_);
        ptr_ = o.ptr_;
        bytes_ = o.bytes_;
        o.ptr_ = nullptr;
        o.bytes_ = 0;
    }
    return *this;
}

PinnedBuffer::PinnedBuffer(std::size_t bytes) : bytes_(bytes) {
    if (bytes) CUDALLM_CUDA(cudaMallocHost(&ptr_, bytes));
}
PinnedBuffer::~PinnedBuffer() {
    if (ptr_) cudaFreeHost(ptr_);
}
PinnedBuffer::PinnedBuffer(PinnedBuffer&& o) noexcept : ptr_(o.ptr_), bytes_(o.bytes_) {
    o.ptr_ = nullptr;
    o.bytes_ = 0;
}
PinnedBuffer& PinnedBuffer::operator=(PinnedBuffer&& o) noexcept {
    if (this != &o) {
        if (ptr_) cudaFreeHost(ptr_);
        ptr_ = o.ptr_;
        bytes_ = o.bytes_;
        o.ptr_ = nullptr;
        o.bytes_ = 0;
    }
    return *this;
}

namespace {
constexpr std::size_t kStagingBytes = 64u << 20;

std::size_t block_of(uint32_t type) {
    switch (type) {
    case kQ5_0: case kQ8_0: return 32;
    case kQ4_K: case kQ5_K: case kQ6_K: return 256;
    default: return 1;
    }
}

float half_to_float_host(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            int e = -1;
            do {
                man <<= 1;
                ++e;
            } while (!(man & 0x400));
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ff) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}
}  // namespace

WeightLoader::WeightLoader(GgufFile& file, Arena& arena, cudaStream_t stream)
    : file_(file), arena_(arena), stream_(stream) {}

WeightLoader::~WeightLoader() {
    if (stream_ && pinned_.get()) cudaStreamSynchronize(stream_);
}

void WeightLoader::finish() {
    if (pinned_.get()) CUDALLM_CUDA(cudaStreamSynchronize(stream_));
}

void WeightLoader::upload(const void* host, std::size_t bytes, void* dst) {
    if (!pinned_.get()) pinned_ = PinnedBuffer(kStagingBytes);
    const char* src = static_cast<const char*>(host);
    for (std::size_t off = 0; off < bytes; off += kStagingBytes) {
        const std::size_t n = std::min(kStagingBytes, bytes - off);
        CUDALLM_CUDA(cudaStreamSynchronize(stream_));
        std::memcpy(pinned_.get(), src + off, n);
        CUDALLM_CUDA(cudaMemcpyAsync(static_cast<char*>(dst) + off, pinned_.get(), n, cudaMemcpyHostToDevice, stream_));
    }
}

DevMat WeightLoader::stacked(const std::vector<Part>& parts) {
    if (parts.empty()) throw std::invalid_argument("empty stacked matrix");
    DevMat m;
    const TensorInfo& first = file_.require(parts[0].name);
    m.type = (int)first.type;
    m.cols = (int)parts[0].cols;
    std::size_t total_rows = 0;
    std::set<std::string> names;  // several row ranges of one tensor (experts) are one load
    for (const Part& p : parts) {
        const TensorInfo& t = file_.require(p.name, p.rows, p.cols);
        if ((int)t.type != m.type || (int)p.cols != m.cols)
            throw std::runtime_error("stacked tensors differ in type or width: " + p.name);
        if (p.row_end > p.rows || p.row_begin > p.row_end) throw std::invalid_argument("bad row range for " + p.name);
        total_rows += p.row_end - p.row_begin;
        if (names.insert(p.name).second) file_.mark_loaded(p.name);
    }
    const long long stride = cl_row_stride(m.type, m.cols);
    if (stride < 0) throw std::runtime_error(std::string("unsupported matrix type ") + ggml_type_name(m.type));
    m.rows = (int)total_rows;
    m.stride = stride;
    m.payload = total_rows * first.row_bytes;
    payload_ += m.payload;
    char* dst = static_cast<char*>(arena_.take(total_rows * (std::size_t)stride));
    m.ptr = dst;
    if (dst == nullptr) return m;
    if (!pinned_.get()) pinned_ = PinnedBuffer(kStagingBytes);
    if (!staging_.get()) staging_ = DeviceBuffer(kStagingBytes);
    const std::size_t rb = first.row_bytes;
    const std::size_t chunk_rows = std::max<std::size_t>(1, kStagingBytes / rb);
    if (rb > kStagingBytes) throw std::runtime_error("row larger than the staging buffer");
    std::size_t out_row = 0;
    for (const Part& p : parts) {
        const TensorInfo& t = file_.require(p.name);
        for (std::size_t r = p.row_begin; r < p.row_end; r += chunk_rows) {
            const std::size_t n = std::min(chunk_rows, p.row_end - r);
            CUDALLM_CUDA(cudaStreamSynchronize(stream_));
            file_.read(t, r * rb, pinned_.get(), n * rb);
            CUDALLM_CUDA(cudaMemcpyAsync(staging_.get(), pinned_.get(), n * rb, cudaMemcpyHostToDevice, stream_));
            CUDALLM_CL(cl_repack_rows(m.type, staging_.get(), dst + out_row * (std::size_t)stride, (int)n, m.cols,
                                      stream_));
            out_row += n;
        }
    }
    return m;
}

DevMat WeightLoader::matrix(const std::string& name, std::size_t rows, std::size_t cols, std::size_t row_begin,
                            std::size_t row_end, std::size_t col_begin, std::size_t col_end) {
    if (row_end == SIZE_MAX) row_end = rows;
    if (col_end == SIZE_MAX) col_end = cols;
    if (col_begin == 0 && col_end == cols) return stacked({Part{name, rows, cols, row_begin, row_end}});
    // Column shard: gather the block-aligned byte range of each row.
    const TensorInfo& t = file_.require(name, rows, cols);
    const std::size_t blk = block_of(t.type);
    if (col_begin % blk || col_end % blk || col_end > cols || col_begin >= col_end || row_end > rows)
        throw std::invalid_argument("column shard of " + name + " is not block aligned");
    file_.mark_loaded(name);
    DevMat m;
    m.type = (int)t.type;
    m.cols = (int)(col_end - col_begin);
    m.rows = (int)(row_end - row_begin);
    m.stride = cl_row_stride(m.type, m.cols);
    if (m.stride < 0) throw std::runtime_error(std::string("unsupported matrix type ") + ggml_type_name(m.type));
    const std::size_t srb = ggml_row_bytes(t.type, m.cols);
    const std::size_t byte0 = ggml_row_bytes(t.type, col_begin);
    m.payload = srb * m.rows;
    payload_ += m.payload;
    char* dst = static_cast<char*>(arena_.take((std::size_t)m.rows * (std::size_t)m.stride));
    m.ptr = dst;
    if (dst == nullptr) return m;
    if (!pinned_.get()) pinned_ = PinnedBuffer(kStagingBytes);
    if (!staging_.get()) staging_ = DeviceBuffer(kStagingBytes);
    const std::size_t chunk_rows = std::max<std::size_t>(1, kStagingBytes / srb);
    for (std::size_t r = 0; r < (std::size_t)m.rows; r += chunk_rows) {
        const std::size_t n = std::min(chunk_rows, (std::size_t)m.rows - r);
        CUDALLM_CUDA(cudaStreamSynchronize(stream_));
        for (std::size_t i = 0; i < n; ++i) {
            file_.read(t, (row_begin + r + i) * t.row_bytes + byte0, static_cast<char*>(pinned_.get()) + i * srb, srb);
        }
        CUDALLM_CUDA(cudaMemcpyAsync(staging_.get(), pinned_.get(), n * srb, cudaMemcpyHostToDevice, stream_));
        CUDALLM_CL(cl_repack_rows(m.type, staging_.get(), dst + r * (std::size_t)m.stride, (int)n, m.cols, stream_));
    }
    return m;
}

float* WeightLoader::matrix_f32(const std::string& name, std::size_t rows, std::size_t cols, std::size_t row_begin,
                                std::size_t row_end) {
    if (row_end == SIZE_MAX) row_end = rows;
    const TensorInfo& t = file_.require(name, rows, cols);
    if (t.type != kF32 && t.type != kF16) throw std::runtime_error(name + " must be F32 or F16");
    file_.mark_loaded(name);
    const std::size_t n = (row_end - row_begin) * cols;
    payload_ += (row_end - row_begin) * t.row_bytes;
    float* dst = static_cast<float*>(arena_.take(n * sizeof(float)));
    if (dst == nullptr) return nullptr;
    std::vector<uint8_t> raw((row_end - row_begin) * t.row_bytes);
    file_.read(t, row_begin * t.row_bytes, raw.data(), raw.size());
    std::vector<float> vals(n);
    if (t.type == kF32) {
        std::memcpy(vals.data(), raw.data(), n * 4);
    } else {
        for (std::size_t i = 0; i < n; ++i) vals[i] = half_to_float_host((uint16_t)(raw[2 * i] | (raw[2 * i + 1] << 8)));
    }
    upload(vals.data(), n * sizeof(float), dst);
    return dst;
}

float* WeightLoader::vector(const std::string& name, std::size_t n, std::size_t begin, std::size_t end) {
    if (end == SIZE_MAX) end = n;
    const TensorInfo& t = file_.require(name);
    if (t.rows * t.cols != n) {
        throw std::runtime_error("unexpected shape for tensor " + name + ": expected " + std::to_string(n) +
                                 " values, got " + std::to_string(t.rows * t.cols));
    }
    if (t.type != kF32 && t.type != kF16) throw std::runtime_error(name + " must be F32 or F16");
    file_.mark_loaded(name);
    const std::size_t esz = t.type == kF32 ? 4 : 2;
    payload_ += (end - begin) * esz;
    float* dst = static_cast<float*>(arena_.take((end - begin) * sizeof(float)));
    if (dst == nullptr) return nullptr;
    std::vector<uint8_t> raw((end - begin) * esz);
    file_.read(t, begin * esz, raw.data(), raw.size());
    std::vector<float> vals(end - begin);
    if (t.type == kF32) {
        std::memcpy(vals.data(), raw.data(), raw.size());
    } else {
        for (std::size_t i = 0; i < vals.size(); ++i)
            vals[i] = half_to_float_host((uint16_t)(raw[2 * i] | (raw[2 * i + 1] << 8)));
    }
    upload(vals.data(), vals.size() * sizeof(float), dst);
    return dst;
}

}  // namespace cudallm
