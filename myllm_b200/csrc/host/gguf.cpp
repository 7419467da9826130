#include "gguf.h"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstring>
#include <limits>
#include <stdexcept>

namespace cudallm {

namespace {

constexpr uint32_t kMagic = 0x46554747u;  // "GGUF"

enum ValueType : uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32v = 6, kBool = 7,
    kString = 8, kArray = 9, kU64 = 10, kI64 = 11, kF64 = 12,
};

std::size_t checked_mul(std::size_t a, std::size_t b, const std::string& what) {
    if (a != 0 && b > std::numeric_limits<std::size_t>::max() / a) {
        throw std::runtime_error(what + " size overflows size_t");
    }
    return a * b;
}

// Buffered little-endian cursor over the file header, refilled with pread.
class Cursor {
public:
    Cursor(int fd, std::size_t file_size) : fd_(fd), size_(file_size) {}

    std::size_t position() const { return base_ + pos_; }

    void need(std::size_t n) {
        if (position() > size_ || n > size_ - position()) throw std::runtime_error("truncated GGUF file");
        if (pos_ + n <= buf_.size()) return;
        base_ += pos_;
        pos_ = 0;
        const std::size_t want = std::max<std::size_t>(n, 1 << 20);
        const std::size_t avail = std::min(want, size_ - base_);
        buf_.resize(avail);
        std::size_t got = 0;
        while (got < avail) {
            const ssize_t r = ::pread(fd_, buf_.data() + got, avail - got, (off_t)(base_ + got));
            if (r <= 0) throw std::runtime_error("cannot read GGUF header");
            got += (std::size_t)r;
        }
    }

    template <typename T>
    T get() {
        need(sizeof(T));
        T v;
        std::memcpy(&v, buf_.data() + pos_, sizeof(T));
        pos_ += sizeof(T);
        return v;
    }

    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (n > size_) throw std::runtime_error("invalid GGUF string length");
        need((std::size_t)n);
        std::string s(reinterpret_cast<const char*>(buf_.data() + pos_), (std::size_t)n);
        pos_ += (std::size_t)n;
        return s;
    }

    void skip(std::size_t n) {
        need(n);
        pos_ += n;
    }

private:
    int fd_;
    std::size_t size_;
    std::vector<uint8_t> buf_;
    std::size_t base_ = 0;
    std::size_t pos_ = 0;
};

// Arrays of arrays are legal GGUF, but no file this reader serves nests
// them; the limit keeps a crafted chain from exhausting the stack.
constexpr int kMaxArrayDepth = 8;

void skip_value(Cursor& c, uint32_t type, int depth = 0) {
    switch (type) {
    case kU8: case kI8: case kBool: c.skip(1); break;
    case kU16: case kI16: c.skip(2); break;
    case kU32: case kI32: case kF32v: c.skip(4); break;
    case kU64: case kI64: case kF64: c.skip(8); break;
    case kString: c.skip((std::size_t)c.get<uint64_t>()); break;
    case kArray: {
        if (depth >= kMaxArrayDepth) throw std::runtime_error("GGUF metadata arrays nested too deeply");
        const uint32_t et = c.get<uint32_t>();
        const uint64_t n = c.get<uint64_t>();
        for (uint64_t i = 0; i < n; ++i) skip_value(c, et, depth + 1);
        break;
    }
    default: throw std::runtime_error("unsupported GGUF metadata type " + std::to_string(type));
    }
}

}  // namespace

const char* ggml_type_name(uint32_t type) noexcept {
    switch (type) {
    case kF32: return "F32";
    case kF16: return "F16";
    case kQ4_0: return "Q4_0";
    case kQ4_1: return "Q4_1";
    case kQ5_0: return "Q5_0";
    case kQ5_1: return "Q5_1";
    case kQ8_0: return "Q8_0";
    case kQ8_1: return "Q8_1";
    case kQ2_K: return "Q2_K";
    case kQ3_K: return "Q3_K";
    case kQ4_K: return "Q4_K";
    case kQ5_K: return "Q5_K";
    case kQ6_K: return "Q6_K";
    case kBF16: return "BF16";
    default: return "UNKNOWN";
    }
}

std::size_t ggml_row_bytes(uint32_t type, std::size_t cols) {
    std::size_t block = 0, size = 0;
    switch (type) {
    case kF32: block = 1; size = 4; break;
    case kF16: case kBF16: block = 1; size = 2; break;
    case kQ4_0: block = 32; size = 18; break;
    case kQ4_1: block = 32; size = 20; break;
    case kQ5_0: block = 32; size = 22; break;
    case kQ5_1: block = 32; size = 24; break;
    case kQ8_0: block = 32; size = 34; break;
    case kQ8_1: block = 32; size = 40; break;
    case kQ2_K: block = 256; size = 84; break;
    case kQ3_K: block = 256; size = 110; break;
    case kQ4_K: block = 256; size = 144; break;
    case kQ5_K: block = 256; size = 176; break;
    case kQ6_K: block = 256; size = 210; break;
    default: throw std::runtime_error("unsupported GGUF tensor type " + std::to_string(type));
    }
    if (cols % block != 0) throw std::runtime_error(std::string(ggml_type_name(type)) + " row is not block aligned");
    return checked_mul(cols / block, size, std::string(ggml_type_name(type)) + " row");
}

GgufFile::GgufFile(const std::string& path) : path_(path) {
    fd_ = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd_ < 0) throw std::runtime_error("cannot open model: " + path);
    try {
        struct stat st {};
        if (::fstat(fd_, &st) != 0 || st.st_size <= 0) throw std::runtime_error("empty model file");
        file_size_ = (std::size_t)st.st_size;
        Cursor c(fd_, file_size_);
        if (c.get<uint32_t>() != kMagic) throw std::runtime_error("not a GGUF file");
        const uint32_t version = c.get<uint32_t>();
        if (version != 2 && version != 3) throw std::runtime_error("unsupported GGUF version");
        const uint64_t n_tensors = c.get<uint64_t>();
        const uint64_t n_kv = c.get<uint64_t>();
        // every metadata entry takes at least 12 bytes (key length, type) and
        // every tensor descriptor at least 32 (name length, rank, one
        // dimension, type, offset): counts beyond that are corrupt, and must
        // not reach an allocation
        if (n_kv > file_size_ / 12 || n_tensors > file_size_ / 32)
            throw std::runtime_error("invalid GGUF header counts");
        for (uint64_t i = 0; i < n_kv; ++i) {
            const std::string key = c.str();
            const uint32_t type = c.get<uint32_t>();
            switch (type) {
            case kU8: ints_[key] = c.get<uint8_t>(); break;
            case kI8: ints_[key] = (uint64_t)(int64_t)c.get<int8_t>(); break;
            case kU16: ints_[key] = c.get<uint16_t>(); break;
            case kI16: ints_[key] = (uint64_t)(int64_t)c.get<int16_t>(); break;
            case kU32: ints_[key] = c.get<uint32_t>(); break;
            case kI32: ints_[key] = (uint64_t)(int64_t)c.get<int32_t>(); break;
            case kU64: ints_[key] = c.get<uint64_t>(); break;
            case kI64: ints_[key] = (uint64_t)c.get<int64_t>(); break;
            case kBool: ints_[key] = c.get<uint8_t>() ? 1 : 0; break;
            case kF32v: reals_[key] = c.get<float>(); break;
            case kF64: reals_[key] = c.get<double>(); break;
            case kString: texts_[key] = c.str(); break;
            case kArray: {
                const uint32_t et = c.get<uint32_t>();
                const uint64_t n = c.get<uint64_t>();
                arrays_[key] = (std::size_t)n;
                if (et == kString) {
                    // every string takes at least its 8-byte length
                    if (n > (file_size_ - c.position()) / 8) throw std::runtime_error("truncated GGUF file");
                    std::vector<std::string>& v = string_arrays_[key];
                    v.reserve((std::size_t)n);
                    for (uint64_t j = 0; j < n; ++j) v.push_back(c.str());
                } else {
                    for (uint64_t j = 0; j < n; ++j) skip_value(c, et);
                }
                break;
            }
            default: throw std::runtime_error("unsupported GGUF metadata type " + std::to_string(type));
            }
        }
        tensors_.reserve((std::size_t)n_tensors);
        std::vector<uint64_t> rel;
        for (uint64_t i = 0; i < n_tensors; ++i) {
            TensorInfo t;
            t.name = c.str();
            const uint32_t nd = c.get<uint32_t>();
            if (nd == 0 || nd > 4) throw std::runtime_error("invalid tensor rank for " + t.name);
            for (uint32_t d = 0; d < nd; ++d) t.dims.push_back(c.get<uint64_t>());
            t.type = c.get<uint32_t>();
            rel.push_back(c.get<uint64_t>());
            t.cols = (std::size_t)t.dims[0];
            t.rows = 1;
            for (uint32_t d = 1; d < nd; ++d) t.rows = checked_mul(t.rows, (std::size_t)t.dims[d], t.name);
            t.row_bytes = ggml_row_bytes(t.type, t.cols);
            t.bytes = checked_mul(t.row_bytes, t.rows, t.name);
            tensors_.push_back(std::move(t));
        }
        const uint64_t align = integer("general.alignment", 32);
        if (align == 0 || (align & (align - 1))) throw std::runtime_error("invalid GGUF alignment");
        const std::size_t data_start = (c.position() + align - 1) / align * align;
        for (std::size_t i = 0; i < tensors_.size(); ++i) {
            TensorInfo& t = tensors_[i];
            if (rel[i] > file_size_ || data_start > file_size_ - rel[i] ||
                t.bytes > file_size_ - data_start - rel[i])
                throw std::runtime_error("GGUF tensor is outside file: " + t.name);
            t.offset = data_start + (std::size_t)rel[i];
            if (!index_.emplace(t.name, i).second) throw std::runtime_error("duplicate GGUF tensor: " + t.name);
        }
    } catch (...) {
        ::close(fd_);
        fd_ = -1;
        throw;
    }
}

GgufFile::~GgufFile() {
    if (fd_ >= 0) ::close(fd_);
}

bool GgufFile::has_tensor(const std::string& name) const noexcept { return index_.count(name) != 0; }

const TensorInfo& GgufFile::require(const std::string& name) const {
    const auto it = index_.find(name);
    if (it == index_.end()) throw std::runtime_error("missing tensor: " + name);
    return tensors_[it->second];
}

const TensorInfo& GgufFile::require(const std::string& name, std::size_t rows, std::size_t cols) const {
    const TensorInfo& t = require(name);
    if (t.rows != rows || t.cols != cols) {
        throw std::runtime_error("unexpected shape for tensor " + name + ": expected " + std::to_string(rows) + "x" +
                                 std::to_string(cols) + ", got " + std::to_string(t.rows) + "x" +
                                 std::to_string(t.cols));
    }
    return t;
}

bool GgufFile::has_key(const std::string& key) const noexcept {
    return ints_.count(key) || reals_.count(key) || texts_.count(key) || arrays_.count(key);
}

uint64_t GgufFile::integer(const std::string& key, uint64_t fallback) const {
    const auto it = ints_.find(key);
    return it == ints_.end() ? fallback : it->second;
}

std::size_t GgufFile::size(const std::string& key) const {
    const auto it = ints_.find(key);
    if (it == ints_.end()) throw std::runtime_error("missing GGUF metadata: " + key);
    if (it->second == 0 || it->second > std::numeric_limits<std::size_t>::max())
        throw std::runtime_error("invalid GGUF metadata: " + key);
    return (std::size_t)it->second;
}

double GgufFile::real(const std::string& key, double fallback) const {
    const auto it = reals_.find(key);
    return it == reals_.end() ? fallback : it->second;
}

std::string GgufFile::text(const std::string& key, const std::string& fallback) const {
    const auto it = texts_.find(key);
    return it == texts_.end() ? fallback : it->second;
}

const std::vector<std::string>& GgufFile::strings(const std::string& key) const {
    static const std::vector<std::string> none;
    const auto it = string_arrays_.find(key);
    return it == string_arrays_.end() ? none : it->second;
}

std::size_t GgufFile::array_length(const std::string& key) const {
    const auto it = arrays_.find(key);
    return it == arrays_.end() ? 0 : it->second;
}

void GgufFile::read(const TensorInfo& t, std::size_t offset, void* dst, std::size_t bytes) const {
    if (offset > t.bytes || bytes > t.bytes - offset) throw std::runtime_error("read outside tensor " + t.name);
    std::size_t done = 0;
    char* out = static_cast<char*>(dst);
    while (done < bytes) {
        const ssize_t r = ::pread(fd_, out + done, bytes - done, (off_t)(t.offset + offset + done));
        if (r < 0 && errno == EINTR) continue;
        if (r <= 0) throw std::runtime_error("cannot read tensor " + t.name);
        done += (std::size_t)r;
    }
}

void GgufFile::mark_loaded(const std::string& name) {
    if (!loaded_.insert(name).second) throw std::runtime_error("tensor loaded more than once: " + name);
}

void GgufFile::ignore_prefix(const std::string& prefix) { ignored_prefixes_.push_back(prefix); }

void GgufFile::validate_all_loaded() const {
    std::string missing;
    for (const TensorInfo& t : tensors_) {
        if (loaded_.count(t.name)) continue;
        bool ignored = false;
        for (const auto& p : ignored_prefixes_) ignored |= t.name.compare(0, p.size(), p) == 0;
        if (!ignored) missing += " " + t.name;
    }
    if (!missing.empty()) throw std::runtime_error("GGUF contains tensors not mapped by the model:" + missing);
}

}  // namespace cudallm
