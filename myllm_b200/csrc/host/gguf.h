// Streaming GGUF reader: parses metadata and tensor descriptors once, then
// reads any byte range of a tensor with pread.  Tensor payloads are never
// materialised as a whole file image (the reference CPU reader reads the
// whole file into memory, model.cpp:378-395; its GPU reader streams one
// tensor at a time, metal_model.cpp:450-562 and 764-790 — this follows the
// streaming behaviour with its own implementation).
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace cudallm {

enum GgmlType : uint32_t {
    kF32 = 0,
    kF16 = 1,
    kQ4_0 = 2,
    kQ4_1 = 3,
    kQ5_0 = 6,
    kQ5_1 = 7,
    kQ8_0 = 8,
    kQ8_1 = 9,
    kQ2_K = 10,
    kQ3_K = 11,
    kQ4_K = 12,
    kQ5_K = 13,
    kQ6_K = 14,
    kBF16 = 30,
};

const char* ggml_type_name(uint32_t type) noexcept;
// Bytes of one row of `cols` elements; throws std::runtime_error when the
// type is unknown or cols is not block aligned (metal_model.cpp:437-448).
std::size_t ggml_row_bytes(uint32_t type, std::size_t cols);

struct TensorInfo {
    std::string name;
    uint32_t type = 0;
    std::vector<uint64_t> dims;  // dims[0] = columns (innermost)
    std::size_t cols = 0;
    std::size_t rows = 0;        // product of dims[1..]
    std::size_t row_bytes = 0;
    std::size_t offset = 0;      // absolute file offset
    std::size_t bytes = 0;
};

class GgufFile {
public:
    explicit GgufFile(const std::string& path);
    ~GgufFile();
    GgufFile(const GgufFile&) = delete;
    GgufFile& operator=(const GgufFile&) = delete;

    const std::string& path() const noexcept { return path_; }
    const std::vector<TensorInfo>& tensors() const noexcept { return tensors_; }
    bool has_tensor(const std::string& name) const noexcept;
    // Descriptor with a shape check: rows x cols (a 1-D tensor has rows == 1).
    const TensorInfo& require(const std::string& name, std::size_t rows, std::size_t cols) const;
    const TensorInfo& require(const std::string& name) const;

    bool has_key(const std::string& key) const noexcept;
    uint64_t integer(const std::string& key, uint64_t fallback) const;
    // Required positive integer (metadata_size semantics, model.cpp:688-697).
    std::size_t size(const std::string& key) const;
    double real(const std::string& key, double fallback) const;
    std::string text(const std::string& key, const std::string& fallback = {}) const;
    std::size_t array_length(const std::string& key) const;  // 0 if absent
    // The elements of a string array (tokenizer vocabulary, merges); empty if
    // the key is absent or not an array of strings.
    const std::vector<std::string>& strings(const std::string& key) const;

    // pread bytes [offset, offset + bytes) of a tensor's payload.
    void read(const TensorInfo& t, std::size_t offset, void* dst, std::size_t bytes) const;

    // "every tensor consumed" bookkeeping (model.cpp:816-828,
    // metal_model.cpp:960-976).
    void mark_loaded(const std::string& name);
    void ignore_prefix(const std::string& prefix);
    void validate_all_loaded() const;

private:
    std::string path_;
    int fd_ = -1;
    std::size_t file_size_ = 0;
    std::unordered_map<std::string, uint64_t> ints_;
    std::unordered_map<std::string, double> reals_;
    std::unordered_map<std::string, std::string> texts_;
    std::unordered_map<std::string, std::size_t> arrays_;
    std::unordered_map<std::string, std::vector<std::string>> string_arrays_;
    std::vector<TensorInfo> tensors_;
    std::unordered_map<std::string, std::size_t> index_;
    std::unordered_set<std::string> loaded_;
    std::vector<std::string> ignored_prefixes_;
};

}  // namespace cudallm
