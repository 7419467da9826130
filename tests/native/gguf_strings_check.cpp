// Reads the tokenizer tables of a GGUF file through the product's reader
// (myllm_b200/csrc/host/gguf.cpp): prints the vocabulary and merge counts,
// their first and last entries and tokenizer.ggml.pre, one per line.
#include <cstdio>
#include <exception>

#include "gguf.h"

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    try {
        const cudallm::GgufFile f(argv[1]);
        const auto& v = f.strings("tokenizer.ggml.tokens");
        const auto& m = f.strings("tokenizer.ggml.merges");
        std::printf("%zu\n%zu\n", v.size(), m.size());
        if (!v.empty()) std::printf("%s\n%s\n", v.front().c_str(), v.back().c_str());
        if (!m.empty()) std::printf("%s\n%s\n", m.front().c_str(), m.back().c_str());
        std::printf("%s\n", f.text("tokenizer.ggml.pre").c_str());
    } catch (const std::exception& e) {
        std::printf("error: %s\n", e.what());
    }
    return 0;
}
