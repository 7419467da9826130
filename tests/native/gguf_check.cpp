// Drives the product's GGUF reader (myllm_b200/csrc/host/gguf.cpp) over the
// files named on the command line, for a build with AddressSanitizer and
// UndefinedBehaviorSanitizer: every file is parsed and its metadata and
// tensor table read back; a rejected file must fail with an exception, never
// with a sanitizer report or a crash.  Prints "<accepted> <rejected>".
#include <cstdio>
#include <exception>

#include "gguf.h"

int main(int argc, char** argv) {
    int accepted = 0, rejected = 0;
    for (int i = 1; i < argc; ++i) {
        try {
            cudallm::GgufFile f(argv[i]);
            std::size_t total = f.text("general.architecture").size() + f.array_length("tokenizer.ggml.tokens");
            for (const cudallm::TensorInfo& t : f.tensors()) total += t.bytes + t.dims.size();
            if (!f.tensors().empty()) {
                const cudallm::TensorInfo& t = f.tensors().front();
                unsigned char b[16];
                if (t.bytes >= sizeof(b)) f.read(t, 0, b, sizeof(b));
            }
            ++accepted;
            (void)total;
        } catch (const std::exception&) {
            ++rejected;
        }
    }
    std::printf("%d %d\n", accepted, rejected);
    return 0;
}
