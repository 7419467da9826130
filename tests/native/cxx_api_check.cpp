// A C++17 host linked against libcudallm.so (tests/test_abi.py builds and
// runs it): the C++ API is exported, and its exceptions cross the library
// boundary with the reference's types.  Runs without a GPU.
#include <cstdio>
#include <stdexcept>

#include "cuda_llm.h"
#include "cuda_moe_llm.h"

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    const cudallm::TensorParallelShard s = cudallm::plan_tensor_parallel(13824, 152064, 40, 8, 128, 256, 8, 7);
    try {
        cudallm::plan_tensor_parallel(13824, 152064, 40, 8, 128, 256, 3, 0);
        return 1;
    } catch (const std::invalid_argument&) {
    }
    const std::string arch = cudallm::gguf_architecture(argv[1]);
    const char* outcome = "constructed";
    try {
        cudallm::CudaLLM llm(argv[1], 16);  // no device here: a runtime_error, not a crash
        if (!llm.available()) return 1;
    } catch (const std::runtime_error&) {
        outcome = "runtime_error";
    }
    std::printf("%s %zu %d %s\n", arch.c_str(), s.q_head0, (int)s.gather_attn, outcome);
    return 0;
}
