/* A plain C host linked against libcudallm.so (tests/test_abi.py builds and
 * runs it): the backend C-ABI's host-only entry points from C, with no GPU. */
#include <stdio.h>
#include <string.h>

#include "cudallm.h"

int main(int argc, char** argv) {
    if (argc < 2) return 2;
    char arch[32];
    uint64_t tensors = 0;
    if (cudallm_gguf_inspect(argv[1], arch, sizeof arch, &tensors) != CUDALLM_OK) {
        fprintf(stderr, "inspect: %s\n", cudallm_last_error());
        return 1;
    }
    cudallm_tp_shard s;
    if (cudallm_tp_plan(13824, 152064, 40, 8, 128, 256, 8, 7, &s) != CUDALLM_OK) return 1;
    if (cudallm_tp_plan(13824, 152064, 40, 8, 128, 256, 3, 0, &s) != CUDALLM_EINVAL) return 1;
    int32_t er[16], el[16], sr[4];
    if (cudallm_ep_plan(16, 4, 4, er, el, sr) != CUDALLM_OK) return 1;
    if (cudallm_create("/nonexistent.gguf", 16, 0, 0, 1, NULL, NULL) != CUDALLM_EINVAL) return 1;
    printf("%s %llu %llu %llu %d %d %d\n", arch, (unsigned long long)tensors, (unsigned long long)s.q_head0,
           (unsigned long long)s.vocab_rows, s.gather_attn, er[13], sr[3]);
    return 0;
}
