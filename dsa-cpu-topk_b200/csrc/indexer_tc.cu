// Stage 1 (tensor-core path): tcgen05 / TMEM Lightning Indexer for bf16 inputs.
// Not enabled yet in this build: every shape runs the fp32 CUDA-core kernel.
#include "common.cuh"

namespace dsa {

bool indexer_tc_supported(int64_t, int64_t, int) { return false; }

int indexer_scores_tc(const void*, const void*, const float*, float*, int64_t, int64_t, int64_t,
                      int64_t, int64_t, int64_t, int, cudaStream_t) {
    return fail(DSA_ERR_UNSUPPORTED, "indexer_scores_tc: tensor-core path not built");
}

}  // namespace dsa
