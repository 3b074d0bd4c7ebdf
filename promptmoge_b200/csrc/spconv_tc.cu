// tcgen05 (5th-generation tensor core) int8 implicit-GEMM path for the submanifold conv and dense layers.
#include "common.cuh"
#include "rowops.cuh"

namespace pmg {

int gemm_i8_tc(const int8_t*, const int32_t*, int64_t, const uint32_t*, const int32_t*, int64_t, int, int, int,
               const int8_t*, const Epi&, cudaStream_t) {
    return PMG_ERR_UNSUPPORTED;
}

}  // namespace pmg
