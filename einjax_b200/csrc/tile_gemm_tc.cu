// Tensor-core tile GEMMs (tcgen05 + TMEM) for the segmented tile einsum.
#include "common.cuh"
#include "tile_gemm_tc.h"

namespace es {

int tc_try_launch(const EinsumDesc&, const void*, int, const void*, int, const int32_t*, const int32_t*,
                  const int64_t*, int64_t, const int32_t*, void*, int, int, cudaStream_t) {
  return ES_ERR_UNSUPPORTED;
}

}  // namespace es
