// Tensor-core (tcgen05 / TMEM) paths of the segmented tile einsum.
#pragma once

#include <cuda_runtime.h>

#include "einsum_desc.h"

namespace es {

// Launches a tensor-core kernel when one covers this contraction (layout,
// dtypes, tile sizes); returns ES_ERR_UNSUPPORTED otherwise so the caller
// can take the SIMT path.
int tc_try_launch(const EinsumDesc& d, const void* lhs, int ldt, const void* rhs, int rdt, const int32_t* pl,
                  const int32_t* pr, const int64_t* seg_off, int64_t nseg, const int32_t* seg_out, void* out,
                  int odt, int precision, cudaStream_t st);

}  // namespace es
