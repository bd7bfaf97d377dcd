// Canonical form of a two-operand per-tile einsum.
//
// Every label of "lhs,rhs->out" falls in one group:
//   B  in lhs, rhs and out      (batch)
//   M  in lhs and out only      (rows)
//   N  in rhs and out only      (columns)
//   K  not in out               (summed; a label present in one operand only
//                                gets stride 0 on the other side, which sums
//                                it exactly as np.einsum does)
// A label repeated inside one operand (a diagonal, "ii,ij->j") gets the sum
// of its strides. out[b,m,n] = sum_k lhs[b,m,k] * rhs[b,k,n] with element
// offsets from per-group mixed-radix tables. This is the contraction that
// kernel_einsum hands to jnp.einsum with a "z" batch label prepended
// (execution/sparse_dispatch.py:118-125).
#pragma once

#include <stdint.h>

#include "einsparse.h"

namespace es {

constexpr int kMaxGroupLabels = 8;

struct EinGroup {
  int n;                        // labels in this group
  int size[kMaxGroupLabels];    // extent per label (outermost first)
  int lstride[kMaxGroupLabels]; // element stride inside an lhs tile
  int rstride[kMaxGroupLabels];
  int ostride[kMaxGroupLabels];
  int total;                    // product of sizes (1 when empty)
};

struct EinsumDesc {
  EinGroup B, M, N, K;
  int lhs_te, rhs_te, out_te;   // elements per tile
  int out_nd;
  int out_tile[ES_MAX_DIMS];
};

// Parses the kernel string against the operand tile shapes. Returns ES_OK or
// ES_ERR_INVALID (no "->", operand rank mismatch, label size conflict, output
// label absent from the inputs or repeated).
int parse_einsum(const char* ks, const int64_t* lhs_tile, int lhs_nd, const int64_t* rhs_tile, int rhs_nd,
                 EinsumDesc* d);

}  // namespace es
