// Tensor-core (tcgen05 / TMEM) path of the segmented tile einsum.
#pragma once

#include <cuda_runtime.h>

#include "einsum_desc.h"

namespace es {

// Geometry of one tensor-core launch, fixed on the host.
struct TcConfig {
  int fp32;        // 1: fp32 operands, 3-pass split TF32; 0: bf16 operands
  int swap;        // 1: compute D^T = panel^T * lhs^T (lhs rows become MMA N)
  int Mt, Kt, Nt;  // tile dims of the plain matmul view
  int G;           // rhs tiles (segments of one strip) per work item
  int slots;       // lhs slots per work item: 1, or 128 / Mt strips stacked
                   // into the 128-row MMA operand (stacked mode)
  int KC;          // k elements per pipeline stage (operand rows of KC elements)
  int swz;         // descriptor layout code of the swizzle: 2 (128 B rows), 4 (64 B), 6 (32 B)
  int stages;
  int halves;      // 128-row MMA halves (M = 128 * halves)
  int n_mma;       // MMA N
  int fold;        // 1 (fp32, swapped, Mt % 32 == 0, 2*Mt <= 256): the lhs hi and lo
                   // copies sit side by side as one N = 2*Mt operand, so
                   // panel_hi x [lhs_hi | lhs_lo] is one MMA; the epilogue adds
                   // the two column blocks
  int col_per_half;  // TMEM columns of one 128-row half of an accumulator
  int acc_bufs;    // TMEM accumulators (2 when they fit: epilogue overlaps the next item)
  int tmem_cols;   // allocated TMEM columns (power of two)
  int lhs_bytes;   // one operand copy of a stage's lhs chunk (all slots)
  int pan_bytes;   // one operand copy of a stage's panel chunk
  int stage_bytes;
  int epi_stage;   // swapped epilogue through shared memory (Nt % 32 == 0): each epilogue
                   // warp transposes its 32 panel rows x 32 lhs rows block and stores
                   // 16-byte row pieces of the output tile
  int epi_dual;    // bf16 operands with the staged epilogue: warps 0-3 (idle without the fp32
                   // split) form a second epilogue group; the groups take alternate blocks
  int epi_warp_bytes;  // staging bytes per epilogue warp (2 KB for bf16 output, 4 KB for fp32)
  int smem_bytes;  // dynamic shared memory per CTA
  int tmem_chain;  // set at launch: fp32 accumulation chains summed in TMEM (one accumulator
                   // at column 0, the running sum at column acc_stride; acc_bufs = 1)
  int rhs_kmajor;  // set by the caller: rhs tiles are stored Nt x Kt (k contiguous), the
                   // transposed form of the contraction's rhs
};

// True when the contraction is a plain tile matmul this path covers:
// lhs (Mt x Kt) k-contiguous, rhs (Kt x Nt) n-contiguous, out (Mt x Nt),
// size-1 batch labels only, both operands f32 or both bf16.
// have_keys: pair_key is available (required for stacked mode).
bool tc_config(const EinsumDesc& d, int ldt, int rdt, int odt, bool have_strips, bool have_keys, TcConfig* c);

// Key blocks of the contracted range for these operands: enough that each
// block's rhs panel fits in L2 (*l2_blocks), and, for few work items, more so
// that a fused launch has several (block, item) units per SM.
int tc_key_blocks(const TcConfig& c, int64_t rhs_rows, bool have_key, int64_t key_extent, int64_t nseg,
                  int* l2_blocks = nullptr);

size_t tc_workspace_size(const TcConfig& c, int64_t rhs_rows, int64_t npairs, int64_t nseg, int nblocks,
                         int64_t key_extent);

int tc_launch(const TcConfig& c, const void* lhs, int64_t lhs_rows, const void* rhs, int64_t rhs_rows,
              const int32_t* pl, const int32_t* pr, int64_t npairs, const int64_t* seg_off, int64_t nseg,
              const int32_t* seg_out, const int64_t* seg_strip, const int32_t* pair_key, int64_t key_extent, void* out,
              int odt, void* ws, size_t ws_bytes, int32_t* err, cudaStream_t st, cudaEvent_t values_ready = nullptr);

}  // namespace es
