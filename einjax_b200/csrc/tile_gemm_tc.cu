// Tensor-core tile GEMM (tcgen05 + TMEM + TMA) for plain block-sparse tile
// matmuls, with the segment-sum fused into the TMEM accumulator.
//
// A work item is up to G segments of one "strip" (segments whose output
// tiles share the lhs-derived coordinates, e.g. one output tile row of a
// block-sparse matmul) -- or, in stacked mode, S = 128 / Mt such sub-strips
// whose lhs tiles are stacked into one 128-row MMA operand. A pre-pass
// (tc_merge_kernel) merges each item's segment pair lists into step records:
// one contracted key, the lhs tile per slot and the rhs tile per segment.
// Each step contributes
//     D(Mt x G*Nt) += lhs(Mt x Kt) * [rhs_0 | ... | rhs_{G-1}](Kt x G*Nt)
// per slot (absent rhs tiles and absent slots are zero), or the transposed
// product when a lone strip has Mt < 128. The item accumulates in TMEM; the
// epilogue writes each segment's output tile once. Summation order over a
// segment's pairs is the join order, as in the reference
// (execution/sparse_dispatch.py:165-169).
//
// fp32 operands use the 3-pass split-TF32 scheme (x = hi + lo; D += A_hi B_hi
// + A_hi B_lo + A_lo B_hi; Ootomo & Yokota, "Recovering single precision
// accuracy from Tensor Cores while surpassing the FP32 theoretical peak
// performance", IJHPCA 2022), giving fp32-level error. hi is x itself, which
// the tensor core reads truncated to TF32, and lo = x - trunc(x); bf16
// operands take one kind::f16 pass with fp32 accumulation. Operands are
// K-major with 32/64/128-byte swizzled rows (the TMA's swizzle modes).
//
// Roles (320 threads): warps 0-3 compute the lo copy of each stage's lhs
// chunk; warp 4 allocates TMEM and issues the MMAs (one elected lane); warp 5
// takes work items from a device-wide queue (largest first), streams their
// step records and issues the TMA loads of the lhs tiles and the bulk copies
// of the rhs "panel" (laid out once per call in the exact shared-memory
// image, hi and lo); warps 6-9 run the epilogue (TMEM lane quadrant = warp %
// 4). Every wait is bounded; on expiry the CTA raises ES_ERR_TIMEOUT, drains
// its own copies and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <climits>
#include <type_traits>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "radix_sort.cuh"
#include "scan.cuh"
#include "tile_gemm_tc.h"

namespace es {
namespace {

constexpr int kProducers = 128;  // warps 0-3: fp32 split / zero-fill of absent tiles
constexpr int kMmaWarp = 4;
constexpr int kSchedWarp = 5;     // work queue, merge, TMA + bulk copies
constexpr int kEpiWarp0 = 6;      // warps 6-9: epilogue (TMEM lane quadrant = warp % 4)
constexpr int kEpilogue = 128;
constexpr int kThreads = 320;
constexpr int kItemLog = 16;
constexpr int kMaxG = 8;
constexpr int kMaxSlots = 8;      // lhs strips stacked into one 128-row MMA operand
constexpr int kMaxStages = 8;
constexpr int kWin = 16;          // prefetched pair entries per segment
constexpr uint64_t kWaitNs = 2000000000ull;   // 2 s without progress: give up
constexpr uint64_t kDrainNs = 100000000ull;   // 100 ms to drain own copies / MMAs
#ifndef EXP_EPI_SLEEP
#define EXP_EPI_SLEEP 0
#endif
constexpr uint32_t kEpiSleepNs = EXP_EPI_SLEEP;
constexpr int64_t kPanelL2Budget = 40ll << 20;  // rhs panel bytes per key block
constexpr int kMaxKeyBlocks = 16;
constexpr int kUnitsPerSm = 4;  // fused launch: (key block, item) units per SM at least
constexpr int kMaxMergeChunks = 64;

// done: 0 data stage, 1 end of a work item, 2 no more items; mask: lhs
// slots present in a data stage (stacked mode)
struct Step {
  int done;
  int mask;
};

// One merge step of a work item, as written by tc_merge_kernel: 16 ints,
// lane j of the scheduler warp loads field j. With S lhs slots and G rhs
// slots: [0, S) lhs tile per slot (-1 absent), [S, S+G) rhs tile per
// segment slot (-1 absent), S+G flags (bit 0: rhs tiles 0..G-1 present and
// consecutive, one copy), S+G+1 first rhs tile. S + G + 2 <= 16.
constexpr int kRecInts = 16;
constexpr int kRecAhead = 4;  // records the scheduler has in flight ahead of use
constexpr int kMaxSplit = 16;  // 16-byte lhs chunks per split thread and stage (lhs operand <= 32 KB)

// A work item: up to S sub-strips (<= G segments of one strip each). The
// scheduler hands the epilogue one entry per accumulation it drains: a
// whole item in one key block, or one chain of it (see TcParams::chain_recs).
struct ItemInfo {
  int s0[kMaxSlots];    // first segment per slot
  int gcnt[kMaxSlots];  // segments per slot (0: empty slot)
  int nsteps;           // records left in this key block (0: nothing in this key block)
  int blk;              // key block of the item
  int acc;              // 1: a chain after the item's first (its earlier chains are summed
                        //    in TMEM, or, without tmem_chain, in the destination)
  int last;             // 1: this accumulation ends the item (written with its end marker)
};

struct Ctrl {
  uint64_t full[kMaxStages];
  uint64_t empty[kMaxStages];
  uint64_t copy[kMaxStages];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  uint32_t progress;  // stages the MMA warp has issued (liveness for long waits)
  Step ring[kMaxStages];
  ItemInfo item_log[kItemLog];  // items in the order this CTA takes them
  int exit_at;                  // item count at which the epilogue stops
};

constexpr int kCtrlBytes = static_cast<int>((sizeof(Ctrl) + 127) / 128 * 128);

struct TcParams {
  TcConfig c;
  const uint8_t* lhs;
  int64_t lhs_rows;
  const uint8_t* pan_hi;
  const uint8_t* pan_lo;
  int64_t rhs_rows;
  const int32_t* recs;      // merge steps, kRecInts ints each
  const int64_t* item_rec;  // per item: nblocks + 1 record boundaries (key blocks)
  int nblocks, blk;         // key blocks, this launch's block
  const uint8_t* zeros;     // zero bytes standing in for absent tiles
  const int64_t* seg_off;
  const int32_t* item_first;
  const int32_t* item_count;
  const int64_t* num_items;
  const int32_t* order;   // item indices, largest work first
  int* queue;             // next position in `order`, zero at launch
  int accumulate;           // 1: add into the output (key blocks after the first)
  int fused;                // 1: one launch over every (key block, item) unit; block b > 0
                            //    writes its sums to part + (b - 1) * part_stride
  int chain_recs;           // > 0: an item's accumulation restarts every chain_recs
                            //    records and the epilogue adds each chain into the
                            //    destination in fp32 (round to nearest), so the tensor
                            //    core's accumulator never sums a long run
  int rn_split;             // fp32: 1 = lo parts rounded to nearest TF32 (lhs: x - trunc(x);
                            //    rhs panel: the tf32_split of x), 0 = truncating split
  float* part;              // fused: per-block partial sums, segment-major rows
  int64_t part_stride;      // elements of one block's partial
  uint8_t* pwritten;        // fused: per (block b > 0, segment) 1 when its partial row was written
  int64_t nseg;             // segments (row stride of pwritten)
  const int32_t* seg_out;
  void* out;
  int odt;
  int32_t* err;
};

// ---------------------------------------------------------------- PTX glue

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// 2-D tiled TMA load (no multicast) completing on an mbarrier.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }


__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// One MMA, issued by one elected lane of a converged warp (all lanes pass
// the same operands).
template <bool F32>
__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accum) {
  if constexpr (F32) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accum)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\telect.sync _|e, 0xffffffff;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accum)
        : "memory");
  }
}

// tcgen05.commit by one elected lane of a converged warp.
__device__ __forceinline__ void umma_commit_warp(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// tcgen05.ld without the wait: the registers are valid only after
// tmem_wait32 on the same array (which names them, so the compiler cannot
// read them earlier).
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_wait32(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// tcgen05.st of 32 consecutive columns of this warp's TMEM lane quadrant
// (one register per column), then the wait for its completion.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])),
      "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
      "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])),
      "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
      "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])),
      "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major operand in a swizzled layout
// (rows of W = 32/64/128 bytes of k, 16-byte chunks XOR-permuted within
// 8-row atoms, SBO = 8 W between atoms), Blackwell descriptor version 1.
// `layout` is the descriptor's layout code (6: 32 B, 4: 64 B, 2: 128 B).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t sbo, uint32_t layout) {
  uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1) << 16;  // LBO (unused for swizzled K-major)
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(layout) << 61;
  return d;
}

// Instruction descriptor: D f32, A/B TF32 (2) or BF16 (1), majors, N>>3, M>>4.
__host__ __device__ constexpr uint32_t make_idesc(bool tf32, bool a_mn, bool b_mn, int M, int N) {
  return (1u << 4) | ((tf32 ? 2u : 1u) << 7) | ((tf32 ? 2u : 1u) << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait. Spins on try_wait (which suspends in hardware) with no
// software sleep while the wait is short, so a pipeline hand-off costs no
// more than the barrier's own latency; backs off after 100 us; gives up
// after kWaitNs without progress. `progress`, when given, is a counter the
// producing side advances; while it moves the wait is not stuck (the
// epilogue waits a whole work item). Returns false when this CTA has
// aborted (here or elsewhere).
__device__ bool wait_bar(uint64_t* bar, uint32_t parity, Ctrl* ctl, int32_t* err,
                         const uint32_t* progress = nullptr, uint32_t sleep_ns = 0) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = global_ns();
  uint32_t seen = progress ? *reinterpret_cast<const volatile uint32_t*>(progress) : 0u;
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (sleep_ns) __nanosleep(sleep_ns);
    if ((i & 31) == 0) {
      if (*reinterpret_cast<volatile int*>(&ctl->abort)) return false;
      const uint64_t now = global_ns();
      if (progress) {
        const uint32_t cur = *reinterpret_cast<const volatile uint32_t*>(progress);
        if (cur != seen) {
          seen = cur;
          t0 = now;
        }
      }
      if (now - t0 > kWaitNs) break;
      if (now - t0 > 100000) __nanosleep(256);
    }
  }
  *reinterpret_cast<volatile int*>(&ctl->abort) = 1;
  if (err) atomicExch(err, ES_ERR_TIMEOUT);
  return false;
}

// wait_bar taken by lane 0 for the whole warp: one poller per warp, and the
// warp stays converged.
__device__ __forceinline__ bool wait_bar_warp(uint64_t* bar, uint32_t parity, Ctrl* ctl, int32_t* err,
                                              const uint32_t* progress = nullptr) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = wait_bar(bar, parity, ctl, err, progress) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Bounded wait that ignores the abort flag (used to drain in-flight work).
__device__ void drain_bar(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return;
    if ((i & 31) == 0 && global_ns() - t0 > kDrainNs) return;
  }
}

// The tensor core reads a kind::tf32 operand as an fp32 container and uses
// its value truncated to TF32 (the low 13 mantissa bits dropped). With x
// itself as the hi operand, the lo operand is the exact fp32 remainder
// x - trunc(x) (|lo| < 2^-10 |x|).
__device__ __forceinline__ float tf32_rem(float x) {
  return x - __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

// x rounded to TF32 (cvt.rna: to nearest, ties away from zero), in an fp32
// container the tensor core reads exactly.
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Rounded split: hi = rna(x), lo = rna(x - hi) (x - hi is exact, |x - hi| <=
// 2^-11 |x|). Both parts round to nearest, so the 3-pass product's error
// (the dropped lo*lo term and lo's rounding, ~2^-22 |ab|) has no sign bias;
// the truncating split (hi = x, lo = x - trunc(x)) errs toward zero.
__device__ __forceinline__ void tf32_split(float x, float& hi, float& lo) {
  hi = tf32_rna(x);
  lo = tf32_rna(x - hi);
}

__device__ __forceinline__ void tf32_split4(const float4& x, bool rn, float4& hi, float4& lo) {
  if (rn) {
    tf32_split(x.x, hi.x, lo.x);
    tf32_split(x.y, hi.y, lo.y);
    tf32_split(x.z, hi.z, lo.z);
    tf32_split(x.w, hi.w, lo.w);
  } else {
    hi = x;
    lo = make_float4(tf32_rem(x.x), tf32_rem(x.y), tf32_rem(x.z), tf32_rem(x.w));
  }
}

// Operand layout of one stage as the MMA warp sees it.
struct MmaArgs {
  uint32_t smem0, tmem;
  int lane;
  uint32_t sbo, layout, col_per_half, acc_stride;
  uint32_t off_m, off_n;  // hi copies of the M and N operands in a stage
  uint32_t lo_m, lo_n;    // distance to their lo copies (fp32)
  uint32_t idesc, idesc2;
};

// Waits (warp-wide) until the epilogue has released the accumulator buffer
// that item item_iter will use; false when the CTA aborted. Kept out of line:
// it only runs for items without steps and at the exit mark.
__device__ __noinline__ bool acc_released(Ctrl* ctl, int32_t* err, uint32_t item_iter, int acc_bufs) {
  if (item_iter < static_cast<uint32_t>(acc_bufs)) return true;
  const uint32_t b = item_iter % acc_bufs;
  return wait_bar_warp(&ctl->acc_empty[b], ((item_iter / acc_bufs) - 1) & 1u, ctl, err);
}

// MMA warp. The whole warp runs this loop on identical values; one elected
// lane issues each MMA. The issue order of a stage is fixed at compile time
// (FOLD, KS k-steps, H halves): with runtime branches between the MMAs each
// one costs several times its tensor-pipe time.
template <bool F32, bool FOLD, int KS, int H>
__device__ void mma_role(const TcParams& p, Ctrl* ctl, const MmaArgs& m) {
  const TcConfig& c = p.c;
  const int lane = m.lane;
  uint32_t it = 0, item_iter = 0;
  int stage = 0;
  uint32_t ph = 0;
  bool first = true, aborted = false;
  uint32_t acc = m.tmem;
  while (true) {
    // fp32 stages pass through the split warps; bf16 stages go straight
    // from the copies to the MMAs
    if (!wait_bar_warp(F32 ? &ctl->full[stage] : &ctl->copy[stage], ph, ctl, p.err)) {
      aborted = true;
      break;
    }
    const int d = __shfl_sync(0xffffffffu, ctl->ring[stage].done, 0);
    if (__builtin_expect(d != 0, 0)) {
      // an item without steps (or the exit mark) still hands accumulator
      // buffer b to the epilogue: wait until the epilogue has released it,
      // so that each of the buffer's barrier phases is consumed once
      if ((d == 2 || first) && !acc_released(ctl, p.err, item_iter, c.acc_bufs)) {
        aborted = true;
        break;
      }
      if (lane == 0) {
        mbar_arrive(&ctl->empty[stage]);
        const int b = static_cast<int>(item_iter % c.acc_bufs);
        if (d == 1) {
          if (first) mbar_arrive(&ctl->acc_full[b]);  // nothing accumulated for this item
          else umma_commit(&ctl->acc_full[b]);
        } else {
          // no more items: wake the epilogue with the exit mark
          *reinterpret_cast<volatile int*>(&ctl->exit_at) = static_cast<int>(item_iter);
          __threadfence_block();
          mbar_arrive(&ctl->acc_full[b]);
        }
      }
      __syncwarp();
      ++it;
      if (++stage == c.stages) {
        stage = 0;
        ph ^= 1u;
      }
      if (d == 2) break;
      ++item_iter;
      first = true;
      continue;
    }
    if (first) {
      // the accumulator buffer must have been read out by the epilogue
      const uint32_t b = item_iter % c.acc_bufs;
      if (item_iter >= static_cast<uint32_t>(c.acc_bufs) &&
          !wait_bar_warp(&ctl->acc_empty[b], ((item_iter / c.acc_bufs) - 1) & 1u, ctl, p.err)) {
        aborted = true;
        break;
      }
      acc = m.tmem + b * m.acc_stride;
    }
    tc_fence_after();
    const uint32_t sb = m.smem0 + static_cast<uint32_t>(stage * c.stage_bytes);
    const uint32_t m0 = sb + m.off_m, n0 = sb + m.off_n;
    const uint32_t acc_first = first ? 0u : 1u;
    if constexpr (FOLD) {
      // per k-step: panel_hi x [lhs_hi | lhs_lo] (N = 2 Mt) for each half,
      // then panel_lo x lhs_hi for each half
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const uint32_t koff = ks * 32;  // one MMA k-step = 32 bytes of a swizzled row
        const uint32_t acc0 = ks == 0 ? acc_first : 1u;
        const uint64_t b_hi = smem_desc(n0 + koff, m.sbo, m.layout);
#pragma unroll
        for (int h = 0; h < H; ++h)
          umma<true>(acc + h * m.col_per_half, smem_desc(m0 + koff + h * 16 * m.sbo, m.sbo, m.layout), b_hi,
                     m.idesc2, acc0);
#pragma unroll
        for (int h = 0; h < H; ++h)
          umma<true>(acc + h * m.col_per_half, smem_desc(m0 + m.lo_m + koff + h * 16 * m.sbo, m.sbo, m.layout), b_hi,
                     m.idesc, 1u);
      }
    } else {
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
        const uint32_t koff = ks * 32;
        const uint32_t acc0 = ks == 0 ? acc_first : 1u;
        const uint64_t b_hi = smem_desc(n0 + koff, m.sbo, m.layout);
#pragma unroll
        for (int h = 0; h < H; ++h) {
          const uint32_t dt = acc + h * m.col_per_half;
          const uint32_t hoff = koff + h * 16 * m.sbo;  // rows 128h.. of the M operand
          const uint64_t a_hi = smem_desc(m0 + hoff, m.sbo, m.layout);
          umma<F32>(dt, a_hi, b_hi, m.idesc, acc0);
          if constexpr (F32) {
            umma<true>(dt, a_hi, smem_desc(n0 + m.lo_n + koff, m.sbo, m.layout), m.idesc, 1u);
            umma<true>(dt, smem_desc(m0 + m.lo_m + hoff, m.sbo, m.layout), b_hi, m.idesc, 1u);
          }
        }
      }
    }
    umma_commit_warp(&ctl->empty[stage]);
    if (lane == 0) *reinterpret_cast<volatile uint32_t*>(&ctl->progress) = it;
    __syncwarp();
    first = false;
    ++it;
    if (++stage == c.stages) {
      stage = 0;
      ph ^= 1u;
    }
  }
  if (aborted && lane == 0) {
    umma_commit(&ctl->drain);
    drain_bar(&ctl->drain, 0);
  }
  __syncwarp();
}

template <bool F32, bool FOLD>
__device__ void mma_dispatch(const TcParams& p, Ctrl* ctl, const MmaArgs& m, int ksteps, int halves) {
  if (halves == 2) {
    switch (ksteps) {
      case 1: mma_role<F32, FOLD, 1, 2>(p, ctl, m); return;
      case 2: mma_role<F32, FOLD, 2, 2>(p, ctl, m); return;
      case 4: mma_role<F32, FOLD, 4, 2>(p, ctl, m); return;
      default: mma_role<F32, FOLD, 8, 2>(p, ctl, m); return;
    }
  }
  switch (ksteps) {
    case 1: mma_role<F32, FOLD, 1, 1>(p, ctl, m); return;
    case 2: mma_role<F32, FOLD, 2, 1>(p, ctl, m); return;
    case 4: mma_role<F32, FOLD, 4, 1>(p, ctl, m); return;
    default: mma_role<F32, FOLD, 8, 1>(p, ctl, m); return;
  }
}

// Split warps (fp32): each data stage's raw lhs chunk (the hi operand as it
// is) gets its lo copy, x - trunc_tf32(x); slots absent from the step
// (stacked mode) become zeros in both copies. PER bounds the 16-byte chunks
// per thread at compile time, so the loads are all issued before the stores.
template <int PER, bool RNLO>
__device__ void split_role(const TcParams& p, Ctrl* ctl, uint8_t* smem, int off_lhs, int slot_bytes, int tid) {
  const TcConfig& c = p.c;
  const int nf = c.lhs_bytes / 16;
  const int slot_f4 = slot_bytes / 16;
  int slot_of[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) slot_of[j] = (tid + j * kProducers) / slot_f4;
  int stage = 0;
  uint32_t ph = 0;
  while (true) {
    if (!wait_bar(&ctl->copy[stage], ph, ctl, p.err)) break;
    const int d = ctl->ring[stage].done;
    if (!d) {
      uint8_t* sbase = smem + stage * c.stage_bytes;
      const int mask = ctl->ring[stage].mask;
      float4 x[PER];
      bool on[PER];
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        const int f = tid + j * kProducers;
        on[j] = f < nf && ((mask >> slot_of[j]) & 1);
        x[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (on[j]) x[j] = *reinterpret_cast<const float4*>(sbase + off_lhs + f * 16);
      }
#pragma unroll
      for (int j = 0; j < PER; ++j) {
        const int f = tid + j * kProducers;
        if (f < nf) {
          // hi stays the raw chunk (read truncated to TF32 by the tensor
          // core); lo = x - trunc(x), rounded to nearest TF32 with RNLO
          float4 lo = make_float4(tf32_rem(x[j].x), tf32_rem(x[j].y), tf32_rem(x[j].z), tf32_rem(x[j].w));
          if (RNLO) lo = make_float4(tf32_rna(lo.x), tf32_rna(lo.y), tf32_rna(lo.z), tf32_rna(lo.w));
          *reinterpret_cast<float4*>(sbase + off_lhs + c.lhs_bytes + f * 16) = lo;
          if (!on[j]) *reinterpret_cast<float4*>(sbase + off_lhs + f * 16) = x[j];  // absent slot: zero hi too
        }
      }
      fence_proxy_async();
    }
    mbar_arrive(&ctl->full[stage]);
    if (++stage == c.stages) {
      stage = 0;
      ph ^= 1u;
    }
    if (d == 2) break;
  }
}

template <bool RNLO>
__device__ void split_dispatch(const TcParams& p, Ctrl* ctl, uint8_t* smem, int off_lhs, int slot_bytes, int tid,
                               int per) {
  if (per <= 1) split_role<1, RNLO>(p, ctl, smem, off_lhs, slot_bytes, tid);
  else if (per <= 2) split_role<2, RNLO>(p, ctl, smem, off_lhs, slot_bytes, tid);
  else if (per <= 4) split_role<4, RNLO>(p, ctl, smem, off_lhs, slot_bytes, tid);
  else if (per <= 8) split_role<8, RNLO>(p, ctl, smem, off_lhs, slot_bytes, tid);
  else split_role<16, RNLO>(p, ctl, smem, off_lhs, slot_bytes, tid);
}

// Swapped epilogue through shared memory (TcConfig::epi_stage): accumulator
// row r = h * 128 + 32 * quad + lane is column n of output tile g = r / Nt,
// and its TMEM columns are the tile's rows m. Per 32 x 32 block the warp
// writes its columns into shared memory (stg: 4 KB for fp32 output, 2 KB for
// bf16) and reads back 16-byte pieces of rows, which it stores (or adds)
// into the output tile.
__device__ __forceinline__ void epi_store_block(const TcParams& p, void* obase, bool accm, const uint32_t (&r)[32],
                                                int64_t tile0, int m0, bool empty, float* stg, int lane) {
  const TcConfig& c = p.c;
  const int rows = c.Mt - m0 < 32 ? c.Mt - m0 : 32;
  if (p.odt == ES_F32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) stg[j * 32 + lane] = empty ? 0.f : __uint_as_float(r[j]);
    __syncwarp();
    // old values are loaded four pieces at a time before their stores (the
    // caller holds two 32-register TMEM blocks, so not all eight)
#pragma unroll
    for (int i0 = 0; i0 < 8; i0 += 4) {
      float4 old[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int j = (i0 + q) * 4 + (lane >> 3), piece = lane & 7;
        old[q] = (accm && j < rows) ? reinterpret_cast<const float4*>(static_cast<float*>(obase) + tile0 +
                                                                      static_cast<int64_t>(m0 + j) * c.Nt)[piece]
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int j = (i0 + q) * 4 + (lane >> 3), piece = lane & 7;
        if (j < rows) {
          float4 x = reinterpret_cast<const float4*>(stg + j * 32)[piece];
          x.x += old[q].x;
          x.y += old[q].y;
          x.z += old[q].z;
          x.w += old[q].w;
          reinterpret_cast<float4*>(static_cast<float*>(obase) + tile0 + static_cast<int64_t>(m0 + j) * c.Nt)[piece] =
              x;
        }
      }
    }
  } else if (accm) {
    // add the old values in fp32 before the one rounding: two passes of 16
    // rows through the 2 KB staging area
#pragma unroll
    for (int pass = 0; pass < 2; ++pass) {
#pragma unroll
      for (int j = 0; j < 16; ++j) stg[j * 32 + lane] = empty ? 0.f : __uint_as_float(r[pass * 16 + j]);
      __syncwarp();
#pragma unroll
      for (int it = 0; it < 2; ++it) {
        const int j = it * 8 + (lane >> 2), piece = lane & 3;
        if (pass * 16 + j < rows) {
          uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(obase) + tile0 +
                                                static_cast<int64_t>(m0 + pass * 16 + j) * c.Nt) +
                       piece;
          const uint4 o = *dst;
          const uint32_t ow[4] = {o.x, o.y, o.z, o.w};
          uint32_t nw[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float a0 = stg[j * 32 + piece * 8 + 2 * q] + __uint_as_float(ow[q] << 16);
            const float a1 = stg[j * 32 + piece * 8 + 2 * q + 1] + __uint_as_float(ow[q] & 0xFFFF0000u);
            const __nv_bfloat162 b2 = __floats2bfloat162_rn(a0, a1);
            nw[q] = *reinterpret_cast<const uint32_t*>(&b2);
          }
          *dst = make_uint4(nw[0], nw[1], nw[2], nw[3]);
        }
      }
      __syncwarp();
    }
    return;
  } else {
    __nv_bfloat16* sb16 = reinterpret_cast<__nv_bfloat16*>(stg);
#pragma unroll
    for (int j = 0; j < 32; ++j) sb16[j * 32 + lane] = __float2bfloat16_rn(empty ? 0.f : __uint_as_float(r[j]));
    __syncwarp();
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int j = it * 8 + (lane >> 2), piece = lane & 3;
      if (j < rows)
        reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(obase) + tile0 + static_cast<int64_t>(m0 + j) * c.Nt)
            [piece] = reinterpret_cast<const uint4*>(sb16 + j * 32)[piece];
    }
  }
  __syncwarp();
}

// The blocks t0, t0 + tstep, ... (block t: half t / nmb, lhs rows 32 (t %
// nmb)..) of one item for one epilogue warp; with two epilogue groups each
// takes every other block. tacc: the accumulator's first column, in this
// warp's TMEM lane quadrant. The next block's TMEM load is in flight while
// a block is stored.
__device__ void epi_swap_staged(const TcParams& p, const ItemInfo& info, void* obase, const int32_t* oseg, bool accm,
                                uint32_t tacc, int quad, int lane, float* stg, bool empty, int t0, int tstep) {
  const TcConfig& c = p.c;
  const int s0 = info.s0[0], gcnt = info.gcnt[0];
  const int nmb = (c.Mt + 31) / 32;
  const int nblk = c.halves * nmb;
  uint32_t ra[32], rb[32];
  // per half: the output tile's column-n0 offset, or -1 when the warp's
  // rows are past the item's segments
  int64_t t0a = -1, t0b = -1;
  for (int h = 0; h < c.halves; ++h) {
    const int r0 = h * 128 + quad * 32;
    const int g0 = r0 / c.Nt;
    if (g0 < gcnt) {
      const int64_t row = oseg ? oseg[s0 + g0] : static_cast<int64_t>(s0 + g0);
      (h == 0 ? t0a : t0b) = row * c.Mt * c.Nt + r0 % c.Nt;
    }
  }
  auto tile_of = [&](int t) { return t / nmb == 0 ? t0a : t0b; };
  auto addr = [&](int t) {
    return tacc + static_cast<uint32_t>((t / nmb) * c.col_per_half + (t % nmb) * 32);
  };
  if (t0 >= nblk) return;
  tmem_ld32_async(addr(t0), ra);
  tmem_wait32(ra);
  for (int t = t0; t < nblk; t += 2 * tstep) {
    const int u = t + tstep;
    if (u < nblk) tmem_ld32_async(addr(u), rb);
    if (tile_of(t) >= 0) epi_store_block(p, obase, accm, ra, tile_of(t), (t % nmb) * 32, empty, stg, lane);
    if (u < nblk) {
      tmem_wait32(rb);
      if (u + tstep < nblk) tmem_ld32_async(addr(u + tstep), ra);
      if (tile_of(u) >= 0) epi_store_block(p, obase, accm, rb, tile_of(u), (u % nmb) * 32, empty, stg, lane);
      if (u + tstep < nblk) tmem_wait32(ra);
    }
  }
}

template <bool F32>
__global__ void __launch_bounds__(kThreads, 1) tc_strip_kernel(const TcParams p,
                                                               const __grid_constant__ CUtensorMap lhs_map) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // swizzled operands need 1024-byte aligned atoms; offset the shared array
  // itself (not through an integer) so accesses stay shared-memory accesses
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const TcConfig& c = p.c;
  Ctrl* ctl = reinterpret_cast<Ctrl*>(smem + c.stages * c.stage_bytes);  // after the aligned ring
  uint8_t* epi_stg = smem + c.stages * c.stage_bytes + kCtrlBytes;      // swapped epilogue staging
  const bool dual = !F32 && c.epi_stage && c.epi_dual;  // warps 0-3: second epilogue group
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t W = *p.num_items;

  constexpr int NH = F32 ? 2 : 1;      // operand copies: hi (and lo)
  constexpr int KSTEP = F32 ? 8 : 16;  // k per MMA instruction
  constexpr int ESZ = F32 ? 4 : 2;
  // both operands are K-major and swizzled: rows of W = KC * ESZ bytes,
  // atoms of 8 rows (SBO = 8 W)
  const int sbo = 8 * c.KC * ESZ;
  const int blk_bytes = c.Nt * c.KC * ESZ;  // one rhs tile's k-chunk = one panel slot
  const int nchunks = c.Kt / c.KC;
  // stage layout: [lhs hi | lhs lo | panel hi | panel lo] (bf16: [lhs | panel]);
  // the TMA lands the raw lhs chunk, already in canonical order, in the last
  // lhs buffer, where the fp32 split rewrites it chunk by chunk in place.
  // Stacked mode: slot s owns rows [s*Mt, s*Mt + Mt) of the lhs operand.
  const int off_lhs = 0;
  const int off_raw = off_lhs;  // the TMA lands the raw lhs chunk in the hi buffer
  const int off_pan = NH * c.lhs_bytes;
  const int slot_bytes = c.lhs_bytes / c.slots;  // one slot's rows of the lhs operand
  const int col_per_half = c.col_per_half;
  const int acc_stride = c.halves * col_per_half;  // TMEM columns of one accumulator

  if (tid == 0) {
    for (int s = 0; s < c.stages; ++s) {
      mbar_init(&ctl->full[s], kProducers);
      mbar_init(&ctl->empty[s], 1);
      mbar_init(&ctl->copy[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->acc_full[b], 1);
      mbar_init(&ctl->acc_empty[b], dual ? 2 * kEpilogue : kEpilogue);
    }
    mbar_init(&ctl->drain, 1);
    ctl->abort = 0;
    ctl->progress = 0;
    ctl->exit_at = -1;
    fence_mbar_init();
  }
  if (warp == kMmaWarp) tmem_alloc(&ctl->tmem_base, static_cast<uint32_t>(c.tmem_cols));
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp == kSchedWarp) {
    // ------------------- scheduler: work queue, merge-step records, copies
    // Records of an item are streamed kRecAhead ahead: lane j < kRecInts
    // holds field j of a record, so one coalesced 64-byte load brings a
    // whole step. Absent rhs tiles are copied from the zero buffer; absent
    // lhs slots (stacked mode) are zeroed by the split warps.
    const int S = c.slots, G = c.G;
    const int64_t W1 = W;                      // sub-strips
    const int64_t nitems = (W1 + S - 1) / S;  // work items of S sub-strips
    // units handed out by the queue: the items of this launch's key block, or
    // (fused) every (key block, item) pair, block-major so that the CTAs in
    // flight share one or two blocks' rhs panel in L2
    const int64_t nunits = p.fused ? nitems * p.nblocks : nitems;
    uint32_t it = 0;
    int stage = 0;
    uint32_t ph = 0;
    bool aborted = false;
    const int jslot = lane / NH;  // panel slot this lane copies when tiles are not consecutive
    const int jhl = lane % NH;
    uint64_t zmask = 0;  // bit stage * kMaxG + g: panel slot g of the stage holds zeros (bf16)
    // Work-item prefetch. With many items per CTA (deep) the queue position
    // of item i+2 is claimed at the start of item i and the metadata and
    // first records follow one item behind, so every dependent load has a
    // whole item's copies to complete behind. With few items per CTA a
    // claim held that long unbalances the largest-first queue, so the next
    // item is claimed during the current item's last kRecAhead steps and its
    // metadata and records are loaded at the item's end.
    const bool deep = nunits >= 16 * static_cast<int64_t>(gridDim.x);
    int nq_raw = 0;  // lane 0: raw atomic result
    int nq = 0, n_ss = -1, n_s0 = 0, n_gcnt = 0, pf = 0;  // next item (A)
    int64_t n_rb = 0, n_re = 0;
    int n_ahead[kRecAhead] = {};
    int bq = 0, b_ss = -1;  // deep: the item after next (B)
    int64_t b_rb = 0, b_re = 0;
    auto load_meta = [&](int q_, int64_t& rb_, int64_t& re_, int& ss_) {
      if (q_ < nunits) {
        const int64_t qi = p.fused ? q_ % nitems : q_;
        const int blk_ = p.fused ? static_cast<int>(q_ / nitems) : p.blk;
        const int64_t* ib = p.item_rec + qi * (p.nblocks + 1) + blk_;
        rb_ = ib[0];
        re_ = ib[1];
        const int64_t sub = qi * S + lane;
        ss_ = (lane < S && sub < W1) ? p.order[sub] : -1;
      }
    };
    auto load_info = [&]() {
      if (nq < nunits) {
        n_s0 = n_ss >= 0 ? p.item_first[n_ss] : 0;
        n_gcnt = n_ss >= 0 ? p.item_count[n_ss] : 0;
#pragma unroll
        for (int a = 0; a < kRecAhead; ++a)
          n_ahead[a] = (lane < kRecInts && n_rb + a < n_re) ? __ldg(p.recs + (n_rb + a) * kRecInts + lane) : 0;
      }
    };
    auto pf_advance = [&]() {  // shallow mode: one stage for the next item
      if (pf == 0) {
        if (lane == 0) nq_raw = atomicAdd(p.queue, 1);
      } else if (pf == 1) {
        nq = __shfl_sync(0xffffffffu, nq_raw, 0);
        load_meta(nq, n_rb, n_re, n_ss);
      } else if (pf == 2) {
        load_info();
      }
      ++pf;
    };
    if (deep) {
      int v0 = 0, v1 = 0;
      if (lane == 0) {
        v0 = atomicAdd(p.queue, 1);
        v1 = atomicAdd(p.queue, 1);
        nq_raw = atomicAdd(p.queue, 1);
      }
      nq = __shfl_sync(0xffffffffu, v0, 0);
      bq = __shfl_sync(0xffffffffu, v1, 0);
      load_meta(nq, n_rb, n_re, n_ss);
      load_meta(bq, b_rb, b_re, b_ss);
      load_info();
    } else {
      pf_advance();
      pf_advance();
      pf_advance();
    }
    // item_iter counts the items handed to the MMA warp and the epilogue
    for (uint32_t item_iter = 0; !aborted;) {
      const int q = nq;
      const int64_t rb = n_rb, re = n_re;
      const int s0_cur = n_s0, gcnt_cur = n_gcnt;
      int ahead[kRecAhead];
#pragma unroll
      for (int a = 0; a < kRecAhead; ++a) ahead[a] = n_ahead[a];
      if (deep) {
        // B becomes the next item; claim the one after it
        nq = bq;
        n_rb = b_rb;
        n_re = b_re;
        n_ss = b_ss;
        bq = __shfl_sync(0xffffffffu, nq_raw, 0);
        if (lane == 0 && bq < nunits) nq_raw = atomicAdd(p.queue, 1);
        load_meta(bq, b_rb, b_re, b_ss);
        load_info();
        pf = 3;
      } else {
        pf = 0;
      }
      if (q >= nunits) {
        // no more items: exit marker
        if (!wait_bar(&ctl->empty[stage], ph ^ 1u, ctl, p.err)) {
          aborted = true;
          break;
        }
        if (lane == 0) {
          ctl->ring[stage].done = 2;
          mbar_arrive_expect_tx(&ctl->copy[stage], 0);
        }
        __syncwarp();
        break;
      }
      const int cur_blk = p.fused ? static_cast<int>(q / nitems) : p.blk;
      if (p.fused && cur_blk > 0) {
        // every unit is visited once: its segments' partial rows are marked
        // written (it has records, so its epilogue writes them) or not, and
        // the ordered addition skips the unwritten ones
        uint8_t* wr = p.pwritten + static_cast<int64_t>(cur_blk - 1) * p.nseg + s0_cur;
        const uint8_t v = re > rb ? 1 : 0;
        for (int g = 0; g < gcnt_cur; ++g) wr[g] = v;
      }
      if ((p.accumulate || cur_blk > 0) && re == rb) {
        // nothing to add from this key block: the item is not handed on
        while (pf < 3) pf_advance();
        continue;
      }
      auto log_item = [&](int64_t left, int acc) {
        if (lane < kMaxSlots) {
          ItemInfo& info = ctl->item_log[item_iter % kItemLog];
          info.s0[lane] = s0_cur;
          info.gcnt[lane] = gcnt_cur;
          if (lane == 0) {
            info.nsteps = static_cast<int>(left);
            info.blk = cur_blk;
            info.acc = acc;
          }
        }
        __syncwarp();
      };
      log_item(re - rb, 0);
      int since = 0;  // records of the current chain
      // ahead[] is a ring indexed at compile time (the loop below is
      // unrolled by kRecAhead): record r sits in ahead[r % kRecAhead] and is
      // replaced by record r + kRecAhead as soon as it is read, so no step
      // waits on the load issued by the step before it
      for (int64_t r = rb; r < re && !aborted;) {
        if (pf == 0 && re - r <= kRecAhead) pf_advance();  // shallow: claim the next item near the end
#pragma unroll
        for (int a = 0; a < kRecAhead; ++a) {
        if (r >= re || aborted) break;
        const int cur = ahead[a];
        ahead[a] = (lane < kRecInts && r + kRecAhead < re) ? __ldg(p.recs + (r + kRecAhead) * kRecInts + lane) : 0;
        ++r;
        const int my_lhs = __shfl_sync(0xffffffffu, cur, lane & (kMaxSlots - 1));  // lanes < S: slot lane
        const int flags = __shfl_sync(0xffffffffu, cur, S + G);
        const int rhs0 = __shfl_sync(0xffffffffu, cur, S + G + 1);
        const int my_rhs = __shfl_sync(0xffffffffu, cur, S + (jslot & (kMaxG - 1)));
        const bool my_lok = lane < S && my_lhs >= 0 && my_lhs < p.lhs_rows;
        const uint32_t mask = __ballot_sync(0xffffffffu, my_lok);
        // fp32: absent slots are zeroed by the split warps; bf16 (one slot):
        // an absent lhs tile is copied from the zero buffer
        const uint32_t lhs_tx = F32 ? static_cast<uint32_t>(__popc(mask)) * static_cast<uint32_t>(slot_bytes)
                                    : static_cast<uint32_t>(c.lhs_bytes);
        const bool consec = (flags & 1) != 0;
        // bf16, scattered rhs tiles: absent panel slots are zero-filled in
        // shared memory by this warp (and left alone when the stage's slot
        // already holds zeros) instead of copied from the zero buffer
        const bool zfill = !F32 && !consec;
        const uint32_t present =
            zfill ? __ballot_sync(0xffffffffu, lane < G && my_rhs >= 0 && my_rhs < p.rhs_rows) : 0u;
        const uint32_t absent = zfill ? (((1u << G) - 1u) & ~present) : 0u;
        const uint32_t pan_tx =
            zfill ? static_cast<uint32_t>(__popc(present) * blk_bytes) : static_cast<uint32_t>(G * NH * blk_bytes);
        for (int chunk = 0; chunk < nchunks; ++chunk) {
          if (!wait_bar(&ctl->empty[stage], ph ^ 1u, ctl, p.err)) {
            aborted = true;
            break;
          }
          const int k0 = chunk * c.KC;
          uint8_t* sbase = smem + stage * c.stage_bytes;
          if (!F32 && !zfill) {
            // the copy below overwrites every panel slot of this stage
            zmask &= ~(0xFFull << (stage * kMaxG));
          }
          if (zfill) {
            const int sh = stage * kMaxG;
            uint32_t need = absent & ~static_cast<uint32_t>((zmask >> sh) & 0xFFull);
            zmask = (zmask & ~(0xFFull << sh)) | (static_cast<uint64_t>(absent) << sh);
            if (need) {
              while (need) {
                const int g = __ffs(need) - 1;
                need &= need - 1;
                uint4* z = reinterpret_cast<uint4*>(sbase + off_pan + g * blk_bytes);
                for (int i = lane; i < blk_bytes / 16; i += 32) z[i] = make_uint4(0u, 0u, 0u, 0u);
              }
              fence_proxy_async();  // the MMAs read these zeros through the async proxy
              __syncwarp();
            }
          }
          if (lane == 0) {
            ctl->ring[stage].done = 0;
            ctl->ring[stage].mask = static_cast<int>(mask);
            mbar_arrive_expect_tx(&ctl->copy[stage], lhs_tx + pan_tx);
          }
          __syncwarp();
          // raw lhs chunk of slot s straight into the canonical K-major
          // layout, at the slot's rows of the operand
          if (my_lok)
            tma_load_2d(sbase + off_raw + lane * slot_bytes, &lhs_map, k0, my_lhs * c.Mt, &ctl->copy[stage]);
          else if (!F32 && lane == 0)
            bulk_g2s(sbase + off_raw, p.zeros, static_cast<uint32_t>(c.lhs_bytes), &ctl->copy[stage]);
          // panel: per k-chunk the pre-laid rhs tiles sit tile after tile, so
          // consecutive rhs tiles (a dense rhs row) arrive in one copy
          const int64_t cbase = static_cast<int64_t>(chunk) * p.rhs_rows;
          if (consec) {
            if (lane < NH)
              bulk_g2s(sbase + off_pan + lane * c.pan_bytes, (lane ? p.pan_lo : p.pan_hi) + (cbase + rhs0) * blk_bytes,
                       static_cast<uint32_t>(G * blk_bytes), &ctl->copy[stage]);
          } else if (lane < G * NH) {
            const bool ok = my_rhs >= 0 && my_rhs < p.rhs_rows;
            if (ok || !zfill)
              bulk_g2s(sbase + off_pan + jhl * c.pan_bytes + jslot * blk_bytes,
                       ok ? (jhl ? p.pan_lo : p.pan_hi) + (cbase + my_rhs) * blk_bytes : p.zeros,
                       static_cast<uint32_t>(blk_bytes), &ctl->copy[stage]);
          }
          __syncwarp();
          ++it;
          if (++stage == c.stages) {
            stage = 0;
            ph ^= 1u;
          }
        }
        }
        // chains end on a multiple of kRecAhead records, outside the unrolled
        // loop above (ahead[] is a ring indexed at compile time, and the
        // scheduler's per-record path stays as short as without chains)
        if (p.chain_recs > 0 && r < re && !aborted && (since += kRecAhead) >= p.chain_recs) {
          // end of a chain: the MMA warp commits this accumulation and starts
          // the rest of the item in a fresh accumulator; the epilogue adds
          // each chain into the running sum
          since = 0;
          if (!wait_bar(&ctl->empty[stage], ph ^ 1u, ctl, p.err)) {
            aborted = true;
            break;
          }
          if (lane == 0) {
            ctl->item_log[item_iter % kItemLog].last = 0;
            ctl->ring[stage].done = 1;
            mbar_arrive_expect_tx(&ctl->copy[stage], 0);
          }
          __syncwarp();
          ++it;
          ++item_iter;
          if (++stage == c.stages) {
            stage = 0;
            ph ^= 1u;
          }
          log_item(re - r, 1);
        }
      }
      if (aborted) break;
      while (pf < 3) pf_advance();
      // end of the item
      if (!wait_bar(&ctl->empty[stage], ph ^ 1u, ctl, p.err)) {
        aborted = true;
        break;
      }
      if (lane == 0) {
        ctl->item_log[item_iter % kItemLog].last = 1;
        ctl->ring[stage].done = 1;
        mbar_arrive_expect_tx(&ctl->copy[stage], 0);
      }
      __syncwarp();
      ++it;
      ++item_iter;
      if (++stage == c.stages) {
        stage = 0;
        ph ^= 1u;
      }
    }
    if (aborted && lane == 0) {
      // the last `stages` stages may still have copies landing
      const uint32_t n = static_cast<uint32_t>(c.stages);
      for (uint32_t i = it > n ? it - n : 0u; i < it; ++i) drain_bar(&ctl->copy[i % n], (i / n) & 1u);
    }
    __syncwarp();
  } else if (warp < 4 && !dual) {
    // ----------------------------------------- fp32 split of the lhs chunk
    if constexpr (F32) {
      const int nf = c.lhs_bytes / 16;  // 16-byte chunks of the lhs operand (all slots)
      const int per = (nf + kProducers - 1) / kProducers;
      if (p.rn_split) split_dispatch<true>(p, ctl, smem, off_lhs, slot_bytes, tid, per);
      else split_dispatch<false>(p, ctl, smem, off_lhs, slot_bytes, tid, per);
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA warp
    MmaArgs m;
    m.smem0 = smem_u32(smem);
    m.tmem = tmem;
    m.lane = lane;
    m.sbo = static_cast<uint32_t>(sbo);
    m.layout = static_cast<uint32_t>(c.swz);
    m.col_per_half = static_cast<uint32_t>(col_per_half);
    m.acc_stride = static_cast<uint32_t>(acc_stride);
    const bool swap = c.swap != 0;
    m.lo_m = swap ? static_cast<uint32_t>(c.pan_bytes) : static_cast<uint32_t>(c.lhs_bytes);
    m.lo_n = swap ? static_cast<uint32_t>(c.lhs_bytes) : static_cast<uint32_t>(c.pan_bytes);
    m.off_m = static_cast<uint32_t>(swap ? off_pan : off_lhs);
    m.off_n = static_cast<uint32_t>(swap ? off_lhs : off_pan);
    m.idesc = make_idesc(F32, false, false, 128, swap ? c.Mt : c.n_mma);
    m.idesc2 = make_idesc(F32, false, false, 128, 2 * c.Mt);
    const int ksteps = c.KC / KSTEP;
    if constexpr (F32) {
      if (c.fold) mma_dispatch<true, true>(p, ctl, m, ksteps, c.halves);
      else mma_dispatch<true, false>(p, ctl, m, ksteps, c.halves);
    } else {
      mma_dispatch<false, false>(p, ctl, m, ksteps, c.halves);
    }
  } else if ((warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) || warp < 4) {
    // ---------------------------------------------------------- epilogue
    // group 0: warps 6-9; group 1 (dual only): warps 0-3
    const int quad = warp & 3;  // TMEM lanes [32*quad, 32*quad+32)
    const int grp = warp < 4 ? 1 : 0;
    float* stg = reinterpret_cast<float*>(epi_stg + (grp * 4 + quad) * c.epi_warp_bytes);
    for (uint32_t item_iter = 0;; ++item_iter) {
      const uint32_t b = item_iter % c.acc_bufs;
      if (!wait_bar(&ctl->acc_full[b], (item_iter / c.acc_bufs) & 1u, ctl, p.err, &ctl->progress, kEpiSleepNs)) break;
      if (*reinterpret_cast<volatile int*>(&ctl->exit_at) == static_cast<int>(item_iter)) break;
      const ItemInfo& info = ctl->item_log[item_iter % kItemLog];
      const bool empty = info.nsteps == 0;  // zeros: written by the first key block only
      // destination: the output (rows through seg_out), or in a fused launch
      // block b's partial sums (segment rows); chains after an item's first
      // and key blocks after the first of sequential launches add into it
      // chains summed in TMEM (tmem_chain): an accumulation that does not end
      // its item is added into the running sum S at column acc_stride and
      // released; the last one adds S and goes out
      const bool tchain = c.tmem_chain != 0;
      const bool accm = p.accumulate || (info.acc && !tchain);
      const bool flush = tchain && !info.last;
      const bool add_s = tchain && info.acc;
      void* obase = p.out;
      const int32_t* oseg = p.seg_out;
      if (p.fused && info.blk > 0) {
        obase = p.part + static_cast<int64_t>(info.blk - 1) * p.part_stride;
        oseg = nullptr;
      }
      tc_fence_after();
      for (int h = 0; h < c.halves && !(empty && accm); ++h) {
        const uint32_t tbase =
            tmem + (static_cast<uint32_t>(quad * 32) << 16) + b * acc_stride + h * col_per_half;
        if (!c.swap) {
          // accumulator row = (lhs slot, row of that slot's tile)
          const int mm = h * 128 + quad * 32 + lane;
          const int slot = mm / c.Mt, m = mm - slot * c.Mt;
          const bool live_slot = slot < c.slots;
          const int s0 = live_slot ? info.s0[slot] : 0, gcnt = live_slot ? info.gcnt[slot] : 0;
          for (int c0 = 0; c0 < c.n_mma; c0 += 32) {
            float v[32];
            tmem_ld32(tbase + c0, v);
            if (empty) {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = 0.f;
            }
            if (add_s) {
              uint32_t sv[32];
              tmem_ld32_async(tbase + acc_stride + c0, sv);
              tmem_wait32(sv);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += __uint_as_float(sv[j]);
            }
            if (flush) {
              tmem_st32(tbase + acc_stride + c0, v);
              continue;
            }
            if (gcnt > 0 && p.odt == ES_F32) {
              // the 8 pieces' old values are all loaded before any store, so
              // an accumulating epilogue waits one memory round trip per 32
              // columns instead of one per piece
              auto piece = [&](int q) -> float4* {
                const int col = c0 + 4 * q;
                const int g = col / c.Nt, n = col % c.Nt;
                if (col >= c.n_mma || g >= gcnt) return nullptr;
                const int64_t row = oseg ? oseg[s0 + g] : static_cast<int64_t>(s0 + g);
                return reinterpret_cast<float4*>(static_cast<float*>(obase) + row * c.Mt * c.Nt +
                                                 static_cast<int64_t>(m) * c.Nt + n);
              };
              if (accm) {
                float4 old[8];
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                  const float4* d = piece(q);
                  old[q] = d ? *d : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                  float4* d = piece(q);
                  if (d)
                    *d = make_float4(v[4 * q] + old[q].x, v[4 * q + 1] + old[q].y, v[4 * q + 2] + old[q].z,
                                     v[4 * q + 3] + old[q].w);
                }
              } else {
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                  float4* d = piece(q);
                  if (d) *d = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                }
              }
            } else if (gcnt > 0) {
#pragma unroll
              for (int j = 0; j < 32; j += 4) {
                const int col = c0 + j;
                const int g = col / c.Nt, n = col % c.Nt;
                if (col >= c.n_mma || g >= gcnt) continue;
                const int64_t row = oseg ? oseg[s0 + g] : static_cast<int64_t>(s0 + g);
                const int64_t o = row * c.Mt * c.Nt + static_cast<int64_t>(m) * c.Nt + n;
                {
                  __nv_bfloat16* ob = static_cast<__nv_bfloat16*>(obase) + o;
#pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    float x = v[j + q];
                    if (accm) x += __bfloat162float(ob[q]);
                    ob[q] = __float2bfloat16_rn(x);
                  }
                }
              }
            }
          }
        } else if (c.epi_stage) {
          // all halves at once (see epi_swap_staged)
          if (h == 0)
            epi_swap_staged(p, info, obase, oseg, accm, tmem + (static_cast<uint32_t>(quad * 32) << 16) + b * acc_stride,
                            quad, lane, stg, empty, grp, dual ? 2 : 1);
        } else {
          const int s0 = info.s0[0], gcnt = info.gcnt[0];
          const int r = h * 128 + quad * 32 + lane;  // panel row = (g, n)
          const int g = r / c.Nt, n = r % c.Nt;
          const bool live = g < gcnt;
          const int64_t row = live ? (oseg ? oseg[s0 + g] : static_cast<int64_t>(s0 + g)) : 0;
          for (int m0 = 0; m0 < c.Mt; m0 += 32) {
            float v[32];
            tmem_ld32(tbase + m0, v);
            if (c.fold) {
              // the panel_hi x lhs_lo block sits Mt columns to the right
              float w[32];
              tmem_ld32(tbase + c.Mt + m0, w);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += w[j];
            }
            if (live && p.odt == ES_F32) {
              // old values in groups of 8 loads before their stores
              float* ob = static_cast<float*>(obase) + row * c.Mt * c.Nt + n;
#pragma unroll
              for (int j0 = 0; j0 < 32; j0 += 8) {
                float old[8];
#pragma unroll
                for (int j = 0; j < 8; ++j)
                  old[j] = (accm && m0 + j0 + j < c.Mt) ? ob[static_cast<int64_t>(m0 + j0 + j) * c.Nt] : 0.f;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                  if (m0 + j0 + j >= c.Mt) break;  // Mt < 32: the tail columns are not part of the tile
                  const float x = (empty ? 0.f : v[j0 + j]) + old[j];
                  ob[static_cast<int64_t>(m0 + j0 + j) * c.Nt] = x;
                }
              }
            } else if (live) {
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                if (m0 + j >= c.Mt) break;  // Mt < 32: the tail columns are not part of the tile
                const int64_t o = row * c.Mt * c.Nt + static_cast<int64_t>(m0 + j) * c.Nt + n;
                float x = empty ? 0.f : v[j];
                {
                  __nv_bfloat16* ob = static_cast<__nv_bfloat16*>(obase) + o;
                  if (accm) x += __bfloat162float(*ob);
                  *ob = __float2bfloat16_rn(x);
                }
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&ctl->acc_empty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, static_cast<uint32_t>(c.tmem_cols));
  }
}

// ------------------------------------------------------- preparation kernels

// rhs tile t -> per k-chunk c of KC rows a K-major swizzled block: row n
// holds the tile's column n over the chunk's k (W = KC * element bytes), its
// 16-byte pieces XOR-permuted by the row's address bits 7.. (the layout the
// TMA's swizzle modes produce for a block starting on a 1024-byte boundary),
// i.e. exactly the image one panel slot has in shared memory. Blocks are
// stored chunk-major ([c][t]) so consecutive tiles of one chunk are
// contiguous.
// Source tiles are Kt x Nt with n contiguous, or (KMAJOR) Nt x Kt with k
// contiguous, which is already the image's row order. fp32 writes the raw
// value (read as TF32 by the tensor core) to hi and x - trunc_tf32(x) to lo.
template <bool F32, bool KMAJOR>
__global__ void __launch_bounds__(256) layout_rhs_kernel(const void* __restrict__ rhs, int64_t rows, int Kt, int Nt,
                                                         int KC, void* __restrict__ hi, void* __restrict__ lo, int rn) {
  using E = typename std::conditional<F32, float, __nv_bfloat16>::type;
  constexpr int ESZ = F32 ? 4 : 2;
  constexpr int EPU = 16 / ESZ;  // elements per 16-byte piece
  const int W = KC * ESZ;        // bytes per image row
  const int pieces = W / 16;
  const int nck = Kt / KC;
  const E* src = static_cast<const E*>(rhs);
  auto put = [&](int64_t dst, const E (&v)[EPU]) {
    if constexpr (F32) {
      float4 h, l;
      tf32_split4(make_float4(v[0], v[1], v[2], v[3]), rn != 0, h, l);
      *reinterpret_cast<float4*>(static_cast<uint8_t*>(hi) + dst) = h;
      *reinterpret_cast<float4*>(static_cast<uint8_t*>(lo) + dst) = l;
    } else {
      *reinterpret_cast<uint4*>(static_cast<uint8_t*>(hi) + dst) = *reinterpret_cast<const uint4*>(v);
    }
  };
  if constexpr (KMAJOR) {
    // one thread per 16-byte piece, pieces of one row adjacent: a straight
    // (swizzled) copy of the source rows
    const int64_t total = rows * nck * static_cast<int64_t>(Nt) * pieces;
    for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < total; q += (int64_t)gridDim.x * blockDim.x) {
      const int j = static_cast<int>(q % pieces);
      int64_t r = q / pieces;
      const int n = static_cast<int>(r % Nt);
      r /= Nt;
      const int c = static_cast<int>(r % nck);
      const int64_t t = r / nck;
      __align__(16) E v[EPU];
      *reinterpret_cast<uint4*>(v) = *reinterpret_cast<const uint4*>(
          src + (t * Nt + n) * static_cast<int64_t>(Kt) + static_cast<int64_t>(c) * KC + j * EPU);
      const int sw = ((n * W) >> 7) & (pieces - 1);
      put(((static_cast<int64_t>(c) * rows + t) * Nt + n) * W + ((j ^ sw) * 16), v);
    }
  } else {
    // one thread per image row (tile t, k-chunk c, row n): the row's pieces
    // are W contiguous bytes, so a warp (32 consecutive n) stores 32 * W
    // contiguous bytes; n varies fastest, so every column read of a warp is
    // one coalesced row segment of the source tile
    const int64_t total = rows * nck * static_cast<int64_t>(Nt);
    for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < total; q += (int64_t)gridDim.x * blockDim.x) {
      const int n = static_cast<int>(q % Nt);
      const int64_t r = q / Nt;
      const int c = static_cast<int>(r % nck);
      const int64_t t = r / nck;
      const E* col = src + t * static_cast<int64_t>(Kt) * Nt + static_cast<int64_t>(c) * KC * Nt + n;
      const int sw = ((n * W) >> 7) & (pieces - 1);
      const int64_t row = ((static_cast<int64_t>(c) * rows + t) * Nt + n) * W;
      constexpr int kBatch = 4;  // pieces with loads in flight together
      for (int j0 = 0; j0 < pieces; j0 += kBatch) {
        __align__(16) E v[kBatch][EPU];
#pragma unroll
        for (int jj = 0; jj < kBatch; ++jj)
#pragma unroll
          for (int e = 0; e < EPU; ++e)
            if (j0 + jj < pieces) v[jj][e] = col[static_cast<int64_t>((j0 + jj) * EPU + e) * Nt];
#pragma unroll
        for (int jj = 0; jj < kBatch; ++jj)
          if (j0 + jj < pieces) put(row + (((j0 + jj) ^ sw) * 16), v[jj]);
      }
    }
  }
}

// layout_rhs_kernel for wide row-major tiles (Nt >= 128): one CTA per
// (tile, chunk, 32 columns) reads the KC x 32 block with coalesced row
// segments into shared memory and writes its 32 image rows -- 32 * W
// contiguous bytes -- as consecutive 16-byte pieces (the per-piece mapping
// scatters each warp's stores over 32 rows of W bytes).
constexpr int kLayoutCols = 32;

template <bool F32>
__global__ void __launch_bounds__(256) layout_rhs_wide_kernel(const void* __restrict__ rhs, int64_t rows, int Kt,
                                                              int Nt, int KC, void* __restrict__ hi,
                                                              void* __restrict__ lo, int rn) {
  using E = typename std::conditional<F32, float, __nv_bfloat16>::type;
  constexpr int ESZ = F32 ? 4 : 2;
  constexpr int EPU = 16 / ESZ;
  const int W = KC * ESZ;
  const int pieces = W / 16;
  const int nck = Kt / KC;
  const E* src = static_cast<const E*>(rhs);
  __shared__ float blk[64][kLayoutCols + 1];
  const int nb = (Nt + kLayoutCols - 1) / kLayoutCols;
  const int64_t nblk = rows * nck * nb;
  for (int64_t b = blockIdx.x; b < nblk; b += gridDim.x) {
    const int cb = static_cast<int>(b % nb);
    const int64_t r = b / nb;
    const int c = static_cast<int>(r % nck);
    const int64_t t = r / nck;
    const int n0 = cb * kLayoutCols;
    const int ncols = Nt - n0 < kLayoutCols ? Nt - n0 : kLayoutCols;
    const E* tile = src + t * static_cast<int64_t>(Kt) * Nt + static_cast<int64_t>(c) * KC * Nt + n0;
    for (int e = threadIdx.x; e < KC * kLayoutCols; e += blockDim.x) {
      const int k = e / kLayoutCols, nn = e % kLayoutCols;
      if (nn < ncols) blk[k][nn] = static_cast<float>(tile[static_cast<int64_t>(k) * Nt + nn]);
    }
    __syncthreads();
    for (int pq = threadIdx.x; pq < ncols * pieces; pq += blockDim.x) {
      const int nn = pq / pieces, j = pq % pieces;
      const int n = n0 + nn;
      __align__(16) E v[EPU];
#pragma unroll
      for (int e = 0; e < EPU; ++e) v[e] = static_cast<E>(blk[j * EPU + e][nn]);
      const int sw = ((n * W) >> 7) & (pieces - 1);
      const int64_t dst = ((static_cast<int64_t>(c) * rows + t) * Nt + n) * W + ((j ^ sw) * 16);
      if constexpr (F32) {
        float4 h, l;
        tf32_split4(make_float4(v[0], v[1], v[2], v[3]), rn != 0, h, l);
        *reinterpret_cast<float4*>(static_cast<uint8_t*>(hi) + dst) = h;
        *reinterpret_cast<float4*>(static_cast<uint8_t*>(lo) + dst) = l;
      } else {
        *reinterpret_cast<uint4*>(static_cast<uint8_t*>(hi) + dst) = *reinterpret_cast<const uint4*>(v);
      }
    }
    __syncthreads();
  }
}

__global__ void item_heads_kernel(const int64_t* __restrict__ strip, int64_t nseg, int G, uint32_t* __restrict__ flags,
                                  int32_t* __restrict__ cnt, ZeroSpans zs) {
  zero_spans(zs);
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s < nseg; s += (int64_t)gridDim.x * blockDim.x) {
    const int64_t key = strip[s];
    int64_t lo = 0, hi = s;  // first index with strip >= key
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (strip[mid] < key) lo = mid + 1; else hi = mid;
    }
    const int64_t first = lo;
    lo = s + 1;
    hi = nseg;  // first index with strip > key
    while (lo < hi) {
      const int64_t mid = (lo + hi) >> 1;
      if (strip[mid] <= key) lo = mid + 1; else hi = mid;
    }
    const int64_t pos = s - first;
    flags[s] = (pos % G == 0) ? 1u : 0u;
    const int64_t left = lo - s;
    cnt[s] = static_cast<int32_t>(left < G ? left : G);
  }
}

__global__ void item_place_kernel(const uint32_t* __restrict__ flags, const uint32_t* __restrict__ excl,
                                  const int32_t* __restrict__ cnt, int64_t nseg, int32_t* __restrict__ first,
                                  int32_t* __restrict__ count) {
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s < nseg; s += (int64_t)gridDim.x * blockDim.x) {
    if (!flags[s]) continue;
    first[excl[s]] = static_cast<int32_t>(s);
    count[excl[s]] = cnt[s];
  }
}

__global__ void item_identity_kernel(int64_t nseg, int32_t* __restrict__ first, int32_t* __restrict__ count,
                                     int64_t* __restrict__ num, ZeroSpans zs) {
  zero_spans(zs);
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s < nseg; s += (int64_t)gridDim.x * blockDim.x) {
    first[s] = static_cast<int32_t>(s);
    count[s] = 1;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) *num = nseg;
}

// Sort key per item slot: items (slot < W) by descending pair count, empty
// slots last.
__global__ void item_work_keys_kernel(const int32_t* __restrict__ first, const int32_t* __restrict__ count,
                                      const int64_t* __restrict__ seg_off, const int64_t* __restrict__ num_items,
                                      int64_t nslots, uint32_t* __restrict__ keys, uint32_t* __restrict__ vals) {
  const int64_t W = *num_items;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nslots; i += (int64_t)gridDim.x * blockDim.x) {
    // 8-bit key, largest work first: half-octave buckets of the pair count
    // (bit length and the next bit), so one stable radix pass orders them;
    // empty items and padding slots go last
    uint32_t key = 0xFFu;
    if (i < W) {
      const int s0 = first[i], g = count[i];
      const int64_t work = seg_off[s0 + g] - seg_off[s0];
      if (work > 0) {
        const int b = 64 - __clzll(static_cast<unsigned long long>(work));
        const int frac = b >= 2 ? static_cast<int>((work >> (b - 2)) & 1) : 0;
        const int level = 2 * b + frac;  // 2 .. 129
        key = static_cast<uint32_t>(250 - level);
      } else {
        key = 0xFEu;
      }
    }
    keys[i] = key;
    vals[i] = static_cast<uint32_t>(i);
  }
}

// Merge of a work item's segment pair lists into step records. An item is S
// sub-strips (queue position q takes order[q*S + s]) of up to G segments;
// lane s*G + g walks segment g of sub-strip s. With one slot the lists merge
// on the lhs tile; with several on the contracted key. Each step takes the
// smallest pending value; the sub-strips holding it whose rhs tiles (per
// segment slot, -1 absent) equal those of the first such sub-strip share the
// step, the others follow in later steps. Each list keeps its own order, so a
// segment's pairs are summed in join order.
//
// With keys, an item's key range is cut into C chunks merged by separate
// warps (warp w: item w / C, chunk w % C): COUNT writes the steps of each
// (item, chunk) to cnt, the fill pass writes the records from off[] (the
// exclusive scan of cnt). Without keys C = 1. Records of an item are in
// ascending key, chunks in order, so a key block (a run of chunks) is a run
// of records.
constexpr int kMergeWarps = 4;

template <bool COUNT>
__global__ void __launch_bounds__(kMergeWarps * 32) tc_merge_kernel(
    const int32_t* __restrict__ pl, const int32_t* __restrict__ pr, const int32_t* __restrict__ pair_key,
    const int64_t* __restrict__ seg_off, const int32_t* __restrict__ item_first, const int32_t* __restrict__ item_count,
    const uint32_t* __restrict__ order, const int64_t* __restrict__ num_sub, int S, int G, int64_t lhs_rows,
    int64_t rhs_rows, int C, int64_t key_extent, int64_t nw, uint32_t* __restrict__ cnt,
    const uint32_t* __restrict__ off, int32_t* __restrict__ recs, int32_t* __restrict__ err, ZeroSpans zs) {
  zero_spans(zs);
  // [entry][lane]: a step's reads (one entry per lane) and a refill's
  // stores (entry qq of every refilling lane) touch 32 distinct banks
  __shared__ int win_l[kMergeWarps][kWin][32];
  __shared__ int win_r[kMergeWarps][kWin][32];
  __shared__ int win_k[kMergeWarps][kWin][32];
  const int wib = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t W1 = *num_sub;
  const int64_t nitems = (W1 + S - 1) / S;
  const bool keyed = pair_key != nullptr;
  const int ls = lane / G, lg = lane - ls * G;  // this lane's sub-strip and segment slot
  // nw covers the slots of every possible item; those past the real items
  // count zero steps, so the scan over all nw entries stays exact
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * kMergeWarps + wib; w < nw;
       w += static_cast<int64_t>(gridDim.x) * kMergeWarps) {
    if (w >= nitems * C) {
      if (COUNT && lane == 0) cnt[w] = 0;
      continue;
    }
    const int64_t q = w / C;
    const int ck = static_cast<int>(w - q * C);
    const int64_t sub = q * S + ls;
    int64_t cur = 0, end = 0;
    if (ls < S && sub < W1) {
      const int ss = static_cast<int>(order[sub]);
      if (lg < item_count[ss]) {
        const int s0 = item_first[ss];
        cur = seg_off[s0 + lg];
        end = seg_off[s0 + lg + 1];
        if (C > 1) {
          // this chunk's pairs: keys increase inside a segment
          const int64_t klo = key_extent * ck / C, khi = key_extent * (ck + 1) / C;
          int64_t lo = cur, hi = end;
          while (lo < hi) {
            const int64_t mid = (lo + hi) >> 1;
            if (pair_key[mid] < klo) lo = mid + 1; else hi = mid;
          }
          const int64_t a = lo;
          hi = end;
          while (lo < hi) {
            const int64_t mid = (lo + hi) >> 1;
            if (pair_key[mid] < khi) lo = mid + 1; else hi = mid;
          }
          cur = a;
          end = lo;
        }
      }
    }
    const int64_t base = COUNT ? 0 : off[w];
    int64_t n = 0;
    int wpos = kWin;
    bool bad = false, contract = false;
    while (true) {
      if (wpos == kWin && cur < end) {
        int tl[kWin], tr[kWin], tk[kWin];
#pragma unroll
        for (int qq = 0; qq < kWin; ++qq) {
          const int64_t i = cur + qq;
          tl[qq] = i < end ? __ldg(pl + i) : INT_MAX;
          tr[qq] = i < end ? __ldg(pr + i) : -1;
          tk[qq] = (keyed && i < end) ? __ldg(pair_key + i) : 0;
        }
#pragma unroll
        for (int qq = 0; qq < kWin; ++qq) {
          win_l[wib][qq][lane] = tl[qq];
          win_r[wib][qq][lane] = tr[qq];
          win_k[wib][qq][lane] = tk[qq];
        }
        wpos = 0;
      }
      __syncwarp();
      const bool live = cur < end;
      const int hl = live ? win_l[wib][wpos][lane] : INT_MAX;
      const int hk = live ? win_k[wib][wpos][lane] : INT_MAX;
      const int v = S > 1 ? hk : hl;
      const int vmin = __reduce_min_sync(0xffffffffu, v);
      if (vmin == INT_MAX) break;
      const bool matched = live && v == vmin;
      const int hr = matched ? win_r[wib][wpos][lane] : -1;
      // the first sub-strip holding vmin sets the rhs tiles of the step
      const uint32_t mm = __ballot_sync(0xffffffffu, matched);
      const int ref = (__ffs(mm) - 1) / G;
      const int ref_r = __shfl_sync(0xffffffffu, hr, (ref * G + lg) & 31);
      const uint32_t eqm = __ballot_sync(0xffffffffu, ls >= S || hr == ref_r);
      const uint32_t gmask = (G == 32) ? 0xffffffffu : ((1u << G) - 1u);
      const uint32_t my_grp = gmask << (ls * G);
      const bool strip_has = (mm & my_grp) != 0u;
      const bool joins = ls < S && strip_has && (eqm & my_grp) == my_grp;
      // lhs tile of each joining sub-strip: from its lowest matched lane
      const int src = joins ? (__ffs(mm & my_grp) - 1) : lane;
      const int slot_lhs = __shfl_sync(0xffffffffu, hl, src & 31);
      // the key must name one lhs tile per sub-strip (caller's contract)
      if (joins && matched && hl != slot_lhs) contract = true;
      if (joins && matched) {
        ++cur;
        ++wpos;
      }
      if (!COUNT) {
        // rhs slot g of the step: lane g holds it after this shuffle
        int rg = __shfl_sync(0xffffffffu, hr, (ref * G + (lane % G)) & 31);
        if (lane < G && (rg < -1 || rg >= rhs_rows)) {
          bad = true;
          rg = -1;
        }
        const int first = __shfl_sync(0xffffffffu, rg, 0);
        const bool cons = __all_sync(0xffffffffu, lane >= G || (rg >= 0 && rg == first + lane)) && first >= 0 &&
                          first + G <= rhs_rows;
        // lhs tile per slot: lane s (< S) takes sub-strip s's value
        const int lhs_s = __shfl_sync(0xffffffffu, slot_lhs, (lane * G) & 31);
        const bool joins_s = __shfl_sync(0xffffffffu, joins ? 1 : 0, (lane * G) & 31) != 0;
        int32_t* rec = recs + (base + n) * kRecInts;
        if (lane < S) {
          const int lv = joins_s ? lhs_s : -1;
          if (joins_s && (lv < 0 || lv >= lhs_rows)) bad = true;
          rec[lane] = lv;
        }
        if (lane < G) rec[S + lane] = rg;
        if (lane == 0) {
          rec[S + G] = cons ? 1 : 0;
          rec[S + G + 1] = first;
        }
      }
      ++n;
    }
    if (COUNT) {
      if (lane == 0) cnt[w] = static_cast<uint32_t>(n);
    } else {
      if (__any_sync(0xffffffffu, bad) && lane == 0 && err) atomicExch(err, ES_ERR_INDEX);
      if (__any_sync(0xffffffffu, contract) && lane == 0 && err) atomicExch(err, ES_ERR_INVALID);
    }
  }
}

// Record boundaries of each item's key blocks: block b of item q starts at
// the record offset of chunk b * (C / nblocks); the last boundary is the
// next item's first record (or the total).
__global__ void item_rec_kernel(const uint32_t* __restrict__ off, const uint32_t* __restrict__ total,
                                const int64_t* __restrict__ num_sub, int S, int C, int nblocks, int64_t nw,
                                int64_t* __restrict__ item_rec, ZeroSpans zs) {
  zero_spans(zs);
  const int64_t W1 = *num_sub;
  const int64_t nitems = (W1 + S - 1) / S;
  const int m = C / nblocks;
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < nitems; q += (int64_t)gridDim.x * blockDim.x) {
    for (int b = 0; b <= nblocks; ++b) {
      const int64_t w = q * C + static_cast<int64_t>(b) * m;
      item_rec[q * (nblocks + 1) + b] = w < nw ? off[w] : *total;
    }
  }
}

// Key chunks of the merge pass: a multiple of the key blocks, about
// kMergeChunkKeys keys each (1 without keys). Smaller chunks measured slower
// on C2 (fill pass 342 us with 256 keys per chunk, 414 us with 32). A
// chunk's merge is one warp's serial loop, so with few items (one rank's
// share of the strips) the chunks are cut finer until about
// kMergeTargetWarps warps run: the pass then takes the longest chunk's
// time, not the longest item's.
constexpr int64_t kMergeChunkKeys = 256;
constexpr int64_t kMergeTargetWarps = 148 * 16;

int merge_chunks(int nblocks, bool have_key, int64_t key_extent, int64_t items) {
  if (!have_key || key_extent <= 1) return 1;
  int64_t keys = kMergeChunkKeys;
  // EINSPARSE_MERGE_KEYS overrides the keys per chunk (tuning, tests)
  const char* env = std::getenv("EINSPARSE_MERGE_KEYS");
  if (env) {
    const long long v = std::atoll(env);
    if (v > 0) keys = v;
  }
  int64_t m = key_extent / (keys * nblocks);
  if (!env && items > 0) {
    const int64_t want = (kMergeTargetWarps + items * nblocks - 1) / (items * nblocks);
    if (want > m) m = want;
  }
  if (m > key_extent / nblocks) m = key_extent / nblocks;  // at least one key per chunk
  if (m < 1) m = 1;
  // EINSPARSE_MERGE_MAXCHUNKS overrides the cap on chunks (tuning, tests)
  int64_t cap = kMaxMergeChunks;
  if (const char* e = std::getenv("EINSPARSE_MERGE_MAXCHUNKS")) {
    const long long v = std::atoll(e);
    if (v > 0) cap = v;
  }
  while (nblocks * m > cap) --m;
  if (m < 1) m = 1;
  return static_cast<int>(nblocks * m);
}

// Work items a launch forms from nseg segments (upper estimate: every strip
// fills its G segment slots).
int64_t items_estimate(const TcConfig& c, int64_t nseg) {
  const int64_t per_item = static_cast<int64_t>(c.G > 0 ? c.G : 1) * (c.slots > 0 ? c.slots : 1);
  return (nseg + per_item - 1) / per_item;
}

// Fused key blocks: one launch takes every (key block, item) unit; blocks
// after the first write partial sums (fp32, one row per segment) that a last
// pass adds into the output in block order. Used when the partials fit in
// this budget (and the output is fp32); else one launch per block.
constexpr int64_t kMaxPartialBytes = 4ll << 30;

bool fused_blocks_possible(const TcConfig& c, int nblocks, int64_t nseg) {
  if (nblocks <= 1) return false;
  const int64_t bytes = static_cast<int64_t>(nblocks - 1) * nseg * c.Mt * c.Nt * 4;
  return bytes <= kMaxPartialBytes;
}

// Accumulation chains (fp32): the tensor core adds each MMA's products into
// its fp32 accumulator with truncation, a bias that grows with the number of
// MMAs summed into one accumulator. Restarting the accumulator every
// kChainKsteps k-steps (K = 8 each) and adding the chains in fp32 with
// round-to-nearest keeps a long contraction within plain fp32 accuracy.
constexpr int kChainKsteps = 128;

int chain_records(const TcConfig& c) {
  if (!c.fp32) return 0;
  int64_t ks = kChainKsteps;
  // EINSPARSE_CHAIN_KSTEPS overrides the chain length (0: no chains; tuning, tests)
  if (const char* e = std::getenv("EINSPARSE_CHAIN_KSTEPS")) ks = std::atoll(e);
  if (ks <= 0) return 0;
  const int per = c.Kt / 8 > 0 ? c.Kt / 8 : 1;  // k-steps per record
  int64_t r = ks / per;
  r = (r + kRecAhead - 1) / kRecAhead * kRecAhead;  // the scheduler ends chains every kRecAhead records
  return static_cast<int>(r < kRecAhead ? kRecAhead : r);
}

// out[row(s)] += part[0][s] + part[1][s] + ... in block order (float4 pieces),
// over the partial rows marked written.
__global__ void add_partials_kernel(float* __restrict__ out, const float* __restrict__ part,
                                    const uint8_t* __restrict__ written, int64_t nseg, int64_t te4, int nparts,
                                    int64_t stride, const int32_t* __restrict__ seg_out) {
  const int64_t nv = nseg * te4;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nv; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t sg = v / te4, e = v - sg * te4;
    const int64_t row = seg_out ? static_cast<int64_t>(seg_out[sg]) : sg;
    float4* o = reinterpret_cast<float4*>(out) + row * te4 + e;
    float4 a = *o;
    for (int b = 0; b < nparts; ++b) {
      if (!written[b * nseg + sg]) continue;
      const float4 x = __ldcs(reinterpret_cast<const float4*>(part + b * stride) + v);
      a.x += x.x;
      a.y += x.y;
      a.z += x.z;
      a.w += x.w;
    }
    *o = a;
  }
}

struct TcWs {
  float* part;
  uint8_t* pwritten;
  uint8_t* pan_hi;
  uint8_t* pan_lo;
  uint8_t* zeros;
  int32_t* recs;
  int64_t* item_rec;
  uint32_t* ipairs;
  uint32_t* rec_base;
  uint32_t* rec_total;
  uint32_t* scan2;
  int32_t* item_first;
  int32_t* item_count;
  uint32_t* flags;
  uint32_t* excl;
  int32_t* cnt;
  uint32_t* scan;
  int64_t* num_items;
  uint32_t* sort_keys;
  uint32_t* order;
  RadixBuffers<uint32_t> rb;
  int* queue;
};

int64_t zero_bytes(const TcConfig& c) {
  const int blk = c.Nt * c.KC * (c.fp32 ? 4 : 2);
  return c.lhs_bytes > blk ? c.lhs_bytes : blk;
}

template <typename C>
void tc_layout(C& cv, TcWs& w, const TcConfig& c, int64_t rhs_rows, int64_t npairs, int64_t nseg, int nblocks,
               int64_t key_extent) {
  const int64_t pan_elems = rhs_rows * c.Kt * c.Nt;
  const int esz = c.fp32 ? 4 : 2;
  w.pan_hi = cv.template take<uint8_t>(pan_elems * esz);
  w.pan_lo = c.fp32 ? cv.template take<uint8_t>(pan_elems * esz) : nullptr;
  w.zeros = cv.template take<uint8_t>(zero_bytes(c));
  w.recs = cv.template take<int32_t>(npairs * kRecInts);
  w.item_rec = cv.template take<int64_t>(nseg * (nblocks + 1));
  const int nck = merge_chunks(nblocks, key_extent > 0, key_extent, items_estimate(c, nseg));
  w.ipairs = cv.template take<uint32_t>(nseg * nck);    // steps per (item, key chunk)
  w.rec_base = cv.template take<uint32_t>(nseg * nck);  // their record offsets
  w.rec_total = cv.template take<uint32_t>(1);
  w.scan2 = cv.template take<uint32_t>(scan_scratch_elems(nseg * nck));
  w.item_first = cv.template take<int32_t>(nseg);
  w.item_count = cv.template take<int32_t>(nseg);
  w.flags = cv.template take<uint32_t>(nseg);
  w.excl = cv.template take<uint32_t>(nseg);
  w.cnt = cv.template take<int32_t>(nseg);
  w.scan = cv.template take<uint32_t>(scan_scratch_elems(nseg));
  w.num_items = cv.template take<int64_t>(1);
  w.sort_keys = cv.template take<uint32_t>(nseg);
  w.order = cv.template take<uint32_t>(nseg);
  w.rb.keys_alt = cv.template take<uint32_t>(nseg);
  w.rb.vals_alt = cv.template take<uint32_t>(nseg);
  w.rb.hist = cv.template take<uint32_t>(RadixScratchSize::hist_elems(nseg));
  w.rb.scan = cv.template take<uint32_t>(RadixScratchSize::scan_elems(nseg));
  w.queue = cv.template take<int>(1);
  const bool fb = fused_blocks_possible(c, nblocks, nseg);
  w.part = fb ? cv.template take<float>(static_cast<int64_t>(nblocks - 1) * nseg * c.Mt * c.Nt) : nullptr;
  w.pwritten = fb ? cv.template take<uint8_t>(static_cast<int64_t>(nblocks - 1) * nseg) : nullptr;
}

struct SizeOnly {
  Sizer s;
  template <typename T>
  T* take(int64_t n) {
    s.take<T>(n);
    return nullptr;
  }
};

// Flattened offsets of one label group (mixed radix, outermost first).
std::vector<int64_t> group_offsets(const EinGroup& g, int which) {
  std::vector<int64_t> out(g.total);
  for (int idx = 0; idx < g.total; ++idx) {
    int rem = idx;
    int64_t o = 0;
    for (int q = g.n - 1; q >= 0; --q) {
      const int x = rem % g.size[q];
      rem /= g.size[q];
      const int st = which == 0 ? g.lstride[q] : which == 1 ? g.rstride[q] : g.ostride[q];
      o += static_cast<int64_t>(x) * st;
    }
    out[idx] = o;
  }
  return out;
}

}  // namespace

// Largest k-chunk that leaves >= 3 pipeline stages (else >= 2) for an lhs
// operand of lhs_rows rows (slots of mt rows) and a panel of pan_rows rows
// (tiles of nt rows); fills KC, the swizzle and the stage geometry. Rows are
// W = KC * element bytes (32, 64 or 128: the swizzle span); every slot and
// panel tile must start on a 1024-byte boundary. False when no chunk fits.
bool pick_stages(int lhs_rows, int mt, int pan_rows, int nt, int Kt, bool f32, TcConfig* c) {
  const int esz = f32 ? 4 : 2, nh = f32 ? 2 : 1, kstep = f32 ? 8 : 16;
  const int ctrl = kCtrlBytes + (c->epi_stage ? (c->epi_dual ? 8 : 4) * c->epi_warp_bytes : 0);
  const int budget = 227 * 1024 - ctrl - 1024;  // 1024: alignment of the stage ring
  for (int min_stages : {3, 2}) {
    for (int kc : {64, 32, 16, 8}) {
      const int W = kc * esz;
      if (kc % kstep || Kt % kc || W < 32 || W > 128) continue;
      if ((mt * W) % 1024 || (nt * W) % 1024) continue;
      const int lb = lhs_rows * W, pb = pan_rows * W;
      if (f32 && lb > kMaxSplit * kProducers * 16) continue;  // the split warps hold a stage's chunks in registers
      const int sb = (nh * (lb + pb) + 1023) / 1024 * 1024;
      int stages = budget / sb;
      if (stages > kMaxStages) stages = kMaxStages;
      if (stages < min_stages) continue;
      c->KC = kc;
      c->swz = W == 128 ? 2 : W == 64 ? 4 : 6;
      c->lhs_bytes = lb;
      c->pan_bytes = pb;
      c->stage_bytes = sb;
      c->stages = stages;
      // at least half the SM's shared memory, so one CTA runs per SM and its
      // TMEM allocation never waits on another CTA's
      c->smem_bytes = stages * sb + ctrl + 1024;
      if (c->smem_bytes < 116 * 1024) c->smem_bytes = 116 * 1024;
      return true;
    }
  }
  return false;
}

// Stacked mode: 128 / Mt strips share each step's rhs panel as the rows of
// one M = 128 operand, against N = G * Nt panel columns.
bool stacked_config(int Mt, int Kt, int Nt, TcConfig* c) {
  if (Mt != 16 && Mt != 32 && Mt != 64) return false;
  const int S = 128 / Mt;
  int G = 256 / Nt;
  if (G > kMaxG) G = kMaxG;
  if (G > 32 / S) G = 32 / S;
  while (G > 1 && (G * Nt) % 16 != 0) --G;
  if (G < 1 || (G * Nt) % 16 != 0 || S + G + 2 > kRecInts) return false;
  if (!pick_stages(128, Mt, G * Nt, Nt, Kt, true, c) || c->stages < 3) return false;
  c->swap = 0;
  c->halves = 1;
  c->slots = S;
  c->G = G;
  c->n_mma = G * Nt;
  c->fold = 0;
  c->col_per_half = c->n_mma;
  c->acc_bufs = 2 * c->n_mma <= 512 ? 2 : 1;
  c->tmem_cols = 512;
  return true;
}

bool tc_config(const EinsumDesc& d, int ldt, int rdt, int odt, bool have_strips, bool have_keys, TcConfig* c) {
  std::memset(c, 0, sizeof(*c));
  const bool f32 = ldt == ES_F32 && rdt == ES_F32;
  const bool b16 = ldt == ES_BF16 && rdt == ES_BF16;
  if (!f32 && !b16) return false;
  if (odt != ES_F32 && odt != ES_BF16) return false;
  if (d.B.total != 1) return false;
  const int Mt = d.M.total, Kt = d.K.total, Nt = d.N.total;
  // plain matmul layout: lhs m*Kt + k, rhs k*Nt + n, out m*Nt + n
  auto lm = group_offsets(d.M, 0), om = group_offsets(d.M, 2);
  auto lk = group_offsets(d.K, 0), rk = group_offsets(d.K, 1);
  auto rn = group_offsets(d.N, 1), on = group_offsets(d.N, 2);
  for (int m = 0; m < Mt; ++m)
    if (lm[m] != static_cast<int64_t>(m) * Kt || om[m] != static_cast<int64_t>(m) * Nt) return false;
  for (int k = 0; k < Kt; ++k)
    if (lk[k] != k || rk[k] != static_cast<int64_t>(k) * Nt) return false;
  for (int n = 0; n < Nt; ++n)
    if (rn[n] != n || on[n] != n) return false;
  const int kstep = f32 ? 8 : 16;
  if (Kt % kstep != 0 || Mt % 8 != 0 || Nt % 8 != 0) return false;
  c->fp32 = f32 ? 1 : 0;
  c->Mt = Mt;
  c->Kt = Kt;
  c->Nt = Nt;
  c->slots = 1;
  if (f32 && have_strips && have_keys && !std::getenv("EINSPARSE_NO_STACK") && stacked_config(Mt, Kt, Nt, c))
    return true;
  // orientation
  if (Mt % 128 == 0 && Mt <= 256) {
    c->swap = 0;
    c->halves = Mt / 128;
    int G = have_strips ? 256 / Nt : 1;
    if (G > kMaxG) G = kMaxG;
    if (G < 1) return false;
    while (G > 1 && (G * Nt) % 16 != 0) --G;
    if ((G * Nt) % 16 != 0 || G * Nt > 256 || G * Nt < 16) return false;
    c->G = G;
    c->n_mma = G * Nt;
  } else if (Mt % 16 == 0 && Mt <= 256 && Mt >= 16) {
    c->swap = 1;
    c->n_mma = Mt;
    int G = 0;
    // EINSPARSE_TC_MAXG caps the rhs tiles per item (tuning experiments)
    const char* gcap = std::getenv("EINSPARSE_TC_MAXG");
    const int maxg = gcap ? std::atoi(gcap) : kMaxG;
    if (256 % Nt == 0 && 256 / Nt <= kMaxG && 256 / Nt <= maxg && (have_strips || 256 / Nt == 1)) {
      G = 256 / Nt;
      c->halves = 2;
    } else if (128 % Nt == 0 && 128 / Nt <= kMaxG && (have_strips || 128 / Nt == 1)) {
      G = 128 / Nt;
      c->halves = 1;
    } else {
      return false;
    }
    c->G = G;
  } else {
    return false;
  }
  c->fold = (f32 && c->swap && Mt % 32 == 0 && 2 * Mt <= 256) ? 1 : 0;
  c->epi_stage = (c->swap && !c->fold && Nt % 32 == 0) ? 1 : 0;
  c->epi_dual = (c->epi_stage && !f32) ? 1 : 0;
  c->epi_warp_bytes = odt == ES_BF16 ? 2048 : 4096;
  c->col_per_half = c->swap ? (c->fold ? 2 * Mt : Mt) : c->n_mma;
  const int acc_cols = c->halves * c->col_per_half;
  if (acc_cols > 512) return false;
  c->acc_bufs = 2 * acc_cols <= 512 ? 2 : 1;
  // one CTA per SM (shared memory is sized for it), so all 512 columns are
  // free; the epilogue reads in 32-column groups that may run past a small
  // accumulator
  c->tmem_cols = 512;
  return pick_stages(Mt, Mt, c->G * Nt, Nt, Kt, f32, c);
}

// Key blocks: the rhs operand re-read by every strip is split along the
// contracted range into slices that fit in L2; one launch per slice, in
// order, later slices adding into the output.
int tc_key_blocks(const TcConfig& c, int64_t rhs_rows, bool have_key, int64_t key_extent, int64_t nseg,
                  int* l2_blocks) {
  if (l2_blocks) *l2_blocks = 1;
  if (!have_key || key_extent <= 1) return 1;
  const int64_t panel_bytes = rhs_rows * c.Kt * c.Nt * (c.fp32 ? 8 : 2);
  // EINSPARSE_KBLOCK_BYTES overrides the per-block panel budget (tuning, tests)
  int64_t budget = kPanelL2Budget;
  if (const char* e = std::getenv("EINSPARSE_KBLOCK_BYTES")) {
    const long long v = std::atoll(e);
    if (v > 0) budget = v;
  }
  int64_t nb = (panel_bytes + budget - 1) / budget;
  if (nb > key_extent) nb = key_extent;
  if (nb > kMaxKeyBlocks) nb = kMaxKeyBlocks;
  if (nb < 1) nb = 1;
  if (l2_blocks) *l2_blocks = static_cast<int>(nb);
  // the fused launch hands out (key block, item) units; with few items (e.g.
  // one rank's share of the strips) split the contracted range further so
  // that every SM gets several units and the launch does not end in a tail
  if (nb > 1 && nseg > 0) {
    int dev = 0, sms = kSMs;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t items = items_estimate(c, nseg);
    // EINSPARSE_UNITS_PER_SM overrides the units per SM (tuning, tests)
    int64_t per_sm = kUnitsPerSm;
    if (const char* e = std::getenv("EINSPARSE_UNITS_PER_SM")) {
      const long long v = std::atoll(e);
      if (v > 0) per_sm = v;
    }
    const int64_t want = (per_sm * sms + items - 1) / items;
    if (want > nb) nb = want;
    if (nb > key_extent) nb = key_extent;
    if (nb > kMaxKeyBlocks) nb = kMaxKeyBlocks;
  }
  return static_cast<int>(nb);
}

size_t tc_workspace_size(const TcConfig& c, int64_t rhs_rows, int64_t npairs, int64_t nseg, int nblocks,
                         int64_t key_extent) {
  SizeOnly s;
  TcWs w;
  tc_layout(s, w, c, rhs_rows, npairs, nseg, nblocks, key_extent);
  return s.s.used + 256;
}

int tc_launch(const TcConfig& c, const void* lhs, int64_t lhs_rows, const void* rhs, int64_t rhs_rows,
              const int32_t* pl, const int32_t* pr, int64_t npairs, const int64_t* seg_off, int64_t nseg,
              const int32_t* seg_out, const int64_t* seg_strip, const int32_t* pair_key, int64_t key_extent, void* out,
              int odt, void* ws, size_t ws_bytes, int32_t* err, cudaStream_t st, cudaEvent_t values_ready) {
  if (nseg <= 0) return ES_OK;
  if (nseg >= INT32_MAX || rhs_rows >= INT32_MAX || lhs_rows >= INT32_MAX) return ES_ERR_UNSUPPORTED;
  int l2_blocks = 1;
  const int nblocks = tc_key_blocks(c, rhs_rows, pair_key != nullptr, key_extent, nseg, &l2_blocks);
  Carver cv(ws, ws_bytes);
  TcWs w;
  tc_layout(cv, w, c, rhs_rows, npairs, nseg, nblocks, pair_key ? key_extent : 0);
  if (cv.overflow) return ES_ERR_WORKSPACE;
  // the clears the steps below need ride on launches that are there anyway:
  // the first item kernel clears the zero tile, the item count and the item
  // scan's and item sort's scratch; the merge count pass the record scan's
  // scratch; item_rec the work queue
  const bool grouped = seg_strip && c.G > 1;
  ZeroSpans z0 = no_zero_spans();
  if (!add_zero_span(z0, w.zeros, zero_bytes(c) / 4) || !add_zero_span(z0, w.rb.hist, radix_clear_words(nseg)) ||
      (grouped && (!add_zero_span(z0, w.num_items, 2) || !add_zero_span(z0, w.scan, scan_clear_words(nseg)))))
    return ES_ERR_INVALID;
  // 2. work items
  if (grouped) {
    ES_LAUNCH(item_heads_kernel, grid_for(nseg, 256), 256, 0, st, seg_strip, nseg, c.G, w.flags, w.cnt, z0);
    ES_TRY(exclusive_scan<uint32_t>(w.flags, w.excl, nseg, reinterpret_cast<uint32_t*>(w.num_items), w.scan, st,
                                    nullptr, true));
    ES_LAUNCH(item_place_kernel, grid_for(nseg, 256), 256, 0, st, w.flags, w.excl, w.cnt, nseg, w.item_first,
              w.item_count);
  } else {
    if (c.G != 1) return ES_ERR_INVALID;
    ES_LAUNCH(item_identity_kernel, grid_for(nseg, 256), 256, 0, st, nseg, w.item_first, w.item_count, w.num_items,
              z0);
  }
  // 3. largest items first, handed out by a device-wide queue
  ES_LAUNCH(item_work_keys_kernel, grid_for(nseg, 256), 256, 0, st, w.item_first, w.item_count, seg_off, w.num_items,
            nseg, w.sort_keys, w.order);
  // the sorted order stays in whichever buffer the sort left it
  const uint32_t* order = w.order;
  {
    uint32_t* k = w.sort_keys;
    uint32_t* v = w.order;
    ES_TRY(radix_sort_pairs<uint32_t>(&k, &v, w.rb, nseg, 0, 8, st, err, true));
    order = v;
  }
  // 4. merge steps of every item (all items and key chunks in parallel);
  //    item q takes the sub-strips order[q*S .. q*S+S-1], so items come
  //    largest first
  {
    const int S = c.slots;
    const int64_t nslots = (nseg + S - 1) / S;
    const int C = merge_chunks(nblocks, pair_key != nullptr, key_extent, items_estimate(c, nseg));
    const int32_t* keys = (c.slots > 1 || C > 1) ? pair_key : nullptr;
    const int64_t nw = nslots * C;
    // grid-stride: nw counts a slot per possible item (most are past the real
    // items and only write a zero count), so a grid of a few blocks per SM
    // walks them instead of launching one mostly empty block per 4 slots
    int64_t nb = (nw + kMergeWarps - 1) / kMergeWarps;
    const int blocks = static_cast<int>(nb < 148 * 8 ? nb : 148 * 8);
    ZeroSpans z1 = no_zero_spans(), z2 = no_zero_spans();
    add_zero_span(z1, w.scan2, scan_clear_words(nw));
    add_zero_span(z2, w.queue, 1);
    ES_LAUNCH(tc_merge_kernel<true>, blocks, kMergeWarps * 32, 0, st, pl, pr, keys, seg_off, w.item_first,
              w.item_count, order, w.num_items, S, c.G, lhs_rows, rhs_rows, C, key_extent, nw, w.ipairs,
              (const uint32_t*)nullptr, w.recs, err, z1);
    ES_TRY(exclusive_scan<uint32_t>(w.ipairs, w.rec_base, nw, w.rec_total, w.scan2, st, nullptr, true));
    ES_LAUNCH(tc_merge_kernel<false>, blocks, kMergeWarps * 32, 0, st, pl, pr, keys, seg_off, w.item_first,
              w.item_count, order, w.num_items, S, c.G, lhs_rows, rhs_rows, C, key_extent, nw, w.ipairs,
              (const uint32_t*)w.rec_base, w.recs, err, no_zero_spans());
    ES_LAUNCH(item_rec_kernel, grid_for(nslots, 256), 256, 0, st, (const uint32_t*)w.rec_base,
              (const uint32_t*)w.rec_total, w.num_items, S, C, nblocks, nw, w.item_rec, z2);
  }
  // the steps above read only the pair lists; the values may still be in
  // flight (values_ready: e.g. a tiling's fill on another stream)
  if (values_ready && cudaStreamWaitEvent(st, values_ready, 0) != cudaSuccess) return ES_ERR_CUDA;
  // 5. rhs tiles into the shared-memory image (split for fp32)
  // EINSPARSE_TF32_SPLIT=trunc: the truncating split (comparisons, tests)
  const char* split_env = std::getenv("EINSPARSE_TF32_SPLIT");
  const int rn = (split_env && std::strcmp(split_env, "trunc") == 0) ? 0 : 1;
  const int64_t pe = rhs_rows * c.Kt * c.Nt / (c.fp32 ? 4 : 8);  // 16-byte pieces of the image
  if (pe > 0) {
    if (c.rhs_kmajor) {
      if (c.fp32)
        ES_LAUNCH((layout_rhs_kernel<true, true>), grid_for(pe, 256), 256, 0, st, rhs, rhs_rows, c.Kt, c.Nt, c.KC,
                  w.pan_hi, w.pan_lo, rn);
      else
        ES_LAUNCH((layout_rhs_kernel<false, true>), grid_for(pe, 256), 256, 0, st, rhs, rhs_rows, c.Kt, c.Nt, c.KC,
                  w.pan_hi, (void*)nullptr, rn);
    } else if (c.fp32 && c.Nt >= 128) {
      const int64_t nblk = rhs_rows * (c.Kt / c.KC) * ((c.Nt + kLayoutCols - 1) / kLayoutCols);
      const int g = static_cast<int>(nblk < 148 * 16 ? nblk : 148 * 16);
      ES_LAUNCH(layout_rhs_wide_kernel<true>, g, 256, 0, st, rhs, rhs_rows, c.Kt, c.Nt, c.KC, w.pan_hi, w.pan_lo, rn);
    } else {
      const int64_t prow = rhs_rows * (c.Kt / c.KC) * c.Nt;  // image rows, one thread each
      if (c.fp32)
        ES_LAUNCH((layout_rhs_kernel<true, false>), grid_for(prow, 256), 256, 0, st, rhs, rhs_rows, c.Kt, c.Nt, c.KC,
                  w.pan_hi, w.pan_lo, rn);
      else
        ES_LAUNCH((layout_rhs_kernel<false, false>), grid_for(prow, 256), 256, 0, st, rhs, rhs_rows, c.Kt, c.Nt,
                  c.KC, w.pan_hi, (void*)nullptr, rn);
    }
  }
  // 6. persistent tensor-core kernel, one CTA per SM
  TcParams prm;
  prm.c = c;
  // the staged epilogue stores 16-byte pieces (its shared memory stays reserved)
  if ((reinterpret_cast<uintptr_t>(out) & 15u) != 0) {
    prm.c.epi_stage = 0;
    prm.c.epi_dual = 0;
  }
  prm.lhs = static_cast<const uint8_t*>(lhs);
  prm.lhs_rows = lhs_rows;
  prm.pan_hi = w.pan_hi;
  prm.pan_lo = w.pan_lo;
  prm.rhs_rows = rhs_rows;
  prm.recs = w.recs;
  prm.item_rec = w.item_rec;
  prm.nblocks = nblocks;
  prm.zeros = w.zeros;
  prm.seg_off = seg_off;
  prm.item_first = w.item_first;
  prm.item_count = w.item_count;
  prm.num_items = w.num_items;
  prm.order = reinterpret_cast<const int32_t*>(order);
  prm.queue = w.queue;
  prm.seg_out = seg_out;
  prm.out = out;
  prm.odt = odt;
  prm.err = err;
  prm.chain_recs = chain_records(c);
  prm.rn_split = rn;
  if (prm.chain_recs > 0) {
    // chains only pay for long items: records per item, estimated from the
    // pairs per segment (stacked steps carry about S / 2 lhs tiles)
    const double spp = c.slots > 1 ? c.slots / 2.0 : 1.0;
    const double recs_per_unit = static_cast<double>(npairs) * spp / static_cast<double>(nseg) / l2_blocks;
    if (recs_per_unit < 2.0 * prm.chain_recs) {
      prm.chain_recs = 0;
    } else if (c.fp32 && !c.swap && c.halves * c.col_per_half <= 256) {
      // the running sum of the chains lives in the second half of TMEM
      prm.c.tmem_chain = 1;
      prm.c.acc_bufs = 1;
    }
  }
  prm.part = w.part;
  prm.part_stride = nseg * c.Mt * c.Nt;
  prm.pwritten = w.pwritten;
  prm.nseg = nseg;
  // EINSPARSE_NO_FUSED_BLOCKS: one launch per key block (tuning, tests)
  prm.fused = (w.part != nullptr && odt == ES_F32 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0 &&
               !std::getenv("EINSPARSE_NO_FUSED_BLOCKS"))
                  ? 1
                  : 0;
  // 2-D view of the lhs values for the TMA: (k, row over all tiles); a box
  // of (KC, Mt) lands one tile's k-chunk in shared memory as Mt swizzled
  // rows of W bytes, the operand layout of the MMA.
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess || !fn)
      return ES_ERR_CUDA;
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  const int esz = c.fp32 ? 4 : 2;
  CUtensorMap lhs_map;
  std::memset(&lhs_map, 0, sizeof(lhs_map));
  cuuint64_t gdim[2] = {static_cast<cuuint64_t>(c.Kt), static_cast<cuuint64_t>(lhs_rows) * c.Mt};
  cuuint64_t gstride[1] = {static_cast<cuuint64_t>(c.Kt) * esz};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(c.KC), static_cast<cuuint32_t>(c.Mt)};
  cuuint32_t estride[2] = {1, 1};
  const CUtensorMapSwizzle swz = c.swz == 2 ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : c.swz == 4 ? CU_TENSOR_MAP_SWIZZLE_64B
                                              : CU_TENSOR_MAP_SWIZZLE_32B;
  if (lhs_rows <= 0) return ES_OK;
  CUresult cr = encode(&lhs_map, c.fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                       const_cast<void*>(lhs), gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                       CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return ES_ERR_UNSUPPORTED;
  int dev = 0, sms = kSMs;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t grid = nseg < sms ? nseg : sms;
  {
    // the kernel's dynamic shared memory limit: per device, raised once to
    // the largest configuration (any smaller one then fits)
    static int attr_bytes[2][kMaxAttrDevices] = {};
    const int fi = c.fp32 ? 1 : 0;
    if (dev < 0 || dev >= kMaxAttrDevices || attr_bytes[fi][dev] < c.smem_bytes) {
      const cudaError_t e =
          c.fp32 ? cudaFuncSetAttribute(tc_strip_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        c.smem_bytes)
                 : cudaFuncSetAttribute(tc_strip_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        c.smem_bytes);
      if (e != cudaSuccess) return ES_ERR_CUDA;
      if (dev >= 0 && dev < kMaxAttrDevices) attr_bytes[fi][dev] = c.smem_bytes;
    }
  }
  if (prm.fused) {
    prm.blk = 0;
    prm.accumulate = 0;
    if (c.fp32)
      ES_LAUNCH(tc_strip_kernel<true>, (int)grid, kThreads, c.smem_bytes, st, prm, lhs_map);
    else
      ES_LAUNCH(tc_strip_kernel<false>, (int)grid, kThreads, c.smem_bytes, st, prm, lhs_map);
    const int64_t te4 = static_cast<int64_t>(c.Mt) * c.Nt / 4;
    const int64_t nv = nseg * te4;
    const int pg = static_cast<int>(nv / 256 + 1 < 148 * 8 ? nv / 256 + 1 : 148 * 8);
    ES_LAUNCH(add_partials_kernel, pg, 256, 0, st, static_cast<float*>(out), w.part, w.pwritten, nseg, te4,
              nblocks - 1, prm.part_stride, seg_out);
    return ES_OK;
  }
  for (int b = 0; b < nblocks; ++b) {
    prm.blk = b;
    prm.accumulate = b > 0 ? 1 : 0;
    if (b > 0 && cudaMemsetAsync(w.queue, 0, sizeof(int), st) != cudaSuccess) return ES_ERR_CUDA;
    if (c.fp32)
      ES_LAUNCH(tc_strip_kernel<true>, (int)grid, kThreads, c.smem_bytes, st, prm, lhs_map);
    else
      ES_LAUNCH(tc_strip_kernel<false>, (int)grid, kThreads, c.smem_bytes, st, prm, lhs_map);
  }
  return ES_OK;
}

}  // namespace es
