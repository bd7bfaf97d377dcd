// Stable LSD radix sort of (key, uint32 payload) pairs, 8 bits per pass,
// "onesweep" style (Adinets & Merrill, "Onesweep: A Faster Least Significant
// Digit Radix Sort for GPUs", 2022): one upsweep reads the keys once and
// builds the global digit histogram of every pass; then each pass is ONE
// launch. A CTA takes the next 4096-key tile from an atomic counter, ranks
// its keys stably -- warp w owns keys [w*512, w*512+512) of the tile and
// walks them 32 at a time, eight ballots group lanes with equal digits and a
// per-warp digit counter gives the running rank -- publishes the
// tile's per-digit counts, finds the counts of all earlier tiles by a
// decoupled look-back over their per-digit status words (one thread per
// digit), and writes the tile reordered through shared memory so every
// digit's run leaves as one coalesced store.
//
// Status word (64 bits): the count in the low 32 bits, a code in the high 32
// -- 2p+1 "aggregate of this tile" or 2p+2 "inclusive prefix up to this
// tile" for pass p. The words are cleared once per sort; codes only grow
// from pass to pass, so a word left from the previous pass reads as "not yet
// published". Waits are bounded: after kScanSpin polls the CTA records
// ES_ERR_TIMEOUT and takes 0 (the output is then invalid).
#pragma once

#include "common.cuh"
#include "scan.cuh"

namespace es {

constexpr int kRsThreads = 256;
constexpr int kRsWarps = kRsThreads / 32;
constexpr int kRsChunks = 16;  // chunks of 32 keys per warp
constexpr int kRsTile = kRsThreads * kRsChunks;
constexpr int kRsBins = 256;
constexpr int kRsMaxPasses = 8;
constexpr int kRsLook = 8;  // status words read per look-back step

__device__ __forceinline__ void st_relaxed_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Lanes of this warp whose key has the same digit (valid lanes only; the
// result of an invalid lane is unused): eight ballots, one per digit bit
// (warp-level multisplit, in place of __match_any_sync).
__device__ __forceinline__ unsigned warp_peers(uint32_t dig, int nbits, bool valid) {
  unsigned peers = __ballot_sync(0xffffffffu, valid);
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    if (b < nbits) {  // nbits is the same for the whole warp
      const bool bit = (dig >> b) & 1u;
      const unsigned bb = __ballot_sync(0xffffffffu, bit);
      peers &= bit ? bb : ~bb;
    }
  }
  return peers;
}

// Global digit histograms of every pass: ghist[p * 256 + d]. A warp whose 32
// keys share a digit adds 32 once; otherwise each lane adds 1.
template <typename K>
__global__ void __launch_bounds__(kRsThreads) rs_upsweep_kernel(const K* __restrict__ keys, int64_t n, int begin_bit,
                                                                int end_bit, uint32_t* __restrict__ ghist) {
  __shared__ uint32_t h[kRsMaxPasses * kRsBins];
  const int npass = (end_bit - begin_bit + 7) / 8;
  for (int i = threadIdx.x; i < npass * kRsBins; i += kRsThreads) h[i] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kRsThreads;
  // every lane of a warp runs the same number of iterations (the votes need them all)
  const int64_t n_pad = (n + 31) & ~static_cast<int64_t>(31);
  for (int64_t g = blockIdx.x * static_cast<int64_t>(kRsThreads) + threadIdx.x; g < n_pad; g += stride) {
    const bool valid = g < n;
    const K k = valid ? keys[g] : K(0);
    for (int p = 0; p < npass; ++p) {
      const int shift = begin_bit + 8 * p;
      const int nb = end_bit - shift < 8 ? end_bit - shift : 8;
      const uint32_t dig = static_cast<uint32_t>(k >> shift) & ((1u << nb) - 1u);
      const uint32_t d0 = __shfl_sync(0xffffffffu, dig, 0);
      const unsigned vb = __ballot_sync(0xffffffffu, valid);
      if (__all_sync(0xffffffffu, !valid || dig == d0)) {
        if (lane == 0 && vb) atomicAdd(&h[p * kRsBins + d0], static_cast<uint32_t>(__popc(vb)));
      } else if (valid) {
        atomicAdd(&h[p * kRsBins + dig], 1u);
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < npass * kRsBins; i += kRsThreads)
    if (h[i]) atomicAdd(&ghist[i], h[i]);
}

template <typename K>
__global__ void __launch_bounds__(kRsThreads, 3) rs_onesweep_kernel(const K* __restrict__ keys_in,
                                                                 const uint32_t* __restrict__ vals_in,
                                                                 K* __restrict__ keys_out,
                                                                 uint32_t* __restrict__ vals_out, int64_t n, int shift,
                                                                 uint32_t mask, int pass,
                                                                 const uint32_t* __restrict__ ghist_pass,
                                                                 uint64_t* __restrict__ status,
                                                                 uint32_t* __restrict__ next_tile, int32_t* err) {
  extern __shared__ __align__(16) unsigned char rs_smem[];
  K* skeys = reinterpret_cast<K*>(rs_smem);
  uint32_t* svals = reinterpret_cast<uint32_t*>(skeys + kRsTile);
  uint32_t* wcnt = svals + kRsTile;           // [warp][digit]
  uint32_t* bstart = wcnt + kRsWarps * kRsBins;
  uint32_t* goff = bstart + kRsBins;
  __shared__ uint32_t wtot[kRsWarps];
  __shared__ uint32_t tile_sh;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nbits = __popc(mask);
  if (tid == 0) tile_sh = atomicAdd(next_tile, 1u);
  for (int i = tid; i < kRsWarps * kRsBins; i += kRsThreads) wcnt[i] = 0;
  __syncthreads();
  const int64_t tile = tile_sh;
  const int64_t base = tile * kRsTile;

  // keys and ranks stay in registers; payloads are read again at the scatter
  // (three CTAs per SM fit that way)
  K k[kRsChunks];
  uint32_t rank[kRsChunks];
  const unsigned lt = (1u << lane) - 1u;
  uint32_t* my = wcnt + warp * kRsBins;
  const int64_t wbase = base + warp * (kRsChunks * 32) + lane;
#pragma unroll
  for (int c = 0; c < kRsChunks; ++c) {  // all loads in flight before the ranking
    const int64_t g = wbase + c * 32;
    k[c] = g < n ? keys_in[g] : K(0);
  }
#pragma unroll
  for (int c = 0; c < kRsChunks; ++c) {
    const bool valid = wbase + c * 32 < n;
    uint32_t dig = static_cast<uint32_t>(k[c] >> shift) & mask;
    const uint32_t d0 = __shfl_sync(0xffffffffu, dig, 0);
    unsigned peers = __all_sync(0xffffffffu, !valid || dig == d0) ? __ballot_sync(0xffffffffu, valid)
                                                                   : warp_peers(dig, nbits, valid);
    uint32_t r = __popc(peers & lt);
    uint32_t b = valid ? my[dig] : 0u;
    __syncwarp();
    if (valid && r == 0) my[dig] = b + __popc(peers);
    __syncwarp();
    rank[c] = b + r;
  }
  __syncthreads();
  const uint64_t code_agg = static_cast<uint64_t>(2 * pass + 1) << 32;
  const uint64_t code_inc = static_cast<uint64_t>(2 * pass + 2) << 32;
  {
    const int d = tid;  // kRsThreads == kRsBins: thread d owns digit d
    // digit d: exclusive prefix over warps (in place) and the tile's count
    uint32_t run = 0;
#pragma unroll
    for (int w = 0; w < kRsWarps; ++w) {
      uint32_t t = wcnt[w * kRsBins + d];
      wcnt[w * kRsBins + d] = run;
      run += t;
    }
    uint64_t* sw = status + tile * kRsBins + d;
    st_relaxed_u64(sw, (tile == 0 ? code_inc : code_agg) | run);
    // the tile-local start of digit d (exclusive scan of the counts over digits)
    uint32_t incl = warp_inclusive_scan(run);
    if (lane == 31) wtot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      uint32_t x = lane < kRsWarps ? wtot[lane] : 0u;
      uint32_t xi = warp_inclusive_scan(x);
      if (lane < kRsWarps) wtot[lane] = xi - x;
    }
    __syncthreads();
    bstart[d] = wtot[warp] + incl - run;
    __syncthreads();
    // the global start of digit d over the whole pass (same scan over the global histogram)
    const uint32_t gd = ghist_pass[d];
    uint32_t gincl = warp_inclusive_scan(gd);
    if (lane == 31) wtot[warp] = gincl;
    __syncthreads();
    if (warp == 0) {
      uint32_t x = lane < kRsWarps ? wtot[lane] : 0u;
      uint32_t xi = warp_inclusive_scan(x);
      if (lane < kRsWarps) wtot[lane] = xi - x;
    }
    __syncthreads();
    uint32_t before = wtot[warp] + gincl - gd;
    // look back over earlier tiles' counts of digit d, kRsLook status words
    // per step (independent loads in flight; each word carries its own count,
    // so relaxed loads suffice)
    if (tile > 0) {
      uint32_t excl = 0;
      int64_t j = tile - 1;
      int spins = 0;
      bool timed_out = false;
      while (true) {
        uint64_t w[kRsLook];
#pragma unroll
        for (int q = 0; q < kRsLook; ++q)
          w[q] = j - q >= 0 ? ld_relaxed_u64(status + (j - q) * kRsBins + d) : code_inc;
        int q = 0;  // words consumed, in order from tile j down
        bool done = false, stalled = false;
#pragma unroll
        for (int qq = 0; qq < kRsLook; ++qq) {
          const uint64_t code = w[qq] & 0xFFFFFFFF00000000ull;
          if (code < code_agg) {  // not published yet: wait for it below
            stalled = true;
            break;
          }
          excl += static_cast<uint32_t>(w[qq]);
          q = qq + 1;
          if (code == code_inc) {
            done = true;
            break;
          }
        }
        if (done) break;
        j -= q;
        if (stalled) {  // tile j has not published for this pass
          if (++spins > kScanSpin) {
            timed_out = true;
            break;
          }
          if (spins > 64) __nanosleep(64);
        }
      }
      if (timed_out) atomicExch(err ? err : &g_scan_timeout, ES_ERR_TIMEOUT);
      st_relaxed_u64(sw, code_inc | (excl + run));
      before += excl;
    }
    goff[d] = before;
  }
  __syncthreads();
#pragma unroll
  for (int c = 0; c < kRsChunks; ++c) {
    int64_t g = base + warp * (kRsChunks * 32) + c * 32 + lane;
    if (g < n) {
      uint32_t dig = static_cast<uint32_t>(k[c] >> shift) & mask;
      uint32_t pos = bstart[dig] + my[dig] + rank[c];
      skeys[pos] = k[c];
      svals[pos] = vals_in[g];
    }
  }
  __syncthreads();
  const int cnt = static_cast<int>(min(static_cast<int64_t>(kRsTile), n - base));
  for (int i = tid; i < cnt; i += kRsThreads) {
    K kk = skeys[i];
    uint32_t dig = static_cast<uint32_t>(kk >> shift) & mask;
    uint32_t dst = goff[dig] + (static_cast<uint32_t>(i) - bstart[dig]);
    keys_out[dst] = kk;
    vals_out[dst] = svals[i];
  }
}

template <typename K>
constexpr size_t rs_scatter_smem() {
  return kRsTile * sizeof(K) + kRsTile * sizeof(uint32_t) + (kRsWarps * kRsBins + 2 * kRsBins) * sizeof(uint32_t);
}

// Scratch of a sort of n pairs, carved by callers as uint32 elements:
// hist = the per-(tile, digit) status words (2 uint32 each), then the
// per-pass tile counters and global histograms; scan = unused (1 element,
// kept so callers' workspace layouts stay put).
struct RadixScratchSize {
  static int64_t tiles(int64_t n) { return (n + kRsTile - 1) / kRsTile; }
  static int64_t status_words(int64_t n) { return kRsBins * (tiles(n) > 0 ? tiles(n) : 1); }
  static int64_t hist_elems(int64_t n) { return 2 * status_words(n) + kRsMaxPasses + kRsMaxPasses * kRsBins; }
  static int64_t scan_elems(int64_t) { return 1; }
};

// Workspace slices a radix sort of n pairs needs (besides the input arrays).
template <typename K>
inline void radix_reserve(Sizer& sz, int64_t n) {
  sz.take<K>(n);
  sz.take<uint32_t>(n);
  sz.take<uint32_t>(RadixScratchSize::hist_elems(n));
  sz.take<uint32_t>(RadixScratchSize::scan_elems(n));
}

template <typename K>
struct RadixBuffers {
  K* keys_alt = nullptr;
  uint32_t* vals_alt = nullptr;
  uint32_t* hist = nullptr;
  uint32_t* scan = nullptr;
  void carve(Carver& c, int64_t n) {
    keys_alt = c.take<K>(n);
    vals_alt = c.take<uint32_t>(n);
    hist = c.take<uint32_t>(RadixScratchSize::hist_elems(n));
    scan = c.take<uint32_t>(RadixScratchSize::scan_elems(n));
  }
};

// 32-bit words of rb.hist that a sort of n keys needs cleared before it runs.
inline int64_t radix_clear_words(int64_t n) { return RadixScratchSize::hist_elems(n); }

// Sorts bits [begin_bit, end_bit) of the keys, stable. On return *keys/*vals
// point at whichever buffer holds the sorted data (the alternate buffers when
// the number of 8-bit passes is odd). Launches: one clear of the scratch
// (none when precleared: an earlier launch on the stream cleared
// radix_clear_words(n) words of rb.hist), the upsweep, one kernel per pass.
// A look-back timeout is recorded in *err when given.
template <typename K>
int radix_sort_pairs(K** keys, uint32_t** vals, RadixBuffers<K>& rb, int64_t n, int begin_bit, int end_bit,
                     cudaStream_t st, int32_t* err = nullptr, bool precleared = false) {
  if (n <= 1 || begin_bit >= end_bit) return ES_OK;
  if (n >= static_cast<int64_t>(UINT32_MAX)) return ES_ERR_UNSUPPORTED;
  const int npass = (end_bit - begin_bit + 7) / 8;
  if (npass > kRsMaxPasses) return ES_ERR_UNSUPPORTED;
  // the attribute is per device: set once on each
  static bool attr_set[kMaxAttrDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return ES_ERR_CUDA;
  if (dev < 0 || dev >= kMaxAttrDevices || !attr_set[dev]) {
    if (cudaFuncSetAttribute(rs_onesweep_kernel<K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(rs_scatter_smem<K>())) != cudaSuccess)
      return ES_ERR_CUDA;
    if (dev >= 0 && dev < kMaxAttrDevices) attr_set[dev] = true;
  }
  const int64_t tiles = RadixScratchSize::tiles(n);
  uint64_t* status = reinterpret_cast<uint64_t*>(rb.hist);
  uint32_t* counters = rb.hist + 2 * RadixScratchSize::status_words(n);
  uint32_t* ghist = counters + kRsMaxPasses;
  const size_t clear = (2 * RadixScratchSize::status_words(n) + kRsMaxPasses + npass * kRsBins) * sizeof(uint32_t);
  if (!precleared && cudaMemsetAsync(rb.hist, 0, clear, st) != cudaSuccess) return ES_ERR_CUDA;
  const int up_grid = static_cast<int>(tiles < 148 * 8 ? tiles : 148 * 8);
  ES_LAUNCH(rs_upsweep_kernel<K>, up_grid, kRsThreads, 0, st, *keys, n, begin_bit, end_bit, ghist);
  K* kin = *keys;
  uint32_t* vin = *vals;
  K* kout = rb.keys_alt;
  uint32_t* vout = rb.vals_alt;
  for (int p = 0; p < npass; ++p) {
    const int shift = begin_bit + 8 * p;
    const int nbits = end_bit - shift < 8 ? end_bit - shift : 8;
    const uint32_t mask = (1u << nbits) - 1u;
    ES_LAUNCH(rs_onesweep_kernel<K>, (int)tiles, kRsThreads, rs_scatter_smem<K>(), st, kin, vin, kout, vout, n, shift,
              mask, p, ghist + p * kRsBins, status, counters + p, err);
    K* tk = kin; kin = kout; kout = tk;
    uint32_t* tv = vin; vin = vout; vout = tv;
  }
  *keys = kin;
  *vals = vin;
  return ES_OK;
}

}  // namespace es
