// Stable LSD radix sort of (key, uint32 payload) pairs, 8 bits per pass.
//
// Per pass: (1) per-tile digit histograms (4096 keys per CTA, warp-aggregated
// shared atomics), (2) one exclusive scan over the digit-major histogram
// matrix gives every (digit, tile) its global offset, (3) each CTA ranks its
// keys stably — warp w owns keys [w*512, w*512+512) of the tile and walks
// them 32 at a time, __match_any_sync groups lanes with equal digits and a
// per-warp digit counter gives the running rank — then reorders the tile in
// shared memory so every digit's run leaves as one coalesced store.
#pragma once

#include "common.cuh"
#include "scan.cuh"

namespace es {

constexpr int kRsThreads = 256;
constexpr int kRsWarps = kRsThreads / 32;
constexpr int kRsChunks = 16;  // chunks of 32 keys per warp
constexpr int kRsTile = kRsThreads * kRsChunks;
constexpr int kRsBins = 256;

template <typename K>
__global__ void __launch_bounds__(kRsThreads) rs_hist_kernel(const K* __restrict__ keys, int64_t n, int shift,
                                                             uint32_t mask, uint32_t* __restrict__ hist,
                                                             int64_t num_tiles) {
  __shared__ uint32_t h[kRsBins];
  for (int i = threadIdx.x; i < kRsBins; i += kRsThreads) h[i] = 0;
  __syncthreads();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kRsTile;
  const int lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kRsTile; i += kRsThreads) {
    int64_t g = base + i;
    bool valid = g < n;
    uint32_t dig = valid ? (static_cast<uint32_t>(keys[g] >> shift) & mask) : (kRsBins + lane);
    unsigned peers = __match_any_sync(0xffffffffu, dig);
    if (valid && (__ffs(peers) - 1) == lane) atomicAdd(&h[dig], static_cast<uint32_t>(__popc(peers)));
  }
  __syncthreads();
  for (int d = threadIdx.x; d < kRsBins; d += kRsThreads) hist[static_cast<int64_t>(d) * num_tiles + blockIdx.x] = h[d];
}

template <typename K>
__global__ void __launch_bounds__(kRsThreads) rs_scatter_kernel(const K* __restrict__ keys_in,
                                                                const uint32_t* __restrict__ vals_in,
                                                                K* __restrict__ keys_out,
                                                                uint32_t* __restrict__ vals_out, int64_t n,
                                                                int shift, uint32_t mask,
                                                                const uint32_t* __restrict__ offsets,
                                                                int64_t num_tiles) {
  extern __shared__ __align__(16) unsigned char rs_smem[];
  K* skeys = reinterpret_cast<K*>(rs_smem);
  uint32_t* svals = reinterpret_cast<uint32_t*>(skeys + kRsTile);
  uint32_t* wcnt = svals + kRsTile;           // [warp][digit]
  uint32_t* bstart = wcnt + kRsWarps * kRsBins;
  uint32_t* goff = bstart + kRsBins;
  __shared__ uint32_t wtot[kRsWarps];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kRsTile;
  for (int i = tid; i < kRsWarps * kRsBins; i += kRsThreads) wcnt[i] = 0;
  for (int d = tid; d < kRsBins; d += kRsThreads) goff[d] = offsets[static_cast<int64_t>(d) * num_tiles + blockIdx.x];
  __syncthreads();

  K k[kRsChunks];
  uint32_t v[kRsChunks];
  uint32_t rank[kRsChunks];
  const unsigned lt = (1u << lane) - 1u;
  uint32_t* my = wcnt + warp * kRsBins;
#pragma unroll
  for (int c = 0; c < kRsChunks; ++c) {
    int64_t g = base + warp * (kRsChunks * 32) + c * 32 + lane;
    bool valid = g < n;
    k[c] = valid ? keys_in[g] : K(0);
    v[c] = valid ? vals_in[g] : 0u;
    uint32_t dig = valid ? (static_cast<uint32_t>(k[c] >> shift) & mask) : (kRsBins + lane);
    unsigned peers = __match_any_sync(0xffffffffu, dig);
    uint32_t r = __popc(peers & lt);
    uint32_t b = valid ? my[dig] : 0u;
    __syncwarp();
    if (valid && r == 0) my[dig] = b + __popc(peers);
    __syncwarp();
    rank[c] = b + r;
  }
  __syncthreads();
  // digit d: exclusive prefix over warps (in place) and the tile total
  {
    const int d = tid;  // kRsThreads == kRsBins
    uint32_t run = 0;
#pragma unroll
    for (int w = 0; w < kRsWarps; ++w) {
      uint32_t t = wcnt[w * kRsBins + d];
      wcnt[w * kRsBins + d] = run;
      run += t;
    }
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
  }
  __syncthreads();
#pragma unroll
  for (int c = 0; c < kRsChunks; ++c) {
    int64_t g = base + warp * (kRsChunks * 32) + c * 32 + lane;
    if (g < n) {
      uint32_t dig = static_cast<uint32_t>(k[c] >> shift) & mask;
      uint32_t pos = bstart[dig] + my[dig] + rank[c];
      skeys[pos] = k[c];
      svals[pos] = v[c];
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

struct RadixScratchSize {
  static int64_t tiles(int64_t n) { return (n + kRsTile - 1) / kRsTile; }
  static int64_t hist_elems(int64_t n) { return kRsBins * (tiles(n) > 0 ? tiles(n) : 1); }
  static int64_t scan_elems(int64_t n) { return scan_scratch_elems(hist_elems(n)); }
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

// Sorts bits [begin_bit, end_bit) of the keys, stable. On return *keys/*vals
// point at whichever buffer holds the sorted data.
template <typename K>
int radix_sort_pairs(K** keys, uint32_t** vals, RadixBuffers<K>& rb, int64_t n, int begin_bit, int end_bit,
                     cudaStream_t st) {
  if (n <= 1 || begin_bit >= end_bit) return ES_OK;
  // The attribute is per device; setting it is a cheap host call.
  if (cudaFuncSetAttribute(rs_scatter_kernel<K>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(rs_scatter_smem<K>())) != cudaSuccess)
    return ES_ERR_CUDA;
  const int64_t tiles = RadixScratchSize::tiles(n);
  K* kin = *keys;
  uint32_t* vin = *vals;
  K* kout = rb.keys_alt;
  uint32_t* vout = rb.vals_alt;
  for (int shift = begin_bit; shift < end_bit; shift += 8) {
    int nbits = end_bit - shift < 8 ? end_bit - shift : 8;
    uint32_t mask = (1u << nbits) - 1u;
    ES_LAUNCH(rs_hist_kernel<K>, (int)tiles, kRsThreads, 0, st, kin, n, shift, mask, rb.hist, tiles);
    ES_TRY(exclusive_scan<uint32_t>(rb.hist, rb.hist, kRsBins * tiles, (uint32_t*)nullptr, rb.scan, st));
    ES_LAUNCH(rs_scatter_kernel<K>, (int)tiles, kRsThreads, rs_scatter_smem<K>(), st, kin, vin, kout, vout, n, shift,
              mask, rb.hist, tiles);
    K* tk = kin; kin = kout; kout = tk;
    uint32_t* tv = vin; vin = vout; vout = tv;
  }
  *keys = kin;
  *vals = vin;
  return ES_OK;
}

}  // namespace es
