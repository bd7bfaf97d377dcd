// Device-wide exclusive prefix sum (single pass, 4096 elements per CTA).
#pragma once

#include "common.cuh"

namespace es {

constexpr int kScanThreads = 512;
constexpr int kScanItems = 8;
constexpr int kScanTile = kScanThreads * kScanItems;

template <typename T>
__device__ __forceinline__ T warp_inclusive_scan(T v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

// Exclusive scan of one tile held in shared memory (kScanTile elements);
// returns the tile total to every thread.
template <typename T>
__device__ T block_exclusive_scan_tile(T* s) {
  __shared__ T warp_tot[kScanThreads / 32];
  const int tid = threadIdx.x;
  T local[kScanItems];
  T run = 0;
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    local[i] = s[tid * kScanItems + i];
    run += local[i];
  }
  T incl = warp_inclusive_scan(run);
  const int lane = tid & 31, warp = tid >> 5;
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    T w = lane < kScanThreads / 32 ? warp_tot[lane] : T(0);
    T wi = warp_inclusive_scan(w);
    if (lane < kScanThreads / 32) warp_tot[lane] = wi - w;
  }
  __syncthreads();
  T base = warp_tot[warp] + incl - run;
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kScanItems; ++i) {
    s[tid * kScanItems + i] = base;
    base += local[i];
  }
  // last thread holds the grand total in `base`
  __shared__ T grand;
  if (tid == kScanThreads - 1) grand = base;
  __syncthreads();
  return grand;
}

// Scans each tile; adds tile_offsets[blockIdx.x] (if given). Writes the
// grand total to *total when this is a single-tile scan.
template <typename T>
__global__ void scan_tiles_kernel(const T* in, T* out, int64_t n,
                                  const T* __restrict__ tile_offsets, T* __restrict__ total) {
  __shared__ T s[kScanTile];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile;
  for (int i = threadIdx.x; i < kScanTile; i += kScanThreads) {
    int64_t g = base + i;
    s[i] = g < n ? in[g] : T(0);
  }
  __syncthreads();
  T grand = block_exclusive_scan_tile<T>(s);
  __syncthreads();
  T off = tile_offsets ? tile_offsets[blockIdx.x] : T(0);
  for (int i = threadIdx.x; i < kScanTile; i += kScanThreads) {
    int64_t g = base + i;
    if (g < n) out[g] = s[i] + off;
  }
  if (total && tile_offsets == nullptr && threadIdx.x == 0) *total = grand;
}

// Single-pass scan over tiles with decoupled look-back (Merrill & Garland,
// "Single-pass Parallel Prefix Scan with Decoupled Look-back", 2016). Each
// CTA takes the next tile from an atomic counter -- so every earlier tile
// belongs to a CTA that is already running, and the look-back always ends
// -- scans it in shared memory, publishes the tile's aggregate, then walks
// back over the status words of earlier tiles (a warp at a time, 32 tiles
// per step) until it meets an inclusive prefix, and publishes its own.
// Status word: flag in bits 62-63 (0 none, 1 aggregate, 2 inclusive
// prefix), value in bits 0-61 (the sums scanned here are non-negative
// counts, below 2^62). The wait on a tile without status is bounded: after
// kScanSpin polls the CTA records ES_ERR_TIMEOUT and takes 0 for it.
constexpr uint64_t kScanAgg = 1ull << 62, kScanInc = 2ull << 62, kScanVal = (1ull << 62) - 1;
constexpr int kScanSpin = 1 << 22;

__device__ int32_t g_scan_timeout;

__device__ __forceinline__ void st_release_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_acquire_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

template <typename T>
__global__ void scan_lookback_kernel(const T* in, T* out, int64_t n, uint64_t* __restrict__ status,
                                     uint32_t* __restrict__ next_tile, T* __restrict__ total, int32_t* err) {
  __shared__ T s[kScanTile];
  __shared__ uint32_t tile_sh;
  __shared__ T excl_sh;
  if (threadIdx.x == 0) tile_sh = atomicAdd(next_tile, 1u);
  __syncthreads();
  const int64_t tile = tile_sh;
  const int64_t base = tile * kScanTile;
  for (int i = threadIdx.x; i < kScanTile; i += kScanThreads) {
    const int64_t g = base + i;
    s[i] = g < n ? in[g] : T(0);
  }
  __syncthreads();
  const T agg = block_exclusive_scan_tile<T>(s);
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    T excl = 0;
    if (tile == 0) {
      if (lane == 0) st_release_u64(status, kScanInc | (static_cast<uint64_t>(agg) & kScanVal));
    } else {
      if (lane == 0) st_release_u64(status + tile, kScanAgg | (static_cast<uint64_t>(agg) & kScanVal));
      int64_t hi = tile - 1;  // window [hi - 31, hi], lane l reads tile hi - l
      int spins = 0;
      bool timed_out = false;
      while (true) {
        const int64_t t = hi - lane;
        uint64_t w = t >= 0 ? ld_acquire_u64(status + t) : kScanInc;
        const bool missing = (w >> 62) == 0;
        if (__any_sync(0xffffffffu, missing)) {
          if (++spins > kScanSpin) {
            timed_out = true;
            if (missing) w = kScanInc;  // give up: counts as 0
          } else {
            if (spins > 64) __nanosleep(64);
            continue;
          }
        }
        // closest inclusive prefix in the window, if any
        const uint32_t inc = __ballot_sync(0xffffffffu, (w >> 62) == 2);
        const int stop = inc ? __ffs(inc) - 1 : 32;
        T v = lane <= stop ? static_cast<T>(w & kScanVal) : T(0);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        excl += v;
        if (inc) break;
        hi -= 32;
      }
      if (lane == 0) {
        if (timed_out) atomicExch(err ? err : &g_scan_timeout, ES_ERR_TIMEOUT);
        st_release_u64(status + tile, kScanInc | (static_cast<uint64_t>(excl + agg) & kScanVal));
      }
    }
    if (lane == 0) excl_sh = excl;
  }
  __syncthreads();
  const T off = excl_sh;
  for (int i = threadIdx.x; i < kScanTile; i += kScanThreads) {
    const int64_t g = base + i;
    if (g < n) out[g] = s[i] + off;
  }
  if (total && threadIdx.x == 0 && base + kScanTile >= n) *total = off + agg;
}

// Scratch elements (of T, 4 or 8 bytes) that exclusive_scan needs for n
// inputs: one status word per tile and the tile counter.
inline int64_t scan_scratch_elems(int64_t n) {
  if (n <= kScanTile) return 1;
  const int64_t nb = (n + kScanTile - 1) / kScanTile;
  return 2 * nb + 2;
}

// out[i] = sum(in[0..i)); *total (device, optional) = sum(in). In-place
// allowed. Inputs are non-negative. One launch (plus a clear of the tile
// status) at any size; a look-back timeout is recorded in *err when given.
// 32-bit words of `scratch` that a scan of n inputs needs cleared before it
// runs (0: the single-tile scan needs none).
inline int64_t scan_clear_words(int64_t n) {
  if (n <= kScanTile) return 0;
  const int64_t nb = (n + kScanTile - 1) / kScanTile;
  return 2 * nb + 1;
}

// precleared: an earlier launch on the stream cleared scan_clear_words(n)
// words of scratch (no clear of its own here).
template <typename T>
int exclusive_scan(const T* in, T* out, int64_t n, T* total, T* scratch, cudaStream_t st, int32_t* err = nullptr,
                   bool precleared = false) {
  if (n <= 0) {
    if (total) {
      if (cudaMemsetAsync(total, 0, sizeof(T), st) != cudaSuccess) return ES_ERR_CUDA;
    }
    return ES_OK;
  }
  if (n <= kScanTile) {
    ES_LAUNCH(scan_tiles_kernel<T>, 1, kScanThreads, 0, st, in, out, n, (const T*)nullptr, total);
    return ES_OK;
  }
  const int64_t nb = (n + kScanTile - 1) / kScanTile;
  uint64_t* status = reinterpret_cast<uint64_t*>(scratch);
  uint32_t* next_tile = reinterpret_cast<uint32_t*>(status + nb);
  if (!precleared && cudaMemsetAsync(status, 0, nb * sizeof(uint64_t) + sizeof(uint32_t), st) != cudaSuccess)
    return ES_ERR_CUDA;
  ES_LAUNCH(scan_lookback_kernel<T>, static_cast<int>(nb), kScanThreads, 0, st, in, out, n, status, next_tile, total,
            err);
  return ES_OK;
}

}  // namespace es
