// Device-wide exclusive prefix sum (reduce-then-scan, 4096 elements per CTA).
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

template <typename T>
__global__ void scan_tile_sums_kernel(const T* __restrict__ in, int64_t n, T* __restrict__ sums) {
  __shared__ T red[kScanThreads / 32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile;
  T acc = 0;
  for (int i = threadIdx.x; i < kScanTile; i += kScanThreads) {
    int64_t g = base + i;
    if (g < n) acc += in[g];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_down_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    T v = threadIdx.x < kScanThreads / 32 ? red[threadIdx.x] : T(0);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) sums[blockIdx.x] = v;
  }
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

template <typename T>
__global__ void write_total_kernel(const T* sums_scanned, const T* sums_raw, int64_t nb, T* total) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *total = sums_scanned[nb - 1] + sums_raw[nb - 1];
}

// Scratch elements (of T) that exclusive_scan needs for n inputs.
inline int64_t scan_scratch_elems(int64_t n) {
  int64_t total = 0;
  while (n > kScanTile) {
    int64_t nb = (n + kScanTile - 1) / kScanTile;
    total += 2 * nb;  // raw sums + scanned sums
    n = nb;
  }
  return total + 1;
}

// out[i] = sum(in[0..i)); *total (device, optional) = sum(in). In-place allowed.
template <typename T>
int exclusive_scan(const T* in, T* out, int64_t n, T* total, T* scratch, cudaStream_t st) {
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
  int64_t nb = (n + kScanTile - 1) / kScanTile;
  T* sums = scratch;
  T* sums_scanned = scratch + nb;
  ES_LAUNCH(scan_tile_sums_kernel<T>, (int)nb, kScanThreads, 0, st, in, n, sums);
  ES_TRY(exclusive_scan<T>(sums, sums_scanned, nb, (T*)nullptr, scratch + 2 * nb, st));
  if (total) ES_LAUNCH(write_total_kernel<T>, 1, 32, 0, st, (const T*)sums_scanned, (const T*)sums, nb, total);
  ES_LAUNCH(scan_tiles_kernel<T>, (int)nb, kScanThreads, 0, st, in, out, n, (const T*)sums_scanned, (T*)nullptr);
  return ES_OK;
}

}  // namespace es
