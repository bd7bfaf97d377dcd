// Shared helpers for the einsparse library (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include <atomic>

#include "einsparse.h"

namespace es {

extern std::atomic<int64_t> g_launches;

inline void count_launch(int n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

// Returns ES_ERR_CUDA if the last launch failed to start.
inline int check_launch() {
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ES_OK : ES_ERR_CUDA;
}

#define ES_TRY(expr)             \
  do {                           \
    int _st = (expr);            \
    if (_st != ES_OK) return _st; \
  } while (0)

#define ES_LAUNCH(kernel, grid, block, smem, stream, ...)                 \
  do {                                                                   \
    kernel<<<(grid), (block), (smem), (stream)>>>(__VA_ARGS__);          \
    ::es::count_launch();                                                \
    int _st = ::es::check_launch();                                      \
    if (_st != ES_OK) return _st;                                        \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

constexpr int kSMs = 148;
constexpr int kMaxAttrDevices = 64;  // devices whose once-per-device kernel attributes are tracked

// Up to four device ranges of 32-bit words that a kernel clears for the
// launches after it: folds a cudaMemsetAsync (an API call and a device
// operation of its own) into a launch that is already there.
struct ZeroSpans {
  uint32_t* p[4];
  int64_t words[4];
};

inline ZeroSpans no_zero_spans() {
  ZeroSpans z;
  for (int i = 0; i < 4; ++i) {
    z.p[i] = nullptr;
    z.words[i] = 0;
  }
  return z;
}

// Adds a range (nothing for nwords <= 0); false when all four are taken.
inline bool add_zero_span(ZeroSpans& z, void* ptr, int64_t nwords) {
  if (nwords <= 0) return true;
  for (int i = 0; i < 4; ++i)
    if (!z.p[i]) {
      z.p[i] = static_cast<uint32_t*>(ptr);
      z.words[i] = nwords;
      return true;
    }
  return false;
}

__device__ __forceinline__ void zero_spans(const ZeroSpans& z) {
  const int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t nt = static_cast<int64_t>(gridDim.x) * blockDim.x;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (z.p[i])
      for (int64_t j = t; j < z.words[i]; j += nt) z.p[i][j] = 0u;
}

inline int grid_for(int64_t n, int threads, int64_t cap = 148LL * 32) {
  int64_t g = (n + threads - 1) / threads;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return static_cast<int>(g);
}

// Bump allocator over a caller-owned workspace, 256-byte aligned slices.
struct Carver {
  char* base;
  size_t cap;
  size_t used = 0;
  bool overflow = false;
  Carver(void* b, size_t c) : base(static_cast<char*>(b)), cap(c) {}
  template <typename T>
  T* take(int64_t count) {
    size_t bytes = static_cast<size_t>(count > 0 ? count : 1) * sizeof(T);
    size_t off = (used + 255) & ~static_cast<size_t>(255);
    used = off + bytes;
    if (used > cap || base == nullptr) {
      overflow = true;
      return nullptr;
    }
    return reinterpret_cast<T*>(base + off);
  }
};

// Size-only twin of Carver, used by the *_workspace_size queries.
struct Sizer {
  size_t used = 0;
  template <typename T>
  void take(int64_t count) {
    size_t bytes = static_cast<size_t>(count > 0 ? count : 1) * sizeof(T);
    used = ((used + 255) & ~static_cast<size_t>(255)) + bytes;
  }
};

inline int bit_length(uint64_t v) {
  int b = 0;
  while (v) {
    ++b;
    v >>= 1;
  }
  return b;
}

// ---- value loads / stores by runtime dtype -------------------------------
__device__ __forceinline__ float load_as_f32(const void* p, int dtype, int64_t i) {
  if (dtype == ES_F32) return static_cast<const float*>(p)[i];
  if (dtype == ES_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return static_cast<float>(static_cast<const double*>(p)[i]);
}

__device__ __forceinline__ bool is_nonzero(const void* p, int dtype, int64_t i) {
  if (dtype == ES_F32) return static_cast<const float*>(p)[i] != 0.0f;
  if (dtype == ES_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]) != 0.0f;
  return static_cast<const double*>(p)[i] != 0.0;
}

inline int dtype_size(int dtype) {
  switch (dtype) {
    case ES_F32: return 4;
    case ES_BF16: return 2;
    case ES_F64: return 8;
    case ES_I32: return 4;
    case ES_I64: return 8;
    default: return 0;
  }
}

}  // namespace es
