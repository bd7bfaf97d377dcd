// Coordinate join of two tile-COO relations on tile-coordinate keys.
//
// Reproduces coordinate_join (execution/sparse_dispatch.py:29-82) including
// its pair order: for each RHS tile j in order, every LHS tile with an equal
// key in ascending LHS index. Plan: the join columns of each LHS tile are
// packed into one integer key (mixed radix over the key extents) and stably
// radix-sorted with the LHS index as payload, so every key group lists its
// LHS tiles in ascending order; each RHS tile binary-searches its group and
// the group sizes are prefix-summed into pair offsets. Fill: one thread per
// output pair finds its RHS tile by binary search over the offsets
// (load-balanced however skewed the groups are) and writes (i, j).
#include <cmath>
#include <mutex>

#include "common.cuh"
#include "radix_sort.cuh"
#include "scan.cuh"

namespace es {

struct JoinKeys {
  int nkeys;
  int lhs_nd, rhs_nd;
  int ld[ES_MAX_DIMS];
  int rd[ES_MAX_DIMS];
  int64_t ext[ES_MAX_DIMS];
};

struct JoinHeader {
  int32_t sorted_in_alt;
};

struct JoinWs {
  JoinHeader* hdr;
  uint64_t* keys;
  uint32_t* idx;
  RadixBuffers<uint64_t> rb;
  int64_t* counts;  // per rhs tile, scanned in place into offsets
  uint32_t* lo;
  int64_t* scan;
};

template <typename C>
static void join_layout(C& c, JoinWs& w, int64_t n_l, int64_t n_r) {
  w.hdr = c.template take<JoinHeader>(1);
  w.keys = c.template take<uint64_t>(n_l);
  w.idx = c.template take<uint32_t>(n_l);
  w.rb.keys_alt = c.template take<uint64_t>(n_l);
  w.rb.vals_alt = c.template take<uint32_t>(n_l);
  w.rb.hist = c.template take<uint32_t>(RadixScratchSize::hist_elems(n_l));
  w.rb.scan = c.template take<uint32_t>(RadixScratchSize::scan_elems(n_l));
  w.counts = c.template take<int64_t>(n_r);
  w.lo = c.template take<uint32_t>(n_r);
  w.scan = c.template take<int64_t>(scan_scratch_elems(n_r));
}

struct JoinSizer {
  Sizer s;
  template <typename T>
  T* take(int64_t n) {
    s.take<T>(n);
    return nullptr;
  }
};

__global__ void join_flag_kernel(JoinHeader* h, int32_t v) {
  if (threadIdx.x == 0 && blockIdx.x == 0) h->sorted_in_alt = v;
}

__device__ __forceinline__ bool pack_key(const int32_t* row, const int* dims, const JoinKeys& jk, uint64_t* out) {
  uint64_t k = 0;
  bool ok = true;
  for (int q = 0; q < jk.nkeys; ++q) {
    int64_t c = row[dims[q]];
    if (c < 0 || c >= jk.ext[q]) ok = false;
    k = k * static_cast<uint64_t>(jk.ext[q]) + static_cast<uint64_t>(c);
  }
  *out = k;
  return ok;
}

__global__ void join_lhs_keys_kernel(const int32_t* __restrict__ coords, int64_t n, JoinKeys jk,
                                     uint64_t* __restrict__ keys, uint32_t* __restrict__ idx, int32_t* err) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    uint64_t k;
    if (!pack_key(coords + i * jk.lhs_nd, jk.ld, jk, &k) && err) atomicExch(err, ES_ERR_INDEX);
    keys[i] = k;
    idx[i] = static_cast<uint32_t>(i);
  }
}

__global__ void join_count_kernel(const JoinHeader* hdr, const uint64_t* k0, const uint64_t* k1, int64_t n_l,
                                  const int32_t* __restrict__ rcoords, int64_t n_r, JoinKeys jk,
                                  int64_t* __restrict__ counts, uint32_t* __restrict__ lo_out, int32_t* err) {
  const uint64_t* keys = hdr->sorted_in_alt ? k1 : k0;
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n_r; j += (int64_t)gridDim.x * blockDim.x) {
    uint64_t k;
    if (!pack_key(rcoords + j * jk.rhs_nd, jk.rd, jk, &k)) {
      if (err) atomicExch(err, ES_ERR_INDEX);
      counts[j] = 0;
      lo_out[j] = 0;
      continue;
    }
    int64_t lo = 0, hi = n_l;  // lower_bound
    while (lo < hi) {
      int64_t mid = (lo + hi) >> 1;
      if (keys[mid] < k) lo = mid + 1; else hi = mid;
    }
    int64_t a = lo;
    hi = n_l;  // upper_bound
    while (lo < hi) {
      int64_t mid = (lo + hi) >> 1;
      if (keys[mid] <= k) lo = mid + 1; else hi = mid;
    }
    counts[j] = lo - a;
    lo_out[j] = static_cast<uint32_t>(a);
  }
}

template <typename IdxT>
__global__ void join_fill_kernel(const JoinHeader* hdr, const uint32_t* i0, const uint32_t* i1,
                                 const int64_t* __restrict__ offsets, const uint32_t* __restrict__ lo, int64_t n_r,
                                 int64_t P, IdxT* __restrict__ li, IdxT* __restrict__ ri) {
  const uint32_t* sidx = hdr->sorted_in_alt ? i1 : i0;
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < P; p += (int64_t)gridDim.x * blockDim.x) {
    int64_t a = 0, b = n_r;  // last j with offsets[j] <= p
    while (b - a > 1) {
      int64_t m = (a + b) >> 1;
      if (offsets[m] <= p) a = m; else b = m;
    }
    const int64_t j = a;
    li[p] = static_cast<IdxT>(sidx[lo[j] + (p - offsets[j])]);
    ri[p] = static_cast<IdxT>(j);
  }
}

template <typename IdxT>
__global__ void cross_fill_kernel(int64_t n_r, int64_t P, IdxT* __restrict__ li, IdxT* __restrict__ ri) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < P; p += (int64_t)gridDim.x * blockDim.x) {
    li[p] = static_cast<IdxT>(p / n_r);
    ri[p] = static_cast<IdxT>(p % n_r);
  }
}

__global__ void write_i64_kernel(int64_t* p, int64_t v) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *p = v;
}

}  // namespace es

using namespace es;

extern "C" size_t es_join_workspace_size(int64_t n_lhs, int64_t n_rhs) {
  JoinSizer s;
  JoinWs w;
  join_layout(s, w, n_lhs, n_rhs);
  return s.s.used + 256;
}

extern "C" int es_join_plan(const int32_t* lhs_coords, int64_t n_lhs, int lhs_ndim, const int32_t* rhs_coords,
                            int64_t n_rhs, int rhs_ndim, const int32_t* join_keys, int nkeys,
                            const int64_t* key_extents, void* workspace, size_t workspace_bytes,
                            int64_t* num_pairs_dev, int32_t* error_dev, void* stream) {
  cudaStream_t st = as_stream(stream);
  if (n_lhs < 0 || n_rhs < 0 || nkeys < 0 || nkeys > ES_MAX_DIMS) return ES_ERR_INVALID;
  if (n_lhs >= (int64_t)UINT32_MAX || n_rhs >= (int64_t)UINT32_MAX) return ES_ERR_UNSUPPORTED;
  if (nkeys == 0) {
    ES_LAUNCH(write_i64_kernel, 1, 32, 0, st, num_pairs_dev, n_lhs * n_rhs);
    return ES_OK;
  }
  if (n_lhs == 0 || n_rhs == 0) {
    ES_LAUNCH(write_i64_kernel, 1, 32, 0, st, num_pairs_dev, (int64_t)0);
    return ES_OK;
  }
  JoinKeys jk;
  jk.nkeys = nkeys;
  jk.lhs_nd = lhs_ndim;
  jk.rhs_nd = rhs_ndim;
  double bits_f = 0;
  uint64_t prod = 1;
  for (int q = 0; q < nkeys; ++q) {
    jk.ld[q] = join_keys[2 * q];
    jk.rd[q] = join_keys[2 * q + 1];
    jk.ext[q] = key_extents[q];
    if (jk.ld[q] < 0 || jk.ld[q] >= lhs_ndim || jk.rd[q] < 0 || jk.rd[q] >= rhs_ndim) return ES_ERR_INVALID;
    if (key_extents[q] <= 0) return ES_ERR_INVALID;
    bits_f += std::log2(static_cast<double>(key_extents[q]));
    if (bits_f > 62) return ES_ERR_UNSUPPORTED;
    prod *= static_cast<uint64_t>(key_extents[q]);
  }
  const int bits = bit_length(prod - 1);
  JoinWs w;
  Carver c(workspace, workspace_bytes);
  join_layout(c, w, n_lhs, n_rhs);
  if (c.overflow) return ES_ERR_WORKSPACE;
  ES_LAUNCH(join_lhs_keys_kernel, grid_for(n_lhs, 256), 256, 0, st, lhs_coords, n_lhs, jk, w.keys, w.idx, error_dev);
  uint64_t* k = w.keys;
  uint32_t* v = w.idx;
  ES_TRY(radix_sort_pairs<uint64_t>(&k, &v, w.rb, n_lhs, 0, bits, st, error_dev));
  ES_LAUNCH(join_flag_kernel, 1, 32, 0, st, w.hdr, k != w.keys ? 1 : 0);
  ES_LAUNCH(join_count_kernel, grid_for(n_rhs, 256), 256, 0, st, w.hdr, w.keys, w.rb.keys_alt, n_lhs, rhs_coords,
            n_rhs, jk, w.counts, w.lo, error_dev);
  ES_TRY(exclusive_scan<int64_t>(w.counts, w.counts, n_rhs, num_pairs_dev, w.scan, st));
  return ES_OK;
}

extern "C" int es_join_fill(int64_t n_lhs, int64_t n_rhs, int nkeys, void* workspace, size_t workspace_bytes,
                            int64_t num_pairs, void* lhs_idx_out, void* rhs_idx_out, int index_dtype, void* stream) {
  cudaStream_t st = as_stream(stream);
  if (num_pairs <= 0) return ES_OK;
  if (index_dtype != ES_I32 && index_dtype != ES_I64) return ES_ERR_UNSUPPORTED;
  if (index_dtype == ES_I32 && (n_lhs > INT32_MAX || n_rhs > INT32_MAX)) return ES_ERR_UNSUPPORTED;
  const int grid = grid_for(num_pairs, 256);
  if (nkeys == 0) {
    if (index_dtype == ES_I32)
      ES_LAUNCH(cross_fill_kernel<int32_t>, grid, 256, 0, st, n_rhs, num_pairs, (int32_t*)lhs_idx_out,
                (int32_t*)rhs_idx_out);
    else
      ES_LAUNCH(cross_fill_kernel<int64_t>, grid, 256, 0, st, n_rhs, num_pairs, (int64_t*)lhs_idx_out,
                (int64_t*)rhs_idx_out);
    return ES_OK;
  }
  JoinWs w;
  Carver c(workspace, workspace_bytes);
  join_layout(c, w, n_lhs, n_rhs);
  if (c.overflow) return ES_ERR_WORKSPACE;
  if (index_dtype == ES_I32)
    ES_LAUNCH(join_fill_kernel<int32_t>, grid, 256, 0, st, w.hdr, w.idx, w.rb.vals_alt, w.counts, w.lo, n_rhs,
              num_pairs, (int32_t*)lhs_idx_out, (int32_t*)rhs_idx_out);
  else
    ES_LAUNCH(join_fill_kernel<int64_t>, grid, 256, 0, st, w.hdr, w.idx, w.rb.vals_alt, w.counts, w.lo, n_rhs,
              num_pairs, (int64_t*)lhs_idx_out, (int64_t*)rhs_idx_out);
  return ES_OK;
}

// ---------------------------------------------------------------------------
// es_join_static: the coordinate join without any allocation.
//
// Some callers cannot allocate device memory at the moment they join: code
// running inside a host callback or a custom allocator hook, an engine that
// hands out all device memory up front and forbids cudaMalloc afterwards, or
// a plugin whose host framework owns every buffer. For them this entry point
// takes the join's scratch (sort keys, sort buffers, per-RHS counts) from a
// fixed array in the library's own device memory instead of a workspace. The
// caller still provides the outputs (pair index arrays with a capacity) and
// the device int64 that receives the pair count; nothing is synchronised,
// so the count can be read whenever the caller next waits on the stream.
//
// Limits and sharing: at most kStaticMaxTiles tiles on each side (larger
// inputs are refused with ES_ERR_UNSUPPORTED). The array lives once per GPU
// that loads the library, for the life of the process, and every call on
// that GPU uses the same bytes: two calls whose kernels overlap on the GPU
// (different streams, no ordering between them) race and corrupt each
// other; serialise them. Each call rewrites everything it reads from the
// array, so leftovers from an earlier call cannot leak into a result.
// The first call on a device looks up the array's device address with
// cudaGetSymbolAddress (once per device, with that device current); make
// that first call before any stream capture.

namespace es {
namespace {

constexpr int64_t kStaticMaxTiles = 65536;
constexpr size_t kStaticScratchBytes = 3u << 20;
static __device__ __align__(256) unsigned char g_join_scratch[kStaticScratchBytes];

// Identity of the current device's primary context. A context that is torn
// down and made again (cudaDeviceReset, then any runtime call) gets a new
// identity, so an address looked up in the old one is never reused. The
// driver's cuCtxGetCurrent / cuCtxGetId come through the runtime's entry-point
// query (no link against the driver library); 0 when they are unavailable.
unsigned long long current_context_id() {
  typedef int (*GetCurrentFn)(void**);
  typedef int (*GetIdFn)(void*, unsigned long long*);
  static GetCurrentFn get_current = nullptr;
  static GetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrentFn>(f);
    f = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &f, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetIdFn>(f);
  });
  void* ctx = nullptr;
  unsigned long long id = 0;
  if (get_current && get_id && get_current(&ctx) == 0 && ctx && get_id(ctx, &id) == 0) return id;
  return 0;
}

// Device address of g_join_scratch in the current device's context, looked up
// with cudaGetSymbolAddress once per (device, context) and kept. Without a
// context identity (no context current yet, or the driver query missing) the
// address is looked up on every call.
void* static_scratch_ptr(int* status) {
  constexpr int kMaxDevices = 64;
  static void* ptrs[kMaxDevices] = {nullptr};
  static unsigned long long ctx_ids[kMaxDevices] = {0};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *status = ES_ERR_CUDA;
    return nullptr;
  }
  const unsigned long long ctx = current_context_id();
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev] || ctx == 0 || ctx_ids[dev] != ctx) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_join_scratch) != cudaSuccess || !p) {
      ptrs[dev] = nullptr;
      *status = ES_ERR_CUDA;
      return nullptr;
    }
    ptrs[dev] = p;
    ctx_ids[dev] = ctx;
  }
  *status = ES_OK;
  return ptrs[dev];
}

// Fill from the device-side pair count, writing at most `capacity` pairs.
template <typename IdxT>
__global__ void join_fill_capped_kernel(const JoinHeader* hdr, const uint32_t* i0, const uint32_t* i1,
                                        const int64_t* __restrict__ offsets, const uint32_t* __restrict__ lo,
                                        int64_t n_r, const int64_t* __restrict__ num_pairs, int64_t capacity,
                                        IdxT* __restrict__ li, IdxT* __restrict__ ri, int32_t* err) {
  const int64_t P = *num_pairs;
  if (P > capacity && err && blockIdx.x == 0 && threadIdx.x == 0) atomicExch(err, ES_ERR_WORKSPACE);
  const int64_t n = P < capacity ? P : capacity;
  const uint32_t* sidx = hdr->sorted_in_alt ? i1 : i0;
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < n; p += (int64_t)gridDim.x * blockDim.x) {
    int64_t a = 0, b = n_r;
    while (b - a > 1) {
      const int64_t m = (a + b) >> 1;
      if (offsets[m] <= p) a = m; else b = m;
    }
    li[p] = static_cast<IdxT>(sidx[lo[a] + (p - offsets[a])]);
    ri[p] = static_cast<IdxT>(a);
  }
}

template <typename IdxT>
__global__ void cross_fill_capped_kernel(int64_t n_r, int64_t P, int64_t capacity, IdxT* __restrict__ li,
                                         IdxT* __restrict__ ri, int32_t* err) {
  if (P > capacity && err && blockIdx.x == 0 && threadIdx.x == 0) atomicExch(err, ES_ERR_WORKSPACE);
  const int64_t n = P < capacity ? P : capacity;
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < n; p += (int64_t)gridDim.x * blockDim.x) {
    li[p] = static_cast<IdxT>(p / n_r);
    ri[p] = static_cast<IdxT>(p % n_r);
  }
}

}  // namespace
}  // namespace es

extern "C" int es_join_static(const int32_t* lhs_coords, int64_t n_lhs, int lhs_ndim, const int32_t* rhs_coords,
                              int64_t n_rhs, int rhs_ndim, const int32_t* join_keys, int nkeys,
                              const int64_t* key_extents, void* lhs_idx_out, void* rhs_idx_out, int index_dtype,
                              int64_t capacity, int64_t* num_pairs_dev, int32_t* error_dev, void* stream) {
  cudaStream_t st = as_stream(stream);
  if (n_lhs < 0 || n_rhs < 0 || nkeys < 0 || nkeys > ES_MAX_DIMS || capacity < 0) return ES_ERR_INVALID;
  if (index_dtype != ES_I32 && index_dtype != ES_I64) return ES_ERR_UNSUPPORTED;
  if (n_lhs > kStaticMaxTiles || n_rhs > kStaticMaxTiles) return ES_ERR_UNSUPPORTED;
  int status = ES_OK;
  void* scratch = static_scratch_ptr(&status);
  if (status != ES_OK) return status;
  if (nkeys == 0 || n_lhs == 0 || n_rhs == 0) {
    const int64_t P = nkeys == 0 ? n_lhs * n_rhs : 0;
    ES_LAUNCH(write_i64_kernel, 1, 32, 0, st, num_pairs_dev, P);
    if (P > 0) {
      const int grid = grid_for(P < capacity ? P : capacity, 256);
      if (index_dtype == ES_I32)
        ES_LAUNCH(cross_fill_capped_kernel<int32_t>, grid, 256, 0, st, n_rhs, P, capacity, (int32_t*)lhs_idx_out,
                  (int32_t*)rhs_idx_out, error_dev);
      else
        ES_LAUNCH(cross_fill_capped_kernel<int64_t>, grid, 256, 0, st, n_rhs, P, capacity, (int64_t*)lhs_idx_out,
                  (int64_t*)rhs_idx_out, error_dev);
    }
    return ES_OK;
  }
  JoinKeys jk;
  jk.nkeys = nkeys;
  jk.lhs_nd = lhs_ndim;
  jk.rhs_nd = rhs_ndim;
  double bits_f = 0;
  uint64_t prod = 1;
  for (int q = 0; q < nkeys; ++q) {
    jk.ld[q] = join_keys[2 * q];
    jk.rd[q] = join_keys[2 * q + 1];
    jk.ext[q] = key_extents[q];
    if (jk.ld[q] < 0 || jk.ld[q] >= lhs_ndim || jk.rd[q] < 0 || jk.rd[q] >= rhs_ndim) return ES_ERR_INVALID;
    if (key_extents[q] <= 0) return ES_ERR_INVALID;
    bits_f += std::log2(static_cast<double>(key_extents[q]));
    if (bits_f > 62) return ES_ERR_UNSUPPORTED;
    prod *= static_cast<uint64_t>(key_extents[q]);
  }
  JoinWs w;
  Carver c(scratch, kStaticScratchBytes);
  join_layout(c, w, n_lhs, n_rhs);
  if (c.overflow) return ES_ERR_UNSUPPORTED;
  ES_LAUNCH(join_lhs_keys_kernel, grid_for(n_lhs, 256), 256, 0, st, lhs_coords, n_lhs, jk, w.keys, w.idx, error_dev);
  uint64_t* k = w.keys;
  uint32_t* v = w.idx;
  ES_TRY(radix_sort_pairs<uint64_t>(&k, &v, w.rb, n_lhs, 0, bit_length(prod - 1), st, error_dev));
  ES_LAUNCH(join_flag_kernel, 1, 32, 0, st, w.hdr, k != w.keys ? 1 : 0);
  ES_LAUNCH(join_count_kernel, grid_for(n_rhs, 256), 256, 0, st, w.hdr, w.keys, w.rb.keys_alt, n_lhs, rhs_coords,
            n_rhs, jk, w.counts, w.lo, error_dev);
  ES_TRY(exclusive_scan<int64_t>(w.counts, w.counts, n_rhs, num_pairs_dev, w.scan, st));
  const int grid = 148 * 8;
  if (index_dtype == ES_I32)
    ES_LAUNCH(join_fill_capped_kernel<int32_t>, grid, 256, 0, st, w.hdr, w.idx, w.rb.vals_alt, w.counts, w.lo, n_rhs,
              num_pairs_dev, capacity, (int32_t*)lhs_idx_out, (int32_t*)rhs_idx_out, error_dev);
  else
    ES_LAUNCH(join_fill_capped_kernel<int64_t>, grid, 256, 0, st, w.hdr, w.idx, w.rb.vals_alt, w.counts, w.lo, n_rhs,
              num_pairs_dev, capacity, (int64_t*)lhs_idx_out, (int64_t*)rhs_idx_out, error_dev);
  return ES_OK;
}
