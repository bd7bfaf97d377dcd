// COO ingestion: coalescing repeated coordinates on the device.
//
// The reference takes element COO as it comes (tensor/sparse.py:234-270) and
// its tiling lets the last of repeated coordinates win (NumPy fancy
// assignment, tensor/sparse.py:211-212); scipy's CSR / torch's uncoalesced
// sparse tensors instead add repeated coordinates. es_coo_coalesce makes the
// policy explicit: one entry per distinct non-zero coordinate, in row-major
// coordinate order, holding either the last value in input order or the sum
// of all of them (accumulated in float64, in input order -- the order
// scipy's sum_duplicates and numpy's add.at use, so float64 sums agree bit
// for bit).
//
// Pipeline: a 64-bit row-major element key per non-zero entry (zeros and
// out-of-range entries get the sentinel), one stable radix sort of the keys
// with their input positions, a last-of-run flag per sorted entry, a scan of
// the flags for output slots, and one pass writing coordinates and values.
#include "common.cuh"
#include "radix_sort.cuh"
#include "scan.cuh"

namespace es {

struct CooGeom {
  int ndim;
  int64_t shape[ES_MAX_DIMS];
  int shape_sh[ES_MAX_DIMS];  // log2(shape[d]) for a power of two, else -1
  int64_t total;
};

// x / d: a shift for powers of two, 32-bit division when both fit, else 64-bit.
__device__ __forceinline__ uint64_t coo_udiv(uint64_t x, uint64_t d, int sh) {
  if (sh >= 0) return x >> sh;
  if ((x >> 32) == 0 && (d >> 32) == 0) return static_cast<uint32_t>(x) / static_cast<uint32_t>(d);
  return x / d;
}

struct CoalesceWs {
  uint64_t* keys;
  uint32_t* perm;
  RadixBuffers<uint64_t> rb;
  uint32_t* flags;
  uint32_t* excl;
  uint32_t* scan;
  int32_t* alt;
};

template <typename C>
static void coalesce_layout(C& c, CoalesceWs& w, int64_t nnz) {
  w.keys = c.template take<uint64_t>(nnz);
  w.perm = c.template take<uint32_t>(nnz);
  w.rb.keys_alt = c.template take<uint64_t>(nnz);
  w.rb.vals_alt = c.template take<uint32_t>(nnz);
  w.rb.hist = c.template take<uint32_t>(RadixScratchSize::hist_elems(nnz));
  w.rb.scan = c.template take<uint32_t>(RadixScratchSize::scan_elems(nnz));
  w.flags = c.template take<uint32_t>(nnz);
  w.excl = c.template take<uint32_t>(nnz);
  w.scan = c.template take<uint32_t>(scan_scratch_elems(nnz));
  w.alt = c.template take<int32_t>(1);
}

struct CoalesceSizer {
  Sizer s;
  template <typename T>
  T* take(int64_t k) {
    s.take<T>(k);
    return nullptr;
  }
};

static int make_coo_geom(int ndim, const int64_t* shape, CooGeom* g) {
  if (ndim < 1 || ndim > ES_MAX_DIMS || !shape) return ES_ERR_INVALID;
  g->ndim = ndim;
  g->total = 1;
  for (int d = 0; d < ndim; ++d) {
    if (shape[d] <= 0) return ES_ERR_INVALID;
    if (g->total > (INT64_MAX / 4) / shape[d]) return ES_ERR_UNSUPPORTED;
    g->shape[d] = shape[d];
    g->total *= shape[d];
  }
  for (int d = ndim; d < ES_MAX_DIMS; ++d) g->shape[d] = 1;
  for (int d = 0; d < ES_MAX_DIMS; ++d) {
    const int64_t v = g->shape[d];
    int sh = -1;
    if ((v & (v - 1)) == 0)
      for (sh = 0; (int64_t{1} << sh) != v; ++sh) {
      }
    g->shape_sh[d] = sh;
  }
  return ES_OK;
}

__device__ __forceinline__ double load_as_f64(const void* p, int dtype, int64_t i) {
  if (dtype == ES_F64) return static_cast<const double*>(p)[i];
  return static_cast<double>(load_as_f32(p, dtype, i));
}

__global__ void coalesce_keys_kernel(const int32_t* __restrict__ idx, const void* __restrict__ vals, int vdtype,
                                     int64_t nnz, CooGeom g, uint64_t* __restrict__ keys,
                                     uint32_t* __restrict__ perm, int32_t* err) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < nnz; e += (int64_t)gridDim.x * blockDim.x) {
    uint64_t key = static_cast<uint64_t>(g.total);
    if (is_nonzero(vals, vdtype, e)) {
      uint64_t lin = 0;
      bool ok = true;
      for (int d = 0; d < g.ndim; ++d) {
        const int64_t x = idx[e * g.ndim + d];
        if (x < 0 || x >= g.shape[d]) ok = false;
        lin = lin * static_cast<uint64_t>(g.shape[d]) + static_cast<uint64_t>(x);
      }
      if (ok) {
        key = lin;
      } else if (err) {
        atomicExch(err, ES_ERR_INDEX);
      }
    }
    keys[e] = key;
    perm[e] = static_cast<uint32_t>(e);
  }
}

// flags[s] = 1 where sorted entry s is the last of its coordinate's run;
// counts[1] = number of non-zero entries (the position of the first sentinel).
__global__ void coalesce_flags_kernel(const int32_t* alt, const uint64_t* k0, const uint64_t* k1, int64_t n,
                                      uint64_t sentinel, uint32_t* __restrict__ flags, int64_t* __restrict__ counts) {
  const uint64_t* keys = *alt ? k1 : k0;
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s < n; s += (int64_t)gridDim.x * blockDim.x) {
    const uint64_t k = keys[s];
    const uint64_t nx = s + 1 < n ? keys[s + 1] : sentinel;
    flags[s] = (k != sentinel && nx != k) ? 1u : 0u;
    if (k != sentinel && nx == sentinel) counts[1] = s + 1;
  }
}

template <typename OutT>
__device__ __forceinline__ void store_value(void* out, int64_t i, double v) {
  if constexpr (sizeof(OutT) == 8) {
    static_cast<double*>(out)[i] = v;
  } else if constexpr (sizeof(OutT) == 4) {
    static_cast<float*>(out)[i] = static_cast<float>(v);
  } else {
    static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(static_cast<float>(v));
  }
}

// One thread per last-of-run entry: decode the key into coordinates and write
// the run's value (last in input order, or the float64 sum of the run in input
// order; the stable sort kept a run's entries in input order).
template <typename OutT>
__global__ void coalesce_write_kernel(const int32_t* alt, const uint64_t* k0, const uint64_t* k1, const uint32_t* p0,
                                      const uint32_t* p1, int64_t n, const uint32_t* __restrict__ flags,
                                      const uint32_t* __restrict__ excl, const void* __restrict__ vals, int vdtype,
                                      int policy, CooGeom g, int32_t* __restrict__ idx_out, void* __restrict__ out) {
  const uint64_t* keys = *alt ? k1 : k0;
  const uint32_t* perm = *alt ? p1 : p0;
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s < n; s += (int64_t)gridDim.x * blockDim.x) {
    if (!flags[s]) continue;
    const uint64_t k = keys[s];
    const int64_t o = excl[s];
    uint64_t lin = k;
    for (int d = g.ndim - 1; d >= 0; --d) {
      const uint64_t q = coo_udiv(lin, static_cast<uint64_t>(g.shape[d]), g.shape_sh[d]);
      idx_out[o * g.ndim + d] = static_cast<int32_t>(lin - q * static_cast<uint64_t>(g.shape[d]));
      lin = q;
    }
    double v;
    if (policy == ES_DUP_SUM) {
      int64_t r = s;
      while (r > 0 && keys[r - 1] == k) --r;
      v = 0.0;
      for (int64_t i = r; i <= s; ++i) v += load_as_f64(vals, vdtype, perm[i]);
    } else {
      v = load_as_f64(vals, vdtype, perm[s]);
    }
    store_value<OutT>(out, o, v);
  }
}

}  // namespace es

using namespace es;

extern "C" size_t es_coo_coalesce_workspace_size(int64_t nnz, int ndim, const int64_t* shape) {
  CooGeom g;
  if (make_coo_geom(ndim, shape, &g) != ES_OK || nnz < 0) return 0;
  CoalesceSizer s;
  CoalesceWs w;
  coalesce_layout(s, w, nnz > 0 ? nnz : 1);
  return s.s.used + 256;
}

extern "C" int es_coo_coalesce(const int32_t* indices, const void* values, int values_dtype, int64_t nnz, int ndim,
                               const int64_t* shape, int policy, void* workspace, size_t workspace_bytes,
                               int32_t* indices_out, void* values_out, int out_dtype, int64_t* counts_dev,
                               int32_t* error_dev, void* stream) {
  CooGeom g;
  ES_TRY(make_coo_geom(ndim, shape, &g));
  if (policy != ES_DUP_LAST && policy != ES_DUP_SUM) return ES_ERR_INVALID;
  if (nnz < 0 || nnz >= (int64_t)UINT32_MAX) return ES_ERR_UNSUPPORTED;
  if (values_dtype != ES_F32 && values_dtype != ES_F64 && values_dtype != ES_BF16) return ES_ERR_UNSUPPORTED;
  if (out_dtype != ES_F32 && out_dtype != ES_F64 && out_dtype != ES_BF16) return ES_ERR_UNSUPPORTED;
  cudaStream_t st = as_stream(stream);
  if (cudaMemsetAsync(counts_dev, 0, 2 * sizeof(int64_t), st) != cudaSuccess) return ES_ERR_CUDA;
  if (nnz == 0) return ES_OK;
  CoalesceWs w;
  Carver c(workspace, workspace_bytes);
  coalesce_layout(c, w, nnz);
  if (c.overflow) return ES_ERR_WORKSPACE;
  const uint64_t sentinel = static_cast<uint64_t>(g.total);
  ES_LAUNCH(coalesce_keys_kernel, grid_for(nnz, 256), 256, 0, st, indices, values, values_dtype, nnz, g, w.keys,
            w.perm, error_dev);
  uint64_t* k = w.keys;
  uint32_t* p = w.perm;
  ES_TRY(radix_sort_pairs<uint64_t>(&k, &p, w.rb, nnz, 0, bit_length(sentinel), st, error_dev));
  // non-zero when the sorted data sits in the radix sort's alternate buffers
  if (cudaMemsetAsync(w.alt, k != w.keys ? 1 : 0, sizeof(int32_t), st) != cudaSuccess) return ES_ERR_CUDA;
  ES_LAUNCH(coalesce_flags_kernel, grid_for(nnz, 256), 256, 0, st, w.alt, w.keys, w.rb.keys_alt, nnz, sentinel,
            w.flags, counts_dev);
  // the distinct count (uint32) accumulates into the low word of counts_dev[0]
  ES_TRY(exclusive_scan<uint32_t>(w.flags, w.excl, nnz, reinterpret_cast<uint32_t*>(counts_dev), w.scan, st));
  if (out_dtype == ES_F64) {
    ES_LAUNCH(coalesce_write_kernel<double>, grid_for(nnz, 256), 256, 0, st, w.alt, w.keys, w.rb.keys_alt, w.perm,
              w.rb.vals_alt, nnz, w.flags, w.excl, values, values_dtype, policy, g, indices_out, values_out);
  } else if (out_dtype == ES_F32) {
    ES_LAUNCH(coalesce_write_kernel<float>, grid_for(nnz, 256), 256, 0, st, w.alt, w.keys, w.rb.keys_alt, w.perm,
              w.rb.vals_alt, nnz, w.flags, w.excl, values, values_dtype, policy, g, indices_out, values_out);
  } else {
    ES_LAUNCH(coalesce_write_kernel<__nv_bfloat16>, grid_for(nnz, 256), 256, 0, st, w.alt, w.keys, w.rb.keys_alt,
              w.perm, w.rb.vals_alt, nnz, w.flags, w.excl, values, values_dtype, policy, g, indices_out, values_out);
  }
  return ES_OK;
}
