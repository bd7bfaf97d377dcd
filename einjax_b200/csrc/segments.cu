// Output-tile grouping, standalone segment-sum and deterministic scatter-add.
//
// Grouping follows _compute_output_coords + segment_sum
// (execution/sparse_dispatch.py:174-223, 129-171): each pair's output tile
// coordinate is packed into one integer (mixed radix over the output grid,
// so integer order == lexicographic coordinate order, as `sorted` at :161),
// pairs are stably radix-sorted by it (inside a group they stay in join
// order, the order the reference adds them in at :167-169) and group heads
// are prefix-summed into segment ids.
#include <cmath>

#include <type_traits>

#include "common.cuh"
#include "radix_sort.cuh"
#include "scan.cuh"

namespace es {

struct AggKeys {
  int out_nd, lhs_nd, rhs_nd;
  int src[ES_MAX_DIMS];
  int dim[ES_MAX_DIMS];
  int64_t ext[ES_MAX_DIMS];
};

struct SegHeader {
  int32_t sorted_in_alt;
};

struct SegWs {
  SegHeader* hdr;
  uint64_t* keys;
  uint32_t* perm;
  RadixBuffers<uint64_t> rb;
  uint32_t* flags;
  uint32_t* excl;
  uint32_t* scan;
  int64_t* seg_off;  // used by segsum / scatter-add
  int64_t* nseg;
};

template <typename C>
static void seg_layout(C& c, SegWs& w, int64_t n) {
  w.hdr = c.template take<SegHeader>(1);
  w.keys = c.template take<uint64_t>(n);
  w.perm = c.template take<uint32_t>(n);
  w.rb.keys_alt = c.template take<uint64_t>(n);
  w.rb.vals_alt = c.template take<uint32_t>(n);
  w.rb.hist = c.template take<uint32_t>(RadixScratchSize::hist_elems(n));
  w.rb.scan = c.template take<uint32_t>(RadixScratchSize::scan_elems(n));
  w.flags = c.template take<uint32_t>(n);
  w.excl = c.template take<uint32_t>(n);
  w.scan = c.template take<uint32_t>(scan_scratch_elems(n));
  w.seg_off = c.template take<int64_t>(n + 1);
  w.nseg = c.template take<int64_t>(1);
}

struct SegSizer {
  Sizer s;
  template <typename T>
  T* take(int64_t n) {
    s.take<T>(n);
    return nullptr;
  }
};

__global__ void seg_flag_kernel(SegHeader* h, int32_t v) {
  if (threadIdx.x == 0 && blockIdx.x == 0) h->sorted_in_alt = v;
}

__global__ void pair_out_keys_kernel(const int32_t* __restrict__ lc, const int32_t* __restrict__ rc,
                                     const int32_t* __restrict__ li, const int32_t* __restrict__ ri, int64_t P,
                                     AggKeys ak, uint64_t* __restrict__ keys, uint32_t* __restrict__ perm,
                                     int32_t* err) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < P; p += (int64_t)gridDim.x * blockDim.x) {
    uint64_t k = 0;
    bool ok = true;
    const int64_t a = li[p], b = ri[p];
    for (int d = 0; d < ak.out_nd; ++d) {
      int64_t c = ak.src[d] == 0 ? lc[a * ak.lhs_nd + ak.dim[d]] : rc[b * ak.rhs_nd + ak.dim[d]];
      if (c < 0 || c >= ak.ext[d]) ok = false;
      k = k * static_cast<uint64_t>(ak.ext[d]) + static_cast<uint64_t>(c);
    }
    if (!ok && err) atomicExch(err, ES_ERR_INDEX);
    keys[p] = k;
    perm[p] = static_cast<uint32_t>(p);
  }
}

__global__ void row_keys_kernel(const int32_t* __restrict__ coords, int64_t n, int nd, AggKeys ak,
                                uint64_t* __restrict__ keys, uint32_t* __restrict__ perm, int32_t* err) {
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < n; r += (int64_t)gridDim.x * blockDim.x) {
    uint64_t k = 0;
    bool ok = true;
    for (int d = 0; d < nd; ++d) {
      int64_t c = coords[r * nd + d];
      if (c < 0 || c >= ak.ext[d]) ok = false;
      k = k * static_cast<uint64_t>(ak.ext[d]) + static_cast<uint64_t>(c);
    }
    if (!ok && err) atomicExch(err, ES_ERR_INDEX);
    keys[r] = k;
    perm[r] = static_cast<uint32_t>(r);
  }
}

__global__ void heads_kernel(const SegHeader* hdr, const uint64_t* k0, const uint64_t* k1, int64_t n,
                             uint32_t* __restrict__ flags) {
  const uint64_t* keys = hdr->sorted_in_alt ? k1 : k0;
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s < n; s += (int64_t)gridDim.x * blockDim.x)
    flags[s] = (s == 0 || keys[s] != keys[s - 1]) ? 1u : 0u;
}

// Segment offsets and (optionally) decoded unique coordinates.
__global__ void seg_offsets_kernel(const SegHeader* hdr, const uint64_t* k0, const uint64_t* k1, int64_t n,
                                   const uint32_t* __restrict__ flags, const uint32_t* __restrict__ excl,
                                   AggKeys ak, int32_t* __restrict__ out_coords, int64_t* __restrict__ seg_off,
                                   int64_t* nseg) {
  const uint64_t* keys = hdr->sorted_in_alt ? k1 : k0;
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s < n; s += (int64_t)gridDim.x * blockDim.x) {
    if (flags[s]) {
      const int64_t sid = excl[s];
      seg_off[sid] = s;
      if (out_coords) {
        uint64_t k = keys[s];
        for (int d = ak.out_nd - 1; d >= 0; --d) {
          out_coords[sid * ak.out_nd + d] = static_cast<int32_t>(k % static_cast<uint64_t>(ak.ext[d]));
          k /= static_cast<uint64_t>(ak.ext[d]);
        }
      }
    }
    if (s == n - 1) {
      const int64_t total = static_cast<int64_t>(excl[s]) + flags[s];
      seg_off[total] = n;
      if (nseg) *nseg = total;
    }
  }
}

// Strip key of each segment: its output key with the trailing
// (out_nd - strip_dims) coordinates divided out, i.e. the packed leading
// strip_dims output coordinates. Non-decreasing in segment order.
__global__ void seg_strip_kernel(const SegHeader* hdr, const uint64_t* k0, const uint64_t* k1, int64_t n,
                                 const uint32_t* __restrict__ flags, const uint32_t* __restrict__ excl,
                                 uint64_t divisor, int64_t* __restrict__ strip) {
  const uint64_t* keys = hdr->sorted_in_alt ? k1 : k0;
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s < n; s += (int64_t)gridDim.x * blockDim.x)
    if (flags[s]) strip[excl[s]] = static_cast<int64_t>(keys[s] / divisor);
}

__global__ void gather_pairs_kernel(const SegHeader* hdr, const uint32_t* p0, const uint32_t* p1, int64_t n,
                                    const int32_t* __restrict__ li, const int32_t* __restrict__ ri,
                                    int32_t* __restrict__ sli, int32_t* __restrict__ sri, int32_t* __restrict__ spi) {
  const uint32_t* perm = hdr->sorted_in_alt ? p1 : p0;
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s < n; s += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t p = perm[s];
    if (sli) sli[s] = li[p];
    if (sri) sri[s] = ri[p];
    if (spi) spi[s] = static_cast<int32_t>(p);
  }
}

// Sum rows of each segment in sorted (== original) order. One CTA per segment
// (grid-stride over segments, bound read on device); threads stride the row.
template <typename OutT>
__global__ void segment_reduce_kernel(const SegHeader* hdr, const uint32_t* p0, const uint32_t* p1,
                                      const int64_t* __restrict__ seg_off, const int64_t* __restrict__ nseg,
                                      const void* __restrict__ vals, int vdtype, int64_t te,
                                      const uint64_t* k0, const uint64_t* k1, int add_into_key_row,
                                      OutT* __restrict__ out) {
  const uint32_t* perm = hdr->sorted_in_alt ? p1 : p0;
  const uint64_t* keys = hdr->sorted_in_alt ? k1 : k0;
  const int64_t ns = *nseg;
  for (int64_t sg = blockIdx.x; sg < ns; sg += gridDim.x) {
    const int64_t a = seg_off[sg], b = seg_off[sg + 1];
    const int64_t orow = add_into_key_row ? static_cast<int64_t>(keys[a]) : sg;
    for (int64_t e = threadIdx.x; e < te; e += blockDim.x) {
      float acc = 0.f;
      for (int64_t s = a; s < b; ++s) acc += load_as_f32(vals, vdtype, static_cast<int64_t>(perm[s]) * te + e);
      if (add_into_key_row) {
        out[orow * te + e] = static_cast<OutT>(static_cast<float>(out[orow * te + e]) + acc);
      } else {
        out[orow * te + e] = static_cast<OutT>(acc);
      }
    }
  }
}

template <>
__global__ void segment_reduce_kernel<__nv_bfloat16>(const SegHeader* hdr, const uint32_t* p0, const uint32_t* p1,
                                                     const int64_t* __restrict__ seg_off,
                                                     const int64_t* __restrict__ nseg, const void* __restrict__ vals,
                                                     int vdtype, int64_t te, const uint64_t* k0, const uint64_t* k1,
                                                     int add_into_key_row, __nv_bfloat16* __restrict__ out) {
  const uint32_t* perm = hdr->sorted_in_alt ? p1 : p0;
  const int64_t ns = *nseg;
  for (int64_t sg = blockIdx.x; sg < ns; sg += gridDim.x) {
    const int64_t a = seg_off[sg], b = seg_off[sg + 1];
    for (int64_t e = threadIdx.x; e < te; e += blockDim.x) {
      float acc = 0.f;
      for (int64_t s = a; s < b; ++s) acc += load_as_f32(vals, vdtype, static_cast<int64_t>(perm[s]) * te + e);
      out[sg * te + e] = __float2bfloat16_rn(acc);
    }
  }
}

// Vectorised form of segment_reduce_kernel for rows of 4-element groups
// (fp32 rows: 16-byte loads; bf16 rows: 8-byte loads). Each thread owns one
// 4-element column group of the tile and walks the segment's rows with
// kSegRowU independent loads in flight; the adds stay in row order, so the
// sums are bit-identical to the scalar kernel's.
constexpr int kSegRowU = 8;

__device__ __forceinline__ float4 load4_f32(const void* v, int64_t i) {
  return __ldcs(reinterpret_cast<const float4*>(static_cast<const float*>(v) + i));
}

__device__ __forceinline__ float4 load4_bf16(const void* v, int64_t i) {
  const uint2 u = __ldcs(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(v) + i));
  float4 f;
  f.x = __uint_as_float(u.x << 16);
  f.y = __uint_as_float(u.x & 0xFFFF0000u);
  f.z = __uint_as_float(u.y << 16);
  f.w = __uint_as_float(u.y & 0xFFFF0000u);
  return f;
}

template <bool BF16_IN, typename OutT>
__global__ void segment_reduce_vec_kernel(const SegHeader* hdr, const uint32_t* p0, const uint32_t* p1,
                                          const int64_t* __restrict__ seg_off, const int64_t* __restrict__ nseg,
                                          const void* __restrict__ vals, int64_t te, const uint64_t* k0,
                                          const uint64_t* k1, int add_into_key_row, OutT* __restrict__ out) {
  const uint32_t* perm = hdr->sorted_in_alt ? p1 : p0;
  const uint64_t* keys = hdr->sorted_in_alt ? k1 : k0;
  const int64_t ns = *nseg;
  const int64_t nv = te >> 2;
  for (int64_t sg = blockIdx.x; sg < ns; sg += gridDim.x) {
    const int64_t a = seg_off[sg], b = seg_off[sg + 1];
    const int64_t orow = add_into_key_row ? static_cast<int64_t>(keys[a]) : sg;
    for (int64_t v = threadIdx.x; v < nv; v += blockDim.x) {
      const int64_t col = v << 2;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      int64_t s = a;
      for (; s + kSegRowU <= b; s += kSegRowU) {
        float4 x[kSegRowU];
#pragma unroll
        for (int u = 0; u < kSegRowU; ++u) {
          const int64_t r = static_cast<int64_t>(perm[s + u]) * te + col;
          x[u] = BF16_IN ? load4_bf16(vals, r) : load4_f32(vals, r);
        }
#pragma unroll
        for (int u = 0; u < kSegRowU; ++u) {
          acc.x += x[u].x;
          acc.y += x[u].y;
          acc.z += x[u].z;
          acc.w += x[u].w;
        }
      }
      for (; s < b; ++s) {
        const int64_t r = static_cast<int64_t>(perm[s]) * te + col;
        const float4 x = BF16_IN ? load4_bf16(vals, r) : load4_f32(vals, r);
        acc.x += x.x;
        acc.y += x.y;
        acc.z += x.z;
        acc.w += x.w;
      }
      OutT* o = out + orow * te + col;
      if (add_into_key_row) {
        o[0] = static_cast<OutT>(static_cast<float>(o[0]) + acc.x);
        o[1] = static_cast<OutT>(static_cast<float>(o[1]) + acc.y);
        o[2] = static_cast<OutT>(static_cast<float>(o[2]) + acc.z);
        o[3] = static_cast<OutT>(static_cast<float>(o[3]) + acc.w);
      } else if constexpr (std::is_same<OutT, float>::value) {
        *reinterpret_cast<float4*>(o) = acc;
      } else {
        o[0] = __float2bfloat16_rn(acc.x);
        o[1] = __float2bfloat16_rn(acc.y);
        o[2] = __float2bfloat16_rn(acc.z);
        o[3] = __float2bfloat16_rn(acc.w);
      }
    }
  }
}

// Launches the vectorised reduce when every row starts on a 4-element group
// (tile_elems % 4 == 0, 16-byte aligned buffers), else the scalar one.
template <typename OutT>
static int launch_segment_reduce(const SegWs& w, const void* values, int vdtype, int64_t te, int64_t num_segments,
                                 int add_into_key_row, OutT* out, cudaStream_t st) {
  const int64_t g = num_segments < 148 * 8 ? num_segments : 148 * 8;
  const int grid = static_cast<int>(g > 0 ? g : 1);
  const bool aligned = (reinterpret_cast<uintptr_t>(values) & 15u) == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
  if (te % 4 == 0 && aligned && (vdtype == ES_F32 || vdtype == ES_BF16)) {
    const int64_t nv = te / 4;
    const int threads = nv >= 256 ? 256 : (nv >= 128 ? 128 : (nv >= 64 ? 64 : 32));
    if (vdtype == ES_F32)
      ES_LAUNCH((segment_reduce_vec_kernel<false, OutT>), grid, threads, 0, st, w.hdr, w.perm, w.rb.vals_alt,
                w.seg_off, w.nseg, values, te, w.keys, w.rb.keys_alt, add_into_key_row, out);
    else
      ES_LAUNCH((segment_reduce_vec_kernel<true, OutT>), grid, threads, 0, st, w.hdr, w.perm, w.rb.vals_alt,
                w.seg_off, w.nseg, values, te, w.keys, w.rb.keys_alt, add_into_key_row, out);
    return ES_OK;
  }
  const int threads = te >= 256 ? 256 : (te >= 64 ? 64 : 32);
  ES_LAUNCH(segment_reduce_kernel<OutT>, grid, threads, 0, st, w.hdr, w.perm, w.rb.vals_alt, w.seg_off, w.nseg,
            values, vdtype, te, w.keys, w.rb.keys_alt, add_into_key_row, out);
  return ES_OK;
}

static int make_agg(const int32_t* agg_keys, int out_nd, int lhs_nd, int rhs_nd, const int64_t* ext, AggKeys* ak,
                    int* bits) {
  if (out_nd < 1 || out_nd > ES_MAX_DIMS) return ES_ERR_INVALID;
  ak->out_nd = out_nd;
  ak->lhs_nd = lhs_nd;
  ak->rhs_nd = rhs_nd;
  double bf = 0;
  uint64_t prod = 1;
  for (int d = 0; d < out_nd; ++d) {
    if (agg_keys) {
      ak->src[d] = agg_keys[2 * d];
      ak->dim[d] = agg_keys[2 * d + 1];
      const int nd = ak->src[d] == 0 ? lhs_nd : rhs_nd;
      if ((ak->src[d] != 0 && ak->src[d] != 1) || ak->dim[d] < 0 || ak->dim[d] >= nd) return ES_ERR_INVALID;
    } else {
      ak->src[d] = 0;
      ak->dim[d] = d;
    }
    if (ext[d] <= 0) return ES_ERR_INVALID;
    ak->ext[d] = ext[d];
    bf += std::log2(static_cast<double>(ext[d]));
    if (bf > 62) return ES_ERR_UNSUPPORTED;
    prod *= static_cast<uint64_t>(ext[d]);
  }
  *bits = bit_length(prod - 1);
  return ES_OK;
}

// Sort keys already in w.keys/w.perm, mark heads, scan them. *count_dev gets
// the number of groups (low 32 bits of an int64 zeroed first); a sort whose
// bounded wait ran out records ES_ERR_TIMEOUT in *err.
static int sort_and_group(SegWs& w, int64_t n, int bits, int64_t* count_dev, int32_t* err, cudaStream_t st) {
  uint64_t* k = w.keys;
  uint32_t* v = w.perm;
  ES_TRY(radix_sort_pairs<uint64_t>(&k, &v, w.rb, n, 0, bits, st, err));
  ES_LAUNCH(seg_flag_kernel, 1, 32, 0, st, w.hdr, k != w.keys ? 1 : 0);
  ES_LAUNCH(heads_kernel, grid_for(n, 256), 256, 0, st, w.hdr, w.keys, w.rb.keys_alt, n, w.flags);
  if (count_dev && cudaMemsetAsync(count_dev, 0, sizeof(int64_t), st) != cudaSuccess) return ES_ERR_CUDA;
  ES_TRY(exclusive_scan<uint32_t>(w.flags, w.excl, n, reinterpret_cast<uint32_t*>(count_dev), w.scan, st));
  return ES_OK;
}

}  // namespace es

using namespace es;

extern "C" size_t es_segments_workspace_size(int64_t num_pairs) {
  SegSizer s;
  SegWs w;
  seg_layout(s, w, num_pairs);
  return s.s.used + 256;
}

extern "C" int es_segments_plan(const int32_t* lhs_coords, int lhs_ndim, const int32_t* rhs_coords, int rhs_ndim,
                                const int32_t* lhs_idx, const int32_t* rhs_idx, int64_t num_pairs,
                                const int32_t* agg_keys, int out_ndim, const int64_t* out_extents, void* workspace,
                                size_t workspace_bytes, int64_t* num_segments_dev, int32_t* error_dev, void* stream) {
  cudaStream_t st = as_stream(stream);
  if (num_pairs < 0 || num_pairs >= (int64_t)UINT32_MAX) return ES_ERR_UNSUPPORTED;
  AggKeys ak;
  int bits = 0;
  ES_TRY(make_agg(agg_keys, out_ndim, lhs_ndim, rhs_ndim, out_extents, &ak, &bits));
  if (num_pairs == 0) {
    if (cudaMemsetAsync(num_segments_dev, 0, sizeof(int64_t), st) != cudaSuccess) return ES_ERR_CUDA;
    return ES_OK;
  }
  SegWs w;
  Carver c(workspace, workspace_bytes);
  seg_layout(c, w, num_pairs);
  if (c.overflow) return ES_ERR_WORKSPACE;
  ES_LAUNCH(pair_out_keys_kernel, grid_for(num_pairs, 256), 256, 0, st, lhs_coords, rhs_coords, lhs_idx, rhs_idx,
            num_pairs, ak, w.keys, w.perm, error_dev);
  return sort_and_group(w, num_pairs, bits, num_segments_dev, error_dev, st);
}

extern "C" int es_segments_fill(const int32_t* lhs_idx, const int32_t* rhs_idx, int64_t num_pairs, int out_ndim,
                                const int64_t* out_extents, void* workspace, size_t workspace_bytes,
                                int64_t num_segments, int32_t* out_coords, int64_t* seg_offsets,
                                int32_t* seg_lhs_idx, int32_t* seg_rhs_idx, int32_t* seg_pair_idx, int strip_dims,
                                int64_t* seg_strip, void* stream) {
  cudaStream_t st = as_stream(stream);
  if (num_pairs <= 0 || num_segments <= 0) return ES_OK;
  AggKeys ak;
  int bits = 0;
  ES_TRY(make_agg(nullptr, out_ndim, out_ndim, out_ndim, out_extents, &ak, &bits));
  SegWs w;
  Carver c(workspace, workspace_bytes);
  seg_layout(c, w, num_pairs);
  if (c.overflow) return ES_ERR_WORKSPACE;
  ES_LAUNCH(seg_offsets_kernel, grid_for(num_pairs, 256), 256, 0, st, w.hdr, w.keys, w.rb.keys_alt, num_pairs, w.flags,
            w.excl, ak, out_coords, seg_offsets, (int64_t*)nullptr);
  ES_LAUNCH(gather_pairs_kernel, grid_for(num_pairs, 256), 256, 0, st, w.hdr, w.perm, w.rb.vals_alt, num_pairs,
            lhs_idx, rhs_idx, seg_lhs_idx, seg_rhs_idx, seg_pair_idx);
  if (seg_strip) {
    if (strip_dims < 0 || strip_dims > out_ndim) return ES_ERR_INVALID;
    uint64_t div = 1;
    for (int d = strip_dims; d < out_ndim; ++d) div *= static_cast<uint64_t>(out_extents[d]);
    ES_LAUNCH(seg_strip_kernel, grid_for(num_pairs, 256), 256, 0, st, w.hdr, w.keys, w.rb.keys_alt, num_pairs, w.flags,
              w.excl, div, seg_strip);
  }
  return ES_OK;
}

__global__ void output_coords_kernel(const int32_t* __restrict__ lc, const int32_t* __restrict__ rc,
                                     const int32_t* __restrict__ li, const int32_t* __restrict__ ri, int64_t P,
                                     AggKeys ak, int32_t* __restrict__ out) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < P; p += (int64_t)gridDim.x * blockDim.x) {
    const int64_t a = li[p], b = ri[p];
    for (int d = 0; d < ak.out_nd; ++d)
      out[p * ak.out_nd + d] = ak.src[d] == 0 ? lc[a * ak.lhs_nd + ak.dim[d]] : rc[b * ak.rhs_nd + ak.dim[d]];
  }
}

extern "C" int es_output_coords(const int32_t* lhs_coords, int lhs_ndim, const int32_t* rhs_coords, int rhs_ndim,
                                const int32_t* lhs_idx, const int32_t* rhs_idx, int64_t num_pairs,
                                const int32_t* agg_keys, int out_ndim, int32_t* out_coords, void* stream) {
  if (num_pairs <= 0) return ES_OK;
  AggKeys ak;
  int bits = 0;
  int64_t ext[ES_MAX_DIMS];
  for (int d = 0; d < ES_MAX_DIMS; ++d) ext[d] = 1;
  ES_TRY(make_agg(agg_keys, out_ndim, lhs_ndim, rhs_ndim, ext, &ak, &bits));
  cudaStream_t st = as_stream(stream);
  ES_LAUNCH(output_coords_kernel, grid_for(num_pairs, 256), 256, 0, st, lhs_coords, rhs_coords, lhs_idx, rhs_idx,
            num_pairs, ak, out_coords);
  return ES_OK;
}

extern "C" size_t es_segsum_workspace_size(int64_t num_rows) { return es_segments_workspace_size(num_rows); }

extern "C" int es_segsum_plan(const int32_t* coords, int64_t num_rows, int nd, const int64_t* extents,
                              void* workspace, size_t workspace_bytes, int64_t* num_segments_dev, int32_t* error_dev,
                              void* stream) {
  cudaStream_t st = as_stream(stream);
  if (num_rows < 0 || num_rows >= (int64_t)UINT32_MAX) return ES_ERR_UNSUPPORTED;
  AggKeys ak;
  int bits = 0;
  ES_TRY(make_agg(nullptr, nd, nd, nd, extents, &ak, &bits));
  if (num_rows == 0) {
    if (cudaMemsetAsync(num_segments_dev, 0, sizeof(int64_t), st) != cudaSuccess) return ES_ERR_CUDA;
    return ES_OK;
  }
  SegWs w;
  Carver c(workspace, workspace_bytes);
  seg_layout(c, w, num_rows);
  if (c.overflow) return ES_ERR_WORKSPACE;
  ES_LAUNCH(row_keys_kernel, grid_for(num_rows, 256), 256, 0, st, coords, num_rows, nd, ak, w.keys, w.perm, error_dev);
  return sort_and_group(w, num_rows, bits, num_segments_dev, error_dev, st);
}

extern "C" int es_segsum_fill(const void* values, int values_dtype, int64_t num_rows, int64_t tile_elems, int nd,
                              const int64_t* extents, void* workspace, size_t workspace_bytes, int64_t num_segments,
                              int32_t* out_coords, void* out_values, int out_dtype, void* stream) {
  cudaStream_t st = as_stream(stream);
  if (num_rows <= 0 || num_segments <= 0) return ES_OK;
  if (out_dtype != ES_F32 && out_dtype != ES_BF16) return ES_ERR_UNSUPPORTED;
  AggKeys ak;
  int bits = 0;
  ES_TRY(make_agg(nullptr, nd, nd, nd, extents, &ak, &bits));
  SegWs w;
  Carver c(workspace, workspace_bytes);
  seg_layout(c, w, num_rows);
  if (c.overflow) return ES_ERR_WORKSPACE;
  ES_LAUNCH(seg_offsets_kernel, grid_for(num_rows, 256), 256, 0, st, w.hdr, w.keys, w.rb.keys_alt, num_rows, w.flags,
            w.excl, ak, out_coords, w.seg_off, w.nseg);
  if (out_dtype == ES_F32)
    ES_TRY(launch_segment_reduce<float>(w, values, values_dtype, tile_elems, num_segments, 0,
                                        static_cast<float*>(out_values), st));
  else
    ES_TRY(launch_segment_reduce<__nv_bfloat16>(w, values, values_dtype, tile_elems, num_segments, 0,
                                                static_cast<__nv_bfloat16*>(out_values), st));
  return ES_OK;
}

// Group index of every input row: its sorted position s lies in group
// excl[s] + flags[s] - 1 (flags mark group heads, excl is their exclusive scan).
__global__ void row_group_kernel(const SegHeader* hdr, const uint32_t* p0, const uint32_t* p1, int64_t n,
                                 const uint32_t* __restrict__ flags, const uint32_t* __restrict__ excl,
                                 int32_t* __restrict__ row_group) {
  const uint32_t* perm = hdr->sorted_in_alt ? p1 : p0;
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s < n; s += (int64_t)gridDim.x * blockDim.x)
    row_group[perm[s]] = static_cast<int32_t>(excl[s] + flags[s]) - 1;
}

extern "C" int es_segsum_groups(int64_t num_rows, int nd, const int64_t* extents, void* workspace,
                                size_t workspace_bytes, int64_t num_segments, int32_t* out_coords, int32_t* row_group,
                                void* stream) {
  cudaStream_t st = as_stream(stream);
  if (num_rows <= 0 || num_segments <= 0) return ES_OK;
  if (num_segments > INT32_MAX) return ES_ERR_UNSUPPORTED;
  AggKeys ak;
  int bits = 0;
  ES_TRY(make_agg(nullptr, nd, nd, nd, extents, &ak, &bits));
  SegWs w;
  Carver c(workspace, workspace_bytes);
  seg_layout(c, w, num_rows);
  if (c.overflow) return ES_ERR_WORKSPACE;
  if (out_coords)
    ES_LAUNCH(seg_offsets_kernel, grid_for(num_rows, 256), 256, 0, st, w.hdr, w.keys, w.rb.keys_alt, num_rows,
              w.flags, w.excl, ak, out_coords, w.seg_off, w.nseg);
  if (row_group)
    ES_LAUNCH(row_group_kernel, grid_for(num_rows, 256), 256, 0, st, w.hdr, w.perm, w.rb.vals_alt, num_rows, w.flags,
              w.excl, row_group);
  return ES_OK;
}

extern "C" size_t es_scatter_add_workspace_size(int64_t num_rows) { return es_segments_workspace_size(num_rows); }

extern "C" int es_scatter_add_rows(const void* values, int values_dtype, const int32_t* idx, int64_t num_rows,
                                   int64_t tile_elems, int64_t num_out_rows, void* workspace, size_t workspace_bytes,
                                   float* out, int32_t* error_dev, void* stream) {
  cudaStream_t st = as_stream(stream);
  if (num_rows <= 0) return ES_OK;
  if (num_rows >= (int64_t)UINT32_MAX || num_out_rows <= 0) return ES_ERR_UNSUPPORTED;
  AggKeys ak;
  int bits = 0;
  int64_t ext = num_out_rows;
  ES_TRY(make_agg(nullptr, 1, 1, 1, &ext, &ak, &bits));
  SegWs w;
  Carver c(workspace, workspace_bytes);
  seg_layout(c, w, num_rows);
  if (c.overflow) return ES_ERR_WORKSPACE;
  ES_LAUNCH(row_keys_kernel, grid_for(num_rows, 256), 256, 0, st, idx, num_rows, 1, ak, w.keys, w.perm, error_dev);
  ES_TRY(sort_and_group(w, num_rows, bits, nullptr, error_dev, st));
  ES_LAUNCH(seg_offsets_kernel, grid_for(num_rows, 256), 256, 0, st, w.hdr, w.keys, w.rb.keys_alt, num_rows, w.flags,
            w.excl, ak, (int32_t*)nullptr, w.seg_off, w.nseg);
  ES_TRY(launch_segment_reduce<float>(w, values, values_dtype, tile_elems, 148 * 8, 1, out, st));
  return ES_OK;
}
