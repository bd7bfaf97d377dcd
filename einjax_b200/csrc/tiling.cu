// Tiling: element COO / dense arrays -> tile-COO (coords int32 (T, nd), values (T, tile)).
//
// Follows SparseTensor.to_relation (tensor/sparse.py:160-219). Each non-zero
// entry gets a 64-bit element key  tile_linear * tile_elems + in_tile_linear
// (row-major over the tile grid and inside the tile), so sorting the keys puts
// tiles in lexicographic coordinate order (np.unique, :204-206) and, inside a
// tile, entries in row-major position order. A stable sort keeps repeated
// coordinates in input order; the last of each run is the one written, which
// is what NumPy's fancy assignment at :211-212 leaves. Tiles are then written
// densely chunk by chunk: a CTA zero-fills 8192 output elements in shared
// memory, drops in the entries that land there and streams the chunk out
// with 16-byte stores, so every output byte is written exactly once.
#include "common.cuh"
#include "radix_sort.cuh"
#include "scan.cuh"

namespace es {

struct TileGeom {
  int ndim;
  int64_t shape[ES_MAX_DIMS];
  int64_t tile[ES_MAX_DIMS];
  int64_t grid[ES_MAX_DIMS];
  int64_t tile_elems;
  int64_t grid_tiles;
  int64_t total_elems;
  // log2 of tile[d], grid[d], tile_elems when a power of two, else -1
  int tile_sh[ES_MAX_DIMS];
  int grid_sh[ES_MAX_DIMS];
  int te_sh;
};

static int pow2_shift(int64_t v) {
  if (v <= 0 || (v & (v - 1)) != 0) return -1;
  int s = 0;
  while ((int64_t{1} << s) != v) ++s;
  return s;
}

// x / d: a shift for powers of two, 32-bit division when both fit (the
// common case: tile and grid extents, tile-linear indices), else 64-bit.
__device__ __forceinline__ uint64_t udiv(uint64_t x, uint64_t d, int sh) {
  if (sh >= 0) return x >> sh;
  if ((x >> 32) == 0 && (d >> 32) == 0) return static_cast<uint32_t>(x) / static_cast<uint32_t>(d);
  return x / d;
}

static int make_geom(int ndim, const int64_t* shape, const int64_t* tile, TileGeom* g) {
  if (ndim < 1 || ndim > ES_MAX_DIMS || !shape || !tile) return ES_ERR_INVALID;
  g->ndim = ndim;
  g->tile_elems = 1;
  g->grid_tiles = 1;
  g->total_elems = 1;
  for (int d = 0; d < ndim; ++d) {
    if (shape[d] <= 0 || tile[d] <= 0) return ES_ERR_INVALID;
    if (shape[d] % tile[d] != 0) return ES_ERR_INVALID;
    g->shape[d] = shape[d];
    g->tile[d] = tile[d];
    g->grid[d] = shape[d] / tile[d];
    g->tile_elems *= tile[d];
    g->grid_tiles *= g->grid[d];
    if (g->total_elems > (INT64_MAX / 4) / shape[d]) return ES_ERR_UNSUPPORTED;
    g->total_elems *= shape[d];
  }
  for (int d = ndim; d < ES_MAX_DIMS; ++d) g->shape[d] = g->tile[d] = g->grid[d] = 1;
  for (int d = 0; d < ES_MAX_DIMS; ++d) {
    g->tile_sh[d] = pow2_shift(g->tile[d]);
    g->grid_sh[d] = pow2_shift(g->grid[d]);
  }
  g->te_sh = pow2_shift(g->tile_elems);
  return ES_OK;
}

constexpr int kChunk = 8192;  // output elements per densify CTA

// Header kept at the start of the tiling workspace between plan and fill.
struct TileHeader {
  int32_t sorted_in_alt;
};

struct CooWs {
  TileHeader* hdr;
  uint64_t* keys;
  uint32_t* perm;
  RadixBuffers<uint64_t> rb;
  uint32_t* flags;
  uint32_t* excl;
  uint32_t* scan;
  int64_t* chunk_start;
};

static int64_t max_chunks_for(int64_t nnz, int64_t tile_elems) {
  // T <= nnz, so the values array holds at most nnz*tile_elems elements.
  return (nnz * tile_elems + kChunk - 1) / kChunk + 1;
}

struct SizeCarver {
  Sizer s;
  template <typename T>
  T* take(int64_t n) {
    s.take<T>(n);
    return nullptr;
  }
};

}  // namespace es

namespace es {

__global__ void set_flag_kernel(int32_t* p, int32_t v) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *p = v;
}

__global__ void coo_keys_kernel(const int32_t* __restrict__ idx, const void* __restrict__ vals, int vdtype,
                                int64_t nnz, TileGeom g, uint64_t sentinel, uint64_t* __restrict__ keys,
                                uint32_t* __restrict__ perm, int32_t* err) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < nnz; e += (int64_t)gridDim.x * blockDim.x) {
    uint64_t key = sentinel;
    if (is_nonzero(vals, vdtype, e)) {
      uint64_t tl = 0, w = 0;
      bool ok = true;
      for (int d = 0; d < g.ndim; ++d) {
        int64_t x = idx[e * g.ndim + d];
        if (x < 0 || x >= g.shape[d]) ok = false;
        const uint64_t q = udiv(static_cast<uint64_t>(x), static_cast<uint64_t>(g.tile[d]), g.tile_sh[d]);
        tl = tl * g.grid[d] + q;
        w = w * g.tile[d] + (static_cast<uint64_t>(x) - q * static_cast<uint64_t>(g.tile[d]));
      }
      if (ok) {
        key = tl * static_cast<uint64_t>(g.tile_elems) + w;
      } else if (err) {
        atomicExch(err, ES_ERR_INDEX);
      }
    }
    keys[e] = key;
    perm[e] = static_cast<uint32_t>(e);
  }
}

// flags[s] = 1 where entry s starts a new tile (valid entries only).
__global__ void tile_heads_kernel(const TileHeader* hdr, const uint64_t* k0, const uint64_t* k1, int64_t n,
                                  uint64_t tile_elems, int te_sh, uint64_t sentinel, uint32_t* __restrict__ flags) {
  const uint64_t* keys = hdr->sorted_in_alt ? k1 : k0;
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s < n; s += (int64_t)gridDim.x * blockDim.x) {
    uint64_t k = keys[s];
    uint32_t f = 0;
    if (k != sentinel)
      f = (s == 0 || udiv(keys[s - 1], tile_elems, te_sh) != udiv(k, tile_elems, te_sh)) ? 1u : 0u;
    flags[s] = f;
  }
}

// One pass over the sorted entries (s = 0 .. n):
// * a tile's first entry writes the tile's coordinates (coords row excl[s];
//   skipped when coords is null);
// * chunk_start[c] = first sorted entry whose output position lies in chunk c,
//   chunk_start[num_chunks] = number of valid entries.
__global__ void tile_coords_bounds_kernel(const TileHeader* hdr, const uint64_t* k0, const uint64_t* k1, int64_t n,
                                          const uint32_t* __restrict__ flags, const uint32_t* __restrict__ excl,
                                          TileGeom g, uint64_t sentinel, int64_t num_chunks,
                                          int32_t* __restrict__ coords, int64_t* __restrict__ chunk_start) {
  const uint64_t* keys = hdr->sorted_in_alt ? k1 : k0;
  const uint64_t te = static_cast<uint64_t>(g.tile_elems);
  for (int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; s <= n; s += (int64_t)gridDim.x * blockDim.x) {
    auto chunk_of = [&](int64_t i) -> int64_t {
      uint64_t k = keys[i];
      if (k == sentinel) return num_chunks;
      int64_t tid = static_cast<int64_t>(excl[i]) + flags[i] - 1;
      int64_t f = tid * static_cast<int64_t>(te) + static_cast<int64_t>(k - udiv(k, te, g.te_sh) * te);
      return f / kChunk;
    };
    int64_t prev = s == 0 ? -1 : chunk_of(s - 1);
    int64_t cur = s == n ? num_chunks : chunk_of(s);
    for (int64_t c = prev + 1; c <= cur; ++c) chunk_start[c] = s;
    if (coords && s < n && flags[s]) {
      uint64_t tl = udiv(keys[s], te, g.te_sh);
      const int64_t t = excl[s];
      for (int d = g.ndim - 1; d >= 0; --d) {
        const uint64_t q = udiv(tl, static_cast<uint64_t>(g.grid[d]), g.grid_sh[d]);
        coords[t * g.ndim + d] = static_cast<int32_t>(tl - q * static_cast<uint64_t>(g.grid[d]));
        tl = q;
      }
    }
  }
}

template <typename OutT>
__device__ __forceinline__ OutT cvt_out(float v);
template <>
__device__ __forceinline__ float cvt_out<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 cvt_out<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// One CTA per kChunk elements of the tile value array: the chunk is first
// written as zeros with 16-byte stores, then (after the block barrier, which
// orders the zero stores before them) the chunk's entries are stored over it
// -- the last of repeated coordinates only. Every output byte goes to L2 once
// as a full line; the few entry stores land on lines still in L2.
template <typename OutT>
__global__ void __launch_bounds__(256) densify_kernel(const TileHeader* hdr, const uint64_t* k0, const uint64_t* k1,
                                                      const uint32_t* p0, const uint32_t* p1, int64_t n,
                                                      const uint32_t* __restrict__ flags,
                                                      const uint32_t* __restrict__ excl,
                                                      const int64_t* __restrict__ chunk_start,
                                                      const void* __restrict__ vals, int vdtype, uint64_t tile_elems,
                                                      int te_sh, int64_t total_out, int vec_ok,
                                                      OutT* __restrict__ out) {
  const uint64_t* keys = hdr->sorted_in_alt ? k1 : k0;
  const uint32_t* perm = hdr->sorted_in_alt ? p1 : p0;
  const int64_t c = blockIdx.x;
  const int64_t base = c * kChunk;
  constexpr int kVec = 16 / sizeof(OutT);
  const int64_t len = min(static_cast<int64_t>(kChunk), total_out - base);
  // with a 16-byte aligned value array (vec_ok) a full chunk is whole
  // 16-byte pieces (kChunk is a multiple of kVec)
  if (len == kChunk && vec_ok) {
#pragma unroll 4
    for (int i = threadIdx.x * kVec; i < kChunk; i += blockDim.x * kVec)
      *reinterpret_cast<uint4*>(&out[base + i]) = make_uint4(0u, 0u, 0u, 0u);
  } else {
    for (int64_t i = threadIdx.x; i < len; i += blockDim.x) out[base + i] = cvt_out<OutT>(0.f);
  }
  __syncthreads();
  const int64_t s0 = chunk_start[c], s1 = chunk_start[c + 1];
  for (int64_t s = s0 + threadIdx.x; s < s1; s += blockDim.x) {
    const uint64_t k = keys[s];
    const bool last = (s + 1 >= n) || keys[s + 1] != k;
    if (!last) continue;
    const int64_t tid = static_cast<int64_t>(excl[s]) + flags[s] - 1;
    const int64_t f = tid * static_cast<int64_t>(tile_elems) +
                      static_cast<int64_t>(k - udiv(k, tile_elems, te_sh) * tile_elems);
    out[f] = cvt_out<OutT>(load_as_f32(vals, vdtype, perm[s]));
  }
}

// ---- dense -> tiles -------------------------------------------------------

struct DenseWs {
  uint32_t* flags;
  uint32_t* excl;
  uint32_t* scan;
};

template <typename C>
static void dense_layout(C& c, DenseWs& w, int64_t grid_tiles) {
  w.flags = c.template take<uint32_t>(grid_tiles);
  w.excl = c.template take<uint32_t>(grid_tiles);
  w.scan = c.template take<uint32_t>(scan_scratch_elems(grid_tiles));
}

__device__ __forceinline__ int64_t dense_offset(const TileGeom& g, int64_t tile_lin, int64_t e) {
  // element e of grid tile tile_lin -> row-major offset in the dense array
  int64_t off = 0, stride = 1;
  for (int d = g.ndim - 1; d >= 0; --d) {
    const int64_t tq = static_cast<int64_t>(udiv(tile_lin, g.grid[d], g.grid_sh[d]));
    const int64_t td = tile_lin - tq * g.grid[d];
    tile_lin = tq;
    const int64_t eq = static_cast<int64_t>(udiv(e, g.tile[d], g.tile_sh[d]));
    const int64_t wd = e - eq * g.tile[d];
    e = eq;
    off += (td * g.tile[d] + wd) * stride;
    stride *= g.shape[d];
  }
  return off;
}

__global__ void dense_flags_kernel(const void* __restrict__ dense, int dtype, TileGeom g, uint32_t* __restrict__ flags) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t t = warp; t < g.grid_tiles; t += nwarps) {
    bool any = false;
    for (int64_t e0 = 0; e0 < g.tile_elems && !any; e0 += 32) {
      int64_t e = e0 + lane;
      bool nz = e < g.tile_elems && is_nonzero(dense, dtype, dense_offset(g, t, e));
      any = __any_sync(0xffffffffu, nz);
    }
    if (lane == 0) flags[t] = any ? 1u : 0u;
  }
}

// Coordinates of the non-zero tiles: thread t writes grid tile t's row
// excl[t] when flags[t] is set.
__global__ void dense_coords_kernel(TileGeom g, const uint32_t* __restrict__ flags,
                                    const uint32_t* __restrict__ excl, int32_t* __restrict__ coords) {
  for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < g.grid_tiles;
       t += (int64_t)gridDim.x * blockDim.x) {
    if (!flags[t]) continue;
    const int64_t r = excl[t];
    int64_t tl = t;
    for (int d = g.ndim - 1; d >= 0; --d) {
      const int64_t q = static_cast<int64_t>(udiv(tl, g.grid[d], g.grid_sh[d]));
      coords[r * g.ndim + d] = static_cast<int32_t>(tl - q * g.grid[d]);
      tl = q;
    }
  }
}

// Values of the non-zero tiles, any input dtype: one block per grid tile at a
// time, row excl[t] of out.
template <typename OutT>
__global__ void dense_fill_kernel(const void* __restrict__ dense, int dtype, TileGeom g,
                                  const uint32_t* __restrict__ flags, const uint32_t* __restrict__ excl,
                                  OutT* __restrict__ out) {
  for (int64_t t = blockIdx.x; t < g.grid_tiles; t += gridDim.x) {
    if (!flags[t]) continue;
    const int64_t r = excl[t];
    for (int64_t e = threadIdx.x; e < g.tile_elems; e += blockDim.x)
      out[r * g.tile_elems + e] = cvt_out<OutT>(load_as_f32(dense, dtype, dense_offset(g, t, e)));
  }
}

// fp32 -> fp32 in whole 16-byte pieces (both arrays 16-byte aligned, tile
// rows a multiple of four floats, so four consecutive elements of a tile row
// are four consecutive floats of the dense array). A block takes
// kDenseBatch consecutive grid tiles at a time; each thread keeps kPer
// pieces of them in flight, all loads of a round issued before its stores.
constexpr int kDenseBatch = 4;

__global__ void __launch_bounds__(256) dense_fill_vec_kernel(const float* __restrict__ dense, TileGeom g,
                                                             const uint32_t* __restrict__ flags,
                                                             const uint32_t* __restrict__ excl,
                                                             float* __restrict__ out) {
  constexpr int kPer = 4;
  const uint32_t pieces = static_cast<uint32_t>(g.tile_elems / 4);
  const uint32_t span = pieces * kDenseBatch;
  for (int64_t t0 = blockIdx.x * static_cast<int64_t>(kDenseBatch); t0 < g.grid_tiles;
       t0 += static_cast<int64_t>(gridDim.x) * kDenseBatch) {
    for (uint32_t q0 = threadIdx.x; q0 < span; q0 += blockDim.x * kPer) {
      float4 v[kPer];
      int64_t dst[kPer];
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        dst[j] = -1;
        const uint32_t q = q0 + j * blockDim.x;
        if (q < span) {
          const uint32_t bt = q / pieces, p = q - bt * pieces;
          const int64_t t = t0 + bt;
          if (t < g.grid_tiles && flags[t]) {
            v[j] = *reinterpret_cast<const float4*>(dense + dense_offset(g, t, 4 * static_cast<int64_t>(p)));
            dst[j] = static_cast<int64_t>(excl[t]) * pieces + p;
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kPer; ++j)
        if (dst[j] >= 0) reinterpret_cast<float4*>(out)[dst[j]] = v[j];
    }
  }
}

}  // namespace es

using namespace es;

extern "C" size_t es_tile_coo_workspace_size(int64_t nnz, int ndim, const int64_t* shape, const int64_t* tile) {
  TileGeom g;
  if (make_geom(ndim, shape, tile, &g) != ES_OK) return 0;
  SizeCarver sc;
  CooWs w;
  w.hdr = sc.take<TileHeader>(1);
  sc.take<uint64_t>(nnz);
  sc.take<uint32_t>(nnz);
  radix_reserve<uint64_t>(sc.s, nnz);
  sc.take<uint32_t>(nnz);
  sc.take<uint32_t>(nnz);
  sc.take<uint32_t>(scan_scratch_elems(nnz));
  sc.take<int64_t>(max_chunks_for(nnz, g.tile_elems) + 1);
  return sc.s.used + 256;
}

static int carve_coo(void* ws, size_t bytes, int64_t nnz, int64_t tile_elems, CooWs* w) {
  Carver c(ws, bytes);
  w->hdr = c.take<TileHeader>(1);
  w->keys = c.take<uint64_t>(nnz);
  w->perm = c.take<uint32_t>(nnz);
  w->rb.carve(c, nnz);
  w->flags = c.take<uint32_t>(nnz);
  w->excl = c.take<uint32_t>(nnz);
  w->scan = c.take<uint32_t>(scan_scratch_elems(nnz));
  w->chunk_start = c.take<int64_t>(max_chunks_for(nnz, tile_elems) + 1);
  return c.overflow ? ES_ERR_WORKSPACE : ES_OK;
}

extern "C" int es_tile_coo_plan(const int32_t* indices, const void* values, int values_dtype, int64_t nnz, int ndim,
                                const int64_t* shape, const int64_t* tile, void* workspace, size_t workspace_bytes,
                                int64_t* num_tiles_dev, int32_t* error_dev, void* stream) {
  TileGeom g;
  ES_TRY(make_geom(ndim, shape, tile, &g));
  if (nnz < 0 || nnz >= (int64_t)UINT32_MAX) return ES_ERR_UNSUPPORTED;
  if (values_dtype != ES_F32 && values_dtype != ES_F64 && values_dtype != ES_BF16) return ES_ERR_UNSUPPORTED;
  cudaStream_t st = as_stream(stream);
  // the status slot needs no initialisation by the caller
  if (error_dev && cudaMemsetAsync(error_dev, 0, sizeof(int32_t), st) != cudaSuccess) return ES_ERR_CUDA;
  if (nnz == 0) {
    if (cudaMemsetAsync(num_tiles_dev, 0, sizeof(int64_t), st) != cudaSuccess) return ES_ERR_CUDA;
    return ES_OK;
  }
  CooWs w;
  ES_TRY(carve_coo(workspace, workspace_bytes, nnz, g.tile_elems, &w));
  const uint64_t sentinel = static_cast<uint64_t>(g.total_elems);
  const int bits = bit_length(sentinel);
  ES_LAUNCH(coo_keys_kernel, grid_for(nnz, 256), 256, 0, st, indices, values, values_dtype, nnz, g, sentinel, w.keys,
            w.perm, error_dev);
  uint64_t* k = w.keys;
  uint32_t* p = w.perm;
  ES_TRY(radix_sort_pairs<uint64_t>(&k, &p, w.rb, nnz, 0, bits, st, error_dev));
  const int alt = (k != w.keys) ? 1 : 0;
  ES_LAUNCH(set_flag_kernel, 1, 32, 0, st, &w.hdr->sorted_in_alt, alt);
  ES_LAUNCH(tile_heads_kernel, grid_for(nnz, 256), 256, 0, st, w.hdr, w.keys, w.rb.keys_alt, nnz,
            static_cast<uint64_t>(g.tile_elems), g.te_sh, sentinel, w.flags);
  // T (uint32) is accumulated into the low word of *num_tiles_dev.
  if (cudaMemsetAsync(num_tiles_dev, 0, sizeof(int64_t), st) != cudaSuccess) return ES_ERR_CUDA;
  ES_TRY(exclusive_scan<uint32_t>(w.flags, w.excl, nnz, reinterpret_cast<uint32_t*>(num_tiles_dev), w.scan, st));
  return ES_OK;
}

extern "C" int es_tile_coo_fill(const void* values, int values_dtype, int64_t nnz, int ndim, const int64_t* shape,
                                const int64_t* tile, void* workspace, size_t workspace_bytes, int64_t num_tiles,
                                int32_t* coords_out, void* values_out, int out_dtype, void* stream) {
  TileGeom g;
  ES_TRY(make_geom(ndim, shape, tile, &g));
  if (out_dtype != ES_F32 && out_dtype != ES_BF16) return ES_ERR_UNSUPPORTED;
  if (num_tiles <= 0 || nnz <= 0) return ES_OK;
  cudaStream_t st = as_stream(stream);
  CooWs w;
  ES_TRY(carve_coo(workspace, workspace_bytes, nnz, g.tile_elems, &w));
  const uint64_t sentinel = static_cast<uint64_t>(g.total_elems);
  const int64_t total_out = num_tiles * g.tile_elems;
  const int64_t num_chunks = (total_out + kChunk - 1) / kChunk;
  if (num_chunks > max_chunks_for(nnz, g.tile_elems)) return ES_ERR_INVALID;
  // coords_out null: the values alone, from the chunk bounds an earlier call
  // with coords_out left in this workspace; values_out null: coords (and the
  // bounds) alone
  if (coords_out)
    ES_LAUNCH(tile_coords_bounds_kernel, grid_for(nnz + 1, 256), 256, 0, st, w.hdr, w.keys, w.rb.keys_alt, nnz,
              w.flags, w.excl, g, sentinel, num_chunks, coords_out, w.chunk_start);
  if (!values_out) return ES_OK;
  const int vec_ok = (reinterpret_cast<uintptr_t>(values_out) & 15u) == 0 ? 1 : 0;
  if (out_dtype == ES_F32) {
    ES_LAUNCH(densify_kernel<float>, (int)num_chunks, 256, 0, st, w.hdr, w.keys, w.rb.keys_alt, w.perm,
              w.rb.vals_alt, nnz, w.flags, w.excl, w.chunk_start, values, values_dtype,
              static_cast<uint64_t>(g.tile_elems), g.te_sh, total_out, vec_ok, static_cast<float*>(values_out));
  } else {
    ES_LAUNCH(densify_kernel<__nv_bfloat16>, (int)num_chunks, 256, 0, st, w.hdr, w.keys, w.rb.keys_alt, w.perm,
              w.rb.vals_alt, nnz, w.flags, w.excl, w.chunk_start, values, values_dtype,
              static_cast<uint64_t>(g.tile_elems), g.te_sh, total_out, vec_ok,
              static_cast<__nv_bfloat16*>(values_out));
  }
  return ES_OK;
}

extern "C" size_t es_tile_dense_workspace_size(int ndim, const int64_t* shape, const int64_t* tile) {
  TileGeom g;
  if (make_geom(ndim, shape, tile, &g) != ES_OK) return 0;
  SizeCarver sc;
  DenseWs w;
  dense_layout(sc, w, g.grid_tiles);
  return sc.s.used + 256;
}

extern "C" int es_tile_dense_plan(const void* dense, int dtype, int ndim, const int64_t* shape, const int64_t* tile,
                                  void* workspace, size_t workspace_bytes, int64_t* num_tiles_dev, void* stream) {
  TileGeom g;
  ES_TRY(make_geom(ndim, shape, tile, &g));
  if (dtype != ES_F32 && dtype != ES_F64 && dtype != ES_BF16) return ES_ERR_UNSUPPORTED;
  if (g.grid_tiles >= (int64_t)UINT32_MAX) return ES_ERR_UNSUPPORTED;
  cudaStream_t st = as_stream(stream);
  Carver c(workspace, workspace_bytes);
  DenseWs w;
  dense_layout(c, w, g.grid_tiles);
  if (c.overflow) return ES_ERR_WORKSPACE;
  ES_LAUNCH(dense_flags_kernel, grid_for(g.grid_tiles * 32, 256), 256, 0, st, dense, dtype, g, w.flags);
  if (cudaMemsetAsync(num_tiles_dev, 0, sizeof(int64_t), st) != cudaSuccess) return ES_ERR_CUDA;
  ES_TRY(exclusive_scan<uint32_t>(w.flags, w.excl, g.grid_tiles, reinterpret_cast<uint32_t*>(num_tiles_dev), w.scan,
                                  st));
  return ES_OK;
}

extern "C" int es_tile_dense_fill(const void* dense, int dtype, int ndim, const int64_t* shape, const int64_t* tile,
                                  void* workspace, size_t workspace_bytes, int64_t num_tiles, int32_t* coords_out,
                                  void* values_out, int out_dtype, void* stream) {
  TileGeom g;
  ES_TRY(make_geom(ndim, shape, tile, &g));
  if (out_dtype != ES_F32 && out_dtype != ES_BF16) return ES_ERR_UNSUPPORTED;
  if (num_tiles <= 0) return ES_OK;
  cudaStream_t st = as_stream(stream);
  Carver c(workspace, workspace_bytes);
  DenseWs w;
  dense_layout(c, w, g.grid_tiles);
  if (c.overflow) return ES_ERR_WORKSPACE;
  // coords_out / values_out null: that output is not written
  if (coords_out)
    ES_LAUNCH(dense_coords_kernel, grid_for(g.grid_tiles, 256), 256, 0, st, g, w.flags, w.excl, coords_out);
  if (!values_out) return ES_OK;
  const int grid = static_cast<int>(g.grid_tiles < 148 * 16 ? g.grid_tiles : 148 * 16);
  const bool vec = dtype == ES_F32 && out_dtype == ES_F32 && g.tile[ndim - 1] % 4 == 0 &&
                   g.shape[ndim - 1] % 4 == 0 && g.tile_elems < (1LL << 28) &&
                   (reinterpret_cast<uintptr_t>(dense) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(values_out) & 15u) == 0;
  if (vec) {
    const int64_t nb = (g.grid_tiles + kDenseBatch - 1) / kDenseBatch;
    ES_LAUNCH(dense_fill_vec_kernel, static_cast<int>(nb < 148 * 16 ? nb : 148 * 16), 256, 0, st,
              static_cast<const float*>(dense), g, w.flags, w.excl, static_cast<float*>(values_out));
  } else if (out_dtype == ES_F32) {
    ES_LAUNCH(dense_fill_kernel<float>, grid, 256, 0, st, dense, dtype, g, w.flags, w.excl,
              static_cast<float*>(values_out));
  } else {
    ES_LAUNCH(dense_fill_kernel<__nv_bfloat16>, grid, 256, 0, st, dense, dtype, g, w.flags, w.excl,
              static_cast<__nv_bfloat16*>(values_out));
  }
  return ES_OK;
}
