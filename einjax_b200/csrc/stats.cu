// Sparsity statistics per tiling scheme, the planner's input
// (tensor/stats.py:25-80, SparseTensor._compute_sparsity_metrics
// tensor/sparse.py:122-158, DenseTensor's tensor/dense.py:44-94): for every
// tile shape U, T(U) = tiles that hold a non-zero entry and V(l, U) = distinct
// tile coordinates along dimension l. The reference runs one np.unique per
// scheme (or a Python loop over entries x schemes for dense input).
//
// Here:
//  * V: one pass over the entries marks, per dimension l, a bitmap of the
//    coordinates that hold a non-zero (shape_l bits); V(l, U) is the number of
//    groups of t_l consecutive coordinates with a set bit (one warp per
//    (scheme, dimension)).
//  * T: schemes go in batches whose tile-grid bitmaps (one bit per tile) fit
//    the bitmap budget; one pass over the entries sets each entry's tile bit in
//    every bitmap of the batch, then a popcount per scheme gives T.
//  * A scheme whose grid does not fit the budget counts the distinct tile keys
//    of its entries after a radix sort.
// Entries come as COO (int32 indices (n, ndim) and values) or as a dense
// row-major array of `shape` (indices NULL); zeros do not count, repeated
// coordinates count once.
#include <vector>

#include "common.cuh"
#include "radix_sort.cuh"
#include "scan.cuh"

namespace es {

constexpr int kStatsBatch = 16;                              // schemes per marking pass
constexpr int64_t kStatsBitmapWords = int64_t(1) << 27;       // 512 MB of tile bits per pass

// floor(c / t) for 0 <= c < 2^31, 1 <= t < 2^31 as (c * m) >> sh with
// m = ceil(2^(31+k) / t), k = ceil(log2 t), sh = 31 + k (Granlund &
// Montgomery, "Division by invariant integers using multiplication", 1994):
// c*m / 2^sh exceeds c/t by less than 2^31 / 2^sh = 2^-k <= 1/t, which
// cannot carry c/t = q + r/t (r <= t - 1) past q + 1; m < 2^32 + 1 and
// c * m < 2^64.
struct FastDiv {
  uint64_t m;
  int sh;
};

static FastDiv make_fastdiv(int64_t t) {
  int k = 0;
  while ((int64_t(1) << k) < t) ++k;
  FastDiv f;
  f.sh = 31 + k;
  const unsigned __int128 num = static_cast<unsigned __int128>(1) << f.sh;
  f.m = static_cast<uint64_t>((num + static_cast<unsigned __int128>(t) - 1) / static_cast<unsigned __int128>(t));
  return f;
}

__device__ __forceinline__ uint32_t fdiv(uint32_t c, const FastDiv& f) {
  return static_cast<uint32_t>((static_cast<uint64_t>(c) * f.m) >> f.sh);
}

struct StatsGeom {
  int nd;
  int64_t shape[ES_MAX_DIMS];
  int64_t cbm_off[ES_MAX_DIMS];    // word offset of dimension l's coordinate bitmap
};

struct StatsBatch {
  int n;
  int sidx[kStatsBatch];  // output index of each scheme
  FastDiv tdiv[kStatsBatch][ES_MAX_DIMS];
  int64_t grid[kStatsBatch][ES_MAX_DIMS];
  int64_t word_off[kStatsBatch + 1];  // bitmap words of scheme j: [word_off[j], word_off[j+1])
};

// Coordinates of entry e (COO row e, or the dense array's linear index e);
// false when it holds a zero.
__device__ __forceinline__ bool stats_entry(const int32_t* __restrict__ idx, const void* __restrict__ vals, int vdt,
                                            int64_t e, const StatsGeom& g, uint32_t (&c)[ES_MAX_DIMS],
                                            int32_t* err) {
  if (vals && !is_nonzero(vals, vdt, e)) return false;
  if (idx) {
    const int32_t* row = idx + e * g.nd;
    for (int d = 0; d < g.nd; ++d) {
      const int32_t x = row[d];
      if (x < 0 || x >= g.shape[d]) {
        if (err) atomicExch(err, ES_ERR_INDEX);
        return false;
      }
      c[d] = static_cast<uint32_t>(x);
    }
  } else {
    uint64_t lin = static_cast<uint64_t>(e);
    for (int d = g.nd - 1; d >= 0; --d) {
      const uint64_t q = lin / static_cast<uint64_t>(g.shape[d]);
      c[d] = static_cast<uint32_t>(lin - q * static_cast<uint64_t>(g.shape[d]));
      lin = q;
    }
  }
  return true;
}

// Sets a bit, skipping the atomic when a plain read already sees it set:
// bits only go from 0 to 1 during a pass, so a stale read can only cost a
// redundant atomic. Coarse tilings (few tiles, every entry on a handful of
// words) would otherwise serialise millions of atomics on one L2 line.
__device__ __forceinline__ void set_bit(uint32_t* bm, uint64_t bit) {
  uint32_t* w = bm + (bit >> 5);
  const uint32_t m = 1u << (bit & 31);
  if (!(*reinterpret_cast<volatile uint32_t*>(w) & m)) atomicOr(w, m);
}

// Per-dimension coordinate bitmaps.
__global__ void stats_coords_kernel(const int32_t* __restrict__ idx, const void* __restrict__ vals, int vdt,
                                    int64_t n, StatsGeom g, uint32_t* __restrict__ cbm, int32_t* err) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    uint32_t c[ES_MAX_DIMS];
    if (!stats_entry(idx, vals, vdt, e, g, c, err)) continue;
    for (int d = 0; d < g.nd; ++d) set_bit(cbm + g.cbm_off[d], c[d]);
  }
}

// Tile bits of every scheme of the batch.
__global__ void stats_mark_kernel(const int32_t* __restrict__ idx, const void* __restrict__ vals, int vdt, int64_t n,
                                  StatsGeom g, StatsBatch b, uint32_t* __restrict__ bm) {
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    uint32_t c[ES_MAX_DIMS];
    if (!stats_entry(idx, vals, vdt, e, g, c, nullptr)) continue;
    for (int j = 0; j < b.n; ++j) {
      uint64_t lin = 0;
      for (int d = 0; d < g.nd; ++d) lin = lin * static_cast<uint64_t>(b.grid[j][d]) + fdiv(c[d], b.tdiv[j][d]);
      set_bit(bm + b.word_off[j], lin);
    }
  }
}

// T of each scheme of the batch: popcount of its bitmap words.
__global__ void stats_popcount_kernel(const uint32_t* __restrict__ bm, StatsBatch b,
                                      int64_t* __restrict__ num_tuples) {
  const int64_t nw = b.word_off[b.n];
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t w0 = ((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5) * 32; w0 < nw; w0 += warps * 32) {
    const int64_t w = w0 + lane;
    int j = 0;
    if (w < nw)
      while (j + 1 < b.n && b.word_off[j + 1] <= w) ++j;
    const uint32_t pc = w < nw ? static_cast<uint32_t>(__popc(bm[w])) : 0u;
    const int j0 = __shfl_sync(0xffffffffu, j, 0);
    if (__all_sync(0xffffffffu, j == j0 || w >= nw)) {
      uint32_t s = pc;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0 && s) atomicAdd(reinterpret_cast<unsigned long long*>(num_tuples + b.sidx[j0]), s);
    } else if (pc) {
      atomicAdd(reinterpret_cast<unsigned long long*>(num_tuples + b.sidx[j]), pc);
    }
  }
}

// V(l, U) for scheme s, dimension l: groups of t_l coordinates with a set
// bit in l's coordinate bitmap. One warp per (scheme, dimension).
__global__ void stats_vcount_kernel(const uint32_t* __restrict__ cbm, StatsGeom g, const int64_t* __restrict__ tiles,
                                    int nschemes, int64_t* __restrict__ value_count) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t u = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5; u < static_cast<int64_t>(nschemes) * g.nd;
       u += warps) {
    const int64_t s = u / g.nd;
    const int d = static_cast<int>(u - s * g.nd);
    const int64_t t = tiles[s * g.nd + d], len = g.shape[d];
    const int64_t groups = (len + t - 1) / t;
    const uint32_t* bm = cbm + g.cbm_off[d];
    int64_t cnt = 0;
    for (int64_t gi = lane; gi < groups; gi += 32) {
      const int64_t lo = gi * t, hi = lo + t < len ? lo + t : len;
      bool any = false;
      for (int64_t bit = lo; bit < hi && !any;) {
        const int64_t word = bit >> 5;
        const int b0 = static_cast<int>(bit & 31);
        const int64_t take = (hi - bit) < (32 - b0) ? (hi - bit) : (32 - b0);
        const uint32_t mask = take == 32 ? 0xffffffffu : (((1u << take) - 1u) << b0);
        any = (bm[word] & mask) != 0u;
        bit += take;
      }
      cnt += any ? 1 : 0;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    if (lane == 0) value_count[u] = cnt;
  }
}

// Sort path: tile key of every entry (zeros get the sentinel `grid_total`).
__global__ void stats_keys_kernel(const int32_t* __restrict__ idx, const void* __restrict__ vals, int vdt, int64_t n,
                                  StatsGeom g, StatsBatch b, uint64_t* __restrict__ keys, uint32_t* __restrict__ perm) {
  uint64_t total = 1;
  for (int d = 0; d < g.nd; ++d) total *= static_cast<uint64_t>(b.grid[0][d]);
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    uint32_t c[ES_MAX_DIMS];
    uint64_t lin = total;
    if (stats_entry(idx, vals, vdt, e, g, c, nullptr)) {
      lin = 0;
      for (int d = 0; d < g.nd; ++d) lin = lin * static_cast<uint64_t>(b.grid[0][d]) + fdiv(c[d], b.tdiv[0][d]);
    }
    keys[e] = lin;
    perm[e] = static_cast<uint32_t>(e);
  }
}

// Distinct sorted keys below the sentinel.
__global__ void stats_distinct_kernel(const uint64_t* __restrict__ keys, int64_t n, uint64_t sentinel,
                                      int64_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  for (int64_t i0 = ((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5) * 32; i0 < n;
       i0 += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = i0 + lane;
    const bool head = i < n && keys[i] != sentinel && (i == 0 || keys[i - 1] != keys[i]);
    const uint32_t c = static_cast<uint32_t>(__popc(__ballot_sync(0xffffffffu, head)));
    if (lane == 0 && c) atomicAdd(reinterpret_cast<unsigned long long*>(out), static_cast<unsigned long long>(c));
  }
}

// ------------------------------------------------------------ host planning

struct StatsPlan {
  StatsGeom g;
  int64_t cbm_words = 0;
  int64_t bm_words = 0;    // tile bitmap words of the largest batch
  bool need_sort = false;
  std::vector<std::vector<int>> batches;  // bitmap schemes per pass
  std::vector<int> sorted;                // schemes counted by the sort path
};

static int plan_stats(int64_t n, int nd, const int64_t* shape, const int64_t* tiles, int nschemes, StatsPlan* p) {
  if (nd < 1 || nd > ES_MAX_DIMS || nschemes < 0 || n < 0) return ES_ERR_INVALID;
  p->g.nd = nd;
  for (int d = 0; d < nd; ++d) {
    if (shape[d] <= 0 || shape[d] >= INT32_MAX) return ES_ERR_UNSUPPORTED;
    p->g.shape[d] = shape[d];
    p->g.cbm_off[d] = p->cbm_words;
    p->cbm_words += (shape[d] + 31) / 32;
  }
  std::vector<int> cur;
  int64_t cur_words = 0;
  for (int s = 0; s < nschemes; ++s) {
    long double total = 1;
    for (int d = 0; d < nd; ++d) {
      const int64_t t = tiles[s * nd + d];
      if (t <= 0 || t >= INT32_MAX) return ES_ERR_INVALID;
      total *= static_cast<long double>((shape[d] + t - 1) / t);
    }
    if (total > static_cast<long double>(kStatsBitmapWords) * 32) {
      p->sorted.push_back(s);
      p->need_sort = true;
      continue;
    }
    const int64_t words = (static_cast<int64_t>(total) + 31) / 32;
    if (!cur.empty() && (cur_words + words > kStatsBitmapWords || static_cast<int>(cur.size()) == kStatsBatch)) {
      p->batches.push_back(cur);
      cur.clear();
      cur_words = 0;
    }
    cur.push_back(s);
    cur_words += words;
    if (cur_words > p->bm_words) p->bm_words = cur_words;
  }
  if (!cur.empty()) p->batches.push_back(cur);
  if (p->need_sort && n >= static_cast<int64_t>(UINT32_MAX)) return ES_ERR_UNSUPPORTED;
  return ES_OK;
}

struct StatsWs {
  int64_t* tiles;  // (schemes, ndim) tile shapes on the device
  uint32_t* cbm;
  uint32_t* bm;
  uint64_t* keys;
  uint32_t* perm;
  RadixBuffers<uint64_t> rb;
};

template <typename C>
static void stats_layout(C& c, StatsWs& w, const StatsPlan& p, int64_t n, int nschemes) {
  w.tiles = c.template take<int64_t>(static_cast<int64_t>(nschemes) * p.g.nd);
  w.cbm = c.template take<uint32_t>(p.cbm_words);
  w.bm = c.template take<uint32_t>(p.bm_words);
  if (p.need_sort) {
    w.keys = c.template take<uint64_t>(n);
    w.perm = c.template take<uint32_t>(n);
    w.rb.keys_alt = c.template take<uint64_t>(n);
    w.rb.vals_alt = c.template take<uint32_t>(n);
    w.rb.hist = c.template take<uint32_t>(RadixScratchSize::hist_elems(n));
    w.rb.scan = c.template take<uint32_t>(RadixScratchSize::scan_elems(n));
  }
}

struct StatsSizer {
  Sizer s;
  template <typename T>
  T* take(int64_t k) {
    s.take<T>(k);
    return nullptr;
  }
};

static StatsBatch make_batch(const StatsPlan& p, const std::vector<int>& schemes, const int64_t* tiles) {
  StatsBatch b;
  b.n = static_cast<int>(schemes.size());
  int64_t off = 0;
  for (int j = 0; j < b.n; ++j) {
    const int s = schemes[j];
    int64_t total = 1;
    for (int d = 0; d < p.g.nd; ++d) {
      const int64_t t = tiles[s * p.g.nd + d];
      b.tdiv[j][d] = make_fastdiv(t);
      b.grid[j][d] = (p.g.shape[d] + t - 1) / t;
      total *= b.grid[j][d];
    }
    b.sidx[j] = s;
    b.word_off[j] = off;
    off += (total + 31) / 32;
  }
  b.word_off[b.n] = off;
  return b;
}

}  // namespace es

using namespace es;

extern "C" size_t es_sparsity_stats_workspace_size(int64_t num_entries, int ndim, const int64_t* shape,
                                                   const int64_t* tile_shapes, int num_schemes) {
  StatsPlan p;
  if (plan_stats(num_entries, ndim, shape, tile_shapes, num_schemes, &p) != ES_OK) return 0;
  StatsSizer s;
  StatsWs w;
  stats_layout(s, w, p, num_entries, num_schemes);
  return s.s.used + 256;
}

extern "C" int es_sparsity_stats(const int32_t* indices, const void* values, int values_dtype, int64_t num_entries,
                                 int ndim, const int64_t* shape, const int64_t* tile_shapes, int num_schemes,
                                 void* workspace, size_t workspace_bytes, int64_t* num_tuples_dev,
                                 int64_t* value_count_dev, int32_t* error_dev, void* stream) {
  cudaStream_t st = as_stream(stream);
  StatsPlan p;
  ES_TRY(plan_stats(num_entries, ndim, shape, tile_shapes, num_schemes, &p));
  if (!indices && !values) return ES_ERR_INVALID;
  if (values && values_dtype != ES_F32 && values_dtype != ES_BF16 && values_dtype != ES_F64) return ES_ERR_UNSUPPORTED;
  if (!indices) {
    int64_t total = 1;
    for (int d = 0; d < ndim; ++d) total *= shape[d];
    if (total != num_entries) return ES_ERR_INVALID;
  }
  if (num_schemes == 0) return ES_OK;
  if (cudaMemsetAsync(num_tuples_dev, 0, num_schemes * sizeof(int64_t), st) != cudaSuccess) return ES_ERR_CUDA;
  if (cudaMemsetAsync(value_count_dev, 0, static_cast<size_t>(num_schemes) * ndim * sizeof(int64_t), st) !=
      cudaSuccess)
    return ES_ERR_CUDA;
  if (num_entries == 0) return ES_OK;
  Carver cv(workspace, workspace_bytes);
  StatsWs w;
  stats_layout(cv, w, p, num_entries, num_schemes);
  if (cv.overflow) return ES_ERR_WORKSPACE;
  const int grid = grid_for(num_entries, 256);
  // V: coordinate bitmaps, then per (scheme, dimension) group counts
  if (cudaMemsetAsync(w.cbm, 0, p.cbm_words * sizeof(uint32_t), st) != cudaSuccess) return ES_ERR_CUDA;
  ES_LAUNCH(stats_coords_kernel, grid, 256, 0, st, indices, values, values_dtype, num_entries, p.g, w.cbm, error_dev);
  if (cudaMemcpyAsync(w.tiles, tile_shapes, static_cast<size_t>(num_schemes) * ndim * sizeof(int64_t),
                      cudaMemcpyHostToDevice, st) != cudaSuccess)
    return ES_ERR_CUDA;
  ES_LAUNCH(stats_vcount_kernel, grid_for(static_cast<int64_t>(num_schemes) * ndim * 32, 256), 256, 0, st, w.cbm, p.g,
            w.tiles, num_schemes, value_count_dev);
  // T: bitmap batches
  for (const auto& sch : p.batches) {
    const StatsBatch b = make_batch(p, sch, tile_shapes);
    if (cudaMemsetAsync(w.bm, 0, b.word_off[b.n] * sizeof(uint32_t), st) != cudaSuccess) return ES_ERR_CUDA;
    ES_LAUNCH(stats_mark_kernel, grid, 256, 0, st, indices, values, values_dtype, num_entries, p.g, b, w.bm);
    ES_LAUNCH(stats_popcount_kernel, grid_for(b.word_off[b.n], 256), 256, 0, st, w.bm, b, num_tuples_dev);
  }
  // T: sort path for grids beyond the bitmap budget
  for (int s : p.sorted) {
    const StatsBatch b = make_batch(p, std::vector<int>{s}, tile_shapes);
    uint64_t total = 1;
    for (int d = 0; d < ndim; ++d) total *= static_cast<uint64_t>(b.grid[0][d]);
    int bits = 0;
    while (bits < 64 && (uint64_t(1) << bits) <= total) ++bits;
    ES_LAUNCH(stats_keys_kernel, grid, 256, 0, st, indices, values, values_dtype, num_entries, p.g, b, w.keys, w.perm);
    uint64_t* k = w.keys;
    uint32_t* v = w.perm;
    ES_TRY(radix_sort_pairs<uint64_t>(&k, &v, w.rb, num_entries, 0, bits, st, error_dev));
    ES_LAUNCH(stats_distinct_kernel, grid_for(num_entries, 256), 256, 0, st, k, num_entries, total,
              num_tuples_dev + s);
  }
  return ES_OK;
}
