// Join + output grouping in one go for contractions of the form
//     lhs (strip..., k) x rhs (k, col...) -> out (strip..., col...)
// i.e. one join key that is the last lhs coordinate and the first rhs
// coordinate, the output coordinates being the other lhs coordinates then
// the other rhs coordinates (execute_sparse's join + _compute_output_coords
// + segment_sum grouping, execution/sparse_dispatch.py:29-82, 174-223,
// 129-171, for "ij,jk->ik", "ijk,kl->ijl", ...).
//
// The lhs relation is in lexicographic coordinate order (its invariant,
// checked here), so a strip's tiles are contiguous and in ascending k. The
// rhs tiles go into a dense (k, col) -> tile table. Output tile (strip s,
// column c) pairs each lhs tile i of strip s whose (k(i), c) table entry
// exists with that rhs tile, in ascending k -- the join's order inside a
// segment (for one rhs tile per pair, rhs ascending). With the hit matrix
// H[c][i] (1 where the entry exists) and its exclusive scan E, segment (s, c)
// has E[c][end(s)] - E[c][start(s)] pairs and the pair of lhs tile i goes to
// offset(s, c) + E[c][i] - E[c][start(s)]: no sort at all.
#include "common.cuh"
#include "scan.cuh"

namespace es {

struct DirectGeom {
  int lhs_nd, rhs_nd;
  int64_t kext;                 // contracted tile extent
  int64_t cext;                 // product of the rhs column extents
  int64_t col_ext[ES_MAX_DIMS]; // rhs grid extents of dims 1..rhs_nd-1
};

struct DirectWs {
  int32_t* table;      // (kext * cext) rhs tile or -1
  uint32_t* colflag;   // (cext) column present
  uint32_t* colrank;   // (cext) exclusive scan of colflag
  uint32_t* colids;    // (cext) present columns in order
  uint32_t* sflag;     // (T_L) strip head
  uint32_t* sexcl;     // (T_L) exclusive scan: strip of a head
  uint32_t* sstart;    // (T_L + 1) first lhs tile of each strip, then T_L
  uint32_t* hit;       // (cext * T_L + 1) H, c-major
  uint32_t* hscan;     // (cext * T_L + 1) E
  uint32_t* counts;    // (T_L * cext) pairs per (strip, column)
  uint32_t* nzflag;    // (T_L * cext)
  uint32_t* segid;     // (T_L * cext) exclusive scan of nzflag
  uint32_t* off;       // (T_L * cext + 1) exclusive scan of counts
  uint32_t* scan;      // scan scratch (largest length)
  uint32_t* ncols;     // (1) present columns
  uint32_t* nstrips;   // (1)
  uint32_t* total;     // (1) scratch totals
  int32_t* bad;        // (1) lhs not in lexicographic order / duplicate coordinates
};

template <typename C>
static void direct_layout(C& c, DirectWs& w, int64_t nl, const DirectGeom& g) {
  const int64_t hn = g.cext * nl + 1;
  const int64_t sc = nl * g.cext;
  w.table = c.template take<int32_t>(g.kext * g.cext);
  w.colflag = c.template take<uint32_t>(g.cext);
  w.colrank = c.template take<uint32_t>(g.cext);
  w.colids = c.template take<uint32_t>(g.cext);
  w.sflag = c.template take<uint32_t>(nl);
  w.sexcl = c.template take<uint32_t>(nl);
  w.sstart = c.template take<uint32_t>(nl + 1);
  w.hit = c.template take<uint32_t>(hn);
  w.hscan = c.template take<uint32_t>(hn);
  w.counts = c.template take<uint32_t>(sc);
  w.nzflag = c.template take<uint32_t>(sc);
  w.segid = c.template take<uint32_t>(sc);
  w.off = c.template take<uint32_t>(sc + 1);
  int64_t mx = hn > sc + 1 ? hn : sc + 1;
  if (g.cext > mx) mx = g.cext;
  if (nl > mx) mx = nl;
  w.scan = c.template take<uint32_t>(scan_scratch_elems(mx));
  w.ncols = c.template take<uint32_t>(1);
  w.nstrips = c.template take<uint32_t>(1);
  w.total = c.template take<uint32_t>(1);
  w.bad = c.template take<int32_t>(1);
}

struct DirectSizer {
  Sizer s;
  template <typename T>
  T* take(int64_t n) {
    s.take<T>(n);
    return nullptr;
  }
};

__device__ __forceinline__ int64_t col_linear(const int32_t* row, const DirectGeom& g, bool* ok) {
  int64_t c = 0;
  for (int d = 1; d < g.rhs_nd; ++d) {
    const int64_t x = row[d];
    if (x < 0 || x >= g.col_ext[d - 1]) *ok = false;
    c = c * g.col_ext[d - 1] + x;
  }
  return c;
}

__global__ void direct_table_kernel(const int32_t* __restrict__ rc, int64_t nr, DirectGeom g,
                                    int32_t* __restrict__ table, uint32_t* __restrict__ colflag, int32_t* err) {
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < nr; j += (int64_t)gridDim.x * blockDim.x) {
    const int32_t* row = rc + j * g.rhs_nd;
    bool ok = row[0] >= 0 && row[0] < g.kext;
    const int64_t c = col_linear(row, g, &ok);
    if (!ok) {
      if (err) atomicExch(err, ES_ERR_INDEX);
      continue;
    }
    table[static_cast<int64_t>(row[0]) * g.cext + c] = static_cast<int32_t>(j);
    colflag[c] = 1u;
  }
}

__global__ void direct_colids_kernel(const uint32_t* __restrict__ colflag, const uint32_t* __restrict__ colrank,
                                     int64_t cext, uint32_t* __restrict__ colids) {
  for (int64_t c = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < cext; c += (int64_t)gridDim.x * blockDim.x)
    if (colflag[c]) colids[colrank[c]] = static_cast<uint32_t>(c);
}

// Strip heads of the lhs; flags lhs tiles out of lexicographic order (or
// repeated) and keys outside the contracted range.
__global__ void direct_strips_kernel(const int32_t* __restrict__ lc, int64_t nl, DirectGeom g,
                                     uint32_t* __restrict__ sflag, int32_t* __restrict__ bad, int32_t* err) {
  const int nd = g.lhs_nd;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nl; i += (int64_t)gridDim.x * blockDim.x) {
    const int32_t* row = lc + i * nd;
    if (row[nd - 1] < 0 || row[nd - 1] >= g.kext) {
      if (err) atomicExch(err, ES_ERR_INDEX);
    }
    uint32_t head = 1u;
    if (i > 0) {
      const int32_t* prev = row - nd;
      int cmp = 0;  // lexicographic compare over all dims; strip = dims 0..nd-2
      bool same_strip = true;
      for (int d = 0; d < nd && cmp == 0; ++d) {
        if (row[d] != prev[d]) {
          cmp = row[d] > prev[d] ? 1 : -1;
          if (d < nd - 1) same_strip = false;
        }
      }
      if (cmp <= 0) *bad = 1;
      head = same_strip ? 0u : 1u;
    }
    sflag[i] = head;
  }
}

__global__ void direct_sstart_kernel(const uint32_t* __restrict__ sflag, const uint32_t* __restrict__ sexcl,
                                     int64_t nl, const uint32_t* __restrict__ nstrips, uint32_t* __restrict__ sstart) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nl; i += (int64_t)gridDim.x * blockDim.x) {
    if (sflag[i]) sstart[sexcl[i]] = static_cast<uint32_t>(i);
    if (i == 0) sstart[*nstrips] = static_cast<uint32_t>(nl);
  }
}

// H[c][i] = 1 when rhs tile (k(i), column c) exists; H[C][0] (the slot after
// the last used row) = 0 so the scan's tail reads a total.
__global__ void direct_hits_kernel(const int32_t* __restrict__ lc, int64_t nl, DirectGeom g,
                                   const int32_t* __restrict__ table, const uint32_t* __restrict__ colids,
                                   const uint32_t* __restrict__ ncols, uint32_t* __restrict__ hit) {
  const int64_t C = *ncols;
  const int64_t n = C * nl;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e <= n; e += (int64_t)gridDim.x * blockDim.x) {
    if (e == n) {
      hit[e] = 0u;
      continue;
    }
    const int64_t c = e / nl, i = e - c * nl;
    const int32_t k = lc[i * g.lhs_nd + g.lhs_nd - 1];
    uint32_t h = 0u;
    if (k >= 0 && k < g.kext) h = table[static_cast<int64_t>(k) * g.cext + colids[c]] >= 0 ? 1u : 0u;
    hit[e] = h;
  }
}

// Pairs per (strip, present column), strip-major.
__global__ void direct_counts_kernel(const uint32_t* __restrict__ hscan, const uint32_t* __restrict__ sstart,
                                     const uint32_t* __restrict__ nstrips, const uint32_t* __restrict__ ncols,
                                     int64_t nl, uint32_t* __restrict__ counts, uint32_t* __restrict__ nzflag) {
  const int64_t S = *nstrips, C = *ncols;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < S * C; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t s = e / C, c = e - s * C;
    const uint32_t n = hscan[c * nl + sstart[s + 1]] - hscan[c * nl + sstart[s]];
    counts[e] = n;
    nzflag[e] = n ? 1u : 0u;
  }
}

// Counts of the host's sizes: [0] pairs, [1] output tiles.
__global__ void direct_totals_kernel(const uint32_t* __restrict__ off, const uint32_t* __restrict__ segid,
                                     const uint32_t* __restrict__ counts, const uint32_t* __restrict__ nzflag,
                                     const uint32_t* __restrict__ nstrips, const uint32_t* __restrict__ ncols,
                                     const int32_t* __restrict__ bad, int64_t* __restrict__ out) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const int64_t n = static_cast<int64_t>(*nstrips) * (*ncols);
  if (n == 0) {
    out[0] = 0;
    out[1] = 0;
  } else {
    out[0] = static_cast<int64_t>(off[n - 1]) + counts[n - 1];
    out[1] = static_cast<int64_t>(segid[n - 1]) + nzflag[n - 1];
  }
  out[2] = *bad;
}

__global__ void direct_pairs_kernel(const int32_t* __restrict__ lc, int64_t nl, DirectGeom g,
                                    const int32_t* __restrict__ table, const uint32_t* __restrict__ colids,
                                    const uint32_t* __restrict__ ncols, const uint32_t* __restrict__ hit,
                                    const uint32_t* __restrict__ hscan, const uint32_t* __restrict__ sflag,
                                    const uint32_t* __restrict__ sexcl, const uint32_t* __restrict__ sstart,
                                    const uint32_t* __restrict__ off, int32_t* __restrict__ seg_lhs,
                                    int32_t* __restrict__ seg_rhs, int32_t* __restrict__ seg_key) {
  const int64_t C = *ncols;
  const int64_t n = C * nl;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    if (!hit[e]) continue;
    const int64_t c = e / nl, i = e - c * nl;
    const int64_t s = static_cast<int64_t>(sexcl[i]) + sflag[i] - 1;  // strip of lhs tile i
    const int64_t pos = static_cast<int64_t>(off[s * C + c]) + (hscan[e] - hscan[c * nl + sstart[s]]);
    const int32_t k = lc[i * g.lhs_nd + g.lhs_nd - 1];
    seg_lhs[pos] = static_cast<int32_t>(i);
    seg_rhs[pos] = table[static_cast<int64_t>(k) * g.cext + colids[c]];
    if (seg_key) seg_key[pos] = k;
  }
}

__global__ void direct_segments_kernel(const int32_t* __restrict__ lc, DirectGeom g,
                                       const uint32_t* __restrict__ colids, const uint32_t* __restrict__ ncols,
                                       const uint32_t* __restrict__ nstrips, const uint32_t* __restrict__ sstart,
                                       const uint32_t* __restrict__ nzflag, const uint32_t* __restrict__ segid,
                                       const uint32_t* __restrict__ off, int32_t* __restrict__ out_coords,
                                       int64_t* __restrict__ seg_off, int64_t* __restrict__ seg_strip) {
  const int64_t S = *nstrips, C = *ncols;
  const int out_nd = (g.lhs_nd - 1) + (g.rhs_nd - 1);
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < S * C; e += (int64_t)gridDim.x * blockDim.x) {
    if (!nzflag[e]) continue;
    const int64_t s = e / C, c = e - s * C;
    const int64_t o = segid[e];
    const int32_t* row = lc + static_cast<int64_t>(sstart[s]) * g.lhs_nd;
    int32_t* oc = out_coords + o * out_nd;
    for (int d = 0; d < g.lhs_nd - 1; ++d) oc[d] = row[d];
    int64_t cl = colids[c];
    for (int d = g.rhs_nd - 2; d >= 0; --d) {
      oc[g.lhs_nd - 1 + d] = static_cast<int32_t>(cl % g.col_ext[d]);
      cl /= g.col_ext[d];
    }
    seg_off[o] = off[e];
    if (seg_strip) seg_strip[o] = s;
  }
}

__global__ void direct_last_offset_kernel(int64_t* seg_off, int64_t O, int64_t P) {
  if (threadIdx.x == 0 && blockIdx.x == 0) seg_off[O] = P;
}

static int make_direct_geom(int lhs_nd, int rhs_nd, const int64_t* lhs_grid, const int64_t* rhs_grid,
                            DirectGeom* g) {
  if (lhs_nd < 1 || rhs_nd < 1 || lhs_nd > ES_MAX_DIMS || rhs_nd > ES_MAX_DIMS) return ES_ERR_INVALID;
  if (lhs_nd + rhs_nd - 2 < 1) return ES_ERR_UNSUPPORTED;
  g->lhs_nd = lhs_nd;
  g->rhs_nd = rhs_nd;
  g->kext = lhs_grid[lhs_nd - 1] > rhs_grid[0] ? lhs_grid[lhs_nd - 1] : rhs_grid[0];
  g->cext = 1;
  for (int d = 1; d < rhs_nd; ++d) {
    g->col_ext[d - 1] = rhs_grid[d];
    g->cext *= rhs_grid[d];
  }
  if (g->kext <= 0 || g->cext <= 0) return ES_ERR_INVALID;
  return ES_OK;
}

}  // namespace es

using namespace es;

extern "C" size_t es_direct_workspace_size(int64_t n_lhs, int lhs_ndim, int64_t n_rhs, int rhs_ndim,
                                           const int64_t* lhs_grid, const int64_t* rhs_grid) {
  DirectGeom g;
  if (make_direct_geom(lhs_ndim, rhs_ndim, lhs_grid, rhs_grid, &g) != ES_OK) return 0;
  (void)n_rhs;
  DirectSizer s;
  DirectWs w;
  direct_layout(s, w, n_lhs, g);
  return s.s.used + 256;
}

extern "C" int es_direct_plan(const int32_t* lhs_coords, int64_t n_lhs, int lhs_ndim, const int32_t* rhs_coords,
                              int64_t n_rhs, int rhs_ndim, const int64_t* lhs_grid, const int64_t* rhs_grid,
                              void* workspace, size_t workspace_bytes, int64_t* counts_dev, int32_t* error_dev,
                              void* stream) {
  cudaStream_t st = as_stream(stream);
  DirectGeom g;
  ES_TRY(make_direct_geom(lhs_ndim, rhs_ndim, lhs_grid, rhs_grid, &g));
  if (n_lhs <= 0 || n_rhs <= 0) return ES_ERR_INVALID;
  if (g.cext * n_lhs + 1 >= static_cast<int64_t>(UINT32_MAX) || g.kext * g.cext >= static_cast<int64_t>(INT32_MAX) ||
      n_rhs >= static_cast<int64_t>(INT32_MAX))
    return ES_ERR_UNSUPPORTED;
  Carver cv(workspace, workspace_bytes);
  DirectWs w;
  direct_layout(cv, w, n_lhs, g);
  if (cv.overflow) return ES_ERR_WORKSPACE;
  if (cudaMemsetAsync(w.table, 0xFF, g.kext * g.cext * sizeof(int32_t), st) != cudaSuccess) return ES_ERR_CUDA;
  if (cudaMemsetAsync(w.colflag, 0, g.cext * sizeof(uint32_t), st) != cudaSuccess) return ES_ERR_CUDA;
  if (cudaMemsetAsync(w.bad, 0, sizeof(int32_t), st) != cudaSuccess) return ES_ERR_CUDA;
  ES_LAUNCH(direct_table_kernel, grid_for(n_rhs, 256), 256, 0, st, rhs_coords, n_rhs, g, w.table, w.colflag,
            error_dev);
  ES_TRY(exclusive_scan<uint32_t>(w.colflag, w.colrank, g.cext, w.ncols, w.scan, st));
  ES_LAUNCH(direct_colids_kernel, grid_for(g.cext, 256), 256, 0, st, w.colflag, w.colrank, g.cext, w.colids);
  ES_LAUNCH(direct_strips_kernel, grid_for(n_lhs, 256), 256, 0, st, lhs_coords, n_lhs, g, w.sflag, w.bad, error_dev);
  ES_TRY(exclusive_scan<uint32_t>(w.sflag, w.sexcl, n_lhs, w.nstrips, w.scan, st));
  ES_LAUNCH(direct_sstart_kernel, grid_for(n_lhs, 256), 256, 0, st, w.sflag, w.sexcl, n_lhs, w.nstrips, w.sstart);
  const int64_t hn = g.cext * n_lhs + 1;  // the used part is ncols * n_lhs + 1 (device count)
  ES_LAUNCH(direct_hits_kernel, grid_for(hn, 256), 256, 0, st, lhs_coords, n_lhs, g, w.table, w.colids, w.ncols,
            w.hit);
  ES_TRY(exclusive_scan<uint32_t>(w.hit, w.hscan, hn, w.total, w.scan, st));
  const int64_t sc = n_lhs * g.cext;
  ES_LAUNCH(direct_counts_kernel, grid_for(sc, 256), 256, 0, st, w.hscan, w.sstart, w.nstrips, w.ncols, n_lhs,
            w.counts, w.nzflag);
  // the scans run over the upper bound; entries past nstrips * ncols are not
  // written and only ever enter prefixes past the used length
  ES_TRY(exclusive_scan<uint32_t>(w.counts, w.off, sc, w.total, w.scan, st));
  ES_TRY(exclusive_scan<uint32_t>(w.nzflag, w.segid, sc, w.total, w.scan, st));
  ES_LAUNCH(direct_totals_kernel, 1, 32, 0, st, w.off, w.segid, w.counts, w.nzflag, w.nstrips, w.ncols, w.bad,
            counts_dev);
  return ES_OK;
}

extern "C" int es_direct_fill(const int32_t* lhs_coords, int64_t n_lhs, int lhs_ndim, int rhs_ndim,
                              const int64_t* lhs_grid, const int64_t* rhs_grid, void* workspace,
                              size_t workspace_bytes, int64_t num_pairs, int64_t num_segments, int32_t* out_coords,
                              int64_t* seg_offsets, int32_t* seg_lhs, int32_t* seg_rhs, int64_t* seg_strip,
                              int32_t* seg_key, void* stream) {
  cudaStream_t st = as_stream(stream);
  DirectGeom g;
  ES_TRY(make_direct_geom(lhs_ndim, rhs_ndim, lhs_grid, rhs_grid, &g));
  if (n_lhs <= 0) return ES_ERR_INVALID;
  Carver cv(workspace, workspace_bytes);
  DirectWs w;
  direct_layout(cv, w, n_lhs, g);
  if (cv.overflow) return ES_ERR_WORKSPACE;
  const int64_t hn = g.cext * n_lhs;
  if (num_pairs > 0)
    ES_LAUNCH(direct_pairs_kernel, grid_for(hn, 256), 256, 0, st, lhs_coords, n_lhs, g, w.table, w.colids, w.ncols,
              w.hit, w.hscan, w.sflag, w.sexcl, w.sstart, w.off, seg_lhs, seg_rhs, seg_key);
  const int64_t sc = n_lhs * g.cext;
  if (num_segments > 0)
    ES_LAUNCH(direct_segments_kernel, grid_for(sc, 256), 256, 0, st, lhs_coords, g, w.colids, w.ncols, w.nstrips,
              w.sstart, w.nzflag, w.segid, w.off, out_coords, seg_offsets, seg_strip);
  ES_LAUNCH(direct_last_offset_kernel, 1, 32, 0, st, seg_offsets, num_segments, num_pairs);
  return ES_OK;
}
