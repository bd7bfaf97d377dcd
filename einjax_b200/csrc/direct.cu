// Join + output grouping in one go for contractions of the form
//     lhs (batch..., strip..., k) x rhs (batch..., k, col...)
//         -> out (batch..., strip..., col...)
// i.e. join keys that pair the leading batch coordinates of both sides and
// the last lhs coordinate with the rhs coordinate after the batch ones, the
// output coordinates being the other lhs coordinates then the other rhs
// coordinates (execute_sparse's join + _compute_output_coords + segment_sum
// grouping, execution/sparse_dispatch.py:29-82, 174-223, 129-171, for
// "ij,jk->ik", "ijk,kl->ijl", "bij,bjk->bik", ...).
//
// Both relations are in lexicographic coordinate order (their invariant,
// checked here), so a strip -- the lhs coordinates but the last, batch
// included -- has its tiles contiguous and in ascending k. The rhs tiles go
// into a dense ((batch, k), col) -> tile table. Output tile (strip s, column
// c) pairs each lhs tile i of strip s whose ((batch, k)(i), c) table entry
// exists with that rhs tile, in ascending k -- the join's order inside a
// segment (rhs-major over an rhs in lexicographic order).
//
// Positions without a sort: the lhs tiles are cut into chunks of 32 (one
// warp). For every present column c a warp ballots which tiles of its chunk
// hit, giving a 32-bit hit mask per (column, chunk) and its popcount; one
// exclusive scan of the popcounts (column-major) gives G_c(t) = hits of
// column c among tiles [0, t) (plus a per-column constant) for any t, as the
// chunk's scanned count plus the popcount of its mask below t. Segment
// (s, c) then holds G_c(end s) - G_c(start s) pairs, and the pair of tile i
// goes to offset(s, c) + G_c(i) - G_c(start s). Nothing of size pairs or
// (columns x lhs tiles) is materialised besides the pair arrays themselves:
// the masks are (columns x tiles / 32) words.
#include <cstdlib>

#include "common.cuh"
#include "scan.cuh"

namespace es {

struct DirectGeom {
  int lhs_nd, rhs_nd, nb;       // nb: leading batch dims joined pairwise
  int64_t kx;                   // contracted tile extent
  int64_t kext;                 // table rows: batch extents x kx
  int64_t cext;                 // product of the rhs column extents
  int64_t sext;                 // product of the lhs strip extents (dims 0..lhs_nd-2)
  int64_t bat_ext[ES_MAX_DIMS]; // grid extents of the batch dims
  int64_t col_ext[ES_MAX_DIMS]; // rhs grid extents of dims nb+1..rhs_nd-1
};

struct DirectWs {
  int32_t* table;      // (kext * cext) rhs tile or -1
  uint32_t* colflag;   // (cext) column present
  uint32_t* colrank;   // (cext) exclusive scan of colflag
  uint32_t* colids;    // (cext) present columns in order
  uint32_t* sflag;     // (T_L) strip head
  uint32_t* sexcl;     // (T_L) exclusive scan: strip of a head
  uint32_t* sstart;    // (T_L + 1) first lhs tile of each strip, then T_L
  uint32_t* mask;      // (CB * (NCH + 1)) hit mask per (present column, 32-tile chunk), column-major
  uint32_t* ccnt;      // (CB * (NCH + 1)) popcount of mask
  uint32_t* cscan;     // (CB * (NCH + 1)) exclusive scan of ccnt
  uint64_t* cnz;       // (SC) per (strip, present column), strip-major: pairs | (pairs > 0) << 32
  uint64_t* pos;       // (SC) exclusive scan of cnz: first pair | output tile index << 32
  uint32_t* gstart;    // (SC) G_c(first tile of the strip)
  uint32_t* scan_c;    // scratch of the column-flag scan
  uint32_t* scan_s;    // scratch of the strip-head scan
  uint32_t* scan_m;    // scratch of the mask-count scan
  uint32_t* scan_p;    // scratch of the pair-count scan (64-bit values)
  uint32_t* ncols;     // (1) present columns
  uint32_t* nstrips;   // (1)
  uint32_t* total;     // (1) scratch totals
  uint64_t* total64;   // (1)
  int32_t* bad;        // (1) a relation not in lexicographic order / repeated coordinates
};

// Upper bound of present columns: min(T_R, column extent).
static int64_t direct_col_bound(const DirectGeom& g, int64_t nr) { return nr < g.cext ? nr : g.cext; }

// Upper bound of strips x present columns: strips <= min(T_L, strip extent).
static int64_t direct_sc_bound(const DirectGeom& g, int64_t nl, int64_t nr) {
  const int64_t s = nl < g.sext ? nl : g.sext;
  return s * direct_col_bound(g, nr);
}

// 32-tile chunks of the lhs plus one empty chunk per column (so that
// G_c(T_L) reads a chunk of its own when T_L is a multiple of 32).
static int64_t direct_chunks(int64_t nl) { return (nl + 31) / 32 + 1; }

template <typename C>
static void direct_layout(C& c, DirectWs& w, int64_t nl, int64_t nr, const DirectGeom& g) {
  const int64_t sc = direct_sc_bound(g, nl, nr);
  w.table = c.template take<int32_t>(g.kext * g.cext);
  w.colflag = c.template take<uint32_t>(g.cext);
  w.colrank = c.template take<uint32_t>(g.cext);
  w.colids = c.template take<uint32_t>(g.cext);
  w.sflag = c.template take<uint32_t>(nl);
  w.sexcl = c.template take<uint32_t>(nl);
  w.sstart = c.template take<uint32_t>(nl + 1);
  const int64_t hm = direct_col_bound(g, nr) * direct_chunks(nl);
  w.mask = c.template take<uint32_t>(hm);
  w.ccnt = c.template take<uint32_t>(hm);
  w.cscan = c.template take<uint32_t>(hm);
  w.cnz = c.template take<uint64_t>(sc);
  w.pos = c.template take<uint64_t>(sc);
  w.gstart = c.template take<uint32_t>(sc);
  // one scratch per scan, so the init launch clears all four up front
  w.scan_c = c.template take<uint32_t>(scan_scratch_elems(g.cext));
  w.scan_s = c.template take<uint32_t>(scan_scratch_elems(nl));
  w.scan_m = c.template take<uint32_t>(scan_scratch_elems(hm));
  w.scan_p = c.template take<uint32_t>(2 * scan_scratch_elems(sc));
  w.ncols = c.template take<uint32_t>(1);
  w.nstrips = c.template take<uint32_t>(1);
  w.total = c.template take<uint32_t>(1);
  w.total64 = c.template take<uint64_t>(1);
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

// Table row of a tile: its batch coordinates (row[0..nb)) then its
// contracted coordinate row[kdim], linearised; -1 when out of range.
__device__ __forceinline__ int64_t key_of(const int32_t* row, int kdim, const DirectGeom& g) {
  int64_t key = 0;
  for (int d = 0; d < g.nb; ++d) {
    const int64_t x = row[d];
    if (x < 0 || x >= g.bat_ext[d]) return -1;
    key = key * g.bat_ext[d] + x;
  }
  const int64_t k = row[kdim];
  if (k < 0 || k >= g.kx) return -1;
  return key * g.kx + k;
}

__device__ __forceinline__ int64_t col_linear(const int32_t* row, const DirectGeom& g, bool* ok) {
  int64_t c = 0;
  for (int d = g.nb + 1; d < g.rhs_nd; ++d) {
    const int64_t x = row[d];
    const int64_t e = g.col_ext[d - g.nb - 1];
    if (x < 0 || x >= e) *ok = false;
    c = c * e + x;
  }
  return c;
}

// Lexicographic comparison of two coordinate rows: -1, 0, 1; *first_diff =
// the first dimension where they differ (nd when equal).
__device__ __forceinline__ int lex_cmp(const int32_t* a, const int32_t* b, int nd, int* first_diff) {
  for (int d = 0; d < nd; ++d)
    if (a[d] != b[d]) {
      *first_diff = d;
      return a[d] > b[d] ? 1 : -1;
    }
  *first_diff = nd;
  return 0;
}

// Clears the table (-1), the column flags, the order flag and the caller's
// status slot.
__global__ void direct_init_kernel(int32_t* __restrict__ table, int64_t tn, uint32_t* __restrict__ colflag,
                                   int64_t cext, int32_t* __restrict__ bad, int32_t* __restrict__ err,
                                   ZeroSpans zs) {
  zero_spans(zs);
  const int64_t n = tn > cext ? tn : cext;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    if (i < tn) table[i] = -1;
    if (i < cext) colflag[i] = 0u;
    if (i == 0) {
      *bad = 0;
      if (err) *err = 0;
    }
  }
}

// Threads [0, nr): rhs tile j into the table (flags an rhs out of
// lexicographic order). Threads [nr, nr + nl): strip head flag of lhs tile
// i (flags lhs tiles out of lexicographic order or repeated, and keys
// outside the table).
// (Each phase below is a device function over threads t0, t0 + nt, ...: the
// multi-CTA kernels call it with the grid's threads, the one-CTA plan for
// small inputs with the block's.)
__device__ __forceinline__ void direct_inputs_body(const int32_t* __restrict__ rc, int64_t nr,
                                                   const int32_t* __restrict__ lc, int64_t nl, const DirectGeom& g,
                                                   int32_t* __restrict__ table, uint32_t* __restrict__ colflag,
                                                   uint32_t* __restrict__ sflag, int32_t* __restrict__ bad,
                                                   int32_t* err, int64_t t0, int64_t nt) {
  for (int64_t q = t0; q < nr + nl; q += nt) {
    if (q < nr) {
      const int64_t j = q;
      const int32_t* row = rc + j * g.rhs_nd;
      int fd;
      if (j > 0 && lex_cmp(row, row - g.rhs_nd, g.rhs_nd, &fd) <= 0) *bad = 1;
      const int64_t key = key_of(row, g.nb, g);
      bool ok = key >= 0;
      const int64_t c = col_linear(row, g, &ok);
      if (!ok) {
        if (err) atomicExch(err, ES_ERR_INDEX);
        continue;
      }
      table[key * g.cext + c] = static_cast<int32_t>(j);
      colflag[c] = 1u;
    } else {
      const int64_t i = q - nr;
      const int nd = g.lhs_nd;
      const int32_t* row = lc + i * nd;
      if (key_of(row, nd - 1, g) < 0) {
        if (err) atomicExch(err, ES_ERR_INDEX);
      }
      uint32_t head = 1u;
      if (i > 0) {
        int fd;
        if (lex_cmp(row, row - nd, nd, &fd) <= 0) *bad = 1;
        head = fd < nd - 1 ? 1u : 0u;  // strip = dims 0..nd-2
      }
      sflag[i] = head;
    }
  }
}

__global__ void direct_inputs_kernel(const int32_t* __restrict__ rc, int64_t nr, const int32_t* __restrict__ lc,
                                     int64_t nl, DirectGeom g, int32_t* __restrict__ table,
                                     uint32_t* __restrict__ colflag, uint32_t* __restrict__ sflag,
                                     int32_t* __restrict__ bad, int32_t* err) {
  direct_inputs_body(rc, nr, lc, nl, g, table, colflag, sflag, bad, err, blockIdx.x * (int64_t)blockDim.x + threadIdx.x,
                     (int64_t)gridDim.x * blockDim.x);
}

// Threads [0, cext): present column ids in order; threads [0, nl): first lhs
// tile of each strip, then sstart[nstrips] = nl.
__device__ __forceinline__ void direct_index_body(const uint32_t* __restrict__ colflag,
                                                  const uint32_t* __restrict__ colrank, int64_t cext,
                                                  uint32_t* __restrict__ colids, const uint32_t* __restrict__ sflag,
                                                  const uint32_t* __restrict__ sexcl, int64_t nl,
                                                  const uint32_t* __restrict__ nstrips, uint32_t* __restrict__ sstart,
                                                  int64_t t0, int64_t nt) {
  const int64_t n = nl > cext ? nl : cext;
  for (int64_t i = t0; i < n; i += nt) {
    if (i < cext && colflag[i]) colids[colrank[i]] = static_cast<uint32_t>(i);
    if (i < nl) {
      if (sflag[i]) sstart[sexcl[i]] = static_cast<uint32_t>(i);
      if (i == 0) sstart[*nstrips] = static_cast<uint32_t>(nl);
    }
  }
}

__global__ void direct_index_kernel(const uint32_t* __restrict__ colflag, const uint32_t* __restrict__ colrank,
                                    int64_t cext, uint32_t* __restrict__ colids, const uint32_t* __restrict__ sflag,
                                    const uint32_t* __restrict__ sexcl, int64_t nl,
                                    const uint32_t* __restrict__ nstrips, uint32_t* __restrict__ sstart) {
  direct_index_body(colflag, colrank, cext, colids, sflag, sexcl, nl, nstrips, sstart,
                    blockIdx.x * (int64_t)blockDim.x + threadIdx.x, (int64_t)gridDim.x * blockDim.x);
}

// Table lookup of a tile's key for column col: the rhs tile or -1. NC: read
// through the read-only path, valid when an earlier launch wrote the table
// (not within the kernel that writes it).
template <bool NC = true>
__device__ __forceinline__ int32_t direct_lookup(const DirectGeom& g, const int32_t* __restrict__ table, int64_t key,
                                                 int64_t col) {
  if (key < 0) return -1;
  return NC ? __ldg(table + key * g.cext + col) : table[key * g.cext + col];
}

// Table row of lhs tile i (-1 out of range); *k = its contracted coordinate.
__device__ __forceinline__ int64_t direct_key(const int32_t* __restrict__ lc, const DirectGeom& g, int64_t i,
                                              int32_t* k) {
  const int nd = g.lhs_nd;
  const int32_t* row = lc + i * nd;
  *k = __ldg(row + nd - 1);
  if (g.nb == 0) return (*k >= 0 && *k < g.kx) ? *k : -1;
  return key_of(row, nd - 1, g);
}

// Columns one warp looks up per unit of work (independent loads in flight).
constexpr int kDirCols = 8;

// Hit masks: one warp per (32-tile chunk, group of kDirCols present
// columns); chunks run to nch inclusive, the last one past every tile.
template <bool NC>
__device__ __forceinline__ void direct_masks_body(const int32_t* __restrict__ lc, int64_t nl, const DirectGeom& g,
                                                  const int32_t* __restrict__ table,
                                                  const uint32_t* __restrict__ colids,
                                                  const uint32_t* __restrict__ ncols, int64_t nchp1,
                                                  uint32_t* __restrict__ mask, uint32_t* __restrict__ ccnt, int64_t t0,
                                                  int64_t nt) {
  const int64_t C = *ncols;
  const int64_t groups = (C + kDirCols - 1) / kDirCols;
  const int lane = threadIdx.x & 31;
  const int64_t nw = nt >> 5;
  for (int64_t u = t0 >> 5; u < nchp1 * groups; u += nw) {
    const int64_t ch = u / groups, c0 = (u - ch * groups) * kDirCols;
    const int64_t i = ch * 32 + lane;
    int32_t k;
    const int64_t key = i < nl ? direct_key(lc, g, i, &k) : -1;
    int32_t r[kDirCols];
#pragma unroll
    for (int j = 0; j < kDirCols; ++j)
      r[j] = c0 + j < C ? direct_lookup<NC>(g, table, key, colids[c0 + j]) : -1;
#pragma unroll
    for (int j = 0; j < kDirCols; ++j) {
      const uint32_t m = __ballot_sync(0xffffffffu, r[j] >= 0);
      if (lane == j && c0 + j < C) {
        mask[(c0 + j) * nchp1 + ch] = m;
        ccnt[(c0 + j) * nchp1 + ch] = __popc(m);
      }
    }
  }
}

__global__ void direct_masks_kernel(const int32_t* __restrict__ lc, int64_t nl, DirectGeom g,
                                    const int32_t* __restrict__ table, const uint32_t* __restrict__ colids,
                                    const uint32_t* __restrict__ ncols, int64_t nchp1, uint32_t* __restrict__ mask,
                                    uint32_t* __restrict__ ccnt) {
  direct_masks_body<true>(lc, nl, g, table, colids, ncols, nchp1, mask, ccnt,
                          blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x,
                          static_cast<int64_t>(gridDim.x) * blockDim.x);
}

// G_c(t): hits of present column c among lhs tiles [0, t), plus a constant
// per column.
__device__ __forceinline__ uint32_t direct_g(const uint32_t* __restrict__ mask, const uint32_t* __restrict__ cscan,
                                             int64_t nchp1, int64_t c, int64_t t) {
  const int64_t idx = c * nchp1 + (t >> 5);
  return cscan[idx] + __popc(mask[idx] & ((1u << (t & 31)) - 1u));
}

// Pairs per (strip, present column), strip-major, one thread per entry.
__device__ __forceinline__ void direct_counts_body(const uint32_t* __restrict__ mask,
                                                   const uint32_t* __restrict__ cscan, int64_t nchp1,
                                                   const uint32_t* __restrict__ ncols,
                                                   const uint32_t* __restrict__ nstrips,
                                                   const uint32_t* __restrict__ sstart, uint64_t* __restrict__ cnz,
                                                   uint32_t* __restrict__ gstart, int64_t t0, int64_t nt) {
  const int64_t S = *nstrips, C = *ncols;
  for (int64_t e = t0; e < S * C; e += nt) {
    const int64_t s = e / C, c = e - s * C;
    const uint32_t ga = direct_g(mask, cscan, nchp1, c, sstart[s]);
    const uint32_t n = direct_g(mask, cscan, nchp1, c, sstart[s + 1]) - ga;
    cnz[e] = static_cast<uint64_t>(n) | (n ? (1ull << 32) : 0ull);
    gstart[e] = ga;
  }
}

__global__ void direct_counts_kernel(const uint32_t* __restrict__ mask, const uint32_t* __restrict__ cscan,
                                     int64_t nchp1, const uint32_t* __restrict__ ncols,
                                     const uint32_t* __restrict__ nstrips, const uint32_t* __restrict__ sstart,
                                     uint64_t* __restrict__ cnz, uint32_t* __restrict__ gstart) {
  direct_counts_body(mask, cscan, nchp1, ncols, nstrips, sstart, cnz, gstart,
                     blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x,
                     static_cast<int64_t>(gridDim.x) * blockDim.x);
}

// Counts of the host's sizes: [0] pairs, [1] output tiles, [2] out of order.
__device__ __forceinline__ void direct_totals_body(const uint64_t* __restrict__ pos,
                                                   const uint64_t* __restrict__ cnz,
                                                   const uint32_t* __restrict__ nstrips,
                                                   const uint32_t* __restrict__ ncols, const int32_t* __restrict__ bad,
                                                   int64_t* __restrict__ out) {
  const int64_t n = static_cast<int64_t>(*nstrips) * (*ncols);
  const uint64_t t = n == 0 ? 0ull : pos[n - 1] + cnz[n - 1];
  out[0] = static_cast<int64_t>(t & 0xFFFFFFFFull);
  out[1] = static_cast<int64_t>(t >> 32);
  out[2] = *bad;
}

__global__ void direct_totals_kernel(const uint64_t* __restrict__ pos, const uint64_t* __restrict__ cnz,
                                     const uint32_t* __restrict__ nstrips, const uint32_t* __restrict__ ncols,
                                     const int32_t* __restrict__ bad, int64_t* __restrict__ out) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  direct_totals_body(pos, cnz, nstrips, ncols, bad, out);
}

// Fill. Threads first write the output-tile records of the (strip, present
// column) entries with pairs (coordinates, first pair, strip; the last
// record also writes seg_off[O] = P). Then, one warp per (32-tile chunk,
// column group) as in the mask pass, a hit of tile i for column c goes to
// first(s, c) + G_c(i) - G_c(start s).
__global__ void direct_pairs_kernel(const int32_t* __restrict__ lc, int64_t nl, DirectGeom g,
                                    const int32_t* __restrict__ table, const uint32_t* __restrict__ colids,
                                    const uint32_t* __restrict__ ncols, const uint32_t* __restrict__ nstrips,
                                    const uint32_t* __restrict__ sstart, int64_t nchp1,
                                    const uint32_t* __restrict__ cscan, const uint32_t* __restrict__ sflag,
                                    const uint32_t* __restrict__ sexcl, const uint64_t* __restrict__ cnz,
                                    const uint64_t* __restrict__ posw, const uint32_t* __restrict__ gstart,
                                    int64_t num_pairs, int64_t num_segments, int32_t* __restrict__ seg_lhs,
                                    int32_t* __restrict__ seg_rhs, int32_t* __restrict__ seg_key,
                                    int32_t* __restrict__ out_coords, int64_t* __restrict__ seg_off,
                                    int64_t* __restrict__ seg_strip) {
  const int64_t C = *ncols;
  {
    const int64_t S = *nstrips;
    const int ncd = g.rhs_nd - 1 - g.nb;  // rhs column dims
    const int out_nd = (g.lhs_nd - 1) + ncd;
    for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < S * C;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      if ((cnz[e] & 0xFFFFFFFFull) == 0) continue;
      const int64_t s = e / C, c = e - s * C;
      const int64_t o = static_cast<int64_t>(posw[e] >> 32);
      const int32_t* row = lc + static_cast<int64_t>(sstart[s]) * g.lhs_nd;
      int32_t* oc = out_coords + o * out_nd;
      for (int d = 0; d < g.lhs_nd - 1; ++d) oc[d] = row[d];
      int64_t cl = colids[c];
      for (int d = ncd - 1; d >= 0; --d) {
        oc[g.lhs_nd - 1 + d] = static_cast<int32_t>(cl % g.col_ext[d]);
        cl /= g.col_ext[d];
      }
      seg_off[o] = static_cast<int64_t>(posw[e] & 0xFFFFFFFFull);
      if (seg_strip) seg_strip[o] = s;
      if (o + 1 == num_segments) seg_off[num_segments] = num_pairs;
    }
  }
  const int64_t groups = (C + kDirCols - 1) / kDirCols;
  const int lane = threadIdx.x & 31;
  const uint32_t below = (1u << lane) - 1u;
  const int64_t nch = nchp1 - 1;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t u = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; u < nch * groups; u += nw) {
    const int64_t ch = u / groups, c0 = (u - ch * groups) * kDirCols;
    const int64_t i = ch * 32 + lane;
    int32_t k = -1;
    int64_t key = -1, s = 0;
    if (i < nl) {
      key = direct_key(lc, g, i, &k);
      s = static_cast<int64_t>(sexcl[i]) + sflag[i] - 1;
    }
    int32_t r[kDirCols];
#pragma unroll
    for (int j = 0; j < kDirCols; ++j)
      r[j] = c0 + j < C ? direct_lookup(g, table, key, colids[c0 + j]) : -1;
    // the (strip, column) bases of every hit first, all loads in flight together
    int64_t pb[kDirCols];
    uint32_t gb[kDirCols];
#pragma unroll
    for (int j = 0; j < kDirCols; ++j) {
      pb[j] = 0;
      gb[j] = 0;
      if (r[j] >= 0) {
        const int64_t c = c0 + j;
        const int64_t e = s * C + c;
        pb[j] = static_cast<int64_t>(posw[e] & 0xFFFFFFFFull);
        gb[j] = cscan[c * nchp1 + ch] - gstart[e];
      }
    }
#pragma unroll
    for (int j = 0; j < kDirCols; ++j) {
      const uint32_t m = __ballot_sync(0xffffffffu, r[j] >= 0);
      if (r[j] >= 0) {
        // first(s, c) + G_c(i) - G_c(start s), as uint32 (non-negative for a hit)
        const int64_t p = pb[j] + static_cast<uint32_t>(gb[j] + __popc(m & below));
        seg_lhs[p] = static_cast<int32_t>(i);
        seg_rhs[p] = r[j];
        if (seg_key) seg_key[p] = k;
      }
    }
  }
}

// Exclusive scan of n values by one CTA (every thread of the block calls
// it): thread t sums a contiguous run, the runs' sums are scanned across the
// block, then each run is written. In place allowed; *total gets the sum.
template <typename T>
__device__ void block_exclusive_scan(const T* in, T* out, int64_t n, T* total, T* sh) {
  const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31, warp = tid >> 5, nwarp = nth >> 5;
  const int64_t per = (n + nth - 1) / nth;
  const int64_t b = min(n, static_cast<int64_t>(tid) * per), e = min(n, b + per);
  T s = 0;
  for (int64_t i = b; i < e; ++i) s += in[i];
  T incl = s;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) sh[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const T v = lane < nwarp ? sh[lane] : T(0);
    T iv = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const T u = __shfl_up_sync(0xffffffffu, iv, o);
      if (lane >= o) iv += u;
    }
    if (lane < nwarp) sh[lane] = iv - v;
  }
  __syncthreads();
  T run = sh[warp] + incl - s;
  if (tid == nth - 1 && total) *total = run + s;
  for (int64_t i = b; i < e; ++i) {
    const T v = in[i];
    out[i] = run;
    run += v;
  }
  __syncthreads();
}

// The whole plan in one CTA for small inputs: the phases of the multi-CTA
// launches, separated by block barriers (which order the global writes of
// one phase before the next phase's reads), with block scans. The table is
// written inside this kernel, so its lookups use plain loads.
constexpr int kDirSmallThreads = 1024;
constexpr int64_t kDirSmallTiles = 8192;   // n_lhs + n_rhs at most
constexpr int64_t kDirSmallTable = 65536;  // table, mask and (strip, column) entries at most

__global__ void __launch_bounds__(kDirSmallThreads) direct_plan_small_kernel(
    const int32_t* __restrict__ rc, int64_t nr, const int32_t* __restrict__ lc, int64_t nl, DirectGeom g, DirectWs w,
    int64_t tn, int64_t nchp1, int64_t* __restrict__ counts, int32_t* err) {
  __shared__ uint32_t sh32[32];
  __shared__ uint64_t sh64[32];
  const int64_t t0 = threadIdx.x, nt = blockDim.x;
  const int64_t ni = tn > g.cext ? tn : g.cext;
  for (int64_t i = t0; i < ni; i += nt) {
    if (i < tn) w.table[i] = -1;
    if (i < g.cext) w.colflag[i] = 0u;
  }
  if (t0 == 0) {
    *w.bad = 0;
    if (err) *err = 0;
  }
  __syncthreads();
  direct_inputs_body(rc, nr, lc, nl, g, w.table, w.colflag, w.sflag, w.bad, err, t0, nt);
  __syncthreads();
  block_exclusive_scan<uint32_t>(w.colflag, w.colrank, g.cext, w.ncols, sh32);
  block_exclusive_scan<uint32_t>(w.sflag, w.sexcl, nl, w.nstrips, sh32);
  direct_index_body(w.colflag, w.colrank, g.cext, w.colids, w.sflag, w.sexcl, nl, w.nstrips, w.sstart, t0, nt);
  __syncthreads();
  direct_masks_body<false>(lc, nl, g, w.table, w.colids, w.ncols, nchp1, w.mask, w.ccnt, t0, nt);
  __syncthreads();
  // only the present columns' masks (column-major) and the (strip, present
  // column) entries are scanned
  block_exclusive_scan<uint32_t>(w.ccnt, w.cscan, static_cast<int64_t>(*w.ncols) * nchp1, w.total, sh32);
  direct_counts_body(w.mask, w.cscan, nchp1, w.ncols, w.nstrips, w.sstart, w.cnz, w.gstart, t0, nt);
  __syncthreads();
  block_exclusive_scan<uint64_t>(w.cnz, w.pos, static_cast<int64_t>(*w.nstrips) * (*w.ncols), w.total64, sh64);
  if (t0 == 0) direct_totals_body(w.pos, w.cnz, w.nstrips, w.ncols, w.bad, counts);
}

static int make_direct_geom(int lhs_nd, int rhs_nd, int nb, const int64_t* lhs_grid, const int64_t* rhs_grid,
                            DirectGeom* g) {
  if (lhs_nd < 1 || rhs_nd < 1 || lhs_nd > ES_MAX_DIMS || rhs_nd > ES_MAX_DIMS) return ES_ERR_INVALID;
  if (nb < 0 || nb >= lhs_nd || nb >= rhs_nd) return ES_ERR_INVALID;
  if (lhs_nd + rhs_nd - 2 - nb < 1) return ES_ERR_UNSUPPORTED;
  g->lhs_nd = lhs_nd;
  g->rhs_nd = rhs_nd;
  g->nb = nb;
  g->kx = lhs_grid[lhs_nd - 1] > rhs_grid[nb] ? lhs_grid[lhs_nd - 1] : rhs_grid[nb];
  g->kext = g->kx;
  for (int d = 0; d < nb; ++d) {
    g->bat_ext[d] = lhs_grid[d] > rhs_grid[d] ? lhs_grid[d] : rhs_grid[d];
    if (g->bat_ext[d] <= 0) return ES_ERR_INVALID;
    g->kext *= g->bat_ext[d];
  }
  g->cext = 1;
  for (int d = nb + 1; d < rhs_nd; ++d) {
    g->col_ext[d - nb - 1] = rhs_grid[d];
    g->cext *= rhs_grid[d];
  }
  g->sext = 1;
  for (int d = 0; d + 1 < lhs_nd; ++d) g->sext *= lhs_grid[d];
  if (g->kx <= 0 || g->cext <= 0 || g->sext <= 0) return ES_ERR_INVALID;
  return ES_OK;
}

}  // namespace es

using namespace es;

extern "C" size_t es_direct_workspace_size(int64_t n_lhs, int lhs_ndim, int64_t n_rhs, int rhs_ndim,
                                           int batch_ndim, const int64_t* lhs_grid, const int64_t* rhs_grid) {
  DirectGeom g;
  if (make_direct_geom(lhs_ndim, rhs_ndim, batch_ndim, lhs_grid, rhs_grid, &g) != ES_OK) return 0;
  DirectSizer s;
  DirectWs w;
  direct_layout(s, w, n_lhs, n_rhs, g);
  return s.s.used + 256;
}

extern "C" int es_direct_plan(const int32_t* lhs_coords, int64_t n_lhs, int lhs_ndim, const int32_t* rhs_coords,
                              int64_t n_rhs, int rhs_ndim, int batch_ndim, const int64_t* lhs_grid,
                              const int64_t* rhs_grid, void* workspace, size_t workspace_bytes, int64_t* counts_dev,
                              int32_t* error_dev, void* stream) {
  cudaStream_t st = as_stream(stream);
  DirectGeom g;
  ES_TRY(make_direct_geom(lhs_ndim, rhs_ndim, batch_ndim, lhs_grid, rhs_grid, &g));
  if (n_lhs <= 0 || n_rhs <= 0) return ES_ERR_INVALID;
  // pairs <= n_lhs * present columns must fit the int32 pair arrays
  const int64_t cmax = n_rhs < g.cext ? n_rhs : g.cext;
  if (n_lhs >= static_cast<int64_t>(INT32_MAX) / cmax || g.kext * g.cext >= static_cast<int64_t>(INT32_MAX) ||
      n_rhs >= static_cast<int64_t>(INT32_MAX))
    return ES_ERR_UNSUPPORTED;
  Carver cv(workspace, workspace_bytes);
  DirectWs w;
  direct_layout(cv, w, n_lhs, n_rhs, g);
  if (cv.overflow) return ES_ERR_WORKSPACE;
  const int64_t tn = g.kext * g.cext;
  const int64_t nchp1 = direct_chunks(n_lhs);
  const int64_t cb = direct_col_bound(g, n_rhs);
  const int64_t sc = direct_sc_bound(g, n_lhs, n_rhs);
  // EINSPARSE_NO_SMALL_PLAN: always the multi-launch plan (tests)
  if (n_lhs + n_rhs <= kDirSmallTiles && tn <= kDirSmallTable && cb * nchp1 <= kDirSmallTable &&
      sc <= kDirSmallTable && !std::getenv("EINSPARSE_NO_SMALL_PLAN")) {
    // small inputs: one launch instead of about ten
    ES_LAUNCH(direct_plan_small_kernel, 1, kDirSmallThreads, 0, st, rhs_coords, n_rhs, lhs_coords, n_lhs, g, w, tn,
              nchp1, counts_dev, error_dev);
    return ES_OK;
  }
  ZeroSpans zs = no_zero_spans();
  add_zero_span(zs, w.scan_c, scan_clear_words(g.cext));
  add_zero_span(zs, w.scan_s, scan_clear_words(n_lhs));
  add_zero_span(zs, w.scan_m, scan_clear_words(cb * nchp1));
  add_zero_span(zs, w.scan_p, 2 * scan_clear_words(sc));
  ES_LAUNCH(direct_init_kernel, grid_for(tn > g.cext ? tn : g.cext, 256), 256, 0, st, w.table, tn, w.colflag, g.cext,
            w.bad, error_dev, zs);
  ES_LAUNCH(direct_inputs_kernel, grid_for(n_rhs + n_lhs, 256), 256, 0, st, rhs_coords, n_rhs, lhs_coords, n_lhs, g,
            w.table, w.colflag, w.sflag, w.bad, error_dev);
  ES_TRY(exclusive_scan<uint32_t>(w.colflag, w.colrank, g.cext, w.ncols, w.scan_c, st, nullptr, true));
  ES_TRY(exclusive_scan<uint32_t>(w.sflag, w.sexcl, n_lhs, w.nstrips, w.scan_s, st, nullptr, true));
  ES_LAUNCH(direct_index_kernel, grid_for(n_lhs > g.cext ? n_lhs : g.cext, 256), 256, 0, st, w.colflag, w.colrank,
            g.cext, w.colids, w.sflag, w.sexcl, n_lhs, w.nstrips, w.sstart);
  // hit masks per (present column, chunk), their scan, then the per-(strip,
  // column) counts; the column count lives on the device, so grids cover the
  // upper bound and stride over the used part
  ES_LAUNCH(direct_masks_kernel, grid_for(nchp1 * ((cb + kDirCols - 1) / kDirCols) * 32, 256), 256, 0, st,
            lhs_coords, n_lhs, g, w.table, w.colids, w.ncols, nchp1, w.mask, w.ccnt);
  // column-major: entries of columns past ncols are not written and only
  // ever enter prefixes past the used part
  ES_TRY(exclusive_scan<uint32_t>(w.ccnt, w.cscan, cb * nchp1, w.total, w.scan_m, st, nullptr, true));
  ES_LAUNCH(direct_counts_kernel, grid_for(sc, 256), 256, 0, st, w.mask, w.cscan, nchp1, w.ncols, w.nstrips,
            w.sstart, w.cnz, w.gstart);
  // one scan gives first pairs (low word) and output tile indices (high);
  // it runs over the upper bound: entries past nstrips * ncols are not
  // written and only ever enter prefixes past the used length
  ES_TRY(exclusive_scan<uint64_t>(w.cnz, w.pos, sc, w.total64, reinterpret_cast<uint64_t*>(w.scan_p), st, nullptr,
                                  true));
  ES_LAUNCH(direct_totals_kernel, 1, 32, 0, st, w.pos, w.cnz, w.nstrips, w.ncols, w.bad, counts_dev);
  return ES_OK;
}

extern "C" int es_direct_fill(const int32_t* lhs_coords, int64_t n_lhs, int lhs_ndim, int64_t n_rhs, int rhs_ndim,
                              int batch_ndim, const int64_t* lhs_grid, const int64_t* rhs_grid, void* workspace,
                              size_t workspace_bytes, int64_t num_pairs, int64_t num_segments, int32_t* out_coords,
                              int64_t* seg_offsets, int32_t* seg_lhs, int32_t* seg_rhs, int64_t* seg_strip,
                              int32_t* seg_key, void* stream) {
  cudaStream_t st = as_stream(stream);
  DirectGeom g;
  ES_TRY(make_direct_geom(lhs_ndim, rhs_ndim, batch_ndim, lhs_grid, rhs_grid, &g));
  if (n_lhs <= 0 || n_rhs <= 0) return ES_ERR_INVALID;
  Carver cv(workspace, workspace_bytes);
  DirectWs w;
  direct_layout(cv, w, n_lhs, n_rhs, g);
  if (cv.overflow) return ES_ERR_WORKSPACE;
  if (num_segments == 0) {
    // no pairs: the single offset 0
    if (cudaMemsetAsync(seg_offsets, 0, sizeof(int64_t), st) != cudaSuccess) return ES_ERR_CUDA;
    return ES_OK;
  }
  const int64_t nchp1 = direct_chunks(n_lhs);
  const int64_t cb = direct_col_bound(g, n_rhs);
  const int64_t sc = direct_sc_bound(g, n_lhs, n_rhs);
  const int64_t units = (nchp1 - 1) * ((cb + kDirCols - 1) / kDirCols) * 32;
  ES_LAUNCH(direct_pairs_kernel, grid_for(units > sc ? units : sc, 256), 256, 0, st, lhs_coords, n_lhs, g, w.table,
            w.colids, w.ncols, w.nstrips, w.sstart, nchp1, w.cscan, w.sflag, w.sexcl, w.cnz, w.pos, w.gstart,
            num_pairs, num_segments, seg_lhs, seg_rhs, seg_key, out_coords, seg_offsets, seg_strip);
  return ES_OK;
}
