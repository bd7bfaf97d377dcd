/*
 * einsparse — C ABI of the B200 (sm_100a) sparse tensor-relational einsum path.
 *
 * Each entry point replaces one step of einjax's sparse execution path
 * (paths below are relative to the einjax project root). All pointers are
 * device pointers unless stated; all sizes are element counts; every call is
 * asynchronous on `stream` (a cudaStream_t, 0 = legacy default stream) and
 * returns an es_status. No entry point allocates memory: multi-phase steps
 * take a caller-owned workspace whose size the matching *_workspace_size
 * query reports, and data-dependent output sizes are written to a device
 * int64 that the caller reads before allocating the outputs of the *_fill
 * phase. Device-side checks (an index outside its grid) set *error_dev to a
 * non-zero es_status; the caller reads it together with the size. The
 * caller clears *error_dev (and the counts) before a call, except for
 * es_tile_coo_plan, es_tile_dense_plan, es_direct_plan and es_tile_einsum(_ev),
 * which clear their own count and status outputs first.
 *
 * Threading: calls on different streams may run concurrently as long as
 * they do not share a workspace. The library holds no global mutable state
 * apart from a launch counter (es_launch_count).
 */
#ifndef EINSPARSE_H
#define EINSPARSE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum es_status {
  ES_OK = 0,
  ES_ERR_INVALID = 1,     /* bad shape / argument; the reference raises ValueError */
  ES_ERR_INDEX = 2,       /* a coordinate outside the grid its shape defines */
  ES_ERR_WORKSPACE = 3,   /* workspace smaller than *_workspace_size reported */
  ES_ERR_CUDA = 4,        /* CUDA runtime error (launch or async) */
  ES_ERR_UNSUPPORTED = 5, /* dtype / rank / size this build does not handle */
  ES_ERR_TIMEOUT = 6      /* a bounded device-side wait ran out; outputs are invalid */
} es_status;

typedef enum es_dtype { ES_F32 = 0, ES_BF16 = 1, ES_F64 = 2, ES_I32 = 3, ES_I64 = 4 } es_dtype;

/* Arithmetic of the tile contraction. EXACT: fp32 FFMA (SIMT); TC: tensor
 * cores (bf16 inputs: kind::f16; fp32 inputs: 3-pass split TF32, fp32-level
 * error); AUTO: TC where a tensor-core kernel covers the shape, else EXACT. */
typedef enum es_precision { ES_PREC_AUTO = 0, ES_PREC_EXACT = 1, ES_PREC_TC = 2 } es_precision;

#define ES_MAX_DIMS 8

/* Library version and a count of kernels launched since load (or since the
 * last es_launch_count_reset). */
int es_version(void);
int64_t es_launch_count(void);
void es_launch_count_reset(void);
const char* es_status_string(int status);

/* ---------------------------------------------------------------------------
 * Tiling: element COO -> tile-COO.
 * Replaces SparseTensor.to_relation (tensor/sparse.py:160-219) together with
 * the COO extraction it consumes (tensor/sparse.py:234-270).
 * indices: int32 (nnz, ndim) row-major; values: (nnz) of values_dtype
 * (F32/F64/BF16). Entries equal to zero are dropped (sparse.py:185-187);
 * tiles come out in lexicographic coordinate order (np.unique, :204-206);
 * when a coordinate repeats, the entry that comes last in input order
 * wins (NumPy fancy assignment, :211-212). shape[d] % tile[d] != 0 gives
 * ES_ERR_INVALID (:174-179). Plan writes the tile count T to *num_tiles_dev;
 * fill writes coords int32 (T, ndim) and values (T, prod(tile)) of out_dtype.
 * Either fill output may be NULL: with values_out NULL the call writes the
 * coords (and keeps the value bounds in the workspace); with coords_out NULL
 * it writes the values from the bounds that an earlier coords call left in
 * the same workspace (so the values can be filled later, e.g. while the host
 * waits for other counts).
 * ------------------------------------------------------------------------- */
size_t es_tile_coo_workspace_size(int64_t nnz, int ndim, const int64_t* shape, const int64_t* tile);
int es_tile_coo_plan(const int32_t* indices, const void* values, int values_dtype, int64_t nnz,
                     int ndim, const int64_t* shape, const int64_t* tile,
                     void* workspace, size_t workspace_bytes,
                     int64_t* num_tiles_dev, int32_t* error_dev, void* stream);
int es_tile_coo_fill(const void* values, int values_dtype, int64_t nnz, int ndim,
                     const int64_t* shape, const int64_t* tile,
                     void* workspace, size_t workspace_bytes, int64_t num_tiles,
                     int32_t* coords_out, void* values_out, int out_dtype, void* stream);

/* ---------------------------------------------------------------------------
 * COO ingestion: coalescing repeated coordinates.
 * The reference feeds element COO to its tiling as it comes
 * (_extract_coo, tensor/sparse.py:234-270) and the last repeated coordinate
 * wins there (:211-212); scipy CSR and torch's uncoalesced sparse tensors add
 * repeated coordinates instead. es_coo_coalesce states the policy: it writes
 * one entry per distinct coordinate holding a non-zero value, in row-major
 * coordinate order -- ES_DUP_LAST: the value that comes last in input order;
 * ES_DUP_SUM: the sum of the run, accumulated in float64 in input order (what
 * scipy's sum_duplicates and numpy.add.at compute). Zero entries are dropped
 * before coalescing (tensor/sparse.py:185-187); a sum that cancels to zero is
 * written as 0 (the tiling drops it). indices_out int32 (nnz, ndim) and
 * values_out (nnz) of out_dtype (F32/F64/BF16) are caller buffers of the input
 * size; counts_dev[0] = entries written, counts_dev[1] = non-zero input
 * entries (they differ exactly when a coordinate repeats). A coordinate
 * outside `shape` sets *error_dev to ES_ERR_INDEX. This entry point has no
 * counterpart in the reference (it is the explicit form of its implicit
 * last-wins policy).
 * ------------------------------------------------------------------------- */
typedef enum es_dup_policy { ES_DUP_LAST = 0, ES_DUP_SUM = 1 } es_dup_policy;
size_t es_coo_coalesce_workspace_size(int64_t nnz, int ndim, const int64_t* shape);
int es_coo_coalesce(const int32_t* indices, const void* values, int values_dtype, int64_t nnz,
                    int ndim, const int64_t* shape, int policy,
                    void* workspace, size_t workspace_bytes,
                    int32_t* indices_out, void* values_out, int out_dtype,
                    int64_t* counts_dev, int32_t* error_dev, void* stream);

/* Dense array (row-major `shape`) -> tile-COO of the tiles holding any
 * non-zero. Same result as SparseTensor(dense).to_relation(tile)
 * (tensor/sparse.py:104-117,160-219, via np.nonzero at :260-268). Fill:
 * coords_out or values_out may be NULL (that output is not written; the
 * other one only needs the plan's workspace and the dense array). */
size_t es_tile_dense_workspace_size(int ndim, const int64_t* shape, const int64_t* tile);
int es_tile_dense_plan(const void* dense, int dtype, int ndim, const int64_t* shape,
                       const int64_t* tile, void* workspace, size_t workspace_bytes,
                       int64_t* num_tiles_dev, void* stream);
int es_tile_dense_fill(const void* dense, int dtype, int ndim, const int64_t* shape,
                       const int64_t* tile, void* workspace, size_t workspace_bytes,
                       int64_t num_tiles, int32_t* coords_out, void* values_out, int out_dtype,
                       void* stream);

/* ---------------------------------------------------------------------------
 * Coordinate join. Replaces coordinate_join (execution/sparse_dispatch.py:29-82)
 * and coordinate_join_hash (kernels/pallas_gather.py:19-76).
 * join_keys: nkeys pairs (lhs_dim, rhs_dim); key_extents[k]: the tile-grid
 * extent of key k (coordinates must lie in [0, extent), else ES_ERR_INDEX in
 * *error_dev). Pair order is the reference's: RHS tile j ascending, and for
 * each j every LHS tile with an equal key, LHS index ascending; nkeys == 0
 * gives the LHS-major cross product (:53-59). Plan writes P to *num_pairs_dev;
 * fill writes lhs_idx/rhs_idx as index_dtype (ES_I32 or ES_I64).
 * ------------------------------------------------------------------------- */
size_t es_join_workspace_size(int64_t n_lhs, int64_t n_rhs);
int es_join_plan(const int32_t* lhs_coords, int64_t n_lhs, int lhs_ndim,
                 const int32_t* rhs_coords, int64_t n_rhs, int rhs_ndim,
                 const int32_t* join_keys, int nkeys, const int64_t* key_extents,
                 void* workspace, size_t workspace_bytes,
                 int64_t* num_pairs_dev, int32_t* error_dev, void* stream);
int es_join_fill(int64_t n_lhs, int64_t n_rhs, int nkeys, void* workspace, size_t workspace_bytes,
                 int64_t num_pairs, void* lhs_idx_out, void* rhs_idx_out, int index_dtype,
                 void* stream);

/* Allocation-free coordinate join (no counterpart in the reference; an
 * addition for callers that may not allocate device memory when they join,
 * e.g. code in a host callback or an engine that reserves all memory up
 * front). Same pairs and order as es_join_plan + es_join_fill, but the sort
 * and count scratch comes from a fixed array inside the library (one per
 * GPU, kept until the process exits) instead of a workspace. At most 65536
 * tiles per side, else ES_ERR_UNSUPPORTED. The caller passes the outputs:
 * lhs_idx_out / rhs_idx_out with room for `capacity` pairs and the device
 * int64 *num_pairs_dev that receives P; if P > capacity only `capacity`
 * pairs are written and *error_dev becomes ES_ERR_WORKSPACE. Nothing is
 * allocated or synchronised. Calls whose kernels overlap on one GPU share the
 * array and race: order them on one stream. The first call on a device looks
 * up the array's address (cudaGetSymbolAddress); make it before any stream
 * capture. */
int es_join_static(const int32_t* lhs_coords, int64_t n_lhs, int lhs_ndim,
                   const int32_t* rhs_coords, int64_t n_rhs, int rhs_ndim,
                   const int32_t* join_keys, int nkeys, const int64_t* key_extents,
                   void* lhs_idx_out, void* rhs_idx_out, int index_dtype, int64_t capacity,
                   int64_t* num_pairs_dev, int32_t* error_dev, void* stream);

/* ---------------------------------------------------------------------------
 * Output-tile grouping. Replaces _compute_output_coords + the grouping half of
 * segment_sum (execution/sparse_dispatch.py:174-223, 129-171): the output
 * coordinate of each pair is gathered through agg_keys (pairs (src, dim),
 * src 0 = lhs, 1 = rhs); pairs are stably sorted by it, so inside each group
 * they keep join order (the reference sums each group in pair order,
 * :165-169). Plan writes the group count O to *num_segments_dev; fill writes
 * out_coords int32 (O, out_ndim) sorted lexicographically (:161),
 * seg_offsets int64 (O+1) and the pairs regrouped (seg_lhs_idx,
 * seg_rhs_idx int32, P each; seg_pair_idx int32 = original pair index, may
 * be NULL). lhs_idx/rhs_idx are int32. With seg_strip non-NULL, fill also
 * writes per segment the packed value of its first strip_dims output
 * coordinates (int64, non-decreasing): segments with equal values form a
 * "strip" that shares its lhs-derived coordinates, which es_tile_einsum
 * batches into one tensor-core tile.
 * ------------------------------------------------------------------------- */
size_t es_segments_workspace_size(int64_t num_pairs);
int es_segments_plan(const int32_t* lhs_coords, int lhs_ndim, const int32_t* rhs_coords, int rhs_ndim,
                     const int32_t* lhs_idx, const int32_t* rhs_idx, int64_t num_pairs,
                     const int32_t* agg_keys, int out_ndim, const int64_t* out_extents,
                     void* workspace, size_t workspace_bytes,
                     int64_t* num_segments_dev, int32_t* error_dev, void* stream);
int es_segments_fill(const int32_t* lhs_idx, const int32_t* rhs_idx, int64_t num_pairs, int out_ndim,
                     const int64_t* out_extents, void* workspace, size_t workspace_bytes,
                     int64_t num_segments, int32_t* out_coords, int64_t* seg_offsets,
                     int32_t* seg_lhs_idx, int32_t* seg_rhs_idx, int32_t* seg_pair_idx,
                     int strip_dims, int64_t* seg_strip, void* stream);

/* Per-pair output tile coordinates, int32 (P, out_ndim): the gather of
 * _compute_output_coords (execution/sparse_dispatch.py:174-223). */
int es_output_coords(const int32_t* lhs_coords, int lhs_ndim, const int32_t* rhs_coords, int rhs_ndim,
                     const int32_t* lhs_idx, const int32_t* rhs_idx, int64_t num_pairs,
                     const int32_t* agg_keys, int out_ndim, int32_t* out_coords, void* stream);

/* ---------------------------------------------------------------------------
 * Segmented tile einsum — the per-pair kernel einsum fused with the
 * segment-sum (execution/sparse_dispatch.py:85-126 + 129-171; the batched
 * tile einsum of kernels/pallas_matmul.py:33-113).
 * kernel_string: the per-tile einsum ("ij,jk->ik", "bij,bjk->bik",
 * "ijk,kl->ijl", ...; any two-operand string with an explicit "->").
 * For segment s, out[s_out] = sum over p in [seg_offsets[s], seg_offsets[s+1])
 * of einsum(lhs_values[pair_lhs[p]], rhs_values[pair_rhs[p]]), accumulated
 * in fp32, where s_out = seg_out_index ? seg_out_index[s] : s.
 * seg_offsets == NULL means every pair is its own segment (the unfused
 * per-pair kernel_einsum, output (P, *out_tile)). Output rows that no segment
 * writes are left untouched. lhs_rows / rhs_rows: tiles in each values array
 * (pair indices outside them raise ES_ERR_INDEX in *error_dev and read as
 * zero tiles). Values dtypes: F32 / BF16 / F64 inputs; F32 / BF16 outputs.
 * seg_strip (optional, from es_segments_fill): strip key per segment; the
 * tensor-core path computes up to 8 segments of one strip in one tile.
 * pair_key (optional): the contracted tile coordinate of each pair, with
 * key_extent its range. Contract: inside a segment keys increase strictly,
 * and segments of one strip (seg_strip) pair the same lhs tile with a given
 * key. When given, the tensor-core path may stack up to 128 / Mt strips
 * into one 128-row operand that shares each step's rhs tiles (fp32, Mt 16,
 * 32 or 64, Kt 32 or 64), and splits the contracted range into blocks whose
 * rhs operand fits in L2, adding the blocks' partial sums into the output
 * in block order. A broken contract sets *error_dev to ES_ERR_INVALID.
 * A contraction that is a plain tile matmul after swapping the last two tile
 * dims of an operand ("ik,jk->ij", "ij,ik->jk": the autodiff strings) also
 * takes the tensor-core path; the swapped operand is transposed into the
 * workspace first (a copy, no rounding).
 * workspace: es_tile_einsum_workspace_size bytes (0 for the SIMT path),
 * sized for the same lhs_rows, rhs_rows, num_pairs, num_segments and
 * key_extent (0 when no pair_key is passed). A device-side wait that runs
 * out sets *error_dev to ES_ERR_TIMEOUT.
 * ------------------------------------------------------------------------- */
size_t es_tile_einsum_workspace_size(const char* kernel_string,
                                     const int64_t* lhs_tile, int lhs_nd, const int64_t* rhs_tile, int rhs_nd,
                                     int lhs_dtype, int rhs_dtype, int64_t lhs_rows, int64_t rhs_rows,
                                     int64_t num_pairs, int64_t num_segments, int64_t key_extent, int precision);
int es_tile_einsum(const char* kernel_string,
                   const int64_t* lhs_tile, int lhs_nd, const int64_t* rhs_tile, int rhs_nd,
                   const void* lhs_values, int lhs_dtype, int64_t lhs_rows,
                   const void* rhs_values, int rhs_dtype, int64_t rhs_rows,
                   const int32_t* pair_lhs, const int32_t* pair_rhs, int64_t num_pairs,
                   const int64_t* seg_offsets, int64_t num_segments, const int32_t* seg_out_index,
                   const int64_t* seg_strip, const int32_t* pair_key, int64_t key_extent,
                   void* out_values, int out_dtype, int precision,
                   void* workspace, size_t workspace_bytes, int32_t* error_dev, void* stream);

/* es_tile_einsum that waits for the cudaEvent_t values_ready (NULL: no
 * wait) on `stream` right before its first launch that reads lhs_values or
 * rhs_values: the grouping of the pairs into work items and step records
 * runs first, so values written on another stream (e.g. a tiling's value
 * fill) overlap it. status_host (NULL: none): pinned host int32 that
 * receives *error_dev by an asynchronous copy behind the call's launches,
 * so a caller can check the status later without a copy of its own. */
int es_tile_einsum_ev(const char* kernel_string,
                      const int64_t* lhs_tile, int lhs_nd, const int64_t* rhs_tile, int rhs_nd,
                      const void* lhs_values, int lhs_dtype, int64_t lhs_rows,
                      const void* rhs_values, int rhs_dtype, int64_t rhs_rows,
                      const int32_t* pair_lhs, const int32_t* pair_rhs, int64_t num_pairs,
                      const int64_t* seg_offsets, int64_t num_segments, const int32_t* seg_out_index,
                      const int64_t* seg_strip, const int32_t* pair_key, int64_t key_extent,
                      void* out_values, int out_dtype, int precision,
                      void* workspace, size_t workspace_bytes, int32_t* error_dev, void* stream,
                      void* values_ready, int32_t* status_host);

/* Which path es_tile_einsum takes for these arguments: 1 tensor cores,
 * 0 SIMT, negative es_status if the call would be rejected. Host-side. */
int es_tile_einsum_path(const char* kernel_string, const int64_t* lhs_tile, int lhs_nd,
                        const int64_t* rhs_tile, int rhs_nd, int lhs_dtype, int rhs_dtype, int precision);

/* ---------------------------------------------------------------------------
 * Join + output grouping in one pass for
 *     lhs (batch..., strip..., k) x rhs (batch..., k, col...)
 *         -> out (batch..., strip..., col...)
 * with batch_ndim >= 0 leading batch dims joined pairwise (lhs dim d with rhs
 * dim d), the last lhs coordinate joined with rhs coordinate batch_ndim, and
 * output = the other lhs then the other rhs coordinates (the matmul-like
 * calls of execute_sparse: coordinate_join + _compute_output_coords +
 * segment_sum grouping, execution/sparse_dispatch.py:29-82, 174-223,
 * 129-171). No reference counterpart as one function: it replaces
 * es_join_plan/_fill + es_segments_plan/_fill for these shapes with no sort.
 * Both coordinate arrays must be in lexicographic order without repeats (a
 * relation's invariant); lhs_grid / rhs_grid are the tile-grid extents.
 * plan writes counts_dev[0] = pairs P, [1] = output tiles O, [2] = 1 when a
 * relation is not in lexicographic order (then use the general path); fill
 * writes out_coords (O, out_nd) lexicographic, seg_offsets (O+1), seg_lhs /
 * seg_rhs (P) grouped by output tile (pairs of a tile in ascending k = join
 * order), and optionally seg_strip (O) strip index and seg_key (P) the
 * contracted k. fill takes the same sizes, grids and workspace as plan (the
 * workspace carries the plan's per-(strip, column) offsets).
 * ------------------------------------------------------------------------- */
size_t es_direct_workspace_size(int64_t n_lhs, int lhs_ndim, int64_t n_rhs, int rhs_ndim, int batch_ndim,
                                const int64_t* lhs_grid, const int64_t* rhs_grid);
int es_direct_plan(const int32_t* lhs_coords, int64_t n_lhs, int lhs_ndim, const int32_t* rhs_coords,
                   int64_t n_rhs, int rhs_ndim, int batch_ndim, const int64_t* lhs_grid, const int64_t* rhs_grid,
                   void* workspace, size_t workspace_bytes, int64_t* counts_dev, int32_t* error_dev,
                   void* stream);
int es_direct_fill(const int32_t* lhs_coords, int64_t n_lhs, int lhs_ndim, int64_t n_rhs, int rhs_ndim,
                   int batch_ndim, const int64_t* lhs_grid, const int64_t* rhs_grid, void* workspace,
                   size_t workspace_bytes, int64_t num_pairs, int64_t num_segments, int32_t* out_coords,
                   int64_t* seg_offsets, int32_t* seg_lhs, int32_t* seg_rhs, int64_t* seg_strip, int32_t* seg_key,
                   void* stream);

/* Out tile shape of a kernel string (_infer_output_tile_shape,
 * execution/sparse_dispatch.py:506-545). Host-side; returns the out rank or
 * a negative es_status. */
int es_out_tile_shape(const char* kernel_string, const int64_t* lhs_tile, int lhs_nd,
                      const int64_t* rhs_tile, int rhs_nd, int64_t* out_tile);

/* ---------------------------------------------------------------------------
 * Standalone segment-sum (execution/sparse_dispatch.py:129-171): values
 * (P, tile_elems) grouped by coords (P, nd) int32 with per-dim extents.
 * Plan (es_segsum_plan) writes O; fill writes unique coords (O, nd) sorted
 * lexicographically and the per-group sums, added in row order in fp32.
 * Scatter-add by index (the `.at[idx].add` of autodiff/custom_vjp.py:272-273)
 * is the nd == 1 case with out rows chosen by the caller via es_tile_einsum's
 * seg_out_index; see es_scatter_add_rows.
 * ------------------------------------------------------------------------- */
size_t es_segsum_workspace_size(int64_t num_rows);
int es_segsum_plan(const int32_t* coords, int64_t num_rows, int nd, const int64_t* extents,
                   void* workspace, size_t workspace_bytes, int64_t* num_segments_dev,
                   int32_t* error_dev, void* stream);
int es_segsum_fill(const void* values, int values_dtype, int64_t num_rows, int64_t tile_elems, int nd,
                   const int64_t* extents, void* workspace, size_t workspace_bytes, int64_t num_segments,
                   int32_t* out_coords, void* out_values, int out_dtype, void* stream);

/* Groups of an es_segsum_plan without a reduction: unique coordinates
 * (O, nd) sorted lexicographically into out_coords (may be NULL) and, for
 * each input row r, its group index into row_group[r] (int32, may be NULL).
 * This is the grouping half of segment_sum (execution/sparse_dispatch.py:
 * 154-161: the unique output keys and which key each row belongs to); the
 * sharded path uses it to lay every rank's partial output tiles out in the
 * order of the union of all ranks' output coordinates before the
 * reduce-scatter. Same workspace as the plan, which must have run first. */
int es_segsum_groups(int64_t num_rows, int nd, const int64_t* extents, void* workspace, size_t workspace_bytes,
                     int64_t num_segments, int32_t* out_coords, int32_t* row_group, void* stream);

/* out[idx[r]] += values[r] for r in row order, rows of tile_elems
 * (autodiff/custom_vjp.py:272-273). out must be F32. Deterministic: rows
 * are grouped by a stable sort, each group is summed in row order, then
 * added once. */
size_t es_scatter_add_workspace_size(int64_t num_rows);
int es_scatter_add_rows(const void* values, int values_dtype, const int32_t* idx, int64_t num_rows,
                        int64_t tile_elems, int64_t num_out_rows, void* workspace,
                        size_t workspace_bytes, float* out, int32_t* error_dev, void* stream);

/* ---------------------------------------------------------------------------
 * Sparsity statistics per tiling scheme, the contraction planner's input
 * (tensor/stats.py:25-80 compute_sparsity_stats_coo; the metrics
 * SparseTensor / DenseTensor compute for every scheme, tensor/sparse.py:122-158,
 * tensor/dense.py:44-94). For each of num_schemes tile shapes U
 * (tile_shapes: host int64 (num_schemes, ndim), sides >= 1):
 *   num_tuples_dev[u]            = T(U), tiles holding a non-zero entry;
 *   value_count_dev[u*ndim + l]  = V(l, U), distinct tile coordinates along l.
 * Entries: COO (indices int32 (num_entries, ndim), values of values_dtype or
 * NULL when every entry counts), or with indices == NULL a dense row-major
 * array `values` of `shape` (num_entries = its element count). Zeros do not
 * count; repeated coordinates count once. A coordinate outside the shape sets
 * *error_dev to ES_ERR_INDEX. Tile grids up to 2^32 tiles use a bitmap (the
 * workspace holds up to 512 MB of them per pass, several schemes per pass);
 * larger grids count distinct tile keys after a radix sort of the entries.
 * workspace: es_sparsity_stats_workspace_size bytes for the same arguments.
 * ------------------------------------------------------------------------- */
size_t es_sparsity_stats_workspace_size(int64_t num_entries, int ndim, const int64_t* shape,
                                        const int64_t* tile_shapes, int num_schemes);
int es_sparsity_stats(const int32_t* indices, const void* values, int values_dtype, int64_t num_entries, int ndim,
                      const int64_t* shape, const int64_t* tile_shapes, int num_schemes, void* workspace,
                      size_t workspace_bytes, int64_t* num_tuples_dev, int64_t* value_count_dev,
                      int32_t* error_dev, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* EINSPARSE_H */
