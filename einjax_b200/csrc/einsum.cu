// Segmented tile einsum: per-pair tile contraction fused with the segment-sum.
//
// es_tile_einsum computes, for every segment s (a run of pairs that share an
// output tile, in join order), out[s] = sum_p einsum(lhs[pair_lhs[p]],
// rhs[pair_rhs[p]]) — kernel_einsum followed by segment_sum
// (execution/sparse_dispatch.py:85-171) without materialising the (P, tile)
// per-pair partials. This file holds the string parser, the generic SIMT
// kernel (fp32 FFMA, any label layout, the ES_PREC_EXACT path) and the
// dispatcher; tensor-core kernels live in tile_gemm_tc.cu.
#include <string.h>

#include <string>

#include "common.cuh"
#include "einsum_desc.h"
#include "tile_gemm_tc.h"

namespace es {

int parse_einsum(const char* ks, const int64_t* lhs_tile, int lhs_nd, const int64_t* rhs_tile, int rhs_nd,
                 EinsumDesc* d) {
  if (!ks) return ES_ERR_INVALID;
  std::string s(ks);
  std::string clean;
  for (char c : s)
    if (c != ' ') clean.push_back(c);
  size_t arrow = clean.find("->");
  if (arrow == std::string::npos) return ES_ERR_INVALID;
  std::string ins = clean.substr(0, arrow), out = clean.substr(arrow + 2);
  size_t comma = ins.find(',');
  if (comma == std::string::npos || ins.find(',', comma + 1) != std::string::npos) return ES_ERR_INVALID;
  std::string L = ins.substr(0, comma), R = ins.substr(comma + 1);
  if ((int)L.size() != lhs_nd || (int)R.size() != rhs_nd) return ES_ERR_INVALID;
  if ((int)out.size() > ES_MAX_DIMS) return ES_ERR_UNSUPPORTED;
  auto is_label = [](char c) { return (c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z'); };
  int64_t size[128];
  int64_t lst[128], rst[128], ost[128];
  bool inL[128], inR[128], inO[128];
  for (int i = 0; i < 128; ++i) {
    size[i] = -1;
    lst[i] = rst[i] = ost[i] = 0;
    inL[i] = inR[i] = inO[i] = false;
  }
  int64_t stride = 1;
  d->lhs_te = 1;
  for (int i = lhs_nd - 1; i >= 0; --i) {
    unsigned char c = L[i];
    if (!is_label(c) || lhs_tile[i] <= 0) return ES_ERR_INVALID;
    if (size[c] >= 0 && size[c] != lhs_tile[i]) return ES_ERR_INVALID;
    size[c] = lhs_tile[i];
    lst[c] += stride;
    inL[c] = true;
    stride *= lhs_tile[i];
  }
  d->lhs_te = (int)stride;
  stride = 1;
  for (int i = rhs_nd - 1; i >= 0; --i) {
    unsigned char c = R[i];
    if (!is_label(c) || rhs_tile[i] <= 0) return ES_ERR_INVALID;
    if (size[c] >= 0 && size[c] != rhs_tile[i]) return ES_ERR_INVALID;
    size[c] = rhs_tile[i];
    rst[c] += stride;
    inR[c] = true;
    stride *= rhs_tile[i];
  }
  d->rhs_te = (int)stride;
  stride = 1;
  d->out_nd = (int)out.size();
  for (int i = (int)out.size() - 1; i >= 0; --i) {
    unsigned char c = out[i];
    if (!is_label(c) || size[c] < 0 || inO[c]) return ES_ERR_INVALID;
    ost[c] = stride;
    inO[c] = true;
    d->out_tile[i] = (int)size[c];
    stride *= size[c];
  }
  d->out_te = (int)stride;
  EinGroup* groups[4] = {&d->B, &d->M, &d->N, &d->K};
  for (auto* g : groups) {
    g->n = 0;
    g->total = 1;
  }
  // Group members in order of first appearance: output order for B/M/N,
  // lhs-then-rhs order for K.
  std::string order = out + L + R;
  bool seen[128] = {false};
  for (char cc : order) {
    unsigned char c = cc;
    if (seen[c]) continue;
    seen[c] = true;
    EinGroup* g;
    if (inO[c]) {
      if (inL[c] && inR[c]) g = &d->B;
      else if (inL[c]) g = &d->M;
      else g = &d->N;
    } else {
      g = &d->K;
    }
    if (g->n >= kMaxGroupLabels) return ES_ERR_UNSUPPORTED;
    g->size[g->n] = (int)size[c];
    g->lstride[g->n] = (int)lst[c];
    g->rstride[g->n] = (int)rst[c];
    g->ostride[g->n] = (int)ost[c];
    g->total *= (int)size[c];
    g->n++;
  }
  return ES_OK;
}

// ---------------------------------------------------------------------------
// Generic SIMT kernel: 64x64 output block per CTA, 4x4 per thread, K in
// steps of 16 through shared memory; offsets come from per-group tables.

constexpr int kBM = 64, kBN = 64, kBK = 16;

struct SimtTables {
  int *lb, *rb, *ob;  // B: lhs, rhs, out offsets
  int *lm, *om;       // M
  int *rn, *on;       // N
  int *lk, *rk;       // K
};

__device__ void fill_group_tables(const EinGroup& g, int* a, int* b, int* c, int which_a, int which_b, int which_c) {
  for (int idx = threadIdx.x; idx < g.total; idx += blockDim.x) {
    int rem = idx;
    int oa = 0, ob = 0, oc = 0;
    for (int q = g.n - 1; q >= 0; --q) {
      int x = rem % g.size[q];
      rem /= g.size[q];
      const int st[3] = {g.lstride[q], g.rstride[q], g.ostride[q]};
      oa += x * st[which_a];
      ob += x * st[which_b];
      oc += x * st[which_c];
    }
    if (a) a[idx] = oa;
    if (b) b[idx] = ob;
    if (c) c[idx] = oc;
  }
}

__device__ __forceinline__ float ld_val(const void* p, int dtype, int64_t i) { return load_as_f32(p, dtype, i); }

__global__ void __launch_bounds__(256) einsum_simt_kernel(EinsumDesc d, const void* __restrict__ lhs, int ldt,
                                                          const void* __restrict__ rhs, int rdt,
                                                          const int32_t* __restrict__ pl,
                                                          const int32_t* __restrict__ pr,
                                                          const int64_t* __restrict__ seg_off, int64_t nseg,
                                                          const int32_t* __restrict__ seg_out, void* __restrict__ out,
                                                          int odt) {
  extern __shared__ int simt_tab[];
  __shared__ float As[kBK][kBM + 4];
  __shared__ float Bs[kBK][kBN + 4];
  SimtTables t;
  int* p = simt_tab;
  t.lb = p; p += d.B.total;
  t.rb = p; p += d.B.total;
  t.ob = p; p += d.B.total;
  t.lm = p; p += d.M.total;
  t.om = p; p += d.M.total;
  t.rn = p; p += d.N.total;
  t.on = p; p += d.N.total;
  t.lk = p; p += d.K.total;
  t.rk = p;
  fill_group_tables(d.B, t.lb, t.rb, t.ob, 0, 1, 2);
  fill_group_tables(d.M, t.lm, nullptr, t.om, 0, 1, 2);
  fill_group_tables(d.N, t.rn, nullptr, t.on, 1, 0, 2);
  fill_group_tables(d.K, t.lk, t.rk, nullptr, 0, 1, 2);
  __syncthreads();

  const int M = d.M.total, N = d.N.total, K = d.K.total, Bt = d.B.total;
  const int mb = (M + kBM - 1) / kBM, nb = (N + kBN - 1) / kBN;
  const int64_t items = nseg * Bt * mb * nb;
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
  for (int64_t it = blockIdx.x; it < items; it += gridDim.x) {
    int64_t r = it;
    const int nbi = r % nb; r /= nb;
    const int mbi = r % mb; r /= mb;
    const int b = r % Bt; r /= Bt;
    const int64_t s = r;
    const int64_t p0 = seg_off ? seg_off[s] : s;
    const int64_t p1 = seg_off ? seg_off[s + 1] : s + 1;
    const int m0 = mbi * kBM, n0 = nbi * kBN;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    for (int64_t pp = p0; pp < p1; ++pp) {
      const int64_t lbase = static_cast<int64_t>(pl[pp]) * d.lhs_te + t.lb[b];
      const int64_t rbase = static_cast<int64_t>(pr[pp]) * d.rhs_te + t.rb[b];
      for (int k0 = 0; k0 < K; k0 += kBK) {
        __syncthreads();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int e = tid + q * 256;
          const int kk = e % kBK, mm = e / kBK;  // A: k fastest
          const int m = m0 + mm, k = k0 + kk;
          As[kk][mm] = (m < M && k < K) ? ld_val(lhs, ldt, lbase + t.lm[m] + t.lk[k]) : 0.f;
          const int nn = e % kBN, kb = e / kBN;  // B: n fastest
          const int n = n0 + nn, k2 = k0 + kb;
          Bs[kb][nn] = (n < N && k2 < K) ? ld_val(rhs, rdt, rbase + t.rk[k2] + t.rn[n]) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < kBK; ++kk) {
          float a[4], bv[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
          for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bv[j], acc[i][j]);
        }
      }
    }
    const int64_t orow = seg_out ? static_cast<int64_t>(seg_out[s]) : s;
    const int64_t obase = orow * d.out_te + t.ob[b];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int m = m0 + ty * 4 + i;
      if (m >= M) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + tx * 4 + j;
        if (n >= N) continue;
        const int64_t o = obase + t.om[m] + t.on[n];
        if (odt == ES_F32) static_cast<float*>(out)[o] = acc[i][j];
        else static_cast<__nv_bfloat16*>(out)[o] = __float2bfloat16_rn(acc[i][j]);
      }
    }
  }
}

static int launch_simt(const EinsumDesc& d, const void* lhs, int ldt, const void* rhs, int rdt, const int32_t* pl,
                       const int32_t* pr, const int64_t* seg_off, int64_t nseg, const int32_t* seg_out, void* out,
                       int odt, cudaStream_t st) {
  const int64_t tab_ints = 3LL * d.B.total + 2LL * d.M.total + 2LL * d.N.total + 2LL * d.K.total;
  const size_t smem = static_cast<size_t>(tab_ints) * sizeof(int);
  if (smem > 160 * 1024) return ES_ERR_UNSUPPORTED;
  {
    // raised once per device to the largest size asked for
    static int attr_bytes[kMaxAttrDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return ES_ERR_CUDA;
    if (dev < 0 || dev >= kMaxAttrDevices || attr_bytes[dev] < static_cast<int>(smem)) {
      if (cudaFuncSetAttribute(einsum_simt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess)
        return ES_ERR_CUDA;
      if (dev >= 0 && dev < kMaxAttrDevices) attr_bytes[dev] = static_cast<int>(smem);
    }
  }
  const int64_t mb = (d.M.total + kBM - 1) / kBM, nb = (d.N.total + kBN - 1) / kBN;
  const int64_t items = nseg * d.B.total * mb * nb;
  if (items <= 0) return ES_OK;
  const int grid = static_cast<int>(items < 148LL * 8 ? items : 148LL * 8);
  ES_LAUNCH(einsum_simt_kernel, grid, 256, smem, st, d, lhs, ldt, rhs, rdt, pl, pr, seg_off, nseg, seg_out, out, odt);
  return ES_OK;
}

}  // namespace es

using namespace es;

extern "C" int es_out_tile_shape(const char* kernel_string, const int64_t* lhs_tile, int lhs_nd,
                                 const int64_t* rhs_tile, int rhs_nd, int64_t* out_tile) {
  EinsumDesc d;
  int st = parse_einsum(kernel_string, lhs_tile, lhs_nd, rhs_tile, rhs_nd, &d);
  if (st != ES_OK) return -st;
  for (int i = 0; i < d.out_nd; ++i) out_tile[i] = d.out_tile[i];
  return d.out_nd;
}

static bool want_tc(int precision) { return precision == ES_PREC_AUTO || precision == ES_PREC_TC; }

// A contraction the tensor-core path covers after swapping the last two tile
// dims of the lhs and/or rhs operand (e.g. the autodiff strings
// "ik,jk->ij" = g . rhs^T and "ij,ik->jk" = lhs^T . g): a swapped lhs is
// transposed into the workspace (a pure copy); a swapped rhs is read in its
// own (k-contiguous) layout when the panel image is built.
struct TcVariant {
  int tl = 0, tr = 0;  // transpose lhs / rhs
  std::string ks;
  int64_t lt[ES_MAX_DIMS], rt[ES_MAX_DIMS];
  EinsumDesc d;
};

static bool tc_variant(const char* kernel_string, const int64_t* lhs_tile, int lhs_nd, const int64_t* rhs_tile,
                       int rhs_nd, int ldt, int rdt, int odt, bool strips, bool keys, TcVariant* v, TcConfig* c) {
  std::string clean;
  for (const char* p = kernel_string; *p; ++p)
    if (*p != ' ') clean.push_back(*p);
  const size_t comma = clean.find(','), arrow = clean.find("->");
  if (comma == std::string::npos || arrow == std::string::npos || comma > arrow) return false;
  if (lhs_nd > ES_MAX_DIMS || rhs_nd > ES_MAX_DIMS) return false;
  for (int t = 0; t < 4; ++t) {
    const int tl = t & 1, tr = (t >> 1) & 1;
    if ((tl && lhs_nd < 2) || (tr && rhs_nd < 2)) continue;
    std::string ks = clean;
    for (int i = 0; i < lhs_nd; ++i) v->lt[i] = lhs_tile[i];
    for (int i = 0; i < rhs_nd; ++i) v->rt[i] = rhs_tile[i];
    if (tl) {
      std::swap(ks[comma - 2], ks[comma - 1]);
      std::swap(v->lt[lhs_nd - 2], v->lt[lhs_nd - 1]);
    }
    if (tr) {
      std::swap(ks[arrow - 2], ks[arrow - 1]);
      std::swap(v->rt[rhs_nd - 2], v->rt[rhs_nd - 1]);
    }
    if (parse_einsum(ks.c_str(), v->lt, lhs_nd, v->rt, rhs_nd, &v->d) != ES_OK) continue;
    if (!tc_config(v->d, ldt, rdt, odt, strips, keys, c)) continue;
    v->tl = tl;
    v->tr = tr;
    v->ks = ks;
    return true;
  }
  return false;
}

// out[m][c][r] = in[m][r][c] for nmat matrices of R x C elements of esz
// bytes (4 or 2): 32 x 32 blocks through shared memory, coalesced both ways.
template <typename T>
__global__ void __launch_bounds__(256) tiles_transpose_kernel(const T* __restrict__ in, T* __restrict__ out,
                                                              int64_t nmat, int R, int C) {
  __shared__ T blk[32][33];
  const int br = (R + 31) / 32, bc = (C + 31) / 32;
  const int64_t nblk = nmat * br * bc;
  for (int64_t b = blockIdx.x; b < nblk; b += gridDim.x) {
    const int64_t m = b / (br * bc);
    const int rem = static_cast<int>(b - m * br * bc);
    const int r0 = (rem / bc) * 32, c0 = (rem % bc) * 32;
    const T* src = in + m * R * C;
    T* dst = out + m * R * C;
    for (int i = threadIdx.y; i < 32; i += 8) {
      const int r = r0 + i, cc = c0 + threadIdx.x;
      if (r < R && cc < C) blk[i][threadIdx.x] = src[static_cast<int64_t>(r) * C + cc];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += 8) {
      const int cc = c0 + i, r = r0 + threadIdx.x;
      if (r < R && cc < C) dst[static_cast<int64_t>(cc) * R + r] = blk[threadIdx.x][i];
    }
    __syncthreads();
  }
}

static int transpose_tiles(const void* in, void* out, int dtype, int64_t rows, const int64_t* tile, int nd,
                           cudaStream_t st) {
  int64_t lead = 1;
  for (int i = 0; i + 2 < nd; ++i) lead *= tile[i];
  const int64_t nmat = rows * lead;
  const int R = static_cast<int>(tile[nd - 2]), C = static_cast<int>(tile[nd - 1]);
  const int64_t nblk = nmat * ((R + 31) / 32) * ((C + 31) / 32);
  const int grid = static_cast<int>(nblk < 148 * 64 ? nblk : 148 * 64);
  if (nblk <= 0) return ES_OK;
  if (dtype == ES_F32)
    ES_LAUNCH(tiles_transpose_kernel<float>, grid, dim3(32, 8), 0, st, static_cast<const float*>(in),
              static_cast<float*>(out), nmat, R, C);
  else
    ES_LAUNCH(tiles_transpose_kernel<uint16_t>, grid, dim3(32, 8), 0, st, static_cast<const uint16_t*>(in),
              static_cast<uint16_t*>(out), nmat, R, C);
  return ES_OK;
}

static size_t round256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

extern "C" int es_tile_einsum_path(const char* kernel_string, const int64_t* lhs_tile, int lhs_nd,
                                   const int64_t* rhs_tile, int rhs_nd, int lhs_dtype, int rhs_dtype,
                                   int precision) {
  EinsumDesc d;
  int st = parse_einsum(kernel_string, lhs_tile, lhs_nd, rhs_tile, rhs_nd, &d);
  if (st != ES_OK) return -st;
  TcConfig c;
  TcVariant v;
  if (want_tc(precision) && tc_variant(kernel_string, lhs_tile, lhs_nd, rhs_tile, rhs_nd, lhs_dtype, rhs_dtype,
                                       ES_F32, true, false, &v, &c))
    return 1;
  if (precision == ES_PREC_TC) return -ES_ERR_UNSUPPORTED;
  return 0;
}

extern "C" size_t es_tile_einsum_workspace_size(const char* kernel_string, const int64_t* lhs_tile, int lhs_nd,
                                                const int64_t* rhs_tile, int rhs_nd, int lhs_dtype, int rhs_dtype,
                                                int64_t lhs_rows, int64_t rhs_rows, int64_t num_pairs,
                                                int64_t num_segments, int64_t key_extent, int precision) {
  EinsumDesc d;
  if (parse_einsum(kernel_string, lhs_tile, lhs_nd, rhs_tile, rhs_nd, &d) != ES_OK) return 0;
  if (!want_tc(precision)) return 0;
  // the launch's geometry depends on whether strips (seg_strip) and keys
  // (pair_key) are passed; size for the largest of the candidates
  size_t best = 0;
  for (int strips = 0; strips < 2; ++strips) {
    for (int keys = 0; keys < (key_extent > 0 ? 2 : 1); ++keys) {
      TcConfig c;
      TcVariant v;
      if (!tc_variant(kernel_string, lhs_tile, lhs_nd, rhs_tile, rhs_nd, lhs_dtype, rhs_dtype, ES_F32, strips != 0,
                      keys != 0, &v, &c))
        continue;
      const int64_t ke = keys ? key_extent : 0;
      size_t sz = tc_workspace_size(c, rhs_rows, num_pairs, num_segments,
                                    tc_key_blocks(c, rhs_rows, keys != 0, ke, num_segments), ke);
      if (v.tl) sz += round256(static_cast<size_t>(lhs_rows) * d.lhs_te * dtype_size(lhs_dtype)) + 256;
      if (sz > best) best = sz;
    }
  }
  return best;
}

static int tile_einsum_impl(const char* kernel_string, const int64_t* lhs_tile, int lhs_nd, const int64_t* rhs_tile,
                            int rhs_nd, const void* lhs_values, int lhs_dtype, int64_t lhs_rows,
                            const void* rhs_values, int rhs_dtype, int64_t rhs_rows, const int32_t* pair_lhs,
                            const int32_t* pair_rhs, int64_t num_pairs, const int64_t* seg_offsets,
                            int64_t num_segments, const int32_t* seg_out_index, const int64_t* seg_strip,
                            const int32_t* pair_key, int64_t key_extent, void* out_values, int out_dtype,
                            int precision, void* workspace, size_t workspace_bytes, int32_t* error_dev,
                            void* stream, void* values_ready);

extern "C" int es_tile_einsum_ev(const char* kernel_string, const int64_t* lhs_tile, int lhs_nd,
                                 const int64_t* rhs_tile, int rhs_nd, const void* lhs_values, int lhs_dtype,
                                 int64_t lhs_rows, const void* rhs_values, int rhs_dtype, int64_t rhs_rows,
                                 const int32_t* pair_lhs, const int32_t* pair_rhs, int64_t num_pairs,
                                 const int64_t* seg_offsets, int64_t num_segments, const int32_t* seg_out_index,
                                 const int64_t* seg_strip, const int32_t* pair_key, int64_t key_extent,
                                 void* out_values, int out_dtype, int precision, void* workspace,
                                 size_t workspace_bytes, int32_t* error_dev, void* stream, void* values_ready,
                                 int32_t* status_host) {
  const int r = tile_einsum_impl(kernel_string, lhs_tile, lhs_nd, rhs_tile, rhs_nd, lhs_values, lhs_dtype, lhs_rows,
                                 rhs_values, rhs_dtype, rhs_rows, pair_lhs, pair_rhs, num_pairs, seg_offsets,
                                 num_segments, seg_out_index, seg_strip, pair_key, key_extent, out_values, out_dtype,
                                 precision, workspace, workspace_bytes, error_dev, stream, values_ready);
  // the device status follows into pinned host memory behind the launches
  if (r == ES_OK && status_host && error_dev &&
      cudaMemcpyAsync(status_host, error_dev, sizeof(int32_t), cudaMemcpyDeviceToHost, as_stream(stream)) !=
          cudaSuccess)
    return ES_ERR_CUDA;
  return r;
}

static int tile_einsum_impl(const char* kernel_string, const int64_t* lhs_tile, int lhs_nd, const int64_t* rhs_tile,
                            int rhs_nd, const void* lhs_values, int lhs_dtype, int64_t lhs_rows,
                            const void* rhs_values, int rhs_dtype, int64_t rhs_rows, const int32_t* pair_lhs,
                            const int32_t* pair_rhs, int64_t num_pairs, const int64_t* seg_offsets,
                            int64_t num_segments, const int32_t* seg_out_index, const int64_t* seg_strip,
                            const int32_t* pair_key, int64_t key_extent, void* out_values, int out_dtype,
                            int precision, void* workspace, size_t workspace_bytes, int32_t* error_dev,
                            void* stream, void* values_ready) {
  cudaEvent_t ready = static_cast<cudaEvent_t>(values_ready);
  EinsumDesc d;
  ES_TRY(parse_einsum(kernel_string, lhs_tile, lhs_nd, rhs_tile, rhs_nd, &d));
  if (out_dtype != ES_F32 && out_dtype != ES_BF16) return ES_ERR_UNSUPPORTED;
  auto ok_in = [](int t) { return t == ES_F32 || t == ES_BF16 || t == ES_F64; };
  if (!ok_in(lhs_dtype) || !ok_in(rhs_dtype)) return ES_ERR_UNSUPPORTED;
  cudaStream_t st = as_stream(stream);
  // the status slot needs no initialisation by the caller
  if (error_dev && cudaMemsetAsync(error_dev, 0, sizeof(int32_t), st) != cudaSuccess) return ES_ERR_CUDA;
  const int64_t nseg = seg_offsets ? num_segments : num_pairs;
  if (nseg <= 0 || num_pairs <= 0) return ES_OK;
  if (want_tc(precision)) {
    TcConfig c;
    TcVariant v;
    // the tensor-core path walks each segment's pairs as one sorted lhs
    // sequence; per-pair calls (no segments) stay on the SIMT path
    if (seg_offsets && tc_variant(kernel_string, lhs_tile, lhs_nd, rhs_tile, rhs_nd, lhs_dtype, rhs_dtype, out_dtype,
                                  seg_strip != nullptr, pair_key != nullptr && key_extent > 0, &v, &c)) {
      char* ws = static_cast<char*>(workspace);
      size_t left = workspace_bytes;
      const void* lv = lhs_values;
      const void* rv = rhs_values;
      auto take = [&](size_t bytes) -> void* {
        char* p = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(ws) + 255) & ~static_cast<uintptr_t>(255));
        const size_t used = static_cast<size_t>(p - ws) + round256(bytes);
        if (used > left) return nullptr;
        ws += used;
        left -= used;
        return p;
      };
      if (v.tl) {
        void* t = take(static_cast<size_t>(lhs_rows) * d.lhs_te * dtype_size(lhs_dtype));
        if (!t) return ES_ERR_WORKSPACE;
        if (ready && cudaStreamWaitEvent(st, ready, 0) != cudaSuccess) return ES_ERR_CUDA;
        ES_TRY(transpose_tiles(lhs_values, t, lhs_dtype, lhs_rows, lhs_tile, lhs_nd, st));
        lv = t;
      }
      // a transposed rhs needs no copy: the panel image is built from its
      // k-contiguous rows directly
      if (v.tr) c.rhs_kmajor = 1;
      const int r = tc_launch(c, lv, lhs_rows, rv, rhs_rows, pair_lhs, pair_rhs, num_pairs, seg_offsets, nseg,
                              seg_out_index, seg_strip, pair_key, key_extent, out_values, out_dtype, ws, left,
                              error_dev, st, ready);
      if (r != ES_ERR_UNSUPPORTED || precision == ES_PREC_TC) return r;
    }
    if (precision == ES_PREC_TC) return ES_ERR_UNSUPPORTED;
  }
  if (ready && cudaStreamWaitEvent(st, ready, 0) != cudaSuccess) return ES_ERR_CUDA;
  return launch_simt(d, lhs_values, lhs_dtype, rhs_values, rhs_dtype, pair_lhs, pair_rhs, seg_offsets, nseg,
                     seg_out_index, out_values, out_dtype, st);
}

extern "C" int es_tile_einsum(const char* kernel_string, const int64_t* lhs_tile, int lhs_nd, const int64_t* rhs_tile,
                              int rhs_nd, const void* lhs_values, int lhs_dtype, int64_t lhs_rows,
                              const void* rhs_values, int rhs_dtype, int64_t rhs_rows, const int32_t* pair_lhs,
                              const int32_t* pair_rhs, int64_t num_pairs, const int64_t* seg_offsets,
                              int64_t num_segments, const int32_t* seg_out_index, const int64_t* seg_strip,
                              const int32_t* pair_key, int64_t key_extent, void* out_values, int out_dtype,
                              int precision, void* workspace, size_t workspace_bytes, int32_t* error_dev,
                              void* stream) {
  return es_tile_einsum_ev(kernel_string, lhs_tile, lhs_nd, rhs_tile, rhs_nd, lhs_values, lhs_dtype, lhs_rows,
                           rhs_values, rhs_dtype, rhs_rows, pair_lhs, pair_rhs, num_pairs, seg_offsets, num_segments,
                           seg_out_index, seg_strip, pair_key, key_extent, out_values, out_dtype, precision, workspace,
                           workspace_bytes, error_dev, stream, nullptr, nullptr);
}
