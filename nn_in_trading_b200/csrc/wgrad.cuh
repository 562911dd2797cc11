// Weight-gradient reductions shared by the dense and convolution update
// kernels.  A batched update first reduces the per-sample weight gradients
// sum_b A(m,b..) B(b..,n) with a split-K SIMT GEMM into per-split partials,
// then an apply kernel sums the partials, scales by 1/batch and runs the
// reference update arithmetic on every weight.  In a data-parallel update
// region the summed, scaled gradient is written to the gradient arena
// instead, averaged over ranks, and applied afterwards.
#pragma once
#include "gemm_fast.cuh"
#include "tc_gemm.cuh"
#include "gemm_simt.cuh"
#include "nn_device.cuh"
#include "nn_internal.h"

namespace nn {

struct PartialStore {
  float *p;
  int M, N, nz;
  __device__ void operator()(int m, int n, int z, int split, float acc) const {
    p[(((size_t)split * nz + z) * M + m) * N + n] = acc;
  }
};

// Gradient source for an apply kernel: G(idx) = scale * sum_s p[s*stride + idx].
struct GradSrc {
  const float *p;
  int splits;
  size_t stride;
  float scale;
  // rows of `ncol` gradient entries stored `ld` floats apart (ld == ncol: dense, the default)
  int ld = 0, ncol = 0;
  __device__ __forceinline__ size_t at(size_t i) const {
    return ld == ncol ? i : (i / (size_t)ncol) * (size_t)ld + i % (size_t)ncol;
  }
  __device__ __forceinline__ float operator()(size_t idx) const {
    const size_t j = at(idx);
    float s = 0.f;
#pragma unroll 4
    for (int k = 0; k < splits; ++k) s += p[k * stride + j];
    return s * scale;
  }
};

__global__ void reduce_partials_kernel(float *out, GradSrc src, size_t n);

// NormalizeWeights (defined with the dense kernels): rows of `dim` weights rescaled to unit norm.
__global__ void normalize_weights_kernel(float *buf, int rows, int dim);

// A single-sample weight update followed by NormalizeWeights of the rows it updated
// (NeuroNet_Core.mqh:15971-15977), in one kernel: one block of 256 threads per row of `dim` weights;
// step(i) applies the update arithmetic to weight i of the row-major matrix, stores it and returns what
// it stored; each thread accumulates the squares of its own columns, the block sums them (in another
// order than normalize_weights_kernel, so the norm may differ in its last bit), and the row is
// rescaled when its norm exceeds 1, with normalize_weights_kernel's retry when the sum overflows.
template <class Step>
__global__ void __launch_bounds__(256) update_normalize_rows_flat_kernel(float *w, int rows, int dim, Step step) {
  __shared__ float part[8];
  __shared__ float row_d;
  const int row = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  pdl_wait();  // a no-op unless launched with programmatic dependent launch
  pdl_trigger();
  if (row >= rows) return;
  float *wr = w + (size_t)row * dim;
  float s = 0.f;
  for (int col = t; col < dim; col += 256) {
    const float q = nan0(step((size_t)row * dim + col));
    s += q * q;
  }
  s = warp_sum(s);
  if (lane == 0) part[warp] = s;
  __syncthreads();
  if (warp == 0) {
    s = lane < 8 ? part[lane] : 0.f;
    s = warp_sum(s);
    float k = 1.f;
    for (int guard = 1; !isfinite(s) && guard < 64; ++guard) {
      k *= 10.f;
      s = 0.f;
      for (int i = lane; i < dim; i += 32) {
        const float q = nan0(wr[i]) / k;
        s += q * q;
      }
      s = warp_sum(s);
    }
    if (lane == 0) row_d = k * sqrtf(s);
  }
  __syncthreads();
  const float d = row_d;
  if (d > 1.f)
    for (int i = t; i < dim; i += 256) wr[i] = nan0(wr[i]) / d;
}



// Partial store for the fast GEMM: N computed columns inside rows of `ldp` (the bias
// column N of each row is filled by colsum_partial_kernel).
struct PartialStoreLd {
  float *p;
  int M, ldp, nz;
  __device__ void operator()(int m, int n, int z, int split, float acc) const {
    p[(((size_t)split * nz + z) * M + m) * ldp + n] = acc;
  }
  __device__ __forceinline__ long long row(int m, int z, int split) const {
    return (((long long)split * nz + z) * M + m) * ldp;
  }
  __device__ __forceinline__ float col(int, int) const { return 0.f; }
  template <int R>
  __device__ __forceinline__ void put_rows(const long long (&rb)[R], int n, const float (&v)[R], float,
                                           unsigned mask) const {
#pragma unroll
    for (int j = 0; j < R; ++j)
      if (mask >> j & 1u) p[rb[j] + n] = v[j];
  }
  __host__ __device__ bool aligned4() const { return (ldp) % 4 == 0 && ((uintptr_t)p & 15) == 0; }
  __device__ __forceinline__ float4 col4(int, int) const { return make_float4(0.f, 0.f, 0.f, 0.f); }
  template <int R>
  __device__ __forceinline__ void put_rows4(const long long (&rb)[R], int n, const float4 (&v)[R], float4,
                                            unsigned mask) const {
#pragma unroll
    for (int j = 0; j < R; ++j)
      if (mask >> j & 1u) *reinterpret_cast<float4 *>(p + rb[j] + n) = v[j];
  }
};

// PartialStoreLd through TMA stores: rows padded to a multiple of 4 floats (16-byte row stride), the
// split as the tensor's outer coordinate.
struct PartialStoreTma : PartialStoreLd {
  static constexpr bool kTmaStore = true;
  static constexpr bool kRowSum = true;
  template <class F>
  __device__ __forceinline__ void transform(F &&f) const {
    f([](float x, float, float) { return x; });
  }
  __device__ __forceinline__ int zc(int z, int split) const { return split * nz + z; }
  bool out_map(CUtensorMap *tm, int rows, int cols, int outer) const {
    return make_tmap(tm, p, ldp, (long long)M * ldp, cols, rows, outer, 32, false);
  }
};

// Partial store of a transposed product: the GEMM computed C^T (its rows are the gradient's columns
// n, its columns the gradient's rows m); element (n, m) of split s goes to p[(s*M + m)*ldp + n].
// The tensor-core epilogue stores it column by column from the accumulator rows (kColMajor), so
// the lanes (consecutive n) write consecutive addresses.
struct PartialStoreT {
  static constexpr bool kColMajor = true;
  float *p;
  int M, ldp;
  __device__ void operator()(int n, int m, int, int split, float acc) const {
    p[((size_t)split * M + m) * ldp + n] = acc;
  }
  __device__ __forceinline__ long long row(int n, int, int split) const { return (long long)split * M * ldp + n; }
  __device__ __forceinline__ void put_col(long long rowoff, int m, float v) const { p[rowoff + (long long)m * ldp] = v; }
  // (the row-major protocol, unused when kColMajor)
  __host__ __device__ bool aligned4() const { return false; }
  __device__ __forceinline__ float col(int, int) const { return 0.f; }
  __device__ __forceinline__ float4 col4(int, int) const { return make_float4(0.f, 0.f, 0.f, 0.f); }
  template <int R>
  __device__ __forceinline__ void put_rows(const long long (&rb)[R], int m, const float (&v)[R], float,
                                           unsigned mask) const {
#pragma unroll
    for (int j = 0; j < R; ++j)
      if (mask >> j & 1u) put_col(rb[j], m, v[j]);
  }
  template <int R>
  __device__ __forceinline__ void put_rows4(const long long (&rb)[R], int m, const float4 (&v)[R], float4,
                                            unsigned mask) const {}
};

// Bias column of a weight gradient: per split, sum over the split's reduction
// rows r of nan0(g[r*ld + m]) into p[(split*M + m)*ldp + col].
__global__ void colsum_partial_kernel(float *p, const float *g, int M, int rows, long long ld, int kchunk, int ldp,
                                      int col);
// Same, 32 columns x 8 row lanes per block (block 32 x 8, grid (ceil(M/32), splits)).
__global__ void colsum_rows_kernel(float *p, const float *g, int M, int rows, long long ld, int kchunk, int ldp,
                                   int col);

// Weight gradient with at most kSmallM outputs: per split, G[m][n] = sum_r nan0(A[r*lda + m])
// nan0(X[r*ldx + n]) for n < N and the bias column G[m][N] = sum_r nan0(A[r*lda + m]), into
// p[(split*M + m)*ldp + n].  Block (32 columns, 8 row lanes), grid (ceil((N+1)/32), splits).
constexpr int kSmallM = 16;
__global__ void wgrad_small_m_kernel(float *p, const float *A, long long lda, const float *X, long long ldx, int M,
                                     int N, int rows, int kchunk, int ldp);

// Split-K count of a product with `tiles` output tiles: the fewest splits (at most `cap`) whose work
// items fill whole waves of the 148 SMs within 3 % of the best of one, two or three waves.  The time of
// a split product goes as tiles / (SMs x wave efficiency), so equal efficiencies cost the same and the
// fewer partials to sum win.
inline int wave_splits(long long tiles, long long cap) {
  const long long sms = 148;
  if (tiles >= sms) return 1;
  if (cap < 1) cap = 1;
  long long cand[3];
  double eff[3], best = 0.0;
  for (int w = 1; w <= 3; ++w) {
    long long sp = w * sms / tiles;
    if (sp > cap) sp = cap;
    if (sp < 1) sp = 1;
    const long long items = tiles * sp;
    cand[w - 1] = sp;
    eff[w - 1] = (double)items / (double)(sms * ((items + sms - 1) / sms));
    if (eff[w - 1] > best) best = eff[w - 1];
  }
  long long pick = cand[2];
  for (int i = 0; i < 3; ++i)
    if (eff[i] >= best - 0.03 && cand[i] < pick) pick = cand[i];
  return (int)pick;
}

// Split-K count of a weight gradient (the reduction runs over the batch's rows, few 128 x 128 output
// tiles): whole waves as above, at least 256 rows per split.  (A fixed target of two waves capped at 64
// splits left 64 of 148 SMs busy for a single tile over a million rows.)
inline int wgrad_splits(int M, int N, int K) {
  const long long tiles = (long long)((M + 127) / 128) * ((N + 127) / 128);
  return wave_splits(tiles, K / 256);
}

// Weight gradient of a plain GEMM: G[m][n] = sum_r A[r*lda + m] * X[r*ldx + n] for n < N, and
// G[m][N] = sum_r A[r*lda + m] (the bias column, input 1).  Partials per split into scratch 0.
inline int wgrad_fast(Launch &L, const float *A, long long lda, const float *X, long long ldx, int M, int N, int rows,
                      GradSrc *out) {
  int splits = wgrad_splits(M, N, rows);
  // tensor-core path: split boundaries on its 32-deep stages (so TMA can load whole stages)
  const int gran = tc_path(FastShape{M, N, rows, 1, 1, 0, A, lda, 0, X, ldx, 0}) ? 32 : 8;
  int kchunk = ((rows + splits - 1) / splits + gran - 1) / gran * gran;
  splits = (rows + kchunk - 1) / kchunk;
  if (splits < 1) splits = 1;
  FastShape fs{M, N, rows, 1, splits, kchunk, A, lda, 0, X, ldx, 0};
  const bool tc = tc_path(fs), transposed = tc && M < 128 && N >= 128;
  // partial rows: N + 1 entries, padded to a multiple of 4 floats when the GEMM's epilogue writes
  // them with TMA stores (the tensor-core product with the bias column folded in)
  const int ldp = (tc && !transposed) ? (N + 1 + 3) / 4 * 4 : N + 1;
  size_t per = (size_t)M * ldp;
  float *part = L.scratch(0, per * splits);
  if (!part) return NN_ERR_CUDA;
  out->ld = out->ncol = 0;
  if (transposed) {
    // few outputs, many inputs: the transposed product X^T A^T fills the 128-row tiles with the
    // inputs instead of padding the outputs; the bias column is a separate column sum of A
    FastShape ft{N, M, rows, 1, splits, kchunk, X, ldx, 0, A, lda, 0};
    cudaError_t e = tcgemm<true, true>(ft, PartialStoreT{part, M, ldp}, L.stream, device_status());
    if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
    L.counted();
    NN_LAUNCH_PDL(L, colsum_rows_kernel, dim3((M + 31) / 32, splits), dim3(32, 32), 0, L.stream, part, A, M, rows, lda, kchunk, ldp, N);
  } else if (tc) {
    if (N % 32 == 0 && tcgemm_row_sum_ok(fs)) {
      // the bias input (1): its gradient column is the row sum of A, which the GEMM's producer warps
      // accumulate while they split A, so the MMAs cover the N real columns only.  The epilogue's
      // 32-column TMA-store boxes then end at column N: a box clipped inside a row would share a
      // 16-byte chunk with the bias column, and its store could land after the producers' one.
      fs.rowsum_col = N;
    } else {
      // the bias input (1) is column N of X: one GEMM writes all N + 1 gradient columns
      fs.N = N + 1;
      fs.ones_col = N;
    }
    cudaError_t e = tcgemm<true, true>(fs, PartialStoreTma{{part, M, ldp, 1}}, L.stream, device_status());
    if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
    L.counted();
    out->ld = ldp;
    out->ncol = N + 1;
  } else if (M <= kSmallM) {
    // few outputs: one pass over X computes every output row (a 128-row GEMM tile would be mostly
    // padding); the bias column is column N of the same pass
    NN_LAUNCH_PDL(L, wgrad_small_m_kernel, dim3((N + 1 + 31) / 32, splits), dim3(32, 8), 0, L.stream, part, A, lda, X, ldx, M, N, rows, kchunk, ldp);
  } else {
    cudaError_t e = sgemm_fast<true, true>(fs, PartialStoreLd{part, M, ldp, 1}, L.stream);
    if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
    L.counted();
    dim3 grid((M + 255) / 256, splits);
    NN_LAUNCH_PDL(L, colsum_partial_kernel, grid, 256, 0, L.stream, part, A, M, rows, lda, kchunk, ldp, N);
  }
  out->p = part;
  out->splits = splits;
  out->stride = per;
  out->scale = 1.f;
  return NN_OK;
}

// Runs the split-K GEMM into scratch slot 0 and returns the gradient source
// (not yet scaled).  M x N per z problem, K reduction length.
template <bool AK, bool BN, class LA, class LB>
inline int wgrad_partials(Launch &L, int M, int N, int K, int nz, LA la, LB lb, GradSrc *out) {
  int splits = pick_splits(M, N, K, nz);
  size_t per = (size_t)M * N * nz;
  float *part = L.scratch(0, per * splits);
  if (!part) return NN_ERR_CUDA;
  GemmShape sh{M, N, K, nz, splits};
  cudaError_t e = gemm_simt<AK, BN>(sh, la, lb, PartialStore{part, M, N, nz}, L.stream);
  if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
  L.counted();
  out->p = part;
  out->splits = splits;
  out->stride = per;
  out->scale = 1.f;
  return NN_OK;
}

// Either hands `src` to `apply` directly, or (inside a data-parallel update
// region) reduces it into an arena slot and defers `apply` until the ranks'
// gradients have been averaged.
inline int finish_update(Launch &L, GradSrc src, size_t n, int (*apply)(const Launch &, const float *),
                         int (*apply_src)(const Launch &, GradSrc)) {
  if (L.deferred()) {
    float *slot = L.grad_slot(n);
    if (!slot) return NN_ERR_BOUNDS;
    NN_LAUNCH_PDL(L, reduce_partials_kernel, (unsigned)((n + 31) / 32), dim3(32, 8), 0, L.stream, slot, src, n);
    L.defer(apply, slot);
    return NN_OK;
  }
  return apply_src(L, src);
}

}  // namespace nn
