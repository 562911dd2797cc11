// General matrix products of the reference library, for the layers that multiply activations by
// activations (or by a weight matrix held as a plain buffer):
//   MatMult      result[v] = matr1[v] . matr2[v or 0]                    NeuroNet.cl:5969-6013
//   MatMultGrad  matr1_gr[v] = result_gr[v] . matr2[v or 0]^T,
//                matr2_gr[v] = matr1[v]^T . result_gr[v]  (summed over v when matr2 is shared)
//                                                                        NeuroNet.cl:6018-6060
// NDRange (rows, cols, variables); matr1 is [v][rows][dimension], matr2 [v][dimension][cols] when
// multvarsecond is set (one shared [dimension][cols] matrix otherwise), result [v][rows][cols], each
// at its raw-buffer offset.  Every product passes through IsNaNOrInf(., 0): a product with a
// non-finite operand adds nothing, which the GEMM cores reproduce by zeroing non-finite operands.
// MatMultGrad also passes each finished sum through IsNaNOrInf(., 0).
//
// Both run on the library's GEMM cores (tcgen05 3xTF32 tiles for large products, the SIMT tile
// below that); a product whose output tiles cannot fill the GPU but whose reduction is long is
// split along k into partial products summed in split order by a second kernel (deterministic).
//
// With numeric flags (MatMult's flags_enabled), flags[v][row][col] = 1 where an operand, a
// product or the running sum was not finite.  An operand that is not finite makes its product
// not finite, so the flag is (row of matr1 not finite) | (column of matr2 not finite) | (sum not
// finite) | (a product of two finite operands overflowed).  The last can only happen where
// max|row| * max|column| reaches FLT_MAX; those outputs are recomputed in the reference's order,
// dropping the overflowing products as it does, so flags and results match it exactly.
//
// Batches: the variables dimension is the batch of these kernels (a per-sample matr2 with
// multvarsecond = 1, a shared one with 0, whose gradient MatMultGrad then sums over the batch), so
// nn_set_batch > 1 is refused.
#include <cfloat>

#include "../../include/nn_b200.h"
#include "gemm_fast.cuh"
#include "nn_device.cuh"
#include "nn_internal.h"
#include "tc_gemm.cuh"

namespace nn {

// Output of a product (or of one k split of it): element (m, n) of matrix z of split `split`
// at o + ((split * nz + z) * M + m) * ld + n, optionally through IsNaNOrInf(., 0).
template <bool NAN0>
struct MatEpi {
  float *o;
  long long ld, M;
  int nz;
  __device__ __forceinline__ float fix(float x) const { return NAN0 ? nan0(x) : x; }
  __device__ __forceinline__ long long row(int m, int z, int split) const {
    return (((long long)split * nz + z) * M + m) * ld;
  }
  __device__ __forceinline__ void operator()(int m, int n, int z, int split, float acc) const {
    o[row(m, z, split) + n] = fix(acc);
  }
  __device__ __forceinline__ float col(int, int) const { return 0.f; }
  __device__ __forceinline__ float4 col4(int, int) const { return make_float4(0.f, 0.f, 0.f, 0.f); }
  template <int R>
  __device__ __forceinline__ void put_rows(const long long (&rb)[R], int n, const float (&v)[R], float,
                                           unsigned mask) const {
#pragma unroll
    for (int j = 0; j < R; ++j)
      if (mask >> j & 1u) o[rb[j] + n] = fix(v[j]);
  }
  __host__ __device__ bool aligned4() const { return ld % 4 == 0 && ((uintptr_t)o & 15) == 0; }
  template <int R>
  __device__ __forceinline__ void put_rows4(const long long (&rb)[R], int n, const float4 (&v)[R], float4,
                                            unsigned mask) const {
#pragma unroll
    for (int j = 0; j < R; ++j)
      if (mask >> j & 1u)
        *reinterpret_cast<float4 *>(o + rb[j] + n) = make_float4(fix(v[j].x), fix(v[j].y), fix(v[j].z), fix(v[j].w));
  }
};

// Sum of the k splits in split order: e enumerates (z, m, n) of the compact partials.
template <bool NAN0>
__global__ void mat_split_sum_kernel(const float *__restrict__ part, int splits, long long per_split, int N,
                                     float *__restrict__ o, long long ld) {
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < per_split;
       e += (long long)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int sp = 0; sp < splits; ++sp) s += part[sp * per_split + e];
    const long long r = e / N;
    o[r * ld + (e - r * N)] = NAN0 ? nan0(s) : s;
  }
}

// k splits for an M x N (x nz) product with reduction length K: only when its tiles leave most SMs
// idle and the reduction is long enough to share.
static int mat_splits(int M, int N, int K, int nz) {
  const long long tiles = (long long)((M + 127) / 128) * ((N + 127) / 128) * nz;
  if (tiles >= 148 || K < 2048) return 1;
  return fast_splits(M, N, K, nz);
}

// out[z][m][n] (rows ld apart, M rows per z) = sum_k A(m,k) B(k,n) for the layouts of `s`.
template <bool A_MCONTIG, bool B_NCONTIG, bool NAN0>
static int mat_product(Launch &L, FastShape s, float *out, long long ld, int scratch_slot) {
  if (s.M <= 0 || s.N <= 0 || s.nz <= 0) return NN_OK;
  s.splits = mat_splits(s.M, s.N, s.K, s.nz);
  s.kchunk = 0;
  cudaError_t e;
  if (s.splits == 1) {
    e = gemm_f32<A_MCONTIG, B_NCONTIG>(s, MatEpi<NAN0>{out, ld, s.M, s.nz}, L.stream);
    if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
    L.counted();
    return NN_OK;
  }
  const long long per_split = (long long)s.nz * s.M * s.N;
  float *part = L.scratch(scratch_slot, (size_t)per_split * s.splits);
  if (!part) return L.fail(NN_ERR_CUDA, "MatMult: split-K scratch allocation failed");
  e = gemm_f32<A_MCONTIG, B_NCONTIG>(s, MatEpi<false>{part, s.N, s.M, s.nz}, L.stream);
  if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
  L.counted();
  const long long blocks = std::min<long long>((per_split + 255) / 256, 148LL * 16);
  mat_split_sum_kernel<NAN0><<<(unsigned)blocks, 256, 0, L.stream>>>(part, s.splits, per_split, s.N, out, ld);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

// ------------------------------------------------------------- numeric flags
// Per (v, row) of matr1: whether an entry is not finite, and the largest finite |entry|.  A warp
// per row.
__global__ void mat_row_stats_kernel(const float *__restrict__ a, long long nrows, int dim, float *__restrict__ amax,
                                     int *__restrict__ abad) {
  const long long r = (blockIdx.x * (long long)blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (r >= nrows) return;
  const float *p = a + r * dim;
  float mx = 0.f;
  int bad = 0;
  for (int i = lane; i < dim; i += 32) {
    const float x = p[i];
    if (isfinite(x)) mx = fmaxf(mx, fabsf(x));
    else bad = 1;
  }
  for (int o = 16; o > 0; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    bad |= __shfl_xor_sync(0xffffffffu, bad, o);
  }
  if (lane == 0) {
    amax[r] = mx;
    abad[r] = bad;
  }
}

// Per (v, col) of matr2 ([nv][dim][cols]): 32 columns per block, 8 thread rows sharing the k range.
__global__ void __launch_bounds__(256) mat_col_stats_kernel(const float *__restrict__ b, int dim, int cols,
                                                            float *__restrict__ bmax, int *__restrict__ bbad) {
  __shared__ float smx[8][33];
  __shared__ int sbad[8][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + tx, v = blockIdx.y;
  float mx = 0.f;
  int bad = 0;
  if (c < cols) {
    const float *p = b + (long long)v * dim * cols + c;
    for (int i = ty; i < dim; i += 8) {
      const float x = p[(long long)i * cols];
      if (isfinite(x)) mx = fmaxf(mx, fabsf(x));
      else bad = 1;
    }
  }
  smx[ty][tx] = mx;
  sbad[ty][tx] = bad;
  __syncthreads();
  if (ty == 0 && c < cols) {
    for (int j = 1; j < 8; ++j) {
      mx = fmaxf(mx, smx[j][tx]);
      bad |= sbad[j][tx];
    }
    bmax[(long long)v * cols + c] = mx;
    bbad[(long long)v * cols + c] = bad;
  }
}

// One thread per output: the flag, and the reference-order sum where a product may overflow.
__global__ void mat_flags_kernel(const float *__restrict__ a, const float *__restrict__ b, float *__restrict__ res,
                                 float *__restrict__ flags, int rows, int cols, int dim, int var, int mvs,
                                 const float *__restrict__ amax, const int *__restrict__ abad,
                                 const float *__restrict__ bmax, const int *__restrict__ bbad) {
  const long long total = (long long)var * rows * cols;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < total;
       e += (long long)gridDim.x * blockDim.x) {
    const long long vr = e / cols;
    const int c = (int)(e - vr * cols);
    const int v = (int)(vr / rows);
    const long long bc = (long long)(mvs ? v : 0) * cols + c;
    int invalid = abad[vr] | bbad[bc];
    if ((double)amax[vr] * (double)bmax[bc] >= (double)FLT_MAX) {
      const float *ar = a + vr * dim;
      const float *bp = b + (long long)(mvs ? v : 0) * dim * cols + c;
      float s = 0.f;
      for (int i = 0; i < dim; ++i) {
        const float p = __fmul_rn(ar[i], bp[(long long)i * cols]);
        if (isfinite(p)) s = __fadd_rn(s, p);
        else invalid = 1;
      }
      res[e] = s;
    }
    if (!isfinite(res[e])) invalid = 1;
    flags[e] = invalid ? 1.f : 0.f;
  }
}

// ------------------------------------------------------------------- MatMult
static int k_mat_mult(Launch &L) {
  if (L.B != 1) return L.fail(NN_ERR_UNSUPPORTED, "MatMult: the batch goes in global[2] (variables)");
  const int rows = (int)L.nd.g[0], cols = L.nd.dims > 1 ? (int)L.nd.g[1] : 1;
  const int var = L.nd.dims > 2 ? (int)L.nd.g[2] : 1;
  const int dim = L.i(3), mvs = L.i(4) != 0, off1 = L.i(5), off2 = L.i(6), offr = L.i(7);
  const int flags_on = L.i(9) != 0;
  if (dim < 0 || off1 < 0 || off2 < 0 || offr < 0) return L.fail(NN_ERR_ARG, "MatMult: negative size or offset");
  const size_t n_out = (size_t)var * rows * cols;
  float *m1 = L.buf(0, off1 + (size_t)var * rows * dim);
  float *m2 = L.buf(1, off2 + (size_t)(mvs ? var : 1) * dim * cols);
  float *r = L.buf(2, offr + n_out);
  if (!m1 || !m2 || !r) return NN_ERR_BOUNDS;
  float *flags = nullptr;
  if (flags_on) {
    if (L.handle(8) == L.handle(0) || L.handle(8) == L.handle(1) || L.handle(8) == L.handle(2))
      return L.fail(NN_ERR_ARG, "MatMult: numeric_flags must be its own buffer");
    flags = L.buf(8, n_out);
    if (!flags) return NN_ERR_BOUNDS;
  }
  const float *A = m1 + off1, *Bm = m2 + off2;
  float *R = r + offr;
  FastShape fs{rows, cols, dim, var, 1, 0, A, dim, (long long)rows * dim, Bm, cols, mvs ? (long long)dim * cols : 0};
  int st = mat_product<false, true, false>(L, fs, R, cols, 0);
  if (st != NN_OK || !flags_on) return st;
  const long long nrows = (long long)var * rows, nbv = mvs ? var : 1;
  float *amax = L.scratch(1, (size_t)(nrows + nbv * cols) * 2);
  if (!amax) return L.fail(NN_ERR_CUDA, "MatMult: flag scratch allocation failed");
  float *bmax = amax + nrows;
  int *abad = reinterpret_cast<int *>(bmax + nbv * cols);
  int *bbad = abad + nrows;
  mat_row_stats_kernel<<<grid1d((size_t)nrows * 32, 256), 256, 0, L.stream>>>(A, nrows, dim, amax, abad);
  NN_CHECK_LAUNCH(L);
  mat_col_stats_kernel<<<dim3((cols + 31) / 32, (unsigned)nbv), 256, 0, L.stream>>>(Bm, dim, cols, bmax, bbad);
  NN_CHECK_LAUNCH(L);
  const long long blocks = std::min<long long>(((long long)n_out + 255) / 256, 148LL * 16);
  mat_flags_kernel<<<(unsigned)blocks, 256, 0, L.stream>>>(A, Bm, R, flags, rows, cols, dim, var, mvs, amax, abad,
                                                           bmax, bbad);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

// --------------------------------------------------------------- MatMultGrad
static int k_mat_mult_grad(Launch &L) {
  if (L.B != 1) return L.fail(NN_ERR_UNSUPPORTED, "MatMultGrad: the batch goes in global[2] (variables)");
  const int rows = (int)L.nd.g[0], cols = L.nd.dims > 1 ? (int)L.nd.g[1] : 1;
  const int var = L.nd.dims > 2 ? (int)L.nd.g[2] : 1;
  const int dim = L.i(5), mvs = L.i(6) != 0;
  const int off1 = L.i(7), off1g = L.i(8), off2 = L.i(9), off2g = L.i(10), offr = L.i(11);
  if (dim < 0 || off1 < 0 || off1g < 0 || off2 < 0 || off2g < 0 || offr < 0)
    return L.fail(NN_ERR_ARG, "MatMultGrad: negative size or offset");
  const size_t n1 = (size_t)var * rows * dim, n2 = (size_t)(mvs ? var : 1) * dim * cols;
  float *m1 = L.buf(0, off1 + n1), *m1g = L.buf(1, off1g + n1);
  float *m2 = L.buf(2, off2 + n2), *m2g = L.buf(3, off2g + n2);
  float *rg = L.buf(4, offr + (size_t)var * rows * cols);
  if (!m1 || !m1g || !m2 || !m2g || !rg) return NN_ERR_BOUNDS;
  const float *A = m1 + off1, *Bm = m2 + off2, *G = rg + offr;
  // matr1_gr[v] (rows x dim) = G[v] (rows x cols) . matr2[v]^T: B(k = i, n = f) = matr2[f * cols + i]
  FastShape da{rows, dim, cols, var, 1, 0, G, cols, (long long)rows * cols,
               Bm, cols, mvs ? (long long)dim * cols : 0};
  int st = mat_product<false, false, true>(L, da, m1g + off1g, dim, 0);
  if (st != NN_OK) return st;
  // matr2_gr (dim x cols) = matr1^T . G per variable, or over the variables stacked along k
  FastShape db = mvs ? FastShape{dim, cols, rows, var, 1, 0, A, dim, (long long)rows * dim, G, cols,
                                 (long long)rows * cols}
                     : FastShape{dim, cols, rows * var, 1, 1, 0, A, dim, 0, G, cols, 0};
  return mat_product<true, true, true>(L, db, m2g + off2g, cols, 0);
}

const KernelDef kMatKernels[] = {
    {"MatMult", "pppiiiiipi", k_mat_mult, false},
    {"MatMultGrad", "pppppiiiiiii", k_mat_mult_grad, false},
};
const int kNumMatKernels = sizeof(kMatKernels) / sizeof(kMatKernels[0]);

}  // namespace nn
