// fp32 SIMT GEMM for operands with plain strided layouts:
//   acc[m][n] = sum_k A(m,k) B(k,n)
//   A(m,k) = A[m*lda + k]  (A_MCONTIG = false)   or  A[k*lda + m]  (A_MCONTIG = true)
//   B(k,n) = B[k*ldb + n]  (B_NCONTIG = true)    or  B[n*ldb + k]  (B_NCONTIG = false)
// with blockIdx.z enumerating (split, z): z offsets A and B by strideA/strideB,
// split partitions K into chunks of `kchunk` (a multiple of BK).
//
// CTA tile 128 x BN (BN = 128 or 64), BK = 8, 256 threads, each thread an
// 8 x (BN/16) register tile read from shared memory as float4 (two 4-row and
// two or one 4-column groups, 64 rows / 64 columns apart), the next k-slice
// fetched into registers while the current one is multiplied.  Every loaded
// element is passed through nan0 (the reference sanitises its operands).
// VEC_A / VEC_B: the contiguous dimension is 16-byte aligned at every row
// (ld % 4 == 0 and an aligned base) so global loads can be float4.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "nn_device.cuh"

namespace nn {

struct FastShape {
  int M, N, K;
  int nz, splits, kchunk;
  const float *A;
  long long lda, strideA;
  const float *B;
  long long ldb, strideB;
  // Tensor-core path only: when >= 0, column `ones_col` of B is all ones (not read from memory) and
  // B holds ones_col real columns -- the bias input of a weight gradient folded into the GEMM.
  int ones_col = -1;
  // Tensor-core path with TMA-loaded A and B only: when >= 0, the producers also write the sum of
  // A(m, k) over each split's k range into column `rowsum_col` of the output (the bias column of a
  // weight gradient, without an MMA column for it).  The epilogue functor stores single elements;
  // N must be a multiple of 32, so that no TMA-store box of the epilogue covers that column.
  int rowsum_col = -1;
};

template <int BN, bool A_MCONTIG, bool B_NCONTIG, bool VEC_A, bool VEC_B, class EP>
__global__ void __launch_bounds__(256) sgemm_fast_kernel(FastShape s, EP ep) {
  constexpr int BM = 128, BK = 8;
  constexpr int TN = BN / 16;  // 8 or 4 columns per thread
  __shared__ __align__(16) float As[2][BK][BM];
  __shared__ __align__(16) float Bs[2][BK][BN];
  const int tid = threadIdx.x;
  const int z = blockIdx.z % s.nz;
  const int split = blockIdx.z / s.nz;
  const int kbeg = split * s.kchunk;
  const int kend = min(s.K, kbeg + s.kchunk);
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const float *A = s.A + (size_t)z * s.strideA;
  const float *B = s.B + (size_t)z * s.strideB;

  // --- global -> register fetch mapping (each thread: 4 A values, BN/32 B values x 4 ... )
  float ra[4];
  float rb[BN / 32];
  auto fetchA = [&](int k0) {
    if (A_MCONTIG) {  // k = tid / 32, m = (tid % 32) * 4
      int k = k0 + tid / 32, m = m0 + (tid % 32) * 4;
      const float *p = A + (size_t)k * s.lda + m;
      if (VEC_A && k < kend && m + 3 < s.M) {
        float4 v = *reinterpret_cast<const float4 *>(p);
        ra[0] = v.x; ra[1] = v.y; ra[2] = v.z; ra[3] = v.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) ra[i] = (k < kend && m + i < s.M) ? p[i] : 0.f;
      }
    } else {  // m = tid / 2, k = (tid % 2) * 4
      int m = m0 + tid / 2, k = k0 + (tid % 2) * 4;
      const float *p = A + (size_t)m * s.lda + k;
      if (VEC_A && m < s.M && k + 3 < kend) {
        float4 v = *reinterpret_cast<const float4 *>(p);
        ra[0] = v.x; ra[1] = v.y; ra[2] = v.z; ra[3] = v.w;
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) ra[i] = (m < s.M && k + i < kend) ? p[i] : 0.f;
      }
    }
  };
  auto stashA = [&](int buf) {
    if (A_MCONTIG) {
      int k = tid / 32, m = (tid % 32) * 4;
      *reinterpret_cast<float4 *>(&As[buf][k][m]) = make_float4(nan0(ra[0]), nan0(ra[1]), nan0(ra[2]), nan0(ra[3]));
    } else {
      int m = tid / 2, k = (tid % 2) * 4;
#pragma unroll
      for (int i = 0; i < 4; ++i) As[buf][k + i][m] = nan0(ra[i]);
    }
  };
  auto fetchB = [&](int k0) {
    if (B_NCONTIG) {  // BN/32 floats per thread along n: k = tid / (BN/4), n = (tid % (BN/4)) * 4 ... for BN=128: 1 float4
      if (BN == 128) {
        int k = k0 + tid / 32, n = n0 + (tid % 32) * 4;
        const float *p = B + (size_t)k * s.ldb + n;
        if (VEC_B && k < kend && n + 3 < s.N) {
          float4 v = *reinterpret_cast<const float4 *>(p);
          rb[0] = v.x; rb[1] = v.y; rb[2] = v.z; rb[3] = v.w;
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) rb[i] = (k < kend && n + i < s.N) ? p[i] : 0.f;
        }
      } else {  // BN == 64: k = tid / 32, n = (tid % 32) * 2
        int k = k0 + tid / 32, n = n0 + (tid % 32) * 2;
        const float *p = B + (size_t)k * s.ldb + n;
#pragma unroll
        for (int i = 0; i < 2; ++i) rb[i] = (k < kend && n + i < s.N) ? p[i] : 0.f;
      }
    } else {  // k contiguous: n = tid / 2 (BN=128) or tid / 4 (BN=64)
      if (BN == 128) {
        int n = n0 + tid / 2, k = k0 + (tid % 2) * 4;
        const float *p = B + (size_t)n * s.ldb + k;
        if (VEC_B && n < s.N && k + 3 < kend) {
          float4 v = *reinterpret_cast<const float4 *>(p);
          rb[0] = v.x; rb[1] = v.y; rb[2] = v.z; rb[3] = v.w;
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) rb[i] = (n < s.N && k + i < kend) ? p[i] : 0.f;
        }
      } else {
        int n = n0 + tid / 4, k = k0 + (tid % 4) * 2;
        const float *p = B + (size_t)n * s.ldb + k;
#pragma unroll
        for (int i = 0; i < 2; ++i) rb[i] = (n < s.N && k + i < kend) ? p[i] : 0.f;
      }
    }
  };
  auto stashB = [&](int buf) {
    if (B_NCONTIG) {
      if (BN == 128) {
        int k = tid / 32, n = (tid % 32) * 4;
        *reinterpret_cast<float4 *>(&Bs[buf][k][n]) = make_float4(nan0(rb[0]), nan0(rb[1]), nan0(rb[2]), nan0(rb[3]));
      } else {
        int k = tid / 32, n = (tid % 32) * 2;
        Bs[buf][k][n] = nan0(rb[0]);
        Bs[buf][k][n + 1] = nan0(rb[1]);
      }
    } else {
      if (BN == 128) {
        int n = tid / 2, k = (tid % 2) * 4;
#pragma unroll
        for (int i = 0; i < 4; ++i) Bs[buf][k + i][n] = nan0(rb[i]);
      } else {
        int n = tid / 4, k = (tid % 4) * 2;
        Bs[buf][k][n] = nan0(rb[0]);
        Bs[buf][k + 1][n] = nan0(rb[1]);
      }
    }
  };

  // thread tile: rows ty*4 + {0..3} and 64 + ty*4 + {0..3}; columns tx*4 + {0..3} (+ BN/2)
  const int tx = tid % 16, ty = tid / 16;
  float acc[8][TN];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  int buf = 0;
  if (kbeg < kend) {
    fetchA(kbeg);
    fetchB(kbeg);
    stashA(0);
    stashB(0);
  }
  __syncthreads();
  for (int k0 = kbeg; k0 < kend; k0 += BK) {
    const bool more = k0 + BK < kend;
    if (more) {
      fetchA(k0 + BK);
      fetchB(k0 + BK);
    }
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[8], b[TN];
      float4 a0 = *reinterpret_cast<const float4 *>(&As[buf][kk][ty * 4]);
      float4 a1 = *reinterpret_cast<const float4 *>(&As[buf][kk][64 + ty * 4]);
      a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
      a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
      float4 b0 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][tx * 4]);
      b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
      if (TN == 8) {
        float4 b1 = *reinterpret_cast<const float4 *>(&Bs[buf][kk][BN / 2 + tx * 4]);
        b[TN - 4] = b1.x; b[TN - 3] = b1.y; b[TN - 2] = b1.z; b[TN - 1] = b1.w;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (more) {
      stashA(buf ^ 1);
      stashB(buf ^ 1);
    }
    __syncthreads();
    buf ^= 1;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    int m = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (m >= s.M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      int n = n0 + (j < 4 ? tx * 4 + j : BN / 2 + tx * 4 + (j - 4));
      if (n < s.N) ep(m, n, z, split, acc[i][j]);
    }
  }
}

// Launch with the tile width that wastes least of N, and split-K to fill the GPU.
template <bool A_MCONTIG, bool B_NCONTIG, class EP>
inline cudaError_t sgemm_fast(FastShape s, EP ep, cudaStream_t st) {
  auto aligned = [](const float *p, long long ld) { return ((uintptr_t)p % 16 == 0) && (ld % 4 == 0); };
  const bool va = aligned(s.A, s.lda) && (s.strideA % 4 == 0);
  const bool vb = aligned(s.B, s.ldb) && (s.strideB % 4 == 0);
  const bool narrow = s.N <= 64 || (s.N % 128 != 0 && s.N % 128 <= 64);
  if (s.splits < 1) s.splits = 1;
  if (s.kchunk <= 0) s.kchunk = ((s.K + s.splits - 1) / s.splits + 7) / 8 * 8;
  const int bn = narrow ? 64 : 128;
  dim3 grid((s.N + bn - 1) / bn, (s.M + 127) / 128, s.nz * s.splits);
#define NN_SGEMM_LAUNCH(BNV, VA, VB) \
  sgemm_fast_kernel<BNV, A_MCONTIG, B_NCONTIG, VA, VB><<<grid, 256, 0, st>>>(s, ep)
  if (narrow) {
    if (va && vb) NN_SGEMM_LAUNCH(64, true, true);
    else if (va) NN_SGEMM_LAUNCH(64, true, false);
    else if (vb) NN_SGEMM_LAUNCH(64, false, true);
    else NN_SGEMM_LAUNCH(64, false, false);
  } else {
    if (va && vb) NN_SGEMM_LAUNCH(128, true, true);
    else if (va) NN_SGEMM_LAUNCH(128, true, false);
    else if (vb) NN_SGEMM_LAUNCH(128, false, true);
    else NN_SGEMM_LAUNCH(128, false, false);
  }
#undef NN_SGEMM_LAUNCH
  return cudaGetLastError();
}

// split-K count for an M x N (x nz) output and reduction length K.
inline int fast_splits(int M, int N, int K, int nz) {
  long long tiles = (long long)((M + 127) / 128) * ((N + 127) / 128) * nz;
  long long want = (2 * 148 + tiles - 1) / tiles;
  long long cap = K / 512;
  if (cap < 1) cap = 1;
  if (want > cap) want = cap;
  if (want > 64) want = 64;
  return (int)(want < 1 ? 1 : want);
}

}  // namespace nn
