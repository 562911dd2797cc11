// fp32 SIMT tiled GEMM used by the dense, convolution and weight-gradient
// kernels: C[m,n] = sum_k A(m,k) B(k,n), with A and B supplied by loader
// functors (so that im2col views, per-sample strides, bias columns and the
// reference's NaN/Inf sanitising happen in the load) and the result handed to
// an epilogue functor (activation, activation derivative, Adam ...).
//
// Tiles of BM x BN outputs per CTA, BK-deep k-slices staged in shared memory
// (double buffered through registers), TM x TN outputs per thread.
// blockIdx.z enumerates (split, z) pairs: z is a per-launch batch index
// (variables of a convolution), split partitions K for split-K reductions.
#pragma once
#include <cuda_runtime.h>

namespace nn {

struct GemmShape {
  int M, N, K;
  int nz;      // number of independent z problems
  int splits;  // K partitions
};

template <int BM, int BN, int BK, int TM, int TN, bool A_KCONTIG, bool B_NCONTIG, class LA, class LB, class EP>
__global__ void __launch_bounds__((BM / TM) * (BN / TN))
gemm_simt_kernel(GemmShape sh, LA la, LB lb, EP ep) {
  constexpr int NT = (BM / TM) * (BN / TN);
  constexpr int A_PER = (BM * BK) / NT;
  constexpr int B_PER = (BK * BN) / NT;
  static_assert((BM * BK) % NT == 0 && (BK * BN) % NT == 0, "tile/thread mismatch");
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];

  const int z = blockIdx.z % sh.nz;
  const int split = blockIdx.z / sh.nz;
  const int kchunk = (sh.K + sh.splits - 1) / sh.splits;
  const int kbeg = split * kchunk;
  const int kend = min(sh.K, kbeg + kchunk);
  const int m0 = blockIdx.y * BM;
  const int n0 = blockIdx.x * BN;
  const int tid = threadIdx.x;
  const int tx = tid % (BN / TN);
  const int ty = tid / (BN / TN);

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  float ra[A_PER], rb[B_PER];
  auto fetch = [&](int k0) {
#pragma unroll
    for (int r = 0; r < A_PER; ++r) {
      int e = tid + r * NT;
      int m, k;
      if (A_KCONTIG) { k = e % BK; m = e / BK; } else { m = e % BM; k = e / BM; }
      int gm = m0 + m, gk = k0 + k;
      ra[r] = (gm < sh.M && gk < kend) ? la(gm, gk, z) : 0.f;
    }
#pragma unroll
    for (int r = 0; r < B_PER; ++r) {
      int e = tid + r * NT;
      int k, n;
      if (B_NCONTIG) { n = e % BN; k = e / BN; } else { k = e % BK; n = e / BK; }
      int gn = n0 + n, gk = k0 + k;
      rb[r] = (gn < sh.N && gk < kend) ? lb(gk, gn, z) : 0.f;
    }
  };
  auto stash = [&]() {
#pragma unroll
    for (int r = 0; r < A_PER; ++r) {
      int e = tid + r * NT;
      int m, k;
      if (A_KCONTIG) { k = e % BK; m = e / BK; } else { m = e % BM; k = e / BM; }
      As[k][m] = ra[r];
    }
#pragma unroll
    for (int r = 0; r < B_PER; ++r) {
      int e = tid + r * NT;
      int k, n;
      if (B_NCONTIG) { n = e % BN; k = e / BN; } else { k = e % BK; n = e / BK; }
      Bs[k][n] = rb[r];
    }
  };

  if (kbeg < kend) fetch(kbeg);
  for (int k0 = kbeg; k0 < kend; k0 += BK) {
    stash();
    __syncthreads();
    if (k0 + BK < kend) fetch(k0 + BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) a[i] = As[kk][ty + i * (BM / TM)];
#pragma unroll
      for (int j = 0; j < TN; ++j) b[j] = Bs[kk][tx + j * (BN / TN)];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    int gm = m0 + ty + i * (BM / TM);
    if (gm >= sh.M) continue;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      int gn = n0 + tx + j * (BN / TN);
      if (gn < sh.N) ep(gm, gn, z, split, acc[i][j]);
    }
  }
}

// Host launcher: picks the tile and the grid.
template <bool A_KCONTIG, bool B_NCONTIG, class LA, class LB, class EP>
inline cudaError_t gemm_simt(const GemmShape &sh, LA la, LB lb, EP ep, cudaStream_t s) {
  constexpr int BM = 64, BN = 64, BK = 16, TM = 4, TN = 4;
  dim3 grid((sh.N + BN - 1) / BN, (sh.M + BM - 1) / BM, sh.nz * sh.splits);
  gemm_simt_kernel<BM, BN, BK, TM, TN, A_KCONTIG, B_NCONTIG><<<grid, (BM / TM) * (BN / TN), 0, s>>>(sh, la, lb,
                                                                                                    ep);
  return cudaGetLastError();
}

// Number of K partitions that fills the machine with at least ~2 waves of CTAs
// while keeping every partition at least `min_chunk` deep.
inline int pick_splits(int M, int N, int K, int nz, int min_chunk = 256) {
  long long tiles = (long long)((M + 63) / 64) * ((N + 63) / 64) * nz;
  long long want = (2 * 148 + tiles - 1) / tiles;
  long long cap = K / min_chunk;
  if (cap < 1) cap = 1;
  if (want > cap) want = cap;
  if (want > 64) want = 64;
  return (int)(want < 1 ? 1 : want);
}

}  // namespace nn
