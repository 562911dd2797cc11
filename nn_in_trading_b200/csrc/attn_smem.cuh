// Shared-memory-resident attention kernels: one CTA per (sample, head) holds
// the head's whole score matrix and its Q/K/V/gradient slices on chip, so each
// operand crosses HBM once.  Used when units^2 + a few units*dim floats fit in
// shared memory (units up to ~180 at dim 32); larger shapes take the streaming
// kernels in k_attn.cu.
//
// Thread mapping of every product: a warp owns blocks of 4 output rows, its
// lanes own the feature (or key) columns; the row operand is read as float4
// broadcasts along k and the column operand conflict-free across lanes, i.e.
// 8 shared loads per 16 FMAs.
#pragma once
#include <cstdint>

#include "nn_device.cuh"

namespace nn {

// rows of an smem matrix padded to a multiple of 4 floats (float4 alignment)
__host__ __device__ __forceinline__ int pad4(int n) { return (n + 3) & ~3; }

// Load `rows` vectors of `dim` floats from global (row r at src + r*stride) into
// smem dst[r*ld + d], optionally sanitised.
__device__ __forceinline__ void load_rows(float *dst, int ld, const float *src, size_t stride, int rows, int dim,
                                          bool sanitize) {
  for (int e = threadIdx.x; e < rows * dim; e += blockDim.x) {
    int r = e / dim, d = e - r * dim;
    float v = src[(size_t)r * stride + d];
    dst[r * ld + d] = sanitize ? nan0(v) : v;
  }
}

// Copy `rows` rows of `cols` floats (row r at src + r*stride) into smem dst[r*ld + c]
// with 16-byte cp.async when every row start is 16-byte aligned, else plain loads.
// Warps take rows, lanes take 16-byte chunks: no division, many copies in flight.
// The caller waits with async_wait_all() and a __syncthreads().
__device__ __forceinline__ void async_rows(float *dst, int ld, const float *src, size_t stride, int rows, int cols) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const bool vec = (cols % 4 == 0) && (ld % 4 == 0) && (stride % 4 == 0) && ((uintptr_t)src % 16 == 0);
  if (vec) {
    const int c4 = cols / 4;
    for (int r = warp; r < rows; r += nw) {
      const float *s = src + (size_t)r * stride;
      float *d = dst + r * ld;
      for (int c = lane; c < c4; c += 32) {
        unsigned saddr = (unsigned)__cvta_generic_to_shared(d + 4 * c);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(saddr), "l"(s + 4 * c));
      }
    }
    asm volatile("cp.async.commit_group;\n" ::);
  } else {  // rows not 16-byte aligned: 4-byte copies, still all in flight
    for (int r = warp; r < rows; r += nw) {
      const float *s = src + (size_t)r * stride;
      float *d = dst + r * ld;
      for (int c = lane; c < cols; c += 32) {
        unsigned saddr = (unsigned)__cvta_generic_to_shared(d + c);
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(saddr), "l"(s + c));
      }
    }
    asm volatile("cp.async.commit_group;\n" ::);
  }
}
__device__ __forceinline__ void async_wait_all() { asm volatile("cp.async.wait_group 0;\n" ::); }

// out[r][c] (r < R, c < N) = sum_k A[r*lda + k] * Bm[k*ldb + c], A rows via float4,
// computed by warps over 4-row blocks and lanes over columns c = lane + 32 j.
// The functor `emit(r, c, acc)` receives each result.  DPL = ceil(N / 32) <= 4.
// SUB = 2 (N <= 16): each half-warp takes its own 4-row block, lanes c = lane % 16.
template <int DPL, class Emit, int SUB = 1>
__device__ __forceinline__ void rows_times_cols(const float *A, int lda, const float *Bm, int ldb, int R, int N,
                                                int K, Emit emit) {
  constexpr int CL = 32 / SUB;  // column lanes
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int cl = lane % CL, sub = lane / CL;
  for (int rb = warp * 4 * SUB; rb < R; rb += nw * 4 * SUB) {
    const int r0 = rb + 4 * sub;
    float acc[4][DPL];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < DPL; ++j) acc[i][j] = 0.f;
    const int nr = max(0, min(4, R - r0));
    int k = 0;
    for (; k + 4 <= K; k += 4) {
      float4 a[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        a[i] = (i < nr) ? *reinterpret_cast<const float4 *>(A + (r0 + i) * lda + k) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < DPL; ++j) {
        int c = cl + CL * j;
        if (c < N) {
          float b0 = Bm[(k + 0) * ldb + c], b1 = Bm[(k + 1) * ldb + c];
          float b2 = Bm[(k + 2) * ldb + c], b3 = Bm[(k + 3) * ldb + c];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            acc[i][j] = fmaf(a[i].x, b0, acc[i][j]);
            acc[i][j] = fmaf(a[i].y, b1, acc[i][j]);
            acc[i][j] = fmaf(a[i].z, b2, acc[i][j]);
            acc[i][j] = fmaf(a[i].w, b3, acc[i][j]);
          }
        }
      }
    }
    for (; k < K; ++k) {
#pragma unroll
      for (int j = 0; j < DPL; ++j) {
        int c = cl + CL * j;
        if (c < N) {
          float b = Bm[k * ldb + c];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (i < nr) acc[i][j] = fmaf(A[(r0 + i) * lda + k], b, acc[i][j]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (i >= nr) break;
#pragma unroll
      for (int j = 0; j < DPL; ++j) {
        int c = cl + CL * j;
        if (c < N) emit(r0 + i, c, acc[i][j]);
      }
    }
  }
}

// out[r][c] = sum_k At[k*lda + r] * Bm[k*ldb + c]  (A given transposed: column
// blocks of At read as float4 broadcasts).  SUB as in rows_times_cols.
template <int DPL, class Emit, int SUB = 1>
__device__ __forceinline__ void cols_times_cols(const float *At, int lda, const float *Bm, int ldb, int R, int N,
                                                int K, Emit emit) {
  constexpr int CL = 32 / SUB;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int cl = lane % CL, sub = lane / CL;
  for (int rb = warp * 4 * SUB; rb < R; rb += nw * 4 * SUB) {
    const int r0 = rb + 4 * sub;
    float acc[4][DPL];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < DPL; ++j) acc[i][j] = 0.f;
    const int nr = max(0, min(4, R - r0));
    const bool live = nr > 0;  // the float4 column block lies in the padded row
    int k = 0;
    for (; k + 4 <= K; k += 4) {  // four k per iteration: all loads issued before the FMAs
      float4 a[4];
      float b[4][DPL];
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        a[kk] = live ? *reinterpret_cast<const float4 *>(At + (k + kk) * lda + r0) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
          int c = cl + CL * j;
          b[kk][j] = c < N ? Bm[(k + kk) * ldb + c] : 0.f;
        }
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
#pragma unroll
        for (int j = 0; j < DPL; ++j) {
          acc[0][j] = fmaf(a[kk].x, b[kk][j], acc[0][j]);
          acc[1][j] = fmaf(a[kk].y, b[kk][j], acc[1][j]);
          acc[2][j] = fmaf(a[kk].z, b[kk][j], acc[2][j]);
          acc[3][j] = fmaf(a[kk].w, b[kk][j], acc[3][j]);
        }
    }
    for (; k < K; ++k) {
      float4 a = live ? *reinterpret_cast<const float4 *>(At + k * lda + r0) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < DPL; ++j) {
        int c = cl + CL * j;
        if (c < N) {
          float b = Bm[k * ldb + c];
          acc[0][j] = fmaf(a.x, b, acc[0][j]);
          acc[1][j] = fmaf(a.y, b, acc[1][j]);
          acc[2][j] = fmaf(a.z, b, acc[2][j]);
          acc[3][j] = fmaf(a.w, b, acc[3][j]);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (i >= nr) break;
#pragma unroll
      for (int j = 0; j < DPL; ++j) {
        int c = cl + CL * j;
        if (c < N) emit(r0 + i, c, acc[i][j]);
      }
    }
  }
}

// out[r][c] for r < R, c < N (N a multiple of 4) = sum_k A(r, k) * Bm[k*ldb + c], with
// A(r, k) = At[k*lda + r] (A_T) or A[r*lda + k].  Each thread owns a tile of 4 rows x 4 columns and
// reads both operands as float4, four k at a time (64 FMAs per 8 shared loads).  When the tiles are
// fewer than half the block's threads, the k range is split across thread groups (slices of a
// multiple of 4) and the partial tiles are summed through `red` (blockDim.x * 16 floats of shared
// memory).  Block-wide: every thread of the block calls it; rows past R are computed from the
// last row and never emitted.  Requires lda and ldb multiples of 4 and 16-byte aligned operands.
template <bool A_T, class Emit>
__device__ __forceinline__ void tile_product(const float *A, int lda, const float *Bm, int ldb, int R, int N, int K,
                                             float *red, Emit emit) {
  const int cgs = N >> 2, rgs = (R + 3) >> 2, tiles = rgs * cgs;
  const int nt = blockDim.x;
  int ks = nt / tiles;
  if (ks > 8) ks = 8;
  if (ks < 2) ks = 1;
  const int kc = ks == 1 ? K : (((K + ks - 1) / ks + 3) & ~3);
  for (int t0 = 0; t0 < (ks == 1 ? tiles : 1); t0 += nt) {
    const int t = t0 + (int)threadIdx.x;
    const int tile = ks == 1 ? t : t % tiles, split = ks == 1 ? 0 : t / tiles;
    const bool live = ks == 1 ? t < tiles : split < ks;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
    const int rg = tile / cgs, cg = tile - rg * cgs;
    const int r0 = 4 * rg, c0 = 4 * cg;
    // rows of the tile: 4 consecutive (A_T: one float4 of At per k) or, for row-major A, every
    // rgs-th row, so that a warp's eight row groups read eight consecutive rows (conflict-free
    // when lda is not a multiple of 32 floats)
    auto row_of = [&](int i) { return A_T ? r0 + i : rg + i * rgs; };
    if (live) {
      const int kb = split * kc, ke = min(K, kb + kc);
      int rr[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) rr[i] = min(row_of(i), R - 1);
      int k = kb;
      for (; k + 4 <= ke; k += 4) {
        float a[4][4];  // a[kk][i] = A(r0 + i, k + kk)
        if (A_T) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const float4 v = *reinterpret_cast<const float4 *>(A + (k + kk) * lda + r0);
            a[kk][0] = v.x, a[kk][1] = v.y, a[kk][2] = v.z, a[kk][3] = v.w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 v = *reinterpret_cast<const float4 *>(A + rr[i] * lda + k);
            a[0][i] = v.x, a[1][i] = v.y, a[2][i] = v.z, a[3][i] = v.w;
          }
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const float4 b = *reinterpret_cast<const float4 *>(Bm + (k + kk) * ldb + c0);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            acc[i][0] = fmaf(a[kk][i], b.x, acc[i][0]);
            acc[i][1] = fmaf(a[kk][i], b.y, acc[i][1]);
            acc[i][2] = fmaf(a[kk][i], b.z, acc[i][2]);
            acc[i][3] = fmaf(a[kk][i], b.w, acc[i][3]);
          }
        }
      }
      for (; k < ke; ++k) {
        const float4 b = *reinterpret_cast<const float4 *>(Bm + k * ldb + c0);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float av = A_T ? A[k * lda + min(r0 + i, lda - 1)] : A[rr[i] * lda + k];
          acc[i][0] = fmaf(av, b.x, acc[i][0]);
          acc[i][1] = fmaf(av, b.y, acc[i][1]);
          acc[i][2] = fmaf(av, b.z, acc[i][2]);
          acc[i][3] = fmaf(av, b.w, acc[i][3]);
        }
      }
    }
    if (ks > 1) {
      // partial tile rows float4-major ([row i][split][tile]): consecutive threads, consecutive 16 bytes
      float4 *red4 = reinterpret_cast<float4 *>(red);
      const int slots = (ks - 1) * tiles;
      if (live && split > 0) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
          red4[(size_t)i * slots + (split - 1) * tiles + tile] = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
      }
      __syncthreads();
      if (live && split == 0)
        for (int sp = 1; sp < ks; ++sp) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float4 v = red4[(size_t)i * slots + (sp - 1) * tiles + tile];
            acc[i][0] += v.x, acc[i][1] += v.y, acc[i][2] += v.z, acc[i][3] += v.w;
          }
        }
      __syncthreads();  // `red` is free again for the next product
    }
    if (live && split == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = row_of(i);
        if (r >= R) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) emit(r, c0 + j, acc[i][j]);
      }
    }
  }
}

// ------------------------------------------------------------ score (smem)
// S[q,h,k] of MHAttentionScore (NeuroNet.cl:1662-1719) for one (sample, head).
// smem: Q [U][ldq] (ldq = pad4(D)), Kt [D][ldk] (ldk = pad4(U)).
template <int KPL>
__global__ void mh_score_smem_kernel(const float *__restrict__ qkv, float *__restrict__ score, int U, int H, int D,
                                     int mask, float koef) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float4 sm4[];
  float *sm = reinterpret_cast<float *>(sm4);
  const int ldq = pad4(D), ldk = pad4(U);
  float *Qs = sm;             // [U][ldq]
  float *Kt = sm + U * ldq;   // [D][ldk]
  const int h = blockIdx.x;
  const size_t b = blockIdx.y;
  const float *base = qkv + b * (size_t)U * 3 * H * D;
  const size_t rs = (size_t)3 * H * D;
  async_rows(Qs, ldq, base + (size_t)h * D, rs, U, D);
  // K transposed into smem: eight loads of a thread in flight before its stores
  for (int e0 = threadIdx.x; e0 < U * D; e0 += 8 * blockDim.x) {
    float kv[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = e0 + j * blockDim.x;
      kv[j] = e < U * D ? base[(size_t)(e / D) * rs + (size_t)(H + h) * D + e % D] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = e0 + j * blockDim.x;
      if (e < U * D) Kt[(e % D) * ldk + e / D] = nan0(kv[j]);
    }
  }
  for (int e = threadIdx.x; e < U * (ldq - D); e += blockDim.x) Qs[(e / (ldq - D)) * ldq + D + e % (ldq - D)] = 0.f;
  async_wait_all();
  __syncthreads();
  for (int e = threadIdx.x; e < U * D; e += blockDim.x) {  // IsNaNOrInf on the query operand
    float *q = Qs + (e / D) * ldq + e % D;
    *q = nan0(*q);
  }
  __syncthreads();
  float *sbase = score + b * (size_t)U * H * U + (size_t)h * U;  // row q at sbase + q*H*U
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int q0 = warp * 4; q0 < U; q0 += nw * 4) {
    const int nr = min(4, U - q0);
    float acc[4][KPL];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < KPL; ++j) acc[i][j] = 0.f;
    for (int d = 0; d < ldq; d += 4) {
      float4 a[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        a[i] = (i < nr) ? *reinterpret_cast<const float4 *>(Qs + (q0 + i) * ldq + d) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < KPL; ++j) {
        int k = lane + 32 * j;
        if (k < U) {
          float b0 = d + 0 < D ? Kt[(d + 0) * ldk + k] : 0.f, b1 = d + 1 < D ? Kt[(d + 1) * ldk + k] : 0.f;
          float b2 = d + 2 < D ? Kt[(d + 2) * ldk + k] : 0.f, b3 = d + 3 < D ? Kt[(d + 3) * ldk + k] : 0.f;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            acc[i][j] = fmaf(a[i].x, b0, acc[i][j]);
            acc[i][j] = fmaf(a[i].y, b1, acc[i][j]);
            acc[i][j] = fmaf(a[i].z, b2, acc[i][j]);
            acc[i][j] = fmaf(a[i].w, b3, acc[i][j]);
          }
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (i >= nr) break;
      const int q = q0 + i;
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < KPL; ++j) {
        int k = lane + 32 * j;
        float r = 0.f;
        if (k < U && !(mask > 0 && k > q)) {
          r = expf(clampf(acc[i][j] / koef, -100.f, 100.f));
          if (isnan(r)) r = 0.f;
          sum += r;
        }
        acc[i][j] = r;
      }
      sum = warp_sum(sum);
      float *row = sbase + (size_t)q * H * U;
#pragma unroll
      for (int j = 0; j < KPL; ++j) {
        int k = lane + 32 * j;
        if (k < U) row[k] = sum > 1.f ? acc[i][j] / sum : acc[i][j];
      }
    }
  }
}

// -------------------------------------------------------------- out (smem)
// O = S V for one (sample, head) (MHAttentionOut, NeuroNet.cl:1730-1759).
// Row stride of a shared [U][.] score matrix: U rounded up to 4 floats, plus 4 when that is a multiple
// of 32 floats (row-major float4 reads of consecutive rows then hit distinct banks).
__host__ __device__ __forceinline__ int score_lds(int U) {
  const int l = pad4(U);
  return (l % 32 == 0) ? l + 4 : l;
}

template <int DPL, int SUB>
__global__ void __launch_bounds__(256, 4) mh_out_smem_kernel(const float *__restrict__ scores, const float *__restrict__ qkv,
                                   float *__restrict__ out, int U, int H, int D) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float4 sm4[];
  float *sm = reinterpret_cast<float *>(sm4);
  const int lds = D % 4 == 0 ? score_lds(U) : pad4(U);
  float *Ss = sm;              // [U][lds]
  float *Vs = sm + U * lds;    // [U][D]
  const int h = blockIdx.x;
  const size_t b = blockIdx.y;
  const float *base = qkv + b * (size_t)U * 3 * H * D;
  async_rows(Ss, lds, scores + b * (size_t)U * H * U + (size_t)h * U, (size_t)H * U, U, U);
  async_rows(Vs, D, base + (size_t)(2 * H + h) * D, (size_t)3 * H * D, U, D);
  async_wait_all();
  __syncthreads();
  float *ob = out + b * (size_t)U * H * D + (size_t)h * D;
  auto emit = [&](int u, int d, float acc) { ob[(size_t)u * H * D + d] = acc; };
  if (D % 4 == 0)  // 4 x 4 register tiles; `red` (blockDim.x * 16 floats) follows V
    tile_product<false>(Ss, lds, Vs, D, U, D, U, Vs + U * D, emit);
  else
    rows_times_cols<DPL, decltype(emit), SUB>(Ss, lds, Vs, D, U, D, U, emit);
}

// ------------------------------------------------- inside gradients (smem)
// MHAttentionInsideGradients (NeuroNet.cl:1777-1845) for one (sample, head), in
// the reassociated form dV = S^T g, A = S V0, C = S o (V0^T - A),
// dQ = g o (C K) / koef, dK = C^T (g o Q) / koef.
template <int DPL, int SUB>
__global__ void mh_grad_smem_kernel(const float *__restrict__ qkv, float *__restrict__ qkv_g,
                                    const float *__restrict__ scores, const float *__restrict__ grad, int U, int H,
                                    int D, float koef) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float4 sm4[];
  float *sm = reinterpret_cast<float *>(sm4);
  const int lds = D % 4 == 0 ? score_lds(U) : pad4(U);
  float *Cs = sm;                 // [U][lds]  S, then C
  float *Ks = Cs + U * lds;       // [U][D]
  float *Gs = Ks + U * D;         // [U][D]
  float *GQ = Gs + U * D;         // [U][D]   Q, then g o Q
  float *V0 = GQ + U * D;         // [lds]
  float *red = V0 + 2 * lds;      // [blockDim.x * 16] partial tiles of the tile products (D % 4 == 0)
  const bool tiled = D % 4 == 0;
  const int h = blockIdx.x;
  const size_t b = blockIdx.y;
  const size_t rs = (size_t)3 * H * D;
  const float *base = qkv + b * (size_t)U * rs;
  async_rows(Cs, lds, scores + b * (size_t)U * H * U + (size_t)h * U, (size_t)H * U, U, U);
  async_rows(Ks, D, base + (size_t)(H + h) * D, rs, U, D);
  async_rows(GQ, D, base + (size_t)h * D, rs, U, D);
  async_rows(Gs, D, grad + b * (size_t)U * H * D + (size_t)h * D, (size_t)H * D, U, D);
  for (int u = threadIdx.x; u < lds; u += blockDim.x) V0[u] = u < U ? base[(size_t)u * rs + (size_t)(2 * H + h) * D] : 0.f;
  if (lds > U)  // zero the padding columns of S (read by the float4 column loads)
    for (int q = threadIdx.x; q < U; q += blockDim.x)
      for (int c = U; c < lds; ++c) Cs[q * lds + c] = 0.f;
  async_wait_all();
  __syncthreads();
  float *gb = qkv_g + b * (size_t)U * rs;
  // dV[u][d] = sum_i S[i][u] g[i][d]
  auto emit_v = [&](int u, int d, float acc) { gb[(size_t)u * rs + (size_t)(2 * H + h) * D + d] = acc; };
  if (tiled)
    tile_product<true>(Cs, lds, Gs, D, U, D, U, red, emit_v);
  else
    cols_times_cols<DPL, decltype(emit_v), SUB>(Cs, lds, Gs, D, U, D, U, emit_v);
  for (int e = threadIdx.x; e < U * D; e += blockDim.x) GQ[e] *= Gs[e];  // g o Q
  __syncthreads();  // every dV read of S is done before S becomes C
  // per query row (one warp): A[q] = sum_v S[q][v] V0[v], then C[q][u] = S[q][u] (V0[u] - A[q])
  {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int q = warp; q < U; q += nw) {
      float *row = Cs + q * lds;
      float a = 0.f;
      for (int v = lane; v < U; v += 32) a += row[v] * V0[v];
      a = warp_sum(a);
      for (int u = lane; u < U; u += 32) row[u] *= (V0[u] - a);
    }
  }
  __syncthreads();
  const float inv = 1.f / koef;
  // dK[u][d] = sum_q C[q][u] (g o Q)[q][d] / koef
  auto emit_k = [&](int u, int d, float acc) { gb[(size_t)u * rs + (size_t)(H + h) * D + d] = acc * inv; };
  // dQ[u][d] = g[u][d] / koef * sum_k C[u][k] K[k][d]
  auto emit_q = [&](int u, int d, float acc) { gb[(size_t)u * rs + (size_t)h * D + d] = Gs[u * D + d] * acc * inv; };
  if (tiled) {
    tile_product<true>(Cs, lds, GQ, D, U, D, U, red, emit_k);
    tile_product<false>(Cs, lds, Ks, D, U, D, U, red, emit_q);
  } else {
    cols_times_cols<DPL, decltype(emit_k), SUB>(Cs, lds, GQ, D, U, D, U, emit_k);
    rows_times_cols<DPL, decltype(emit_q), SUB>(Cs, lds, Ks, D, U, D, U, emit_q);
  }
}

}  // namespace nn
