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

// ------------------------------------------------------------ score (smem)
// S[q,h,k] of MHAttentionScore (NeuroNet.cl:1662-1719) for one (sample, head).
// smem: Q [U][ldq] (ldq = pad4(D)), Kt [D][ldk] (ldk = pad4(U)).
template <int KPL>
__global__ void mh_score_smem_kernel(const float *__restrict__ qkv, float *__restrict__ score, int U, int H, int D,
                                     int mask, float koef) {
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
template <int DPL, int SUB>
__global__ void mh_out_smem_kernel(const float *__restrict__ scores, const float *__restrict__ qkv,
                                   float *__restrict__ out, int U, int H, int D) {
  extern __shared__ float4 sm4[];
  float *sm = reinterpret_cast<float *>(sm4);
  const int lds = pad4(U);
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
  extern __shared__ float4 sm4[];
  float *sm = reinterpret_cast<float *>(sm4);
  const int lds = pad4(U);
  float *Cs = sm;                 // [U][lds]  S, then C
  float *Ks = Cs + U * lds;       // [U][D]
  float *Gs = Ks + U * D;         // [U][D]
  float *GQ = Gs + U * D;         // [U][D]   Q, then g o Q
  float *V0 = GQ + U * D;         // [lds]
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
  cols_times_cols<DPL, decltype(emit_k), SUB>(Cs, lds, GQ, D, U, D, U, emit_k);
  // dQ[u][d] = g[u][d] / koef * sum_k C[u][k] K[k][d]
  auto emit_q = [&](int u, int d, float acc) { gb[(size_t)u * rs + (size_t)h * D + d] = Gs[u * D + d] * acc * inv; };
  rows_times_cols<DPL, decltype(emit_q), SUB>(Cs, lds, Ks, D, U, D, U, emit_q);
}

}  // namespace nn
