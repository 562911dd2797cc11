// Attention-layer kernels (CNeuronMLMHAttentionOCL path) and the row-wise
// kernels around them: MHAttentionScore, MHAttentionOut,
// MHAttentionInsideGradients, SumMatrix, Normalize, SoftMax_FeedForward,
// SoftMax_HiddenGradient, SoftMax_OutputGradient, Transpose,
// ConcatenateBuffers, DeconcatenateBuffers.
//
// qkv layout is the reference's [unit][3][head][dimension]
// (NeuroNet.cl:1674, 1693, 1754); scores are [query][head][key].
#include <algorithm>

#include "../../include/nn_b200.h"
#include "attn_smem.cuh"
#include "tc_attn.cuh"
#include "nn_device.cuh"
#include "nn_internal.h"

namespace nn {

constexpr size_t kSmemCap = 200 * 1024;  // dynamic shared memory one CTA may use

// ------------------------------------------------------- MHAttentionScore
// NeuroNet.cl:1662-1719: S[q,h,k] = exp(clamp(q.k / sqrt(d), +-100)) (NaN -> 0),
// masked keys (k > q when mask) are 0 and excluded from the row sum, and the
// row is divided by its sum only when that sum exceeds 1.
// One warp per query row, keys of a tile of KT staged in shared memory.
constexpr int kScoreKT = 128;

__global__ void mh_score_kernel(const float *__restrict__ qkv, float *__restrict__ score, int units, int heads,
                                int dim, int mask, float koef) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float sm[];
  const int dp = dim + 1;
  float *Ks = sm;                    // [kScoreKT][dim+1]
  float *Qs = sm + kScoreKT * dp;    // [warps][dim]
  const int h = blockIdx.y;
  const size_t b = blockIdx.z;
  const int warps = blockDim.x >> 5;
  const int wv = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = blockIdx.x * warps + wv;
  const float *base = qkv + b * (size_t)units * 3 * heads * dim;
  float *srow = score + (b * units + (size_t)min(q, units - 1)) * heads * units + (size_t)h * units;
  if (q < units)
    for (int d = lane; d < dim; d += 32) Qs[wv * dim + d] = nan0(base[((size_t)q * 3 * heads + h) * dim + d]);
  float rowsum = 0.f;
  for (int k0 = 0; k0 < units; k0 += kScoreKT) {
    int kt = min(kScoreKT, units - k0);
    __syncthreads();
    for (int e = threadIdx.x; e < kt * dim; e += blockDim.x) {
      int kk = e / dim, d = e - kk * dim;
      Ks[kk * dp + d] = nan0(base[((size_t)(k0 + kk) * 3 * heads + heads + h) * dim + d]);
    }
    __syncthreads();
    if (q < units) {
      for (int kk = lane; kk < kt; kk += 32) {
        int k = k0 + kk;
        float r;
        if (mask > 0 && k > q) {
          r = 0.f;
        } else {
          float s = 0.f;
          const float *kr = Ks + kk * dp;
          const float *qr = Qs + wv * dim;
          for (int d = 0; d < dim; ++d) s = fmaf(qr[d], kr[d], s);
          r = expf(clampf(s / koef, -100.f, 100.f));
          if (isnan(r)) r = 0.f;
          rowsum += r;
        }
        srow[k] = r;
      }
    }
  }
  if (q >= units) return;
  rowsum = warp_sum(rowsum);
  if (rowsum > 1.f) {
    __syncwarp();
    for (int k = lane; k < units; k += 32) srow[k] /= rowsum;
  }
}

static int k_mh_attention_score(Launch &L) {
  const int units = (int)L.nd.g[0], heads = L.nd.dims > 1 ? (int)L.nd.g[1] : 1;
  const int dim = L.i(2), mask = L.i(3);
  if (dim <= 0 || dim > 1024) return L.fail(NN_ERR_ARG, "MHAttentionScore: dimension outside [1, 1024]");
  float *qkv = L.buf(0, (size_t)L.B * units * 3 * heads * dim);
  float *score = L.buf(1, (size_t)L.B * units * heads * units);
  if (!qkv || !score) return NN_ERR_BOUNDS;
  float koef = sqrtf((float)dim);
  if (koef < 1.f) koef = 1.f;
  if (attn_tc_ok(qkv, score, units, heads, dim)) {
    cudaError_t e = attn_tc<tc::kAttnScore>(qkv, score, score, L.B, units, heads, mask, koef, L.stream);
    if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
    L.counted();
    return NN_OK;
  }
  {
    size_t sm = (size_t)(units * pad4(dim) + dim * pad4(units)) * sizeof(float);
    int kpl = (units + 31) / 32;
    if (sm <= kSmemCap && kpl <= 4) {
      auto fn = kpl <= 1 ? mh_score_smem_kernel<1> : kpl == 2 ? mh_score_smem_kernel<2>
              : kpl == 3 ? mh_score_smem_kernel<3> : mh_score_smem_kernel<4>;
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
      NN_LAUNCH_PDL(L, fn, dim3(heads, L.B), 256, sm, L.stream, qkv, score, units, heads, dim, mask, koef);
      return NN_OK;
    }
  }
  const int warps = 8;
  size_t smem = (size_t)(kScoreKT * (dim + 1) + warps * dim) * sizeof(float);
  if (smem > 200 * 1024) return L.fail(NN_ERR_UNSUPPORTED, "MHAttentionScore: key dimension too large");
  if (smem > 48 * 1024) cudaFuncSetAttribute(mh_score_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(ceil_div(units, warps), heads, L.B);
  NN_LAUNCH_PDL(L, mh_score_kernel, grid, warps * 32, smem, L.stream, qkv, score, units, heads, dim, mask, koef);
  return NN_OK;
}

// --------------------------------------------------------- MHAttentionOut
// NeuroNet.cl:1730-1759: O[u,h,:] = sum_v S[u,h,v] V[v,h,:] (no sanitising).
constexpr int kOutVT = 64;
__global__ void mh_out_kernel(const float *__restrict__ scores, const float *__restrict__ qkv, float *__restrict__ out,
                              int units, int heads, int dim) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ float sm[];
  float *Vs = sm;                         // [kOutVT][dim]
  float *Ss = sm + kOutVT * dim;          // [warps][kOutVT]
  const int h = blockIdx.y;
  const size_t b = blockIdx.z;
  const int warps = blockDim.x >> 5;
  const int wv = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u = blockIdx.x * warps + wv;
  const float *base = qkv + b * (size_t)units * 3 * heads * dim;
  const float *srow = scores + (b * units + (size_t)min(u, units - 1)) * heads * units + (size_t)h * units;
  constexpr int MAXD = 8;  // dim up to 256 in registers (dim / 32 per lane)
  float acc[MAXD];
#pragma unroll
  for (int j = 0; j < MAXD; ++j) acc[j] = 0.f;
  for (int v0 = 0; v0 < units; v0 += kOutVT) {
    int vt = min(kOutVT, units - v0);
    __syncthreads();
    for (int e = threadIdx.x; e < vt * dim; e += blockDim.x) {
      int vv = e / dim, d = e - vv * dim;
      Vs[vv * dim + d] = base[((size_t)(v0 + vv) * 3 * heads + 2 * heads + h) * dim + d];
    }
    if (u < units)
      for (int vv = lane; vv < vt; vv += 32) Ss[wv * kOutVT + vv] = srow[v0 + vv];
    __syncthreads();
    if (u < units) {
      for (int vv = 0; vv < vt; ++vv) {
        float s = Ss[wv * kOutVT + vv];
#pragma unroll
        for (int j = 0; j < MAXD; ++j) {
          int d = lane + 32 * j;
          if (d < dim) acc[j] = fmaf(s, Vs[vv * dim + d], acc[j]);
        }
      }
    }
  }
  if (u >= units) return;
  float *orow = out + ((b * units + u) * heads + h) * (size_t)dim;
#pragma unroll
  for (int j = 0; j < MAXD; ++j) {
    int d = lane + 32 * j;
    if (d < dim) orow[d] = acc[j];
  }
}

static int k_mh_attention_out(Launch &L) {
  const int units = (int)L.nd.g[0], heads = L.nd.dims > 1 ? (int)L.nd.g[1] : 1;
  const int dim = L.i(3);
  if (dim <= 0 || dim > 256) return L.fail(NN_ERR_UNSUPPORTED, "MHAttentionOut: dimension outside [1, 256]");
  float *scores = L.buf(0, (size_t)L.B * units * heads * units);
  float *qkv = L.buf(1, (size_t)L.B * units * 3 * heads * dim);
  float *out = L.buf(2, (size_t)L.B * units * heads * dim);
  if (!scores || !qkv || !out) return NN_ERR_BOUNDS;
  if (attn_tc_ok(qkv, scores, units, heads, dim) && ((uintptr_t)out & 15) == 0) {
    cudaError_t e = attn_tc<tc::kAttnOut>(qkv, scores, out, L.B, units, heads, 0, 1.f, L.stream);
    if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
    L.counted();
    return NN_OK;
  }
  {
    // head dimensions that are multiples of 4 take the tiled product, with 16 floats per thread
    // of partial tiles after V
    const int lds = dim % 4 == 0 ? score_lds(units) : pad4(units);
    size_t sm = (size_t)(units * lds + units * dim + (dim % 4 == 0 ? 256 * 16 : 0)) * sizeof(float);
    int dpl = (dim + 31) / 32;
    if (sm <= kSmemCap && dpl <= 2) {
      // head dimensions up to 16: half-warps take separate row blocks (no idle lanes)
      auto fn = dim <= 16 ? mh_out_smem_kernel<1, 2> : dpl <= 1 ? mh_out_smem_kernel<1, 1> : mh_out_smem_kernel<2, 1>;
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
      NN_LAUNCH_PDL(L, fn, dim3(heads, L.B), 256, sm, L.stream, scores, qkv, out, units, heads, dim);
      return NN_OK;
    }
  }
  const int warps = 8;
  size_t smem = (size_t)(kOutVT * dim + warps * kOutVT) * sizeof(float);
  if (smem > 48 * 1024) cudaFuncSetAttribute(mh_out_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(ceil_div(units, warps), heads, L.B);
  NN_LAUNCH_PDL(L, mh_out_kernel, grid, warps * 32, smem, L.stream, scores, qkv, out, units, heads, dim);
  return NN_OK;
}

// --------------------------------------------- MHAttentionInsideGradients
// NeuroNet.cl:1777-1845.  With V0[k] = V[k,h,0] (the reference reads V without
// the +d offset, NeuroNet.cl:1822/1840) and A[q] = sum_v S[q,v] V0[v], the
// reference's triple loops are, exactly reassociated:
//   dV[u,d] = sum_i S[i,u] g[i,d]
//   dQ[u,d] = g[u,d]/koef * sum_k S[u,k] (V0[k]-A[u]) K[k,d]
//   dK[u,d] = 1/koef * sum_q S[q,u] (V0[u]-A[q]) g[q,d] Q[q,d]
__global__ void mh_grad_rowsum_kernel(const float *__restrict__ qkv, const float *__restrict__ scores,
                                      float *__restrict__ A, int units, int heads, int dim, int B) {
  pdl_wait();
  pdl_trigger();
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  int rows = B * units * heads;  // (b, q, h)
  if (warp >= rows) return;
  int h = warp % heads;
  int bq = warp / heads;
  int b = bq / units;
  const float *srow = scores + (size_t)warp * units;
  const float *base = qkv + (size_t)b * units * 3 * heads * dim;
  float s = 0.f;
  for (int v = lane; v < units; v += 32) s += srow[v] * base[((size_t)v * 3 * heads + 2 * heads + h) * dim];
  s = warp_sum(s);
  if (lane == 0) A[warp] = s;
}

__global__ void mh_grad_kernel(const float *__restrict__ qkv, float *__restrict__ qkv_g,
                               const float *__restrict__ scores, const float *__restrict__ grad,
                               const float *__restrict__ A, int units, int heads, int dim, float koef, int B) {
  pdl_wait();
  pdl_trigger();
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t total = (size_t)B * units * heads * dim;
  if (t >= total) return;
  int d = (int)(t % dim);
  size_t r = t / dim;
  int h = (int)(r % heads);
  r /= heads;
  int u = (int)(r % units);
  size_t b = r / units;
  const float *base = qkv + b * (size_t)units * 3 * heads * dim;
  const float *S = scores + b * (size_t)units * heads * units;  // [q][h][k]
  const float *G = grad + b * (size_t)units * heads * dim;      // [u][h][d]
  const float *Ab = A + b * (size_t)units * heads;              // [q][h]
  const size_t qstride = (size_t)3 * heads * dim;
  float v0u = base[u * qstride + (2 * heads + h) * (size_t)dim];
  float au = Ab[(size_t)u * heads + h];
  float dv = 0.f, dq = 0.f, dk = 0.f;
  for (int i = 0; i < units; ++i) {
    float s_iu = S[((size_t)i * heads + h) * units + u];
    float g_id = G[((size_t)i * heads + h) * dim + d];
    dv = fmaf(s_iu, g_id, dv);
    float q_id = base[i * qstride + (size_t)h * dim + d];
    dk = fmaf(s_iu * (v0u - Ab[(size_t)i * heads + h]), g_id * q_id, dk);
    float s_ui = S[((size_t)u * heads + h) * units + i];
    float v0i = base[i * qstride + (2 * heads + h) * (size_t)dim];
    float k_id = base[i * qstride + (heads + h) * (size_t)dim + d];
    dq = fmaf(s_ui * (v0i - au), k_id, dq);
  }
  float g_ud = G[((size_t)u * heads + h) * dim + d];
  float *og = qkv_g + b * (size_t)units * 3 * heads * dim + u * qstride;
  og[(size_t)h * dim + d] = g_ud * dq / koef;
  og[(size_t)(heads + h) * dim + d] = dk / koef;
  og[(size_t)(2 * heads + h) * dim + d] = dv;
}

static int k_mh_attention_inside_gradients(Launch &L) {
  const int units = (int)L.nd.g[0];
  const int heads = L.nd.dims > 1 ? (int)L.nd.g[1] : 1;
  const int dim = L.nd.dims > 2 ? (int)L.nd.g[2] : 1;
  size_t nqkv = (size_t)L.B * units * 3 * heads * dim;
  float *qkv = L.buf(0, nqkv), *qkv_g = L.buf(1, nqkv);
  float *scores = L.buf(2, (size_t)L.B * units * heads * units);
  float *grad = L.buf(3, (size_t)L.B * units * heads * dim);
  if (!qkv || !qkv_g || !scores || !grad) return NN_ERR_BOUNDS;
  float koef = sqrtf((float)dim);
  if (koef < 1.f) koef = 1.f;
  if (attn_tc_ok(qkv, scores, units, heads, dim) && ((uintptr_t)grad & 15) == 0 && ((uintptr_t)qkv_g & 31) == 0) {
    cudaError_t e = attn_grad_tc(qkv, qkv_g, scores, grad, L.B, units, heads, koef, L.stream);
    if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
    L.counted();
    return NN_OK;
  }
  {
    const int lds = dim % 4 == 0 ? score_lds(units) : pad4(units);
    size_t sm = (size_t)(units * lds + 3 * units * dim + 2 * lds + (dim % 4 == 0 ? 256 * 16 : 0)) * sizeof(float);
    int dpl = (dim + 31) / 32;
    if (sm <= kSmemCap && dpl <= 2) {
      auto fn = dim <= 16 ? mh_grad_smem_kernel<1, 2>
                          : dpl <= 1 ? mh_grad_smem_kernel<1, 1> : mh_grad_smem_kernel<2, 1>;
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
      NN_LAUNCH_PDL(L, fn, dim3(heads, L.B), 256, sm, L.stream, qkv, qkv_g, scores, grad, units, heads, dim, koef);
      return NN_OK;
    }
  }
  size_t rows = (size_t)L.B * units * heads;
  float *A = L.scratch(2, rows);
  if (!A) return NN_ERR_CUDA;
  NN_LAUNCH_PDL(L, mh_grad_rowsum_kernel, ceil_div(rows * 32, 256), 256, 0, L.stream, qkv, scores, A, units, heads, dim, L.B);
  size_t total = rows * dim;
  NN_LAUNCH_PDL(L, mh_grad_kernel, grid1d(total, 256), 256, 0, L.stream, qkv, qkv_g, scores, grad, A, units, heads, dim, koef, L.B);
  return NN_OK;
}

// -------------------------------------------------------------- SumMatrix
// NeuroNet.cl:1314-1347: out[i*so + i*dim + k] = nan0((a[i*s1 + i*dim + k] + b[i*s2 + i*dim + k]) * mult)
__global__ void sum_matrix_kernel(const float *a, const float *bm, float *out, float *flags, int rows, int dim,
                                  float mult, int s1, int s2, int so, int fe) {
  pdl_wait();
  pdl_trigger();
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)rows * dim) return;
  size_t i = t / dim;
  size_t index = t;
  float v1 = a[i * s1 + index], v2 = bm[i * s2 + index];
  float raw = (v1 + v2) * mult;
  if (fe) flags[index] = (!isfinite(v1) || !isfinite(v2) || !isfinite(v1 + v2) || !isfinite(raw)) ? 1.f : 0.f;
  out[i * so + index] = nan0(raw);
}

// Same with zero row shifts (the encoder's residual sums): a flat float4 stream.
__global__ void sum_matrix_flat4_kernel(const float4 *a, const float4 *bm, float4 *out, float4 *flags, size_t n4,
                                        float mult) {
  pdl_wait();
  pdl_trigger();
  for (size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x; t < n4; t += (size_t)gridDim.x * blockDim.x) {
    const float4 x = a[t], y = bm[t];
    const float r[4] = {(x.x + y.x) * mult, (x.y + y.y) * mult, (x.z + y.z) * mult, (x.w + y.w) * mult};
    if (flags) {
      const float xs[4] = {x.x, x.y, x.z, x.w}, ys[4] = {y.x, y.y, y.z, y.w};
      float f[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        f[e] = (!isfinite(xs[e]) || !isfinite(ys[e]) || !isfinite(xs[e] + ys[e]) || !isfinite(r[e])) ? 1.f : 0.f;
      flags[t] = make_float4(f[0], f[1], f[2], f[3]);
    }
    out[t] = make_float4(nan0(r[0]), nan0(r[1]), nan0(r[2]), nan0(r[3]));
  }
}

static int k_sum_matrix(Launch &L) {
  const int rows = (int)L.nd.g[0] * L.B;
  const int dim = L.i(3), s1 = L.i(5), s2 = L.i(6), so = L.i(7), fe = L.i(9);
  if (dim < 0 || s1 < 0 || s2 < 0 || so < 0) return L.fail(NN_ERR_ARG, "SumMatrix: bad shape");
  if (rows == 0 || dim == 0) return NN_OK;
  auto need = [&](int s) { return (size_t)(rows - 1) * (s + dim) + dim; };
  float *a = L.buf(0, need(s1)), *b = L.buf(1, need(s2)), *o = L.buf(2, need(so));
  if (!a || !b || !o) return NN_ERR_BOUNDS;
  float *flags = nullptr;
  if (fe) {
    flags = L.buf(8, (size_t)rows * dim);
    if (!flags) return NN_ERR_BOUNDS;
  }
  size_t n = (size_t)rows * dim;
  auto al16 = [](const void *p) { return ((uintptr_t)p & 15) == 0; };
  if (s1 == 0 && s2 == 0 && so == 0 && n % 4 == 0 && al16(a) && al16(b) && al16(o) && (!flags || al16(flags))) {
    const size_t n4 = n / 4;
    const unsigned blocks = (unsigned)std::min<size_t>((n4 + 255) / 256, 148 * 16);
    NN_LAUNCH_PDL(L, sum_matrix_flat4_kernel, blocks, 256, 0, L.stream, reinterpret_cast<const float4 *>(a), reinterpret_cast<const float4 *>(b), reinterpret_cast<float4 *>(o), reinterpret_cast<float4 *>(flags), n4, L.f(4));
    return NN_OK;
  }
  NN_LAUNCH_PDL(L, sum_matrix_kernel, grid1d(n, 256), 256, 0, L.stream, a, b, o, flags, rows, dim, L.f(4), s1, s2, so, fe);
  return NN_OK;
}

// -------------------------------------------------------------- Normalize
// NeuroNet.cl:1455-1486: per row, centre on the mean and divide by the
// unbiased *variance* (not its root) only when it exceeds 1.  One warp per row.
__global__ void normalize_rows_kernel(float *buf, int rows, int dim) {
  pdl_wait();
  pdl_trigger();
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  float *row = buf + (size_t)warp * dim;
  float s = 0.f;
  for (int i = lane; i < dim; i += 32) s += nan0(row[i]);
  float mean = warp_sum(s) / (float)dim;
  float m2 = 0.f;
  for (int i = lane; i < dim; i += 32) {
    float c = nan0(row[i]) - mean;
    m2 += c * c;
  }
  float variance = warp_sum(m2) / (float)(dim - 1);
  __syncwarp();
  bool scale = variance > 1.f;
  for (int i = lane; i < dim; i += 32) {
    float c = row[i] - mean;
    row[i] = nan0(scale ? c / variance : c);
  }
}

// Same for rows of at most 32*EPL floats: the row is read once into registers.
template <int EPL>
__global__ void normalize_rows_reg_kernel(float *buf, int rows, int dim) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  float *row = buf + (size_t)warp * dim;
  float x[EPL];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int i = lane + 32 * j;
    x[j] = i < dim ? row[i] : 0.f;
    s += i < dim ? nan0(x[j]) : 0.f;
  }
  const float mean = warp_sum(s) / (float)dim;
  float m2 = 0.f;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int i = lane + 32 * j;
    const float c = nan0(x[j]) - mean;
    m2 += i < dim ? c * c : 0.f;
  }
  const float variance = warp_sum(m2) / (float)(dim - 1);
  const bool scale = variance > 1.f;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int i = lane + 32 * j;
    const float c = x[j] - mean;
    if (i < dim) row[i] = nan0(scale ? c / variance : c);
  }
}

static int k_normalize(Launch &L) {
  const int rows = (int)L.nd.g[0] * L.B, dim = L.i(1);
  if (dim < 1) return NN_OK;  // the reference returns without touching the buffer
  float *b = L.buf(0, (size_t)rows * dim);
  if (!b) return NN_ERR_BOUNDS;
  const unsigned blocks = ceil_div((size_t)rows * 32, 256);
  if (dim <= 64)
    NN_LAUNCH_PDL(L, normalize_rows_reg_kernel<2>, blocks, 256, 0, L.stream, b, rows, dim);
  else if (dim <= 128)
    NN_LAUNCH_PDL(L, normalize_rows_reg_kernel<4>, blocks, 256, 0, L.stream, b, rows, dim);
  else
    NN_LAUNCH_PDL(L, normalize_rows_kernel, blocks, 256, 0, L.stream, b, rows, dim);
  return NN_OK;
}

// SumMatrix (zero row shifts, no numeric flags) immediately followed by Normalize of its output
// (CNeuronBaseOCL::SumAndNormalize, NeuroNet_Core.mqh:17976-18075): one pass instead of two.  Each
// warp takes one row, forms out = IsNaNOrInf((a + b) * mult) as SumMatrix does, then normalises the
// row in registers exactly as normalize_rows_reg_kernel does, and writes it once.
template <int EPL>
__global__ void sum_normalize_rows_kernel(const float *__restrict__ a, const float *__restrict__ bm,
                                          float *__restrict__ out, int rows, int dim, float mult) {
  pdl_wait();
  pdl_trigger();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const size_t base = (size_t)warp * dim;
  float x[EPL];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int i = lane + 32 * j;
    x[j] = i < dim ? nan0((a[base + i] + bm[base + i]) * mult) : 0.f;
    s += x[j];
  }
  const float mean = warp_sum(s) / (float)dim;
  float m2 = 0.f;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int i = lane + 32 * j;
    const float c = x[j] - mean;
    m2 += i < dim ? c * c : 0.f;
  }
  const float variance = warp_sum(m2) / (float)(dim - 1);
  const bool scale = variance > 1.f;
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int i = lane + 32 * j;
    const float c = x[j] - mean;
    if (i < dim) out[base + i] = nan0(scale ? c / variance : c);
  }
}

// Whether a recorded SumMatrix and the Normalize after it can run as sum_normalize_rows_kernel: the
// Normalize normalises exactly the rows the SumMatrix wrote (same buffer, row length and row count),
// with no row shifts, no flags and rows of at most 128 floats.
bool sum_normalize_fusable(const KernelInst &sm, const NDR &nsm, const KernelInst &nm, const NDR &nnm) {
  if (sm.args[5].i != 0 || sm.args[6].i != 0 || sm.args[7].i != 0 || sm.args[9].i != 0) return false;
  if (nm.args[0].i != sm.args[2].i || nm.args[1].i != sm.args[3].i) return false;
  if (nm.batch != sm.batch || nnm.g[0] != nsm.g[0]) return false;
  const int dim = sm.args[3].i;
  return dim >= 2 && dim <= 128;
}

// The fused pair, launched for the SumMatrix execution `L` (its Normalize is skipped).
int sum_normalize_launch(Launch &L) {
  const int rows = (int)L.nd.g[0] * L.B, dim = L.i(3);
  if (rows == 0) return NN_OK;
  const size_t n = (size_t)rows * dim;
  float *a = L.buf(0, n), *b = L.buf(1, n), *o = L.buf(2, n);
  if (!a || !b || !o) return NN_ERR_BOUNDS;
  const unsigned blocks = ceil_div((size_t)rows * 32, 256);
  if (dim <= 64)
    NN_LAUNCH_PDL(L, sum_normalize_rows_kernel<2>, blocks, 256, 0, L.stream, a, b, o, rows, dim, L.f(4));
  else
    NN_LAUNCH_PDL(L, sum_normalize_rows_kernel<4>, blocks, 256, 0, L.stream, a, b, o, rows, dim, L.f(4));
  return NN_OK;
}

// ---------------------------------------------------------------- SoftMax
// NeuroNet.cl:2479-2520 (LocalSoftMax / LocalSoftMaxGrad, NeuroNet.cl:392-420).
// Row length is the local size of dimension 0; one warp per (sample, head) row.
__global__ void softmax_fwd_kernel(const float *in, float *out, int rows, int size) {
  pdl_wait();
  pdl_trigger();
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float *x = in + (size_t)warp * size;
  float *y = out + (size_t)warp * size;
  float mx = kMinValue;
  for (int i = lane; i < size; i += 32) mx = fmaxf(mx, nan0(x[i], kMinValue));
  mx = warp_max(mx);
  if (mx == kMinValue) {
    for (int i = lane; i < size; i += 32) y[i] = 0.f;
    return;
  }
  float s = 0.f;
  for (int i = lane; i < size; i += 32) {
    float v = nan0(x[i], kMinValue);
    s += (v == kMinValue) ? 0.f : nan0(expf(v - mx));
  }
  s = nan0(warp_sum(s));
  __syncwarp();
  for (int i = lane; i < size; i += 32) {
    float v = nan0(x[i], kMinValue);
    float e = (v == kMinValue) ? 0.f : nan0(expf(v - mx));
    y[i] = (s == 0.f) ? 0.f : nan0(e / s);
  }
}

__global__ void softmax_bwd_kernel(const float *outp, const float *og, float *ig, int rows, int size) {
  pdl_wait();
  pdl_trigger();
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float *y = outp + (size_t)warp * size;
  const float *g = og + (size_t)warp * size;
  float s = 0.f;
  for (int i = lane; i < size; i += 32) s += nan0(nan0(y[i]) * nan0(g[i]));
  s = nan0(warp_sum(s));
  __syncwarp();
  for (int i = lane; i < size; i += 32) {
    float yy = nan0(y[i]), gg = nan0(g[i]);
    ig[(size_t)warp * size + i] = nan0(yy * (gg - s));
  }
}

static int softmax_shape(Launch &L, int *size, int *rows) {
  int sz = L.nd.has_local ? (int)L.nd.l[0] : (int)L.nd.g[0];
  if ((int)L.nd.g[0] != sz) return L.fail(NN_ERR_UNSUPPORTED, "SoftMax: global size 0 must equal local size 0");
  *size = sz;
  *rows = (L.nd.dims > 1 ? (int)L.nd.g[1] : 1) * L.B;
  return NN_OK;
}

static int k_softmax_ff(Launch &L) {
  int size, rows;
  int rc = softmax_shape(L, &size, &rows);
  if (rc) return rc;
  float *in = L.buf(0, (size_t)size * rows), *out = L.buf(1, (size_t)size * rows);
  if (!in || !out) return NN_ERR_BOUNDS;
  NN_LAUNCH_PDL(L, softmax_fwd_kernel, ceil_div((size_t)rows * 32, 256), 256, 0, L.stream, in, out, rows, size);
  return NN_OK;
}

static int k_softmax_hg(Launch &L) {
  int size, rows;
  int rc = softmax_shape(L, &size, &rows);
  if (rc) return rc;
  size_t n = (size_t)size * rows;
  float *y = L.buf(0, n), *og = L.buf(1, n), *ig = L.buf(2, n);
  if (!y || !og || !ig) return NN_ERR_BOUNDS;
  NN_LAUNCH_PDL(L, softmax_bwd_kernel, ceil_div((size_t)rows * 32, 256), 256, 0, L.stream, y, og, ig, rows, size);
  return NN_OK;
}

__global__ void softmax_og_kernel(const float *y, const float *t, float *g, size_t n) {
  pdl_wait();
  pdl_trigger();
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) g[i] = (y[i] == 0.f) ? 0.f : t[i] / y[i];
}
static int k_softmax_og(Launch &L) {
  size_t n = (size_t)L.nd.g[0] * L.B;
  float *y = L.buf(0, n), *t = L.buf(1, n), *g = L.buf(2, n);
  if (!y || !t || !g) return NN_ERR_BOUNDS;
  NN_LAUNCH_PDL(L, softmax_og_kernel, grid1d(n, 256), 256, 0, L.stream, y, t, g, n);
  return NN_OK;
}

// -------------------------------------------------------------- Transpose
// NeuroNet.cl:4237-4248, smem-tiled, per sample.
__global__ void transpose_kernel(const float *in, float *out, int rows, int cols) {
  pdl_wait();
  pdl_trigger();
  __shared__ float tile[32][33];
  size_t b = blockIdx.z;
  const float *src = in + b * (size_t)rows * cols;
  float *dst = out + b * (size_t)rows * cols;
  int c = blockIdx.x * 32 + threadIdx.x;
  for (int r = blockIdx.y * 32 + threadIdx.y; r < min(rows, (int)blockIdx.y * 32 + 32); r += 8)
    if (c < cols) tile[r - blockIdx.y * 32][threadIdx.x] = src[(size_t)r * cols + c];
  __syncthreads();
  int r = blockIdx.y * 32 + threadIdx.x;
  for (int cc = blockIdx.x * 32 + threadIdx.y; cc < min(cols, (int)blockIdx.x * 32 + 32); cc += 8)
    if (r < rows) dst[(size_t)cc * rows + r] = tile[threadIdx.x][cc - blockIdx.x * 32];
}
static int k_transpose(Launch &L) {
  int rows = (int)L.nd.g[0], cols = L.nd.dims > 1 ? (int)L.nd.g[1] : 1;
  size_t n = (size_t)rows * cols * L.B;
  float *in = L.buf(0, n), *out = L.buf(1, n);
  if (!in || !out) return NN_ERR_BOUNDS;
  dim3 grid(ceil_div(cols, 32), ceil_div(rows, 32), L.B);
  NN_LAUNCH_PDL(L, transpose_kernel, grid, dim3(32, 8), 0, L.stream, in, out, rows, cols);
  return NN_OK;
}

// ------------------------------------------------ Concatenate/Deconcatenate
// NeuroNet.cl:1538-1576 / 1601-1650: row-wise join / split of up to 4 buffers.
struct Parts {
  float *p[4];
  int w[4];
};
__global__ void concat_kernel(Parts parts, float *out, int n, int tot, int split) {
  pdl_wait();
  pdl_trigger();
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)n * tot) return;
  int row = (int)(t / tot), c = (int)(t % tot);
  int j = 0, off = 0;
  while (c >= off + parts.w[j]) {
    off += parts.w[j];
    ++j;
  }
  float *src = parts.p[j] + (size_t)row * parts.w[j] + (c - off);
  if (split)
    *src = nan0(out[t]);
  else
    out[t] = nan0(*src);
}
static int concat_common(Launch &L, bool split) {
  int n = (int)L.nd.g[0] * L.B;
  Parts parts;
  int tot = 0;
  for (int j = 0; j < 4; ++j) {
    parts.w[j] = L.i(2 * j + 1);
    if (parts.w[j] < 0) return L.fail(NN_ERR_ARG, "Concatenate: negative window");
    parts.p[j] = nullptr;
    if (parts.w[j] > 0) {
      parts.p[j] = L.buf(2 * j, (size_t)n * parts.w[j]);
      if (!parts.p[j]) return NN_ERR_BOUNDS;
    }
    tot += parts.w[j];
  }
  if (tot == 0 || n == 0) return NN_OK;
  float *o = L.buf(8, (size_t)n * tot);
  if (!o) return NN_ERR_BOUNDS;
  NN_LAUNCH_PDL(L, concat_kernel, grid1d((size_t)n * tot, 256), 256, 0, L.stream, parts, o, n, tot, split ? 1 : 0);
  return NN_OK;
}
static int k_concat(Launch &L) { return concat_common(L, false); }
static int k_deconcat(Launch &L) { return concat_common(L, true); }

const KernelDef kAttnKernels[] = {
    {"MHAttentionScore", "ppii", k_mh_attention_score, false},
    {"MHAttentionOut", "pppi", k_mh_attention_out, false},
    {"MHAttentionInsideGradients", "pppp", k_mh_attention_inside_gradients, false},
    {"SumMatrix", "pppifiiipi", k_sum_matrix, false},
    {"Normalize", "pi", k_normalize, false},
    {"SoftMax_FeedForward", "pp", k_softmax_ff, false},
    {"SoftMax_HiddenGradient", "ppp", k_softmax_hg, false},
    {"SoftMax_OutputGradient", "ppp", k_softmax_og, false},
    {"Transpose", "pp", k_transpose, false},
    {"ConcatenateBuffers", "pipipipip", k_concat, false},
    {"DeconcatenateBuffers", "pipipipip", k_deconcat, false},
};
const int kNumAttnKernels = sizeof(kAttnKernels) / sizeof(kAttnKernels[0]);

}  // namespace nn
