// Dense-layer kernels of the library (CNeuronBaseOCL path) and the
// elementwise kernels: FeedForward, CalcOutputGradient, CalcHiddenGradient,
// UpdateWeightsMomentum, UpdateWeightsAdam, NormalizeWeights, Activation,
// DeActivation, SoftUpdate, SoftUpdateAdam.
//
// Weight layout is the reference's: W[out][in+1] row-major with the bias in
// the last column, stored on the *source* layer (NeuroNet_Core.mqh:15568).
#include <cstring>
#include "../../include/nn_b200.h"
#include "gemm_fast.cuh"
#include "tc_gemm.cuh"
#include "gemm_simt.cuh"
#include "nn_device.cuh"
#include "nn_internal.h"
#include "wgrad.cuh"
#include "epi_dense.cuh"

namespace nn {

// out[i] = scale * sum_k p[k * stride + i]: block (32 entries, 8 split groups), each thread summing
// every 8th partial of one entry, then a shared-memory reduction.
__global__ void reduce_partials_kernel(float *out, GradSrc src, size_t n) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[8][33];
  const size_t i = blockIdx.x * (size_t)32 + threadIdx.x;
  float s = 0.f;
  if (i < n) {
    const size_t j = src.at(i);
#pragma unroll 4
    for (int k = threadIdx.y; k < src.splits; k += 8) s += src.p[k * src.stride + j];
  }
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y != 0 || i >= n) return;
  float t = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) t += red[j][threadIdx.x];
  out[i] = t * src.scale;
}

__global__ void colsum_partial_kernel(float *p, const float *g, int M, int rows, long long ld, int kchunk, int ldp,
                                      int col) {
  pdl_wait();
  pdl_trigger();
  int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= M) return;
  int r0 = blockIdx.y * kchunk, r1 = min(rows, r0 + kchunk);
  float s = 0.f;
  for (int r = r0; r < r1; ++r) s += nan0(g[(size_t)r * ld + m]);
  p[((size_t)blockIdx.y * M + m) * ldp + col] = s;
}

__global__ void colsum_rows_kernel(float *p, const float *g, int M, int rows, long long ld, int kchunk, int ldp,
                                   int col) {
  pdl_wait();
  pdl_trigger();
  // block (32 columns, 32 row groups): every warp reads one 128-byte row segment per load, and each
  // thread keeps four independent sums so that four loads are in flight
  __shared__ float red[32][33];
  const int m = blockIdx.x * 32 + threadIdx.x;
  const int r0 = blockIdx.y * kchunk, r1 = min(rows, r0 + kchunk);
  float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
  if (m < M) {
    int r = r0 + (int)threadIdx.y;
    for (; r + 96 < r1; r += 128) {
      s0 += nan0(g[(size_t)r * ld + m]);
      s1 += nan0(g[(size_t)(r + 32) * ld + m]);
      s2 += nan0(g[(size_t)(r + 64) * ld + m]);
      s3 += nan0(g[(size_t)(r + 96) * ld + m]);
    }
    for (; r < r1; r += 32) s0 += nan0(g[(size_t)r * ld + m]);
  }
  red[threadIdx.y][threadIdx.x] = (s0 + s1) + (s2 + s3);
  __syncthreads();
  if (threadIdx.y == 0 && m < M) {
    float t = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) t += red[j][threadIdx.x];
    p[((size_t)blockIdx.y * M + m) * ldp + col] = t;
  }
}

__global__ void wgrad_small_m_kernel(float *p, const float *A, long long lda, const float *X, long long ldx, int M,
                                     int N, int rows, int kchunk, int ldp) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[8][kSmallM][33];
  const int n = blockIdx.x * 32 + threadIdx.x;  // n == N: the bias column (input 1)
  const int r0 = blockIdx.y * kchunk, r1 = min(rows, r0 + kchunk);
  float s[kSmallM];
#pragma unroll
  for (int m = 0; m < kSmallM; ++m) s[m] = 0.f;
  if (n <= N) {
#pragma unroll 4
    for (int r = r0 + (int)threadIdx.y; r < r1; r += 8) {
      const float x = n < N ? nan0(X[(size_t)r * ldx + n]) : 1.f;
      const float *a = A + (size_t)r * lda;  // the same M values for the whole warp (broadcast)
#pragma unroll
      for (int m = 0; m < kSmallM; ++m)
        if (m < M) s[m] += nan0(a[m]) * x;
    }
  }
#pragma unroll
  for (int m = 0; m < kSmallM; ++m) red[threadIdx.y][m][threadIdx.x] = s[m];
  __syncthreads();
  if (threadIdx.y != 0 || n > N) return;
  for (int m = 0; m < M; ++m) {
    float t = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) t += red[j][m][threadIdx.x];
    p[((size_t)blockIdx.y * M + m) * ldp + n] = t;
  }
}

// ------------------------------------------------------------ FeedForward
// NeuroNet.cl:430-512.  y[b,o] = act(sum_k nan0(nan0(x[b,k]) w[o,k]) + nan0(w[o,in]))
// Small batches: one warp per output row, lanes striding the row (coalesced).  Launched with
// programmatic dependent launch, like the other kernels of a batch-1 step (the output gradient, the
// hidden gradient, the fused update): each waits for its predecessor's writes before its first read
// and lets its successor launch at once.
template <int MAXB>
__global__ void ff_rows_kernel(const float *__restrict__ w, const float *__restrict__ x, float *__restrict__ y,
                               int inputs, int outputs, int B, int act) {
  pdl_wait();
  pdl_trigger();
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  if (warp >= outputs) return;
  const float *row = w + (size_t)warp * (inputs + 1);
  float s[MAXB];
#pragma unroll
  for (int b = 0; b < MAXB; ++b) s[b] = 0.f;
#pragma unroll 4
  for (int k = lane; k < inputs; k += 32) {
    float wk = row[k];
#pragma unroll
    for (int b = 0; b < MAXB; ++b)
      if (b < B) s[b] += nan0(nan0(x[(size_t)b * inputs + k]) * wk);
  }
  float bias = nan0(row[inputs]);
#pragma unroll
  for (int b = 0; b < MAXB; ++b) {
    if (b >= B) break;
    float t = warp_sum(s[b]);
    if (lane == 0) y[(size_t)b * outputs + warp] = activate(t + bias, act);
  }
}

// Many samples, at most kSkinny outputs (a value head, an action head): one warp per sample, lanes
// striding its inputs, every output's dot product kept in registers; the same arithmetic as
// ff_rows_kernel.
constexpr int kSkinny = 16;
__global__ void ff_skinny_kernel(const float *__restrict__ w, const float *__restrict__ x, float *__restrict__ y,
                                 int inputs, int outputs, int B, int act) {
  pdl_wait();
  pdl_trigger();
  const int b = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (b >= B) return;
  const float *xb = x + (size_t)b * inputs;
  float s[kSkinny];
#pragma unroll
  for (int o = 0; o < kSkinny; ++o) s[o] = 0.f;
#pragma unroll 4
  for (int k = lane; k < inputs; k += 32) {
    const float xk = nan0(xb[k]);
#pragma unroll
    for (int o = 0; o < kSkinny; ++o)
      if (o < outputs) s[o] += nan0(xk * w[(size_t)o * (inputs + 1) + k]);
  }
#pragma unroll
  for (int o = 0; o < kSkinny; ++o) {
    if (o >= outputs) break;
    const float t = warp_sum(s[o]);
    if (lane == 0) y[(size_t)b * outputs + o] = activate(t + nan0(w[(size_t)o * (inputs + 1) + inputs]), act);
  }
}

// Many samples, at most kSkinny outputs of the next layer: one thread per (sample, input), k
// ascending.
__global__ void chg_skinny_kernel(const float *__restrict__ w, const float *__restrict__ g, const float *__restrict__ o,
                                  float *__restrict__ ig, int inputs, int outputs, int B, int act) {
  pdl_wait();
  pdl_trigger();
  const size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)B * inputs) return;
  const int i = (int)(t % inputs);
  const float *gb = g + (t / inputs) * outputs;  // the same row for a warp's inputs (broadcast)
  float s = 0.f;
#pragma unroll 4
  for (int k = 0; k < outputs; ++k) s += nan0(w[(size_t)k * (inputs + 1) + i]) * nan0(gb[k]);
  ig[t] = deactivate(s, o[t], act);
}

struct FFLoadX {
  const float *x;
  int inputs;
  __device__ __forceinline__ float operator()(int m, int k, int) const { return nan0(x[(size_t)m * inputs + k]); }
};
struct FFLoadW {  // B(k, n) = W[n][k]
  const float *w;
  int ld;
  __device__ __forceinline__ float operator()(int k, int n, int) const { return nan0(w[(size_t)n * ld + k]); }
};
__global__ void ff_flags_kernel(const float *w, const float *x, const float *y, float *flags, int inputs,
                                int outputs, int B) {
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)B * outputs) return;
  int b = (int)(t / outputs), o = (int)(t % outputs);
  const float *row = w + (size_t)o * (inputs + 1);
  bool bad = false;
  float s = 0.f;
  for (int k = 0; k < inputs; ++k) {
    float xi = x[(size_t)b * inputs + k], wk = row[k];
    bad |= !isfinite(xi) || !isfinite(wk) || !isfinite(xi * wk);
    s += nan0(nan0(xi) * wk);
  }
  bad |= !isfinite(row[inputs]) || !isfinite(s) || !isfinite(y[t]);
  flags[t] = bad ? 1.f : 0.f;
}

static int k_feedforward(Launch &L) {
  const int outputs = (int)L.nd.g[0];
  const int inputs = L.i(3), act = L.i(4), fe = L.i(6);
  if (inputs < 0) return L.fail(NN_ERR_ARG, "FeedForward: negative inputs");
  const int ld = inputs + 1;
  float *w = L.buf(0, (size_t)outputs * ld);
  float *x = L.buf(1, (size_t)L.B * inputs);
  float *y = L.buf(2, (size_t)L.B * outputs);
  if (!w || !x || !y) return NN_ERR_BOUNDS;
  float *flags = nullptr;
  if (fe) {
    flags = L.buf(5, (size_t)L.B * outputs);
    if (!flags) return NN_ERR_BOUNDS;
  }
  if (L.B <= 4) {
    unsigned blocks = ceil_div((size_t)outputs * 32, 256);
    NN_LAUNCH_PDL(L, ff_rows_kernel<4>, blocks, 256, 0, L.stream, w, x, y, inputs, outputs, L.B, act);
  } else if (outputs <= kSkinny) {
    NN_LAUNCH_PDL(L, ff_skinny_kernel, ceil_div((size_t)L.B * 32, 256), 256, 0, L.stream, w, x, y, inputs, outputs, L.B, act);
  } else {
    FastShape fs{L.B, outputs, inputs, 1, 1, 0, x, inputs, 0, w, ld, 0};
    cudaError_t e = tma_store_ok(y, outputs, 0, 1, outputs)
                        ? gemm_f32_wb<false, false>(L, fs, FFEpiTma{{w, y, ld, inputs, outputs, act}})
                        : gemm_f32_wb<false, false>(L, fs, FFEpi{w, y, ld, inputs, outputs, act});
    if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
    L.counted();
  }
  if (fe) {
    ff_flags_kernel<<<grid1d((size_t)L.B * outputs, 256), 256, 0, L.stream>>>(w, x, y, flags, inputs, outputs, L.B);
    NN_CHECK_LAUNCH(L);
  }
  return NN_OK;
}

// ----------------------------------------------------- CalcOutputGradient
// NeuroNet.cl:523-536.  ig = Deactivation(t - o, o, act); the `error` argument is unused.
__global__ void out_grad_kernel(const float *t, const float *o, float *ig, size_t n, int act) {
  pdl_wait();
  pdl_trigger();
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  float out = o[i];
  ig[i] = isfinite(out) ? deactivate(t[i] - out, out, act) : 0.f;
}

static int k_calc_output_gradient(Launch &L) {
  size_t n = (size_t)L.nd.g[0] * L.B;
  float *t = L.buf(0, n), *o = L.buf(1, n), *ig = L.buf(2, n);
  if (!t || !o || !ig) return NN_ERR_BOUNDS;
  NN_LAUNCH_PDL(L, out_grad_kernel, grid1d(n, 256), 256, 0, L.stream, t, o, ig, n, L.i(3));
  return NN_OK;
}

// ----------------------------------------------------- CalcHiddenGradient
// NeuroNet.cl:547-613.  ig[b,i] = Deactivation(sum_k nan0(w[k,i]) nan0(g[b,k]), o[b,i], act)
// Small batches: a CTA of 16 warps per CPB columns.  Lane l of a warp takes column l % CPB and k
// lane l / CPB, so the CTA splits the k range KS = 16 * 32 / CPB ways (each thread sums its k in
// ascending order, KS apart); a warp load reads 32 / CPB rows of W, CPB floats each.  Narrow
// column groups spread a batch-1 product of a few hundred columns over about a hundred CTAs
// instead of a dozen.  The KS partials of each (sample, column) are summed by one warp in a fixed
// shuffle order.
constexpr int kChgWarps = 16;
template <int MAXB, int CPB>
__global__ void __launch_bounds__(kChgWarps * 32) chg_cols_kernel(const float *__restrict__ w,
                                                                  const float *__restrict__ g,
                                                                  const float *__restrict__ o, float *__restrict__ ig,
                                                                  int inputs, int outputs, int B, int act) {
  constexpr int KL = 32 / CPB, KS = kChgWarps * KL;
  __shared__ float part[MAXB][CPB][KS + 1];
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, wv = threadIdx.x >> 5;
  const int c = lane % CPB, kid = wv * KL + lane / CPB;
  const int col = blockIdx.x * CPB + c;
  float s[MAXB];
#pragma unroll
  for (int b = 0; b < MAXB; ++b) s[b] = 0.f;
  if (col < inputs) {
    const size_t ld = (size_t)inputs + 1;
#pragma unroll 4
    for (int k = kid; k < outputs; k += KS) {
      const float wk = nan0(w[(size_t)k * ld + col]);
#pragma unroll
      for (int b = 0; b < MAXB; ++b)
        if (b < B) s[b] += wk * nan0(g[(size_t)b * outputs + k]);
    }
  }
#pragma unroll
  for (int b = 0; b < MAXB; ++b) part[b][c][kid] = s[b];
  __syncthreads();
  // warp wv reduces the (sample, column) pairs wv, wv + 16, ...
  for (int pr = wv; pr < B * CPB; pr += kChgWarps) {
    const int b = pr / CPB, cc = pr % CPB, col2 = blockIdx.x * CPB + cc;
    float t = 0.f;
    for (int r = lane; r < KS; r += 32) t += part[b][cc][r];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) t += __shfl_down_sync(0xffffffffu, t, off);
    if (lane == 0 && col2 < inputs) {
      const size_t idx = (size_t)b * inputs + col2;
      ig[idx] = deactivate(t, o[idx], act);
    }
  }
}

struct CHGLoadG {
  const float *g;
  int outputs;
  __device__ __forceinline__ float operator()(int m, int k, int) const { return nan0(g[(size_t)m * outputs + k]); }
};
struct CHGLoadW {  // B(k, n) = W[k][n]
  const float *w;
  int ld;
  __device__ __forceinline__ float operator()(int k, int n, int) const { return nan0(w[(size_t)k * ld + n]); }
};
static int k_calc_hidden_gradient(Launch &L) {
  const int inputs = (int)L.nd.g[0];
  const int outputs = L.i(4), act = L.i(5);
  if (outputs < 0) return L.fail(NN_ERR_ARG, "CalcHiddenGradient: negative outputs");
  const int ld = inputs + 1;
  float *w = L.buf(0, (size_t)outputs * ld);
  float *g = L.buf(1, (size_t)L.B * outputs);
  float *o = L.buf(2, (size_t)L.B * inputs);
  float *ig = L.buf(3, (size_t)L.B * inputs);
  if (!w || !g || !o || !ig) return NN_ERR_BOUNDS;
  if (L.B <= 4) {
    // column groups as wide as still give most SMs a CTA
    if (inputs >= 32 * 148)
      NN_LAUNCH_PDL(L, (chg_cols_kernel<4, 32>), ceil_div(inputs, 32), kChgWarps * 32, 0, L.stream, w, g, o, ig,
                    inputs, outputs, L.B, act);
    else if (inputs >= 8 * 74)
      NN_LAUNCH_PDL(L, (chg_cols_kernel<4, 8>), ceil_div(inputs, 8), kChgWarps * 32, 0, L.stream, w, g, o, ig, inputs,
                    outputs, L.B, act);
    else
      NN_LAUNCH_PDL(L, (chg_cols_kernel<4, 4>), ceil_div(inputs, 4), kChgWarps * 32, 0, L.stream, w, g, o, ig, inputs,
                    outputs, L.B, act);
    return NN_OK;
  }
  if (outputs <= kSkinny) {
    NN_LAUNCH_PDL(L, chg_skinny_kernel, grid1d((size_t)L.B * inputs, 256), 256, 0, L.stream, w, g, o, ig, inputs, outputs, L.B, act);
    return NN_OK;
  }
  FastShape fs{L.B, inputs, outputs, 1, 1, 0, g, outputs, 0, w, ld, 0};
  cudaError_t e = tma_store_ok(ig, inputs, 0, 1, inputs) && ((uintptr_t)o & 15) == 0
                      ? gemm_f32_wb<false, true>(L, fs, CHGEpiTma{{o, ig, inputs, act}})
                      : gemm_f32_wb<false, true>(L, fs, CHGEpi{o, ig, inputs, act});
  if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
  L.counted();
  return NN_OK;
}

// ---------------------------------------------------------- dense updates
// Batch weight gradient G[o][j] = (1/B) sum_b gsrc(b,o) * inp(b,j), inp(b, inputs) = 1.
struct WGLoadG {  // A(m=o, k=b)
  const float *g;
  int outputs;
  int clamp_g;  // momentum path clamps the node gradient per sample
  __device__ __forceinline__ float operator()(int m, int k, int) const {
    float v = g[(size_t)k * outputs + m];
    return clamp_g ? clampf(v, -kMaxGrad, kMaxGrad) : nan0(v);
  }
};
struct WGLoadX {  // B(k=b, n=j)
  const float *x;
  int inputs;
  __device__ __forceinline__ float operator()(int k, int n, int) const {
    return n < inputs ? nan0(x[(size_t)k * inputs + n]) : 1.f;
  }
};

// UpdateWeightsAdam arithmetic (NeuroNet.cl:678-693) with a given pre-clamp gradient.
// UpdateWeightsAdam arithmetic for one weight, given its (batch-mean) gradient before clamping.
__device__ __forceinline__ void adam_dense_step(float *w, float *m, float *v, size_t wi, float graw, float l, float b1,
                                                float b2) {
  float weight = nan0(w[wi]);
  float mm = nan0(m[wi]);
  float vv = nan0(v[wi]);
  float g = clampf(nan0(graw), -kMaxGrad, kMaxGrad);
  float mt = nan0(b1 * mm + (1.f - b1) * g);
  float vt = nan0(b2 * vv + (1.f - b2) * (g * g));
  float delta = nan0(l * (mt / (sqrtf(vt) + 1.0e-37f) - (kL1 * signf(weight) + kL2 * weight)));
  if (fabsf(delta) > 0.f) w[wi] = nan0(w[wi] + delta);
  m[wi] = mt;
  v[wi] = vt;
}

__global__ void adam_dense_apply_kernel(float *w, float *m, float *v, GradSrc G, int n_out, int n_col, int inputs,
                                        float l, float b1, float b2) {
  pdl_wait();
  pdl_trigger();
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)n_out * n_col) return;
  int i = (int)(t / n_col), j = (int)(t % n_col);
  adam_dense_step(w, m, v, (size_t)i * (inputs + 1) + j, G(t), l, b1, b2);
}

// The same with many split-K partials: block (32 weights, 8 split groups), as reduce_partials_kernel.
__global__ void adam_dense_apply_split_kernel(float *w, float *m, float *v, GradSrc G, int n_out, int n_col,
                                              int inputs, float l, float b1, float b2) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[8][33];
  const size_t t = blockIdx.x * (size_t)32 + threadIdx.x, n = (size_t)n_out * n_col;
  float s = 0.f;
  if (t < n) {
    const size_t ga = G.at(t);
#pragma unroll 4
    for (int k = threadIdx.y; k < G.splits; k += 8) s += G.p[k * G.stride + ga];
  }
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y != 0 || t >= n) return;
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) sum += red[j][threadIdx.x];
  const int i = (int)(t / n_col), j = (int)(t % n_col);
  adam_dense_step(w, m, v, (size_t)i * (inputs + 1) + j, sum * G.scale, l, b1, b2);
}

// Single-sample fused kernel: exactly the reference's per-weight arithmetic.
__global__ void adam_dense_fused_kernel(float *w, const float *g, const float *x, float *m, float *v, int n_out,
                                        int n_col, int inputs, float l, float b1, float b2) {
  pdl_wait();
  pdl_trigger();
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)n_out * n_col) return;
  int i = (int)(t / n_col), j = (int)(t % n_col);
  size_t wi = (size_t)i * (inputs + 1) + j;
  float inp = nan0(j == inputs ? 1.f : x[j]);
  float weight = nan0(w[wi]);
  float mm = nan0(m[wi]);
  float vv = nan0(v[wi]);
  float gg = clampf(nan0(g[i] * inp), -kMaxGrad, kMaxGrad);
  float mt = nan0(b1 * mm + (1.f - b1) * gg);
  float vt = nan0(b2 * vv + (1.f - b2) * (gg * gg));
  float delta = nan0(l * (mt / (sqrtf(vt) + 1.0e-37f) - (kL1 * signf(weight) + kL2 * weight)));
  if (fabsf(delta) > 0.f) w[wi] = nan0(w[wi] + delta);
  m[wi] = mt;
  v[wi] = vt;
}

struct AdamDenseShape {
  int n_out, n_col, inputs;
};
static AdamDenseShape adam_dense_shape(const Launch &L) {
  return AdamDenseShape{(int)L.nd.g[0], L.nd.dims > 1 ? (int)L.nd.g[1] : 1, L.i(5)};
}

// UpdateWeightsAdam on weight idx of [n_out][inputs+1] (whole rows: n_col == inputs + 1) from one
// sample's output gradient and inputs, the reference kernel's own arithmetic, for
// update_normalize_rows_flat_kernel.
struct DenseAdamSampleStep {
  float *w, *m, *v;
  const float *g, *x;
  int n_col, inputs;
  float l, b1, b2;
  __device__ float operator()(size_t idx) const {
    const int i = (int)(idx / n_col), j = (int)(idx % n_col);
    float inp = nan0(j == inputs ? 1.f : x[j]);
    float weight = nan0(w[idx]);
    float mm = nan0(m[idx]);
    float vv = nan0(v[idx]);
    float gg = clampf(nan0(g[i] * inp), -kMaxGrad, kMaxGrad);
    float mt = nan0(b1 * mm + (1.f - b1) * gg);
    float vt = nan0(b2 * vv + (1.f - b2) * (gg * gg));
    float delta = nan0(l * (mt / (sqrtf(vt) + 1.0e-37f) - (kL1 * signf(weight) + kL2 * weight)));
    if (fabsf(delta) > 0.f) w[idx] = nan0(w[idx] + delta);
    m[idx] = mt;
    v[idx] = vt;
    return w[idx];
  }
};

static int adam_dense_apply_src(const Launch &Lc, GradSrc G) {
  Launch &L = const_cast<Launch &>(Lc);
  AdamDenseShape s = adam_dense_shape(L);
  size_t nw = (size_t)(s.n_out - 1) * (s.inputs + 1) + s.n_col;
  float *w = L.buf(0, nw), *m = L.buf(3, nw), *v = L.buf(4, nw);
  if (!w || !m || !v) return NN_ERR_BOUNDS;
  size_t n = (size_t)s.n_out * s.n_col;
  if (G.splits > 4)
    NN_LAUNCH_PDL(L, adam_dense_apply_split_kernel, (unsigned)((n + 31) / 32), dim3(32, 8), 0, L.stream, w, m, v, G,
                  s.n_out, s.n_col, s.inputs, L.f(6), L.f(7), L.f(8));
  else
    NN_LAUNCH_PDL(L, adam_dense_apply_kernel, grid1d(n, 256), 256, 0, L.stream, w, m, v, G, s.n_out, s.n_col, s.inputs, L.f(6), L.f(7), L.f(8));
  if (L.norm_rows > 0) {
    // the folded NormalizeWeights after a batched update (see adam_conv_apply_src)
    NN_LAUNCH_PDL(L, normalize_weights_kernel, ceil_div((size_t)L.norm_rows * 32, 256), 256, 0, L.stream, w, L.norm_rows, L.norm_dim);
  }
  return NN_OK;
}
static int adam_dense_apply(const Launch &L, const float *grad) {
  return adam_dense_apply_src(L, GradSrc{grad, 1, 0, 1.f});
}

static int k_update_weights_adam(Launch &L) {
  AdamDenseShape s = adam_dense_shape(L);
  if (s.inputs < 0 || s.n_col > s.inputs + 1) return L.fail(NN_ERR_ARG, "UpdateWeightsAdam: bad shape");
  size_t nw = (size_t)(s.n_out - 1) * (s.inputs + 1) + s.n_col;
  float *w = L.buf(0, nw), *g = L.buf(1, (size_t)L.B * s.n_out), *x = L.buf(2, (size_t)L.B * s.inputs);
  float *m = L.buf(3, nw), *v = L.buf(4, nw);
  if (!w || !g || !x || !m || !v) return NN_ERR_BOUNDS;
  if (L.B == 1 && !L.deferred()) {
    if (L.norm_rows > 0) {
      NN_LAUNCH_PDL(L, update_normalize_rows_flat_kernel<DenseAdamSampleStep>, L.norm_rows, 256, 0, L.stream, w,
                    L.norm_rows, L.norm_dim,
                    DenseAdamSampleStep{w, m, v, g, x, s.n_col, s.inputs, L.f(6), L.f(7), L.f(8)});
      return NN_OK;
    }
    size_t n = (size_t)s.n_out * s.n_col;
    NN_LAUNCH_PDL(L, adam_dense_fused_kernel, grid1d(n, 256), 256, 0, L.stream, w, g, x, m, v, s.n_out, s.n_col, s.inputs, L.f(6), L.f(7), L.f(8));
    return NN_OK;
  }
  GradSrc src;
  int rc = s.n_col == s.inputs + 1
               ? wgrad_fast(L, g, s.n_out, x, s.inputs, s.n_out, s.inputs, L.B, &src)
               : wgrad_partials<false, true>(L, s.n_out, s.n_col, L.B, 1, WGLoadG{g, s.n_out, 0},
                                             WGLoadX{x, s.inputs}, &src);
  if (rc) return rc;
  src.scale = 1.f / (float)L.B;
  return finish_update(L, src, (size_t)s.n_out * s.n_col, adam_dense_apply, adam_dense_apply_src);
}

// UpdateWeightsAdamMini (NeuroNet.cl:7515-7612), one sample: global (inputs+1, outputs), local
// (inputs+1, 1).  Every output row shares the scale s of the reference's local reduction of
// inp^2 / inputs: slot t of ls = min(64, inputs) sums local ids t, t + ls, ... that its count loop
// reaches (the bias input 1 only when inputs % ls != 0), then the folding loop, which stops before
// its last step, leaves s in slot 0.  One block of 64 threads reproduces that order.
__global__ void adam_mini_scale_kernel(const float *__restrict__ x, int inputs, float *__restrict__ s_out) {
  __shared__ float temp[64];
  const int ls = min(64, inputs), t = threadIdx.x;
  if (t < ls) {
    const int counts = (inputs + ls - 1) / ls;
    float acc = 0.f;
    for (int count = 0; count < counts; ++count) {
      const int i = count * ls + t;
      if (i > inputs) break;
      const float inp = i < inputs ? x[i] : 1.f;
      const float term = isfinite(inp) ? inp * inp / (float)inputs : 0.f;
      acc = (count == 0 ? 0.f : acc) + term;
    }
    temp[t] = acc;
  }
  __syncthreads();
  int count = (ls + 1) / 2;
  while (true) {
    if (t < count && t + count < ls) {
      temp[t] += temp[t + count];
      temp[t + count] = 0.f;
    }
    count = (count + 1) / 2;
    __syncthreads();
    if (!(count > 1)) break;
  }
  if (t == 0) *s_out = temp[0];
}

// One block per output row: its second moment from the shared scale, then every weight of the row.
__global__ void adam_mini_apply_kernel(float *w, const float *g, const float *x, float *m, float *v,
                                       const float *s_in, int inputs, float l, float b1, float b2) {
  __shared__ float vt_s, g_s;
  const int o = blockIdx.x;
  if (threadIdx.x == 0) {
    float gg = g[o];
    if (!isfinite(gg)) gg = 0.f;
    float t0 = *s_in;
    if (!isfinite(t0)) t0 = 1.f;
    float vv = v[o];
    if (!isfinite(vv)) vv = 1.f;
    t0 = b2 * vv + (1.f - b2) * (gg * gg) * t0;
    v[o] = t0;
    vt_s = t0;
    g_s = gg;
  }
  __syncthreads();
  const float vt = vt_s, gg = g_s;
  for (int i = threadIdx.x; i <= inputs; i += blockDim.x) {
    const size_t wi = (size_t)o * (inputs + 1) + i;
    const float inp = i < inputs ? x[i] : 1.f;
    float weight = w[wi];
    if (!isfinite(weight)) weight = 0.f;
    float mm = m[wi];
    if (!isfinite(mm)) mm = 0.f;
    mm = b1 * mm + (1.f - b1) * gg * inp;
    if (!isfinite(mm)) mm = 0.f;
    float delta = l * (mm / (sqrtf(vt) + 1.0e-37f) - (kL1 * signf(weight) + kL2 * weight));
    if (!isfinite(delta)) delta = 0.f;
    if (delta > 0.f) w[wi] = weight + delta;
    m[wi] = mm;
  }
}

static int k_update_weights_adam_mini(Launch &L) {
  if (!L.nd.has_local || L.nd.dims < 2)
    return L.fail(NN_ERR_ARG, "UpdateWeightsAdamMini: needs global (inputs+1, outputs) and local (inputs+1, 1)");
  const int inputs = (int)L.nd.l[0] - 1, outputs = (int)L.nd.g[1];
  if (inputs < 1 || (int)L.nd.g[0] != inputs + 1)
    return L.fail(NN_ERR_ARG, "UpdateWeightsAdamMini: global size 0 must equal local size 0 (inputs + 1)");
  if (L.B != 1 || L.deferred())
    return L.fail(NN_ERR_UNSUPPORTED, "UpdateWeightsAdamMini: one sample per execution (the reference's "
                                      "per-row second moment has no batch-mean form here)");
  const size_t nw = (size_t)outputs * (inputs + 1);
  float *w = L.buf(0, nw), *g = L.buf(1, outputs), *x = L.buf(2, inputs), *m = L.buf(3, nw);
  float *v = L.buf(4, outputs);
  if (!w || !g || !x || !m || !v) return NN_ERR_BOUNDS;
  float *s = L.scratch(3, 1);
  if (!s) return NN_ERR_CUDA;
  adam_mini_scale_kernel<<<1, 64, 0, L.stream>>>(x, inputs, s);
  NN_CHECK_LAUNCH(L);
  adam_mini_apply_kernel<<<outputs, 256, 0, L.stream>>>(w, g, x, m, v, s, inputs, L.f(5), L.f(6), L.f(7));
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

// UpdateWeightsMomentum (NeuroNet.cl:624-645); batch: G = mean_b clamp(g_b) x_b.
__global__ void momentum_dense_kernel(float *w, float *dw, GradSrc G, const float *g, const float *x, int n_out,
                                      int n_col, int inputs, float lr, float mom, int fused) {
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)n_out * n_col) return;
  int i = (int)(t / n_col), j = (int)(t % n_col);
  size_t wi = (size_t)i * (inputs + 1) + j;
  float term;
  if (fused) {
    float grad = clampf(g[i], -kMaxGrad, kMaxGrad);
    term = nan0(lr * grad * (j < inputs ? x[j] : 1.f));
  } else {
    term = nan0(lr * G(t));
  }
  float delta = term + nan0(mom * dw[wi]);
  dw[wi] = delta;
  if (fabsf(delta) > 0.f) w[wi] = nan0(w[wi] + delta);
}

static int momentum_dense_apply_src(const Launch &Lc, GradSrc G) {
  Launch &L = const_cast<Launch &>(Lc);
  int n_out = (int)L.nd.g[0], n_col = L.nd.dims > 1 ? (int)L.nd.g[1] : 1, inputs = L.i(4);
  size_t nw = (size_t)(n_out - 1) * (inputs + 1) + n_col;
  float *w = L.buf(0, nw), *dw = L.buf(3, nw);
  if (!w || !dw) return NN_ERR_BOUNDS;
  size_t n = (size_t)n_out * n_col;
  momentum_dense_kernel<<<grid1d(n, 256), 256, 0, L.stream>>>(w, dw, G, nullptr, nullptr, n_out, n_col, inputs,
                                                              L.f(5), L.f(6), 0);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}
static int momentum_dense_apply(const Launch &L, const float *grad) {
  return momentum_dense_apply_src(L, GradSrc{grad, 1, 0, 1.f});
}

static int k_update_weights_momentum(Launch &L) {
  int n_out = (int)L.nd.g[0], n_col = L.nd.dims > 1 ? (int)L.nd.g[1] : 1, inputs = L.i(4);
  if (inputs < 0 || n_col > inputs + 1) return L.fail(NN_ERR_ARG, "UpdateWeightsMomentum: bad shape");
  size_t nw = (size_t)(n_out - 1) * (inputs + 1) + n_col;
  float *w = L.buf(0, nw), *g = L.buf(1, (size_t)L.B * n_out), *x = L.buf(2, (size_t)L.B * inputs);
  float *dw = L.buf(3, nw);
  if (!w || !g || !x || !dw) return NN_ERR_BOUNDS;
  if (L.B == 1 && !L.deferred()) {
    size_t n = (size_t)n_out * n_col;
    momentum_dense_kernel<<<grid1d(n, 256), 256, 0, L.stream>>>(w, dw, GradSrc{nullptr, 0, 0, 1.f}, g, x, n_out,
                                                                n_col, inputs, L.f(5), L.f(6), 1);
    NN_CHECK_LAUNCH(L);
    return NN_OK;
  }
  GradSrc src;
  int rc = wgrad_partials<false, true>(L, n_out, n_col, L.B, 1, WGLoadG{g, n_out, 1}, WGLoadX{x, inputs}, &src);
  if (rc) return rc;
  src.scale = 1.f / (float)L.B;
  return finish_update(L, src, (size_t)n_out * n_col, momentum_dense_apply, momentum_dense_apply_src);
}

// ------------------------------------------------------- NormalizeWeights
// NeuroNet.cl:1498-1525: rows of `dimension` weights rescaled to unit norm when
// the norm exceeds 1; the 10x pre-scaling retry handles overflow.
__global__ void normalize_weights_kernel(float *buf, int rows, int dim) {
  pdl_wait();
  pdl_trigger();
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  float *row = buf + (size_t)warp * dim;
  float k = 1.f;
  float s;
  for (int guard = 0; guard < 64; ++guard) {
    s = 0.f;
    for (int i = lane; i < dim; i += 32) {
      const float q = guard == 0 ? nan0(row[i]) : nan0(row[i]) / k;  // k == 1 on the first pass
      s += q * q;
    }
    s = warp_sum(s);
    if (isfinite(s)) break;
    k *= 10.f;
  }
  s = sqrtf(s);
  float d = k * s;
  if (d > 1.f)
    for (int i = lane; i < dim; i += 32) row[i] = nan0(row[i]) / d;
}

bool update_normalize_fusable(const KernelInst &u, const NDR &nu, const KernelInst &nw, const NDR &nnw) {
  if (nw.args[0].type != ARG_BUF || u.args[0].type != ARG_BUF || nw.args[0].i != u.args[0].i) return false;
  const int dim = nw.args[1].i;
  const size_t rows = nnw.g[0];
  if (dim <= 0 || rows == 0) return false;
  if (std::strcmp(u.def->name, "UpdateWeightsAdam") == 0) {
    const size_t n_out = nu.g[0], n_col = nu.dims > 1 ? nu.g[1] : 1;
    const int inputs = u.args[5].i;
    return n_col == (size_t)inputs + 1 && dim == inputs + 1 && rows == n_out;
  }
  if (std::strcmp(u.def->name, "UpdateWeightsConvAdam") == 0) {
    const int win = u.args[9].i;
    return dim == win + 1 && rows * (size_t)dim == nu.g[0];
  }
  return false;
}

static int k_normalize_weights(Launch &L) {
  int rows = (int)L.nd.g[0], dim = L.i(1);
  if (dim < 0) return L.fail(NN_ERR_ARG, "NormalizeWeights: negative dimension");
  float *b = L.buf(0, (size_t)rows * dim);
  if (!b) return NN_ERR_BOUNDS;
  NN_LAUNCH_PDL(L, normalize_weights_kernel, ceil_div((size_t)rows * 32, 256), 256, 0, L.stream, b, rows, dim);
  return NN_OK;
}

// ------------------------------------------------------------ elementwise
__global__ void activation_kernel(const float *in, float *out, size_t n, int act) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) out[i] = activate(nan0(in[i]), act);
}
static int k_activation(Launch &L) {  // NeuroNet.cl:5796-5808
  size_t n = (size_t)L.nd.g[0] * L.B;
  float *in = L.buf(0, n), *out = L.buf(1, n);
  if (!in || !out) return NN_ERR_BOUNDS;
  activation_kernel<<<grid1d(n, 256), 256, 0, L.stream>>>(in, out, n, L.i(2));
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

__global__ void deactivation_kernel(const float *in, float *in_gr, const float *out_gr, size_t n, int act) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) in_gr[i] = deactivate(nan0(out_gr[i]), in[i], act);
}
static int k_deactivation(Launch &L) {  // NeuroNet.cl:5811-5823
  size_t n = (size_t)L.nd.g[0] * L.B;
  float *in = L.buf(0, n), *ig = L.buf(1, n), *og = L.buf(2, n);
  if (!in || !ig || !og) return NN_ERR_BOUNDS;
  deactivation_kernel<<<grid1d(n, 256), 256, 0, L.stream>>>(in, ig, og, n, L.i(3));
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

__global__ void soft_update_kernel(float *t, const float *s, size_t n, float tau) {
  pdl_wait();
  pdl_trigger();
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) t[i] = s[i] * tau + (1.f - tau) * t[i];
}
static int k_soft_update(Launch &L) {  // NeuroNet.cl:3864-3871
  size_t n = L.nd.g[0];
  float *t = L.buf(0, n), *s = L.buf(1, n);
  if (!t || !s) return NN_ERR_BOUNDS;
  NN_LAUNCH_PDL(L, soft_update_kernel, grid1d(n, 256), 256, 0, L.stream, t, s, n, L.f(2));
  return NN_OK;
}

__global__ void soft_update_adam_kernel(float *t, const float *s, float *m, float *v, size_t n, float tau, float b1,
                                        float b2) {
  pdl_wait();
  pdl_trigger();
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  float mm = m[i], vv = v[i], weight = t[i];
  float g = s[i] - weight;
  mm = b1 * mm + (1.f - b1) * g;
  vv = b2 * vv + (1.f - b2) * (g * g);
  float delta = (1.f - tau) * mm / (vv != 0.f ? sqrtf(vv) : 1.f);
  if (fabsf(delta) > 0.f) t[i] = weight + delta;
  m[i] = mm;
  v[i] = vv;
}
static int k_soft_update_adam(Launch &L) {  // NeuroNet.cl:3875-3899
  size_t n = L.nd.g[0];
  float *t = L.buf(0, n), *s = L.buf(1, n), *m = L.buf(2, n), *v = L.buf(3, n);
  if (!t || !s || !m || !v) return NN_ERR_BOUNDS;
  NN_LAUNCH_PDL(L, soft_update_adam_kernel, grid1d(n, 256), 256, 0, L.stream, t, s, m, v, n, L.f(4), L.f(5), L.f(6));
  return NN_OK;
}

const KernelDef kDenseKernels[] = {
    {"FeedForward", "pppiipi", k_feedforward, false},
    {"CalcOutputGradient", "pppif", k_calc_output_gradient, false},
    {"CalcHiddenGradient", "ppppii", k_calc_hidden_gradient, false},
    {"UpdateWeightsMomentum", "ppppiff", k_update_weights_momentum, false},
    {"UpdateWeightsAdam", "pppppifff", k_update_weights_adam, false},
    {"UpdateWeightsAdamMini", "pppppfff", k_update_weights_adam_mini, false},
    {"NormalizeWeights", "pi", k_normalize_weights, true},
    {"Activation", "ppi", k_activation, false},
    {"DeActivation", "pppi", k_deactivation, false},
    {"SoftUpdate", "ppf", k_soft_update, true},
    {"SoftUpdateAdam", "ppppfff", k_soft_update_adam, true},
};
const int kNumDenseKernels = sizeof(kDenseKernels) / sizeof(kDenseKernels[0]);

}  // namespace nn
