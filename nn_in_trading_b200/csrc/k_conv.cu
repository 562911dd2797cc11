// Convolution kernels (CNeuronConvOCL path and the 1x1 "convolutions" of the
// attention layers): FeedForwardConv, CalcHiddenGradientConv,
// UpdateWeightsConvAdam, UpdateWeightsConvMomentum.
//
// Layout is the reference's: input [variables][inputs], output
// [variables][units][window_out], weights [variables][window_out][window_in+1]
// with the bias last.  With a batch, every per-sample buffer holds `batch`
// consecutive copies of that layout and the weights are shared.
#include "../../include/nn_b200.h"
#include "gemm_fast.cuh"
#include "tc_gemm.cuh"
#include "gemm_simt.cuh"
#include "nn_device.cuh"
#include "nn_internal.h"
#include "wgrad.cuh"

namespace nn {

// -------------------------------------------------------- FeedForwardConv
// NeuroNet.cl:887-932 as a GEMM per variable: rows (sample, unit), columns
// output channel, k the window offset (im2col view of the strided input).
struct ConvLoadX {
  const float *x;
  int units, step, inputs, var;
  __device__ __forceinline__ float operator()(int m, int k, int v) const {
    int b = m / units, u = m - b * units;
    int pos = u * step + k;
    return pos < inputs ? nan0(x[((size_t)b * var + v) * inputs + pos]) : 0.f;
  }
};
struct ConvLoadW {  // B(k, n) = W[v][n][k]
  const float *w;
  int win, wout;
  __device__ __forceinline__ float operator()(int k, int n, int v) const {
    return nan0(w[((size_t)v * wout + n) * (win + 1) + k]);
  }
};
struct ConvEpi {
  const float *w;
  float *o;
  int units, win, wout, var, act;
  __device__ __forceinline__ void operator()(int m, int n, int v, int, float acc) const {
    int b = m / units, u = m - b * units;
    float bias = nan0(w[((size_t)v * wout + n) * (win + 1) + win]);
    o[(((size_t)b * var + v) * units + u) * wout + n] = activate(acc + bias, act);
  }
};

// Plain-layout epilogue: one variable, windows tiling the input (row m at o + m*wout).
struct ConvEpiPlain {
  const float *w;
  float *o;
  int win, wout, act;
  __device__ __forceinline__ void operator()(int m, int n, int, int, float acc) const {
    o[(size_t)m * wout + n] = activate(acc + nan0(w[(size_t)n * (win + 1) + win]), act);
  }
  __device__ __forceinline__ long long row(int m, int, int) const { return (long long)m * wout; }
  __device__ __forceinline__ float col(int n, int) const { return nan0(w[(size_t)n * (win + 1) + win]); }
  template <int R>
  __device__ __forceinline__ void put_rows(const long long (&rb)[R], int n, const float (&v)[R], float bias,
                                           unsigned mask) const {
    act_dispatch(act, [&](auto A) {
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (mask >> j & 1u) o[rb[j] + n] = activate(v[j] + bias, decltype(A)::value);
    });
  }
  __host__ __device__ bool aligned4() const { return wout % 4 == 0 && ((uintptr_t)o & 15) == 0; }
  __device__ __forceinline__ float4 col4(int n, int z) const {
    return make_float4(col(n, z), col(n + 1, z), col(n + 2, z), col(n + 3, z));
  }
  template <int R>
  __device__ __forceinline__ void put_rows4(const long long (&rb)[R], int n, const float4 (&v)[R], float4 b,
                                            unsigned mask) const {
    act_dispatch(act, [&](auto A) {
      constexpr int a = decltype(A)::value;
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (mask >> j & 1u)
          *reinterpret_cast<float4 *>(o + rb[j] + n) = make_float4(
              activate(v[j].x + b.x, a), activate(v[j].y + b.y, a), activate(v[j].z + b.z, a),
              activate(v[j].w + b.w, a));
    });
  }
};

// ConvEpiPlain with the output written by TMA stores on the tensor-core path (rows of wout floats,
// 16-byte aligned, wout and the computed columns multiples of 4; checked with tma_store_ok).
struct ConvEpiTma : ConvEpiPlain {
  static constexpr bool kTmaStore = true;
  template <class F>
  __device__ __forceinline__ void transform(F &&f) const {
    act_dispatch(act, [&](auto A) { f([](float x, float b, float) { return activate(x + b, decltype(A)::value); }); });
  }
  __device__ __forceinline__ int zc(int z, int) const { return z; }
  bool out_map(CUtensorMap *tm, int M, int N, int nz) const { return make_tmap(tm, o, wout, 0, N, M, nz, 32, false); }
};

static int k_feedforward_conv(Launch &L) {
  const int units = (int)L.nd.g[0];
  const int wout_g = L.nd.dims > 1 ? (int)L.nd.g[1] : 1;
  const int var = L.nd.dims > 2 ? (int)L.nd.g[2] : 1;
  const int inputs = L.i(3), step = L.i(4), win = L.i(5), wout = L.i(6), act = L.i(7);
  if (inputs < 0 || step < 0 || win < 0 || wout < wout_g) return L.fail(NN_ERR_ARG, "FeedForwardConv: bad shape");
  float *w = L.buf(0, (size_t)var * wout * (win + 1));
  float *x = L.buf(1, (size_t)L.B * var * inputs);
  float *o = L.buf(2, (size_t)L.B * var * units * wout);
  if (!w || !x || !o) return NN_ERR_BOUNDS;
  cudaError_t e;
  if (var == 1 && step == win && inputs == units * step && win > 0) {
    // windows tile the input: a plain [B*units][win] x W^T GEMM
    FastShape fs{L.B * units, wout_g, win, 1, 1, 0, x, win, 0, w, win + 1, 0};
    if (tma_store_ok(o, wout, 0, 1, wout_g))
      e = gemm_f32_wb<false, false>(L, fs, ConvEpiTma{{w, o, win, wout, act}});
    else
      e = gemm_f32_wb<false, false>(L, fs, ConvEpiPlain{w, o, win, wout, act});
  } else {
    GemmShape sh{L.B * units, wout_g, win, var, 1};
    e = gemm_simt<true, false>(sh, ConvLoadX{x, units, step, inputs, var}, ConvLoadW{w, win, wout},
                               ConvEpi{w, o, units, win, wout, var, act}, L.stream);
  }
  if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
  L.counted();
  return NN_OK;
}

// ------------------------------------------------- CalcHiddenGradientConv
// NeuroNet.cl:941-986.  General form: one thread per (sample, variable, input)
// position summing over the windows that cover it.
__global__ void conv_dgrad_direct_kernel(const float *__restrict__ w, const float *__restrict__ g,
                                         const float *__restrict__ o, float *__restrict__ ig, int inputs, int var,
                                         int outputs, int step, int win, int wout, int act, int shift_out, int B) {
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t total = (size_t)B * var * inputs;
  if (t >= total) return;
  int i = (int)(t % inputs);
  size_t bv = t / inputs;
  int v = (int)(bv % var);
  size_t b = bv / var;
  const float *gs = g + shift_out + b * (size_t)var * outputs + (size_t)v * outputs;
  const float *ws = w + (size_t)v * wout * (win + 1);
  int start = i < win ? 0 : (i - win) / step + 1;
  int stop = min(i / step + 1, outputs / wout);
  float sum = 0.f;
  for (int h = 0; h < wout; ++h)
    for (int k = start; k < stop; ++k) {
      float gr = nan0(gs[k * wout + h]);
      if (fabsf(gr) > 0.f) sum += nan0(gr * ws[h * (win + 1) + i - k * step]);
    }
  ig[t] = deactivate(sum, o[t], act);
}

// Overlapping windows: one CTA of 256 threads per (sample, variable).  The row's output gradient
// (n_win windows x wout channels, nan0) and the variable's weights go to shared memory; each window's
// contribution P[k][r] = sum_h g[k][h] W[h][r] (r < window_in) is formed once, four windows' entries
// per thread at a time, then every input adds the windows that cover it, k ascending, and takes the
// derivative.  Every product keeps the reference's guard (a zero gradient adds nothing) and nan0; the
// sum runs over h per window, then over the windows (the direct form interleaves the two).
// Shared memory: n_win*wout + wout*(win+1) + n_win*win floats.
__global__ void __launch_bounds__(256) conv_dgrad_overlap_kernel(const float *__restrict__ w,
                                                                 const float *__restrict__ g,
                                                                 const float *__restrict__ o, float *__restrict__ ig,
                                                                 int inputs, int var, int outputs, int step, int win,
                                                                 int wout, int act, int shift_out) {
  extern __shared__ float sm[];
  pdl_wait();
  pdl_trigger();
  const int n_win = outputs / wout;
  const size_t bv = blockIdx.x;  // sample b, variable v: bv = b * var + v
  const int v = (int)(bv % var);
  float *gs_s = sm;                      // [n_win][wout]
  float *ws_s = gs_s + n_win * wout;     // [wout][win + 1]
  float *p_s = ws_s + wout * (win + 1);  // [n_win][win]
  const float *gs = g + shift_out + bv * (size_t)outputs;
  const float *ws = w + (size_t)v * wout * (win + 1);
  for (int t = threadIdx.x; t < n_win * wout; t += 256) gs_s[t] = nan0(gs[t]);
  for (int t = threadIdx.x; t < wout * (win + 1); t += 256) ws_s[t] = ws[t];
  __syncthreads();
  const int np = n_win * win;
  for (int q0 = threadIdx.x; q0 < np; q0 += 4 * 256) {
    int kq[4], rq[4];
    float acc[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int q = min(q0 + 256 * j, np - 1);  // past the end: a duplicate, not stored
      kq[j] = q / win;
      rq[j] = q - kq[j] * win;
      acc[j] = 0.f;
    }
#pragma unroll 2
    for (int h = 0; h < wout; ++h) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float gr = gs_s[kq[j] * wout + h];
        if (fabsf(gr) > 0.f) acc[j] += nan0(gr * ws_s[h * (win + 1) + rq[j]]);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (q0 + 256 * j < np) p_s[q0 + 256 * j] = acc[j];
  }
  __syncthreads();
  const float *ob = o + bv * (size_t)inputs;
  float *igb = ig + bv * (size_t)inputs;
  for (int i = threadIdx.x; i < inputs; i += 256) {
    const int start = i < win ? 0 : (i - win) / step + 1;
    const int stop = min(i / step + 1, n_win);
    float sum = 0.f;
    for (int k = start; k < stop; ++k) sum += p_s[k * win + i - k * step];
    igb[i] = deactivate(sum, ob[i], act);
  }
}

// Non-overlapping windows (step == window_in, input fully tiled): one GEMM per
// variable, rows (sample, window), columns window offset, k output channel.
struct CDLoadG {
  const float *g;
  int n_win, wout, outputs, var;
  __device__ __forceinline__ float operator()(int m, int h, int v) const {
    int b = m / n_win, k = m - b * n_win;
    return nan0(g[((size_t)b * var + v) * outputs + (size_t)k * wout + h]);
  }
};
struct CDLoadW {  // B(h, r) = W[v][h][r]
  const float *w;
  int win, wout;
  __device__ __forceinline__ float operator()(int h, int r, int v) const {
    return nan0(w[((size_t)v * wout + h) * (win + 1) + r]);
  }
};
struct CDEpi {
  const float *o;
  float *ig;
  int n_win, win, inputs, var, act;
  __device__ __forceinline__ void operator()(int m, int r, int v, int, float acc) const {
    int b = m / n_win, k = m - b * n_win;
    size_t idx = ((size_t)b * var + v) * inputs + (size_t)k * win + r;
    ig[idx] = deactivate(acc, o[idx], act);
  }
  __device__ __forceinline__ long long row(int m, int v, int) const {
    int b = m / n_win, k = m - b * n_win;
    return ((long long)b * var + v) * inputs + (long long)k * win;
  }
  __device__ __forceinline__ float col(int, int) const { return 0.f; }
  template <int R>
  __device__ __forceinline__ void put_rows(const long long (&rb)[R], int r, const float (&v)[R], float,
                                           unsigned mask) const {
    float y[R];
#pragma unroll
    for (int j = 0; j < R; ++j) y[j] = (mask >> j & 1u) ? o[rb[j] + r] : 0.f;
    act_dispatch(act, [&](auto A) {
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (mask >> j & 1u) ig[rb[j] + r] = deactivate(v[j], y[j], decltype(A)::value);
    });
  }
  __host__ __device__ bool aligned4() const {
    return inputs % 4 == 0 && win % 4 == 0 && ((uintptr_t)o & 15) == 0 && ((uintptr_t)ig & 15) == 0;
  }
  __device__ __forceinline__ float4 col4(int, int) const { return make_float4(0.f, 0.f, 0.f, 0.f); }
  template <int R>
  __device__ __forceinline__ void put_rows4(const long long (&rb)[R], int r, const float4 (&v)[R], float4,
                                            unsigned mask) const {
    float4 y[R];
#pragma unroll
    for (int j = 0; j < R; ++j)
      y[j] = (mask >> j & 1u) ? *reinterpret_cast<const float4 *>(o + rb[j] + r) : make_float4(0.f, 0.f, 0.f, 0.f);
    act_dispatch(act, [&](auto A) {
      constexpr int a = decltype(A)::value;
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (mask >> j & 1u)
          *reinterpret_cast<float4 *>(ig + rb[j] + r) =
              make_float4(deactivate(v[j].x, y[j].x, a), deactivate(v[j].y, y[j].y, a),
                          deactivate(v[j].z, y[j].z, a), deactivate(v[j].w, y[j].w, a));
    });
  }
};

// CDEpi (one variable, rows of `win` inputs) with the input gradient written by TMA stores and the
// activation output read as the aux tensor (checked with tma_store_ok).
struct CDEpiTma : CDEpi {
  static constexpr bool kTmaStore = true, kAux = true;
  template <class F>
  __device__ __forceinline__ void transform(F &&f) const {
    act_dispatch(act, [&](auto A) { f([](float x, float, float y) { return deactivate(x, y, decltype(A)::value); }); });
  }
  __device__ __forceinline__ int zc(int z, int) const { return z; }
  __device__ __forceinline__ float4 aux4(int m, int, int n) const {
    return *reinterpret_cast<const float4 *>(o + (size_t)m * win + n);
  }
  bool out_map(CUtensorMap *tm, int M, int N, int nz) const { return make_tmap(tm, ig, win, 0, N, M, nz, 32, false); }
};

static int k_calc_hidden_gradient_conv(Launch &L) {
  const int inputs = (int)L.nd.g[0];
  const int var = L.nd.dims > 1 ? (int)L.nd.g[1] : 1;
  const int outputs = L.i(4), step = L.i(5), win = L.i(6), wout = L.i(7), act = L.i(8), shift_out = L.i(9);
  if (outputs < 0 || step <= 0 || win < 0 || wout <= 0 || shift_out < 0)
    return L.fail(NN_ERR_ARG, "CalcHiddenGradientConv: bad shape");
  if (L.B > 1 && shift_out != 0) return L.fail(NN_ERR_UNSUPPORTED, "CalcHiddenGradientConv: shift_out with batch");
  float *w = L.buf(0, (size_t)var * wout * (win + 1));
  float *g = L.buf(1, (size_t)shift_out + (size_t)L.B * var * outputs);
  float *o = L.buf(2, (size_t)L.B * var * inputs);
  float *ig = L.buf(3, (size_t)L.B * var * inputs);
  if (!w || !g || !o || !ig) return NN_ERR_BOUNDS;
  const int n_win = outputs / wout;
  if (step == win && shift_out == 0 && outputs == n_win * wout && inputs == n_win * win && win > 0) {
    cudaError_t e;
    if (var == 1) {
      FastShape fs{L.B * n_win, win, wout, 1, 1, 0, g, wout, 0, w, win + 1, 0};
      if (tma_store_ok(ig, win, 0, 1, win) && ((uintptr_t)o & 15) == 0)
        e = gemm_f32_wb<false, true>(L, fs, CDEpiTma{{o, ig, n_win, win, inputs, var, act}});
      else
        e = gemm_f32_wb<false, true>(L, fs, CDEpi{o, ig, n_win, win, inputs, var, act});
    } else {
      GemmShape sh{L.B * n_win, win, wout, var, 1};
      e = gemm_simt<true, true>(sh, CDLoadG{g, n_win, wout, outputs, var}, CDLoadW{w, win, wout},
                                CDEpi{o, ig, n_win, win, inputs, var, act}, L.stream);
    }
    if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
    L.counted();
    return NN_OK;
  }
  const size_t smem = ((size_t)n_win * wout + (size_t)wout * (win + 1) + (size_t)n_win * win) * sizeof(float);
  if (win > 0 && n_win > 0 && smem <= 48 * 1024 && (size_t)L.B * var <= 0x7fffffffu) {
    NN_LAUNCH_PDL(L, conv_dgrad_overlap_kernel, (unsigned)((size_t)L.B * var), 256, smem, L.stream, w, g, o, ig,
                  inputs, var, outputs, step, win, wout, act, shift_out);
    return NN_OK;
  }
  size_t total = (size_t)L.B * var * inputs;
  conv_dgrad_direct_kernel<<<grid1d(total, 256), 256, 0, L.stream>>>(w, g, o, ig, inputs, var, outputs, step, win,
                                                                      wout, act, shift_out, L.B);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

// ---------------------------------------------------- UpdateWeightsConvAdam
// NeuroNet.cl:1053-1098.  Weight (v, o, k): grad = sum_t g[v*total*wout + t*wout + o] *
// x[v*inputs + t*step + k] (x = 1 for the bias column k == window_in), with
// total = (inputs-(window_in-step)+(step-1))/step and the loop stopping, for
// k < window_in, at the first t with k + t*window_in >= inputs.  Batched: the
// mean over samples, then clamp and the reference Adam step (no eps, no l1/l2).
struct CWLoadG {  // A(m=o, kk=(b,t))
  const float *g;
  int total, wout;
  size_t gstride;  // floats per sample
  __device__ __forceinline__ float operator()(int o, int kk, int v) const {
    int b = kk / total, t = kk - b * total;
    return nan0(g[(size_t)b * gstride + ((size_t)v * total + t) * wout + o]);
  }
};
struct CWLoadX {  // B(kk=(b,t), n=k)
  const float *x;
  int total, inputs, step, win, var;
  __device__ __forceinline__ float operator()(int kk, int n, int v) const {
    if (n == win) return 1.f;
    int b = kk / total, t = kk - b * total;
    if (n + t * win >= inputs) return 0.f;  // the reference's loop exit (uses window_in, not step)
    return nan0(x[((size_t)b * var + v) * inputs + n + (size_t)t * step]);
  }
};

// UpdateWeightsConvAdam arithmetic for one weight, given its (batch-mean) gradient before clamping.
__device__ __forceinline__ void adam_conv_step(float *w, float *m, float *v, size_t i, float graw, float l, float b1,
                                               float b2) {
  float grad = clampf(nan0(graw), -kMaxGrad, kMaxGrad);
  float mt = nan0(b1 * m[i] + (1.f - b1) * grad);
  float vt = nan0(b2 * v[i] + (1.f - b2) * (grad * grad), 1.f);
  float weight = nan0(w[i] + nan0(l * mt / sqrtf(vt)));
  w[i] = weight;
  m[i] = mt;
  v[i] = vt;
}

__global__ void adam_conv_apply_kernel(float *w, float *m, float *v, GradSrc G, size_t n, float l, float b1,
                                       float b2) {
  pdl_wait();
  pdl_trigger();
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  adam_conv_step(w, m, v, i, G(i), l, b1, b2);
}

// The same when the gradient is a sum of many split-K partials: block (32 weights, 8 split
// groups), each thread summing every 8th partial of one weight (a warp reads 128 contiguous bytes
// per partial), then a shared-memory reduction and the update by the first group.
__global__ void adam_conv_apply_split_kernel(float *w, float *m, float *v, GradSrc G, size_t n, float l, float b1,
                                             float b2) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[8][33];
  const size_t i = blockIdx.x * (size_t)32 + threadIdx.x;
  float s = 0.f;
  if (i < n) {
    const size_t ga = G.at(i);
#pragma unroll 4
    for (int k = threadIdx.y; k < G.splits; k += 8) s += G.p[k * G.stride + ga];
  }
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y != 0 || i >= n) return;
  float t = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) t += red[j][threadIdx.x];
  adam_conv_step(w, m, v, i, t * G.scale, l, b1, b2);
}

struct ConvUpdShape {
  int nw, var, inputs, win, wout, step, total;
  size_t need_x;   // floats of x per sample read by the loops
  size_t gstride;  // floats of gradient per sample: var * units * wout
};
static int conv_upd_shape(Launch &L, int inputs_idx, int win_idx, int wout_idx, int step_idx, bool adam,
                          ConvUpdShape *s) {
  s->nw = (int)L.nd.g[0];
  s->inputs = L.i(inputs_idx);
  s->win = L.i(win_idx);
  s->wout = L.i(wout_idx);
  s->step = L.i(step_idx);
  if (s->win < 0 || s->wout <= 0 || s->step <= 0 || s->inputs < 0) return L.fail(NN_ERR_ARG, "conv update: bad shape");
  int per_var = s->wout * (s->win + 1);
  if (s->nw % per_var != 0) return L.fail(NN_ERR_ARG, "conv update: weight count not a multiple of wout*(win+1)");
  s->var = s->nw / per_var;
  s->total = adam ? (s->inputs - (s->win - s->step) + (s->step - 1)) / s->step
                  : (s->inputs - s->win + s->step - 1) / s->step;
  if (s->total < 0) s->total = 0;
  // largest x position the gradient loops read, per variable
  long long maxpos = -1;
  for (int k = 0; k < s->win; ++k) {
    long long tend = s->inputs > k ? ((long long)s->inputs - k + s->win - 1) / s->win : 0;
    if (tend > s->total) tend = s->total;
    if (tend > 0) maxpos = std::max(maxpos, (long long)k + (tend - 1) * s->step);
  }
  s->need_x = (size_t)std::max(maxpos + 1, (long long)s->inputs);
  // A batch holds one layer gradient [var][units][wout] per sample, with units the
  // number of complete windows (inputs - window_in) / step + 1.
  int units = s->inputs >= s->win ? (s->inputs - s->win) / s->step + 1 : 1;
  s->gstride = (size_t)s->var * units * s->wout;
  return NN_OK;
}

static int adam_conv_apply_src(const Launch &Lc, GradSrc G) {
  Launch &L = const_cast<Launch &>(Lc);
  size_t n = L.nd.g[0];
  float *w = L.buf(0, n), *m = L.buf(3, n), *v = L.buf(4, n);
  if (!w || !m || !v) return NN_ERR_BOUNDS;
  if (G.splits > 4)
    NN_LAUNCH_PDL(L, adam_conv_apply_split_kernel, (unsigned)((n + 31) / 32), dim3(32, 8), 0, L.stream, w, m, v, G, n,
                  L.f(6), L.f(7), L.f(8));
  else
    NN_LAUNCH_PDL(L, adam_conv_apply_kernel, grid1d(n, 256), 256, 0, L.stream, w, m, v, G, n, L.f(6), L.f(7), L.f(8));
  if (L.norm_rows > 0) {
    // the NormalizeWeights the runner folded into this update: a reduction over many split-K partials
    // keeps every weight its own thread, so the rows are normalised by the usual kernel afterwards
    NN_LAUNCH_PDL(L, normalize_weights_kernel, ceil_div((size_t)L.norm_rows * 32, 256), 256, 0, L.stream, w, L.norm_rows, L.norm_dim);
  }
  return NN_OK;
}
static int adam_conv_apply(const Launch &L, const float *grad) {
  return adam_conv_apply_src(L, GradSrc{grad, 1, 0, 1.f});
}

static int k_update_weights_conv_adam(Launch &L) {
  ConvUpdShape s;
  int rc = conv_upd_shape(L, 5, 9, 10, 11, true, &s);
  if (rc) return rc;
  float *w = L.buf(0, s.nw), *m = L.buf(3, s.nw), *v = L.buf(4, s.nw);
  float *g = L.buf(1, (size_t)(L.B - 1) * s.gstride + (size_t)s.var * s.total * s.wout);
  float *x = L.buf(2, (size_t)(L.B * s.var - 1) * s.inputs + s.need_x);
  if (!w || !m || !v || !g || !x) return NN_ERR_BOUNDS;
  GradSrc src;
  if (s.total == 0 || L.B * s.total == 0) {
    float *z = L.scratch(0, s.nw);
    if (!z) return NN_ERR_CUDA;
    cudaMemsetAsync(z, 0, (size_t)s.nw * sizeof(float), L.stream);
    src = GradSrc{z, 1, 0, 1.f};
  } else if (s.var == 1 && s.step == s.win && s.inputs == s.total * s.win && s.win > 0) {
    // windows tile the input: G = g^T [rows][wout] x X [rows][win], bias = column sums of g
    rc = wgrad_fast(L, g, s.wout, x, s.win, s.wout, s.win, L.B * s.total, &src);
    if (rc) return rc;
    src.scale = 1.f / (float)L.B;
  } else {
    rc = wgrad_partials<false, true>(L, s.wout, s.win + 1, L.B * s.total, s.var,
                                     CWLoadG{g, s.total, s.wout, s.gstride},
                                     CWLoadX{x, s.total, s.inputs, s.step, s.win, s.var}, &src);
    if (rc) return rc;
    src.scale = 1.f / (float)L.B;
  }
  return finish_update(L, src, (size_t)s.nw, adam_conv_apply, adam_conv_apply_src);
}

// ------------------------------------------------ UpdateWeightsConvMomentum
// NeuroNet.cl:996-1043 (with its shift_out = i/(window_in+1) - v indexing and
// total = (inputs-window_in+step-1)/step).  One thread per weight; batched:
// the per-sample sums are averaged.
__global__ void momentum_conv_grad_kernel(float *gout, const float *g, const float *x, int nw, int inputs, int win,
                                          int wout, int step, int total, int var, int B, size_t gstride) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nw) return;
  int v = i / ((win + 1) * wout);
  int shift = i % (win + 1);
  int shift_out = i / (win + 1) - v;
  float acc = 0.f;
  for (int b = 0; b < B; ++b) {
    const float *gs = g + (size_t)b * gstride + (size_t)v * total * wout;
    const float *xs = x + (size_t)b * var * inputs + (size_t)v * inputs;
    float grad = 0.f;
    for (int t = 0; t < total; ++t) {
      if (shift != win && (shift + t * win) >= inputs) break;
      grad += nan0(gs[t * wout + shift_out] * (shift == win ? 1.f : xs[shift + t * step]));
    }
    acc += grad;
  }
  gout[i] = acc / (float)B;
}

__global__ void momentum_conv_apply_kernel(float *w, float *dw, const float *grad, int n, float lr, float mom) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float delta = nan0(lr * grad[i]) + mom * dw[i];
  if (!isnan(delta)) {
    dw[i] = delta;
    if (fabsf(delta) > 0.f) w[i] = nan0(w[i] + delta);
  }
}

static int momentum_conv_apply(const Launch &Lc, const float *grad) {
  Launch &L = const_cast<Launch &>(Lc);
  int n = (int)L.nd.g[0];
  float *w = L.buf(0, n), *dw = L.buf(3, n);
  if (!w || !dw) return NN_ERR_BOUNDS;
  momentum_conv_apply_kernel<<<grid1d(n, 256), 256, 0, L.stream>>>(w, dw, grad, n, L.f(5), L.f(6));
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

static int k_update_weights_conv_momentum(Launch &L) {
  ConvUpdShape s;
  int rc = conv_upd_shape(L, 4, 7, 8, 9, false, &s);
  if (rc) return rc;
  // largest gradient index of the reference formula (ignoring early loop exits)
  size_t need_g = 0;
  if (s.total > 0) {
    long long v = s.var - 1;
    long long mx = (long long)(s.total - 1) * s.wout + (v + 1) * s.wout - 1 - v + v * (long long)s.total * s.wout;
    need_g = (size_t)(mx + 1);
  }
  float *w = L.buf(0, s.nw), *dw = L.buf(3, s.nw);
  float *g = L.buf(1, (size_t)(L.B - 1) * s.gstride + need_g);
  float *x = L.buf(2, (size_t)(L.B * s.var - 1) * s.inputs + s.need_x);
  if (!w || !dw || !g || !x) return NN_ERR_BOUNDS;
  float *grad = L.deferred() ? L.grad_slot(s.nw) : L.scratch(1, s.nw);
  if (!grad) return NN_ERR_BOUNDS;
  momentum_conv_grad_kernel<<<grid1d(s.nw, 256), 256, 0, L.stream>>>(grad, g, x, s.nw, s.inputs, s.win, s.wout,
                                                                      s.step, s.total, s.var, L.B, s.gstride);
  NN_CHECK_LAUNCH(L);
  if (L.deferred()) {
    L.defer(momentum_conv_apply, grad);
    return NN_OK;
  }
  return momentum_conv_apply(L, grad);
}

// UpdateWeightsConvAdamMini (NeuroNet.cl:7615-7731), one sample: global (window_in+1, window_out,
// variables), local (window_in+1, window_out_h, 1).  Per weight, the gradient over
// total = (inputs - window_in + step - 1) / step units, stopping once i + t*window_in >= inputs (the
// reference's test), non-finite terms skipped.
__global__ void conv_adam_mini_grad_kernel(const float *__restrict__ g, const float *__restrict__ x,
                                           float *__restrict__ G, int inputs, int win, int wout, int variables,
                                           int step, int total) {
  const size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)variables * wout * (win + 1)) return;
  const int i = (int)(t % (win + 1));
  const size_t r = t / (win + 1);
  const int f = (int)(r % wout), v = (int)(r / wout);
  const float *gv = g + (size_t)v * total * wout + f;
  const float *xv = x + (size_t)v * inputs;
  float acc = 0.f;
  for (int tt = 0; tt < total; ++tt) {
    if (i != win && i + tt * win >= inputs) break;
    const float gt = gv[(size_t)tt * wout] * (i == win ? 1.f : xv[i + tt * step]);
    if (isfinite(gt)) acc += gt;
  }
  G[t] = acc;
}

// One block per head (window_out_h rows).  The second moment is indexed by head only, so the
// reference's work-groups of different variables race on it; here the variables take their turns in
// order.  Each turn: the reference's slot reduction of grad^2 / (window_in * window_out_h) (rows
// outer, the bias column only when window_in % 64 != 0, the fold stopping one step early), the
// clamped second moment, then the head's weights: m clamped to +-1e5, w += l m / sqrt(v).
__global__ void conv_adam_mini_apply_kernel(float *w, float *m, float *vh, const float *__restrict__ G, int win,
                                            int wout, int wout_h, int variables, float l, float b1, float b2) {
  __shared__ float temp[64];
  __shared__ float vt_s;
  const int head = blockIdx.x, t = threadIdx.x;
  const int ls = min(64, win), counts = (win + ls - 1) / ls;
  const float den = (float)(win * wout_h);
  for (int v = 0; v < variables; ++v) {
    const float *Gh = G + ((size_t)v * wout + (size_t)head * wout_h) * (win + 1);
    if (t < ls) {
      float acc = 0.f;
      for (int h = 0; h < wout_h; ++h)
        for (int count = 0; count < counts; ++count) {
          const int i = count * ls + t;
          if (i > win) break;
          const float gv = Gh[(size_t)h * (win + 1) + i];
          const float term = isfinite(gv) ? gv * gv / den : 0.f;
          acc = ((count == 0 && h == 0) ? 0.f : acc) + term;
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
    if (t == 0) {
      float t0 = temp[0];
      if (!isfinite(t0)) t0 = 1.f;
      float vv = vh[head];
      if (!isfinite(vv)) vv = 1.f;
      t0 = fminf(fmaxf(b2 * vv + (1.f - b2) * t0, 1.0e-6f), 1.0e6f);
      vh[head] = t0;
      vt_s = t0;
    }
    __syncthreads();
    const float vt = vt_s;
    for (int e = t; e < wout_h * (win + 1); e += blockDim.x) {
      const size_t wi = ((size_t)v * wout + (size_t)head * wout_h + e / (win + 1)) * (win + 1) + e % (win + 1);
      float mt = fminf(fmaxf(b1 * m[wi] + (1.f - b1) * G[wi], -1.0e5f), 1.0e5f);
      if (!isfinite(mt)) mt = 0.f;
      const float wv = w[wi] + l * mt / sqrtf(vt);
      if (isfinite(wv)) w[wi] = wv;
      m[wi] = mt;
    }
    __syncthreads();  // temp and vt_s are rewritten by the next variable's turn
  }
}

static int k_update_weights_conv_adam_mini(Launch &L) {
  if (!L.nd.has_local || L.nd.dims < 2)
    return L.fail(NN_ERR_ARG, "UpdateWeightsConvAdamMini: needs global (window_in+1, window_out, variables) "
                              "and local (window_in+1, window_out_h, 1)");
  const int win = (int)L.nd.g[0] - 1, wout = (int)L.nd.g[1];
  const int variables = L.nd.dims > 2 ? (int)L.nd.g[2] : 1, wout_h = (int)L.nd.l[1];
  const int inputs = L.i(5), step = L.i(9);
  if (win < 1 || step < 1 || inputs < win || wout_h < 1 || wout % wout_h || (int)L.nd.l[0] != win + 1)
    return L.fail(NN_ERR_ARG, "UpdateWeightsConvAdamMini: bad window, step, inputs or head size");
  if (L.B != 1 || L.deferred())
    return L.fail(NN_ERR_UNSUPPORTED, "UpdateWeightsConvAdamMini: one sample per execution (the reference's "
                                      "per-head second moment has no batch-mean form here)");
  const int total = (inputs - win + step - 1) / step;
  const size_t nw = (size_t)variables * wout * (win + 1);
  float *w = L.buf(0, nw), *g = L.buf(1, (size_t)variables * total * wout), *x = L.buf(2, (size_t)variables * inputs);
  float *m = L.buf(3, nw), *v = L.buf(4, (size_t)(wout / wout_h));
  if (!w || !g || !x || !m || !v) return NN_ERR_BOUNDS;
  float *G = L.scratch(1, nw);
  if (!G) return NN_ERR_CUDA;
  conv_adam_mini_grad_kernel<<<grid1d(nw, 256), 256, 0, L.stream>>>(g, x, G, inputs, win, wout, variables, step,
                                                                   total);
  NN_CHECK_LAUNCH(L);
  conv_adam_mini_apply_kernel<<<wout / wout_h, 256, 0, L.stream>>>(w, m, v, G, win, wout, wout_h, variables,
                                                                   L.f(6), L.f(7), L.f(8));
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

const KernelDef kConvKernels[] = {
    {"UpdateWeightsConvAdamMini", "pppppifffi", k_update_weights_conv_adam_mini, false},
    {"FeedForwardConv", "pppiiiii", k_feedforward_conv, false},
    {"CalcHiddenGradientConv", "ppppiiiiii", k_calc_hidden_gradient_conv, false},
    {"UpdateWeightsConvAdam", "pppppifffiii", k_update_weights_conv_adam, false},
    {"UpdateWeightsConvMomentum", "ppppiffiii", k_update_weights_conv_momentum, false},
};
const int kNumConvKernels = sizeof(kConvKernels) / sizeof(kConvKernels[0]);

}  // namespace nn
