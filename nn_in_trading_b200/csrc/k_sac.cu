// Concatenate input layer and the soft actor-critic step.
//
// CNeuronConcatenate (NeuroNet_Misc.mqh:286-680) feeds a layer from two inputs at once, the previous
// layer's output x1 and a second buffer x2 (a critic's state and action):
//   Concat_FeedForward           y[i] = act(W[i] . [x1; x2; 1])          NeuroNet.cl:3628-3718
//   Concat_HiddenGradient        ig = Deact(W^T g) into the x1 and x2 gradients   NeuroNet.cl:3724-3785
//   Concat_UpdateWeightsMomentum / Concat_UpdateWeightsAdam              NeuroNet.cl:3790-3862
// W is [outputs][inputs1 + inputs2 + 1], the bias last.  Batches follow the library's contract:
// forward and input gradients per sample, the weight gradient the batch mean of g_b [x1; x2; 1]_b,
// then the reference's update arithmetic once (no gradient clamp in the Concat updates).
//
// Kernels of this library with no reference counterpart, for a squashed-Gaussian soft actor-critic
// update built from the kernels above (the reference trains its SAC agents through quantile heads):
//   SACGaussianPolicy   a = tanh(mu + exp(clamp(log_std)) eps) and log pi(a) per sample
//   SACTargetValue      y = r + gamma (1 - done) (min(q1, q2) - alpha log pi)
//   SACPolicyGradient   gradient of min(q1, q2) - alpha log pi with respect to mu and log_std
// A launch covers global[0] * batch samples.
#include "../../include/nn_b200.h"
#include "gemm_fast.cuh"
#include "nn_device.cuh"
#include "nn_internal.h"
#include "tc_gemm.cuh"
#include "wgrad.cuh"
#include "epi_dense.cuh"

namespace nn {

// ------------------------------------------------------ Concat_FeedForward
// Small batches: one warp per (sample, output row); lanes take the float4 groups of both inputs, a
// group whose sum is NaN is skipped (the reference skips a group that makes its running sum NaN),
// the bias is added unchecked and a NaN total becomes 0.
__global__ void concat_ff_rows_kernel(const float *__restrict__ w, const float *__restrict__ x1,
                                      const float *__restrict__ x2, float *__restrict__ y, int in1, int in2,
                                      int outputs, int B, int act) {
  pdl_wait();
  pdl_trigger();
  const int warp = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (warp >= outputs * B) return;
  const int b = warp / outputs, i = warp % outputs;
  const float *row = w + (size_t)i * (in1 + in2 + 1);
  const float *a = x1 + (size_t)b * in1, *c = x2 + (size_t)b * in2;
  const int g1 = (in1 + 3) / 4, g2 = (in2 + 3) / 4;
  float s = 0.f;
  for (int g = lane; g < g1 + g2; g += 32) {
    const bool first = g < g1;
    const float *x = first ? a : c;
    const float *wr = first ? row : row + in1;
    const int n = first ? in1 : in2, k = (first ? g : g - g1) * 4;
    float d = 0.f;
    for (int u = 0; u < 4 && k + u < n; ++u) d += x[k + u] * wr[k + u];
    if (!isnan(d)) s += d;
  }
  s = warp_sum(s);
  if (lane == 0) {
    s += row[in1 + in2];
    if (isnan(s)) s = 0.f;
    y[(size_t)b * outputs + i] = activate(s, act);
  }
}

// [x1 | x2] per sample, the operand of the batched products, in rows of ldp = inputs1 + inputs2
// rounded up to 4 floats (16-byte rows that TMA can address; the padding columns are zero)
__host__ __device__ __forceinline__ int concat_ldp(int in1, int in2) { return (in1 + in2 + 3) & ~3; }
__global__ void concat_pack_kernel(const float *__restrict__ x1, const float *__restrict__ x2, float *__restrict__ p,
                                   int in1, int in2, int B) {
  pdl_wait();
  pdl_trigger();
  const int ldp = concat_ldp(in1, in2);
  const size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)B * ldp) return;
  const size_t b = t / ldp;
  const int j = (int)(t % ldp);
  p[t] = j < in1 ? x1[b * in1 + j] : (j - in1 < in2 ? x2[b * in2 + (j - in1)] : 0.f);
}

// Batched forward epilogue: y[m][n] = act(acc + W[n][K]), a NaN pre-activation -> 0.
struct ConcatEpi {
  const float *w;
  float *y;
  int ld, K, outputs, act;
  __device__ __forceinline__ float fin(float v, float bias) const {
    v += bias;
    return isnan(v) ? 0.f : v;
  }
  __device__ __forceinline__ void operator()(int m, int n, int, int, float acc) const {
    y[(size_t)m * outputs + n] = activate(fin(acc, w[(size_t)n * ld + K]), act);
  }
  __device__ __forceinline__ long long row(int m, int, int) const { return (long long)m * outputs; }
  __device__ __forceinline__ float col(int n, int) const { return w[(size_t)n * ld + K]; }
  template <int R>
  __device__ __forceinline__ void put_rows(const long long (&rb)[R], int n, const float (&v)[R], float bias,
                                           unsigned mask) const {
    act_dispatch(act, [&](auto A) {
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (mask >> j & 1u) y[rb[j] + n] = activate(fin(v[j], bias), decltype(A)::value);
    });
  }
  __host__ __device__ bool aligned4() const { return outputs % 4 == 0 && ((uintptr_t)y & 15) == 0; }
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
          *reinterpret_cast<float4 *>(y + rb[j] + n) =
              make_float4(activate(fin(v[j].x, b.x), a), activate(fin(v[j].y, b.y), a),
                          activate(fin(v[j].z, b.z), a), activate(fin(v[j].w, b.w), a));
    });
  }
};

static int k_concat_ff(Launch &L) {
  const int outputs = (int)L.nd.g[0];
  const int in1 = L.i(4), in2 = L.i(5), act = L.i(6);
  if (in1 < 0 || in2 < 0) return L.fail(NN_ERR_ARG, "Concat_FeedForward: negative input count");
  const int K = in1 + in2, ld = K + 1;
  float *w = L.buf(0, (size_t)outputs * ld);
  float *x1 = L.buf(1, (size_t)L.B * in1), *x2 = L.buf(2, (size_t)L.B * in2);
  float *y = L.buf(3, (size_t)L.B * outputs);
  if (!w || !x1 || !x2 || !y) return NN_ERR_BOUNDS;
  if (L.B <= 4) {
    NN_LAUNCH_PDL(L, concat_ff_rows_kernel, ceil_div((size_t)outputs * L.B * 32, 256), 256, 0, L.stream, w, x1, x2, y, in1, in2, outputs, L.B, act);
    return NN_OK;
  }
  const int ldp = concat_ldp(in1, in2);
  float *p = L.scratch(2, (size_t)L.B * ldp);
  if (!p) return NN_ERR_CUDA;
  NN_LAUNCH_PDL(L, concat_pack_kernel, grid1d((size_t)L.B * ldp, 256), 256, 0, L.stream, x1, x2, p, in1, in2, L.B);
  FastShape fs{L.B, outputs, K, 1, 1, 0, p, ldp, 0, w, ld, 0};
  cudaError_t e = gemm_f32_wb<false, false>(L, fs, ConcatEpi{w, y, ld, K, outputs, act});
  if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
  L.counted();
  return NN_OK;
}

// --------------------------------------------------- Concat_HiddenGradient
// Small batches: CTA of 16 warps per 32 input columns; warps split the outputs k.  The sum has no
// per-term check; a NaN sum becomes 0 before the derivative.
constexpr int kCatWarps = 16;
template <int MAXB>
__global__ void __launch_bounds__(kCatWarps * 32)
    concat_hg_cols_kernel(const float *__restrict__ w, const float *__restrict__ g, const float *__restrict__ o1,
                          const float *__restrict__ o2, float *__restrict__ ig1, float *__restrict__ ig2, int outputs,
                          int in1, int in2, int B, int act1, int act2) {
  pdl_wait();
  pdl_trigger();
  __shared__ float part[kCatWarps][MAXB][33];
  const int K = in1 + in2;
  const int col = blockIdx.x * 32 + (threadIdx.x & 31), wv = threadIdx.x >> 5;
  float s[MAXB];
#pragma unroll
  for (int b = 0; b < MAXB; ++b) s[b] = 0.f;
  if (col < K)
    for (int k = wv; k < outputs; k += kCatWarps) {
      const float wk = w[(size_t)k * (K + 1) + col];
#pragma unroll
      for (int b = 0; b < MAXB; ++b)
        if (b < B) s[b] += wk * g[(size_t)b * outputs + k];
    }
#pragma unroll
  for (int b = 0; b < MAXB; ++b) part[wv][b][threadIdx.x & 31] = s[b];
  __syncthreads();
  if (wv >= MAXB || wv >= B || col >= K) return;
  float t = 0.f;
#pragma unroll
  for (int r = 0; r < kCatWarps; ++r) t += part[r][wv][threadIdx.x & 31];
  if (isnan(t)) t = 0.f;
  const int b = wv;
  if (col < in1)
    ig1[(size_t)b * in1 + col] = deactivate(t, o1[(size_t)b * in1 + col], act1);
  else
    ig2[(size_t)b * in2 + col - in1] = deactivate(t, o2[(size_t)b * in2 + col - in1], act2);
}

// Batched epilogue: column n < in1 goes to ig1 with act1, the others to ig2 with act2.
struct ConcatHGEpi {
  const float *o1, *o2;
  float *ig1, *ig2;
  int in1, in2, act1, act2;
  __device__ __forceinline__ void put(int m, int n, float acc) const {
    const float s = isnan(acc) ? 0.f : acc;
    if (n < in1) {
      const size_t i = (size_t)m * in1 + n;
      ig1[i] = deactivate(s, o1[i], act1);
    } else {
      const size_t i = (size_t)m * in2 + (n - in1);
      ig2[i] = deactivate(s, o2[i], act2);
    }
  }
  __device__ __forceinline__ void operator()(int m, int n, int, int, float acc) const { put(m, n, acc); }
  __device__ __forceinline__ long long row(int m, int, int) const { return m; }
  __device__ __forceinline__ float col(int, int) const { return 0.f; }
  template <int R>
  __device__ __forceinline__ void put_rows(const long long (&rb)[R], int n, const float (&v)[R], float,
                                           unsigned mask) const {
#pragma unroll
    for (int j = 0; j < R; ++j)
      if (mask >> j & 1u) put((int)rb[j], n, v[j]);
  }
  __host__ __device__ bool aligned4() const { return false; }
  __device__ __forceinline__ float4 col4(int, int) const { return make_float4(0.f, 0.f, 0.f, 0.f); }
  template <int R>
  __device__ __forceinline__ void put_rows4(const long long (&rb)[R], int n, const float4 (&v)[R], float4,
                                            unsigned mask) const {}
};

// Batched gradient of a short second input (inputs2 <= kCatShort): one warp per sample, lanes
// striding the outputs k, one partial sum per second input, NaN sum -> 0, then the derivative.
constexpr int kCatShort = 16;
__global__ void concat_hg_second_kernel(const float *__restrict__ w, const float *__restrict__ g,
                                        const float *__restrict__ o2, float *__restrict__ ig2, int outputs, int in1,
                                        int in2, int B, int act2) {
  pdl_wait();
  pdl_trigger();
  const int b = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
  if (b >= B) return;
  const int ld = in1 + in2 + 1;
  const float *gb = g + (size_t)b * outputs;
  float s[kCatShort];
#pragma unroll
  for (int j = 0; j < kCatShort; ++j) s[j] = 0.f;
#pragma unroll 4
  for (int k = lane; k < outputs; k += 32) {
    const float gk = gb[k];
    const float *wr = w + (size_t)k * ld + in1;
#pragma unroll
    for (int j = 0; j < kCatShort; ++j)
      if (j < in2) s[j] += wr[j] * gk;
  }
#pragma unroll
  for (int j = 0; j < kCatShort; ++j) {
    if (j >= in2) break;
    float t = warp_sum(s[j]);
    if (isnan(t)) t = 0.f;
    if (lane == 0) ig2[(size_t)b * in2 + j] = deactivate(t, o2[(size_t)b * in2 + j], act2);
  }
}

static int k_concat_hg(Launch &L) {
  const int outputs = L.i(6), in1 = L.i(7), in2 = L.i(8), act1 = L.i(9), act2 = L.i(10);
  if (outputs < 0 || in1 < 0 || in2 < 0) return L.fail(NN_ERR_ARG, "Concat_HiddenGradient: negative size");
  const int K = in1 + in2;
  if ((int)L.nd.g[0] < K) return L.fail(NN_ERR_UNSUPPORTED, "Concat_HiddenGradient: global size below inputs1+inputs2");
  float *w = L.buf(0, (size_t)outputs * (K + 1)), *g = L.buf(1, (size_t)L.B * outputs);
  float *o1 = L.buf(2, (size_t)L.B * in1), *o2 = L.buf(3, (size_t)L.B * in2);
  float *ig1 = L.buf(4, (size_t)L.B * in1), *ig2 = L.buf(5, (size_t)L.B * in2);
  if (!w || !g || !o1 || !o2 || !ig1 || !ig2) return NN_ERR_BOUNDS;
  if (L.B <= 4) {
    NN_LAUNCH_PDL(L, concat_hg_cols_kernel<4>, ceil_div(K, 32), kCatWarps * 32, 0, L.stream, w, g, o1, o2, ig1, ig2, outputs, in1, in2, L.B, act1, act2);
    return NN_OK;
  }
  if (in2 <= kCatShort && in1 > 0 && tma_store_ok(ig1, in1, 0, 1, in1) && ((uintptr_t)o1 & 15) == 0) {
    // the first input's gradient as the dense hidden-gradient product (TMA-store epilogue with the
    // activation output as its second input), the short second input by one warp per sample
    FastShape f1{L.B, in1, outputs, 1, 1, 0, g, outputs, 0, w, K + 1, 0};
    cudaError_t e = gemm_f32_wb<false, true>(L, f1, CHGEpiTma{{o1, ig1, in1, act1}});
    if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
    L.counted();
    if (in2 > 0) {
      NN_LAUNCH_PDL(L, concat_hg_second_kernel, ceil_div((size_t)L.B * 32, 256), 256, 0, L.stream, w, g, o2, ig2, outputs, in1, in2, L.B, act2);
    }
    return NN_OK;
  }
  FastShape fs{L.B, K, outputs, 1, 1, 0, g, outputs, 0, w, K + 1, 0};
  cudaError_t e = gemm_f32_wb<false, true>(L, fs, ConcatHGEpi{o1, o2, ig1, ig2, in1, in2, act1, act2});
  if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
  L.counted();
  return NN_OK;
}

// ------------------------------------------------------------ updates
// Weight (i, j) of a row of ld = inputs1 + inputs2 + 1 floats, input [x1; x2; 1][j].
__device__ __forceinline__ float concat_input(const float *x1, const float *x2, int in1, int in2, int j) {
  return j < in1 ? x1[j] : (j - in1 < in2 ? x2[j - in1] : 1.f);
}

// NeuroNet.cl:3849-3861: no clamp, no NaN guards, the weight moves only when |delta| > 0.
__device__ __forceinline__ void concat_adam_step(float *w, float *m, float *v, size_t wi, float g, float l, float b1,
                                                 float b2) {
  const float weight = w[wi];
  const float mt = b1 * m[wi] + (1.f - b1) * g;
  const float vt = b2 * v[wi] + (1.f - b2) * (g * g);
  const float delta = l * (mt / (sqrtf(vt) + 1.0e-37f) - (kL1 * signf(weight) + kL2 * weight));
  if (fabsf(delta) > 0.f) w[wi] = weight + delta;
  m[wi] = mt;
  v[wi] = vt;
}

// NeuroNet.cl:3806-3817: the delta is kept (and applied when non-zero) unless it is NaN.
__device__ __forceinline__ void concat_momentum_step(float *w, float *dw, size_t wi, float lr_g, float mom) {
  const float delta = lr_g + mom * dw[wi];
  if (!isnan(delta)) {
    dw[wi] = delta;
    if (fabsf(delta) > 0.f) w[wi] = w[wi] + delta;
  }
}

__global__ void concat_adam_fused_kernel(float *w, const float *g, const float *x1, const float *x2, float *m,
                                         float *v, int n_out, int n_col, int in1, int in2, float l, float b1,
                                         float b2) {
  pdl_wait();
  pdl_trigger();
  const size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)n_out * n_col) return;
  const int i = (int)(t / n_col), j = (int)(t % n_col);
  concat_adam_step(w, m, v, (size_t)i * (in1 + in2 + 1) + j, g[i] * concat_input(x1, x2, in1, in2, j), l, b1, b2);
}

__global__ void concat_momentum_fused_kernel(float *w, const float *g, const float *x1, const float *x2, float *dw,
                                             int n_out, int n_col, int in1, int in2, float lr, float mom) {
  pdl_wait();
  pdl_trigger();
  const size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)n_out * n_col) return;
  const int i = (int)(t / n_col), j = (int)(t % n_col);
  concat_momentum_step(w, dw, (size_t)i * (in1 + in2 + 1) + j, lr * g[i] * concat_input(x1, x2, in1, in2, j), mom);
}

// Apply kernels over a (batch-mean) gradient source: block of 32 weights x 8 split groups.
template <bool ADAM>
__global__ void concat_apply_kernel(float *w, float *m, float *v, GradSrc G, int n_out, int n_col, int ld, float a,
                                    float b1, float b2) {
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
  const size_t wi = (t / n_col) * (size_t)ld + t % n_col;
  if (ADAM)
    concat_adam_step(w, m, v, wi, sum * G.scale, a, b1, b2);
  else
    concat_momentum_step(w, m, wi, a * (sum * G.scale), b1);  // m = dw, a = lr, b1 = momentum
}

struct ConcatUpdShape {
  int n_out, n_col, in1, in2;
};
template <bool ADAM>
static ConcatUpdShape concat_upd_shape(const Launch &L) {
  // Adam: (w, g, x1, x2, m, v, in1, in2, l, b1, b2); momentum: (w, g, x1, x2, dw, in1, in2, lr, mom)
  return ConcatUpdShape{(int)L.nd.g[0], L.nd.dims > 1 ? (int)L.nd.g[1] : 1, L.i(ADAM ? 6 : 5), L.i(ADAM ? 7 : 6)};
}

template <bool ADAM>
static int concat_apply_src(const Launch &Lc, GradSrc G) {
  Launch &L = const_cast<Launch &>(Lc);
  const ConcatUpdShape s = concat_upd_shape<ADAM>(L);
  const int ld = s.in1 + s.in2 + 1;
  const size_t nw = (size_t)s.n_out * ld;
  float *w = L.buf(0, nw), *m = L.buf(4, nw), *v = ADAM ? L.buf(5, nw) : nullptr;
  if (!w || !m || (ADAM && !v)) return NN_ERR_BOUNDS;
  const size_t n = (size_t)s.n_out * s.n_col;
  if (ADAM)
    NN_LAUNCH_PDL(L, concat_apply_kernel<true>, (unsigned)((n + 31) / 32), dim3(32, 8), 0, L.stream, w, m, v, G,
                  s.n_out, s.n_col, ld, L.f(8), L.f(9), L.f(10));
  else
    NN_LAUNCH_PDL(L, concat_apply_kernel<false>, (unsigned)((n + 31) / 32), dim3(32, 8), 0, L.stream, w, m, nullptr, G, s.n_out, s.n_col, ld, L.f(7), L.f(8), 0.f);
  return NN_OK;
}
template <bool ADAM>
static int concat_apply(const Launch &L, const float *grad) {
  return concat_apply_src<ADAM>(L, GradSrc{grad, 1, 0, 1.f});
}

template <bool ADAM>
static int k_concat_update(Launch &L) {
  const char *name = ADAM ? "Concat_UpdateWeightsAdam" : "Concat_UpdateWeightsMomentum";
  const ConcatUpdShape s = concat_upd_shape<ADAM>(L);
  if (s.in1 < 0 || s.in2 < 0) return L.fail(NN_ERR_ARG, std::string(name) + ": negative input count");
  const int K = s.in1 + s.in2, ld = K + 1;
  if (s.n_col > ld) return L.fail(NN_ERR_ARG, std::string(name) + ": global size 1 above inputs1+inputs2+1");
  const size_t nw = (size_t)s.n_out * ld;
  float *w = L.buf(0, nw), *g = L.buf(1, (size_t)L.B * s.n_out);
  float *x1 = L.buf(2, (size_t)L.B * s.in1), *x2 = L.buf(3, (size_t)L.B * s.in2);
  float *m = L.buf(4, nw), *v = ADAM ? L.buf(5, nw) : nullptr;
  if (!w || !g || !x1 || !x2 || !m || (ADAM && !v)) return NN_ERR_BOUNDS;
  const size_t n = (size_t)s.n_out * s.n_col;
  if (L.B == 1 && !L.deferred()) {
    if (ADAM)
      NN_LAUNCH_PDL(L, concat_adam_fused_kernel, grid1d(n, 256), 256, 0, L.stream, w, g, x1, x2, m, v, s.n_out,
                    s.n_col, s.in1, s.in2, L.f(8), L.f(9), L.f(10));
    else
      NN_LAUNCH_PDL(L, concat_momentum_fused_kernel, grid1d(n, 256), 256, 0, L.stream, w, g, x1, x2, m, s.n_out, s.n_col, s.in1, s.in2, L.f(7), L.f(8));
    return NN_OK;
  }
  if (s.n_col != ld)
    return L.fail(NN_ERR_UNSUPPORTED, std::string(name) + ": a batched update covers whole rows (global size 1 = "
                                                          "inputs1+inputs2+1)");
  const int ldp = concat_ldp(s.in1, s.in2);
  float *p = L.scratch(2, (size_t)L.B * ldp);
  if (!p) return NN_ERR_CUDA;
  NN_LAUNCH_PDL(L, concat_pack_kernel, grid1d((size_t)L.B * ldp, 256), 256, 0, L.stream, x1, x2, p, s.in1, s.in2, L.B);
  GradSrc src;
  int rc = wgrad_fast(L, g, s.n_out, p, ldp, s.n_out, K, L.B, &src);
  if (rc) return rc;
  src.scale = 1.f / (float)L.B;
  return finish_update(L, src, n, concat_apply<ADAM>, concat_apply_src<ADAM>);
}

// ------------------------------------------------------ soft actor-critic
constexpr float kLogStdMin = -20.f, kLogStdMax = 2.f;
constexpr float kHalfLog2Pi = 0.91893853320467274f;
constexpr float kSquashEps = 1.0e-6f;

// outputs [n][2A] = (mu, log_std); noise [n][A]; actions [n][A]; log_probs [n]
__global__ void sac_policy_kernel(const float *__restrict__ out, const float *__restrict__ noise,
                                  float *__restrict__ actions, float *__restrict__ logp, int A, int n) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n) return;
  const float *o = out + (size_t)b * 2 * A;
  float lp = 0.f;
  for (int j = 0; j < A; ++j) {
    const float ls = clampf(o[A + j], kLogStdMin, kLogStdMax);
    const float e = noise[(size_t)b * A + j];
    const float a = tanhf(o[j] + expf(ls) * e);
    actions[(size_t)b * A + j] = a;
    lp += -0.5f * e * e - ls - kHalfLog2Pi - logf(1.f - a * a + kSquashEps);
  }
  logp[b] = lp;
}

static int k_sac_policy(Launch &L) {
  const int A = L.i(4);
  const int n = (int)L.nd.g[0] * L.B;
  if (A <= 0) return L.fail(NN_ERR_ARG, "SACGaussianPolicy: action_dim must be positive");
  float *out = L.buf(0, (size_t)n * 2 * A), *noise = L.buf(1, (size_t)n * A), *act = L.buf(2, (size_t)n * A);
  float *lp = L.buf(3, (size_t)n);
  if (!out || !noise || !act || !lp) return NN_ERR_BOUNDS;
  NN_LAUNCH_PDL(L, sac_policy_kernel, grid1d(n, 256), 256, 0, L.stream, out, noise, act, lp, A, n);
  return NN_OK;
}

__global__ void sac_target_kernel(const float *q1, const float *q2, const float *r, const float *done,
                                  const float *logp, float *y, int n, float gamma, float alpha) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= n) return;
  y[b] = r[b] + gamma * (1.f - done[b]) * (fminf(q1[b], q2[b]) - alpha * logp[b]);
}

static int k_sac_target(Launch &L) {
  const int n = (int)L.nd.g[0] * L.B;
  float *q1 = L.buf(0, n), *q2 = L.buf(1, n), *r = L.buf(2, n), *d = L.buf(3, n), *lp = L.buf(4, n);
  float *y = L.buf(5, n);
  if (!q1 || !q2 || !r || !d || !lp || !y) return NN_ERR_BOUNDS;
  NN_LAUNCH_PDL(L, sac_target_kernel, grid1d(n, 256), 256, 0, L.stream, q1, q2, r, d, lp, y, n, L.f(6), L.f(7));
  return NN_OK;
}

// Gradient (the library's ascent direction, clamped to +-MAX_GRAD like every output gradient) of
// J = min(q1, q2) - alpha log pi with respect to (mu, log_std), dq of the smaller critic:
//   s = dq (1 - a^2) - alpha 2a(1 - a^2)/(1 - a^2 + eps);  dJ/dmu = s;
//   dJ/dlog_std = s std eps + alpha inside the clamp range of log_std, else 0.
__global__ void sac_policy_grad_kernel(const float *__restrict__ out, const float *__restrict__ noise,
                                       const float *__restrict__ actions, const float *__restrict__ q1,
                                       const float *__restrict__ q2, const float *__restrict__ dq1,
                                       const float *__restrict__ dq2, float *__restrict__ grad, int A, int n,
                                       float alpha) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n * A) return;
  const int b = t / A, j = t % A;
  const float *dq = q1[b] <= q2[b] ? dq1 : dq2;
  const float a = actions[t], e = noise[t];
  const float ls_raw = out[(size_t)b * 2 * A + A + j];
  const float ls = clampf(ls_raw, kLogStdMin, kLogStdMax);
  const float one = 1.f - a * a;
  const float s = dq[t] * one - alpha * 2.f * a * one / (one + kSquashEps);
  grad[(size_t)b * 2 * A + j] = clampf(nan0(s), -kMaxGrad, kMaxGrad);
  const bool inside = ls_raw > kLogStdMin && ls_raw < kLogStdMax;
  grad[(size_t)b * 2 * A + A + j] = inside ? clampf(nan0(s * expf(ls) * e + alpha), -kMaxGrad, kMaxGrad) : 0.f;
}

static int k_sac_policy_grad(Launch &L) {
  const int A = L.i(8);
  const int n = (int)L.nd.g[0] * L.B;
  if (A <= 0) return L.fail(NN_ERR_ARG, "SACPolicyGradient: action_dim must be positive");
  float *out = L.buf(0, (size_t)n * 2 * A), *noise = L.buf(1, (size_t)n * A), *act = L.buf(2, (size_t)n * A);
  float *q1 = L.buf(3, n), *q2 = L.buf(4, n), *dq1 = L.buf(5, (size_t)n * A), *dq2 = L.buf(6, (size_t)n * A);
  float *grad = L.buf(7, (size_t)n * 2 * A);
  if (!out || !noise || !act || !q1 || !q2 || !dq1 || !dq2 || !grad) return NN_ERR_BOUNDS;
  NN_LAUNCH_PDL(L, sac_policy_grad_kernel, grid1d((size_t)n * A, 256), 256, 0, L.stream, out, noise, act, q1, q2, dq1, dq2, grad, A, n, L.f(9));
  return NN_OK;
}

const KernelDef kSacKernels[] = {
    {"Concat_FeedForward", "ppppiii", k_concat_ff, false},
    {"Concat_HiddenGradient", "ppppppiiiii", k_concat_hg, false},
    {"Concat_UpdateWeightsMomentum", "pppppiiff", k_concat_update<false>, false},
    {"Concat_UpdateWeightsAdam", "ppppppiifff", k_concat_update<true>, false},
    {"SACGaussianPolicy", "ppppi", k_sac_policy, false},
    {"SACTargetValue", "ppppppff", k_sac_target, false},
    {"SACPolicyGradient", "ppppppppif", k_sac_policy_grad, false},
};
const int kNumSacKernels = sizeof(kSacKernels) / sizeof(kSacKernels[0]);

}  // namespace nn
