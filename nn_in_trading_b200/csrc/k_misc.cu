// Batch-normalisation kernels (CNeuronBatchNormOCL path): BatchFeedForward,
// CalcHiddenGradientBatch, UpdateBatchOptionsAdam, UpdateBatchOptionsMomentum;
// and the RevIN de-normalisation kernels (CNeuronRevINDenormOCL path):
// RevInFeedForward, RevInHiddenGraddient, which read a batch-normalisation
// layer's options.  Options are [neuron][7] (SGD) or [neuron][9] (Adam):
// mean, variance, nx, gamma, beta, then the optimiser state of gamma and beta.
//
// Batched executions: the running statistics are a per-neuron recurrence over
// samples, so BatchFeedForward scans the batch in order, exactly as that many
// consecutive reference calls with the same `batch` argument would, and keeps
// every sample's (mean, variance, nx) in a side buffer attached to the options
// buffer.  CalcHiddenGradientBatch and the option updates read that history,
// so each sample's gradient uses the statistics of its own forward pass, and
// the gamma/beta update averages the per-sample gradients.
#include "../../include/nn_b200.h"
#include "nn_device.cuh"
#include "nn_internal.h"

namespace nn {

// ---------------------------------------------------------- BatchNorm
// NeuroNet.cl:1900-1953
__global__ void bn_ff_kernel(const float *__restrict__ in, float *__restrict__ opt, float *__restrict__ out,
                             float *__restrict__ hist, int N, int B, int batch, int width, int act, int training) {
  pdl_wait();
  pdl_trigger();
  int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float *o = opt + (size_t)n * width;
  const float fb = (float)batch;
  for (int b = 0; b < B; ++b) {
    size_t idx = (size_t)b * N + n;
    float inp = nan0(in[idx]);
    if (training == 0) {
      float mean = nan0(o[0]);
      float variance = nan0(o[1], 1.f);
      if (variance <= 0.f) variance = 1.f;
      float gamma = nan0(o[3], 1.f);
      if (gamma == 0.f) gamma = 1.f;
      float beta = nan0(o[4]);
      float nx = (inp - mean) / sqrtf(variance);
      out[idx] = activate(gamma * nx + beta, act);
      continue;
    }
    if (batch <= 1) {  // the reference leaves the output and the statistics untouched
      if (hist) {          // a batched backward still reads this sample's (unchanged) statistics
        hist[idx * 3 + 0] = o[0];
        hist[idx * 3 + 1] = o[1];
        hist[idx * 3 + 2] = o[2];
      }
      continue;
    }
    float mean = (nan0(o[0]) * fmaxf(fb - 1.f, 0.f) + inp) / fmaxf(fb, 1.f);
    float delt = inp - mean;
    float variance = (nan0(o[1] * fmaxf(fb - 1.f, 0.f)) + delt * delt) / fmaxf(fb, 1.f);
    if (variance <= 0.f) variance = 1.f;
    float nx = delt / sqrtf(variance);
    float gamma = nan0(o[3], 1.f);
    if (gamma == 0.f) {
      o[3] = 1.f;
      gamma = 1.f;
    }
    float beta = nan0(o[4]);
    o[0] = mean;
    o[1] = variance;
    o[2] = nx;
    if (hist) {
      hist[idx * 3 + 0] = mean;
      hist[idx * 3 + 1] = variance;
      hist[idx * 3 + 2] = nx;
    }
    out[idx] = activate(gamma * nx + beta, act);
  }
}

static int bn_width(Launch &L, int opt_idx) { return L.i(opt_idx) == 0 ? 7 : 9; }

static int k_batch_feed_forward(Launch &L) {
  const int N = (int)L.nd.g[0], width = bn_width(L, 4), batch = L.i(3), act = L.i(5), training = L.i(6);
  float *in = L.buf(0, (size_t)L.B * N), *opt = L.buf(1, (size_t)N * width), *out = L.buf(2, (size_t)L.B * N);
  if (!in || !opt || !out) return NN_ERR_BOUNDS;
  float *hist = nullptr;
  if (L.B > 1 && training != 0) {
    hist = L.side(L.handle(1), (size_t)L.B * N * 3);
    if (!hist) return NN_ERR_CUDA;
  }
  NN_LAUNCH_PDL(L, bn_ff_kernel, grid1d(N, 256), 256, 0, L.stream, in, opt, out, hist, N, L.B, batch, width, act, training);
  return NN_OK;
}

static const float *bn_history(Launch &L, int opt_idx, int N) {
  if (L.B == 1) return nullptr;
  size_t have = 0;
  float *h = L.side_existing(L.handle(opt_idx), &have);
  if (!h || have < (size_t)L.B * N * 3) {
    L.fail(NN_ERR_STATE, std::string(L.k->def->name) + ": batched call without a batched BatchFeedForward before it");
    return nullptr;
  }
  return h;
}

// NeuroNet.cl:1964-1998
__global__ void bn_hg_kernel(const float *__restrict__ opt, const float *__restrict__ g, const float *__restrict__ in,
                             float *__restrict__ ig, const float *__restrict__ hist, int N, int B, int width, int act,
                             int batch) {
  pdl_wait();
  pdl_trigger();
  int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const float *o = opt + (size_t)n * width;
  const float gamma = nan0(o[3], 1.f);
  const float ratio = fmaxf((float)(batch - 1), 0.f) / fmaxf((float)batch, 1.f);
  const int bdiv = max(batch, 1);
  for (int b = 0; b < B; ++b) {
    size_t idx = (size_t)b * N + n;
    float mean = hist ? hist[idx * 3] : nan0(o[0]);
    float variance = hist ? hist[idx * 3 + 1] : nan0(o[1], 1.f);
    float inp = nan0(in[idx]);
    float gnx = nan0(g[idx]) * gamma;
    float temp = variance > 0.f ? 1.f / sqrtf(variance) : 0.f;
    float gmu = -temp * gnx;
    float gvar = variance > 0.f ? (mean * inp) / (2.f * powf(variance, 1.5f)) * gnx : 0.f;
    float gx = temp * gnx + gmu / bdiv + gvar * 2.f * inp / bdiv * ratio * ratio;
    ig[idx] = deactivate(gx, inp, act);
  }
}

static int k_calc_hidden_gradient_batch(Launch &L) {
  const int N = (int)L.nd.g[0], width = bn_width(L, 6), act = L.i(4), batch = L.i(5);
  if (batch <= 1) return NN_OK;  // the reference returns without writing
  float *opt = L.buf(0, (size_t)N * width), *g = L.buf(1, (size_t)L.B * N), *in = L.buf(2, (size_t)L.B * N);
  float *ig = L.buf(3, (size_t)L.B * N);
  if (!opt || !g || !in || !ig) return NN_ERR_BOUNDS;
  const float *hist = bn_history(L, 0, N);
  if (L.B > 1 && !hist) return NN_ERR_STATE;
  NN_LAUNCH_PDL(L, bn_hg_kernel, grid1d(N, 256), 256, 0, L.stream, opt, g, in, ig, hist, N, L.B, width, act, batch);
  return NN_OK;
}

// Per-neuron batch-mean gradients of gamma and beta: G[2n] = mean_b clamp(g_b) nx_b, G[2n+1] = mean_b clamp(g_b).
__global__ void bn_grad_kernel(float *G, const float *__restrict__ opt, const float *__restrict__ g,
                               const float *__restrict__ hist, int N, int B, int width) {
  pdl_wait();
  pdl_trigger();
  int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float sg = 0.f, sb = 0.f;
  for (int b = 0; b < B; ++b) {
    size_t idx = (size_t)b * N + n;
    float grad = clampf(nan0(g[idx]), -kMaxGrad, kMaxGrad);
    float nx = hist ? hist[idx * 3 + 2] : nan0(opt[(size_t)n * width + 2]);
    sg += grad * nx;
    sb += grad;
  }
  G[2 * n] = sg / (float)B;
  G[2 * n + 1] = sb / (float)B;
}

// UpdateBatchOptionsAdam arithmetic, NeuroNet.cl:2050-2098 (delta of beta copies delta of gamma).
__global__ void bn_adam_apply_kernel(float *opt, const float *G, int N, float l, float b1, float b2) {
  pdl_wait();
  pdl_trigger();
  int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float *o = opt + (size_t)n * 9;
  float gg = G[2 * n], gb = G[2 * n + 1];
  float gamma = nan0(o[3], 1.f);
  if (gamma == 0.f) gamma = 1.f;
  float beta = nan0(o[4]);
  float mg = b1 * nan0(o[5]) + (1.f - b1) * gg;
  float mb = b1 * nan0(o[6]) + (1.f - b1) * gb;
  float vg = nan0(b2 * nan0(o[7]) + (1.f - b2) * (gg * gg), 1.f);
  float vb = nan0(b2 * nan0(o[8]) + (1.f - b2) * (gb * gb), 1.f);
  float dg = nan0(l * mg / sqrtf(vg));
  float db = dg;  // the reference assigns delta.s1 = IsNaNOrInf(delta.s0)
  float wg = dg - (kL1 * signf(gamma) + kL2 * gamma / (float)N);
  float wb = db - (kL1 * signf(beta) + kL2 * beta / (float)N);
  o[3] = nan0(gamma + wg, 1.f);
  o[4] = nan0(beta + wb);
  o[5] = nan0(mg);
  o[6] = nan0(mb);
  o[7] = vg;
  o[8] = vb;
}

// UpdateBatchOptionsMomentum arithmetic, NeuroNet.cl:2010-2038.
__global__ void bn_momentum_apply_kernel(float *opt, const float *G, int N, float lr, float mom) {
  pdl_wait();
  pdl_trigger();
  int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float *o = opt + (size_t)n * 7;
  float d0 = nan0(lr * G[2 * n] + mom * nan0(o[5]));
  float d1 = nan0(lr * G[2 * n + 1] + mom * nan0(o[6]));
  o[5] = d0;
  float value = nan0(o[3], 1.f);
  o[3] = value + d0 - lr * (kL1 * signf(value) + kL2 * value / (float)N);
  o[6] = d1;
  value = nan0(o[4]);
  o[4] = value + d1 - lr * (kL1 * signf(value) + kL2 * value / (float)N);
}

static int bn_adam_apply(const Launch &Lc, const float *G) {
  Launch &L = const_cast<Launch &>(Lc);
  const int N = (int)L.nd.g[0];
  float *opt = L.buf(0, (size_t)N * 9);
  if (!opt) return NN_ERR_BOUNDS;
  NN_LAUNCH_PDL(L, bn_adam_apply_kernel, grid1d(N, 256), 256, 0, L.stream, opt, G, N, L.f(2), L.f(3), L.f(4));
  return NN_OK;
}
static int bn_momentum_apply(const Launch &Lc, const float *G) {
  Launch &L = const_cast<Launch &>(Lc);
  const int N = (int)L.nd.g[0];
  float *opt = L.buf(0, (size_t)N * 7);
  if (!opt) return NN_ERR_BOUNDS;
  NN_LAUNCH_PDL(L, bn_momentum_apply_kernel, grid1d(N, 256), 256, 0, L.stream, opt, G, N, L.f(2), L.f(3));
  return NN_OK;
}

static int bn_update(Launch &L, int width, int (*apply)(const Launch &, const float *)) {
  const int N = (int)L.nd.g[0];
  float *opt = L.buf(0, (size_t)N * width), *g = L.buf(1, (size_t)L.B * N);
  if (!opt || !g) return NN_ERR_BOUNDS;
  const float *hist = bn_history(L, 0, N);
  if (L.B > 1 && !hist) return NN_ERR_STATE;
  float *G = L.deferred() ? L.grad_slot((size_t)2 * N) : L.scratch(3, (size_t)2 * N);
  if (!G) return NN_ERR_BOUNDS;
  NN_LAUNCH_PDL(L, bn_grad_kernel, grid1d(N, 256), 256, 0, L.stream, G, opt, g, hist, N, L.B, width);
  if (L.deferred()) {
    L.defer(apply, G);
    return NN_OK;
  }
  return apply(L, G);
}
static int k_update_batch_options_adam(Launch &L) { return bn_update(L, 9, bn_adam_apply); }
static int k_update_batch_options_momentum(Launch &L) { return bn_update(L, 7, bn_momentum_apply); }

// NeuroNet.cl:5742-5764: y = sqrt(var) (x - beta) / max(gamma, 1e-3) + mean
__global__ void revin_ff_kernel(const float *in, const float *opt, float *out, int n, int B, int options_size,
                                int width) {
  pdl_wait();
  pdl_trigger();
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)n * B) return;
  int i = (int)(t % n);
  int shift = (int)(((long long)i * width) % options_size);
  float mean = opt[shift], var = opt[shift + 1], k = opt[shift + 3];
  float res = sqrtf(var) * (in[t] - opt[shift + 4]) / fmaxf(k, 0.001f) + mean;
  out[t] = isnan(res) ? 0.f : res;
}

// NeuroNet.cl:5767-5793
__global__ void revin_hg_kernel(const float *in, float *in_gr, const float *opt, const float *out_gr, int n, int B,
                                int options_size, int width, int act) {
  pdl_wait();
  pdl_trigger();
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)n * B) return;
  int i = (int)(t % n);
  int shift = (int)(((long long)i * width) % options_size);
  float var = opt[shift + 1], k = opt[shift + 3];
  float res = sqrtf(var) * out_gr[t];
  if (fabsf(k) > 1.f) res /= k;
  if (isnan(res)) res = 0.f;
  in_gr[t] = deactivate(res, in[t], act);
}

static int revin_opts(Launch &L, int size_idx, int opt_idx, int *width, int *options_size) {
  *options_size = L.i(size_idx);
  *width = L.i(opt_idx) == 0 ? 7 : 9;
  if (*options_size < 5) return L.fail(NN_ERR_ARG, "RevIn: options_size < 5");
  return NN_OK;
}

// shift = (i*width) % options_size reaches options_size-1, and the kernels read shift+4.
static size_t opt_need(int osz, int width) { return (size_t)osz + (osz % width == 0 ? 0 : 4); }

static int k_revin_ff(Launch &L) {
  int n = (int)L.nd.g[0], width, osz;
  int rc = revin_opts(L, 3, 4, &width, &osz);
  if (rc) return rc;
  float *in = L.buf(0, (size_t)n * L.B), *opt = L.buf(1, opt_need(osz, width)), *out = L.buf(2, (size_t)n * L.B);
  if (!in || !opt || !out) return NN_ERR_BOUNDS;
  NN_LAUNCH_PDL(L, revin_ff_kernel, grid1d((size_t)n * L.B, 256), 256, 0, L.stream, in, opt, out, n, L.B, osz, width);
  return NN_OK;
}

static int k_revin_hg(Launch &L) {
  int n = (int)L.nd.g[0], width, osz;
  int rc = revin_opts(L, 4, 5, &width, &osz);
  if (rc) return rc;
  float *in = L.buf(0, (size_t)n * L.B), *ig = L.buf(1, (size_t)n * L.B), *opt = L.buf(2, opt_need(osz, width));
  float *og = L.buf(3, (size_t)n * L.B);
  if (!in || !ig || !opt || !og) return NN_ERR_BOUNDS;
  NN_LAUNCH_PDL(L, revin_hg_kernel, grid1d((size_t)n * L.B, 256), 256, 0, L.stream, in, ig, opt, og, n, L.B, osz, width, L.i(6));
  return NN_OK;
}

const KernelDef kMiscKernels[] = {
    {"BatchFeedForward", "pppiiii", k_batch_feed_forward, false},
    {"CalcHiddenGradientBatch", "ppppiii", k_calc_hidden_gradient_batch, false},
    {"UpdateBatchOptionsAdam", "ppfff", k_update_batch_options_adam, false},
    {"UpdateBatchOptionsMomentum", "ppff", k_update_batch_options_momentum, false},
    {"RevInFeedForward", "pppii", k_revin_ff, false},
    {"RevInHiddenGraddient", "ppppiii", k_revin_hg, false},
};
const int kNumMiscKernels = sizeof(kMiscKernels) / sizeof(kMiscKernels[0]);

}  // namespace nn
