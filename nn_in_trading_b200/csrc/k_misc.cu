// RevIN de-normalisation kernels (CNeuronRevINDenormOCL path):
// RevInFeedForward, RevInHiddenGraddient.  They read the running statistics
// of a referenced batch-normalisation layer's options buffer
// ([neuron][7] for SGD, [neuron][9] for Adam: mean, variance, nx, gamma, beta, ...).
#include "../../include/nn_b200.h"
#include "nn_device.cuh"
#include "nn_internal.h"

namespace nn {

// NeuroNet.cl:5742-5764: y = sqrt(var) (x - beta) / max(gamma, 1e-3) + mean
__global__ void revin_ff_kernel(const float *in, const float *opt, float *out, int n, int B, int options_size,
                                int width) {
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
  revin_ff_kernel<<<grid1d((size_t)n * L.B, 256), 256, 0, L.stream>>>(in, opt, out, n, L.B, osz, width);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

static int k_revin_hg(Launch &L) {
  int n = (int)L.nd.g[0], width, osz;
  int rc = revin_opts(L, 4, 5, &width, &osz);
  if (rc) return rc;
  float *in = L.buf(0, (size_t)n * L.B), *ig = L.buf(1, (size_t)n * L.B), *opt = L.buf(2, opt_need(osz, width));
  float *og = L.buf(3, (size_t)n * L.B);
  if (!in || !ig || !opt || !og) return NN_ERR_BOUNDS;
  revin_hg_kernel<<<grid1d((size_t)n * L.B, 256), 256, 0, L.stream>>>(in, ig, opt, og, n, L.B, osz, width, L.i(6));
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

const KernelDef kMiscKernels[] = {
    {"RevInFeedForward", "pppii", k_revin_ff, false},
    {"RevInHiddenGraddient", "ppppiii", k_revin_hg, false},
};
const int kNumMiscKernels = sizeof(kMiscKernels) / sizeof(kMiscKernels[0]);

}  // namespace nn
