// Element-wise masking and patch embedding of the reference's newer layers.
//   Dropout                 out = inputs * map (CNeuronDropoutOCL / ElementMult)   NeuroNet.cl:1855-1884
//   PatchCreate             patches of a [time][variables] series, per-variable   NeuroNet.cl:5826-5860
//                           linear map + activation (CNeuronPatching)
//   PatchHiddenGradient     its input gradient                                     NeuroNet.cl:5864-5911
//   PatchUpdateWeightsAdam  refused: the reference kernel reads an uninitialised   NeuroNet.cl:5912-5951
//                           index, so it has no defined result to reproduce
// Batches: every per-sample buffer holds `batch` consecutive copies of the per-sample layout; the
// patch weights are shared.
#include <algorithm>

#include "../../include/nn_b200.h"
#include "nn_device.cuh"
#include "nn_internal.h"

namespace nn {
namespace {

// Dropout (NeuroNet.cl:1855-1884) as the reference indexes it: work-item t loops k over
// [4t, min(dimension, 4t + 4)) and reads and writes element 4t + k, i.e. elements 8t + j with
// j < 4 and 4t + j < dimension.  Elements 8t + 4 .. 8t + 7 are never written, and with the host's
// global size (dimension + 3) / 4 (NeuroNet_Core.mqh:19168) the upper work-items reach past
// `dimension`, up to about 2 * dimension.  This kernel writes every element of that set that lies
// below `limit` (the smallest of the three buffers at batch 1, `dimension` per sample in a batch)
// and skips the rest.  out = 0 where the map or the input is 0 (after IsNaNOrInf), else
// IsNaNOrInf(inp * m).  One thread per element.
__global__ void dropout_kernel(const float *__restrict__ in, const float *__restrict__ map, float *__restrict__ out,
                               long long items, int dimension, long long limit, long long stride, int batch) {
  const long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x;  // (sample, work-item, j)
  if (t >= items * 4 * batch) return;
  const int j = (int)(t & 3);
  const long long wi = (t >> 2) % items;
  const long long b = (t >> 2) / items;
  if (4 * wi + j >= dimension) return;
  const long long e = 8 * wi + j;
  if (e >= limit) return;
  const long long at = b * stride + e;
  const float m = nan0(map[at]);
  if (m == 0.f) {
    out[at] = 0.f;
    return;
  }
  const float x = nan0(in[at]);
  out[at] = x == 0.f ? 0.f : nan0(x * m);
}

int k_dropout(Launch &L) {
  const long long items = (long long)L.nd.g[0];
  const int dimension = L.i(3);
  if (dimension < 0) return L.fail(NN_ERR_ARG, "Dropout: negative dimension");
  if (items == 0 || dimension == 0) return NN_OK;
  // highest element the reference touches: 8t + j for the last work-item t that has a j < 4 with
  // 4t + j below dimension
  const long long tmax = std::min<long long>(items - 1, (dimension - 1) / 4);
  const long long reach = 8 * tmax + std::min<long long>(3, dimension - 1 - 4 * tmax) + 1;
  const long long core = std::min<long long>(reach, dimension);  // the elements below dimension
  long long limit, stride;
  if (L.B == 1) {
    // past `dimension` the reference writes wherever its buffers reach; this library stops at the
    // end of the smallest buffer
    limit = std::min<long long>(reach, (long long)std::min(L.floats(0), std::min(L.floats(1), L.floats(2))));
    limit = std::max(limit, core);
    stride = 0;
  } else {
    limit = core;
    stride = dimension;
  }
  const size_t need = L.B == 1 ? (size_t)limit : (size_t)L.B * dimension;
  float *in = L.buf(0, need), *map = L.buf(1, need), *out = L.buf(2, need);
  if (!in || !map || !out) return NN_ERR_BOUNDS;
  const long long n = items * 4 * L.B;
  dropout_kernel<<<grid1d((size_t)n, 256), 256, 0, L.stream>>>(in, map, out, items, dimension, limit, stride, L.B);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

// PatchCreate (NeuroNet.cl:5826-5860) over global (patches, window_out, variables): output
// (i * variables + v) * window_out + w = act(b + sum_p x[(i*step + p) * variables + v] W[p]) with
// the inputs at or past inputs_total left out, W the (window_in + 1)-float row v * window_out + w
// (bias last); a NaN sum becomes 0.  One thread per output, w fastest (coalesced stores; the
// input of a warp is one broadcast address).
__global__ void patch_create_kernel(const float *__restrict__ x, const float *__restrict__ w, float *__restrict__ y,
                                    int inputs_total, int window_in, int step, int act, int patches, int window_out,
                                    int variables, long long per_out, int batch) {
  const long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (t >= per_out * batch) return;
  const long long b = t / per_out;
  const long long o = t % per_out;
  const int wo = (int)(o % window_out);
  const int v = (int)((o / window_out) % variables);
  const int i = (int)(o / ((long long)window_out * variables));
  const float *xs = x + b * inputs_total;
  const int shift_in = i * step * variables + v;
  const float *row = w + (size_t)(window_in + 1) * ((size_t)v * window_out + wo);
  float res = row[window_in];
  for (int p = 0; p < window_in; ++p) {
    const int at = shift_in + p * variables;
    if (at < inputs_total) res += xs[at] * row[p];
  }
  if (isnan(res)) res = 0.f;
  y[b * per_out + o] = activate(res, act);
  (void)patches;
}

int k_patch_create(Launch &L) {
  const int patches = (int)L.nd.g[0];
  const int window_out = L.nd.dims > 1 ? (int)L.nd.g[1] : 1;
  const int variables = L.nd.dims > 2 ? (int)L.nd.g[2] : 1;
  const int inputs_total = L.i(3), window_in = L.i(4), step = L.i(5), act = L.i(6);
  if (inputs_total < 0 || window_in < 0 || step < 0) return L.fail(NN_ERR_ARG, "PatchCreate: negative size");
  const long long per_out = (long long)patches * window_out * variables;
  float *x = L.buf(0, (size_t)L.B * inputs_total);
  float *w = L.buf(1, (size_t)variables * window_out * (window_in + 1));
  float *y = L.buf(2, (size_t)L.B * per_out);
  if (!x || !w || !y) return NN_ERR_BOUNDS;
  patch_create_kernel<<<grid1d((size_t)per_out * L.B, 256), 256, 0, L.stream>>>(
      x, w, y, inputs_total, window_in, step, act, patches, window_out, variables, per_out, L.B);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

// PatchHiddenGradient (NeuroNet.cl:5864-5911) over global (time, variables): input (i, v) collects
// outputs_gr[(row * variables + v) * window_out + wo] * W[v][wo][w_start + (total - p - 1) * step]
// over the `total` patches row = r_start + p (< outputs_total) that the reference's index
// arithmetic assigns to time i, then Deactivation by the input's activation.  One thread per
// input element, v fastest.
__global__ void patch_hidden_grad_kernel(const float *__restrict__ x, float *__restrict__ xg,
                                         const float *__restrict__ w, const float *__restrict__ og, int window_in,
                                         int step, int window_out, int outputs_total, int act, int times,
                                         int variables, long long per_in, long long per_og, int batch) {
  const long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (t >= per_in * batch) return;
  const long long b = t / per_in;
  const long long e = t % per_in;
  const int v = (int)(e % variables);
  const int i = (int)(e / variables);
  const float *g = og + b * per_og;
  const int w_start = i % step;
  const int r_start = max((i - window_in + step) / step, 0);
  int total = (window_in - w_start + step - 1) / step;
  total = min((i + step) / step, total);
  float grad = 0.f;
  for (int p = 0; p < total; ++p) {
    const int row = r_start + p;
    if (row >= outputs_total) break;
    const float *gr = g + ((size_t)row * variables + v) * window_out;
    const float *wr = w + (size_t)v * (window_in + 1) * window_out + w_start + (size_t)(total - p - 1) * step;
    for (int wo = 0; wo < window_out; ++wo) grad += gr[wo] * wr[(size_t)wo * (window_in + 1)];
  }
  xg[b * per_in + e] = deactivate(grad, x[b * per_in + e], act);
  (void)times;
}

int k_patch_hidden_grad(Launch &L) {
  const int times = (int)L.nd.g[0];
  const int variables = L.nd.dims > 1 ? (int)L.nd.g[1] : 1;
  const int window_in = L.i(4), step = L.i(5), window_out = L.i(6), outputs_total = L.i(7), act = L.i(8);
  if (window_in < 0 || window_out < 0 || outputs_total < 0) return L.fail(NN_ERR_ARG, "PatchHiddenGradient: negative size");
  if (step <= 0) return L.fail(NN_ERR_ARG, "PatchHiddenGradient: step must be positive");
  const long long per_in = (long long)times * variables;
  const long long per_og = (long long)outputs_total * variables * window_out;
  float *x = L.buf(0, (size_t)L.B * per_in), *xg = L.buf(1, (size_t)L.B * per_in);
  float *w = L.buf(2, (size_t)variables * window_out * (window_in + 1));
  float *og = L.buf(3, (size_t)L.B * per_og);
  if (!x || !xg || !w || !og) return NN_ERR_BOUNDS;
  patch_hidden_grad_kernel<<<grid1d((size_t)per_in * L.B, 256), 256, 0, L.stream>>>(
      x, xg, w, og, window_in, step, window_out, outputs_total, act, times, variables, per_in, per_og, L.B);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

int k_patch_update_adam(Launch &L) {
  return L.fail(NN_ERR_UNSUPPORTED,
                "PatchUpdateWeightsAdam: the reference kernel (NeuroNet.cl:5912-5951) indexes its inputs with a "
                "variable read before it is initialised and every gradient term with outputs_gr[0], so its "
                "result is undefined; train patch embeddings with a Conv1D layer (FeedForwardConv / "
                "UpdateWeightsConvAdam) instead");
}

}  // namespace

const KernelDef kPatchKernels[] = {
    {"Dropout", "pppi", k_dropout, false},
    {"PatchCreate", "pppiiii", k_patch_create, false},
    {"PatchHiddenGradient", "ppppiiiii", k_patch_hidden_grad, false},
    {"PatchUpdateWeightsAdam", "pppppifffi", k_patch_update_adam, true},
};
const int kNumPatchKernels = sizeof(kPatchKernels) / sizeof(kPatchKernels[0]);

}  // namespace nn
