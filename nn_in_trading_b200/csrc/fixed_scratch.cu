// nn_update_weights_adam_fixed: the batched dense UpdateWeightsAdam with its
// weight-gradient partials in a fixed device array compiled into this library.
//
// Why it exists.  The regular path (nn_execute of UpdateWeightsAdam with
// nn_set_batch > 1) reduces the per-sample weight gradients into per-context
// scratch that grows with cudaMalloc the first time a larger update is seen,
// and a grow first synchronises the stream and frees the old block.  Some
// callers cannot let that happen: a host that hands all free device memory to
// its own pool after start-up (a cudaMalloc then fails), and a latency-bound
// loop (one bar in, one update out) that cannot take the device-wide stall a
// cudaMalloc/cudaFree pair may cause in the middle of a session.  This entry
// point allocates nothing: the partials live in `g_fixed_scratch` below.  The
// CUDA runtime reserves its storage when it loads this file's device module;
// under lazy module loading (the default since CUDA 12.2) that happens on the
// module's first use, so nn_init resolves the array's address (which loads the
// module) before it returns.
//
// Limits and rules of use.
//  * outputs * (inputs + 1) must not exceed kFixedScratchFloats (2 Mi floats,
//    8 MiB); larger updates are rejected with NN_ERR_BOUNDS and a message.
//  * nn_init looks up the array's device address on the context's device
//    (cudaGetSymbolAddress, with that device current).  If that look-up failed,
//    the first call retries it; make that call before any stream capture starts.
//  * There is ONE array per device.  Calls that overlap on the same device
//    (from two threads, or on two streams) race on it and give wrong results;
//    the caller must order them.  Calls made through this library's context
//    are ordered by its single stream.
//  * The update is local: inside a data-parallel update region
//    (nn_dp_update_begin .. end) the call is refused with NN_ERR_STATE, because
//    applying one rank's gradient there would make the ranks' weights diverge.
//  * Nothing in the array has to start at zero: the split-K GEMM writes every
//    partial of the N weight columns, and the bias-column kernel writes every
//    bias partial, before the apply kernel reads them.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "../../include/nn_b200.h"
#include "nn_internal.h"
#include "wgrad.cuh"

namespace nn {

constexpr size_t kFixedScratchFloats = size_t(1) << 21;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_fixed_scratch[kFixedScratchFloats];

// Defined with the dense kernels (UpdateWeightsAdam arithmetic on a given gradient).
__global__ void adam_dense_apply_kernel(float *w, float *m, float *v, GradSrc G, int n_out, int n_col, int inputs,
                                        float l, float b1, float b2);

static std::mutex g_fixed_mu;
static float *g_fixed_ptr[kMaxDevices] = {};

// Looks up the device address of g_fixed_scratch on `device`, making that device current for the
// look-up (the calling thread may have another one current) and restoring the previous one.
static int fixed_scratch_lookup(int device, float **out) {
  if (device < 0 || device >= kMaxDevices) return report_error(NN_ERR_UNSUPPORTED, "device index out of range");
  std::lock_guard<std::mutex> lock(g_fixed_mu);
  if (!g_fixed_ptr[device]) {
    int prev = -1;
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return report_error(NN_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    if (prev != device) {
      e = cudaSetDevice(device);
      if (e != cudaSuccess) return report_error(NN_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
    }
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_fixed_scratch);
    if (prev != device) cudaSetDevice(prev);
    if (e != cudaSuccess || !p)
      return report_error(NN_ERR_CUDA, std::string("cudaGetSymbolAddress(fixed scratch): ") +
                                           cudaGetErrorString(e));
    g_fixed_ptr[device] = static_cast<float *>(p);
  }
  *out = g_fixed_ptr[device];
  return NN_OK;
}

int fixed_scratch_setup(int device) {
  float *p = nullptr;
  return fixed_scratch_lookup(device, &p);
}

}  // namespace nn

extern "C" NN_API int nn_update_weights_adam_fixed(float *matrix_w, const float *matrix_g, const float *matrix_i,
                                                   float *matrix_m, float *matrix_v, int outputs, int inputs,
                                                   int batch, float l, float b1, float b2) {
  using namespace nn;
  cudaStream_t stream = static_cast<cudaStream_t>(nn_stream());
  if (!stream) return report_error(NN_ERR_STATE, "nn_init not called");
  if (!matrix_w || !matrix_g || !matrix_i || !matrix_m || !matrix_v)
    return report_error(NN_ERR_ARG, "nn_update_weights_adam_fixed: null pointer");
  if (outputs < 1 || inputs < 0 || batch < 1)
    return report_error(NN_ERR_ARG, "nn_update_weights_adam_fixed: outputs and batch must be >= 1, inputs >= 0");
  const int N = inputs, ldp = inputs + 1;
  const size_t per = (size_t)outputs * ldp;
  if (per > kFixedScratchFloats)
    return report_error(NN_ERR_BOUNDS, "nn_update_weights_adam_fixed: outputs*(inputs+1) = " + std::to_string(per) +
                                           " floats exceeds the fixed scratch of " +
                                           std::to_string(kFixedScratchFloats) + " floats");
  if (dp_update_open())
    return report_error(NN_ERR_STATE, "nn_update_weights_adam_fixed: a data-parallel update region is open (the "
                                      "update would apply this rank's gradient alone)");
  float *part = nullptr;
  int rc = fixed_scratch_lookup(context_device(), &part);
  if (rc) return rc;

  // Same split-K decomposition as the context-scratch path, capped by what the array holds; on the
  // tensor cores split boundaries fall on the GEMM's 32-deep stages, as they do there.
  int splits = fast_splits(outputs, N + 1, batch, 1);
  const size_t fit = kFixedScratchFloats / per;
  if ((size_t)splits > fit) splits = (int)fit;
  const int gran = tc_path(FastShape{outputs, N, batch, 1, 1, 0, matrix_g, outputs, 0, matrix_i, inputs, 0}) ? 32 : 8;
  int kchunk = ((batch + splits - 1) / splits + gran - 1) / gran * gran;
  splits = (batch + kchunk - 1) / kchunk;
  if (splits < 1) splits = 1;

  // G[m][n] = sum_b g[b][m] * x[b][n]  (n < inputs), partial per split
  if (N > 0) {
    FastShape fs{outputs, N, batch, 1, splits, kchunk, matrix_g, outputs, 0, matrix_i, inputs, 0};
    cudaError_t e = gemm_f32<true, true>(fs, PartialStoreLd{part, outputs, ldp, 1}, stream);
    if (e != cudaSuccess) return report_error(NN_ERR_CUDA, cudaGetErrorString(e));
    add_launches(1);
  }
  // G[m][inputs] = sum_b g[b][m]  (the bias input is 1)
  colsum_partial_kernel<<<dim3((outputs + 255) / 256, splits), 256, 0, stream>>>(part, matrix_g, outputs, batch,
                                                                                outputs, kchunk, ldp, N);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return report_error(NN_ERR_CUDA, cudaGetErrorString(e));
  GradSrc src{part, splits, per, 1.f / (float)batch};
  adam_dense_apply_kernel<<<grid1d(per, 256), 256, 0, stream>>>(matrix_w, matrix_m, matrix_v, src, outputs, ldp,
                                                                inputs, l, b1, b2);
  e = cudaGetLastError();
  if (e != cudaSuccess) return report_error(NN_ERR_CUDA, cudaGetErrorString(e));
  add_launches(2);
  return NN_OK;
}
