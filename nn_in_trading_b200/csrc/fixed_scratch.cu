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
// CUDA runtime reserves its storage when it loads this file's device module,
// and under lazy loading (the default since CUDA 12.2) it loads each kernel on
// its first launch, which also takes device memory.  So the entry point runs
// only two kernels with fixed entry points (its own split-K weight gradient and
// the dense Adam apply), and nn_init resolves the array's address and queries
// both kernels' attributes, which loads the module and the two kernels before
// nn_init returns: no call of the entry point loads anything.
//
// Limits and rules of use.
//  * outputs * (inputs + 1) must not exceed kFixedScratchFloats (2 Mi floats,
//    8 MiB); larger updates are rejected with NN_ERR_BOUNDS and a message.
//  * nn_init looks up the array's device address on the context's device
//    (cudaGetSymbolAddress, with that device current) and loads the two
//    kernels.  If that failed, the first call retries it; make that call before
//    any stream capture starts and before the host takes the free memory.
//  * There is ONE array per device.  Calls that overlap on the same device
//    (from two threads, or on two streams) race on it and give wrong results;
//    the caller must order them.  Calls made through this library's context
//    are ordered by its single stream.
//  * The update is local: inside a data-parallel update region
//    (nn_dp_update_begin .. end) the call is refused with NN_ERR_STATE, because
//    applying one rank's gradient there would make the ranks' weights diverge.
//  * Nothing in the array has to start at zero: the weight-gradient kernel
//    writes every partial of every weight column, the bias column included,
//    before the apply kernel reads them.
#include <cuda_runtime.h>

#include <algorithm>
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

// Split-K weight gradient of the dense layer into the fixed array: for split z (batch rows
// [z*kchunk, (z+1)*kchunk)), part[z][m][n] = sum_b IsNaNOrInf(g[b][m]) * IsNaNOrInf(x[b][n]) for
// n < inputs and part[z][m][inputs] = sum_b IsNaNOrInf(g[b][m]) (the bias input 1), each product
// with a non-finite result dropped as the batched path does.  A 32 x 32 tile of (m, n) per block of
// 32 x 8 threads, 32 batch rows of g and x staged in shared memory at a time.
__global__ void __launch_bounds__(256) fixed_wgrad_kernel(float *__restrict__ part, const float *__restrict__ g,
                                                          const float *__restrict__ x, int outputs, int inputs,
                                                          int batch, int kchunk) {
  __shared__ float gs[32][33], xs[32][33];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int tiles_n = (inputs + 1 + 31) / 32;
  const int m0 = (int)(blockIdx.x / tiles_n) * 32, n0 = (int)(blockIdx.x % tiles_n) * 32, z = blockIdx.y;
  const int b0 = z * kchunk, b1 = min(batch, b0 + kchunk);
  const int ldp = inputs + 1;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int bb = b0; bb < b1; bb += 32) {
    for (int r = ty; r < 32; r += 8) {
      const int b = bb + r;
      const bool in = b < b1;
      gs[r][tx] = in && m0 + tx < outputs ? nan0(g[(size_t)b * outputs + m0 + tx]) : 0.f;
      const int n = n0 + tx;
      xs[r][tx] = !in || n > inputs ? 0.f : (n == inputs ? 1.f : nan0(x[(size_t)b * inputs + n]));
    }
    __syncthreads();
#pragma unroll 8
    for (int r = 0; r < 32; ++r) {
      const float xv = xs[r][tx];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] += nan0(gs[r][ty + 8 * j] * xv);
    }
    __syncthreads();
  }
  const int n = n0 + tx;
  if (n > inputs) return;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int m = m0 + ty + 8 * j;
    if (m < outputs) part[((size_t)z * outputs + m) * ldp + n] = acc[j];
  }
}

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
  int rc = fixed_scratch_lookup(device, &p);
  if (rc) return rc;
  // load both kernels now (under lazy loading a kernel is loaded, taking device memory, at its first use)
  cudaFuncAttributes a;
  cudaError_t e = cudaFuncGetAttributes(&a, fixed_wgrad_kernel);
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&a, adam_dense_apply_kernel);
  if (e != cudaSuccess) return report_error(NN_ERR_CUDA, std::string("loading the fixed-scratch kernels: ") +
                                                             cudaGetErrorString(e));
  return NN_OK;
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

  // split the batch so that the (m, n) tiles times the splits fill the GPU twice, capped by what the
  // array holds
  const long long tiles = (long long)((outputs + 31) / 32) * ((ldp + 31) / 32);
  int splits = (int)((2 * 148 + tiles - 1) / tiles);
  splits = std::min(splits, (batch + 31) / 32);
  const size_t fit = kFixedScratchFloats / per;
  if ((size_t)splits > fit) splits = (int)fit;
  if (splits < 1) splits = 1;
  const int kchunk = (batch + splits - 1) / splits;
  splits = (batch + kchunk - 1) / kchunk;
  fixed_wgrad_kernel<<<dim3((unsigned)tiles, (unsigned)splits), dim3(32, 8), 0, stream>>>(part, matrix_g, matrix_i,
                                                                                         outputs, N, batch, kchunk);
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
