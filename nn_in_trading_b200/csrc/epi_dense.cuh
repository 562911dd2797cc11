// Epilogues of the dense GEMMs, shared by every launcher whose product ends the same way.
// FFEpi (FeedForward, batched): y[m][n] = act(acc + bias(n)), the bias being column `inputs` of
// weight row n (rows of `ld` floats, NeuroNet.cl:430-512 layout).
#pragma once
#include "nn_device.cuh"
#include "tc_gemm.cuh"

namespace nn {

struct FFEpi {
  const float *w;
  float *y;
  int ld, inputs, outputs, act;
  __device__ __forceinline__ void operator()(int m, int n, int, int, float acc) const {
    y[(size_t)m * outputs + n] = activate(acc + nan0(w[(size_t)n * ld + inputs]), act);
  }
  __device__ __forceinline__ long long row(int m, int, int) const { return (long long)m * outputs; }
  __device__ __forceinline__ float col(int n, int) const { return nan0(w[(size_t)n * ld + inputs]); }
  template <int R>
  __device__ __forceinline__ void put_rows(const long long (&rb)[R], int n, const float (&v)[R], float bias,
                                           unsigned mask) const {
    act_dispatch(act, [&](auto A) {
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (mask >> j & 1u) y[rb[j] + n] = activate(v[j] + bias, decltype(A)::value);
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
          *reinterpret_cast<float4 *>(y + rb[j] + n) = make_float4(
              activate(v[j].x + b.x, a), activate(v[j].y + b.y, a), activate(v[j].z + b.z, a),
              activate(v[j].w + b.w, a));
    });
  }
};

// FFEpi with the output written by TMA stores on the tensor-core path (checked with tma_store_ok).
struct FFEpiTma : FFEpi {
  static constexpr bool kTmaStore = true;
  template <class F>
  __device__ __forceinline__ void transform(F &&f) const {
    act_dispatch(act, [&](auto A) { f([](float x, float b, float) { return activate(x + b, decltype(A)::value); }); });
  }
  __device__ __forceinline__ int zc(int z, int) const { return z; }
  bool out_map(CUtensorMap *tm, int M, int N, int nz) const {
    return make_tmap(tm, y, outputs, 0, N, M, nz, 32, false);
  }
};

// Epilogue of the dense hidden gradient (CalcHiddenGradient, batched): ig[m][n] = Deact(acc, o[m][n]),
// o and ig rows of `inputs` floats.
struct CHGEpi {
  const float *o;
  float *ig;
  int inputs, act;
  __device__ __forceinline__ void operator()(int m, int n, int, int, float acc) const {
    size_t idx = (size_t)m * inputs + n;
    ig[idx] = deactivate(acc, o[idx], act);
  }
  __device__ __forceinline__ long long row(int m, int, int) const { return (long long)m * inputs; }
  __device__ __forceinline__ float col(int, int) const { return 0.f; }
  template <int R>
  __device__ __forceinline__ void put_rows(const long long (&rb)[R], int n, const float (&v)[R], float,
                                           unsigned mask) const {
    float yv[R];
#pragma unroll
    for (int j = 0; j < R; ++j) yv[j] = (mask >> j & 1u) ? o[rb[j] + n] : 0.f;
    act_dispatch(act, [&](auto A) {
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (mask >> j & 1u) ig[rb[j] + n] = deactivate(v[j], yv[j], decltype(A)::value);
    });
  }
  __host__ __device__ bool aligned4() const {
    return inputs % 4 == 0 && ((uintptr_t)o & 15) == 0 && ((uintptr_t)ig & 15) == 0;
  }
  __device__ __forceinline__ float4 col4(int, int) const { return make_float4(0.f, 0.f, 0.f, 0.f); }
  template <int R>
  __device__ __forceinline__ void put_rows4(const long long (&rb)[R], int n, const float4 (&v)[R], float4,
                                            unsigned mask) const {
    float4 yv[R];
#pragma unroll
    for (int j = 0; j < R; ++j)
      yv[j] = (mask >> j & 1u) ? *reinterpret_cast<const float4 *>(o + rb[j] + n) : make_float4(0.f, 0.f, 0.f, 0.f);
    act_dispatch(act, [&](auto A) {
      constexpr int a = decltype(A)::value;
#pragma unroll
      for (int j = 0; j < R; ++j)
        if (mask >> j & 1u)
          *reinterpret_cast<float4 *>(ig + rb[j] + n) =
              make_float4(deactivate(v[j].x, yv[j].x, a), deactivate(v[j].y, yv[j].y, a),
                          deactivate(v[j].z, yv[j].z, a), deactivate(v[j].w, yv[j].w, a));
    });
  }
};

// CHGEpi with the input gradient written by TMA stores and the activation output read as the aux
// tensor (checked with tma_store_ok).
struct CHGEpiTma : CHGEpi {
  static constexpr bool kTmaStore = true, kAux = true;
  template <class F>
  __device__ __forceinline__ void transform(F &&f) const {
    act_dispatch(act, [&](auto A) { f([](float x, float, float y) { return deactivate(x, y, decltype(A)::value); }); });
  }
  __device__ __forceinline__ int zc(int z, int) const { return z; }
  __device__ __forceinline__ float4 aux4(int m, int, int n) const {
    return *reinterpret_cast<const float4 *>(o + (size_t)m * inputs + n);
  }
  bool out_map(CUtensorMap *tm, int M, int N, int nz) const {
    return make_tmap(tm, ig, inputs, 0, N, M, nz, 32, false);
  }
};

}  // namespace nn
