// ORACLE TEST INFRASTRUCTURE -- not part of the shipped library.
//
// OpenCL C -> C++ shim used to compile the reference kernel source
// (Experts/NeuroNet_DNG/NeuroNet.cl) for the host CPU, so that the
// reference's own kernels can be executed on the same seeded inputs as the
// CUDA path.  The generated translation unit lives only in oracle/_ref/
// (git-ignored); this header, the executor below and the generator script
// oracle/build_ref.py are the committed recipe.
//
// What the shim provides:
//   * float2 / float4 with .x.y.z.w and .s0..s3 lanes and elementwise math;
//   * the OpenCL built-ins the in-scope kernels call (exp, sqrt, clamp, sign,
//     dot, isnan, ...) with single-precision semantics;
//   * work-item functions (get_global_id, get_local_size, ...) read from a
//     thread-local NDRange context;
//   * barrier() implemented with cooperative fibers: every work-item of a
//     work-group is a fiber on one OS thread and barrier() yields back to the
//     work-group scheduler, so __local arrays (rewritten to thread_local
//     statics by the generator) are shared by exactly one work-group at a time.
#pragma once
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <vector>
#include <ucontext.h>

namespace ocl {

typedef unsigned int uint;
typedef unsigned long ulong;
typedef unsigned char uchar;
typedef unsigned short ushort;

#define CLK_LOCAL_MEM_FENCE 1
#define CLK_GLOBAL_MEM_FENCE 2
#define M_PI_F 3.14159265358979323846f  /* OpenCL: pi as float */

// ----------------------------------------------------------------- vectors
struct float2 {
  union {
    struct { float x, y; };
    struct { float s0, s1; };
  };
  float2() : x(0.f), y(0.f) {}
  explicit float2(float v) : x(v), y(v) {}
  float2(float a, float b) : x(a), y(b) {}
};
struct float4 {
  union {
    struct { float x, y, z, w; };
    struct { float s0, s1, s2, s3; };
  };
  float4() : x(0.f), y(0.f), z(0.f), w(0.f) {}
  explicit float4(float v) : x(v), y(v), z(v), w(v) {}
  float4(float a, float b, float c, float d) : x(a), y(b), z(c), w(d) {}
};

#define OCL_V2_BINOP(op)                                                          \
  inline float2 operator op(const float2 &a, const float2 &b) { return float2(a.x op b.x, a.y op b.y); } \
  inline float2 operator op(const float2 &a, float b) { return float2(a.x op b, a.y op b); }             \
  inline float2 operator op(float a, const float2 &b) { return float2(a op b.x, a op b.y); }
#define OCL_V4_BINOP(op)                                                                               \
  inline float4 operator op(const float4 &a, const float4 &b) {                                        \
    return float4(a.x op b.x, a.y op b.y, a.z op b.z, a.w op b.w);                                     \
  }                                                                                                    \
  inline float4 operator op(const float4 &a, float b) { return float4(a.x op b, a.y op b, a.z op b, a.w op b); } \
  inline float4 operator op(float a, const float4 &b) { return float4(a op b.x, a op b.y, a op b.z, a op b.w); }
OCL_V2_BINOP(+) OCL_V2_BINOP(-) OCL_V2_BINOP(*) OCL_V2_BINOP(/)
OCL_V4_BINOP(+) OCL_V4_BINOP(-) OCL_V4_BINOP(*) OCL_V4_BINOP(/)
inline float2 operator-(const float2 &a) { return float2(-a.x, -a.y); }
inline float4 operator-(const float4 &a) { return float4(-a.x, -a.y, -a.z, -a.w); }
inline float2 &operator+=(float2 &a, const float2 &b) { a = a + b; return a; }
inline float2 &operator-=(float2 &a, const float2 &b) { a = a - b; return a; }
inline float2 &operator*=(float2 &a, const float2 &b) { a = a * b; return a; }
inline float2 &operator/=(float2 &a, const float2 &b) { a = a / b; return a; }
inline float2 &operator*=(float2 &a, float b) { a = a * b; return a; }
inline float2 &operator/=(float2 &a, float b) { a = a / b; return a; }
inline float4 &operator+=(float4 &a, const float4 &b) { a = a + b; return a; }
inline float4 &operator-=(float4 &a, const float4 &b) { a = a - b; return a; }
inline float4 &operator*=(float4 &a, const float4 &b) { a = a * b; return a; }
inline float4 &operator/=(float4 &a, const float4 &b) { a = a / b; return a; }
inline float4 &operator*=(float4 &a, float b) { a = a * b; return a; }
inline float4 &operator/=(float4 &a, float b) { a = a / b; return a; }

// ------------------------------------------------------------ math built-ins
inline float exp(float v) { return ::expf(v); }
inline float log(float v) { return ::logf(v); }
inline float sqrt(float v) { return ::sqrtf(v); }
inline float tanh(float v) { return ::tanhf(v); }
inline float pow(float a, float b) { return ::powf(a, b); }
inline float expm1(float v) { return ::expm1f(v); }
inline float fabs(float v) { return ::fabsf(v); }
inline float sin(float v) { return ::sinf(v); }
inline float cos(float v) { return ::cosf(v); }
inline float fmax(float a, float b) { return ::fmaxf(a, b); }
inline float fmin(float a, float b) { return ::fminf(a, b); }
inline float2 sqrt(const float2 &v) { return float2(::sqrtf(v.x), ::sqrtf(v.y)); }
inline float4 sqrt(const float4 &v) { return float4(::sqrtf(v.x), ::sqrtf(v.y), ::sqrtf(v.z), ::sqrtf(v.w)); }
inline float2 exp(const float2 &v) { return float2(::expf(v.x), ::expf(v.y)); }
inline float4 exp(const float4 &v) { return float4(::expf(v.x), ::expf(v.y), ::expf(v.z), ::expf(v.w)); }
inline int isnan(float v) { return std::isnan(v) ? 1 : 0; }
inline int isinf(float v) { return std::isinf(v) ? 1 : 0; }
inline int isfinite(float v) { return std::isfinite(v) ? 1 : 0; }
// OpenCL sign(): 1, -1, +-0 for +-0, 0 for NaN.
inline float sign(float v) {
  if (std::isnan(v)) return 0.f;
  if (v > 0.f) return 1.f;
  if (v < 0.f) return -1.f;
  return v;
}
inline float2 sign(const float2 &v) { return float2(sign(v.x), sign(v.y)); }
inline float4 sign(const float4 &v) { return float4(sign(v.x), sign(v.y), sign(v.z), sign(v.w)); }
// OpenCL clamp(x, lo, hi) = min(max(x, lo), hi) (fmin/fmax for floats).
inline float clamp(float v, float lo, float hi) { return ::fminf(::fmaxf(v, lo), hi); }
inline float2 clamp(const float2 &v, float lo, float hi) { return float2(clamp(v.x, lo, hi), clamp(v.y, lo, hi)); }
inline float4 clamp(const float4 &v, float lo, float hi) {
  return float4(clamp(v.x, lo, hi), clamp(v.y, lo, hi), clamp(v.z, lo, hi), clamp(v.w, lo, hi));
}
inline float dot(const float4 &a, const float4 &b) { return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w; }
inline float dot(const float2 &a, const float2 &b) { return a.x * b.x + a.y * b.y; }
inline float dot(float a, float b) { return a * b; }
// integer / float min-max as OpenCL overloads: float if either side is float.
inline float max(float a, float b) { return ::fmaxf(a, b); }
inline float min(float a, float b) { return ::fminf(a, b); }
inline int max(int a, int b) { return a > b ? a : b; }
inline int min(int a, int b) { return a < b ? a : b; }
inline uint max(uint a, uint b) { return a > b ? a : b; }
inline uint min(uint a, uint b) { return a < b ? a : b; }
inline long max(long a, long b) { return a > b ? a : b; }
inline long min(long a, long b) { return a < b ? a : b; }
inline ulong max(ulong a, ulong b) { return a > b ? a : b; }
inline ulong min(ulong a, ulong b) { return a < b ? a : b; }
inline long max(int a, long b) { return max((long)a, b); }
inline long max(long a, int b) { return max(a, (long)b); }
inline long min(int a, long b) { return min((long)a, b); }
inline long min(long a, int b) { return min(a, (long)b); }
inline ulong min(ulong a, uint b) { return min(a, (ulong)b); }
inline ulong min(uint a, ulong b) { return min((ulong)a, b); }
inline ulong max(ulong a, uint b) { return max(a, (ulong)b); }
inline ulong max(uint a, ulong b) { return max((ulong)a, b); }
inline long min(int a, uint b) { return min((long)a, (long)b); }
inline long min(uint a, int b) { return min((long)a, (long)b); }
inline long max(int a, uint b) { return max((long)a, (long)b); }
inline long max(uint a, int b) { return max((long)a, (long)b); }
inline ulong min(ulong a, int b) { return min(a, (ulong)b); }
inline ulong min(int a, ulong b) { return min((ulong)a, b); }
inline ulong max(ulong a, int b) { return max(a, (ulong)b); }
inline ulong max(int a, ulong b) { return max((ulong)a, b); }
inline float nan(uint) { return NAN; }

// ------------------------------------------------------------ NDRange state
struct WorkItem {
  size_t lid[3];
  size_t gid[3];
  ucontext_t uc;
  bool done;
  std::vector<char> stack;
};
struct NDRange {
  uint dims;
  size_t global[3];
  size_t local[3];
  size_t group[3];
  WorkItem *cur;
  ucontext_t sched;
  bool fibers;
};
extern thread_local NDRange g_nd;

inline uint get_work_dim() { return g_nd.dims; }
inline size_t get_global_size(uint d) { return d < 3 ? g_nd.global[d] : 1; }
inline size_t get_local_size(uint d) { return d < 3 ? g_nd.local[d] : 1; }
inline size_t get_num_groups(uint d) { return d < 3 ? g_nd.global[d] / g_nd.local[d] : 1; }
inline size_t get_group_id(uint d) { return d < 3 ? g_nd.group[d] : 0; }
inline size_t get_global_id(uint d) { return d < 3 ? g_nd.cur->gid[d] : 0; }
inline size_t get_local_id(uint d) { return d < 3 ? g_nd.cur->lid[d] : 0; }
inline void barrier(int) {
  if (g_nd.fibers) swapcontext(&g_nd.cur->uc, &g_nd.sched);
}
inline void mem_fence(int) {}

}  // namespace ocl
