// Flash multi-head attention of the reference's newer attention layers (CCrossMHFlashAttention and
// the layers built on it):
//   MHFlashAttention      out = softmax(q k^T / sqrt(d)) v per head, online over the keys, and the
//                         log-sum-exp of every row                               NeuroNet.cl:16066-16177
//   MHFlashAttentionGrad  query, key and value gradients from the saved log-sum-exp
//                                                                                NeuroNet.cl:16182-16277
// Layouts: query / output [q][heads][d], key_value [k][2 heads][d] (keys in heads 0..H-1, values in
// H..2H-1), logsumexp [q][heads].  With mask_future a query q sees the keys k >= q (the reference's
// test is q_id <= k_id).  Forward NDRange (queries, local, heads) with local (1, local, 1): only the
// first `local` features of each output row are written; gradient NDRange (rows, d, heads), the
// gradients written for the first `rows` queries and keys (the reference's host passes
// max(queries, keys)).
//
// Reference arithmetic kept: forward scores sum IsNaNOrInf(dot) over float4 groups of the features
// (operands sanitised), each value enters as IsNaNOrInf(p * v), the running sums are sanitised
// after every key tile; the gradient uses p = IsNaNOrInf(exp(clamp(s - lse, -120, 0))), skips pairs
// with p == 0, and sanitises every product and sum as the reference does.
//
// B200 layout: SIMT fp32 (the reference's semantics are per-element sanitised sums).  A group of
// TPQ lanes owns one row (a query, or a key in the key/value pass) with DPT features each; key (or
// query) tiles are staged in shared memory and each score is reduced across the group by
// shuffles.  The forward rescales once per tile with the tile's maximum.  The gradient runs a query
// pass (which also saves D_q = sum g o) and a key/value pass.  Batches: every buffer per sample.
#include <cfloat>

#include "../../include/nn_b200.h"
#include "nn_device.cuh"
#include "nn_internal.h"

namespace nn {
namespace {

constexpr int kFlashThreads = 128;

// sum_i IsNaNOrInf(a_i b_i, 0) over n features, for sanitised (finite) operands.  Products are
// rounded on their own, so one that overflows makes the plain sum non-finite; only then are the
// products sanitised one by one.
template <int N>
__device__ __forceinline__ float dot_sanitised(const float *a, const float *b) {
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i) s = __fadd_rn(s, __fmul_rn(a[i], b[i]));
  if (!isfinite(s)) {
    s = 0.f;
#pragma unroll
    for (int i = 0; i < N; ++i) s += nan0(__fmul_rn(a[i], b[i]));
  }
  return s;
}

template <int TPQ>
__device__ __forceinline__ float group_sum(float x) {
#pragma unroll
  for (int o = TPQ / 2; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Stage rows [r0, r0 + KT) of a matrix whose rows are `stride` floats apart (features 0 .. D-1 from
// `base`) into tile[KT][DP], zero-padded; `sanitise` applies IsNaNOrInf(., 0).
template <int KT, int DP>
__device__ __forceinline__ void stage_rows(float *tile, const float *base, long long stride, int r0, int rows, int D,
                                           bool sanitise) {
  for (int e = threadIdx.x; e < KT * DP; e += kFlashThreads) {
    const int j = e / DP, d = e - j * DP;
    float x = 0.f;
    if (r0 + j < rows && d < D) x = base[(long long)(r0 + j) * stride + d];
    tile[e] = sanitise ? nan0(x) : x;
  }
}

template <int TPQ, int DPT, int KT>
__global__ void __launch_bounds__(kFlashThreads) flash_fwd_kernel(const float *__restrict__ query,
                                                                  const float *__restrict__ kv, float *__restrict__ lse,
                                                                  float *__restrict__ out, int Q, int KV, int H, int D,
                                                                  int loc, int mask) {
  constexpr int DP = TPQ * DPT, QB = kFlashThreads / TPQ;
  __shared__ __align__(16) float ks[KT * DP];
  __shared__ __align__(16) float vs[KT * DP];
  const int h = blockIdx.y, b = blockIdx.z;
  const int t = threadIdx.x % TPQ, qi = blockIdx.x * QB + threadIdx.x / TPQ;
  const bool row_ok = qi < Q;
  const float *qrow = query + (((long long)b * Q + (row_ok ? qi : 0)) * H + h) * D;
  const float *kvb = kv + (long long)b * KV * 2 * H * D;
  float qr[DPT], acc[DPT];
#pragma unroll
  for (int j = 0; j < DPT; ++j) {
    const int d = t * DPT + j;
    qr[j] = (row_ok && d < D) ? nan0(qrow[d]) : 0.f;
    acc[j] = 0.f;
  }
  const float rs = 1.f / sqrtf((float)D);  // scores scaled by 1/sqrt(d)
  float m = -FLT_MAX, sumexp = 0.f;
  for (int k0 = 0; k0 < KV; k0 += KT) {
    __syncthreads();
    stage_rows<KT, DP>(ks, kvb + (long long)h * D, 2LL * H * D, k0, KV, D, true);
    // values sanitised here: with p in [0, 1], p * IsNaNOrInf(v) is IsNaNOrInf(p * v)
    stage_rows<KT, DP>(vs, kvb + (long long)(H + h) * D, 2LL * H * D, k0, KV, D, true);
    __syncthreads();
    float sc[KT];
    float tmax = -FLT_MAX;
#pragma unroll
    for (int j = 0; j < KT; ++j) {
      const float *kr = ks + j * DP + t * DPT;
      // float4 groups of products, rounded on their own: a group that is not finite makes the
      // plain sum non-finite, and only then is each group sanitised as the reference does
      float grp[DPT / 4], part = 0.f;
#pragma unroll
      for (int g = 0; g < DPT; g += 4) {
        grp[g / 4] = __fadd_rn(__fadd_rn(__fmul_rn(qr[g], kr[g]), __fmul_rn(qr[g + 1], kr[g + 1])),
                               __fadd_rn(__fmul_rn(qr[g + 2], kr[g + 2]), __fmul_rn(qr[g + 3], kr[g + 3])));
        part = __fadd_rn(part, grp[g / 4]);
      }
      if (!isfinite(part)) {
        part = 0.f;
#pragma unroll
        for (int g = 0; g < DPT / 4; ++g) part += nan0(grp[g]);
      }
      const float s = group_sum<TPQ>(part) * rs;
      const int kid = k0 + j;
      const bool ok = kid < KV && (mask == 0 || qi <= kid);
      sc[j] = ok ? s : -FLT_MAX;
      tmax = fmaxf(tmax, sc[j]);
    }
    if (tmax == -FLT_MAX) continue;  // every key of the tile masked: nothing changes
    const float mnew = fmaxf(m, tmax);
    const float scale = expf(m - mnew);
    float psum = 0.f;
#pragma unroll
    for (int j = 0; j < KT; ++j) {
      sc[j] = sc[j] > -FLT_MAX ? expf(sc[j] - mnew) : 0.f;
      psum += sc[j];
    }
    sumexp = nan0(scale * sumexp + psum);
#pragma unroll
    for (int i = 0; i < DPT; ++i) {
      float v = 0.f;
#pragma unroll
      for (int j = 0; j < KT; ++j) v = fmaf(sc[j], vs[j * DP + t * DPT + i], v);
      acc[i] = nan0(scale * acc[i] + v);
    }
    m = mnew;
  }
  if (!row_ok) return;
  float *orow = out + (((long long)b * Q + qi) * H + h) * D;
#pragma unroll
  for (int i = 0; i < DPT; ++i) {
    const int d = t * DPT + i;
    if (d < D && d < loc) orow[d] = sumexp > 0.f ? nan0(acc[i] / sumexp) : 0.f;
  }
  if (t == 0) lse[((long long)b * Q + qi) * H + h] = sumexp > 0.f ? nan0(m + logf(sumexp)) : 0.f;
}

// Query pass over every query: saves D_q, and for the first `qwrite` queries writes
// grad_q = sum_k IsNaNOrInf(k ds), ds = IsNaNOrInf(p (dp - D_q)).
template <int TPQ, int DPT, int KT>
__global__ void __launch_bounds__(kFlashThreads) flash_grad_q_kernel(
    const float *__restrict__ query, float *__restrict__ qgr, const float *__restrict__ kv,
    const float *__restrict__ lse, const float *__restrict__ out, const float *__restrict__ ogr,
    float *__restrict__ dsave, int Q, int qwrite, int KV, int H, int D, int mask) {
  constexpr int DP = TPQ * DPT, QB = kFlashThreads / TPQ;
  __shared__ __align__(16) float ks[KT * DP];
  __shared__ __align__(16) float vs[KT * DP];
  const int h = blockIdx.y, b = blockIdx.z;
  const int t = threadIdx.x % TPQ, qi = blockIdx.x * QB + threadIdx.x / TPQ;
  const bool row_ok = qi < Q;
  const long long row = ((long long)b * Q + (row_ok ? qi : 0)) * H + h;
  const float *kvb = kv + (long long)b * KV * 2 * H * D;
  float qr[DPT], gr[DPT], acc[DPT];
  float dpart = 0.f;
#pragma unroll
  for (int j = 0; j < DPT; ++j) {
    const int d = t * DPT + j;
    const bool ok = row_ok && d < D;
    qr[j] = ok ? nan0(query[row * D + d]) : 0.f;
    gr[j] = ok ? nan0(ogr[row * D + d]) : 0.f;
    dpart += nan0(gr[j] * (ok ? nan0(out[row * D + d]) : 0.f));
    acc[j] = 0.f;
  }
  const float Dq = group_sum<TPQ>(dpart);
  const float l = row_ok ? nan0(lse[row]) : 0.f;
  const float rs = 1.f / sqrtf((float)D);  // scores scaled by 1/sqrt(d)
  for (int k0 = 0; k0 < KV; k0 += KT) {
    __syncthreads();
    stage_rows<KT, DP>(ks, kvb + (long long)h * D, 2LL * H * D, k0, KV, D, true);
    stage_rows<KT, DP>(vs, kvb + (long long)(H + h) * D, 2LL * H * D, k0, KV, D, true);
    __syncthreads();
#pragma unroll 4
    for (int j = 0; j < KT; ++j) {
      const float *kr = ks + j * DP + t * DPT;
      const float *vr = vs + j * DP + t * DPT;
      const float s = group_sum<TPQ>(dot_sanitised<DPT>(qr, kr)) * rs;
      const float dp = group_sum<TPQ>(dot_sanitised<DPT>(gr, vr));
      const int kid = k0 + j;
      const float p = nan0(expf(fminf(fmaxf(s - l, -120.f), 0.f)));
      if (kid < KV && (mask == 0 || qi <= kid) && p != 0.f) {
        const float ds = nan0(p * (dp - Dq));
#pragma unroll
        for (int i = 0; i < DPT; ++i) acc[i] += nan0(kr[i] * ds);
      }
    }
  }
  if (!row_ok) return;
  if (t == 0) dsave[row] = Dq;
  if (qi >= qwrite) return;
#pragma unroll
  for (int i = 0; i < DPT; ++i) {
    const int d = t * DPT + i;
    if (d < D) qgr[row * D + d] = nan0(acc[i]);
  }
}

// Key/value pass over the first `kwrite` keys: grad_k = sum_q IsNaNOrInf(q ds),
// grad_v = sum_q IsNaNOrInf(p g).
template <int TPQ, int DPT, int KT>
__global__ void __launch_bounds__(kFlashThreads) flash_grad_kv_kernel(
    const float *__restrict__ query, const float *__restrict__ kv, float *__restrict__ kvgr,
    const float *__restrict__ lse, const float *__restrict__ ogr, const float *__restrict__ dsave, int Q, int KV,
    int kwrite, int H, int D, int mask) {
  constexpr int DP = TPQ * DPT, QB = kFlashThreads / TPQ;
  __shared__ __align__(16) float qs[KT * DP];
  __shared__ __align__(16) float gs[KT * DP];
  __shared__ float ls[KT], dq[KT];
  const int h = blockIdx.y, b = blockIdx.z;
  const int t = threadIdx.x % TPQ, ki = blockIdx.x * QB + threadIdx.x / TPQ;
  const bool row_ok = ki < kwrite;
  const long long krow = ((long long)b * KV + (row_ok ? ki : 0)) * 2 * H;
  const float *qb = query + (long long)b * Q * H * D;
  const float *gb = ogr + (long long)b * Q * H * D;
  float kr[DPT], vr[DPT], gk[DPT], gv[DPT];
#pragma unroll
  for (int j = 0; j < DPT; ++j) {
    const int d = t * DPT + j;
    const bool ok = row_ok && d < D;
    kr[j] = ok ? nan0(kv[(krow + h) * D + d]) : 0.f;
    vr[j] = ok ? nan0(kv[(krow + H + h) * D + d]) : 0.f;
    gk[j] = gv[j] = 0.f;
  }
  const float rs = 1.f / sqrtf((float)D);  // scores scaled by 1/sqrt(d)
  for (int q0 = 0; q0 < Q; q0 += KT) {
    __syncthreads();
    stage_rows<KT, DP>(qs, qb + (long long)h * D, (long long)H * D, q0, Q, D, true);
    stage_rows<KT, DP>(gs, gb + (long long)h * D, (long long)H * D, q0, Q, D, true);
    if (threadIdx.x < KT) {
      const int qi = q0 + threadIdx.x;
      const long long r = ((long long)b * Q + qi) * H + h;
      ls[threadIdx.x] = qi < Q ? nan0(lse[r]) : 0.f;
      dq[threadIdx.x] = qi < Q ? dsave[r] : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int j = 0; j < KT; ++j) {
      const float *qr = qs + j * DP + t * DPT;
      const float *gr = gs + j * DP + t * DPT;
      const float s = group_sum<TPQ>(dot_sanitised<DPT>(qr, kr)) * rs;
      const float dp = group_sum<TPQ>(dot_sanitised<DPT>(gr, vr));
      const int qi = q0 + j;
      const float p = nan0(expf(fminf(fmaxf(s - ls[j], -120.f), 0.f)));
      if (qi < Q && (mask == 0 || qi <= ki) && p != 0.f) {
        const float ds = nan0(p * (dp - dq[j]));
#pragma unroll
        for (int i = 0; i < DPT; ++i) {
          gk[i] += nan0(qr[i] * ds);
          gv[i] = fmaf(p, gr[i], gv[i]);  // p in [0, 1], g sanitised: the product is finite
        }
      }
    }
  }
  if (!row_ok) return;
#pragma unroll
  for (int i = 0; i < DPT; ++i) {
    const int d = t * DPT + i;
    if (d < D) {
      kvgr[(krow + h) * D + d] = nan0(gk[i]);
      kvgr[(krow + H + h) * D + d] = nan0(gv[i]);
    }
  }
}

// (lanes per row, features per lane, rows per staged tile) for a head dimension; false past 1024.
// Fewer lanes per row repeat less of the per-score work (scale, exponent, mask) across the group.
// Each configuration stages 16 KB or less per operand pair.
template <class F>
bool flash_dispatch(int D, F &&f) {
  using std::integral_constant;
  if (D <= 32) f(integral_constant<int, 1>{}, integral_constant<int, 32>{}, integral_constant<int, 32>{});
  else if (D <= 64) f(integral_constant<int, 2>{}, integral_constant<int, 32>{}, integral_constant<int, 32>{});
  else if (D <= 128) f(integral_constant<int, 8>{}, integral_constant<int, 16>{}, integral_constant<int, 16>{});
  else if (D <= 256) f(integral_constant<int, 16>{}, integral_constant<int, 16>{}, integral_constant<int, 8>{});
  else if (D <= 512) f(integral_constant<int, 32>{}, integral_constant<int, 16>{}, integral_constant<int, 4>{});
  else if (D <= 1024) f(integral_constant<int, 32>{}, integral_constant<int, 32>{}, integral_constant<int, 2>{});
  else return false;
  return true;
}

int k_flash(Launch &L) {
  const int Q = (int)L.nd.g[0], loc = L.nd.dims > 1 ? (int)L.nd.g[1] : 1;
  const int H = L.nd.dims > 2 ? (int)L.nd.g[2] : 1;
  const int D = L.i(4), KV = L.i(5), mask = L.i(6);
  if (D <= 0 || KV < 0) return L.fail(NN_ERR_ARG, "MHFlashAttention: bad dimension or total_kv");
  float *q = L.buf(0, (size_t)L.B * Q * H * D), *kv = L.buf(1, (size_t)L.B * KV * 2 * H * D);
  float *lse = L.buf(2, (size_t)L.B * Q * H), *out = L.buf(3, (size_t)L.B * Q * H * D);
  if (!q || !kv || !lse || !out) return NN_ERR_BOUNDS;
  const bool ok = flash_dispatch(D, [&](auto TPQ, auto DPT, auto KT) {
    constexpr int tpq = decltype(TPQ)::value, QB = kFlashThreads / tpq;
    flash_fwd_kernel<tpq, decltype(DPT)::value, decltype(KT)::value>
        <<<dim3((Q + QB - 1) / QB, H, L.B), kFlashThreads, 0, L.stream>>>(q, kv, lse, out, Q, KV, H, D, loc, mask);
  });
  if (!ok) return L.fail(NN_ERR_UNSUPPORTED, "MHFlashAttention: head dimension above 1024");
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

int k_flash_grad(Launch &L) {
  const int rows = (int)L.nd.g[0], gd = L.nd.dims > 1 ? (int)L.nd.g[1] : 1;
  const int H = L.nd.dims > 2 ? (int)L.nd.g[2] : 1;
  const int D = L.i(7), Qt = L.i(8), KVt = L.i(9), mask = L.i(10);
  if (D <= 0 || Qt < 0 || KVt < 0) return L.fail(NN_ERR_ARG, "MHFlashAttentionGrad: bad sizes");
  if (gd != D) return L.fail(NN_ERR_UNSUPPORTED, "MHFlashAttentionGrad: global[1] must equal the dimension");
  const int qwrite = rows < Qt ? rows : Qt, kwrite = rows < KVt ? rows : KVt;
  const size_t nq = (size_t)L.B * Qt * H * D, nkv = (size_t)L.B * KVt * 2 * H * D;
  float *q = L.buf(0, nq), *qg = L.buf(1, nq), *kv = L.buf(2, nkv), *kvg = L.buf(3, nkv);
  float *lse = L.buf(4, (size_t)L.B * Qt * H), *out = L.buf(5, nq), *og = L.buf(6, nq);
  if (!q || !qg || !kv || !kvg || !lse || !out || !og) return NN_ERR_BOUNDS;
  float *dsave = L.scratch(0, (size_t)L.B * Qt * H + 1);
  if (!dsave) return L.fail(NN_ERR_CUDA, "MHFlashAttentionGrad: scratch allocation failed");
  // the query pass covers every query (the key/value pass reads D_q of each)
  const bool ok = flash_dispatch(D, [&](auto TPQ, auto DPT, auto KT) {
    constexpr int tpq = decltype(TPQ)::value, dpt = decltype(DPT)::value, kt = decltype(KT)::value;
    constexpr int QB = kFlashThreads / tpq;
    if (Qt > 0)
      flash_grad_q_kernel<tpq, dpt, kt><<<dim3((Qt + QB - 1) / QB, H, L.B), kFlashThreads, 0, L.stream>>>(
          q, qg, kv, lse, out, og, dsave, Qt, qwrite, KVt, H, D, mask);
    if (kwrite > 0)
      flash_grad_kv_kernel<tpq, dpt, kt><<<dim3((kwrite + QB - 1) / QB, H, L.B), kFlashThreads, 0, L.stream>>>(
          q, kv, kvg, lse, og, dsave, Qt, KVt, kwrite, H, D, mask);
  });
  if (!ok) return L.fail(NN_ERR_UNSUPPORTED, "MHFlashAttentionGrad: head dimension above 1024");
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
  L.counted((Qt > 0 ? 1 : 0) + (kwrite > 0 ? 1 : 0));
  return NN_OK;
}

}  // namespace

const KernelDef kFlashKernels[] = {
    {"MHFlashAttention", "ppppiii", k_flash, false},
    {"MHFlashAttentionGrad", "pppppppiiii", k_flash_grad, false},
};
const int kNumFlashKernels = sizeof(kFlashKernels) / sizeof(kFlashKernels[0]);

}  // namespace nn
