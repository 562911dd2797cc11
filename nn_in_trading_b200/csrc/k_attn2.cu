// Remaining attention kernels: the single-head attention of CNeuronAttentionOCL
// (AttentionScore, AttentionOut, AttentionInsideGradients) and the two-axis
// multi-head attention of CNeuronMH2AttentionOCL (MH2AttentionOut,
// MH2AttentionInsideGradients).  Not on the benchmark's path: straightforward
// SIMT kernels, one thread or one warp per output row.
#include "../../include/nn_b200.h"
#include "nn_device.cuh"
#include "nn_internal.h"

namespace nn {

// ------------------------------------------------------ AttentionScore
// NeuroNet.cl:1237-1275: S[q,k] = exp(q.k/sqrt(d)) (NaN -> 0), masked k > q -> 0,
// divided by the row sum when it is positive.  One warp per query row.
__global__ void att_score_kernel(const float *q, const float *k, float *s, int U, int D, int mask, float koef,
                                 int B) {
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= B * U) return;
  int b = warp / U, qi = warp % U;
  const float *qr = q + ((size_t)b * U + qi) * D;
  const float *kb = k + (size_t)b * U * D;
  float *row = s + ((size_t)b * U + qi) * U;
  float sum = 0.f;
  for (int kk = lane; kk < U; kk += 32) {
    float r = 0.f;
    if (!(mask > 0 && kk > qi)) {
      float acc = 0.f;
      for (int i = 0; i < D; ++i) acc += qr[i] * kb[(size_t)kk * D + i];
      r = nan0(expf(acc / koef));
      sum += r;
    }
    row[kk] = r;
  }
  sum = warp_sum(sum);
  __syncwarp();
  if (sum > 0.f)
    for (int kk = lane; kk < U; kk += 32) row[kk] /= sum;
}

static int k_attention_score(Launch &L) {
  const int U = (int)L.nd.g[0], D = L.i(3), mask = L.i(4);
  if (D < 0) return L.fail(NN_ERR_ARG, "AttentionScore: negative dimension");
  float *q = L.buf(0, (size_t)L.B * U * D), *k = L.buf(1, (size_t)L.B * U * D), *s = L.buf(2, (size_t)L.B * U * U);
  if (!q || !k || !s) return NN_ERR_BOUNDS;
  float koef = fmaxf(sqrtf((float)D), 1.f);
  att_score_kernel<<<ceil_div((size_t)L.B * U * 32, 256), 256, 0, L.stream>>>(q, k, s, U, D, mask, koef, L.B);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

// -------------------------------------------------------- AttentionOut
// NeuroNet.cl:1286-1303: out[u,d] = nan0(sum_i nan0(S[u,i]) nan0(V[i,d])) + inputs[u,d].
__global__ void att_out_kernel(const float *s, const float *v, const float *in, float *out, int U, int D, int B) {
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)B * U * D) return;
  int d = (int)(t % D);
  size_t r = t / D;
  int u = (int)(r % U);
  size_t b = r / U;
  const float *srow = s + (b * U + u) * U;
  const float *vb = v + b * U * D;
  float acc = 0.f;
  for (int i = 0; i < U; ++i) acc += nan0(srow[i]) * nan0(vb[(size_t)i * D + d]);
  out[t] = nan0(acc) + in[t];
}

static int k_attention_out(Launch &L) {
  const int U = (int)L.nd.g[0], D = L.nd.dims > 1 ? (int)L.nd.g[1] : 1;
  size_t n = (size_t)L.B * U * D;
  float *s = L.buf(0, (size_t)L.B * U * U), *v = L.buf(1, n), *in = L.buf(2, n), *out = L.buf(3, n);
  if (!s || !v || !in || !out) return NN_ERR_BOUNDS;
  att_out_kernel<<<grid1d(n, 256), 256, 0, L.stream>>>(s, v, in, out, U, D, L.B);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

// --------------------------------------------- AttentionInsideGradients
// NeuroNet.cl:1395-1443: with P[u][i] = sum_e g[u,e] V[i,e] and f(s) = s(1-s) (1e-4 when s is 0 or 1):
//   vg[u,d] = sum_i S[i,u] g[i,d]
//   qg[u,d] = sum_i f(S[u,i]) P[u][i] K[i,d] / koef
//   kg[u,d] = sum_i f(S[i,u]) P[i][u] Q[i,d] / koef      each clamped to [-1, 1] after nan0.
__global__ void att_p_kernel(const float *g, const float *v, float *P, int U, int D, int B) {
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)B * U * U) return;
  int i = (int)(t % U);
  size_t r = t / U;
  int u = (int)(r % U);
  size_t b = r / U;
  const float *gr = g + (b * U + u) * D, *vr = v + (b * U + i) * D;
  float acc = 0.f;
  for (int e = 0; e < D; ++e) acc += vr[e] * gr[e];
  P[t] = acc;
}

__device__ __forceinline__ float att_f(float s) { return (s == 0.f || s == 1.f) ? 0.0001f : s * (1.f - s); }

__global__ void att_grad_kernel(const float *q, float *qg, const float *k, float *kg, float *vg, const float *s,
                                const float *g, const float *P, int U, int D, float koef, int B) {
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)B * U * D) return;
  int d = (int)(t % D);
  size_t r = t / D;
  int u = (int)(r % U);
  size_t b = r / U;
  const float *S = s + b * U * U, *G = g + b * U * D, *Pb = P + b * U * U;
  const float *Q = q + b * U * D, *K = k + b * U * D;
  float v_ = 0.f, q_ = 0.f, k_ = 0.f;
  for (int i = 0; i < U; ++i) {
    v_ += S[(size_t)i * U + u] * G[(size_t)i * D + d];
    q_ += att_f(S[(size_t)u * U + i]) * Pb[(size_t)u * U + i] * K[(size_t)i * D + d] / koef;
    k_ += att_f(S[(size_t)i * U + u]) * Pb[(size_t)i * U + u] * Q[(size_t)i * D + d] / koef;
  }
  vg[t] = clampf(nan0(v_), -1.f, 1.f);
  qg[t] = clampf(nan0(q_), -1.f, 1.f);
  kg[t] = clampf(nan0(k_), -1.f, 1.f);
}

static int k_attention_inside_gradients(Launch &L) {
  const int U = (int)L.nd.g[0], D = L.nd.dims > 1 ? (int)L.nd.g[1] : 1;
  size_t n = (size_t)L.B * U * D;
  float *q = L.buf(0, n), *qg = L.buf(1, n), *k = L.buf(2, n), *kg = L.buf(3, n), *v = L.buf(4, n);
  float *vg = L.buf(5, n), *s = L.buf(6, (size_t)L.B * U * U), *g = L.buf(7, n);
  if (!q || !qg || !k || !kg || !v || !vg || !s || !g) return NN_ERR_BOUNDS;
  float *P = L.scratch(2, (size_t)L.B * U * U);
  if (!P) return NN_ERR_CUDA;
  float koef = fmaxf(sqrtf((float)D), 1.f);
  att_p_kernel<<<grid1d((size_t)L.B * U * U, 256), 256, 0, L.stream>>>(g, v, P, U, D, L.B);
  NN_CHECK_LAUNCH(L);
  att_grad_kernel<<<grid1d(n, 256), 256, 0, L.stream>>>(q, qg, k, kg, vg, s, g, P, U, D, koef, L.B);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

// ------------------------------------------------------ MH2AttentionOut
// NeuroNet.cl:4252-4304.  q [Q][H][D], kv [K][2][Hkv][D] (keys then values), score [Q][H][K],
// out [Q][H][D]; head h reads kv head h % Hkv; max-subtracted softmax over the keys (masked keys
// k > q excluded); out = sum_k nan0(V[k] * score).  One warp per (sample, query, head).
__global__ void mh2_out_kernel(const float *q, const float *kv, float *score, float *out, int Qn, int Kn, int H,
                               int Hkv, int D, int mask, float koef, int B) {
  int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= B * Qn * H) return;
  int h = warp % H;
  int r = warp / H;
  int qi = r % Qn;
  int b = r / Qn;
  const int hk = h % Hkv;
  const float *qr = q + (((size_t)b * Qn + qi) * H + h) * D;
  const float *kvb = kv + (size_t)b * Kn * 2 * Hkv * D;
  float *srow = score + (((size_t)b * Qn + qi) * H + h) * Kn;
  float mx = kMinValue;
  for (int k = lane; k < Kn; k += 32) {
    float l = kMinValue;
    if (mask == 0 || qi >= k) {
      float acc = 0.f;
      const float *kr = kvb + ((size_t)k * 2 * Hkv + hk) * D;
      for (int d = 0; d < D; ++d) acc += qr[d] * kr[d];
      l = nan0(acc / koef, kMinValue);
    }
    srow[k] = l;  // logits first, probabilities below
    mx = fmaxf(mx, l);
  }
  mx = warp_max(mx);
  __syncwarp();
  float sum = 0.f;
  for (int k = lane; k < Kn; k += 32) {
    float l = srow[k];
    float e = (mx == kMinValue || l == kMinValue) ? 0.f : nan0(expf(l - mx));
    srow[k] = e;
    sum += e;
  }
  sum = nan0(warp_sum(sum));
  __syncwarp();
  for (int k = lane; k < Kn; k += 32) srow[k] = (mx == kMinValue || sum == 0.f) ? 0.f : nan0(srow[k] / sum);
  __syncwarp();
  float *orow = out + (((size_t)b * Qn + qi) * H + h) * D;
  for (int d = 0; d < D; ++d) {
    float acc = 0.f;
    for (int k = lane; k < Kn; k += 32) acc += nan0(kvb[((size_t)k * 2 * Hkv + Hkv + hk) * D + d] * srow[k]);
    acc = nan0(warp_sum(acc));
    if (lane == 0) orow[d] = acc;
  }
}

static int k_mh2_attention_out(Launch &L) {
  if (L.nd.dims < 3 || !L.nd.has_local) return L.fail(NN_ERR_ARG, "MH2AttentionOut: needs a 3-D NDRange with local size");
  const int Qn = (int)L.nd.g[0], Kn = (int)L.nd.l[1], H = (int)L.nd.g[2];
  if ((int)L.nd.g[1] != Kn) return L.fail(NN_ERR_UNSUPPORTED, "MH2AttentionOut: global size 1 must equal local size 1");
  const int D = L.i(4), Hkv = L.i(5), mask = L.i(6);
  if (D <= 0 || Hkv <= 0) return L.fail(NN_ERR_ARG, "MH2AttentionOut: bad dimension / heads_kv");
  float *q = L.buf(0, (size_t)L.B * Qn * H * D), *kv = L.buf(1, (size_t)L.B * Kn * 2 * Hkv * D);
  float *s = L.buf(2, (size_t)L.B * Qn * H * Kn), *out = L.buf(3, (size_t)L.B * Qn * H * D);
  if (!q || !kv || !s || !out) return NN_ERR_BOUNDS;
  float koef = fmaxf(sqrtf((float)D), 1.f);
  mh2_out_kernel<<<ceil_div((size_t)L.B * Qn * H * 32, 256), 256, 0, L.stream>>>(q, kv, s, out, Qn, Kn, H, Hkv, D,
                                                                                  mask, koef, L.B);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

// ------------------------------------------ MH2AttentionInsideGradients
// NeuroNet.cl:4307-4406, with its indexing as written:
//   dV[v,h,d] (h < Hkv) = sum_{hq = h, h+Hkv, ..} sum_g g[g,hq,d] S[g,hq,v]
//   dQ[q,h,d] = g'[q,h,d]/koef * sum_k S[q,h,k] (V[k,hk,d] - A[q,h,d]) K[k,hk,d],
//     g' read at gradient[(q+h)*D + d], A[q,h,d] = sum_v S[q,h,v] V[v,hk,d]
//   dK[k,h,d] (h < Hkv) = (H-h)/koef * V[k,h,d] * sum_r g[(h+r)*D+d] S[r,0,k] (1 - sum_v S[r,0,v])
//                          * q[D*(q0*H + h + r) + d],  q0 = k mod Q
// (the key gradient multiplies by 1 - sum of a softmax row: it is rounding-level by construction).
__global__ void mh2_grad_qv_kernel(const float *q, float *qg, const float *kv, float *kvg, const float *S,
                                   const float *g, int Qn, int Kn, int H, int Hkv, int D, float koef, int B) {
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)B * Qn * H * D) return;
  int d = (int)(t % D);
  size_t r = t / D;
  int h = (int)(r % H);
  r /= H;
  int qi = (int)(r % Qn);
  size_t b = r / Qn;
  const int hk = h % Hkv;
  const float *Sb = S + b * Qn * H * Kn;
  const float *gb = g + b * Qn * H * D;
  const float *kvb = kv + b * Kn * 2 * Hkv * D;
  // query gradient
  const float *srow = Sb + ((size_t)qi * H + h) * Kn;
  float a = 0.f;
  for (int v = 0; v < Kn; ++v) a += srow[v] * kvb[((size_t)v * 2 * Hkv + Hkv + hk) * D + d];
  float acc = 0.f;
  for (int k = 0; k < Kn; ++k) {
    float sc = srow[k];
    if (sc == 0.f) continue;
    acc += sc * (kvb[((size_t)k * 2 * Hkv + Hkv + hk) * D + d] - a) * kvb[((size_t)k * 2 * Hkv + hk) * D + d];
  }
  float outg = gb[(size_t)(qi + h) * D + d];
  qg[t] = outg * acc / koef;
  // value gradient (threads with h < Hkv own values v = qi, qi+Q, ...)
  if (h < Hkv) {
    float *kvgb = kvg + b * Kn * 2 * Hkv * D;
    for (int v = qi; v < Kn; v += Qn) {
      float s = 0.f;
      for (int hq = h; hq < H; hq += Hkv)
        for (int gg = 0; gg < Qn; ++gg) s += gb[((size_t)gg * H + hq) * D + d] * Sb[((size_t)gg * H + hq) * Kn + v];
      kvgb[((size_t)v * 2 * Hkv + Hkv + h) * D + d] = s;
    }
  }
}

__global__ void mh2_grad_k_kernel(const float *q, const float *kv, float *kvg, const float *S, const float *g,
                                  int Qn, int Kn, int H, int Hkv, int D, float koef, int B, size_t qstride) {
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)B * Kn * Hkv * D) return;
  int d = (int)(t % D);
  size_t r = t / D;
  int h = (int)(r % Hkv);
  r /= Hkv;
  int k = (int)(r % Kn);
  size_t b = r / Kn;
  const int q0 = k % Qn;
  const float *Sb = S + b * Qn * H * Kn;
  const float *gb = g + b * Qn * H * D;
  const float *qb = q + b * qstride;
  const float *kvb = kv + b * Kn * 2 * Hkv * D;
  const float val = kvb[((size_t)k * 2 * Hkv + Hkv + h) * D + d];
  float acc = 0.f;
  for (int scr = 0; scr < Qn; ++scr) {
    const float *row = Sb + (size_t)scr * Kn * H;  // head 0's row of query scr, as the reference indexes it
    float sc = row[k];
    if (sc == 0.f) continue;
    float tot = 0.f;
    for (int v = 0; v < Kn; ++v) tot += row[v];
    float scg = gb[(size_t)(h + scr) * D + d] * val * sc * (1.f - tot);
    acc += scg * qb[(size_t)D * ((size_t)q0 * H + h + scr) + d];
  }
  kvg[b * Kn * 2 * Hkv * D + ((size_t)k * 2 * Hkv + h) * D + d] = acc * (float)(H - h) / koef;
}

static int k_mh2_attention_inside_gradients(Launch &L) {
  const int Qn = (int)L.nd.g[0], D = L.nd.dims > 1 ? (int)L.nd.g[1] : 1, H = L.nd.dims > 2 ? (int)L.nd.g[2] : 1;
  const int Kn = L.i(6), Hkv = L.i(7);
  if (Kn <= 0 || Hkv <= 0 || Hkv > H) return L.fail(NN_ERR_ARG, "MH2AttentionInsideGradients: bad kunits / heads_kv");
  const size_t nq = (size_t)Qn * H * D, nkv = (size_t)Kn * 2 * Hkv * D;
  // the key-gradient loop reads q up to D*((Q-1)*(H+1) + Hkv) floats past each sample's start
  const size_t qneed = (size_t)D * ((size_t)(Qn - 1) * (H + 1) + Hkv);
  const size_t qstride = L.B > 1 ? nq : 0;
  float *q = L.buf(0, (size_t)(L.B - 1) * nq + std::max(nq, qneed)), *qg = L.buf(1, (size_t)L.B * nq);
  float *kv = L.buf(2, (size_t)L.B * nkv), *kvg = L.buf(3, (size_t)L.B * nkv);
  float *S = L.buf(4, (size_t)L.B * Qn * H * Kn), *g = L.buf(5, (size_t)L.B * nq);
  if (!q || !qg || !kv || !kvg || !S || !g) return NN_ERR_BOUNDS;
  if (L.B > 1 && qneed > nq)
    return L.fail(NN_ERR_UNSUPPORTED, "MH2AttentionInsideGradients: batched call whose key loop reads past a sample");
  float koef = fmaxf(sqrtf((float)D), 1.f);
  mh2_grad_qv_kernel<<<grid1d((size_t)L.B * nq, 256), 256, 0, L.stream>>>(q, qg, kv, kvg, S, g, Qn, Kn, H, Hkv, D,
                                                                          koef, L.B);
  NN_CHECK_LAUNCH(L);
  mh2_grad_k_kernel<<<grid1d((size_t)L.B * Kn * Hkv * D, 256), 256, 0, L.stream>>>(q, kv, kvg, S, g, Qn, Kn, H, Hkv,
                                                                                   D, koef, L.B, nq);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

const KernelDef kAttn2Kernels[] = {
    {"AttentionScore", "pppii", k_attention_score, false},
    {"AttentionOut", "pppp", k_attention_out, false},
    {"AttentionInsideGradients", "pppppppp", k_attention_inside_gradients, false},
    {"MH2AttentionOut", "ppppiii", k_mh2_attention_out, false},
    {"MH2AttentionInsideGradients", "ppppppii", k_mh2_attention_inside_gradients, false},
};
const int kNumAttn2Kernels = sizeof(kAttn2Kernels) / sizeof(kAttn2Kernels[0]);

}  // namespace nn
