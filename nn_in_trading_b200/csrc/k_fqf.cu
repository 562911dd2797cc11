// Quantile heads of the reference's distributional agents: CNeuronFQF (fully parameterised
// quantile function) and CNeuronSoftActorCritic's quantile-sampled actions.
//   FQF_Cosine             cos(pi i tau_i), tau_i = sum_{t<i} p_t + p_i / 2   NeuroNet.cl:2524-2538
//   FQF_Output             y = sum_i quantile_i dtau_i                        NeuroNet.cl:2543-2553
//   FQF_OutputGradient     quantile and tau gradients of y                   NeuroNet.cl:2560-2573
//   FQF_QuantileGradient   state and tau-embedding gradients of their product NeuroNet.cl:2579-2592
//   FQF_CosineGradient     softmax gradient through every tau_t, t >= i       NeuroNet.cl:2598-2624
//   FQF_CosineGradientSRM  the same for the spectral-risk head              NeuroNet.cl:2630-2651
//   FQF_DistributionTargetGradient  gradient into the quantile nearest a target  NeuroNet.cl:2663-2716
//   FQF_FractionGradient   input gradient of the fraction proposal layer     NeuroNet.cl:3207-3224
//   FQF_SRMForward         spectral risk of the quantile distribution        NeuroNet.cl:2924-3021
//   FQF_SRMGradient        its quantile and probability gradients            NeuroNet.cl:3027-3200
//   FQF_MonotoneRearrange  quantiles in ascending order, with diagnostics    NeuroNet.cl:20716-20817
//   FQF_RearrangeGradient  ordered gradients back to their source quantiles  NeuroNet.cl:20823-20842
//   FQF_Sample             one draw per row from the quantile distribution   NeuroNet.cl:2722-2799
//   SAC_AlphaLogProbs      sample a quantile by its probability, -alpha log p NeuroNet.cl:3903-3933
//   SAC_AlphaGradients     gradient of alpha                                 NeuroNet.cl:3939-3951
//   SAC_OutputGradient     gradient into the quantiles bracketing the action NeuroNet.cl:3957-4000
//   SAC_CalcLogProbs       -alpha log p of an action between two quantiles   NeuroNet.cl:4006-4036
// The FQF kernels run over (quants, actions): one warp per action, the running sums of the
// fractions as warp scans (the reference loops over the prefix in every work-item).  FQF_CosineGradient's
// inner loop is a suffix sum that does not depend on i, so it is one scan too.  The SAC kernels keep
// one thread per action and the reference's sequential searches (the sampled quantile is the first
// whose running probability reaches the random number, so the sums run in its order).
// Batches: every buffer is per sample (FQF_FractionGradient's weights are shared); a launch covers
// actions x batch rows.
#include <cfloat>

#include "../../include/nn_b200.h"
#include "nn_device.cuh"
#include "nn_internal.h"

namespace nn {
namespace {

constexpr float kPiF = 3.14159265358979f;
constexpr unsigned kFull = 0xffffffffu;

// Exclusive prefix of x over the lanes, and the chunk total.
__device__ __forceinline__ float warp_exclusive(float x, int lane, float *chunk_total) {
  float inc = x;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const float y = __shfl_up_sync(kFull, inc, d);
    if (lane >= d) inc += y;
  }
  *chunk_total = __shfl_sync(kFull, inc, 31);
  const float ex = __shfl_up_sync(kFull, inc, 1);
  return lane == 0 ? 0.f : ex;
}

__global__ void fqf_cosine_kernel(const float *__restrict__ sm, float *__restrict__ out, int total, long long rows) {
  const long long a = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (a >= rows) return;
  const float *s = sm + a * total;
  float carry = 0.f;
  for (int c0 = 0; c0 < total; c0 += 32) {
    const int i = c0 + lane;
    const float x = i < total ? s[i] : 0.f;
    float ct;
    const float ex = warp_exclusive(x, lane, &ct);
    if (i < total) out[a * total + i] = cosf((float)i * kPiF * (carry + ex + x / 2.0f));
    carry += ct;
  }
}

__global__ void fqf_output_kernel(const float *__restrict__ q, const float *__restrict__ dt, float *__restrict__ y,
                                  int total, long long rows) {
  const long long a = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (a >= rows) return;
  float s = 0.f;
  for (int i = lane; i < total; i += 32) s += q[a * total + i] * dt[a * total + i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
  if (lane == 0) y[a] = s;
}

// out1[e] = g[e / per] * in1[e], out2[e] = g[e / per] * in2[e]  (per = total: OutputGradient;
// per = 1: QuantileGradient, where g is itself per element)
__global__ void fqf_pair_grad_kernel(const float *__restrict__ in1, const float *__restrict__ in2,
                                     const float *__restrict__ g, float *__restrict__ out1, float *__restrict__ out2,
                                     int per, long long n) {
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
    const float gr = g[e / per];
    out1[e] = gr * in1[e];
    out2[e] = gr * in2[e];
  }
}

// softmax_gr[i] += -pi i sin(pi i tau_i) g_i + sum_{t>i} -pi t sin(pi t tau_t) g_t p_t / tau_t.
// The chunks of 32 fractions run from the last to the first so that the suffix sum is a running
// total (a term that is not finite reaches only the i below it, as in the reference); a chunk's
// starting tau is the row total less the later chunks (exactly 0 for rows of at most 32).
// SRM (FQF_CosineGradientSRM, NeuroNet.cl:2630-2651): the first term halved and the later terms
// without p_t / tau_t.
template <bool SRM>
__global__ void fqf_cosine_grad_kernel(const float *__restrict__ sm, const float *__restrict__ og,
                                       float *__restrict__ sg, int total, long long rows) {
  const long long a = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (a >= rows) return;
  const float *s = sm + a * total;
  const float *g = og + a * total;
  const int last = total > 0 ? (total - 1) / 32 * 32 : -32;
  float total_s = 0.f, ct;
  for (int c0 = 0; c0 <= last; c0 += 32) {
    const int i = c0 + lane;
    warp_exclusive(i < total ? s[i] : 0.f, lane, &ct);
    total_s += ct;
  }
  float after_s = 0.f, after_f = 0.f;
  for (int c0 = last; c0 >= 0; c0 -= 32) {
    const int i = c0 + lane;
    const float x = i < total ? s[i] : 0.f;
    const float ex = warp_exclusive(x, lane, &ct);
    const float tau = (total_s - after_s - ct) + ex + x / 2;
    const float fi = (float)i;
    const float gi = i < total ? g[i] : 0.f;
    const float sn = sinf(kPiF * fi * tau);
    const float first = SRM ? -0.5f * kPiF * fi * sn * gi : -kPiF * fi * sn * gi;
    const float f = i < total && i > 0 ? (SRM ? -kPiF * fi * sn * gi : -kPiF * fi * sn * gi * x / tau) : 0.f;
    float inc = f;  // inclusive suffix over the lanes
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const float y = __shfl_down_sync(kFull, inc, d);
      if (lane + d < 32) inc += y;
    }
    const float later = __shfl_down_sync(kFull, inc, 1);
    if (i < total) sg[a * total + i] += first + (after_f + (lane == 31 ? 0.f : later));
    after_f += __shfl_sync(kFull, inc, 0);
    after_s += ct;
  }
}

__global__ void sac_alpha_log_probs_kernel(float *__restrict__ out, const float *__restrict__ q,
                                           const float *__restrict__ probs, const float *__restrict__ alphas,
                                           float *__restrict__ lp, const float *__restrict__ rnd, int cq, int act,
                                           long long n) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float *p = probs + i * cq;
  const float r = rnd[i];
  float prob = 0.f, value = 0.f, sum = 0.f;
  for (int k = 0; k < cq; ++k) {
    prob = p[k];
    sum += prob;
    if (sum >= r || k == cq - 1) {
      value = q[i * cq + k];
      break;
    }
  }
  out[i] = activate(value, act);
  lp[i] = -alphas[i] * logf(prob);
}

__global__ void sac_alpha_grad_kernel(const float *__restrict__ out, const float *__restrict__ g,
                                      const float *__restrict__ lp, float *__restrict__ ag, int act, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    ag[i] = deactivate(-g[i] * lp[i], out[i], act);
}

__global__ void sac_output_grad_kernel(const float *__restrict__ q, const float *__restrict__ dt,
                                       const float *__restrict__ og, float *__restrict__ qg, float *__restrict__ tg,
                                       const float *__restrict__ out, int cq, int act, long long n) {
  const long long a = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (a >= n) return;
  const long long shift = a * cq;
  float q1 = -1e37f, q2 = 1e37f;
  long long p1 = -1, p2 = -1;
  const float v = out[a];
  for (int k = 0; k < cq; ++k) {
    const float qq = activate(q[shift + k], act);
    if (v >= qq && q1 < qq) {
      q1 = qq;
      p1 = shift + k;
    }
    if (v < qq && q2 > qq) {
      q2 = qq;
      p2 = shift + k;
    }
    qg[shift + k] = 0.f;
    tg[shift + k] = 0.f;
  }
  const float gr = og[a];
  if (q1 > -1e37f) {
    qg[p1] = gr * dt[p1];
    tg[p1] = gr * q1;
  }
  if (q2 < 1e37f) {
    qg[p2] = gr * dt[p2];
    tg[p2] = gr * q2;
  }
}

__global__ void sac_calc_log_probs_kernel(const float *__restrict__ out, const float *__restrict__ q,
                                          const float *__restrict__ probs, const float *__restrict__ alphas,
                                          float *__restrict__ lp, int cq, int act, long long n) {
  const long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (i >= n) return;
  float q1 = -1e37f, q2 = 1e37f, pr1 = 0.f, pr2 = 0.f;
  const float v = out[i];
  for (int k = 0; k < cq; ++k) {
    const float qq = activate(q[i * cq + k], act);
    if (v >= qq && q1 < qq) {
      q1 = qq;
      pr1 = probs[i * cq + k];
    }
    if (v < qq && q2 > qq) {
      q2 = qq;
      pr2 = probs[i * cq + k];
    }
  }
  float prob = fabsf(v - q1) / fabsf(q2 - q1);
  prob = fminf(fmaxf((1.f - prob) * pr1 + prob * pr2, 1.0e-3f), 1.0f);
  lp[i] = -alphas[i] * logf(prob);
}

// FQF_FractionGradient: input_gr[i] = IsNaNOrInf(sum_k W[k][i] g[k], 0), W rows of inputs + 1.
// Operands are summed as they are (a NaN weight zeroes the whole sum, as in the reference).  A CTA of
// 8 warps per 32 columns, the warps splitting k; blockIdx.y is the sample.
__global__ void __launch_bounds__(256) fqf_fraction_grad_kernel(const float *__restrict__ w,
                                                                const float *__restrict__ g,
                                                                float *__restrict__ ig, int inputs, int outputs) {
  __shared__ float part[8][33];
  const int col = blockIdx.x * 32 + (threadIdx.x & 31), wv = threadIdx.x >> 5;
  const float *gb = g + (size_t)blockIdx.y * outputs;
  float s = 0.f;
  if (col < inputs)
    for (int k = wv; k < outputs; k += 8) s += w[(size_t)k * (inputs + 1) + col] * gb[k];
  part[wv][threadIdx.x & 31] = s;
  __syncthreads();
  if (wv == 0 && col < inputs) {
#pragma unroll
    for (int j = 1; j < 8; ++j) s += part[j][threadIdx.x];
    ig[(size_t)blockIdx.y * inputs + col] = nan0(s);
  }
}

// FQF_DistributionTargetGradient: per row v, the quantile nearest the target (ties: the larger
// value, then the lower index) gets value_weight (target - z) and probability_weight / (p + 1e-37);
// every other entry 0, and the whole row 0 when the target or every quantile is not finite.  A
// warp per row, three reductions.
__global__ void fqf_dist_target_grad_kernel(const float *__restrict__ q, const float *__restrict__ pr,
                                            float *__restrict__ qg, float *__restrict__ pg, float target,
                                            float pw, float vw, int total, long long rows) {
  const long long v = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (v >= rows) return;
  const float *z = q + v * total;
  const bool tv = isfinite(target);
  float dmin = FLT_MAX;
  for (int i = lane; i < total; i += 32)
    if (tv && isfinite(z[i])) dmin = fminf(dmin, fabsf(z[i] - target));
  for (int o = 16; o > 0; o >>= 1) dmin = fminf(dmin, __shfl_xor_sync(kFull, dmin, o));
  float cmax = -FLT_MAX;
  bool any = false;
  for (int i = lane; i < total; i += 32)
    if (tv && isfinite(z[i]) && fabsf(z[i] - target) == dmin) {
      cmax = fmaxf(cmax, z[i]);
      any = true;
    }
  for (int o = 16; o > 0; o >>= 1) {
    cmax = fmaxf(cmax, __shfl_xor_sync(kFull, cmax, o));
    any |= __shfl_xor_sync(kFull, (int)any, o) != 0;
  }
  int kmin = total;
  if (any)
    for (int i = lane; i < total; i += 32)
      if (isfinite(z[i]) && z[i] == cmax) kmin = min(kmin, i);
  for (int o = 16; o > 0; o >>= 1) kmin = min(kmin, __shfl_xor_sync(kFull, kmin, o));
  for (int i = lane; i < total; i += 32) {
    const bool hit = tv && i == kmin;
    qg[v * total + i] = hit ? vw * (target - z[i]) : 0.f;
    pg[v * total + i] = hit ? pw / (nan0(pr[v * total + i]) + 1.0e-37f) : 0.f;
  }
}

// FQF_MonotoneRearrange: per row of `total` quants (a power of two up to 64, else nothing is
// written), the quantiles in ascending (value, index) order with their probabilities and source
// indices; a value that is not finite sorts as 3.4e37, a probability that is not finite or below 0
// as 0.  Six diagnostics per row: crossing rate and total magnitude (per adjacent pair), probability
// sum, min and max, and the count of invalid probabilities.  The reference sorts bitonically; the
// keys are distinct, so ranking each element by counting gives the same order.  A warp per row.
constexpr float kRefMaxValue = 3.4e37f;
__global__ void fqf_rearrange_kernel(const float *__restrict__ q, const float *__restrict__ pr,
                                     float *__restrict__ oq, float *__restrict__ op, float *__restrict__ ord,
                                     float *__restrict__ diag, int total, long long rows) {
  const long long task = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (task >= rows) return;
  const float *z = q + task * total;
  const float *p = pr + task * total;
  float cf = 0.f, cm = 0.f, ps = 0.f, pmin = FLT_MAX, pmax = -FLT_MAX, inv = 0.f;
  for (int i = lane; i < total; i += 32) {
    const float zi = isfinite(z[i]) ? z[i] : kRefMaxValue;
    const bool pbad = !isfinite(p[i]) || p[i] < 0.f;
    const float pi = pbad ? 0.f : p[i];
    if (i + 1 < total) {
      const float zn = isfinite(z[i + 1]) ? z[i + 1] : kRefMaxValue;
      cf += zn < zi ? 1.f : 0.f;
      cm += fmaxf(zi - zn, 0.f);
    }
    ps += pi;
    pmin = fminf(pmin, pi);
    pmax = fmaxf(pmax, pi);
    inv += pbad ? 1.f : 0.f;
    int rank = 0;
    for (int j = 0; j < total; ++j) {
      const float zj = isfinite(z[j]) ? z[j] : kRefMaxValue;
      rank += (zj < zi || (zj == zi && j < i)) ? 1 : 0;
    }
    oq[task * total + rank] = zi;
    op[task * total + rank] = pi;
    ord[task * total + rank] = (float)i;
  }
  for (int o = 16; o > 0; o >>= 1) {
    cf += __shfl_xor_sync(kFull, cf, o);
    cm += __shfl_xor_sync(kFull, cm, o);
    ps += __shfl_xor_sync(kFull, ps, o);
    pmin = fminf(pmin, __shfl_xor_sync(kFull, pmin, o));
    pmax = fmaxf(pmax, __shfl_xor_sync(kFull, pmax, o));
    inv += __shfl_xor_sync(kFull, inv, o);
  }
  if (lane == 0) {
    const float dinv = total > 1 ? 1.0f / (float)(total - 1) : 0.f;
    float *d = diag + task * 6;
    d[0] = cf * dinv;
    d[1] = cm * dinv;
    d[2] = ps;
    d[3] = pmin;
    d[4] = pmax;
    d[5] = inv;
  }
}

// FQF_RearrangeGradient: gradients of the ordered entries scattered back to their source index
// (an order entry that is not a valid index is skipped).
__global__ void fqf_rearrange_grad_kernel(const float *__restrict__ oqg, const float *__restrict__ opg,
                                          const float *__restrict__ ord, float *__restrict__ qg,
                                          float *__restrict__ pg, int total, long long n) {
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += (long long)gridDim.x * blockDim.x) {
    const float o = nan0(ord[e], -1.f);
    const int dst = (int)o;
    if (dst < 0 || dst >= total) continue;
    const long long row = e / total;
    qg[row * total + dst] = oqg[e];
    pg[row * total + dst] = opg[e];
  }
}

// SRMCumulative (NeuroNet.cl:2805-2850): the spectral risk measure's cumulative weight at tau for
// the reference's five risk types (mean, CVaR, mean-CVaR mix, exponential, dual power).
__device__ __forceinline__ float srm_cumulative(float u, int type, float param, float mean_w) {
  constexpr float kEps = 1.0e-6f;
  const float tau = fminf(fmaxf(u, 0.f), 1.f);
  switch (type) {
    case 0: return tau;
    case 1: {
      const float alpha = fminf(fmaxf(param, kEps), 1.f);
      return fminf(fmaxf(fminf(tau, alpha) / alpha, 0.f), 1.f);
    }
    case 2: {
      const float alpha = fminf(fmaxf(param, kEps), 1.f);
      const float omega = fminf(fmaxf(mean_w, 0.f), 1.f);
      return fminf(fmaxf(omega * tau + (1.f - omega) * fminf(tau, alpha) / alpha, 0.f), 1.f);
    }
    case 3: {
      const float lambda = fmaxf(param, 0.f);
      if (lambda <= kEps) return tau;
      return fminf(fmaxf(-expm1f(-lambda * tau) / -expm1f(-lambda), 0.f), 1.f);
    }
    case 4: {
      const float nu = fmaxf(param, 1.f);
      return fminf(fmaxf(1.f - powf(1.f - tau, nu), 0.f), 1.f);
    }
    default: return 0.f;
  }
}

// FQF_SRMForward: per row, the spectral risk of the quantile distribution: with P_i the running
// sum of the (sanitised, non-negative) probabilities and M the row's mass, sum_i z_i
// max(F(P_i / M) - F(P_{i-1} / M), 0); 0 when M <= 1e-37.  A warp per row, the running sum as a
// warp scan.
__global__ void fqf_srm_forward_kernel(const float *__restrict__ q, const float *__restrict__ pr,
                                       float *__restrict__ res, int type, float param, float mean_w, int total,
                                       long long rows) {
  const long long task = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (task >= rows) return;
  const float *p = pr + task * total;
  const float *z = q + task * total;
  float mass = 0.f, ct;
  for (int c0 = 0; c0 < total; c0 += 32) {
    const int i = c0 + lane;
    warp_exclusive(i < total ? fmaxf(nan0(p[i]), 0.f) : 0.f, lane, &ct);
    mass += ct;
  }
  if (!(nan0(mass) > 1.0e-37f)) {
    if (lane == 0) res[task] = 0.f;
    return;
  }
  const float inv = 1.0f / mass;
  float carry = 0.f, risk = 0.f;
  for (int c0 = 0; c0 < total; c0 += 32) {
    const int i = c0 + lane;
    const float x = i < total ? fmaxf(nan0(p[i]), 0.f) : 0.f;
    const float ex = warp_exclusive(x, lane, &ct);
    if (i < total) {
      const float hi = fminf(fmaxf((carry + ex + x) * inv, 0.f), 1.f);
      const float lo = i == 0 ? 0.f : fminf(fmaxf((carry + ex) * inv, 0.f), 1.f);
      const float w = fmaxf(srm_cumulative(hi, type, param, mean_w) - srm_cumulative(lo, type, param, mean_w), 0.f);
      risk += w * nan0(z[i]);
    }
    carry += ct;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) risk += __shfl_xor_sync(kFull, risk, o);
  if (lane == 0) res[task] = nan0(risk);
}

// FQF_Sample (NeuroNet.cl:2722-2799): per row (task), the running probability mass C_i of
// max(IsNaNOrInf(p_i), 0) and a uniform u = clamp(IsNaNOrInf(random[task], 0.5), 0, 1); the sample
// is the quantile of the smallest i with C_i >= u * C_last and C_{i-1} < u * C_last (the last one
// if none), 0 when C_last <= 1e-6.  The reference forms C with a Hillis-Steele scan in local
// memory (Temp[i] += Temp[i - d] for d = 1, 2, 4, ... below the row length); the selection
// compares C against the threshold, so this kernel adds in exactly that order to get the same
// rounded C: a warp per row, element i in lane i (a) and lane i - 32 (b), rows of at most 64.
__global__ void fqf_sample_kernel(const float *__restrict__ q, const float *__restrict__ pr,
                                  const float *__restrict__ rnd, float *__restrict__ res, int total, long long rows) {
  const long long task = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (task >= rows) return;
  const float *p = pr + task * total;
  float a = lane < total ? fmaxf(nan0(p[lane]), 0.f) : 0.f;
  float b = lane + 32 < total ? fmaxf(nan0(p[lane + 32]), 0.f) : 0.f;
  for (int d = 1; d < total; d <<= 1) {
    if (d < 32) {
      // every read of the step before any write, as the reference's barrier orders them
      const float a_lo = __shfl_up_sync(kFull, a, d);            // a[lane - d]
      const float b_lo = __shfl_up_sync(kFull, b, d);            // b[lane - d]
      const float a_wrap = __shfl_sync(kFull, a, (lane - d) & 31);  // a[lane - d + 32]
      if (lane >= d) a += a_lo;
      b += lane >= d ? b_lo : a_wrap;
    } else {
      b += a;  // d == 32: element lane + 32 adds element lane
    }
  }
  const float last_a = __shfl_sync(kFull, a, (total - 1) & 31);
  const float last_b = __shfl_sync(kFull, b, (total - 33) & 31);
  const float last = total <= 32 ? last_a : last_b;
  const float mass = nan0(last);
  if (mass <= 1.0e-6f) {
    if (lane == 0) res[task] = 0.f;
    return;
  }
  const float u = fminf(fmaxf(nan0(rnd[task], 0.5f), 0.f), 1.f);
  const float threshold = u * mass;
  // every lane executes every shuffle (a full-mask shuffle reached by only some lanes never completes)
  const float a_prev = __shfl_up_sync(kFull, a, 1);
  const float a_top = __shfl_sync(kFull, a, 31);
  const float b_up = __shfl_up_sync(kFull, b, 1);
  const float b_prev = lane == 0 ? a_top : b_up;
  int pick = total;
  {
    const int i = lane;
    bool sel = i < total && a >= threshold && (i == 0 || a_prev < threshold);
    if (i == total - 1 && a < threshold) sel = true;
    if (sel) pick = i;
  }
  {
    const int i = lane + 32;
    bool sel = i < total && b >= threshold && b_prev < threshold;
    if (i == total - 1 && b < threshold) sel = true;
    if (sel) pick = min(pick, i);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) pick = min(pick, __shfl_xor_sync(kFull, pick, o));
  if (lane == 0 && pick < total) res[task] = nan0(q[task * total + pick]);
}

// SRMDensity (NeuroNet.cl:2855-2900): the derivative of srm_cumulative in tau.
__device__ __forceinline__ float srm_density(float u, int type, float param, float mean_w) {
  constexpr float kEps = 1.0e-6f;
  const float tau = fminf(fmaxf(u, 0.f), 1.f);
  switch (type) {
    case 0: return 1.f;
    case 1: {
      const float alpha = fminf(fmaxf(param, kEps), 1.f);
      return tau < alpha ? 1.f / alpha : 0.f;
    }
    case 2: {
      const float alpha = fminf(fmaxf(param, kEps), 1.f);
      const float omega = fminf(fmaxf(mean_w, 0.f), 1.f);
      return tau < alpha ? omega + (1.f - omega) / alpha : omega;
    }
    case 3: {
      const float lambda = fmaxf(param, 0.f);
      if (lambda <= kEps) return 1.f;
      return fmaxf(lambda * expf(-lambda * tau) / -expm1f(-lambda), 0.f);
    }
    case 4: {
      const float nu = fmaxf(param, 1.f);
      if (nu == 1.f) return 1.f;
      return fmaxf(nu * powf(1.f - tau, nu - 1.f), 0.f);
    }
    default: return 0.f;
  }
}

// FQF_SRMGradient: per row with upstream gradient u (rows with u == 0 or no mass get zeros):
// quantile i gets u w_i (0 for a non-finite quantile); with b_i = u (z_i - z_{i+1}) F'(P_i / M) and
// S_i = sum_{j >= i} b_j, probability i gets (S_i - sum_j (p_j / M) S_j) / M (0 for a non-finite or
// negative probability).  A warp per row: the mass, then weights and b_i (held in the probability
// gradient), then S_i from the last chunk back with the correction sum, then the final values;
// each lane rereads only the entries it wrote.
__global__ void fqf_srm_grad_kernel(const float *__restrict__ q, const float *__restrict__ pr,
                                    const float *__restrict__ rg, float *__restrict__ qg, float *__restrict__ pg,
                                    int type, float param, float mean_w, int total, long long rows) {
  const long long task = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (task >= rows) return;
  const float *p = pr + task * total;
  const float *z = q + task * total;
  float *qo = qg + task * total;
  float *po = pg + task * total;
  const float up = nan0(rg[task]);
  float mass = 0.f, ct;
  for (int c0 = 0; c0 < total; c0 += 32) {
    const int i = c0 + lane;
    warp_exclusive(i < total ? fmaxf(nan0(p[i]), 0.f) : 0.f, lane, &ct);
    mass += ct;
  }
  mass = nan0(mass);
  if (up == 0.f || mass <= 1.0e-37f) {
    for (int i = lane; i < total; i += 32) qo[i] = po[i] = 0.f;
    return;
  }
  const float inv = 1.0f / mass;
  float carry = 0.f;
  for (int c0 = 0; c0 < total; c0 += 32) {
    const int i = c0 + lane;
    const float x = i < total ? fmaxf(nan0(p[i]), 0.f) : 0.f;
    const float ex = warp_exclusive(x, lane, &ct);
    if (i < total) {
      const float hi = fminf(fmaxf((carry + ex + x) * inv, 0.f), 1.f);
      const float lo = i == 0 ? 0.f : fminf(fmaxf((carry + ex) * inv, 0.f), 1.f);
      const float w = fmaxf(srm_cumulative(hi, type, param, mean_w) - srm_cumulative(lo, type, param, mean_w), 0.f);
      qo[i] = isfinite(z[i]) ? nan0(up * w) : 0.f;
      po[i] = i + 1 < total ? nan0(up * (nan0(z[i]) - nan0(z[i + 1])) * srm_density(hi, type, param, mean_w)) : 0.f;
    }
    carry += ct;
  }
  const int last = (total - 1) / 32 * 32;
  float after = 0.f, corr = 0.f;
  for (int c0 = last; c0 >= 0; c0 -= 32) {
    const int i = c0 + lane;
    float inc = i < total ? po[i] : 0.f;  // inclusive suffix over the lanes
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const float y = __shfl_down_sync(kFull, inc, d);
      if (lane + d < 32) inc += y;
    }
    if (i < total) {
      const float suffix = after + inc;
      po[i] = suffix;
      corr += (fmaxf(nan0(p[i]), 0.f) * inv) * suffix;
    }
    after += __shfl_sync(kFull, inc, 0);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) corr += __shfl_xor_sync(kFull, corr, o);
  for (int i = lane; i < total; i += 32) {
    const bool pv = isfinite(p[i]) && p[i] >= 0.f;
    po[i] = pv ? nan0((po[i] - corr) * inv) : 0.f;
  }
}

dim3 warp_grid(long long rows) { return dim3((unsigned)((rows * 32 + 255) / 256)); }

// (quants, actions) kernels: total = global[0], rows = actions x batch.
void quant_shape(const Launch &L, int *total, long long *rows) {
  *total = (int)L.nd.g[0];
  *rows = (long long)(L.nd.dims > 1 ? L.nd.g[1] : 1) * L.B;
}

int k_fqf_cosine(Launch &L) {
  int T;
  long long R;
  quant_shape(L, &T, &R);
  float *sm = L.buf(0, (size_t)R * T), *out = L.buf(1, (size_t)R * T);
  if (!sm || !out) return NN_ERR_BOUNDS;
  fqf_cosine_kernel<<<warp_grid(R), 256, 0, L.stream>>>(sm, out, T, R);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

int k_fqf_output(Launch &L) {
  const long long R = (long long)L.nd.g[0] * L.B;
  const int T = L.i(3);
  if (T < 0) return L.fail(NN_ERR_ARG, "FQF_Output: negative total");
  float *q = L.buf(0, (size_t)R * T), *dt = L.buf(1, (size_t)R * T), *y = L.buf(2, (size_t)R);
  if (!q || !dt || !y) return NN_ERR_BOUNDS;
  fqf_output_kernel<<<warp_grid(R), 256, 0, L.stream>>>(q, dt, y, T, R);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

int k_fqf_output_grad(Launch &L) {
  int T;
  long long R;
  quant_shape(L, &T, &R);
  const size_t n = (size_t)R * T;
  float *q = L.buf(0, n), *dt = L.buf(1, n), *og = L.buf(2, (size_t)R), *qg = L.buf(3, n), *tg = L.buf(4, n);
  if (!q || !dt || !og || !qg || !tg) return NN_ERR_BOUNDS;
  fqf_pair_grad_kernel<<<grid1d(n, 256), 256, 0, L.stream>>>(dt, q, og, qg, tg, T, (long long)n);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

int k_fqf_quantile_grad(Launch &L) {
  int T;
  long long R;
  quant_shape(L, &T, &R);
  const size_t n = (size_t)R * T;
  float *se = L.buf(0, n), *te = L.buf(1, n), *qg = L.buf(2, n), *sg = L.buf(3, n), *tg = L.buf(4, n);
  if (!se || !te || !qg || !sg || !tg) return NN_ERR_BOUNDS;
  fqf_pair_grad_kernel<<<grid1d(n, 256), 256, 0, L.stream>>>(te, se, qg, sg, tg, 1, (long long)n);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

template <bool SRM>
int k_fqf_cosine_grad(Launch &L) {
  int T;
  long long R;
  quant_shape(L, &T, &R);
  const size_t n = (size_t)R * T;
  float *sm = L.buf(0, n), *og = L.buf(1, n), *sg = L.buf(2, n);
  if (!sm || !og || !sg) return NN_ERR_BOUNDS;
  fqf_cosine_grad_kernel<SRM><<<warp_grid(R), 256, 0, L.stream>>>(sm, og, sg, T, R);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

int k_sac_alpha_log_probs(Launch &L) {
  const long long n = (long long)L.nd.g[0] * L.B;
  const int cq = L.i(6), act = L.i(7);
  if (cq < 0) return L.fail(NN_ERR_ARG, "SAC_AlphaLogProbs: negative count_quants");
  float *out = L.buf(0, n), *q = L.buf(1, (size_t)n * cq), *p = L.buf(2, (size_t)n * cq), *al = L.buf(3, n);
  float *lp = L.buf(4, n), *rnd = L.buf(5, n);
  if (!out || !q || !p || !al || !lp || !rnd) return NN_ERR_BOUNDS;
  sac_alpha_log_probs_kernel<<<grid1d(n, 128), 128, 0, L.stream>>>(out, q, p, al, lp, rnd, cq, act, n);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

int k_sac_alpha_grad(Launch &L) {
  const long long n = (long long)L.nd.g[0] * L.B;
  float *out = L.buf(0, n), *g = L.buf(1, n), *lp = L.buf(2, n), *ag = L.buf(3, n);
  if (!out || !g || !lp || !ag) return NN_ERR_BOUNDS;
  sac_alpha_grad_kernel<<<grid1d(n, 256), 256, 0, L.stream>>>(out, g, lp, ag, L.i(4), n);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

int k_sac_output_grad(Launch &L) {
  const long long n = (long long)L.nd.g[0] * L.B;
  const int cq = L.i(6), act = L.i(7);
  if (cq < 0) return L.fail(NN_ERR_ARG, "SAC_OutputGradient: negative count_quants");
  const size_t nq = (size_t)n * cq;
  float *q = L.buf(0, nq), *dt = L.buf(1, nq), *og = L.buf(2, n), *qg = L.buf(3, nq), *tg = L.buf(4, nq);
  float *out = L.buf(5, n);
  if (!q || !dt || !og || !qg || !tg || !out) return NN_ERR_BOUNDS;
  sac_output_grad_kernel<<<grid1d(n, 128), 128, 0, L.stream>>>(q, dt, og, qg, tg, out, cq, act, n);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

int k_sac_calc_log_probs(Launch &L) {
  const long long n = (long long)L.nd.g[0] * L.B;
  const int cq = L.i(5), act = L.i(6);
  if (cq < 0) return L.fail(NN_ERR_ARG, "SAC_CalcLogProbs: negative count_quants");
  float *out = L.buf(0, n), *q = L.buf(1, (size_t)n * cq), *p = L.buf(2, (size_t)n * cq), *al = L.buf(3, n);
  float *lp = L.buf(4, n);
  if (!out || !q || !p || !al || !lp) return NN_ERR_BOUNDS;
  sac_calc_log_probs_kernel<<<grid1d(n, 128), 128, 0, L.stream>>>(out, q, p, al, lp, cq, act, n);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

int k_fqf_fraction_grad(Launch &L) {
  const int inputs = (int)L.nd.g[0], outputs = L.i(3);
  if (outputs < 0) return L.fail(NN_ERR_ARG, "FQF_FractionGradient: negative outputs");
  float *w = L.buf(0, (size_t)outputs * (inputs + 1)), *g = L.buf(1, (size_t)L.B * outputs);
  float *ig = L.buf(2, (size_t)L.B * inputs);
  if (!w || !g || !ig) return NN_ERR_BOUNDS;
  fqf_fraction_grad_kernel<<<dim3((inputs + 31) / 32, L.B), 256, 0, L.stream>>>(w, g, ig, inputs, outputs);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

int k_fqf_dist_target_grad(Launch &L) {
  // global (quants, rows) with the quants in one work-group
  int T;
  long long R;
  quant_shape(L, &T, &R);
  const size_t n = (size_t)R * T;
  float *q = L.buf(0, n), *p = L.buf(1, n), *qg = L.buf(2, n), *pg = L.buf(3, n);
  if (!q || !p || !qg || !pg) return NN_ERR_BOUNDS;
  fqf_dist_target_grad_kernel<<<warp_grid(R), 256, 0, L.stream>>>(q, p, qg, pg, L.f(4), L.f(5), L.f(6), T, R);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

int k_fqf_rearrange(Launch &L) {
  int T;
  long long R;
  quant_shape(L, &T, &R);
  if (T == 0 || (T & (T - 1)) != 0 || T > 64) return NN_OK;  // the reference writes nothing
  const size_t n = (size_t)R * T;
  float *q = L.buf(0, n), *p = L.buf(1, n), *oq = L.buf(2, n), *op = L.buf(3, n), *ord = L.buf(4, n);
  float *diag = L.buf(5, (size_t)R * 6);
  if (!q || !p || !oq || !op || !ord || !diag) return NN_ERR_BOUNDS;
  fqf_rearrange_kernel<<<warp_grid(R), 256, 0, L.stream>>>(q, p, oq, op, ord, diag, T, R);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

int k_fqf_rearrange_grad(Launch &L) {
  int T;
  long long R;
  quant_shape(L, &T, &R);
  const size_t n = (size_t)R * T;
  float *oqg = L.buf(0, n), *opg = L.buf(1, n), *ord = L.buf(2, n), *qg = L.buf(3, n), *pg = L.buf(4, n);
  if (!oqg || !opg || !ord || !qg || !pg) return NN_ERR_BOUNDS;
  fqf_rearrange_grad_kernel<<<grid1d(n, 256), 256, 0, L.stream>>>(oqg, opg, ord, qg, pg, T, (long long)n);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

int k_fqf_srm_forward(Launch &L) {
  int T;
  long long R;
  quant_shape(L, &T, &R);
  const size_t n = (size_t)R * T;
  float *q = L.buf(0, n), *p = L.buf(1, n), *res = L.buf(2, (size_t)R);
  if (!q || !p || !res) return NN_ERR_BOUNDS;
  fqf_srm_forward_kernel<<<warp_grid(R), 256, 0, L.stream>>>(q, p, res, L.i(3), L.f(4), L.f(5), T, R);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

// FQF_Sample over global (quants, tasks) with local (quants, 1): the row length is the local size.
int k_fqf_sample(Launch &L) {
  if (!L.nd.has_local || L.nd.l[0] != L.nd.g[0] || (L.nd.dims > 1 && L.nd.l[1] != 1))
    return L.fail(NN_ERR_UNSUPPORTED, "FQF_Sample: expects local size (quants, 1) with quants = global[0]");
  const int T = (int)L.nd.l[0];
  if (T > 64)
    return L.fail(NN_ERR_UNSUPPORTED, "FQF_Sample: at most 64 quants per row (the reference's local scan array)");
  const long long R = (long long)(L.nd.dims > 1 ? L.nd.g[1] : 1) * L.B;
  const size_t n = (size_t)R * T;
  float *q = L.buf(0, n), *p = L.buf(1, n), *rnd = L.buf(2, (size_t)R), *res = L.buf(3, (size_t)R);
  if (!q || !p || !rnd || !res) return NN_ERR_BOUNDS;
  fqf_sample_kernel<<<warp_grid(R), 256, 0, L.stream>>>(q, p, rnd, res, T, R);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

int k_fqf_srm_grad(Launch &L) {
  int T;
  long long R;
  quant_shape(L, &T, &R);
  if (T == 0) return NN_OK;
  const size_t n = (size_t)R * T;
  float *q = L.buf(0, n), *p = L.buf(1, n), *rg = L.buf(2, (size_t)R), *qg = L.buf(3, n), *pg = L.buf(4, n);
  if (!q || !p || !rg || !qg || !pg) return NN_ERR_BOUNDS;
  fqf_srm_grad_kernel<<<warp_grid(R), 256, 0, L.stream>>>(q, p, rg, qg, pg, L.i(5), L.f(6), L.f(7), T, R);
  NN_CHECK_LAUNCH(L);
  return NN_OK;
}

}  // namespace

const KernelDef kFqfKernels[] = {
    {"FQF_Cosine", "pp", k_fqf_cosine, false},
    {"FQF_Output", "pppi", k_fqf_output, false},
    {"FQF_OutputGradient", "ppppp", k_fqf_output_grad, false},
    {"FQF_QuantileGradient", "ppppp", k_fqf_quantile_grad, false},
    {"FQF_CosineGradient", "ppp", k_fqf_cosine_grad<false>, false},
    {"FQF_CosineGradientSRM", "ppp", k_fqf_cosine_grad<true>, false},
    {"FQF_DistributionTargetGradient", "ppppfff", k_fqf_dist_target_grad, false},
    {"FQF_FractionGradient", "pppi", k_fqf_fraction_grad, false},
    {"FQF_MonotoneRearrange", "pppppp", k_fqf_rearrange, false},
    {"FQF_RearrangeGradient", "ppppp", k_fqf_rearrange_grad, false},
    {"FQF_SRMForward", "pppiff", k_fqf_srm_forward, false},
    {"FQF_SRMGradient", "pppppiff", k_fqf_srm_grad, false},
    {"FQF_Sample", "pppp", k_fqf_sample, false},
    {"SAC_AlphaLogProbs", "ppppppii", k_sac_alpha_log_probs, false},
    {"SAC_AlphaGradients", "ppppi", k_sac_alpha_grad, false},
    {"SAC_OutputGradient", "ppppppii", k_sac_output_grad, false},
    {"SAC_CalcLogProbs", "pppppii", k_sac_calc_log_probs, false},
};
const int kNumFqfKernels = sizeof(kFqfKernels) / sizeof(kFqfKernels[0]);

}  // namespace nn
