// LSTM kernels (CNeuronLSTMOCL path): LSTM_FeedForward, LSTM_ConcatenatedGradient,
// LSTM_HiddenGradient, LSTM_UpdateWeightsAdam.
//
// Layout is the reference's: per variable (independent series) v, inputs
// [v][in], outputs / hidden state [v][H], gate values and gate gradients
// [v][4][H] (forget, input, output, new content), memory [2][v][H] (current,
// then previous cell state), weights [4H][H+in+1] rows of (hidden, input, bias).
// A batch folds into the variables dimension (the reference's own batching).
//
// Reference behaviours kept (NeuroNet.cl:2189-2475): the gate sum of neuron
// `id`, gate `g` uses weight row g+id; gate derivatives are taken from the
// gradient value (g*(1-g), g*(1-g*g)); the "bias" gradient of row i is written
// at (i+1)*(H+in+1); the input loop reads only the first H inputs when in > H.
// Defined here where the reference is racy: every gate reads the previous step's
// hidden state (the reference overwrites it from other work-groups while reading
// it), and the bias write of row i+1 lands after that row's weight gradient; the
// reference's last bias write, one element past a (4H)x(H+in+1) buffer, is performed only
// when the caller's buffer holds that element.
#include "../../include/nn_b200.h"
#include "gemm_fast.cuh"
#include "tc_gemm.cuh"
#include "nn_device.cuh"
#include "nn_internal.h"
#include "wgrad.cuh"
#include "epi_dense.cuh"

namespace nn {

// ------------------------------------------------------------ forward
// gates: one thread per (v, gate, neuron), reads h(t-1) and x(t), writes concatenated.
__global__ void lstm_gates_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                  const float *__restrict__ h, float *__restrict__ cat, int H, int in, int V) {
  pdl_wait();
  pdl_trigger();
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)V * 4 * H) return;
  int id = (int)(t % H);
  size_t r = t / H;
  int gate = (int)(r % 4);
  size_t v = r / 4;
  const int ws = in + H + 1;
  const float *row = w + (size_t)(gate + id) * ws;
  const float *hv = h + v * H;
  const float *xv = x + v * in;
  float sum = 0.f;
  for (int i = 0; i < H; i += 4) {
    if (H - i > 4) {
      float d = hv[i] * row[i] + hv[i + 1] * row[i + 1] + hv[i + 2] * row[i + 2] + hv[i + 3] * row[i + 3];
      sum += nan0(d);
    } else {
      for (int k = i; k < H; ++k) sum += nan0(hv[k] * row[k]);
    }
  }
  const float *rx = row + H;
  for (int i = 0; i < in; i += 4) {
    if ((unsigned)(H - i) > 4u) {  // unsigned, as the reference's uint arithmetic (wraps when i > H)
      float d = xv[i] * rx[i] + xv[i + 1] * rx[i + 1] + xv[i + 2] * rx[i + 2] + xv[i + 3] * rx[i + 3];
      sum += nan0(d);
    } else {
      for (int k = i; k < H; ++k) sum += nan0(xv[k] * rx[k]);
    }
  }
  sum += nan0(rx[in]);
  sum = activate(sum, gate < 3 ? ACT_SIGMOID : ACT_TANH);
  cat[(v * 4 + gate) * H + id] = sum;
}

// cell: memory and output update from the gate values.
__global__ void lstm_cell_kernel(const float *__restrict__ cat, float *__restrict__ mem, float *__restrict__ out,
                                 int H, int V) {
  pdl_wait();
  pdl_trigger();
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)V * H) return;
  int id = (int)(t % H);
  size_t v = t / H;
  const float *c = cat + v * 4 * H;
  float m = mem[t];
  mem[t + (size_t)V * H] = m;
  m = nan0(m * c[id] + c[H + id] * c[3 * H + id]);
  mem[t] = m;
  out[t] = nan0(c[2 * H + id] * activate(m, ACT_TANH));
}

static int lstm_shape(Launch &L, int *H, int *V) {
  *H = (int)L.nd.g[0];
  *V = (L.nd.dims > 2 ? (int)L.nd.g[2] : 1) * L.B;
  return NN_OK;
}

// Tensor-core forward.  Gate g of neuron id reads weight row g+id, so only rows 0..H+2 are ever
// used: one GEMM gives every pre-activation, P[v][r] = [h(t-1) | x](v) . W[r][0:H+in] + W[r][H+in]
// for r < H+4 (row H+3 pads the row stride to a multiple of 4), and a fused kernel applies the gate
// activations and the cell update.  The packed operand keeps exactly the inputs the reference's
// float4 input loop reads: input j belongs to group i = j - j%4, read when (unsigned)(H-i) > 4
// or, in the tail loop that runs otherwise, when j < H.
__global__ void lstm_pack_hx_kernel(const float *__restrict__ h, const float *__restrict__ x,
                                    float *__restrict__ opnd, int H, int in, int V) {
  pdl_wait();
  pdl_trigger();
  const size_t cols = (size_t)H + in;
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)V * cols) return;
  size_t v = t / cols;
  int c = (int)(t % cols);
  float val;
  if (c < H) {
    val = h[v * H + c];
  } else {
    int j = c - H, i = j - (j & 3);
    val = ((unsigned)(H - i) > 4u || j < H) ? x[v * in + j] : 0.f;
  }
  opnd[t] = val;
}

// P = the GEMM's K-slice partials [splits][V][ldp] of the pre-activations of rows r < H+4; the
// pre-activation of row r is their sum plus the bias nan0(W[r][H+in]).
__global__ void lstm_gates_cell_kernel(const float *__restrict__ P, int splits, size_t pstride, int ldp,
                                       const float *__restrict__ w, int ws, int bcol, float *__restrict__ cat,
                                       float *__restrict__ mem, float *__restrict__ out, int H, int V) {
  pdl_wait();
  pdl_trigger();
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)V * H) return;
  int id = (int)(t % H);
  size_t v = t / H;
  float pre[4];
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    float a = 0.f;
#pragma unroll 4
    for (int sp = 0; sp < splits; ++sp) a += P[sp * pstride + v * ldp + id + g];
    pre[g] = a + nan0(w[(size_t)(id + g) * ws + bcol]);
  }
  const float f = activate(pre[0], ACT_SIGMOID), ig = activate(pre[1], ACT_SIGMOID);
  const float og = activate(pre[2], ACT_SIGMOID), nc = activate(pre[3], ACT_TANH);
  float *c = cat + v * 4 * H + id;
  c[0] = f;
  c[H] = ig;
  c[2 * H] = og;
  c[3 * H] = nc;
  float m = mem[t];
  mem[t + (size_t)V * H] = m;
  m = nan0(m * f + ig * nc);
  mem[t] = m;
  out[t] = nan0(og * activate(m, ACT_TANH));
}

// K slices of the gate product over 128 x 64 tiles: whole waves of the SMs, each slice at least 128
// deep, at most 8 slices.
static int lstm_ff_splits(int V, int N, int K) {
  const long long tiles = (long long)((V + 127) / 128) * ((N + 63) / 64);
  return wave_splits(tiles, std::min(K / 128, 8));
}

static int k_lstm_feed_forward(Launch &L) {
  int H = (int)L.nd.g[0];
  int V = (L.nd.dims > 2 ? (int)L.nd.g[2] : 1) * L.B;
  const int in = L.i(1);
  if (in < 0 || (in % 4) != 0)
    return L.fail(NN_ERR_UNSUPPORTED, "LSTM_FeedForward: inputs_size must be a multiple of 4 "
                                      "(the reference's float4 input loop reads past the row otherwise)");
  if (L.nd.dims < 2 || L.nd.g[1] != 4) return L.fail(NN_ERR_ARG, "LSTM_FeedForward: global size 1 must be 4");
  const int ws = in + H + 1;
  // read extent of the input loop: float4 blocks while H - i > 4, else up to H
  int xneed = 0;
  for (int i = 0; i < in; i += 4) xneed = std::max(xneed, (unsigned)(H - i) > 4u ? i + 4 : H);
  float *x = L.buf(0, (size_t)(V - 1) * in + (size_t)xneed);
  float *w = L.buf(2, (size_t)(H + 3) * ws);
  float *cat = L.buf(3, (size_t)V * 4 * H), *mem = L.buf(4, (size_t)2 * V * H), *out = L.buf(5, (size_t)V * H);
  if (!x || !w || !cat || !mem || !out) return NN_ERR_BOUNDS;
  const int ldp = H + 4;
  if (H % 4 == 0 && xneed <= in && L.floats(2) >= (size_t)ldp * ws) {
    const size_t nop = (size_t)V * (H + in);
    const int K = H + in;
    FastShape fs{V, ldp, K, 1, 1, 0, nullptr, (long long)K, 0, w, ws, 0};
    int splits = lstm_ff_splits(V, ldp, K);
    fs.kchunk = splits > 1 ? ((K + splits - 1) / splits + 31) / 32 * 32 : K;
    splits = (K + fs.kchunk - 1) / fs.kchunk;
    fs.splits = splits;
    const size_t pstride = (size_t)V * ldp;
    float *opnd = L.scratch(1, nop + pstride * splits);
    if (!opnd) return NN_ERR_CUDA;
    float *P = opnd + nop;  // 16-byte aligned: H + in is a multiple of 4
    fs.A = opnd;
    NN_LAUNCH_PDL(L, lstm_pack_hx_kernel, grid1d(nop, 256), 256, 0, L.stream, out, x, opnd, H, in, V);
    // the product's K-slice partials; the gate kernel sums them and adds the bias column
    cudaError_t e = gemm_f32_wb<false, false>(L, fs, PartialStoreTma{{P, V, ldp, 1}});
    if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
    L.counted();
    NN_LAUNCH_PDL(L, lstm_gates_cell_kernel, grid1d((size_t)V * H, 256), 256, 0, L.stream, P, splits, pstride, ldp, w, ws, K, cat, mem, out, H, V);
    return NN_OK;
  }
  NN_LAUNCH_PDL(L, lstm_gates_kernel, grid1d((size_t)V * 4 * H, 256), 256, 0, L.stream, x, w, out, cat, H, in, V);
  NN_LAUNCH_PDL(L, lstm_cell_kernel, grid1d((size_t)V * H, 256), 256, 0, L.stream, cat, mem, out, H, V);
  return NN_OK;
}

// ----------------------------------------------- concatenated gradient
// NeuroNet.cl:2265-2297
__global__ void lstm_cat_grad_kernel(const float *__restrict__ grad, float *__restrict__ cg,
                                     const float *__restrict__ mem, const float *__restrict__ cat, int H, int V) {
  pdl_wait();
  pdl_trigger();
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)V * H) return;
  int id = (int)(t % H);
  size_t v = t / H;
  float th = tanhf(mem[t]);
  float gr = grad[t];
  float *c = cg + v * 4 * H;
  const float *a = cat + v * 4 * H;
  c[2 * H + id] = gr * th;
  float mg = gr * a[2 * H + id];
  mg *= 1.f - th * th;
  c[3 * H + id] = mg * a[H + id];
  c[H + id] = mg * a[3 * H + id];
  c[id] = mg * mem[t + (size_t)V * H];
}

static int k_lstm_concatenated_gradient(Launch &L) {
  int H = (int)L.nd.g[0];
  int V = (L.nd.dims > 1 ? (int)L.nd.g[1] : 1) * L.B;
  float *g = L.buf(0, (size_t)V * H), *cg = L.buf(1, (size_t)V * 4 * H), *mem = L.buf(2, (size_t)2 * V * H);
  float *cat = L.buf(3, (size_t)V * 4 * H);
  if (!g || !cg || !mem || !cat) return NN_ERR_BOUNDS;
  NN_LAUNCH_PDL(L, lstm_cat_grad_kernel, grid1d((size_t)V * H, 256), 256, 0, L.stream, g, cg, mem, cat, H, V);
  return NN_OK;
}

// -------------------------------------------------------- hidden gradient
// NeuroNet.cl:2301-2441.  Derivative factors a[v][g] = cg(1-cg) (g < 3H) or cg(1-cg^2);
// operands [v][H+in] = (h(t-1), x); then hidden_state <- output.
__global__ void lstm_hg_prep_kernel(const float *__restrict__ cg, float *__restrict__ a, float *__restrict__ opnd,
                                    float *__restrict__ hidden, const float *__restrict__ out,
                                    const float *__restrict__ x, int H, int in, int V) {
  pdl_wait();
  pdl_trigger();
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  const size_t na = (size_t)V * 4 * H;
  if (t < na) {
    int g = (int)(t % (4 * H));
    float c = cg[t];
    a[t] = g < 3 * H ? c * (1.f - c) : c * (1.f - c * c);
  }
  const size_t cols = (size_t)H + in;
  if (t < (size_t)V * cols) {
    size_t v = t / cols;
    int i = (int)(t % cols);
    if (i < H) {
      size_t hi = v * H + i;
      opnd[t] = hidden[hi];
      hidden[hi] = out[hi];
    } else {
      opnd[t] = x[v * in + (i - H)];
    }
  }
}

// bias row sums: col0 of row i+1 = sum_v (i < 3H ? cg(1-cg) : 1-cg^2), for i < rows.  Block of
// 32 gate columns x 32 series lanes; each lane sums its series in order, then the 32 lane sums.
__global__ void __launch_bounds__(1024) lstm_bias_kernel(const float *__restrict__ cg, float *__restrict__ wg, int H,
                                                         int V, int ws, int rows) {
  pdl_wait();
  pdl_trigger();
  __shared__ float part[32][33];
  const int i = blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (i < rows) {
    const bool sig = i < 3 * H;
    for (int v = threadIdx.y; v < V; v += 32) {
      float c = cg[(size_t)v * 4 * H + i];
      s += sig ? c * (1.f - c) : 1.f - c * c;
    }
  }
  part[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y != 0 || i >= rows) return;
  float t = 0.f;
#pragma unroll 8
  for (int r = 0; r < 32; ++r) t += part[r][threadIdx.x];
  wg[(size_t)(i + 1) * ws] = t;
}

// weight-gradient rows from split-K partials: wg[g][i] = sum_s part[s][g][i] for i < N (the last
// column of each (H+in+1)-float row is not a gradient the reference writes)
__global__ void lstm_wg_reduce_kernel(float *__restrict__ wg, GradSrc src, int rows, int N, int ws) {
  pdl_wait();
  pdl_trigger();
  const size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)rows * N) return;
  const size_t g = t / N, i = t % N;
  wg[g * ws + i] = src(t);
}

struct StoreStrided {
  float *p;
  long long ld;
  __device__ __forceinline__ void operator()(int m, int n, int, int, float acc) const { p[(size_t)m * ld + n] = acc; }
  __device__ __forceinline__ long long row(int m, int, int) const { return (long long)m * ld; }
  __device__ __forceinline__ float col(int, int) const { return 0.f; }
  template <int R>
  __device__ __forceinline__ void put_rows(const long long (&rb)[R], int n, const float (&v)[R], float,
                                           unsigned mask) const {
#pragma unroll
    for (int j = 0; j < R; ++j)
      if (mask >> j & 1u) p[rb[j] + n] = v[j];
  }
  __host__ __device__ bool aligned4() const { return (ld) % 4 == 0 && ((uintptr_t)p & 15) == 0; }
  __device__ __forceinline__ float4 col4(int, int) const { return make_float4(0.f, 0.f, 0.f, 0.f); }
  template <int R>
  __device__ __forceinline__ void put_rows4(const long long (&rb)[R], int n, const float4 (&v)[R], float4,
                                            unsigned mask) const {
#pragma unroll
    for (int j = 0; j < R; ++j)
      if (mask >> j & 1u) *reinterpret_cast<float4 *>(p + rb[j] + n) = v[j];
  }
};
struct StoreInputGrad {
  float *p;
  int in;
  __device__ __forceinline__ void operator()(int m, int n, int, int, float acc) const { p[(size_t)m * in + n] = acc; }
  __device__ __forceinline__ long long row(int m, int, int) const { return (long long)m * in; }
  __device__ __forceinline__ float col(int, int) const { return 0.f; }
  template <int R>
  __device__ __forceinline__ void put_rows(const long long (&rb)[R], int n, const float (&v)[R], float,
                                           unsigned mask) const {
#pragma unroll
    for (int j = 0; j < R; ++j)
      if (mask >> j & 1u) p[rb[j] + n] = v[j];
  }
  __host__ __device__ bool aligned4() const { return (in) % 4 == 0 && ((uintptr_t)p & 15) == 0; }
  __device__ __forceinline__ float4 col4(int, int) const { return make_float4(0.f, 0.f, 0.f, 0.f); }
  template <int R>
  __device__ __forceinline__ void put_rows4(const long long (&rb)[R], int n, const float4 (&v)[R], float4,
                                            unsigned mask) const {
#pragma unroll
    for (int j = 0; j < R; ++j)
      if (mask >> j & 1u) *reinterpret_cast<float4 *>(p + rb[j] + n) = v[j];
  }
};

// Split-K count for a product of `tiles` 128x128 output tiles over a reduction of K: whole waves of
// the SMs, each slice at least 128 deep, at most 16 slices.
static int lstm_splits(long long tiles, int K) { return wave_splits(tiles, std::min(K / 128, 16)); }

static int k_lstm_hidden_gradient(Launch &L) {
  int H = (int)L.nd.g[0];
  int V = (L.nd.dims > 1 ? (int)L.nd.g[1] : 1) * L.B;
  const int hs = L.i(7), in = L.i(8);
  if (hs != H) return L.fail(NN_ERR_ARG, "LSTM_HiddenGradient: hidden_size must equal global size 0");
  if (in < 0) return L.fail(NN_ERR_ARG, "LSTM_HiddenGradient: negative inputs_size");
  const int ws = H + in + 1;
  float *cg = L.buf(0, (size_t)V * 4 * H), *ig = L.buf(1, (size_t)V * in), *wg = L.buf(2, (size_t)4 * H * ws);
  float *hidden = L.buf(3, (size_t)V * H), *x = L.buf(4, (size_t)V * in), *w = L.buf(5, (size_t)4 * H * ws);
  float *out = L.buf(6, (size_t)V * H);
  if (!cg || !ig || !wg || !hidden || !x || !w || !out) return NN_ERR_BOUNDS;
  const size_t na = (size_t)V * 4 * H, nop = (size_t)V * (H + in);
  float *a = L.scratch(1, na + nop);
  if (!a) return NN_ERR_CUDA;
  float *opnd = a + na;
  NN_LAUNCH_PDL(L, lstm_hg_prep_kernel, grid1d(std::max(na, nop), 256), 256, 0, L.stream, cg, a, opnd, hidden, out, x, H, in, V);
  // input gradient: dx[v][j] = sum_g a[v][g] w[g][H+j]; on the tensor cores in K slices whose
  // partials (16-byte rows when in % 4 == 0) are summed into dx
  if (in > 0) {
    FastShape fs{V, in, 4 * H, 1, 1, 0, a, 4LL * H, 0, w + H, ws, 0};
    const long long tiles = (long long)((V + 127) / 128) * ((in + 127) / 128);
    const int splits = lstm_splits(tiles, 4 * H);
    if (tc_path(fs) && splits > 1 && in % 4 == 0) {
      fs.splits = splits;
      fs.kchunk = ((4 * H + splits - 1) / splits + 31) / 32 * 32;
      fs.splits = (4 * H + fs.kchunk - 1) / fs.kchunk;
      const size_t per = (size_t)V * in;
      float *part = L.scratch(2, per * fs.splits);
      if (!part) return NN_ERR_CUDA;
      cudaError_t e = gemm_f32_wb<false, true>(L, fs, PartialStoreTma{{part, V, in, 1}});
      if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
      L.counted();
      GradSrc src{part, fs.splits, per, 1.f};
      NN_LAUNCH_PDL(L, reduce_partials_kernel, (unsigned)((per + 31) / 32), dim3(32, 8), 0, L.stream, ig, src, per);
    } else {
      cudaError_t e = gemm_f32_wb<false, true>(L, fs, StoreInputGrad{ig, in});
      if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
      L.counted();
    }
  }
  // weight gradient: wg[g][i] = sum_v a[v][g] opnd[v][i], i < H+in (summed over the series), in
  // K slices of the series on the tensor cores
  {
    const int N = H + in;
    FastShape fs{4 * H, N, V, 1, 1, 0, a, 4LL * H, 0, opnd, (long long)N, 0};
    const long long tiles = (long long)((4 * H + 127) / 128) * ((N + 127) / 128);
    const int splits = lstm_splits(tiles, V);
    if (tc_path(fs) && splits > 1 && N % 4 == 0) {
      fs.kchunk = ((V + splits - 1) / splits + 31) / 32 * 32;
      fs.splits = (V + fs.kchunk - 1) / fs.kchunk;
      const size_t per = (size_t)4 * H * N;
      float *part = L.scratch(0, per * fs.splits);
      if (!part) return NN_ERR_CUDA;
      cudaError_t e = tcgemm<true, true>(fs, PartialStoreTma{{part, 4 * H, N, 1}}, L.stream, device_status());
      if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
      L.counted();
      GradSrc src{part, fs.splits, per, 1.f};
      NN_LAUNCH_PDL(L, lstm_wg_reduce_kernel, grid1d(per, 256), 256, 0, L.stream, wg, src, 4 * H, N, ws);
    } else {
      cudaError_t e = gemm_f32<true, true>(fs, StoreStrided{wg, ws}, L.stream);
      if (e != cudaSuccess) return L.fail(NN_ERR_CUDA, cudaGetErrorString(e));
      L.counted();
    }
  }
  // the last bias write lands one element past the (4H)x(H+in+1) matrix: done only when the buffer holds it
  const int bias_rows = L.floats(2) > (size_t)4 * H * ws ? 4 * H : 4 * H - 1;
  NN_LAUNCH_PDL(L, lstm_bias_kernel, (unsigned)((bias_rows + 31) / 32), dim3(32, 32), 0, L.stream, cg, wg, H, V, ws, bias_rows);
  return NN_OK;
}

// ------------------------------------------------------- Adam update
// NeuroNet.cl:2450-2475: elementwise over global (total, rows), l2 decay / total, raw rate.
__global__ void lstm_adam_kernel(float *w, const float *wg, float *m, float *v, int total, int rows, float l, float b1,
                                 float b2) {
  pdl_wait();
  pdl_trigger();
  size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (t >= (size_t)total * rows) return;
  float g = clampf(nan0(wg[t]), -kMaxGrad, kMaxGrad);
  float mt = b1 * nan0(m[t]) + (1.f - b1) * g;
  float vt = b2 * nan0(v[t], 1.f) + (1.f - b2) * (g * g);
  float weight = nan0(w[t]);
  float delta = l * (mt / (sqrtf(vt) + 1.0e-37f) - (kL1 * signf(weight) + kL2 * weight / (float)total));
  w[t] = nan0(weight + delta);
  m[t] = mt;
  v[t] = vt;
}

static int lstm_adam_apply(const Launch &Lc, const float *grad) {
  Launch &L = const_cast<Launch &>(Lc);
  int total = (int)L.nd.g[0], rows = L.nd.dims > 1 ? (int)L.nd.g[1] : 1;
  size_t n = (size_t)total * rows;
  float *w = L.buf(0, n), *m = L.buf(2, n), *v = L.buf(3, n);
  if (!w || !m || !v) return NN_ERR_BOUNDS;
  NN_LAUNCH_PDL(L, lstm_adam_kernel, grid1d(n, 256), 256, 0, L.stream, w, grad, m, v, total, rows, L.f(4), L.f(5), L.f(6));
  return NN_OK;
}

__global__ void scaled_copy_kernel(float *dst, const float *src, size_t n, float s) {
  pdl_wait();
  pdl_trigger();
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (i < n) dst[i] = src[i] * s;
}

static int k_lstm_update_weights_adam(Launch &L) {
  int total = (int)L.nd.g[0], rows = L.nd.dims > 1 ? (int)L.nd.g[1] : 1;
  size_t n = (size_t)total * rows;
  float *wg = L.buf(1, n);
  if (!wg) return NN_ERR_BOUNDS;
  if (L.deferred()) {
    // the weight gradient is a sum over series: the ranks' sums are summed (mean x world)
    float *slot = L.grad_slot(n);
    if (!slot) return NN_ERR_BOUNDS;
    NN_LAUNCH_PDL(L, scaled_copy_kernel, grid1d(n, 256), 256, 0, L.stream, slot, wg, n, (float)dp_world());
    L.defer(lstm_adam_apply, slot);
    return NN_OK;
  }
  return lstm_adam_apply(L, wg);
}

const KernelDef kLstmKernels[] = {
    {"LSTM_FeedForward", "pipppp", k_lstm_feed_forward, false},
    {"LSTM_ConcatenatedGradient", "pppp", k_lstm_concatenated_gradient, false},
    {"LSTM_HiddenGradient", "pppppppii", k_lstm_hidden_gradient, false},
    {"LSTM_UpdateWeightsAdam", "ppppfff", k_lstm_update_weights_adam, false},
};
const int kNumLstmKernels = sizeof(kLstmKernels) / sizeof(kLstmKernels[0]);

}  // namespace nn
