// Multi-head attention score and output products on the tensor cores (tcgen05, 3xTF32), for the
// MHAttentionScore / MHAttentionOut shapes of one (sequence, head) pair per work item: up to 128
// units and a head dimension of 32.
//
//   score:  S[q][k] = softmax_k(Q[q] . K[k] / koef)   M = q (128), N = k (128), K = d (32), 1 stage
//   out:    O[q][d] = sum_k S[q][k] V[k][d]            M = q (128), N = d (32),  K = k (128), 4 stages
//
// Persistent CTAs walk the B*H work items; per CTA 448 threads in the roles of tc_gemm.cuh:
// warps 0-7 epilogue (one output row per thread; two warps per tensor-memory lane quarter, one
// per half of the columns), warps 8-11 split the TMA-loaded raw tiles into hi / lo in place, warp
// 12 issues the MMAs into one of two tensor-memory accumulators, warp 13 issues the TMA loads.  Rows and keys past `units` are loaded (they belong to the next sequence,
// or are zero-filled past the end of the tensor) and computed, but never stored: the score
// epilogue excludes keys >= units from the normalisation, and the out product reads scores whose
// columns >= units are zero-filled by TMA (the score tensor's inner extent is `units`).
#pragma once
#include "tc_gemm.cuh"

namespace nn {
namespace tc {

constexpr int kAttnScore = 0, kAttnOut = 1;

template <int MODE>
struct AttnCfg {
  static constexpr int BM = 128, BK = 32;
  static constexpr int BN = MODE == kAttnScore ? 128 : 32;
  static constexpr int NK = MODE == kAttnScore ? 1 : 4;         // k stages per item
  static constexpr int STAGES = MODE == kAttnScore ? 2 : 4;
  static constexpr uint32_t A_BYTES = BM * BK * 4, B_BYTES = BN * BK * 4;
  static constexpr uint32_t STAGE_BYTES = 2 * (A_BYTES + B_BYTES);
  static constexpr uint32_t EPI_OFF = STAGES * STAGE_BYTES;
  // TMA-store boxes of 32 rows x 32 floats (128-byte swizzle, 4 KB, 1024-byte aligned).  score: two
  // per epilogue warp (its 32 rows x 64 keys) plus the two partial row sums, double-buffered by
  // item parity; out: one per lane quarter
  static constexpr uint32_t PSUM_OFF = 8 * 8192;
  static constexpr uint32_t EPI_BYTES = MODE == kAttnScore ? PSUM_OFF + 2 * 256 * 4 : 4 * 4096;
  static constexpr uint32_t SMEM = EPI_OFF + EPI_BYTES + 1024;
  static constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;
  static_assert(SMEM <= 232448, "shared memory per CTA");
  static_assert((TMEM_COLS & (TMEM_COLS - 1)) == 0, "tensor-memory columns");
  static_assert(EPI_OFF % 1024 == 0, "store boxes use the 128-byte swizzle");
};

// tmQ:  qkv as [B*U rows][3*H*D], box 32 x 128, 128-byte swizzle (K-major Q and K tiles)
// tmS:  scores as [B*U][H][U],    box 32 x 1 x 128, 128-byte swizzle (K-major score tiles)
// tmV:  qkv as [B*U rows][3*H*D], box 32 x 32, 128-byte swizzle / 32-byte granules (MN-major V)
// tmO:  the output as [B][U][H][U] (score) or [B][U][H][D] (out), box 32 x 1 x 32 x 1, 128-byte
//       swizzle: TMA stores clip keys and rows past `units`
template <int MODE>
__global__ void __launch_bounds__(448, 1)
    attn_tc_kernel(int *err, int U, int H, int items, int mask, float koef, const __grid_constant__ CUtensorMap tmQ,
                   const __grid_constant__ CUtensorMap tmS, const __grid_constant__ CUtensorMap tmV,
                   const __grid_constant__ CUtensorMap tmO) {
  using C = AttnCfg<MODE>;
  constexpr int BM = C::BM, BN = C::BN, BK = C::BK, NK = C::NK, STAGES = C::STAGES;
  constexpr int D = 32;
  // A: K-major, 128-byte swizzle.  B: K-major swizzled (score) or MN-major 32-byte granules (out).
  constexpr uint32_t A_LBO = 16u, A_SBO = 1024u, A_LAY = 2u, A_STEP = 32u;
  constexpr bool B_MN = MODE == kAttnOut;
  constexpr uint32_t B_LBO = B_MN ? 128u * BK : 16u, B_SBO = B_MN ? 512u : 1024u, B_LAY = B_MN ? 1u : 2u;
  constexpr uint32_t B_STEP = B_MN ? 1024u : 32u;
  constexpr uint32_t IDESC = instr_desc_tf32(BM, BN, false, B_MN);

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], tmaf[STAGES], accf[2], acce[2], drain;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  // roles: warps 0-7 epilogue (lane quarter w % 4, column half w / 4), 8-11 split, 12 MMA, 13 TMA
  constexpr int kMmaWarp = 12, kLoadWarp = 13;
  __shared__ __align__(8) uint64_t esync;
  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  auto fail = [&](int code) {
    abort_flag = 1;
    atomicExch(err, code);
  };
  if (tid == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 128);
      mbar_init(&empty[i], 1);
      mbar_init(&tmaf[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], 256);
    }
    mbar_init(&esync, 256);
    mbar_init(&drain, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  pdl_wait();
  pdl_trigger();

  if (warp == kLoadWarp) {
    // ------------------------------------------------------------ loader
    if (lane == 0) {
      int it = 0;
      for (int t = blockIdx.x; t < items && !abort_flag; t += gridDim.x) {
        const int b = t / H, h = t % H;
        bool ok = true;
        for (int kk = 0; kk < NK; ++kk, ++it) {
          const int st = it % STAGES;
          if (it >= STAGES && !mbar_wait(&empty[st], ((it / STAGES) - 1) & 1, &abort_flag)) {
            fail(kErrEmptyWait);
            ok = false;
            break;
          }
          uint8_t *base = smem + st * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&tmaf[st], C::A_BYTES + C::B_BYTES);
          if (MODE == kAttnScore) {
            tma_load_3d(base, &tmQ, h * D, b * U, 0, &tmaf[st]);                          // Q rows
            tma_load_3d(base + 2 * C::A_BYTES, &tmQ, (H + h) * D, b * U, 0, &tmaf[st]);   // K rows
          } else {
            tma_load_3d(base, &tmS, 32 * kk, h, b * U, &tmaf[st]);                        // S[:, 32kk..]
            tma_load_3d(base + 2 * C::A_BYTES, &tmV, (2 * H + h) * D, b * U + 32 * kk, 0, &tmaf[st]);
          }
        }
        if (!ok) break;
      }
      for (int st = 0; st < STAGES && st < it; ++st) {
        const int issued = (it - st - 1) / STAGES + 1;
        if (!mbar_wait_drain(&tmaf[st], (issued - 1) & 1) && !abort_flag) fail(kErrFullWait);
      }
    }
  } else if (warp >= 8 && warp < 12) {
    // ------------------------------------------------------------ split raw tiles into hi / lo
    const int ptid = tid - 256;
    int it = 0;
    for (int t = blockIdx.x; t < items && !abort_flag; t += gridDim.x) {
      bool ok = true;
      for (int kk = 0; kk < NK; ++kk, ++it) {
        const int st = it % STAGES;
        if (it >= STAGES && !mbar_wait(&empty[st], ((it / STAGES) - 1) & 1, &abort_flag)) {
          fail(kErrEmptyWait);
          ok = false;
          break;
        }
        if (!mbar_wait(&tmaf[st], (it / STAGES) & 1, &abort_flag)) {
          fail(kErrFullWait);
          ok = false;
          break;
        }
        uint8_t *base = smem + st * C::STAGE_BYTES;
        static_assert(C::A_BYTES % 2048 == 0 && C::B_BYTES % 2048 == 0, "whole chunks per producer thread");
        split_chunks<C::A_BYTES / 2048>(base, base + C::A_BYTES, 16u * ptid, 2048u);
        split_chunks<C::B_BYTES / 2048>(base + 2 * C::A_BYTES, base + 2 * C::A_BYTES + C::B_BYTES, 16u * ptid, 2048u);
        fence_proxy_async_smem();
        mbar_arrive(&full[st]);
      }
      if (!ok) break;
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    int it = 0, tl = 0;
    for (int t = blockIdx.x; t < items && !abort_flag; t += gridDim.x, ++tl) {
      const int b = tl & 1, u = tl >> 1;
      if (tl >= 2 && !mbar_wait(&acce[b], (u - 1) & 1, &abort_flag)) {
        if (lane == 0) fail(kErrDoneWait);
        break;
      }
      tc_fence_after();
      const uint32_t d = tmem + (uint32_t)(b * BN);
      bool ok = true;
      for (int kk = 0; kk < NK; ++kk, ++it) {
        const int st = it % STAGES;
        if (!mbar_wait(&full[st], (it / STAGES) & 1, &abort_flag)) {
          if (lane == 0) fail(kErrFullWait);
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t base = smem_u32(smem + st * C::STAGE_BYTES);
          const uint32_t a_hi = base, a_lo = base + C::A_BYTES;
          const uint32_t b_hi = base + 2 * C::A_BYTES, b_lo = b_hi + C::B_BYTES;
#pragma unroll
          for (int sub = 0; sub < BK / 8; ++sub) {
            const uint64_t ah = smem_desc(a_hi + sub * A_STEP, A_LBO, A_SBO, A_LAY);
            const uint64_t al = smem_desc(a_lo + sub * A_STEP, A_LBO, A_SBO, A_LAY);
            const uint64_t bh = smem_desc(b_hi + sub * B_STEP, B_LBO, B_SBO, B_LAY);
            const uint64_t bl = smem_desc(b_lo + sub * B_STEP, B_LBO, B_SBO, B_LAY);
            mma_tf32(d, al, bh, IDESC, (kk | sub) != 0 ? 1u : 0u);
            mma_tf32(d, ah, bl, IDESC, 1u);
            mma_tf32(d, ah, bh, IDESC, 1u);
          }
          mma_commit(&empty[st]);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (lane == 0) mma_commit(&accf[b]);
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ epilogue (thread = row q)
    const int quarter = warp & 3, half = warp >> 2;
    int tl = 0;
    const float inv_koef = 1.f / koef;
    for (int t = blockIdx.x; t < items && !abort_flag; t += gridDim.x, ++tl) {
      const int bb = t / H, h = t % H;
      const int b = tl & 1, u = tl >> 1;
      if (!mbar_wait(&accf[b], u & 1, &abort_flag)) {
        fail(kErrDoneWait);
        break;
      }
      tc_fence_after();
      const uint32_t trow = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * BN);
      const int q = quarter * 32 + lane;  // this thread's row
      if (MODE == kAttnScore) {
        // MHAttentionScore (NeuroNet.cl:1662-1719): e = exp(clamp(s / koef, -100, 100)) over the
        // unmasked keys, divided by their sum when the sum exceeds 1.  The two warps of a lane
        // quarter each exponentiate one half of the keys (kept in registers) and publish a partial
        // sum per row; after a bounded barrier each thread writes its row of the two store boxes,
        // scaled, and lane 0 hands the boxes to TMA.
        uint8_t *bx = smem + C::EPI_OFF + warp * 8192;
        float *psum = reinterpret_cast<float *>(smem + C::EPI_OFF + C::PSUM_OFF) + (tl & 1) * 256;  // [2][128]
        const int kmax = mask > 0 ? min(U, q + 1) : U;  // keys that take part in row q
        float e[2][32];
        tmem_ld32(trow + (uint32_t)(half * 64), e[0]);
        tmem_ld32(trow + (uint32_t)(half * 64 + 32), e[1]);
        float sum = 0.f;
#pragma unroll
        for (int cb = 0; cb < 2; ++cb)
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            float x = 0.f;
            if (half * 64 + 32 * cb + j < kmax) {
              x = exp2f(clampf(e[cb][j] * inv_koef, -100.f, 100.f) * 1.4426950408889634f);
              if (isnan(x)) x = 0.f;
              sum += x;
            }
            e[cb][j] = x;
          }
        psum[half * 128 + q] = sum;
        mbar_arrive(&esync);
        const bool ok = mbar_wait(&esync, tl & 1, &abort_flag);
        if (!ok) {
          fail(kErrDoneWait);
          break;
        }
        const float tot = psum[q] + psum[128 + q];
        const float sc = tot > 1.f ? 1.f / tot : 1.f;
        if (lane == 0) bulk_wait_read<0>();  // the previous item's stores have read the boxes
        __syncwarp();
#pragma unroll
        for (int cb = 0; cb < 2; ++cb)
#pragma unroll
          for (int g = 0; g < 8; ++g)
            *reinterpret_cast<float4 *>(bx + cb * 4096 + lane * 128 + (((g ^ lane) & 7) << 4)) =
                make_float4(e[cb][4 * g] * sc, e[cb][4 * g + 1] * sc, e[cb][4 * g + 2] * sc, e[cb][4 * g + 3] * sc);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && quarter * 32 < U) {
#pragma unroll
          for (int cb = 0; cb < 2; ++cb)
            if (half * 64 + 32 * cb < U) tma_store_4d(&tmO, bx + cb * 4096, half * 64 + 32 * cb, h, quarter * 32, bb);
          bulk_commit();
        }
      } else if (half == 0) {
        // MHAttentionOut (NeuroNet.cl:1730-1759): O[q][h][d], the quarter's 32 rows as one box
        uint8_t *bx = smem + C::EPI_OFF + quarter * 4096;
        float v[32];
        tmem_ld32(trow, v);
        if (lane == 0) bulk_wait_read<0>();
        __syncwarp();
#pragma unroll
        for (int g = 0; g < 8; ++g)
          *reinterpret_cast<float4 *>(bx + lane * 128 + (((g ^ lane) & 7) << 4)) =
              make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && quarter * 32 < U) {
          tma_store_4d(&tmO, bx, 0, h, quarter * 32, bb);
          bulk_commit();
        }
      }
      tc_fence_before();
      mbar_arrive(&acce[b]);
    }
    // the boxes must be read, and the stores complete, before the CTA exits
    if (lane == 0) bulk_wait<0>();
    __syncwarp();
  }

  // ------------------------------------------------------------ teardown
  if (warp == kMmaWarp) {
    if (lane == 0) mma_commit(&drain);
    __syncwarp();
    if (!mbar_wait_drain(&drain, 0) && lane == 0) atomicExch(err, kErrDoneWait);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ gradient
// MHAttentionInsideGradients (NeuroNet.cl:1777-1845) for one (sequence, head) per work item, with
// V0[u] = V[u][0] and A[q] = sum_u S[q][u] V0[u]:
//   dV = S^T G,   C = S o (V0^T - A),   dK = C^T (G o Q) / koef,   dQ = G o (C K) / koef.
// Shared memory (one item at a time, 210 KB):
//   SH / SL  S, then C: hi / lo, [u-group (4)][q row (128)][32 u], 64 KB each
//   GH / GL and XH / XL  two 32 KB hi / lo pairs [q row][32 d] that swap roles from item to item:
//            one holds G (later K, dQ's B operand), the other G o Q
//   QR       raw Q, later raw K, [row][32 d], 16 KB
//   V0, AV   128 floats each;  VR: V[u][0..3] per row (TMA), the source of V0
// Tensor memory (512 columns): dV, dK, dQ accumulators at columns 0, 32, 64; C's rows hi / lo at
// 128-255 / 256-383 (lane q = row q, column u), dQ's A operand.
// S, G, Q and K tiles use the 128-byte swizzle with 32-byte granules (MN-major operands of dV and
// dK).  Score rows q >= units (the next sequence) are zeroed, so they contribute nothing to the sums
// over q.
// Overlap: dV reduces over q in 8-row steps, so the workers hand S over in 32-row chunks of q, each
// with its own barrier; G o Q and A are formed while dV runs, K is split and C copied into tensor
// memory while dK runs.  The next item's V rows, Q and G load as soon as dK has read G o Q (the next
// G goes into that pair) and K has been split out of QR, and its S once dK has read C and the
// workers have copied it (dQ's factor G is read from global memory, so the epilogue needs no shared
// tile).
struct GradCfg {
  static constexpr uint32_t SH = 0, SL = 65536, GH = 131072, GL = 147456, QR = 163840, XH = 180224, XL = 196608;
  static constexpr uint32_t V0 = 212992, AV = V0 + 512, VR = AV + 512, END = VR + 2048;
  static constexpr uint32_t SMEM = END + 1024;
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

__global__ void __launch_bounds__(320, 1)
    attn_grad_tc_kernel(const float *__restrict__ qkv, const float *__restrict__ grad, float *__restrict__ qkv_g,
                        int *err, int U, int H, int items, float koef, const __grid_constant__ CUtensorMap tmS,
                        const __grid_constant__ CUtensorMap tmQKV, const __grid_constant__ CUtensorMap tmG,
                        const __grid_constant__ CUtensorMap tmV0) {
  using C = GradCfg;
  constexpr int D = 32;
  constexpr uint32_t IDESC_MN = instr_desc_tf32(128, 32, true, true);   // dV, dK
  constexpr uint32_t IDESC_KM = instr_desc_tf32(128, 32, false, true);  // dQ
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *sm = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  float *V0s = reinterpret_cast<float *>(sm + C::V0), *AVs = reinterpret_cast<float *>(sm + C::AV);
  // w1[j]: S and G rows of q-chunk j split (dV may read them); mq[h]: dK has read C's q-chunks 2h,
  // 2h+1; w3: C is in tensor memory and K split (dQ may run, the next S may land); kfree: the workers
  // have split K out of QR
  __shared__ __align__(8) uint64_t ld1, ld2, w1[4], w2, w3, m1, mq[2], accf, qfree, kfree, wsync, drain;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  auto fail = [&](int code) {
    abort_flag = 1;
    atomicExch(err, code);
  };
  if (tid == 0) {
    mbar_init(&ld1, 1);
    mbar_init(&ld2, 1);
    for (int j = 0; j < 4; ++j) mbar_init(&w1[j], 256);
    for (int j = 0; j < 2; ++j) mbar_init(&mq[j], 1);
    mbar_init(&w2, 256);
    mbar_init(&w3, 256);
    mbar_init(&m1, 1);
    mbar_init(&accf, 1);
    mbar_init(&qfree, 256);
    mbar_init(&kfree, 256);
    mbar_init(&wsync, 256);
    mbar_init(&drain, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 8) {
    tmem_alloc(&tmem_slot, 512);  // one CTA per SM (217 KB of shared memory)
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;  // dV at column 0, dK at 32, dQ at 64; C hi at 128, lo at 256
  pdl_wait();
  pdl_trigger();
  const float inv_koef = 1.f / koef;
  const size_t rs = (size_t)3 * H * D;  // qkv row stride

  if (warp == 9) {
    // ------------------------------------------------------------ loader
    // Item n+1's tiles load while item n still runs: its V0 rows, Q and G once item n's dK
    // products have read G o Q (G and G o Q swap buffers from item to item) and its workers have
    // split K out of QR; its S u-groups 0-1 once item n's dQ products have passed them, 2-3 once
    // they are done.  One ld1 phase per item counts all of these copies.
    if (lane == 0) {
      int n = 0, issued1 = 0, issued2 = 0;
      auto load_vqg = [&](int t, int nn) {
        const int b = t / H, h = t % H;
        const uint32_t gbuf = (nn & 1) ? C::XH : C::GH;
        mbar_arrive_expect_tx(&ld1, 65536u + 16384u + 16384u + 2048u);
        tma_load_3d(sm + C::VR, &tmV0, (2 * H + h) * D, b * U, 0, &ld1);
        for (int qc = 0; qc < 4; ++qc) {
          tma_load_3d(sm + gbuf + qc * 4096, &tmG, h * D, b * U + 32 * qc, 0, &ld1);
          tma_load_3d(sm + C::QR + qc * 4096, &tmQKV, h * D, b * U + 32 * qc, 0, &ld1);
        }
      };
      auto load_s = [&](int t, int ug0) {
        const int b = t / H, h = t % H;
        for (int ug = ug0; ug < ug0 + 2; ++ug)
          for (int qc = 0; qc < 4; ++qc)
            tma_load_3d(sm + C::SH + ug * 16384 + qc * 4096, &tmS, 32 * ug, h, b * U + 32 * qc, &ld1);
      };
      int t = blockIdx.x;
      if (t < items) {
        load_vqg(t, 0);
        load_s(t, 0);
        load_s(t, 2);
        ++issued1;
      }
      for (; t < items && !abort_flag; t += gridDim.x, ++n) {
        const int b = t / H, h = t % H;
        const uint32_t par = n & 1;
        // raw K into QR once the workers have consumed Q
        if (!mbar_wait(&qfree, par, &abort_flag)) {
          fail(kErrEmptyWait);
          break;
        }
        mbar_arrive_expect_tx(&ld2, 16384u);
        ++issued2;
        for (int uc = 0; uc < 4; ++uc)
          tma_load_3d(sm + C::QR + uc * 4096, &tmQKV, (H + h) * D, b * U + 32 * uc, 0, &ld2);
        const int tn = t + gridDim.x;
        if (tn >= items) continue;
        if (!mbar_wait(&mq[1], par, &abort_flag) || !mbar_wait(&kfree, par, &abort_flag)) {
          fail(kErrEmptyWait);
          break;
        }
        load_vqg(tn, n + 1);
        ++issued1;
        // S / C's shared tiles are free once dK has read them (mq[1], above) and the workers have
        // copied C into tensor memory (w3)
        if (!mbar_wait(&w3, par, &abort_flag)) {
          fail(kErrEmptyWait);
          break;
        }
        load_s(tn, 0);
        load_s(tn, 2);
      }
      // wait for the last copies into shared memory before exiting
      if (issued1 > 0 && !mbar_wait_drain(&ld1, (issued1 - 1) & 1) && !abort_flag) fail(kErrFullWait);
      if (issued2 > 0 && !mbar_wait_drain(&ld2, (issued2 - 1) & 1) && !abort_flag) fail(kErrFullWait);
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------ MMA issue
    // Operand descriptors from one shared base (address / 16) plus compile-time tile offsets: the
    // issuing lane shares its sub-partition with two busy worker warps, so every issue instruction
    // saved shortens the MMA chain.  MN-major S / C, G (later K) and G o Q tiles: 1024 bytes per
    // 8 rows of q; K-major C: 16384 bytes per u-group, 32 bytes per 8-wide k step.
    const uint32_t b16 = smem_u32(sm) >> 4;
    auto Sm = [&](uint32_t base, int s) { return desc_at<16384u, 512u, 1u>(b16 + (base >> 4) + 64u * s); };
    auto Tm = [&](uint32_t base, int s) { return desc_at<4096u, 512u, 1u>(b16 + (base >> 4) + 64u * s); };
    int n = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < items && ok && !abort_flag; t += gridDim.x, ++n) {
      const uint32_t par = n & 1;
      // G (later K) and G o Q swap their 32 KB buffers from item to item
      const uint32_t gbuf = par ? C::XH : C::GH, xbuf = par ? C::GH : C::XH;
      // dV = S^T G, k-steps s (q rows 8s..8s+7) issued as the workers release each 32-row chunk
      for (int j = 0; j < 4 && ok; ++j) {
        if (!mbar_wait(&w1[j], par, &abort_flag)) {
          if (lane == 0) fail(kErrFullWait);
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int s = 4 * j + i;
            mma_tf32(tmem, Sm(C::SL, s), Tm(gbuf, s), IDESC_MN, s != 0 ? 1u : 0u);
            mma_tf32(tmem, Sm(C::SH, s), Tm(gbuf + 16384u, s), IDESC_MN, 1u);
            mma_tf32(tmem, Sm(C::SH, s), Tm(gbuf, s), IDESC_MN, 1u);
          }
          if (j == 3) mma_commit(&m1);
        }
        __syncwarp();
      }
      if (!ok) break;
      // dK' = C^T (G o Q), with a commit after every second 32-row chunk of q so that the workers
      // can permute the rows it no longer reads
      if (!mbar_wait(&w2, par, &abort_flag)) {
        if (lane == 0) fail(kErrFullWait);
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        for (int j = 0; j < 4; ++j) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int s = 4 * j + i;
            mma_tf32(tmem + 32, Sm(C::SL, s), Tm(xbuf, s), IDESC_MN, s != 0 ? 1u : 0u);
            mma_tf32(tmem + 32, Sm(C::SH, s), Tm(xbuf + 16384u, s), IDESC_MN, 1u);
            mma_tf32(tmem + 32, Sm(C::SH, s), Tm(xbuf, s), IDESC_MN, 1u);
          }
          if (j & 1) mma_commit(&mq[j >> 1]);
        }
      }
      __syncwarp();
      // dQ' = C K  (C from tensor memory, lane q = row q, 8 columns of u per k step; K split in GH/GL)
      if (!mbar_wait(&w3, par, &abort_flag)) {
        if (lane == 0) fail(kErrFullWait);
        break;
      }
      tc_fence_after();
      if (lane == 0) {
#pragma unroll
        for (int s = 0; s < 16; ++s) {
          mma_tf32_ta(tmem + 64, tmem + 256 + 8 * s, Tm(gbuf, s), IDESC_KM, s != 0 ? 1u : 0u);
          mma_tf32_ta(tmem + 64, tmem + 128 + 8 * s, Tm(gbuf + 16384u, s), IDESC_KM, 1u);
          mma_tf32_ta(tmem + 64, tmem + 128 + 8 * s, Tm(gbuf, s), IDESC_KM, 1u);
        }
        mma_commit(&accf);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ workers (warps 0-7)
    const int wt = tid;  // 0..255
    uint32_t nsync = 0;
    // bounded barrier among the 256 workers (an mbarrier phase per use)
    auto worker_sync = [&]() -> bool {
      mbar_arrive(&wsync);
      const bool ok = mbar_wait(&wsync, nsync & 1, &abort_flag);
      ++nsync;
      return ok;
    };
    int n = 0;
    for (int t = blockIdx.x; t < items && !abort_flag; t += gridDim.x, ++n) {
      const int b = t / H, h = t % H;
      const uint32_t par = n & 1;
      // G (later K) and G o Q swap their 32 KB hi / lo buffers from item to item
      const uint32_t gbuf = par ? C::XH : C::GH, xbuf = par ? C::GH : C::XH;
      if (!mbar_wait(&ld1, par, &abort_flag)) {
        fail(kErrFullWait);
        break;
      }
      // V0 (feature 0 of V) for every unit of the tile; zero past `units`
      if (wt < 128) V0s[wt] = wt < U ? nan0(reinterpret_cast<const float *>(sm + C::VR)[4 * wt]) : 0.f;
      // W1, per 32-row chunk j of q: split S (rows q >= units zeroed) and G, then release the chunk
      // to dV.  Thread wt handles row 32j + wt/8 of each u-group, 16 bytes at a time: the same four
      // units u of each u-group for every j (the 32-byte granule order of a row depends on q % 4
      // only), whose V0 it keeps in registers to form its share of A[q] = sum_u S[q][u] V0[u];
      // the eight threads of a row (consecutive lanes) then add their shares.
      float v0r[4][4];
      {
        const float *vr = reinterpret_cast<const float *>(sm + C::VR);  // V[u][0..3] per row u
        const int c = ((((wt & 7) >> 1) ^ (wt >> 3)) & 3) * 8 + (wt & 1) * 4;
#pragma unroll
        for (int ug = 0; ug < 4; ++ug)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int uu = 32 * ug + c + i;
            v0r[ug][i] = uu < U ? nan0(vr[4 * uu]) : 0.f;
          }
      }
      for (int j = 0; j < 4; ++j) {
        const int q = 32 * j + (wt >> 3);
        const uint32_t off = 4096u * j + 16u * wt;
        float a = 0.f;
        if (q >= U) {
#pragma unroll
          for (int ug = 0; ug < 4; ++ug) {
            *reinterpret_cast<float4 *>(sm + C::SH + 16384u * ug + off) = make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4 *>(sm + C::SL + 16384u * ug + off) = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        } else {
          float4 x[4];
#pragma unroll
          for (int ug = 0; ug < 4; ++ug) x[ug] = *reinterpret_cast<const float4 *>(sm + C::SH + 16384u * ug + off);
#pragma unroll
          for (int ug = 0; ug < 4; ++ug) {
            const float4 v = make_float4(nan0(x[ug].x), nan0(x[ug].y), nan0(x[ug].z), nan0(x[ug].w));
            store_split_full(sm + C::SH, sm + C::SL, 16384u * ug + off, v);
            a = fmaf(v.x, v0r[ug][0], a);
            a = fmaf(v.y, v0r[ug][1], a);
            a = fmaf(v.z, v0r[ug][2], a);
            a = fmaf(v.w, v0r[ug][3], a);
          }
        }
        a += __shfl_xor_sync(0xffffffffu, a, 1);
        a += __shfl_xor_sync(0xffffffffu, a, 2);
        a += __shfl_xor_sync(0xffffffffu, a, 4);
        if ((wt & 7) == 0) AVs[q] = a;
        split_chunks<1>(sm + gbuf, sm + gbuf + 16384u, off, 0u);
        fence_proxy_async_smem();
        mbar_arrive(&w1[j]);
      }
      // G o Q -> XH / XL (dK's B operand) while dV runs
      {
        float4 g[4], qv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          g[i] = *reinterpret_cast<const float4 *>(sm + gbuf + 16u * (wt + 256 * i));
          qv[i] = *reinterpret_cast<const float4 *>(sm + C::QR + 16u * (wt + 256 * i));
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
          store_split_full(sm + xbuf, sm + xbuf + 16384u, 16u * (wt + 256 * i),
                           make_float4(g[i].x * qv[i].x, g[i].y * qv[i].y, g[i].z * qv[i].z, g[i].w * qv[i].w));
      }
      fence_proxy_async_smem();
      mbar_arrive(&qfree);  // raw Q consumed: the loader brings raw K into QR
      if (!worker_sync()) {  // V0 and A complete before W2 reads them
        fail(kErrFullWait);
        break;
      }
      // W2: C = S o (V0[u] - A[q]) in place, once the dV MMAs have read S
      if (!mbar_wait(&m1, par, &abort_flag)) {
        fail(kErrDoneWait);
        break;
      }
      tc_fence_after();
      for (int f0 = 0; f0 < 16; f0 += 4) {  // four chunks at a time: their loads overlap
        float4 sv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) sv[i] = *reinterpret_cast<const float4 *>(sm + C::SH + 16u * (wt + 256 * (f0 + i)));
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t off = 16u * (wt + 256 * (f0 + i));
          const int ug = off >> 14, q = (off & 16383u) >> 7;
          const int c0 = ((((off & 127u) >> 5) ^ q) & 3) * 8 + ((off & 31u) >> 2);  // logical column of lane 0
          const float4 hi = sv[i];  // the full fp32 S
          const float aq = AVs[q];
          const float4 v = *reinterpret_cast<const float4 *>(V0s + 32 * ug + c0);
          store_split_full(sm + C::SH, sm + C::SL, off,
                           make_float4(hi.x * (v.x - aq), hi.y * (v.y - aq), hi.z * (v.z - aq), hi.w * (v.w - aq)));
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&w2);
      // Results leave as soon as their products are complete, each warp storing half of its rows'
      // 32 features (warps 0-3 the first 16, warps 4-7 the last): row r of tensor-memory lane
      // quarter w % 4, 64 bytes per row and result.  dV is complete (m1, waited above).
      const int r = (warp & 3) * 32 + lane, f0 = 16 * (warp >> 2);
      const uint32_t tl = tmem + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)f0;
      float *grow = qkv_g + (size_t)(b * U + r) * rs + f0;  // 32-byte aligned: 3*H*D floats per row
      {
        float v[16];
        tmem_ld16(tl + 0, v);
        if (r < U) {
          float *dv = grow + (size_t)(2 * H + h) * D;
          st_global_v8(dv, v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7]);
          st_global_v8(dv + 8, v[8], v[9], v[10], v[11], v[12], v[13], v[14], v[15]);
        }
      }
      // raw K -> GH / GL (dQ's B operand) while dK runs: dV has finished reading G
      if (!mbar_wait(&ld2, par, &abort_flag)) {
        fail(kErrFullWait);
        break;
      }
      {
        float4 kv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) kv[i] = *reinterpret_cast<const float4 *>(sm + C::QR + 16u * (wt + 256 * i));
#pragma unroll
        for (int i = 0; i < 4; ++i) store_split_full(sm + gbuf, sm + gbuf + 16384u, 16u * (wt + 256 * i), kv[i]);
      }
      mbar_arrive(&kfree);  // QR (raw K) and VR read: the loader may bring the next item's Q and V rows
      // W3: C's rows into tensor memory as dQ's A operand (lane q = row q, one column per u: hi at
      // columns 128-255, lo at 256-383), read from the hi tiles W2 wrote (dK reads the same tiles
      // meanwhile; nothing waits for it).  Warp w takes rows 32 (w % 4) .. +31, its tensor-memory
      // lanes, and u-groups 2 (w / 4) and 2 (w / 4) + 1.  Every thread's W2 rows are written first.
      if (!worker_sync()) {
        fail(kErrFullWait);
        break;
      }
      {
        const int q = 32 * (warp & 3) + lane;
        const uint32_t trow = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const int ug = 2 * (warp >> 2) + h2;
          const uint8_t *row = sm + C::SH + 16384u * ug + 128u * q;
          uint32_t hi[32], lo[32];
#pragma unroll
          for (int gi = 0; gi < 4; ++gi)
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              // logical 32-byte granule gi of an MN-major row sits at granule gi ^ (q % 4)
              const float4 v = *reinterpret_cast<const float4 *>(row + 16 * ((((gi ^ q) & 3) << 1) | hf));
              const int u = 8 * gi + 4 * hf;
              hi[u] = __float_as_uint(v.x);
              hi[u + 1] = __float_as_uint(v.y);
              hi[u + 2] = __float_as_uint(v.z);
              hi[u + 3] = __float_as_uint(v.w);
              lo[u] = __float_as_uint(v.x - tf32_hi(v.x));
              lo[u + 1] = __float_as_uint(v.y - tf32_hi(v.y));
              lo[u + 2] = __float_as_uint(v.z - tf32_hi(v.z));
              lo[u + 3] = __float_as_uint(v.w - tf32_hi(v.w));
            }
          tmem_st32(trow + 128 + 32 * ug, hi);
          tmem_st32(trow + 256 + 32 * ug, lo);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      fence_proxy_async_smem();
      mbar_arrive(&w3);
      // dK, once its products are complete, while dQ runs; dQ's factor G (its row in global memory:
      // TMA brought it into L2) loads before the wait for dQ, so its latency overlaps the products
      float4 gq[4];
      if (r < U) {
        const float4 *gr =
            reinterpret_cast<const float4 *>(grad + (size_t)(b * U + r) * H * D + (size_t)h * D + f0);
#pragma unroll
        for (int l16 = 0; l16 < 4; ++l16) gq[l16] = __ldg(gr + l16);
      }
      if (!mbar_wait(&mq[1], par, &abort_flag)) {
        fail(kErrDoneWait);
        break;
      }
      tc_fence_after();
      {
        float k[16];
        tmem_ld16(tl + 32, k);
        if (r < U) {
          float *dk = grow + (size_t)(H + h) * D;
          st_global_v8(dk, k[0] * inv_koef, k[1] * inv_koef, k[2] * inv_koef, k[3] * inv_koef, k[4] * inv_koef,
                       k[5] * inv_koef, k[6] * inv_koef, k[7] * inv_koef);
          st_global_v8(dk + 8, k[8] * inv_koef, k[9] * inv_koef, k[10] * inv_koef, k[11] * inv_koef,
                       k[12] * inv_koef, k[13] * inv_koef, k[14] * inv_koef, k[15] * inv_koef);
        }
      }
      if (!mbar_wait(&accf, par, &abort_flag)) {
        fail(kErrDoneWait);
        break;
      }
      tc_fence_after();
      {
        float v[16];
        tmem_ld16(tl + 64, v);
        if (r < U) {
          float gf[16];
#pragma unroll
          for (int l16 = 0; l16 < 4; ++l16) {
            gf[4 * l16] = nan0(gq[l16].x);
            gf[4 * l16 + 1] = nan0(gq[l16].y);
            gf[4 * l16 + 2] = nan0(gq[l16].z);
            gf[4 * l16 + 3] = nan0(gq[l16].w);
          }
          float *dq = grow + (size_t)h * D;
#pragma unroll
          for (int j = 0; j < 2; ++j)
            st_global_v8(dq + 8 * j, gf[8 * j] * v[8 * j] * inv_koef, gf[8 * j + 1] * v[8 * j + 1] * inv_koef,
                         gf[8 * j + 2] * v[8 * j + 2] * inv_koef, gf[8 * j + 3] * v[8 * j + 3] * inv_koef,
                         gf[8 * j + 4] * v[8 * j + 4] * inv_koef, gf[8 * j + 5] * v[8 * j + 5] * inv_koef,
                         gf[8 * j + 6] * v[8 * j + 6] * inv_koef, gf[8 * j + 7] * v[8 * j + 7] * inv_koef);
        }
      }
      tc_fence_before();
    }
  }

  // ------------------------------------------------------------ teardown
  if (warp == 8) {
    if (lane == 0) mma_commit(&drain);
    __syncwarp();
    if (!mbar_wait_drain(&drain, 0) && lane == 0) atomicExch(err, kErrDoneWait);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace tc

// Whether the tensor-core attention products apply: head dimension 32, at most 128 units, every
// tensor 16-byte aligned (units a multiple of 4 for the score rows).
inline bool attn_tc_ok(const float *qkv, const float *scores, int U, int H, int D) {
  return tensor_gemm_enabled() && tmap_encoder() && D == 32 && U >= 1 && U <= 128 && U % 4 == 0 && H >= 1 &&
         ((uintptr_t)qkv & 15) == 0 && ((uintptr_t)scores & 15) == 0;
}

inline bool make_tmap2(CUtensorMap *tm, const float *p, int rank, const cuuint64_t *dims, const cuuint64_t *strides,
                       const cuuint32_t *box, bool mn_major) {
  cuuint32_t es[5] = {1u, 1u, 1u, 1u, 1u};
  return tmap_encoder()(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank, const_cast<float *>(p), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// MODE kAttnScore: scores = softmax(Q K^T / koef); MODE kAttnOut: out = scores V.
template <int MODE>
inline cudaError_t attn_tc(const float *qkv, const float *scores, float *out, int B, int U, int H, int mask,
                           float koef, cudaStream_t st) {
  using C = tc::AttnCfg<MODE>;
  const int D = 32;
  CUtensorMap tmQ, tmS, tmV, tmO;
  std::memset(&tmQ, 0, sizeof tmQ);
  std::memset(&tmS, 0, sizeof tmS);
  std::memset(&tmV, 0, sizeof tmV);
  {  // the output, [B][U][H][inner] with inner = U keys (score) or D features (out)
    const cuuint64_t inner = MODE == tc::kAttnScore ? (cuuint64_t)U : (cuuint64_t)D;
    cuuint64_t od[4] = {inner, (cuuint64_t)H, (cuuint64_t)U, (cuuint64_t)B};
    cuuint64_t os[3] = {inner * 4, inner * H * 4, inner * H * U * 4};
    cuuint32_t ob[4] = {32u, 1u, 32u, 1u};
    if (!make_tmap2(&tmO, out, 4, od, os, ob, false)) return cudaErrorInvalidValue;
  }
  const cuuint64_t rows = (cuuint64_t)B * U, width = (cuuint64_t)3 * H * D;
  // every map is rank 3 (the loads are 3-d; a trailing extent of 1 where the tensor is 2-d)
  if (MODE == tc::kAttnScore) {
    cuuint64_t dims[3] = {width, rows, 1}, strides[2] = {width * 4, width * 4 * rows};
    cuuint32_t box[3] = {32u, 128u, 1u};
    if (!make_tmap2(&tmQ, qkv, 3, dims, strides, box, false)) return cudaErrorInvalidValue;
  } else {
    cuuint64_t sd[3] = {(cuuint64_t)U, (cuuint64_t)H, rows}, ss[2] = {(cuuint64_t)U * 4, (cuuint64_t)H * U * 4};
    cuuint32_t sb[3] = {32u, 1u, 128u};
    if (!make_tmap2(&tmS, scores, 3, sd, ss, sb, false)) return cudaErrorInvalidValue;
    cuuint64_t vd[3] = {width, rows, 1}, vs[2] = {width * 4, width * 4 * rows};
    cuuint32_t vb[3] = {32u, 32u, 1u};
    if (!make_tmap2(&tmV, qkv, 3, vd, vs, vb, true)) return cudaErrorInvalidValue;
  }
  auto fn = tc::attn_tc_kernel<MODE>;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int items = B * H;
  if (items <= 0) return cudaSuccess;
  const int grid = items < sm_count() ? items : sm_count();
  return launch_pdl(fn, grid, dim3(448), C::SMEM, st, device_status(), U, H, items, mask, koef, tmQ, tmS, tmV, tmO);
}

// MHAttentionInsideGradients on the tensor cores (same applicability as attn_tc_ok; `grad` 16-byte and
// `qkv_g` 32-byte aligned).
inline cudaError_t attn_grad_tc(const float *qkv, float *qkv_g, const float *scores, const float *grad, int B, int U,
                                int H, float koef, cudaStream_t st) {
  const int D = 32;
  CUtensorMap tmS, tmQKV, tmG, tmV0;
  const cuuint64_t rows = (cuuint64_t)B * U, width = (cuuint64_t)3 * H * D, gw = (cuuint64_t)H * D;
  {  // the first 4 features of each V row (feature 0 is V0), no swizzle: row u at 16*u bytes
    cuuint64_t d[3] = {width, rows, 1}, s[2] = {width * 4, width * 4 * rows};
    cuuint32_t bx[3] = {4u, 128u, 1u}, es[3] = {1u, 1u, 1u};
    if (tmap_encoder()(&tmV0, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(qkv), d, s, bx, es,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {
    cuuint64_t d[3] = {(cuuint64_t)U, (cuuint64_t)H, rows}, s[2] = {(cuuint64_t)U * 4, (cuuint64_t)H * U * 4};
    cuuint32_t bx[3] = {32u, 1u, 32u};
    if (!make_tmap2(&tmS, scores, 3, d, s, bx, true)) return cudaErrorInvalidValue;
  }
  {
    cuuint64_t d[3] = {width, rows, 1}, s[2] = {width * 4, width * 4 * rows};
    cuuint32_t bx[3] = {32u, 32u, 1u};
    if (!make_tmap2(&tmQKV, qkv, 3, d, s, bx, true)) return cudaErrorInvalidValue;
  }
  {
    cuuint64_t d[3] = {gw, rows, 1}, s[2] = {gw * 4, gw * 4 * rows};
    cuuint32_t bx[3] = {32u, 32u, 1u};
    if (!make_tmap2(&tmG, grad, 3, d, s, bx, true)) return cudaErrorInvalidValue;
  }
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(tc::attn_grad_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)tc::GradCfg::SMEM);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int items = B * H;
  if (items <= 0) return cudaSuccess;
  const int grid = items < sm_count() ? items : sm_count();
  return launch_pdl(tc::attn_grad_tc_kernel, grid, dim3(320), tc::GradCfg::SMEM, st, qkv, grad, qkv_g,
                    device_status(), U, H, items, koef, tmS, tmQKV, tmG, tmV0);
}

}  // namespace nn
