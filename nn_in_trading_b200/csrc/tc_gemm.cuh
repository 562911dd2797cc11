// FP32 GEMM on the 5th-generation tensor cores (tcgen05, kind::tf32) with the
// 3xTF32 split, for the same strided operands and per-element epilogue as
// sgemm_fast (gemm_fast.cuh):
//   acc[m][n] = sum_k A(m,k) B(k,n)
//   A(m,k) = A[m*lda + k]  (A_MCONTIG = false, K-major)   or  A[k*lda + m]  (true, MN-major)
//   B(k,n) = B[n*ldb + k]  (B_NCONTIG = false, K-major)   or  B[k*ldb + n]  (true, MN-major)
// blockIdx.z enumerates (split, z) exactly as in sgemm_fast.
//
// Accuracy.  Every operand x (after nan0) is split into hi = x with its low 13
// mantissa bits cleared (exactly a TF32 value) and lo = x - hi (exact in FP32);
// the tile product is lo_A*hi_B + hi_A*lo_B + hi_A*hi_B accumulated in FP32 in
// tensor memory.  The dropped lo*lo term and the TF32 truncation of lo are
// below 2^-21 relative per product, the same order as FP32 rounding.
//
// Persistent CTAs (one per SM) walk the 128 x BN output tiles, 9 warps each:
//   warps 4-7  producers: global fp32 -> registers -> nan0 -> hi/lo split ->
//              shared memory in the tensor cores' canonical layout, one
//              mbarrier arrive per thread per stage of a STAGES-deep ring.
//   warp 8     allocates 2*BN tensor-memory columns (two accumulators), issues
//              the MMAs from one lane (3 per 8-wide k step), releases a stage
//              with tcgen05.commit, and frees the columns at the end.
//   warps 0-3  epilogue: tcgen05.ld of their 32 tensor-memory lanes, a
//              transpose through shared memory, and the epilogue functor with
//              lanes along n (coalesced stores), while the MMAs of the next
//              tile run into the other accumulator.
// A operand in tensor memory.  When TMA brings the A tiles in (every variant whose A tensor TMA can
// address), the producers do not split A in shared memory: each thread reads its row's 16 k values of
// the raw tile, writes hi and lo into tensor-memory columns of the stage (tcgen05.st, 32 lanes per
// warp; lane m = row m, one column per k) and the MMAs read A from there (tcgen05.mma with [a_tmem]).
// Shared memory then carries the raw A tile and B only, and the tensor cores read only B from it: the
// CTA allocates all 512 columns (two accumulators of BN columns, then 2 x 32 columns of A per stage),
// which also frees shared memory for 4 stages at BN = 128 and 6 at BN = 64 (3 and 4 with A split in
// shared memory).  An MMA
// that reads a stage's A columns completes before the stage's empty barrier fires (tcgen05.commit), so
// the producers overwrite the columns only after that wait; they wait for their own stores
// (tcgen05.wait::st) before they signal the stage full.
// Every mbarrier wait is bounded (about one second of clock, plus an
// iteration cap): on expiry the thread raises a CTA-wide abort flag and writes
// a code to `err` (read back by nn_finish), and all roles drain to the common
// exit, where the MMA warp waits (again bounded) for the MMAs it issued
// before freeing tensor memory.
//
// Shared-memory layout of one operand tile (R rows of the MN extent, BK k),
// per float4 chunk q (a warp's 32 consecutive chunks fill 512 contiguous
// bytes: no bank conflicts):
//   K-major, no swizzle (8-row x 16-byte core matrices): chunk q at byte 16*q,
//     row 8*(q / (2*BK)) + q%8, k 4*((q/8) % (BK/4)); core-matrix strides
//     K (LBO) 128 B, MN (SBO) 32*BK B.  Global: eight 64-byte row segments.
//   MN-major, the 128-byte swizzle with 32-byte granules (layout type 1, the
//     one layout the tensor cores accept for MN-major 32-bit operands): atoms
//     of 4 k-rows x 32 MN elements (512 B), the four 32-byte granules of row r
//     of an atom XOR-permuted by r.  Chunk q: atom a = q/32 (k-group
//     a % (BK/4), MN-group a / (BK/4)), row (q%32)/8, granule/half from q%8.
//     Strides: MN groups (LBO) 128*BK B, k groups (SBO) 512 B.  Global: four
//     128-byte row segments.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <type_traits>
#include <utility>

#include "gemm_fast.cuh"
#include "nn_device.cuh"
#include "nn_internal.h"

namespace nn {
namespace tc {

constexpr long long kWaitCycles = 2000000000LL;  // ~1 s at 1.9 GHz
constexpr uint32_t kWaitIters = 1u << 26;

// codes written to the status word
constexpr int kErrFullWait = 1, kErrEmptyWait = 2, kErrDoneWait = 3;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity; false on expiry or abort.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  const long long t0 = clock64();
  for (uint32_t it = 0; it < kWaitIters; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) return false;
  }
  return false;
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// One contiguous global -> shared copy by the bulk-copy engine, counted on `bar` (no multicast).
__device__ __forceinline__ void bulk_copy_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// Bounded wait that ignores the abort flag: used only to drain this CTA's own asynchronous copies and
// MMAs before it exits.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t *bar, uint32_t parity) {
  const long long t0 = clock64();
  for (uint32_t it = 0; it < kWaitIters; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - t0 > kWaitCycles) return false;
  }
  return false;
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Shared-memory matrix descriptor (sm100 version 1): layout 0 = no swizzle, 1 = 128-byte swizzle
// with 32-byte granules.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)(layout & 7u) << 61);
}

// Byte offset of float4 chunk q in an operand tile, and the (row, k) of its first element.
template <bool KMAJ, int R, int BK>
__device__ __forceinline__ uint32_t chunk_place(int q, int &row, int &k) {
  if (KMAJ) {
    row = 8 * (q / (2 * BK)) + q % 8;
    k = 4 * ((q / 8) % (BK / 4));
    return 16u * (uint32_t)q;
  }
  const int a = q / 32, w = q % 32;
  const int g = a % (BK / 4), h = a / (BK / 4);
  const int kr = w / 8, c = w % 8;
  row = 32 * h + 4 * c;
  k = 4 * g + kr;
  return (uint32_t)(h * 128 * BK + g * 512 + kr * 128 + (((c >> 1) ^ kr) * 32) + (c & 1) * 16);
}

// Instruction descriptor of kind::tf32: D f32, A/B tf32, majors, N>>3, M>>4.
__host__ __device__ constexpr uint32_t instr_desc_tf32(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// smem_desc with the strides and layout as compile-time constants and the address already divided
// by 16: the 64-bit descriptor is one 32-bit add away from a shared base, so a loop of MMAs keeps
// one register for all its operand tiles instead of a 64-bit descriptor per tile.
template <uint32_t LBO, uint32_t SBO, uint32_t LAYOUT>
__device__ __forceinline__ uint64_t desc_at(uint32_t addr16) {
  constexpr uint32_t lo = ((LBO >> 4) & 0x3FFFu) << 16;
  constexpr uint32_t hi = ((SBO >> 4) & 0x3FFFu) | (1u << 14) | ((LAYOUT & 7u) << 29);
  return ((uint64_t)hi << 32) | (uint64_t)((addr16 & 0x3FFFu) | lo);
}
__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same with A read from tensor memory: tmem_a addresses the 8 columns (one k step) of the A
// tile, row m of A in lane m.
__device__ __forceinline__ void mma_tf32_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// tcgen05.st of 16 consecutive 32-bit columns into this warp's 32 lanes (lane l gets r[] of thread l).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
// tcgen05.st of 32 consecutive 32-bit columns into this warp's 32 lanes.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// every tcgen05.st this thread issued has completed
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive fp32 columns of this warp's 32 lanes: v[j] = D[lane][col + j].
// tcgen05.ld of 32 columns of the warp's 32 lanes, not yet waited for
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// tcgen05.wait::ld (every load this thread issued), naming r so that no use of it is scheduled before
__device__ __forceinline__ void tmem_wait_into(uint32_t (&r)[32], float (&v)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
        "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
        "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
        "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}
// 16 consecutive fp32 columns of this warp's 32 lanes, waited for: v[j] = D[lane][col + j].
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  tmem_ld32_issue(taddr, r);
  tmem_wait_into(r, v);
}

__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u); }

// One float4 chunk of an operand tile, zero outside [0, rows) x [kbeg, kend), and 1 in row
// `ones_row` (for k < kend) when that row is the all-ones column of B.
//   KMAJ: element (row, k) at G[row*ld + k];  else at G[k*ld + row].
template <bool KMAJ>
__device__ __forceinline__ float4 load_chunk(const float *G, long long ld, int row, int k, int rows, int kend,
                                             bool vec, int ones_row = -1) {
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (KMAJ) {
    if (row == ones_row) {
      v.x = k < kend ? 1.f : 0.f;
      v.y = k + 1 < kend ? 1.f : 0.f;
      v.z = k + 2 < kend ? 1.f : 0.f;
      v.w = k + 3 < kend ? 1.f : 0.f;
      return v;
    }
    if (row >= rows) return v;
    const float *p = G + (size_t)row * ld + k;
    if (vec && k + 3 < kend) return *reinterpret_cast<const float4 *>(p);
    if (k < kend) v.x = p[0];
    if (k + 1 < kend) v.y = p[1];
    if (k + 2 < kend) v.z = p[2];
    if (k + 3 < kend) v.w = p[3];
  } else {
    if (k >= kend) return v;
    const float *p = G + (size_t)k * ld + row;
    if (vec && row + 3 < rows) return *reinterpret_cast<const float4 *>(p);
    if (row < rows) v.x = p[0];
    if (row + 1 < rows) v.y = p[1];
    if (row + 2 < rows) v.z = p[2];
    if (row + 3 < rows) v.w = p[3];
    const int o = ones_row - row;
    if (o >= 0 && o < 4) (&v.x)[o] = 1.f;
  }
  return v;
}

__device__ __forceinline__ void store_split(uint8_t *hi, uint8_t *lo, uint32_t off, float4 v) {
  float x[4] = {nan0(v.x), nan0(v.y), nan0(v.z), nan0(v.w)};
  float4 h = make_float4(tf32_hi(x[0]), tf32_hi(x[1]), tf32_hi(x[2]), tf32_hi(x[3]));
  float4 l = make_float4(x[0] - h.x, x[1] - h.y, x[2] - h.z, x[3] - h.w);
  *reinterpret_cast<float4 *>(hi + off) = h;
  *reinterpret_cast<float4 *>(lo + off) = l;
}

// Epilogue functors that store column by column straight from the accumulator rows (no transpose).
template <class T, class = void>
struct ep_col_major : std::false_type {};
template <class T>
struct ep_col_major<T, std::void_t<decltype(T::kColMajor)>> : std::integral_constant<bool, T::kColMajor> {};

// Epilogue functors whose output is a plain [z][row][column] fp32 tensor (row stride a multiple of 4
// elements, 16-byte aligned base): the epilogue stages each 32 x 32 chunk in shared memory and the
// TMA engine writes it out (kTmaStore), clipping rows and columns past the end.  Such a functor
// provides `transform(f)`, which calls f with the per-element map (accumulator, column constant,
// aux) -> output (activation dispatched once), `zc(z, split)`, the tensor's outer coordinate, and on
// the host `out_map(tm, M, N, nz)`, which encodes the tensor map with a 32 x 32 box and the 128-byte
// swizzle.  A functor with kAux also reads a second tensor element by element (`aux4(m, z, n)`: the
// 4 values at row m, columns n..n+3, e.g. the activation output a derivative is taken at); aux is 0
// for the others.
template <class T, class = void>
struct ep_tma_store : std::false_type {};
template <class T>
struct ep_tma_store<T, std::void_t<decltype(T::kTmaStore)>> : std::integral_constant<bool, T::kTmaStore> {};
// Functors that store single elements (operator()(m, n, z, split, value)) and accept the producers'
// row sums of A as column rowsum_col (kRowSum).
template <class T, class = void>
struct ep_row_sum : std::false_type {};
template <class T>
struct ep_row_sum<T, std::void_t<decltype(T::kRowSum)>> : std::integral_constant<bool, T::kRowSum> {};
template <class T, class = void>
struct ep_has_aux : std::false_type {};
template <class T>
struct ep_has_aux<T, std::void_t<decltype(T::kAux)>> : std::integral_constant<bool, T::kAux> {};

// Epilogue warps of a tcgemm_kernel variant: 8 (two per tensor-memory lane quarter, one per half of
// the tile's columns) when TMA or bulk copies feed the stages; 4 when producer warps load operands
// through registers (their double-buffered loads need the register budget of a 320-thread CTA).
__host__ __device__ constexpr int epi_warps(int a_mode, int b_mode) { return (a_mode == 0 || b_mode == 0) ? 4 : 8; }
// Producer warps: 4 when they load operands through registers; 8 when they only split tiles that TMA
// or bulk copies brought in (more warps, fewer chunks each, a larger share of the issue slots).
__host__ __device__ constexpr int prod_warps(int a_mode, int b_mode) { return (a_mode == 0 || b_mode == 0) ? 4 : 8; }

// Shared memory an epilogue of EPIW warps reserves (TMA-store boxes, or transpose buffers plus the
// column-constant table).
__host__ __device__ constexpr uint32_t epi_bytes(int epiw, bool tma_st) {
  return tma_st ? (uint32_t)epiw * 4096u : (uint32_t)epiw * 32u * 36u * 4u + 2048u * 4u;
}

// Stages of a variant whose A tiles are split into tensor memory: as many as both the shared memory
// (raw A + split B per stage) and the 512 tensor-memory columns (two BN-column accumulators, then
// 2 * BK columns of A hi / lo per stage) hold, at most 6.
__host__ __device__ constexpr int atm_stages(int bn, int bk, int epiw, bool tma_st) {
  const int by_smem = (int)((232448u - 1024u - epi_bytes(epiw, tma_st)) / (uint32_t)(128 * bk * 4 + 2 * bn * bk * 4));
  const int by_tmem = (512 - 2 * bn) / (2 * bk);
  const int s = by_smem < by_tmem ? by_smem : by_tmem;
  return s > 6 ? 6 : s;
}

// A_TM: the A operand's hi / lo halves live in tensor memory (the MMAs read A from there and only B
// from shared memory); a stage's shared memory then holds the raw A tile as TMA wrote it, and B.
template <int BN, int BK, int STAGES, int EPIW = 4, bool TMA_ST = false, bool A_TM = false>
struct Cfg {
  static constexpr int BM = 128;
  static constexpr uint32_t A_BYTES = BM * BK * 4;  // one of hi / lo
  static constexpr uint32_t B_BYTES = BN * BK * 4;
  static constexpr uint32_t B_OFF = (A_TM ? 1 : 2) * A_BYTES;  // B hi, then B lo, within a stage
  static constexpr uint32_t STAGE_BYTES = B_OFF + 2 * B_BYTES;
  static constexpr uint32_t EPI_OFF = STAGES * STAGE_BYTES;
  // per epilogue warp: one 32 x 36 transpose buffer, or one 4 KB TMA-store box (1024-byte aligned)
  static constexpr uint32_t EPI_BYTES = TMA_ST ? EPIW * 4096 : EPIW * 32 * 36 * 4;
  static constexpr uint32_t COL_OFF = EPI_OFF + EPI_BYTES;  // column constants of the whole product
  // (none with TMA stores: their shared memory goes to one more stage, and the constants come
  // through L1, where every lane of a warp reads the same address)
  static constexpr int COL_FLOATS = TMA_ST ? 0 : 2048;
  static constexpr uint32_t SMEM = COL_OFF + COL_FLOATS * 4 + 1024;  // + alignment slack
  static constexpr int A_CHUNKS = BM * BK / 4 / 128;            // float4 chunks per producer thread per stage
  static constexpr int B_CHUNKS = BN * BK / 4 / 128;
  // two accumulators (epilogue of one tile || MMAs of the next), then with A_TM the A stages
  static constexpr uint32_t A_COL0 = 2 * BN;
  static constexpr uint32_t TMEM_COLS = A_TM ? 512u : 2 * BN;
  static_assert(BK == 32, "a stage row of a K-major tile is one 128-byte swizzle row");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "tile");
  static_assert(A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "swizzle atoms must stay 1024-byte aligned");
  static_assert((BM * BK / 4) % 128 == 0 && (BN * BK / 4) % 128 == 0, "chunks per thread");
  static_assert((TMEM_COLS & (TMEM_COLS - 1)) == 0 && TMEM_COLS >= 32 && TMEM_COLS <= 512, "tensor-memory columns");
  static_assert(SMEM <= 232448, "shared memory per CTA");
  static_assert(!A_TM || A_COL0 + 2 * BK * STAGES <= TMEM_COLS, "A stages in tensor memory");
  // a CTA that holds all 512 columns must be alone on its SM (no second allocation can wait on it)
  static_assert(!A_TM || SMEM > 232448 / 2, "one CTA per SM");
  static_assert(!TMA_ST || EPI_OFF % 1024 == 0, "TMA-store boxes use the 128-byte swizzle");
};

// Where an operand's stage tiles come from.
//   OP_REGS   producer warps load fp32 into registers, split, and store hi and lo.
//   OP_PACKED (B only) a pre-split image in global memory, one bulk copy per stage.
//   OP_TMA    the loader warp copies the raw fp32 tile with TMA straight into the hi slot; the
//             producer warps then sanitise it in place and write lo = x - trunc(x).  The tensor cores
//             read a TF32 operand by truncating the fp32 bit pattern (measured on this part), so the
//             raw tile is the hi half as it stands.
enum OpMode : int { OP_REGS = 0, OP_PACKED = 1, OP_TMA = 2 };

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// 3-d tiled TMA load of box (c0, c1, c2) into shared memory, counted on `bar` (no multicast).
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *tm, int c0, int c1, int c2, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// Sanitised value -> (hi = the full fp32 value, lo = value - trunc(value)): for tiles whose hi half
// is also read as fp32 by the CUDA cores (the tensor cores truncate it themselves).
__device__ __forceinline__ void store_split_full(uint8_t *hi, uint8_t *lo, uint32_t off, float4 v) {
  v = make_float4(nan0(v.x), nan0(v.y), nan0(v.z), nan0(v.w));
  *reinterpret_cast<float4 *>(hi + off) = v;
  *reinterpret_cast<float4 *>(lo + off) =
      make_float4(v.x - tf32_hi(v.x), v.y - tf32_hi(v.y), v.z - tf32_hi(v.z), v.w - tf32_hi(v.w));
}

// 256-bit global store of 8 consecutive floats (32-byte aligned): a whole 32-byte sector per lane,
// where two 16-byte stores would each write half of one.
__device__ __forceinline__ void st_global_v8(float *p, float a0, float a1, float a2, float a3, float a4, float a5,
                                             float a6, float a7) {
  asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "f"(a0), "f"(a1), "f"(a2),
               "f"(a3), "f"(a4), "f"(a5), "f"(a6), "f"(a7)
               : "memory");
}

// 3-d tiled TMA store of one box from shared memory into the tensor (bulk-group completion).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *tm, const void *src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tm)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
// 4-d tiled TMA store of one box from shared memory into the tensor (bulk-group completion).
__device__ __forceinline__ void tma_store_4d(const CUtensorMap *tm, const void *src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tm)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// at most N committed bulk groups may still be reading their shared-memory source
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// at most N committed bulk groups may still be incomplete
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// NCH chunks first, first + stride, ...: every load is issued before the first store, so the
// shared-memory latencies overlap instead of forming a load -> store chain per chunk.
template <int NCH>
__device__ __forceinline__ void split_chunks(uint8_t *hi, uint8_t *lo, uint32_t first, uint32_t stride) {
  float4 x[NCH];
#pragma unroll
  for (int i = 0; i < NCH; ++i) x[i] = *reinterpret_cast<const float4 *>(hi + first + i * stride);
#pragma unroll
  for (int i = 0; i < NCH; ++i) {
    const uint32_t off = first + i * stride;
    float4 v = x[i];
    if (!(isfinite(v.x) && isfinite(v.y) && isfinite(v.z) && isfinite(v.w))) {
      v = make_float4(nan0(v.x), nan0(v.y), nan0(v.z), nan0(v.w));
      *reinterpret_cast<float4 *>(hi + off) = v;
    }
    *reinterpret_cast<float4 *>(lo + off) =
        make_float4(v.x - tf32_hi(v.x), v.y - tf32_hi(v.y), v.z - tf32_hi(v.z), v.w - tf32_hi(v.w));
  }
}

// Persistent kernel: CTA i processes tiles i, i + gridDim.x, ... (n-tile fastest, so the CTAs in
// flight share their A rows in L2).  320 threads:
//   warps 0-3  epilogue (tensor-memory lanes 32w..32w+31 = tile rows), one accumulator at a time
//   warps 4-7  producers (OP_REGS loads and splits; OP_TMA: A into tensor memory, B split in place), stage ring of STAGES
//   warp 8     tensor-memory owner and MMA issuer, alternating two accumulators
//   warp 9     loader: TMA tiles and packed-image bulk copies
// Epilogue functors give a per-row offset (`row`, computed once per tile by the lane that owns the
// row and broadcast with shuffles), a per-column constant (`col`, e.g. the bias, once per 32-column
// chunk), and store 8 rows of one column at a time (`put_rows`: any per-element inputs are loaded
// for all 8 rows first, and the activation is dispatched once per call, not per element).  When
// every output row starts on a 16-byte boundary (`aligned4`, checked on the host) full 32-column
// chunks go out as float4s instead (`col4` / `put_rows4`: a lane stores 4 columns of 8 rows, a warp
// instruction 4 rows x 128 bytes).
template <int BN, int BK, int STAGES, bool A_MCONTIG, bool B_NCONTIG, int A_MODE, int B_MODE, class EP>
__global__ void __launch_bounds__(32 * (epi_warps(A_MODE, B_MODE) + prod_warps(A_MODE, B_MODE) + 2), 1)
    tcgemm_kernel(FastShape s, EP ep, int *err, int vec_a, int vec_b, int vec_out, int tiles_n, int tiles_m,
                  int total, const uint8_t *bimg, int kstages, const __grid_constant__ CUtensorMap tmA,
                  const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmO) {
  constexpr int EPIW = epi_warps(A_MODE, B_MODE);
  constexpr bool TMA_ST = ep_tma_store<EP>::value && EPIW == 8;
  // roles: warps [0, EPIW) epilogue, then 4 producer warps, the MMA warp and the loader warp
  constexpr int PW = prod_warps(A_MODE, B_MODE), NPT = 32 * PW;
  constexpr int kProd0 = EPIW, kMma = EPIW + PW, kLoad = EPIW + PW + 1;
  static_assert(NPT == 128 || (A_MODE != OP_REGS && B_MODE != OP_REGS), "register loads assume 128 producers");
  // TMA-loaded A tiles are split into tensor memory; only B is read by the MMAs from shared memory
  constexpr bool A_TM = A_MODE == OP_TMA;
  static_assert(!A_TM || PW == 8, "A in tensor memory: two producer warps per lane quarter");
  // with a TMA-loaded B, four producer warps put A into tensor memory and four split B
  constexpr bool A_SPLIT4 = A_TM && B_MODE == OP_TMA;
  using C = Cfg<BN, BK, STAGES, EPIW, TMA_ST, A_TM>;
  constexpr int BM = C::BM;
  constexpr bool A_K = !A_MCONTIG, B_K = !B_NCONTIG;
  static_assert(A_MODE != OP_PACKED, "only the B operand is packed");
  // Descriptor strides (bytes), layout types and the start offset of each 8-wide k step.
  //   K-major TMA tiles: 128-byte swizzle, 16-byte granules (layout 2): 8-row groups 1024 B apart,
  //   a k step moves the start 32 B along the swizzled row.  K-major register / packed tiles: no
  //   swizzle (layout 0).  MN-major tiles in every mode: 128-byte swizzle, 32-byte granules (layout 1).
  constexpr bool A_SW = A_K && A_MODE == OP_TMA, B_SW = B_K && B_MODE == OP_TMA;
  constexpr uint32_t A_LBO = A_K ? (A_SW ? 16u : 128u) : 128u * BK, A_SBO = A_K ? (A_SW ? 1024u : 32u * BK) : 512u;
  constexpr uint32_t B_LBO = B_K ? (B_SW ? 16u : 128u) : 128u * BK, B_SBO = B_K ? (B_SW ? 1024u : 32u * BK) : 512u;
  constexpr uint32_t A_LAY = A_K ? (A_SW ? 2u : 0u) : 1u, B_LAY = B_K ? (B_SW ? 2u : 0u) : 1u;
  constexpr uint32_t A_STEP = A_K ? (A_SW ? 32u : 256u) : 1024u, B_STEP = B_K ? (B_SW ? 32u : 256u) : 1024u;
  // A in tensor memory is K-major: lane m holds row m, one column per k
  constexpr uint32_t IDESC = instr_desc_tf32(BM, BN, A_TM ? false : A_MCONTIG, B_NCONTIG);
  constexpr bool ANY_TMA = A_MODE == OP_TMA || B_MODE == OP_TMA;
  constexpr bool LOADER = ANY_TMA || B_MODE == OP_PACKED;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // swizzle atoms are located by absolute address bits: start the stages on a 1024-byte boundary
  uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], tmaf[STAGES], accf[2], acce[2], drain;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const int per_z = tiles_m * tiles_n;
  auto decode = [&](int t, int &m0, int &n0, int &z, int &split, int &kbeg, int &kend, int &nk) {
    const int zs = t / per_z, rem = t - zs * per_z;
    m0 = (rem / tiles_n) * BM;
    n0 = (rem % tiles_n) * BN;
    z = zs % s.nz;
    split = zs / s.nz;
    kbeg = split * s.kchunk;
    kend = min(s.K, kbeg + s.kchunk);
    nk = kend > kbeg ? (kend - kbeg + BK - 1) / BK : 0;
  };
  auto fail = [&](int code) {
    abort_flag = 1;
    atomicExch(err, code);
  };

  if (tid == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], NPT);
      mbar_init(&empty[i], 1);
      mbar_init(&tmaf[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&accf[i], 1);
      mbar_init(&acce[i], 32 * EPIW);
    }
    mbar_init(&drain, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kMma) {
    tmem_alloc(&tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const int n_real = s.ones_col >= 0 ? s.ones_col : s.N;
  pdl_wait();
  pdl_trigger();

  if (warp >= kProd0 && warp < kProd0 + PW) {
    // ------------------------------------------------------------ producers
    // OP_REGS operands are loaded one stage ahead: the global loads of the next stage are in
    // flight while the current one is split and stored (two register sets, used alternately).
    const int ptid = tid - 32 * kProd0;
    struct PState {
      int t, kk, nk, kbeg, kend, Ma, Nb, ones, m0, n0, z, split;
      const float *Ab, *Bb;
    };
    auto start_tile = [&](PState &p) -> bool {
      for (; p.t < total; p.t += gridDim.x) {
        int m0, n0, z, split;
        decode(p.t, m0, n0, z, split, p.kbeg, p.kend, p.nk);
        if (p.nk == 0) continue;  // nothing to load; the MMA warp signals the empty accumulator
        const float *A = s.A + (size_t)z * s.strideA;
        const float *B = s.B + (size_t)z * s.strideB;
        p.Ab = A + (A_K ? (size_t)m0 * s.lda : (size_t)m0);
        p.Bb = B + (B_K ? (size_t)n0 * s.ldb : (size_t)n0);
        p.Ma = s.M - m0;
        p.Nb = n_real - n0;
        p.ones = s.ones_col >= 0 ? s.ones_col - n0 : -1;
        p.m0 = m0;
        p.n0 = n0;
        p.z = z;
        p.split = split;
        p.kk = 0;
        return true;
      }
      return false;
    };
    auto advance = [&](PState &p) -> bool {
      if (++p.kk < p.nk) return true;
      p.t += gridDim.x;
      return start_tile(p);
    };
    auto load = [&](const PState &p, float4 (&va)[C::A_CHUNKS], float4 (&vb)[C::B_CHUNKS]) {
      const int k0 = p.kbeg + p.kk * BK;
      if (A_MODE == OP_REGS) {
#pragma unroll
        for (int i = 0; i < C::A_CHUNKS; ++i) {
          int row, k;
          chunk_place<A_K, BM, BK>(ptid + 128 * i, row, k);
          va[i] = load_chunk<A_K>(p.Ab, s.lda, row, k0 + k, p.Ma, p.kend, vec_a != 0);
        }
      }
      if (B_MODE == OP_REGS) {
#pragma unroll
        for (int i = 0; i < C::B_CHUNKS; ++i) {
          int row, k;
          chunk_place<B_K, BN, BK>(ptid + 128 * i, row, k);
          vb[i] = load_chunk<B_K>(p.Bb, s.ldb, row, k0 + k, p.Nb, p.kend, vec_b != 0, p.ones);
        }
      }
    };
    int it = 0;
    float rsum = 0.f;  // A_SPLIT4: this thread's row sum of A over the current tile's k range
    auto put = [&](const PState &p, const float4 (&va)[C::A_CHUNKS], const float4 (&vb)[C::B_CHUNKS]) -> bool {
      const int st = it % STAGES;
      if (it >= STAGES && !mbar_wait(&empty[st], ((it / STAGES) - 1) & 1, &abort_flag)) {
        fail(kErrEmptyWait);
        return false;
      }
      if (LOADER && !mbar_wait(&tmaf[st], (it / STAGES) & 1, &abort_flag)) {
        fail(kErrFullWait);
        return false;
      }
      uint8_t *base = smem + st * C::STAGE_BYTES;
      uint8_t *b_hi = base + C::B_OFF, *b_lo = b_hi + C::B_BYTES;
      int row, k;
      if (A_MODE == OP_REGS) {
#pragma unroll
        for (int i = 0; i < C::A_CHUNKS; ++i)
          store_split(base, base + C::A_BYTES, chunk_place<A_K, BM, BK>(ptid + 128 * i, row, k), va[i]);
      } else if constexpr (A_TM) {
        // raw A tile -> registers -> nan0 -> hi / lo -> tensor memory.  Warp w may address lanes
        // 32 (w % 4) .. +31 (A rows 32 (w % 4) + lane).  With a TMA-loaded B the first four producer
        // warps take all 32 k of their rows (in two passes of 16) and the other four split B; with a
        // packed B (nothing to split) the two warps of a lane quarter take the stage's k halves.
        // The MMAs that read this stage's columns last time have completed (the empty barrier above
        // is their commit).
        tc_fence_after();
        const int pw = warp - kProd0, q = warp & 3, m = 32 * q + lane;
        if (!A_SPLIT4 || pw < 4) {
#pragma unroll
          for (int pass = 0; pass < (A_SPLIT4 ? 2 : 1); ++pass) {
            const int half = A_SPLIT4 ? pass : (pw >> 2);
            float v[16];
            if constexpr (A_K) {
              // K-major, 128-byte swizzle: row m at m * 128, its 16-byte granule j at (j ^ (m % 8)) * 16
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float4 x =
                    *reinterpret_cast<const float4 *>(base + m * 128 + ((((4 * half + j) ^ (m & 7))) << 4));
                v[4 * j] = x.x;
                v[4 * j + 1] = x.y;
                v[4 * j + 2] = x.z;
                v[4 * j + 3] = x.w;
              }
            } else {
              // MN-major, 128-byte swizzle with 32-byte granules (the layout of chunk_place<false>): a
              // warp reads one 128-byte k row per load, conflict-free
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int kk = 16 * half + j;
                v[j] = *reinterpret_cast<const float *>(base + q * 128 * BK + (kk >> 2) * 512 + (kk & 3) * 128 +
                                                        ((((lane >> 3) ^ (kk & 3))) << 5) + ((lane >> 2) & 1) * 16 +
                                                        (lane & 3) * 4);
              }
            }
            uint32_t hi[16], lo[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float x = nan0(v[j]);
              if constexpr (A_SPLIT4 && ep_row_sum<EP>::value) rsum += x;  // k ascending within the row
              hi[j] = __float_as_uint(x);  // the tensor cores truncate it to TF32 themselves
              lo[j] = __float_as_uint(x - tf32_hi(x));
            }
            const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + C::A_COL0 + (uint32_t)(st * 2 * BK + 16 * half);
            tmem_st16(ta, hi);
            tmem_st16(ta + BK, lo);
          }
          if constexpr (A_SPLIT4 && ep_row_sum<EP>::value) {
            // the row sums of A over the split's k range: column rowsum_col of the output (written
            // once per (m-tile, split), by the first n-tile's CTA)
            if (p.kk + 1 == p.nk) {
              if (s.rowsum_col >= 0 && p.n0 == 0 && m < p.Ma) ep(p.m0 + m, s.rowsum_col, p.z, p.split, rsum);
              rsum = 0.f;
            }
          }
        }
      } else {
        split_chunks<C::A_BYTES / 16 / NPT>(base, base + C::A_BYTES, 16u * ptid, 16u * NPT);
      }
      if (B_MODE == OP_REGS) {
#pragma unroll
        for (int i = 0; i < C::B_CHUNKS; ++i)
          store_split(b_hi, b_lo, chunk_place<B_K, BN, BK>(ptid + 128 * i, row, k), vb[i]);
      } else if (B_MODE == OP_TMA) {
        // A_SPLIT4: producer warps 4-7 split B; otherwise all of them
        constexpr int BT = A_SPLIT4 ? 128 : NPT;
        const int bt = A_SPLIT4 ? ptid - 128 : ptid;
        if (bt >= 0) {
          split_chunks<C::B_BYTES / 16 / BT>(b_hi, b_lo, 16u * bt, 16u * BT);
          // the all-ones column lies outside the B tensor, so TMA filled it with zeros
          if (p.ones >= 0 && p.ones < BN && bt < BK && p.kbeg + p.kk * BK + bt < p.kend) {
            const int kr = bt, j = p.ones;
            const uint32_t off = B_K ? (uint32_t)(j * 128 + ((((kr >> 2) ^ (j & 7))) << 4) + (kr & 3) * 4)
                                     : (uint32_t)((j >> 5) * 128 * BK + kr * 128 +
                                                  ((((j & 31) >> 3) ^ (kr & 3)) << 5) + (j & 7) * 4);
            *reinterpret_cast<float *>(b_hi + off) = 1.f;
          }
        }
      }
      fence_proxy_async_smem();
      if constexpr (A_TM) {
        tmem_wait_st();
        tc_fence_before();
      }
      mbar_arrive(&full[st]);
      ++it;
      return true;
    };
    float4 va0[C::A_CHUNKS], vb0[C::B_CHUNKS], va1[C::A_CHUNKS], vb1[C::B_CHUNKS];
    PState p;
    p.t = blockIdx.x;
    bool have = start_tile(p);
    if (have) load(p, va0, vb0);
    PState cur;
    while (have && !abort_flag) {
      cur = p;
      have = advance(p);
      if (have) load(p, va1, vb1);
      if (!put(cur, va0, vb0) || !have) break;
      cur = p;
      have = advance(p);
      if (have) load(p, va0, vb0);
      if (!put(cur, va1, vb1)) break;
    }
  } else if (warp == kLoad) {
    // ------------------------------------------------------------ loader
    if (LOADER && lane == 0) {
      int it = 0;
      for (int t = blockIdx.x; t < total && !abort_flag; t += gridDim.x) {
        int m0, n0, z, split, kbeg, kend, nk;
        decode(t, m0, n0, z, split, kbeg, kend, nk);
        bool ok = true;
        for (int kk = 0; kk < nk; ++kk, ++it) {
          const int st = it % STAGES;
          if (it >= STAGES && !mbar_wait(&empty[st], ((it / STAGES) - 1) & 1, &abort_flag)) {
            fail(kErrEmptyWait);
            ok = false;
            break;
          }
          uint8_t *base = smem + st * C::STAGE_BYTES;
          const int k0 = kbeg + kk * BK;
          // every copy of the stage completes on tmaf[st]; the producers wait for it before they
          // split and release the stage to the MMA warp
          mbar_arrive_expect_tx(&tmaf[st], (A_MODE == OP_TMA ? C::A_BYTES : 0u) + (B_MODE == OP_TMA ? C::B_BYTES : 0u) +
                                               (B_MODE == OP_PACKED ? 2 * C::B_BYTES : 0u));
          {
            if (A_MODE == OP_TMA) {
              if (A_K) {
                tma_load_3d(base, &tmA, k0, m0, z, &tmaf[st]);
              } else {
#pragma unroll
                for (int h = 0; h < BM / 32; ++h) tma_load_3d(base + h * 128 * BK, &tmA, m0 + 32 * h, k0, z, &tmaf[st]);
              }
            }
            if (B_MODE == OP_TMA) {
              uint8_t *bdst = base + C::B_OFF;
              if (B_K) {
                tma_load_3d(bdst, &tmB, k0, n0, z, &tmaf[st]);
              } else {
#pragma unroll
                for (int h = 0; h < BN / 32; ++h) tma_load_3d(bdst + h * 128 * BK, &tmB, n0 + 32 * h, k0, z, &tmaf[st]);
              }
            }
          }
          if (B_MODE == OP_PACKED) {
            // the weight tile of this stage, already split and laid out, in one bulk copy
            const size_t img = ((size_t)(n0 / BN) * kstages + (kbeg / BK + kk)) * (2 * C::B_BYTES);
            bulk_copy_g2s(base + C::B_OFF, bimg + img, 2 * C::B_BYTES, &tmaf[st]);
          }
        }
        if (!ok) break;
      }
      // before exiting, wait for every copy still in flight into this CTA's shared memory
      for (int st = 0; st < STAGES && st < it; ++st) {
        const int issued = (it - st - 1) / STAGES + 1;
        if (!mbar_wait_drain(&tmaf[st], (issued - 1) & 1) && !abort_flag) fail(kErrFullWait);
      }
    }
  } else if (warp == kMma) {
    // ------------------------------------------------------------ MMA issue
    int it = 0, tl = 0;
    for (int t = blockIdx.x; t < total && !abort_flag; t += gridDim.x, ++tl) {
      int m0, n0, z, split, kbeg, kend, nk;
      decode(t, m0, n0, z, split, kbeg, kend, nk);
      const int b = tl & 1, u = tl >> 1;
      if (tl >= 2 && !mbar_wait(&acce[b], (u - 1) & 1, &abort_flag)) {
        if (lane == 0) fail(kErrDoneWait);
        break;
      }
      tc_fence_after();
      const uint32_t d = tmem + (uint32_t)(b * BN);
      bool ok = true;
      for (int kk = 0; kk < nk; ++kk, ++it) {
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
          const uint32_t b_hi = base + C::B_OFF, b_lo = b_hi + C::B_BYTES;
          // A_TM: the stage's A hi / lo columns in tensor memory (8 columns per k step)
          const uint32_t ta_hi = tmem + C::A_COL0 + (uint32_t)(st * 2 * BK), ta_lo = ta_hi + BK;
          const int kv = min(BK, kend - (kbeg + kk * BK));
          const int nsub = (kv + 7) / 8;
          for (int sub = 0; sub < nsub; ++sub) {
            const uint64_t bh = smem_desc(b_hi + sub * B_STEP, B_LBO, B_SBO, B_LAY);
            const uint64_t bl = smem_desc(b_lo + sub * B_STEP, B_LBO, B_SBO, B_LAY);
            if constexpr (A_TM) {
              mma_tf32_ta(d, ta_lo + 8 * sub, bh, IDESC, (kk | sub) != 0 ? 1u : 0u);
              mma_tf32_ta(d, ta_hi + 8 * sub, bl, IDESC, 1u);
              mma_tf32_ta(d, ta_hi + 8 * sub, bh, IDESC, 1u);
            } else {
              const uint64_t ah = smem_desc(a_hi + sub * A_STEP, A_LBO, A_SBO, A_LAY);
              const uint64_t al = smem_desc(a_lo + sub * A_STEP, A_LBO, A_SBO, A_LAY);
              mma_tf32(d, al, bh, IDESC, (kk | sub) != 0 ? 1u : 0u);
              mma_tf32(d, ah, bl, IDESC, 1u);
              mma_tf32(d, ah, bh, IDESC, 1u);
            }
          }
          mma_commit(&empty[st]);
        }
        __syncwarp();
      }
      if (!ok) break;
      if (lane == 0) {
        if (nk > 0)
          mma_commit(&accf[b]);
        else
          mbar_arrive(&accf[b]);
      }
      __syncwarp();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    float *buf = reinterpret_cast<float *>(smem + C::EPI_OFF) + warp * 32 * 36;
    // column constants (e.g. the bias of every output) once per CTA into shared memory, so the
    // stores never wait on a global gather; every epilogue thread reaches this barrier exactly
    // once, before any bounded wait
    float *coltab = reinterpret_cast<float *>(smem + C::COL_OFF);
    const bool use_tab = (long long)s.N * s.nz <= C::COL_FLOATS;
    if (use_tab)
      for (int i = tid; i < s.N * s.nz; i += 32 * EPIW) coltab[i] = ep.col(i % s.N, i / s.N);
    asm volatile("bar.sync 2, %0;" ::"r"(32 * EPIW) : "memory");
    const int quarter = warp & 3;  // tensor-memory lane quarter = rows 32*quarter .. +31 of the tile
    const int c_begin = EPIW == 8 ? (warp >> 2) * (BN / 2) : 0, c_end = EPIW == 8 ? c_begin + BN / 2 : BN;
    if constexpr (TMA_ST) {
      // each 32 x 32 chunk: accumulator -> registers -> column constant and activation -> the warp's
      // 4 KB box in shared memory (128-byte swizzle: row r's 16-byte granule g at g ^ (r % 8),
      // conflict-free) -> one TMA store issued by lane 0.  The box is rewritten only after the
      // previous chunk's store has read it.
      uint8_t *box = smem + C::EPI_OFF + warp * 4096;
      ep.transform([&](auto tr) {
        int tl = 0;
        constexpr int NCH = (EPIW == 8 ? BN / 2 : BN) / 32;  // chunks per warp per tile
        for (int t = blockIdx.x; t < total && !abort_flag; t += gridDim.x, ++tl) {
          int m0, n0, z, split, kbeg, kend, nk;
          decode(t, m0, n0, z, split, kbeg, kend, nk);
          const int b = tl & 1, u = tl >> 1;
          // lane j holds the constant of column j of each of the warp's chunks, loaded before the
          // accumulator wait so that the load latency overlaps it
          float colv[NCH];
#pragma unroll
          for (int k = 0; k < NCH; ++k) {
            const int n = n0 + c_begin + 32 * k + lane;
            colv[k] = n < s.N ? ep.col(n, z) : 0.f;
          }
          const int mw = m0 + quarter * 32;
          // the second input of this thread's row for chunk k (zeros without one)
          float y[32];
          auto load_aux = [&](int k) {
#pragma unroll
            for (int j = 0; j < 32; ++j) y[j] = 0.f;
            if constexpr (ep_has_aux<EP>::value) {
              const int nc = n0 + c_begin + 32 * k;
              if (mw + lane < s.M) {
#pragma unroll
                for (int q = 0; q < 8; ++q)
                  if (nc + 4 * q < s.N) {
                    const float4 a4 = ep.aux4(mw + lane, z, nc + 4 * q);
                    y[4 * q] = a4.x;
                    y[4 * q + 1] = a4.y;
                    y[4 * q + 2] = a4.z;
                    y[4 * q + 3] = a4.w;
                  }
              }
            }
          };
          // the first chunk's second input is in flight while the MMAs of the tile finish
          load_aux(0);
          if (!mbar_wait(&accf[b], u & 1, &abort_flag)) {
            fail(kErrDoneWait);
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < NCH; ++k) {
            const int c = c_begin + 32 * k;
            if (n0 + c >= s.N) break;
            const int nc = n0 + c;
            if (k > 0) load_aux(k);  // in flight during the tensor-memory load
            float v[32];
            if (nk > 0) {
              tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * BN + c), v);
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = 0.f;
            }
            if (lane == 0) bulk_wait_read<0>();
            __syncwarp();
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              float cc[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) cc[i] = __shfl_sync(0xffffffffu, colv[k], 4 * q + i);
              *reinterpret_cast<float4 *>(box + lane * 128 + (((q ^ lane) & 7) << 4)) =
                  make_float4(tr(v[4 * q], cc[0], y[4 * q]), tr(v[4 * q + 1], cc[1], y[4 * q + 1]),
                              tr(v[4 * q + 2], cc[2], y[4 * q + 2]), tr(v[4 * q + 3], cc[3], y[4 * q + 3]));
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_3d(&tmO, box, nc, mw, ep.zc(z, split));
              bulk_commit();
            }
          }
          tc_fence_before();
          mbar_arrive(&acce[b]);
        }
      });
      // the boxes must be read, and the stores complete, before the CTA exits
      if (lane == 0) bulk_wait<0>();
      __syncwarp();
    } else {
    int tl = 0;
    for (int t = blockIdx.x; t < total && !abort_flag; t += gridDim.x, ++tl) {
      int m0, n0, z, split, kbeg, kend, nk;
      decode(t, m0, n0, z, split, kbeg, kend, nk);
      const int b = tl & 1, u = tl >> 1;
      if (!mbar_wait(&accf[b], u & 1, &abort_flag)) {
        fail(kErrDoneWait);
        break;
      }
      tc_fence_after();
      const int mw = m0 + quarter * 32;
      const long long my_row = (mw + lane < s.M) ? ep.row(mw + lane, z, split) : 0;
#pragma unroll 1
      for (int c = c_begin; c < c_end && n0 + c < s.N; c += 32) {
        float v[32];
        if (nk > 0) {
          tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(b * BN + c), v);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0.f;
        }
        if constexpr (ep_col_major<EP>::value) {
          // column j of the chunk: the 32 lanes (rows) write consecutive addresses
          if (mw + lane < s.M) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (n0 + c + j < s.N) ep.put_col(my_row, n0 + c + j, v[j]);
          }
          continue;
        }
        // row `lane` of the chunk -> shared row `lane` (36-float stride: conflict-free float4 traffic)
#pragma unroll
        for (int q = 0; q < 8; ++q)
          *reinterpret_cast<float4 *>(&buf[lane * 36 + 4 * q]) =
              make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        __syncwarp();
        const int rows = min(32, s.M - mw);
        if (vec_out && n0 + c + 32 <= s.N) {
          const int cq = lane & 7, rs = lane >> 3;
          const int n = n0 + c + 4 * cq;
          const float *ct = coltab + (size_t)z * s.N + n;
          const float4 cv = use_tab ? make_float4(ct[0], ct[1], ct[2], ct[3]) : ep.col4(n, z);
          long long rb[8];
          float4 vv[8];
          unsigned mask = 0;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int r = rs + 4 * j;
            rb[j] = __shfl_sync(0xffffffffu, my_row, r);
            vv[j] = *reinterpret_cast<const float4 *>(&buf[r * 36 + 4 * cq]);
            mask |= r < rows ? 1u << j : 0u;
          }
          if (mask) ep.put_rows4(rb, n, vv, cv, mask);
        } else {
          const int n = n0 + c + lane;
          const bool col_ok = n < s.N;
          const float cv = !col_ok ? 0.f : use_tab ? coltab[(size_t)z * s.N + n] : ep.col(n, z);
#pragma unroll 1
          for (int r0 = 0; r0 < 32; r0 += 8) {
            long long rb[8];
            float vv[8];
            unsigned mask = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              rb[j] = __shfl_sync(0xffffffffu, my_row, r0 + j);
              vv[j] = buf[(r0 + j) * 36 + lane];
              mask |= (col_ok && r0 + j < rows) ? 1u << j : 0u;
            }
            if (mask) ep.put_rows(rb, n, vv, cv, mask);
          }
        }
        __syncwarp();
      }
      tc_fence_before();
      mbar_arrive(&acce[b]);
    }
    }
  }

  // ------------------------------------------------------------ teardown
  if (warp == kMma) {
    // every MMA this thread issued must be complete before its columns are freed
    if (lane == 0) mma_commit(&drain);
    __syncwarp();
    if (!mbar_wait_drain(&drain, 0) && lane == 0) atomicExch(err, kErrDoneWait);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMma) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// Weight operand image for PACKED_B: for every (n-tile, k-stage) the split hi and lo tiles exactly as
// a stage holds them in shared memory ([hi: BN*BK floats][lo: BN*BK floats]), so that one bulk copy
// fills a stage.  One thread per float4 chunk of the image.
template <int BN, int BK, bool B_K>
__global__ void pack_b_kernel(const float *B, long long ldb, int N, int K, uint8_t *img, int tiles_n,
                              int kstages) {
  constexpr int CH = BN * BK / 4;  // chunks per tile image half
  pdl_trigger();                   // the GEMM that consumes the image may start its prologue
  pdl_wait();                      // the weights are final (the previous kernel may have updated them)
  const long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  if (t >= (long long)tiles_n * kstages * CH) return;
  const int q = (int)(t % CH);
  const long long tile = t / CH;  // nt * kstages + ks
  const int nt = (int)(tile / kstages), ks = (int)(tile % kstages);
  int row, k;
  const uint32_t off = chunk_place<B_K, BN, BK>(q, row, k);
  const int n0 = nt * BN;
  const float *Bb = B + (B_K ? (size_t)n0 * ldb : (size_t)n0);
  const float4 v = load_chunk<B_K>(Bb, ldb, row, ks * BK + k, N - n0, K, false);
  uint8_t *hi = img + (size_t)tile * (2 * BN * BK * 4);
  store_split(hi, hi + BN * BK * 4, off, v);
}

}  // namespace tc

inline int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  }
  return n;
}

// Bytes of the packed weight image tcgemm needs for `s` (0 when the weight operand is not packed:
// split-K slices off the 32-deep stage grid, or an all-ones column).
inline size_t tcgemm_pack_bytes(const FastShape &s) {
  // split-K slices must start on a stage boundary: the loader indexes the image by kbeg / 32 + stage
  if ((s.splits > 1 && (s.kchunk <= 0 || s.kchunk % 32)) || s.ones_col >= 0 || s.rowsum_col >= 0 || s.nz != 1) return 0;
  const bool narrow = s.N <= 64 || (s.N % 128 != 0 && s.N % 128 <= 64);
  const int BN = narrow ? 64 : 128;
  const size_t tiles_n = (s.N + BN - 1) / BN, kstages = (s.K + 31) / 32;
  return tiles_n * kstages * 2 * (size_t)BN * 32 * 4;
}

// Tensor maps for OP_TMA operands (the encoder is the driver's, resolved once through the runtime).
typedef CUresult (*TmapEncodeFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                 const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
inline TmapEncodeFn tmap_encoder() {
  static TmapEncodeFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<TmapEncodeFn>(p);
  }
  return fn;
}

// Whether an operand can be read by TMA: 16-byte aligned base, rows and batch strides multiples of 16
// bytes, and (for split-K) split boundaries on stage boundaries.
inline bool tma_ok(const float *p, long long ld, long long stride_z, int nz, const FastShape &s) {
  if (!tmap_encoder()) return false;
  if (((uintptr_t)p & 15) || ld % 4 || ld <= 0) return false;
  if (nz > 1 && (stride_z % 4 || stride_z <= 0)) return false;
  if (s.splits > 1 && s.kchunk % 32) return false;
  return true;
}

// Fp32 tensor [nz][outer][inner] with row stride ld and batch stride stride_z (elements); box
// 32 x box_outer, 128-byte swizzle with 16-byte (K-major) or 32-byte (MN-major) granules.
inline bool make_tmap(CUtensorMap *tm, const float *p, long long ld, long long stride_z, int inner, int outer, int nz,
                      int box_outer, bool mn_major) {
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)outer, (cuuint64_t)nz};
  cuuint64_t strides[2] = {(cuuint64_t)ld * 4, (cuuint64_t)(nz > 1 ? stride_z : ld * (long long)outer) * 4};
  cuuint32_t box[3] = {32u, (cuuint32_t)box_outer, 1u}, es[3] = {1u, 1u, 1u};
  return tmap_encoder()(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(p), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Whether an output [nz][rows][cols] with row stride ld (elements) can be written by TMA-store
// epilogues: 16-byte aligned base, rows and z strides multiples of 16 bytes, whole float4 column
// groups.
inline bool tma_store_ok(const float *p, long long ld, long long stride_z, int nz, int cols) {
  return tmap_encoder() && ((uintptr_t)p & 15) == 0 && ld % 4 == 0 && ld > 0 && cols % 4 == 0 &&
         (nz <= 1 || (stride_z % 4 == 0 && stride_z > 0));
}

template <int BN, bool A_MCONTIG, bool B_NCONTIG, int A_MODE, int B_MODE, class EP>
inline cudaError_t tcgemm_launch(const FastShape &s, EP ep, cudaStream_t st, int *err, int va, int vb,
                                 uint8_t *img) {
  constexpr int BK = 32;
  constexpr int EPIW = tc::epi_warps(A_MODE, B_MODE);
  constexpr bool TMA_ST = tc::ep_tma_store<EP>::value && EPIW == 8;
  // stages fill what the epilogue buffers leave of the 227 KB
  constexpr bool A_TM = A_MODE == tc::OP_TMA;
  constexpr int STAGES = A_TM     ? tc::atm_stages(BN, BK, EPIW, TMA_ST)
                         : TMA_ST ? (BN == 128 ? 3 : 4)
                         : BN == 128 ? (EPIW == 8 ? 2 : 3)
                                     : (EPIW == 8 ? 3 : 4);
  using C = tc::Cfg<BN, BK, STAGES, EPIW, TMA_ST, A_TM>;
  auto fn = tc::tcgemm_kernel<BN, BK, STAGES, A_MCONTIG, B_NCONTIG, A_MODE, B_MODE, EP>;
  static bool attr = false;  // per instantiation; setting it twice is harmless
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  const int tiles_n = (s.N + BN - 1) / BN, tiles_m = (s.M + 127) / 128;
  const long long total = (long long)tiles_n * tiles_m * s.nz * s.splits;
  if (total <= 0) return cudaSuccess;
  if (total > (1LL << 30)) return cudaErrorInvalidValue;
  const int grid = (int)(total < sm_count() ? total : sm_count());
  const int kstages = (s.K + BK - 1) / BK;
  CUtensorMap tmA, tmB, tmO;
  std::memset(&tmA, 0, sizeof tmA);
  std::memset(&tmB, 0, sizeof tmB);
  std::memset(&tmO, 0, sizeof tmO);
  if constexpr (TMA_ST) {
    if (!ep.out_map(&tmO, s.M, s.N, s.nz * s.splits)) return cudaErrorInvalidValue;
  }
  if (A_MODE == tc::OP_TMA) {
    const bool ok = A_MCONTIG ? make_tmap(&tmA, s.A, s.lda, s.strideA, s.M, s.K, s.nz, 32, true)
                              : make_tmap(&tmA, s.A, s.lda, s.strideA, s.K, s.M, s.nz, 128, false);
    if (!ok) return cudaErrorInvalidValue;
  }
  if (B_MODE == tc::OP_TMA) {
    const int n_real = s.ones_col >= 0 ? s.ones_col : s.N;
    const bool ok = B_NCONTIG ? make_tmap(&tmB, s.B, s.ldb, s.strideB, n_real, s.K, s.nz, 32, true)
                              : make_tmap(&tmB, s.B, s.ldb, s.strideB, s.K, n_real, s.nz, BN, false);
    if (!ok) return cudaErrorInvalidValue;
  }
  if (B_MODE == tc::OP_PACKED) {
    const long long n = (long long)tiles_n * kstages * (BN * BK / 4);
    cudaError_t pe = launch_pdl(tc::pack_b_kernel<BN, BK, !B_NCONTIG>, (unsigned)((n + 255) / 256), 256, 0, st, s.B,
                                s.ldb, s.N, s.K, img, tiles_n, kstages);
    if (pe != cudaSuccess) return pe;
  }
  return launch_pdl(fn, grid, dim3(32 * (EPIW + tc::prod_warps(A_MODE, B_MODE) + 2)), C::SMEM, st, s, ep, err, va,
                    vb, ep.aligned4() ? 1 : 0, tiles_n, tiles_m, (int)total, img, kstages, tmA, tmB, tmO);
}

template <int BN, bool A_MCONTIG, bool B_NCONTIG, class EP>
inline cudaError_t tcgemm_modes(const FastShape &s, EP ep, cudaStream_t st, int *err, int va, int vb, uint8_t *img,
                                bool a_tma, bool b_tma) {
  using namespace tc;
  if (img) {
    if (a_tma) return tcgemm_launch<BN, A_MCONTIG, B_NCONTIG, OP_TMA, OP_PACKED>(s, ep, st, err, va, vb, img);
    return tcgemm_launch<BN, A_MCONTIG, B_NCONTIG, OP_REGS, OP_PACKED>(s, ep, st, err, va, vb, img);
  }
  if (a_tma && b_tma)
    return tcgemm_launch<BN, A_MCONTIG, B_NCONTIG, OP_TMA, OP_TMA>(s, ep, st, err, va, vb, nullptr);
  return tcgemm_launch<BN, A_MCONTIG, B_NCONTIG, OP_REGS, OP_REGS>(s, ep, st, err, va, vb, nullptr);
}

// Tile width by N (64 when that wastes less), split-K as given in `s`.  With `img` (at least
// tcgemm_pack_bytes(s) bytes, 16-byte aligned) the B operand is packed first and streamed into the
// stages by bulk copies; otherwise B is loaded like A.  Operands TMA can address are copied by
// TMA, the others by the producer warps.
template <bool A_MCONTIG, bool B_NCONTIG, class EP>
inline cudaError_t tcgemm(FastShape s, EP ep, cudaStream_t st, int *err, uint8_t *img = nullptr) {
  constexpr int BK = 32;
  if (s.M <= 0 || s.N <= 0 || s.nz <= 0) return cudaSuccess;
  if (s.splits < 1) s.splits = 1;
  if (s.kchunk <= 0) s.kchunk = ((s.K + s.splits - 1) / s.splits + BK - 1) / BK * BK;
  auto aligned = [](const float *p, long long ld) { return ((uintptr_t)p % 16 == 0) && (ld % 4 == 0); };
  const int va = aligned(s.A, s.lda) && (s.strideA % 4 == 0);
  const int vb = aligned(s.B, s.ldb) && (s.strideB % 4 == 0);
  const bool narrow = s.N <= 64 || (s.N % 128 != 0 && s.N % 128 <= 64);
  const bool packed = img != nullptr && tcgemm_pack_bytes(s) > 0 && ((uintptr_t)img & 15) == 0;
  const bool a_tma = tma_ok(s.A, s.lda, s.strideA, s.nz, s);
  const bool b_tma = !packed && tma_ok(s.B, s.ldb, s.strideB, s.nz, s);
  // row sums come from the producers of the TMA path only (callers check tcgemm_row_sum_ok)
  if (s.rowsum_col >= 0 && !(a_tma && b_tma && tensor_gemm_enabled() && s.N % 32 == 0 && s.rowsum_col >= s.N))
    return cudaErrorInvalidValue;
  if (narrow) return tcgemm_modes<64, A_MCONTIG, B_NCONTIG>(s, ep, st, err, va, vb, packed ? img : nullptr, a_tma, b_tma);
  return tcgemm_modes<128, A_MCONTIG, B_NCONTIG>(s, ep, st, err, va, vb, packed ? img : nullptr, a_tma, b_tma);
}

// Whether tcgemm can compute the row sums of A (FastShape::rowsum_col) for this product: both
// operands loaded by TMA and B not packed.
inline bool tcgemm_row_sum_ok(const FastShape &s) {
  return tensor_gemm_enabled() && tma_ok(s.A, s.lda, s.strideA, s.nz, s) && tma_ok(s.B, s.ldb, s.strideB, s.nz, s);
}

// Whether a call site's FP32 GEMM runs on the tensor cores: unless the context was created with
// NN_INIT_SIMT_GEMM or the product is too small for a 128-row tile to pay off.
inline bool tc_path(const FastShape &s) {
  return tensor_gemm_enabled() && s.M >= 64 && (long long)s.M * s.N * s.K >= (1LL << 20);
}

template <bool A_MCONTIG, bool B_NCONTIG, class EP>
inline cudaError_t gemm_f32(FastShape s, EP ep, cudaStream_t st) {
  if (tc_path(s)) return tcgemm<A_MCONTIG, B_NCONTIG>(s, ep, st, device_status());
  return sgemm_fast<A_MCONTIG, B_NCONTIG>(s, ep, st);
}

// Same, for a B operand that every row tile re-reads (a weight matrix): on the tensor-core path B
// is packed once into scratch slot 4 and streamed by bulk copies.
template <bool A_MCONTIG, bool B_NCONTIG, class EP>
inline cudaError_t gemm_f32_wb(Launch &L, FastShape s, EP ep) {
  if (!tc_path(s)) return sgemm_fast<A_MCONTIG, B_NCONTIG>(s, ep, L.stream);
  const size_t bytes = tcgemm_pack_bytes(s);
  uint8_t *img = nullptr;
  if (bytes > 0) {
    img = reinterpret_cast<uint8_t *>(L.scratch(4, (bytes + 3) / 4));
    if (!img) return cudaErrorMemoryAllocation;
    L.counted();  // the pack kernel
  }
  return tcgemm<A_MCONTIG, B_NCONTIG>(s, ep, L.stream, device_status(), img);
}

}  // namespace nn
