// Internal runtime interfaces of libnn_b200.so (not part of the C ABI).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>
#include <utility>
#include <vector>

namespace nn {

constexpr int kMaxArgs = 16;
constexpr int kScratchSlots = 5;

enum ArgType : uint8_t { ARG_UNSET = 0, ARG_BUF, ARG_INT, ARG_FLOAT };

struct Arg {
  ArgType type = ARG_UNSET;
  int i = 0;    // buffer handle or int value
  float f = 0;  // float value
};

struct KernelDef;

struct KernelInst {
  const KernelDef *def = nullptr;
  Arg args[kMaxArgs];
  int batch = 1;
};

struct NDR {
  int dims = 1;
  size_t g[3] = {1, 1, 1};
  size_t l[3] = {1, 1, 1};
  bool has_local = false;
};

struct Context;

// What a kernel launcher sees: resolved arguments plus validation helpers.
// Launchers return NN_OK or a negative status after calling fail().
struct Launch {
  Context *ctx;
  const KernelInst *k;
  NDR nd;
  cudaStream_t stream;
  int B;  // batch
  // When > 0: a NormalizeWeights of norm_rows rows of norm_dim weights follows this weight update on
  // the same matrix and is done by the update's apply kernel (the runner skips the NormalizeWeights).
  int norm_rows = 0, norm_dim = 0;

  // Device pointer of buffer argument `idx`, checked to hold at least
  // `need` floats.  Returns nullptr (and records the error) otherwise.
  float *buf(int idx, size_t need);
  // Buffer argument that may legitimately be unused (flags disabled).
  float *buf_opt(int idx);
  int i(int idx) const { return k->args[idx].i; }
  float f(int idx) const { return k->args[idx].f; }
  int fail(int status, const std::string &msg);
  // Per-context scratch of at least `floats` floats (slots 0..kScratchSlots-1 independent; slot 4
  // holds the packed weight operand of the tensor-core GEMMs).
  float *scratch(int slot, size_t floats);
  // Persistent side buffer attached to a buffer handle (created or grown on
  // demand, lives until the handle is freed); `fresh` tells whether it was (re)made.
  float *side(int key_handle, size_t floats, bool *fresh = nullptr);
  // Existing side buffer of a handle, or nullptr; `floats` receives its size.
  float *side_existing(int key_handle, size_t *floats);
  // Size in floats of the buffer bound to argument idx (0 if none).
  size_t floats(int idx) const;
  // Buffer handle bound to argument idx.
  int handle(int idx) const { return k->args[idx].i; }
  // Data-parallel deferred-update hooks (see nn_dp_update_begin).
  bool deferred() const;
  // Arena slot for a weight gradient of n floats, or nullptr when not deferring.
  float *grad_slot(size_t n);
  // Queue the apply half of a deferred update.
  void defer(int (*apply)(const Launch &, const float *grad), const float *grad);
  // Count of CUDA launches issued (for the launch counter).
  void counted(int n = 1);
};

typedef int (*LaunchFn)(Launch &);

struct KernelDef {
  const char *name;
  const char *argtypes;  // p = buffer, i = int, f = float, one char per argument
  LaunchFn fn;
  bool param_only;       // touches only parameter buffers (deferrable in DP mode)
};

// Kernel tables of the translation units.
extern const KernelDef kDenseKernels[];
extern const int kNumDenseKernels;
extern const KernelDef kConvKernels[];
extern const int kNumConvKernels;
extern const KernelDef kAttnKernels[];
extern const int kNumAttnKernels;
extern const KernelDef kMiscKernels[];
extern const int kNumMiscKernels;
extern const KernelDef kLstmKernels[];
extern const int kNumLstmKernels;
extern const KernelDef kAttn2Kernels[];
extern const int kNumAttn2Kernels;
extern const KernelDef kSacKernels[];
extern const int kNumSacKernels;
extern const KernelDef kMatKernels[];
extern const int kNumMatKernels;
extern const KernelDef kFqfKernels[];
extern const int kNumFqfKernels;
extern const KernelDef kFlashKernels[];
extern const int kNumFlashKernels;
extern const KernelDef kPatchKernels[];
extern const int kNumPatchKernels;

// Number of data-parallel ranks (1 without a communicator).
int dp_world();

// Records `msg` as the message nn_last_error returns and gives back `status`
// (for entry points that run outside a kernel Launch).
int report_error(int status, const std::string &msg);

// Device word that kernels with bounded waits set when a wait expires (checked by nn_finish).
int *device_status();
// True unless the context was created with NN_INIT_SIMT_GEMM.
bool tensor_gemm_enabled();
// CUDA ordinal of the context (-1 without one).
int context_device();
// True while a data-parallel update region (nn_dp_update_begin .. end) is open.
bool dp_update_open();
// Adds n launches to the context's launch counter (for entry points outside a kernel Launch).
void add_launches(int n);
// Resolves the device address of the fixed scratch array on `device` (which is current), so that
// its module is loaded at nn_init rather than at the first call that uses it.
int fixed_scratch_setup(int device);

const KernelDef *find_kernel(const char *name);

// Pairs of recorded executions that a command list runs as one kernel (the reference issues them back
// to back): SumMatrix then Normalize of its output.
bool sum_normalize_fusable(const KernelInst &sum, const NDR &nsum, const KernelInst &norm, const NDR &nnorm);
// ... and a dense or convolution Adam update then NormalizeWeights of the same weight rows.
bool update_normalize_fusable(const KernelInst &upd, const NDR &nupd, const KernelInst &norm, const NDR &nnorm);
int sum_normalize_launch(Launch &L);

inline unsigned int ceil_div(size_t a, size_t b) { return (unsigned int)((a + b - 1) / b); }

// Launch-config helper: grid of `n` threads with `threads` per block.
inline dim3 grid1d(size_t n, int threads) { return dim3(ceil_div(n, threads)); }

#define NN_CHECK_LAUNCH(L)                                                            \
  do {                                                                                \
    cudaError_t e_ = cudaGetLastError();                                              \
    if (e_ != cudaSuccess) return (L).fail(NN_ERR_CUDA, cudaGetErrorString(e_));      \
    (L).counted();                                                                    \
  } while (0)

// Launch with programmatic stream serialization (the kernel must call pdl_wait before it
// touches global data).
template <class... KArgs, class... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  return e != cudaSuccess ? e : cudaGetLastError();
}

// Launch with programmatic stream serialization from a reference-kernel implementation (a function
// with a Launch `L` that returns an NN_ status): failures return through L.fail, successes count as
// one of the library's launches.  A kernel name with template commas goes in parentheses.
#define NN_LAUNCH_PDL(L, ...)                                                        \
  do {                                                                               \
    cudaError_t e_ = launch_pdl(__VA_ARGS__);                                        \
    if (e_ != cudaSuccess) return (L).fail(NN_ERR_CUDA, cudaGetErrorString(e_));     \
    (L).counted();                                                                   \
  } while (0)


}  // namespace nn
