// Runtime of libnn_b200.so: the C ABI declared in include/nn_b200.h.
//
// One context per process (the reference drives one OpenCL context from a
// single-threaded MQL5 event loop, NeuroNet_Core.mqh:241-326), one in-order
// CUDA stream, buffers as int handles, kernels by id with persistent
// positional arguments, and nn_execute mapping a NeuroNet.cl kernel name plus
// NDRange onto this library's CUDA launches.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>
#include <unordered_map>
#include <vector>

#include "../../include/nn_b200.h"
#include "nn_internal.h"

namespace nn {

struct Buffer {
  float *ptr = nullptr;
  size_t bytes = 0;
  bool live = false;
};

struct Recorded {
  KernelInst k;
  NDR nd;
};

struct CmdList {
  std::vector<Recorded> ops;
  bool live = false;
};

struct DeferredOp {
  KernelInst k;
  NDR nd;
  int (*apply)(const Launch &, const float *) = nullptr;  // null: plain launch
  const float *grad = nullptr;
  int norm_rows = 0, norm_dim = 0;  // NormalizeWeights done by the apply (see Launch)
};

// ---- NCCL, resolved at nn_dp_init so the library loads without it ----------
typedef struct ncclComm *ncclComm_t;
struct NcclUid { char internal[128]; };
typedef int (*PfnGetUniqueId)(NcclUid *);
typedef int (*PfnCommInitRank)(ncclComm_t *, int, NcclUid, int);
typedef int (*PfnAllReduce)(const void *, void *, size_t, int, int, ncclComm_t, cudaStream_t);
typedef int (*PfnCommDestroy)(ncclComm_t);
typedef const char *(*PfnGetErrorString)(int);
struct Nccl {
  void *lib = nullptr;
  PfnGetUniqueId get_unique_id = nullptr;
  PfnCommInitRank comm_init_rank = nullptr;
  PfnAllReduce all_reduce = nullptr;
  PfnCommDestroy comm_destroy = nullptr;
  PfnGetErrorString error_string = nullptr;
};
constexpr int kNcclFloat32 = 7;  // ncclFloat32
constexpr int kNcclSum = 0;      // ncclSum
constexpr int kNcclAvg = 4;      // ncclAvg (NCCL >= 2.10)

struct Context {
  int device = 0;
  cudaStream_t stream = nullptr;
  std::vector<Buffer> bufs;
  std::vector<int> free_bufs;
  std::unordered_map<int, KernelInst> kernels;
  std::vector<CmdList> lists;
  bool recording = false;
  std::vector<Recorded> rec;
  float *scratch[kScratchSlots] = {};
  size_t scratch_n[kScratchSlots] = {};
  std::unordered_map<int, std::pair<float *, size_t>> sides;  // side buffers keyed by buffer handle
  long long launches = 0;
  // data parallel
  Nccl nccl;
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  bool deferring = false;
  float *arena = nullptr;
  size_t arena_cap = 0, arena_used = 0;
  // gradient buckets: [0, arena_flushed) has been handed to NCCL on comm_stream; a bucket is
  // flushed once kBucketFloats of new gradients have been deferred, while backward goes on
  size_t arena_flushed = 0;
  static constexpr size_t kBucketFloats = size_t(1) << 18;  // 1 MB
  cudaStream_t comm_stream = nullptr;
  cudaEvent_t ev_grads = nullptr, ev_reduced = nullptr;
  int dp_pending = NN_OK;  // first error of a bucket flush inside the open region
  std::string dp_pending_msg;
  std::vector<DeferredOp> deferred;
  // device status word written by kernels whose bounded waits expired (0 = fine)
  int *status = nullptr;
  bool simt_gemm = false;  // NN_INIT_SIMT_GEMM: FP32 SIMT GEMMs instead of 3xTF32 tensor cores
  // overlapped transfers (nn_buffer_write_async / nn_buffer_read_async), created on first use
  cudaStream_t xfer_in = nullptr, xfer_out = nullptr;
  cudaEvent_t ev_in = nullptr, ev_exec = nullptr;
  static constexpr int kReadSlots = 64;
  cudaEvent_t ev_read[kReadSlots] = {};
  long long reads_issued = 0;
};

static Context *g_ctx = nullptr;
static std::string g_err;

static int set_err(int status, const std::string &msg) {
  g_err = msg;
  return status;
}

#define CUDA_TRY(expr)                                                              \
  do {                                                                              \
    cudaError_t e_ = (expr);                                                        \
    if (e_ != cudaSuccess) return set_err(NN_ERR_CUDA, std::string(#expr ": ") + cudaGetErrorString(e_)); \
  } while (0)

// ---------------------------------------------------------------- Launch ----
float *Launch::buf(int idx, size_t need) {
  const Arg &a = k->args[idx];
  if (a.type != ARG_BUF) {
    fail(NN_ERR_ARG, std::string(k->def->name) + ": argument " + std::to_string(idx) + " is not a buffer");
    return nullptr;
  }
  if (a.i < 0 || a.i >= (int)ctx->bufs.size() || !ctx->bufs[a.i].live) {
    fail(NN_ERR_HANDLE, std::string(k->def->name) + ": argument " + std::to_string(idx) + " has no buffer");
    return nullptr;
  }
  const Buffer &b = ctx->bufs[a.i];
  if (need * sizeof(float) > b.bytes) {
    fail(NN_ERR_BOUNDS, std::string(k->def->name) + ": argument " + std::to_string(idx) + " needs " +
                            std::to_string(need) + " floats, buffer holds " + std::to_string(b.bytes / 4));
    return nullptr;
  }
  return b.ptr;
}

float *Launch::buf_opt(int idx) {
  const Arg &a = k->args[idx];
  if (a.type != ARG_BUF || a.i < 0 || a.i >= (int)ctx->bufs.size() || !ctx->bufs[a.i].live) return nullptr;
  return ctx->bufs[a.i].ptr;
}

int Launch::fail(int status, const std::string &msg) { return set_err(status, msg); }

size_t Launch::floats(int idx) const {
  const Arg &a = k->args[idx];
  if (a.type != ARG_BUF || a.i < 0 || a.i >= (int)ctx->bufs.size() || !ctx->bufs[a.i].live) return 0;
  return ctx->bufs[a.i].bytes / sizeof(float);
}

float *Launch::scratch(int slot, size_t floats) {
  if (ctx->scratch_n[slot] < floats) {
    if (ctx->scratch[slot]) {
      cudaStreamSynchronize(ctx->stream);
      cudaFree(ctx->scratch[slot]);
    }
    size_t n = floats + floats / 4 + 1024;
    if (cudaMalloc(&ctx->scratch[slot], n * sizeof(float)) != cudaSuccess) {
      ctx->scratch[slot] = nullptr;
      ctx->scratch_n[slot] = 0;
      fail(NN_ERR_CUDA, "scratch allocation failed");
      return nullptr;
    }
    ctx->scratch_n[slot] = n;
  }
  return ctx->scratch[slot];
}

float *Launch::side(int key, size_t floats, bool *fresh) {
  auto it = ctx->sides.find(key);
  if (it != ctx->sides.end() && it->second.second >= floats) {
    if (fresh) *fresh = false;
    return it->second.first;
  }
  if (it != ctx->sides.end()) {
    cudaStreamSynchronize(ctx->stream);
    cudaFree(it->second.first);
    ctx->sides.erase(it);
  }
  float *p = nullptr;
  if (cudaMalloc(&p, floats * sizeof(float)) != cudaSuccess) {
    fail(NN_ERR_CUDA, "side buffer allocation failed");
    return nullptr;
  }
  cudaMemsetAsync(p, 0, floats * sizeof(float), ctx->stream);
  ctx->sides[key] = {p, floats};
  if (fresh) *fresh = true;
  return p;
}

float *Launch::side_existing(int key, size_t *floats) {
  auto it = ctx->sides.find(key);
  if (it == ctx->sides.end()) return nullptr;
  if (floats) *floats = it->second.second;
  return it->second.first;
}

bool Launch::deferred() const { return ctx->deferring; }

float *Launch::grad_slot(size_t n) {
  if (!ctx->deferring) return nullptr;
  size_t start = (ctx->arena_used + 63) & ~size_t(63);  // 256-byte aligned slots
  if (start + n > ctx->arena_cap) {
    fail(NN_ERR_BOUNDS, "data-parallel gradient arena too small: call nn_dp_update_end and retry");
    return nullptr;
  }
  ctx->arena_used = start + n;
  return ctx->arena + start;
}

static int flush_bucket(Context *c);

void Launch::defer(int (*apply)(const Launch &, const float *), const float *grad) {
  DeferredOp op;
  op.k = *k;
  op.nd = nd;
  op.apply = apply;
  op.grad = grad;
  op.norm_rows = norm_rows;
  op.norm_dim = norm_dim;
  ctx->deferred.push_back(op);
  // every gradient written so far is final for this step: once a bucket's worth has gathered,
  // its allreduce starts on the communication stream while the rest of backward runs
  if (ctx->arena_used - ctx->arena_flushed >= Context::kBucketFloats && ctx->dp_pending == NN_OK) {
    std::string saved = g_err;
    int rc = flush_bucket(ctx);
    if (rc) {
      ctx->dp_pending = rc;
      ctx->dp_pending_msg = g_err;
    }
    g_err = saved;
  }
}

void Launch::counted(int n) { ctx->launches += n; }

const KernelDef *find_kernel(const char *name) {
  struct Table { const KernelDef *t; int n; };
  const Table tables[] = {{kDenseKernels, kNumDenseKernels}, {kConvKernels, kNumConvKernels},
                          {kAttnKernels, kNumAttnKernels}, {kMiscKernels, kNumMiscKernels},
                          {kLstmKernels, kNumLstmKernels}, {kAttn2Kernels, kNumAttn2Kernels},
                          {kSacKernels, kNumSacKernels}, {kMatKernels, kNumMatKernels},
                          {kFqfKernels, kNumFqfKernels},
                          {kFlashKernels, kNumFlashKernels}, {kPatchKernels, kNumPatchKernels}};
  for (const Table &t : tables)
    for (int i = 0; i < t.n; ++i)
      if (std::strcmp(t.t[i].name, name) == 0) return &t.t[i];
  return nullptr;
}

int dp_world() { return g_ctx ? g_ctx->world : 1; }

int report_error(int status, const std::string &msg) { return set_err(status, msg); }

int *device_status() { return g_ctx ? g_ctx->status : nullptr; }

bool tensor_gemm_enabled() { return g_ctx && !g_ctx->simt_gemm && g_ctx->status; }

int context_device() { return g_ctx ? g_ctx->device : -1; }

bool dp_update_open() { return g_ctx && g_ctx->deferring; }

void add_launches(int n) {
  if (g_ctx) g_ctx->launches += n;
}

static int run_one(Context *c, const KernelInst &k, const NDR &nd, int norm_rows = 0, int norm_dim = 0) {
  Launch L;
  L.ctx = c;
  L.k = &k;
  L.nd = nd;
  L.stream = c->stream;
  L.B = k.batch;
  L.norm_rows = norm_rows;
  L.norm_dim = norm_dim;
  for (size_t i = 0; i < std::strlen(k.def->argtypes); ++i) {
    if (k.args[i].type == ARG_UNSET)
      return set_err(NN_ERR_ARG, std::string(k.def->name) + ": argument " + std::to_string(i) + " not set");
  }
  return k.def->fn(L);
}

// run_one with another launcher for the same arguments (a fused pair of recorded executions).
static int run_as(Context *c, const KernelInst &k, const NDR &nd, LaunchFn fn) {
  Launch L;
  L.ctx = c;
  L.k = &k;
  L.nd = nd;
  L.stream = c->stream;
  L.B = k.batch;
  for (size_t i = 0; i < std::strlen(k.def->argtypes); ++i) {
    if (k.args[i].type == ARG_UNSET)
      return set_err(NN_ERR_ARG, std::string(k.def->name) + ": argument " + std::to_string(i) + " not set");
  }
  return fn(L);
}

static int run_deferred(Context *c, const DeferredOp &op) {
  if (!op.apply) return run_one(c, op.k, op.nd);
  Launch L;
  L.ctx = c;
  L.k = &op.k;
  L.nd = op.nd;
  L.stream = c->stream;
  L.B = op.k.batch;
  L.norm_rows = op.norm_rows;
  L.norm_dim = op.norm_dim;
  return op.apply(L, op.grad);
}

// Average arena[arena_flushed, arena_used) over the ranks on the communication stream, after the
// context stream's launches so far (which wrote those gradients).  Every rank defers the same
// updates in the same order, so every rank issues the same sequence of bucket allreduces.
static int flush_bucket(Context *c) {
  const size_t n = c->arena_used - c->arena_flushed;
  if (n == 0) return NN_OK;
  if (c->comm && c->world > 1) {
    CUDA_TRY(cudaEventRecord(c->ev_grads, c->stream));
    CUDA_TRY(cudaStreamWaitEvent(c->comm_stream, c->ev_grads, 0));
    float *p = c->arena + c->arena_flushed;
    int r = c->nccl.all_reduce(p, p, n, kNcclFloat32, kNcclAvg, c->comm, c->comm_stream);
    if (r)
      return set_err(NN_ERR_NCCL, std::string("ncclAllReduce (gradient bucket): ") +
                                      (c->nccl.error_string ? c->nccl.error_string(r) : ""));
  }
  c->arena_flushed = c->arena_used;
  return NN_OK;
}

}  // namespace nn

using namespace nn;

#define NEED_CTX()                                                  \
  do {                                                              \
    if (!g_ctx) return set_err(NN_ERR_STATE, "nn_init not called"); \
  } while (0)

extern "C" {

int nn_init(int device, int flags) {
  if (g_ctx) return set_err(NN_ERR_STATE, "context already initialised");
  if (flags & ~NN_INIT_SIMT_GEMM) return set_err(NN_ERR_ARG, "nn_init: unknown flag bits");
  int n = 0;
  CUDA_TRY(cudaGetDeviceCount(&n));
  if (device < 0 || device >= n) return set_err(NN_ERR_ARG, "no such CUDA device");
  CUDA_TRY(cudaSetDevice(device));
  Context *c = new Context();
  c->device = device;
  cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete c;
    return set_err(NN_ERR_CUDA, cudaGetErrorString(e));
  }
  c->simt_gemm = (flags & NN_INIT_SIMT_GEMM) != 0;
  e = cudaMalloc(&c->status, 256);
  if (e == cudaSuccess) e = cudaMemset(c->status, 0, 256);
  if (e != cudaSuccess) {
    if (c->status) cudaFree(c->status);
    cudaStreamDestroy(c->stream);
    delete c;
    return set_err(NN_ERR_CUDA, cudaGetErrorString(e));
  }
  g_ctx = c;
  // Load the module of the fixed scratch array now: under lazy module loading it would otherwise
  // be loaded (and its array reserved) inside the first nn_update_weights_adam_fixed call, after a
  // host may have handed all free device memory to its own pool.  A failure here is not fatal:
  // that entry point retries the look-up and reports it.
  if (fixed_scratch_setup(device) != NN_OK) {
    cudaGetLastError();
    g_err.clear();
  }
  return NN_OK;
}

int nn_shutdown(void) {
  NEED_CTX();
  Context *c = g_ctx;
  cudaStreamSynchronize(c->stream);
  for (Buffer &b : c->bufs)
    if (b.live) cudaFree(b.ptr);
  for (int i = 0; i < kScratchSlots; ++i)
    if (c->scratch[i]) cudaFree(c->scratch[i]);
  for (auto &kv : c->sides) cudaFree(kv.second.first);
  if (c->arena) cudaFree(c->arena);
  if (c->status) cudaFree(c->status);
  if (c->comm_stream) cudaStreamSynchronize(c->comm_stream);
  if (c->comm && c->nccl.comm_destroy) c->nccl.comm_destroy(c->comm);
  if (c->comm_stream) {
    cudaStreamDestroy(c->comm_stream);
    cudaEventDestroy(c->ev_grads);
    cudaEventDestroy(c->ev_reduced);
  }
  if (c->xfer_in) {
    cudaStreamSynchronize(c->xfer_in);
    cudaStreamSynchronize(c->xfer_out);
    cudaStreamDestroy(c->xfer_in);
    cudaStreamDestroy(c->xfer_out);
    cudaEventDestroy(c->ev_in);
    cudaEventDestroy(c->ev_exec);
    for (cudaEvent_t &e : c->ev_read) cudaEventDestroy(e);
  }
  cudaStreamDestroy(c->stream);
  delete c;
  g_ctx = nullptr;
  return NN_OK;
}

int nn_last_error(char *buf, int len) {
  if (!buf || len <= 0) return NN_ERR_ARG;
  std::snprintf(buf, (size_t)len, "%s", g_err.c_str());
  return NN_OK;
}

int nn_max_local_size(int dim) {
  (void)dim;
  return 1024;
}

// After the stream drained: a kernel whose bounded wait expired left a code in the status word.
static int check_status(Context *c) {
  int code = 0;
  CUDA_TRY(cudaMemcpy(&code, c->status, sizeof(int), cudaMemcpyDeviceToHost));
  if (code == 0) return NN_OK;
  CUDA_TRY(cudaMemset(c->status, 0, sizeof(int)));
  return set_err(NN_ERR_TIMEOUT, "a tensor-core GEMM gave up waiting on its pipeline (code " +
                                     std::to_string(code) + "); its output is incomplete");
}

int nn_finish(int timeout_ms) {
  NEED_CTX();
  if (timeout_ms <= 0) {
    CUDA_TRY(cudaStreamSynchronize(g_ctx->stream));
    return check_status(g_ctx);
  }
  auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaStreamQuery(g_ctx->stream);
    if (e == cudaSuccess) return check_status(g_ctx);
    if (e != cudaErrorNotReady) return set_err(NN_ERR_CUDA, cudaGetErrorString(e));
    auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count();
    if (ms > timeout_ms) return set_err(NN_ERR_TIMEOUT, "nn_finish: stream still busy after timeout");
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

void *nn_stream(void) { return g_ctx ? (void *)g_ctx->stream : nullptr; }

// ---------------------------------------------------------------- buffers
int nn_buffer_create(long long bytes) {
  NEED_CTX();
  if (bytes <= 0) return set_err(NN_ERR_ARG, "buffer size must be positive");
  float *p = nullptr;
  size_t padded = ((size_t)bytes + 255) & ~size_t(255);
  CUDA_TRY(cudaMalloc(&p, padded));
  CUDA_TRY(cudaMemsetAsync(p, 0, padded, g_ctx->stream));
  Context *c = g_ctx;
  int h;
  if (!c->free_bufs.empty()) {
    h = c->free_bufs.back();
    c->free_bufs.pop_back();
  } else {
    h = (int)c->bufs.size();
    c->bufs.push_back(Buffer());
  }
  c->bufs[h].ptr = p;
  c->bufs[h].bytes = (size_t)bytes;
  c->bufs[h].live = true;
  return h;
}

static Buffer *get_buf(int h) {
  if (!g_ctx || h < 0 || h >= (int)g_ctx->bufs.size() || !g_ctx->bufs[h].live) return nullptr;
  return &g_ctx->bufs[h];
}

int nn_buffer_free(int h) {
  NEED_CTX();
  Buffer *b = get_buf(h);
  if (!b) return set_err(NN_ERR_HANDLE, "nn_buffer_free: unknown buffer");
  CUDA_TRY(cudaStreamSynchronize(g_ctx->stream));
  CUDA_TRY(cudaFree(b->ptr));
  *b = Buffer();
  g_ctx->free_bufs.push_back(h);
  auto it = g_ctx->sides.find(h);
  if (it != g_ctx->sides.end()) {
    cudaFree(it->second.first);
    g_ctx->sides.erase(it);
  }
  return NN_OK;
}

static int check_range(Buffer *b, long long offset, long long count, const char *who) {
  if (!b) return set_err(NN_ERR_HANDLE, std::string(who) + ": unknown buffer");
  if (offset < 0 || count < 0 || (size_t)(offset + count) * sizeof(float) > b->bytes)
    return set_err(NN_ERR_BOUNDS, std::string(who) + ": range outside the buffer");
  return NN_OK;
}

int nn_buffer_write(int h, const float *src, long long offset, long long count) {
  NEED_CTX();
  Buffer *b = get_buf(h);
  int rc = check_range(b, offset, count, "nn_buffer_write");
  if (rc) return rc;
  if (count == 0) return NN_OK;
  if (!src) return set_err(NN_ERR_ARG, "nn_buffer_write: null source");
  // src may be pageable: the copy is staged before return.  Pinned sources
  // still go asynchronously through the DMA engine.
  CUDA_TRY(cudaMemcpyAsync(b->ptr + offset, src, (size_t)count * sizeof(float), cudaMemcpyHostToDevice,
                           g_ctx->stream));
  return NN_OK;
}

int nn_buffer_read(int h, float *dst, long long offset, long long count) {
  NEED_CTX();
  Buffer *b = get_buf(h);
  int rc = check_range(b, offset, count, "nn_buffer_read");
  if (rc) return rc;
  if (count == 0) return NN_OK;
  if (!dst) return set_err(NN_ERR_ARG, "nn_buffer_read: null destination");
  CUDA_TRY(cudaMemcpyAsync(dst, b->ptr + offset, (size_t)count * sizeof(float), cudaMemcpyDeviceToHost,
                           g_ctx->stream));
  CUDA_TRY(cudaStreamSynchronize(g_ctx->stream));
  return NN_OK;
}

// COpenCL::BufferWrite / BufferRead with the reference's meaning of their two offsets: the
// device position is a BYTE offset into the buffer (CLBufferWrite's buffer_offset), the host
// position an element index into the caller's array (data_offset).  Floats only, so the byte
// offset must be a multiple of 4.
static int ex_range(long long byte_offset, long long start, long long *elem, const char *who) {
  if (byte_offset < 0 || (byte_offset & 3))
    return set_err(NN_ERR_ARG, std::string(who) + ": buffer byte offset must be a non-negative multiple of 4");
  if (start < 0) return set_err(NN_ERR_ARG, std::string(who) + ": negative array start");
  *elem = byte_offset / 4;
  return NN_OK;
}

int nn_buffer_write_ex(int h, const float *data, long long byte_offset, long long start, long long count) {
  long long elem = 0;
  int rc = ex_range(byte_offset, start, &elem, "nn_buffer_write_ex");
  if (rc) return rc;
  return nn_buffer_write(h, data ? data + start : nullptr, elem, count);
}

int nn_buffer_read_ex(int h, float *data, long long byte_offset, long long start, long long count) {
  long long elem = 0;
  int rc = ex_range(byte_offset, start, &elem, "nn_buffer_read_ex");
  if (rc) return rc;
  return nn_buffer_read(h, data ? data + start : nullptr, elem, count);
}

// Transfer streams and events of the overlapped copies (once per context).
static int transfers_ready(Context *c) {
  if (c->xfer_in) return NN_OK;
  cudaError_t e = cudaStreamCreateWithFlags(&c->xfer_in, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->xfer_out, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_in, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->ev_exec, cudaEventDisableTiming);
  for (int i = 0; i < Context::kReadSlots && e == cudaSuccess; ++i)
    e = cudaEventCreateWithFlags(&c->ev_read[i], cudaEventDisableTiming);
  if (e != cudaSuccess) return set_err(NN_ERR_CUDA, cudaGetErrorString(e));
  return NN_OK;
}

int nn_buffer_write_async(int h, const float *src, long long offset, long long count) {
  NEED_CTX();
  Context *c = g_ctx;
  Buffer *b = get_buf(h);
  int rc = check_range(b, offset, count, "nn_buffer_write_async");
  if (rc) return rc;
  if (count == 0) return NN_OK;
  if (!src) return set_err(NN_ERR_ARG, "nn_buffer_write_async: null source");
  rc = transfers_ready(c);
  if (rc) return rc;
  // on the input transfer stream, concurrent with the executions already enqueued; everything
  // enqueued on the execution stream from now on waits for it
  CUDA_TRY(cudaMemcpyAsync(b->ptr + offset, src, (size_t)count * sizeof(float), cudaMemcpyHostToDevice, c->xfer_in));
  CUDA_TRY(cudaEventRecord(c->ev_in, c->xfer_in));
  CUDA_TRY(cudaStreamWaitEvent(c->stream, c->ev_in, 0));
  return NN_OK;
}

int nn_buffer_read_async(int h, float *dst, long long offset, long long count) {
  NEED_CTX();
  Context *c = g_ctx;
  Buffer *b = get_buf(h);
  int rc = check_range(b, offset, count, "nn_buffer_read_async");
  if (rc) return rc;
  if (!dst && count > 0) return set_err(NN_ERR_ARG, "nn_buffer_read_async: null destination");
  rc = transfers_ready(c);
  if (rc) return rc;
  // the range as every execution enqueued so far leaves it, copied on the output transfer stream
  // while later executions run; a ticket names the read for nn_transfer_wait
  const long long ticket = c->reads_issued;
  cudaEvent_t done = c->ev_read[ticket % Context::kReadSlots];
  CUDA_TRY(cudaEventRecord(c->ev_exec, c->stream));
  CUDA_TRY(cudaStreamWaitEvent(c->xfer_out, c->ev_exec, 0));
  if (count > 0)
    CUDA_TRY(cudaMemcpyAsync(dst, b->ptr + offset, (size_t)count * sizeof(float), cudaMemcpyDeviceToHost,
                             c->xfer_out));
  CUDA_TRY(cudaEventRecord(done, c->xfer_out));
  c->reads_issued++;
  return (int)(ticket % 0x40000000LL);
}

int nn_transfer_wait(int ticket) {
  NEED_CTX();
  Context *c = g_ctx;
  if (ticket < 0) return set_err(NN_ERR_ARG, "nn_transfer_wait: negative ticket");
  // tickets are issued in order; only the last kReadSlots reads can still be waited on
  const long long issued = c->reads_issued;
  long long t = (issued & ~0x3fffffffLL) | ticket;
  if (t >= issued) t -= 0x40000000LL;
  if (t < 0 || t >= issued || issued - t > Context::kReadSlots)
    return set_err(NN_ERR_ARG, "nn_transfer_wait: ticket not among the last 64 reads");
  CUDA_TRY(cudaEventSynchronize(c->ev_read[t % Context::kReadSlots]));
  return NN_OK;
}

__global__ void fill_kernel(float *p, float v, size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) p[i] = v;
}

int nn_buffer_fill(int h, float value, long long offset, long long count) {
  NEED_CTX();
  Buffer *b = get_buf(h);
  int rc = check_range(b, offset, count, "nn_buffer_fill");
  if (rc) return rc;
  if (count == 0) return NN_OK;
  unsigned int blocks = (unsigned int)std::min<long long>((count + 255) / 256, 148 * 16);
  fill_kernel<<<blocks, 256, 0, g_ctx->stream>>>(b->ptr + offset, value, (size_t)count);
  CUDA_TRY(cudaGetLastError());
  g_ctx->launches++;
  return NN_OK;
}

int nn_buffer_copy(int dst, long long dst_offset, int src, long long src_offset, long long count) {
  NEED_CTX();
  Buffer *d = get_buf(dst), *s = get_buf(src);
  int rc = check_range(d, dst_offset, count, "nn_buffer_copy");
  if (rc) return rc;
  rc = check_range(s, src_offset, count, "nn_buffer_copy");
  if (rc) return rc;
  if (count == 0) return NN_OK;
  CUDA_TRY(cudaMemcpyAsync(d->ptr + dst_offset, s->ptr + src_offset, (size_t)count * sizeof(float),
                           cudaMemcpyDeviceToDevice, g_ctx->stream));
  return NN_OK;
}

long long nn_buffer_bytes(int h) {
  NEED_CTX();
  Buffer *b = get_buf(h);
  if (!b) return set_err(NN_ERR_HANDLE, "nn_buffer_bytes: unknown buffer");
  return (long long)b->bytes;
}

void *nn_buffer_device_ptr(int h) {
  Buffer *b = get_buf(h);
  return b ? (void *)b->ptr : nullptr;
}

// ---------------------------------------------------------------- kernels
int nn_kernel_create(int id, const char *name) {
  NEED_CTX();
  if (id < 0 || id > 65535) return set_err(NN_ERR_ARG, "kernel id outside [0, 65535]");
  if (!name) return set_err(NN_ERR_ARG, "null kernel name");
  const KernelDef *d = find_kernel(name);
  if (!d) return set_err(NN_ERR_KERNEL, std::string("kernel not in library: ") + name);
  KernelInst k;
  k.def = d;
  g_ctx->kernels[id] = k;
  return NN_OK;
}

int nn_kernel_create_w(int id, const unsigned short *name_utf16) {
  if (!name_utf16) return set_err(NN_ERR_ARG, "null kernel name");
  char name[128];
  int n = 0;
  for (; name_utf16[n] && n < 127; ++n) {
    if (name_utf16[n] > 127) return set_err(NN_ERR_KERNEL, "kernel names are ASCII");
    name[n] = (char)name_utf16[n];
  }
  name[n] = 0;
  return nn_kernel_create(id, name);
}

int nn_kernel_free(int id) {
  NEED_CTX();
  if (!g_ctx->kernels.erase(id)) return set_err(NN_ERR_HANDLE, "unknown kernel id");
  return NN_OK;
}

static KernelInst *get_kernel(int id) {
  if (!g_ctx) return nullptr;
  auto it = g_ctx->kernels.find(id);
  return it == g_ctx->kernels.end() ? nullptr : &it->second;
}

static int set_arg(int id, int idx, ArgType t, int iv, float fv) {
  NEED_CTX();
  KernelInst *k = get_kernel(id);
  if (!k) return set_err(NN_ERR_HANDLE, "unknown kernel id " + std::to_string(id));
  int nargs = (int)std::strlen(k->def->argtypes);
  if (idx < 0 || idx >= nargs)
    return set_err(NN_ERR_ARG, std::string(k->def->name) + ": argument index out of range");
  char want = k->def->argtypes[idx];
  if ((t == ARG_BUF) != (want == 'p'))
    return set_err(NN_ERR_ARG, std::string(k->def->name) + ": argument " + std::to_string(idx) +
                                   (want == 'p' ? " is a buffer" : " is a scalar"));
  Arg &a = k->args[idx];
  a.type = t;
  if (t == ARG_INT && want == 'f') {  // MQL5 may pass an int for a float parameter
    a.type = ARG_FLOAT;
    a.f = (float)iv;
  } else if (t == ARG_FLOAT && want == 'i') {
    a.type = ARG_INT;
    a.i = (int)fv;
  } else {
    a.i = iv;
    a.f = fv;
  }
  return NN_OK;
}

int nn_set_arg_buffer(int id, int idx, int h) {
  NEED_CTX();
  if (!get_buf(h)) return set_err(NN_ERR_HANDLE, "nn_set_arg_buffer: unknown buffer");
  return set_arg(id, idx, ARG_BUF, h, 0.f);
}
int nn_set_arg_int(int id, int idx, int v) { return set_arg(id, idx, ARG_INT, v, (float)v); }
int nn_set_arg_float(int id, int idx, float v) { return set_arg(id, idx, ARG_FLOAT, (int)v, v); }

int nn_set_batch(int id, int batch) {
  NEED_CTX();
  KernelInst *k = get_kernel(id);
  if (!k) return set_err(NN_ERR_HANDLE, "unknown kernel id");
  if (batch < 1) return set_err(NN_ERR_ARG, "batch must be >= 1");
  k->batch = batch;
  return NN_OK;
}

int nn_execute(int id, int dims, const unsigned int *offset, const unsigned int *global,
               const unsigned int *local) {
  NEED_CTX();
  KernelInst *k = get_kernel(id);
  if (!k) return set_err(NN_ERR_HANDLE, "unknown kernel id " + std::to_string(id));
  if (dims < 1 || dims > 3 || !global) return set_err(NN_ERR_ARG, "nn_execute: bad work dimensions");
  NDR nd;
  nd.dims = dims;
  for (int d = 0; d < dims; ++d) {
    if (offset && offset[d] != 0) return set_err(NN_ERR_UNSUPPORTED, "nn_execute: non-zero global offset");
    nd.g[d] = global[d];
    nd.l[d] = local ? local[d] : 1;
    if (nd.l[d] == 0) return set_err(NN_ERR_ARG, "nn_execute: zero local size");
  }
  nd.has_local = local != nullptr;
  for (int d = 0; d < dims; ++d)
    if (nd.g[d] == 0) return NN_OK;  // empty NDRange: nothing to run
  Context *c = g_ctx;
  if (c->recording) {
    c->rec.push_back(Recorded{*k, nd});
    return NN_OK;
  }
  if (c->deferring && k->def->param_only) {
    DeferredOp op;
    op.k = *k;
    op.nd = nd;
    c->deferred.push_back(op);
    return NN_OK;
  }
  return run_one(c, *k, nd);
}

long long nn_launch_count(void) { return g_ctx ? g_ctx->launches : 0; }

// ----------------------------------------------------------- command lists
int nn_cmdlist_begin(void) {
  NEED_CTX();
  if (g_ctx->recording) return set_err(NN_ERR_STATE, "already recording");
  g_ctx->recording = true;
  g_ctx->rec.clear();
  return NN_OK;
}

int nn_cmdlist_end(void) {
  NEED_CTX();
  if (!g_ctx->recording) return set_err(NN_ERR_STATE, "not recording");
  g_ctx->recording = false;
  CmdList l;
  l.ops.swap(g_ctx->rec);
  l.live = true;
  for (size_t i = 0; i < g_ctx->lists.size(); ++i)
    if (!g_ctx->lists[i].live) {
      g_ctx->lists[i] = std::move(l);
      return (int)i;
    }
  g_ctx->lists.push_back(std::move(l));
  return (int)g_ctx->lists.size() - 1;
}

static CmdList *get_list(int id) {
  if (!g_ctx || id < 0 || id >= (int)g_ctx->lists.size() || !g_ctx->lists[id].live) return nullptr;
  return &g_ctx->lists[id];
}

int nn_cmdlist_run(int id) {
  NEED_CTX();
  CmdList *l = get_list(id);
  if (!l) return set_err(NN_ERR_HANDLE, "unknown command list");
  static const KernelDef *k_sum = find_kernel("SumMatrix"), *k_norm = find_kernel("Normalize");
  static const KernelDef *k_normw = find_kernel("NormalizeWeights");
  for (size_t i = 0; i < l->ops.size(); ++i) {
    Context *c = g_ctx;
    const Recorded &r = l->ops[i];
    int rc;
    if (r.k.def == k_sum && i + 1 < l->ops.size() && l->ops[i + 1].k.def == k_norm &&
        sum_normalize_fusable(r.k, r.nd, l->ops[i + 1].k, l->ops[i + 1].nd)) {
      // SumMatrix + Normalize of its output: one pass over the rows
      rc = run_as(c, r.k, r.nd, sum_normalize_launch);
      if (rc) return set_err(rc, "command list position " + std::to_string(i) + ": " + g_err);
      ++i;
      continue;
    }
    if (i + 1 < l->ops.size() && l->ops[i + 1].k.def == k_normw &&
        update_normalize_fusable(r.k, r.nd, l->ops[i + 1].k, l->ops[i + 1].nd)) {
      // a weight update then NormalizeWeights of its rows: the apply kernel normalises them
      const Recorded &n = l->ops[i + 1];
      rc = run_one(c, r.k, r.nd, (int)n.nd.g[0], n.k.args[1].i);
      if (rc) return set_err(rc, "command list position " + std::to_string(i) + ": " + g_err);
      ++i;
      continue;
    }
    if (c->deferring && r.k.def->param_only) {
      DeferredOp op;
      op.k = r.k;
      op.nd = r.nd;
      c->deferred.push_back(op);
      rc = NN_OK;
    } else {
      rc = run_one(c, r.k, r.nd);
    }
    if (rc) return set_err(rc, "command list position " + std::to_string(i) + ": " + g_err);
  }
  return NN_OK;
}

static int list_set(int id, int pos, int idx, ArgType t, int iv, float fv) {
  NEED_CTX();
  CmdList *l = get_list(id);
  if (!l) return set_err(NN_ERR_HANDLE, "unknown command list");
  if (pos < 0 || pos >= (int)l->ops.size()) return set_err(NN_ERR_ARG, "position outside the list");
  KernelInst &k = l->ops[pos].k;
  int nargs = (int)std::strlen(k.def->argtypes);
  if (idx < 0 || idx >= nargs || k.def->argtypes[idx] == 'p')
    return set_err(NN_ERR_ARG, "not a scalar argument");
  Arg &a = k.args[idx];
  if (k.def->argtypes[idx] == 'f') {
    a.type = ARG_FLOAT;
    a.f = (t == ARG_FLOAT) ? fv : (float)iv;
  } else {
    a.type = ARG_INT;
    a.i = (t == ARG_INT) ? iv : (int)fv;
  }
  return NN_OK;
}

int nn_cmdlist_set_float(int id, int pos, int idx, float v) { return list_set(id, pos, idx, ARG_FLOAT, 0, v); }
int nn_cmdlist_set_int(int id, int pos, int idx, int v) { return list_set(id, pos, idx, ARG_INT, v, 0.f); }

int nn_cmdlist_size(int id) {
  NEED_CTX();
  CmdList *l = get_list(id);
  if (!l) return set_err(NN_ERR_HANDLE, "unknown command list");
  return (int)l->ops.size();
}

int nn_cmdlist_free(int id) {
  NEED_CTX();
  CmdList *l = get_list(id);
  if (!l) return set_err(NN_ERR_HANDLE, "unknown command list");
  l->ops.clear();
  l->live = false;
  return NN_OK;
}

// ------------------------------------------------------------ data parallel
static int load_nccl(Nccl &n) {
  if (n.lib) return NN_OK;
  const char *names[] = {"libnccl.so.2", "libnccl.so"};
  for (const char *nm : names) {
    n.lib = dlopen(nm, RTLD_NOW | RTLD_GLOBAL);
    if (n.lib) break;
  }
  if (!n.lib) return set_err(NN_ERR_NCCL, "libnccl.so.2 not found");
  n.get_unique_id = (PfnGetUniqueId)dlsym(n.lib, "ncclGetUniqueId");
  n.comm_init_rank = (PfnCommInitRank)dlsym(n.lib, "ncclCommInitRank");
  n.all_reduce = (PfnAllReduce)dlsym(n.lib, "ncclAllReduce");
  n.comm_destroy = (PfnCommDestroy)dlsym(n.lib, "ncclCommDestroy");
  n.error_string = (PfnGetErrorString)dlsym(n.lib, "ncclGetErrorString");
  if (!n.get_unique_id || !n.comm_init_rank || !n.all_reduce || !n.comm_destroy)
    return set_err(NN_ERR_NCCL, "libnccl.so.2 lacks required symbols");
  return NN_OK;
}

static int nccl_err(int r, const char *what) {
  const char *s = (g_ctx && g_ctx->nccl.error_string) ? g_ctx->nccl.error_string(r) : "";
  return set_err(NN_ERR_NCCL, std::string(what) + ": " + s);
}

int nn_dp_unique_id(unsigned char *id128) {
  NEED_CTX();
  if (!id128) return set_err(NN_ERR_ARG, "null id buffer");
  int rc = load_nccl(g_ctx->nccl);
  if (rc) return rc;
  NcclUid uid;
  int r = g_ctx->nccl.get_unique_id(&uid);
  if (r) return nccl_err(r, "ncclGetUniqueId");
  std::memcpy(id128, uid.internal, 128);
  return NN_OK;
}

int nn_dp_init(int rank, int world, const unsigned char *id128) {
  NEED_CTX();
  if (world < 1 || rank < 0 || rank >= world || !id128) return set_err(NN_ERR_ARG, "bad rank/world/id");
  if (g_ctx->comm) return set_err(NN_ERR_STATE, "data parallelism already initialised");
  int rc = load_nccl(g_ctx->nccl);
  if (rc) return rc;
  NcclUid uid;
  std::memcpy(uid.internal, id128, 128);
  if (!g_ctx->comm_stream) {
    CUDA_TRY(cudaStreamCreateWithFlags(&g_ctx->comm_stream, cudaStreamNonBlocking));
    CUDA_TRY(cudaEventCreateWithFlags(&g_ctx->ev_grads, cudaEventDisableTiming));
    CUDA_TRY(cudaEventCreateWithFlags(&g_ctx->ev_reduced, cudaEventDisableTiming));
  }
  int r = g_ctx->nccl.comm_init_rank(&g_ctx->comm, world, uid, rank);
  if (r) {
    g_ctx->comm = nullptr;
    return nccl_err(r, "ncclCommInitRank");
  }
  g_ctx->rank = rank;
  g_ctx->world = world;
  return NN_OK;
}

int nn_dp_shutdown(void) {
  NEED_CTX();
  if (!g_ctx->comm) return NN_OK;
  cudaStreamSynchronize(g_ctx->stream);
  if (g_ctx->comm_stream) cudaStreamSynchronize(g_ctx->comm_stream);
  g_ctx->nccl.comm_destroy(g_ctx->comm);
  g_ctx->comm = nullptr;
  g_ctx->world = 1;
  g_ctx->rank = 0;
  return NN_OK;
}

__global__ void scale_kernel(float *p, float s, size_t n) {
  size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  size_t stride = (size_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) p[i] *= s;
}

static int allreduce_ptr(float *p, size_t n, float scale) {
  Context *c = g_ctx;
  if (n == 0) return NN_OK;
  if (c->comm && c->world > 1) {
    int r = c->nccl.all_reduce(p, p, n, kNcclFloat32, kNcclSum, c->comm, c->stream);
    if (r) return nccl_err(r, "ncclAllReduce");
  }
  if (scale != 1.f) {
    unsigned int blocks = (unsigned int)std::min<size_t>((n + 255) / 256, 148 * 8);
    scale_kernel<<<blocks, 256, 0, c->stream>>>(p, scale, n);
    CUDA_TRY(cudaGetLastError());
    c->launches++;
  }
  return NN_OK;
}

int nn_dp_allreduce(int h, long long offset, long long count, float scale) {
  NEED_CTX();
  Buffer *b = get_buf(h);
  int rc = check_range(b, offset, count, "nn_dp_allreduce");
  if (rc) return rc;
  return allreduce_ptr(b->ptr + offset, (size_t)count, scale);
}

int nn_dp_update_begin(void) {
  NEED_CTX();
  Context *c = g_ctx;
  if (c->deferring) return set_err(NN_ERR_STATE, "update region already open");
  if (!c->arena) {
    c->arena_cap = size_t(64) << 20;  // 64 Mi floats (256 MB) of weight gradients per step
    cudaError_t e = cudaMalloc(&c->arena, c->arena_cap * sizeof(float));
    if (e != cudaSuccess) {
      c->arena = nullptr;
      return set_err(NN_ERR_CUDA, cudaGetErrorString(e));
    }
  }
  c->arena_used = 0;
  c->arena_flushed = 0;
  c->dp_pending = NN_OK;
  c->dp_pending_msg.clear();
  c->deferred.clear();
  c->deferring = true;
  return NN_OK;
}

int nn_dp_update_end(void) {
  NEED_CTX();
  Context *c = g_ctx;
  if (!c->deferring) return set_err(NN_ERR_STATE, "no update region open");
  c->deferring = false;
  if (c->dp_pending) {
    c->deferred.clear();
    return set_err(c->dp_pending, c->dp_pending_msg);
  }
  int rc = flush_bucket(c);
  if (rc) return rc;
  if (c->comm && c->world > 1) {
    // the applies read every bucket: the context stream waits for the last allreduce
    CUDA_TRY(cudaEventRecord(c->ev_reduced, c->comm_stream));
    CUDA_TRY(cudaStreamWaitEvent(c->stream, c->ev_reduced, 0));
  }
  for (size_t i = 0; i < c->deferred.size(); ++i) {
    rc = run_deferred(c, c->deferred[i]);
    if (rc) return rc;
  }
  c->deferred.clear();
  return NN_OK;
}

}  // extern "C"
