// ORACLE TEST INFRASTRUCTURE -- not part of the shipped library.
//
// NDRange executor for the reference kernels compiled by oracle/build_ref.py.
// A launch runs every work-group of the NDRange; work-groups are spread over
// OpenMP threads.  Kernels that use barrier() run their work-items as
// cooperative fibers (ucontext), kernels without barriers run work-items as a
// plain loop.  Exported C entry points (used through ctypes by the tests, the
// golden-vector generator and the CPU baseline of bench.py):
//
//   int  nnref_launch(const char *kernel, int work_dim, const size_t *global,
//                     const size_t *local /* nullable */, void **args);
//   int  nnref_kernel_count(void);
//   const char *nnref_kernel_name(int i);
//   int  nnref_kernel_nargs(int i);
//   const char *nnref_kernel_argtypes(int i);   // one char per arg: p=pointer, i=int, u=uint, f=float
//
// args[i] is the buffer pointer itself for pointer parameters and a pointer to
// the scalar value for scalar parameters.
#include "ref_shim.h"

#include <omp.h>

#include <cstdio>
#include <cstring>

namespace ocl {
thread_local NDRange g_nd;
}

struct RefKernel {
  const char *name;
  void (*call)(void **);
  int uses_barrier;
  int nargs;
  const char *argtypes;
  int serial;  // work-groups in order on one thread (kernels whose groups write the same elements)
};
extern "C" const RefKernel nnref_table[];
extern "C" const int nnref_table_size;

namespace {

constexpr size_t kFiberStack = 64 * 1024;

thread_local void (*t_call)(void **) = nullptr;
thread_local void **t_args = nullptr;
thread_local std::vector<ocl::WorkItem> *t_pool = nullptr;

void fiber_main() {
  ocl::WorkItem *w = ocl::g_nd.cur;
  t_call(t_args);
  w->done = true;
}

void run_group(const RefKernel &k, void **args, const size_t group[3]) {
  using namespace ocl;
  NDRange &nd = g_nd;
  nd.group[0] = group[0];
  nd.group[1] = group[1];
  nd.group[2] = group[2];
  const size_t n = nd.local[0] * nd.local[1] * nd.local[2];
  if (!k.uses_barrier) {
    WorkItem wi;
    nd.cur = &wi;
    nd.fibers = false;
    for (size_t l2 = 0; l2 < nd.local[2]; ++l2)
      for (size_t l1 = 0; l1 < nd.local[1]; ++l1)
        for (size_t l0 = 0; l0 < nd.local[0]; ++l0) {
          wi.lid[0] = l0;
          wi.lid[1] = l1;
          wi.lid[2] = l2;
          for (int d = 0; d < 3; ++d) wi.gid[d] = group[d] * nd.local[d] + wi.lid[d];
          k.call(args);
        }
    return;
  }
  if (!t_pool) t_pool = new std::vector<WorkItem>();
  std::vector<WorkItem> &pool = *t_pool;
  if (pool.size() < n) pool.resize(n);
  nd.fibers = true;
  t_call = k.call;
  t_args = args;
  size_t idx = 0;
  for (size_t l2 = 0; l2 < nd.local[2]; ++l2)
    for (size_t l1 = 0; l1 < nd.local[1]; ++l1)
      for (size_t l0 = 0; l0 < nd.local[0]; ++l0, ++idx) {
        WorkItem &wi = pool[idx];
        wi.lid[0] = l0;
        wi.lid[1] = l1;
        wi.lid[2] = l2;
        for (int d = 0; d < 3; ++d) wi.gid[d] = group[d] * nd.local[d] + wi.lid[d];
        wi.done = false;
        if (wi.stack.size() < kFiberStack) wi.stack.resize(kFiberStack);
        getcontext(&wi.uc);
        wi.uc.uc_stack.ss_sp = wi.stack.data();
        wi.uc.uc_stack.ss_size = wi.stack.size();
        wi.uc.uc_link = &nd.sched;
        makecontext(&wi.uc, fiber_main, 0);
      }
  bool pending = true;
  while (pending) {
    pending = false;
    for (size_t i = 0; i < n; ++i) {
      WorkItem &wi = pool[i];
      if (wi.done) continue;
      nd.cur = &wi;
      swapcontext(&nd.sched, &wi.uc);
      if (!wi.done) pending = true;
    }
  }
}

}  // namespace

extern "C" int nnref_kernel_count(void) { return nnref_table_size; }
extern "C" const char *nnref_kernel_name(int i) {
  return (i >= 0 && i < nnref_table_size) ? nnref_table[i].name : nullptr;
}
extern "C" int nnref_kernel_nargs(int i) {
  return (i >= 0 && i < nnref_table_size) ? nnref_table[i].nargs : -1;
}
extern "C" const char *nnref_kernel_argtypes(int i) {
  return (i >= 0 && i < nnref_table_size) ? nnref_table[i].argtypes : nullptr;
}
extern "C" int nnref_max_threads(void) { return omp_get_max_threads(); }

extern "C" int nnref_launch(const char *name, int work_dim, const size_t *global, const size_t *local,
                            void **args) {
  const RefKernel *k = nullptr;
  for (int i = 0; i < nnref_table_size; ++i)
    if (std::strcmp(nnref_table[i].name, name) == 0) k = &nnref_table[i];
  if (!k) return -1;
  if (work_dim < 1 || work_dim > 3) return -2;
  size_t g[3] = {1, 1, 1}, l[3] = {1, 1, 1}, ng[3];
  for (int d = 0; d < work_dim; ++d) {
    g[d] = global[d];
    l[d] = local ? local[d] : 1;
    if (l[d] == 0 || g[d] % l[d] != 0) return -3;
  }
  size_t total = 1;
  for (int d = 0; d < 3; ++d) {
    ng[d] = g[d] / l[d];
    total *= ng[d];
  }
  if (total == 0) return 0;
#pragma omp parallel for schedule(dynamic, 1) if (!k->serial)
  for (long long gi = 0; gi < (long long)total; ++gi) {
    ocl::NDRange &nd = ocl::g_nd;
    nd.dims = (ocl::uint)work_dim;
    for (int d = 0; d < 3; ++d) {
      nd.global[d] = g[d];
      nd.local[d] = l[d];
    }
    size_t grp[3];
    size_t rem = (size_t)gi;
    grp[0] = rem % ng[0];
    rem /= ng[0];
    grp[1] = rem % ng[1];
    grp[2] = rem / ng[1];
    run_group(*k, args, grp);
  }
  return 0;
}
