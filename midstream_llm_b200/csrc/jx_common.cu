// Host-side plumbing shared by all entry points: per-thread error text,
// the device status word kernels set when a bounded wait expires, SM count.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>
#include <mutex>

#include "jx_common.cuh"
#include "jx_host.h"

namespace jx {

static thread_local char g_last_error[512] = "";
static std::atomic<long long> g_launches{0};

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

// One status word per device. Kernels that abandon work after a bounded
// wait write a non-zero code here; jx_device_status() reads it back.
static __device__ int g_device_status;

static std::mutex g_mu;
static int g_sms[64];

// Driver calls reached through the runtime's entry-point query (the library does not link libcuda).
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

uint64_t current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  if (!get_current || !get_id) return 0;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  unsigned long long id = 0;
  if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

void* SymbolCache::get(const void* symbol) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  const uint64_t ctx = current_context_id();
  std::lock_guard<std::mutex> lock(mu_);
  Entry& e = entries_[dev];
  if (e.ptr == nullptr || ctx == 0 || e.ctx != ctx) {
    // The lookup also creates the device's context if this thread had none yet; its id is read after.
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, symbol) != cudaSuccess) return nullptr;
    e.ptr = p;
    e.ctx = current_context_id();
  }
  return e.ptr;
}

static SymbolCache g_status_cache;

int* status_ptr() { return static_cast<int*>(g_status_cache.get(reinterpret_cast<const void*>(&g_device_status))); }

int num_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_sms[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sms[dev] = n;
  }
  return g_sms[dev];
}

// SMs a host thread leaves free for other work while its persistent kernels run (jx_set_sm_reserve).
static thread_local int g_sm_reserve = 0;

int persistent_sms() {
  const int n = num_sms() - g_sm_reserve;
  return n < 8 ? 8 : n;
}

}  // namespace jx

extern "C" int jx_set_sm_reserve(int sms) {
  JX_CHECK_ARG(sms >= 0 && sms <= 64, "jx_set_sm_reserve: reserve must be in [0, 64] (got %d)", sms);
  jx::g_sm_reserve = sms;
  return JX_OK;
}

extern "C" int jx_version(void) { return 100; }

extern "C" const char* jx_last_error(void) { return jx::g_last_error; }

extern "C" int64_t jx_launch_count(void) { return jx::g_launches.load(std::memory_order_relaxed); }

extern "C" int jx_device_status(int* status_out, int clear) {
  JX_CHECK_ARG(status_out != nullptr, "jx_device_status: status_out is NULL");
  JX_CUDA_TRY(cudaDeviceSynchronize(), "jx_device_status: synchronize");
  int v = 0;
  JX_CUDA_TRY(cudaMemcpyFromSymbol(&v, jx::g_device_status, sizeof(int)), "jx_device_status: read");
  *status_out = v;
  if (clear) {
    int z = 0;
    JX_CUDA_TRY(cudaMemcpyToSymbol(jx::g_device_status, &z, sizeof(int)), "jx_device_status: clear");
  }
  return JX_OK;
}
