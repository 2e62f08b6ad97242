// Status plumbing of the C ABI: per-host-thread last-error message and version.
#include "common.cuh"
#include "tmap.cuh"

#include <atomic>
#include <mutex>
#include <stdarg.h>
#include <stdio.h>

namespace verace {

static thread_local char g_last_error[512] = "no error";
static std::atomic<unsigned long long> g_launches{0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int check_launch(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: kernel launch failed: %s", what, cudaGetErrorString(e));
    return VERACE_ERR_CUDA;
  }
  return VERACE_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

}  // namespace verace

extern "C" int verace_version(void) { return 1 * 10000 + 0 * 100 + 0; }

extern "C" const char* verace_last_error(void) { return verace::g_last_error; }

extern "C" unsigned long long verace_kernel_launches(void) {
  return verace::g_launches.load(std::memory_order_relaxed);
}
