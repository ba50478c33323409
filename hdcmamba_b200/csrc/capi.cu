// C ABI glue: error state, version queries and the slot-scan dispatcher.
#include <stdarg.h>
#include <stdio.h>

#include <atomic>

#include "common.cuh"

namespace hdc {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

static std::atomic<long long> g_launches{0};

int launch_status(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return (int)e;
  }
  return 0;
}

static int (*g_err_readers[16])(int) = {nullptr};
static int g_n_err_readers = 0;

void register_dev_error_reader(int (*reader)(int reset)) {
  if (g_n_err_readers < 16) g_err_readers[g_n_err_readers++] = reader;
}

}  // namespace hdc

extern "C" int hdc_device_error(int reset) {
  int first = 0;
  for (int i = 0; i < hdc::g_n_err_readers; ++i) {
    const int v = hdc::g_err_readers[i](reset);
    if (v != 0 && first == 0) first = v;
  }
  return first;
}

extern "C" int hdc_version(void) { return 100; }

extern "C" int hdc_built_arch(void) {
#if defined(HDC_BUILT_ARCH)
  return HDC_BUILT_ARCH;
#else
  return 0;
#endif
}

extern "C" const char* hdc_error_string(void) { return hdc::g_err; }

extern "C" long long hdc_launch_count(void) { return hdc::g_launches.load(std::memory_order_relaxed); }
