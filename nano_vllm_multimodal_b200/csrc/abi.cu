// ABI plumbing: version, per-thread error message, launch status, SM count.
#include <cstdarg>
#include <cstdlib>
#include <cstdio>

#include "nib_common.cuh"

namespace nib {

static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

static thread_local cudaError_t g_launch_error = cudaSuccess;

void note_launch_error(cudaError_t e) {
  if (g_launch_error == cudaSuccess) g_launch_error = e;
}

// Off unless NIB_B200_PDL=1. Measured on B200: a captured 28-layer decode step
// of Qwen3-0.6B shapes gets 4% faster with it, the Qwen3-VL-2B one 2.5% slower;
// and a step whose inputs and outputs cross PCIe on other streams while the
// kernels run (the end-to-end bench) loses the overlap of one copy: 101.7 ->
// 117.6 ms per C5 step.
bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("NIB_B200_PDL");
    return v && (v[0] == '1' || v[0] == 'y' || v[0] == 'Y' || v[0] == 't' || v[0] == 'T');
  }();
  return on;
}

int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (g_launch_error != cudaSuccess) {
    e = g_launch_error;
    g_launch_error = cudaSuccess;
  }
  if (e != cudaSuccess) {
    set_error("%s: kernel launch failed: %s", what, cudaGetErrorString(e));
    return NIB_ERR_CUDA;
  }
  return NIB_OK;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

}  // namespace nib

extern "C" int nib_abi_version(void) { return NIB_ABI_VERSION; }

extern "C" const char* nib_last_error(void) { return nib::g_last_error; }
