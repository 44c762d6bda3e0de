// Library-wide plumbing of the C ABI: error messages, version, device queries.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "common.cuh"

namespace v1x {

static thread_local char g_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
}

void clear_error() { g_error[0] = '\0'; }

int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return V1X_ERR_CUDA;
  }
  return V1X_OK;
}

int greatest_priority() {
  static int cached[64] = {};
  static bool have[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (!have[dev]) {
    int least = 0, greatest = 0;
    if (cudaDeviceGetStreamPriorityRange(&least, &greatest) != cudaSuccess) greatest = 0;
    cached[dev] = greatest;
    have[dev] = true;
  }
  return cached[dev];
}

int num_sms() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
      sms = v;
  }
  return sms;
}

}  // namespace v1x

extern "C" int v1x_version(void) { return 0x000100; }

extern "C" const char* v1x_last_error(void) { return v1x::g_error; }
