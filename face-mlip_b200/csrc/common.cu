// Error reporting and device queries for libfacek.so.
#include "common.cuh"

namespace facek {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return FACEK_ELAUNCH;
  }
  return FACEK_OK;
}

static int query_attr(cudaDeviceAttr a) {
  int dev = 0, v = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&v, a, dev);
  return v;
}

int sm_count() {
  static thread_local int cached_dev = -1, cached = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_dev) {
    cached = query_attr(cudaDevAttrMultiProcessorCount);
    cached_dev = dev;
  }
  return cached > 0 ? cached : 148;
}

int max_smem_optin() { return query_attr(cudaDevAttrMaxSharedMemoryPerBlockOptin); }

}  // namespace facek

extern "C" const char* facek_last_error(void) { return facek::g_err; }
extern "C" int facek_version(void) { return 1; }
