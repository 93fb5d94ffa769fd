// Error reporting and version for the C ABI.
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

namespace gdn {

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

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  g_err[0] = 0;
  return GDN_OK;
}

}  // namespace gdn

extern "C" const char* gdn_last_error(void) { return gdn::g_err; }

extern "C" int gdn_version(void) { return 100; }
