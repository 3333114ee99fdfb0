// Library-wide status handling: version, per-thread last-error message, launch checks.
#include <cstdarg>
#include <cstdio>

#include "mmp_common.cuh"

static thread_local char g_last_error[512] = "";

int mmp_set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int mmp_check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return mmp_set_error(MMP_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return MMP_OK;
}

static int g_pdl = 1;  // measured: helps the GEMMs (weight prefetch), hurts the short kernels

bool mmp::pdl_enabled(int kind) { return (g_pdl & (kind == 1 ? 1 : 2)) != 0; }

extern "C" int mmp_set_pdl(int enable) {
  const int prev = g_pdl;
  g_pdl = enable & 3;
  return prev;
}

extern "C" int mmp_version(void) { return 100; }

extern "C" const char* mmp_last_error(void) { return g_last_error; }
