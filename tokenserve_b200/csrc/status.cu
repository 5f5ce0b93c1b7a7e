// Status and error-message plumbing behind ts_last_error().
#include <cstdarg>
#include <cstdio>
#include <string>

#include "common.cuh"

namespace ts {

namespace {
thread_local std::string g_last_error;
}

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int ok() {
  g_last_error.clear();
  return TS_OK;
}

int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(static_cast<int>(e), "%s: %s", what, cudaGetErrorString(e));
  return ok();
}

}  // namespace ts

extern "C" int ts_version(void) { return TS_ABI_VERSION; }

extern "C" const char* ts_last_error(void) { return ts::g_last_error.c_str(); }
