// Library-level entry points: version and the per-thread error text.
#include <string>
#include <string.h>

#include "common.cuh"

namespace jb {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

int launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: CUDA error %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
    return JANUS_ERR_CUDA;
  }
  return JANUS_OK;
}

}  // namespace jb

extern "C" int janus_b200_version(void) { return 100; }

extern "C" int janus_b200_last_error(char* buf, size_t len) {
  const std::string& s = jb::g_last_error;
  if (buf && len) {
    size_t n = s.size() < len - 1 ? s.size() : len - 1;
    memcpy(buf, s.data(), n);
    buf[n] = 0;
  }
  return (int)s.size();
}
