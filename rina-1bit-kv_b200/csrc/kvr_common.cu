// Error state and version of the kvr_b200 C ABI.
#include "kvr_common.cuh"

namespace kvr {

static thread_local char g_last_error[512] = {0};

int set_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

void clear_error() { g_last_error[0] = 0; }

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(KVR_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return KVR_OK;
}

}  // namespace kvr

extern "C" const char *kvr_last_error(void) { return kvr::g_last_error; }
extern "C" int kvr_abi_version(void) { return (1 << 16) | 0; }
