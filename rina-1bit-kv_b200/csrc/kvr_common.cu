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

// ------------------------------------------------------------ self-test ----
// Exercises the bounded-wait failure path of the kernels on the device: an
// mbarrier that expects two arrivals gets one, so its phase never completes;
// the bounded wait (the same helper the bulk-copy waits use) gives up after
// `spin_limit` polls, records the failure in the workspace's error word the
// way the attention kernels do, and the kernel returns.  No copy is in
// flight, nothing faults, the context stays usable; the host then sees
// KVR_ETIMEOUT from kvr_workspace_status.
namespace kvr {
__global__ void bounded_wait_selftest_kernel(unsigned *err, uint32_t spin_limit) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 2);
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&bar)) : "memory");
    if (!mbar_wait_bounded(&bar, 0, spin_limit)) atomicOr(err, 1u);
  }
}
}  // namespace kvr

extern "C" int kvr_selftest_bounded_wait(void *workspace, uint32_t spin_limit, kvr_stream_t stream) {
  kvr::clear_error();
  KVR_REQUIRE(workspace, "kvr_selftest_bounded_wait: null workspace");
  KVR_REQUIRE(spin_limit > 0 && spin_limit <= (1u << 16), "kvr_selftest_bounded_wait: spin_limit in [1, 65536]");
  kvr::bounded_wait_selftest_kernel<<<1, 32, 0, kvr::as_cuda(stream)>>>(reinterpret_cast<unsigned *>(workspace),
                                                                        spin_limit);
  return kvr::check_launch("kvr_selftest_bounded_wait");
}
