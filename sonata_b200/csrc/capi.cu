// Library-level C entry points (version, status strings).
#include "common.cuh"

namespace sn {
namespace {

// One thread initialises an mbarrier that nothing ever arrives on and waits
// for its first phase with the kernels' bounded wait, limited to limit_ns.
// The wait runs out, the thread records SN_ERR_TIMEOUT in this unit's status
// word and the kernel returns: no copy, MMA or TMEM allocation is involved.
__global__ void bounded_wait_probe_kernel(uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    if (!mbar_wait_bounded(&bar, 0, limit_ns)) record_status(SN_ERR_TIMEOUT);
  }
}

}  // namespace

int tu_status_gemv(bool reset, cudaStream_t st, int* out);
int tu_status_bmm(bool reset, cudaStream_t st, int* out);
int tu_status_snake(bool reset, cudaStream_t st, int* out);
}  // namespace sn

extern "C" {

int sn_device_status(int reset, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int (*units[])(bool, cudaStream_t, int*) = {sn::tu_status_gemv, sn::tu_status_bmm, sn::tu_status_snake,
                                              sn::read_tu_status};
  int first = SN_OK;
  for (auto f : units) {
    int v = SN_OK;
    const int rc = f(reset != 0, st, &v);
    if (rc != SN_OK) return rc;
    if (first == SN_OK && v != SN_OK) first = v;
  }
  return first;
}

int sn_diag_bounded_wait(uint64_t limit_ns, void* stream) {
  if (limit_ns < 1000 || limit_ns > 1000000000ull) return SN_ERR_INVALID_ARGUMENT;
  return sn::launch(sn::bounded_wait_probe_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), false,
                    limit_ns);
}

int sn_version(void) { return 100; }  // 0.1.0

const char* sn_status_string(int status) {
  switch (status) {
    case SN_OK: return "ok";
    case SN_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer or inconsistent shape)";
    case SN_ERR_MISALIGNED: return "pointer or stride not aligned as the kernel requires";
    case SN_ERR_UNSUPPORTED: return "shape outside what the kernels implement";
    case SN_ERR_LAUNCH: return "CUDA kernel launch failed";
    case SN_ERR_DEVICE: return "current device is not an sm_100 (B200) GPU";
    case SN_ERR_TIMEOUT: return "a bounded device-side wait ran out";
    case SN_ERR_SCRATCH_LIMIT:
      return "problem needs more scratch than the allocation-free entry point's static array holds";
    case SN_ERR_SCRATCH_ADDRESS:
      return "could not look up the device address of the allocation-free entry point's static array "
             "(make the first call on a device outside stream capture)";
    default: return "unknown status";
  }
}

}  // extern "C"
