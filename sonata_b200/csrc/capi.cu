// Library-level C entry points (version, status strings).
#include "common.cuh"

namespace sn {
int tu_status_gemv(bool reset, cudaStream_t st, int* out);
int tu_status_bmm(bool reset, cudaStream_t st, int* out);
int tu_status_snake(bool reset, cudaStream_t st, int* out);
}  // namespace sn

extern "C" {

int sn_device_status(int reset, void* stream) {
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int (*units[])(bool, cudaStream_t, int*) = {sn::tu_status_gemv, sn::tu_status_bmm, sn::tu_status_snake};
  int first = SN_OK;
  for (auto f : units) {
    int v = SN_OK;
    const int rc = f(reset != 0, st, &v);
    if (rc != SN_OK) return rc;
    if (first == SN_OK && v != SN_OK) first = v;
  }
  return first;
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
    default: return "unknown status";
  }
}

}  // extern "C"
