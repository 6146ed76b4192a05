// Error state and version of the deltaphase_b200 C ABI.
#include "dp_common.cuh"

namespace dp {

static thread_local std::string g_last_error;

// Device-side error word: kernels record DP_ERR_TIMEOUT here when a bounded wait
// expires (one word per device, read and cleared by dp_device_error).
__device__ int g_device_error;

int *device_error_ptr() {
  static int *ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!ptrs[dev]) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int *>(p);
  }
  return ptrs[dev];
}

int set_error(int status, const std::string &msg) {
  g_last_error = msg;
  return status;
}

int check_launch(const char *what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return set_error(DP_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
  }
  return DP_OK;
}

}  // namespace dp

extern "C" {

const char *dp_version(void) { return "deltaphase_b200 0.1.0 (sm_100a)"; }

const char *dp_last_error(void) { return dp::g_last_error.c_str(); }

int dp_device_error(int clear) {
  int v = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  if (cudaMemcpyFromSymbol(&v, dp::g_device_error, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(dp::g_device_error, &zero, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

const char *dp_status_string(int status) {
  switch (status) {
    case DP_OK: return "ok";
    case DP_ERR_INVALID_ARGUMENT: return "invalid argument";
    case DP_ERR_UNSUPPORTED: return "unsupported shape";
    case DP_ERR_MISALIGNED: return "misaligned pointer or stride";
    case DP_ERR_CUDA: return "CUDA error";
    case DP_ERR_TIMEOUT: return "device-side wait timed out";
    case DP_ERR_WORKSPACE: return "workspace too small";
    case DP_ERR_RANGE: return "value outside the range of 16-bit operand tiles";
    default: return "unknown status";
  }
}

}  // extern "C"
