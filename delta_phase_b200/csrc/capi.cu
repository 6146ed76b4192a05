// Error state and version of the deltaphase_b200 C ABI.
#include "dp_common.cuh"

namespace dp {

static thread_local std::string g_last_error;

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

const char *dp_status_string(int status) {
  switch (status) {
    case DP_OK: return "ok";
    case DP_ERR_INVALID_ARGUMENT: return "invalid argument";
    case DP_ERR_UNSUPPORTED: return "unsupported shape";
    case DP_ERR_MISALIGNED: return "misaligned pointer or stride";
    case DP_ERR_CUDA: return "CUDA error";
    case DP_ERR_TIMEOUT: return "device-side wait timed out";
    case DP_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}

}  // extern "C"
