// lr_capi.cu -- status reporting for the C ABI.
#include "lr_common.cuh"

namespace lr {
static thread_local int g_last_cuda_error = 0;

int record_cuda_error(cudaError_t e) {
  g_last_cuda_error = static_cast<int>(e);
  return LR_ERR_CUDA;
}
}  // namespace lr

extern "C" int lr_last_cuda_error(void) { return lr::g_last_cuda_error; }

extern "C" int lr_abi_version(void) { return 3; }

extern "C" const char* lr_status_string(int status) {
  switch (status) {
    case LR_OK:
      return "ok";
    case LR_ERR_INVALID_ARGUMENT:
      return "invalid argument (shape, alignment or null pointer)";
    case LR_ERR_UNSUPPORTED:
      return "unsupported configuration";
    case LR_ERR_CUDA: {
      const int e = lr::g_last_cuda_error;
      return e ? cudaGetErrorString(static_cast<cudaError_t>(e)) : "CUDA error";
    }
    case LR_ERR_WORKSPACE:
      return "workspace missing or too small";
    case LR_ERR_NO_DEVICE:
      return "no sm_100 device";
    case LR_ERR_TOO_LARGE:
      return "size exceeds the 1 MiB static scratch of the allocation-free entry point";
    default:
      return "unknown status";
  }
}
