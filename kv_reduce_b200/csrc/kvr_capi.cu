// Status strings, version and per-thread CUDA error text of the C ABI.
#include "kvr_common.cuh"

#include <cstring>

namespace kvr {
static thread_local char g_last_error[256] = {0};

void set_last_cuda_error(cudaError_t e) {
  const char* s = cudaGetErrorString(e);
  std::strncpy(g_last_error, s ? s : "unknown CUDA error", sizeof(g_last_error) - 1);
  g_last_error[sizeof(g_last_error) - 1] = 0;
}
}  // namespace kvr

extern "C" int kvr_version(void) { return 100; }  // 0.1.0

extern "C" const char* kvr_last_error(void) { return kvr::g_last_error; }

extern "C" int kvr_host_mapped(const void* p, int* mapped) {
  if (!mapped) return KVR_ERR_INVALID_ARGUMENT;
  *mapped = 0;
  if (!p) return KVR_OK;
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    (void)cudaGetLastError();   // memory the runtime does not know: not mapped
    return KVR_OK;
  }
  *mapped = (attr.type == cudaMemoryTypeHost && attr.devicePointer == p) ? 1 : 0;
  return KVR_OK;
}

extern "C" const char* kvr_status_string(int status) {
  switch (status) {
    case KVR_OK: return "ok";
    case KVR_ERR_INVALID_ARGUMENT: return "invalid argument";
    case KVR_ERR_UNSUPPORTED: return "unsupported configuration";
    case KVR_ERR_MISALIGNED: return "pointer or stride not 16-byte aligned";
    case KVR_ERR_CUDA: return "CUDA runtime error";
    case KVR_ERR_CAPACITY: return "cache capacity exceeded";
    case KVR_ERR_WORKSPACE: return "workspace too small";
    default: return "unknown status";
  }
}
