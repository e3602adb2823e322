// Exchange buffers for the cross-GPU decode merge: device memory shared between the ranks'
// processes with CUDA IPC, so the decode kernel can store into other GPUs' buffers over NVLink.
#include <cuda_runtime.h>

#include <cstring>
#include <string>

#include "../../include/sunshape_b200.h"

namespace sunshape {
int set_last_error(int code, const char* msg);   // defined in capi.cu
}

namespace {
int cuda_fail(const char* what, cudaError_t e) {
  return sunshape::set_last_error(SUNSHAPE_E_CUDA, (std::string(what) + ": " + cudaGetErrorString(e)).c_str());
}
}  // namespace

extern "C" {

int sunshape_peer_alloc(int64_t bytes, void** dev_ptr, void* ipc_handle) {
  if (bytes <= 0 || !dev_ptr || !ipc_handle) return sunshape::set_last_error(SUNSHAPE_E_INVALID, "bad peer_alloc args.");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e != cudaSuccess) return cuda_fail("cudaMalloc(peer buffer)", e);
  e = cudaMemset(p, 0, (size_t)bytes);
  if (e != cudaSuccess) { cudaFree(p); return cuda_fail("cudaMemset(peer buffer)", e); }
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) { cudaFree(p); return cuda_fail("cudaIpcGetMemHandle", e); }
  static_assert(sizeof(h) == 64, "IPC handle size");
  std::memcpy(ipc_handle, &h, sizeof(h));
  *dev_ptr = p;
  return SUNSHAPE_OK;
}

int sunshape_peer_open(const void* ipc_handle, void** dev_ptr) {
  if (!ipc_handle || !dev_ptr) return sunshape::set_last_error(SUNSHAPE_E_INVALID, "bad peer_open args.");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail("cudaIpcOpenMemHandle", e);
  *dev_ptr = p;
  return SUNSHAPE_OK;
}

int sunshape_peer_close(void* dev_ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  return e == cudaSuccess ? SUNSHAPE_OK : cuda_fail("cudaIpcCloseMemHandle", e);
}

int sunshape_peer_free(void* dev_ptr) {
  const cudaError_t e = cudaFree(dev_ptr);
  return e == cudaSuccess ? SUNSHAPE_OK : cuda_fail("cudaFree(peer buffer)", e);
}

}  // extern "C"
