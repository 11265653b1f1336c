// Peer memory for the fused output gather: device buffers that the other
// processes of this node (one per GPU) map with CUDA IPC and write to over
// NVLink.  Set-up calls only; nothing here runs on the decode path.
#include <string.h>

#include "common.cuh"

extern "C" int clover_b200_ipc_alloc(int64_t bytes, void** dev_ptr, void* handle) {
  using namespace clover;
  if (bytes <= 0 || !dev_ptr || !handle)
    return set_error(CLOVER_B200_ERR_INVALID_ARG, "ipc_alloc: bad arguments");
  void* p = nullptr;
  int rc = check_cuda(cudaMalloc(&p, (size_t)bytes), "ipc_alloc cudaMalloc");
  if (rc) return rc;
  rc = check_cuda(cudaMemset(p, 0, (size_t)bytes), "ipc_alloc cudaMemset");
  if (rc) {
    cudaFree(p);
    return rc;
  }
  cudaIpcMemHandle_t h;
  rc = check_cuda(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
  if (rc) {
    cudaFree(p);
    return rc;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == CLOVER_B200_IPC_HANDLE_BYTES, "handle size");
  memcpy(handle, &h, sizeof(h));
  *dev_ptr = p;
  return CLOVER_B200_OK;
}

extern "C" int clover_b200_ipc_open(const void* handle, void** dev_ptr) {
  using namespace clover;
  if (!handle || !dev_ptr) return set_error(CLOVER_B200_ERR_INVALID_ARG, "ipc_open: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return check_cuda(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess),
                    "cudaIpcOpenMemHandle");
}

extern "C" int clover_b200_ipc_close(void* dev_ptr) {
  using namespace clover;
  if (!dev_ptr) return CLOVER_B200_OK;
  return check_cuda(cudaIpcCloseMemHandle(dev_ptr), "cudaIpcCloseMemHandle");
}

extern "C" int clover_b200_ipc_free(void* dev_ptr) {
  using namespace clover;
  if (!dev_ptr) return CLOVER_B200_OK;
  return check_cuda(cudaFree(dev_ptr), "ipc_free cudaFree");
}
