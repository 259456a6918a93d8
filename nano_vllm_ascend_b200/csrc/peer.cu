// Peer buffers for the KV-head-sharded decode: device memory that the other
// processes of a node map through CUDA IPC, so that one rank's kernel can
// store into another rank's buffer over NVLink. Plain allocations and plain
// loads/stores only: no multicast object is created.
#include <cstring>

#include "host_common.h"

static_assert(sizeof(cudaIpcMemHandle_t) == NVK_PEER_HANDLE_BYTES, "IPC handle size");

extern "C" int nvk_peer_alloc(size_t bytes, void** ptr) {
  using namespace nvk;
  if (!ptr || bytes == 0) return fail(NVK_ERR_INVALID_ARGUMENT, "peer_alloc: null output or zero size");
  *ptr = nullptr;
  void* p = nullptr;
  int rc = check_cuda(cudaMalloc(&p, bytes), "peer_alloc: cudaMalloc");
  if (rc != NVK_OK) return rc;
  rc = check_cuda(cudaMemset(p, 0, bytes), "peer_alloc: cudaMemset");
  if (rc != NVK_OK) {
    cudaFree(p);
    return rc;
  }
  *ptr = p;
  return NVK_OK;
}

extern "C" int nvk_peer_free(void* ptr) {
  if (!ptr) return NVK_OK;
  return nvk::check_cuda(cudaFree(ptr), "peer_free: cudaFree");
}

extern "C" int nvk_peer_export(const void* ptr, void* handle) {
  using namespace nvk;
  if (!ptr || !handle) return fail(NVK_ERR_INVALID_ARGUMENT, "peer_export: null pointer");
  cudaIpcMemHandle_t h;
  const int rc = check_cuda(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)), "peer_export: cudaIpcGetMemHandle");
  if (rc != NVK_OK) return rc;
  std::memcpy(handle, &h, sizeof(h));
  return NVK_OK;
}

extern "C" int nvk_peer_import(const void* handle, void** ptr) {
  using namespace nvk;
  if (!ptr || !handle) return fail(NVK_ERR_INVALID_ARGUMENT, "peer_import: null pointer");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return check_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "peer_import: cudaIpcOpenMemHandle");
}

extern "C" int nvk_peer_close(void* ptr) {
  if (!ptr) return NVK_OK;
  return nvk::check_cuda(cudaIpcCloseMemHandle(ptr), "peer_close: cudaIpcCloseMemHandle");
}
