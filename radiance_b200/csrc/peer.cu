// Peer buffers for the multi-GPU paths, shared between the processes of one box through CUDA IPC.
//
// The fused N-split all-gather (rb_nvfp4_gemm_allgather) stores every output tile into the other
// GPUs' copies of the output over NVLink, so each rank needs pointers to its peers' buffers.  These
// entry points give them without any NVLink multicast object: a buffer is one plain cudaMalloc
// allocation (legacy CUDA IPC requires exactly that), its 64-byte IPC handle travels between the
// processes by whatever channel the caller has (torch.distributed's object collectives here), and
// each peer maps it with cudaIpcOpenMemHandle.  Only ordinary loads and stores ever touch a mapping
// (no TMA multicast, no multimem), so a rank that dies leaves its peers with nothing bound to a
// multicast object.
#include <string.h>

#include "common.cuh"
#include "../../include/radiance_nvfp4.h"

extern "C" {

int rb_peer_alloc(size_t bytes, void** ptr_out) {
  if (ptr_out == nullptr || bytes == 0) {
    rb_host::set_error("peer_alloc: needs bytes > 0 and an output pointer");
    return RB_ERR_ARG;
  }
  *ptr_out = nullptr;
  const cudaError_t e = cudaMalloc(ptr_out, bytes);
  if (e != cudaSuccess) {
    rb_host::set_error("peer_alloc: cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

int rb_peer_free(void* ptr) {
  if (ptr == nullptr) return RB_OK;
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) {
    rb_host::set_error("peer_free: cudaFree failed: %s", cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

int rb_peer_handle(void* ptr, void* handle_out) {
  if (ptr == nullptr || handle_out == nullptr) {
    rb_host::set_error("peer_handle: null argument");
    return RB_ERR_ARG;
  }
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) {
    rb_host::set_error("peer_handle: cudaIpcGetMemHandle failed: %s", cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  static_assert(sizeof(h) == RB_PEER_HANDLE_BYTES, "IPC handle size");
  memcpy(handle_out, &h, sizeof(h));
  return RB_OK;
}

int rb_peer_open(const void* handle, void** ptr_out) {
  if (handle == nullptr || ptr_out == nullptr) {
    rb_host::set_error("peer_open: null argument");
    return RB_ERR_ARG;
  }
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  *ptr_out = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    rb_host::set_error("peer_open: cudaIpcOpenMemHandle failed: %s", cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

int rb_peer_close(void* ptr) {
  if (ptr == nullptr) return RB_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) {
    rb_host::set_error("peer_close: cudaIpcCloseMemHandle failed: %s", cudaGetErrorString(e));
    return RB_ERR_CUDA;
  }
  return RB_OK;
}

}  // extern "C"
