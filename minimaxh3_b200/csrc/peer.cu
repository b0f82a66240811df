// Exchange buffers shared between the processes of one node through CUDA IPC.
//
// A head-parallel (Ulysses) step moves every rank's quantised sequence shard
// to the rank that owns its heads and the attention output back.  With these
// entry points each rank allocates its send buffers once, exports them, maps
// its peers' buffers into its own device context, and pulls the chunks
// addressed to it with copy-engine copies (mh3_copy_rows on a peer pointer):
// no SM time, so a pull can run while the attention kernel holds every SM,
// and the output lands directly in its strided place.  Plain peer mappings
// only (no multicast objects).

#include <cuda_runtime.h>

#include <cstring>

#include "mh3_internal.h"

static_assert(sizeof(cudaIpcMemHandle_t) == MH3_PEER_HANDLE_BYTES, "IPC handle size");

extern "C" int mh3_peer_alloc(int64_t bytes, void** ptr) {
  if (ptr == nullptr || bytes <= 0) return mh3::fail(MH3_ERR_INVALID, "mh3_peer_alloc: bad size or null ptr");
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, (size_t)bytes);
  return e == cudaSuccess ? MH3_OK : mh3::fail_cuda(e, "mh3_peer_alloc");
}

extern "C" int mh3_peer_free(void* ptr) {
  if (ptr == nullptr) return MH3_OK;
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? MH3_OK : mh3::fail_cuda(e, "mh3_peer_free");
}

extern "C" int mh3_peer_handle(const void* ptr, void* handle) {
  if (ptr == nullptr || handle == nullptr) return mh3::fail(MH3_ERR_INVALID, "mh3_peer_handle: null pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) return mh3::fail_cuda(e, "mh3_peer_handle");
  std::memcpy(handle, &h, sizeof(h));
  return MH3_OK;
}

extern "C" int mh3_peer_open(const void* handle, void** ptr) {
  if (ptr == nullptr || handle == nullptr) return mh3::fail(MH3_ERR_INVALID, "mh3_peer_open: null pointer");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? MH3_OK : mh3::fail_cuda(e, "mh3_peer_open");
}

extern "C" int mh3_peer_close(void* ptr) {
  if (ptr == nullptr) return MH3_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? MH3_OK : mh3::fail_cuda(e, "mh3_peer_close");
}
