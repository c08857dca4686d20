// Exchange buffers of the tensor-parallel peer sum (the decode kernel's PEER form):
// allocation, CUDA IPC export / import between the ranks' processes, and reset.
//
// Each rank allocates one buffer on its own GPU, exports it with cudaIpcGetMemHandle,
// the ranks exchange the 64-byte handles over the host (torch.distributed), and each
// rank maps every peer's buffer with cudaIpcOpenMemHandle; the device array of the
// world mapped pointers (own buffer at index rank) is what the kernel takes.  Peer
// access over NVLink is enabled lazily by the mapping.
#include <string.h>

#include "common.cuh"
#include "gemm_args.cuh"

extern "C" int64_t tq_peer_buffer_bytes(int world, int slots) {
  if (world < 1 || world > TQ_PEER_MAX_WORLD || slots < 1 || slots > TQ_PEER_MAX_SLOTS) return 0;
  return tq::peer_buffer_bytes(world, slots);
}

extern "C" int tq_peer_alloc(int world, int slots, void** buf) {
  if (!buf) return tq_set_error(TQ_ERR_INVALID, "peer buffer: null result pointer");
  *buf = nullptr;
  const int64_t bytes = tq_peer_buffer_bytes(world, slots);
  if (bytes == 0) return tq_set_error(TQ_ERR_INVALID, "peer buffer: need 1 <= world <= 8 and 1 <= slots <= 65536");
  void* p = nullptr;
  TQ_CUDA_TRY(cudaMalloc(&p, (size_t)bytes));
  if (cudaMemset(p, 0, (size_t)bytes) != cudaSuccess) {
    cudaFree(p);
    return tq_set_error(TQ_ERR_CUDA, "peer buffer: cudaMemset failed");
  }
  TQ_CUDA_TRY(cudaDeviceSynchronize());  // zeroed before any peer can map it
  *buf = p;
  return TQ_OK;
}

extern "C" int tq_peer_free(void* buf) {
  if (!buf) return TQ_OK;
  TQ_CUDA_TRY(cudaFree(buf));
  return TQ_OK;
}

extern "C" int tq_peer_ipc_handle(void* buf, void* handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) == TQ_IPC_HANDLE_BYTES, "IPC handle size");
  if (!buf || !handle) return tq_set_error(TQ_ERR_INVALID, "peer buffer: null buffer or handle");
  cudaIpcMemHandle_t h;
  TQ_CUDA_TRY(cudaIpcGetMemHandle(&h, buf));
  memcpy(handle, &h, sizeof(h));
  return TQ_OK;
}

extern "C" int tq_peer_ipc_open(const void* handle, void** buf) {
  if (!handle || !buf) return tq_set_error(TQ_ERR_INVALID, "peer buffer: null handle or result pointer");
  *buf = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  TQ_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  *buf = p;
  return TQ_OK;
}

extern "C" int tq_peer_ipc_close(void* buf) {
  if (!buf) return TQ_OK;
  TQ_CUDA_TRY(cudaIpcCloseMemHandle(buf));
  return TQ_OK;
}

extern "C" int tq_peer_reset(void* buf, int world, int slots, uint32_t* epochs, void* stream) {
  const int64_t bytes = tq_peer_buffer_bytes(world, slots);
  if (!buf || !epochs || bytes == 0) return tq_set_error(TQ_ERR_INVALID, "peer reset: bad buffer, counters or sizes");
  cudaStream_t st = (cudaStream_t)stream;
  TQ_CUDA_TRY(cudaMemsetAsync(buf, 0, (size_t)bytes, st));
  TQ_CUDA_TRY(cudaMemsetAsync(epochs, 0, (size_t)slots * sizeof(uint32_t), st));
  return TQ_OK;
}
