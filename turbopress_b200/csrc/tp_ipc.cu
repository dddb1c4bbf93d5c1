// Peer memory for tensor-parallel engine programs: plain device allocations
// shared between the processes of one node through CUDA IPC handles.
#include <cstring>

#include "tp_common.cuh"

using namespace tp;

static_assert(sizeof(cudaIpcMemHandle_t) == TP_IPC_HANDLE_BYTES, "IPC handle size");

extern "C" tp_status tp_ipc_alloc(int64_t bytes, void** ptr) {
  if (!ptr || bytes <= 0) return fail(TP_ERR_ARG, "tp_ipc_alloc: bad arguments");
  TP_CUDA_TRY(cudaMalloc(ptr, static_cast<size_t>(bytes)), "cudaMalloc(ipc)");
  TP_CUDA_TRY(cudaMemset(*ptr, 0, static_cast<size_t>(bytes)), "cudaMemset(ipc)");
  return clear_ok();
}

extern "C" tp_status tp_ipc_free(void* ptr) {
  if (!ptr) return clear_ok();
  TP_CUDA_TRY(cudaFree(ptr), "cudaFree(ipc)");
  return clear_ok();
}

extern "C" tp_status tp_ipc_get_handle(void* ptr, void* handle) {
  if (!ptr || !handle) return fail(TP_ERR_ARG, "tp_ipc_get_handle: bad arguments");
  cudaIpcMemHandle_t h;
  TP_CUDA_TRY(cudaIpcGetMemHandle(&h, ptr), "cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof(h));
  return clear_ok();
}

extern "C" tp_status tp_ipc_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return fail(TP_ERR_ARG, "tp_ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  TP_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return clear_ok();
}

extern "C" tp_status tp_ipc_close(void* ptr) {
  if (!ptr) return clear_ok();
  TP_CUDA_TRY(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
  return clear_ok();
}
