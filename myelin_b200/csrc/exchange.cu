// Device buffers shared between the processes of a multi-GPU job through
// CUDA IPC handles: the gather buffers of the fused pack + all-gather
// (mb_pack_count_scatter). One process per GPU allocates its buffer with
// mb_ipc_alloc, the handles travel between processes on the host (any
// channel: torch.distributed in the Python layer), and each process maps the
// others' buffers with mb_ipc_open. Plain peer-to-peer memory over
// NVLink / NVSwitch: no multicast object is created.
#include <cstring>

#include "common.cuh"

using namespace mb;

extern "C" int mb_ipc_alloc(int64_t bytes, void** ptr, void* handle) {
  clear_error();
  MB_CHECK_ARG(bytes > 0 && ptr != nullptr && handle != nullptr, "mb_ipc_alloc: bad arguments");
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, static_cast<size_t>(bytes));
  if (e != cudaSuccess) {
    set_error("mb_ipc_alloc: cudaMalloc of %lld bytes failed: %s", (long long)bytes,
              cudaGetErrorString(e));
    return 1;
  }
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    set_error("mb_ipc_alloc: cudaIpcGetMemHandle failed: %s", cudaGetErrorString(e));
    return 1;
  }
  memcpy(handle, &h, sizeof(h));
  return 0;
}

extern "C" int mb_ipc_open(const void* handle, void** ptr) {
  clear_error();
  MB_CHECK_ARG(handle != nullptr && ptr != nullptr, "mb_ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    *ptr = nullptr;
    set_error("mb_ipc_open: cudaIpcOpenMemHandle failed: %s", cudaGetErrorString(e));
    return 1;
  }
  return 0;
}

extern "C" int mb_ipc_close(void* ptr) {
  clear_error();
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) {
    set_error("mb_ipc_close: %s", cudaGetErrorString(e));
    return 1;
  }
  return 0;
}

extern "C" int mb_ipc_free(void* ptr) {
  clear_error();
  const cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) {
    set_error("mb_ipc_free: %s", cudaGetErrorString(e));
    return 1;
  }
  return 0;
}

extern "C" int mb_ipc_handle_bytes(void) { return static_cast<int>(sizeof(cudaIpcMemHandle_t)); }
