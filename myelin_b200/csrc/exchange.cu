// Device buffers shared between the processes of a multi-GPU job through
// CUDA IPC handles: the gather buffers of the fused pack + all-gather
// (mb_pack_count_scatter). One process per GPU allocates its buffer with
// mb_ipc_alloc, the handles travel between processes on the host (any
// channel: torch.distributed in the Python layer), and each process maps the
// others' buffers with mb_ipc_open. Plain peer-to-peer memory over
// NVLink / NVSwitch: no switch-replicated (NVLS) mapping is created.
#include <cstring>

#include "common.cuh"
#include "exchange.cuh"

namespace mb {

namespace {

template <typename W>
struct PushPeers {
  W* p[kMaxPushPeers];
};

constexpr int kPushUnroll = 4;

// Grid-stride copy of n units (16 or 4 bytes) from src to NPEER peers: each
// thread keeps kPushUnroll loads in flight, then stores every unit to every
// peer (a warp stores 512 contiguous bytes per peer per instruction with
// 16-byte units).
template <typename W, int NPEER>
__global__ void __launch_bounds__(256) push_kernel(const W* __restrict__ src,
                                                   const PushPeers<W> peers, int64_t n) {
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; i + (kPushUnroll - 1) * stride < n; i += kPushUnroll * stride) {
    W v[kPushUnroll];
#pragma unroll
    for (int u = 0; u < kPushUnroll; ++u) v[u] = src[i + u * stride];
#pragma unroll
    for (int u = 0; u < kPushUnroll; ++u) {
#pragma unroll
      for (int d = 0; d < NPEER; ++d) peers.p[d][i + u * stride] = v[u];
    }
  }
  for (; i < n; i += stride) {
    const W v = src[i];
#pragma unroll
    for (int d = 0; d < NPEER; ++d) peers.p[d][i] = v;
  }
  __threadfence_system();  // peer stores ordered before the kernel's end
}

template <typename W>
void launch_push(const void* src, void* const* peers, int num_peers, int64_t n, cudaStream_t s) {
  PushPeers<W> pp{};
  for (int d = 0; d < num_peers; ++d) pp.p[d] = static_cast<W*>(peers[d]);
  int64_t blocks = ceil_div(n, 256 * kPushUnroll);
  if (blocks > 148 * 4) blocks = 148 * 4;
  if (blocks < 1) blocks = 1;
  const auto* in = static_cast<const W*>(src);
  const unsigned g = static_cast<unsigned>(blocks);
  switch (num_peers) {
    case 1: push_kernel<W, 1><<<g, 256, 0, s>>>(in, pp, n); break;
    case 2: push_kernel<W, 2><<<g, 256, 0, s>>>(in, pp, n); break;
    case 3: push_kernel<W, 3><<<g, 256, 0, s>>>(in, pp, n); break;
    case 4: push_kernel<W, 4><<<g, 256, 0, s>>>(in, pp, n); break;
    case 5: push_kernel<W, 5><<<g, 256, 0, s>>>(in, pp, n); break;
    case 6: push_kernel<W, 6><<<g, 256, 0, s>>>(in, pp, n); break;
    case 7: push_kernel<W, 7><<<g, 256, 0, s>>>(in, pp, n); break;
    default: break;
  }
}

}  // namespace

void push_to_peers(const void* src, void* const* peers, int num_peers, size_t bytes,
                   cudaStream_t s) {
  if (num_peers <= 0 || bytes == 0) return;
  bool vec = bytes % 16 == 0 && aligned_to(src, 16);
  for (int d = 0; d < num_peers; ++d) vec = vec && aligned_to(peers[d], 16);
  if (vec) {
    launch_push<uint4>(src, peers, num_peers, static_cast<int64_t>(bytes / 16), s);
  } else {
    launch_push<uint32_t>(src, peers, num_peers, static_cast<int64_t>(bytes / 4), s);
  }
}

}  // namespace mb

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
