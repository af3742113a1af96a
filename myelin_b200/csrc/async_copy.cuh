// Bulk asynchronous global->shared copies (the TMA engine's 1-D form) tracked
// by shared-memory mbarriers, for sm_100a. Every wait is bounded: a wait that
// runs out records an error code in a device status word that the host reads
// with mb_device_status(), and returns false instead of spinning forever.
#pragma once

#include "common.cuh"

namespace mb {

// Device status word of this translation unit: 0 = ok. Set (first error
// wins) by kernels whose bounded waits ran out. The library is built without
// relocatable device code, so every .cu file that includes this header has
// its own copy of the word; each such file defines one host accessor (below)
// and mb_device_status() combines all of them.
static __device__ int g_device_status = 0;

// Host accessors, one per translation unit that includes this header: read
// (and with `clear`, reset) that unit's status word; -1 if it can't be read.
int scan_unit_status(bool clear);       // scan.cu
int scan_fast_unit_status(bool clear);  // scan_fast.cu
int gemm_unit_status(bool clear);       // gemm_tcgen05.cu

// Launchers of each unit's wait-timeout probe (wait_timeout_probe_kernel).
cudaError_t scan_unit_wait_probe(uint32_t polls, cudaStream_t stream);
cudaError_t scan_fast_unit_wait_probe(uint32_t polls, cudaStream_t stream);
cudaError_t gemm_unit_wait_probe(uint32_t polls, cudaStream_t stream);

enum DeviceStatus : int {
  kStatusOk = 0,
  kStatusWaitTimeout = 1,
};

__device__ __forceinline__ void record_status(int code) { atomicCAS(&g_device_status, 0, code); }

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// Make initialised barriers visible to the async proxy (the copy engine).
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy accesses (a buffer that was read is about to be refilled).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// Plain arrival (count 1) on a barrier, e.g. "this warp is done with a stage".
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// One contiguous copy of `bytes` (multiple of 16, both addresses 16-byte
// aligned) from global memory into this CTA's shared memory; completion is
// signalled on `bar` as transaction bytes.
__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// One contiguous copy of `bytes` (multiple of 16, both addresses 16-byte
// aligned) from this CTA's shared memory to global memory, tracked in the
// issuing thread's bulk async-group. Shared-memory writes that feed it must be
// ordered first with fence_proxy_async_smem by the threads that made them.
__device__ __forceinline__ void bulk_copy_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(smem_addr(src)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until this thread's committed bulk stores have finished reading their
// shared-memory sources (the buffer may then be reused).
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Wait until this thread's committed bulk stores have completed.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n"
      "  .reg .pred p;\n"
      "  mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "  selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Upper bound on try_wait polls (each poll may itself suspend the thread for a
// bounded, hardware-defined time). Far above any legitimate wait here: a chunk
// copy is tens of kilobytes.
constexpr uint32_t kMaxWaitPolls = 1u << 22;

__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint32_t max_polls = kMaxWaitPolls) {
  for (uint32_t i = 0; i < max_polls; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  record_status(kStatusWaitTimeout);
  return false;
}

namespace {

// Diagnostic: one thread waits, with a poll budget of `polls`, for phase 0 of
// a freshly initialised barrier that nothing ever arrives at, so the wait runs
// out through the same path as the kernels' own waits (the unit's status word
// becomes kStatusWaitTimeout) and the kernel returns. Nothing faults and
// nothing spins without bound.
__global__ void wait_timeout_probe_kernel(uint32_t polls) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
    mbar_wait_bounded(&bar, 0, polls);
  }
}

}  // namespace

// Host side: read (and optionally clear) this translation unit's status word.
// Synchronises with the device.
static inline int read_device_status(bool clear) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int)) != cudaSuccess) return -1;
  if (clear && v != 0) {
    const int zero = 0;
    if (cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int)) != cudaSuccess) return -1;
  }
  return v;
}

}  // namespace mb
