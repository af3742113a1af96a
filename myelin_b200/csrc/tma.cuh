// Tensor-map (TMA descriptor) creation shared by the kernels that move tiles
// with cp.async.bulk.tensor: the driver's cuTensorMapEncodeTiled, looked up
// once through the runtime (no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

namespace mb {

inline PFN_cuTensorMapEncodeTiled_v12000 tma_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

// 2-D bulk tensor store of a dense shared-memory box to global memory, tracked
// in the issuing thread's bulk async-group (committed here). Elements of the
// box outside the tensor are not written.
__device__ __forceinline__ void tma_store_box_2d(const CUtensorMap* map, const void* src, int c0,
                                                 int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(c0), "r"(c1), "r"(static_cast<uint32_t>(__cvta_generic_to_shared(src)))
      : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// 2-D bulk tensor load of one box at (c0, c1) into dense shared memory (128-byte
// aligned), completing as transaction bytes on the mbarrier `bar`. The whole
// box is written: elements outside the tensor read as zero, and the
// transaction count is the full box size. Loads of this GPU's own memory only.
__device__ __forceinline__ void tma_load_box_2d(void* dst, const CUtensorMap* map, int c0, int c1,
                                                uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1),
      "r"(static_cast<uint32_t>(__cvta_generic_to_shared(bar)))
      : "memory");
}

}  // namespace mb
