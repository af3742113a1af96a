// Shared device/host helpers for the myelin_b200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/myelin_b200.h"

namespace mb {

// ---------------------------------------------------------------------------
// Error reporting: every C entry point returns an int status and records a
// thread-local message for mb_last_error().
// ---------------------------------------------------------------------------
void set_error(const char* fmt, ...);
void clear_error();

#define MB_CHECK_ARG(cond, ...)       \
  do {                                \
    if (!(cond)) {                    \
      ::mb::set_error(__VA_ARGS__);   \
      return 1;                       \
    }                                 \
  } while (0)

#define MB_CHECK_LAUNCH(what)                                                    \
  do {                                                                           \
    cudaError_t err__ = cudaGetLastError();                                      \
    if (err__ != cudaSuccess) {                                                  \
      ::mb::set_error("%s: CUDA launch failed: %s", what, cudaGetErrorString(err__)); \
      return 2;                                                                  \
    }                                                                            \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ---------------------------------------------------------------------------
// I/O element conversion. The scan always computes in fp32; 16-bit tensors are
// widened on load and rounded to nearest-even on store.
// ---------------------------------------------------------------------------
template <typename T>
struct Elem;

template <>
struct Elem<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
  static __device__ __forceinline__ float one() { return 1.0f; }
  static __device__ __forceinline__ float zero() { return 0.0f; }
};

template <>
struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ __nv_bfloat16 one() { return __float2bfloat16_rn(1.0f); }
  static __device__ __forceinline__ __nv_bfloat16 zero() { return __float2bfloat16_rn(0.0f); }
};

template <>
struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ __half one() { return __float2half_rn(1.0f); }
  static __device__ __forceinline__ __half zero() { return __float2half_rn(0.0f); }
};

// A run of NPT consecutive elements moved with one vector instruction.
template <typename T, int NPT>
struct alignas(sizeof(T) * NPT) Vec {
  T v[NPT];
};

template <typename T, int NPT>
__device__ __forceinline__ Vec<T, NPT> load_vec(const T* p) {
  return *reinterpret_cast<const Vec<T, NPT>*>(p);
}

template <typename T, int NPT>
__device__ __forceinline__ void store_vec(T* p, const Vec<T, NPT>& v) {
  *reinterpret_cast<Vec<T, NPT>*>(p) = v;
}

__host__ __device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline bool aligned_to(const void* p, int64_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) % static_cast<uintptr_t>(bytes)) == 0;
}

}  // namespace mb
