// Operand preparation for the tensor-core GEMM and the bias gradient.
//
// mb_split_bf16: an fp32 matrix becomes 1-3 bf16 matrices whose sum is the
// original value exactly (part p holds the bits 8p below the leading ones),
// so that mb_gemm can form fp32 products on the 16-bit tensor cores; 16-bit
// inputs are copied (one part), which also serves to re-lay out an operand
// whose strides the tensor-map copies cannot take (a transposed view, or rows
// not a multiple of 16 bytes, as for a 10-wide readout layer).
//
// mb_column_sums: per-column sums of a [rows, cols] matrix in fp32 with a
// fixed summation order (row slices summed in order, then the slices in
// order), e.g. the bias gradient db = sum over t, b of dL/dcurrents.
#include <type_traits>

#include "common.cuh"

namespace mb {
namespace {

template <typename TS>
__device__ __forceinline__ float load_as_float(const TS* p) {
  if constexpr (std::is_same<TS, float>::value) return __ldg(p);
  else return Elem<TS>::to_f(*p);
}

// One element -> up to 3 bf16 parts; returns a bitmask of nonzero parts.
// (A float16 destination is a plain one-part conversion.)
template <typename TD>
__device__ __forceinline__ uint32_t split_one(float x, int parts, TD* out, int64_t part_stride) {
  if constexpr (std::is_same<TD, __half>::value) {
    out[0] = __float2half_rn(x);
    return x != 0.0f ? 1u : 0u;
  } else {
    if (!isfinite(x)) {  // inf / nan stay in the leading part, the rest are zero
      out[0] = __float2bfloat16_rn(x);
      for (int p = 1; p < parts; ++p) out[p * part_stride] = __float2bfloat16_rn(0.0f);
      return 1u;
    }
    uint32_t nz = 0;
    float rest = x;
    for (int p = 0; p < parts; ++p) {
      const __nv_bfloat16 h = __float2bfloat16_rn(rest);
      out[p * part_stride] = h;
      const float hf = __bfloat162float(h);
      nz |= (hf != 0.0f) ? (1u << p) : 0u;
      rest = __fsub_rn(rest, hf);  // exact: the rounding error of a bf16 rounding
    }
    return nz;
  }
}

// Destination region [dst_rows, dst_cols] (each >= the source's): element
// (r, c) is the split of src(r, c) inside the source and zero outside it.
// Rows are spread over blockIdx.y (grid-stride), columns over the threads of
// blockIdx.x: consecutive threads touch consecutive columns (coalesced loads
// for a row-major source, coalesced stores of every part).
template <typename TS, typename TD>
__global__ void split_bf16_kernel(const TS* __restrict__ src, int64_t rows, int64_t cols,
                                  int64_t rs, int64_t cs, int parts,
                                  TD* __restrict__ dst, int64_t dst_rows,
                                  int64_t dst_cols, int64_t ld, int64_t part_stride,
                                  int32_t* nonzero) {
  uint32_t nz = 0;
  const int64_t c0 = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t cstep = int64_t(gridDim.x) * blockDim.x;
  for (int64_t r = blockIdx.y; r < dst_rows; r += gridDim.y) {
    const TS* srow = src + r * rs;
    TD* drow = dst + r * ld;
    for (int64_t c = c0; c < dst_cols; c += cstep) {
      const float x = (r < rows && c < cols) ? load_as_float(srow + c * cs) : 0.0f;
      nz |= split_one(x, parts, drow + c, part_stride);
    }
  }
  if (nonzero != nullptr) {
    nz = __reduce_or_sync(0xffffffffu, nz);
    if ((threadIdx.x & 31) == 0) {
      for (int p = 0; p < parts; ++p) {
        if (nz & (1u << p)) atomicOr(nonzero + p, 1);
      }
    }
  }
}

// Vector form of split_bf16_kernel for an fp32 source with unit column
// stride and 16-byte aligned rows, 4-aligned widths and a 4-aligned
// destination pitch: thread = 4 consecutive columns (one 16-byte load, one
// 8-byte store per part), rows on blockIdx.y, four rows' loads in flight.
template <int PARTS>
__device__ __forceinline__ uint32_t split_store4(const float4 v, __nv_bfloat16* out,
                                                 int64_t part_stride) {
  float rest[4] = {v.x, v.y, v.z, v.w};
  uint32_t nz = 0;
  bool finite[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) finite[e] = isfinite(rest[e]);
#pragma unroll
  for (int p = 0; p < PARTS; ++p) {
    __nv_bfloat16 h[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      // inf / nan stay in the leading part, the rest are zero
      h[e] = (p == 0 || finite[e]) ? __float2bfloat16_rn(rest[e]) : __float2bfloat16_rn(0.0f);
      const float hf = __bfloat162float(h[e]);
      nz |= (hf != 0.0f || (p == 0 && !finite[e])) ? (1u << p) : 0u;
      rest[e] = finite[e] ? __fsub_rn(rest[e], hf) : 0.0f;  // exact: a bf16 rounding error
    }
    uint2 w;
    w.x = uint32_t(__bfloat16_as_ushort(h[0])) | (uint32_t(__bfloat16_as_ushort(h[1])) << 16);
    w.y = uint32_t(__bfloat16_as_ushort(h[2])) | (uint32_t(__bfloat16_as_ushort(h[3])) << 16);
    *reinterpret_cast<uint2*>(out + p * part_stride) = w;
  }
  return nz;
}

template <int PARTS>
__global__ void split_bf16_vec4_kernel(const float* __restrict__ src, int64_t rows, int64_t cols,
                                       int64_t rs, __nv_bfloat16* __restrict__ dst,
                                       int64_t dst_rows, int64_t dst_cols, int64_t ld,
                                       int64_t part_stride, int32_t* nonzero) {
  uint32_t nz = 0;
  const int64_t c = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (c < dst_cols) {
    const bool in_cols = c < cols;  // cols % 4 == 0: a group is wholly in or out
    const int64_t step = gridDim.y;
    auto load = [&](int64_t r) {
      return (in_cols && r < rows) ? __ldg(reinterpret_cast<const float4*>(src + r * rs + c))
                                   : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    };
    int64_t r = blockIdx.y;
    for (; r + 3 * step < dst_rows; r += 4 * step) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) v[u] = load(r + u * step);
#pragma unroll
      for (int u = 0; u < 4; ++u) nz |= split_store4<PARTS>(v[u], dst + (r + u * step) * ld + c, part_stride);
    }
    for (; r < dst_rows; r += step) nz |= split_store4<PARTS>(load(r), dst + r * ld + c, part_stride);
  }
  if (nonzero != nullptr) {
    nz = __reduce_or_sync(0xffffffffu, nz);
    if ((threadIdx.x & 31) == 0) {
      for (int p = 0; p < PARTS; ++p) {
        if (nz & (1u << p)) atomicOr(nonzero + p, 1);
      }
    }
  }
}

// Column sums, stage 1: block (cb, slice) sums rows [slice * rows_per_slice,
// ...) of 256 consecutive columns, one column per thread, in row order.
template <typename TS>
__global__ void column_sums_partial_kernel(const TS* __restrict__ src, int64_t rows, int64_t cols,
                                           int64_t ld, int64_t rows_per_slice,
                                           float* __restrict__ partial) {
  const int64_t c = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t r0 = int64_t(blockIdx.y) * rows_per_slice;
  const int64_t r1 = imin64(rows, r0 + rows_per_slice);
  if (c >= cols) return;
  float acc = 0.0f;
  int64_t r = r0;
  // eight loads in flight, then their sums in row order
  for (; r + 8 <= r1; r += 8) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = load_as_float(src + (r + j) * ld + c);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc += v[j];
  }
  for (; r < r1; ++r) acc += load_as_float(src + r * ld + c);
  partial[int64_t(blockIdx.y) * cols + c] = acc;
}

// Vector form of stage 1 (16-byte rows, widths a multiple of the vector):
// thread = 16 bytes of consecutive columns (4 fp32 or 8 16-bit values),
// eight rows' loads in flight, each column summed in row order as above.
template <typename TS>
__device__ __forceinline__ void add_row16(float* acc, const uint4 v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  if constexpr (std::is_same<TS, float>::value) {
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[e] += __uint_as_float(w[e]);
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if constexpr (std::is_same<TS, __nv_bfloat16>::value) {
        acc[2 * e] += __uint_as_float(w[e] << 16);
        acc[2 * e + 1] += __uint_as_float(w[e] & 0xffff0000u);
      } else {
        acc[2 * e] += __half2float(__ushort_as_half(static_cast<uint16_t>(w[e] & 0xffffu)));
        acc[2 * e + 1] += __half2float(__ushort_as_half(static_cast<uint16_t>(w[e] >> 16)));
      }
    }
  }
}

template <typename TS>
__global__ void column_sums_partial_vec_kernel(const TS* __restrict__ src, int64_t rows,
                                               int64_t cols, int64_t ld, int64_t rows_per_slice,
                                               float* __restrict__ partial) {
  constexpr int kVec = 16 / int(sizeof(TS));
  const int64_t c = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) * kVec;
  const int64_t r0 = int64_t(blockIdx.y) * rows_per_slice;
  const int64_t r1 = imin64(rows, r0 + rows_per_slice);
  if (c >= cols) return;
  float acc[kVec];
#pragma unroll
  for (int e = 0; e < kVec; ++e) acc[e] = 0.0f;
  int64_t r = r0;
  for (; r + 8 <= r1; r += 8) {
    uint4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __ldg(reinterpret_cast<const uint4*>(src + (r + j) * ld + c));
#pragma unroll
    for (int j = 0; j < 8; ++j) add_row16<TS>(acc, v[j]);
  }
  for (; r < r1; ++r) add_row16<TS>(acc, __ldg(reinterpret_cast<const uint4*>(src + r * ld + c)));
  float* out = partial + int64_t(blockIdx.y) * cols + c;
#pragma unroll
  for (int e = 0; e < kVec; ++e) out[e] = acc[e];
}

// Stage 2: sum the slices of each column in slice order, write out.
template <typename TO>
__global__ void column_sums_final_kernel(const float* __restrict__ partial, int64_t slices,
                                         int64_t cols, TO* __restrict__ out) {
  const int64_t c = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (c >= cols) return;
  float acc = 0.0f;
  int64_t s = 0;
  for (; s + 32 <= slices; s += 32) {  // 32 loads in flight, summed in slice order
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = partial[(s + j) * cols + c];
#pragma unroll
    for (int j = 0; j < 32; ++j) acc += v[j];
  }
  for (; s < slices; ++s) acc += partial[s * cols + c];
  out[c] = Elem<TO>::from_f(acc);
}

int64_t column_slices(int64_t rows, int64_t cols) {
  // about 8 blocks per SM when a thread reads 4 columns (fp32 vector loads;
  // 16-bit ones read 8, so half as many blocks with twice the bytes each)
  const int64_t col_blocks = ceil_div(cols, 256 * 4);
  int64_t slices = ceil_div(148 * 8, col_blocks);
  const int64_t max_by_rows = ceil_div(rows, 128);  // at least 128 rows per slice
  if (slices > max_by_rows) slices = max_by_rows;
  return slices < 1 ? 1 : slices;
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" int mb_split_bf16(int src_dtype, const void* src, int64_t rows, int64_t cols,
                             int64_t src_row_stride, int64_t src_col_stride, int parts, void* dst,
                             int64_t dst_rows, int64_t dst_cols, int64_t dst_ld,
                             int64_t dst_part_stride, int32_t* nonzero, void* stream) {
  clear_error();
  MB_CHECK_ARG(src_dtype == MB_F32 || src_dtype == MB_BF16 || src_dtype == MB_F16,
               "mb_split_bf16: source must be float32, bfloat16 or float16");
  MB_CHECK_ARG(parts >= 1 && parts <= 3, "mb_split_bf16: parts must be 1, 2 or 3");
  MB_CHECK_ARG(src_dtype == MB_F32 || parts == 1,
               "mb_split_bf16: a 16-bit source is copied in one part (of its own type)");
  MB_CHECK_ARG(rows >= 0 && cols >= 0, "mb_split_bf16: negative size");
  MB_CHECK_ARG(dst_rows >= rows && dst_cols >= cols && dst_ld >= dst_cols,
               "mb_split_bf16: destination region smaller than the source");
  MB_CHECK_ARG(parts == 1 || dst_part_stride >= dst_rows * dst_ld,
               "mb_split_bf16: part stride smaller than a part");
  cudaStream_t s = as_stream(stream);
  if (nonzero != nullptr) cudaMemsetAsync(nonzero, 0, sizeof(int32_t) * parts, s);
  if (dst_rows == 0 || dst_cols == 0) {
    MB_CHECK_LAUNCH("mb_split_bf16");
    return 0;
  }
  MB_CHECK_ARG((src != nullptr || rows * cols == 0) && dst != nullptr,
               "mb_split_bf16: null pointer");
  if (src_dtype == MB_F32 && src_col_stride == 1 && aligned_to(src, 16) && src_row_stride % 4 == 0 &&
      cols % 4 == 0 && dst_cols % 4 == 0 && dst_ld % 4 == 0 && dst_part_stride % 4 == 0 &&
      aligned_to(dst, 8)) {
    // 4 columns per thread, about 8 blocks of 256 threads per SM
    const int64_t col_blocks = ceil_div(dst_cols / 4, 256);
    const dim3 grid(static_cast<unsigned>(col_blocks),
                    static_cast<unsigned>(imin64(dst_rows, imin64(65535, ceil_div(148 * 8, col_blocks)))));
    auto* out = static_cast<__nv_bfloat16*>(dst);
    const auto* in = static_cast<const float*>(src);
    if (parts == 1) {
      split_bf16_vec4_kernel<1><<<grid, 256, 0, s>>>(in, rows, cols, src_row_stride, out, dst_rows,
                                                     dst_cols, dst_ld, dst_part_stride, nonzero);
    } else if (parts == 2) {
      split_bf16_vec4_kernel<2><<<grid, 256, 0, s>>>(in, rows, cols, src_row_stride, out, dst_rows,
                                                     dst_cols, dst_ld, dst_part_stride, nonzero);
    } else {
      split_bf16_vec4_kernel<3><<<grid, 256, 0, s>>>(in, rows, cols, src_row_stride, out, dst_rows,
                                                     dst_cols, dst_ld, dst_part_stride, nonzero);
    }
    MB_CHECK_LAUNCH("mb_split_bf16");
    return 0;
  }
  // enough blocks for about 16 per SM: columns in blocks of 256, rows on y
  const int64_t col_blocks = imin64(ceil_div(dst_cols, 256), 148 * 16);
  const dim3 grid(static_cast<unsigned>(col_blocks),
                  static_cast<unsigned>(imin64(dst_rows, imin64(65535, ceil_div(148 * 16, col_blocks)))));
  auto* out = static_cast<__nv_bfloat16*>(dst);
  switch (src_dtype) {
    case MB_F32:
      split_bf16_kernel<float, __nv_bfloat16><<<grid, 256, 0, s>>>(
          static_cast<const float*>(src), rows, cols, src_row_stride, src_col_stride, parts, out,
          dst_rows, dst_cols, dst_ld, dst_part_stride, nonzero);
      break;
    case MB_BF16:
      split_bf16_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(src), rows, cols, src_row_stride, src_col_stride,
          parts, out, dst_rows, dst_cols, dst_ld, dst_part_stride, nonzero);
      break;
    default:  // float16 stays float16 (one part)
      split_bf16_kernel<__half, __half><<<grid, 256, 0, s>>>(
          static_cast<const __half*>(src), rows, cols, src_row_stride, src_col_stride, parts,
          static_cast<__half*>(dst), dst_rows, dst_cols, dst_ld, dst_part_stride, nonzero);
      break;
  }
  MB_CHECK_LAUNCH("mb_split_bf16");
  return 0;
}

extern "C" int64_t mb_column_sums_workspace_bytes(int64_t rows, int64_t cols) {
  if (rows <= 0 || cols <= 0) return 0;
  return column_slices(rows, cols) * cols * int64_t(sizeof(float));
}

extern "C" int mb_column_sums(int dtype, const void* src, int64_t rows, int64_t cols, int64_t ld,
                              int out_dtype, void* out, void* workspace, int64_t workspace_bytes,
                              void* stream) {
  clear_error();
  MB_CHECK_ARG(dtype == MB_F32 || dtype == MB_BF16 || dtype == MB_F16,
               "mb_column_sums: source must be float32, bfloat16 or float16");
  MB_CHECK_ARG(out_dtype == MB_F32 || out_dtype == MB_BF16 || out_dtype == MB_F16,
               "mb_column_sums: output must be float32, bfloat16 or float16");
  MB_CHECK_ARG(rows >= 0 && cols >= 0 && ld >= cols, "mb_column_sums: bad shape");
  cudaStream_t s = as_stream(stream);
  if (cols == 0) return 0;
  MB_CHECK_ARG(out != nullptr, "mb_column_sums: null output");
  if (rows == 0) {
    cudaMemsetAsync(out, 0, cols * (out_dtype == MB_F32 ? 4 : 2), s);
    MB_CHECK_LAUNCH("mb_column_sums");
    return 0;
  }
  MB_CHECK_ARG(src != nullptr, "mb_column_sums: null source");
  const int64_t slices = column_slices(rows, cols);
  const int64_t need = slices * cols * int64_t(sizeof(float));
  MB_CHECK_ARG(workspace != nullptr && workspace_bytes >= need && aligned_to(workspace, 4),
               "mb_column_sums: workspace of %lld bytes required, got %lld", (long long)need,
               (long long)workspace_bytes);
  float* partial = static_cast<float*>(workspace);
  const dim3 grid1(static_cast<unsigned>(ceil_div(cols, 256)), static_cast<unsigned>(slices));
  const int64_t per = ceil_div(rows, slices);
  const int64_t vec = dtype == MB_F32 ? 4 : 8;  // elements per 16-byte load
  // wide rows (config 5: 51200 x 4096 bf16 103 -> 79 us); narrower ones keep a
  // thread per column, whose many warps hide the latency better
  if (cols >= 2048 && cols % vec == 0 && ld % vec == 0 && aligned_to(src, 16) &&
      aligned_to(workspace, 16)) {
    // narrower blocks when the slices alone leave the SMs short of blocks
    unsigned bs = 256;
    while (bs > 32 && ceil_div(cols / vec, bs) * slices < 148 * 4) bs /= 2;
    const dim3 gridv(static_cast<unsigned>(ceil_div(cols / vec, bs)), static_cast<unsigned>(slices));
    if (dtype == MB_F32) {
      column_sums_partial_vec_kernel<float><<<gridv, bs, 0, s>>>(
          static_cast<const float*>(src), rows, cols, ld, per, partial);
    } else if (dtype == MB_BF16) {
      column_sums_partial_vec_kernel<__nv_bfloat16><<<gridv, bs, 0, s>>>(
          static_cast<const __nv_bfloat16*>(src), rows, cols, ld, per, partial);
    } else {
      column_sums_partial_vec_kernel<__half><<<gridv, bs, 0, s>>>(
          static_cast<const __half*>(src), rows, cols, ld, per, partial);
    }
  } else switch (dtype) {
    case MB_F32:
      column_sums_partial_kernel<float><<<grid1, 256, 0, s>>>(static_cast<const float*>(src),
                                                              rows, cols, ld, per, partial);
      break;
    case MB_BF16:
      column_sums_partial_kernel<__nv_bfloat16><<<grid1, 256, 0, s>>>(
          static_cast<const __nv_bfloat16*>(src), rows, cols, ld, per, partial);
      break;
    default:
      column_sums_partial_kernel<__half><<<grid1, 256, 0, s>>>(static_cast<const __half*>(src),
                                                               rows, cols, ld, per, partial);
      break;
  }
  const unsigned grid2 = static_cast<unsigned>(ceil_div(cols, 256));
  switch (out_dtype) {
    case MB_F32:
      column_sums_final_kernel<float><<<grid2, 256, 0, s>>>(partial, slices, cols,
                                                            static_cast<float*>(out));
      break;
    case MB_BF16:
      column_sums_final_kernel<__nv_bfloat16><<<grid2, 256, 0, s>>>(
          partial, slices, cols, static_cast<__nv_bfloat16*>(out));
      break;
    default:
      column_sums_final_kernel<__half><<<grid2, 256, 0, s>>>(partial, slices, cols,
                                                             static_cast<__half*>(out));
      break;
  }
  MB_CHECK_LAUNCH("mb_column_sums");
  return 0;
}

// ---------------------------------------------------------------------------
// fp32 product with a short contraction (K <= 32), e.g. the input gradient of
// a 10-wide readout layer: C[M, N] = A[M, K] * B[N, K]^T in fp32 FMAs, k in
// order (deterministic). Block = 256 threads over 256 columns n and 32 rows m:
// a thread keeps its B row in registers and takes each A row from shared
// memory (one broadcast per k); a warp's stores of a row are 128 contiguous
// bytes.
// ---------------------------------------------------------------------------
namespace mb {
namespace {

constexpr int kSmallK = 32;
constexpr int kSmallRows = 32;

// C[m, n] = sum_k A[m, k] * B[n, k] for K <= KP (KP = 8, 16 or 32): one thread
// per output column n holds B's row n in registers, the block's kSmallRows
// rows of A sit in shared memory, both zero-padded to KP, and k is summed in
// order with fmaf. The padded terms add 0 * 0 to an accumulator that is never
// -0 (it starts at +0 and round-to-nearest sums give +0 for x + -x), so they
// change nothing. Each row of A is read as KP / 4 broadcast 16-byte loads.
template <int KP>
__global__ void gemm_small_k_kernel(const float* __restrict__ A, int64_t lda,
                                    const float* __restrict__ B, int64_t ldb, float* __restrict__ C,
                                    int64_t ldc, int64_t M, int64_t N, int K) {
  __shared__ __align__(16) float sa[kSmallRows][KP];
  const int64_t n = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t m0 = int64_t(blockIdx.y) * kSmallRows;
  for (int i = threadIdx.x; i < kSmallRows * KP; i += blockDim.x) {
    const int r = i / KP, k = i % KP;
    sa[r][k] = (m0 + r < M && k < K) ? A[(m0 + r) * lda + k] : 0.0f;
  }
  float b[KP];
#pragma unroll
  for (int k = 0; k < KP; ++k) b[k] = (n < N && k < K) ? B[n * ldb + k] : 0.0f;
  __syncthreads();
  if (n >= N) return;
  const int rows = static_cast<int>(M - m0 < kSmallRows ? M - m0 : kSmallRows);
  float* c = C + m0 * ldc + n;
#pragma unroll 4
  for (int r = 0; r < rows; ++r) {
    float acc = 0.0f;
#pragma unroll
    for (int q = 0; q < KP / 4; ++q) {
      const float4 a = *reinterpret_cast<const float4*>(&sa[r][4 * q]);
      acc = __fmaf_rn(a.x, b[4 * q], acc);
      acc = __fmaf_rn(a.y, b[4 * q + 1], acc);
      acc = __fmaf_rn(a.z, b[4 * q + 2], acc);
      acc = __fmaf_rn(a.w, b[4 * q + 3], acc);
    }
    c[r * ldc] = acc;
  }
}

}  // namespace
}  // namespace mb

extern "C" int mb_gemm_small_k(const float* A, int64_t lda, const float* B, int64_t ldb, float* C,
                               int64_t ldc, int64_t M, int64_t N, int64_t K, void* stream) {
  clear_error();
  MB_CHECK_ARG(M >= 0 && N >= 0 && K >= 0 && K <= kSmallK,
               "mb_gemm_small_k: K must be in [0, %d]", kSmallK);
  MB_CHECK_ARG(lda >= K && ldb >= K && ldc >= N, "mb_gemm_small_k: leading dimension too small");
  if (M == 0 || N == 0) return 0;
  MB_CHECK_ARG(A != nullptr && B != nullptr && C != nullptr, "mb_gemm_small_k: null pointer");
  const dim3 grid(static_cast<unsigned>(ceil_div(N, 256)), static_cast<unsigned>(ceil_div(M, kSmallRows)));
  cudaStream_t s = as_stream(stream);
  const int k = static_cast<int>(K);
  if (K <= 8) gemm_small_k_kernel<8><<<grid, 256, 0, s>>>(A, lda, B, ldb, C, ldc, M, N, k);
  else if (K <= 16) gemm_small_k_kernel<16><<<grid, 256, 0, s>>>(A, lda, B, ldb, C, ldc, M, N, k);
  else gemm_small_k_kernel<kSmallK><<<grid, 256, 0, s>>>(A, lda, B, ldb, C, ldc, M, N, k);
  MB_CHECK_LAUNCH("mb_gemm_small_k");
  return 0;
}
