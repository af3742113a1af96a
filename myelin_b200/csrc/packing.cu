// Bit-packed spike words: pack, unpack, per-row and per-neuron counts.
//
// Word format (src/myelin/packing.py:45-71): spikes[..., n] -> int32 words
// [..., ceil(n / 32)], bit j of word w holds neuron 32*w + j (LSB first),
// padding bits are zero, bit 31 makes the word negative.
//
// All kernels are HBM-streaming integer work. When the last dimension is a
// multiple of 32 and the base pointer is 16-byte aligned, every thread moves
// exactly 16 bytes per access (fully coalesced); other shapes take a scalar
// path with the same results.
#include <mutex>

#include "common.cuh"
#include "exchange.cuh"

namespace mb {

// ---------------------------------------------------------------------------
// Nonzero test on the raw bits of one element ("spikes != 0" in torch: -0.0
// is zero, NaN is nonzero).
// ---------------------------------------------------------------------------
template <int DT>
struct Raw;
template <> struct Raw<MB_U8>   { using U = uint8_t;  static __device__ __forceinline__ bool nz(U v) { return v != 0; } };
template <> struct Raw<MB_I16>  { using U = uint16_t; static __device__ __forceinline__ bool nz(U v) { return v != 0; } };
template <> struct Raw<MB_F16>  { using U = uint16_t; static __device__ __forceinline__ bool nz(U v) { return (v & 0x7fffu) != 0; } };
template <> struct Raw<MB_BF16> { using U = uint16_t; static __device__ __forceinline__ bool nz(U v) { return (v & 0x7fffu) != 0; } };
template <> struct Raw<MB_I32>  { using U = uint32_t; static __device__ __forceinline__ bool nz(U v) { return v != 0; } };
template <> struct Raw<MB_F32>  { using U = uint32_t; static __device__ __forceinline__ bool nz(U v) { return (v & 0x7fffffffu) != 0; } };
template <> struct Raw<MB_I64>  { using U = uint64_t; static __device__ __forceinline__ bool nz(U v) { return v != 0; } };
template <> struct Raw<MB_F64>  { using U = uint64_t; static __device__ __forceinline__ bool nz(U v) { return (v & 0x7fffffffffffffffull) != 0; } };

// The value 1 in each element type, as raw bits.
template <int DT> __device__ __forceinline__ typename Raw<DT>::U raw_one();
template <> __device__ __forceinline__ uint8_t raw_one<MB_U8>() { return 1; }
template <> __device__ __forceinline__ uint16_t raw_one<MB_I16>() { return 1; }
template <> __device__ __forceinline__ uint16_t raw_one<MB_F16>() { return 0x3c00u; }
template <> __device__ __forceinline__ uint16_t raw_one<MB_BF16>() { return 0x3f80u; }
template <> __device__ __forceinline__ uint32_t raw_one<MB_I32>() { return 1u; }
template <> __device__ __forceinline__ uint32_t raw_one<MB_F32>() { return 0x3f800000u; }
template <> __device__ __forceinline__ uint64_t raw_one<MB_I64>() { return 1ull; }
template <> __device__ __forceinline__ uint64_t raw_one<MB_F64>() { return 0x3ff0000000000000ull; }

// ---------------------------------------------------------------------------
// Pack, vector path: n % 32 == 0, 16-byte aligned. Each thread loads 16 bytes
// (kEPT elements) and contributes kEPT bits; the kLPW lanes that share one
// word OR their bits together with shuffles, and the first lane stores it.
// ---------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(256) pack_vec_kernel(const uint4* __restrict__ in,
                                                       int32_t* __restrict__ words,
                                                       int64_t n_vec) {
  using U = typename Raw<DT>::U;
  constexpr int kEPT = 16 / sizeof(U);
  constexpr int kLPW = 32 / kEPT;  // lanes per word
  const int lane = threadIdx.x & 31;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  // The grid-stride loop keeps whole warps together (n_vec is a multiple of
  // kLPW and every warp starts on a word boundary), so the shuffles below are
  // executed by full warps only when all lanes are in range.
  for (int64_t i0 = int64_t(blockIdx.x) * blockDim.x; i0 < n_vec; i0 += stride) {
    const int64_t i = i0 + threadIdx.x;
    uint32_t bits = 0;
    if (i < n_vec) {
      const uint4 v = in[i];
      U el[kEPT];
      *reinterpret_cast<uint4*>(el) = v;
      if (DT == MB_U8) {
        // four bytes at a time: high bit of each byte set iff the byte != 0
        const uint32_t* w4 = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t h = (((w4[q] & 0x7f7f7f7fu) + 0x7f7f7f7fu) | w4[q]) & 0x80808080u;
          h >>= 7;
          h = (h | (h >> 7) | (h >> 14) | (h >> 21)) & 0xfu;
          bits |= h << (4 * q);
        }
      } else {
#pragma unroll
        for (int k = 0; k < kEPT; ++k) bits |= uint32_t(Raw<DT>::nz(el[k])) << k;
      }
    }
    uint32_t word = bits << ((lane % kLPW) * kEPT);
#pragma unroll
    for (int off = 1; off < kLPW; off <<= 1) word |= __shfl_xor_sync(0xffffffffu, word, off);
    if (i < n_vec && (lane % kLPW) == 0) words[i / kLPW] = static_cast<int32_t>(word);
  }
}

// Pack, scalar path: one thread per output word.
template <int DT>
__global__ void __launch_bounds__(256) pack_scalar_kernel(const typename Raw<DT>::U* __restrict__ in,
                                                          int32_t* __restrict__ words, int64_t rows,
                                                          int64_t n, int64_t W) {
  const int64_t total = rows * W;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t wi = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; wi < total; wi += stride) {
    const int64_t r = wi / W;
    const int64_t w = wi - r * W;
    const int64_t n0 = w * 32;
    const int cnt = static_cast<int>(imin64(32, n - n0));
    const typename Raw<DT>::U* src = in + r * n + n0;
    uint32_t word = 0;
    for (int k = 0; k < cnt; ++k) word |= uint32_t(Raw<DT>::nz(src[k])) << k;
    words[wi] = static_cast<int32_t>(word);
  }
}

// ---------------------------------------------------------------------------
// Unpack.
// ---------------------------------------------------------------------------
template <int DT>
__global__ void __launch_bounds__(256) unpack_vec_kernel(const uint32_t* __restrict__ words,
                                                         uint4* __restrict__ out, int64_t n_vec) {
  using U = typename Raw<DT>::U;
  constexpr int kEPT = 16 / sizeof(U);
  constexpr int kLPW = 32 / kEPT;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n_vec; i += stride) {
    const uint32_t word = words[i / kLPW] >> ((i % kLPW) * kEPT);
    U el[kEPT];
#pragma unroll
    for (int k = 0; k < kEPT; ++k) el[k] = ((word >> k) & 1u) ? raw_one<DT>() : U(0);
    out[i] = *reinterpret_cast<const uint4*>(el);
  }
}

template <int DT>
__global__ void __launch_bounds__(256) unpack_scalar_kernel(const uint32_t* __restrict__ words,
                                                            typename Raw<DT>::U* __restrict__ out,
                                                            int64_t rows, int64_t n, int64_t W) {
  using U = typename Raw<DT>::U;
  const int64_t total = rows * n;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / n;
    const int64_t c = i - r * n;
    const uint32_t word = words[r * W + (c >> 5)];
    out[i] = ((word >> (c & 31)) & 1u) ? raw_one<DT>() : U(0);
  }
}

// ---------------------------------------------------------------------------
// Per-row counts: one warp per row, popcount over the row's words with the
// padding bits of the last word masked off.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) count_rows_kernel(const uint32_t* __restrict__ words,
                                                         int64_t* __restrict__ counts,
                                                         int64_t rows, int64_t W,
                                                         uint32_t last_mask) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t r = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < rows; r += warps) {
    const uint32_t* src = words + r * W;
    int64_t c = 0;
    for (int64_t w = lane; w < W; w += 32) {
      uint32_t v = src[w];
      if (w == W - 1) v &= last_mask;
      c += __popc(v);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) c += __shfl_xor_sync(0xffffffffu, c, off);
    if (lane == 0) counts[r] = c;
  }
}

// ---------------------------------------------------------------------------
// Per-neuron counts over all rows (column popcount). Each lane owns one word
// column; its 32 bit positions are counted in 8 SWAR registers holding four
// 8-bit counters each (bit k, k+8, k+16, k+24), flushed into 32 int32
// counters before any 8-bit counter can overflow. The 8 warps of a block take
// interleaved rows of the same 32 word columns and are reduced through shared
// memory; every (row slice, neuron) partial is written to the workspace and a
// second kernel sums the slices.
// ---------------------------------------------------------------------------
constexpr int kColWarps = 8;

__global__ void __launch_bounds__(256) count_columns_partial_kernel(
    const uint32_t* __restrict__ words, int32_t* __restrict__ partial, int64_t rows, int64_t W,
    int64_t n, int64_t rows_per_slice) {
  __shared__ int32_t red[kColWarps][32 * 33];
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  const int64_t w = int64_t(blockIdx.x) * 32 + lane;
  const int64_t r_begin = int64_t(blockIdx.y) * rows_per_slice;
  const int64_t r_end = imin64(rows, r_begin + rows_per_slice);

  int32_t acc[32];
#pragma unroll
  for (int k = 0; k < 32; ++k) acc[k] = 0;
  uint32_t swar[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) swar[k] = 0;
  int pending = 0;

  if (w < W) {
    for (int64_t r = r_begin + wid; r < r_end; r += kColWarps) {
      const uint32_t v = words[r * W + w];
#pragma unroll
      for (int k = 0; k < 8; ++k) swar[k] += (v >> k) & 0x01010101u;
      if (++pending == 255) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
#pragma unroll
          for (int q = 0; q < 4; ++q) acc[k + 8 * q] += (swar[k] >> (8 * q)) & 0xffu;
          swar[k] = 0;
        }
        pending = 0;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[k + 8 * q] += (swar[k] >> (8 * q)) & 0xffu;
  }
  // padding stride 33 keeps the transposed reads below conflict-free
#pragma unroll
  for (int k = 0; k < 32; ++k) red[wid][lane * 33 + k] = acc[k];
  __syncthreads();
  // thread t sums neuron (t) of this block's 32*32 = 1024 neurons, 4 per thread
  for (int j = threadIdx.x; j < 1024; j += blockDim.x) {
    const int wl = j >> 5;  // word column within block
    const int bit = j & 31;
    int32_t s = 0;
#pragma unroll
    for (int q = 0; q < kColWarps; ++q) s += red[q][wl * 33 + bit];
    const int64_t neuron = int64_t(blockIdx.x) * 1024 + j;
    if (neuron < n) partial[int64_t(blockIdx.y) * n + neuron] = s;
  }
}

// Sum of the per-slice partial counts: block = 32 neurons, its 8 warps take
// interleaved slices (coalesced 128-byte rows), then warp 0 adds the 8 warp
// sums in a fixed order (deterministic).
__global__ void __launch_bounds__(256) count_columns_final_kernel(const int32_t* __restrict__ partial,
                                                                  int64_t slices, int64_t n,
                                                                  int64_t* __restrict__ out64,
                                                                  int32_t* __restrict__ out32) {
  __shared__ int64_t red[8][32];
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  const int64_t j = int64_t(blockIdx.x) * 32 + lane;
  int64_t s = 0;
  if (j < n) {
#pragma unroll 4
    for (int64_t q = wid; q < slices; q += 8) s += partial[q * n + j];
  }
  red[wid][lane] = s;
  __syncthreads();
  if (wid == 0 && j < n) {
    int64_t t = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w][lane];
    if (out64) out64[j] = t;
    if (out32) out32[j] = static_cast<int32_t>(t);
  }
}

// ---------------------------------------------------------------------------
// Fused pack + per-neuron count for 1-byte spikes (bool / uint8 / int8),
// n % 32 == 0, 16-byte aligned: one pass over the spikes instead of a pack
// pass plus a count pass over the words.
//
// Thread = one word column (32 neurons = 32 bytes of every row); a block's
// kPackCountThreads threads take consecutive word columns of the rows of its
// slice. Per row and 4 bytes w:
//   m   = ((w & 0x7f7f7f7f) + 0x7f7f7f7f | w) & 0x80808080   bit 7 of each
//         byte set iff the byte is nonzero (no carry crosses a byte)
//   b   = m >> 7                                             0/1 per byte
//   (b * 0x01020408) >> 24                                   the 4 bits, LSB =
//         first byte: each byte's term lands on bit 24 + k; the other
//         products fall on distinct bits below 24 (no carry) or above 31
//   acc += b                                                 four 8-bit counters
// The 8-bit counters are flushed every 255 rows into 32 int32 counters per
// thread kept in shared memory (registers go to loads in flight instead: rows
// are processed kRowUnroll at a time, kRowUnroll x 32 bytes per thread).
// Per-slice partial counts go to the workspace and
// count_columns_final_kernel sums the slices (deterministic).
// ---------------------------------------------------------------------------
constexpr int kRowUnroll = 8;
constexpr int kPackCountThreads = 128;

__device__ __forceinline__ uint32_t nonzero_bytes(uint32_t w) {
  return ((((w & 0x7f7f7f7fu) + 0x7f7f7f7fu) | w) & 0x80808080u) >> 7;
}

// Further destinations of the packed words: this rank's [rows, W] slot in
// the other ranks' gather buffers (peer memory over NVLink).
constexpr int kMaxPeerSlots = 7;
struct PeerSlots {
  uint32_t* p[kMaxPeerSlots];
};

// COUNT = false packs only (the plain pack of 1-byte spikes: no counters, no
// partials). NPEER > 0 also stores each word to the first NPEER peer slots
// (plain stores; a compile-time count, so a word costs exactly 1 + NPEER
// stores and no predicates).
template <bool COUNT, int NPEER>
__global__ void __launch_bounds__(kPackCountThreads) pack_count_u8_kernel(
    const uint4* __restrict__ in, uint32_t* __restrict__ words,
    unsigned long long* __restrict__ counts64, unsigned int* __restrict__ counts32, int64_t rows,
    int64_t W, int64_t rows_per_slice, const PeerSlots peers) {
  // [neuron in word][thread], one pad column: conflict-free both for a thread
  // walking its own 32 counters and for a warp reading one thread's 32
  __shared__ int32_t cnt[32][kPackCountThreads + 1];
  const int tid = threadIdx.x;
  const int64_t wc = int64_t(blockIdx.x) * kPackCountThreads + tid;  // word column
  const int64_t r_begin = int64_t(blockIdx.y) * rows_per_slice;
  // with counters, columns past W take no rows (they still meet the block
  // barrier below); without, they leave at once
  if (!COUNT && wc >= W) return;
  const int64_t r_end = COUNT && wc >= W ? r_begin : imin64(rows, r_begin + rows_per_slice);

  if (COUNT) {
#pragma unroll
    for (int k = 0; k < 32; ++k) cnt[k][tid] = 0;
  }
  uint32_t acc[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) acc[q] = 0;
  int pending = 0;  // rows added to the 8-bit counters since the last flush

  auto flush = [&]() {
    if constexpr (COUNT) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
#pragma unroll
        for (int k = 0; k < 4; ++k) cnt[4 * q + k][tid] += (acc[q] >> (8 * k)) & 0xffu;
        acc[q] = 0;
      }
    }
    pending = 0;
  };
  auto consume = [&](uint4 lo, uint4 hi, int64_t r) {
    const uint32_t v[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
    uint32_t word = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint32_t b = nonzero_bytes(v[q]);
      word |= ((b * 0x01020408u) >> 24) << (4 * q);
      if (COUNT) acc[q] += b;
    }
    words[r * W + wc] = word;
#pragma unroll
    for (int d = 0; d < NPEER; ++d) peers.p[d][r * W + wc] = word;
  };

  const uint4* src = in + wc * 2;  // 2 x 16 bytes per row
  const int64_t row_vec = W * 2;
  int64_t r = r_begin;
  for (; r + kRowUnroll <= r_end; r += kRowUnroll) {
    uint4 lo[kRowUnroll], hi[kRowUnroll];
#pragma unroll
    for (int u = 0; u < kRowUnroll; ++u) {
      lo[u] = src[(r + u) * row_vec];
      hi[u] = src[(r + u) * row_vec + 1];
    }
#pragma unroll
    for (int u = 0; u < kRowUnroll; ++u) consume(lo[u], hi[u], r + u);
    pending += kRowUnroll;
    if (pending > 255 - kRowUnroll) flush();
  }
  for (; r < r_end; ++r) {
    consume(src[r * row_vec], src[r * row_vec + 1], r);
    if (++pending == 255) flush();
  }
  if (NPEER > 0) __threadfence_system();  // peer stores ordered before the kernel's end
  if (!COUNT) return;
  flush();
  __syncthreads();
  // The slice's counts go straight into the per-neuron totals: warp w reads
  // the 32 counters of each of its threads' word columns in turn, so each
  // reduction instruction covers 32 consecutive neurons (one 128-byte line of
  // int32 totals). Integer adds: the totals do not depend on their order.
  const int w = tid >> 5, lane = tid & 31;
  for (int j = 0; j < 32; ++j) {
    const int t = 32 * w + j;
    const int64_t col = int64_t(blockIdx.x) * kPackCountThreads + t;
    if (col >= W) break;  // uniform over the warp
    const unsigned int v = static_cast<unsigned int>(cnt[lane][t]);
    const int64_t neuron = col * 32 + lane;
    if (v != 0) {
      if (counts64) atomicAdd(counts64 + neuron, static_cast<unsigned long long>(v));
      if (counts32) atomicAdd(counts32 + neuron, v);
    }
  }
}

// ---------------------------------------------------------------------------
// Full-row variant of the fused kernel for the exchange: a block's THREADS
// threads cover every word column of its rows (W == THREADS), so the words of
// kRowUnroll consecutive rows are one contiguous run of kRowUnroll * W words
// in every destination (this rank's slot in its own gather buffer and in each
// peer's). The threads stage each group of rows in shared memory and one
// thread sends the group to all NDST destinations as bulk copies
// (cp.async.bulk shared -> global, no multicast), so NVLink carries runs of
// kRowUnroll * W * 4 bytes instead of one 128-byte warp store per row and
// peer, and the threads go on packing the next group while the copies drain.
// Two staging buffers alternate; a buffer is rewritten only after the copies
// of two groups ago have read it. Counting is the same as in
// pack_count_u8_kernel.
// ---------------------------------------------------------------------------
constexpr int kMaxDstSlots = 1 + kMaxPeerSlots;
struct DstSlots {
  uint32_t* p[kMaxDstSlots];
};

__device__ __forceinline__ void rows_fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <int THREADS, int NDST>
__global__ void __launch_bounds__(THREADS) pack_count_rows_kernel(
    const uint4* __restrict__ in, const DstSlots dst, unsigned long long* __restrict__ counts64,
    unsigned int* __restrict__ counts32, int64_t rows, int64_t rows_per_slice) {
  extern __shared__ __align__(128) unsigned char rows_smem[];
  constexpr int kStageWords = kRowUnroll * THREADS;
  uint32_t* stage = reinterpret_cast<uint32_t*>(rows_smem);           // [2][kRowUnroll][THREADS]
  auto cnt = reinterpret_cast<int32_t(*)[THREADS + 1]>(rows_smem + 2 * kStageWords * 4);
  const int tid = threadIdx.x;
  const int64_t r_begin = int64_t(blockIdx.x) * rows_per_slice;
  const int64_t r_end = imin64(rows, r_begin + rows_per_slice);

#pragma unroll
  for (int k = 0; k < 32; ++k) cnt[k][tid] = 0;
  uint32_t acc[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) acc[q] = 0;
  int pending = 0;
  auto flush = [&]() {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
#pragma unroll
      for (int k = 0; k < 4; ++k) cnt[4 * q + k][tid] += (acc[q] >> (8 * k)) & 0xffu;
      acc[q] = 0;
    }
    pending = 0;
  };

  const uint4* src = in + tid * 2;  // 2 x 16 bytes of every row
  constexpr int64_t row_vec = THREADS * 2;
  int group = 0;
  for (int64_t r = r_begin; r < r_end; r += kRowUnroll, ++group) {
    const int nr = static_cast<int>(imin64(kRowUnroll, r_end - r));
    uint32_t* st = stage + (group & 1) * kStageWords;
    if (group >= 2) {
      // the copies of two groups ago have read this buffer
      if (tid == 0) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
      __syncthreads();
    }
    uint4 lo[kRowUnroll], hi[kRowUnroll];
#pragma unroll
    for (int u = 0; u < kRowUnroll; ++u) {
      if (u < nr) {
        lo[u] = src[(r + u) * row_vec];
        hi[u] = src[(r + u) * row_vec + 1];
      }
    }
#pragma unroll
    for (int u = 0; u < kRowUnroll; ++u) {
      if (u < nr) {
        const uint32_t v[8] = {lo[u].x, lo[u].y, lo[u].z, lo[u].w, hi[u].x, hi[u].y, hi[u].z, hi[u].w};
        uint32_t word = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint32_t b = nonzero_bytes(v[q]);
          word |= ((b * 0x01020408u) >> 24) << (4 * q);
          acc[q] += b;
        }
        st[u * THREADS + tid] = word;
      }
    }
    pending += nr;
    if (pending > 255 - kRowUnroll) flush();
    rows_fence_proxy_async();  // this thread's staged words, before the copies read them
    __syncthreads();
    if (tid == 0) {
      const uint32_t bytes = static_cast<uint32_t>(nr) * THREADS * 4u;
#pragma unroll
      for (int d = 0; d < NDST; ++d) {
        asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
                         dst.p[d] + r * THREADS),
                     "r"(static_cast<uint32_t>(__cvta_generic_to_shared(st))), "r"(bytes)
                     : "memory");
      }
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
  }
  if (tid == 0) {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // every copy has landed
    __threadfence_system();  // and is ordered before the kernel's end for the other GPUs
  }
  flush();
  __syncthreads();
  const int w = tid >> 5, lane = tid & 31;
  for (int j = 0; j < 32; ++j) {
    const int t = 32 * w + j;
    const unsigned int v = static_cast<unsigned int>(cnt[lane][t]);
    const int64_t neuron = int64_t(t) * 32 + lane;
    if (v != 0) {
      if (counts64) atomicAdd(counts64 + neuron, static_cast<unsigned long long>(v));
      if (counts32) atomicAdd(counts32 + neuron, v);
    }
  }
}

template <int THREADS>
constexpr size_t rows_kernel_smem() {
  return size_t(2) * kRowUnroll * THREADS * 4 + size_t(32) * (THREADS + 1) * 4;
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
static int grid_for(int64_t work_items, int block = 256) {
  const int64_t cap = 148 * 32;  // grid-stride loops beyond ~32 blocks per SM
  int64_t g = ceil_div(work_items, block);
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

static int64_t pack_count_slices(int64_t rows, int64_t n);

template <int DT>
static void launch_pack(const void* spikes, int32_t* words, int64_t rows, int64_t n,
                        cudaStream_t s) {
  using U = typename Raw<DT>::U;
  const int64_t W = ceil_div(n, 32);
  if (DT == MB_U8 && n % 32 == 0 && aligned_to(spikes, 16)) {
    // 1-byte spikes: the fused kernel without its counters (8 rows in flight)
    const int64_t slices = pack_count_slices(rows, n);
    dim3 grid(static_cast<unsigned>(ceil_div(W, kPackCountThreads)),
              static_cast<unsigned>(slices));
    pack_count_u8_kernel<false, 0><<<grid, kPackCountThreads, 0, s>>>(
        static_cast<const uint4*>(spikes), reinterpret_cast<uint32_t*>(words), nullptr, nullptr,
        rows, W, ceil_div(rows, slices), PeerSlots{});
  } else if (n % 32 == 0 && aligned_to(spikes, 16)) {
    const int64_t n_vec = rows * n * int64_t(sizeof(U)) / 16;
    pack_vec_kernel<DT><<<grid_for(n_vec), 256, 0, s>>>(static_cast<const uint4*>(spikes), words,
                                                        n_vec);
  } else {
    pack_scalar_kernel<DT><<<grid_for(rows * W), 256, 0, s>>>(static_cast<const U*>(spikes),
                                                             words, rows, n, W);
  }
}

template <int DT>
static void launch_unpack(const int32_t* words, void* out, int64_t rows, int64_t n,
                          cudaStream_t s) {
  using U = typename Raw<DT>::U;
  const int64_t W = ceil_div(n, 32);
  const uint32_t* uw = reinterpret_cast<const uint32_t*>(words);
  if (n % 32 == 0 && aligned_to(out, 16)) {
    const int64_t n_vec = rows * n * int64_t(sizeof(U)) / 16;
    unpack_vec_kernel<DT><<<grid_for(n_vec), 256, 0, s>>>(uw, static_cast<uint4*>(out), n_vec);
  } else {
    unpack_scalar_kernel<DT><<<grid_for(rows * n), 256, 0, s>>>(uw, static_cast<U*>(out), rows, n,
                                                               W);
  }
}

#define MB_DISPATCH_DTYPE(dtype, FN, ...)              \
  switch (dtype) {                                     \
    case MB_F32: FN<MB_F32>(__VA_ARGS__); break;       \
    case MB_BF16: FN<MB_BF16>(__VA_ARGS__); break;     \
    case MB_F16: FN<MB_F16>(__VA_ARGS__); break;       \
    case MB_F64: FN<MB_F64>(__VA_ARGS__); break;       \
    case MB_U8: FN<MB_U8>(__VA_ARGS__); break;         \
    case MB_I16: FN<MB_I16>(__VA_ARGS__); break;       \
    case MB_I32: FN<MB_I32>(__VA_ARGS__); break;       \
    default: FN<MB_I64>(__VA_ARGS__); break;           \
  }

// Row slices for the column count: enough blocks for ~4 per SM, at least
// 64 rows per slice.
static int64_t column_slices(int64_t rows, int64_t n) {
  const int64_t col_blocks = ceil_div(ceil_div(n, 32), 32);
  int64_t slices = ceil_div(148 * 4, col_blocks);
  const int64_t max_by_rows = ceil_div(rows, 64);
  if (slices > max_by_rows) slices = max_by_rows;
  if (slices < 1) slices = 1;
  return slices;
}

int launch_count_columns(const int32_t* words, int64_t rows, int64_t n, int64_t* counts64,
                         int32_t* counts32, int32_t* workspace, cudaStream_t s) {
  const int64_t W = ceil_div(n, 32);
  const int64_t slices = column_slices(rows, n);
  const int64_t rows_per_slice = ceil_div(rows, slices);
  dim3 grid(static_cast<unsigned>(ceil_div(W, 32)), static_cast<unsigned>(slices));
  count_columns_partial_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const uint32_t*>(words),
                                                    workspace, rows, W, n, rows_per_slice);
  count_columns_final_kernel<<<static_cast<unsigned>(ceil_div(n, 32)), 256, 0, s>>>(workspace, slices, n, counts64, counts32);
  return 0;
}

int64_t count_columns_workspace_bytes(int64_t rows, int64_t n) {
  if (rows <= 0 || n <= 0) return 0;
  return column_slices(rows, n) * n * int64_t(sizeof(int32_t));
}

// Row slices of the fused pack + count: about five blocks per SM (the register
// limit; each thread keeps kRowUnroll x 32 bytes in flight), at least 64 rows
// each.
static int64_t pack_count_slices(int64_t rows, int64_t n) {
  const int64_t col_blocks = ceil_div(n / 32, kPackCountThreads);
  int64_t slices = ceil_div(148 * 5, col_blocks);
  const int64_t max_by_rows = ceil_div(rows, 64);
  if (slices > max_by_rows) slices = max_by_rows;
  if (slices < 1) slices = 1;
  return slices;
}

static bool pack_count_fused_ok(int dtype, const void* spikes, int64_t n) {
  return dtype == MB_U8 && n % 32 == 0 && aligned_to(spikes, 16);
}

// The fused kernel needs no scratch; the pack-then-count path (other dtypes,
// ragged or unaligned spikes) needs the column count's.
int64_t pack_count_workspace_bytes(int64_t rows, int64_t n) {
  if (rows <= 0 || n <= 0) return 0;
  return count_columns_workspace_bytes(rows, n);
}

// Pack + per-neuron count: one fused pass for aligned 1-byte spikes with
// n % 32 == 0, else the pack kernel followed by the column count of the words.
// The fused pack + count of aligned 1-byte spikes (n % 32 == 0): the totals
// are zeroed, then one kernel packs (words to `words` and to `npeer` peer
// slots) and adds each row slice's counts into them.
static void launch_pack_count_u8(const void* spikes, int32_t* words, const PeerSlots& peers,
                                 int npeer, int64_t rows, int64_t n, int64_t* counts64,
                                 int32_t* counts32, cudaStream_t s) {
  const int64_t W = n / 32;
  const int64_t slices = pack_count_slices(rows, n);
  const dim3 grid(static_cast<unsigned>(ceil_div(W, kPackCountThreads)),
                  static_cast<unsigned>(slices));
  const auto* in = static_cast<const uint4*>(spikes);
  auto* out = reinterpret_cast<uint32_t*>(words);
  auto* c64 = reinterpret_cast<unsigned long long*>(counts64);
  auto* c32 = reinterpret_cast<unsigned int*>(counts32);
  if (c64) cudaMemsetAsync(c64, 0, size_t(n) * sizeof(int64_t), s);
  if (c32) cudaMemsetAsync(c32, 0, size_t(n) * sizeof(int32_t), s);
  const int64_t per_slice = ceil_div(rows, slices);
  switch (npeer) {
#define MB_PACK_PEERS(K)                                                                     \
  case K:                                                                                    \
    pack_count_u8_kernel<true, K>                                                            \
        <<<grid, kPackCountThreads, 0, s>>>(in, out, c64, c32, rows, W, per_slice, peers);  \
    break;
    MB_PACK_PEERS(0)
    MB_PACK_PEERS(1)
    MB_PACK_PEERS(2)
    MB_PACK_PEERS(3)
    MB_PACK_PEERS(4)
    MB_PACK_PEERS(5)
    MB_PACK_PEERS(6)
    MB_PACK_PEERS(7)
#undef MB_PACK_PEERS
    default: break;
  }
}

// The full-row exchange kernel applies when a row is 128 or 256 words
// (n = 4096 or 8192 neurons) and every destination is 16-byte aligned.
static bool pack_count_rows_ok(int64_t n, int32_t* words, void* const* peers, int num_peers) {
  const int64_t W = n / 32;
  if (W != 128 && W != 256) return false;
  if (!aligned_to(words, 16)) return false;
  for (int d = 0; d < num_peers; ++d) {
    if (!aligned_to(peers[d], 16)) return false;
  }
  return true;
}

template <int THREADS>
static void launch_pack_count_rows_t(const void* spikes, const DstSlots& dst, int ndst,
                                     int64_t rows, int64_t rows_per_slice, int64_t slices,
                                     unsigned long long* c64, unsigned int* c32, cudaStream_t s) {
  const auto* in = static_cast<const uint4*>(spikes);
  constexpr size_t smem = rows_kernel_smem<THREADS>();
  const unsigned grid = static_cast<unsigned>(slices);
  switch (ndst) {
#define MB_PACK_ROWS(K)                                                                        \
  case K: {                                                                                    \
    auto kern = pack_count_rows_kernel<THREADS, K>;                                            \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));        \
    kern<<<grid, THREADS, smem, s>>>(in, dst, c64, c32, rows, rows_per_slice);                 \
    break;                                                                                     \
  }
    MB_PACK_ROWS(1)
    MB_PACK_ROWS(2)
    MB_PACK_ROWS(3)
    MB_PACK_ROWS(4)
    MB_PACK_ROWS(5)
    MB_PACK_ROWS(6)
    MB_PACK_ROWS(7)
    MB_PACK_ROWS(8)
#undef MB_PACK_ROWS
    default: break;
  }
}

// Rows per block: a multiple of kRowUnroll, at most 4 blocks per SM's worth
// of slices, at least 16 rows per block.
static void launch_pack_count_rows(const void* spikes, int32_t* words, void* const* peers,
                                   int num_peers, int64_t rows, int64_t n, int64_t* counts64,
                                   int32_t* counts32, cudaStream_t s) {
  DstSlots dst{};
  dst.p[0] = reinterpret_cast<uint32_t*>(words);
  for (int d = 0; d < num_peers; ++d) dst.p[1 + d] = static_cast<uint32_t*>(peers[d]);
  auto* c64 = reinterpret_cast<unsigned long long*>(counts64);
  auto* c32 = reinterpret_cast<unsigned int*>(counts32);
  if (c64) cudaMemsetAsync(c64, 0, size_t(n) * sizeof(int64_t), s);
  if (c32) cudaMemsetAsync(c32, 0, size_t(n) * sizeof(int32_t), s);
  int64_t slices = imin64(ceil_div(rows, 16), 148 * 4);
  if (slices < 1) slices = 1;
  const int64_t per = ceil_div(ceil_div(rows, slices), kRowUnroll) * kRowUnroll;
  slices = ceil_div(rows, per);
  if (n / 32 == 256) {
    launch_pack_count_rows_t<256>(spikes, dst, 1 + num_peers, rows, per, slices, c64, c32, s);
  } else {
    launch_pack_count_rows_t<128>(spikes, dst, 1 + num_peers, rows, per, slices, c64, c32, s);
  }
}

template <int DT>
static void launch_pack_count(const void* spikes, int32_t* words, int64_t rows, int64_t n,
                              int64_t* counts64, int32_t* counts32, void* workspace,
                              cudaStream_t s) {
  if (pack_count_fused_ok(DT, spikes, n) && pack_count_rows_ok(n, words, nullptr, 0)) {
    // whole rows per block, words out as bulk copies (config 4 on one GPU:
    // 0.230 -> 0.213 ms against the per-thread word stores below)
    launch_pack_count_rows(spikes, words, nullptr, 0, rows, n, counts64, counts32, s);
    return;
  }
  if (pack_count_fused_ok(DT, spikes, n)) {
    launch_pack_count_u8(spikes, words, PeerSlots{}, 0, rows, n, counts64, counts32, s);
    return;
  }
  launch_pack<DT>(spikes, words, rows, n, s);
  launch_count_columns(words, rows, n, counts64, counts32, static_cast<int32_t*>(workspace), s);
}

}  // namespace mb

using namespace mb;

static bool valid_io_dtype(int dtype) { return dtype >= MB_F32 && dtype <= MB_I64; }

extern "C" int mb_pack_spikes(int dtype, const void* spikes, int32_t* words, int64_t rows,
                              int64_t n, void* stream) {
  clear_error();
  MB_CHECK_ARG(valid_io_dtype(dtype), "mb_pack_spikes: unknown dtype %d", dtype);
  MB_CHECK_ARG(rows >= 0 && n > 0, "mb_pack_spikes: cannot pack an empty last dimension");
  if (rows == 0) return 0;
  MB_CHECK_ARG(spikes != nullptr && words != nullptr, "mb_pack_spikes: null pointer");
  cudaStream_t s = as_stream(stream);
  MB_DISPATCH_DTYPE(dtype, launch_pack, spikes, words, rows, n, s);
  MB_CHECK_LAUNCH("mb_pack_spikes");
  return 0;
}

extern "C" int mb_unpack_spikes(const int32_t* words, int dtype, void* out, int64_t rows,
                                int64_t n, void* stream) {
  clear_error();
  MB_CHECK_ARG(valid_io_dtype(dtype), "mb_unpack_spikes: unknown dtype %d", dtype);
  MB_CHECK_ARG(rows >= 0 && n > 0, "mb_unpack_spikes: packed.original_shape must have non-empty last dimension");
  if (rows == 0) return 0;
  MB_CHECK_ARG(words != nullptr && out != nullptr, "mb_unpack_spikes: null pointer");
  cudaStream_t s = as_stream(stream);
  MB_DISPATCH_DTYPE(dtype, launch_unpack, words, out, rows, n, s);
  MB_CHECK_LAUNCH("mb_unpack_spikes");
  return 0;
}

extern "C" int mb_count_rows(const int32_t* words, int64_t rows, int64_t n, int64_t* counts,
                             void* stream) {
  clear_error();
  MB_CHECK_ARG(rows >= 0 && n > 0, "mb_count_rows: packed.original_shape must have non-empty last dimension");
  if (rows == 0) return 0;
  MB_CHECK_ARG(words != nullptr && counts != nullptr, "mb_count_rows: null pointer");
  const int64_t W = ceil_div(n, 32);
  const uint32_t last_mask = (n % 32 == 0) ? 0xffffffffu : ((1u << (n % 32)) - 1u);
  count_rows_kernel<<<grid_for(rows * 32), 256, 0, as_stream(stream)>>>(
      reinterpret_cast<const uint32_t*>(words), counts, rows, W, last_mask);
  MB_CHECK_LAUNCH("mb_count_rows");
  return 0;
}

extern "C" int64_t mb_count_columns_workspace_bytes(int64_t rows, int64_t n) {
  return count_columns_workspace_bytes(rows, n);
}

extern "C" int mb_count_columns(const int32_t* words, int64_t rows, int64_t n, int64_t* counts64,
                                int32_t* counts32, void* workspace, int64_t workspace_bytes,
                                void* stream) {
  clear_error();
  MB_CHECK_ARG(rows >= 0 && n > 0, "mb_count_columns: packed.original_shape must have non-empty last dimension");
  MB_CHECK_ARG(counts64 != nullptr || counts32 != nullptr, "mb_count_columns: no output");
  MB_CHECK_ARG(aligned_to(counts64, 8) && aligned_to(counts32, 4),
               "mb_count_columns: counts misaligned");
  cudaStream_t s = as_stream(stream);
  if (rows == 0) {
    if (counts64) cudaMemsetAsync(counts64, 0, n * sizeof(int64_t), s);
    if (counts32) cudaMemsetAsync(counts32, 0, n * sizeof(int32_t), s);
    MB_CHECK_LAUNCH("mb_count_columns");
    return 0;
  }
  MB_CHECK_ARG(words != nullptr, "mb_count_columns: null words");
  const int64_t need = count_columns_workspace_bytes(rows, n);
  MB_CHECK_ARG(workspace != nullptr && workspace_bytes >= need,
               "mb_count_columns: workspace of %lld bytes required, got %lld", (long long)need,
               (long long)workspace_bytes);
  MB_CHECK_ARG(aligned_to(workspace, 4), "mb_count_columns: workspace misaligned");
  launch_count_columns(words, rows, n, counts64, counts32, static_cast<int32_t*>(workspace), s);
  MB_CHECK_LAUNCH("mb_count_columns");
  return 0;
}

extern "C" int64_t mb_pack_count_workspace_bytes(int64_t rows, int64_t n) {
  return pack_count_workspace_bytes(rows, n);
}

extern "C" int mb_pack_count_spikes(int dtype, const void* spikes, int32_t* words, int64_t rows,
                                    int64_t n, int64_t* counts64, int32_t* counts32,
                                    void* workspace, int64_t workspace_bytes, void* stream) {
  clear_error();
  MB_CHECK_ARG(valid_io_dtype(dtype), "mb_pack_count_spikes: unknown dtype %d", dtype);
  MB_CHECK_ARG(rows >= 0 && n > 0, "mb_pack_count_spikes: cannot pack an empty last dimension");
  MB_CHECK_ARG(counts64 != nullptr || counts32 != nullptr, "mb_pack_count_spikes: no output");
  MB_CHECK_ARG(aligned_to(counts64, 8) && aligned_to(counts32, 4),
               "mb_pack_count_spikes: counts misaligned");
  cudaStream_t s = as_stream(stream);
  if (rows == 0) {
    if (counts64) cudaMemsetAsync(counts64, 0, n * sizeof(int64_t), s);
    if (counts32) cudaMemsetAsync(counts32, 0, n * sizeof(int32_t), s);
    MB_CHECK_LAUNCH("mb_pack_count_spikes");
    return 0;
  }
  MB_CHECK_ARG(spikes != nullptr && words != nullptr, "mb_pack_count_spikes: null pointer");
  const int64_t need = pack_count_workspace_bytes(rows, n);
  MB_CHECK_ARG(workspace != nullptr && workspace_bytes >= need,
               "mb_pack_count_spikes: workspace of %lld bytes required, got %lld",
               (long long)need, (long long)workspace_bytes);
  MB_CHECK_ARG(aligned_to(workspace, 4), "mb_pack_count_spikes: workspace misaligned");
  MB_DISPATCH_DTYPE(dtype, launch_pack_count, spikes, words, rows, n, counts64, counts32,
                    workspace, s);
  MB_CHECK_LAUNCH("mb_pack_count_spikes");
  return 0;
}

extern "C" int mb_pack_count_scatter(int dtype, const void* spikes, int32_t* words,
                                     int64_t rows, int64_t n, void* const* peers, int num_peers,
                                     int64_t* counts64, int32_t* counts32, void* workspace,
                                     int64_t workspace_bytes, void* stream) {
  clear_error();
  MB_CHECK_ARG(valid_io_dtype(dtype), "mb_pack_count_scatter: unknown dtype %d", dtype);
  MB_CHECK_ARG(rows >= 0 && n > 0, "mb_pack_count_scatter: cannot pack an empty last dimension");
  MB_CHECK_ARG(counts64 != nullptr || counts32 != nullptr, "mb_pack_count_scatter: no output");
  MB_CHECK_ARG(aligned_to(counts64, 8) && aligned_to(counts32, 4),
               "mb_pack_count_scatter: counts misaligned");
  MB_CHECK_ARG(words != nullptr && aligned_to(words, 4),
               "mb_pack_count_scatter: words null or misaligned");
  MB_CHECK_ARG(num_peers >= 0 && num_peers <= kMaxPeerSlots && (num_peers == 0 || peers),
               "mb_pack_count_scatter: 0 to %d peer slots required", kMaxPeerSlots);
  for (int d = 0; d < num_peers; ++d) {
    MB_CHECK_ARG(peers[d] != nullptr && aligned_to(peers[d], 4),
                 "mb_pack_count_scatter: peer slot %d null or misaligned", d);
  }
  cudaStream_t s = as_stream(stream);
  if (rows == 0) {
    if (counts64) cudaMemsetAsync(counts64, 0, n * sizeof(int64_t), s);
    if (counts32) cudaMemsetAsync(counts32, 0, n * sizeof(int32_t), s);
    MB_CHECK_LAUNCH("mb_pack_count_scatter");
    return 0;
  }
  MB_CHECK_ARG(spikes != nullptr, "mb_pack_count_scatter: null spikes");
  const int64_t need = pack_count_workspace_bytes(rows, n);
  MB_CHECK_ARG(workspace != nullptr && workspace_bytes >= need,
               "mb_pack_count_scatter: workspace of %lld bytes required, got %lld",
               (long long)need, (long long)workspace_bytes);
  MB_CHECK_ARG(aligned_to(workspace, 4), "mb_pack_count_scatter: workspace misaligned");
  if (pack_count_fused_ok(dtype, spikes, n) && pack_count_rows_ok(n, words, peers, num_peers)) {
    // whole rows per block: each group of rows goes to every slot as one bulk copy
    launch_pack_count_rows(spikes, words, peers, num_peers, rows, n, counts64, counts32, s);
  } else if (pack_count_fused_ok(dtype, spikes, n)) {
    PeerSlots slots{};
    for (int d = 0; d < num_peers; ++d) slots.p[d] = static_cast<uint32_t*>(peers[d]);
    launch_pack_count_u8(spikes, words, slots, num_peers, rows, n, counts64, counts32, s);
  } else {
    // other shapes: pack + count into `words`, then one kernel stores them
    // into every peer slot (over NVLink)
    MB_DISPATCH_DTYPE(dtype, launch_pack_count, spikes, words, rows, n, counts64, counts32,
                      workspace, s);
    push_to_peers(words, peers, num_peers,
                  size_t(rows) * size_t(ceil_div(n, 32)) * sizeof(int32_t), s);
  }
  MB_CHECK_LAUNCH("mb_pack_count_scatter");
  return 0;
}

// ---------------------------------------------------------------------------
// Column counts without any allocation.
//
// Some callers cannot allocate device memory at the point where they need a
// count: code running under a host runtime that owns every byte of device
// memory through its own fixed arena (and forbids other allocations), or a
// latency-critical loop where an allocation call would block on the device.
// For them the column count's per-slice partial sums live in this file-scope
// device array instead of a caller-provided workspace. The array is part of
// the library's device image: every GPU that loads the library holds it until
// the process exits.
//
// Every call shares the one array and overwrites it. Each partial sum is
// written before it is read within the same call, so nothing has to start at
// zero and stale contents from an earlier call are never used. Two calls
// whose kernels overlap on the GPU (different streams, or different host
// threads on the same device) race on the array and give wrong counts: keep
// such calls ordered on one stream.
// ---------------------------------------------------------------------------
namespace mb {

constexpr int64_t kNoAllocScratchBytes = MB_COUNT_COLUMNS_NOALLOC_MAX_BYTES;
static __device__ __align__(256) int32_t g_count_columns_scratch[kNoAllocScratchBytes / 4];

constexpr int kMaxDevices = 64;
static int32_t* g_scratch_ptr[kMaxDevices] = {nullptr};
static std::mutex g_scratch_mutex;

// Device address of the scratch array on the current device, looked up once
// per device (the host-side name of a __device__ array is not a device
// address). Returns nullptr and sets the error message on failure.
static int32_t* noalloc_scratch_for_current_device() {
  int dev = -1;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_error("mb_count_columns_noalloc: cannot query the current device (%s)",
              err != cudaSuccess ? cudaGetErrorString(err) : "device index out of range");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_count_columns_scratch);
    if (err != cudaSuccess || p == nullptr) {
      set_error("mb_count_columns_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
                cudaGetErrorString(err));
      return nullptr;
    }
    g_scratch_ptr[dev] = static_cast<int32_t*>(p);
  }
  return g_scratch_ptr[dev];
}

}  // namespace mb

extern "C" int mb_count_columns_noalloc(const int32_t* words, int64_t rows, int64_t n,
                                        int64_t* counts64, int32_t* counts32, void* stream) {
  clear_error();
  MB_CHECK_ARG(rows >= 0 && n > 0,
               "mb_count_columns_noalloc: packed.original_shape must have non-empty last dimension");
  MB_CHECK_ARG(counts64 != nullptr || counts32 != nullptr, "mb_count_columns_noalloc: no output");
  MB_CHECK_ARG(rows == 0 || words != nullptr, "mb_count_columns_noalloc: null words");
  MB_CHECK_ARG(aligned_to(counts64, 8) && aligned_to(counts32, 4),
               "mb_count_columns_noalloc: counts misaligned");
  // every row slice holds n partial sums of 4 bytes: reject an n whose single
  // slice already exceeds the scratch before the size product can overflow
  MB_CHECK_ARG(rows == 0 || n <= kNoAllocScratchBytes / 4,
               "mb_count_columns_noalloc: n = %lld needs more scratch than the built-in %lld "
               "bytes; use mb_count_columns with a caller-provided workspace",
               (long long)n, (long long)kNoAllocScratchBytes);
  const int64_t need = count_columns_workspace_bytes(rows, n);
  MB_CHECK_ARG(need <= kNoAllocScratchBytes,
               "mb_count_columns_noalloc: this shape needs %lld bytes of scratch, more than the "
               "built-in %lld; use mb_count_columns with a caller-provided workspace",
               (long long)need, (long long)kNoAllocScratchBytes);
  cudaStream_t s = as_stream(stream);
  if (rows == 0) {
    if (counts64) cudaMemsetAsync(counts64, 0, n * sizeof(int64_t), s);
    if (counts32) cudaMemsetAsync(counts32, 0, n * sizeof(int32_t), s);
    MB_CHECK_LAUNCH("mb_count_columns_noalloc");
    return 0;
  }
  int32_t* scratch = noalloc_scratch_for_current_device();
  if (scratch == nullptr) return 3;
  launch_count_columns(words, rows, n, counts64, counts32, scratch, s);
  MB_CHECK_LAUNCH("mb_count_columns_noalloc");
  return 0;
}
