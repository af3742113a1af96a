// Dense projection GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
//   C[M, N] = A[M, K] * B[N, K]^T (+ bias[N]),   A, B bf16 or f16 (K contiguous),
//   fp32 accumulation in tensor memory, C written as fp32 or the input type.
//
// This is the stream-synapse projection of the spiking layers: currents of all
// time steps at once, x[T*B, F] * W^T, feeding the scan; and the input
// gradient G[T*B, N] * W[F, N]^T of the backward.
//
// One persistent CTA per SM, 6 warps:
//   warp 0    copy engine driver: 2-D tiled bulk tensor copies (TMA) of A and
//             B K-slices into a 4-stage shared-memory ring (128-byte swizzle);
//   warp 1    allocates 2*BN TMEM columns and issues tcgen05.mma (one thread),
//             M=128 x N=BN x K=16 per instruction, committing each stage back
//             to the producer and each finished tile to the epilogue;
//   warps 2-5 epilogue: tcgen05.ld of the accumulator (each warp reads its own
//             32-lane quarter of TMEM), bias add, conversion, global stores.
// Two TMEM accumulators let the epilogue of one tile overlap the MMAs of the
// next. Every mbarrier wait is bounded. Large problems (M, N >= 256, enough
// tiles for every SM pair) run the two-SM variant, gemm_tn_pair_kernel, below.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "async_copy.cuh"
#include "common.cuh"
#include "tma.cuh"

namespace mb {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 64;  // one 128-byte swizzle row of 16-bit elements
constexpr int kStages = 4;
constexpr int kThreads = 192;
constexpr int kUmmaK = 16;

// Up to this many (A part, B part) products summed into one accumulator.
constexpr int kMaxSegments = 6;

struct GemmArgs {
  const void* bias;
  void* C;
  int64_t ldc;
  int64_t M, N, K;
  int bias_dtype;  // MB_F32 / MB_BF16 / MB_F16
  int vec_ok;      // C rows 16-byte aligned: 16-byte stores
  int tma_store;   // write C through smem + bulk tensor stores (tma_c valid)
  // C = sum over segments q of A[seg_a[q]] * B[seg_b[q]]^T: the K loop runs
  // over every enabled segment in turn. Segment q > 0 is skipped when a_nonzero
  // or b_nonzero (device flags, one int per part, nullable) says its A or B
  // part is all zeros; segment 0 always runs.
  int nseg;
  int8_t seg_a[kMaxSegments];
  int8_t seg_b[kMaxSegments];
  const int32_t* a_nonzero;
  const int32_t* b_nonzero;
  // Split K: each output tile is computed as k_slices independent partial
  // sums (k-blocks [s * kb_per_slice, (s + 1) * kb_per_slice) for slice s),
  // written as fp32 to slice s of C = a [k_slices, M, ldc] workspace (no
  // bias); a second kernel sums the slices in order. k_slices == 1: plain.
  // Work unit u is tile u % tiles of slice u / tiles: the units running at
  // once share one slice's rows of both operands, which stay in L2.
  int k_slices;
  int kb_per_slice;
  // Tail slicing (two-SM kernel, long K): units [0, full_units) are whole
  // tiles 0 .. full_units-1, written to C; the remaining tiles (the last,
  // partial wave) run as k_slices slices each, unit full_units + v being
  // slice v / tail_tiles of tile full_units + v % tail_tiles, written as fp32
  // partial sums through the second output map (a [k_slices, M - p_row0,
  // ldp] workspace holding rows p_row0 .. M-1); a second kernel adds them into
  // C. full_units == 0: the plain scheme above.
  int64_t full_units;
  int64_t p_row0;
};

// One work unit: its tile, K range and where its result goes.
struct WorkUnit {
  int64_t tile;
  int slice;
  int kb0, kb1;
  bool partial;  // a slice of a tail tile (tail slicing): fp32 to the workspace
};

__device__ __forceinline__ int64_t unit_count(const GemmArgs& a, int64_t tiles) {
  return a.full_units + (tiles - a.full_units) * a.k_slices;
}

__device__ __forceinline__ WorkUnit decode_unit(const GemmArgs& a, int64_t unit, int64_t tiles,
                                                int kblocks) {
  WorkUnit w;
  const int64_t v = unit - a.full_units;
  if (v < 0) {  // a whole tile of the full waves
    w.tile = unit;
    w.slice = 0;
    w.kb0 = 0;
    w.kb1 = kblocks;
    w.partial = false;
    return w;
  }
  const int64_t tail = tiles - a.full_units;
  w.tile = a.full_units + v % tail;
  w.slice = static_cast<int>(v / tail);
  w.kb0 = w.slice * a.kb_per_slice;
  w.kb1 = min(kblocks, w.kb0 + a.kb_per_slice);
  w.partial = a.full_units > 0;
  return w;
}

// Which segments this launch runs (bit q = segment q); read once per thread
// that walks the K loop, so the copy and MMA threads agree.
__device__ __forceinline__ uint32_t segment_mask(const GemmArgs& a) {
  uint32_t m = 1u;
  for (int q = 1; q < a.nseg; ++q) {
    const bool on = (a.a_nonzero == nullptr || __ldg(a.a_nonzero + a.seg_a[q]) != 0) &&
                    (a.b_nonzero == nullptr || __ldg(a.b_nonzero + a.seg_b[q]) != 0);
    m |= on ? (1u << q) : 0u;
  }
  return m;
}

template <int BN>
struct Layout {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarrierBytes = 256;
  // epilogue staging: 4 warps x 2 slots x (32 rows x 32 columns x up to 4 B)
  static constexpr int kEpiSlotBytes = 32 * 32 * 4;
  static constexpr int kEpiBytes = 4 * 2 * kEpiSlotBytes;
  static constexpr size_t kSmem =
      size_t(kStages) * kStageBytes + kEpiBytes + kBarrierBytes + 1024;
  static constexpr uint32_t kTmemCols = 2 * BN;  // two accumulators
};

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int c0,
                                             int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(src))
      : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0,
                                             int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(c0), "r"(c1), "r"(smem_addr(src))
      : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N of this thread's bulk stores still read shared memory.
template <int N>
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void tma_store_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// 3-D tiled loads: {inner, outer, part} coordinates over an operand stored as
// [parts, outer, ld] (the part dimension has extent 1 for plain operands).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar))
      : "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of
// 128 bytes, 8-row groups 1024 bytes apart (the layout the TMA copy writes).
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3fffu);  // start address
  d |= uint64_t(1) << 16;                  // leading byte offset (16 B; unused for this layout)
  d |= uint64_t(1024 >> 4) << 32;          // stride byte offset: 8 rows x 128 B
  d |= uint64_t(1) << 46;                  // descriptor version
  d |= uint64_t(2) << 61;                  // 128-byte swizzle
  return d;
}

// Bytes of one MN-major swizzle block in shared memory: 64 MN-elements
// (128 B) x kBK K-rows, as one TMA box writes it.
constexpr uint32_t kMnBlockBytes = 128 * kBK;

// Shared-memory matrix descriptor: MN-major operand (the M or N index is the
// contiguous one), 128-byte swizzle. A K-row holds 64 consecutive M/N
// elements (128 B); 8 K-rows form one 1024-byte swizzle atom (stride byte
// offset); the next 64 M/N elements start kMnBlockBytes further on (leading
// byte offset), the next TMA box.
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3fffu);       // start address
  d |= uint64_t(kMnBlockBytes >> 4) << 16;      // leading byte offset: next 64 M/N elements
  d |= uint64_t(1024 >> 4) << 32;               // stride byte offset: next 8 K-rows
  d |= uint64_t(1) << 46;                       // descriptor version
  d |= uint64_t(2) << 61;                       // 128-byte swizzle
  return d;
}

// Descriptor of the k-th 16-deep K step of a staged operand tile.
template <bool MN>
__device__ __forceinline__ uint64_t operand_desc(uint32_t base, int k) {
  if constexpr (MN) {
    return sw128_mnmajor_desc(base + uint32_t(k) * kUmmaK * 128);  // 16 K-rows of 128 B
  } else {
    return sw128_kmajor_desc(base + uint32_t(k) * kUmmaK * 2);  // 16 elements along a row
  }
}

// Stage one operand tile (ROWS M/N-elements x kBK K-elements of part `part`)
// into shared memory: one box of kBK x ROWS for a K-major operand, ROWS/64
// boxes of 64 x kBK (kMnBlockBytes apart) for an MN-major one.
template <bool MN, int ROWS>
__device__ __forceinline__ void load_operand(uint8_t* dst, const CUtensorMap* map, int64_t mn0,
                                             int kb, int part, uint64_t* bar) {
  if constexpr (MN) {
#pragma unroll
    for (int j = 0; j < ROWS / 64; ++j) {
      tma_load_3d(dst + j * kMnBlockBytes, map, static_cast<int>(mn0) + 64 * j, kb * kBK, part,
                  bar);
    }
  } else {
    tma_load_3d(dst, map, kb * kBK, static_cast<int>(mn0), part, bar);
  }
}

// Instruction descriptor of kind::f16: fp32 accumulate, A/B type, A/B major.
template <typename TIn, int BN, bool A_MN = false, bool B_MN = false>
__device__ __forceinline__ uint32_t mma_idesc() {
  constexpr uint32_t ab = std::is_same<TIn, __nv_bfloat16>::value ? 1u : 0u;
  return (1u << 4)            // D = F32
         | (ab << 7)          // A format
         | (ab << 10)         // B format
         | (uint32_t(A_MN) << 15)  // A MN-major
         | (uint32_t(B_MN) << 16)  // B MN-major
         | (uint32_t(BN >> 3) << 17)
         | (uint32_t(kBM >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Arrive on `bar` once every MMA issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Issue a 32-column TMEM load of this warp's 32 lanes; complete it with tmem_wait_ld().
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// The bias of a warp's NC 32-column chunks starting at column j0, one column
// per lane per chunk (lane l holds column j0 + 32 c + l in bcol[c]; zero past
// N or without bias). Loaded before the warp waits for its accumulator, so the
// load latency overlaps the wait; the epilogue broadcasts each value across
// the warp with shuffles.
template <int NC>
__device__ __forceinline__ void load_bias_cols(const GemmArgs& args, int64_t j0, int lane,
                                               float (&bcol)[NC]) {
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int64_t j = j0 + 32 * c + lane;
    float v = 0.0f;
    if (args.bias != nullptr && j < args.N) {
      if (args.bias_dtype == MB_F32) v = __ldg(static_cast<const float*>(args.bias) + j);
      else if (args.bias_dtype == MB_BF16) v = __bfloat162float(static_cast<const __nv_bfloat16*>(args.bias)[j]);
      else v = __half2float(static_cast<const __half*>(args.bias)[j]);
    }
    bcol[c] = v;
  }
}

template <typename TOut>
__device__ __forceinline__ void store_row32(TOut* dst, const float (&v)[32], int valid,
                                            bool vec_ok) {
  if (vec_ok && valid == 32) {
    if constexpr (std::is_same<TOut, float>::value) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        reinterpret_cast<float4*>(dst)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      }
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t w[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float a = v[8 * q + 2 * h], b = v[8 * q + 2 * h + 1];
          if constexpr (std::is_same<TOut, __nv_bfloat16>::value) {
            const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
            w[h] = *reinterpret_cast<const uint32_t*>(&p);
          } else {
            const __half2 p = __floats2half2_rn(a, b);
            w[h] = *reinterpret_cast<const uint32_t*>(&p);
          }
        }
        reinterpret_cast<uint4*>(dst)[q] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
    return;
  }
  // unrolled with a predicate per element: a loop bounded by `valid` would
  // index v at run time and move it (and every chunk's values) to local memory
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (j < valid) {
      if constexpr (std::is_same<TOut, float>::value) dst[j] = v[j];
      else if constexpr (std::is_same<TOut, __nv_bfloat16>::value) dst[j] = __float2bfloat16_rn(v[j]);
      else dst[j] = __float2half_rn(v[j]);
    }
  }
}

// One lane's 32 values of output row r (a 32-column chunk) into a staging slot
// of 32 rows x 128 bytes laid out as the bulk tensor store expects with the
// 128-byte swizzle: 16-byte chunk q of row r sits at chunk q ^ (r & 7), so the
// 32 lanes of a warp writing their rows hit distinct banks. fp32 chunks fill a
// row; 16-bit chunks fill half `h` of it (two chunks per store, so every
// store writes whole 128-byte lines).
template <typename TOut>
__device__ __forceinline__ void stage_row32(uint8_t* slot, int r, int h, const float (&v)[32]) {
  if constexpr (std::is_same<TOut, float>::value) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int pq = q ^ (r & 7);
      *reinterpret_cast<float4*>(slot + r * 128 + pq * 16) =
          make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float a = v[8 * q + 2 * e], b = v[8 * q + 2 * e + 1];
        if constexpr (std::is_same<TOut, __nv_bfloat16>::value) {
          const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
          w[e] = *reinterpret_cast<const uint32_t*>(&p);
        } else {
          const __half2 p = __floats2half2_rn(a, b);
          w[e] = *reinterpret_cast<const uint32_t*>(&p);
        }
      }
      const int pq = (4 * h + q) ^ (r & 7);
      *reinterpret_cast<uint4*>(slot + r * 128 + pq * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

// Epilogue of one tile for one warp: its 32 accumulator rows (TMEM lanes
// taddr's quarter, columns b*BN ..) -> bias add in fp32 (bcol from
// load_bias_cols) -> one rounding to TOut
// -> global memory, either staged in swizzled shared memory and written with
// bulk tensor stores of 32 rows x 128 bytes (tma_store: one store per 32 fp32
// or 64 16-bit columns) or with direct row stores. TMEM loads are
// double-buffered: chunk ci+1 loads while chunk ci is converted. With split K
// (args.k_slices > 1, fp32 only) the tile goes to slice `slice` of the fp32
// workspace (a 3-D tensor map over [k_slices, M, ldc]).
// Where a drained tile goes: `map` (2-D over C, or 3-D over a slices
// workspace when `sliced`, with tile row r stored at row r - row_base of the
// slice); `bias`: add the bias columns.
struct DrainTarget {
  const CUtensorMap* map;
  bool sliced;
  bool bias;
  int64_t row_base;
};

template <typename TOut, int BN, int WARP_STAGE_BYTES = 2 * 32 * 32 * 4>
__device__ __forceinline__ void drain_tile(uint32_t tbase, int64_t row0, int64_t col_tile0,
                                           int lane, const GemmArgs& args,
                                           const float (&bcol)[BN / 32], const DrainTarget& tgt,
                                           uint8_t* slots, uint32_t& nstore, int slice) {
  constexpr int kPerStore = sizeof(TOut) == 4 ? 1 : 2;  // 32-column chunks per store
  constexpr int kSlotBytes = 32 * 128;
  constexpr int kSlots = WARP_STAGE_BYTES / kSlotBytes;  // staging slots of this warp
  static_assert(kSlots >= 1 && (BN / 32) % kPerStore == 0, "epilogue staging layout");
  const bool has_bias = tgt.bias;
  const bool vec_ok = args.vec_ok != 0;
  const bool use_tma = args.tma_store != 0;
  const int64_t row = row0 + lane;
  const bool sliced = tgt.sliced;
  const CUtensorMap* tma_c = tgt.map;
  const int store_row0 = static_cast<int>(row0 - tgt.row_base);
  TOut* crow = static_cast<TOut*>(args.C) + (row + (sliced ? slice * args.M : 0)) * args.ldc;
  uint32_t r[2][32];
  uint8_t* slot = slots;
  tmem_ld32_issue(tbase, r[0]);
#pragma unroll
  for (int ci = 0; ci < BN / 32; ++ci) {
    const int c = ci * 32;
    tmem_wait_ld();  // chunk ci has landed
    if (ci + 1 < BN / 32) tmem_ld32_issue(tbase + c + 32, r[(ci + 1) & 1]);  // overlap the next
    const uint32_t(&rc)[32] = r[ci & 1];
    const int64_t col0 = col_tile0 + c;
    const int64_t store_col0 = col_tile0 + (ci / kPerStore) * kPerStore * 32;
    if (store_col0 >= args.N || row0 >= args.M) continue;  // warp-uniform
    const int valid = col0 < args.N ? static_cast<int>(imin64(32, args.N - col0)) : 0;
    float v[32];
    if (has_bias) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(rc[j]) + __shfl_sync(0xffffffffu, bcol[ci], j);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(rc[j]);
    }
    if (use_tma) {
      const int part = ci % kPerStore;
      if (part == 0) {
        // the slot used kSlots stores ago must have been read out
        if (lane == 0) tma_store_wait_read<kSlots - 1>();
        __syncwarp();
        slot = slots + (nstore % kSlots) * kSlotBytes;
      }
      // columns past N are staged too; the store does not write them
      stage_row32<TOut>(slot, lane, part, v);
      if (part == kPerStore - 1) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (sliced) tma_store_3d(tma_c, slot, static_cast<int>(store_col0), store_row0, slice);
          else tma_store_2d(tma_c, slot, static_cast<int>(store_col0), store_row0);
        }
        ++nstore;
      }
    } else if (row < args.M && valid > 0) {
      store_row32<TOut>(crow + col0, v, valid, vec_ok);
    }
  }
}

template <typename TIn, typename TOut, int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tn_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
                   const __grid_constant__ CUtensorMap tma_c, const __grid_constant__ GemmArgs args) {
  using L = Layout<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + kStages * L::kABytes;
  uint8_t* sepi = sb + kStages * L::kBBytes;  // epilogue staging slots (1 KB aligned)
  uint64_t* full = reinterpret_cast<uint64_t*>(sepi + L::kEpiBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint64_t* drained = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t m_tiles = (args.M + kBM - 1) / kBM;
  const int64_t n_tiles = (args.N + BN - 1) / BN;
  const int64_t tiles = m_tiles * n_tiles;
  const int64_t units = unit_count(args, tiles);  // (tile, K slice) work units
  const int kblocks = static_cast<int>((args.K + kBK - 1) / kBK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    mbar_init(drained, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(L::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      const uint32_t segs = segment_mask(args);
      for (int64_t unit = blockIdx.x; unit < units && ok; unit += gridDim.x) {
        const WorkUnit wu = decode_unit(args, unit, tiles, kblocks);
        const int64_t tile = wu.tile;
        const int kb0 = wu.kb0, kb1 = wu.kb1;
        const int64_t tm = tile / n_tiles;
        const int64_t tn = tile % n_tiles;
        // smallest products first: they are summed while the accumulator is small
        for (int q = args.nseg - 1; q >= 0 && ok; --q) {
          if (((segs >> q) & 1u) == 0) continue;
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s = static_cast<int>(it % kStages);
            const uint32_t use = it / kStages;
            if (use > 0 && !mbar_wait_bounded(&empty[s], (use - 1) & 1)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&full[s], L::kStageBytes);
            load_operand<A_MN, kBM>(sa + s * L::kABytes, &tma_a, tm * kBM, kb, args.seg_a[q],
                                    &full[s]);
            load_operand<B_MN, BN>(sb + s * L::kBBytes, &tma_b, tn * BN, kb, args.seg_b[q],
                                   &full[s]);
          }
        }
      }
      // every issued copy has landed before the CTA can retire; a wait that
      // runs out is already recorded in the status word, and the remaining
      // waits still run (each bounded) so that no copy is left in flight
      const uint32_t issued = it;
      for (uint32_t j = issued > kStages ? issued - kStages : 0; j < issued; ++j) {
        (void)mbar_wait_bounded(&full[j % kStages], (j / kStages) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = mma_idesc<TIn, BN, A_MN, B_MN>();
      const uint32_t segs = segment_mask(args);
      uint32_t it = 0, local = 0;
      bool ok = true;
      for (int64_t unit = blockIdx.x; unit < units && ok; unit += gridDim.x, ++local) {
        const WorkUnit wu = decode_unit(args, unit, tiles, kblocks);
        const int kb0 = wu.kb0, kb1 = wu.kb1;
        const uint32_t b = local & 1;
        const uint32_t use_b = local >> 1;
        if (use_b > 0 && !mbar_wait_bounded(&acc_empty[b], (use_b - 1) & 1)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * BN;
        bool acc = false;  // the tile's first MMA overwrites the accumulator
        for (int q = args.nseg - 1; q >= 0 && ok; --q) {
          if (((segs >> q) & 1u) == 0) continue;
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s = static_cast<int>(it % kStages);
            if (!mbar_wait_bounded(&full[s], (it / kStages) & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_addr(sa + s * L::kABytes);
            const uint32_t b0 = smem_addr(sb + s * L::kBBytes);
#pragma unroll
            for (int k = 0; k < kBK / kUmmaK; ++k) {
              mma_f16(d_tmem, operand_desc<A_MN>(a0, k), operand_desc<B_MN>(b0, k), idesc,
                      (acc || k != 0) ? 1u : 0u);
            }
            acc = true;
            mma_commit(&empty[s]);  // the stage is free once these MMAs finish
          }
        }
        if (ok) mma_commit(&acc_full[b]);  // the tile's accumulator is complete
      }
      // all issued MMAs have finished before TMEM is released (a timeout is
      // recorded in the status word; the exit path is the same either way)
      mma_commit(drained);
      (void)mbar_wait_bounded(drained, 0);
    }
  } else {
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const bool use_tma = args.tma_store != 0;
    uint8_t* slots = sepi + (warp - 2) * 2 * L::kEpiSlotBytes;
    uint32_t nstore = 0;
    uint32_t local = 0;
    for (int64_t unit = blockIdx.x; unit < units; unit += gridDim.x, ++local) {
      const uint32_t b = local & 1;
      const WorkUnit wu = decode_unit(args, unit, tiles, kblocks);
      const int64_t tm = wu.tile / n_tiles;
      const int64_t tn = wu.tile % n_tiles;
      float bcol[BN / 32];
      load_bias_cols(args, tn * BN, lane, bcol);
      if (!mbar_wait_bounded(&acc_full[b], (local >> 1) & 1)) break;
      tc_fence_after();
      const DrainTarget tgt{&tma_c, args.k_slices > 1, args.bias != nullptr, 0};
      drain_tile<TOut, BN>(tmem_base + (uint32_t(quarter * 32) << 16) + b * BN,
                           tm * kBM + quarter * 32, tn * BN, lane, args, bcol, tgt, slots,
                           nstore, wu.slice);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
    if (use_tma && lane == 0) tma_store_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(L::kTmemCols));
  }
}


// ---------------------------------------------------------------------------
// Two-SM variant: a cluster of 2 CTAs (on 2 SMs) computes a 256 x 256 tile
// with tcgen05.mma.cta_group::2 (M = 256, N = 256 per instruction). CTA r of
// the pair loads rows [128 r, 128 r + 128) of the A tile and of the B tile
// (32 KB per stage instead of 48 KB per 128 x 256 tile on one SM: half the
// operand traffic per SM) and holds its 128 rows x 256 columns of the
// accumulator in its own TMEM. The pair's leader (rank 0):
//   - arms its "full" barrier with both CTAs' bytes; both CTAs' TMA loads
//     (the .cta_group::2 form) complete on the leader's barrier;
//   - issues the MMAs from one thread and commits stage release and tile
//     completion to the barriers of both CTAs (one commit per CTA);
//   - waits on its "acc_empty" barrier, which the epilogue warps of both
//     CTAs arrive on through cluster addresses.
// Each CTA drains its accumulator with 8 epilogue warps (two per TMEM lane
// quarter, 128 columns each), so draining a tile keeps up with its MMAs even
// at small K.
// Every wait is bounded; no thread leaves early (failed waits fall through),
// and a cluster barrier before TMEM release keeps both CTAs alive until
// neither can touch the other's shared memory.
// ---------------------------------------------------------------------------
constexpr int k2Stages = 6;
constexpr int k2EpiWarps = 8;  // two per TMEM lane quarter, 128 columns each
constexpr int k2Threads = 64 + 32 * k2EpiWarps;
constexpr int k2BM = 256;  // rows per pair tile (128 per CTA)
constexpr int k2BN = 256;  // columns per pair tile (B rows: 128 per CTA)

struct Layout2 {
  static constexpr int kABytes = 128 * kBK * 2;  // this CTA's A rows
  static constexpr int kBBytes = 128 * kBK * 2;  // this CTA's B rows
  static constexpr int kStageBytes = kABytes + kBBytes;
  // epilogue staging per warp: one block of 32 rows x 128 bytes
  static constexpr int kEpiWarpBytes = 32 * 128;
  static constexpr int kEpiBytes = k2EpiWarps * kEpiWarpBytes;
  static constexpr int kBarrierBytes = 256;
  static constexpr size_t kSmem =
      size_t(k2Stages) * kStageBytes + kEpiBytes + kBarrierBytes + 1024;
  static constexpr uint32_t kTmemCols = 2 * k2BN;  // two accumulators
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address in the cluster's shared window of `local` (a shared::cta address)
// as seen in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// 3-D tiled load ({inner, outer, part}) into this CTA's shared memory whose
// completion bytes are counted on the barrier at cluster address
// `bar_cluster` (the leader's). Loads of this GPU's own memory only.
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, int c0, int c1,
                                                 int c2, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar_cluster)
      : "memory");
}

// load_operand for one CTA of the pair: its 128 M/N-elements of the tile.
template <bool MN>
__device__ __forceinline__ void load_operand_pair(uint8_t* dst, const CUtensorMap* map,
                                                  int64_t mn0, int kb, int part,
                                                  uint32_t bar_cluster) {
  if constexpr (MN) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      tma_load_3d_pair(dst + j * kMnBlockBytes, map, static_cast<int>(mn0) + 64 * j, kb * kBK,
                       part, bar_cluster);
    }
  } else {
    tma_load_3d_pair(dst, map, kb * kBK, static_cast<int>(mn0), part, bar_cluster);
  }
}

__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Arrive once on the barrier at shared offset `bar` in both CTAs of the pair
// (one multicast commit) when every pair MMA issued so far by this thread has
// completed.
__device__ __forceinline__ void mma_commit_pair_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_addr(bar)),
      "h"(static_cast<uint16_t>(0x3))
      : "memory");
}

// Arrive once on the barrier at cluster address `bar_cluster` when every
// pair MMA issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar_cluster)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster)
               : "memory");
}

template <typename TIn, bool A_MN, bool B_MN>
__device__ __forceinline__ uint32_t mma_idesc_pair() {
  constexpr uint32_t ab = std::is_same<TIn, __nv_bfloat16>::value ? 1u : 0u;
  return (1u << 4) | (ab << 7) | (ab << 10) | (uint32_t(A_MN) << 15) | (uint32_t(B_MN) << 16) |
         (uint32_t(k2BN >> 3) << 17) | (uint32_t(k2BM >> 4) << 24);
}

template <typename TIn, typename TOut, bool A_MN, bool B_MN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(k2Threads, 1)
    gemm_tn_pair_kernel(const __grid_constant__ CUtensorMap tma_a,
                        const __grid_constant__ CUtensorMap tma_b,
                        const __grid_constant__ CUtensorMap tma_c, const __grid_constant__ GemmArgs args,
                        const __grid_constant__ CUtensorMap tma_p) {
  using L = Layout2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + k2Stages * L::kABytes;
  uint8_t* sepi = sb + k2Stages * L::kBBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sepi + L::kEpiBytes);
  uint64_t* empty = full + k2Stages;
  uint64_t* acc_full = empty + k2Stages;  // [2]
  uint64_t* acc_empty = acc_full + 2;     // [2]
  uint64_t* drained = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int64_t pair = blockIdx.x >> 1;
  const int64_t pairs = gridDim.x >> 1;
  const int64_t m_tiles = (args.M + k2BM - 1) / k2BM;
  const int64_t n_tiles = (args.N + k2BN - 1) / k2BN;
  const int64_t tiles = m_tiles * n_tiles;
  const int64_t units = unit_count(args, tiles);  // (tile, K slice) work units
  const int kblocks = static_cast<int>((args.K + kBK - 1) / kBK);

  if (threadIdx.x == 0) {
    for (int s = 0; s < k2Stages; ++s) {
      mbar_init(&full[s], 1);   // the leader's arm (its expect_tx); peer's unused
      mbar_init(&empty[s], 1);  // one commit per use, from the leader's MMA thread
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);   // one commit per tile
      mbar_init(&acc_empty[b], 2 * k2EpiWarps);  // epilogue warps of both CTAs (leader's used)
    }
    mbar_init(drained, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(tmem_slot)),
                 "r"(L::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers initialised before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      const uint32_t segs = segment_mask(args);
      for (int64_t unit = pair; unit < units && ok; unit += pairs) {
        const WorkUnit wu = decode_unit(args, unit, tiles, kblocks);
        const int64_t tile = wu.tile;
        const int kb0 = wu.kb0, kb1 = wu.kb1;
        const int64_t tm = tile / n_tiles;
        const int64_t tn = tile % n_tiles;
        for (int q = args.nseg - 1; q >= 0 && ok; --q) {
          if (((segs >> q) & 1u) == 0) continue;
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s = static_cast<int>(it % k2Stages);
            const uint32_t use = it / k2Stages;
            if (use > 0 && !mbar_wait_bounded(&empty[s], (use - 1) & 1)) {
              ok = false;
              break;
            }
            const uint32_t bar = cluster_addr(smem_addr(&full[s]), 0);
            if (leader) mbar_arrive_expect_tx(&full[s], 2 * L::kStageBytes);
            load_operand_pair<A_MN>(sa + s * L::kABytes, &tma_a, tm * k2BM + int64_t(rank) * 128,
                                    kb, args.seg_a[q], bar);
            load_operand_pair<B_MN>(sb + s * L::kBBytes, &tma_b, tn * k2BN + int64_t(rank) * 128,
                                    kb, args.seg_b[q], bar);
          }
        }
      }
      if (leader) {
        // both CTAs' copies complete on the leader's barriers: once the last
        // phases have completed nothing is in flight into either CTA
        // (a wait that runs out is recorded; the rest still run, each bounded)
        const uint32_t issued = it;
        for (uint32_t j = issued > k2Stages ? issued - k2Stages : 0; j < issued; ++j) {
          (void)mbar_wait_bounded(&full[j % k2Stages], (j / k2Stages) & 1);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      const uint32_t idesc = mma_idesc_pair<TIn, A_MN, B_MN>();
      const uint32_t segs = segment_mask(args);
      uint32_t it = 0, local = 0;
      bool ok = true;
      for (int64_t unit = pair; unit < units && ok; unit += pairs, ++local) {
        const WorkUnit wu = decode_unit(args, unit, tiles, kblocks);
        const int kb0 = wu.kb0, kb1 = wu.kb1;
        const uint32_t b = local & 1;
        const uint32_t use_b = local >> 1;
        if (use_b > 0 && !mbar_wait_bounded(&acc_empty[b], (use_b - 1) & 1)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + b * k2BN;
        bool acc = false;  // the tile's first MMA overwrites the accumulator
        for (int q = args.nseg - 1; q >= 0 && ok; --q) {
          if (((segs >> q) & 1u) == 0) continue;
          for (int kb = kb0; kb < kb1; ++kb, ++it) {
            const int s = static_cast<int>(it % k2Stages);
            if (!mbar_wait_bounded(&full[s], (it / k2Stages) & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a0 = smem_addr(sa + s * L::kABytes);
            const uint32_t b0 = smem_addr(sb + s * L::kBBytes);
#pragma unroll
            for (int k = 0; k < kBK / kUmmaK; ++k) {
              mma_f16_pair(d_tmem, operand_desc<A_MN>(a0, k), operand_desc<B_MN>(b0, k), idesc,
                           (acc || k != 0) ? 1u : 0u);
            }
            acc = true;
            // the stage is free in both CTAs once these MMAs finish
            mma_commit_pair_both(&empty[s]);
          }
        }
        if (ok) mma_commit_pair_both(&acc_full[b]);  // both CTAs' accumulator halves are complete
      }
      mma_commit_pair(cluster_addr(smem_addr(drained), 0));
      // all MMAs done before TMEM is released (a timeout is recorded in the
      // status word; the exit path is the same either way)
      (void)mbar_wait_bounded(drained, 0);
    }
  } else {
    const int quarter = warp & 3;      // TMEM lanes this warp may access (warp id % 4)
    const int half = (warp - 2) >> 2;  // which 128 of the 256 columns it drains
    const bool use_tma = args.tma_store != 0;
    uint8_t* slots = sepi + (warp - 2) * L::kEpiWarpBytes;
    uint32_t nstore = 0;
    uint32_t local = 0;
    for (int64_t unit = pair; unit < units; unit += pairs, ++local) {
      const uint32_t b = local & 1;
      const WorkUnit wu = decode_unit(args, unit, tiles, kblocks);
      const int64_t tm = wu.tile / n_tiles;
      const int64_t tn = wu.tile % n_tiles;
      const int64_t col_tile0 = tn * k2BN + half * (k2BN / 2);
      const uint32_t taddr = tmem_base + (uint32_t(quarter * 32) << 16) + b * k2BN + half * (k2BN / 2);
      const int64_t row0 = tm * k2BM + int64_t(rank) * 128 + quarter * 32;
      float bcol[k2BN / 2 / 32];
      load_bias_cols(args, col_tile0, lane, bcol);
      if (!mbar_wait_bounded(&acc_full[b], (local >> 1) & 1)) break;
      tc_fence_after();
      if (wu.partial) {
        // a slice of a tail tile: fp32 partial sums to the workspace (no bias)
        const DrainTarget tgt{&tma_p, true, false, args.p_row0};
        drain_tile<float, k2BN / 2, L::kEpiWarpBytes>(taddr, row0, col_tile0, lane, args, bcol,
                                                      tgt, slots, nstore, wu.slice);
      } else {
        const DrainTarget tgt{&tma_c, args.k_slices > 1 && args.full_units == 0,
                              args.bias != nullptr, 0};
        drain_tile<TOut, k2BN / 2, L::kEpiWarpBytes>(taddr, row0, col_tile0, lane, args, bcol,
                                                     tgt, slots, nstore, wu.slice);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(cluster_addr(smem_addr(&acc_empty[b]), 0));
    }
    if (use_tma && lane == 0) tma_store_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA touches the other's shared memory or TMEM after this
  tc_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(L::kTmemCols));
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() { return tma_encode_fn(); }

// One GEMM operand in global memory: `parts` matrices of 16-bit elements, part
// p starting p * part_stride elements after `ptr`. K-major: rows of K
// contiguous elements, row r at r * ld; MN-major: K rows of M (or N)
// contiguous elements, row k at k * ld.
struct Operand {
  const void* ptr;
  int64_t ld;
  int64_t part_stride;
  int parts;
  bool mn_major;
};

// 3-D map {inner, outer, part} over an operand whose M/N extent is `mn`:
// K-major box 64 K-elements x box_rows rows, MN-major box 64 M/N-elements x
// kBK K-rows; 128-byte swizzle either way. Elements outside the operand
// (K and M/N tails) read as zero.
bool make_operand_map(CUtensorMap* map, const Operand& op, int64_t mn, int64_t k, int box_rows,
                      bool bf16) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const int64_t inner = op.mn_major ? mn : k;
  const int64_t outer = op.mn_major ? k : mn;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer),
                        static_cast<cuuint64_t>(op.parts)};
  const int64_t part_bytes = (op.parts > 1 ? op.part_stride : outer * op.ld) * 2;
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(op.ld * 2), static_cast<cuuint64_t>(part_bytes)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(kBK),
                       static_cast<cuuint32_t>(op.mn_major ? kBK : box_rows), 1};
  cuuint32_t estride[3] = {1, 1, 1};
  const CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        3, const_cast<void*>(op.ptr), dims, strides, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D map over C[M, N] (leading dimension ldc elements) for the epilogue's
// bulk tensor stores: boxes of 32 rows x 128 bytes (32 fp32 or 64 16-bit
// columns), 128-byte swizzle matching stage_row32.
bool make_c_map(CUtensorMap* map, void* ptr, int64_t M, int64_t N, int64_t ldc, int out_dtype) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  const int elt = out_dtype == MB_F32 ? 4 : 2;
  if (!aligned_to(ptr, 16) || (ldc * elt) % 16 != 0) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldc * elt)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / elt), 32};
  cuuint32_t estride[2] = {1, 1};
  const CUtensorMapDataType dt = out_dtype == MB_F32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : out_dtype == MB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = fn(map, dt, 2, ptr, dims, strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 3-D map over the split-K workspace [k_slices, M, ldc] of fp32 partial sums
// for the epilogue's bulk tensor stores (box 32 x 32 x 1, 128-byte swizzle).
bool make_slices_map(CUtensorMap* map, void* ptr, int64_t M, int64_t N, int64_t ldc, int slices) {
  auto fn = encode_fn();
  if (fn == nullptr) return false;
  if (!aligned_to(ptr, 16) || (ldc * 4) % 16 != 0) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(M),
                        static_cast<cuuint64_t>(slices)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(ldc * 4), static_cast<cuuint64_t>(M * ldc * 4)};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estride[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, ptr, dims, strides, box, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Sum of the split-K partial sums in slice order (+ bias), one rounding to TOut.
template <typename TOut>
__global__ void slices_reduce_kernel(const float* __restrict__ partial, int slices, int64_t M,
                                     int64_t N, int64_t pld, const void* bias, int bias_dtype,
                                     TOut* __restrict__ C, int64_t ldc) {
  const int64_t total = M * N;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t m = i / N;
    const int64_t n = i - m * N;
    float acc = 0.0f;
    for (int sl = 0; sl < slices; ++sl) acc += partial[(sl * M + m) * pld + n];
    if (bias != nullptr) {
      if (bias_dtype == MB_F32) acc += static_cast<const float*>(bias)[n];
      else if (bias_dtype == MB_BF16) acc += __bfloat162float(static_cast<const __nv_bfloat16*>(bias)[n]);
      else acc += __half2float(static_cast<const __half*>(bias)[n]);
    }
    C[m * ldc + n] = Elem<TOut>::from_f(acc);
  }
}

// The tail tiles of a tail-sliced launch: for every element of rows
// p_row0 .. M-1 whose tile index is >= full_units, the sum of its slices'
// partial sums in slice order (+ bias), one rounding to TOut. Elements of
// whole tiles in those rows are left as the GEMM wrote them.
template <typename TOut>
__global__ void tail_reduce_kernel(const float* __restrict__ partial, int slices, int64_t M,
                                   int64_t N, int64_t pld, int64_t p_row0, int64_t full_units,
                                   int64_t n_tiles, const void* bias, int bias_dtype,
                                   TOut* __restrict__ C, int64_t ldc) {
  const int64_t rows = M - p_row0;
  const int64_t total = rows * N;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / N;
    const int64_t n = i - r * N;
    const int64_t m = p_row0 + r;
    if ((m / k2BM) * n_tiles + n / k2BN < full_units) continue;
    float acc = 0.0f;
    for (int sl = 0; sl < slices; ++sl) acc += partial[(sl * rows + r) * pld + n];
    if (bias != nullptr) {
      if (bias_dtype == MB_F32) acc += static_cast<const float*>(bias)[n];
      else if (bias_dtype == MB_BF16) acc += __bfloat162float(static_cast<const __nv_bfloat16*>(bias)[n]);
      else acc += __half2float(static_cast<const __half*>(bias)[n]);
    }
    C[m * ldc + n] = Elem<TOut>::from_f(acc);
  }
}

int sm_count();

// K slices for a launch (each slice's partial sums go to an fp32 workspace and
// a second kernel adds them in order):
//  - accuracy: fp32 output from split (fp32) operands is summed in slices of
//    at most kSliceKBlocks k-blocks. The tensor cores' fp32 accumulation of
//    each MMA is not correctly rounded, so its error grows with the number of
//    MMAs summed into one accumulator; slices bound that count and are added
//    in fp32 (correctly rounded) afterwards;
//  - parallelism: when the output has too few tiles to occupy half of the SMs
//    and K is long (a weight gradient of a narrow or small layer: K = T * B),
//    K is split until the (tile, slice) units fill the SMs, each slice at
//    least kMinSliceKBlocks k-blocks long.
// (Long K with many tiles is handled by tail slicing, tail_plan below, from
// kWaveSliceKBlocks k-blocks on.)
constexpr int kSliceKBlocks = 32;     // K = 2048 per slice
constexpr int kMinSliceKBlocks = 8;   // K = 512
constexpr int kWaveSliceKBlocks = 128;  // K = 8192

int k_slices_for(int64_t M, int64_t N, int64_t K, int a_parts, int b_parts, int out_dtype,
                 bool occupancy, int* kb_per_slice) {
  const int kblocks = static_cast<int>((K + kBK - 1) / kBK);
  int slices = 1;
  if (out_dtype == MB_F32 && (a_parts > 1 || b_parts > 1) && kblocks > kSliceKBlocks) {
    slices = (kblocks + kSliceKBlocks - 1) / kSliceKBlocks;
  }
  const int bn = N >= 192 ? 256 : (N > 64 ? 128 : 64);
  const int64_t tiles = ((M + kBM - 1) / kBM) * ((N + bn - 1) / bn);
  const int sms = sm_count();
  if (occupancy && tiles * slices < sms / 2 && kblocks >= 2 * kMinSliceKBlocks) {
    const int64_t want = (sms + tiles - 1) / tiles;
    const int64_t most = kblocks / kMinSliceKBlocks;
    slices = static_cast<int>(std::max<int64_t>(slices, std::min(want, most)));
  }
  const int per = (kblocks + slices - 1) / slices;
  *kb_per_slice = per;
  return (kblocks + per - 1) / per;
}

int64_t slices_pld(int64_t N) { return (N + 3) / 4 * 4; }

// Tail slicing for long K on the two-SM kernel (a weight gradient, K = T * B):
// the whole waves of pair tiles run unsliced, and only the tiles of the last,
// partial wave are split into `slices` K slices (as many as fit one wave of
// pairs, at most 4), so that wave ends after 1/slices of a tile's time. (256
// pair tiles on 74 pairs: 3 whole waves of 74 tiles, then 34 tiles x 2
// slices; slicing every tile instead wrote and re-read fp32 partials of the
// whole output.) Their partial sums go to a workspace covering rows p_row0 ..
// M-1 of the output.
struct TailPlan {
  int64_t full_units = 0;
  int slices = 1;
  int kb_per_slice = 0;
  int64_t p_row0 = 0;
};

bool tail_plan(int64_t M, int64_t N, int64_t K, TailPlan* plan) {
  const int kblocks = static_cast<int>((K + kBK - 1) / kBK);
  if (kblocks < kWaveSliceKBlocks || M < k2BM || N < k2BN) return false;
  const int64_t pairs = sm_count() / 2;
  const int64_t n_tiles = (N + k2BN - 1) / k2BN;
  const int64_t ptiles = ((M + k2BM - 1) / k2BM) * n_tiles;
  const int64_t tail = ptiles % pairs;
  if (ptiles <= pairs || tail == 0) return false;
  const int slices = static_cast<int>(std::min<int64_t>(4, pairs / tail));
  if (slices < 2 || kblocks / slices < kMinSliceKBlocks) return false;
  plan->full_units = ptiles - tail;
  plan->slices = slices;
  plan->kb_per_slice = (kblocks + slices - 1) / slices;
  plan->p_row0 = (plan->full_units / n_tiles) * k2BM;
  return true;
}

int64_t tail_workspace_bytes(int64_t M, int64_t N, const TailPlan& plan) {
  return int64_t(plan.slices) * (M - plan.p_row0) * slices_pld(N) * int64_t(sizeof(float));
}

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

template <typename TIn, typename TOut, int BN, bool A_MN, bool B_MN>
int launch(const CUtensorMap& ma, const CUtensorMap& mb_, const CUtensorMap& mc,
           const GemmArgs& args, cudaStream_t s) {
  auto kern = gemm_tn_kernel<TIn, TOut, BN, A_MN, B_MN>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(Layout<BN>::kSmem));
  const int64_t tiles = ((args.M + kBM - 1) / kBM) * ((args.N + BN - 1) / BN);
  const int grid = static_cast<int>(imin64(tiles * args.k_slices, sm_count()));
  kern<<<grid, kThreads, Layout<BN>::kSmem, s>>>(ma, mb_, mc, args);
  return 0;
}

template <typename TIn, typename TOut, bool A_MN, bool B_MN>
int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb_, const CUtensorMap& mc,
                const CUtensorMap& mp, const GemmArgs& args, cudaStream_t s) {
  auto kern = gemm_tn_pair_kernel<TIn, TOut, A_MN, B_MN>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       static_cast<int>(Layout2::kSmem));
  const int64_t tiles = ((args.M + k2BM - 1) / k2BM) * ((args.N + k2BN - 1) / k2BN);
  const int64_t units = args.full_units + (tiles - args.full_units) * args.k_slices;
  const int pairs = static_cast<int>(imin64(units, sm_count() / 2));
  kern<<<2 * pairs, k2Threads, Layout2::kSmem, s>>>(ma, mb_, mc, args, mp);
  return 0;
}

// Kernel choice, from measurements on B200 (bf16, CUDA events):
//  - the pair kernel halves operand traffic per SM (each SM loads half of B)
//    and drains its accumulator with twice the warps; with 16-bit output it
//    is faster at every K measured (51200 x 4096 x K: K = 256 662 vs 608
//    TFLOP/s, 512 1212 vs 1150, 1024 1517 vs 1387, 2048 1662 on par);
//  - fp32 output (one 4 KB staging block per drain warp in the pair kernel)
//    goes to the pair kernel when the main loop dominates (K per unit >= 2048)
//    or the problem is small (under two waves of one-SM tiles).
// `k_eff` is the K loop length of one work unit summed over the segments.
bool use_pair(const GemmArgs& args, int64_t k_eff, bool out_f32) {
  const int sms = sm_count();
  const int64_t pair_tiles = ((args.M + k2BM - 1) / k2BM) * ((args.N + k2BN - 1) / k2BN);
  const int64_t single_tiles = ((args.M + kBM - 1) / kBM) * ((args.N + 255) / 256);
  if (args.M < k2BM || args.N < k2BN || pair_tiles * args.k_slices < sms / 2) return false;
  return !out_f32 || k_eff >= 2048 || single_tiles < 2 * sms;
}

template <typename TIn, typename TOut, bool A_MN, bool B_MN>
int launch_majors(const Operand& A, const Operand& B, GemmArgs args, int out_dtype,
                  void* partials, cudaStream_t s) {
  const bool bf16 = std::is_same<TIn, __nv_bfloat16>::value;
  CUtensorMap ma, mbm, mc, mp;
  memset(&mc, 0, sizeof(mc));
  memset(&mp, 0, sizeof(mp));
  if (args.full_units > 0) {
    // tail slicing (two-SM kernel only): whole tiles to C, the tail's slices
    // to the workspace rows p_row0 .. M-1, both through bulk tensor stores
    if (!make_c_map(&mc, args.C, args.M, args.N, args.ldc, out_dtype) ||
        !make_slices_map(&mp, partials, args.M - args.p_row0, args.N, slices_pld(args.N),
                         args.k_slices) ||
        !make_operand_map(&ma, A, args.M, args.K, 128, bf16) ||
        !make_operand_map(&mbm, B, args.N, args.K, 128, bf16)) {
      set_error("mb_gemm: cuTensorMapEncodeTiled failed (shape or alignment)");
      return 1;
    }
    args.tma_store = 1;
    return launch_pair<TIn, TOut, A_MN, B_MN>(ma, mbm, mc, mp, args, s);
  }
  args.tma_store = (args.k_slices > 1
                        ? make_slices_map(&mc, args.C, args.M, args.N, args.ldc, args.k_slices)
                        : make_c_map(&mc, args.C, args.M, args.N, args.ldc, out_dtype))
                       ? 1
                       : 0;
  const int64_t k_unit = std::min<int64_t>(args.K, int64_t(args.kb_per_slice) * kBK);
  if (use_pair(args, k_unit * args.nseg, out_dtype == MB_F32)) {
    // both operand maps: each CTA's 128 rows (K-major) / 64-wide blocks (MN-major)
    if (!make_operand_map(&ma, A, args.M, args.K, 128, bf16) ||
        !make_operand_map(&mbm, B, args.N, args.K, 128, bf16)) {
      set_error("mb_gemm: cuTensorMapEncodeTiled failed (shape or alignment)");
      return 1;
    }
    return launch_pair<TIn, TOut, A_MN, B_MN>(ma, mbm, mc, mp, args, s);
  }
  const int bn = args.N >= 192 ? 256 : (args.N > 64 ? 128 : 64);
  if (!make_operand_map(&ma, A, args.M, args.K, kBM, bf16) ||
      !make_operand_map(&mbm, B, args.N, args.K, bn, bf16)) {
    set_error("mb_gemm: cuTensorMapEncodeTiled failed (shape or alignment)");
    return 1;
  }
  if (bn == 256) return launch<TIn, TOut, 256, A_MN, B_MN>(ma, mbm, mc, args, s);
  if (bn == 128) return launch<TIn, TOut, 128, A_MN, B_MN>(ma, mbm, mc, args, s);
  return launch<TIn, TOut, 64, A_MN, B_MN>(ma, mbm, mc, args, s);
}

template <typename TIn, typename TOut>
int launch_typed(const Operand& A, const Operand& B, const GemmArgs& args, int out_dtype,
                 void* partials, cudaStream_t s) {
  if (!A.mn_major && !B.mn_major) {
    return launch_majors<TIn, TOut, false, false>(A, B, args, out_dtype, partials, s);
  }
  if (!A.mn_major && B.mn_major) {
    return launch_majors<TIn, TOut, false, true>(A, B, args, out_dtype, partials, s);
  }
  return launch_majors<TIn, TOut, true, true>(A, B, args, out_dtype, partials, s);
}

// Check one operand's layout; `mn` is its M (A) or N (B) extent.
bool operand_ok(const Operand& op, int64_t mn, int64_t K, const char* name) {
  if (op.parts < 1 || op.parts > 3) {
    set_error("mb_gemm: %s parts must be 1, 2 or 3 (got %d)", name, op.parts);
    return false;
  }
  if (op.ptr == nullptr || !aligned_to(op.ptr, 16)) {
    set_error("mb_gemm: %s must be a 16-byte aligned device pointer", name);
    return false;
  }
  if (op.ld % 8 != 0) {
    set_error("mb_gemm: leading dimension of %s must be a multiple of 8 (16-byte rows)", name);
    return false;
  }
  if (op.mn_major ? op.ld < mn : (op.ld < K || K % 8 != 0)) {
    set_error(op.mn_major ? "mb_gemm: %s: leading dimension smaller than its M/N extent"
                          : "mb_gemm: %s: K must be a multiple of 8 and at most the leading "
                            "dimension",
              name);
    return false;
  }
  const int64_t rows = op.mn_major ? K : mn;
  if (op.parts > 1 && (op.part_stride % 8 != 0 || op.part_stride < rows * op.ld)) {
    set_error("mb_gemm: %s part stride must be a multiple of 8 covering a whole part", name);
    return false;
  }
  return true;
}

}  // namespace
}  // namespace mb

using namespace mb;

extern "C" int64_t mb_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int a_parts,
                                           int b_parts, int out_dtype) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  int per = 0;
  const int slices = k_slices_for(M, N, K, a_parts, b_parts, out_dtype, true, &per);
  if (slices > 1) return int64_t(slices) * M * slices_pld(N) * int64_t(sizeof(float));
  TailPlan plan;
  return tail_plan(M, N, K, &plan) ? tail_workspace_bytes(M, N, plan) : 0;
}

extern "C" int mb_gemm(int in_dtype, const void* A, int a_major, int64_t lda, int64_t a_part_stride,
                       int a_parts, const int32_t* a_nonzero, const void* B, int b_major,
                       int64_t ldb, int64_t b_part_stride, int b_parts, const int32_t* b_nonzero,
                       const void* bias, int bias_dtype, int out_dtype, void* C, int64_t ldc,
                       int64_t M, int64_t N, int64_t K, void* workspace, int64_t workspace_bytes,
                       void* stream) {
  clear_error();
  MB_CHECK_ARG(in_dtype == MB_BF16 || in_dtype == MB_F16,
               "mb_gemm: inputs must be bfloat16 or float16 (got dtype %d)", in_dtype);
  MB_CHECK_ARG(out_dtype == MB_F32 || out_dtype == in_dtype,
               "mb_gemm: output must be float32 or the input type");
  MB_CHECK_ARG(bias == nullptr || bias_dtype == MB_F32 || bias_dtype == MB_BF16 ||
                   bias_dtype == MB_F16,
               "mb_gemm: bias must be float32, bfloat16 or float16");
  MB_CHECK_ARG((a_major == MB_KMAJOR || a_major == MB_MNMAJOR) &&
                   (b_major == MB_KMAJOR || b_major == MB_MNMAJOR),
               "mb_gemm: unknown operand major");
  MB_CHECK_ARG(!(a_major == MB_MNMAJOR && b_major == MB_KMAJOR),
               "mb_gemm: an M-major A needs an N-major B");
  MB_CHECK_ARG(M >= 0 && N >= 0 && K >= 0, "mb_gemm: negative size");
  if (M == 0 || N == 0) return 0;
  MB_CHECK_ARG(K > 0, "mb_gemm: K must be positive");
  MB_CHECK_ARG(M < (int64_t(1) << 31) && N < (int64_t(1) << 31) && K < (int64_t(1) << 31),
               "mb_gemm: M, N or K too large");
  MB_CHECK_ARG(ldc >= N, "mb_gemm: ldc < N");
  MB_CHECK_ARG(C != nullptr, "mb_gemm: null C");
  const Operand a{A, lda, a_part_stride, a_parts, a_major == MB_MNMAJOR};
  const Operand b{B, ldb, b_part_stride, b_parts, b_major == MB_MNMAJOR};
  if (!operand_ok(a, M, K, "A") || !operand_ok(b, N, K, "B")) return 1;

  const int64_t out_elt = out_dtype == MB_F32 ? 4 : 2;
  GemmArgs args{};
  args.bias = bias;
  args.C = C;
  args.ldc = ldc;
  args.M = M;
  args.N = N;
  args.K = K;
  args.bias_dtype = bias_dtype;
  args.vec_ok = (ldc * out_elt) % 16 == 0 && aligned_to(C, 16) ? 1 : 0;
  args.a_nonzero = a_nonzero;
  args.b_nonzero = b_nonzero;
  // (A part i, B part j) products with i + j <= 2: part p of a 3-way split
  // carries the bits 8p below the leading ones, so the dropped products sit
  // under 2^-24 of the result (bf16x6 for two 3-way split fp32 operands)
  args.nseg = 0;
  for (int order = 0; order <= 2; ++order) {
    for (int i = 0; i <= order; ++i) {
      const int j = order - i;
      if (i < a_parts && j < b_parts) {
        args.seg_a[args.nseg] = static_cast<int8_t>(i);
        args.seg_b[args.nseg] = static_cast<int8_t>(j);
        ++args.nseg;
      }
    }
  }
  cudaStream_t s = as_stream(stream);
  const int64_t pld = slices_pld(N);
  args.k_slices = k_slices_for(M, N, K, a_parts, b_parts, out_dtype, true, &args.kb_per_slice);
  if (args.k_slices > 1 &&
      (workspace == nullptr ||
       workspace_bytes < int64_t(args.k_slices) * M * pld * int64_t(sizeof(float)))) {
    // no room for the slices that would only add parallelism (e.g. through
    // mb_gemm_tn, which takes no workspace): keep the ones accuracy needs
    args.k_slices = k_slices_for(M, N, K, a_parts, b_parts, out_dtype, false, &args.kb_per_slice);
  }
  args.full_units = 0;
  args.p_row0 = 0;
  TailPlan plan;
  if (args.k_slices == 1 && tail_plan(M, N, K, &plan) && workspace != nullptr &&
      workspace_bytes >= tail_workspace_bytes(M, N, plan) && aligned_to(workspace, 16) &&
      aligned_to(C, 16) && (ldc * out_elt) % 16 == 0) {
    args.full_units = plan.full_units;
    args.k_slices = plan.slices;
    args.kb_per_slice = plan.kb_per_slice;
    args.p_row0 = plan.p_row0;
  }
  int rc;
  if (args.k_slices > 1 && args.full_units == 0) {
    // fp32 partial sums per K slice into the workspace, then their ordered sum
    const int64_t need = int64_t(args.k_slices) * M * pld * int64_t(sizeof(float));
    MB_CHECK_ARG(workspace != nullptr && workspace_bytes >= need && aligned_to(workspace, 16),
                 "mb_gemm: workspace of %lld bytes (16-byte aligned) required, got %lld",
                 (long long)need, (long long)workspace_bytes);
    GemmArgs part = args;
    part.C = workspace;
    part.ldc = pld;
    part.bias = nullptr;
    part.vec_ok = 1;
    rc = in_dtype == MB_BF16 ? launch_typed<__nv_bfloat16, float>(a, b, part, MB_F32, nullptr, s)
                             : launch_typed<__half, float>(a, b, part, MB_F32, nullptr, s);
    if (rc != 0) return rc;
    const unsigned grid = static_cast<unsigned>(imin64(ceil_div(M * N, 256), 148 * 8));
    const float* ws = static_cast<const float*>(workspace);
    if (out_dtype == MB_F32) {
      slices_reduce_kernel<float><<<grid, 256, 0, s>>>(ws, args.k_slices, M, N, pld, bias,
                                                       bias_dtype, static_cast<float*>(C), ldc);
    } else if (out_dtype == MB_BF16) {
      slices_reduce_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
          ws, args.k_slices, M, N, pld, bias, bias_dtype, static_cast<__nv_bfloat16*>(C), ldc);
    } else {
      slices_reduce_kernel<__half><<<grid, 256, 0, s>>>(ws, args.k_slices, M, N, pld, bias,
                                                        bias_dtype, static_cast<__half*>(C), ldc);
    }
    MB_CHECK_LAUNCH("mb_gemm");
    return 0;
  }
  void* partials = args.full_units > 0 ? workspace : nullptr;
  if (in_dtype == MB_BF16) {
    rc = out_dtype == MB_F32 ? launch_typed<__nv_bfloat16, float>(a, b, args, out_dtype, partials, s)
                             : launch_typed<__nv_bfloat16, __nv_bfloat16>(a, b, args, out_dtype, partials, s);
  } else {
    rc = out_dtype == MB_F32 ? launch_typed<__half, float>(a, b, args, out_dtype, partials, s)
                             : launch_typed<__half, __half>(a, b, args, out_dtype, partials, s);
  }
  if (rc != 0) return rc;
  if (args.full_units > 0) {
    // the tail tiles: their slices' partial sums added in order, + bias
    const int64_t rows = M - args.p_row0;
    const unsigned grid = static_cast<unsigned>(imin64(ceil_div(rows * N, 256), 148 * 8));
    const float* ws = static_cast<const float*>(workspace);
    const int64_t n_tiles = (N + k2BN - 1) / k2BN;
    if (out_dtype == MB_F32) {
      tail_reduce_kernel<float><<<grid, 256, 0, s>>>(ws, args.k_slices, M, N, pld, args.p_row0,
                                                     args.full_units, n_tiles, bias, bias_dtype,
                                                     static_cast<float*>(C), ldc);
    } else if (out_dtype == MB_BF16) {
      tail_reduce_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
          ws, args.k_slices, M, N, pld, args.p_row0, args.full_units, n_tiles, bias, bias_dtype,
          static_cast<__nv_bfloat16*>(C), ldc);
    } else {
      tail_reduce_kernel<__half><<<grid, 256, 0, s>>>(ws, args.k_slices, M, N, pld, args.p_row0,
                                                      args.full_units, n_tiles, bias, bias_dtype,
                                                      static_cast<__half*>(C), ldc);
    }
  }
  MB_CHECK_LAUNCH("mb_gemm");
  return 0;
}

extern "C" int mb_gemm_tn(int in_dtype, const void* A, int64_t lda, const void* B, int64_t ldb,
                          const void* bias, int bias_dtype, int out_dtype, void* C, int64_t ldc,
                          int64_t M, int64_t N, int64_t K, void* stream) {
  return mb_gemm(in_dtype, A, MB_KMAJOR, lda, 0, 1, nullptr, B, MB_KMAJOR, ldb, 0, 1, nullptr,
                 bias, bias_dtype, out_dtype, C, ldc, M, N, K, nullptr, 0, stream);
}

namespace mb {

int gemm_unit_status(bool clear) { return read_device_status(clear); }

cudaError_t gemm_unit_wait_probe(uint32_t polls, cudaStream_t stream) {
  wait_timeout_probe_kernel<<<1, 32, 0, stream>>>(polls);
  return cudaGetLastError();
}

}  // namespace mb
