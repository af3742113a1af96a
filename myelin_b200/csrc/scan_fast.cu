// Warp-specialized LIF/ALIF scan kernels for 16-byte-aligned [T, B*N] rows.
//
// CTA = kWarps compute warps over a tile of kTileN consecutive flat neurons
// (two per thread). Every kChunk-step chunk of the tile travels through a
// ring of shared-memory stages: one 2-D bulk tensor copy (TMA) per input
// array brings a [kChunk x kTileN] box in, completing on the stage's "full"
// mbarrier. There is no copy warp: the compute warp that finishes a stage
// last (a counter per stage, acquire-release) writes it back (dense outputs,
// one bulk tensor store) and refills it with the chunk RING steps ahead, so
// every warp of the CTA computes and no CTA-wide barrier is taken after
// set-up. Compute threads own two neighbouring neurons each, so every smem
// read, global store and bf16 conversion moves a pair.
//
// Forward: the state is carried in fp32 registers; per step it writes dense
// spikes (into the stage, over the inputs they came from) and/or packed words
// and/or spike counts, and at each chunk start the fp32 checkpoint.
// Backward: chunks run last to first; each is replayed from its checkpoint
// into registers (bit-identical to the forward) and then walked in reverse.
#include <climits>
#include <cstring>
#include <initializer_list>
#include <type_traits>

#include "async_copy.cuh"
#include "common.cuh"
#include "scan_common.cuh"
#include "tma.cuh"

namespace mb {

namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kTileN = kWarps * 32 * 2;  // neurons per CTA

// Stages in flight and resident CTAs per SM (the register budget the kernel is
// compiled for), per element type: the forward's stage is one input box, the
// backward's two input boxes plus the chunk's fp32 checkpoints.
// (Measured on B200 at BASELINE config 3, ALIF bf16: forward 5 stages x 5
// CTAs 0.1068 ms against 4 x 6 0.1088 and 3 x 8 0.1108; backward 2 stages x
// 4 CTAs 0.1398 against 3 x 4 0.1417 and 2 x 5 0.1434.)
template <typename T>
struct FwdCfg {
  static constexpr int kRing = sizeof(T) == 2 ? 5 : 3;
  static constexpr int kMinBlocks = sizeof(T) == 2 ? 5 : 4;
};

template <typename T>
__host__ __device__ constexpr size_t fwd_smem(int ring) {
  return size_t(ring) * kChunk * kTileN * sizeof(T) + ring * (sizeof(uint64_t) + sizeof(uint32_t));
}

// Backward stage: kChunk rows of x, kChunk rows of grad_spikes, then the fp32
// checkpoint rows (membrane, adaptation) of the chunk.
template <typename T>
__host__ __device__ constexpr size_t bwd_stage_bytes() {
  return size_t(2) * kChunk * kTileN * sizeof(T) + 2 * kTileN * sizeof(float);
}

template <typename T>
struct BwdCfg {
  static constexpr int kRing = 2;
};

template <typename T>
__host__ __device__ constexpr size_t bwd_smem(int ring) {
  return size_t(ring) * bwd_stage_bytes<T>() + ring * (sizeof(uint64_t) + sizeof(uint32_t));
}

// Output modes of the forward (what the caller asked for), fixed at compile
// time so the per-step code has no branches: dense spikes, packed words,
// spike rates, or any combination (checked at run time).
enum FwdMode { kFwdDense = 0, kFwdPacked = 1, kFwdRates = 2, kFwdAny = 3 };
// Backward inputs: spike gradients, rate gradients, or any combination.
enum BwdMode { kBwdSpikes = 0, kBwdRates = 1, kBwdAny = 2 };

// Resident CTAs per SM the backward is compiled for (a register budget). LIF
// fits 4 without spilling. ALIF (two state adjoints, two replayed states)
// also runs at 4 for one gradient input: a small spill costs less than the
// occupancy lost at 3 (measured 0.155 vs 0.179 ms at config 3). With both
// spike and rate gradients the spill grows past 100 bytes, so that mode runs
// at 3; the exp-based surrogates (sigmoid, multi-Gaussian) hold more
// temporaries and run at 2.
constexpr int bwd_min_blocks(int kind, int surr, int mode) {
  return kind == MB_LIF ? 4
         : (surr == MB_SURR_SIGMOID || surr == MB_SURR_MULTI_GAUSSIAN) ? 2
         : mode == kBwdAny ? 3
                           : 4;
}

// Per-launch fp32 constants, each duplicated into both lanes of a float2 for
// the packed instructions; passed as a kernel parameter.
struct PairConsts {
  float2 decay, nthr, adapt_decay, nbeta, reset, k0, k1, one;
};

inline float2 dup2(float v) { return make_float2(v, v); }

template <int SURR>
PairConsts pair_consts(float decay, float thr, float adapt_decay, float beta, float reset,
                       float slope) {
  const SurrogateD<SURR> sd(slope);
  return PairConsts{dup2(decay), dup2(-thr), dup2(adapt_decay), dup2(-beta), dup2(reset),
                    dup2(sd.k0), dup2(sd.k1), dup2(1.0f)};
}

// Called by every compute thread when it is done with a stage (its reads of
// the inputs and its writes of the outputs). Orders the thread's shared-memory
// accesses before later async-proxy accesses (the store that reads the stage,
// the copies that refill it), then counts the warp in on the stage's counter
// with an acquire-release add at CTA scope. Returns true in lane 0 of the warp
// that arrives last: every other warp's accesses to the stage happen before
// what that lane does next. The last lane puts the counter back to 0 (before
// any refill of the stage, whose completion the next users acquire).
__device__ __forceinline__ bool last_warp_done(uint32_t* counter) {
  fence_proxy_async_smem();
  __syncwarp();
  if ((threadIdx.x & 31) != 0) return false;
  uint32_t old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
               : "=r"(old)
               : "r"(smem_addr(counter))
               : "memory");
  if (old != kWarps - 1) return false;
  *counter = 0;
  return true;
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
template <typename T, int KIND, int RESET, int MODE, int RING, int MINB>
__global__ void __launch_bounds__(kThreads, MINB) scan_fwd_fast_kernel(
    const ScanFwdArgs a, const PairConsts c, const __grid_constant__ CUtensorMap in_map,
    const __grid_constant__ CUtensorMap out_map) {
  using P = Pair<T>;
  using V = typename P::V;
  constexpr int kRing = RING;
  constexpr uint32_t kStageBytes = uint32_t(kChunk) * kTileN * sizeof(T);
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* ring = reinterpret_cast<T*>(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + size_t(kRing) * kStageBytes);
  uint32_t* done = reinterpret_cast<uint32_t*>(full + kRing);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t e0 = int64_t(blockIdx.x) * kTileN;
  const int tile_n = static_cast<int>(imin64(kTileN, a.BN - e0));
  const int64_t K = (a.T + kChunk - 1) / kChunk;
  constexpr bool kDense = MODE == kFwdDense || MODE == kFwdAny;
  const bool do_dense = kDense && (MODE != kFwdAny || a.spikes != nullptr);

  // chunk k into stage k % kRing: one box of kChunk rows x kTileN neurons
  // (rows past T and neurons past B*N read as zero and are never used)
  auto refill = [&](int64_t k) {
    const int st = static_cast<int>(k % kRing);
    mbar_arrive_expect_tx(&full[st], kStageBytes);
    tma_load_box_2d(ring + size_t(st) * kChunk * kTileN, &in_map, static_cast<int>(e0),
                    static_cast<int>(k * kChunk), &full[st]);
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&full[s], 1);
      done[s] = 0;
    }
    fence_barrier_init();
    for (int64_t k = 0; k < imin64(kRing, K); ++k) refill(k);
  }
  __syncthreads();

  const int tid = threadIdx.x;  // 0 .. kThreads - 1
  // Neurons of a thread: the adjacent pair e, e + 1 (e = e0 + 2 tid), so that
  // one vector access moves both; or, for packed output only (kSplit), lane l
  // of warp w owns neurons l and l + 32 of the warp's 64 (ea = e0 + 64 w + l,
  // eb = ea + 32), so that each ballot over the warp is already a finished
  // 32-neuron word (no bit interleaving per step). Packed output needs
  // N % 32 == 0, so tile_n is a multiple of 32 and both halves of a warp are
  // wholly inside or outside the tile.
  constexpr bool kSplit = MODE == kFwdPacked;
  using E = Elem<T>;
  const bool valid = kSplit ? 64 * warp < tile_n : 2 * tid < tile_n;  // tile_n is even
  const bool valid_b = kSplit ? 64 * warp + 32 < tile_n : valid;
  const int64_t e = e0 + 2 * tid;
  const int64_t ea = e0 + 64 * warp + lane, eb = ea + 32;
  constexpr bool kTwoStates = KIND != MB_LIF;  // ALIF adaptation / Izhikevich recovery
  F2 m = f2(0.0f), ad = f2(0.0f);
  int c0 = 0, c1 = 0;
  if constexpr (kSplit) {
    const T* v0 = static_cast<const T*>(a.v0);
    const T* a0 = static_cast<const T*>(a.a0);
    m = f2(make_float2(valid ? E::to_f(v0[ea]) : 0.0f, valid_b ? E::to_f(v0[eb]) : 0.0f));
    if (kTwoStates) {
      ad = f2(make_float2(valid ? E::to_f(a0[ea]) : 0.0f, valid_b ? E::to_f(a0[eb]) : 0.0f));
    }
  } else if (valid) {
    m = f2(P::to_f2(reinterpret_cast<const V*>(a.v0)[e >> 1]));
    if (kTwoStates) ad = f2(P::to_f2(reinterpret_cast<const V*>(a.a0)[e >> 1]));
  }
  const F2 decay = c.decay, nthr = c.nthr, adapt_decay = c.adapt_decay, nbeta = c.nbeta;
  const float reset_v = a.reset;

  constexpr bool kPacked = MODE == kFwdPacked || MODE == kFwdAny;
  constexpr bool kRates = MODE == kFwdRates || MODE == kFwdAny;
  const bool do_packed = kPacked && (MODE != kFwdAny || a.packed != nullptr);
  // Dense spikes overwrite the x values they came from in the stage (each
  // thread its own pair); the warp that finishes the chunk last writes the
  // whole stage [16 rows x 256 neurons] with one bulk tensor store (clipped
  // at the tensor's edges) before refilling it.
  // packed words: this warp's 64 neurons are flat words q and q+1; with
  // N % 32 == 0 every word lies wholly inside or wholly outside the tile
  const int64_t words_per_t = a.BN >> 5;
  const int64_t q = (e0 >> 5) + 2 * warp + (kSplit ? lane : lane >> 4);
  int32_t* pk = do_packed ? a.packed + q : nullptr;
  // pair layout: lanes 0 and 16 store words q and q + 1 (built from the even
  // and odd ballots); split layout: lanes 0 and 1 store the two ballots
  const bool pk_lane = kSplit ? (lane == 0 && valid) || (lane == 1 && valid_b)
                              : (lane & 15) == 0 && (q << 5) < a.BN;
  const int sh = lane & 16;  // pair layout: lanes 0-15 -> word q, lanes 16-31 -> word q+1

  // a register copy: referring to the parameter block itself would place it
  // in local memory
  const IzhConsts izc = a.izh;
  auto step = [&](float2 xf, V* slot) {
    Step2<KIND == kIzhikevich ? MB_LIF : KIND, RESET> st;
    if constexpr (KIND == kIzhikevich) {
      st.s0 = izh_step(m.x, ad.x, xf.x, izc);
      st.s1 = izh_step(m.y, ad.y, xf.y, izc);
      st.sf = f2(st.s0 ? 1.0f : 0.0f, st.s1 ? 1.0f : 0.0f);
    } else {
      st.run(m, ad, f2(xf), decay, nthr, reset_v, adapt_decay, nbeta);
    }
    if (kRates) {
      c0 += st.s0 ? 1 : 0;
      c1 += st.s1 ? 1 : 0;
    }
    if (kDense && (MODE != kFwdAny || do_dense)) {
      const float2 sf = split(st.sf);
      *slot = P::from_f2(sf.x, sf.y);  // exact 0 / 1 in every I/O type
    }
    if (kPacked && (MODE != kFwdAny || pk != nullptr)) {
      const uint32_t even = __ballot_sync(0xffffffffu, st.s0);
      const uint32_t odd = __ballot_sync(0xffffffffu, st.s1);
      const uint32_t word =
          kSplit ? (lane == 0 ? even : odd)
                 : spread_even_bits(even >> sh) | (spread_even_bits(odd >> sh) << 1);
      if (pk_lane) *pk = static_cast<int32_t>(word);
      pk += words_per_t;
    }
  };

  for (int64_t k = 0; k < K; ++k) {
    const int s = static_cast<int>(k % kRing);
    if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>((k / kRing) & 1))) {
      bulk_wait_all();  // stores of earlier chunks finish before the early exit
      return;
    }
    if constexpr (kSplit) {
      if (a.ckpt_v != nullptr) {
        if (valid) a.ckpt_v[k * a.BN + ea] = split(m).x;
        if (valid_b) a.ckpt_v[k * a.BN + eb] = split(m).y;
        if (kTwoStates) {
          if (valid) a.ckpt_a[k * a.BN + ea] = split(ad).x;
          if (valid_b) a.ckpt_a[k * a.BN + eb] = split(ad).y;
        }
      }
    } else if (a.ckpt_v != nullptr && valid) {
      reinterpret_cast<float2*>(a.ckpt_v + k * a.BN)[e >> 1] = split(m);
      if (kTwoStates) reinterpret_cast<float2*>(a.ckpt_a + k * a.BN)[e >> 1] = split(ad);
    }
    T* stage = ring + size_t(s) * kChunk * kTileN;
    V* row = reinterpret_cast<V*>(stage) + tid;
    const T* srow = stage + 64 * warp + lane;  // split layout: neurons l and l + 32
    const int len = static_cast<int>(imin64(kChunk, a.T - k * kChunk));
    if constexpr (kSplit) {
      if (len == kChunk) {
        V xv[kChunk];  // the two neurons' inputs joined as one pair value
#pragma unroll
        for (int j = 0; j < kChunk; ++j) xv[j] = P::join(srow[j * kTileN], srow[j * kTileN + 32]);
#pragma unroll
        for (int j = 0; j < kChunk; ++j) step(P::to_f2(xv[j]), nullptr);
      } else {
        for (int j = 0; j < len; ++j) {
          step(P::to_f2(P::join(srow[j * kTileN], srow[j * kTileN + 32])), nullptr);
        }
      }
    } else if (len == kChunk) {
      // all loads first: the spike stores below alias the same stage
      V xv[kChunk];
#pragma unroll
      for (int j = 0; j < kChunk; ++j) xv[j] = row[j * (kTileN / 2)];
#pragma unroll
      for (int j = 0; j < kChunk; ++j) step(P::to_f2(xv[j]), row + j * (kTileN / 2));
    } else {
      for (int j = 0; j < len; ++j) step(P::to_f2(row[j * (kTileN / 2)]), row + j * (kTileN / 2));
    }
    if (last_warp_done(&done[s])) {
      if (kDense && (MODE != kFwdAny || do_dense)) {
        tma_store_box_2d(&out_map, stage, static_cast<int>(e0), static_cast<int>(k * kChunk));
        bulk_wait_read_all();  // the stage may be refilled once the store has read it
      }
      if (k + kRing < K) refill(k + kRing);
    }
    __syncwarp();
  }
  if (kDense && (MODE != kFwdAny || do_dense)) bulk_wait_all();

  if constexpr (kSplit) {
    T* vT = static_cast<T*>(a.vT);
    T* aT = static_cast<T*>(a.aT);
    if (vT && valid) vT[ea] = E::from_f(split(m).x);
    if (vT && valid_b) vT[eb] = E::from_f(split(m).y);
    if (kTwoStates && aT && valid) aT[ea] = E::from_f(split(ad).x);
    if (kTwoStates && aT && valid_b) aT[eb] = E::from_f(split(ad).y);
    return;
  }
  if (!valid) return;
  if (a.vT) reinterpret_cast<V*>(a.vT)[e >> 1] = P::from_f2(split(m).x, split(m).y);
  if (kTwoStates && a.aT) reinterpret_cast<V*>(a.aT)[e >> 1] = P::from_f2(split(ad).x, split(ad).y);
  if (kRates && a.rates) {
    const float tf = static_cast<float>(a.T);
    reinterpret_cast<V*>(a.rates)[e >> 1] =
        P::from_f2(__fdiv_rn(static_cast<float>(c0), tf), __fdiv_rn(static_cast<float>(c1), tf));
  }
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------
template <typename T, int KIND, int RESET, int SURR, int MODE, int RING, int MINB>
__global__ void __launch_bounds__(kThreads, MINB) scan_bwd_fast_kernel(
    const ScanBwdArgs a, const PairConsts c, const __grid_constant__ CUtensorMap x_map,
    const __grid_constant__ CUtensorMap g_map, const __grid_constant__ CUtensorMap out_map) {
  using P = Pair<T>;
  using V = typename P::V;
  constexpr int kRing = RING;
  constexpr uint32_t kBoxBytes = uint32_t(kChunk) * kTileN * sizeof(T);
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + kRing * bwd_stage_bytes<T>());
  uint32_t* done = reinterpret_cast<uint32_t*>(full + kRing);
  auto stage_x = [&](int s) { return reinterpret_cast<T*>(smem_raw + s * bwd_stage_bytes<T>()); };
  auto stage_g = [&](int s) { return stage_x(s) + kChunk * kTileN; };
  auto stage_c = [&](int s) { return reinterpret_cast<float*>(stage_g(s) + kChunk * kTileN); };

  // Tiles in reverse block order: the forward runs tiles in block order, so
  // the backward's first CTAs take the tiles the forward finished last, whose
  // last chunks (inputs and checkpoints, read first here) are still in L2
  // (config 3, ALIF bf16: forward + backward 0.2415 -> 0.2303 ms).
  const int64_t e0 = int64_t(gridDim.x - 1 - blockIdx.x) * kTileN;
  const int tile_n = static_cast<int>(imin64(kTileN, a.BN - e0));
  const int64_t K = (a.T + kChunk - 1) / kChunk;
  constexpr bool kSpikes = MODE == kBwdSpikes || MODE == kBwdAny;
  constexpr bool kRateGrad = MODE == kBwdRates || MODE == kBwdAny;
  const bool has_gs = kSpikes && (MODE != kBwdAny || a.grad_spikes != nullptr);
  const bool has_alif = KIND == MB_ALIF;

  // the i-th chunk from the end into stage i % kRing: a box of x rows, a box
  // of grad_spikes rows (rows past T and neurons past B*N read as zero and
  // are never used) and the chunk's checkpoint rows (exactly the tile)
  auto refill = [&](int64_t i) {
    const int st = static_cast<int>(i % kRing);
    const int64_t k = K - 1 - i;
    const uint32_t ckpt_bytes = uint32_t(tile_n) * 4u;
    mbar_arrive_expect_tx(&full[st], kBoxBytes * (has_gs ? 2u : 1u) +
                                         ckpt_bytes * (has_alif ? 2u : 1u));
    tma_load_box_2d(stage_x(st), &x_map, static_cast<int>(e0), static_cast<int>(k * kChunk),
                    &full[st]);
    if (has_gs) {
      tma_load_box_2d(stage_g(st), &g_map, static_cast<int>(e0), static_cast<int>(k * kChunk),
                      &full[st]);
    }
    bulk_copy_g2s(stage_c(st), a.ckpt_v + k * a.BN + e0, ckpt_bytes, &full[st]);
    if (has_alif) bulk_copy_g2s(stage_c(st) + kTileN, a.ckpt_a + k * a.BN + e0, ckpt_bytes, &full[st]);
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&full[s], 1);
      done[s] = 0;
    }
    fence_barrier_init();
    for (int64_t i = 0; i < imin64(kRing, K); ++i) refill(i);
  }
  __syncthreads();

  const int tid = threadIdx.x;
  const bool valid = 2 * tid < tile_n;
  const int64_t e = e0 + 2 * tid;
  const F2 decay = c.decay, nthr = c.nthr, adapt_decay = c.adapt_decay, nbeta = c.nbeta;
  const F2 reset2 = c.reset;
  const float reset_v = a.reset;
  const SurrogateD2<SURR> dfun(a.slope, c.k0, c.k1, c.one);

  F2 gm = f2(0.0f), ga = f2(0.0f), gr = f2(0.0f);
  if (valid) {
    if (a.grad_vT) gm = f2(P::to_f2(reinterpret_cast<const V*>(a.grad_vT)[e >> 1]));
    if (KIND == MB_ALIF && a.grad_aT) {
      ga = f2(P::to_f2(reinterpret_cast<const V*>(a.grad_aT)[e >> 1]));
    }
    if (kRateGrad && a.grad_rates) {
      // the grad of a rate output reaches every step as grad_rates / T
      // (src/myelin/autograd.py:842-844)
      const float2 v = P::to_f2(reinterpret_cast<const V*>(a.grad_rates)[e >> 1]);
      const float tf = static_cast<float>(a.T);
      gr = f2(__fdiv_rn(v.x, tf), __fdiv_rn(v.y, tf));
    }
  }

  // One reverse step for a pair of neurons; returns dL/dx_t and updates gm, ga.
  // pv is what the replay kept: p - theta (subtractive reset) or p (hard
  // reset); nth = -theta. The spike is diff >= 0, which equals p >= theta for
  // finite values (a NaN or infinite membrane gives NaN gradients either way).
  auto adjoint = [&](F2 pv, F2 nth, F2 gsum) -> F2 {
    const F2 diff = (RESET == MB_RESET_SUBTRACT) ? pv : add2(pv, nth);
    const F2 d = dfun(diff);
    F2 gp;
    if (KIND == MB_LIF) {
      if (RESET == MB_RESET_HARD) {
        const F2 nsf = f2(lt_f(diff.x, 0.0f), lt_f(diff.y, 0.0f));  // 1 - s
        gp = fma2(gm, fma2(sub2(reset2, pv), d, nsf), mul2(gsum, d));
      } else {
        gp = fma2(fma2(gm, nth, gsum), d, gm);
      }
    } else {
      if (RESET == MB_RESET_HARD) {
        const F2 nsf = f2(lt_f(diff.x, 0.0f), lt_f(diff.y, 0.0f));  // 1 - s
        const F2 Gd = mul2(add2(fma2(gm, sub2(reset2, pv), gsum), ga), d);
        gp = fma2(gm, nsf, Gd);
        ga = fma2(nbeta, Gd, mul2(ga, adapt_decay));
      } else {
        const F2 sf = f2(ge_f(diff.x, 0.0f), ge_f(diff.y, 0.0f));
        const F2 Gd = mul2(add2(fma2(gm, nth, gsum), ga), d);
        gp = add2(gm, Gd);
        ga = fma2(nbeta, fma2(sf, gm, Gd), mul2(ga, adapt_decay));
      }
    }
    gm = mul2(gp, decay);
    return gp;
  };

  // Per-neuron sum over t of grad_x (LIF only: the bias gradient of a
  // stream-synapse layer, db = sum over t and batch rows), from the last
  // step to the first, of the values as stored.
  const bool do_sum = KIND == MB_LIF && a.grad_sum != nullptr;
  F2 gsum = f2(0.0f);

  // grad_x overwrites the x values of the stage (x is dead once the chunk is
  // replayed; each thread its own pair) and the finished stage goes out with
  // one bulk tensor store.
  for (int64_t i = 0; i < K; ++i) {
    const int s = static_cast<int>(i % kRing);
    const int64_t k = K - 1 - i;
    const int64_t t0 = k * kChunk;
    const int len = static_cast<int>(imin64(kChunk, a.T - t0));
    if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>((i / kRing) & 1))) {
      bulk_wait_all();  // stores of earlier chunks finish before the early exit
      return;
    }
    V* xrow = reinterpret_cast<V*>(stage_x(s)) + tid;
    const V* grow = reinterpret_cast<const V*>(stage_g(s)) + tid;
    if (valid) {
      F2 m = f2(reinterpret_cast<const float2*>(stage_c(s))[tid]), av = f2(0.0f);
      if (KIND == MB_ALIF) av = f2(reinterpret_cast<const float2*>(stage_c(s) + kTileN)[tid]);
      F2 PV[kChunk], TH[kChunk];
      auto replay = [&](int j) {
        Step2<KIND, RESET> st;
        st.run(m, av, f2(P::to_f2(xrow[j * (kTileN / 2)])), decay, nthr, reset_v, adapt_decay,
               nbeta);
        PV[j] = (RESET == MB_RESET_SUBTRACT) ? st.diff : st.p;
        TH[j] = st.nth;
      };
      // tag: also add the stored grad_x to the per-neuron sum over t
      auto reverse = [&](int j, auto tag) {
        F2 g = gr;
        if (MODE == kBwdSpikes) {
          g = f2(P::to_f2(grow[j * (kTileN / 2)]));
        } else if (has_gs) {
          g = add2(g, f2(P::to_f2(grow[j * (kTileN / 2)])));
        }
        const float2 gp = split(adjoint(PV[j], TH[j], g));
        const V stored = P::from_f2(gp.x, gp.y);
        xrow[j * (kTileN / 2)] = stored;
        if constexpr (decltype(tag)::value) gsum = add2(gsum, f2(P::to_f2(stored)));
      };
      auto reverse_chunk = [&](auto tag) {
        if (len == kChunk) {
#pragma unroll
          for (int j = kChunk - 1; j >= 0; --j) reverse(j, tag);
        } else {
#pragma unroll
          for (int j = kChunk - 1; j >= 0; --j) {
            if (j < len) reverse(j, tag);
          }
        }
      };
      if (len == kChunk) {
#pragma unroll
        for (int j = 0; j < kChunk; ++j) replay(j);
      } else {
#pragma unroll
        for (int j = 0; j < kChunk; ++j) {
          if (j < len) replay(j);
        }
      }
      if constexpr (KIND == MB_LIF) {
        if (do_sum) reverse_chunk(std::true_type{});
        else reverse_chunk(std::false_type{});
      } else {
        reverse_chunk(std::false_type{});
      }
    }
    // the warp done last with the chunk writes grad_x (it overwrote x in the
    // stage) and refills the stage with the chunk kRing further back
    if (last_warp_done(&done[s])) {
      tma_store_box_2d(&out_map, stage_x(s), static_cast<int>(e0), static_cast<int>(t0));
      bulk_wait_read_all();
      if (i + kRing < K) refill(i + kRing);
    }
    __syncwarp();
  }
  bulk_wait_all();
  if (!valid) return;
  if (do_sum) reinterpret_cast<float2*>(a.grad_sum)[e >> 1] = split(gsum);
  if (a.grad_v0) reinterpret_cast<V*>(a.grad_v0)[e >> 1] = P::from_f2(split(gm).x, split(gm).y);
  if (KIND == MB_ALIF && a.grad_a0) {
    reinterpret_cast<V*>(a.grad_a0)[e >> 1] = P::from_f2(split(ga).x, split(ga).y);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
template <typename Kern>
void allow_smem(Kern k, size_t bytes) {
  if (bytes > 48 * 1024) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  }
}

bool fast_layout_ok(int64_t BN, size_t elt, std::initializer_list<const void*> rows,
                    std::initializer_list<const void*> pairs) {
  if ((BN * int64_t(elt)) % 16 != 0) return false;
  for (const void* p : rows) {
    if (p != nullptr && !aligned_to(p, 16)) return false;
  }
  for (const void* p : pairs) {  // two-element accesses
    if (p != nullptr && !aligned_to(p, 2 * elt < 8 ? 8 : 2 * elt)) return false;
  }
  return true;
}

using Map = CUtensorMap;

// The tensor maps of one launch: the input rows the stages load (x), the
// spike-gradient rows (backward), and the output rows the stages store.
struct Maps {
  Map in, g, out;
};

template <typename T, int KIND, int RESET, int MODE, int RING = FwdCfg<T>::kRing,
          int MINB = FwdCfg<T>::kMinBlocks>
void fwd_fast_mode(const ScanFwdArgs& a, const Maps& om, cudaStream_t stream) {
  auto k = scan_fwd_fast_kernel<T, KIND, RESET, MODE, RING, MINB>;
  allow_smem(k, fwd_smem<T>(RING));
  k<<<static_cast<unsigned>(ceil_div(a.BN, kTileN)), kThreads, fwd_smem<T>(RING), stream>>>(
      a, pair_consts<MB_SURR_NONE>(a.decay, a.threshold, a.adapt_decay, a.beta, a.reset, 0.0f),
      om.in, om.out);
}

template <typename T, int KIND, int RESET>
void fwd_fast(const ScanFwdArgs& a, const Maps& om, cudaStream_t stream) {
  const bool d = a.spikes != nullptr, p = a.packed != nullptr, r = a.rates != nullptr;
  if (d && !p && !r) fwd_fast_mode<T, KIND, RESET, kFwdDense>(a, om, stream);
  else if (!d && p && !r) fwd_fast_mode<T, KIND, RESET, kFwdPacked>(a, om, stream);
  else if (!d && !p && r) fwd_fast_mode<T, KIND, RESET, kFwdRates>(a, om, stream);
  else fwd_fast_mode<T, KIND, RESET, kFwdAny>(a, om, stream);
}

template <typename T>
void fwd_fast_dispatch(int neuron, int reset_mode, const ScanFwdArgs& a, const Maps& om,
                       cudaStream_t stream) {
  if (neuron == kIzhikevich) {
    fwd_fast<T, kIzhikevich, MB_RESET_HARD>(a, om, stream);
  } else if (neuron == MB_LIF) {
    if (reset_mode == MB_RESET_HARD) fwd_fast<T, MB_LIF, MB_RESET_HARD>(a, om, stream);
    else fwd_fast<T, MB_LIF, MB_RESET_SUBTRACT>(a, om, stream);
  } else {
    if (reset_mode == MB_RESET_HARD) fwd_fast<T, MB_ALIF, MB_RESET_HARD>(a, om, stream);
    else fwd_fast<T, MB_ALIF, MB_RESET_SUBTRACT>(a, om, stream);
  }
}

template <typename T, int KIND, int RESET, int SURR, int MODE, int RING = BwdCfg<T>::kRing,
          int MINB = bwd_min_blocks(KIND, SURR, MODE)>
void bwd_fast_mode(const ScanBwdArgs& a, const Maps& om, cudaStream_t stream) {
  auto k = scan_bwd_fast_kernel<T, KIND, RESET, SURR, MODE, RING, MINB>;
  allow_smem(k, bwd_smem<T>(RING));
  k<<<static_cast<unsigned>(ceil_div(a.BN, kTileN)), kThreads, bwd_smem<T>(RING), stream>>>(
      a, pair_consts<SURR>(a.decay, a.threshold, a.adapt_decay, a.beta, a.reset, a.slope),
      om.in, om.g, om.out);
}

template <typename T, int KIND, int RESET, int SURR>
void bwd_fast(const ScanBwdArgs& a, const Maps& om, cudaStream_t stream) {
  const bool g = a.grad_spikes != nullptr, r = a.grad_rates != nullptr;
  if (g && !r) bwd_fast_mode<T, KIND, RESET, SURR, kBwdSpikes>(a, om, stream);
  else if (!g && r) bwd_fast_mode<T, KIND, RESET, SURR, kBwdRates>(a, om, stream);
  else bwd_fast_mode<T, KIND, RESET, SURR, kBwdAny>(a, om, stream);
}

template <typename T, int KIND, int RESET>
void bwd_fast_surr(int surrogate, const ScanBwdArgs& a, const Maps& om, cudaStream_t stream) {
  switch (surrogate) {
    case MB_SURR_SIGMOID: bwd_fast<T, KIND, RESET, MB_SURR_SIGMOID>(a, om, stream); break;
    case MB_SURR_FAST_SIGMOID: bwd_fast<T, KIND, RESET, MB_SURR_FAST_SIGMOID>(a, om, stream); break;
    case MB_SURR_ATAN: bwd_fast<T, KIND, RESET, MB_SURR_ATAN>(a, om, stream); break;
    case MB_SURR_TRIANGULAR: bwd_fast<T, KIND, RESET, MB_SURR_TRIANGULAR>(a, om, stream); break;
    case MB_SURR_SUPERSPIKE: bwd_fast<T, KIND, RESET, MB_SURR_SUPERSPIKE>(a, om, stream); break;
    case MB_SURR_MULTI_GAUSSIAN:
      bwd_fast<T, KIND, RESET, MB_SURR_MULTI_GAUSSIAN>(a, om, stream);
      break;
    default: bwd_fast<T, KIND, RESET, MB_SURR_NONE>(a, om, stream); break;
  }
}

template <typename T>
void bwd_fast_dispatch(int neuron, int reset_mode, int surrogate, const ScanBwdArgs& a,
                       const Maps& om, cudaStream_t stream) {
  if (neuron == MB_LIF) {
    if (reset_mode == MB_RESET_HARD) bwd_fast_surr<T, MB_LIF, MB_RESET_HARD>(surrogate, a, om, stream);
    else bwd_fast_surr<T, MB_LIF, MB_RESET_SUBTRACT>(surrogate, a, om, stream);
  } else {
    if (reset_mode == MB_RESET_HARD) bwd_fast_surr<T, MB_ALIF, MB_RESET_HARD>(surrogate, a, om, stream);
    else bwd_fast_surr<T, MB_ALIF, MB_RESET_SUBTRACT>(surrogate, a, om, stream);
  }
}

size_t dtype_size(int dtype) { return dtype == MB_F32 ? 4 : 2; }

// Tensor map over [T, BN] rows moved stage by stage (loaded inputs, stored
// outputs): box = one stage (kTileN neurons x kChunk rows), no swizzle (the
// stage is dense row-major).
bool make_stage_map(Map* map, const void* cptr, int dtype, int64_t BN, int64_t T) {
  void* ptr = const_cast<void*>(cptr);
  std::memset(map, 0, sizeof(Map));
  if (ptr == nullptr) return true;  // no such output: the kernel never uses the map
  auto fn = tma_encode_fn();
  if (fn == nullptr) return false;
  // coordinates are 32-bit in the store instruction
  if (BN > INT32_MAX || T > INT32_MAX) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(BN), static_cast<cuuint64_t>(T)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(BN) * dtype_size(dtype)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kTileN), static_cast<cuuint32_t>(kChunk)};
  cuuint32_t estride[2] = {1, 1};
  const CUtensorMapDataType dt = dtype == MB_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == MB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return fn(map, dt, 2, ptr, dims, strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool launch_scan_fwd_fast(int dtype, int neuron, int reset_mode, const ScanFwdArgs& a,
                          cudaStream_t stream) {
  const size_t elt = dtype_size(dtype);
  if (a.T <= 0) return false;
  if (a.packed != nullptr && (a.N % 32) != 0) return false;
  if (!fast_layout_ok(a.BN, elt, {a.x, a.spikes}, {a.v0, a.a0, a.vT, a.aT, a.rates, a.ckpt_v,
                                                   a.ckpt_a})) {
    return false;
  }
  Maps om;
  if (!make_stage_map(&om.in, a.x, dtype, a.BN, a.T) ||
      !make_stage_map(&om.out, a.spikes, dtype, a.BN, a.T)) {
    return false;
  }
  std::memset(&om.g, 0, sizeof(Map));
  switch (dtype) {
    case MB_F32: fwd_fast_dispatch<float>(neuron, reset_mode, a, om, stream); break;
    case MB_BF16: fwd_fast_dispatch<__nv_bfloat16>(neuron, reset_mode, a, om, stream); break;
    default: fwd_fast_dispatch<__half>(neuron, reset_mode, a, om, stream); break;
  }
  return true;
}

bool launch_scan_bwd_fast(int dtype, int neuron, int reset_mode, int surrogate,
                          const ScanBwdArgs& a, cudaStream_t stream) {
  const size_t elt = dtype_size(dtype);
  if (a.T <= 0) return false;
  if (!fast_layout_ok(a.BN, elt, {a.x, a.grad_x, a.grad_spikes, a.ckpt_v, a.ckpt_a},
                      {a.grad_rates, a.grad_vT, a.grad_aT, a.grad_v0, a.grad_a0})) {
    return false;
  }
  Maps om;
  if (!make_stage_map(&om.in, a.x, dtype, a.BN, a.T) ||
      !make_stage_map(&om.g, a.grad_spikes, dtype, a.BN, a.T) ||
      !make_stage_map(&om.out, a.grad_x, dtype, a.BN, a.T)) {
    return false;
  }
  switch (dtype) {
    case MB_F32: bwd_fast_dispatch<float>(neuron, reset_mode, surrogate, a, om, stream); break;
    case MB_BF16:
      bwd_fast_dispatch<__nv_bfloat16>(neuron, reset_mode, surrogate, a, om, stream);
      break;
    default: bwd_fast_dispatch<__half>(neuron, reset_mode, surrogate, a, om, stream); break;
  }
  return true;
}

int scan_fast_unit_status(bool clear) { return read_device_status(clear); }

cudaError_t scan_fast_unit_wait_probe(uint32_t polls, cudaStream_t stream) {
  wait_timeout_probe_kernel<<<1, 32, 0, stream>>>(polls);
  return cudaGetLastError();
}

}  // namespace mb
