// Warp-specialized LIF/ALIF scan kernels for 16-byte-aligned [T, B*N] rows.
//
// CTA = kConsumerWarps compute warps + 1 copy warp. The copy warp streams the
// CTA's tile (kTileN consecutive flat neurons) of every kChunk-step chunk into
// a ring of shared-memory stages with 1-D bulk async copies (the TMA engine);
// each stage has a "full" mbarrier (copy bytes landed) and an "empty" mbarrier
// (every compute warp is done with it). Compute threads own two neighbouring
// neurons each, so every smem read, global store and bf16 conversion moves a
// pair. No CTA-wide barrier is taken after set-up.
//
// Forward: the state is carried in fp32 registers; per step it writes dense
// spikes (a pair per store) and/or packed words (two ballots interleaved into
// two 32-neuron words per warp), and at each chunk start the fp32 checkpoint.
// Backward: chunks run last to first; each is replayed from its checkpoint
// into registers (bit-identical to the forward) and then walked in reverse.
#include <initializer_list>

#include "async_copy.cuh"
#include "common.cuh"
#include "scan_common.cuh"

namespace mb {

namespace {

constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kTileN = kConsumerWarps * 32 * 2;  // neurons per CTA
constexpr int kFwdRing = 4;                      // stages (chunks) in flight, forward
constexpr int kBwdRing = 3;                      // stages in flight, backward

template <typename T>
__host__ __device__ constexpr size_t fwd_smem() {
  return size_t(kFwdRing) * kChunk * kTileN * sizeof(T) + 2 * kFwdRing * sizeof(uint64_t);
}

// Backward stage: kChunk rows of x, kChunk rows of grad_spikes, then the fp32
// checkpoint rows (membrane, adaptation) of the chunk.
template <typename T>
__host__ __device__ constexpr size_t bwd_stage_bytes() {
  return size_t(2) * kChunk * kTileN * sizeof(T) + 2 * kTileN * sizeof(float);
}

template <typename T>
__host__ __device__ constexpr size_t bwd_smem() {
  return size_t(kBwdRing) * bwd_stage_bytes<T>() + 2 * kBwdRing * sizeof(uint64_t);
}

// Output modes of the forward (what the caller asked for), fixed at compile
// time so the per-step code has no branches: dense spikes, packed words,
// spike rates, or any combination (checked at run time).
enum FwdMode { kFwdDense = 0, kFwdPacked = 1, kFwdRates = 2, kFwdAny = 3 };
// Backward inputs: spike gradients, rate gradients, or any combination.
enum BwdMode { kBwdSpikes = 0, kBwdRates = 1, kBwdAny = 2 };

template <typename T>
__device__ __forceinline__ void queue_chunk_rows(T* dst, const T* src, int64_t t0, int len,
                                                 int64_t BN, int64_t e0, uint32_t row_bytes,
                                                 uint64_t* bar) {
  for (int j = 0; j < len; ++j) {
    bulk_copy_g2s(dst + j * kTileN, src + (t0 + j) * BN + e0, row_bytes, bar);
  }
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
template <typename T, int KIND, int RESET, int MODE>
__global__ void __launch_bounds__(kThreads) scan_fwd_fast_kernel(const ScanFwdArgs a) {
  using P = Pair<T>;
  using V = typename P::V;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* ring = reinterpret_cast<T*>(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + size_t(kFwdRing) * kChunk * kTileN * sizeof(T));
  uint64_t* empty = full + kFwdRing;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t e0 = int64_t(blockIdx.x) * kTileN;
  const int tile_n = static_cast<int>(imin64(kTileN, a.BN - e0));
  const int64_t K = (a.T + kChunk - 1) / kChunk;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFwdRing; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // copy warp: one lane streams every chunk of this tile through the ring
    if (lane == 0) {
      const T* x = static_cast<const T*>(a.x);
      const uint32_t row_bytes = uint32_t(tile_n) * uint32_t(sizeof(T));
      for (int64_t k = 0; k < K; ++k) {
        const int s = static_cast<int>(k % kFwdRing);
        if (k >= kFwdRing &&
            !mbar_wait_bounded(&empty[s], static_cast<uint32_t>(((k / kFwdRing) - 1) & 1))) {
          break;
        }
        const int64_t t0 = k * kChunk;
        const int len = static_cast<int>(imin64(kChunk, a.T - t0));
        mbar_arrive_expect_tx(&full[s], row_bytes * uint32_t(len));
        queue_chunk_rows(ring + s * kChunk * kTileN, x, t0, len, a.BN, e0, row_bytes, &full[s]);
      }
    }
    return;
  }

  const int tid = threadIdx.x;  // 0 .. 32*kConsumerWarps-1
  const bool valid = 2 * tid < tile_n;  // tile_n is even
  const int64_t e = e0 + 2 * tid;
  const int64_t half_bn = a.BN >> 1;  // BN is even on this path

  float m0 = 0.f, m1 = 0.f, ad0 = 0.f, ad1 = 0.f;
  int c0 = 0, c1 = 0;
  if (valid) {
    const float2 v = P::to_f2(reinterpret_cast<const V*>(a.v0)[e >> 1]);
    m0 = v.x;
    m1 = v.y;
    if (KIND == MB_ALIF) {
      const float2 av = P::to_f2(reinterpret_cast<const V*>(a.a0)[e >> 1]);
      ad0 = av.x;
      ad1 = av.y;
    }
  }
  const float decay = a.decay, thr = a.threshold, reset_v = a.reset;
  const float adapt_decay = a.adapt_decay, beta = a.beta;

  constexpr bool kDense = MODE == kFwdDense || MODE == kFwdAny;
  constexpr bool kPacked = MODE == kFwdPacked || MODE == kFwdAny;
  constexpr bool kRates = MODE == kFwdRates || MODE == kFwdAny;
  const bool do_dense = kDense && (MODE != kFwdAny || a.spikes != nullptr);
  const bool do_packed = kPacked && (MODE != kFwdAny || a.packed != nullptr);
  V* sp = do_dense ? reinterpret_cast<V*>(a.spikes) + (e >> 1) : nullptr;
  // packed words: this warp's 64 neurons are flat words q and q+1; with
  // N % 32 == 0 every word lies wholly inside or wholly outside the tile
  const int64_t words_per_t = a.BN >> 5;
  const int64_t q = (e0 >> 5) + 2 * warp + (lane >> 4);
  int32_t* pk = do_packed ? a.packed + q : nullptr;
  const bool pk_lane = (lane & 15) == 0 && (q << 5) < a.BN;
  const int sh = lane & 16;  // lanes 0-15 -> word q, lanes 16-31 -> word q+1

  auto step = [&](V xv) {
    const float2 xf = P::to_f2(xv);
    Step<KIND, RESET> s0, s1;
    s0.run(m0, ad0, xf.x, decay, thr, reset_v, adapt_decay, beta);
    s1.run(m1, ad1, xf.y, decay, thr, reset_v, adapt_decay, beta);
    if (kRates) {
      c0 += s0.s ? 1 : 0;
      c1 += s1.s ? 1 : 0;
    }
    if (kDense && (MODE != kFwdAny || sp != nullptr)) {
      if (valid) *sp = P::spikes(s0.s, s1.s);
      sp += half_bn;
    }
    if (kPacked && (MODE != kFwdAny || pk != nullptr)) {
      const uint32_t even = __ballot_sync(0xffffffffu, s0.s);
      const uint32_t odd = __ballot_sync(0xffffffffu, s1.s);
      const uint32_t word = spread_even_bits(even >> sh) | (spread_even_bits(odd >> sh) << 1);
      if (pk_lane) *pk = static_cast<int32_t>(word);
      pk += words_per_t;
    }
  };

  for (int64_t k = 0; k < K; ++k) {
    const int s = static_cast<int>(k % kFwdRing);
    if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>((k / kFwdRing) & 1))) return;
    if (a.ckpt_v != nullptr && valid) {
      reinterpret_cast<float2*>(a.ckpt_v + k * a.BN)[e >> 1] = make_float2(m0, m1);
      if (KIND == MB_ALIF) reinterpret_cast<float2*>(a.ckpt_a + k * a.BN)[e >> 1] = make_float2(ad0, ad1);
    }
    const V* row = reinterpret_cast<const V*>(ring + s * kChunk * kTileN) + tid;
    const int len = static_cast<int>(imin64(kChunk, a.T - k * kChunk));
    if (len == kChunk) {
#pragma unroll
      for (int j = 0; j < kChunk; ++j) step(row[j * (kTileN / 2)]);
    } else {
      for (int j = 0; j < len; ++j) step(row[j * (kTileN / 2)]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  if (!valid) return;
  if (a.vT) reinterpret_cast<V*>(a.vT)[e >> 1] = P::from_f2(m0, m1);
  if (KIND == MB_ALIF && a.aT) reinterpret_cast<V*>(a.aT)[e >> 1] = P::from_f2(ad0, ad1);
  if (kRates && a.rates) {
    const float tf = static_cast<float>(a.T);
    reinterpret_cast<V*>(a.rates)[e >> 1] =
        P::from_f2(__fdiv_rn(static_cast<float>(c0), tf), __fdiv_rn(static_cast<float>(c1), tf));
  }
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------
template <typename T, int KIND, int RESET, int SURR, int MODE>
__global__ void __launch_bounds__(kThreads, KIND == MB_ALIF ? 3 : 4) scan_bwd_fast_kernel(const ScanBwdArgs a) {
  using P = Pair<T>;
  using V = typename P::V;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + kBwdRing * bwd_stage_bytes<T>());
  uint64_t* empty = full + kBwdRing;
  auto stage_x = [&](int s) { return reinterpret_cast<T*>(smem_raw + s * bwd_stage_bytes<T>()); };
  auto stage_g = [&](int s) { return stage_x(s) + kChunk * kTileN; };
  auto stage_c = [&](int s) { return reinterpret_cast<float*>(stage_g(s) + kChunk * kTileN); };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t e0 = int64_t(blockIdx.x) * kTileN;
  const int tile_n = static_cast<int>(imin64(kTileN, a.BN - e0));
  const int64_t K = (a.T + kChunk - 1) / kChunk;
  constexpr bool kSpikes = MODE == kBwdSpikes || MODE == kBwdAny;
  constexpr bool kRateGrad = MODE == kBwdRates || MODE == kBwdAny;
  const bool has_gs = kSpikes && (MODE != kBwdAny || a.grad_spikes != nullptr);
  const bool has_alif = KIND == MB_ALIF;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kBwdRing; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    if (lane == 0) {
      const T* x = static_cast<const T*>(a.x);
      const T* gs = static_cast<const T*>(a.grad_spikes);
      const uint32_t row_bytes = uint32_t(tile_n) * uint32_t(sizeof(T));
      for (int64_t i = 0; i < K; ++i) {
        const int s = static_cast<int>(i % kBwdRing);
        if (i >= kBwdRing &&
            !mbar_wait_bounded(&empty[s], static_cast<uint32_t>(((i / kBwdRing) - 1) & 1))) {
          break;
        }
        const int64_t k = K - 1 - i;
        const int64_t t0 = k * kChunk;
        const int len = static_cast<int>(imin64(kChunk, a.T - t0));
        const uint32_t ckpt_bytes = uint32_t(tile_n) * 4u;
        mbar_arrive_expect_tx(&full[s], row_bytes * uint32_t(len) * (has_gs ? 2u : 1u) +
                                            ckpt_bytes * (has_alif ? 2u : 1u));
        queue_chunk_rows(stage_x(s), x, t0, len, a.BN, e0, row_bytes, &full[s]);
        if (has_gs) queue_chunk_rows(stage_g(s), gs, t0, len, a.BN, e0, row_bytes, &full[s]);
        bulk_copy_g2s(stage_c(s), a.ckpt_v + k * a.BN + e0, ckpt_bytes, &full[s]);
        if (has_alif) bulk_copy_g2s(stage_c(s) + kTileN, a.ckpt_a + k * a.BN + e0, ckpt_bytes, &full[s]);
      }
    }
    return;
  }

  const int tid = threadIdx.x;
  const bool valid = 2 * tid < tile_n;
  const int64_t e = e0 + 2 * tid;
  const int64_t half_bn = a.BN >> 1;
  const float decay = a.decay, thr = a.threshold, reset_v = a.reset;
  const float adapt_decay = a.adapt_decay, beta = a.beta;
  const SurrogateD<SURR> dfun(a.slope);

  float gm0 = 0.f, gm1 = 0.f, ga0 = 0.f, ga1 = 0.f, gr0 = 0.f, gr1 = 0.f;
  if (valid) {
    if (a.grad_vT) {
      const float2 v = P::to_f2(reinterpret_cast<const V*>(a.grad_vT)[e >> 1]);
      gm0 = v.x;
      gm1 = v.y;
    }
    if (KIND == MB_ALIF && a.grad_aT) {
      const float2 v = P::to_f2(reinterpret_cast<const V*>(a.grad_aT)[e >> 1]);
      ga0 = v.x;
      ga1 = v.y;
    }
    if (kRateGrad && a.grad_rates) {
      // the grad of a rate output reaches every step as grad_rates / T
      // (src/myelin/autograd.py:842-844)
      const float2 v = P::to_f2(reinterpret_cast<const V*>(a.grad_rates)[e >> 1]);
      const float tf = static_cast<float>(a.T);
      gr0 = __fdiv_rn(v.x, tf);
      gr1 = __fdiv_rn(v.y, tf);
    }
  }

  // One reverse step for one neuron; returns dL/dx_t and updates gm, ga.
  auto adjoint = [&](float p, float th, float gsum, float& gm, float& ga) -> float {
    const float d = dfun(p - th);
    float gp;
    if (KIND == MB_LIF) {
      if (RESET == MB_RESET_HARD) {
        const float sf = p >= th ? 1.0f : 0.0f;
        gp = gm * ((1.0f - sf) + (reset_v - p) * d) + gsum * d;
      } else {
        gp = gm + (gsum - gm * th) * d;
      }
    } else {
      if (RESET == MB_RESET_HARD) {
        const float Gs = gsum + gm * (reset_v - p) + ga;
        const float Gd = Gs * d;
        gp = (p >= th ? 0.0f : gm) + Gd;
        ga = ga * adapt_decay - beta * Gd;
      } else {
        const float Gs = gsum - gm * th + ga;
        const float Gd = Gs * d;
        gp = gm + Gd;
        ga = ga * adapt_decay - beta * ((p >= th ? gm : 0.0f) + Gd);
      }
    }
    gm = gp * decay;
    return gp;
  };

  V* gxp = reinterpret_cast<V*>(a.grad_x) + (e >> 1);
  for (int64_t i = 0; i < K; ++i) {
    const int s = static_cast<int>(i % kBwdRing);
    const int64_t k = K - 1 - i;
    const int64_t t0 = k * kChunk;
    const int len = static_cast<int>(imin64(kChunk, a.T - t0));
    if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>((i / kBwdRing) & 1))) return;
    const V* xrow = reinterpret_cast<const V*>(stage_x(s)) + tid;
    const V* grow = reinterpret_cast<const V*>(stage_g(s)) + tid;
    if (valid) {
      const float2 mv = reinterpret_cast<const float2*>(stage_c(s))[tid];
      float m0 = mv.x, m1 = mv.y, av0 = 0.f, av1 = 0.f;
      if (KIND == MB_ALIF) {
        const float2 avv = reinterpret_cast<const float2*>(stage_c(s) + kTileN)[tid];
        av0 = avv.x;
        av1 = avv.y;
      }
      float P0[kChunk], P1[kChunk], TH0[kChunk], TH1[kChunk];
      V* out = gxp + (t0 + len - 1) * half_bn;
      auto replay = [&](int j) {
        const float2 xf = P::to_f2(xrow[j * (kTileN / 2)]);
        Step<KIND, RESET> s0, s1;
        s0.run(m0, av0, xf.x, decay, thr, reset_v, adapt_decay, beta);
        s1.run(m1, av1, xf.y, decay, thr, reset_v, adapt_decay, beta);
        P0[j] = s0.p;
        P1[j] = s1.p;
        TH0[j] = s0.theta;
        TH1[j] = s1.theta;
      };
      auto reverse = [&](int j) {
        float g0 = gr0, g1 = gr1;
        if (MODE == kBwdSpikes) {
          const float2 gf = P::to_f2(grow[j * (kTileN / 2)]);
          g0 = gf.x;
          g1 = gf.y;
        } else if (has_gs) {
          const float2 gf = P::to_f2(grow[j * (kTileN / 2)]);
          g0 += gf.x;
          g1 += gf.y;
        }
        const float gp0 = adjoint(P0[j], TH0[j], g0, gm0, ga0);
        const float gp1 = adjoint(P1[j], TH1[j], g1, gm1, ga1);
        *out = P::from_f2(gp0, gp1);
        out -= half_bn;
      };
      if (len == kChunk) {
#pragma unroll
        for (int j = 0; j < kChunk; ++j) replay(j);
#pragma unroll
        for (int j = kChunk - 1; j >= 0; --j) reverse(j);
      } else {
#pragma unroll
        for (int j = 0; j < kChunk; ++j) {
          if (j < len) replay(j);
        }
#pragma unroll
        for (int j = kChunk - 1; j >= 0; --j) {
          if (j < len) reverse(j);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (!valid) return;
  if (a.grad_v0) reinterpret_cast<V*>(a.grad_v0)[e >> 1] = P::from_f2(gm0, gm1);
  if (KIND == MB_ALIF && a.grad_a0) reinterpret_cast<V*>(a.grad_a0)[e >> 1] = P::from_f2(ga0, ga1);
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

template <typename T, int KIND, int RESET, int MODE>
void fwd_fast_mode(const ScanFwdArgs& a, cudaStream_t stream) {
  auto k = scan_fwd_fast_kernel<T, KIND, RESET, MODE>;
  allow_smem(k, fwd_smem<T>());
  k<<<static_cast<unsigned>(ceil_div(a.BN, kTileN)), kThreads, fwd_smem<T>(), stream>>>(a);
}

template <typename T, int KIND, int RESET>
void fwd_fast(const ScanFwdArgs& a, cudaStream_t stream) {
  const bool d = a.spikes != nullptr, p = a.packed != nullptr, r = a.rates != nullptr;
  if (d && !p && !r) fwd_fast_mode<T, KIND, RESET, kFwdDense>(a, stream);
  else if (!d && p && !r) fwd_fast_mode<T, KIND, RESET, kFwdPacked>(a, stream);
  else if (!d && !p && r) fwd_fast_mode<T, KIND, RESET, kFwdRates>(a, stream);
  else fwd_fast_mode<T, KIND, RESET, kFwdAny>(a, stream);
}

template <typename T>
void fwd_fast_dispatch(int neuron, int reset_mode, const ScanFwdArgs& a, cudaStream_t stream) {
  if (neuron == MB_LIF) {
    if (reset_mode == MB_RESET_HARD) fwd_fast<T, MB_LIF, MB_RESET_HARD>(a, stream);
    else fwd_fast<T, MB_LIF, MB_RESET_SUBTRACT>(a, stream);
  } else {
    if (reset_mode == MB_RESET_HARD) fwd_fast<T, MB_ALIF, MB_RESET_HARD>(a, stream);
    else fwd_fast<T, MB_ALIF, MB_RESET_SUBTRACT>(a, stream);
  }
}

template <typename T, int KIND, int RESET, int SURR, int MODE>
void bwd_fast_mode(const ScanBwdArgs& a, cudaStream_t stream) {
  auto k = scan_bwd_fast_kernel<T, KIND, RESET, SURR, MODE>;
  allow_smem(k, bwd_smem<T>());
  k<<<static_cast<unsigned>(ceil_div(a.BN, kTileN)), kThreads, bwd_smem<T>(), stream>>>(a);
}

template <typename T, int KIND, int RESET, int SURR>
void bwd_fast(const ScanBwdArgs& a, cudaStream_t stream) {
  const bool g = a.grad_spikes != nullptr, r = a.grad_rates != nullptr;
  if (g && !r) bwd_fast_mode<T, KIND, RESET, SURR, kBwdSpikes>(a, stream);
  else if (!g && r) bwd_fast_mode<T, KIND, RESET, SURR, kBwdRates>(a, stream);
  else bwd_fast_mode<T, KIND, RESET, SURR, kBwdAny>(a, stream);
}

template <typename T, int KIND, int RESET>
void bwd_fast_surr(int surrogate, const ScanBwdArgs& a, cudaStream_t stream) {
  switch (surrogate) {
    case MB_SURR_SIGMOID: bwd_fast<T, KIND, RESET, MB_SURR_SIGMOID>(a, stream); break;
    case MB_SURR_FAST_SIGMOID: bwd_fast<T, KIND, RESET, MB_SURR_FAST_SIGMOID>(a, stream); break;
    case MB_SURR_ATAN: bwd_fast<T, KIND, RESET, MB_SURR_ATAN>(a, stream); break;
    case MB_SURR_TRIANGULAR: bwd_fast<T, KIND, RESET, MB_SURR_TRIANGULAR>(a, stream); break;
    case MB_SURR_SUPERSPIKE: bwd_fast<T, KIND, RESET, MB_SURR_SUPERSPIKE>(a, stream); break;
    case MB_SURR_MULTI_GAUSSIAN: bwd_fast<T, KIND, RESET, MB_SURR_MULTI_GAUSSIAN>(a, stream); break;
    default: bwd_fast<T, KIND, RESET, MB_SURR_NONE>(a, stream); break;
  }
}

template <typename T>
void bwd_fast_dispatch(int neuron, int reset_mode, int surrogate, const ScanBwdArgs& a,
                       cudaStream_t stream) {
  if (neuron == MB_LIF) {
    if (reset_mode == MB_RESET_HARD) bwd_fast_surr<T, MB_LIF, MB_RESET_HARD>(surrogate, a, stream);
    else bwd_fast_surr<T, MB_LIF, MB_RESET_SUBTRACT>(surrogate, a, stream);
  } else {
    if (reset_mode == MB_RESET_HARD) bwd_fast_surr<T, MB_ALIF, MB_RESET_HARD>(surrogate, a, stream);
    else bwd_fast_surr<T, MB_ALIF, MB_RESET_SUBTRACT>(surrogate, a, stream);
  }
}

size_t dtype_size(int dtype) { return dtype == MB_F32 ? 4 : 2; }

}  // namespace

bool launch_scan_fwd_fast(int dtype, int neuron, int reset_mode, const ScanFwdArgs& a,
                          cudaStream_t stream) {
  const size_t elt = dtype_size(dtype);
  if (a.T <= 0) return false;
  if (a.packed != nullptr && (a.N % 32) != 0) return false;
  if (!fast_layout_ok(a.BN, elt, {a.x}, {a.v0, a.a0, a.vT, a.aT, a.spikes, a.rates, a.ckpt_v,
                                        a.ckpt_a})) {
    return false;
  }
  switch (dtype) {
    case MB_F32: fwd_fast_dispatch<float>(neuron, reset_mode, a, stream); break;
    case MB_BF16: fwd_fast_dispatch<__nv_bfloat16>(neuron, reset_mode, a, stream); break;
    default: fwd_fast_dispatch<__half>(neuron, reset_mode, a, stream); break;
  }
  return true;
}

bool launch_scan_bwd_fast(int dtype, int neuron, int reset_mode, int surrogate,
                          const ScanBwdArgs& a, cudaStream_t stream) {
  const size_t elt = dtype_size(dtype);
  if (a.T <= 0) return false;
  if (!fast_layout_ok(a.BN, elt, {a.x, a.grad_spikes, a.ckpt_v, a.ckpt_a},
                      {a.grad_x, a.grad_rates, a.grad_vT, a.grad_aT, a.grad_v0, a.grad_a0})) {
    return false;
  }
  switch (dtype) {
    case MB_F32: bwd_fast_dispatch<float>(neuron, reset_mode, surrogate, a, stream); break;
    case MB_BF16: bwd_fast_dispatch<__nv_bfloat16>(neuron, reset_mode, surrogate, a, stream); break;
    default: bwd_fast_dispatch<__half>(neuron, reset_mode, surrogate, a, stream); break;
  }
  return true;
}

}  // namespace mb
