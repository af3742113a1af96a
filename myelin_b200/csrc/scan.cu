// Fused-time LIF / ALIF membrane scan and its reverse-time surrogate backward.
//
// Layout: x, spikes, grad tensors are time-major [T, B, N] (C-contiguous), the
// state is [B, N]. One warp owns 32*NPT consecutive neurons of one batch row
// for all T steps, so every time step is one coalesced vector load per thread
// and the 32-neuron spike words of the packed output are formed inside the
// warp (ballot / shuffle-OR) and stored with one int32 store per word.
//
// Numerics (bit-exact contract with the reference forward,
// src/myelin/neurons.py:106-128): the recurrence is evaluated in fp32 with
// two roundings and no FMA contraction, p = fl(fl(m*decay) + x),
// theta = fl(thr + fl(beta*a)), s = p >= theta. 16-bit I/O is widened to fp32
// on load; the carry stays fp32.
#include <cstdio>

#include "async_copy.cuh"
#include "common.cuh"
#include "exchange.cuh"
#include "scan_common.cuh"

namespace mb {

// ---------------------------------------------------------------------------
// Forward scan.
// ---------------------------------------------------------------------------
template <typename T, int NPT, int KIND, int RESET>
__global__ void __launch_bounds__(kBlock) scan_fwd_kernel(const ScanFwdArgs a) {
  using E = Elem<T>;
  constexpr int kLanesPerWord = 32 / NPT;
  constexpr int kDepth = 8;  // time steps of loads issued ahead of the math

  const int lane = threadIdx.x & 31;
  const int64_t warp = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t row = warp / a.groups_per_row;
  if (row >= a.B) return;  // warp-uniform
  const int64_t g = warp - row * a.groups_per_row;
  const int64_t n0 = g * (32 * NPT) + int64_t(lane) * NPT;
  const bool valid = n0 < a.N;  // NPT > 1 is only used when N % NPT == 0
  const int64_t e = row * a.N + n0;

  const T* __restrict__ x = static_cast<const T*>(a.x);
  float m[NPT], ad[NPT];
  int cnt[NPT];
#pragma unroll
  for (int i = 0; i < NPT; ++i) {
    m[i] = 0.0f;
    ad[i] = 0.0f;
    cnt[i] = 0;
  }
  if (valid) {
    const Vec<T, NPT> v = load_vec<T, NPT>(static_cast<const T*>(a.v0) + e);
#pragma unroll
    for (int i = 0; i < NPT; ++i) m[i] = E::to_f(v.v[i]);
    if (KIND == MB_ALIF) {
      const Vec<T, NPT> av = load_vec<T, NPT>(static_cast<const T*>(a.a0) + e);
#pragma unroll
      for (int i = 0; i < NPT; ++i) ad[i] = E::to_f(av.v[i]);
    }
  }

  const float decay = a.decay, thr = a.threshold, reset_v = a.reset;
  const float adapt_decay = a.adapt_decay, beta = a.beta;
  T* __restrict__ spikes = static_cast<T*>(a.spikes);

  for (int64_t t0 = 0; t0 < a.T; t0 += kDepth) {
    Vec<T, NPT> xb[kDepth];
#pragma unroll
    for (int j = 0; j < kDepth; ++j) {
      if (valid && t0 + j < a.T) {
        xb[j] = load_vec<T, NPT>(x + (t0 + j) * a.BN + e);
      } else {
#pragma unroll
        for (int i = 0; i < NPT; ++i) xb[j].v[i] = E::zero();
      }
    }
#pragma unroll
    for (int j = 0; j < kDepth; ++j) {
      const int64_t t = t0 + j;
      if (t >= a.T) break;  // warp-uniform
      if (a.ckpt_v != nullptr && (t % kChunk) == 0 && valid) {
        const int64_t c = (t / kChunk) * a.BN + e;
#pragma unroll
        for (int i = 0; i < NPT; ++i) a.ckpt_v[c + i] = m[i];
        if (KIND == MB_ALIF) {
#pragma unroll
          for (int i = 0; i < NPT; ++i) a.ckpt_a[c + i] = ad[i];
        }
      }
      uint32_t bits = 0;
      Vec<T, NPT> sv;
#pragma unroll
      for (int i = 0; i < NPT; ++i) {
        Step<KIND, RESET> st;
        st.run(m[i], ad[i], E::to_f(xb[j].v[i]), decay, thr, reset_v, adapt_decay, beta);
        bits |= uint32_t(st.s) << i;
        cnt[i] += st.s ? 1 : 0;
        sv.v[i] = st.s ? E::one() : E::zero();
      }
      if (spikes != nullptr && valid) store_vec<T, NPT>(spikes + t * a.BN + e, sv);
      if (a.packed != nullptr) {
        uint32_t word;
        if (NPT == 1) {
          word = __ballot_sync(0xffffffffu, bits != 0);
        } else {
          word = bits << ((lane % kLanesPerWord) * NPT);
#pragma unroll
          for (int off = 1; off < kLanesPerWord; off <<= 1) {
            word |= __shfl_xor_sync(0xffffffffu, word, off);
          }
        }
        if ((lane % kLanesPerWord) == 0) {
          const int64_t wi = g * NPT + lane / kLanesPerWord;
          if (wi < a.words_per_row) {
            a.packed[(t * a.B + row) * a.words_per_row + wi] = static_cast<int32_t>(word);
          }
        }
      }
    }
  }

  if (!valid) return;
  if (a.vT != nullptr) {
    Vec<T, NPT> v;
#pragma unroll
    for (int i = 0; i < NPT; ++i) v.v[i] = E::from_f(m[i]);
    store_vec<T, NPT>(static_cast<T*>(a.vT) + e, v);
  }
  if (KIND == MB_ALIF && a.aT != nullptr) {
    Vec<T, NPT> v;
#pragma unroll
    for (int i = 0; i < NPT; ++i) v.v[i] = E::from_f(ad[i]);
    store_vec<T, NPT>(static_cast<T*>(a.aT) + e, v);
  }
  if (a.rates != nullptr) {
    const float tf = static_cast<float>(a.T);
    Vec<T, NPT> v;
#pragma unroll
    for (int i = 0; i < NPT; ++i) v.v[i] = E::from_f(__fdiv_rn(static_cast<float>(cnt[i]), tf));
    store_vec<T, NPT>(static_cast<T*>(a.rates) + e, v);
  }
}

// ---------------------------------------------------------------------------
// Tiled kernels: one CTA owns kTile consecutive flat neurons (index b*N + n)
// for all T steps, one neuron per thread. The x (and grad_spikes) rows of a
// chunk of kChunk steps are staged in shared memory, by the copy engine
// (1-D bulk async copies, one per row, tracked by an mbarrier) when every row
// is 16-byte aligned, else by the threads themselves. Staging keeps the loads
// in flight off the register file, which the backward needs for its replay.
// ---------------------------------------------------------------------------
constexpr int kTile = 256;
constexpr int kFwdStages = 3;
constexpr int kBwdStages = 2;

template <typename T>
__host__ __device__ constexpr size_t fwd_smem_bytes() {
  return size_t(kFwdStages) * kChunk * kTile * sizeof(T) + kFwdStages * sizeof(uint64_t);
}

template <typename T>
__host__ __device__ constexpr size_t bwd_smem_bytes() {
  return size_t(2) * kBwdStages * kChunk * kTile * sizeof(T) + kBwdStages * sizeof(uint64_t);
}

// Thread 0 of a CTA queues the rows [t0, t0 + len) of one [T, BN] tensor
// (tile columns [e0, e0 + tile_n)) into smem rows of stride kTile.
template <typename T>
__device__ __forceinline__ void queue_rows(T* dst, const T* src, int64_t t0, int len, int64_t BN,
                                           int64_t e0, uint32_t row_bytes, uint64_t* bar) {
  for (int j = 0; j < len; ++j) {
    bulk_copy_g2s(dst + j * kTile, src + (t0 + j) * BN + e0, row_bytes, bar);
  }
}

// Every thread copies its own column of the rows (no cross-thread sharing).
template <typename T>
__device__ __forceinline__ void fill_rows(T* dst, const T* src, int64_t t0, int len, int64_t BN,
                                          int64_t e, int tid) {
#pragma unroll 4
  for (int j = 0; j < len; ++j) dst[j * kTile + tid] = src[(t0 + j) * BN + e];
}

template <typename T, int KIND, int RESET, bool TMA>
__global__ void __launch_bounds__(kTile) scan_fwd_tiled_kernel(const ScanFwdArgs a) {
  using E = Elem<T>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* xs = reinterpret_cast<T*>(smem_raw);  // [kFwdStages][kChunk][kTile]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + size_t(kFwdStages) * kChunk * kTile * sizeof(T));

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int64_t e0 = int64_t(blockIdx.x) * kTile;
  const int tile_n = static_cast<int>(imin64(kTile, a.BN - e0));
  const bool valid = tid < tile_n;
  const int64_t e = e0 + tid;
  const int64_t K = (a.T + kChunk - 1) / kChunk;
  const T* __restrict__ x = static_cast<const T*>(a.x);
  T* __restrict__ spikes = static_cast<T*>(a.spikes);
  const uint32_t row_bytes = uint32_t(tile_n) * uint32_t(sizeof(T));

  if (TMA) {
    if (tid == 0) {
      for (int s = 0; s < kFwdStages; ++s) mbar_init(&bars[s], 1);
      fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) {
      for (int64_t k = 0; k < imin64(kFwdStages, K); ++k) {
        const int64_t t0 = k * kChunk;
        const int len = static_cast<int>(imin64(kChunk, a.T - t0));
        mbar_arrive_expect_tx(&bars[k], row_bytes * len);
        queue_rows(xs + k * kChunk * kTile, x, t0, len, a.BN, e0, row_bytes, &bars[k]);
      }
    }
  }

  float m = 0.0f, ad = 0.0f;
  int cnt = 0;
  if (valid) {
    m = E::to_f(static_cast<const T*>(a.v0)[e]);
    if (KIND == MB_ALIF) ad = E::to_f(static_cast<const T*>(a.a0)[e]);
  }
  const float decay = a.decay, thr = a.threshold, reset_v = a.reset;
  const float adapt_decay = a.adapt_decay, beta = a.beta;
  const int64_t words_per_t = a.BN >> 5;  // packed path requires N % 32 == 0

  for (int64_t k = 0; k < K; ++k) {
    const int s = static_cast<int>(k % kFwdStages);
    const int64_t t0 = k * kChunk;
    const int len = static_cast<int>(imin64(kChunk, a.T - t0));
    T* stage = xs + s * kChunk * kTile;
    bool ok = true;
    if (TMA) {
      ok = mbar_wait_bounded(&bars[s], static_cast<uint32_t>((k / kFwdStages) & 1));
    } else if (valid) {
      fill_rows(stage, x, t0, len, a.BN, e, tid);
    }
    if (a.ckpt_v != nullptr && valid) {
      a.ckpt_v[k * a.BN + e] = m;
      if (KIND == MB_ALIF) a.ckpt_a[k * a.BN + e] = ad;
    }
#pragma unroll 4
    for (int j = 0; j < len; ++j) {
      const int64_t t = t0 + j;
      Step<KIND, RESET> st;
      st.run(m, ad, E::to_f(stage[j * kTile + tid]), decay, thr, reset_v, adapt_decay, beta);
      const bool sp = valid && st.s;
      cnt += sp ? 1 : 0;
      if (spikes != nullptr && valid) spikes[t * a.BN + e] = sp ? E::one() : E::zero();
      if (a.packed != nullptr) {
        const uint32_t word = __ballot_sync(0xffffffffu, sp);
        const int64_t q = (e0 >> 5) + (tid >> 5);
        if (lane == 0 && (q << 5) < a.BN) a.packed[t * words_per_t + q] = static_cast<int32_t>(word);
      }
    }
    if (TMA) {
      // every thread is done with this stage; refill it with chunk k + kFwdStages
      if (__syncthreads_or(!ok)) {
        if (tid == 0) {
          for (int64_t kk = k + 1; kk < imin64(k + kFwdStages, K); ++kk) {
            mbar_wait_bounded(&bars[kk % kFwdStages], static_cast<uint32_t>((kk / kFwdStages) & 1));
          }
        }
        return;
      }
      const int64_t kn = k + kFwdStages;
      if (tid == 0 && kn < K) {
        fence_proxy_async_smem();
        const int64_t tn = kn * kChunk;
        const int ln = static_cast<int>(imin64(kChunk, a.T - tn));
        mbar_arrive_expect_tx(&bars[s], row_bytes * ln);
        queue_rows(stage, x, tn, ln, a.BN, e0, row_bytes, &bars[s]);
      }
    }
  }

  if (!valid) return;
  if (a.vT != nullptr) static_cast<T*>(a.vT)[e] = E::from_f(m);
  if (KIND == MB_ALIF && a.aT != nullptr) static_cast<T*>(a.aT)[e] = E::from_f(ad);
  if (a.rates != nullptr) {
    static_cast<T*>(a.rates)[e] =
        E::from_f(__fdiv_rn(static_cast<float>(cnt), static_cast<float>(a.T)));
  }
}

// Backward: chunks from last to first. Each chunk is replayed from its fp32
// checkpoint into registers (P, TH: bit-identical to the forward) and then
// walked in reverse with the adjoint recurrence.
template <typename T, int KIND, int RESET, int SURR, bool TMA>
__global__ void __launch_bounds__(kTile) scan_bwd_tiled_kernel(const ScanBwdArgs a) {
  using E = Elem<T>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  T* xs = reinterpret_cast<T*>(smem_raw);          // [kBwdStages][kChunk][kTile]
  T* gss = xs + kBwdStages * kChunk * kTile;       // [kBwdStages][kChunk][kTile]
  uint64_t* bars = reinterpret_cast<uint64_t*>(gss + kBwdStages * kChunk * kTile);

  const int tid = threadIdx.x;
  const int64_t e0 = int64_t(blockIdx.x) * kTile;
  const int tile_n = static_cast<int>(imin64(kTile, a.BN - e0));
  const bool valid = tid < tile_n;
  const int64_t e = e0 + tid;
  const int64_t K = (a.T + kChunk - 1) / kChunk;
  const T* __restrict__ x = static_cast<const T*>(a.x);
  const T* __restrict__ gs = static_cast<const T*>(a.grad_spikes);
  T* __restrict__ gx = static_cast<T*>(a.grad_x);
  const uint32_t row_bytes = uint32_t(tile_n) * uint32_t(sizeof(T));
  const int n_src = gs != nullptr ? 2 : 1;

  auto queue_chunk = [&](int64_t i, int s) {
    const int64_t k = K - 1 - i;
    const int64_t t0 = k * kChunk;
    const int len = static_cast<int>(imin64(kChunk, a.T - t0));
    mbar_arrive_expect_tx(&bars[s], row_bytes * len * n_src);
    queue_rows(xs + s * kChunk * kTile, x, t0, len, a.BN, e0, row_bytes, &bars[s]);
    if (gs != nullptr) queue_rows(gss + s * kChunk * kTile, gs, t0, len, a.BN, e0, row_bytes, &bars[s]);
  };

  if (TMA) {
    if (tid == 0) {
      for (int s = 0; s < kBwdStages; ++s) mbar_init(&bars[s], 1);
      fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) {
      for (int64_t i = 0; i < imin64(kBwdStages, K); ++i) queue_chunk(i, static_cast<int>(i));
    }
  }

  const float decay = a.decay, thr = a.threshold, reset_v = a.reset;
  const float adapt_decay = a.adapt_decay, beta = a.beta, slope = a.slope;
  float gm = 0.0f, ga = 0.0f, gr = 0.0f;
  if (valid) {
    if (a.grad_vT) gm = E::to_f(static_cast<const T*>(a.grad_vT)[e]);
    if (KIND == MB_ALIF && a.grad_aT) ga = E::to_f(static_cast<const T*>(a.grad_aT)[e]);
    // the grad of a rate output reaches every step as grad_rates / T
    // (src/myelin/autograd.py:842-844)
    if (a.grad_rates) {
      gr = __fdiv_rn(E::to_f(static_cast<const T*>(a.grad_rates)[e]), static_cast<float>(a.T));
    }
  }

  for (int64_t i = 0; i < K; ++i) {
    const int s = static_cast<int>(i % kBwdStages);
    const int64_t k = K - 1 - i;
    const int64_t t0 = k * kChunk;
    const int len = static_cast<int>(imin64(kChunk, a.T - t0));
    const T* xstage = xs + s * kChunk * kTile;
    const T* gstage = gss + s * kChunk * kTile;
    bool ok = true;
    if (TMA) {
      ok = mbar_wait_bounded(&bars[s], static_cast<uint32_t>((i / kBwdStages) & 1));
    } else if (valid) {
      fill_rows(xs + s * kChunk * kTile, x, t0, len, a.BN, e, tid);
      if (gs != nullptr) fill_rows(gss + s * kChunk * kTile, gs, t0, len, a.BN, e, tid);
    }
    if (valid) {
      float m = a.ckpt_v[k * a.BN + e];
      float av = (KIND == MB_ALIF) ? a.ckpt_a[k * a.BN + e] : 0.0f;
      float P[kChunk];
      float TH[kChunk];
#pragma unroll
      for (int j = 0; j < kChunk; ++j) {
        if (j < len) {
          Step<KIND, RESET> st;
          st.run(m, av, E::to_f(xstage[j * kTile + tid]), decay, thr, reset_v, adapt_decay, beta);
          P[j] = st.p;
          TH[j] = st.theta;
        }
      }
#pragma unroll
      for (int j = kChunk - 1; j >= 0; --j) {
        if (j < len) {
          const float p = P[j];
          const float th = TH[j];
          const float sf = p >= th ? 1.0f : 0.0f;
          const float gsum = (gs != nullptr ? E::to_f(gstage[j * kTile + tid]) : 0.0f) + gr;
          const float d = slope * surrogate_grad<SURR>(slope * (p - th));
          float gp;
          if (KIND == MB_LIF) {
            if (RESET == MB_RESET_HARD) {
              // reference order: src/myelin/triton/lif.py:283-284
              gp = gm * ((1.0f - sf) + (reset_v - p) * d) + gsum * d;
            } else {
              gp = gm + (gsum - gm * th) * d;
            }
          } else {
            if (RESET == MB_RESET_HARD) {
              const float Gs = gsum + gm * (reset_v - p) + ga;
              gp = gm * (1.0f - sf) + Gs * d;
              ga = ga * adapt_decay - beta * (Gs * d);
            } else {
              const float Gs = gsum - gm * th + ga;
              gp = gm + Gs * d;
              ga = ga * adapt_decay - beta * (gm * sf + Gs * d);
            }
          }
          gx[(t0 + j) * a.BN + e] = E::from_f(gp);
          gm = gp * decay;
        }
      }
    }
    if (TMA) {
      if (__syncthreads_or(!ok)) {
        if (tid == 0) {
          for (int64_t ii = i + 1; ii < imin64(i + kBwdStages, K); ++ii) {
            mbar_wait_bounded(&bars[ii % kBwdStages], static_cast<uint32_t>((ii / kBwdStages) & 1));
          }
        }
        return;
      }
      if (tid == 0 && i + kBwdStages < K) {
        fence_proxy_async_smem();
        queue_chunk(i + kBwdStages, s);
      }
    }
  }
  if (!valid) return;
  if (a.grad_v0) static_cast<T*>(a.grad_v0)[e] = E::from_f(gm);
  if (KIND == MB_ALIF && a.grad_a0) static_cast<T*>(a.grad_a0)[e] = E::from_f(ga);
}

// ---------------------------------------------------------------------------
// Host dispatch.
// ---------------------------------------------------------------------------
template <typename Kern>
static void set_smem(Kern k, size_t bytes) {
  if (bytes > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
}

static bool rows_bulk_copyable(const void* base, int64_t BN, size_t elt) {
  return base != nullptr && aligned_to(base, 16) && (BN * int64_t(elt)) % 16 == 0;
}

template <typename T, int NPT, int KIND, int RESET>
static void launch_fwd_direct(ScanFwdArgs a, cudaStream_t stream) {
  a.groups_per_row = ceil_div(a.N, 32 * NPT);
  const int64_t threads = a.B * a.groups_per_row * 32;
  const int64_t blocks = ceil_div(threads, kBlock);
  scan_fwd_kernel<T, NPT, KIND, RESET><<<static_cast<unsigned>(blocks), kBlock, 0, stream>>>(a);
}

template <typename T, int KIND, int RESET>
static void dispatch_fwd_kr(const ScanFwdArgs& a, cudaStream_t stream) {
  const bool packed_ok = a.packed == nullptr || (a.N % 32) == 0;
  if (packed_ok) {
    const unsigned blocks = static_cast<unsigned>(ceil_div(a.BN, kTile));
    const size_t smem = fwd_smem_bytes<T>();
    if (a.T > 0 && rows_bulk_copyable(a.x, a.BN, sizeof(T))) {
      auto k = scan_fwd_tiled_kernel<T, KIND, RESET, true>;
      set_smem(k, smem);
      k<<<blocks, kTile, smem, stream>>>(a);
    } else {
      auto k = scan_fwd_tiled_kernel<T, KIND, RESET, false>;
      set_smem(k, smem);
      k<<<blocks, kTile, smem, stream>>>(a);
    }
    return;
  }
  constexpr int kVec = 16 / sizeof(T);
  bool vec_ok = (a.N % kVec) == 0;
  const void* ptrs[] = {a.x, a.v0, a.a0, a.vT, a.aT, a.spikes, a.rates};
  for (const void* p : ptrs) vec_ok = vec_ok && (p == nullptr || aligned_to(p, 16));
  if (vec_ok) {
    launch_fwd_direct<T, kVec, KIND, RESET>(a, stream);
  } else {
    launch_fwd_direct<T, 1, KIND, RESET>(a, stream);
  }
}

template <typename T>
static void dispatch_fwd(int neuron, int reset_mode, const ScanFwdArgs& a, cudaStream_t stream) {
  if (neuron == MB_LIF) {
    if (reset_mode == MB_RESET_HARD) dispatch_fwd_kr<T, MB_LIF, MB_RESET_HARD>(a, stream);
    else dispatch_fwd_kr<T, MB_LIF, MB_RESET_SUBTRACT>(a, stream);
  } else {
    if (reset_mode == MB_RESET_HARD) dispatch_fwd_kr<T, MB_ALIF, MB_RESET_HARD>(a, stream);
    else dispatch_fwd_kr<T, MB_ALIF, MB_RESET_SUBTRACT>(a, stream);
  }
}

template <typename T, int KIND, int RESET, int SURR>
static void launch_bwd(const ScanBwdArgs& a, cudaStream_t stream) {
  const unsigned blocks = static_cast<unsigned>(ceil_div(a.BN, kTile));
  const size_t smem = bwd_smem_bytes<T>();
  const bool tma = a.T > 0 && rows_bulk_copyable(a.x, a.BN, sizeof(T)) &&
                   (a.grad_spikes == nullptr || rows_bulk_copyable(a.grad_spikes, a.BN, sizeof(T)));
  if (tma) {
    auto k = scan_bwd_tiled_kernel<T, KIND, RESET, SURR, true>;
    set_smem(k, smem);
    k<<<blocks, kTile, smem, stream>>>(a);
  } else {
    auto k = scan_bwd_tiled_kernel<T, KIND, RESET, SURR, false>;
    set_smem(k, smem);
    k<<<blocks, kTile, smem, stream>>>(a);
  }
}

template <typename T, int KIND, int RESET>
static void dispatch_bwd_surr(int surrogate, const ScanBwdArgs& a, cudaStream_t stream) {
  switch (surrogate) {
    case MB_SURR_SIGMOID: launch_bwd<T, KIND, RESET, MB_SURR_SIGMOID>(a, stream); break;
    case MB_SURR_FAST_SIGMOID: launch_bwd<T, KIND, RESET, MB_SURR_FAST_SIGMOID>(a, stream); break;
    case MB_SURR_ATAN: launch_bwd<T, KIND, RESET, MB_SURR_ATAN>(a, stream); break;
    case MB_SURR_TRIANGULAR: launch_bwd<T, KIND, RESET, MB_SURR_TRIANGULAR>(a, stream); break;
    case MB_SURR_SUPERSPIKE: launch_bwd<T, KIND, RESET, MB_SURR_SUPERSPIKE>(a, stream); break;
    case MB_SURR_MULTI_GAUSSIAN: launch_bwd<T, KIND, RESET, MB_SURR_MULTI_GAUSSIAN>(a, stream); break;
    default: launch_bwd<T, KIND, RESET, MB_SURR_NONE>(a, stream); break;
  }
}

template <typename T>
static void dispatch_bwd(int neuron, int reset_mode, int surrogate, const ScanBwdArgs& a,
                         cudaStream_t stream) {
  if (neuron == MB_LIF) {
    if (reset_mode == MB_RESET_HARD) dispatch_bwd_surr<T, MB_LIF, MB_RESET_HARD>(surrogate, a, stream);
    else dispatch_bwd_surr<T, MB_LIF, MB_RESET_SUBTRACT>(surrogate, a, stream);
  } else {
    if (reset_mode == MB_RESET_HARD) dispatch_bwd_surr<T, MB_ALIF, MB_RESET_HARD>(surrogate, a, stream);
    else dispatch_bwd_surr<T, MB_ALIF, MB_RESET_SUBTRACT>(surrogate, a, stream);
  }
}

static int check_common(const char* fn, int neuron, int dtype, int64_t T, int64_t B, int64_t N,
                        int reset_mode) {
  MB_CHECK_ARG(neuron == MB_LIF || neuron == MB_ALIF, "%s: unknown neuron model %d", fn, neuron);
  MB_CHECK_ARG(dtype == MB_F32 || dtype == MB_BF16 || dtype == MB_F16,
               "%s: unsupported dtype %d (float32, bfloat16 or float16)", fn, dtype);
  MB_CHECK_ARG(T >= 0 && B >= 0 && N >= 0, "%s: negative size (T=%lld, B=%lld, N=%lld)", fn,
               (long long)T, (long long)B, (long long)N);
  MB_CHECK_ARG(reset_mode == MB_RESET_HARD || reset_mode == MB_RESET_SUBTRACT,
               "%s: unknown reset mode %d", fn, reset_mode);
  MB_CHECK_ARG(ceil_div(B * ceil_div(N, 32) * 32, kTile) < (int64_t(1) << 31),
               "%s: B*N too large for one launch", fn);
  return 0;
}

}  // namespace mb

using namespace mb;

extern "C" int64_t mb_scan_num_checkpoints(int64_t T) { return T <= 0 ? 0 : ceil_div(T, kChunk); }

extern "C" int mb_scan_forward(int neuron, int dtype, const void* x, const void* v0,
                               const void* a0, void* vT, void* aT, void* spikes, int32_t* packed,
                               void* rates, float* ckpt_v, float* ckpt_a, int64_t T, int64_t B,
                               int64_t N, float decay, float threshold, float reset,
                               float adapt_decay, float beta, int reset_mode, void* stream) {
  clear_error();
  if (check_common("mb_scan_forward", neuron, dtype, T, B, N, reset_mode)) return 1;
  if (B == 0 || N == 0) return 0;
  MB_CHECK_ARG(v0 != nullptr, "mb_scan_forward: v0 is required");
  MB_CHECK_ARG(T == 0 || x != nullptr, "mb_scan_forward: x is required");
  MB_CHECK_ARG(neuron == MB_LIF || a0 != nullptr, "mb_scan_forward: ALIF requires a0");
  MB_CHECK_ARG(neuron == MB_LIF || ckpt_v == nullptr || ckpt_a != nullptr,
               "mb_scan_forward: ALIF checkpoints need both ckpt_v and ckpt_a");
  MB_CHECK_ARG(packed == nullptr || aligned_to(packed, 4), "mb_scan_forward: packed misaligned");
  ScanFwdArgs a{};
  a.x = x; a.v0 = v0; a.a0 = a0; a.vT = vT; a.aT = aT;
  a.spikes = spikes; a.packed = packed; a.rates = rates;
  a.ckpt_v = ckpt_v; a.ckpt_a = ckpt_a;
  a.T = T; a.B = B; a.N = N; a.BN = B * N;
  a.words_per_row = ceil_div(N, 32);
  a.decay = decay; a.threshold = threshold; a.reset = reset;
  a.adapt_decay = adapt_decay; a.beta = beta;
  cudaStream_t s = as_stream(stream);
  if (launch_scan_fwd_fast(dtype, neuron, reset_mode, a, s)) {
    MB_CHECK_LAUNCH("mb_scan_forward");
    return 0;
  }
  switch (dtype) {
    case MB_F32: dispatch_fwd<float>(neuron, reset_mode, a, s); break;
    case MB_BF16: dispatch_fwd<__nv_bfloat16>(neuron, reset_mode, a, s); break;
    default: dispatch_fwd<__half>(neuron, reset_mode, a, s); break;
  }
  MB_CHECK_LAUNCH("mb_scan_forward");
  return 0;
}

extern "C" int mb_scan_forward_packed_scatter(int neuron, int dtype, const void* x,
                                              const void* v0, const void* a0, void* vT, void* aT,
                                              int32_t* packed, void* const* peers, int num_peers,
                                              int64_t T, int64_t B, int64_t N, float decay,
                                              float threshold, float reset, float adapt_decay,
                                              float beta, int reset_mode, void* stream) {
  clear_error();
  MB_CHECK_ARG(neuron == MB_LIF || neuron == MB_ALIF,
               "mb_scan_forward_packed_scatter: LIF or ALIF only");
  MB_CHECK_ARG(num_peers >= 0 && num_peers <= kMaxPushPeers && (num_peers == 0 || peers),
               "mb_scan_forward_packed_scatter: 0 to %d peer slots required", kMaxPushPeers);
  MB_CHECK_ARG(packed != nullptr || T * B * N == 0,
               "mb_scan_forward_packed_scatter: packed is required");
  MB_CHECK_ARG(aligned_to(packed, 4), "mb_scan_forward_packed_scatter: packed misaligned");
  for (int d = 0; d < num_peers; ++d) {
    MB_CHECK_ARG(peers[d] != nullptr && aligned_to(peers[d], 4),
                 "mb_scan_forward_packed_scatter: peer slot %d null or misaligned", d);
  }
  // The scan writes the words into this GPU's slot at full speed; one push
  // kernel then stores the slot into every peer's buffer, all peers at once.
  // (Stores of the words from the scan itself reach NVLink as 4- to 32-byte
  // pieces, one step of one 256-neuron tile, which made the step slower;
  // copy-engine copies one peer after another reached about 210 GB/s in
  // aggregate at 8 GPUs.)
  const int rc = mb_scan_forward(neuron, dtype, x, v0, a0, vT, aT, nullptr, packed, nullptr,
                                 nullptr, nullptr, T, B, N, decay, threshold, reset, adapt_decay,
                                 beta, reset_mode, stream);
  if (rc != 0) return rc;
  const size_t bytes = size_t(T) * size_t(B) * size_t(ceil_div(N, 32)) * sizeof(int32_t);
  if (bytes == 0) return 0;
  push_to_peers(packed, peers, num_peers, bytes, as_stream(stream));
  MB_CHECK_LAUNCH("mb_scan_forward_packed_scatter");
  return 0;
}

namespace mb {
namespace {

// Sum over t (last step first) of grad_x[t, i] as stored: the path for the
// neuron kinds and layouts whose backward kernel does not form it itself.
template <typename T>
__global__ void sum_over_t_kernel(const T* __restrict__ grad_x, int64_t steps, int64_t BN,
                                  float* __restrict__ out) {
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < BN;
       i += int64_t(gridDim.x) * blockDim.x) {
    float acc = 0.0f;
    for (int64_t t = steps - 1; t >= 0; --t) acc += Elem<T>::to_f(grad_x[t * BN + i]);
    out[i] = acc;
  }
}

int scan_backward_impl(int neuron, int dtype, const void* x, const float* ckpt_v,
                       const float* ckpt_a, const void* grad_spikes, const void* grad_rates,
                       const void* grad_vT, const void* grad_aT, void* grad_x, void* grad_v0,
                       void* grad_a0, float* grad_sum, int64_t T, int64_t B, int64_t N,
                       float decay, float threshold, float reset, float adapt_decay, float beta,
                       int reset_mode, int surrogate, float slope, void* stream) {
  clear_error();
  if (check_common("mb_scan_backward", neuron, dtype, T, B, N, reset_mode)) return 1;
  MB_CHECK_ARG(surrogate >= MB_SURR_SIGMOID && surrogate <= MB_SURR_NONE,
               "mb_scan_backward: unknown surrogate id %d", surrogate);
  if (B == 0 || N == 0) return 0;
  MB_CHECK_ARG(T == 0 || (x != nullptr && ckpt_v != nullptr && grad_x != nullptr),
               "mb_scan_backward: x, ckpt_v and grad_x are required");
  MB_CHECK_ARG(neuron == MB_LIF || T == 0 || ckpt_a != nullptr,
               "mb_scan_backward: ALIF requires ckpt_a");
  MB_CHECK_ARG(aligned_to(grad_sum, 8), "mb_scan_backward: grad_sum must be 8-byte aligned");
  cudaStream_t s = as_stream(stream);
  if (T == 0 && grad_sum != nullptr) cudaMemsetAsync(grad_sum, 0, size_t(B * N) * sizeof(float), s);
  ScanBwdArgs a{};
  a.x = x; a.ckpt_v = ckpt_v; a.ckpt_a = ckpt_a;
  a.grad_spikes = grad_spikes; a.grad_rates = grad_rates;
  a.grad_vT = grad_vT; a.grad_aT = grad_aT;
  a.grad_x = grad_x; a.grad_v0 = grad_v0; a.grad_a0 = grad_a0;
  // the fast LIF backward adds up grad_x as it stores it
  a.grad_sum = neuron == MB_LIF ? grad_sum : nullptr;
  a.T = T; a.B = B; a.N = N; a.BN = B * N;
  a.decay = decay; a.threshold = threshold; a.reset = reset;
  a.adapt_decay = adapt_decay; a.beta = beta; a.slope = slope;
  const bool fast = launch_scan_bwd_fast(dtype, neuron, reset_mode, surrogate, a, s);
  if (!fast) {
    switch (dtype) {
      case MB_F32: dispatch_bwd<float>(neuron, reset_mode, surrogate, a, s); break;
      case MB_BF16: dispatch_bwd<__nv_bfloat16>(neuron, reset_mode, surrogate, a, s); break;
      default: dispatch_bwd<__half>(neuron, reset_mode, surrogate, a, s); break;
    }
  }
  if (grad_sum != nullptr && T > 0 && !(fast && a.grad_sum != nullptr)) {
    const int64_t BN = B * N;
    const unsigned grid = static_cast<unsigned>(imin64(ceil_div(BN, 256), 148 * 16));
    switch (dtype) {
      case MB_F32:
        sum_over_t_kernel<float><<<grid, 256, 0, s>>>(static_cast<const float*>(grad_x), T, BN, grad_sum);
        break;
      case MB_BF16:
        sum_over_t_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
            static_cast<const __nv_bfloat16*>(grad_x), T, BN, grad_sum);
        break;
      default:
        sum_over_t_kernel<__half><<<grid, 256, 0, s>>>(static_cast<const __half*>(grad_x), T, BN,
                                                       grad_sum);
        break;
    }
  }
  MB_CHECK_LAUNCH("mb_scan_backward");
  return 0;
}

}  // namespace
}  // namespace mb

extern "C" int mb_scan_backward(int neuron, int dtype, const void* x, const float* ckpt_v,
                                const float* ckpt_a, const void* grad_spikes,
                                const void* grad_rates, const void* grad_vT, const void* grad_aT,
                                void* grad_x, void* grad_v0, void* grad_a0, int64_t T, int64_t B,
                                int64_t N, float decay, float threshold, float reset,
                                float adapt_decay, float beta, int reset_mode, int surrogate,
                                float slope, void* stream) {
  return scan_backward_impl(neuron, dtype, x, ckpt_v, ckpt_a, grad_spikes, grad_rates, grad_vT,
                            grad_aT, grad_x, grad_v0, grad_a0, nullptr, T, B, N, decay,
                            threshold, reset, adapt_decay, beta, reset_mode, surrogate, slope,
                            stream);
}

extern "C" int mb_scan_backward_sum(int neuron, int dtype, const void* x, const float* ckpt_v,
                                    const float* ckpt_a, const void* grad_spikes,
                                    const void* grad_rates, const void* grad_vT,
                                    const void* grad_aT, void* grad_x, void* grad_v0,
                                    void* grad_a0, float* grad_sum, int64_t T, int64_t B,
                                    int64_t N, float decay, float threshold, float reset,
                                    float adapt_decay, float beta, int reset_mode, int surrogate,
                                    float slope, void* stream) {
  return scan_backward_impl(neuron, dtype, x, ckpt_v, ckpt_a, grad_spikes, grad_rates, grad_vT,
                            grad_aT, grad_x, grad_v0, grad_a0, grad_sum, T, B, N, decay,
                            threshold, reset, adapt_decay, beta, reset_mode, surrogate, slope,
                            stream);
}

namespace mb {

int scan_unit_status(bool clear) { return read_device_status(clear); }

cudaError_t scan_unit_wait_probe(uint32_t polls, cudaStream_t stream) {
  wait_timeout_probe_kernel<<<1, 32, 0, stream>>>(polls);
  return cudaGetLastError();
}

}  // namespace mb
