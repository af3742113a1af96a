// Fused-time Izhikevich forward over time-major [T, B*N] currents.
//
// The step is the reference's (src/myelin/neurons.py:131-156), evaluated in
// the order the torch expression does with one fp32 rounding per operation
// and no FMA, so spikes and final states are bit-exact with
// functional.izhikevich_unroll for fp32 inputs (16-bit inputs: fp32 carry,
// one rounding on output, like the LIF/ALIF scans):
//   dv  = ((c2 * v) * v + c1 * v) + bias - u + I
//   p_v = v + dt * dv
//   p_u = u + dt * (a * (b * v - u))
//   s   = p_v >= threshold
//   v'  = s ? reset_voltage : p_v;   u' = s ? p_u + jump : p_u
//
// Forward only, like the reference's generated kernel
// (src/myelin/triton/generated.py:1192-1227). Rows that are 16-byte aligned
// run the warp-specialized scan forward (scan_fast.cu, TMA-streamed chunks);
// the kernels here serve the other shapes: two neighbouring neurons per thread
// with kIzhUnroll steps of loads in flight, or one neuron per thread.
#include "common.cuh"
#include "scan_common.cuh"

namespace mb {

namespace {

constexpr int kIzhUnroll = 8;

// Two neurons per thread (BN even, pair-aligned pointers).
template <typename T>
__global__ void __launch_bounds__(256) izh_fwd_pair_kernel(const T* __restrict__ x,
                                                           const T* __restrict__ v0,
                                                           const T* __restrict__ u0,
                                                           T* __restrict__ vT, T* __restrict__ uT,
                                                           T* __restrict__ spikes, int64_t steps,
                                                           int64_t half, IzhConsts cp) {
  using P = Pair<T>;
  const IzhConsts c = cp;  // register copy (see izh_step's callers in scan_fast.cu)
  using V = typename P::V;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < half; i += stride) {
    const float2 vv = P::to_f2(reinterpret_cast<const V*>(v0)[i]);
    const float2 uu = P::to_f2(reinterpret_cast<const V*>(u0)[i]);
    float va = vv.x, vb = vv.y, ua = uu.x, ub = uu.y;
    const V* xp = reinterpret_cast<const V*>(x) + i;
    V* sp = spikes ? reinterpret_cast<V*>(spikes) + i : nullptr;
    auto step = [&](V xv, int64_t t) {
      const float2 xf = P::to_f2(xv);
      const bool sa = izh_step(va, ua, xf.x, c);
      const bool sb = izh_step(vb, ub, xf.y, c);
      if (sp) sp[t * half] = P::spikes(sa, sb);
    };
    int64_t t = 0;
    for (; t + kIzhUnroll <= steps; t += kIzhUnroll) {
      V xv[kIzhUnroll];
#pragma unroll
      for (int k = 0; k < kIzhUnroll; ++k) xv[k] = xp[(t + k) * half];
#pragma unroll
      for (int k = 0; k < kIzhUnroll; ++k) step(xv[k], t + k);
    }
    for (; t < steps; ++t) step(xp[t * half], t);
    if (vT) reinterpret_cast<V*>(vT)[i] = P::from_f2(va, vb);
    if (uT) reinterpret_cast<V*>(uT)[i] = P::from_f2(ua, ub);
  }
}

// One neuron per thread (any shape or alignment).
template <typename T>
__global__ void __launch_bounds__(256) izh_fwd_scalar_kernel(const T* __restrict__ x,
                                                             const T* __restrict__ v0,
                                                             const T* __restrict__ u0,
                                                             T* __restrict__ vT, T* __restrict__ uT,
                                                             T* __restrict__ spikes,
                                                             int64_t steps, int64_t BN,
                                                             IzhConsts cp) {
  using E = Elem<T>;
  const IzhConsts c = cp;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t e = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; e < BN; e += stride) {
    float v = E::to_f(v0[e]), u = E::to_f(u0[e]);
    for (int64_t t = 0; t < steps; ++t) {
      const bool s = izh_step(v, u, E::to_f(x[t * BN + e]), c);
      if (spikes) spikes[t * BN + e] = E::from_f(s ? 1.0f : 0.0f);
    }
    if (vT) vT[e] = E::from_f(v);
    if (uT) uT[e] = E::from_f(u);
  }
}

int izh_grid(int64_t items) {
  int64_t g = ceil_div(items, 256);
  const int64_t cap = 148 * 16;
  if (g > cap) g = cap;
  return static_cast<int>(g < 1 ? 1 : g);
}

template <typename T>
void launch_izh(const void* x, const void* v0, const void* u0, void* vT, void* uT, void* spikes,
                int64_t steps, int64_t BN, const IzhConsts& c, cudaStream_t s) {
  const size_t pair = 2 * sizeof(T);
  const bool pairs_ok = BN % 2 == 0 && aligned_to(x, pair) && aligned_to(v0, pair) &&
                        aligned_to(u0, pair) && (vT == nullptr || aligned_to(vT, pair)) &&
                        (uT == nullptr || aligned_to(uT, pair)) &&
                        (spikes == nullptr || aligned_to(spikes, pair));
  const T* xt = static_cast<const T*>(x);
  if (pairs_ok) {
    izh_fwd_pair_kernel<T><<<izh_grid(BN / 2), 256, 0, s>>>(
        xt, static_cast<const T*>(v0), static_cast<const T*>(u0), static_cast<T*>(vT),
        static_cast<T*>(uT), static_cast<T*>(spikes), steps, BN / 2, c);
  } else {
    izh_fwd_scalar_kernel<T><<<izh_grid(BN), 256, 0, s>>>(
        xt, static_cast<const T*>(v0), static_cast<const T*>(u0), static_cast<T*>(vT),
        static_cast<T*>(uT), static_cast<T*>(spikes), steps, BN, c);
  }
}

}  // namespace

}  // namespace mb

using namespace mb;

extern "C" int mb_izhikevich_forward(int dtype, const void* x, const void* v0, const void* u0,
                                     void* vT, void* uT, void* spikes, int64_t T, int64_t B,
                                     int64_t N, const mb_izhikevich_params* params,
                                     void* stream) {
  clear_error();
  MB_CHECK_ARG(dtype == MB_F32 || dtype == MB_BF16 || dtype == MB_F16,
               "mb_izhikevich_forward: dtype must be float32, bfloat16 or float16 (got %d)",
               dtype);
  MB_CHECK_ARG(T >= 0 && B >= 0 && N >= 0, "mb_izhikevich_forward: negative shape");
  MB_CHECK_ARG(params != nullptr, "mb_izhikevich_forward: params is required");
  MB_CHECK_ARG(params->dt > 0.0f, "mb_izhikevich_forward: dt must be positive");
  if (B == 0 || N == 0) return 0;
  MB_CHECK_ARG(v0 != nullptr && u0 != nullptr, "mb_izhikevich_forward: v0 and u0 are required");
  MB_CHECK_ARG(T == 0 || x != nullptr, "mb_izhikevich_forward: x is required");
  const IzhConsts c{params->recovery_decay, params->recovery_coupling, params->reset_voltage,
                    params->recovery_jump,  params->threshold,         params->dt,
                    params->voltage_square_coeff, params->voltage_coeff, params->voltage_bias};
  cudaStream_t s = as_stream(stream);
  const int64_t BN = B * N;
  if (T > 0) {
    // 16-byte-aligned rows: the warp-specialized forward (TMA-streamed chunks)
    ScanFwdArgs a{};
    a.x = x; a.v0 = v0; a.a0 = u0; a.vT = vT; a.aT = uT; a.spikes = spikes;
    a.T = T; a.B = B; a.N = N; a.BN = BN;
    a.words_per_row = ceil_div(N, 32);
    a.izh = c;
    if (launch_scan_fwd_fast(dtype, kIzhikevich, MB_RESET_HARD, a, s)) {
      MB_CHECK_LAUNCH("mb_izhikevich_forward");
      return 0;
    }
  }
  switch (dtype) {
    case MB_F32: launch_izh<float>(x, v0, u0, vT, uT, spikes, T, BN, c, s); break;
    case MB_BF16: launch_izh<__nv_bfloat16>(x, v0, u0, vT, uT, spikes, T, BN, c, s); break;
    default: launch_izh<__half>(x, v0, u0, vT, uT, spikes, T, BN, c, s); break;
  }
  MB_CHECK_LAUNCH("mb_izhikevich_forward");
  return 0;
}
