// Shared definitions of the LIF/ALIF scan kernels: argument blocks, the
// bit-exact neuron step, and the closed-form surrogate derivatives.
#pragma once

#include "common.cuh"

namespace mb {

constexpr int kChunk = MB_SCAN_CHUNK;
constexpr int kBlock = 256;

// Izhikevich constants (mb_izhikevich_params) and the internal neuron-kind id
// the forward kernels use for it (the public mb_neuron enum covers the scans
// with a backward; Izhikevich has its own entry point).
constexpr int kIzhikevich = 2;

struct IzhConsts {
  float a, b, reset_v, jump, thr, dt, c2, c1, bias;
};

// One Izhikevich step (src/myelin/neurons.py:131-156) in the torch
// expression's order, one fp32 rounding per operation, no FMA:
//   dv = ((c2 * v) * v + c1 * v) + bias - u + x;  p_v = v + dt * dv
//   p_u = u + dt * (a * (b * v - u));  s = p_v >= thr
//   v = s ? reset_v : p_v;  u = s ? p_u + jump : p_u
__device__ __forceinline__ bool izh_step(float& v, float& u, float x, const IzhConsts& c) {
  float dv = __fmul_rn(__fmul_rn(c.c2, v), v);
  dv = __fadd_rn(dv, __fmul_rn(c.c1, v));
  dv = __fadd_rn(dv, c.bias);
  dv = __fsub_rn(dv, u);
  dv = __fadd_rn(dv, x);
  const float pv = __fadd_rn(v, __fmul_rn(c.dt, dv));
  const float pu = __fadd_rn(u, __fmul_rn(c.dt, __fmul_rn(c.a, __fsub_rn(__fmul_rn(c.b, v), u))));
  const bool s = pv >= c.thr;
  v = s ? c.reset_v : pv;
  u = s ? __fadd_rn(pu, c.jump) : pu;
  return s;
}

struct ScanFwdArgs {
  const void* x;
  const void* v0;
  const void* a0;
  void* vT;
  void* aT;
  void* spikes;
  int32_t* packed;
  void* rates;
  float* ckpt_v;
  float* ckpt_a;
  int64_t T, B, N, BN;
  int64_t words_per_row;   // ceil(N / 32)
  int64_t groups_per_row;  // ceil(N / (32 * NPT))
  float decay, threshold, reset, adapt_decay, beta;
  IzhConsts izh;  // kIzhikevich only
};

struct ScanBwdArgs {
  const void* x;
  const float* ckpt_v;
  const float* ckpt_a;
  const void* grad_spikes;
  const void* grad_rates;
  const void* grad_vT;
  const void* grad_aT;
  void* grad_x;
  void* grad_v0;
  void* grad_a0;
  // optional: sum over t of grad_x (as stored, in the I/O type), fp32 [B*N],
  // summed from the last step to the first
  float* grad_sum;
  int64_t T, B, N, BN;
  int64_t groups_per_row;  // ceil(N / 32)
  float decay, threshold, reset, adapt_decay, beta, slope;
};

// One step of the neuron recurrence, shared by the forward and the backward
// replay so that both produce bit-identical membranes and spike decisions.
template <int KIND, int RESET>
struct Step {
  float p;      // pre-reset membrane
  float theta;  // (adaptive) threshold used for this step
  bool s;       // spike
  __device__ __forceinline__ void run(float& m, float& a, float x, const float decay,
                                      const float thr, const float reset_v,
                                      const float adapt_decay, const float beta) {
    p = __fadd_rn(__fmul_rn(m, decay), x);
    theta = (KIND == MB_ALIF) ? __fadd_rn(thr, __fmul_rn(beta, a)) : thr;
    s = p >= theta;
    if (RESET == MB_RESET_HARD) {
      m = s ? reset_v : p;
    } else {
      m = s ? __fsub_rn(p, theta) : p;
    }
    if (KIND == MB_ALIF) {
      a = __fadd_rn(__fmul_rn(a, adapt_decay), s ? 1.0f : 0.0f);
    }
  }
};

// Closed-form surrogate derivatives, as src/myelin/surrogates.py:78-102 and
// src/myelin/triton/lif.py:225-249 (ids 0..5). MB_SURR_NONE returns 0: the
// gradient of the hard threshold itself.
template <int SURR>
__device__ __forceinline__ float surrogate_grad(float c) {
  if constexpr (SURR == MB_SURR_SIGMOID) {
    const float v = __fdividef(1.0f, 1.0f + __expf(-c));
    return v * (1.0f - v);
  } else if constexpr (SURR == MB_SURR_FAST_SIGMOID) {
    const float dn = 1.0f + fabsf(c);
    return __fdividef(0.5f, dn * dn);
  } else if constexpr (SURR == MB_SURR_ATAN) {
    const float u = 1.5707963267948966f * c;  // (pi / 2) * c
    return __fdividef(0.5f, 1.0f + u * u);
  } else if constexpr (SURR == MB_SURR_TRIANGULAR) {
    const float sgn = c > 0.0f ? 1.0f : (c < 0.0f ? -1.0f : 0.0f);
    return fabsf(c) < 1.0f ? -sgn : 0.0f;
  } else if constexpr (SURR == MB_SURR_SUPERSPIKE) {
    const float dn = 1.0f + fabsf(c);
    return __fdividef(1.0f, dn * dn);
  } else if constexpr (SURR == MB_SURR_MULTI_GAUSSIAN) {
    // 0.6 * N(c; 0, 0.5) + 0.2 * N(c; 1, 1) + 0.2 * N(c; -1, 1)
    const float cm = c - 1.0f;
    const float cp = c + 1.0f;
    const float center = 0.47873073648171924f * __expf(-2.0f * c * c);
    const float right = 0.07978845608028655f * __expf(-0.5f * cm * cm);
    const float left = 0.07978845608028655f * __expf(-0.5f * cp * cp);
    return center + right + left;
  } else {
    return 0.0f;
  }
}


// Surrogate derivative with the slope folded in: d(diff) = slope * sg(slope * diff)
// where diff = p - theta. Same functions as surrogate_grad, with the
// constants pre-multiplied so the hot loop spends as few instructions as
// possible (one reciprocal, a few multiply-adds).
template <int SURR>
struct SurrogateD {
  float k0, k1;
  __host__ __device__ __forceinline__ explicit SurrogateD(float slope) {
    if (SURR == MB_SURR_ATAN) {
      k0 = 1.5707963267948966f * slope;  // u = (pi/2) * slope * diff
      k1 = 0.5f * slope;                 // d = 0.5 * slope / (1 + u^2)
    } else if (SURR == MB_SURR_FAST_SIGMOID) {
      k0 = slope;
      k1 = 0.5f * slope;                 // d = 0.5 * slope / (1 + |slope diff|)^2
    } else if (SURR == MB_SURR_SUPERSPIKE) {
      k0 = slope;
      k1 = slope;                        // d = slope / (1 + |slope diff|)^2
    } else {
      k0 = slope;
      k1 = slope;
    }
  }
  __device__ __forceinline__ float operator()(float diff) const {
    if constexpr (SURR == MB_SURR_ATAN) {
      const float u = k0 * diff;
      return __fdividef(k1, 1.0f + u * u);
    } else if constexpr (SURR == MB_SURR_FAST_SIGMOID || SURR == MB_SURR_SUPERSPIKE) {
      const float dn = 1.0f + fabsf(k0 * diff);
      return __fdividef(k1, dn * dn);
    } else if constexpr (SURR == MB_SURR_NONE) {
      return 0.0f;
    } else {
      return k1 * surrogate_grad<SURR>(k0 * diff);
    }
  }
};

// Two neighbouring neurons' I/O values moved as one 4- or 8-byte word.
template <typename T>
struct Pair;

template <>
struct Pair<float> {
  using V = float2;
  static __device__ __forceinline__ float2 join(float a, float b) { return make_float2(a, b); }
  static __device__ __forceinline__ float2 to_f2(float2 v) { return v; }
  static __device__ __forceinline__ float2 from_f2(float a, float b) { return make_float2(a, b); }
  static __device__ __forceinline__ float2 spikes(bool s0, bool s1) {
    return make_float2(s0 ? 1.0f : 0.0f, s1 ? 1.0f : 0.0f);
  }
};

template <>
struct Pair<__nv_bfloat16> {
  using V = uint32_t;  // bf16x2, low half = first neuron
  static __device__ __forceinline__ uint32_t join(__nv_bfloat16 a, __nv_bfloat16 b) {
    return uint32_t(__bfloat16_as_ushort(a)) | (uint32_t(__bfloat16_as_ushort(b)) << 16);
  }
  static __device__ __forceinline__ float2 to_f2(uint32_t v) {
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
  }
  static __device__ __forceinline__ uint32_t from_f2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  static __device__ __forceinline__ uint32_t spikes(bool s0, bool s1) {
    return (s0 ? 0x00003f80u : 0u) | (s1 ? 0x3f800000u : 0u);
  }
};

template <>
struct Pair<__half> {
  using V = uint32_t;  // f16x2, low half = first neuron
  static __device__ __forceinline__ uint32_t join(__half a, __half b) {
    return uint32_t(__half_as_ushort(a)) | (uint32_t(__half_as_ushort(b)) << 16);
  }
  static __device__ __forceinline__ float2 to_f2(uint32_t v) {
    return __half22float2(*reinterpret_cast<const __half2*>(&v));
  }
  static __device__ __forceinline__ uint32_t from_f2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  static __device__ __forceinline__ uint32_t spikes(bool s0, bool s1) {
    return (s0 ? 0x00003c00u : 0u) | (s1 ? 0x3c000000u : 0u);
  }
};

// ---------------------------------------------------------------------------
// Two fp32 lanes (a float2) operated on by the sm_100 packed instructions
// through the builtins __fadd2_rn / __fmul2_rn / __ffma2_rn: one instruction
// for both lanes, each lane rounded like the scalar __fadd_rn / __fmul_rn /
// __fmaf_rn. A packed product followed by a packed sum is contracted into a
// fused multiply-add by the compiler (measured on B200 with CUDA 12.9 for the
// builtins and for PTX mul.rn/add.rn .f32x2 alike, despite the explicit
// rounding modes), while a scalar __fmul_rn is never merged. So the bit-exact
// neuron step multiplies lane by lane (mul2_exact) and adds in pairs.
// ---------------------------------------------------------------------------
using F2 = float2;

__device__ __forceinline__ F2 f2(float lo, float hi) { return make_float2(lo, hi); }
__device__ __forceinline__ F2 f2(float both) { return make_float2(both, both); }
__device__ __forceinline__ F2 f2(float2 v) { return v; }
__device__ __forceinline__ float2 split(F2 x) { return x; }
__device__ __forceinline__ F2 add2(F2 a, F2 b) { return __fadd2_rn(a, b); }
// a - b == a + (-b) exactly (negation is exact)
__device__ __forceinline__ F2 sub2(F2 a, F2 b) { return __fadd2_rn(a, make_float2(-b.x, -b.y)); }
__device__ __forceinline__ F2 mul2(F2 a, F2 b) { return __fmul2_rn(a, b); }
// a * b + c, one rounding per lane
__device__ __forceinline__ F2 fma2(F2 a, F2 b, F2 c) { return __ffma2_rn(a, b, c); }
// a * b per lane with the scalar __fmul_rn, which is never merged into a
// fused multiply-add (see the note above)
__device__ __forceinline__ F2 mul2_exact(F2 a, F2 b) {
  return make_float2(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y));
}
// 1.0f where a >= b, else 0.0f (NaN compares false)
__device__ __forceinline__ float ge_f(float a, float b) {
  float r;
  asm("set.ge.f32.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
// 1.0f where a < b, else 0.0f (NaN compares false)
__device__ __forceinline__ float lt_f(float a, float b) {
  float r;
  asm("set.lt.f32.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
// Approximate reciprocal (PTX rcp.approx: max 1 ulp error, subnormals flushed).
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Step for a pair of neurons: per lane the same operations and roundings as
// Step, so membranes and spike decisions are bit-identical. It works with the
// negated threshold nth = -theta (exact: fl(-thr + fl(-beta * a)) is
// -fl(thr + fl(beta * a))), so that p - theta = p + nth needs no negation.
//
// The spike is also produced as a float 0/1 (sf, one set instruction per lane)
// so that the subtractive reset is one packed fused multiply-add,
// m = sf * nth + p: exactly fl(p + nth) = fl(p - theta) where sf = 1 and p
// where sf = 0 (the only difference from a select: a membrane of -0 that does
// not spike comes back as +0 when the threshold is negative; values compare
// equal). The adaptation adds sf directly.
template <int KIND, int RESET>
struct Step2 {
  F2 p;     // pre-reset membranes
  F2 nth;   // minus the thresholds used this step
  F2 diff;  // p - theta (subtractive reset only)
  F2 sf;    // spikes as 1.0f / 0.0f
  bool s0, s1;
  __device__ __forceinline__ void run(F2& m, F2& a, F2 x, const F2 decay, const F2 nthr,
                                      const float reset_v, const F2 adapt_decay,
                                      const F2 nbeta) {
    p = add2(mul2_exact(m, decay), x);
    nth = (KIND == MB_ALIF) ? add2(nthr, mul2_exact(nbeta, a)) : nthr;
    s0 = p.x >= -nth.x;
    s1 = p.y >= -nth.y;
    sf = f2(ge_f(p.x, -nth.x), ge_f(p.y, -nth.y));
    if (RESET == MB_RESET_HARD) {
      m = f2(s0 ? reset_v : p.x, s1 ? reset_v : p.y);
    } else {
      diff = add2(p, nth);
      m = fma2(sf, nth, p);
    }
    if (KIND == MB_ALIF) {
      a = add2(mul2_exact(a, adapt_decay), sf);
    }
  }
};

// SurrogateD on a pair of differences p - theta; k0, k1 are SurrogateD's
// constants in both lanes, `one` is 1.0f in both lanes.
template <int SURR>
struct SurrogateD2 {
  SurrogateD<SURR> scalar;
  F2 k0, k1, one;
  __device__ __forceinline__ SurrogateD2(float slope, F2 k0_, F2 k1_, F2 one_)
      : scalar(slope), k0(k0_), k1(k1_), one(one_) {}
  __device__ __forceinline__ F2 operator()(F2 diff) const {
    if constexpr (SURR == MB_SURR_ATAN) {
      const F2 u = mul2(k0, diff);
      const float2 dn = split(fma2(u, u, one));
      return mul2(k1, f2(rcp_approx(dn.x), rcp_approx(dn.y)));
    } else if constexpr (SURR == MB_SURR_FAST_SIGMOID || SURR == MB_SURR_SUPERSPIKE) {
      const float2 u = split(mul2(k0, diff));
      const F2 dn = add2(one, f2(fabsf(u.x), fabsf(u.y)));
      const float2 dd = split(mul2(dn, dn));
      return mul2(k1, f2(rcp_approx(dd.x), rcp_approx(dd.y)));
    } else if constexpr (SURR == MB_SURR_NONE) {
      return f2(0.0f);
    } else {
      const float2 df = split(diff);
      return f2(scalar(df.x), scalar(df.y));
    }
  }
};

// Spread the low 16 bits of x to the even bit positions of a 32-bit word.
__device__ __forceinline__ uint32_t spread_even_bits(uint32_t x) {
  x &= 0xffffu;
  x = (x | (x << 8)) & 0x00ff00ffu;
  x = (x | (x << 4)) & 0x0f0f0f0fu;
  x = (x | (x << 2)) & 0x33333333u;
  x = (x | (x << 1)) & 0x55555555u;
  return x;
}

// Host launchers of the warp-specialized two-neurons-per-thread kernels
// (scan_fast.cu). They return false when the shape or alignment does not fit
// their layout (the caller then uses the general kernels).
bool launch_scan_fwd_fast(int dtype, int neuron, int reset_mode, const ScanFwdArgs& a,
                          cudaStream_t stream);
bool launch_scan_bwd_fast(int dtype, int neuron, int reset_mode, int surrogate,
                          const ScanBwdArgs& a, cudaStream_t stream);

}  // namespace mb
