/*
 * TEST INFRASTRUCTURE ONLY — the CPU oracle for myelin_b200's parity tests
 * and the CPU baseline timed by bench.py. Nothing in the product path links,
 * loads or calls this file.
 *
 * A plain-C restatement of the reference's fused-time LIF/ALIF scan and its
 * surrogate-gradient backward (djsaunde/myelin):
 *   forward  src/myelin/neurons.py:106-128 (_lif_step_unchecked,
 *            _alif_step_unchecked), src/myelin/functional.py:21-78 (lif_unroll,
 *            alif_unroll), src/myelin/triton/lif.py:16-41 (fused forward);
 *   backward src/myelin/triton/lif.py:252-288 (LIF adjoint),
 *            src/myelin/autograd.py:536-556 (rate/linear adjoint order), and the
 *            adjoint of src/myelin/functional.py:149-189 (surrogate ALIF);
 *   surrogate derivatives src/myelin/surrogates.py:78-102 and
 *            src/myelin/triton/lif.py:225-249.
 * Extension restated here (no reference counterpart): reset_mode SUBTRACT,
 * m <- p - theta after a spike, theta = threshold (+ beta * a for ALIF).
 *
 * Numerics: float32 throughout, every operation rounded separately (build with
 * -ffp-contract=off), which is what the reference's per-op torch kernels do;
 * this makes the forward bit-exact with lif_unroll / alif_unroll.
 *
 * Loop order is time-outer / neuron-inner over a per-thread neuron range, so
 * the CPU streams [T, B, N] memory like the reference's per-step torch ops.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { OR_LIF = 0, OR_ALIF = 1 };
enum { OR_HARD = 0, OR_SUBTRACT = 1 };

static float surrogate_grad(int id, float c) {
  switch (id) {
    case 0: { /* sigmoid */
      const float v = 1.0f / (1.0f + expf(-c));
      return v * (1.0f - v);
    }
    case 1: { /* fast_sigmoid */
      const float dn = 1.0f + fabsf(c);
      return 0.5f / (dn * dn);
    }
    case 2: { /* atan */
      const float u = 1.5707963267948966f * c;
      return 0.5f / (1.0f + u * u);
    }
    case 3: { /* triangular */
      const float sgn = c > 0.0f ? 1.0f : (c < 0.0f ? -1.0f : 0.0f);
      return fabsf(c) < 1.0f ? -sgn : 0.0f;
    }
    case 4: { /* superspike */
      const float dn = 1.0f + fabsf(c);
      return 1.0f / (dn * dn);
    }
    case 5: { /* multi_gaussian */
      const float h = c / 0.5f;
      return 0.47873073648171924f * expf(-0.5f * h * h) +
             0.07978845608028655f * expf(-0.5f * (c - 1.0f) * (c - 1.0f)) +
             0.07978845608028655f * expf(-0.5f * (c + 1.0f) * (c + 1.0f));
    }
    default:
      return 0.0f; /* exact gradient of the hard threshold */
  }
}

static int resolve_threads(int nthreads) {
#ifdef _OPENMP
  return nthreads > 0 ? nthreads : omp_get_max_threads();
#else
  (void)nthreads;
  return 1;
#endif
}

/* Neuron range [lo, hi) of thread `tid` out of `nt` over `total` neurons. */
static void thread_range(int64_t total, int tid, int nt, int64_t* lo, int64_t* hi) {
  const int64_t per = (total + nt - 1) / nt;
  *lo = (int64_t)tid * per;
  *hi = *lo + per < total ? *lo + per : total;
  if (*lo > total) *lo = total;
}

/* One step for neurons [lo, hi) at time t. Writes p/theta if requested. */
static void step_range(int neuron, int reset_mode, const float* xt, float* m, float* a,
                       uint8_t* st, float* pt, float* tht, int64_t* cnt, int64_t lo, int64_t hi,
                       float decay, float thr, float reset, float adapt_decay, float beta) {
  for (int64_t e = lo; e < hi; ++e) {
    const float p = m[e] * decay + xt[e];
    const float th = neuron == OR_ALIF ? thr + beta * a[e] : thr;
    const int s = p >= th;
    if (st) st[e] = (uint8_t)s;
    if (pt) pt[e] = p;
    if (tht) tht[e] = th;
    if (cnt) cnt[e] += s;
    m[e] = s ? (reset_mode == OR_HARD ? reset : p - th) : p;
    if (neuron == OR_ALIF) a[e] = a[e] * adapt_decay + (s ? 1.0f : 0.0f);
  }
}

/*
 * Forward scan. x [T,B,N]; v0/a0 [B,N]; outputs vT/aT [B,N], spikes [T,B,N]
 * as 0/1 bytes, counts [B,N] int64 (any output may be NULL except vT).
 */
void oracle_scan_forward(int neuron, int reset_mode, const float* x, const float* v0,
                         const float* a0, float* vT, float* aT, uint8_t* spikes, int64_t* counts,
                         int64_t T, int64_t B, int64_t N, float decay, float thr, float reset,
                         float adapt_decay, float beta, int nthreads) {
  const int64_t BN = B * N;
  float* a = (float*)calloc((size_t)(BN > 0 ? BN : 1), sizeof(float));
  memcpy(vT, v0, (size_t)BN * sizeof(float));
  if (neuron == OR_ALIF) memcpy(a, a0, (size_t)BN * sizeof(float));
  if (counts) memset(counts, 0, (size_t)BN * sizeof(int64_t));
  const int nt = resolve_threads(nthreads);
#pragma omp parallel num_threads(nt)
  {
    int tid = 0, n_t = 1;
#ifdef _OPENMP
    tid = omp_get_thread_num();
    n_t = omp_get_num_threads();
#endif
    int64_t lo, hi;
    thread_range(BN, tid, n_t, &lo, &hi);
    for (int64_t t = 0; t < T; ++t) {
      step_range(neuron, reset_mode, x + t * BN, vT, a, spikes ? spikes + t * BN : NULL, NULL,
                 NULL, counts, lo, hi, decay, thr, reset, adapt_decay, beta);
    }
  }
  if (aT) memcpy(aT, a, (size_t)BN * sizeof(float));
  free(a);
}

/*
 * Surrogate backward (full reverse-time adjoint). Replays the forward in
 * chunks of `chunk` steps from saved states (exact replay, so the chunk size
 * does not change any value) and walks each chunk in reverse:
 *   d = slope * sg(slope * (p - theta))
 *   LIF  HARD: gp = gm*((1-s) + (reset-p)*d) + gs*d
 *   LIF  SUB : gp = gm + (gs - gm*theta)*d
 *   ALIF HARD: Gs = gs + gm*(reset-p) + ga; gp = gm*(1-s) + Gs*d; ga = ga*rho - beta*(Gs*d)
 *   ALIF SUB : Gs = gs - gm*theta + ga;     gp = gm + Gs*d;       ga = ga*rho - beta*(gm*s + Gs*d)
 *   grad_x = gp; gm = gp*decay
 * gs = grad_spikes[t] (if any) + grad_rates/T (if any).
 */
void oracle_scan_backward(int neuron, int reset_mode, int surrogate, const float* x,
                          const float* v0, const float* a0, const float* grad_spikes,
                          const float* grad_rates, const float* grad_vT, const float* grad_aT,
                          float* grad_x, float* grad_v0, float* grad_a0, int64_t T, int64_t B,
                          int64_t N, float decay, float thr, float reset, float adapt_decay,
                          float beta, float slope, int64_t chunk, int nthreads) {
  const int64_t BN = B * N;
  if (chunk <= 0) chunk = 16;
  const int64_t K = T > 0 ? (T + chunk - 1) / chunk : 0;
  const int nt = resolve_threads(nthreads);
#pragma omp parallel num_threads(nt)
  {
    int tid = 0, n_t = 1;
#ifdef _OPENMP
    tid = omp_get_thread_num();
    n_t = omp_get_num_threads();
#endif
    int64_t lo, hi;
    thread_range(BN, tid, n_t, &lo, &hi);
    const int64_t R = hi - lo;
    float* m = (float*)malloc((size_t)(R > 0 ? R : 1) * sizeof(float));
    float* a = (float*)calloc((size_t)(R > 0 ? R : 1), sizeof(float));
    float* cm = (float*)malloc((size_t)((K > 0 ? K : 1) * (R > 0 ? R : 1)) * sizeof(float));
    float* ca = (float*)calloc((size_t)((K > 0 ? K : 1) * (R > 0 ? R : 1)), sizeof(float));
    float* P = (float*)malloc((size_t)(chunk * (R > 0 ? R : 1)) * sizeof(float));
    float* TH = (float*)malloc((size_t)(chunk * (R > 0 ? R : 1)) * sizeof(float));
    float* gm = (float*)malloc((size_t)(R > 0 ? R : 1) * sizeof(float));
    float* ga = (float*)malloc((size_t)(R > 0 ? R : 1) * sizeof(float));
    const float tf = (float)T;
    for (int64_t i = 0; i < R; ++i) {
      m[i] = v0[lo + i];
      if (neuron == OR_ALIF) a[i] = a0[lo + i];
      gm[i] = grad_vT ? grad_vT[lo + i] : 0.0f;
      ga[i] = (neuron == OR_ALIF && grad_aT) ? grad_aT[lo + i] : 0.0f;
    }
    /* forward pass saving chunk-start states */
    for (int64_t t = 0; t < T; ++t) {
      if (t % chunk == 0) {
        memcpy(cm + (t / chunk) * R, m, (size_t)R * sizeof(float));
        memcpy(ca + (t / chunk) * R, a, (size_t)R * sizeof(float));
      }
      step_range(neuron, reset_mode, x + t * BN + lo, m, a, NULL, NULL, NULL, NULL, 0, R, decay,
                 thr, reset, adapt_decay, beta);
    }
    for (int64_t k = K - 1; k >= 0; --k) {
      const int64_t t0 = k * chunk;
      const int64_t len = t0 + chunk <= T ? chunk : T - t0;
      memcpy(m, cm + k * R, (size_t)R * sizeof(float));
      memcpy(a, ca + k * R, (size_t)R * sizeof(float));
      for (int64_t j = 0; j < len; ++j) {
        step_range(neuron, reset_mode, x + (t0 + j) * BN + lo, m, a, NULL, P + j * R, TH + j * R,
                   NULL, 0, R, decay, thr, reset, adapt_decay, beta);
      }
      for (int64_t j = len - 1; j >= 0; --j) {
        const int64_t t = t0 + j;
        for (int64_t i = 0; i < R; ++i) {
          const float p = P[j * R + i];
          const float th = TH[j * R + i];
          const float s = p >= th ? 1.0f : 0.0f;
          float gs = grad_spikes ? grad_spikes[t * BN + lo + i] : 0.0f;
          if (grad_rates) gs = gs + grad_rates[lo + i] / tf;
          const float d = slope * surrogate_grad(surrogate, slope * (p - th));
          float gp;
          if (neuron == OR_LIF) {
            if (reset_mode == OR_HARD) {
              gp = gm[i] * ((1.0f - s) + (reset - p) * d) + gs * d;
            } else {
              gp = gm[i] + (gs - gm[i] * th) * d;
            }
          } else {
            if (reset_mode == OR_HARD) {
              const float Gs = gs + gm[i] * (reset - p) + ga[i];
              gp = gm[i] * (1.0f - s) + Gs * d;
              ga[i] = ga[i] * adapt_decay - beta * (Gs * d);
            } else {
              const float Gs = gs - gm[i] * th + ga[i];
              gp = gm[i] + Gs * d;
              ga[i] = ga[i] * adapt_decay - beta * (gm[i] * s + Gs * d);
            }
          }
          grad_x[t * BN + lo + i] = gp;
          gm[i] = gp * decay;
        }
      }
    }
    for (int64_t i = 0; i < R; ++i) {
      if (grad_v0) grad_v0[lo + i] = gm[i];
      if (grad_a0 && neuron == OR_ALIF) grad_a0[lo + i] = ga[i];
    }
    free(m); free(a); free(cm); free(ca); free(P); free(TH); free(gm); free(ga);
  }
}

int oracle_num_threads(void) { return resolve_threads(0); }
