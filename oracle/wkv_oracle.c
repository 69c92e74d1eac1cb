/*
 * CPU oracle for the RWKV-4 WKV recurrence -- TEST INFRASTRUCTURE ONLY.
 *
 * This file is a plain-C restatement of the reference's WKV arithmetic. It is
 * the checker for the CUDA path (tests, smoke(), and the CPU-baseline leg of
 * bench.py); nothing in the shipped library links it or calls it.
 *
 * Parity of this oracle is pinned by tests/test_oracle_golden.py against golden
 * vectors produced by the reference itself (tests/golden/make_golden.py runs
 * spikegpt.language.weighted_key_value_loop with float64 autograd).
 *
 * Reference semantics restated here (paths relative to the reference project):
 *   forward : src/spikegpt/language.py:399-449 (weighted_key_value_loop), which
 *             is also the recurrence of src/spikegpt/wkv_triton.py:34-58.
 *   backward: src/spikegpt/wkv_triton.py:60-142 (pass 1: forward replay with
 *             forward-mode dp/dw, dq/dw; pass 2: reverse-time adjoint), and
 *             src/spikegpt/wkv_triton.py:117,194 (g_time_decay = sum_b gw*w).
 *
 * Layout: k, v, y, gy, gk, gv are row-major [B, T, C]; element (b, t, c) sits
 * at b*T*C + t*C + c. time_decay / time_first / w / u / g_* are [C].
 *
 * Both a double and a float instantiation are exported. The double one is the
 * parity oracle; the float one is what the CPU baseline times (the reference's
 * CPU path runs in float32). Lanes (b, c) are independent, so they are spread
 * over OpenMP threads; the per-channel reductions over b run in a fixed order so
 * the result does not depend on the thread count.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define WKV_ORACLE_DEFINE(REAL, SUF, EXP, INIT_LOG_SCALE)                                   \
  /* Forward: language.py:399-449. The log-scale starts at the dtype's most            \
   * negative finite value (finfo.min, language.py:422-427). */                         \
  int wkv_oracle_forward_##SUF(const REAL* k, const REAL* v, const REAL* time_decay,     \
                               const REAL* time_first, REAL* y, int64_t B, int64_t T,   \
                               int64_t C, int nthreads) {                               \
    if (B < 0 || T < 0 || C < 0) return 1;                                              \
    int64_t lanes = B * C;                                                              \
    _Pragma("omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)") \
    for (int64_t lane = 0; lane < lanes; ++lane) {                                      \
      int64_t b = lane / C, c = lane % C;                                               \
      REAL w = -EXP(time_decay[c]);                                                     \
      REAL u = time_first[c];                                                           \
      REAL num = 0, den = 0, o = INIT_LOG_SCALE;                                        \
      const int64_t base = b * T * C + c;                                               \
      for (int64_t t = 0; t < T; ++t) {                                                 \
        const REAL kt = k[base + t * C], vt = v[base + t * C];                          \
        REAL no = o > u + kt ? o : u + kt;                                              \
        REAL a = EXP(o - no), e = EXP(u + kt - no);                                     \
        y[base + t * C] = (a * num + e * vt) / (a * den + e);                           \
        REAL wo = o + w;                                                                \
        no = wo > kt ? wo : kt;                                                         \
        a = EXP(wo - no);                                                               \
        e = EXP(kt - no);                                                               \
        num = a * num + e * vt;                                                         \
        den = a * den + e;                                                              \
        o = no;                                                                         \
      }                                                                                 \
    }                                                                                   \
    return 0;                                                                           \
  }                                                                                     \
                                                                                        \
  /* Backward: wkv_triton.py:60-142. w = -exp(time_decay), u = time_first.           \
   * g_time_decay[c] = sum_b gw[b,c] * w[c] (wkv_triton.py:117,194);                   \
   * g_time_first[c] = sum_b gu[b,c]. The replay buffers y/z/zexp are per-lane         \
   * scratch (wkv_triton.py:170-172), reduced here to O(T) per thread. */              \
  int wkv_oracle_backward_##SUF(const REAL* gy, const REAL* w, const REAL* u,            \
                                const REAL* k, const REAL* v, REAL* gk, REAL* gv,        \
                                REAL* g_time_decay, REAL* g_time_first, int64_t B,       \
                                int64_t T, int64_t C, int nthreads) {                    \
    if (B < 0 || T < 0 || C < 0) return 1;                                              \
    int64_t lanes = B * C;                                                              \
    REAL* gw_lane = (REAL*)calloc((size_t)(lanes > 0 ? lanes : 1), sizeof(REAL));       \
    REAL* gu_lane = (REAL*)calloc((size_t)(lanes > 0 ? lanes : 1), sizeof(REAL));       \
    if (!gw_lane || !gu_lane) { free(gw_lane); free(gu_lane); return 2; }               \
    int failed = 0;                                                                     \
    _Pragma("omp parallel num_threads(nthreads > 0 ? nthreads : 1)")                     \
    {                                                                                   \
      REAL* ys = (REAL*)malloc((size_t)(T > 0 ? T : 1) * 3 * sizeof(REAL));             \
      if (!ys) {                                                                        \
        _Pragma("omp atomic write") failed = 1;                                         \
      }                                                                                 \
      REAL* zs = ys ? ys + (T > 0 ? T : 1) : NULL;                                      \
      REAL* zx = ys ? zs + (T > 0 ? T : 1) : NULL;                                      \
      _Pragma("omp for schedule(static)")                                               \
      for (int64_t lane = 0; lane < lanes; ++lane) {                                    \
        if (!ys) continue;                                                              \
        int64_t b = lane / C, c = lane % C;                                             \
        const REAL wc = w[c], uc = u[c];                                                \
        const int64_t base = b * T * C + c;                                             \
        /* pass 1: forward replay (wkv_triton.py:85-118) */                             \
        REAL p = 0, q = 0, dpdw = 0, dqdw = 0, o = (REAL)-1e38, gws = 0, gus = 0;       \
        for (int64_t t = 0; t < T; ++t) {                                               \
          const int64_t off = base + t * C;                                             \
          const REAL kt = k[off], vt = v[off], gyt = gy[off];                           \
          REAL no = o > kt + uc ? o : kt + uc;                                          \
          REAL a = EXP(o - no), e = EXP(kt + uc - no);                                  \
          REAL iden = (REAL)1 / (a * q + e);                                            \
          REAL yt = (a * p + e * vt) * iden;                                            \
          ys[t] = yt; zs[t] = iden; zx[t] = kt + uc - no;                               \
          gws += gyt * (dpdw - dqdw * yt) * iden * a;                                   \
          gus += gyt * (vt - yt) * e * iden;                                            \
          no = wc + o > kt ? wc + o : kt;                                               \
          a = EXP(wc + o - no);                                                         \
          e = EXP(kt - no);                                                             \
          dpdw = a * (p + dpdw);                                                        \
          dqdw = a * (q + dqdw);                                                        \
          p = a * p + e * vt;                                                           \
          q = a * q + e;                                                                \
          o = no;                                                                       \
        }                                                                               \
        gw_lane[lane] = gws * wc;                                                       \
        gu_lane[lane] = gus;                                                            \
        /* pass 2: reverse accumulation (wkv_triton.py:120-142) */                      \
        REAL gp = 0, gq = 0;                                                            \
        o = (REAL)-1e38;                                                                \
        for (int64_t ti = 0; ti < T; ++ti) {                                            \
          const int64_t t = T - 1 - ti;                                                 \
          const int64_t off = base + t * C;                                             \
          const REAL kt = k[off], vt = v[off], gyt = gy[off];                           \
          const REAL yt = ys[t], zt = zs[t], zxt = zx[t];                               \
          REAL a = gyt * zt * EXP(zxt);                                                 \
          REAL e = EXP(kt + o);                                                         \
          gk[off] = a * (vt - yt) + e * (gp * vt + gq);                                 \
          gv[off] = a + e * gp;                                                         \
          REAL no = wc + o > zxt - kt - uc ? wc + o : zxt - kt - uc;                    \
          a = EXP(wc + o - no);                                                         \
          e = gyt * zt * EXP(zxt - kt - uc - no);                                       \
          gp = a * gp + e;                                                              \
          gq = a * gq - e * yt;                                                         \
          o = no;                                                                       \
        }                                                                               \
      }                                                                                 \
      free(ys);                                                                         \
    }                                                                                   \
    if (!failed) {                                                                      \
      for (int64_t c = 0; c < C; ++c) {                                                 \
        REAL sw = 0, su = 0;                                                            \
        for (int64_t b = 0; b < B; ++b) { sw += gw_lane[b * C + c]; su += gu_lane[b * C + c]; } \
        g_time_decay[c] = sw;                                                           \
        g_time_first[c] = su;                                                           \
      }                                                                                 \
    }                                                                                   \
    free(gw_lane);                                                                      \
    free(gu_lane);                                                                      \
    return failed ? 2 : 0;                                                              \
  }

WKV_ORACLE_DEFINE(double, f64, exp, -1.7976931348623157e308)
WKV_ORACLE_DEFINE(float, f32, expf, -3.4028234663852886e38f)

/*
 * One recurrent step (generation): the WKV part of SpikeTimeMix.step, reference
 * src/spikegpt/language.py:993-1010, in REAL arithmetic, with the reference's
 * state (numerator, denominator, log_scale; natural-log scale). key, value,
 * numerator, denominator, log_scale, y: [B, C]; time_decay, time_first: [C].
 * The state is updated in place; y receives the step's output before the
 * receptance gate.
 */
#define WKV_ORACLE_STEP_DEFINE(REAL, SUF, EXP)                                               \
  void wkv_oracle_step_##SUF(const REAL* key, const REAL* value, const REAL* time_decay,     \
                             const REAL* time_first, REAL* num, REAL* den, REAL* log_scale,  \
                             REAL* y, int64_t B, int64_t C) {                                \
    for (int64_t b = 0; b < B; ++b) {                                                        \
      for (int64_t c = 0; c < C; ++c) {                                                      \
        const int64_t i = b * C + c;                                                         \
        const REAL k = key[i], v = value[i], s = log_scale[i];                               \
        const REAL w = -EXP(time_decay[c]), u = time_first[c];                               \
        const REAL uk = u + k;                                                               \
        const REAL ns = s > uk ? s : uk;                                                     \
        REAL a = EXP(s - ns), e = EXP(uk - ns);                                              \
        y[i] = (a * num[i] + e * v) / (a * den[i] + e);                                      \
        const REAL ds = s + w;                                                               \
        const REAL rs = ds > k ? ds : k;                                                     \
        a = EXP(ds - rs);                                                                    \
        e = EXP(k - rs);                                                                     \
        num[i] = a * num[i] + e * v;                                                         \
        den[i] = a * den[i] + e;                                                             \
        log_scale[i] = rs;                                                                   \
      }                                                                                      \
    }                                                                                        \
  }

WKV_ORACLE_STEP_DEFINE(double, f64, exp)
WKV_ORACLE_STEP_DEFINE(float, f32, expf)

/*
 * LIF sequence op (reference SpikingSequenceLIF, src/spikegpt/language.py:766-918),
 * per (b, c) over t, in the operation order of the reference's step
 * (language.py:831-841):
 *   v = v * decay + x_t;  centered = slope * (v - threshold);
 *   s_t = centered >= 0;  v = v * (1 - s_t) + reset * s_t
 * with decay = 1 - 1/tau and v = 0 at t = 0. x, s: [B, T, C].
 * The backward is the gradient of that loop under autograd with the spike's
 * surrogate derivative slope * surrogate'(centered), surrogate'(x) =
 * 1 / (2 (1 + (pi/2 x)^2)) (the published arc-tangent surrogate; the
 * reference's own definition lives in myelin@68b8ebb, not available here):
 *   dL/dv_t = ds/dv (gs_t + g (reset - v_t)) + g (1 - s_t),  dL/dx_t = dL/dv_t,
 *   g <- decay * dL/dv_t  (g = dL/d(membrane after step t), 0 after the last step)
 */
#define LIF_ORACLE_DEFINE(REAL, SUF)                                                          \
  void lif_oracle_forward_##SUF(const REAL* x, REAL* spikes, int64_t B, int64_t T, int64_t C, \
                                REAL tau, REAL threshold, REAL reset, REAL slope) {           \
    const REAL decay = (REAL)(1.0 - 1.0 / (double)tau);                                     \
    for (int64_t b = 0; b < B; ++b)                                                           \
      for (int64_t c = 0; c < C; ++c) {                                                       \
        REAL v = 0;                                                                           \
        for (int64_t t = 0; t < T; ++t) {                                                     \
          const int64_t i = (b * T + t) * C + c;                                              \
          v = v * decay + x[i];                                                               \
          const REAL centered = slope * (v - threshold);                                      \
          const REAL s = centered >= 0 ? (REAL)1 : (REAL)0;                                   \
          spikes[i] = s;                                                                      \
          v = v * ((REAL)1 - s) + reset * s;                                                  \
        }                                                                                     \
      }                                                                                       \
  }                                                                                           \
  int lif_oracle_backward_##SUF(const REAL* gs, const REAL* x, REAL* gx, int64_t B, int64_t T, \
                                int64_t C, REAL tau, REAL threshold, REAL reset, REAL slope) { \
    const REAL decay = (REAL)(1.0 - 1.0 / (double)tau);                                     \
    REAL* vs = (REAL*)malloc(sizeof(REAL) * (size_t)(T > 0 ? T : 1));                         \
    if (!vs) return 1;                                                                        \
    for (int64_t b = 0; b < B; ++b)                                                           \
      for (int64_t c = 0; c < C; ++c) {                                                       \
        REAL v = 0;                                                                           \
        for (int64_t t = 0; t < T; ++t) {                                                     \
          const int64_t i = (b * T + t) * C + c;                                              \
          v = v * decay + x[i];                                                               \
          vs[t] = v;                                                                          \
          const REAL s = slope * (v - threshold) >= 0 ? (REAL)1 : (REAL)0;                    \
          v = v * ((REAL)1 - s) + reset * s;                                                  \
        }                                                                                     \
        REAL g = 0;                                                                           \
        for (int64_t t = T - 1; t >= 0; --t) {                                                \
          const int64_t i = (b * T + t) * C + c;                                              \
          const REAL centered = slope * (vs[t] - threshold);                                  \
          const REAL s = centered >= 0 ? (REAL)1 : (REAL)0;                                   \
          const REAL h = (REAL)1.5707963267948966 * centered;                                 \
          const REAL dsdv = slope * ((REAL)0.5 / ((REAL)1 + h * h));                          \
          const REAL gv = dsdv * (gs[i] + g * (reset - vs[t])) + g * ((REAL)1 - s);           \
          gx[i] = gv;                                                                         \
          g = decay * gv;                                                                     \
        }                                                                                     \
      }                                                                                       \
    free(vs);                                                                                 \
    return 0;                                                                                 \
  }

LIF_ORACLE_DEFINE(double, f64)
LIF_ORACLE_DEFINE(float, f32)

/* Number of OpenMP threads the runtime would use by default (1 without OpenMP). */
int wkv_oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
