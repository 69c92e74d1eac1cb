// Device-side building blocks of the WKV recurrence for sm_100a: PTX wrappers
// (MUFU ex2/rcp, mbarrier, TMA bulk-tensor copies), I/O dtype traits, and the
// per-sub-chunk arithmetic shared by the forward, checkpoint and backward
// kernels in wkv_kernels.cuh.
//
// The recurrence is the RWKV-4 WKV of the reference (src/spikegpt/language.py:
// 399-449, src/spikegpt/wkv_triton.py:34-142). Per lane (b, c), with
// P_t = sum_{s<t} e^{w(t-1-s)+k_s} v_s and Q_t likewise with v = 1:
//     y_t     = (P_t + e^{u+k_t} v_t) / (Q_t + e^{u+k_t})
//     P_{t+1} = e^w P_t + e^{k_t} v_t,   Q_{t+1} = e^w Q_t + e^{k_t}
// State is carried as (S, p, q) with P = 2^S p, Q = 2^S q (log2 units).
//
// Fast path ("fixed sub-chunk scale"): for a sub-chunk of kSub steps the lane
// picks one scale s = max(S, max_t k_t*log2e) and runs the recurrence with one
// ex2 and one rcp per step and no per-step max/select. It is taken only when a
// cheap check proves every denominator stays >= 2^-kMargin (no underflow) and no
// term can overflow; otherwise the warp runs the exact per-step-rescaling
// arithmetic of the reference for that sub-chunk ("slow path").
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace wkv {

constexpr float kL2E = 1.4426950408889634f;  // log2(e)
constexpr float kNegBig = -1e38f;            // "log2 of zero" (reference wkv_triton.py:43)
constexpr int kLanes = 32;                   // channels per CTA: one warp, one lane each
constexpr int kSub = 16;                     // steps per sub-chunk = checkpoint interval
constexpr int kTile = 32;                    // steps per staged tile
constexpr int kSubPerTile = kTile / kSub;
constexpr float kMargin = 60.f;              // log2 headroom kept above fp32's normal range
constexpr unsigned kFull = 0xffffffffu;
constexpr long long kWaitLimitCycles = 4000000000ll;  // ~2 s at 2 GHz

static_assert(kTile % kSub == 0, "tile must hold whole sub-chunks");

// ---------------------------------------------------------------- PTX helpers

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase: returns false (and never spins forever)
// when the phase has not completed within kWaitLimitCycles.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - start > kWaitLimitCycles) return false;
  }
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x,
                                             int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(x), "r"(y), "r"(z), "r"(smem_u32(src))
      : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N committed bulk stores still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------------ I/O dtype traits

template <typename T>
struct IOType;
template <>
struct IOType<float> {
  static __device__ __forceinline__ float ld(float x) { return x; }
  static __device__ __forceinline__ float st(float x) { return x; }
};
template <>
struct IOType<__nv_bfloat16> {
  static __device__ __forceinline__ float ld(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 st(float x) { return __float2bfloat16_rn(x); }
};
template <>
struct IOType<__half> {
  static __device__ __forceinline__ float ld(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half st(float x) { return __float2half_rn(x); }
};

// ------------------------------------------------------------------- state

// Per-channel constants. w = -exp(time_decay) <= 0 (reference wkv_triton.py:152).
struct Lane {
  float w;   // natural-log decay per step
  float w2;  // w * log2(e)
  float u2;  // time_first * log2(e)
  float ew;  // e^w
  float eu;  // e^u
};

__device__ __forceinline__ Lane make_lane(float w, float u) {
  Lane l;
  l.w = w;
  l.w2 = w * kL2E;
  l.u2 = u * kL2E;
  l.ew = expf(w);
  l.eu = expf(u);
  return l;
}

struct Fwd {  // P = 2^S p, Q = 2^S q
  float S, p, q;
};
struct Adj {  // dL/dP = 2^G gp, dL/dQ = 2^G gq
  float G, gp, gq;
};

__device__ __forceinline__ Fwd fwd_identity() { return Fwd{kNegBig, 0.f, 0.f}; }
__device__ __forceinline__ Adj adj_zero() { return Adj{kNegBig, 0.f, 0.f}; }

// State after `delta` more steps of pure decay from g, plus a local state l
// that was accumulated from zero over those same steps (P is linear in the
// history, so the two parts add).
__device__ __forceinline__ Fwd fwd_combine(const Fwd& g, int delta, const Lane& lc,
                                           const Fwd& l) {
  const float sg = g.S + lc.w2 * static_cast<float>(delta);
  const float s = fmaxf(sg, l.S);
  const float a = ex2(sg - s), b = ex2(l.S - s);
  return Fwd{s, fmaf(g.p, a, l.p * b), fmaf(g.q, a, l.q * b)};
}

// Adjoint at the start of a segment of `len` steps: its own contribution
// `local` (accumulated from a zero adjoint) plus the adjoint at the segment end
// decayed through the segment.
__device__ __forceinline__ Adj adj_combine(const Adj& local, const Adj& end, int len,
                                           const Lane& lc) {
  const float ge = end.G + lc.w2 * static_cast<float>(len);
  const float g = fmaxf(ge, local.G);
  const float a = ex2(ge - g), b = ex2(local.G - g);
  return Adj{g, fmaf(end.gp, a, local.gp * b), fmaf(end.gq, a, local.gq * b)};
}

// One exact step of the state update with per-step rescaling (the second half
// of the reference loop body, wkv_triton.py:53-58), in log2 units.
__device__ __forceinline__ void slow_update(float& o, float& p, float& q, float k, float v,
                                            const Lane& lc) {
  const float k2 = k * kL2E;
  const float wo = lc.w2 + o;
  const float no = fmaxf(wo, k2);
  const float a = ex2(wo - no), b = ex2(k2 - no);
  p = fmaf(a, p, b * v);
  q = fmaf(a, q, b);
  o = no;
}

// Fast-path admissibility for a sub-chunk of L steps starting from state st.
// s: the sub-chunk scale; p, q: the carried state rescaled to s.
__device__ __forceinline__ bool fast_ok(const Fwd& st, float kmax, float kmin, int L,
                                        const Lane& lc, float& s, float& p, float& q) {
  s = fmaxf(st.S, kmax * kL2E);
  const float c = ex2(st.S - s);
  p = st.p * c;
  q = st.q * c;
  // den_t >= max(q e^{w t}, e^{u + k_t}) / 2^s; e^{k_t}/2^s bounds the q update.
  const float decayed = q * ex2(lc.w2 * static_cast<float>(L));
  const float low = fmaf(kmin, kL2E, -s) + fminf(lc.u2, 0.f);
  return (lc.w2 <= 0.f) && (fabsf(lc.u2) <= 64.f) && (s < 1e30f) &&
         (decayed >= 0x1p-60f || low >= -kMargin);
}

// Masked tree reductions over a sub-chunk held in registers.
template <bool kTail>
__device__ __forceinline__ void minmax16(const float (&x)[kSub], int L, float& mx, float& mn) {
  float a[kSub / 2], b[kSub / 2];
#pragma unroll
  for (int i = 0; i < kSub / 2; ++i) {
    const bool i0 = !kTail || i < L, i1 = !kTail || i + kSub / 2 < L;
    const float x0 = x[i], x1 = x[i + kSub / 2];
    a[i] = fmaxf(i0 ? x0 : -INFINITY, i1 ? x1 : -INFINITY);
    b[i] = fminf(i0 ? x0 : INFINITY, i1 ? x1 : INFINITY);
  }
#pragma unroll
  for (int w = kSub / 4; w > 0; w /= 2) {
#pragma unroll
    for (int i = 0; i < w; ++i) {
      a[i] = fmaxf(a[i], a[i + w]);
      b[i] = fminf(b[i], b[i + w]);
    }
  }
  mx = a[0];
  mn = b[0];
}

template <bool kTail>
__device__ __forceinline__ float absmax16(const float (&x)[kSub], int L) {
  float a[kSub / 2];
#pragma unroll
  for (int i = 0; i < kSub / 2; ++i) {
    const bool i0 = !kTail || i < L, i1 = !kTail || i + kSub / 2 < L;
    a[i] = fmaxf(i0 ? fabsf(x[i]) : 0.f, i1 ? fabsf(x[i + kSub / 2]) : 0.f);
  }
#pragma unroll
  for (int w = kSub / 4; w > 0; w /= 2) {
#pragma unroll
    for (int i = 0; i < w; ++i) a[i] = fmaxf(a[i], a[i + w]);
  }
  return a[0];
}

// Loads a sub-chunk column (kSub rows, stride kLanes) into registers. Rows past
// L inside the staged tile are zero-filled or stale; they are masked by callers.
template <typename T>
__device__ __forceinline__ void load16(float (&r)[kSub], const T* src) {
#pragma unroll
  for (int i = 0; i < kSub; ++i) r[i] = IOType<T>::ld(src[i * kLanes]);
}

// ------------------------------------------------------ forward sub-chunk
//
// Advances st over L (<= kSub) steps whose k/v sit in shared memory at
// ks[i*kLanes], vs[i*kLanes]; with kY writes y to ys[i*kLanes]. Inputs are
// staged into registers first and outputs written last, so the 16 steps are
// free to overlap (the only true dependency is the p/q recurrence).
template <typename T, bool kTail, bool kY>
__device__ __forceinline__ void fwd_sub(Fwd& st, const T* ks, const T* vs, T* ys, int L,
                                        const Lane& lc, bool force_slow) {
  using io = IOType<T>;
  float kr[kSub], vr[kSub], yr[kSub];
  load16(kr, ks);
  load16(vr, vs);
  float kmax, kmin;
  minmax16<kTail>(kr, L, kmax, kmin);
  float s, p, q;
  const bool ok = fast_ok(st, kmax, kmin, kTail ? L : kSub, lc, s, p, q) && !force_slow;
  if (__all_sync(kFull, ok)) {
#pragma unroll
    for (int i = 0; i < kSub; ++i) {
      if (kTail && i >= L) break;
      const float ek = ex2(fmaf(kr[i], kL2E, -s));
      if (kY) {
        const float eb = ek * lc.eu;
        yr[i] = fmaf(eb, vr[i], p) * rcp(q + eb);
      }
      p = fmaf(lc.ew, p, ek * vr[i]);
      q = fmaf(lc.ew, q, ek);
    }
    st = Fwd{s, p, q};
  } else {
    float o = st.S;
    p = st.p;
    q = st.q;
#pragma unroll
    for (int i = 0; i < kSub; ++i) {
      if (kTail && i >= L) break;
      if (kY) {  // reference wkv_triton.py:49-52
        const float uk = lc.u2 + kr[i] * kL2E;
        const float no = fmaxf(o, uk);
        const float a = ex2(o - no), b = ex2(uk - no);
        yr[i] = fmaf(a, p, b * vr[i]) * rcp(fmaf(a, q, b));
      }
      slow_update(o, p, q, kr[i], vr[i], lc);
    }
    st = Fwd{o, p, q};
  }
  if (kY) {
#pragma unroll
    for (int i = 0; i < kSub; ++i)
      if (!kTail || i < L) ys[i * kLanes] = io::st(yr[i]);
  }
}

// ----------------------------------------------------- backward sub-chunk
//
// Given the forward state st0 at the sub-chunk start and the adjoint at its end,
// produces grad_key / grad_value for its L steps (kOut), accumulates
// gwacc += sum_t (dL/dP_{t+1} P_t + dL/dQ_{t+1} Q_t)  (dL/dw = e^w gwacc) and
// gu += dL/du, and leaves the adjoint at the sub-chunk start in adj.
template <typename T, bool kTail, bool kOut>
__device__ __forceinline__ void bwd_sub(const Fwd& st0, Adj& adj, const T* ks, const T* vs,
                                        const T* gys, T* gks, T* gvs, int L, const Lane& lc,
                                        float& gwacc, float& gu, bool force_slow) {
  using io = IOType<T>;
  float kr[kSub], vr[kSub], gr[kSub];
  load16(kr, ks);
  load16(vr, vs);
  load16(gr, gys);
  float kmax, kmin;
  minmax16<kTail>(kr, L, kmax, kmin);
  const float gymax = absmax16<kTail>(gr, L);
  float s, p, q;
  bool ok = fast_ok(st0, kmax, kmin, kTail ? L : kSub, lc, s, p, q) && !force_slow;
  // Adjoint rescaled to the sub-chunk scale: dL/dP = 2^{-s} gp.
  const float f = ex2(adj.G + s);
  float gp = adj.gp * f, gq = adj.gq * f;
  ok = ok && (gymax <= 0x1p40f) && (fabsf(gp) <= 0x1p80f) && (fabsf(gq) <= 0x1p80f);
  if (__all_sync(kFull, ok)) {
    float ry[kSub], rg[kSub], re[kSub], rp[kSub], rq[kSub];
    // forward recompute of the sub-chunk
#pragma unroll
    for (int i = 0; i < kSub; ++i) {
      if (kTail && i >= L) break;
      const float ek = ex2(fmaf(kr[i], kL2E, -s));
      const float eb = ek * lc.eu;
      const float rd = rcp(q + eb);
      ry[i] = fmaf(eb, vr[i], p) * rd;
      rg[i] = gr[i] * rd;  // gy * 2^s / D_t
      re[i] = ek;
      rp[i] = p;
      rq[i] = q;
      p = fmaf(lc.ew, p, ek * vr[i]);
      q = fmaf(lc.ew, q, ek);
    }
    // reverse sweep
#pragma unroll
    for (int i = kSub - 1; i >= 0; --i) {
      if (kTail && i >= L) continue;
      const float v = vr[i];
      const float a = rg[i] * re[i] * lc.eu;  // gy e^{u+k} / D
      const float av = a * (v - ry[i]);
      gu += av;
      gwacc = fmaf(gp, rp[i], fmaf(gq, rq[i], gwacc));
      if (kOut) {
        gvs[i * kLanes] = io::st(fmaf(re[i], gp, a));
        gks[i * kLanes] = io::st(fmaf(re[i], fmaf(gp, v, gq), av));
      }
      gq = fmaf(lc.ew, gq, -rg[i] * ry[i]);
      gp = fmaf(lc.ew, gp, rg[i]);
    }
    adj = Adj{-s, gp, gq};
  } else {
    // Exact path: for each step (last to first) replay the forward from st0 with
    // per-step rescaling (reference wkv_triton.py:93-115), then take the reverse
    // step of wkv_triton.py:124-142 with its own adjoint log-scale G.
    float G = adj.G;
    gp = adj.gp;
    gq = adj.gq;
#pragma unroll 1
    for (int i = L - 1; i >= 0; --i) {
      float o = st0.S, pp = st0.p, qq = st0.q;
#pragma unroll 1
      for (int j = 0; j < i; ++j)
        slow_update(o, pp, qq, io::ld(ks[j * kLanes]), io::ld(vs[j * kLanes]), lc);
      const float k = io::ld(ks[i * kLanes]), v = io::ld(vs[i * kLanes]);
      const float gy = io::ld(gys[i * kLanes]);
      const float k2 = k * kL2E, uk = lc.u2 + k2;
      const float no = fmaxf(o, uk);
      const float a = ex2(o - no), b = ex2(uk - no);
      const float iden = rcp(fmaf(a, qq, b));
      const float y = fmaf(a, pp, b * v) * iden;
      const float A = gy * iden * b;
      const float av = A * (v - y);
      gu += av;
      const float t = fmaf(gp, pp, gq * qq);
      if (t != 0.f) gwacc = fmaf(ex2(o + G), t, gwacc);
      if (kOut) {
        const float ekg = (gp != 0.f || gq != 0.f) ? ex2(k2 + G) : 0.f;
        gvs[i * kLanes] = io::st(fmaf(ekg, gp, A));
        gks[i * kLanes] = io::st(fmaf(ekg, fmaf(gp, v, gq), av));
      }
      // dL/dP_t = gy / D_t + e^w dL/dP_{t+1}, with 1/D_t = iden 2^{-no}
      const float ng = fmaxf(lc.w2 + G, -no);
      const float aa = ex2(lc.w2 + G - ng);
      const float bb = ex2(-no - ng) * gy * iden;
      gp = fmaf(aa, gp, bb);
      gq = fmaf(aa, gq, -bb * y);
      G = ng;
    }
    adj = Adj{G, gp, gq};
  }
}

}  // namespace wkv
