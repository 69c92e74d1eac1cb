// Device-side building blocks of the WKV recurrence for sm_100a: PTX wrappers
// (MUFU ex2/rcp, packed f32x2 FMA/MUL/ADD, mbarrier, TMA bulk-tensor copies),
// I/O dtype traits, and the per-sub-chunk arithmetic shared by the forward,
// checkpoint and backward kernels in wkv_kernels.cuh.
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
//
// Each thread owns two adjacent channels ("a lane pair"): their recurrences
// advance together with Blackwell's packed fma/mul/add.f32x2, and their I/O
// moves as one 32-bit bf16x2/f16x2 (or 64-bit float2) word.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace wkv {

constexpr float kL2E = 1.4426950408889634f;  // log2(e)
constexpr float kNegBig = -1e38f;            // "log2 of zero" (reference wkv_triton.py:43)
constexpr int kThreads = 32;                 // one warp per CTA
constexpr int kLanes = 2 * kThreads;         // channels per CTA (two per thread)
constexpr int kSub = 16;                     // steps per sub-chunk = checkpoint interval
constexpr int kSegAlign = 32;                // segment lengths are multiples of this
constexpr float kMargin = 60.f;              // log2 headroom kept above fp32's normal range
constexpr unsigned kFull = 0xffffffffu;
constexpr long long kWaitLimitCycles = 4000000000ll;  // ~2 s at 2 GHz

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

struct f2 {
  float x, y;
};

// Packed two-wide fp32 arithmetic (sm_100: one FFMA2/FMUL2/FADD2 per pair).
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
  f2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
  f2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
  f2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ f2 sub2(f2 a, f2 b) {
  f2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "sub.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ f2 ex2x2(f2 a) { return f2{ex2(a.x), ex2(a.y)}; }
__device__ __forceinline__ f2 rcpx2(f2 a) { return f2{rcp(a.x), rcp(a.y)}; }
__device__ __forceinline__ f2 splat(float a) { return f2{a, a}; }

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
// when the phase has not completed within `limit` cycles.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  long long limit = kWaitLimitCycles) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (clock64() - start > limit) return false;
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

// Predicated forms: only the threads with `on` set issue the copy, with no
// branch (the elected-lane `if` of a warp otherwise costs a convergence region).
__device__ __forceinline__ void mbar_arrive_expect_tx_if(bool on, uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %2, 0;\n\t"
      "@p mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes), "r"((uint32_t)on)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d_if(bool on, void* dst, const CUtensorMap* map,
                                               uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %6, 0;\n\t"
      "@p cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];\n\t}" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)),
      "r"((uint32_t)on)
      : "memory");
}
__device__ __forceinline__ void tma_store_3d_if(bool on, const CUtensorMap* map, const void* src,
                                                int x, int y, int z) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.u32 p, %5, 0;\n\t"
      "@p cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];\n\t}" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(x), "r"(y), "r"(z), "r"(smem_u32(src)), "r"((uint32_t)on)
      : "memory");
}

// Bulk groups are per thread: committing or waiting on a thread that issued no
// bulk copy is a no-op, so whole warps may execute these.
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
//
// Pair<T>::raw is the in-memory form of two adjacent elements; unpack widens it
// to f2 (element c in .x, c+1 in .y), pack rounds to nearest even. hi/lo give a
// raw pair the packed max/min identity for the prescan.

template <typename T>
struct Pair;

// Widens the two 16-bit floats of a packed word (element c in the low half) to
// float32 with sm_100's mixed-precision add, d = a + (-0.0) with a 16-bit
// source: one FP32-pipe instruction per value instead of a shift or a mask on
// the integer pipe, and exact (adding -0.0 keeps every value, signed zeros,
// subnormals and infinities included).
template <bool kHalf>
__device__ __forceinline__ f2 unpack16(uint32_t r) {
  f2 d;
  if constexpr (kHalf)
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
        "add.rn.f32.f16 %0, l, 0f80000000;\n\tadd.rn.f32.f16 %1, h, 0f80000000;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "r"(r));
  else
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
        "add.rn.f32.bf16 %0, l, 0f80000000;\n\tadd.rn.f32.bf16 %1, h, 0f80000000;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "r"(r));
  return d;
}

template <>
struct Pair<float> {
  using raw = float2;
  static constexpr int kTileRows = 16;  // 16 rows x 64 channels x 4 B = 4 KB tiles
  static __device__ __forceinline__ raw ld(const float* p) {
    return *reinterpret_cast<const float2*>(p);
  }
  static __device__ __forceinline__ void st(float* p, raw r) { *reinterpret_cast<float2*>(p) = r; }
  static __device__ __forceinline__ f2 unpack(raw r) { return f2{r.x, r.y}; }
  static __device__ __forceinline__ raw pack(f2 v) { return make_float2(v.x, v.y); }
  // (p0 ? 1 : 0, p1 ? 1 : 0) by integer selects of the constant's bits
  static __device__ __forceinline__ raw ones(bool p0, bool p1) {
    return make_float2(__int_as_float(p0 ? 0x3f800000 : 0), __int_as_float(p1 ? 0x3f800000 : 0));
  }
  static __device__ __forceinline__ float scalar(float x) { return x; }
  static __device__ __forceinline__ float from_float(float x) { return x; }
};

template <>
struct Pair<__nv_bfloat16> {
  using raw = uint32_t;
  static constexpr int kTileRows = 32;  // 32 rows x 64 channels x 2 B = 4 KB tiles
  static __device__ __forceinline__ raw ld(const __nv_bfloat16* p) {
    return *reinterpret_cast<const uint32_t*>(p);
  }
  static __device__ __forceinline__ void st(__nv_bfloat16* p, raw r) {
    *reinterpret_cast<uint32_t*>(p) = r;
  }
  static __device__ __forceinline__ f2 unpack(raw r) { return unpack16<false>(r); }
  static __device__ __forceinline__ raw pack(f2 v) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(v.y), "f"(v.x));
    return d;
  }
  static __device__ __forceinline__ raw ones(bool p0, bool p1) {
    return (p0 ? 0x3f80u : 0u) | (p1 ? 0x3f800000u : 0u);
  }
  static __device__ __forceinline__ float scalar(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_float(float x) { return __float2bfloat16_rn(x); }
};

template <>
struct Pair<__half> {
  using raw = uint32_t;
  static constexpr int kTileRows = 32;
  static __device__ __forceinline__ raw ld(const __half* p) {
    return *reinterpret_cast<const uint32_t*>(p);
  }
  static __device__ __forceinline__ void st(__half* p, raw r) { *reinterpret_cast<uint32_t*>(p) = r; }
  static __device__ __forceinline__ f2 unpack(raw r) { return unpack16<true>(r); }
  static __device__ __forceinline__ raw pack(f2 v) {
    uint32_t d;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(v.y), "f"(v.x));
    return d;
  }
  static __device__ __forceinline__ raw ones(bool p0, bool p1) {
    return (p0 ? 0x3c00u : 0u) | (p1 ? 0x3c000000u : 0u);
  }
  static __device__ __forceinline__ float scalar(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_float(float x) { return __float2half_rn(x); }
};

// ------------------------------------------------------------------- state

// Decay over n steps, ew^n = m 2^e (m in [0.5, 1), e an integer; m = 0 and
// e = kNegBig once it underflows), where ew is the float32 per-step factor the recurrences
// multiply by. The power is formed in double from that same float, so a state
// decayed by a combine and a state decayed step by step carry the same
// systematic rounding of ew. The backward's adjoint decays step by step with
// ew; states whose decay differs from ew^n by even a few ulps (e.g. 2^{w n
// log2 e} through ex2) make the gradients near dominant keys several times less
// accurate, because the adjoint sums cancel.
struct Decay1 {
  float m, e;
};
__device__ __forceinline__ Decay1 ew_decay(float ew, int n) {
  double x = static_cast<double>(ew), r = 1.0;
  for (int k = n; k > 0; k >>= 1) {
    if (k & 1) r *= x;
    x *= x;
  }
  if (!(r > 0.0)) return Decay1{0.f, kNegBig};
  int ex = 0;
  const double m = frexp(r, &ex);
  return Decay1{static_cast<float>(m), static_cast<float>(ex)};
}

// Per-channel constants of a lane pair. w = -exp(time_decay) <= 0 (reference
// wkv_triton.py:152).
struct Lane2 {
  f2 w;     // natural-log decay per step
  f2 w2;    // w * log2(e)
  f2 u2;    // time_first * log2(e)
  f2 ew;    // e^w
  f2 eu;    // e^u
  f2 dm16;  // ew^kSub = dm16 2^de16 (see ew_decay)
  f2 de16;
};

__device__ __forceinline__ Lane2 make_lane2(f2 w, f2 u) {
  Lane2 l;
  l.w = w;
  l.w2 = f2{w.x * kL2E, w.y * kL2E};
  l.u2 = f2{u.x * kL2E, u.y * kL2E};
  l.ew = f2{expf(w.x), expf(w.y)};
  l.eu = f2{expf(u.x), expf(u.y)};
  const Decay1 dx = ew_decay(l.ew.x, kSub), dy = ew_decay(l.ew.y, kSub);
  l.dm16 = f2{dx.m, dy.m};
  l.de16 = f2{dx.e, dy.e};
  return l;
}

struct Fwd2 {  // P = 2^S p, Q = 2^S q, per lane of the pair
  f2 S, p, q;
};
// Adjoint at a step boundary t: dL/dP_t = 2^G gp, dL/dQ_t = 2^G gq, and their
// derivatives with respect to w, d(dL/dP_t)/dw = 2^G hp, d(dL/dQ_t)/dw = 2^G hq.
// With H_t = d(dL/dP_t)/dw = e^w (dL/dP_{t+1} + H_{t+1}), the decay gradient is
// dL/dw = sum_s e^{k_s} (v_s H^P_{s+1} + H^Q_{s+1}).
struct Adj2 {
  f2 G, gp, gq, hp, hq;
};

__device__ __forceinline__ Fwd2 fwd_identity2() {
  return Fwd2{splat(kNegBig), splat(0.f), splat(0.f)};
}
__device__ __forceinline__ Adj2 adj_zero2() {
  return Adj2{splat(kNegBig), splat(0.f), splat(0.f), splat(0.f), splat(0.f)};
}

// State after `delta` more steps of pure decay from g, plus a local state l
// that was accumulated from zero over those same steps (P is linear in the
// history, so the two parts add); d = ew^delta (ew_decay). One lane.
// All scales are integers (see fast_ok1), so the new scale s is exact and each
// part is rescaled by one rounding: g by d.m 2^{gS + d.e - s}, l by 2^{lS - s}.
__device__ __forceinline__ void fwd_combine1(float gS, float gp, float gq, Decay1 d, float& lS,
                                             float& lp, float& lq) {
  const float ge = gS + d.e;
  const float s = fmaxf(ge, lS);
  const float a = d.m * ex2(ge - s), b = ex2(lS - s);
  lp = fmaf(gp, a, lp * b);
  lq = fmaf(gq, a, lq * b);
  lS = s;
}

// The decay ew^delta of both lanes as (mantissas, integer exponents).
__device__ __forceinline__ void ew_decay2(const Lane2& lc, int delta, f2& m, f2& e) {
  if (delta == kSub) {
    m = lc.dm16;
    e = lc.de16;
  } else {
    const Decay1 dx = ew_decay(lc.ew.x, delta), dy = ew_decay(lc.ew.y, delta);
    m = f2{dx.m, dy.m};
    e = f2{dx.e, dy.e};
  }
}

// fwd_combine1 for both lanes of the pair with packed arithmetic (the same
// roundings lane by lane).
__device__ __forceinline__ Fwd2 fwd_combine2(const Fwd2& g, int delta, const Lane2& lc,
                                             Fwd2 l) {
  f2 dm, de;
  ew_decay2(lc, delta, dm, de);
  const f2 ge = add2(g.S, de);
  const f2 s = f2{fmaxf(ge.x, l.S.x), fmaxf(ge.y, l.S.y)};
  const f2 a = mul2(dm, ex2x2(sub2(ge, s)));
  const f2 b = ex2x2(sub2(l.S, s));
  l.p = fma2(g.p, a, mul2(l.p, b));
  l.q = fma2(g.q, a, mul2(l.q, b));
  l.S = s;
  return l;
}

// fwd_combine2 over exactly kSub steps (the decay ew^kSub precomputed in lc):
// branch-free, so a run of them schedules as one short chain of scales, ex2s
// that do not wait on each other, and multiply-add chains. Same roundings.
__device__ __forceinline__ Fwd2 fwd_combine16(const Fwd2& g, const Lane2& lc, Fwd2 l) {
  const f2 ge = add2(g.S, lc.de16);
  const f2 s = f2{fmaxf(ge.x, l.S.x), fmaxf(ge.y, l.S.y)};
  const f2 a = mul2(lc.dm16, ex2x2(sub2(ge, s)));
  const f2 b = ex2x2(sub2(l.S, s));
  l.p = fma2(g.p, a, mul2(l.p, b));
  l.q = fma2(g.q, a, mul2(l.q, b));
  l.S = s;
  return l;
}

// Adjoint at the start of a segment of `len` steps: its own contribution
// `local` (accumulated from a zero adjoint) plus the adjoint at the segment end
// decayed through the segment, e^{w len} dL/dP_end; the w-derivatives pick up
// the product rule term len e^{w len} dL/dP_end. d = ew^len (ew_decay). One
// lane; l = local, e = end (overwritten with the result).
__device__ __forceinline__ void adj_combine1(const float (&l)[5], float (&e)[5], int len,
                                             Decay1 d) {
  const float fl = static_cast<float>(len);
  const float ge = e[0] + d.e;
  const float g = fmaxf(ge, l[0]);
  const float a = d.m * ex2(ge - g), b = ex2(l[0] - g);
  const float hp = fmaf(fl, e[1], e[3]), hq = fmaf(fl, e[2], e[4]);
  e[1] = fmaf(e[1], a, l[1] * b);
  e[2] = fmaf(e[2], a, l[2] * b);
  e[3] = fmaf(hp, a, l[3] * b);
  e[4] = fmaf(hq, a, l[4] * b);
  e[0] = g;
}

// One exact step of the state update with per-step rescaling (the second half
// of the reference loop body, wkv_triton.py:53-58), in log2 units. One lane.
__device__ __forceinline__ void slow_update(float& o, float& p, float& q, float k, float v,
                                            float w2) {
  const float k2 = k * kL2E;
  const float wo = w2 + o;
  const float no = fmaxf(wo, k2);
  const float a = ex2(wo - no), b = ex2(k2 - no);
  p = fmaf(a, p, b * v);
  q = fmaf(a, q, b);
  o = no;
}

// Fast-path admissibility for one lane over a sub-chunk of L steps starting
// from state (S, p, q). Outputs the sub-chunk scale s and the carried state
// rescaled to it.
//
// Scales are integers (log2 units) throughout: a change of scale then
// multiplies by an exact power of two (ex2 of an integer argument is exact on
// sm_100a), so state and adjoint pick up no rounding when consecutive
// sub-chunks use different scales. Non-integer scales cost ~2^-22 relative per
// change, which accumulates along T in the adjoint chain.
__device__ __forceinline__ bool fast_ok1(float S, float p0, float q0, float kmax, float kmin,
                                         int L, float w2, float u2, float& s, float& p,
                                         float& q) {
  s = fmaxf(S, ceilf(kmax * kL2E));
  const float c = ex2(S - s);
  p = p0 * c;
  q = q0 * c;
  // den_t >= max(q e^{w t}, e^{u + k_t}) / 2^s; e^{k_t}/2^s bounds the q update.
  const float decayed = q * ex2(w2 * static_cast<float>(L));
  const float low = fmaf(kmin, kL2E, -s) + fminf(u2, 0.f);
  return (w2 <= 0.f) && (fabsf(u2) <= 64.f) && (s < 1e30f) &&
         (decayed >= 0x1p-60f || low >= -kMargin);
}

}  // namespace wkv
