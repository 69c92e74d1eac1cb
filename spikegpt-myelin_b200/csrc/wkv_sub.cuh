// Per-sub-chunk arithmetic of the WKV recurrence for one lane pair (two adjacent
// channels per thread). A sub-chunk is kSub consecutive time steps of a staged
// shared-memory tile: element (row r, channel pair of this thread) sits at
// tile[r * kLanes + 2 * threadIdx.x]. See wkv_device.cuh for the state
// representation and the fast/exact split.
#pragma once

#include "wkv_device.cuh"

namespace wkv {

// Packed prescan: max/min of k and max|grad_y| over the rows of a sub-chunk, on
// the raw I/O words (bf16x2/f16x2 compares are exact on the stored values).
template <typename T>
struct Scan;

template <>
struct Scan<__nv_bfloat16> {
  using raw = uint32_t;
  static constexpr raw kLo = 0xff80ff80u;  // (-inf, -inf)
  static constexpr raw kHi = 0x7f807f80u;  // (+inf, +inf)
  static __device__ __forceinline__ raw vmax(raw a, raw b) {
    raw d;
    asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  static __device__ __forceinline__ raw vmin(raw a, raw b) {
    raw d;
    asm("min.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  static __device__ __forceinline__ raw vabs(raw a) { return a & 0x7fff7fffu; }
};

template <>
struct Scan<__half> {
  using raw = uint32_t;
  static constexpr raw kLo = 0xfc00fc00u;
  static constexpr raw kHi = 0x7c007c00u;
  static __device__ __forceinline__ raw vmax(raw a, raw b) {
    raw d;
    asm("max.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  static __device__ __forceinline__ raw vmin(raw a, raw b) {
    raw d;
    asm("min.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
  static __device__ __forceinline__ raw vabs(raw a) { return a & 0x7fff7fffu; }
};

template <>
struct Scan<float> {
  using raw = float2;
  static __device__ __forceinline__ raw lo() { return make_float2(-INFINITY, -INFINITY); }
  static __device__ __forceinline__ raw hi() { return make_float2(INFINITY, INFINITY); }
  static __device__ __forceinline__ raw vmax(raw a, raw b) {
    return make_float2(fmaxf(a.x, b.x), fmaxf(a.y, b.y));
  }
  static __device__ __forceinline__ raw vmin(raw a, raw b) {
    return make_float2(fminf(a.x, b.x), fminf(a.y, b.y));
  }
  static __device__ __forceinline__ raw vabs(raw a) { return make_float2(fabsf(a.x), fabsf(a.y)); }
};

template <typename T>
__device__ __forceinline__ typename Pair<T>::raw scan_lo() {
  if constexpr (sizeof(T) == 4) return Scan<T>::lo(); else return Scan<T>::kLo;
}
template <typename T>
__device__ __forceinline__ typename Pair<T>::raw scan_hi() {
  if constexpr (sizeof(T) == 4) return Scan<T>::hi(); else return Scan<T>::kHi;
}

// Checkpoint rows of 3 [C] planes ([row][3][C] floats: S, p, q) for the two
// channels c, c+1 of a lane pair.
__device__ __forceinline__ void store_state(float* base, size_t row, int C, int c, bool v0, bool v1,
                                            f2 S, f2 p, f2 q) {
  float* r = base + row * 3 * (size_t)C + c;
  if (v0) {
    r[0] = S.x;
    r[C] = p.x;
    r[2 * (size_t)C] = q.x;
  }
  if (v1) {
    r[1] = S.y;
    r[C + 1] = p.y;
    r[2 * (size_t)C + 1] = q.y;
  }
}

// Range summary of one sub-chunk.
struct Pre {
  f2 kmax, kmin, gymax;
};

// Tree max/min of k (and max |grad_y| when gys != nullptr) over rows [0, L) of a
// sub-chunk in shared memory, rows RS elements apart (rows past L excluded when
// kTail).
template <typename T, bool kTail, bool kGy, int RS = kLanes>
__device__ __forceinline__ Pre prescan(const T* ks, const T* gys, int L) {
  using S = Scan<T>;
  using P = Pair<T>;
  using raw = typename P::raw;
  raw a[kSub / 2], b[kSub / 2], g[kSub / 2];
#pragma unroll
  for (int i = 0; i < kSub / 2; ++i) {
    const bool i0 = !kTail || i < L, i1 = !kTail || i + kSub / 2 < L;
    const raw x0 = P::ld(ks + i * RS), x1 = P::ld(ks + (i + kSub / 2) * RS);
    a[i] = S::vmax(i0 ? x0 : scan_lo<T>(), i1 ? x1 : scan_lo<T>());
    b[i] = S::vmin(i0 ? x0 : scan_hi<T>(), i1 ? x1 : scan_hi<T>());
    if (kGy) {
      const raw g0 = P::ld(gys + i * RS), g1 = P::ld(gys + (i + kSub / 2) * RS);
      g[i] = S::vmax(S::vabs(i0 ? g0 : scan_lo<T>()), S::vabs(i1 ? g1 : scan_lo<T>()));
    }
  }
#pragma unroll
  for (int w = kSub / 4; w > 0; w /= 2) {
#pragma unroll
    for (int i = 0; i < w; ++i) {
      a[i] = S::vmax(a[i], a[i + w]);
      b[i] = S::vmin(b[i], b[i + w]);
      if (kGy) g[i] = S::vmax(g[i], g[i + w]);
    }
  }
  Pre r;
  r.kmax = P::unpack(a[0]);
  r.kmin = P::unpack(b[0]);
  r.gymax = kGy ? P::unpack(g[0]) : splat(0.f);
  return r;
}

// ---------------------------------------------------------- exact (slow) path

// Forward over L steps of one lane with per-step rescaling (reference
// wkv_triton.py:45-58). ks/vs/ys point at this lane's element of row 0; input
// rows are `stride` elements apart, output rows `ystride` (kLanes in a staged
// tile, C in global memory).
template <typename T, bool kY>
__device__ __noinline__ void fwd_slow1(float& S, float& p, float& q, const T* ks, const T* vs,
                                       T* ys, int L, float w2, float u2, int stride = kLanes,
                                       int ystride = kLanes) {
  using P = Pair<T>;
  float o = S;
  for (int i = 0; i < L; ++i) {
    const size_t r = (size_t)i * stride;
    const float k = P::scalar(ks[r]), v = P::scalar(vs[r]);
    if (kY) {
      const float uk = u2 + k * kL2E;
      const float no = fmaxf(o, uk);
      const float a = ex2(o - no), b = ex2(uk - no);
      ys[(size_t)i * ystride] = P::from_float(fmaf(a, p, b * v) * rcp(fmaf(a, q, b)));
    }
    slow_update(o, p, q, k, v, w2);
  }
  // back to an integer scale (see fast_ok1)
  S = ceilf(o);
  const float f = ex2(o - S);
  p *= f;
  q *= f;
}

// Backward over L steps of one lane: for each step (last to first) replay the
// forward from the sub-chunk start with per-step rescaling (reference
// wkv_triton.py:93-115), then take the reverse step of wkv_triton.py:124-142
// with its own adjoint log-scale G (adj = {G, gp, gq, hp, hq}, see Adj2).
// O(L^2) work; only taken when the fast path's range checks fail.
// Inputs are read at rows `istride` elements apart, outputs written `ostride`
// apart (kLanes in a staged tile, C in global memory).
template <typename T, bool kOut>
__device__ __noinline__ void bwd_slow1(float S0, float p0, float q0, float (&adj)[5], const T* ks,
                                       const T* vs, const T* gys, T* gks, T* gvs, int L, float w2,
                                       float u2, float& gwacc, float& gu, int istride = kLanes,
                                       int ostride = kLanes) {
  using P = Pair<T>;
  float G = adj[0], gp = adj[1], gq = adj[2], hp = adj[3], hq = adj[4];
  for (int i = L - 1; i >= 0; --i) {
    float o = S0, pp = p0, qq = q0;
    for (int j = 0; j < i; ++j)
      slow_update(o, pp, qq, P::scalar(ks[(size_t)j * istride]), P::scalar(vs[(size_t)j * istride]), w2);
    const size_t ri = (size_t)i * istride;
    const float k = P::scalar(ks[ri]), v = P::scalar(vs[ri]);
    const float gy = P::scalar(gys[ri]);
    const float k2 = k * kL2E, uk = u2 + k2;
    const float no = fmaxf(o, uk);
    const float a = ex2(o - no), b = ex2(uk - no);
    const float iden = rcp(fmaf(a, qq, b));
    const float y = fmaf(a, pp, b * v) * iden;
    const float A = gy * iden * b;
    const float av = A * (v - y);
    gu += av;
    const bool live = gp != 0.f || gq != 0.f || hp != 0.f || hq != 0.f;
    const float ekg = live ? ex2(k2 + G) : 0.f;  // e^k 2^G
    gwacc = fmaf(ekg, fmaf(v, hp, hq), gwacc);
    if (kOut) {
      gvs[(size_t)i * ostride] = P::from_float(fmaf(ekg, gp, A));
      gks[(size_t)i * ostride] = P::from_float(fmaf(ekg, fmaf(gp, v, gq), av));
    }
    // dL/dP_t = gy / D_t + e^w dL/dP_{t+1} with 1/D_t = iden 2^{-no};
    // H_t = e^w (dL/dP_{t+1} + H_{t+1})
    const float ng = fmaxf(w2 + G, -no);
    const float aa = ex2(w2 + G - ng);
    const float bb = ex2(-no - ng) * gy * iden;
    hp = aa * (gp + hp);
    hq = aa * (gq + hq);
    gp = fmaf(aa, gp, bb);
    gq = fmaf(aa, gq, -bb * y);
    G = ng;
  }
  // back to an integer scale (see fast_ok1)
  const float Gi = ceilf(G);
  const float f = ex2(G - Gi);
  adj[0] = Gi;
  adj[1] = gp * f;
  adj[2] = gq * f;
  adj[3] = hp * f;
  adj[4] = hq * f;
}

// ------------------------------------------------------------- forward tile
//
// Advances st over the `rows` steps of one staged tile (k/v pairs at
// ks[i*RS], vs[i*RS]); with kY writes y pairs to ys[i*RS]; with
// ck != nullptr stores the state at every sub-chunk start (rows 0, kSub, ...)
// to checkpoint rows ck_row0, ck_row0 + 1, ... The range check and the scale
// choice are made once per tile. The fast path is computed unconditionally (it
// cannot fault on any input); if any lane of the warp fails the range check the
// exact path recomputes the tile and its results (and checkpoints) replace the
// fast ones.
template <typename T, bool kTail, bool kY, int RS = kLanes>
__device__ __forceinline__ void fwd_tile2(Fwd2& st, const T* ks, const T* vs, T* ys, int rows,
                                          const Lane2& lc, bool force_slow, float* ck,
                                          size_t ck_row0, int C, int c, bool v0, bool v1) {
  using P = Pair<T>;
  using Sc = Scan<T>;
  using raw = typename P::raw;
  constexpr int R = P::kTileRows;
  raw kr[R], vr[R];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    kr[i] = P::ld(ks + i * RS);
    vr[i] = P::ld(vs + i * RS);
  }
  raw mx[R / 2], mn[R / 2];
#pragma unroll
  for (int i = 0; i < R / 2; ++i) {
    const bool i0 = !kTail || i < rows, i1 = !kTail || i + R / 2 < rows;
    mx[i] = Sc::vmax(i0 ? kr[i] : scan_lo<T>(), i1 ? kr[i + R / 2] : scan_lo<T>());
    mn[i] = Sc::vmin(i0 ? kr[i] : scan_hi<T>(), i1 ? kr[i + R / 2] : scan_hi<T>());
  }
#pragma unroll
  for (int w = R / 4; w > 0; w /= 2) {
#pragma unroll
    for (int i = 0; i < w; ++i) {
      mx[i] = Sc::vmax(mx[i], mx[i + w]);
      mn[i] = Sc::vmin(mn[i], mn[i + w]);
    }
  }
  const f2 kmax = P::unpack(mx[0]), kmin = P::unpack(mn[0]);
  const int n = kTail ? rows : R;
  f2 s, p, q;
  const bool ok =
      fast_ok1(st.S.x, st.p.x, st.q.x, kmax.x, kmin.x, n, lc.w2.x, lc.u2.x, s.x, p.x, q.x) &&
      fast_ok1(st.S.y, st.p.y, st.q.y, kmax.y, kmin.y, n, lc.w2.y, lc.u2.y, s.y, p.y, q.y) &&
      !force_slow;
  const f2 ns = f2{-s.x, -s.y};
  const f2 l2e = splat(kL2E);
  f2 yr[R];
#pragma unroll
  for (int i = 0; i < R; ++i) {
    if (kTail && i >= rows) break;
    if (ck != nullptr && i % kSub == 0) store_state(ck, ck_row0 + i / kSub, C, c, v0, v1, s, p, q);
    const f2 v = P::unpack(vr[i]);
    const f2 ek = ex2x2(fma2(P::unpack(kr[i]), l2e, ns));
    if (kY) {
      const f2 eb = mul2(ek, lc.eu);
      yr[i] = mul2(fma2(eb, v, p), rcpx2(add2(q, eb)));
    }
    p = fma2(lc.ew, p, mul2(ek, v));
    q = fma2(lc.ew, q, ek);
  }
  if (__all_sync(kFull, ok)) {
    st = Fwd2{s, p, q};
    if (kY) {
#pragma unroll
      for (int i = 0; i < R; ++i)
        if (!kTail || i < rows) P::st(ys + i * RS, P::pack(yr[i]));
    }
  } else {
#pragma unroll 1
    for (int r0 = 0; r0 < rows; r0 += kSub) {
      if (ck != nullptr) store_state(ck, ck_row0 + r0 / kSub, C, c, v0, v1, st.S, st.p, st.q);
      const int L = min(kSub, rows - r0);
      const int o = r0 * RS;
      fwd_slow1<T, kY>(st.S.x, st.p.x, st.q.x, ks + o, vs + o, ys + o, L, lc.w2.x, lc.u2.x, RS, RS);
      fwd_slow1<T, kY>(st.S.y, st.p.y, st.q.y, ks + o + 1, vs + o + 1, ys + o + 1, L, lc.w2.y,
                       lc.u2.y, RS, RS);
    }
  }
}

// ----------------------------------------------------- backward sub-chunk
//
// Given the forward state st0 at the sub-chunk start and the adjoint at its end,
// produces grad_key / grad_value pairs for its L steps (kOut), accumulates
// gwacc += dL/dw = sum_s e^{k_s} (v_s H^P_{s+1} + H^Q_{s+1}) and gu += dL/du,
// and leaves the adjoint at the sub-chunk start in adj.
// Fast path, with every adjoint quantity scaled by 2^s (the sub-chunk scale):
//   A  = gy e^{u+k}/D            gv = A + e^k dL/dP_{t+1}
//   gk = A (v - y) + e^k (dL/dP_{t+1} v + dL/dQ_{t+1})
//   dL/dP_t = gy/D_t + e^w dL/dP_{t+1},  dL/dQ_t = -gy y/D_t + e^w dL/dQ_{t+1}
//   H_t = e^w (dL/dP_{t+1} + H_{t+1})    (likewise for Q)
template <typename T, bool kTail, bool kOut, int RS = kLanes>
__device__ __forceinline__ void bwd_sub2(const Fwd2& st0, const Pre& pre, Adj2& adj, const T* ks,
                                         const T* vs, const T* gys, T* gks, T* gvs, int L,
                                         const Lane2& lc, f2& gwacc, f2& gu, bool force_slow) {
  using P = Pair<T>;
  const int n = kTail ? L : kSub;
  f2 s, p, q;
  bool ok =
      fast_ok1(st0.S.x, st0.p.x, st0.q.x, pre.kmax.x, pre.kmin.x, n, lc.w2.x, lc.u2.x, s.x, p.x, q.x) &&
      fast_ok1(st0.S.y, st0.p.y, st0.q.y, pre.kmax.y, pre.kmin.y, n, lc.w2.y, lc.u2.y, s.y, p.y, q.y) &&
      !force_slow;
  // Adjoint rescaled to the sub-chunk scale 2^{-s}.
  const f2 f = ex2x2(add2(adj.G, s));
  f2 gp = mul2(adj.gp, f), gq = mul2(adj.gq, f), hp = mul2(adj.hp, f), hq = mul2(adj.hq, f);
  const float amax = fmaxf(fmaxf(fmaxf(fabsf(gp.x), fabsf(gp.y)), fmaxf(fabsf(gq.x), fabsf(gq.y))),
                           fmaxf(fmaxf(fabsf(hp.x), fabsf(hp.y)), fmaxf(fabsf(hq.x), fabsf(hq.y))));
  ok = ok && fmaxf(pre.gymax.x, pre.gymax.y) <= 0x1p40f && amax <= 0x1p80f;
  const f2 ns = f2{-s.x, -s.y};
  const f2 l2e = splat(kL2E);
  const f2 gw0 = gwacc, gu0 = gu;
  f2 ry[kSub], rg[kSub], re[kSub];
  // forward recompute of the sub-chunk (k, v, gy read from shared memory once
  // here and v once more in the reverse sweep; e^{k-s} kept in registers)
#pragma unroll
  for (int i = 0; i < kSub; ++i) {
    if (kTail && i >= L) break;
    const f2 v = P::unpack(P::ld(vs + i * RS));
    const f2 ek = ex2x2(fma2(P::unpack(P::ld(ks + i * RS)), l2e, ns));
    re[i] = ek;
    const f2 eb = mul2(ek, lc.eu);
    const f2 rd = rcpx2(add2(q, eb));
    ry[i] = mul2(fma2(eb, v, p), rd);
    rg[i] = mul2(P::unpack(P::ld(gys + i * RS)), rd);  // gy 2^s / D_t
    p = fma2(lc.ew, p, mul2(ek, v));
    q = fma2(lc.ew, q, ek);
  }
  // reverse sweep
#pragma unroll
  for (int i = kSub - 1; i >= 0; --i) {
    if (kTail && i >= L) continue;
    const f2 v = P::unpack(P::ld(vs + i * RS));
    const f2 ek = re[i];
    const f2 a = mul2(mul2(rg[i], ek), lc.eu);  // gy e^{u+k} / D
    const f2 av = mul2(a, sub2(v, ry[i]));
    gu = add2(gu, av);
    gwacc = fma2(ek, fma2(v, hp, hq), gwacc);
    if (kOut) {
      P::st(gvs + i * RS, P::pack(fma2(ek, gp, a)));
      P::st(gks + i * RS, P::pack(fma2(ek, fma2(gp, v, gq), av)));
    }
    hp = mul2(lc.ew, add2(gp, hp));
    hq = mul2(lc.ew, add2(gq, hq));
    gq = sub2(mul2(lc.ew, gq), mul2(rg[i], ry[i]));
    gp = fma2(lc.ew, gp, rg[i]);
  }
  if (__all_sync(kFull, ok)) {
    adj = Adj2{ns, gp, gq, hp, hq};
  } else {
    gwacc = gw0;
    gu = gu0;
    float ax[5] = {adj.G.x, adj.gp.x, adj.gq.x, adj.hp.x, adj.hq.x};
    float ay[5] = {adj.G.y, adj.gp.y, adj.gq.y, adj.hp.y, adj.hq.y};
    bwd_slow1<T, kOut>(st0.S.x, st0.p.x, st0.q.x, ax, ks, vs, gys, gks, gvs, L, lc.w2.x, lc.u2.x,
                       gwacc.x, gu.x, RS, RS);
    bwd_slow1<T, kOut>(st0.S.y, st0.p.y, st0.q.y, ay, ks + 1, vs + 1, gys + 1, gks + 1, gvs + 1, L,
                       lc.w2.y, lc.u2.y, gwacc.y, gu.y, RS, RS);
    adj = Adj2{f2{ax[0], ay[0]}, f2{ax[1], ay[1]}, f2{ax[2], ay[2]}, f2{ax[3], ay[3]},
               f2{ax[4], ay[4]}};
  }
}

}  // namespace wkv
