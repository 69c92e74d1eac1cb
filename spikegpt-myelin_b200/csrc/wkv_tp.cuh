// Time-parallel WKV kernels for sm_100a (TMA path).
//
// The single-warp kernels of wkv_kernels.cuh give each SM only as many
// independent recurrence chains as there are (batch row, 64-channel block)
// lanes, 3-4 warps per SM at B*C = 32768, which leaves every warp's serial
// chain exposed. Here a CTA of W warps works on W consecutive kSub-step tiles of
// the same 64 channels at once, in rounds of W tiles:
//
//   A. each warp summarises its tile from a zero state, at the tile's own scale
//      (the state a zero state reaches after the tile: the update is linear in
//      the history, so summaries compose with fwd_combine2);
//   B. after one CTA barrier every warp folds the round's summaries, in time
//      order, into the state at the round start: the prefix up to its own tile
//      is its carry-in, the full fold is the next round's start state (every
//      warp computes the same fold, in the same order);
//   C. each warp produces its tile's outputs from its carry-in.
//
// HBM traffic is unchanged (one TMA box per tensor per round, read once); the
// extra work is the summary pass (one ex2 and three FMAs per element; the
// e^{k-s} values are kept in registers for phase C) and W combines per round.
#pragma once

#include "wkv_kernels.cuh"

namespace wkv {

// Warps per CTA: 4 for 16-bit I/O (4 CTAs of 54 KB shared memory fit an SM, so
// B*C = 32768 runs in one wave), 2 for float32 (twice the bytes per box).
template <typename T>
constexpr int tp_warps() {
  return sizeof(T) == 4 ? 2 : 4;
}

template <typename T, int W>
struct Tp {
  static constexpr int kRoundRows = W * kSub;  // steps per round = rows of one TMA box
  static constexpr int kBoxElems = kRoundRows * kLanes;
  static constexpr uint32_t kBoxBytes = kBoxElems * sizeof(T);
  static constexpr int kFwdStages = 3;
  static constexpr int kSumFloats = 2 * W * 3 * kLanes;  // [2 rounds][W tiles][S,p,q][lanes]
  static_assert(kSegAlign % kSub == 0, "segments start on tile boundaries");
};

template <typename T, int W>
constexpr size_t fwd_tp_smem_bytes() {
  using G = Tp<T, W>;
  return (size_t)2 * G::kFwdStages * G::kBoxBytes + G::kSumFloats * sizeof(float) +
         8 * G::kFwdStages;
}

// Packed max/min of k over rows [0, n) of a register tile (all kSub rows
// unless kTail).
template <typename T, bool kTail>
__device__ __forceinline__ void tile_kminmax(const typename Pair<T>::raw (&kr)[kSub], int n, f2& kmax,
                                             f2& kmin) {
  using Sc = Scan<T>;
  using raw = typename Pair<T>::raw;
  raw mx[kSub / 2], mn[kSub / 2];
#pragma unroll
  for (int i = 0; i < kSub / 2; ++i) {
    const bool i0 = !kTail || i < n, i1 = !kTail || i + kSub / 2 < n;
    mx[i] = Sc::vmax(i0 ? kr[i] : scan_lo<T>(), i1 ? kr[i + kSub / 2] : scan_lo<T>());
    mn[i] = Sc::vmin(i0 ? kr[i] : scan_hi<T>(), i1 ? kr[i + kSub / 2] : scan_hi<T>());
  }
#pragma unroll
  for (int w = kSub / 4; w > 0; w /= 2) {
#pragma unroll
    for (int i = 0; i < w; ++i) {
      mx[i] = Sc::vmax(mx[i], mx[i + w]);
      mn[i] = Sc::vmin(mn[i], mn[i + w]);
    }
  }
  kmax = Pair<T>::unpack(mx[0]);
  kmin = Pair<T>::unpack(mn[0]);
}

// Phase A of the forward for one tile held in registers: its range and its
// summary from a zero state, (sj, lp, lq) with P = 2^sj lp, sj = ceil(max k log2 e);
// ek[i] = e^{k_i} 2^-sj is kept for phase C. Rows >= n (kTail) contribute
// nothing.
template <typename T, bool kTail>
__device__ __forceinline__ void fwd_tp_summary(const typename Pair<T>::raw (&kr)[kSub],
                                               const typename Pair<T>::raw (&vr)[kSub], int n,
                                               const Lane2& lc, f2& kmax, f2& kmin, f2& sj,
                                               f2 (&ek)[kSub], f2& lp, f2& lq) {
  using P = Pair<T>;
  tile_kminmax<T, kTail>(kr, n, kmax, kmin);
  const f2 l2e = splat(kL2E);
  sj = f2{ceilf(kmax.x * kL2E), ceilf(kmax.y * kL2E)};  // integer scale: see fast_ok1
  const f2 nsj = f2{-sj.x, -sj.y};
  lp = splat(0.f);
  lq = splat(0.f);
#pragma unroll
  for (int i = 0; i < kSub; ++i) {
    if (kTail && i >= n) {
      ek[i] = splat(0.f);
      continue;
    }
    ek[i] = ex2x2(fma2(P::unpack(kr[i]), l2e, nsj));
    lp = fma2(lc.ew, lp, mul2(ek[i], P::unpack(vr[i])));
    lq = fma2(lc.ew, lq, ek[i]);
  }
}

// Phase C of the forward: y for the n rows of the tile from the carry-in
// (sc, p, q), with e^{k_i - sc} = ek[i] * c2.
template <typename T, bool kTail>
__device__ __forceinline__ void fwd_tp_y(const typename Pair<T>::raw (&vr)[kSub],
                                         const f2 (&ek)[kSub], int n, const Lane2& lc, f2 c2, f2 p,
                                         f2 q, T* yrow, size_t ystride, bool v0, bool v1) {
  using P = Pair<T>;
#pragma unroll
  for (int i = 0; i < kSub; ++i) {
    if (kTail && i >= n) break;
    const f2 v = P::unpack(vr[i]);
    const f2 e = mul2(ek[i], c2);
    const f2 eb = mul2(e, lc.eu);
    const f2 y = mul2(fma2(eb, v, p), rcpx2(add2(q, eb)));
    if (v1)
      P::st(yrow + i * ystride, P::pack(y));
    else if (v0)
      yrow[i * ystride] = P::from_float(y.x);
    p = fma2(lc.ew, p, mul2(e, v));
    q = fma2(lc.ew, q, e);
  }
}

// A state (S, p, q) of the channels c, c+1 as one checkpoint row ([3][C]
// floats), with 8-byte stores when both channels are valid and C is even.
__device__ __forceinline__ void store_state2(float* base, size_t row, int C, int c, bool v0,
                                             bool v1, const Fwd2& st) {
  if (v1 && (C & 1) == 0) {
    f2* r = reinterpret_cast<f2*>(base + row * 3 * (size_t)C + c);
    const size_t pl = (size_t)C / 2;
    r[0] = st.S;
    r[pl] = st.p;
    r[2 * pl] = st.q;
  } else {
    store_state(base, row, C, c, v0, v1, st.S, st.p, st.q);
  }
}

// Forward. kY: write y (and checkpoints when a.ckpt != null); !kY: the state
// sweep (checkpoints and/or segment-end states only). Grid (B * ncblk, nseg),
// W warps per CTA; reference wkv_triton.py:34-58.
template <typename T, int W, bool kY>
__global__ void __launch_bounds__(32 * W, 4)
    wkv_fwd_tp_kernel(const FwdArgs a, const __grid_constant__ CUtensorMap tk,
                      const __grid_constant__ CUtensorMap tv) {
  using G = Tp<T, W>;
  using P = Pair<T>;
  using raw = typename P::raw;
  constexpr int NS = G::kFwdStages;
  constexpr int R = kSub;
  extern __shared__ __align__(128) unsigned char smem[];
  T* kbuf = reinterpret_cast<T*>(smem);
  T* vbuf = kbuf + NS * G::kBoxElems;
  float* sum = reinterpret_cast<float*>(vbuf + NS * G::kBoxElems);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sum + G::kSumFloats);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cb = blockIdx.x % a.ncblk, b = blockIdx.x / a.ncblk;
  const int c = cb * kLanes + 2 * lane;
  const int seg = blockIdx.y + a.seg_base;
  const bool v0 = c < a.C, v1 = c + 1 < a.C;
  f2 dec = splat(0.f), uu = splat(0.f);
  if (v0) {
    dec.x = a.decay[c];
    uu.x = a.u[c];
  }
  if (v1) {
    dec.y = a.decay[c + 1];
    uu.y = a.u[c + 1];
  }
  if (!a.decay_is_w) dec = f2{-expf(dec.x), -expf(dec.y)};
  const Lane2 lc = make_lane2(dec, uu);
  const int t_begin = seg * a.seg_len;
  const int t_end = min(a.T, t_begin + a.seg_len);
  const int nrounds = (t_end - t_begin + G::kRoundRows - 1) / G::kRoundRows;
  const bool force_slow = a.force_slow != 0;

  if (a.zero_tickets != nullptr && blockIdx.x == 0 && blockIdx.y == 0)
    for (int i = threadIdx.x; i < a.nzero; i += blockDim.x) a.zero_tickets[i] = 0u;

  Fwd2 st = fwd_identity2();
  if (a.seg_start != nullptr)
    load3(a.seg_start, (size_t)b * a.nseg + seg, a.C, c, v0, v1, st.S, st.p, st.q);

  auto issue = [&](int r) {
    const int s = r % NS;
    mbar_arrive_expect_tx(&bars[s], 2 * G::kBoxBytes);
    const int t0 = t_begin + r * G::kRoundRows;
    tma_load_3d(kbuf + s * G::kBoxElems, &tk, &bars[s], cb * kLanes, t0, b);
    tma_load_3d(vbuf + s * G::kBoxElems, &tv, &bars[s], cb * kLanes, t0, b);
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
    prefetch_tensormap(&tk);
    prefetch_tensormap(&tv);
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int r = 0; r < min(NS, nrounds); ++r) issue(r);

#pragma unroll 1
  for (int r = 0; r < nrounds; ++r) {
    const int s = r % NS;
    const int t0 = t_begin + r * G::kRoundRows + warp * R;  // this warp's tile
    const int n = max(0, min(R, t_end - t0));
    const bool arrived = mbar_wait_bounded(&bars[s], (r / NS) & 1);

    // A. summary of the tile from a zero state, scaled by 2^-sj, sj = ceil(max k log2 e)
    raw kr[R], vr[R];
    const T* kt = kbuf + s * G::kBoxElems + warp * R * kLanes + 2 * lane;
    const T* vt = vbuf + s * G::kBoxElems + warp * R * kLanes + 2 * lane;
#pragma unroll
    for (int i = 0; i < R; ++i) {
      kr[i] = P::ld(kt + i * kLanes);
      vr[i] = P::ld(vt + i * kLanes);
    }
    f2 kmax, kmin, sj, lp, lq;
    f2 ek[R];
    if (n == R) {
      fwd_tp_summary<T, false>(kr, vr, n, lc, kmax, kmin, sj, ek, lp, lq);
    } else {
      fwd_tp_summary<T, true>(kr, vr, n, lc, kmax, kmin, sj, ek, lp, lq);
      if (n == 0) sj = splat(kNegBig);
    }
    {
      f2* sw = reinterpret_cast<f2*>(sum + ((r & 1) * W + warp) * 3 * kLanes) + lane;
      sw[0] = sj;
      sw[kLanes / 2] = lp;
      sw[kLanes] = lq;
    }
    // Every warp has its tile in registers and its summary in shared memory.
    if (!__syncthreads_and(arrived)) {
      if (threadIdx.x == 0) {
        report_timeout(a.err);
        for (int q = r; q < min(r + NS, nrounds); ++q) mbar_wait_bounded(&bars[q % NS], (q / NS) & 1);
      }
      return;
    }
    if (threadIdx.x == 0 && r + NS < nrounds) issue(r + NS);

    // B. carry-in of this warp's tile; st becomes the state after the round
    Fwd2 sin = st;
#pragma unroll
    for (int m = 0; m < W; ++m) {
      const f2* sm = reinterpret_cast<const f2*>(sum + ((r & 1) * W + m) * 3 * kLanes) + lane;
      const Fwd2 l{sm[0], sm[kLanes / 2], sm[kLanes]};
      const int nm = max(0, min(R, t_end - (t_begin + r * G::kRoundRows + m * R)));
      if (m == warp) sin = st;
      st = fwd_combine2(st, nm, lc, l);
    }

    // C. outputs of the tile from its carry-in
    if (n > 0) {
      if (a.ckpt != nullptr) store_state2(a.ckpt, (size_t)b * a.nsub + t0 / kSub, a.C, c, v0, v1, sin);
      if (kY) {
        f2 sc, p, q;
        const bool ok = fast_ok1(sin.S.x, sin.p.x, sin.q.x, kmax.x, kmin.x, n, lc.w2.x, lc.u2.x,
                                 sc.x, p.x, q.x) &&
                        fast_ok1(sin.S.y, sin.p.y, sin.q.y, kmax.y, kmin.y, n, lc.w2.y, lc.u2.y,
                                 sc.y, p.y, q.y) &&
                        !force_slow;
        const f2 c2 = ex2x2(sub2(sj, sc));  // e^{k - sj} -> e^{k - sc}
        T* yrow = static_cast<T*>(a.y) + ((size_t)b * a.T + t0) * a.C + c;
        if (n == R)
          fwd_tp_y<T, false>(vr, ek, n, lc, c2, p, q, yrow, (size_t)a.C, v0, v1);
        else
          fwd_tp_y<T, true>(vr, ek, n, lc, c2, p, q, yrow, (size_t)a.C, v0, v1);
        if (!__all_sync(kFull, ok)) {
          // exact per-step rescaling from the carry-in, reading k, v from memory
          const size_t base = ((size_t)b * a.T + t0) * a.C + c;
          const T* kg = static_cast<const T*>(a.k) + base;
          const T* vg = static_cast<const T*>(a.v) + base;
          if (v0) {
            float S0 = sin.S.x, p0 = sin.p.x, q0 = sin.q.x;
            fwd_slow1<T, true>(S0, p0, q0, kg, vg, yrow, n, lc.w2.x, lc.u2.x, a.C);
          }
          if (v1) {
            float S1 = sin.S.y, p1 = sin.p.y, q1 = sin.q.y;
            fwd_slow1<T, true>(S1, p1, q1, kg + 1, vg + 1, yrow + 1, n, lc.w2.y, lc.u2.y, a.C);
          }
        }
      }
    }
  }
  if (a.seg_end != nullptr && warp == 0)
    store3(a.seg_end, (size_t)b * a.nseg + seg, a.C, c, v0, v1, st.S, st.p, st.q);
}

}  // namespace wkv
