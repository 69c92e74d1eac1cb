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

// Warps per CTA: 4 for 16-bit I/O (4 CTAs of 47 KB shared memory fit an SM, so
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
  // Two stages: a stage is read only in phase A, so the box of round r+2 is
  // requested a whole round before it is needed.
  static constexpr int kFwdStages = 2;
  // [2 rounds][W tile summaries][S, p, q][lanes]
  static constexpr int kSumFloats = 2 * W * 3 * kLanes;
  static constexpr uint32_t kYTileBytes = kSub * kLanes * sizeof(T);  // one warp's staged y tile
  static_assert(kSegAlign % kSub == 0, "segments start on tile boundaries");
  static_assert(kBoxBytes % 128 == 0 && (kSumFloats * 4) % 128 == 0 && kYTileBytes % 128 == 0,
                "bulk-copy buffers start on 128-byte boundaries");
};

// Shared memory: k stages | v stages | summaries | y tiles | barriers.
template <typename T, int W>
constexpr size_t fwd_tp_smem_bytes() {
  using G = Tp<T, W>;
  return (size_t)2 * G::kFwdStages * G::kBoxBytes + G::kSumFloats * sizeof(float) +
         W * G::kYTileBytes + 8 * G::kFwdStages;
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
// (sc, p, q), with e^{k_i - sc} = ek[i] * c2 (kScale; else c2 = 1), into a
// staged tile. Per step: ekv = e v; y = (p + u' ekv) / (q + u' e) with u' = e^u,
// both as one fused multiply-add; then p, q decay and take the step's terms.
template <typename T, bool kTail, bool kScale>
__device__ __forceinline__ void fwd_tp_y(const typename Pair<T>::raw (&vr)[kSub],
                                         const f2 (&ek)[kSub], int n, const Lane2& lc, f2 c2, f2 p,
                                         f2 q, T* ys) {
  using P = Pair<T>;
#pragma unroll
  for (int i = 0; i < kSub; ++i) {
    if (kTail && i >= n) break;
    const f2 v = P::unpack(vr[i]);
    const f2 e = kScale ? mul2(ek[i], c2) : ek[i];
    const f2 ekv = mul2(e, v);
    const f2 y = mul2(fma2(lc.eu, ekv, p), rcpx2(fma2(e, lc.eu, q)));
    P::st(ys + i * kLanes, P::pack(y));  // staged [kSub][kLanes] tile
    p = fma2(lc.ew, p, ekv);
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

// Exact (per-step rescaling) y of a tile from its carry-in, reading k, v from
// global memory and writing the staged y tile. Rare: only when the fast path's
// range checks fail.
template <typename T>
__device__ __noinline__ void fwd_tp_exact(const FwdArgs& a, int b, int t0, int c, bool v0, bool v1,
                                          int n, Fwd2 sin, Lane2 lc, T* ys) {
  const size_t base = ((size_t)b * a.T + t0) * a.C + c;
  const T* kg = static_cast<const T*>(a.k) + base;
  const T* vg = static_cast<const T*>(a.v) + base;
  if (v0) fwd_slow1<T, true>(sin.S.x, sin.p.x, sin.q.x, kg, vg, ys, n, lc.w2.x, lc.u2.x, a.C, kLanes);
  if (v1)
    fwd_slow1<T, true>(sin.S.y, sin.p.y, sin.q.y, kg + 1, vg + 1, ys + 1, n, lc.w2.y, lc.u2.y, a.C,
                       kLanes);
}

// Forward. kY: write y (and checkpoints when a.ckpt != null); !kY: the state
// sweep (checkpoints and/or segment-end states only). Grid (B * ncblk, nseg),
// W warps per CTA; reference wkv_triton.py:34-58.
template <typename T, int W, bool kY>
__global__ void __launch_bounds__(32 * W, 4)
    wkv_fwd_tp_kernel(const FwdArgs a, const __grid_constant__ CUtensorMap tk,
                      const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap ty) {
  using G = Tp<T, W>;
  using P = Pair<T>;
  using raw = typename P::raw;
  constexpr int NS = G::kFwdStages;
  constexpr int R = kSub;
  extern __shared__ __align__(128) unsigned char smem[];
  T* kbuf = reinterpret_cast<T*>(smem);
  T* vbuf = kbuf + NS * G::kBoxElems;
  float* sum = reinterpret_cast<float*>(vbuf + NS * G::kBoxElems);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  T* ys = reinterpret_cast<T*>(sum + G::kSumFloats) + warp * kSub * kLanes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<unsigned char*>(sum + G::kSumFloats) +
                                               W * G::kYTileBytes);

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

  Fwd2 start = fwd_identity2();  // state at the segment start
  if (a.seg_start != nullptr)
    load3(a.seg_start, (size_t)b * a.nseg + seg, a.C, c, v0, v1, start.S, start.p, start.q);
  else if (a.seg_sums != nullptr && seg > 0)
    start = fold_state_summaries(a.seg_sums, b, a.nseg, seg, a.seg_len, a.C, c, v0, v1, lc);

  // (a.withhold_first: debug only, the first round's copies are never issued)
  auto withheld = [&](int r) { return a.withhold_first != 0 && r == 0; };
  auto issue = [&](bool on, int r) {  // by the threads with `on` (one per CTA)
    const int s = r % NS;
    on = on && !withheld(r);
    mbar_arrive_expect_tx_if(on, &bars[s], 2 * G::kBoxBytes);
    const int t0 = t_begin + r * G::kRoundRows;
    tma_load_3d_if(on, kbuf + s * G::kBoxElems, &tk, &bars[s], cb * kLanes, t0, b);
    tma_load_3d_if(on, vbuf + s * G::kBoxElems, &tv, &bars[s], cb * kLanes, t0, b);
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
    prefetch_tensormap(&tk);
    prefetch_tensormap(&tv);
    if (kY) prefetch_tensormap(&ty);
  }
  __syncthreads();
  for (int r = 0; r < min(NS, nrounds); ++r) issue(threadIdx.x == 0, r);

  Fwd2 cur = start;  // the state at the start of the current round (every warp)
#pragma unroll 1
  for (int r = 0; r < nrounds; ++r) {
    const int s = r % NS;
    const int rt0 = t_begin + r * G::kRoundRows;
    const int t0 = rt0 + warp * R;  // this warp's tile
    const int n = max(0, min(R, t_end - t0));
    float* sr = sum + (r & 1) * W * 3 * kLanes;  // this round's summaries
    const bool arrived = mbar_wait_bounded(&bars[s], (r / NS) & 1, a.wait_limit);

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
      f2* sw = reinterpret_cast<f2*>(sr + warp * 3 * kLanes) + lane;
      sw[0] = sj;
      sw[kLanes / 2] = lp;
      sw[kLanes] = lq;
    }
    // Every warp has its tile in registers and its summary in shared memory.
    if (!__syncthreads_and(arrived)) {
      if (threadIdx.x == 0) {
        report_timeout(a.err);
        // every copy this CTA issued lands before it exits
        for (int q = r; q < min(r + NS, nrounds); ++q)
          if (!withheld(q)) mbar_wait_bounded(&bars[q % NS], (q / NS) & 1);
      }
      if (kY) bulk_wait_all();
      return;
    }
    if (r + NS < nrounds) issue(threadIdx.x == 0, r + NS);

    // B. carry-in of this warp's tile: the round's start state folded with the
    // summaries of the earlier tiles of the round. Every warp folds all W
    // summaries (so every warp holds the next round's start state), and a
    // round of full tiles takes the branch-free 16-step combine: the fold's
    // latency is then one short chain, not W dependent combines.
    Fwd2 sin = cur;
    {
      Fwd2 sm[W];
#pragma unroll
      for (int m = 0; m < W; ++m) {
        const f2* q = reinterpret_cast<const f2*>(sr + m * 3 * kLanes) + lane;
        sm[m] = Fwd2{q[0], q[kLanes / 2], q[kLanes]};
      }
      if (rt0 + W * R <= t_end) {
#pragma unroll
        for (int m = 0; m < W; ++m) {
          cur = fwd_combine16(cur, lc, sm[m]);
          if (m + 1 == warp) sin = cur;
        }
      } else {
#pragma unroll
        for (int m = 0; m < W; ++m) {
          const int nm = min(R, max(0, t_end - (rt0 + m * R)));
          if (nm > 0) cur = fwd_combine2(cur, nm, lc, sm[m]);
          if (m + 1 == warp) sin = cur;
        }
      }
    }

    // C. outputs of the tile from its carry-in
    if (n > 0) {
      if (a.ckpt != nullptr) store_state2(a.ckpt, (size_t)b * a.nsub + t0 / kSub, a.C, c, v0, v1, sin);
      if (kY) {
        bulk_wait_read<0>();  // the previous tile's store (lane 0's group) has read ys
        __syncwarp();
        f2 sc, p, q;
        const bool ok = fast_ok1(sin.S.x, sin.p.x, sin.q.x, kmax.x, kmin.x, n, lc.w2.x, lc.u2.x,
                                 sc.x, p.x, q.x) &&
                        fast_ok1(sin.S.y, sin.p.y, sin.q.y, kmax.y, kmin.y, n, lc.w2.y, lc.u2.y,
                                 sc.y, p.y, q.y) &&
                        !force_slow;
        if (__all_sync(kFull, ok)) {
          // e^{k - sj} -> e^{k - sc}: an exact power of two, 1 unless the
          // carried state's scale exceeds the tile's own
          if (__all_sync(kFull, sc.x == sj.x && sc.y == sj.y)) {
            if (n == R)
              fwd_tp_y<T, false, false>(vr, ek, n, lc, splat(1.f), p, q, ys + 2 * lane);
            else
              fwd_tp_y<T, true, false>(vr, ek, n, lc, splat(1.f), p, q, ys + 2 * lane);
          } else {
            const f2 c2 = ex2x2(sub2(sj, sc));  // integer exponents: exact
            if (n == R)
              fwd_tp_y<T, false, true>(vr, ek, n, lc, c2, p, q, ys + 2 * lane);
            else
              fwd_tp_y<T, true, true>(vr, ek, n, lc, c2, p, q, ys + 2 * lane);
          }
        } else {
          fwd_tp_exact<T>(a, b, t0, c, v0, v1, n, sin, lc, ys + 2 * lane);
        }
        fence_proxy_async_smem();
        __syncwarp();
        tma_store_3d_if(lane == 0, &ty, ys, cb * kLanes, t0, b);
        bulk_commit();
      }
    }
  }
  if (kY) bulk_wait_all();
  if (a.seg_end != nullptr && warp == W - 1)
    store3(a.seg_end, (size_t)b * a.nseg + seg, a.C, c, v0, v1, cur.S, cur.p, cur.q);
}

// ----------------------------------------------------------------- backward
//
// Rounds go backwards in time; warp w of a round takes the w-th of its W tiles
// (in time order), so warp W-1 holds the latest tile.
//   A. from the tile's checkpoint (its forward state, saved by the forward or the
//      state sweep) recompute y_t and gy_t/D_t over the tile, then run the
//      adjoint recurrence backwards over the tile from a zero adjoint: the
//      tile's local adjoint summary (the adjoint recurrence is linear in the
//      adjoint, so summaries compose with adj_combine1);
//   B. fold the summaries, latest tile first, into the adjoint entering the
//      round: the fold down to a warp's tile end is its incoming adjoint, the
//      full fold enters the next round;
//   C. rerun the reverse recurrence from the incoming adjoint, writing
//      grad_key / grad_value and accumulating dL/dw, dL/du.

// Warps per backward CTA: a tile's records (e^{k-s}, gy/D, -gy y/D) stay in
// registers across the round barrier (~237 registers a thread), so an SM runs
// 4 CTAs of 2 warps and B*C = 32768 fits one wave. A full tile's k and grad_y
// rows are loaded into registers once, for the range scan and the recompute;
// v is read from the staged box where it is used (recompute and outputs).
template <typename T>
constexpr int tp_bwd_warps() {
  return 2;
}

template <typename T, int W>
struct TpB {
  static constexpr int kRoundRows = W * kSub;
  static constexpr int kBoxElems = kRoundRows * kLanes;
  static constexpr uint32_t kBoxBytes = kBoxElems * sizeof(T);
  static constexpr uint32_t kCkBytes = W * 3 * kLanes * sizeof(float);  // W checkpoint rows
  static constexpr uint32_t kStageBytes = 3 * kBoxBytes + kCkBytes;     // k, v, gy, ckpt
  // A stage's round r + NS - 1 copy is issued once every warp has passed round
  // r's barrier (the stage was last read, and its staged outputs stored, in
  // round r - 1). Three stages for 16-bit I/O (47 KB a CTA), two for float32.
  static constexpr int kStages = sizeof(T) == 4 ? 2 : 3;
  static constexpr int kSumFloats = 2 * W * 5 * kLanes;  // [2 rounds][W][G,gp,gq,hp,hq][lanes]
  static_assert(kStages >= 2, "a stage is refilled one round after it was read");
  static_assert(kBoxBytes % 128 == 0 && kCkBytes % 128 == 0 && kStageBytes % 128 == 0 &&
                    (kSumFloats * 4) % 128 == 0 && (W * 2 * kLanes * 4) % 128 == 0 &&
                    (kSub * kLanes * sizeof(T)) % 128 == 0,
                "bulk-copy buffers start on 128-byte boundaries");
};

// Shared memory: stages | summaries | per-warp partial sums | barriers. A
// warp's grad_key / grad_value tiles are staged over its own rows of the
// round's k and grad_y boxes, which phase A was the last to read.
template <typename T, int W>
constexpr size_t bwd_tp_smem_bytes() {
  using G = TpB<T, W>;
  return (size_t)G::kStages * G::kStageBytes + G::kSumFloats * sizeof(float) +
         W * 2 * kLanes * sizeof(float) + 8 * G::kStages;
}

// Forward recompute of a tile from its start state rescaled to the tile scale
// s, keeping for the reverse pass re = e^{k_t - s}, rg = gy_t 2^s / D_t and
// rn = -rg_t y_t (the two adjoint increments of step t: dL/dP_t and dL/dQ_t
// take rg_t and rn_t, and the output formulas need y_t only through rn_t).
template <typename T, bool kTail>
__device__ __forceinline__ void bwd_tp_recompute(const T* ks, const T* vs, const T* gys, int n,
                                                 const Lane2& lc, f2 s, f2 p, f2 q,
                                                 f2 (&re)[kSub], f2 (&rg)[kSub], f2 (&rn)[kSub]) {
  using P = Pair<T>;
  const f2 l2e = splat(kL2E), ns = f2{-s.x, -s.y};
#pragma unroll
  for (int i = 0; i < kSub; ++i) {
    if (kTail && i >= n) {
      re[i] = splat(0.f);
      rg[i] = splat(0.f);
      rn[i] = splat(0.f);
      continue;
    }
    const f2 v = P::unpack(P::ld(vs + i * kLanes));
    const f2 ek = ex2x2(fma2(P::unpack(P::ld(ks + i * kLanes)), l2e, ns));
    re[i] = ek;
    const f2 ekv = mul2(ek, v);
    const f2 rd = rcpx2(fma2(ek, lc.eu, q));  // 1 / D
    const f2 y = mul2(fma2(lc.eu, ekv, p), rd);
    const f2 g = mul2(P::unpack(P::ld(gys + i * kLanes)), rd);
    rg[i] = g;
    rn[i] = f2{-(g.x * y.x), -(g.y * y.y)};
    p = fma2(lc.ew, p, ekv);
    q = fma2(lc.ew, q, ek);
  }
}

// bwd_tp_recompute for a full tile whose k and grad_y rows are already in
// registers (loaded once for the range scan), v read from the staged box.
template <typename T>
__device__ __forceinline__ void bwd_tp_recompute_regs(const typename Pair<T>::raw (&kr)[kSub],
                                                      const typename Pair<T>::raw (&gr)[kSub], const T* vs,
                                                      const Lane2& lc, f2 s, f2 p, f2 q, f2 (&re)[kSub],
                                                      f2 (&rg)[kSub], f2 (&rn)[kSub]) {
  using P = Pair<T>;
  const f2 l2e = splat(kL2E), ns = f2{-s.x, -s.y};
#pragma unroll
  for (int i = 0; i < kSub; ++i) {
    const f2 v = P::unpack(P::ld(vs + i * kLanes));
    const f2 ek = ex2x2(fma2(P::unpack(kr[i]), l2e, ns));
    re[i] = ek;
    const f2 ekv = mul2(ek, v);
    const f2 rd = rcpx2(fma2(ek, lc.eu, q));  // 1 / D
    const f2 y = mul2(fma2(lc.eu, ekv, p), rd);
    const f2 g = mul2(P::unpack(gr[i]), rd);
    rg[i] = g;
    rn[i] = f2{-(g.x * y.x), -(g.y * y.y)};
    p = fma2(lc.ew, p, ekv);
    q = fma2(lc.ew, q, ek);
  }
}

// Packed max |grad_y| over the rows of a full register tile.
template <typename T>
__device__ __forceinline__ f2 tile_absmax(const typename Pair<T>::raw (&gr)[kSub]) {
  using Sc = Scan<T>;
  using raw = typename Pair<T>::raw;
  raw g[kSub / 2];
#pragma unroll
  for (int i = 0; i < kSub / 2; ++i) g[i] = Sc::vmax(Sc::vabs(gr[i]), Sc::vabs(gr[i + kSub / 2]));
#pragma unroll
  for (int w = kSub / 4; w > 0; w /= 2) {
#pragma unroll
    for (int i = 0; i < w; ++i) g[i] = Sc::vmax(g[i], g[i + w]);
  }
  return Pair<T>::unpack(g[0]);
}

// The tile's adjoint summary: the reverse recurrence over its rows from a zero
// adjoint at the tile end (scaled by 2^s, like rg). The w-derivatives are
// carried as K with H = e^w K (K_t = G_{t+1} + H_{t+1}, so K_t = G_{t+1} +
// e^w K_{t+1}: one multiply-add per step instead of an add and a multiply).
template <bool kTail>
__device__ __forceinline__ void bwd_tp_summary(const f2 (&rg)[kSub], const f2 (&rn)[kSub], int n,
                                               const Lane2& lc, f2& gp, f2& gq, f2& hp, f2& hq) {
  f2 kp = splat(0.f), kq = splat(0.f);
  gp = gq = splat(0.f);
#pragma unroll
  for (int i = kSub - 1; i >= 0; --i) {
    if (kTail && i >= n) continue;
    kp = fma2(lc.ew, kp, gp);
    kq = fma2(lc.ew, kq, gq);
    gq = fma2(lc.ew, gq, rn[i]);
    gp = fma2(lc.ew, gp, rg[i]);
  }
  hp = mul2(lc.ew, kp);
  hq = mul2(lc.ew, kq);
}

// Reverse pass of a tile from the adjoint at its end (scaled by 2^s): grad_key /
// grad_value of its rows (kOut) and dL/dw, dL/du accumulated into gw, gu.
// Per step, with X = dL/dP_{t+1} + e^u rg_t and Y = dL/dQ_{t+1} + e^u rn_t:
//   grad_value = e^k X,  grad_key = grad_value v + e^k Y,
//   dL/du += e^u e^k (rg v + rn),  dL/dw += e^k (v H^P_{t+1} + H^Q_{t+1}).
// Full tiles take the top row with the incoming H and the rest with K
// (H = e^w K, see bwd_tp_summary), the factors e^u and e^w applied once per
// tile; partial tiles carry H itself.
template <typename T, bool kTail, bool kOut>
__device__ __forceinline__ void bwd_tp_outputs(const f2 (&re)[kSub], const T* vs,
                                               const f2 (&rg)[kSub], const f2 (&rn)[kSub], int n,
                                               const Lane2& lc, f2 gp, f2 gq, f2 hp, f2 hq,
                                               T* gks, T* gvs, f2& gw, f2& gu) {
  using P = Pair<T>;
  f2 tu = splat(0.f);
  auto row = [&](int i, f2 v, f2 ek) {
    const f2 gv = mul2(ek, fma2(lc.eu, rg[i], gp));
    const f2 gk = fma2(gv, v, mul2(ek, fma2(lc.eu, rn[i], gq)));
    tu = fma2(ek, fma2(rg[i], v, rn[i]), tu);
    if (kOut) {  // staged [kSub][kLanes] tiles
      P::st(gvs + i * kLanes, P::pack(gv));
      P::st(gks + i * kLanes, P::pack(gk));
    }
  };
  if (kTail) {
#pragma unroll
    for (int i = kSub - 1; i >= 0; --i) {
      if (i >= n) continue;
      const f2 v = P::unpack(P::ld(vs + i * kLanes)), ek = re[i];
      row(i, v, ek);
      gw = fma2(ek, fma2(v, hp, hq), gw);
      hp = mul2(lc.ew, add2(gp, hp));
      hq = mul2(lc.ew, add2(gq, hq));
      gq = fma2(lc.ew, gq, rn[i]);
      gp = fma2(lc.ew, gp, rg[i]);
    }
  } else {
    constexpr int top = kSub - 1;
    f2 kp, kq, tw = splat(0.f);
    {
      const f2 v = P::unpack(P::ld(vs + top * kLanes)), ek = re[top];
      row(top, v, ek);
      gw = fma2(ek, fma2(v, hp, hq), gw);
      kp = add2(gp, hp);
      kq = add2(gq, hq);
      gq = fma2(lc.ew, gq, rn[top]);
      gp = fma2(lc.ew, gp, rg[top]);
    }
#pragma unroll
    for (int i = top - 1; i >= 0; --i) {
      const f2 v = P::unpack(P::ld(vs + i * kLanes)), ek = re[i];
      row(i, v, ek);
      tw = fma2(ek, fma2(v, kp, kq), tw);
      kp = fma2(lc.ew, kp, gp);
      kq = fma2(lc.ew, kq, gq);
      gq = fma2(lc.ew, gq, rn[i]);
      gp = fma2(lc.ew, gp, rg[i]);
    }
    gw = fma2(lc.ew, tw, gw);
  }
  gu = fma2(lc.eu, tu, gu);
}

// adj_combine1 for both lanes of the pair with packed arithmetic (the same
// roundings lane by lane).
__device__ __forceinline__ Adj2 adj_combine2(const Adj2& l, Adj2 e, int len, const Lane2& lc) {
  f2 dm, de;
  ew_decay2(lc, len, dm, de);
  const f2 fl = splat(static_cast<float>(len));
  const f2 ge = add2(e.G, de);
  const f2 g = f2{fmaxf(ge.x, l.G.x), fmaxf(ge.y, l.G.y)};
  const f2 a = mul2(dm, ex2x2(sub2(ge, g)));
  const f2 b = ex2x2(sub2(l.G, g));
  const f2 hp = fma2(fl, e.gp, e.hp), hq = fma2(fl, e.gq, e.hq);
  e.gp = fma2(e.gp, a, mul2(l.gp, b));
  e.gq = fma2(e.gq, a, mul2(l.gq, b));
  e.hp = fma2(hp, a, mul2(l.hp, b));
  e.hq = fma2(hq, a, mul2(l.hq, b));
  e.G = g;
  return e;
}

// adj_combine2 over exactly kSub steps: branch-free (see fwd_combine16).
__device__ __forceinline__ Adj2 adj_combine16(const Adj2& l, Adj2 e, const Lane2& lc) {
  const f2 fl = splat(static_cast<float>(kSub));
  const f2 ge = add2(e.G, lc.de16);
  const f2 g = f2{fmaxf(ge.x, l.G.x), fmaxf(ge.y, l.G.y)};
  const f2 a = mul2(lc.dm16, ex2x2(sub2(ge, g)));
  const f2 b = ex2x2(sub2(l.G, g));
  const f2 hp = fma2(fl, e.gp, e.hp), hq = fma2(fl, e.gq, e.hq);
  e.gp = fma2(e.gp, a, mul2(l.gp, b));
  e.gq = fma2(e.gq, a, mul2(l.gq, b));
  e.hp = fma2(hp, a, mul2(l.hp, b));
  e.hq = fma2(hq, a, mul2(l.hq, b));
  e.G = g;
  return e;
}

__device__ __forceinline__ Adj2 fold_adjoint_summaries(const float* sums, int b, int nseg, int seg,
                                                       int seg_len, int T, int C, int c, bool v0,
                                                       bool v1, const Lane2& lc) {
  Adj2 e = adj_zero2();
  const int last_len = T - (nseg - 1) * seg_len;
  constexpr int K = 4;
  for (int s0 = nseg - 1; s0 > seg; s0 -= K) {
    Adj2 l[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      l[k] = adj_zero2();
      if (s0 - k > seg) load_adj(sums, (size_t)b * nseg + s0 - k, C, c, v0, v1, l[k]);
    }
#pragma unroll
    for (int k = 0; k < K; ++k)
      if (s0 - k > seg) e = adj_combine2(l[k], e, s0 - k == nseg - 1 ? last_len : seg_len, lc);
  }
  return e;
}

// Exact (per-step rescaling) adjoint summary of a staged tile from a zero
// adjoint, both channels of the lane pair. Rare: only when the fast path's
// range checks fail.
template <typename T>
__device__ __noinline__ Adj2 bwd_tp_exact_summary(const T* ks, const T* vs, const T* gys, int n,
                                                  Fwd2 st0, Lane2 lc) {
  float lx[5] = {kNegBig, 0.f, 0.f, 0.f, 0.f}, ly[5] = {kNegBig, 0.f, 0.f, 0.f, 0.f};
  float d0 = 0.f, d1 = 0.f;
  bwd_slow1<T, false>(st0.S.x, st0.p.x, st0.q.x, lx, ks, vs, gys, nullptr, nullptr, n, lc.w2.x,
                      lc.u2.x, d0, d1);
  bwd_slow1<T, false>(st0.S.y, st0.p.y, st0.q.y, ly, ks + 1, vs + 1, gys + 1, nullptr, nullptr, n,
                      lc.w2.y, lc.u2.y, d0, d1);
  return Adj2{f2{lx[0], ly[0]}, f2{lx[1], ly[1]}, f2{lx[2], ly[2]}, f2{lx[3], ly[3]}, f2{lx[4], ly[4]}};
}

// Exact reverse pass of a tile from its incoming adjoint, reading k, v, gy from
// global memory and writing grad_key / grad_value into the staged tiles. Rare.
template <typename T>
__device__ __noinline__ void bwd_tp_exact(const BwdArgs& a, int b, int t0, int c, bool v0, bool v1,
                                          int n, Fwd2 st0, Adj2 ein, Lane2 lc, T* gks, T* gvs,
                                          f2& gw, f2& gu) {
  const size_t row = ((size_t)b * a.T + t0) * a.C + c;
  const T* kg = static_cast<const T*>(a.k) + row;
  const T* vg = static_cast<const T*>(a.v) + row;
  const T* gg = static_cast<const T*>(a.gy) + row;
  if (v0) {
    float ax[5] = {ein.G.x, ein.gp.x, ein.gq.x, ein.hp.x, ein.hq.x};
    bwd_slow1<T, true>(st0.S.x, st0.p.x, st0.q.x, ax, kg, vg, gg, gks, gvs, n, lc.w2.x, lc.u2.x,
                       gw.x, gu.x, a.C, kLanes);
  }
  if (v1) {
    float ay[5] = {ein.G.y, ein.gp.y, ein.gq.y, ein.hp.y, ein.hq.y};
    bwd_slow1<T, true>(st0.S.y, st0.p.y, st0.q.y, ay, kg + 1, vg + 1, gg + 1, gks + 1, gvs + 1, n,
                       lc.w2.y, lc.u2.y, gw.y, gu.y, a.C, kLanes);
  }
}

// Adjoints (G, gp, gq, hp, hq) of the kLanes channels as [5][kLanes] floats.
__device__ __forceinline__ Adj2 adj_ld(const float* slot, int lane) {
  const f2* q = reinterpret_cast<const f2*>(slot) + lane;
  return Adj2{q[0], q[kLanes / 2], q[kLanes], q[3 * kLanes / 2], q[2 * kLanes]};
}
__device__ __forceinline__ void adj_st(float* slot, int lane, const Adj2& x) {
  f2* q = reinterpret_cast<f2*>(slot) + lane;
  q[0] = x.G;
  q[kLanes / 2] = x.gp;
  q[kLanes] = x.gq;
  q[3 * kLanes / 2] = x.hp;
  q[2 * kLanes] = x.hq;
}

// Backward. kOut: grad_key/grad_value, per-lane partial sums and (last CTA per
// column block) the time gradients; !kOut: only the adjoint at the segment
// start (a.adj_out), for the segmented plan. Grid (B * ncblk, nseg), W warps
// per CTA; reference wkv_triton.py:60-142.
//
// Shared memory: NS stages | summaries [2][W][5][kLanes] | per-warp partial
// sums [W][2][kLanes] | barriers.
template <typename T, int W, bool kOut>
__global__ void __launch_bounds__(32 * W, 4)
    wkv_bwd_tp_kernel(const BwdArgs a, const __grid_constant__ CUtensorMap tk,
                      const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tgy,
                      const __grid_constant__ CUtensorMap tck, const __grid_constant__ CUtensorMap tgk,
                      const __grid_constant__ CUtensorMap tgv) {
  using G = TpB<T, W>;
  constexpr int NS = G::kStages;
  constexpr int R = kSub;
  extern __shared__ __align__(128) unsigned char smem[];
  float* sum = reinterpret_cast<float*>(smem + NS * G::kStageBytes);
  float* red = sum + G::kSumFloats;  // [W][2][kLanes]
  uint64_t* bars = reinterpret_cast<uint64_t*>(red + W * 2 * kLanes);
  auto slot = [&](int parity, int m) { return sum + (parity * W + m) * 5 * kLanes; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cb = blockIdx.x % a.ncblk, b = blockIdx.x / a.ncblk;
  const int c = cb * kLanes + 2 * lane;
  const int seg = blockIdx.y + a.seg_base;
  const bool v0 = c < a.C, v1 = c + 1 < a.C;
  const int t_begin = seg * a.seg_len;
  const int t_end = min(a.T, t_begin + a.seg_len);
  const int ntiles = (t_end - t_begin + R - 1) / R;
  const int nrounds = (ntiles + W - 1) / W;
  const bool force_slow = a.force_slow != 0;
  const size_t lseg = (size_t)b * a.nseg + seg;
  const bool seg_local = a.seg_start != nullptr || a.seg_sums != nullptr;  // checkpoints from the segment start

  f2 ww = splat(0.f), uu = splat(0.f);
  if (v0) {
    ww.x = a.w[c];
    uu.x = a.u[c];
  }
  if (v1) {
    ww.y = a.w[c + 1];
    uu.y = a.u[c + 1];
  }
  const Lane2 lc = make_lane2(ww, uu);
  Adj2 adj = adj_zero2();  // adjoint entering the current round (at its last tile's end)
  if (a.adj_in != nullptr)
    load_adj(a.adj_in, lseg, a.C, c, v0, v1, adj);
  else if (a.adj_sums != nullptr && seg + 1 < a.nseg)
    adj = fold_adjoint_summaries(a.adj_sums, b, a.nseg, seg, a.seg_len, a.T, a.C, c, v0, v1, lc);
  Fwd2 segst = fwd_identity2();
  if (a.seg_start != nullptr)
    load3(a.seg_start, lseg, a.C, c, v0, v1, segst.S, segst.p, segst.q);
  else if (a.seg_sums != nullptr && seg > 0)
    segst = fold_state_summaries(a.seg_sums, b, a.nseg, seg, a.seg_len, a.C, c, v0, v1, lc);
  f2 gwacc = splat(0.f), gu = splat(0.f);

  auto issue = [&](bool on, int r) {  // by the threads with `on` (one per CTA)
    const int st = r % NS;
    unsigned char* base = smem + st * G::kStageBytes;
    const int jb = ntiles - (r + 1) * W;  // first tile of the round (may be < 0)
    const int t0 = t_begin + jb * R;
    mbar_arrive_expect_tx_if(on, &bars[st], 3 * G::kBoxBytes + G::kCkBytes);
    tma_load_3d_if(on, base, &tk, &bars[st], cb * kLanes, t0, b);
    tma_load_3d_if(on, base + G::kBoxBytes, &tv, &bars[st], cb * kLanes, t0, b);
    tma_load_3d_if(on, base + 2 * G::kBoxBytes, &tgy, &bars[st], cb * kLanes, t0, b);
    tma_load_3d_if(on, base + 3 * G::kBoxBytes, &tck, &bars[st], cb * kLanes, 0,
                   b * a.nsub + t_begin / kSub + jb);
  };
  if (threadIdx.x == 0) {
    for (int st = 0; st < NS; ++st) mbar_init(&bars[st], 1);
    fence_barrier_init();
    prefetch_tensormap(&tk);
    prefetch_tensormap(&tv);
    prefetch_tensormap(&tgy);
    prefetch_tensormap(&tck);
    if (kOut) {
      prefetch_tensormap(&tgk);
      prefetch_tensormap(&tgv);
    }
  }
  __syncthreads();
  for (int r = 0; r < min(NS - 1, nrounds); ++r) issue(threadIdx.x == 0, r);

#pragma unroll 1
  for (int r = 0; r < nrounds; ++r) {
    const int st = r % NS;
    unsigned char* base = smem + st * G::kStageBytes;
    const int jb = ntiles - (r + 1) * W;
    const int j = jb + warp;
    const int t0 = t_begin + j * R;
    const int n = j < 0 ? 0 : min(R, t_end - t0);
    const bool arrived = mbar_wait_bounded(&bars[st], (r / NS) & 1);

    // A. recompute and local adjoint summary, reading this warp's rows of the
    // staged boxes; grad_key / grad_value are later staged over its k and
    // grad_y rows
    T* ktw = reinterpret_cast<T*>(base) + warp * R * kLanes;
    T* gtw = reinterpret_cast<T*>(base + 2 * G::kBoxBytes) + warp * R * kLanes;
    const T* kt = ktw + 2 * lane;
    const T* vt = reinterpret_cast<const T*>(base + G::kBoxBytes) + warp * R * kLanes + 2 * lane;
    const T* gt = gtw + 2 * lane;
    Fwd2 st0;  // forward state at the tile start
    {
      const f2* ck = reinterpret_cast<const f2*>(base + 3 * G::kBoxBytes) + warp * 3 * (kLanes / 2) + lane;
      st0 = Fwd2{ck[0], ck[kLanes / 2], ck[kLanes]};
    }
    if (seg_local && n > 0)
      st0 = (t0 == t_begin) ? segst : fwd_combine2(segst, t0 - t_begin, lc, st0);
    f2 s, p, q;
    bool ok;
    f2 re[R], rg[R], rn[R];
    Adj2 loc;
    auto check = [&](f2 kmax, f2 kmin, f2 gymax) {
      return fast_ok1(st0.S.x, st0.p.x, st0.q.x, kmax.x, kmin.x, n, lc.w2.x, lc.u2.x, s.x, p.x, q.x) &&
             fast_ok1(st0.S.y, st0.p.y, st0.q.y, kmax.y, kmin.y, n, lc.w2.y, lc.u2.y, s.y, p.y, q.y) &&
             fmaxf(gymax.x, gymax.y) <= 0x1p40f && !force_slow;
    };
    if (n == R) {  // k and grad_y rows read once, into registers, for the range scan and the recompute
      typename Pair<T>::raw kr[R], gr[R];
#pragma unroll
      for (int i = 0; i < R; ++i) {
        kr[i] = Pair<T>::ld(kt + i * kLanes);
        gr[i] = Pair<T>::ld(gt + i * kLanes);
      }
      f2 kmax, kmin;
      tile_kminmax<T, false>(kr, n, kmax, kmin);
      ok = check(kmax, kmin, tile_absmax<T>(gr));
      bwd_tp_recompute_regs<T>(kr, gr, vt, lc, s, p, q, re, rg, rn);
      bwd_tp_summary<false>(rg, rn, n, lc, loc.gp, loc.gq, loc.hp, loc.hq);
    } else {
      const Pre pre = prescan<T, true, true>(kt, gt, n);
      ok = n == 0 || check(pre.kmax, pre.kmin, pre.gymax);
      if (n == 0) s = p = q = splat(0.f);
      bwd_tp_recompute<T, true>(kt, vt, gt, n, lc, s, p, q, re, rg, rn);
      bwd_tp_summary<true>(rg, rn, n, lc, loc.gp, loc.gq, loc.hp, loc.hq);
    }
    loc.G = f2{-s.x, -s.y};
    const bool fast = __all_sync(kFull, ok);
    if (!fast && n > 0) loc = bwd_tp_exact_summary<T>(kt, vt, gt, n, st0, lc);
    // the previous round's staged outputs (lane 0's bulk group) have been read
    // out of the stage the next copy refills
    if (kOut) bulk_wait_read<0>();
    adj_st(slot(r & 1, warp), lane, loc);
    if (!__syncthreads_and(arrived)) {
      if (threadIdx.x == 0) {
        report_timeout(a.err);
        for (int q2 = r; q2 < min(r + NS - 1, nrounds); ++q2)
          mbar_wait_bounded(&bars[q2 % NS], (q2 / NS) & 1);
      }
      if (kOut) bulk_wait_all();
      return;
    }
    // every warp is past its last read of stage (r - 1) % NS
    if (r + NS - 1 < nrounds) issue(threadIdx.x == 0, r + NS - 1);

    // B. the adjoint at this warp's tile end; adj becomes the adjoint entering
    // the next round (every warp folds all of the round's summaries, in the
    // same order; a round of full tiles takes the branch-free 16-step combine)
    Adj2 ein = adj;
    {
      Adj2 sm[W];
#pragma unroll
      for (int m = 0; m < W; ++m) sm[m] = adj_ld(slot(r & 1, m), lane);
      if (jb >= 0 && t_begin + (jb + W) * R <= t_end) {
#pragma unroll
        for (int m = W - 1; m >= 0; --m) {
          if (m == warp) ein = adj;
          adj = adj_combine16(sm[m], adj, lc);
        }
      } else {
#pragma unroll
        for (int m = W - 1; m >= 0; --m) {
          const int nm = (jb + m) < 0 ? 0 : min(R, t_end - (t_begin + (jb + m) * R));
          if (m == warp) ein = adj;
          if (nm > 0) adj = adj_combine2(sm[m], adj, nm, lc);
        }
      }
    }

    // C. outputs from the incoming adjoint, staged over this warp's k and
    // grad_y rows and written with one bulk tensor store per tensor
    if (kOut && n > 0) {
      T* gks = ktw;
      T* gvs = gtw;
      const f2 f = ex2x2(add2(ein.G, s));  // integer exponents: exact
      const f2 gp = mul2(ein.gp, f), gq = mul2(ein.gq, f), hp = mul2(ein.hp, f), hq = mul2(ein.hq, f);
      const float amax = fmaxf(fmaxf(fmaxf(fabsf(gp.x), fabsf(gp.y)), fmaxf(fabsf(gq.x), fabsf(gq.y))),
                               fmaxf(fmaxf(fabsf(hp.x), fabsf(hp.y)), fmaxf(fabsf(hq.x), fabsf(hq.y))));
      if (fast && __all_sync(kFull, amax <= 0x1p80f)) {
        if (n == R)
          bwd_tp_outputs<T, false, kOut>(re, vt, rg, rn, n, lc, gp, gq, hp, hq, gks + 2 * lane,
                                         gvs + 2 * lane, gwacc, gu);
        else
          bwd_tp_outputs<T, true, kOut>(re, vt, rg, rn, n, lc, gp, gq, hp, hq, gks + 2 * lane,
                                        gvs + 2 * lane, gwacc, gu);
      } else {
        bwd_tp_exact<T>(a, b, t0, c, v0, v1, n, st0, ein, lc, gks + 2 * lane, gvs + 2 * lane,
                        gwacc, gu);
      }
      fence_proxy_async_smem();
      __syncwarp();
      tma_store_3d_if(lane == 0, &tgk, gks, cb * kLanes, t0, b);
      tma_store_3d_if(lane == 0, &tgv, gvs, cb * kLanes, t0, b);
      bulk_commit();
    }
  }
  if (kOut) bulk_wait_all();
  if (a.adj_out != nullptr && warp == 0) store_adj(a.adj_out, lseg, a.C, c, v0, v1, adj);
  if (!kOut || a.partial == nullptr) return;

  // per-lane partial sums of the CTA, summed over its warps in a fixed order
  {
    f2* rw = reinterpret_cast<f2*>(red + warp * 2 * kLanes) + lane;
    rw[0] = gwacc;
    rw[kLanes / 2] = gu;
  }
  __syncthreads();
  if (warp != 0) return;
  f2 sw = splat(0.f), su = splat(0.f);
#pragma unroll
  for (int m = 0; m < W; ++m) {
    const f2* rw = reinterpret_cast<const f2*>(red + m * 2 * kLanes) + lane;
    sw = add2(sw, rw[0]);
    su = add2(su, rw[kLanes / 2]);
  }
  {
    float* rp = a.partial + lseg * 2 * (size_t)a.C + c;
    if (v0) {
      rp[0] = sw.x;
      rp[a.C] = su.x;
    }
    if (v1) {
      rp[1] = sw.y;
      rp[a.C + 1] = su.y;
    }
  }
  if (a.tickets == nullptr) return;
  // The last CTA of this column block to finish sums every (b, segment) row in
  // a fixed order: grad_time_decay = w sum dL/dw (reference wkv_triton.py:117,
  // 194), grad_time_first = sum dL/du. No CTA waits for another.
  __threadfence();
  __syncwarp();
  unsigned ticket = 0;
  if (lane == 0) ticket = atomicAdd(&a.tickets[cb], 1u);
  ticket = __shfl_sync(kFull, ticket, 0);
  const int rows = a.B * a.nseg;
  if (ticket + 1 != static_cast<unsigned>(rows)) return;
  __threadfence();
  if (lane == 0) a.tickets[cb] = 0u;  // ready for a later call that reuses the counters
  reduce_time_grads(a, c, v0, v1, lc.w, rows);
}

}  // namespace wkv
