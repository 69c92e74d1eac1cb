// WKV kernels for sm_100a.
//
// One CTA = one warp = 64 consecutive channels of one batch row; each thread
// owns two adjacent channels (a lane pair). A CTA walks its time range in tiles
// of Pair<T>::kTileRows steps. On the TMA path a single elected lane streams
// [rows x 64] tiles of every input through a multi-stage ring of shared-memory
// buffers (cp.async.bulk.tensor + mbarrier complete_tx) and writes output tiles
// back with bulk tensor stores; on the generic path (C*sizeof(dtype) not a
// multiple of 16, or unaligned pointers) the lanes fill the same tiles with
// plain loads.
//
// Time can be split into segments (blockIdx.y) so that small B*C still fills
// the GPU: a segment is processed from a start state produced by a carry pass
// over per-segment summaries (the WKV state update is linear in the history, so
// segment summaries combine associatively).
//
// Kernels:
//   wkv_fwd_kernel<T, kY=true>   y for a segment (reference wkv_triton.py:34-58)
//   wkv_fwd_kernel<T, kY=false>  state only: per-sub-chunk checkpoints and/or
//                                the segment-end summary
//   wkv_bwd_kernel<T, kOut>      reverse sweep over sub-chunks with forward
//                                recompute from checkpoints (reference
//                                wkv_triton.py:60-142); its last CTA per
//                                column block reduces grad_time_decay/first;
//                                kOut=false only produces the segment's
//                                adjoint summary
//   wkv_carry_fwd_kernel         segment summaries -> segment start states
//   wkv_carry_adj_kernel         adjoint summaries -> adjoint at segment ends
#pragma once

#include "wkv_sub.cuh"

namespace wkv {

template <typename T>
struct Cfg {
  static constexpr int kRows = Pair<T>::kTileRows;  // steps per staged tile
  static constexpr int kTileElems = kRows * kLanes;
  static constexpr uint32_t kTileBytes = kTileElems * sizeof(T);
  static constexpr int kSubPerTile = kRows / kSub;
  static constexpr int kFwdStages = 4;
  static constexpr int kBwdStages = 3;
  static_assert(kRows % kSub == 0 && kSegAlign % kRows == 0, "tile/segment alignment");
};

template <typename T>
constexpr size_t fwd_smem_bytes(bool y) {
  return (size_t)(2 * Cfg<T>::kFwdStages + (y ? 2 : 0)) * Cfg<T>::kTileBytes +
         8 * Cfg<T>::kFwdStages;
}
template <typename T>
constexpr size_t bwd_smem_bytes(bool out) {
  return (size_t)(3 * Cfg<T>::kBwdStages + (out ? 4 : 0)) * Cfg<T>::kTileBytes +
         8 * Cfg<T>::kBwdStages;
}

struct FwdArgs {
  const void* k;
  const void* v;
  void* y;
  const float* decay;  // time_decay (decay_is_w == 0) or w = -exp(time_decay)
  const float* u;      // time_first
  int decay_is_w;
  int B, T, C;
  int ncblk;     // ceil(C / kLanes)
  int seg_len;   // steps per segment (a multiple of kSegAlign unless nseg == 1)
  int nseg;      // segments per lane
  int seg_base;  // segment of blockIdx.y == 0
  int nsub;      // checkpoint rows per batch row: ceil(T / kSub)
  float* ckpt;             // [B][nsub][3][C] states at sub-chunk starts, or null
  const float* seg_start;  // [B][nseg][3][C] segment start states, or null (zero state)
  float* seg_end;          // [B][nseg][3][C] segment end states, or null
  unsigned* zero_tickets;  // counters the first CTA resets for a later wkv_bwd_kernel, or null
  int nzero;
  const float* seg_sums;   // [B][nseg][3][C] segment summaries (from zero) to fold into the start state, or null
  int force_slow;
  unsigned* err;
  // Debug (wkv_set_debug_pipeline): the consumers' copy-wait limit in cycles,
  // and withholding the first round's copies so that wait runs out.
  long long wait_limit;
  int withhold_first;
};

struct BwdArgs {
  const void* k;
  const void* v;
  const void* gy;
  void* gk;
  void* gv;
  const float* w;
  const float* u;
  int B, T, C;
  int ncblk, seg_len, nseg, seg_base, nsub;
  const float* ckpt;       // [B][nsub][3][C]: true states, or states local to the segment
  const float* seg_start;  // [B][nseg][3][C] (ckpt is segment-local when non-null)
  const float* adj_in;     // [B][nseg][5][C] adjoint at segment ends, or null (zero)
  const float* seg_sums;   // [B][nseg][3][C] state summaries to fold into the segment start, or null
  const float* adj_sums;   // [B][nseg][5][C] adjoint summaries (s >= 1) to fold into the segment end, or null
  float* adj_out;          // [B][nseg][5][C] adjoint at segment starts, or null
  float* partial;          // [B][nseg][2][C] (gwacc, gu) per lane-segment, or null
  unsigned* tickets;       // [ncblk] arrival counters (zeroed beforehand), or null
  float* gtd;              // [C] grad_time_decay, written by the last CTA of a column block
  float* gtf;              // [C] grad_time_first
  int force_slow;
  unsigned* err;
};

// Rows of 3 [C] planes ([row][3][C] floats) for the two channels c, c+1.
__device__ __forceinline__ void load3(const float* base, size_t row, int C, int c, bool v0,
                                      bool v1, f2& a, f2& b, f2& d) {
  const float* r = base + row * 3 * (size_t)C + c;
  if (v0) {
    a.x = r[0];
    b.x = r[C];
    d.x = r[2 * (size_t)C];
  }
  if (v1) {
    a.y = r[1];
    b.y = r[C + 1];
    d.y = r[2 * (size_t)C + 1];
  }
}
__device__ __forceinline__ void store3(float* base, size_t row, int C, int c, bool v0, bool v1,
                                       f2 a, f2 b, f2 d) {
  float* r = base + row * 3 * (size_t)C + c;
  if (v0) {
    r[0] = a.x;
    r[C] = b.x;
    r[2 * (size_t)C] = d.x;
  }
  if (v1) {
    r[1] = a.y;
    r[C + 1] = b.y;
    r[2 * (size_t)C + 1] = d.y;
  }
}

// Rows of 5 [C] planes (an Adj2) for the two channels c, c+1.
__device__ __forceinline__ void load_adj(const float* base, size_t row, int C, int c, bool v0,
                                         bool v1, Adj2& a) {
  f2* f[5] = {&a.G, &a.gp, &a.gq, &a.hp, &a.hq};
  const float* r = base + row * 5 * (size_t)C + c;
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    if (v0) f[i]->x = r[i * (size_t)C];
    if (v1) f[i]->y = r[i * (size_t)C + 1];
  }
}
__device__ __forceinline__ void store_adj(float* base, size_t row, int C, int c, bool v0, bool v1,
                                          const Adj2& a) {
  const f2 f[5] = {a.G, a.gp, a.gq, a.hp, a.hq};
  float* r = base + row * 5 * (size_t)C + c;
#pragma unroll
  for (int i = 0; i < 5; ++i) {
    if (v0) r[i * (size_t)C] = f[i].x;
    if (v1) r[i * (size_t)C + 1] = f[i].y;
  }
}

// Generic path: the warp fills rows [0, rows) of a [rows][kLanes] tile.
// State at the start of segment `seg` of batch row b: the summaries of segments
// 0 .. seg-1 (each the state the segment reaches from zero) folded in order,
// every one decayed over a full segment. Loaded four at a time ahead of the
// serial fold. (The carry kernel does the same for all segments at once.)
__device__ __forceinline__ Fwd2 fold_state_summaries(const float* sums, int b, int nseg, int seg,
                                                     int seg_len, int C, int c, bool v0, bool v1,
                                                     const Lane2& lc) {
  Fwd2 st = fwd_identity2();
  constexpr int K = 4;
  for (int s0 = 0; s0 < seg; s0 += K) {
    Fwd2 l[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      l[k] = fwd_identity2();
      if (s0 + k < seg) load3(sums, (size_t)b * nseg + s0 + k, C, c, v0, v1, l[k].S, l[k].p, l[k].q);
    }
#pragma unroll
    for (int k = 0; k < K; ++k)
      if (s0 + k < seg) st = fwd_combine2(st, seg_len, lc, l[k]);
  }
  return st;
}

// Adjoint at the end of segment `seg`: the adjoint summaries of segments
// nseg-1 down to seg+1 (each accumulated from a zero adjoint at its own end)
// folded from a zero adjoint at T; the last segment may be shorter.
__device__ __forceinline__ Adj2 fold_adjoint_summaries(const float* sums, int b, int nseg, int seg,
                                                       int seg_len, int T, int C, int c, bool v0,
                                                       bool v1, const Lane2& lc);

template <typename T>
__device__ __forceinline__ void fill_tile(T* tile, const T* src, int b, int t0, int rows, int T_,
                                          int C, int c, bool v0, bool v1, int lane) {
  const size_t base = ((size_t)b * T_ + t0) * C + c;
  const T zero = Pair<T>::from_float(0.f);
#pragma unroll 4
  for (int r = 0; r < rows; ++r) {
    tile[r * kLanes + 2 * lane] = v0 ? src[base + (size_t)r * C] : zero;
    tile[r * kLanes + 2 * lane + 1] = v1 ? src[base + (size_t)r * C + 1] : zero;
  }
}
template <typename T>
__device__ __forceinline__ void drain_tile(const T* tile, T* dst, int b, int t0, int rows, int T_,
                                           int C, int c, bool v0, bool v1, int lane) {
  const size_t base = ((size_t)b * T_ + t0) * C + c;
#pragma unroll 4
  for (int r = 0; r < rows; ++r) {
    if (v0) dst[base + (size_t)r * C] = tile[r * kLanes + 2 * lane];
    if (v1) dst[base + (size_t)r * C + 1] = tile[r * kLanes + 2 * lane + 1];
  }
}

__device__ __forceinline__ void report_timeout(unsigned* err) {
  if (err) atomicOr(err, 1u);
}

// The last CTA of a column block: sum the per-lane partials of all rows (batch
// row x segment) in a fixed order, in double, and write grad_time_decay =
// w * sum dL/dw and grad_time_first = sum dL/du for the lane's two channels.
__device__ __forceinline__ void reduce_time_grads(const BwdArgs& a, int c, bool v0, bool v1, f2 w,
                                                  int rows) {
  double sw0 = 0.0, su0 = 0.0, sw1 = 0.0, su1 = 0.0;
  const float* base = a.partial + c;
  for (int r0 = 0; r0 < rows; r0 += 8) {
    float pw0[8], pu0[8], pw1[8], pu1[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const bool in = r0 + i < rows;
      const size_t o = (size_t)(r0 + i) * 2 * a.C;
      pw0[i] = (in && v0) ? __ldcg(base + o) : 0.f;
      pu0[i] = (in && v0) ? __ldcg(base + o + a.C) : 0.f;
      pw1[i] = (in && v1) ? __ldcg(base + o + 1) : 0.f;
      pu1[i] = (in && v1) ? __ldcg(base + o + a.C + 1) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      sw0 += pw0[i];
      su0 += pu0[i];
      sw1 += pw1[i];
      su1 += pu1[i];
    }
  }
  if (v0) {
    a.gtd[c] = static_cast<float>(static_cast<double>(w.x) * sw0);
    a.gtf[c] = static_cast<float>(su0);
  }
  if (v1) {
    a.gtd[c + 1] = static_cast<float>(static_cast<double>(w.y) * sw1);
    a.gtf[c + 1] = static_cast<float>(su1);
  }
}

// ------------------------------------------------------------------ forward

template <typename T, bool kY, bool kTma>
__global__ void __launch_bounds__(kThreads)
    wkv_fwd_kernel(const FwdArgs a, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap ty) {
  using G = Cfg<T>;
  constexpr int S = G::kFwdStages;
  extern __shared__ __align__(128) unsigned char smem[];
  T* kbuf = reinterpret_cast<T*>(smem);
  T* vbuf = kbuf + S * G::kTileElems;
  T* ybuf = vbuf + S * G::kTileElems;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ybuf + (kY ? 2 : 0) * G::kTileElems);

  const int lane = threadIdx.x;
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
  const int ntiles = (t_end - t_begin + G::kRows - 1) / G::kRows;
  const bool force_slow = a.force_slow != 0;

  if (a.zero_tickets != nullptr && blockIdx.x == 0 && blockIdx.y == 0)
    for (int i = lane; i < a.nzero; i += kThreads) a.zero_tickets[i] = 0u;

  Fwd2 st = fwd_identity2();
  if (a.seg_start != nullptr)
    load3(a.seg_start, (size_t)b * a.nseg + seg, a.C, c, v0, v1, st.S, st.p, st.q);

  auto issue = [&](int j) {
    const int s = j % S;
    mbar_arrive_expect_tx(&bars[s], 2 * G::kTileBytes);
    const int t0 = t_begin + j * G::kRows;
    tma_load_3d(kbuf + s * G::kTileElems, &tk, &bars[s], cb * kLanes, t0, b);
    tma_load_3d(vbuf + s * G::kTileElems, &tv, &bars[s], cb * kLanes, t0, b);
  };
  // Makes tile j resident (waits for its copy, or fills it on the generic path).
  // On a copy timeout it records the error, drains the copies it issued and
  // returns false; the caller then exits.
  auto acquire = [&](int j) -> bool {
    const int s = j % S;
    if (kTma) {
      const bool ok = mbar_wait_bounded(&bars[s], (j / S) & 1);
      if (!__all_sync(kFull, ok)) {
        if (lane == 0) report_timeout(a.err);
        for (int r = j + 1; r < min(j + S, ntiles); ++r) mbar_wait_bounded(&bars[r % S], (r / S) & 1);
        if (kY && lane == 0) bulk_wait_all();
        return false;
      }
    } else {
      const int t0 = t_begin + j * G::kRows;
      const int rows = min(G::kRows, t_end - t0);
      fill_tile(kbuf + s * G::kTileElems, static_cast<const T*>(a.k), b, t0, rows, a.T, a.C, c, v0, v1, lane);
      fill_tile(vbuf + s * G::kTileElems, static_cast<const T*>(a.v), b, t0, rows, a.T, a.C, c, v0, v1, lane);
      __syncwarp();
    }
    return true;
  };
  if (kTma) {
    if (lane == 0) {
      for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
      fence_barrier_init();
      prefetch_tensormap(&tk);
      prefetch_tensormap(&tv);
      if (kY) prefetch_tensormap(&ty);
    }
    __syncwarp();
    if (lane == 0)
      for (int j = 0; j < min(S, ntiles); ++j) issue(j);
  }

#pragma unroll 1
  for (int j = 0; j < ntiles; ++j) {
    const int sidx = j % S;
    const int t0 = t_begin + j * G::kRows;
    const int rows = min(G::kRows, t_end - t0);
    if (!acquire(j)) return;
    T* ys = ybuf + (j & 1) * G::kTileElems;
    if (kY && kTma && j >= 2) {  // ys was last read by the store of tile j-2
      if (lane == 0) bulk_wait_read<1>();
      __syncwarp();
    }
    const int off = 2 * lane;
    const size_t ck_row0 = (size_t)b * a.nsub + t0 / kSub;
    if (rows == G::kRows)
      fwd_tile2<T, false, kY>(st, kbuf + sidx * G::kTileElems + off, vbuf + sidx * G::kTileElems + off,
                              ys + off, rows, lc, force_slow, a.ckpt, ck_row0, a.C, c, v0, v1);
    else
      fwd_tile2<T, true, kY>(st, kbuf + sidx * G::kTileElems + off, vbuf + sidx * G::kTileElems + off,
                             ys + off, rows, lc, force_slow, a.ckpt, ck_row0, a.C, c, v0, v1);
    if (kY) {
      if (kTma) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(&ty, ys, cb * kLanes, t0, b);
          bulk_commit();
        }
      } else {
        __syncwarp();
        drain_tile(ys, static_cast<T*>(a.y), b, t0, rows, a.T, a.C, c, v0, v1, lane);
      }
    }
    __syncwarp();
    if (kTma && lane == 0 && j + S < ntiles) issue(j + S);
  }
  if (kTma && kY && lane == 0) bulk_wait_all();
  if (a.seg_end != nullptr)
    store3(a.seg_end, (size_t)b * a.nseg + seg, a.C, c, v0, v1, st.S, st.p, st.q);
}

// ----------------------------------------------------------------- backward

template <typename T, bool kOut, bool kTma>
__global__ void __launch_bounds__(kThreads)
    wkv_bwd_kernel(const BwdArgs a, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tgy,
                   const __grid_constant__ CUtensorMap tgk,
                   const __grid_constant__ CUtensorMap tgv) {
  using G = Cfg<T>;
  constexpr int S = G::kBwdStages;
  extern __shared__ __align__(128) unsigned char smem[];
  T* kbuf = reinterpret_cast<T*>(smem);
  T* vbuf = kbuf + S * G::kTileElems;
  T* gybuf = vbuf + S * G::kTileElems;
  T* gkbuf = gybuf + S * G::kTileElems;  // [2][tile] when kOut
  T* gvbuf = gkbuf + (kOut ? 2 : 0) * G::kTileElems;
  uint64_t* bars = reinterpret_cast<uint64_t*>(gvbuf + (kOut ? 2 : 0) * G::kTileElems);

  const int lane = threadIdx.x;
  const int cb = blockIdx.x % a.ncblk, b = blockIdx.x / a.ncblk;
  const int c = cb * kLanes + 2 * lane;
  const int seg = blockIdx.y + a.seg_base;
  const bool v0 = c < a.C, v1 = c + 1 < a.C;
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
  const int t_begin = seg * a.seg_len;
  const int t_end = min(a.T, t_begin + a.seg_len);
  const int ntiles = (t_end - t_begin + G::kRows - 1) / G::kRows;
  const bool force_slow = a.force_slow != 0;
  const size_t lseg = (size_t)b * a.nseg + seg;

  Adj2 adj = adj_zero2();
  if (a.adj_in != nullptr) load_adj(a.adj_in, lseg, a.C, c, v0, v1, adj);
  Fwd2 segst = fwd_identity2();
  if (a.seg_start != nullptr) load3(a.seg_start, lseg, a.C, c, v0, v1, segst.S, segst.p, segst.q);
  f2 gwacc = splat(0.f), gu = splat(0.f);
  // Checkpoints are loaded one sub-chunk ahead of their use (sub-chunks are
  // visited last to first, kSub steps apart).
  const int t_last = t_begin + ((t_end - t_begin - 1) / kSub) * kSub;
  Fwd2 pend = fwd_identity2();
  load3(a.ckpt, (size_t)b * a.nsub + t_last / kSub, a.C, c, v0, v1, pend.S, pend.p, pend.q);

  // Tiles are visited last to first; the jj-th visited tile is j = ntiles-1-jj.
  auto issue = [&](int jj) {
    const int s = jj % S;
    const int t0 = t_begin + (ntiles - 1 - jj) * G::kRows;
    mbar_arrive_expect_tx(&bars[s], 3 * G::kTileBytes);
    tma_load_3d(kbuf + s * G::kTileElems, &tk, &bars[s], cb * kLanes, t0, b);
    tma_load_3d(vbuf + s * G::kTileElems, &tv, &bars[s], cb * kLanes, t0, b);
    tma_load_3d(gybuf + s * G::kTileElems, &tgy, &bars[s], cb * kLanes, t0, b);
  };
  auto acquire = [&](int jj) -> bool {
    const int s = jj % S;
    if (kTma) {
      const bool ok = mbar_wait_bounded(&bars[s], (jj / S) & 1);
      if (!__all_sync(kFull, ok)) {
        if (lane == 0) report_timeout(a.err);
        for (int r = jj + 1; r < min(jj + S, ntiles); ++r)
          mbar_wait_bounded(&bars[r % S], (r / S) & 1);
        if (kOut && lane == 0) bulk_wait_all();
        return false;
      }
    } else {
      const int t0 = t_begin + (ntiles - 1 - jj) * G::kRows;
      const int rows = min(G::kRows, t_end - t0);
      fill_tile(kbuf + s * G::kTileElems, static_cast<const T*>(a.k), b, t0, rows, a.T, a.C, c, v0, v1, lane);
      fill_tile(vbuf + s * G::kTileElems, static_cast<const T*>(a.v), b, t0, rows, a.T, a.C, c, v0, v1, lane);
      fill_tile(gybuf + s * G::kTileElems, static_cast<const T*>(a.gy), b, t0, rows, a.T, a.C, c, v0, v1, lane);
      __syncwarp();
    }
    return true;
  };
  if (kTma) {
    if (lane == 0) {
      for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
      fence_barrier_init();
      prefetch_tensormap(&tk);
      prefetch_tensormap(&tv);
      prefetch_tensormap(&tgy);
      if (kOut) {
        prefetch_tensormap(&tgk);
        prefetch_tensormap(&tgv);
      }
    }
    __syncwarp();
    if (lane == 0)
      for (int jj = 0; jj < min(S, ntiles); ++jj) issue(jj);
  }

#pragma unroll 1
  for (int jj = 0; jj < ntiles; ++jj) {
    const int j = ntiles - 1 - jj;
    const int sidx = jj % S;
    const int t0 = t_begin + j * G::kRows;
    const int rows = min(G::kRows, t_end - t0);
    if (!acquire(jj)) return;
    T* gks = gkbuf + (jj & 1) * G::kTileElems;
    T* gvs = gvbuf + (jj & 1) * G::kTileElems;
    if (kOut && kTma && jj >= 2) {
      if (lane == 0) bulk_wait_read<1>();  // gks/gvs were last read by tile jj-2's store
      __syncwarp();
    }
#pragma unroll 1
    for (int sb = G::kSubPerTile - 1; sb >= 0; --sb) {
      const int r0 = sb * kSub;
      if (r0 >= rows) continue;
      const int L = min(kSub, rows - r0);
      const int t = t0 + r0;
      Fwd2 st = pend;
      if (t - kSub >= t_begin)
        load3(a.ckpt, (size_t)b * a.nsub + (t - kSub) / kSub, a.C, c, v0, v1, pend.S, pend.p, pend.q);
      if (a.seg_start != nullptr) st = (t == t_begin) ? segst : fwd_combine2(segst, t - t_begin, lc, st);
      const int off = r0 * kLanes + 2 * lane;
      const T* ks = kbuf + sidx * G::kTileElems + off;
      const T* vs = vbuf + sidx * G::kTileElems + off;
      const T* gys = gybuf + sidx * G::kTileElems + off;
      if (L == kSub) {
        const Pre pre = prescan<T, false, true>(ks, gys, L);
        bwd_sub2<T, false, kOut>(st, pre, adj, ks, vs, gys, gks + off, gvs + off, L, lc, gwacc, gu,
                                 force_slow);
      } else {
        const Pre pre = prescan<T, true, true>(ks, gys, L);
        bwd_sub2<T, true, kOut>(st, pre, adj, ks, vs, gys, gks + off, gvs + off, L, lc, gwacc, gu,
                                force_slow);
      }
    }
    if (kOut) {
      if (kTma) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(&tgk, gks, cb * kLanes, t0, b);
          tma_store_3d(&tgv, gvs, cb * kLanes, t0, b);
          bulk_commit();
        }
      } else {
        __syncwarp();
        drain_tile(gks, static_cast<T*>(a.gk), b, t0, rows, a.T, a.C, c, v0, v1, lane);
        drain_tile(gvs, static_cast<T*>(a.gv), b, t0, rows, a.T, a.C, c, v0, v1, lane);
      }
    }
    __syncwarp();
    if (kTma && lane == 0 && jj + S < ntiles) issue(jj + S);
  }
  if (kTma && kOut && lane == 0) bulk_wait_all();
  if (a.adj_out != nullptr) store_adj(a.adj_out, lseg, a.C, c, v0, v1, adj);
  if (a.partial == nullptr) return;
  {
    float* r = a.partial + lseg * 2 * (size_t)a.C + c;
    if (v0) {
      r[0] = gwacc.x;
      r[a.C] = gu.x;
    }
    if (v1) {
      r[1] = gwacc.y;
      r[a.C + 1] = gu.y;
    }
  }
  if (a.tickets == nullptr) return;
  // The last CTA of this column block to finish sums every (b, segment) row in
  // a fixed order: grad_time_decay = w sum gwacc (dL/dw * w, reference
  // wkv_triton.py:117,194), grad_time_first = sum gu. No CTA waits for another.
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

// ------------------------------------------------------------------- carries

__device__ __forceinline__ void load3s(const float* base, size_t row, int C, int c, float& a,
                                       float& b, float& d) {
  const float* r = base + row * 3 * (size_t)C + c;
  a = r[0];
  b = r[C];
  d = r[2 * (size_t)C];
}
__device__ __forceinline__ void store3s(float* base, size_t row, int C, int c, float a, float b,
                                        float d) {
  float* r = base + row * 3 * (size_t)C + c;
  r[0] = a;
  r[C] = b;
  r[2 * (size_t)C] = d;
}

// In place over seg[B][nseg][3][C]: entry s holds the state a segment reaches
// from zero (its summary); on exit it holds the true state at the segment start.
__global__ void wkv_carry_fwd_kernel(float* seg, const float* decay, int decay_is_w, int B, int T,
                                     int C, int nseg, int seg_len) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)B * C) return;
  const int b = static_cast<int>(i / C), c = static_cast<int>(i % C);
  const float d = decay[c];
  const float ew = expf(decay_is_w ? d : -expf(d));  // as make_lane2
  // every combined segment is a full one (only the last may be shorter, and
  // nothing follows it)
  const Decay1 dfull = ew_decay(ew, seg_len);
  float S = kNegBig, p = 0.f, q = 0.f;
  constexpr int K = 8;  // summaries loaded K at a time, ahead of the serial chain
  for (int s0 = 0; s0 < nseg; s0 += K) {
    float lS[K], lp[K], lq[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      lS[k] = kNegBig;
      lp[k] = lq[k] = 0.f;
      if (s0 + k + 1 < nseg) load3s(seg, (size_t)b * nseg + s0 + k, C, c, lS[k], lp[k], lq[k]);
    }
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int s = s0 + k;
      if (s >= nseg) break;
      store3s(seg, (size_t)b * nseg + s, C, c, S, p, q);
      if (s + 1 < nseg) {
        fwd_combine1(S, p, q, dfull, lS[k], lp[k], lq[k]);
        S = lS[k];
        p = lp[k];
        q = lq[k];
      }
    }
  }
}

// In place over adj[B][nseg][5][C]: entry s (s >= 1) holds the adjoint at the
// start of segment s accumulated from a zero adjoint at its end; on exit entry s
// holds the true adjoint at the end of segment s.
__global__ void wkv_carry_adj_kernel(float* adj, const float* w, int B, int T, int C, int nseg,
                                     int seg_len) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)B * C) return;
  const int b = static_cast<int>(i / C), c = static_cast<int>(i % C);
  const float ew = expf(w[c]);  // as make_lane2
  const int last_len = T - (nseg - 1) * seg_len;  // the last segment may be shorter
  const Decay1 dfull = ew_decay(ew, seg_len), dlast = ew_decay(ew, last_len);
  float e[5] = {kNegBig, 0.f, 0.f, 0.f, 0.f};
  constexpr int K = 4;  // summaries loaded K at a time, ahead of the serial chain
  for (int s0 = nseg - 1; s0 >= 0; s0 -= K) {
    float l[K][5];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int s = s0 - k;
      l[k][0] = kNegBig;
      l[k][1] = l[k][2] = l[k][3] = l[k][4] = 0.f;
      if (s > 0) {
        const float* r = adj + ((size_t)b * nseg + s) * 5 * (size_t)C + c;
#pragma unroll
        for (int f = 0; f < 5; ++f) l[k][f] = r[f * (size_t)C];
      }
    }
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int s = s0 - k;
      if (s < 0) break;
      float* r = adj + ((size_t)b * nseg + s) * 5 * (size_t)C + c;
#pragma unroll
      for (int f = 0; f < 5; ++f) r[f * (size_t)C] = e[f];
      if (s > 0) {
        const bool last = s == nseg - 1;
        adj_combine1(l[k], e, last ? last_len : seg_len, last ? dlast : dfull);
      }
    }
  }
}

}  // namespace wkv
