// WKV kernels for sm_100a.
//
// One CTA = one warp = 32 consecutive channels of one batch row; one thread per
// (b, c) lane. Each CTA walks its time range in tiles of kTile steps. On the TMA
// path a single elected lane streams [kTile x 32] tiles of every input through a
// multi-stage ring of shared-memory buffers (cp.async.bulk.tensor + mbarrier
// complete_tx) and writes output tiles back with bulk tensor stores; on the
// generic path (C*sizeof(dtype) not a multiple of 16, or unaligned pointers) the
// lanes fill the same tiles with plain loads.
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

#include "wkv_device.cuh"

namespace wkv {

template <typename T>
struct Stages {
  static constexpr int fwd = sizeof(T) == 4 ? 3 : 4;
  static constexpr int bwd = sizeof(T) == 4 ? 2 : 3;
};

template <typename T>
constexpr size_t fwd_smem_bytes(bool y) {
  return (size_t)(2 * Stages<T>::fwd + (y ? 2 : 0)) * kTile * kLanes * sizeof(T) +
         8 * Stages<T>::fwd;
}
template <typename T>
constexpr size_t bwd_smem_bytes(bool out) {
  return (size_t)(3 * Stages<T>::bwd + (out ? 4 : 0)) * kTile * kLanes * sizeof(T) +
         8 * Stages<T>::bwd;
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
  int seg_len;   // steps per segment (a multiple of kTile unless nseg == 1)
  int nseg;      // segments per lane
  int seg_base;  // segment of blockIdx.y == 0
  int nsub;      // checkpoint rows per batch row: ceil(T / kSub)
  float* ckpt;             // [B][nsub][3][C] states at sub-chunk starts, or null
  const float* seg_start;  // [B][nseg][3][C] segment start states, or null (zero state)
  float* seg_end;          // [B][nseg][3][C] segment end states, or null
  unsigned* zero_tickets;  // counters the first CTA resets for a later wkv_bwd_kernel, or null
  int nzero;
  int force_slow;
  unsigned* err;
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
  const float* adj_in;     // [B][nseg][3][C] adjoint at segment ends, or null (zero)
  float* adj_out;          // [B][nseg][3][C] adjoint at segment starts, or null
  float* partial;          // [B][nseg][2][C] (gwacc, gu) per lane-segment, or null
  unsigned* tickets;       // [ncblk] arrival counters (zeroed beforehand), or null
  float* gtd;              // [C] grad_time_decay, written by the last CTA of a column block
  float* gtf;              // [C] grad_time_first
  int force_slow;
  unsigned* err;
};

__device__ __forceinline__ Fwd load_fwd(const float* base, size_t row, int C, int c) {
  const float* r = base + row * 3 * (size_t)C + c;
  return Fwd{r[0], r[C], r[2 * (size_t)C]};
}
__device__ __forceinline__ void store_fwd(float* base, size_t row, int C, int c, const Fwd& s) {
  float* r = base + row * 3 * (size_t)C + c;
  r[0] = s.S;
  r[C] = s.p;
  r[2 * (size_t)C] = s.q;
}
__device__ __forceinline__ Adj load_adj(const float* base, size_t row, int C, int c) {
  const float* r = base + row * 3 * (size_t)C + c;
  return Adj{r[0], r[C], r[2 * (size_t)C]};
}
__device__ __forceinline__ void store_adj(float* base, size_t row, int C, int c, const Adj& s) {
  float* r = base + row * 3 * (size_t)C + c;
  r[0] = s.G;
  r[C] = s.gp;
  r[2 * (size_t)C] = s.gq;
}

// Generic path: the warp fills rows [0, rows) of a [kTile][kLanes] tile.
template <typename T>
__device__ __forceinline__ void fill_tile(T* tile, const T* src, int b, int t0, int rows, int T_,
                                          int C, int c, bool cval, int lane) {
  const size_t base = ((size_t)b * T_ + t0) * C + c;
#pragma unroll 4
  for (int r = 0; r < rows; ++r) tile[r * kLanes + lane] = cval ? src[base + (size_t)r * C] : T(0.f);
}
template <typename T>
__device__ __forceinline__ void drain_tile(const T* tile, T* dst, int b, int t0, int rows, int T_,
                                           int C, int c, bool cval, int lane) {
  if (!cval) return;
  const size_t base = ((size_t)b * T_ + t0) * C + c;
#pragma unroll 4
  for (int r = 0; r < rows; ++r) dst[base + (size_t)r * C] = tile[r * kLanes + lane];
}

__device__ __forceinline__ void report_timeout(unsigned* err) {
  if (err) atomicOr(err, 1u);
}

// ------------------------------------------------------------------ forward

template <typename T, bool kY, bool kTma>
__global__ void __launch_bounds__(kLanes)
    wkv_fwd_kernel(const FwdArgs a, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap ty) {
  constexpr int S = Stages<T>::fwd;
  constexpr int kTileElems = kTile * kLanes;
  constexpr uint32_t kTileBytes = kTileElems * sizeof(T);
  extern __shared__ __align__(128) unsigned char smem[];
  T* kbuf = reinterpret_cast<T*>(smem);
  T* vbuf = kbuf + S * kTileElems;
  T* ybuf = vbuf + S * kTileElems;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ybuf + (kY ? 2 : 0) * kTileElems);

  const int lane = threadIdx.x;
  const int cb = blockIdx.x % a.ncblk, b = blockIdx.x / a.ncblk;
  const int c = cb * kLanes + lane;
  const int seg = blockIdx.y + a.seg_base;
  const bool cval = c < a.C;
  const float dec = cval ? a.decay[c] : 0.f;
  const Lane lc = make_lane(a.decay_is_w ? dec : -expf(dec), cval ? a.u[c] : 0.f);
  const int t_begin = seg * a.seg_len;
  const int t_end = min(a.T, t_begin + a.seg_len);
  const int ntiles = (t_end - t_begin + kTile - 1) / kTile;
  const bool force_slow = a.force_slow != 0;

  if (a.zero_tickets != nullptr && blockIdx.x == 0 && blockIdx.y == 0)
    for (int i = lane; i < a.nzero; i += kLanes) a.zero_tickets[i] = 0u;

  Fwd st = fwd_identity();
  if (a.seg_start != nullptr && cval) st = load_fwd(a.seg_start, (size_t)b * a.nseg + seg, a.C, c);

  auto issue = [&](int j) {
    const int s = j % S;
    mbar_arrive_expect_tx(&bars[s], 2 * kTileBytes);
    const int t0 = t_begin + j * kTile;
    tma_load_3d(kbuf + s * kTileElems, &tk, &bars[s], cb * kLanes, t0, b);
    tma_load_3d(vbuf + s * kTileElems, &tv, &bars[s], cb * kLanes, t0, b);
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

  for (int j = 0; j < ntiles; ++j) {
    const int s = j % S;
    const int t0 = t_begin + j * kTile;
    const int rows = min(kTile, t_end - t0);
    T* ks = kbuf + s * kTileElems;
    T* vs = vbuf + s * kTileElems;
    T* ys = ybuf + (j & 1) * kTileElems;
    if (kTma) {
      const bool ok = mbar_wait_bounded(&bars[s], (j / S) & 1);
      if (!__all_sync(kFull, ok)) {
        if (lane == 0) report_timeout(a.err);
        for (int r = j + 1; r < min(j + S, ntiles); ++r) mbar_wait_bounded(&bars[r % S], (r / S) & 1);
        if (kY && lane == 0) bulk_wait_all();
        return;
      }
      if (kY && j >= 2) {  // ys was last read by the store of tile j-2
        if (lane == 0) bulk_wait_read<1>();
        __syncwarp();
      }
    } else {
      fill_tile(ks, static_cast<const T*>(a.k), b, t0, rows, a.T, a.C, c, cval, lane);
      fill_tile(vs, static_cast<const T*>(a.v), b, t0, rows, a.T, a.C, c, cval, lane);
      __syncwarp();
    }
#pragma unroll 1
    for (int sb = 0; sb < kSubPerTile; ++sb) {
      const int r0 = sb * kSub;
      if (r0 >= rows) break;
      const int L = min(kSub, rows - r0);
      if (!kY && a.ckpt != nullptr && cval)
        store_fwd(a.ckpt, (size_t)b * a.nsub + (t0 + r0) / kSub, a.C, c, st);
      const int off = r0 * kLanes + lane;
      if (L == kSub)
        fwd_sub<T, false, kY>(st, ks + off, vs + off, ys + off, L, lc, force_slow);
      else
        fwd_sub<T, true, kY>(st, ks + off, vs + off, ys + off, L, lc, force_slow);
    }
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
        drain_tile(ys, static_cast<T*>(a.y), b, t0, rows, a.T, a.C, c, cval, lane);
      }
    }
    __syncwarp();
    if (kTma && lane == 0 && j + S < ntiles) issue(j + S);
  }
  if (kTma && kY && lane == 0) bulk_wait_all();
  if (a.seg_end != nullptr && cval) store_fwd(a.seg_end, (size_t)b * a.nseg + seg, a.C, c, st);
}

// ----------------------------------------------------------------- backward

template <typename T, bool kOut, bool kTma>
__global__ void __launch_bounds__(kLanes)
    wkv_bwd_kernel(const BwdArgs a, const __grid_constant__ CUtensorMap tk,
                   const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tgy,
                   const __grid_constant__ CUtensorMap tgk,
                   const __grid_constant__ CUtensorMap tgv) {
  constexpr int S = Stages<T>::bwd;
  constexpr int kTileElems = kTile * kLanes;
  constexpr uint32_t kTileBytes = kTileElems * sizeof(T);
  extern __shared__ __align__(128) unsigned char smem[];
  T* kbuf = reinterpret_cast<T*>(smem);
  T* vbuf = kbuf + S * kTileElems;
  T* gybuf = vbuf + S * kTileElems;
  T* gkbuf = gybuf + S * kTileElems;  // [2][tile] when kOut
  T* gvbuf = gkbuf + (kOut ? 2 : 0) * kTileElems;
  uint64_t* bars = reinterpret_cast<uint64_t*>(gvbuf + (kOut ? 2 : 0) * kTileElems);

  const int lane = threadIdx.x;
  const int cb = blockIdx.x % a.ncblk, b = blockIdx.x / a.ncblk;
  const int c = cb * kLanes + lane;
  const int seg = blockIdx.y + a.seg_base;
  const bool cval = c < a.C;
  const Lane lc = make_lane(cval ? a.w[c] : 0.f, cval ? a.u[c] : 0.f);
  const int t_begin = seg * a.seg_len;
  const int t_end = min(a.T, t_begin + a.seg_len);
  const int ntiles = (t_end - t_begin + kTile - 1) / kTile;
  const bool force_slow = a.force_slow != 0;
  const size_t lseg = (size_t)b * a.nseg + seg;

  Adj adj = adj_zero();
  if (a.adj_in != nullptr && cval) adj = load_adj(a.adj_in, lseg, a.C, c);
  Fwd segst = fwd_identity();
  if (a.seg_start != nullptr && cval) segst = load_fwd(a.seg_start, lseg, a.C, c);
  float gwacc = 0.f, gu = 0.f;
  // Checkpoints are loaded one sub-chunk ahead of their use (sub-chunks are
  // visited last to first, kSub steps apart).
  const int t_last = t_begin + ((t_end - t_begin - 1) / kSub) * kSub;
  Fwd pend = fwd_identity();
  if (cval) pend = load_fwd(a.ckpt, (size_t)b * a.nsub + t_last / kSub, a.C, c);

  // Tiles are visited last to first; the jj-th visited tile is j = ntiles-1-jj.
  auto issue = [&](int jj) {
    const int s = jj % S;
    const int t0 = t_begin + (ntiles - 1 - jj) * kTile;
    mbar_arrive_expect_tx(&bars[s], 3 * kTileBytes);
    tma_load_3d(kbuf + s * kTileElems, &tk, &bars[s], cb * kLanes, t0, b);
    tma_load_3d(vbuf + s * kTileElems, &tv, &bars[s], cb * kLanes, t0, b);
    tma_load_3d(gybuf + s * kTileElems, &tgy, &bars[s], cb * kLanes, t0, b);
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

  for (int jj = 0; jj < ntiles; ++jj) {
    const int j = ntiles - 1 - jj;
    const int s = jj % S;
    const int t0 = t_begin + j * kTile;
    const int rows = min(kTile, t_end - t0);
    T* ks = kbuf + s * kTileElems;
    T* vs = vbuf + s * kTileElems;
    T* gys = gybuf + s * kTileElems;
    T* gks = gkbuf + (jj & 1) * kTileElems;
    T* gvs = gvbuf + (jj & 1) * kTileElems;
    if (kTma) {
      const bool ok = mbar_wait_bounded(&bars[s], (jj / S) & 1);
      if (!__all_sync(kFull, ok)) {
        if (lane == 0) report_timeout(a.err);
        for (int r = jj + 1; r < min(jj + S, ntiles); ++r)
          mbar_wait_bounded(&bars[r % S], (r / S) & 1);
        if (kOut && lane == 0) bulk_wait_all();
        return;
      }
      if (kOut && jj >= 2) {
        if (lane == 0) bulk_wait_read<1>();
        __syncwarp();
      }
    } else {
      fill_tile(ks, static_cast<const T*>(a.k), b, t0, rows, a.T, a.C, c, cval, lane);
      fill_tile(vs, static_cast<const T*>(a.v), b, t0, rows, a.T, a.C, c, cval, lane);
      fill_tile(gys, static_cast<const T*>(a.gy), b, t0, rows, a.T, a.C, c, cval, lane);
      __syncwarp();
    }
#pragma unroll 1
    for (int sb = kSubPerTile - 1; sb >= 0; --sb) {
      const int r0 = sb * kSub;
      if (r0 >= rows) continue;
      const int L = min(kSub, rows - r0);
      const int t = t0 + r0;
      Fwd st = pend;
      if (cval && t - kSub >= t_begin) pend = load_fwd(a.ckpt, (size_t)b * a.nsub + (t - kSub) / kSub, a.C, c);
      if (a.seg_start != nullptr) st = (t == t_begin) ? segst : fwd_combine(segst, t - t_begin, lc, st);
      const int off = r0 * kLanes + lane;
      if (L == kSub)
        bwd_sub<T, false, kOut>(st, adj, ks + off, vs + off, gys + off, gks + off, gvs + off, L,
                                lc, gwacc, gu, force_slow);
      else
        bwd_sub<T, true, kOut>(st, adj, ks + off, vs + off, gys + off, gks + off, gvs + off, L,
                               lc, gwacc, gu, force_slow);
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
        drain_tile(gks, static_cast<T*>(a.gk), b, t0, rows, a.T, a.C, c, cval, lane);
        drain_tile(gvs, static_cast<T*>(a.gv), b, t0, rows, a.T, a.C, c, cval, lane);
      }
    }
    __syncwarp();
    if (kTma && lane == 0 && jj + S < ntiles) issue(jj + S);
  }
  if (kTma && kOut && lane == 0) bulk_wait_all();
  if (cval && a.adj_out != nullptr) store_adj(a.adj_out, lseg, a.C, c, adj);
  if (a.partial == nullptr) return;
  if (cval) {
    float* r = a.partial + lseg * 2 * (size_t)a.C + c;
    r[0] = gwacc;
    r[a.C] = gu;
  }
  if (a.tickets == nullptr) return;
  // The last CTA of this column block to finish sums every (b, segment) row in
  // a fixed order: grad_time_decay = w e^w sum gwacc (dL/dw * w, reference
  // wkv_triton.py:117,194), grad_time_first = sum gu. No CTA waits for another.
  __threadfence();
  __syncwarp();
  unsigned ticket = 0;
  if (lane == 0) ticket = atomicAdd(&a.tickets[cb], 1u);
  ticket = __shfl_sync(kFull, ticket, 0);
  const int rows = a.B * a.nseg;
  if (ticket + 1 != static_cast<unsigned>(rows)) return;
  __threadfence();
  if (!cval) return;
  double sw = 0.0, su = 0.0;
  const float* base = a.partial + c;
  for (int r0 = 0; r0 < rows; r0 += 16) {
    float pw[16], pu[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const bool in = r0 + i < rows;
      pw[i] = in ? __ldcg(base + (size_t)(r0 + i) * 2 * a.C) : 0.f;
      pu[i] = in ? __ldcg(base + ((size_t)(r0 + i) * 2 + 1) * a.C) : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      sw += pw[i];
      su += pu[i];
    }
  }
  a.gtd[c] = static_cast<float>(static_cast<double>(lc.w) * static_cast<double>(lc.ew) * sw);
  a.gtf[c] = static_cast<float>(su);
}

// ------------------------------------------------------------------- carries

// In place over seg[B][nseg][3][C]: entry s holds the state a segment reaches
// from zero (its summary); on exit it holds the true state at the segment start.
__global__ void wkv_carry_fwd_kernel(float* seg, const float* decay, int decay_is_w, int B, int T,
                                     int C, int nseg, int seg_len) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)B * C) return;
  const int b = static_cast<int>(i / C), c = static_cast<int>(i % C);
  const float d = decay[c];
  const Lane lc = make_lane(decay_is_w ? d : -expf(d), 0.f);
  Fwd st = fwd_identity();
  for (int s = 0; s < nseg; ++s) {
    const size_t row = (size_t)b * nseg + s;
    Fwd sum = fwd_identity();
    if (s + 1 < nseg) sum = load_fwd(seg, row, C, c);
    store_fwd(seg, row, C, c, st);
    if (s + 1 < nseg) st = fwd_combine(st, min(seg_len, T - s * seg_len), lc, sum);
  }
}

// In place over adj[B][nseg][3][C]: entry s (s >= 1) holds the adjoint at the
// start of segment s accumulated from a zero adjoint at its end; on exit entry s
// holds the true adjoint at the end of segment s.
__global__ void wkv_carry_adj_kernel(float* adj, const float* w, int B, int T, int C, int nseg,
                                     int seg_len) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)B * C) return;
  const int b = static_cast<int>(i / C), c = static_cast<int>(i % C);
  const Lane lc = make_lane(w[c], 0.f);
  Adj a = adj_zero();
  for (int s = nseg - 1; s >= 0; --s) {
    const size_t row = (size_t)b * nseg + s;
    Adj local = adj_zero();
    if (s > 0) local = load_adj(adj, row, C, c);
    store_adj(adj, row, C, c, a);
    if (s > 0) a = adj_combine(local, a, min(seg_len, T - s * seg_len), lc);
  }
}

}  // namespace wkv
