// LIF sequence op for sm_100a: the spiking activation of SpikeGPT blocks,
// reference SpikingSequenceLIF (src/spikegpt/language.py:766-918).
//
// Per (b, c) over t, in the operation order of the reference's step
// (language.py:831-841), with the membrane carried in float32:
//   v = v * decay + x_t;  centered = slope * (v - threshold);
//   s_t = (centered >= 0);  v = s_t ? reset : v
// (decay = 1 - 1/tau; the reset form v*(1-s) + reset*s is exactly this select).
// Backward (gradient of that loop under autograd, with the spike's surrogate
// derivative slope * surrogate'(centered), surrogate'(x) = 1 / (2 (1 + (pi/2 x)^2))):
//   dL/dv_t = ds/dv (gs_t + g (reset - v_t)) + g (1 - s_t);  dL/dx_t = dL/dv_t;
//   g <- decay * dL/dv_t  (g = dL/d(membrane after step t), 0 after the last step).
//
// One warp per (64-channel block, batch row), two channels per lane; kSub-step
// tiles stream through a ring of shared-memory stages with TMA (or plain loads
// on the generic path); spikes / input gradients go out through staged tiles.
// The forward stores the membrane at every tile start ([B][ntiles][C] float32);
// the backward recomputes each tile's membranes from it, last tile first.
// Memory-bound: forward 2 * sizeof(T) bytes per element, backward 3 *.
#pragma once

#include "wkv_kernels.cuh"

namespace wkv {

struct LifArgs {
  const void* x;
  const void* gs;
  void* s;
  void* gx;
  float* state;  // [B][ntiles][C] membrane at each tile start (forward output, backward input)
  float decay, threshold, reset, slope;
  int B, T, C, ncblk, ntiles;
  unsigned* err;
};

// Stages of the input ring: 24 KB of the forward's x (12 bf16 tiles) and 32 KB
// of the backward's (x, grad) pairs in flight per warp whatever the dtype.
template <typename T>
__host__ __device__ constexpr int lif_fwd_stages() {
  return 24 / static_cast<int>(sizeof(T));
}
template <typename T>
__host__ __device__ constexpr int lif_bwd_stages() {
  return 16 / static_cast<int>(sizeof(T));
}
template <typename T>
constexpr size_t lif_fwd_smem_bytes() {
  return (size_t)(lif_fwd_stages<T>() + 2) * kSub * kLanes * sizeof(T) + 8 * lif_fwd_stages<T>();
}
template <typename T>
constexpr size_t lif_bwd_smem_bytes() {
  return (size_t)(2 * lif_bwd_stages<T>() + 2) * kSub * kLanes * sizeof(T) + 8 * lif_bwd_stages<T>();
}

__device__ __forceinline__ f2 lif_spike(f2 v, f2 thr, f2 slope) {
  const f2 cen = mul2(slope, sub2(v, thr));
  return f2{cen.x >= 0.f ? 1.f : 0.f, cen.y >= 0.f ? 1.f : 0.f};
}

template <typename T, bool kTma>
__global__ void __launch_bounds__(32) lif_fwd_kernel(const LifArgs a,
                                                     const __grid_constant__ CUtensorMap tx,
                                                     const __grid_constant__ CUtensorMap ts) {
  using P = Pair<T>;
  constexpr int S = lif_fwd_stages<T>();
  constexpr int R = kSub;
  constexpr int E = R * kLanes;
  extern __shared__ __align__(128) unsigned char smem[];
  T* xbuf = reinterpret_cast<T*>(smem);
  T* sbuf = xbuf + S * E;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sbuf + 2 * E);
  const int lane = threadIdx.x;
  const int cb = blockIdx.x % a.ncblk, b = blockIdx.x / a.ncblk;
  const int c = cb * kLanes + 2 * lane;
  const bool v0 = c < a.C, v1 = c + 1 < a.C;
  const f2 decay = splat(a.decay), thr = splat(a.threshold), slope = splat(a.slope);
  const int nt = a.ntiles;

  auto issue = [&](int j) {
    mbar_arrive_expect_tx_if(lane == 0, &bars[j % S], E * sizeof(T));
    tma_load_3d_if(lane == 0, xbuf + (j % S) * E, &tx, &bars[j % S], cb * kLanes, j * R, b);
  };
  if (kTma) {
    if (lane == 0) {
      for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
      fence_barrier_init();
      prefetch_tensormap(&tx);
      prefetch_tensormap(&ts);
    }
    __syncwarp();
    for (int j = 0; j < min(S, nt); ++j) issue(j);
  }
  f2 v = splat(0.f);
#pragma unroll 1
  for (int j = 0; j < nt; ++j) {
    const int t0 = j * R;
    const int rows = min(R, a.T - t0);
    T* xs = xbuf + (j % S) * E;
    if (kTma) {
      if (!__all_sync(kFull, mbar_wait_bounded(&bars[j % S], (j / S) & 1))) {
        if (lane == 0) {
          report_timeout(a.err);
          for (int q = j + 1; q < min(j + S, nt); ++q) mbar_wait_bounded(&bars[q % S], (q / S) & 1);
        }
        bulk_wait_all();
        return;
      }
    } else {
      fill_tile(xs, static_cast<const T*>(a.x), b, t0, rows, a.T, a.C, c, v0, v1, lane);
      __syncwarp();
    }
    if (a.state != nullptr && v1) {  // membrane entering the tile
      *reinterpret_cast<f2*>(a.state + ((size_t)b * nt + j) * a.C + c) = v;
    } else if (a.state != nullptr && v0) {
      a.state[((size_t)b * nt + j) * a.C + c] = v.x;
    }
    T* ss = sbuf + (j & 1) * E;
    if (kTma) {
      bulk_wait_read<1>();  // the store of tile j-2 has read ss
      __syncwarp();
    }
    const T* xr = xs + 2 * lane;
#pragma unroll
    for (int i = 0; i < R; ++i) {
      if (i < rows) {
        v = add2(mul2(v, decay), P::unpack(P::ld(xr + i * kLanes)));
        const f2 sp = lif_spike(v, thr, slope);
        v = f2{sp.x != 0.f ? a.reset : v.x, sp.y != 0.f ? a.reset : v.y};
        P::st(ss + 2 * lane + i * kLanes, P::pack(sp));
      }
    }
    if (kTma) {
      fence_proxy_async_smem();
      __syncwarp();
      tma_store_3d_if(lane == 0, &ts, ss, cb * kLanes, t0, b);
      bulk_commit();
      if (j + S < nt) issue(j + S);
    } else {
      __syncwarp();
      drain_tile(ss, static_cast<T*>(a.s), b, t0, rows, a.T, a.C, c, v0, v1, lane);
    }
  }
  if (kTma) bulk_wait_all();
}

template <typename T, bool kTma>
__global__ void __launch_bounds__(32) lif_bwd_kernel(const LifArgs a,
                                                     const __grid_constant__ CUtensorMap tx,
                                                     const __grid_constant__ CUtensorMap tgs,
                                                     const __grid_constant__ CUtensorMap tgx) {
  using P = Pair<T>;
  constexpr int S = lif_bwd_stages<T>();
  constexpr int R = kSub;
  constexpr int E = R * kLanes;
  extern __shared__ __align__(128) unsigned char smem[];
  T* xbuf = reinterpret_cast<T*>(smem);
  T* gbuf = xbuf + S * E;
  T* obuf = gbuf + S * E;
  uint64_t* bars = reinterpret_cast<uint64_t*>(obuf + 2 * E);
  const int lane = threadIdx.x;
  const int cb = blockIdx.x % a.ncblk, b = blockIdx.x / a.ncblk;
  const int c = cb * kLanes + 2 * lane;
  const bool v0 = c < a.C, v1 = c + 1 < a.C;
  const f2 decay = splat(a.decay), thr = splat(a.threshold), slope = splat(a.slope);
  const f2 reset = splat(a.reset), half_pi = splat(1.5707963267948966f), half = splat(0.5f);
  const int nt = a.ntiles;

  // the jj-th visited tile is j = nt - 1 - jj
  auto issue = [&](int jj) {
    const int s = jj % S, t0 = (nt - 1 - jj) * R;
    mbar_arrive_expect_tx_if(lane == 0, &bars[s], 2 * E * sizeof(T));
    tma_load_3d_if(lane == 0, xbuf + s * E, &tx, &bars[s], cb * kLanes, t0, b);
    tma_load_3d_if(lane == 0, gbuf + s * E, &tgs, &bars[s], cb * kLanes, t0, b);
  };
  if (kTma) {
    if (lane == 0) {
      for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
      fence_barrier_init();
      prefetch_tensormap(&tx);
      prefetch_tensormap(&tgs);
      prefetch_tensormap(&tgx);
    }
    __syncwarp();
    for (int jj = 0; jj < min(S, nt); ++jj) issue(jj);
  }
  auto load_state = [&](int j) -> f2 {
    f2 r = splat(0.f);
    const float* p = a.state + ((size_t)b * nt + j) * a.C + c;
    if (v1) r = *reinterpret_cast<const f2*>(p);
    else if (v0) r.x = *p;
    return r;
  };
  f2 g = splat(0.f);  // dL/d(membrane after the current step), from later steps
  f2 vin_next = nt > 0 ? load_state(nt - 1) : splat(0.f);
#pragma unroll 1
  for (int jj = 0; jj < nt; ++jj) {
    const int j = nt - 1 - jj;
    const int s = jj % S;
    const int t0 = j * R;
    const int rows = min(R, a.T - t0);
    const f2 vin = vin_next;
    if (j > 0) vin_next = load_state(j - 1);
    T* xs = xbuf + s * E;
    T* gss = gbuf + s * E;
    if (kTma) {
      if (!__all_sync(kFull, mbar_wait_bounded(&bars[s], (jj / S) & 1))) {
        if (lane == 0) {
          report_timeout(a.err);
          for (int q = jj + 1; q < min(jj + S, nt); ++q) mbar_wait_bounded(&bars[q % S], (q / S) & 1);
        }
        bulk_wait_all();
        return;
      }
    } else {
      fill_tile(xs, static_cast<const T*>(a.x), b, t0, rows, a.T, a.C, c, v0, v1, lane);
      fill_tile(gss, static_cast<const T*>(a.gs), b, t0, rows, a.T, a.C, c, v0, v1, lane);
      __syncwarp();
    }
    // recompute the tile's membranes (before reset) from the state entering it
    f2 vp[R];
    {
      f2 v = vin;
#pragma unroll
      for (int i = 0; i < R; ++i) {
        if (i < rows) {
          v = add2(mul2(v, decay), P::unpack(P::ld(xs + 2 * lane + i * kLanes)));
          vp[i] = v;
          const f2 sp = lif_spike(v, thr, slope);
          v = f2{sp.x != 0.f ? a.reset : v.x, sp.y != 0.f ? a.reset : v.y};
        } else {
          vp[i] = splat(0.f);
        }
      }
    }
    T* os = obuf + (jj & 1) * E;
    if (kTma) {
      bulk_wait_read<1>();  // the store of tile jj-2 has read os
      __syncwarp();
    }
#pragma unroll
    for (int i = R - 1; i >= 0; --i) {
      if (i < rows) {
        const f2 cen = mul2(slope, sub2(vp[i], thr));
        const f2 sp = f2{cen.x >= 0.f ? 1.f : 0.f, cen.y >= 0.f ? 1.f : 0.f};
        const f2 h = mul2(half_pi, cen);
        const f2 dsdv = mul2(slope, mul2(half, rcpx2(fma2(h, h, splat(1.f)))));
        const f2 gsi = P::unpack(P::ld(gss + 2 * lane + i * kLanes));
        const f2 gv = fma2(dsdv, fma2(g, sub2(reset, vp[i]), gsi), mul2(g, sub2(splat(1.f), sp)));
        P::st(os + 2 * lane + i * kLanes, P::pack(gv));
        g = mul2(decay, gv);
      }
    }
    if (kTma) {
      fence_proxy_async_smem();
      __syncwarp();
      tma_store_3d_if(lane == 0, &tgx, os, cb * kLanes, t0, b);
      bulk_commit();
      if (jj + S < nt) issue(jj + S);
    } else {
      __syncwarp();
      drain_tile(os, static_cast<T*>(a.gx), b, t0, rows, a.T, a.C, c, v0, v1, lane);
    }
  }
  if (kTma) bulk_wait_all();
}

}  // namespace wkv
