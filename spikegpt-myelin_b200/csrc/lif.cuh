// LIF sequence op for sm_100a: the spiking activation of SpikeGPT blocks,
// reference SpikingSequenceLIF (src/spikegpt/language.py:766-918).
//
// Per (b, c) over t, in the operation order of the reference's step
// (language.py:831-841), with the membrane carried in float32:
//   v = v * decay + x_t;  centered = slope * (v - threshold);
//   s_t = (centered >= 0);  v = v * (1 - s_t) + reset * s_t
// (decay = 1 - 1/tau).
// Backward (gradient of that loop under autograd, with the spike's surrogate
// derivative slope * surrogate'(centered), surrogate'(x) = 1 / (2 (1 + (pi/2 x)^2))):
//   dL/dv_t = ds/dv (gs_t + g (reset - v_t)) + g (1 - s_t);  dL/dx_t = dL/dv_t;
//   g <- decay * dL/dv_t  (g = dL/d(membrane after step t), 0 after the last step).
//
// One warp per (64-channel block, batch row), two channels per lane, kLifWarps
// independent warps per CTA (no CTA-wide synchronization). A warp alone on its
// scheduler issues every instruction of its T steps, and most of them (packed
// f32x2 arithmetic, compares, selects, logic) issue at one per two cycles, so
// the step is written for the fewest instructions: the spike test, the two
// reset branches and the selects in one block that keeps the predicates in
// predicate registers, the branches' products with decay folded into single
// fmas, spikes / gradients staged in shared memory with immediate offsets and
// written by one TMA store per 8 KB tile, and every per-tile cost (barrier
// wait, TMA issue) paid once per lif_rows<T>() steps; the backward's copies
// are issued by a producer warp (lif_bwd_ws_kernel). Sub-tiles of kSub steps
// are the unit of computation and of the checkpoints the forward stores (the
// membrane entering each sub-tile times decay, [B][ceil(T/kSub)][C] float32)
// and the backward recomputes from, last sub-tile first. The generic path (unaligned tensors) stages kSub-row tiles
// with plain loads and stores. With few sequences the forward instead splits
// T into segments run at once and repaired where their speculated starts were
// wrong (lif_fwd_seg_kernel, below), and the backward splits T into segments
// joined by affine adjoint maps. Memory-bound target: forward 2 * sizeof(T)
// bytes per element, backward 3 *.
#pragma once

#include <type_traits>

#include "wkv_kernels.cuh"

namespace wkv {

struct LifArgs {
  const void* x;
  const void* gs;
  void* s;
  void* gx;
  float* state;  // [B][ntiles][C] membrane entering each kSub-step sub-tile times decay (forward output)
  float decay, threshold, reset, slope;
  int B, T, C, ncblk, ntiles;
  unsigned* err;
  // Time-segmented backward (TMA path, few sequences): nseg segments of
  // seg_tiles staged tiles each (nseg 1: one segment, seg_sum unused), and
  // the affine map g_start = A * g_end + B of the adjoint over each segment,
  // [B][nseg][2][C] (A, then B).
  int nseg, seg_tiles;
  float* seg_sum;
};

// Rows of a TMA-staged tile: 8 KB of 64 channels (64 bf16/fp16 rows, 32 fp32 rows).
template <typename T>
__host__ __device__ constexpr int lif_rows() {
  return 8192 / (kLanes * static_cast<int>(sizeof(T)));
}
constexpr int kLifTileBytes = 8192;
constexpr int kLifFwdStages = 4;  // x tiles in flight per warp (forward)
constexpr int kLifOut = 2;        // staged output tiles per warp (forward)
// Independent warps per CTA: one warp lands on each of an SM's 4 schedulers.
constexpr int kLifWarps = 4;
__host__ __device__ constexpr size_t lif_align128(size_t n) { return (n + 127) / 128 * 128; }
// Shared memory of one warp (the CTA holds kLifWarps of these): the stage
// ring, the staged output tiles, the stage barriers. The generic path's
// kSub-row stages fit in the same space.
__host__ __device__ constexpr size_t lif_fwd_smem_bytes() {
  return lif_align128((size_t)(kLifFwdStages + kLifOut) * kLifTileBytes + 8 * kLifFwdStages);
}
// Generic-path backward: two kSub-row stages of x, grad and the checkpoint,
// and one staged gradient tile, per warp.
template <typename T>
__host__ __device__ constexpr size_t lif_bwd_smem_bytes() {
  return lif_align128((size_t)2 * (2 * kSub * kLanes * sizeof(T) + kLanes * sizeof(float)) +
                      (size_t)kSub * kLanes * sizeof(T));
}
static_assert(lif_rows<float>() % kSub == 0 && lif_rows<__nv_bfloat16>() % kSub == 0, "sub-tiles");
static_assert(kLifWarps * lif_bwd_smem_bytes<float>() <= 227 * 1024, "generic LIF backward shared memory");
static_assert(3 * kSub * kLanes * sizeof(float) + 8 <= lif_fwd_smem_bytes(), "generic forward staging");
static_assert(kLifWarps * lif_fwd_smem_bytes() <= 227 * 1024, "LIF forward shared memory");

// Per-lane constants of the step for a pair of channels.
struct LifK {
  f2 decay, thr, slope, reset;
  f2 reset0;  // reset * 0: what the non-spiking branch adds (zero unless reset is not finite)
  f2 rd;      // reset * decay
  f2 rz;      // reset0 * decay
  f2 half_slope, half_pi, hq, cq, zero, one;
};

__device__ __forceinline__ LifK lif_constants(const LifArgs& a) {
  LifK k;
  k.decay = splat(a.decay);
  k.thr = splat(a.threshold);
  k.slope = splat(a.slope);
  k.reset = splat(a.reset);
  k.reset0 = splat(__fmul_rn(a.reset, 0.f));
  k.rd = splat(__fmul_rn(a.reset, a.decay));
  k.rz = splat(__fmul_rn(__fmul_rn(a.reset, 0.f), a.decay));
  k.half_slope = splat(__fmul_rn(a.slope, 0.5f));
  k.half_pi = splat(1.5707963267948966f);
  k.hq = splat(1.5707963267948966f * a.slope * rsqrtf(0.5f * a.slope));  // plain test only (slope >= 1)
  k.cq = splat(2.f / a.slope);
  k.zero = splat(0.f);
  k.one = splat(1.f);
  return k;
}

// Spike words of a lane's pair: a 16-bit type's one in each half, or two
// float ones.
template <typename T>
struct LifOnes {
  static constexpr uint32_t lo = 0x3f80u, hi = 0x3f800000u;  // bf16
};
template <>
struct LifOnes<__half> {
  static constexpr uint32_t lo = 0x3c00u, hi = 0x3c000000u;
};
template <>
struct LifOnes<float> {
  static constexpr uint32_t lo = 0x3f800000u, hi = 0x3f800000u;
};

// The spike test on vn (%2, %3) leaves predicates p0, p1. Exact form:
// centered = slope * (vn - threshold) >= 0. Plain form, vn >= threshold: the
// same predicate whenever slope >= 1 is finite and threshold is finite (then
// vn - threshold rounds to zero only when vn == threshold, to the sign of the
// exact difference otherwise, and slope * d neither flushes a nonzero d to
// zero nor flips its sign, with NaNs comparing false in both).
#define LIF_TEST_EXACT                                 \
  "mov.b64 rk, {%8, %8};\n\t"                          \
  "sub.rn.f32x2 ra, rv, rk;\n\t"                       \
  "mov.b64 rk, {%9, %9};\n\t"                          \
  "mul.rn.f32x2 ra, rk, ra;\n\t"                       \
  "mov.b64 {c0, c1}, ra;\n\t"                          \
  "setp.ge.f32 p0, c0, 0f00000000;\n\t"                \
  "setp.ge.f32 p1, c1, 0f00000000;\n\t"
#define LIF_TEST_PLAIN      \
  "setp.ge.f32 p0, %2, %8;\n\t" \
  "setp.ge.f32 p1, %3, %8;\n\t"
// vn = m + x; spike test; next m = p ? vn * 0 + reset * decay : vn * decay + reset0 * decay
// (the reference's branches times decay, each one fma: vn * 0 is exact, and
// reset0 * decay is zero unless reset is not finite).
#define LIF_STEP_BODY(TEST)                                                         \
  "{\n\t.reg .pred p0, p1;\n\t.reg .b64 rm, rx, rv, ra, rb, rk;\n\t"                  \
  ".reg .f32 a0, a1, b0, b1, c0, c1;\n\t"                                           \
  "mov.b64 rm, {%0, %1};\n\tmov.b64 rx, {%6, %7};\n\t"                              \
  "add.rn.f32x2 rv, rm, rx;\n\tmov.b64 {%2, %3}, rv;\n\t" TEST                        \
  "mov.b64 rk, {%10, %11};\n\tmov.b64 ra, 0;\n\tfma.rn.f32x2 ra, rv, ra, rk;\n\t"  \
  "mov.b64 rk, {%12, %13};\n\tmov.b64 rb, {%14, %15};\n\tfma.rn.f32x2 rb, rv, rk, rb;\n\t" \
  "mov.b64 {a0, a1}, ra;\n\tmov.b64 {b0, b1}, rb;\n\t"                              \
  "selp.f32 %0, a0, b0, p0;\n\tselp.f32 %1, a1, b1, p1;\n\t"
#define LIF_SPIKES_16 "selp.b32 %4, %16, 0, p0;\n\t@p1 or.b32 %4, %4, %17;\n\tmov.b32 %5, 0;\n\t}"
#define LIF_SPIKES_32 "selp.b32 %4, %16, 0, p0;\n\tselp.b32 %5, %17, 0, p1;\n\t}"
#define LIF_STEP_OPERANDS(m, vn, w0, w1, x, k, T)                                             \
  : "+f"(m.x), "+f"(m.y), "=f"(vn.x), "=f"(vn.y), "=r"(w0), "=r"(w1)                             \
  : "f"(x.x), "f"(x.y), "f"(k.thr.x), "f"(k.slope.x), "f"(k.rd.x), "f"(k.rd.y), "f"(k.decay.x), \
    "f"(k.decay.y), "f"(k.rz.x), "f"(k.rz.y), "n"(LifOnes<T>::lo), "n"(LifOnes<T>::hi)

// One step for a lane's pair of channels: m = membrane * decay from the step
// before (updated), vn = membrane before reset, w0 / w1 = spike words
// (LifOnes<T>).
template <typename T, bool kPlain>
__device__ __forceinline__ void lif_step(f2& m, f2 x, const LifK& k, f2& vn, uint32_t& w0, uint32_t& w1) {
  if constexpr (sizeof(T) == 2 && kPlain) {
    asm(LIF_STEP_BODY(LIF_TEST_PLAIN) LIF_SPIKES_16 LIF_STEP_OPERANDS(m, vn, w0, w1, x, k, T));
  } else if constexpr (sizeof(T) == 2) {
    asm(LIF_STEP_BODY(LIF_TEST_EXACT) LIF_SPIKES_16 LIF_STEP_OPERANDS(m, vn, w0, w1, x, k, T));
  } else if constexpr (kPlain) {
    asm(LIF_STEP_BODY(LIF_TEST_PLAIN) LIF_SPIKES_32 LIF_STEP_OPERANDS(m, vn, w0, w1, x, k, T));
  } else {
    asm(LIF_STEP_BODY(LIF_TEST_EXACT) LIF_SPIKES_32 LIF_STEP_OPERANDS(m, vn, w0, w1, x, k, T));
  }
}

// One sub-tile of the forward: rows steps (kSub when kWhole) from m = the
// membrane entering it times decay; x from a staged tile and spikes to a
// staged tile (row stride kLanes, lane offset applied). Returns m for the
// step after the sub-tile.
template <bool kWhole, bool kPlain, typename T, int RS = kLanes>
__device__ __forceinline__ f2 lif_fwd_tile(f2 m, const T* xr, T* out, int rows, const LifK& k) {
  using P = Pair<T>;
  typename P::raw xin[kSub];
#pragma unroll
  for (int i = 0; i < kSub; ++i)
    if (kWhole || i < rows) xin[i] = P::ld(xr + i * RS);
#pragma unroll
  for (int i = 0; i < kSub; ++i) {
    if (kWhole || i < rows) {
      uint32_t w0, w1;
      f2 vn;
      lif_step<T, kPlain>(m, P::unpack(xin[i]), k, vn, w0, w1);
      if constexpr (sizeof(T) == 2) {
        *reinterpret_cast<uint32_t*>(out + i * RS) = w0;
      } else {
        *reinterpret_cast<uint2*>(out + i * RS) = make_uint2(w0, w1);
      }
    }
  }
  return m;
}

// The membranes before reset (vp) of one sub-tile, recomputed from its
// checkpoint m (the membrane entering it times decay).
template <bool kWhole, bool kPlain, typename T, int RS = kLanes>
__device__ __forceinline__ void lif_recompute(f2 m, const T* xr, int rows, const LifK& k, f2 (&vp)[kSub]) {
  using P = Pair<T>;
  typename P::raw xin[kSub];
#pragma unroll
  for (int i = 0; i < kSub; ++i)
    if (kWhole || i < rows) xin[i] = P::ld(xr + i * RS);
#pragma unroll
  for (int i = 0; i < kSub; ++i) {
    if (kWhole || i < rows) {
      uint32_t w0, w1;
      lif_step<T, kPlain>(m, P::unpack(xin[i]), k, vp[i], w0, w1);
    } else {
      vp[i] = k.zero;
    }
  }
}

// The adjoint sweep of one sub-tile, last step first. g = dL/d(membrane after
// the sub-tile's last step); per step
//   dL/dvn = dsdv * (gs + g * (reset - vn)) + g * (1 - s);  dL/dx = dL/dvn;  g <- decay * dL/dvn
// with dsdv = slope * 0.5 / (1 + (pi/2 * centered)^2) (the arc-tangent
// surrogate's derivative; slope * (0.5 * r) == (slope * 0.5) * r exactly) and
// g * (1 - s) as g * 0 or g. With the plain spike test (see lif_step) the
// spike is d = vn - threshold >= 0 and dsdv is formed as 1 / (h'^2 + 2/slope)
// with h' = (pi/2 * slope / sqrt(slope/2)) * d: the same quantity, to a few
// roundings, with one multiply fewer (slope >= 1 there). Input gradients go to a staged tile (row stride kLanes,
// lane offset applied). Returns g entering the sub-tile.
template <bool kWhole, bool kPlain, typename T, int RS = kLanes>
__device__ __forceinline__ f2 lif_grad_tile(f2 g, const f2 (&vp)[kSub], const T* gr, T* out, int rows,
                                            const LifK& k) {
  using P = Pair<T>;
  typename P::raw gin[kSub];
#pragma unroll
  for (int i = 0; i < kSub; ++i)
    if (kWhole || i < rows) gin[i] = P::ld(gr + i * RS);
#pragma unroll
  for (int i = kSub - 1; i >= 0; --i) {
    if (kWhole || i < rows) {
      const f2 d = sub2(vp[i], k.thr);
      const f2 cen = kPlain ? d : mul2(k.slope, d);  // carries the spike test's sign
      f2 dsdv;
      if constexpr (kPlain) {  // slope / 2 / (1 + h^2) = 1 / (h'^2 + 2 / slope), h' = h / sqrt(slope / 2)
        const f2 h = mul2(k.hq, d);
        dsdv = rcpx2(fma2(h, h, k.cq));
      } else {
        const f2 h = mul2(k.half_pi, cen);
        dsdv = mul2(k.half_slope, rcpx2(fma2(h, h, k.one)));
      }
      const f2 g0 = mul2(g, k.zero);
      const f2 gk = f2{cen.x >= 0.f ? g0.x : g.x, cen.y >= 0.f ? g0.y : g.y};
      const f2 gv = fma2(dsdv, fma2(g, sub2(k.reset, vp[i]), P::unpack(gin[i])), gk);
      P::st(out + i * RS, P::pack(gv));
      g = mul2(k.decay, gv);
    }
  }
  return g;
}

template <typename T, bool kTma, bool kPlain>
__global__ void __launch_bounds__(32 * kLifWarps, 1) lif_fwd_kernel(const LifArgs a,
                                                                 const __grid_constant__ CUtensorMap tx,
                                                                 const __grid_constant__ CUtensorMap ts) {
  constexpr int S = kTma ? kLifFwdStages : 1;
  constexpr int RT = kTma ? lif_rows<T>() : kSub;  // rows per staged tile
  constexpr int E = RT * kLanes;
  extern __shared__ __align__(128) unsigned char smem[];
  const int unit = blockIdx.x * kLifWarps + threadIdx.x / 32;  // (channel block, batch row)
  if (unit >= a.ncblk * a.B) return;
  T* xbuf = reinterpret_cast<T*>(smem + (threadIdx.x / 32) * lif_fwd_smem_bytes());
  T* obuf = xbuf + S * E;
  uint64_t* bars = reinterpret_cast<uint64_t*>(obuf + kLifOut * E);
  const int lane = threadIdx.x % 32;
  const int cb = unit % a.ncblk, b = unit / a.ncblk;
  const int c = cb * kLanes + 2 * lane;
  const bool v0 = c < a.C, v1 = c + 1 < a.C;
  const LifK k = lif_constants(a);
  const int ntt = (a.T + RT - 1) / RT;
  // checkpoints: the membrane entering each sub-tile times decay, the first
  // operand of its first step
  float* state = a.state == nullptr ? nullptr : a.state + (size_t)b * a.ntiles * a.C + c;

  auto issue = [&](int j) {
    mbar_arrive_expect_tx_if(lane == 0, &bars[j % S], E * sizeof(T));
    tma_load_3d_if(lane == 0, xbuf + (j % S) * E, &tx, &bars[j % S], cb * kLanes, j * RT, b);
  };
  auto checkpoint = [&](int u0, f2 v) {  // for the sub-tile starting at step u0
    if (state == nullptr) return;
    float* st = state + (size_t)(u0 / kSub) * a.C;
    if (v1) *reinterpret_cast<f2*>(st) = v;
    else if (v0) *st = v.x;
  };
  if (kTma) {
    if (lane == 0) {
      for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
      fence_barrier_init();
      prefetch_tensormap(&tx);
      prefetch_tensormap(&ts);
    }
    __syncwarp();
    for (int j = 0; j < min(S, ntt); ++j) issue(j);
  }
  f2 m = k.zero;  // the initial membrane (zero) times decay
#pragma unroll 1
  for (int j = 0; j < ntt; ++j) {
    const int t0 = j * RT;
    const T* xs = xbuf + (j % S) * E + 2 * lane;
    T* os = obuf + (j % kLifOut) * E;
    if (kTma) {
      if (!__all_sync(kFull, mbar_wait_bounded(&bars[j % S], (j / S) & 1))) {
        if (lane == 0) {
          report_timeout(a.err);
          for (int q = j + 1; q < min(j + S, ntt); ++q) mbar_wait_bounded(&bars[q % S], (q / S) & 1);
        }
        bulk_wait_all();
        return;
      }
      bulk_wait_read<kLifOut - 1>();  // the store of tile j - kLifOut has read os
      __syncwarp();
    } else {
      fill_tile(xbuf, static_cast<const T*>(a.x), b, t0, min(RT, a.T - t0), a.T, a.C, c, v0, v1, lane);
      __syncwarp();
    }
    if (t0 + RT <= a.T) {  // whole sub-tiles only
#pragma unroll 1
      for (int q = 0; q < RT / kSub; ++q) {
        checkpoint(t0 + q * kSub, m);
        m = lif_fwd_tile<true, kPlain>(m, xs + q * kSub * kLanes, os + q * kSub * kLanes + 2 * lane, kSub, k);
      }
    } else {
#pragma unroll 1
      for (int q = 0; q < RT / kSub; ++q) {
        const int u0 = t0 + q * kSub;
        if (u0 >= a.T) break;
        const int rows = min(kSub, a.T - u0);
        checkpoint(u0, m);
        m = rows == kSub
                ? lif_fwd_tile<true, kPlain>(m, xs + q * kSub * kLanes, os + q * kSub * kLanes + 2 * lane, kSub, k)
                : lif_fwd_tile<false, kPlain>(m, xs + q * kSub * kLanes, os + q * kSub * kLanes + 2 * lane, rows, k);
      }
    }
    if (kTma) {
      fence_proxy_async_smem();
      __syncwarp();  // every lane has read stage j % S and written os
      tma_store_3d_if(lane == 0, &ts, os, cb * kLanes, t0, b);
      bulk_commit();
      if (j + S < ntt) issue(j + S);
    } else {
      __syncwarp();
      drain_tile(os, static_cast<T*>(a.s), b, t0, min(RT, a.T - t0), a.T, a.C, c, v0, v1, lane);
      __syncwarp();
    }
  }
  if (kTma) bulk_wait_all();
}

// ------------------------------------------------ time-segmented forward
//
// With few sequences the forward above leaves most SMs idle: one warp per
// (64-channel block, batch row) and a serial chain of T steps, so the launch
// takes T steps of one warp's arithmetic whatever the batch. The segmented
// forward gives a CTA of nseg warps one (block, row); warp j takes the
// sub-tiles [j ls, (j+1) ls) (ls sub-tiles of kSub steps, the last segment
// shorter) and the result is the sequential forward's, bit for bit, whatever
// the input:
//  A. every warp runs its segment from the membrane 0 (warp 0 from the true
//     start, which is 0), writing spikes and checkpoints, and leaves its end
//     membrane in shared memory;
//  B. warp j >= 1 reruns its segment from the end membrane of segment j-1,
//     writing nothing, until each channel's membrane at a sub-tile boundary
//     equals, bit for bit, the checkpoint pass A left there. From that
//     boundary on the two runs are the same computation: a spike sets the
//     membrane to the constant reset * decay, and with decay < 1 a difference
//     that no spike removes shrinks below the rounding within a few dozen
//     steps;
//  V. warp 0 walks the segments in order, per channel: where the start pass
//     B used is the true end of the previous segment, pass B's convergence
//     point and end hold; where it is not (the previous segment never
//     converged), it reruns the segment from the true start itself;
//  C. warp j >= 1 reruns its segment from the true start up to the last
//     boundary at which a channel of its block had not converged, rewriting
//     those sub-tiles' spikes and checkpoints (converged channels write the
//     values pass A wrote).
// Needs the checkpoints (state != null), whole sub-tiles (T % kSub == 0) and
// whole 64-channel blocks (C % 64 == 0, 4-byte aligned pairs).
constexpr int kLifSegMax = 8;

template <typename T>
__device__ __forceinline__ void lif_seg_load(typename Pair<T>::raw (&xin)[kSub], const T* xg, size_t ld) {
#pragma unroll
  for (int i = 0; i < kSub; ++i) xin[i] = Pair<T>::ld(xg + i * ld);
}

// kSub steps from m (the membrane entering them times decay); spikes to sg
// (row stride ld) when kWrite. Returns m after the sub-tile.
template <bool kWrite, bool kPlain, typename T>
__device__ __forceinline__ f2 lif_seg_run(f2 m, const typename Pair<T>::raw (&xin)[kSub], T* sg, size_t ld,
                                          const LifK& k) {
#pragma unroll
  for (int i = 0; i < kSub; ++i) {
    uint32_t w0, w1;
    f2 vn;
    lif_step<T, kPlain>(m, Pair<T>::unpack(xin[i]), k, vn, w0, w1);
    if constexpr (kWrite) {
      if constexpr (sizeof(T) == 2) *reinterpret_cast<uint32_t*>(sg + i * ld) = w0;
      else *reinterpret_cast<uint2*>(sg + i * ld) = make_uint2(w0, w1);
    }
  }
  return m;
}

__device__ __forceinline__ bool lif_same(float a, float b) { return __float_as_uint(a) == __float_as_uint(b); }

template <typename T, bool kPlain>
__global__ void __launch_bounds__(32 * kLifSegMax) lif_fwd_seg_kernel(const LifArgs a, int nseg, int ls) {
  using raw = typename Pair<T>::raw;
  __shared__ f2 s_end[kLifSegMax][32];     // pass A: end membrane (times decay) per segment and lane
  __shared__ f2 s_endb[kLifSegMax][32];    // pass B: end membrane
  __shared__ int2 s_conv[kLifSegMax][32];  // pass B, then V: sub-tiles to recompute per channel
  __shared__ f2 s_start[kLifSegMax][32];   // V: true start membrane
  const int w = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int cb = blockIdx.x % a.ncblk, b = blockIdx.x / a.ncblk;
  const int c = cb * kLanes + 2 * lane;
  const LifK k = lif_constants(a);
  const size_t ld = (size_t)a.C;
  const int ntiles = a.T / kSub;
  const T* xrow = static_cast<const T*>(a.x) + (size_t)b * a.T * ld + c;
  T* srow = static_cast<T*>(a.s) + (size_t)b * a.T * ld + c;
  float* state = a.state + (size_t)b * a.ntiles * ld + c;
  auto seg_begin = [&](int j) { return min(ntiles, j * ls); };
  auto ckpt = [&](int q) { return reinterpret_cast<f2*>(state + (size_t)q * ld); };

  // Runs sub-tiles [q0, q1) from m with the next sub-tile's loads in flight;
  // kWrite: checkpoints and spikes written.
  auto sweep = [&](auto write_tag, f2 m, int q0, int q1) {
    constexpr bool kWrite = decltype(write_tag)::value;
    raw cur[kSub], nxt[kSub];
    if (q0 < q1) lif_seg_load<T>(cur, xrow + (size_t)q0 * kSub * ld, ld);
#pragma unroll 1
    for (int q = q0; q < q1; ++q) {
      if (q + 1 < q1) lif_seg_load<T>(nxt, xrow + (size_t)(q + 1) * kSub * ld, ld);
      if constexpr (kWrite) *ckpt(q) = m;
      m = lif_seg_run<kWrite, kPlain, T>(m, cur, srow + (size_t)q * kSub * ld, ld, k);
#pragma unroll
      for (int i = 0; i < kSub; ++i) cur[i] = nxt[i];
    }
    return m;
  };
  using WriteOn = std::integral_constant<bool, true>;

  // Reruns segment j from m0 without writing, comparing each boundary with
  // pass A's membrane there; returns the end membrane and, per channel, the
  // sub-tiles before the first agreeing boundary (the segment's length when
  // none agrees). Every lane runs until its own channels agree.
  auto converge = [&](int j, f2 m0, int2& conv) {
    const int q0 = seg_begin(j), q1 = seg_begin(j + 1), n = q1 - q0;
    const f2 g = *ckpt(q0);  // pass A's start (the guess)
    conv = make_int2(lif_same(m0.x, g.x) ? 0 : n, lif_same(m0.y, g.y) ? 0 : n);
    f2 m = m0;
    raw cur[kSub], nxt[kSub];
    if (n > 0) lif_seg_load<T>(cur, xrow + (size_t)q0 * kSub * ld, ld);
#pragma unroll 1
    for (int i = 0; i < n && (conv.x == n || conv.y == n); ++i) {
      const int q = q0 + i;
      if (i + 1 < n) lif_seg_load<T>(nxt, xrow + (size_t)(q + 1) * kSub * ld, ld);
      const f2 ref = i + 1 < n ? *ckpt(q + 1) : s_end[j][lane];
      m = lif_seg_run<false, kPlain, T>(m, cur, nullptr, ld, k);
      if (conv.x == n && lif_same(m.x, ref.x)) conv.x = i + 1;
      if (conv.y == n && lif_same(m.y, ref.y)) conv.y = i + 1;
#pragma unroll
      for (int r = 0; r < kSub; ++r) cur[r] = nxt[r];
    }
    // a converged channel ends where pass A ended
    const f2 ea = s_end[j][lane];
    return f2{conv.x < n ? ea.x : m.x, conv.y < n ? ea.y : m.y};
  };

  // A
  if (w < nseg) {
    const f2 m = sweep(WriteOn{}, k.zero, seg_begin(w), seg_begin(w + 1));
    s_end[w][lane] = m;
  }
  __syncthreads();
  // B
  if (w >= 1 && w < nseg) {
    int2 conv;
    s_endb[w][lane] = converge(w, s_end[w - 1][lane], conv);
    s_conv[w][lane] = conv;
  }
  __syncthreads();
  // V
  if (w == 0) {
    f2 te = s_end[0][lane];  // the true end of segment 0
#pragma unroll 1
    for (int j = 1; j < nseg; ++j) {
      const f2 used = s_end[j - 1][lane];
      s_start[j][lane] = te;
      int2 conv = s_conv[j][lane];
      f2 e = s_endb[j][lane];
      if (!lif_same(used.x, te.x) || !lif_same(used.y, te.y)) {  // rerun from the true start
        int2 c2;
        const f2 e2 = converge(j, te, c2);
        if (!lif_same(used.x, te.x)) {
          conv.x = c2.x;
          e.x = e2.x;
        }
        if (!lif_same(used.y, te.y)) {
          conv.y = c2.y;
          e.y = e2.y;
        }
        s_conv[j][lane] = conv;
      }
      te = e;
    }
  }
  __syncthreads();
  // C
  if (w >= 1 && w < nseg) {
    const int2 conv = s_conv[w][lane];
    const int n = __reduce_max_sync(kFull, max(conv.x, conv.y));
    const int q0 = seg_begin(w);
    sweep(WriteOn{}, s_start[w][lane], q0, q0 + n);
  }
}

// Backward on the generic path (unaligned tensors), last sub-tile first,
// software-pipelined by one sub-tile: while the adjoint sweep of sub-tile q
// runs, the membranes of sub-tile q - 1 are recomputed from its checkpoint,
// two independent dependency chains in one straight-line block. Each
// kSub-row sub-tile is staged with plain loads (x, grad, checkpoint) into one
// of two stages and its input gradients leave through a staged tile.
template <typename T, bool kPlain>
__global__ void __launch_bounds__(32 * kLifWarps, 1) lif_bwd_kernel(const LifArgs a) {
  constexpr int E = kSub * kLanes;
  constexpr int SE = 2 * E * sizeof(T) + kLanes * sizeof(float);  // stage bytes
  extern __shared__ __align__(128) unsigned char smem[];
  const int unit = blockIdx.x * kLifWarps + threadIdx.x / 32;  // (channel block, batch row)
  if (unit >= a.ncblk * a.B) return;
  unsigned char* base = smem + (threadIdx.x / 32) * lif_bwd_smem_bytes<T>();
  T* obuf = reinterpret_cast<T*>(base + 2 * SE);
  const int lane = threadIdx.x % 32;
  const int cb = unit % a.ncblk, b = unit / a.ncblk;
  const int c = cb * kLanes + 2 * lane;
  const bool v0 = c < a.C, v1 = c + 1 < a.C;
  const LifK k = lif_constants(a);
  const int nq = a.ntiles;

  auto xs_of = [&](int q) { return reinterpret_cast<T*>(base + (q & 1) * SE); };
  auto gs_of = [&](int q) { return xs_of(q) + E; };
  auto st_of = [&](int q) { return reinterpret_cast<float*>(xs_of(q) + 2 * E); };
  auto stage = [&](int q) {  // sub-tile q into stage q & 1
    const int t0 = q * kSub, rows = min(kSub, a.T - t0);
    fill_tile(xs_of(q), static_cast<const T*>(a.x), b, t0, rows, a.T, a.C, c, v0, v1, lane);
    fill_tile(gs_of(q), static_cast<const T*>(a.gs), b, t0, rows, a.T, a.C, c, v0, v1, lane);
    const float* st = a.state + ((size_t)b * nq + q) * a.C + c;
    st_of(q)[2 * lane] = v0 ? st[0] : 0.f;
    st_of(q)[2 * lane + 1] = v1 ? st[1] : 0.f;
    __syncwarp();
  };
  auto v_sub = [&](int q) -> f2 { return *reinterpret_cast<const f2*>(st_of(q) + 2 * lane); };
  if (nq == 0) return;
  const int last_rows = a.T - (nq - 1) * kSub;
  f2 va[kSub], vb[kSub];
  stage(nq - 1);
  if (last_rows == kSub) lif_recompute<true, kPlain>(v_sub(nq - 1), xs_of(nq - 1) + 2 * lane, kSub, k, va);
  else lif_recompute<false, kPlain>(v_sub(nq - 1), xs_of(nq - 1) + 2 * lane, last_rows, k, va);
  f2 g = k.zero;  // dL/d(membrane after the current step), from later steps
  // sub-tile q: its membranes are in cur; those of q - 1 are recomputed into nxt
  auto body = [&](int q, const f2(&cur)[kSub], f2(&nxt)[kSub]) {
    const int rows = min(kSub, a.T - q * kSub);
    if (q > 0) stage(q - 1);
    T* out = obuf + 2 * lane;
    if (q > 0 && rows == kSub) {
      lif_recompute<true, kPlain>(v_sub(q - 1), xs_of(q - 1) + 2 * lane, kSub, k, nxt);
      g = lif_grad_tile<true, kPlain>(g, cur, gs_of(q) + 2 * lane, out, kSub, k);
    } else {
      g = lif_grad_tile<false, kPlain>(g, cur, gs_of(q) + 2 * lane, out, rows, k);
      if (q > 0) lif_recompute<true, kPlain>(v_sub(q - 1), xs_of(q - 1) + 2 * lane, kSub, k, nxt);
    }
    __syncwarp();
    drain_tile(obuf, static_cast<T*>(a.gx), b, q * kSub, rows, a.T, a.C, c, v0, v1, lane);
    __syncwarp();
  };
#pragma unroll 1
  for (int q = nq - 1; q >= 0; q -= 2) {
    body(q, va, vb);
    if (q == 0) break;
    body(q - 1, vb, va);
  }
}

// ---------------------------------------------- warp-specialized backward (TMA)
//
// The backward's TMA path: a CTA holds kLifWarps consumer warps, one per 64-channel block
// of one batch row (adjacent blocks), and one producer warp. One TMA box of
// kLifWsCols channels per tensor and staged tile serves all consumers, and
// one TMA store per tile writes their outputs, all issued by the producer:
// a TMA operation costs the issuing warp ~150 cycles, which the consumers
// (each alone on its scheduler, paying for every instruction it issues) no
// longer pay (the backward has three loads and a store per staged tile; 47.6
// against 50.9 us at B=64 T=1024 C=512 bf16). The forward, one load and one
// store per 8 KB tile and close to the DRAM bound, stays faster with its
// warps issuing their own copies (25.1 against 29.2 us as warp-specialized). Barriers: full[s] (producer + TMA bytes), empty[s] (one arrival
// per consumer when done with stage s), ofull[o] (one arrival per consumer
// when its part of output buffer o is written and fenced), oempty[o] (the
// producer, once the store from buffer o has read it, reported after the
// next store is issued). All waits are bounded; on a timeout the error is
// recorded, the warp returns, and the producer drains its loads.

constexpr int kLifWsCols = kLifWarps * kLanes;     // channels per CTA (one box wide)
constexpr int kLifWsThreads = 32 * (kLifWarps + 1);
constexpr int kLifWsBwdStages = 4;
constexpr int kLifWsOut = 4;
// Rows of a staged tile: 16 KB boxes (32 bf16/fp16 rows, 16 fp32 rows).
template <typename T>
__host__ __device__ constexpr int lif_ws_rows() {
  return 16384 / (kLifWsCols * static_cast<int>(sizeof(T)));
}
template <typename T>
__host__ __device__ constexpr size_t lif_ws_bwd_stage_bytes() {
  return (size_t)2 * 16384 + (size_t)(lif_ws_rows<T>() / kSub) * kLifWsCols * sizeof(float);
}
template <typename T>
__host__ __device__ constexpr size_t lif_ws_bwd_smem_bytes() {
  return (size_t)kLifWsBwdStages * lif_ws_bwd_stage_bytes<T>() + (size_t)kLifWsOut * 16384 +
         8 * (2 * kLifWsBwdStages + 2 * kLifWsOut);
}
static_assert(lif_ws_bwd_smem_bytes<__nv_bfloat16>() <= 227 * 1024 && lif_ws_bwd_smem_bytes<float>() <= 227 * 1024,
              "LIF backward shared memory");
static_assert(lif_ws_bwd_stage_bytes<float>() % 128 == 0 && lif_ws_bwd_stage_bytes<__nv_bfloat16>() % 128 == 0,
              "TMA stage alignment");

__device__ __forceinline__ void lif_mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

template <typename T, bool kPlain>
__global__ void __launch_bounds__(kLifWsThreads, 1)
    lif_bwd_ws_kernel(const LifArgs a, const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tgs,
                      const __grid_constant__ CUtensorMap tst, const __grid_constant__ CUtensorMap tgx) {
  constexpr int S = kLifWsBwdStages, NO = kLifWsOut;
  constexpr int RT = lif_ws_rows<T>();
  constexpr int QT = RT / kSub;
  constexpr int E = RT * kLifWsCols;
  constexpr int SE = (int)lif_ws_bwd_stage_bytes<T>();
  extern __shared__ __align__(128) unsigned char smem[];
  T* obuf = reinterpret_cast<T*>(smem + S * SE);
  uint64_t* full = reinterpret_cast<uint64_t*>(obuf + NO * E);
  uint64_t* empty = full + S;
  uint64_t* ofull = empty + S;
  uint64_t* oempty = ofull + NO;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncg = (a.ncblk + kLifWarps - 1) / kLifWarps;
  const int cg = blockIdx.x % ncg, b = blockIdx.x / ncg;
  // this CTA's time segment: staged tiles [tt0, tt0 + ntt), sub-tiles [q0, q0 + nq)
  const int seg = blockIdx.y;
  const int ntt_all = (a.T + RT - 1) / RT;
  const int tt0 = a.nseg > 1 ? seg * a.seg_tiles : 0;
  const int ntt = a.nseg > 1 ? min(ntt_all, tt0 + a.seg_tiles) - tt0 : ntt_all;
  const int q0 = tt0 * QT;
  const int nq = min(a.ntiles, q0 + ntt * QT) - q0;
  auto xs_of = [&](int vt) { return reinterpret_cast<T*>(smem + (vt % S) * SE); };
  auto gs_of = [&](int vt) { return xs_of(vt) + E; };
  auto st_of = [&](int vt) { return reinterpret_cast<float*>(xs_of(vt) + 2 * E); };
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kLifWarps);
    }
    for (int i = 0; i < NO; ++i) {
      mbar_init(&ofull[i], kLifWarps);
      mbar_init(&oempty[i], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == kLifWarps) {  // producer; the vt-th visited tile is tile ntt - 1 - vt
    if (lane != 0) return;
    prefetch_tensormap(&tx);
    prefetch_tensormap(&tgs);
    prefetch_tensormap(&tst);
    prefetch_tensormap(&tgx);
    auto issue = [&](int vt) {
      const int jt = tt0 + ntt - 1 - vt;
      uint64_t* bar = &full[vt % S];
      mbar_arrive_expect_tx(bar, SE);
      tma_load_3d(xs_of(vt), &tx, bar, cg * kLifWsCols, jt * RT, b);
      tma_load_3d(gs_of(vt), &tgs, bar, cg * kLifWsCols, jt * RT, b);
      tma_load_3d(st_of(vt), &tst, bar, cg * kLifWsCols, jt * QT, b);
    };
    int issued = min(S, ntt);
    for (int vt = 0; vt < issued; ++vt) issue(vt);
    for (int vt = 0; vt < ntt; ++vt) {
      if (vt + S < ntt) {
        if (!mbar_wait_bounded(&empty[vt % S], (vt / S) & 1)) {
          report_timeout(a.err);
          break;
        }
        issue(vt + S);
        issued = vt + S + 1;
      }
      if (!mbar_wait_bounded(&ofull[vt % NO], (vt / NO) & 1)) {
        report_timeout(a.err);
        break;
      }
      tma_store_3d(&tgx, obuf + (vt % NO) * E, cg * kLifWsCols, (tt0 + ntt - 1 - vt) * RT, b);
      bulk_commit();
      if (vt > 0) {
        bulk_wait_read<1>();
        lif_mbar_arrive(&oempty[(vt - 1) % NO]);
      }
    }
    for (int j = max(0, issued - S); j < issued; ++j) mbar_wait_bounded(&full[j % S], (j / S) & 1);
    bulk_wait_all();
    return;
  }

  // consumers: sub-tiles last first, the recompute of sub-tile q - 1 beside
  // the adjoint sweep of sub-tile q
  const int cb = cg * kLifWarps + warp;
  const LifK k = lif_constants(a);
  const int off = warp * kLanes + 2 * lane;
  (void)cb;
  auto vt_of = [&](int q) { return ntt - 1 - q / QT; };
  auto x_sub = [&](int q) -> const T* { return xs_of(vt_of(q)) + (q % QT) * kSub * kLifWsCols + off; };
  auto g_sub = [&](int q) -> const T* { return gs_of(vt_of(q)) + (q % QT) * kSub * kLifWsCols + off; };
  auto o_sub = [&](int q) -> T* { return obuf + (vt_of(q) % NO) * E + (q % QT) * kSub * kLifWsCols + off; };
  auto v_sub = [&](int q) -> f2 {
    return *reinterpret_cast<const f2*>(st_of(vt_of(q)) + (q % QT) * kLifWsCols + off);
  };
  auto wait_full = [&](int vt) -> bool {
    if (__all_sync(kFull, mbar_wait_bounded(&full[vt % S], (vt / S) & 1))) return true;
    if (lane == 0) report_timeout(a.err);
    return false;
  };
  if (nq == 0) return;
  const int last_rows = a.T - (q0 + nq - 1) * kSub;
  f2 va[kSub], vb[kSub];
  // the adjoint entering the segment from its end: zero for the last one,
  // else the later segments' affine maps applied to zero, last first
  f2 g = k.zero;
  if (a.nseg > 1) {
    const int c = cg * kLifWsCols + off;
    if (c < a.C) {
      for (int s2 = a.nseg - 1; s2 > seg; --s2) {
        const float* p = a.seg_sum + ((size_t)b * a.nseg + s2) * 2 * a.C + c;
        g = fma2(*reinterpret_cast<const f2*>(p), g, *reinterpret_cast<const f2*>(p + a.C));
      }
    }
  }
  if (!wait_full(0)) return;
  if (last_rows == kSub) lif_recompute<true, kPlain, T, kLifWsCols>(v_sub(nq - 1), x_sub(nq - 1), kSub, k, va);
  else lif_recompute<false, kPlain, T, kLifWsCols>(v_sub(nq - 1), x_sub(nq - 1), last_rows, k, va);
  auto body = [&](int q, const f2(&cur)[kSub], f2(&nxt)[kSub]) -> bool {
    const int u0 = (q0 + q) * kSub;
    const int rows = min(kSub, a.T - u0);
    const int vt = vt_of(q);
    if (q > 0 && q % QT == 0 && !wait_full(vt + 1)) return false;
    if ((q == nq - 1 || q % QT == QT - 1) && vt >= NO &&
        !__all_sync(kFull, mbar_wait_bounded(&oempty[vt % NO], ((vt - NO) / NO) & 1))) {
      if (lane == 0) report_timeout(a.err);
      return false;
    }
    if (q > 0 && rows == kSub) {
      lif_recompute<true, kPlain, T, kLifWsCols>(v_sub(q - 1), x_sub(q - 1), kSub, k, nxt);
      g = lif_grad_tile<true, kPlain, T, kLifWsCols>(g, cur, g_sub(q), o_sub(q), kSub, k);
    } else {
      g = lif_grad_tile<false, kPlain, T, kLifWsCols>(g, cur, g_sub(q), o_sub(q), rows, k);
      if (q > 0) lif_recompute<true, kPlain, T, kLifWsCols>(v_sub(q - 1), x_sub(q - 1), kSub, k, nxt);
    }
    if (q % QT == 0) {  // the visited tile is done: release its stage, hand over its gradients
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        lif_mbar_arrive(&empty[vt % S]);
        lif_mbar_arrive(&ofull[vt % NO]);
      }
    }
    return true;
  };
#pragma unroll 1
  for (int q = nq - 1; q >= 0; q -= 2) {
    if (!body(q, va, vb)) return;
    if (q == 0 || !body(q - 1, vb, va)) return;
  }
}

// ------------------------------------------ time-segmented backward (summary)
//
// With few sequences the backward has few units (one per 256-channel group
// and sequence) and each is a serial sweep over T. The adjoint recurrence is
// affine in g: per step, with the membrane recomputed from the checkpoints,
//   g_prev = decay * (dsdv * (g * (reset - vn) + gs) + (spike ? g * 0 : g))
// so a segment of steps maps the adjoint entering from its end, G, to
// g_start = A * G + B. This kernel composes (A, B) for segments 1 .. nseg-1,
// with the operations of lif_grad_tile. A CTA takes one 64-channel block,
// sequence and segment; its kLifWarps warps compose consecutive quarters of
// the segment's sub-tiles (plain coalesced loads, the next sub-tile's loads
// issued before the current one is processed) and warp 0 chains the quarters'
// maps, latest first. The warp-specialized kernel then runs every segment at
// once from its entering adjoint (the later segments' maps applied to zero):
// the last segment's gradients are bit-identical to the one-segment sweep,
// the others agree to rounding.
template <typename T, bool kPlain>
__global__ void __launch_bounds__(32 * kLifWarps) lif_bwd_summary_kernel(const LifArgs a) {
  using P = Pair<T>;
  using raw = typename P::raw;
  __shared__ f2 part[kLifWarps][2][kLanes / 2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cb = blockIdx.x % a.ncblk, b = blockIdx.x / a.ncblk;  // (channel block, sequence)
  const int c = cb * kLanes + 2 * lane;
  const bool on = c < a.C;  // the TMA path has C a multiple of 4: a pair is in or out
  const int s = blockIdx.y + 1;
  constexpr int QT = lif_ws_rows<T>() / kSub;
  const int s_begin = s * a.seg_tiles * QT, s_end = min(a.ntiles, (s + 1) * a.seg_tiles * QT);
  const int per_warp = (s_end - s_begin + kLifWarps - 1) / kLifWarps;
  const int q_begin = min(s_end, s_begin + warp * per_warp), q_end = min(s_end, q_begin + per_warp);
  const LifK k = lif_constants(a);
  const T* xg = static_cast<const T*>(a.x);
  const T* gg = static_cast<const T*>(a.gs);
  const raw zero{};
  auto load = [&](int q, raw (&xo)[kSub], raw (&go)[kSub], f2& m) {
    const int t0 = q * kSub;
#pragma unroll
    for (int i = 0; i < kSub; ++i) {
      const bool ok = on && t0 + i < a.T;
      const size_t r = ((size_t)b * a.T + t0 + i) * a.C + c;
      xo[i] = ok ? P::ld(xg + r) : zero;
      go[i] = ok ? P::ld(gg + r) : zero;
    }
    m = on ? *reinterpret_cast<const f2*>(a.state + ((size_t)b * a.ntiles + q) * a.C + c) : k.zero;
  };
  f2 A = k.one, B = k.zero;
  auto compose = [&](int q, const raw (&xi)[kSub], const raw (&gi)[kSub], f2 m) {
    const int rows = min(kSub, a.T - q * kSub);
    f2 vp[kSub];
#pragma unroll
    for (int i = 0; i < kSub; ++i) {
      if (i < rows) {
        uint32_t w0, w1;
        lif_step<T, kPlain>(m, P::unpack(xi[i]), k, vp[i], w0, w1);
      }
    }
#pragma unroll
    for (int i = kSub - 1; i >= 0; --i) {
      if (i < rows) {
        const f2 d = sub2(vp[i], k.thr);
        const f2 cen = kPlain ? d : mul2(k.slope, d);
        f2 dsdv;
        if constexpr (kPlain) {
          const f2 h = mul2(k.hq, d);
          dsdv = rcpx2(fma2(h, h, k.cq));
        } else {
          const f2 h = mul2(k.half_pi, cen);
          dsdv = mul2(k.half_slope, rcpx2(fma2(h, h, k.one)));
        }
        const f2 rv = sub2(k.reset, vp[i]);
        const f2 a0 = mul2(A, k.zero), b0 = mul2(B, k.zero);
        const f2 as = f2{cen.x >= 0.f ? a0.x : A.x, cen.y >= 0.f ? a0.y : A.y};
        const f2 bs = f2{cen.x >= 0.f ? b0.x : B.x, cen.y >= 0.f ? b0.y : B.y};
        A = mul2(k.decay, fma2(dsdv, mul2(A, rv), as));
        B = mul2(k.decay, fma2(dsdv, fma2(B, rv, P::unpack(gi[i])), bs));
      }
    }
  };
  if (q_begin < q_end) {
    raw xa[kSub], ga[kSub], xb[kSub], gb[kSub];
    f2 ma, mb;
    load(q_end - 1, xa, ga, ma);
#pragma unroll 1
    for (int q = q_end - 1; q >= q_begin; q -= 2) {
      if (q - 1 >= q_begin) load(q - 1, xb, gb, mb);
      compose(q, xa, ga, ma);
      if (q - 1 < q_begin) break;
      if (q - 2 >= q_begin) load(q - 2, xa, ga, ma);
      compose(q - 1, xb, gb, mb);
    }
  }
  part[warp][0][lane] = A;
  part[warp][1][lane] = B;
  __syncthreads();
  if (warp != 0 || !on) return;
  // g_start = A_0 (A_1 ( ... (A_last G + B_last) ... ) + B_1) + B_0
  f2 At = k.one, Bt = k.zero;
  for (int w = kLifWarps - 1; w >= 0; --w) {
    const f2 Aw = part[w][0][lane], Bw = part[w][1][lane];
    Bt = fma2(Aw, Bt, Bw);
    At = mul2(Aw, At);
  }
  float* p = a.seg_sum + ((size_t)b * a.nseg + s) * 2 * a.C + c;
  *reinterpret_cast<f2*>(p) = At;
  *reinterpret_cast<f2*>(p + a.C) = Bt;
}

}  // namespace wkv
