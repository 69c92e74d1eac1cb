// Fused elementwise gates of the SpikeGPT blocks (sm_100a), bf16 tensors.
//
// The receptance gate of time and channel mixing (src/spikegpt/language.py:
// 1022 and 1035 ``sigmoid(receptance(xr)) * wkv``, 1195-1196 ``sigmoid(r) *
// value(k)``) and the channel-mixing activation (language.py:1193
// ``relu(key(xk)).square()``) run under bf16 autocast as two eager kernels
// forward and two or three backward each. Here each is one pass, with the
// eager roundings:
//   gate:        s = bf16(1 / (1 + exp(-r))),  out = bf16(s * x)
//                grad_x = bf16(g * s),  a = bf16(g * x),
//                grad_r = bf16(bf16(a * bf16(1 - s)) * s)
//                (the sigmoid backward in bf16 arithmetic, one rounding per
//                operation, as PyTorch evaluates it for 16-bit types)
//   relu_square: out = bf16(relu(k)^2)
//                grad_k = k <= 0 ? 0 : bf16(g * (2 k))
//   residual_add: out = x + float(s)   (float32 residual stream plus the bf16
//                spikes of a LIF sublayer, language.py:1353-1358; PyTorch's
//                type-promoting add, which converts s exactly and rounds once)
// (products in float32; relu keeps NaN, and its backward zeroes the
// gradient where its output is <= 0, so a NaN key passes g * 2k = NaN on, as
// eagerly). Eight elements per thread per
// iteration (16-byte loads and stores), grid-stride; a scalar tail handles
// n % 8. Memory-bound: gate forward 6 B per element, backward 10 B;
// relu_square 4 B and 6 B; residual_add 10 B.
#pragma once

#include <cuda_bf16.h>

#include <cstdint>

namespace wkv {

constexpr int kGateThreads = 256;

__device__ __forceinline__ float bf(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 rb(float v) { return __float2bfloat16_rn(v); }

__device__ __forceinline__ float gate_sigmoid(float r) { return bf(rb(1.f / (1.f + expf(-r)))); }

__device__ __forceinline__ void gate_grad(float g, float r, float x, __nv_bfloat16& gr, __nv_bfloat16& gx) {
  const float s = gate_sigmoid(r);
  gx = rb(g * s);
  const float a = bf(rb(g * x));
  gr = rb(bf(rb(a * bf(rb(1.f - s)))) * s);
}

struct Gate {
  __device__ static void fwd(const __nv_bfloat16* r, const __nv_bfloat16* x, __nv_bfloat16* out, int64_t i) {
    out[i] = rb(gate_sigmoid(bf(r[i])) * bf(x[i]));
  }
  __device__ static void bwd(const __nv_bfloat16* g, const __nv_bfloat16* r, const __nv_bfloat16* x,
                             __nv_bfloat16* gr, __nv_bfloat16* gx, int64_t i) {
    gate_grad(bf(g[i]), bf(r[i]), bf(x[i]), gr[i], gx[i]);
  }
};

struct ReluSquare {
  __device__ static float act(float k) {
    const float v = k != k ? k : fmaxf(k, 0.f);  // relu, NaN kept
    return v * v;
  }
  __device__ static void fwd(const __nv_bfloat16* k, __nv_bfloat16* out, int64_t i) { out[i] = rb(act(bf(k[i]))); }
  __device__ static __nv_bfloat16 grad(float g, float k) { return k <= 0.f ? rb(0.f) : rb(g * (2.f * k)); }
  __device__ static void bwd(const __nv_bfloat16* g, const __nv_bfloat16* k, __nv_bfloat16* gk, int64_t i) {
    gk[i] = grad(bf(g[i]), bf(k[i]));
  }
};

union Bf8 {
  uint4 u;
  __nv_bfloat16 h[8];
};

__device__ __forceinline__ Bf8 ld8(const __nv_bfloat16* p) {
  Bf8 v;
  v.u = *reinterpret_cast<const uint4*>(p);
  return v;
}
__device__ __forceinline__ void st8(__nv_bfloat16* p, const Bf8& v) { *reinterpret_cast<uint4*>(p) = v.u; }

__global__ void __launch_bounds__(kGateThreads) gate_fwd_kernel(const __nv_bfloat16* r, const __nv_bfloat16* x,
                                                                __nv_bfloat16* out, int64_t n) {
  const int64_t nv = n / 8, stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += stride) {
    const Bf8 a = ld8(r + 8 * v), b = ld8(x + 8 * v);
    Bf8 o;
#pragma unroll
    for (int j = 0; j < 8; ++j) o.h[j] = rb(gate_sigmoid(bf(a.h[j])) * bf(b.h[j]));
    st8(out + 8 * v, o);
  }
  if (blockIdx.x == 0)
    for (int64_t i = 8 * nv + threadIdx.x; i < n; i += blockDim.x) Gate::fwd(r, x, out, i);
}

__global__ void __launch_bounds__(kGateThreads) gate_bwd_kernel(const __nv_bfloat16* g, const __nv_bfloat16* r,
                                                                const __nv_bfloat16* x, __nv_bfloat16* gr,
                                                                __nv_bfloat16* gx, int64_t n) {
  const int64_t nv = n / 8, stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += stride) {
    const Bf8 gg = ld8(g + 8 * v), rr = ld8(r + 8 * v), xx = ld8(x + 8 * v);
    Bf8 a, b;
#pragma unroll
    for (int j = 0; j < 8; ++j) gate_grad(bf(gg.h[j]), bf(rr.h[j]), bf(xx.h[j]), a.h[j], b.h[j]);
    st8(gr + 8 * v, a);
    st8(gx + 8 * v, b);
  }
  if (blockIdx.x == 0)
    for (int64_t i = 8 * nv + threadIdx.x; i < n; i += blockDim.x) Gate::bwd(g, r, x, gr, gx, i);
}

__global__ void __launch_bounds__(kGateThreads) relu_square_fwd_kernel(const __nv_bfloat16* k, __nv_bfloat16* out,
                                                                       int64_t n) {
  const int64_t nv = n / 8, stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += stride) {
    const Bf8 a = ld8(k + 8 * v);
    Bf8 o;
#pragma unroll
    for (int j = 0; j < 8; ++j) o.h[j] = rb(ReluSquare::act(bf(a.h[j])));
    st8(out + 8 * v, o);
  }
  if (blockIdx.x == 0)
    for (int64_t i = 8 * nv + threadIdx.x; i < n; i += blockDim.x) ReluSquare::fwd(k, out, i);
}

__global__ void __launch_bounds__(kGateThreads) relu_square_bwd_kernel(const __nv_bfloat16* g,
                                                                       const __nv_bfloat16* k, __nv_bfloat16* gk,
                                                                       int64_t n) {
  const int64_t nv = n / 8, stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += stride) {
    const Bf8 gg = ld8(g + 8 * v), kk = ld8(k + 8 * v);
    Bf8 o;
#pragma unroll
    for (int j = 0; j < 8; ++j) o.h[j] = ReluSquare::grad(bf(gg.h[j]), bf(kk.h[j]));
    st8(gk + 8 * v, o);
  }
  if (blockIdx.x == 0)
    for (int64_t i = 8 * nv + threadIdx.x; i < n; i += blockDim.x) ReluSquare::bwd(g, k, gk, i);
}

__global__ void __launch_bounds__(kGateThreads) residual_add_kernel(const float* x, const __nv_bfloat16* s,
                                                                    float* out, int64_t n) {
  const int64_t nv = n / 8, stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nv; v += stride) {
    const float4 a = *reinterpret_cast<const float4*>(x + 8 * v), b = *reinterpret_cast<const float4*>(x + 8 * v + 4);
    const Bf8 sp = ld8(s + 8 * v);
    *reinterpret_cast<float4*>(out + 8 * v) =
        make_float4(a.x + bf(sp.h[0]), a.y + bf(sp.h[1]), a.z + bf(sp.h[2]), a.w + bf(sp.h[3]));
    *reinterpret_cast<float4*>(out + 8 * v + 4) =
        make_float4(b.x + bf(sp.h[4]), b.y + bf(sp.h[5]), b.z + bf(sp.h[6]), b.w + bf(sp.h[7]));
  }
  if (blockIdx.x == 0)
    for (int64_t i = 8 * nv + threadIdx.x; i < n; i += blockDim.x) out[i] = x[i] + bf(s[i]);
}

}  // namespace wkv
