// Fused cross-entropy over bf16 logits for the language-model loss (sm_100a).
//
// The reference computes its loss as F.cross_entropy(logits.float(), targets)
// (src/spikegpt/language.py:1475-1480): under bf16 autocast that is a float32
// copy of the [rows, V] logits, a log-softmax forward and backward over the
// copy, and a cast of the gradient back to bf16. Here, per row i with target
// t_i (rows whose target is PyTorch's ignore_index -100 are ignored: loss 0,
// gradient 0; any other target outside [0, V), which PyTorch rejects, gives
// the row a NaN loss and a NaN gradient and sets kXentBadTarget in the sticky
// device error flags, so the mean loss is NaN instead of silently lower):
//   forward:  lse_i = log sum_j exp(x_ij),  loss_i = lse_i - x_i,t_i
//   backward: dx_ij = bf16(g_i * (exp(x_ij - lse_i) - [j == t_i]))
// in float32 from the bf16 logits, read in place (row pitch ld >= V, a
// multiple of 8; the backward writes zeros in the pitch's tail columns). One
// CTA per row: the forward keeps a running (max, sum of exp) per thread over
// 16-byte loads and merges the threads' pairs in a fixed order; the backward
// streams the row once more. Memory-bound: 2 B per logit forward, 4 B back.
#pragma once

#include <cuda_bf16.h>

#include <cstdint>

namespace wkv {

constexpr int kXentThreads = 256;
constexpr int64_t kXentIgnore = -100;
constexpr unsigned kXentBadTarget = 2u;  // WKV_DEVERR_BAD_TARGET

__device__ __forceinline__ void xent_merge(float& m, float& s, float m2, float s2) {
  // (m, s) represents s * exp(m); merge two such sums (an empty one is
  // m = -inf, s = 0; a NaN logit makes the row's sum NaN, as log-softmax does)
  if (!(m2 > -INFINITY)) {
    if (m2 != m2 || s2 != s2) m = s = __int_as_float(0x7fffffff);
    return;
  }
  if (m != m) return;
  if (m2 > m) {
    s = s * expf(m - m2) + s2;
    m = m2;
  } else {
    s = s + s2 * expf(m2 - m);
  }
}

__global__ void __launch_bounds__(kXentThreads) xent_fwd_kernel(const __nv_bfloat16* logits, int64_t ld,
                                                               const int64_t* targets, int64_t V, float* loss,
                                                               float* lse_out, unsigned* err) {
  __shared__ float sm[kXentThreads], ss[kXentThreads];
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* x = logits + row * ld;
  float m = -INFINITY, s = 0.f;
  const int64_t nv = V / 8;
  for (int64_t v = threadIdx.x; v < nv; v += kXentThreads) {
    const uint4 u = *reinterpret_cast<const uint4*>(x + 8 * v);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      xent_merge(m, s, __uint_as_float(w[k] << 16), 1.f);
      xent_merge(m, s, __uint_as_float(w[k] & 0xffff0000u), 1.f);
    }
  }
  for (int64_t j = 8 * nv + threadIdx.x; j < V; j += kXentThreads) xent_merge(m, s, __bfloat162float(x[j]), 1.f);
  sm[threadIdx.x] = m;
  ss[threadIdx.x] = s;
  __syncthreads();
  // fixed-order tree over the threads' pairs
  for (int w = kXentThreads / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) {
      float a = sm[threadIdx.x], b = ss[threadIdx.x];
      xent_merge(a, b, sm[threadIdx.x + w], ss[threadIdx.x + w]);
      sm[threadIdx.x] = a;
      ss[threadIdx.x] = b;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float lse = sm[0] + logf(ss[0]);
    const int64_t t = targets[row];
    lse_out[row] = lse;
    if (t >= 0 && t < V) {
      loss[row] = lse - __bfloat162float(x[t]);
    } else if (t == kXentIgnore) {
      loss[row] = 0.f;
    } else {
      loss[row] = __int_as_float(0x7fffffff);
      if (err) atomicOr(err, kXentBadTarget);
    }
  }
}

__global__ void __launch_bounds__(kXentThreads) xent_bwd_kernel(const __nv_bfloat16* logits, int64_t ld,
                                                               const int64_t* targets, const float* lse_in,
                                                               const float* grad, __nv_bfloat16* dx,
                                                               int64_t V) {
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* x = logits + row * ld;
  __nv_bfloat16* d = dx + row * ld;
  const int64_t t = targets[row];
  const bool on = t >= 0 && t < V;
  const float g = on ? grad[row] : (t == kXentIgnore ? 0.f : __int_as_float(0x7fffffff));
  const float lse = lse_in[row];
  const int64_t nv = ld / 8;
  for (int64_t v = threadIdx.x; v < nv; v += kXentThreads) {
    const uint4 u = *reinterpret_cast<const uint4*>(x + 8 * v);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int64_t j = 8 * v + 2 * k;
      float a = j < V ? expf(__uint_as_float(w[k] << 16) - lse) - (j == t ? 1.f : 0.f) : 0.f;
      float b = j + 1 < V ? expf(__uint_as_float(w[k] & 0xffff0000u) - lse) - (j + 1 == t ? 1.f : 0.f) : 0.f;
      const __nv_bfloat162 p = __floats2bfloat162_rn(g * a, g * b);
      o[k] = *reinterpret_cast<const uint32_t*>(&p);
    }
    *reinterpret_cast<uint4*>(d + 8 * v) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace wkv
