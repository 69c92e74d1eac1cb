// Fused LayerNorm + token-shift mixing for the SpikeGPT blocks (sm_100a).
//
// Every time-mixing and channel-mixing sublayer of the reference model
// (src/spikegpt/language.py:1009-1012, 1190-1192, 344-353) normalises the
// residual stream x [B, T, C] (float32) and forms, for each of its n mixing
// vectors m_i [C], the GEMM input
//   out_i[t] = h[t] * m_i + h[t-1] * (1 - m_i),  h = LayerNorm(x), h[-1] = 0,
// which bf16 autocast then rounds to bf16. ln_mix_fwd does that in one pass
// over x (the products and the sum rounded as the reference's eager float32
// ops round them, then to bf16), keeping the row statistics (mean, 1/std) for
// the backward. ln_mix_bwd takes the n bf16 output gradients and returns
//   dh[t]  = sum_i m_i g_i[t] + (1 - m_i) g_i[t+1]
//   dx     = rstd (dh w - mean(dh w) - xhat mean(dh w xhat))      (LayerNorm)
//   dw     = sum_rows dh xhat,  db = sum_rows dh,  dm_i = sum_rows g_i[t] (h[t] - h[t-1])
// the column sums as per-warp partials reduced in a fixed order by
// ln_mix_reduce (deterministic).
//
// Layout: one warp per chunk of kMixRows consecutive steps of one sequence;
// lane l holds channels g*128 + 4l .. 4l+3 of each 128-channel group g
// (float4 loads of x, 8-byte bf16 stores). C is a multiple of 128, at most
// kMixMaxGroups * 128. Memory-bound: forward reads x (4 B) and writes n bf16
// outputs (2n B) per element; backward reads x and n gradients, writes dx.
#pragma once

#include "wkv_device.cuh"

namespace wkv {

constexpr int kMixMax = 3;         // mixing vectors per call (time mixing: key, value, receptance)
constexpr int kMixRows = 64;       // steps per warp chunk
constexpr int kMixWarps = 4;       // warps per CTA
constexpr int kMixMaxGroups = 8;   // C <= 1024

struct MixArgs {
  const float* x;    // [B*T][C]
  const float* w;    // [C] LayerNorm weight
  const float* b;    // [C] LayerNorm bias
  const float* mix;  // [n][C]
  __nv_bfloat16* out[kMixMax];
  const __nv_bfloat16* gout[kMixMax];
  float* mean;     // [B*T]
  float* rstd;     // [B*T]
  float* gx;       // [B*T][C]
  float* partial;  // [nchunks][2 + n][C]: dw, db, dm_0 .. dm_{n-1} per chunk
  int n, B, T, C, nct;  // nct = chunks per sequence
  float eps;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

template <int G>
__device__ __forceinline__ void mix_load_row(const float* row, int lane, float4 (&v)[G]) {
#pragma unroll
  for (int g = 0; g < G; ++g) v[g] = *reinterpret_cast<const float4*>(row + g * 128 + 4 * lane);
}

// Row statistics as PyTorch's LayerNorm defines them (biased variance).
template <int G>
__device__ __forceinline__ void mix_stats(const float4 (&v)[G], int C, float eps, float& mu, float& rs) {
  float s = 0.f;
#pragma unroll
  for (int g = 0; g < G; ++g) s += (v[g].x + v[g].y) + (v[g].z + v[g].w);
  mu = warp_sum(s) / C;
  float q = 0.f;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float a = v[g].x - mu, b = v[g].y - mu, c = v[g].z - mu, d = v[g].w - mu;
    q += (a * a + b * b) + (c * c + d * d);
  }
  rs = rsqrtf(warp_sum(q) / C + eps);
}

__device__ __forceinline__ float4 mix_norm(float4 v, float mu, float rs, float4 w, float4 b) {
  return make_float4(__fmaf_rn(__fmul_rn(v.x - mu, rs), w.x, b.x), __fmaf_rn(__fmul_rn(v.y - mu, rs), w.y, b.y),
                     __fmaf_rn(__fmul_rn(v.z - mu, rs), w.z, b.z), __fmaf_rn(__fmul_rn(v.w - mu, rs), w.w, b.w));
}

// h * m + p * (1 - m) with the reference's roundings (two products, one sum).
__device__ __forceinline__ float mix1(float h, float p, float m, float om) {
  return __fadd_rn(__fmul_rn(h, m), __fmul_rn(p, om));
}

template <int G>
__global__ void __launch_bounds__(32 * kMixWarps) ln_mix_fwd_kernel(const MixArgs a) {
  const int lane = threadIdx.x & 31;
  const int chunk = blockIdx.x * kMixWarps + (threadIdx.x >> 5);
  if (chunk >= a.B * a.nct) return;
  const int bi = chunk / a.nct, t0 = (chunk % a.nct) * kMixRows;
  const int t1 = min(a.T, t0 + kMixRows);
  float4 wv[G], bv[G];
  mix_load_row<G>(a.w, lane, wv);
  mix_load_row<G>(a.b, lane, bv);
  const size_t row0 = (size_t)bi * a.T;
  float4 hp[G];  // h[t-1]
  if (t0 > 0) {
    float4 v[G];
    mix_load_row<G>(a.x + (row0 + t0 - 1) * a.C, lane, v);
    float mu, rs;
    mix_stats<G>(v, a.C, a.eps, mu, rs);
#pragma unroll
    for (int g = 0; g < G; ++g) hp[g] = mix_norm(v[g], mu, rs, wv[g], bv[g]);
  } else {
#pragma unroll
    for (int g = 0; g < G; ++g) hp[g] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll 1
  for (int t = t0; t < t1; ++t) {
    const size_t r = row0 + t;
    float4 v[G];
    mix_load_row<G>(a.x + r * a.C, lane, v);
    float mu, rs;
    mix_stats<G>(v, a.C, a.eps, mu, rs);
    if (lane == 0) {
      a.mean[r] = mu;
      a.rstd[r] = rs;
    }
    float4 h[G];
#pragma unroll
    for (int g = 0; g < G; ++g) h[g] = mix_norm(v[g], mu, rs, wv[g], bv[g]);
#pragma unroll 1
    for (int i = 0; i < a.n; ++i) {
      const float* mrow = a.mix + (size_t)i * a.C;
      __nv_bfloat16* orow = a.out[i] + r * a.C;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float4 m = *reinterpret_cast<const float4*>(mrow + g * 128 + 4 * lane);
        const float o0 = mix1(h[g].x, hp[g].x, m.x, 1.f - m.x), o1 = mix1(h[g].y, hp[g].y, m.y, 1.f - m.y);
        const float o2 = mix1(h[g].z, hp[g].z, m.z, 1.f - m.z), o3 = mix1(h[g].w, hp[g].w, m.w, 1.f - m.w);
        __nv_bfloat162 lo = __floats2bfloat162_rn(o0, o1), hi = __floats2bfloat162_rn(o2, o3);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&lo);
        pk.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(orow + g * 128 + 4 * lane) = pk;
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) hp[g] = h[g];
  }
}

// Four bf16 values (8 bytes) as floats.
__device__ __forceinline__ float4 mix_grad4(const __nv_bfloat16* p) {
  const uint2 pk = *reinterpret_cast<const uint2*>(p);
  return make_float4(__uint_as_float(pk.x << 16), __uint_as_float(pk.x & 0xffff0000u),
                     __uint_as_float(pk.y << 16), __uint_as_float(pk.y & 0xffff0000u));
}

// Backward of one chunk. The mixing vectors and the output gradients are read
// where used (the next row's gradients again as the current row's one step
// later, from L1/L2); the column accumulators stay in registers.
template <int G, int N>
__global__ void __launch_bounds__(32 * kMixWarps) ln_mix_bwd_kernel(const MixArgs a) {
  const int lane = threadIdx.x & 31;
  const int chunk = blockIdx.x * kMixWarps + (threadIdx.x >> 5);
  if (chunk >= a.B * a.nct) return;
  const int bi = chunk / a.nct, t0 = (chunk % a.nct) * kMixRows;
  const int t1 = min(a.T, t0 + kMixRows);
  float4 wv[G], bv[G];
  mix_load_row<G>(a.w, lane, wv);
  mix_load_row<G>(a.b, lane, bv);
  const size_t row0 = (size_t)bi * a.T;
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  float4 acc_w[G], acc_b[G], acc_m[N][G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    acc_w[g] = acc_b[g] = z4;
#pragma unroll
    for (int i = 0; i < N; ++i) acc_m[i][g] = z4;
  }
  float4 hp[G];  // h[t-1]
  if (t0 > 0) {
    float4 v[G];
    const size_t r = row0 + t0 - 1;
    mix_load_row<G>(a.x + r * a.C, lane, v);
    const float mu = a.mean[r], rs = a.rstd[r];
#pragma unroll
    for (int g = 0; g < G; ++g) hp[g] = mix_norm(v[g], mu, rs, wv[g], bv[g]);
  } else {
#pragma unroll
    for (int g = 0; g < G; ++g) hp[g] = z4;
  }
#pragma unroll 1
  for (int t = t0; t < t1; ++t) {
    const size_t r = row0 + t;
    const bool has_next = t + 1 < a.T;
    float4 xh[G], dw[G];
    float s1 = 0.f, s2 = 0.f;
    const float mu = a.mean[r], rs = a.rstd[r];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int c = g * 128 + 4 * lane;
      const float4 v = *reinterpret_cast<const float4*>(a.x + r * a.C + c);
      const float4 h = mix_norm(v, mu, rs, wv[g], bv[g]);
      xh[g] = make_float4(__fmul_rn(v.x - mu, rs), __fmul_rn(v.y - mu, rs), __fmul_rn(v.z - mu, rs),
                          __fmul_rn(v.w - mu, rs));
      float4 d = z4;
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const float4 m = *reinterpret_cast<const float4*>(a.mix + (size_t)i * a.C + c);
        const float4 gc = mix_grad4(a.gout[i] + r * a.C + c);
        const float4 gn = has_next ? mix_grad4(a.gout[i] + (r + 1) * a.C + c) : z4;
        d.x += m.x * gc.x + (1.f - m.x) * gn.x;
        d.y += m.y * gc.y + (1.f - m.y) * gn.y;
        d.z += m.z * gc.z + (1.f - m.z) * gn.z;
        d.w += m.w * gc.w + (1.f - m.w) * gn.w;
        acc_m[i][g].x += gc.x * (h.x - hp[g].x);
        acc_m[i][g].y += gc.y * (h.y - hp[g].y);
        acc_m[i][g].z += gc.z * (h.z - hp[g].z);
        acc_m[i][g].w += gc.w * (h.w - hp[g].w);
      }
      hp[g] = h;
      acc_w[g].x += d.x * xh[g].x;
      acc_w[g].y += d.y * xh[g].y;
      acc_w[g].z += d.z * xh[g].z;
      acc_w[g].w += d.w * xh[g].w;
      acc_b[g].x += d.x;
      acc_b[g].y += d.y;
      acc_b[g].z += d.z;
      acc_b[g].w += d.w;
      dw[g] = make_float4(d.x * wv[g].x, d.y * wv[g].y, d.z * wv[g].z, d.w * wv[g].w);
      s1 += (dw[g].x + dw[g].y) + (dw[g].z + dw[g].w);
      s2 += (dw[g].x * xh[g].x + dw[g].y * xh[g].y) + (dw[g].z * xh[g].z + dw[g].w * xh[g].w);
    }
    s1 = warp_sum(s1) / a.C;
    s2 = warp_sum(s2) / a.C;
    float* gxr = a.gx + r * a.C;
#pragma unroll
    for (int g = 0; g < G; ++g)
      *reinterpret_cast<float4*>(gxr + g * 128 + 4 * lane) =
          make_float4(rs * (dw[g].x - s1 - xh[g].x * s2), rs * (dw[g].y - s1 - xh[g].y * s2),
                      rs * (dw[g].z - s1 - xh[g].z * s2), rs * (dw[g].w - s1 - xh[g].w * s2));
  }
  float* p = a.partial + (size_t)chunk * (2 + N) * a.C;
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const int c = g * 128 + 4 * lane;
    *reinterpret_cast<float4*>(p + c) = acc_w[g];
    *reinterpret_cast<float4*>(p + a.C + c) = acc_b[g];
#pragma unroll
    for (int i = 0; i < N; ++i) *reinterpret_cast<float4*>(p + (2 + i) * (size_t)a.C + c) = acc_m[i][g];
  }
}

// Column sums of the per-chunk partials: out[k][c] for the 2 + n rows k (dw,
// db, dm_i). A CTA of 32 x 32 threads takes 32 columns of one row k; thread
// (y, x) sums the chunks y, y + 32, ... of column x, then the 32 partial sums
// of a column are added in y order (a fixed order: the result does not depend
// on timing).
__global__ void __launch_bounds__(1024) ln_mix_reduce_kernel(const float* partial, int nchunks, int rows, int C,
                                                             float* gw, float* gb, float* gmix) {
  __shared__ float part[32][33];
  const int k = blockIdx.y;
  const int c = blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (c < C)
    for (int j = threadIdx.y; j < nchunks; j += 32) s += partial[((size_t)j * rows + k) * C + c];
  part[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y != 0 || c >= C) return;
  float t = 0.f;
#pragma unroll 8
  for (int y = 0; y < 32; ++y) t += part[y][threadIdx.x];
  float* dst = k == 0 ? gw + c : k == 1 ? gb + c : gmix + (size_t)(k - 2) * C + c;
  *dst = t;
}

}  // namespace wkv
