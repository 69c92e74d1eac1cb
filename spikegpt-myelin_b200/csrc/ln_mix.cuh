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
// the column sums as per-CTA partials reduced in a fixed order by
// ln_mix_reduce (deterministic). When the sublayer's residual connection
// passes its gradient in (gres), dx also takes that gradient, so the residual
// stream's two gradient contributions need no separate add.
//
// Layout: a CTA of C/4 threads takes `rows` consecutive steps of one sequence,
// one row at a time; thread j holds channels 4j .. 4j+3 (a float4 of x, an
// 8-byte bf16 word of each output or gradient), so a row is one coalesced
// 4C-byte read. Row sums (the statistics in the forward, the two LayerNorm
// backward means) are block reductions: a warp butterfly, then the warps'
// sums added in warp order through shared memory, double-buffered so one
// barrier per reduction suffices. The forward issues the next row's load
// before it processes the current row. The backward, which reads more per row
// (x, the residual gradient, n output gradients), keeps a ring of kMixStages
// rows in shared memory filled by per-thread cp.async copies, so two rows are
// in flight while one is processed: on one B200 (SpikeGPT-41M shapes, C=512,
// n=3, 64 x 1024 rows) 226 -> 140 us per call against one row of register
// prefetch. A thread needs few registers, so many CTAs share an SM; `rows`
// (8..64) is chosen per launch so that a launch has about 8 CTAs per SM
// whatever the batch. C is a multiple of 128, at most kMixMaxC.
// Memory-bound: forward reads x (4 B) and writes n bf16 outputs (2n B) per
// element; backward reads x and n gradients, writes dx (and, on request, its
// bf16 copy: the gradient of the bf16 spikes added to the residual stream
// that x is, which would otherwise take a separate cast pass over dx).
#pragma once

#include "wkv_device.cuh"

namespace wkv {

constexpr int kMixMax = 3;        // mixing vectors per call (time mixing: key, value, receptance)
constexpr int kMixMaxC = 1024;    // channels: a CTA has C/4 <= 256 threads
constexpr int kMixMinRows = 8;    // steps per CTA, at least
constexpr int kMixMaxRows = 64;   // and at most
constexpr int kMixStages = 4;     // backward: rows of a CTA's ring, two in use, the rest in flight

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
  __nv_bfloat16* gx16;  // [B*T][C] or null: bf16(gx) as well
  const float* gres;  // [B*T][C] or null: the residual connection's gradient, added to gx
  float* partial;  // [B*nct][2 + n][C]: dw, db, dm_0 .. dm_{n-1} per CTA
  int n, B, T, C;
  int rows;  // steps per CTA
  int nct;   // CTAs per sequence
  float eps;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

// Sum over the CTA of one value per thread (all threads get it): warp sums,
// then the warps' sums in warp order. `slot` alternates between calls (two
// buffers): a buffer is rewritten only after every thread has passed the
// barrier of the call in between, so its readers are done with it.
__device__ __forceinline__ float block_sum(float v, float (*red)[kMixMaxC / 128], int slot) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[slot][threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[slot][w];
  return s;
}

// Two sums at once (one barrier).
__device__ __forceinline__ float2 block_sum2(float u, float v, float2 (*red)[kMixMaxC / 128], int slot) {
  u = warp_sum(u);
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[slot][threadIdx.x >> 5] = make_float2(u, v);
  __syncthreads();
  float2 s = make_float2(0.f, 0.f);
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
    s.x += red[slot][w].x;
    s.y += red[slot][w].y;
  }
  return s;
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// Row statistics as PyTorch's LayerNorm defines them (biased variance), two
// passes (mean, then the centred squares); uses reduction slots 0 and 1.
__device__ __forceinline__ void mix_stats(float4 v, int C, float eps, float (*red)[kMixMaxC / 128], float& mu,
                                          float& rs) {
  mu = block_sum((v.x + v.y) + (v.z + v.w), red, 0) / C;
  const float a = v.x - mu, b = v.y - mu, c = v.z - mu, d = v.w - mu;
  rs = rsqrtf(block_sum((a * a + b * b) + (c * c + d * d), red, 1) / C + eps);
}

__device__ __forceinline__ float4 mix_norm(float4 v, float mu, float rs, float4 w, float4 b) {
  return make_float4(__fmaf_rn(__fmul_rn(v.x - mu, rs), w.x, b.x), __fmaf_rn(__fmul_rn(v.y - mu, rs), w.y, b.y),
                     __fmaf_rn(__fmul_rn(v.z - mu, rs), w.z, b.z), __fmaf_rn(__fmul_rn(v.w - mu, rs), w.w, b.w));
}

// h * m + p * (1 - m) with the reference's roundings (two products, one sum).
__device__ __forceinline__ float mix1(float h, float p, float m, float om) {
  return __fadd_rn(__fmul_rn(h, m), __fmul_rn(p, om));
}

// Four bf16 values (8 bytes): loaded packed, unpacked to floats where used.
__device__ __forceinline__ uint2 mix_ld8(const __nv_bfloat16* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ float4 mix_unpack4(uint2 pk) {
  return make_float4(__uint_as_float(pk.x << 16), __uint_as_float(pk.x & 0xffff0000u),
                     __uint_as_float(pk.y << 16), __uint_as_float(pk.y & 0xffff0000u));
}

// Steps [t0, t1) of sequence bi taken by this CTA.
__device__ __forceinline__ void mix_span(const MixArgs& a, int& bi, int& t0, int& t1) {
  bi = blockIdx.x / a.nct;
  t0 = (blockIdx.x % a.nct) * a.rows;
  t1 = min(a.T, t0 + a.rows);
}

__global__ void __launch_bounds__(kMixMaxC / 4) ln_mix_fwd_kernel(const MixArgs a) {
  __shared__ float red[2][kMixMaxC / 128];
  const int c = 4 * threadIdx.x;
  int bi, t0, t1;
  mix_span(a, bi, t0, t1);
  const float4 wv = ld4(a.w + c), bv = ld4(a.b + c);
  float4 m[kMixMax];
#pragma unroll
  for (int i = 0; i < kMixMax; ++i) m[i] = i < a.n ? ld4(a.mix + (size_t)i * a.C + c) : make_float4(0, 0, 0, 0);
  const size_t row0 = (size_t)bi * a.T;
  float4 hp = make_float4(0.f, 0.f, 0.f, 0.f);  // h[t-1]
  if (t0 > 0) {
    const float4 v = ld4(a.x + (row0 + t0 - 1) * a.C + c);
    float mu, rs;
    mix_stats(v, a.C, a.eps, red, mu, rs);
    hp = mix_norm(v, mu, rs, wv, bv);
  }
  float4 v = ld4(a.x + (row0 + t0) * a.C + c);
#pragma unroll 1
  for (int t = t0; t < t1; ++t) {
    const size_t r = row0 + t;
    const float4 vn = ld4(a.x + (row0 + min(t + 1, t1 - 1)) * a.C + c);  // next row (last row again at the end)
    float mu, rs;
    mix_stats(v, a.C, a.eps, red, mu, rs);
    if (threadIdx.x == 0) {
      a.mean[r] = mu;
      a.rstd[r] = rs;
    }
    const float4 h = mix_norm(v, mu, rs, wv, bv);
#pragma unroll
    for (int i = 0; i < kMixMax; ++i) {
      if (i < a.n) {
        const float o0 = mix1(h.x, hp.x, m[i].x, 1.f - m[i].x), o1 = mix1(h.y, hp.y, m[i].y, 1.f - m[i].y);
        const float o2 = mix1(h.z, hp.z, m[i].z, 1.f - m[i].z), o3 = mix1(h.w, hp.w, m[i].w, 1.f - m[i].w);
        __nv_bfloat162 lo = __floats2bfloat162_rn(o0, o1), hi = __floats2bfloat162_rn(o2, o3);
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&lo);
        pk.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(a.out[i] + r * a.C + c) = pk;
      }
    }
    hp = h;
    v = vn;
  }
}

// Per-thread asynchronous copies into the CTA's row ring (cp.async: each
// thread copies, and later reads, only its own channels, so a stage needs no
// barrier between its copy and its use).
__device__ __forceinline__ void mix_cp16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void mix_cp8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void mix_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int kPending>
__device__ __forceinline__ void mix_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kPending) : "memory");
}

// Dynamic shared memory of ln_mix_bwd: the ring of kMixStages row stages, each
// x [C] and, with a residual gradient, gres [C] (float32), then the n output
// gradients g_i [C] (bf16).
__host__ __device__ constexpr size_t mix_bwd_stage_bytes(int n, int C, bool res) {
  return (size_t)C * (4 + (res ? 4 : 0) + 2 * n);
}

// Backward of the CTA's steps t0 .. t1-1. Row t needs x[t], gres[t], g_i[t]
// and g_i[t+1]: stage k of the ring holds row t0 + k (mod kMixStages) -- its
// x and gres while the row is one of the CTA's, its g_i while it is < T (row
// t1 contributes only its g_i) -- so row t waits for the copies of rows t and
// t+1 while rows t+2 .. t+kMixStages-1 are still in flight. The row
// statistics of rows t0-1 .. t1-1 are loaded once. The column sums
// accumulate per thread and leave as the CTA's partial row set.
template <int N>
__global__ void __launch_bounds__(kMixMaxC / 4, 3) ln_mix_bwd_kernel(const MixArgs a) {
  __shared__ float2 red[2][kMixMaxC / 128];
  __shared__ float smu[kMixMaxRows + 1], srs[kMixMaxRows + 1];  // rows t0-1 .. t1-1
  extern __shared__ __align__(16) unsigned char mix_dyn[];
  const int c = 4 * threadIdx.x;
  int bi, t0, t1;
  mix_span(a, bi, t0, t1);
  const bool res = a.gres != nullptr;
  const size_t stage = mix_bwd_stage_bytes(N, a.C, res);
  const size_t row0 = (size_t)bi * a.T;
  auto xs = [&](int k) { return reinterpret_cast<float*>(mix_dyn + k * stage) + c; };
  auto rs_ = [&](int k) { return reinterpret_cast<float*>(mix_dyn + k * stage + (size_t)a.C * 4) + c; };
  auto gs = [&](int k, int i) {
    return reinterpret_cast<__nv_bfloat16*>(mix_dyn + k * stage + (size_t)a.C * (res ? 8 : 4)) + (size_t)i * a.C +
           c;
  };
  auto issue = [&](int t) {  // row t into its stage
    const int k = (t - t0) % kMixStages;
    const size_t r = row0 + t;
    if (t < t1) {
      mix_cp16(xs(k), a.x + r * a.C + c);
      if (res) mix_cp16(rs_(k), a.gres + r * a.C + c);
    }
    if (t <= t1 && t < a.T) {
#pragma unroll
      for (int i = 0; i < N; ++i) mix_cp8(gs(k, i), a.gout[i] + r * a.C + c);
    }
    mix_commit();
  };
#pragma unroll 1
  for (int k = 0; k < kMixStages; ++k) issue(t0 + k);
  for (int i = threadIdx.x; i <= t1 - t0; i += blockDim.x) {
    const int t = t0 - 1 + i;
    smu[i] = t >= 0 ? a.mean[row0 + t] : 0.f;
    srs[i] = t >= 0 ? a.rstd[row0 + t] : 0.f;
  }
  const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
  const float4 wv = ld4(a.w + c), bv = ld4(a.b + c);
  float4 m[N];
#pragma unroll
  for (int i = 0; i < N; ++i) m[i] = ld4(a.mix + (size_t)i * a.C + c);
  float4 acc_w = z4, acc_b = z4, acc_m[N];
#pragma unroll
  for (int i = 0; i < N; ++i) acc_m[i] = z4;
  float4 hp = z4;  // h[t-1]
  const float4 xp = t0 > 0 ? ld4(a.x + (row0 + t0 - 1) * a.C + c) : z4;
  __syncthreads();  // the statistics
  if (t0 > 0) hp = mix_norm(xp, smu[0], srs[0], wv, bv);
  const uint2 z2 = make_uint2(0u, 0u);  // four bf16 zeros
  int slot = 0;
#pragma unroll 1
  for (int t = t0; t < t1; ++t) {
    const size_t r = row0 + t;
    const int k = (t - t0) % kMixStages, kn = (t + 1 - t0) % kMixStages;
    mix_wait<kMixStages - 2>();  // rows t and t+1 have landed
    const float4 v = *reinterpret_cast<const float4*>(xs(k));
    const float4 gr = res ? *reinterpret_cast<const float4*>(rs_(k)) : z4;
    uint2 gc[N], gn[N];
#pragma unroll
    for (int i = 0; i < N; ++i) {
      gc[i] = *reinterpret_cast<const uint2*>(gs(k, i));
      gn[i] = t + 1 < a.T ? *reinterpret_cast<const uint2*>(gs(kn, i)) : z2;
    }
    const float mu = smu[t - t0 + 1], rs = srs[t - t0 + 1];

    const float4 h = mix_norm(v, mu, rs, wv, bv);
    const float4 xh = make_float4(__fmul_rn(v.x - mu, rs), __fmul_rn(v.y - mu, rs), __fmul_rn(v.z - mu, rs),
                                  __fmul_rn(v.w - mu, rs));
    float4 d = z4;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      const float4 g = mix_unpack4(gc[i]), gq = mix_unpack4(gn[i]);
      d.x += m[i].x * g.x + (1.f - m[i].x) * gq.x;
      d.y += m[i].y * g.y + (1.f - m[i].y) * gq.y;
      d.z += m[i].z * g.z + (1.f - m[i].z) * gq.z;
      d.w += m[i].w * g.w + (1.f - m[i].w) * gq.w;
      acc_m[i].x += g.x * (h.x - hp.x);
      acc_m[i].y += g.y * (h.y - hp.y);
      acc_m[i].z += g.z * (h.z - hp.z);
      acc_m[i].w += g.w * (h.w - hp.w);
    }
    // stage k is read (its g_i were also row t-1's next row): refill it
    issue(t + kMixStages);
    acc_w.x += d.x * xh.x;
    acc_w.y += d.y * xh.y;
    acc_w.z += d.z * xh.z;
    acc_w.w += d.w * xh.w;
    acc_b.x += d.x;
    acc_b.y += d.y;
    acc_b.z += d.z;
    acc_b.w += d.w;
    const float4 dw = make_float4(d.x * wv.x, d.y * wv.y, d.z * wv.z, d.w * wv.w);
    const float2 s = block_sum2((dw.x + dw.y) + (dw.z + dw.w),
                                (dw.x * xh.x + dw.y * xh.y) + (dw.z * xh.z + dw.w * xh.w), red, slot);
    slot ^= 1;
    const float s1 = s.x / a.C, s2 = s.y / a.C;
    float4 o = make_float4(__fmul_rn(rs, dw.x - s1 - xh.x * s2), __fmul_rn(rs, dw.y - s1 - xh.y * s2),
                           __fmul_rn(rs, dw.z - s1 - xh.z * s2), __fmul_rn(rs, dw.w - s1 - xh.w * s2));
    if (res)  // the skip connection's gradient, one rounded add as autograd's sum
      o = make_float4(__fadd_rn(o.x, gr.x), __fadd_rn(o.y, gr.y), __fadd_rn(o.z, gr.z), __fadd_rn(o.w, gr.w));
    *reinterpret_cast<float4*>(a.gx + r * a.C + c) = o;
    if (a.gx16 != nullptr) {  // round to nearest, as a cast of gx would
      __nv_bfloat162 lo = __floats2bfloat162_rn(o.x, o.y), hi = __floats2bfloat162_rn(o.z, o.w);
      uint2 pk;
      pk.x = *reinterpret_cast<uint32_t*>(&lo);
      pk.y = *reinterpret_cast<uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(a.gx16 + r * a.C + c) = pk;
    }
    hp = h;
  }
  mix_wait<0>();
  float* p = a.partial + (size_t)blockIdx.x * (2 + N) * a.C + c;
  *reinterpret_cast<float4*>(p) = acc_w;
  *reinterpret_cast<float4*>(p + a.C) = acc_b;
#pragma unroll
  for (int i = 0; i < N; ++i) *reinterpret_cast<float4*>(p + (2 + i) * (size_t)a.C) = acc_m[i];
}

// Column sums of the per-CTA partials: out[k][c] for the 2 + n rows k (dw,
// db, dm_i). A CTA of 32 x 32 threads takes 32 columns of one row k; thread
// (y, x) sums the partials j = y (mod 32) of column x into four accumulators
// by j / 32 mod 4 (four independent load chains), adds them in order, then the
// 32 partial sums of a column are added in y order (a fixed order: the result
// does not depend on timing).
__global__ void __launch_bounds__(1024) ln_mix_reduce_kernel(const float* partial, int nchunks, int rows, int C,
                                                             float* gw, float* gb, float* gmix) {
  __shared__ float part[32][33];
  const int k = blockIdx.y;
  const int c = blockIdx.x * 32 + threadIdx.x;
  float s = 0.f;
  if (c < C) {
    const float* col = partial + (size_t)k * C + c;
    const size_t step = (size_t)32 * rows * C;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    int j = threadIdx.y;
    for (; j + 96 < nchunks; j += 128) {
      const float* p = col + (size_t)j * rows * C;
      a0 += p[0];
      a1 += p[step];
      a2 += p[2 * step];
      a3 += p[3 * step];
    }
    for (; j < nchunks; j += 32) a0 += col[(size_t)j * rows * C];
    s = (a0 + a1) + (a2 + a3);
  }
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
