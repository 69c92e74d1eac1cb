// Recurrent (single-token) WKV step for generation: the WKV part of the
// reference's SpikeTimeMix.step, src/spikegpt/language.py:993-1010, on the
// reference's state (numerator, denominator, log_scale with a natural-log
// scale), updated in place.
//
// Per (b, c): with w = -exp(time_decay), u = time_first, s = log_scale,
//   m  = max(s, u + k);  y = (e^{s-m} num + e^{u+k-m} v) / (e^{s-m} den + e^{u+k-m})
//   m' = max(s + w, k);  num = e^{s+w-m'} num + e^{k-m'} v;  den = e^{s+w-m'} den + e^{k-m'};  s = m'
// Arithmetic is float32 whatever the storage types (the reference computes in
// the promoted dtype of its operands; float32 is at least as accurate), with
// the math library's expf and IEEE division. Elementwise and memory-bound: 9
// values move per element (k, v, num, den, s in; y, num, den, s out).
#pragma once

#include "wkv_device.cuh"

namespace wkv {

template <typename T>
struct Conv;
template <>
struct Conv<float> {
  static __device__ __forceinline__ float in(float x) { return x; }
  static __device__ __forceinline__ float out(float x) { return x; }
};
template <>
struct Conv<__nv_bfloat16> {
  static __device__ __forceinline__ float in(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 out(float x) { return __float2bfloat16_rn(x); }
};
template <>
struct Conv<__half> {
  static __device__ __forceinline__ float in(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half out(float x) { return __float2half_rn(x); }
};

struct StepArgs {
  const void* key;
  const void* value;
  const float* time_decay;
  const float* time_first;
  void* num;
  void* den;
  void* log_scale;
  void* y;
  int64_t n;  // B * C
  int C;
};

__device__ __forceinline__ void step1(float k, float v, float w, float u, float& num, float& den,
                                      float& s, float& y) {
  const float uk = u + k;
  const float m = fmaxf(s, uk);
  float a = expf(s - m), e = expf(uk - m);
  y = (a * num + e * v) / (a * den + e);
  const float ds = s + w;
  const float m2 = fmaxf(ds, k);
  a = expf(ds - m2);
  e = expf(k - m2);
  num = a * num + e * v;
  den = a * den + e;
  s = m2;
}

// V consecutive elements per thread per iteration, grid-stride; key/value in
// TK, state and y in TS. With V > 1 the caller guarantees C % V == 0 and
// 16-byte aligned pointers, so every group of V lies in one row and moves with
// 16-byte loads and stores (V * sizeof(TK) == 16 bytes of key; the state takes
// one or two 16-byte words).
template <typename T, int V>
struct VecIO {
  static constexpr int kWords = V * sizeof(T) / 16;
  uint4 w[kWords];
  __device__ __forceinline__ void load(const T* p) {
#pragma unroll
    for (int i = 0; i < kWords; ++i) w[i] = reinterpret_cast<const uint4*>(p)[i];
  }
  __device__ __forceinline__ void store(T* p) const {
#pragma unroll
    for (int i = 0; i < kWords; ++i) reinterpret_cast<uint4*>(p)[i] = w[i];
  }
  __device__ __forceinline__ T* at() { return reinterpret_cast<T*>(w); }
};

template <typename TK, typename TS, int V>
__global__ void __launch_bounds__(256) wkv_step_kernel(const StepArgs a) {
  static_assert(V == 1 || V * sizeof(TK) == 16, "16-byte key vectors");
  using CK = Conv<TK>;
  using CS = Conv<TS>;
  const TK* kp = static_cast<const TK*>(a.key);
  const TK* vp = static_cast<const TK*>(a.value);
  TS* np_ = static_cast<TS*>(a.num);
  TS* dp = static_cast<TS*>(a.den);
  TS* sp = static_cast<TS*>(a.log_scale);
  TS* yp = static_cast<TS*>(a.y);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x * V;
  for (int64_t i0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * V; i0 < a.n; i0 += stride) {
    const int c0 = static_cast<int>(i0 % a.C);
    if constexpr (V == 1) {
      float num = CS::in(np_[i0]), den = CS::in(dp[i0]), s = CS::in(sp[i0]), y;
      step1(CK::in(kp[i0]), CK::in(vp[i0]), -expf(a.time_decay[c0]), a.time_first[c0], num, den, s,
            y);
      yp[i0] = CS::out(y);
      np_[i0] = CS::out(num);
      dp[i0] = CS::out(den);
      sp[i0] = CS::out(s);
    } else {
      VecIO<TK, V> k, v;
      VecIO<TS, V> nu, de, sc, yo;
      k.load(kp + i0);
      v.load(vp + i0);
      nu.load(np_ + i0);
      de.load(dp + i0);
      sc.load(sp + i0);
#pragma unroll
      for (int j = 0; j < V; ++j) {
        float num = CS::in(nu.at()[j]), den = CS::in(de.at()[j]), s = CS::in(sc.at()[j]), y;
        step1(CK::in(k.at()[j]), CK::in(v.at()[j]), -expf(__ldg(a.time_decay + c0 + j)),
              __ldg(a.time_first + c0 + j), num, den, s, y);
        yo.at()[j] = CS::out(y);
        nu.at()[j] = CS::out(num);
        de.at()[j] = CS::out(den);
        sc.at()[j] = CS::out(s);
      }
      yo.store(yp + i0);
      nu.store(np_ + i0);
      de.store(dp + i0);
      sc.store(sp + i0);
    }
  }
}

}  // namespace wkv
