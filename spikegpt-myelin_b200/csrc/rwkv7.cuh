// RWKV-7 DPLR time-mixing recurrence, forward (sm_100a), float32.
//
// The reference has no code for this op (its RWKV-7 experiments called an
// external library); this is the published diagonal-plus-low-rank state
// update, per sequence b and head h with a head_size x head_size state S
// (rows: value channels i, columns: key channels j):
//   S_t = S_{t-1} diag(w_t) + (S_{t-1} a_t) b_t^T + v_t k_t^T,   y_t = S_t r_t,
// S_0 = 0 (or a given initial state), every vector [N] of step t of head h.
// Tensors are [B, T, H, N] float32 (N = 64), the state [B, H, N, N].
//
// Layout: one CTA of 64 threads per (b, h); thread (rb, q) = (tid / 4, tid % 4)
// keeps the 4 x 16 block S[4rb .. 4rb+3][16q .. 16q+15] in registers, so each
// step vector read from shared memory serves four state rows (two rows a
// thread measured slower: twice the shared-memory reads per entry). Per step it
// forms its part of (S a) and of y for its rows, the four partial sums of a
// row meet in two xor shuffles (fixed order), and it updates its 64 entries
// with two fused multiply-adds and a multiply each. The step vectors of
// kChunk steps at a time are staged in shared memory by asynchronous 16-byte
// copies, double-buffered (chunk c+1 lands while chunk c is computed); y
// leaves through shared memory by coalesced float4 stores. Serial in T by
// construction: this is the sequential form of the op on CUDA cores (the
// chunked tensor-core form is not built).
#pragma once

#include "wkv_device.cuh"

namespace wkv {

constexpr int kR7N = 64;           // head size
constexpr int kR7Rows = 4;         // state rows per thread
constexpr int kR7Cols = kR7N / 4;  // state columns per thread
constexpr int kR7Threads = (kR7N / kR7Rows) * 4;
constexpr int kR7Chunk = 8;        // steps staged per pass

struct R7Args {
  const float* r;
  const float* w;
  const float* k;
  const float* v;
  const float* a;
  const float* b;
  const float* s0;  // [B][H][N][N] or null (zero)
  float* y;
  float* s_out;  // [B][H][N][N] or null
  int B, T, H;
};

__device__ __forceinline__ void r7_cp16(float* dst, const float* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

__global__ void __launch_bounds__(kR7Threads) rwkv7_fwd_kernel(const R7Args p) {
  // staged step vectors, two buffers: [r, w, k, a, b, v][kChunk][N]; y [kChunk][N]
  __shared__ __align__(16) float st[2][6][kR7Chunk][kR7N];
  __shared__ __align__(16) float ys[kR7Chunk][kR7N];
  const int tid = threadIdx.x;
  const int rb = tid >> 2, q = tid & 3;
  const int i0 = rb * kR7Rows, j0 = q * kR7Cols;
  const int bh = blockIdx.x, bi = bh / p.H, h = bh % p.H;
  const size_t head = (size_t)h * kR7N;
  const size_t row_stride = (size_t)p.H * kR7N;  // between steps
  const size_t seq = (size_t)bi * p.T * row_stride;
  float S[kR7Rows][kR7Cols];
#pragma unroll
  for (int r = 0; r < kR7Rows; ++r) {
    const float* s0 = p.s0 != nullptr ? p.s0 + ((size_t)bh * kR7N + i0 + r) * kR7N + j0 : nullptr;
#pragma unroll
    for (int j = 0; j < kR7Cols; ++j) S[r][j] = s0 != nullptr ? s0[j] : 0.f;
  }
  const float* src[6] = {p.r, p.w, p.k, p.a, p.b, p.v};
  const int nch = (p.T + kR7Chunk - 1) / kR7Chunk;
  // 6 x kChunk x 16 float4 per chunk over the CTA: thread -> float4 column
  // tid % 16, steps tid / 16 + kR7Threads / 16 * m
  constexpr int kSteps = kR7Threads / 16;  // steps one pass of the CTA covers
  auto issue = [&](int c) {
    const int col = 4 * (tid & 15);
#pragma unroll
    for (int m = 0; m < kR7Chunk / kSteps; ++m) {
      const int u = (tid >> 4) + kSteps * m, t = c * kR7Chunk + u;
      if (t < p.T) {
#pragma unroll
        for (int s6 = 0; s6 < 6; ++s6)
          r7_cp16(&st[c & 1][s6][u][col], src[s6] + seq + (size_t)t * row_stride + head + col);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  if (nch > 0) issue(0);
#pragma unroll 1
  for (int c = 0; c < nch; ++c) {
    const int t0 = c * kR7Chunk, n = min(kR7Chunk, p.T - t0);
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();  // chunk c landed; chunk c-1's buffer and y are consumed
    if (c + 1 < nch) issue(c + 1);
    float(*sv)[kR7Chunk][kR7N] = st[c & 1];
#pragma unroll 1
    for (int u = 0; u < n; ++u) {
      const float* rr = &sv[0][u][j0];
      const float* ww = &sv[1][u][j0];
      const float* kk = &sv[2][u][j0];
      const float* aa = &sv[3][u][j0];
      const float* bb = &sv[4][u][j0];
      const float4 v4 = *reinterpret_cast<const float4*>(&sv[5][u][i0]);
      const float vi[kR7Rows] = {v4.x, v4.y, v4.z, v4.w};
      // (S a) for the rows over this thread's columns (two chains a row),
      // then over the row's four column blocks
      float sa[kR7Rows];
#pragma unroll
      for (int r = 0; r < kR7Rows; ++r) {
        float e = 0.f, o = 0.f;
#pragma unroll
        for (int j = 0; j < kR7Cols; j += 2) {
          e = fmaf(S[r][j], aa[j], e);
          o = fmaf(S[r][j + 1], aa[j + 1], o);
        }
        sa[r] = e + o;
      }
#pragma unroll
      for (int r = 0; r < kR7Rows; ++r) {
        sa[r] += __shfl_xor_sync(0xffffffffu, sa[r], 1);
        sa[r] += __shfl_xor_sync(0xffffffffu, sa[r], 2);
      }
      float y[kR7Rows];
#pragma unroll
      for (int r = 0; r < kR7Rows; ++r) {
        float e = 0.f, o = 0.f;
#pragma unroll
        for (int j = 0; j < kR7Cols; j += 2) {
          S[r][j] = fmaf(vi[r], kk[j], fmaf(S[r][j], ww[j], sa[r] * bb[j]));
          S[r][j + 1] = fmaf(vi[r], kk[j + 1], fmaf(S[r][j + 1], ww[j + 1], sa[r] * bb[j + 1]));
          e = fmaf(S[r][j], rr[j], e);
          o = fmaf(S[r][j + 1], rr[j + 1], o);
        }
        y[r] = e + o;
      }
#pragma unroll
      for (int r = 0; r < kR7Rows; ++r) {
        y[r] += __shfl_xor_sync(0xffffffffu, y[r], 1);
        y[r] += __shfl_xor_sync(0xffffffffu, y[r], 2);
      }
      if (q == 0) *reinterpret_cast<float4*>(&ys[u][i0]) = make_float4(y[0], y[1], y[2], y[3]);
    }
    __syncthreads();
#pragma unroll
    for (int m = 0; m < kR7Chunk / kSteps; ++m) {
      const int u = (tid >> 4) + kSteps * m, col = 4 * (tid & 15);
      if (u < n)
        *reinterpret_cast<float4*>(p.y + seq + (size_t)(t0 + u) * row_stride + head + col) =
            *reinterpret_cast<const float4*>(&ys[u][col]);
    }
  }
  if (p.s_out != nullptr) {
#pragma unroll
    for (int r = 0; r < kR7Rows; ++r) {
      float* so = p.s_out + ((size_t)bh * kR7N + i0 + r) * kR7N + j0;
#pragma unroll
      for (int j = 0; j < kR7Cols; ++j) so[j] = S[r][j];
    }
  }
}

}  // namespace wkv
