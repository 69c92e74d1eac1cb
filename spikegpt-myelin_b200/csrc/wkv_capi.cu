// C ABI of libspikegpt_wkv.so (declared in include/spikegpt_wkv.h).
//
// Host side: argument validation, the execution plan (TMA vs generic tiles,
// number of time segments), the caller-provided workspace carve-up, TMA
// descriptor encoding, and the kernel launch sequence. Every entry point is
// asynchronous on the caller's stream and allocates nothing.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <initializer_list>
#include <mutex>
#include <type_traits>
#include <vector>

#include "spikegpt_wkv.h"
#include "gates.cuh"
#include "lif.cuh"
#include "ln_mix.cuh"
#include "rwkv7.cuh"
#include "xent.cuh"
#include "wkv_step.cuh"
#include "wkv_tp.cuh"

namespace {

using namespace wkv;

thread_local char g_last_error[512] = "";
std::atomic<int> g_force_segments{0};
std::atomic<int> g_force_generic{0};
std::atomic<int> g_force_slow{0};
std::atomic<long long> g_wait_limit{kWaitLimitCycles};
std::atomic<int> g_withhold_first{0};

__device__ unsigned g_device_error_flags = 0;

// ------------------------------------------------ launch accounting / timing
//
// Every kernel launch goes through launch(): it bumps a per-kind counter and,
// while timing is enabled, brackets the launch with CUDA events recorded on the
// launch stream, so per-kernel device time can be read back by the caller.

enum Kind {
  K_FWD_Y, K_FWD_STATE, K_BWD_GRAD, K_BWD_ADJ, K_CARRY_FWD, K_CARRY_ADJ, K_STEP, K_LIF_FWD, K_LIF_BWD,
  K_MIX_FWD, K_MIX_BWD, K_MIX_RED,
  K_GATE_FWD, K_GATE_BWD, K_RSQ_FWD, K_RSQ_BWD, K_RESID, K_LIF_SUM, K_R7_FWD, K_XENT_FWD, K_XENT_BWD,
  K_COUNT
};
const char* const kKindNames[K_COUNT] = {
    "wkv_fwd_kernel<y>",      "wkv_fwd_kernel<state>", "wkv_bwd_kernel<grad>",
    "wkv_bwd_kernel<adjoint>", "wkv_carry_fwd_kernel",  "wkv_carry_adj_kernel",
    "wkv_step_kernel",        "lif_fwd_kernel",        "lif_bwd_kernel",
    "ln_mix_fwd_kernel",      "ln_mix_bwd_kernel",     "ln_mix_reduce_kernel",
    "gate_fwd_kernel",        "gate_bwd_kernel",       "relu_square_fwd_kernel",
    "relu_square_bwd_kernel", "residual_add_kernel",   "lif_bwd_summary_kernel",
    "rwkv7_fwd_kernel",       "xent_fwd_kernel",       "xent_bwd_kernel"};

std::atomic<long long> g_launches[K_COUNT];
std::atomic<bool> g_timing{false};
std::mutex g_timing_mu;
struct TimedLaunch {
  int kind;
  cudaEvent_t start, stop;
};
std::vector<TimedLaunch> g_timed;
std::vector<cudaEvent_t> g_event_pool;

cudaEvent_t pooled_event() {
  std::lock_guard<std::mutex> lk(g_timing_mu);
  if (!g_event_pool.empty()) {
    cudaEvent_t e = g_event_pool.back();
    g_event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

template <class F>
void launch(int kind, cudaStream_t st, F&& f) {
  g_launches[kind].fetch_add(1, std::memory_order_relaxed);
  if (!g_timing.load(std::memory_order_relaxed)) {
    f();
    return;
  }
  cudaEvent_t a = pooled_event(), b = pooled_event();
  if (a) cudaEventRecord(a, st);
  f();
  if (b) cudaEventRecord(b, st);
  if (a && b) {
    std::lock_guard<std::mutex> lk(g_timing_mu);
    g_timed.push_back(TimedLaunch{kind, a, b});
  }
}

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(WKV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

size_t dtype_size(int dtype) {
  switch (dtype) {
    case WKV_DTYPE_F32: return 4;
    case WKV_DTYPE_BF16: return 2;
    case WKV_DTYPE_F16: return 2;
    default: return 0;
  }
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

struct Plan {
  bool tma;
  int nseg;
  int seg_len;
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Segments (the chunked two-level scan across CTAs) against one sequential
// sweep per lane set, chosen from a sweep of measured step times (forward +
// backward, B200, C = 512, bf16, T in {1024, 3072}, B from 1 to 24, segment
// counts from 1 to 24). A CTA covers one (batch row, 64-channel block,
// segment); about 512 CTAs (3.46 per SM: the resident limit of the
// time-parallel kernels is 4) fill the GPU. Segmenting adds a state sweep and
// an adjoint sweep (the TMA kernels fold the segment summaries themselves),
// which pays when the sweep alone leaves most SMs idle: at T = 1024 up to 96
// lane sets (B = 12: 98 us with 6 segments against 111 us with one), not at
// 192 (B = 24: 116 us with one, 144 us with 3); at T = 3072 down to 192 lane
// sets (B = 24: 262 us with 3 against 295 us). The segment count is then
// 512 / lane sets rounded up, at most 16 and with segments of at least 128
// steps (the measured best within 3 % on every swept shape).
Plan make_plan(int dtype, int64_t B, int64_t T, int64_t C, bool ptrs_aligned) {
  Plan p;
  const size_t es = dtype_size(dtype);
  p.tma = g_force_generic.load() == 0 && ptrs_aligned && (C * (int64_t)es) % 16 == 0;
  const int64_t sets = B * ((C + kLanes - 1) / kLanes);  // CTAs of one sweep
  const int64_t want = (int64_t)sm_count() * 346 / 100;     // 512 on 148 SMs
  int64_t nseg = 1;
  if (sets > 0 && sets < want && (T >= 2048 || sets <= 96)) nseg = (want + sets - 1) / sets;
  const int64_t max_seg = std::min<int64_t>(16, T / 128);
  if (nseg > max_seg) nseg = max_seg;
  if (g_force_segments.load() > 0) nseg = g_force_segments.load();
  if (nseg < 1) nseg = 1;
  if (nseg == 1) {
    p.nseg = 1;
    p.seg_len = static_cast<int>(T);
  } else {
    int64_t len = (T + nseg - 1) / nseg;
    len = (len + kSegAlign - 1) / kSegAlign * kSegAlign;
    p.seg_len = static_cast<int>(len);
    p.nseg = static_cast<int>((T + len - 1) / len);
    if (p.nseg == 1) p.seg_len = static_cast<int>(T);
  }
  return p;
}

constexpr size_t kAlign = 256;
size_t round_up(size_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

struct FwdWs {
  float* seg;
  size_t bytes;
};
FwdWs fwd_workspace(const Plan& p, int64_t B, int64_t C, void* base) {
  FwdWs w{nullptr, 0};
  if (p.nseg > 1) {
    w.bytes = round_up((size_t)B * p.nseg * 3 * C * sizeof(float));
    w.seg = static_cast<float*>(base);
  }
  return w;
}

struct BwdWs {
  float* ckpt;
  float* seg;
  float* adj;
  float* partial;
  unsigned* tickets;
  size_t bytes;
};
BwdWs bwd_workspace(const Plan& p, int64_t B, int64_t T, int64_t C, void* base) {
  BwdWs w{};
  char* cur = static_cast<char*>(base);
  auto take = [&](size_t n) {
    char* r = cur;
    const size_t sz = round_up(n);
    if (cur) cur += sz;
    w.bytes += sz;
    return reinterpret_cast<float*>(r);
  };
  const int64_t nsub = (T + kSub - 1) / kSub;
  w.ckpt = take((size_t)B * nsub * 3 * C * sizeof(float));
  if (p.nseg > 1) {
    w.seg = take((size_t)B * p.nseg * 3 * C * sizeof(float));
    w.adj = take((size_t)B * p.nseg * 5 * C * sizeof(float));
  }
  w.partial = take((size_t)B * p.nseg * 2 * C * sizeof(float));
  w.tickets = reinterpret_cast<unsigned*>(take((size_t)((C + kLanes - 1) / kLanes) * sizeof(unsigned)));
  if (!base) {
    w.ckpt = w.seg = w.adj = w.partial = nullptr;
    w.tickets = nullptr;
  }
  return w;
}

// ------------------------------------------------------------ TMA descriptors

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// [B, T, C] tensor as a 3-D map with dims {C, T, B} and a [1][rows][cols] box,
// rows = box_rows, or the dtype's tile height (Pair<T>::kTileRows) when 0.
int make_map(CUtensorMap* m, int dtype, const void* ptr, int64_t B, int64_t T, int64_t C,
             int box_rows = 0, int box_cols = kLanes) {
  std::memset(m, 0, sizeof(*m));
  if (ptr == nullptr) return WKV_OK;
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(WKV_ERR_DRIVER, "cuTensorMapEncodeTiled is not available");
  const size_t es = dtype_size(dtype);
  const CUtensorMapDataType dt = dtype == WKV_DTYPE_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == WKV_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)T, (cuuint64_t)B};
  const cuuint64_t strides[2] = {(cuuint64_t)(C * es), (cuuint64_t)(T * C * es)};
  const cuuint32_t rows = box_rows > 0                 ? (cuuint32_t)box_rows
                          : dtype == WKV_DTYPE_F32 ? Pair<float>::kTileRows
                                                   : Pair<__half>::kTileRows;
  const cuuint32_t box[3] = {(cuuint32_t)box_cols, rows, 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUresult r = fn(m, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(WKV_ERR_DRIVER, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return WKV_OK;
}

// Checkpoint rows [rows][3][C] float32 as a 3-D map with dims {C, 3, rows} and a
// [tiles][3][kLanes] box (the checkpoints of `tiles` consecutive tiles).
int make_ckpt_map(CUtensorMap* m, const float* ptr, int64_t rows, int64_t C, int tiles,
                  int box_cols = kLanes) {
  std::memset(m, 0, sizeof(*m));
  if (ptr == nullptr) return WKV_OK;
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(WKV_ERR_DRIVER, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[3] = {(cuuint64_t)C, 3u, (cuuint64_t)rows};
  const cuuint64_t strides[2] = {(cuuint64_t)(C * 4), (cuuint64_t)(3 * C * 4)};
  const cuuint32_t box[3] = {(cuuint32_t)box_cols, 3u, (cuuint32_t)tiles};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(ptr), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(WKV_ERR_DRIVER, "cuTensorMapEncodeTiled (checkpoints) failed (%d)", (int)r);
  return WKV_OK;
}

// The current CUDA context (driver API through the runtime's entry-point
// query, so the library needs no -lcuda). Device addresses of this module's
// __device__ symbols are cached per (device, context): a device reset creates
// a new primary context, reloads the module and moves the symbols.
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CUcontext current_context() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  CUcontext c = nullptr;
  if (fn == nullptr || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

struct SymbolCache {
  std::mutex mu;
  CUcontext ctx[64] = {};
  void* ptr[64] = {};
};

// Device address of `symbol` in the current context, looked up with
// cudaGetSymbolAddress when the device's context differs from the cached one.
template <class S>
cudaError_t symbol_address(SymbolCache& cache, const S& symbol, void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  // (null before the runtime has bound a context to this thread: the lookup
  // below binds one, and the next call caches again under the real context)
  const CUcontext ctx = current_context();
  std::lock_guard<std::mutex> lk(cache.mu);
  if (cache.ptr[dev] == nullptr || cache.ctx[dev] != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, symbol);
    if (e != cudaSuccess) return e;
    cache.ptr[dev] = p;
    cache.ctx[dev] = ctx;
  }
  *out = cache.ptr[dev];
  return cudaSuccess;
}

// Device address of g_device_error_flags for the current device and context
// (the host-side symbol itself is not a device address).
SymbolCache g_err_cache;
unsigned* device_err_ptr() {
  void* p = nullptr;
  if (symbol_address(g_err_cache, g_device_error_flags, &p) != cudaSuccess) return nullptr;
  return static_cast<unsigned*>(p);
}

int check_dims(int dtype, int64_t B, int64_t T, int64_t C) {
  if (dtype_size(dtype) == 0) return fail(WKV_ERR_INVALID_ARGUMENT, "unknown dtype code %d", dtype);
  if (B < 0 || T < 0 || C < 0)
    return fail(WKV_ERR_INVALID_ARGUMENT, "negative size B=%lld T=%lld C=%lld", (long long)B,
                (long long)T, (long long)C);
  if (T > (1ll << 30) || C > (1ll << 30) || B > (1ll << 30) || B * ((C + 31) / 32) > (1ll << 31) - 1)
    return fail(WKV_ERR_INVALID_ARGUMENT, "size out of range B=%lld T=%lld C=%lld", (long long)B,
                (long long)T, (long long)C);
  return WKV_OK;
}

// Kernels whose dynamic shared memory exceeds the 48 KB default opt in once per
// device.
template <typename K>
cudaError_t allow_smem(K* kernel, size_t bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  static std::mutex mu;
  static std::vector<std::pair<const void*, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(mu);
  for (auto& d : done)
    if (d.first == reinterpret_cast<const void*>(kernel) && d.second == dev) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess) done.emplace_back(reinterpret_cast<const void*>(kernel), dev);
  return e;
}

// ----------------------------------------------------------- launch helpers


template <typename IO>
int launch_forward(const void* k, const void* v, const float* decay, int decay_is_w,
                   const float* u, void* y, int B, int T, int C, const Plan& p, float* seg,
                   float* state, unsigned* state_tickets, cudaStream_t st) {
  CUtensorMap mk, mv, my;
  const int dt = sizeof(IO) == 4 ? WKV_DTYPE_F32
                 : std::is_same<IO, __nv_bfloat16>::value ? WKV_DTYPE_BF16
                                                         : WKV_DTYPE_F16;
  constexpr int TW = tp_warps<IO>();
  int rc;
  if (p.tma) {
    if ((rc = make_map(&mk, dt, k, B, T, C, Tp<IO, TW>::kRoundRows)) ||
        (rc = make_map(&mv, dt, v, B, T, C, Tp<IO, TW>::kRoundRows)) ||
        (rc = make_map(&my, dt, y, B, T, C, kSub)))
      return rc;
  } else {
    std::memset(&mk, 0, sizeof(mk));
    std::memset(&mv, 0, sizeof(mv));
    std::memset(&my, 0, sizeof(my));
  }
  FwdArgs a{};
  a.k = k;
  a.v = v;
  a.y = y;
  a.decay = decay;
  a.u = u;
  a.decay_is_w = decay_is_w;
  a.B = B;
  a.T = T;
  a.C = C;
  a.ncblk = (C + kLanes - 1) / kLanes;
  a.seg_len = p.seg_len;
  a.nseg = p.nseg;
  a.nsub = (T + kSub - 1) / kSub;
  a.force_slow = g_force_slow.load();
  a.err = device_err_ptr();
  a.wait_limit = g_wait_limit.load();
  a.withhold_first = g_withhold_first.load();
  const unsigned gx = (unsigned)a.ncblk * (unsigned)B;
  if (p.nseg > 1) {
    // summaries of segments 0..nseg-2, then the carry
    FwdArgs s = a;
    s.seg_end = seg;
    if (p.tma) {
      const size_t sm = fwd_tp_smem_bytes<IO, TW>();
      const cudaError_t e = allow_smem(wkv_fwd_tp_kernel<IO, TW, false>, sm);
      if (e != cudaSuccess) return cuda_fail(e, "setting the forward kernel's shared memory size");
      launch(K_FWD_STATE, st, [&] {
        wkv_fwd_tp_kernel<IO, TW, false><<<dim3(gx, p.nseg - 1), 32 * TW, sm, st>>>(s, mk, mv, my);
      });
    } else {
      const size_t sm = fwd_smem_bytes<IO>(false);
      launch(K_FWD_STATE, st, [&] {
        wkv_fwd_kernel<IO, false, false><<<dim3(gx, p.nseg - 1), kThreads, sm, st>>>(s, mk, mv, my);
      });
    }
    if (p.tma) {
      a.seg_sums = seg;  // each CTA folds the summaries before its segment itself
    } else {
      const int64_t lanes = (int64_t)B * C;
      launch(K_CARRY_FWD, st, [&] {
        wkv_carry_fwd_kernel<<<(unsigned)((lanes + 127) / 128), 128, 0, st>>>(
            seg, decay, decay_is_w, B, T, C, p.nseg, p.seg_len);
      });
      a.seg_start = seg;
    }
  }
  // The main pass starts every segment from its true state, so the checkpoints
  // it writes are true states; it also zeroes the backward's arrival counters.
  a.ckpt = state;
  a.zero_tickets = state_tickets;
  a.nzero = state_tickets ? a.ncblk : 0;
  if (p.tma) {
    const size_t sm = fwd_tp_smem_bytes<IO, TW>();
    const cudaError_t e = allow_smem(wkv_fwd_tp_kernel<IO, TW, true>, sm);
    if (e != cudaSuccess) return cuda_fail(e, "setting the forward kernel's shared memory size");
    launch(K_FWD_Y, st, [&] {
      wkv_fwd_tp_kernel<IO, TW, true><<<dim3(gx, p.nseg), 32 * TW, sm, st>>>(a, mk, mv, my);
    });
  } else {
    const size_t sm = fwd_smem_bytes<IO>(true);
    launch(K_FWD_Y, st, [&] {
      wkv_fwd_kernel<IO, true, false><<<dim3(gx, p.nseg), kThreads, sm, st>>>(a, mk, mv, my);
    });
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "wkv forward launch");
  return WKV_OK;
}

template <typename IO>
int launch_backward(const void* gy, const float* w, const float* u, const void* k, const void* v,
                    void* gk, void* gv, float* gtd, float* gtf, int B, int T, int C,
                    const Plan& p, const BwdWs& ws, const float* state,
                    unsigned* state_tickets, cudaStream_t st) {
  const int dt = sizeof(IO) == 4 ? WKV_DTYPE_F32
                 : std::is_same<IO, __nv_bfloat16>::value ? WKV_DTYPE_BF16
                                                         : WKV_DTYPE_F16;
  constexpr int BW = tp_bwd_warps<IO>();
  CUtensorMap mk, mv, mgy, mck, mgk, mgv, none;
  std::memset(&none, 0, sizeof(none));
  const int ncblk = (C + kLanes - 1) / kLanes;
  const int nsub = (T + kSub - 1) / kSub;
  const float* ckpt = state ? state : ws.ckpt;
  int rc;
  if (p.tma) {
    constexpr int rows = TpB<IO, BW>::kRoundRows;
    if ((rc = make_map(&mk, dt, k, B, T, C, rows)) || (rc = make_map(&mv, dt, v, B, T, C, rows)) ||
        (rc = make_map(&mgy, dt, gy, B, T, C, rows)) ||
        (rc = make_ckpt_map(&mck, ckpt, (int64_t)B * nsub, C, BW)) ||
        (rc = make_map(&mgk, dt, gk, B, T, C, kSub)) || (rc = make_map(&mgv, dt, gv, B, T, C, kSub)))
      return rc;
  } else {
    mk = mv = mgy = mck = mgk = mgv = none;
  }
  const unsigned gx = (unsigned)ncblk * (unsigned)B;
  unsigned* err = device_err_ptr();
  const int force_slow = g_force_slow.load();

  // 1. forward state sweep: checkpoints at every sub-chunk start (+ segment ends)
  FwdArgs f{};
  f.k = k;
  f.v = v;
  f.decay = w;
  f.u = u;
  f.decay_is_w = 1;
  f.B = B;
  f.T = T;
  f.C = C;
  f.ncblk = ncblk;
  f.seg_len = p.seg_len;
  f.nseg = p.nseg;
  f.nsub = nsub;
  f.ckpt = ws.ckpt;
  f.seg_end = p.nseg > 1 ? ws.seg : nullptr;
  f.zero_tickets = ws.tickets;
  f.nzero = ncblk;
  f.force_slow = force_slow;
  f.err = err;
  if (state == nullptr) {
    if (p.tma) {
      constexpr int TW = tp_warps<IO>();
      CUtensorMap rk, rv;
      if ((rc = make_map(&rk, dt, k, B, T, C, Tp<IO, TW>::kRoundRows)) ||
          (rc = make_map(&rv, dt, v, B, T, C, Tp<IO, TW>::kRoundRows)))
        return rc;
      const size_t fsm = fwd_tp_smem_bytes<IO, TW>();
      const cudaError_t e = allow_smem(wkv_fwd_tp_kernel<IO, TW, false>, fsm);
      if (e != cudaSuccess) return cuda_fail(e, "setting the forward kernel's shared memory size");
      launch(K_FWD_STATE, st, [&] {
        wkv_fwd_tp_kernel<IO, TW, false><<<dim3(gx, p.nseg), 32 * TW, fsm, st>>>(f, rk, rv, none);
      });
    } else {
      const size_t fsm = fwd_smem_bytes<IO>(false);
      launch(K_FWD_STATE, st, [&] {
        wkv_fwd_kernel<IO, false, false><<<dim3(gx, p.nseg), kThreads, fsm, st>>>(f, mk, mv, none);
      });
    }
  }

  BwdArgs a{};
  a.k = k;
  a.v = v;
  a.gy = gy;
  a.gk = gk;
  a.gv = gv;
  a.w = w;
  a.u = u;
  a.B = B;
  a.T = T;
  a.C = C;
  a.ncblk = ncblk;
  a.seg_len = p.seg_len;
  a.nseg = p.nseg;
  a.nsub = nsub;
  a.ckpt = ckpt;
  a.force_slow = force_slow;
  a.err = err;
  const int64_t lanes = (int64_t)B * C;
  const unsigned cgrid = (unsigned)((lanes + 127) / 128);
  if (p.nseg > 1) {
    // 2. segment start states (only when the checkpoints are segment-local);
    // 3. adjoint summaries of segments 1..nseg-1; 4. adjoint at every segment end
    // (TMA kernels fold the summaries themselves; the generic ones take the
    // carried states)
    if (state == nullptr && !p.tma)
      launch(K_CARRY_FWD, st, [&] {
        wkv_carry_fwd_kernel<<<cgrid, 128, 0, st>>>(ws.seg, w, 1, B, T, C, p.nseg, p.seg_len);
      });
    BwdArgs s = a;
    if (p.tma)
      s.seg_sums = state ? nullptr : ws.seg;
    else
      s.seg_start = state ? nullptr : ws.seg;
    s.seg_base = 1;
    s.adj_out = ws.adj;
    if (p.tma) {
      const size_t ssm = bwd_tp_smem_bytes<IO, BW>();
      const cudaError_t e = allow_smem(wkv_bwd_tp_kernel<IO, BW, false>, ssm);
      if (e != cudaSuccess) return cuda_fail(e, "setting the backward kernel's shared memory size");
      launch(K_BWD_ADJ, st, [&] {
        wkv_bwd_tp_kernel<IO, BW, false>
            <<<dim3(gx, p.nseg - 1), 32 * BW, ssm, st>>>(s, mk, mv, mgy, mck, none, none);
      });
    } else {
      const size_t ssm = bwd_smem_bytes<IO>(false);
      launch(K_BWD_ADJ, st, [&] {
        wkv_bwd_kernel<IO, false, false>
            <<<dim3(gx, p.nseg - 1), kThreads, ssm, st>>>(s, mk, mv, mgy, none, none);
      });
    }
    if (p.tma) {
      a.seg_sums = state ? nullptr : ws.seg;
      a.adj_sums = ws.adj;
    } else {
      launch(K_CARRY_ADJ, st, [&] {
        wkv_carry_adj_kernel<<<cgrid, 128, 0, st>>>(ws.adj, w, B, T, C, p.nseg, p.seg_len);
      });
      a.seg_start = state ? nullptr : ws.seg;
      a.adj_in = ws.adj;
    }
  }
  // 5. reverse sweep writing grad_key / grad_value and per-lane partials; the
  // last CTA of each column block reduces the partials into the time gradients
  a.partial = ws.partial;
  a.tickets = state ? state_tickets : ws.tickets;
  a.gtd = gtd;
  a.gtf = gtf;
  if (p.tma) {
    const size_t bsm = bwd_tp_smem_bytes<IO, BW>();
    const cudaError_t e = allow_smem(wkv_bwd_tp_kernel<IO, BW, true>, bsm);
    if (e != cudaSuccess) return cuda_fail(e, "setting the backward kernel's shared memory size");
    launch(K_BWD_GRAD, st, [&] {
      wkv_bwd_tp_kernel<IO, BW, true>
          <<<dim3(gx, p.nseg), 32 * BW, bsm, st>>>(a, mk, mv, mgy, mck, mgk, mgv);
    });
  } else {
    const size_t bsm = bwd_smem_bytes<IO>(true);
    const cudaError_t e = allow_smem(wkv_bwd_kernel<IO, true, false>, bsm);
    if (e != cudaSuccess) return cuda_fail(e, "setting the backward kernel's shared memory size");
    launch(K_BWD_GRAD, st, [&] {
      wkv_bwd_kernel<IO, true, false>
          <<<dim3(gx, p.nseg), kThreads, bsm, st>>>(a, mk, mv, mgy, none, none);
    });
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "wkv backward launch");
  return WKV_OK;
}

}  // namespace

extern "C" {

int wkv_abi_version(void) { return WKV_ABI_VERSION; }

const char* wkv_status_string(int status) {
  switch (status) {
    case WKV_OK: return "ok";
    case WKV_ERR_INVALID_ARGUMENT: return "invalid argument";
    case WKV_ERR_WORKSPACE_TOO_SMALL: return "workspace too small";
    case WKV_ERR_CUDA: return "CUDA error";
    case WKV_ERR_DRIVER: return "CUDA driver (TMA descriptor) error";
    default: return "unknown status";
  }
}

const char* wkv_last_error(void) { return g_last_error; }

int wkv_set_debug_overrides(int force_segments, int force_generic, int force_slow) {
  g_force_segments.store(force_segments > 0 ? force_segments : 0);
  g_force_generic.store(force_generic != 0);
  g_force_slow.store(force_slow != 0);
  return WKV_OK;
}

int wkv_set_debug_pipeline(long long wait_limit_cycles, int withhold_first_copies) {
  g_last_error[0] = '\0';
  if (wait_limit_cycles < 0) return fail(WKV_ERR_INVALID_ARGUMENT, "negative wait limit");
  g_wait_limit.store(wait_limit_cycles == 0 ? kWaitLimitCycles : wait_limit_cycles);
  g_withhold_first.store(withhold_first_copies != 0);
  return WKV_OK;
}

int wkv_plan(int dtype, int64_t B, int64_t T, int64_t C, int* tma, int* segments) {
  int rc = check_dims(dtype, B, T, C);
  if (rc) return rc;
  const Plan p = make_plan(dtype, B, T, C, true);
  if (tma) *tma = p.tma ? 1 : 0;
  if (segments) *segments = p.nseg;
  return WKV_OK;
}

size_t wkv_forward_workspace_size(int dtype, int64_t B, int64_t T, int64_t C) {
  if (check_dims(dtype, B, T, C)) return 0;
  const Plan p = make_plan(dtype, B, T, C, true);
  return fwd_workspace(p, B, C, nullptr).bytes;
}

size_t wkv_backward_workspace_size(int dtype, int64_t B, int64_t T, int64_t C) {
  if (check_dims(dtype, B, T, C)) return 0;
  const Plan p = make_plan(dtype, B, T, C, true);
  return bwd_workspace(p, B, T, C, nullptr).bytes;
}

}  // extern "C"

namespace {

// Saved forward state: checkpoint rows [B][ceil(T/kSub)][3][C] floats, then one
// arrival counter per 64-channel block.
struct StateLayout {
  size_t ckpt_bytes, bytes;
};
StateLayout state_layout(int64_t B, int64_t T, int64_t C) {
  StateLayout l;
  const int64_t nsub = (T + kSub - 1) / kSub;
  l.ckpt_bytes = round_up((size_t)B * nsub * 3 * C * sizeof(float));
  l.bytes = l.ckpt_bytes + round_up((size_t)((C + kLanes - 1) / kLanes) * sizeof(unsigned));
  return l;
}

int forward_impl(int dtype, const void* key, const void* value, const float* time_decay,
                 const float* time_first, void* y, float* state, size_t state_bytes, int64_t B,
                 int64_t T, int64_t C, void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error[0] = '\0';
  int rc = check_dims(dtype, B, T, C);
  if (rc) return rc;
  if (B == 0 || T == 0 || C == 0) return WKV_OK;
  if (!key || !value || !time_decay || !time_first || !y)
    return fail(WKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  const bool al = aligned16(key) && aligned16(value) && aligned16(y);
  const Plan p = make_plan(dtype, B, T, C, al);
  const FwdWs need = fwd_workspace(p, B, C, workspace);
  if (need.bytes > 0 && (workspace == nullptr || workspace_bytes < need.bytes))
    return fail(WKV_ERR_WORKSPACE_TOO_SMALL, "forward needs %zu workspace bytes, got %zu",
                need.bytes, workspace_bytes);
  unsigned* state_tickets = nullptr;
  if (state != nullptr) {
    const StateLayout sl = state_layout(B, T, C);
    if (state_bytes < sl.bytes)
      return fail(WKV_ERR_WORKSPACE_TOO_SMALL, "state needs %zu bytes, got %zu", sl.bytes, state_bytes);
    if (!aligned16(state)) return fail(WKV_ERR_INVALID_ARGUMENT, "state must be 16-byte aligned");
    state_tickets = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(state) + sl.ckpt_bytes);
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int b = (int)B, t = (int)T, c = (int)C;
  switch (dtype) {
    case WKV_DTYPE_F32:
      return launch_forward<float>(key, value, time_decay, 0, time_first, y, b, t, c, p, need.seg,
                                   state, state_tickets, st);
    case WKV_DTYPE_BF16:
      return launch_forward<__nv_bfloat16>(key, value, time_decay, 0, time_first, y, b, t, c, p,
                                           need.seg, state, state_tickets, st);
    default:
      return launch_forward<__half>(key, value, time_decay, 0, time_first, y, b, t, c, p, need.seg,
                                    state, state_tickets, st);
  }
}

int backward_impl(int dtype, const void* grad_y, const float* w, const float* u, const void* key,
                  const void* value, const float* state, size_t state_bytes, void* grad_key,
                  void* grad_value, float* grad_time_decay, float* grad_time_first, int64_t B,
                  int64_t T, int64_t C, void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error[0] = '\0';
  int rc = check_dims(dtype, B, T, C);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (C > 0 && (B == 0 || T == 0)) {
    if (!grad_time_decay || !grad_time_first)
      return fail(WKV_ERR_INVALID_ARGUMENT, "null gradient pointer");
    cudaError_t e = cudaMemsetAsync(grad_time_decay, 0, C * sizeof(float), st);
    if (e == cudaSuccess) e = cudaMemsetAsync(grad_time_first, 0, C * sizeof(float), st);
    return e == cudaSuccess ? WKV_OK : cuda_fail(e, "zeroing time gradients");
  }
  if (B == 0 || T == 0 || C == 0) return WKV_OK;
  if (!grad_y || !w || !u || !key || !value || !grad_key || !grad_value || !grad_time_decay ||
      !grad_time_first)
    return fail(WKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  const bool al = aligned16(grad_y) && aligned16(key) && aligned16(value) && aligned16(grad_key) &&
                  aligned16(grad_value);
  const Plan p = make_plan(dtype, B, T, C, al);
  const BwdWs need = bwd_workspace(p, B, T, C, nullptr);
  if (workspace == nullptr || workspace_bytes < need.bytes)
    return fail(WKV_ERR_WORKSPACE_TOO_SMALL, "backward needs %zu workspace bytes, got %zu",
                need.bytes, workspace_bytes);
  if (!aligned16(workspace))
    return fail(WKV_ERR_INVALID_ARGUMENT, "workspace must be 16-byte aligned");
  const BwdWs ws = bwd_workspace(p, B, T, C, workspace);
  unsigned* state_tickets = nullptr;
  if (state != nullptr) {
    const StateLayout sl = state_layout(B, T, C);
    if (state_bytes < sl.bytes)
      return fail(WKV_ERR_WORKSPACE_TOO_SMALL, "state needs %zu bytes, got %zu", sl.bytes, state_bytes);
    if (!aligned16(state)) return fail(WKV_ERR_INVALID_ARGUMENT, "state must be 16-byte aligned");
    state_tickets = reinterpret_cast<unsigned*>(
        reinterpret_cast<char*>(const_cast<float*>(state)) + sl.ckpt_bytes);
  }
  const int b = (int)B, t = (int)T, c = (int)C;
  switch (dtype) {
    case WKV_DTYPE_F32:
      return launch_backward<float>(grad_y, w, u, key, value, grad_key, grad_value,
                                    grad_time_decay, grad_time_first, b, t, c, p, ws, state,
                                    state_tickets, st);
    case WKV_DTYPE_BF16:
      return launch_backward<__nv_bfloat16>(grad_y, w, u, key, value, grad_key, grad_value,
                                            grad_time_decay, grad_time_first, b, t, c, p, ws,
                                            state, state_tickets, st);
    default:
      return launch_backward<__half>(grad_y, w, u, key, value, grad_key, grad_value,
                                     grad_time_decay, grad_time_first, b, t, c, p, ws, state,
                                     state_tickets, st);
  }
}

// ------------------------------------------------- allocation-free backward
//
// Scratch of wkv_backward_noalloc. The runtime reserves it on each device that
// loads this module and zero-fills it once; after that every call reuses it as
// left by the previous call, so the launch sequence must clear whatever has to
// start at zero (it does: the state sweep zeroes the reduction counters before
// the gradient kernel reads them; checkpoints and partial sums are overwritten).
__device__ __align__(256) unsigned char g_noalloc_scratch[WKV_NOALLOC_SCRATCH_BYTES];

SymbolCache g_noalloc_cache;

// In host code `g_noalloc_scratch` names a host-side shadow of the symbol, not
// device memory: the device address comes from cudaGetSymbolAddress, asked
// with the device current, and is cached per device and context.
int noalloc_scratch(void** base) {
  const cudaError_t e = symbol_address(g_noalloc_cache, g_noalloc_scratch, base);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
  return WKV_OK;
}

}  // namespace

extern "C" {

int wkv_backward_noalloc(int dtype, const void* grad_y, const float* w, const float* u,
                         const void* key, const void* value, void* grad_key, void* grad_value,
                         float* grad_time_decay, float* grad_time_first, int64_t B, int64_t T,
                         int64_t C, void* stream) {
  g_last_error[0] = '\0';
  const int rc = check_dims(dtype, B, T, C);
  if (rc) return rc;
  const bool al = aligned16(grad_y) && aligned16(key) && aligned16(value) && aligned16(grad_key) &&
                  aligned16(grad_value);
  const size_t need = bwd_workspace(make_plan(dtype, B, T, C, al), B, T, C, nullptr).bytes;
  if (need > WKV_NOALLOC_SCRATCH_BYTES)
    return fail(WKV_ERR_INVALID_ARGUMENT,
                "wkv_backward_noalloc: B=%lld T=%lld C=%lld needs %zu scratch bytes but the "
                "static scratch holds %zu; call wkv_backward with a workspace instead",
                (long long)B, (long long)T, (long long)C, need, (size_t)WKV_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if (B > 0 && T > 0 && C > 0) {
    const int src = noalloc_scratch(&scratch);
    if (src) return src;
  }
  return backward_impl(dtype, grad_y, w, u, key, value, nullptr, 0, grad_key, grad_value,
                       grad_time_decay, grad_time_first, B, T, C, scratch,
                       WKV_NOALLOC_SCRATCH_BYTES, stream);
}

int wkv_forward(int dtype, const void* key, const void* value, const float* time_decay,
                const float* time_first, void* y, int64_t B, int64_t T, int64_t C,
                void* workspace, size_t workspace_bytes, void* stream) {
  return forward_impl(dtype, key, value, time_decay, time_first, y, nullptr, 0, B, T, C,
                      workspace, workspace_bytes, stream);
}

int wkv_backward(int dtype, const void* grad_y, const float* w, const float* u, const void* key,
                 const void* value, void* grad_key, void* grad_value, float* grad_time_decay,
                 float* grad_time_first, int64_t B, int64_t T, int64_t C, void* workspace,
                 size_t workspace_bytes, void* stream) {
  return backward_impl(dtype, grad_y, w, u, key, value, nullptr, 0, grad_key, grad_value,
                       grad_time_decay, grad_time_first, B, T, C, workspace, workspace_bytes,
                       stream);
}

size_t wkv_state_size(int dtype, int64_t B, int64_t T, int64_t C) {
  if (check_dims(dtype, B, T, C)) return 0;
  return state_layout(B, T, C).bytes;
}

int wkv_forward_with_state(int dtype, const void* key, const void* value, const float* time_decay,
                           const float* time_first, void* y, float* state, size_t state_bytes,
                           int64_t B, int64_t T, int64_t C, void* workspace,
                           size_t workspace_bytes, void* stream) {
  if (state == nullptr && B > 0 && T > 0 && C > 0)
    return fail(WKV_ERR_INVALID_ARGUMENT, "null state pointer");
  return forward_impl(dtype, key, value, time_decay, time_first, y, state, state_bytes, B, T, C,
                      workspace, workspace_bytes, stream);
}

int wkv_backward_from_state(int dtype, const void* grad_y, const float* w, const float* u,
                            const void* key, const void* value, const float* state,
                            size_t state_bytes, void* grad_key, void* grad_value,
                            float* grad_time_decay, float* grad_time_first, int64_t B, int64_t T,
                            int64_t C, void* workspace, size_t workspace_bytes, void* stream) {
  if (state == nullptr && B > 0 && T > 0 && C > 0)
    return fail(WKV_ERR_INVALID_ARGUMENT, "null state pointer");
  return backward_impl(dtype, grad_y, w, u, key, value, state, state_bytes, grad_key, grad_value,
                       grad_time_decay, grad_time_first, B, T, C, workspace, workspace_bytes,
                       stream);
}

int wkv_step(int dtype, int state_dtype, const void* key, const void* value,
             const float* time_decay, const float* time_first, void* numerator, void* denominator,
             void* log_scale, void* y, int64_t B, int64_t C, void* stream) {
  g_last_error[0] = '\0';
  int rc = check_dims(dtype, B, 1, C);
  if (rc) return rc;
  if (state_dtype != dtype && state_dtype != WKV_DTYPE_F32)
    return fail(WKV_ERR_INVALID_ARGUMENT,
                "state dtype code %d: the state must be float32 or the key/value dtype (%d)",
                state_dtype, dtype);
  if (B == 0 || C == 0) return WKV_OK;
  if (!key || !value || !time_decay || !time_first || !numerator || !denominator || !log_scale || !y)
    return fail(WKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  const int V = static_cast<int>(16 / dtype_size(dtype));
  const bool vec = (C % V) == 0 && aligned16(key) && aligned16(value) && aligned16(numerator) &&
                   aligned16(denominator) && aligned16(log_scale) && aligned16(y) &&
                   aligned16(time_decay) && aligned16(time_first);
  StepArgs a{key, value, time_decay, time_first, numerator, denominator, log_scale, y, B * C, (int)C};
  const int64_t work = vec ? a.n / V : a.n;
  const unsigned grid =
      (unsigned)std::min<int64_t>((work + 255) / 256, (int64_t)sm_count() * 8);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool s32 = state_dtype == WKV_DTYPE_F32;
  launch(K_STEP, st, [&] {
    switch (dtype) {
      case WKV_DTYPE_F32:
        if (vec) wkv_step_kernel<float, float, 4><<<grid, 256, 0, st>>>(a);
        else wkv_step_kernel<float, float, 1><<<grid, 256, 0, st>>>(a);
        break;
      case WKV_DTYPE_BF16:
        if (s32) {
          if (vec) wkv_step_kernel<__nv_bfloat16, float, 8><<<grid, 256, 0, st>>>(a);
          else wkv_step_kernel<__nv_bfloat16, float, 1><<<grid, 256, 0, st>>>(a);
        } else {
          if (vec) wkv_step_kernel<__nv_bfloat16, __nv_bfloat16, 8><<<grid, 256, 0, st>>>(a);
          else wkv_step_kernel<__nv_bfloat16, __nv_bfloat16, 1><<<grid, 256, 0, st>>>(a);
        }
        break;
      default:
        if (s32) {
          if (vec) wkv_step_kernel<__half, float, 8><<<grid, 256, 0, st>>>(a);
          else wkv_step_kernel<__half, float, 1><<<grid, 256, 0, st>>>(a);
        } else {
          if (vec) wkv_step_kernel<__half, __half, 8><<<grid, 256, 0, st>>>(a);
          else wkv_step_kernel<__half, __half, 1><<<grid, 256, 0, st>>>(a);
        }
        break;
    }
  });
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "wkv step launch");
  return WKV_OK;
}

}  // extern "C"

namespace {

// Time segments of the LIF backward's TMA path: with few units (256-channel
// groups x sequences) for the SMs, the sweep over T is split into up to 16
// segments of at least two staged tiles (segment summaries, then every
// segment at once); 1 when the units fill half the GPU or the shape has no
// TMA path. seg_tiles: staged tiles per segment. The debug override
// force_segments (> 1) sets the count.
int lif_bwd_segments(int dtype, int64_t B, int64_t T, int64_t C, int* seg_tiles) {
  const int64_t rt = dtype == WKV_DTYPE_F32 ? lif_ws_rows<float>() : lif_ws_rows<__nv_bfloat16>();
  const int64_t tiles = (T + rt - 1) / rt;
  *seg_tiles = (int)tiles;
  if ((C * (int64_t)dtype_size(dtype)) % 16 != 0 || tiles < 4) return 1;
  const int64_t units = ((C + kLanes - 1) / kLanes + kLifWarps - 1) / kLifWarps * B;
  const int forced = g_force_segments.load();
  int64_t nseg = forced > 1 ? forced : (2 * units <= 148 ? std::min<int64_t>(16, 148 / std::max<int64_t>(1, units)) : 1);
  nseg = std::min<int64_t>(nseg, tiles / 2);
  if (nseg < 2) return 1;
  const int64_t per = (tiles + nseg - 1) / nseg;
  *seg_tiles = (int)per;
  return (int)((tiles + per - 1) / per);
}

size_t lif_ckpt_bytes(int64_t B, int64_t T, int64_t C) {
  return round_up((size_t)B * ((T + kSub - 1) / kSub) * C * sizeof(float));
}

}  // namespace

extern "C" {

size_t lif_state_size(int dtype, int64_t B, int64_t T, int64_t C) {
  if (check_dims(dtype, B, T, C)) return 0;
  int per = 0;
  const int nseg = lif_bwd_segments(dtype, B, T, C, &per);
  const size_t sums = nseg > 1 ? round_up((size_t)B * nseg * 2 * C * sizeof(float)) : 0;
  return lif_ckpt_bytes(B, T, C) + sums;
}

}  // extern "C"

namespace {

// with_device = false: the shape and constants only (no CUDA call; for plans)
int lif_prepare(int dtype, int64_t B, int64_t T, int64_t C, float tau, float threshold,
                float reset, float slope, LifArgs& a, bool with_device = true) {
  int rc = check_dims(dtype, B, T, C);
  if (rc) return rc;
  if (!(tau > 0.f)) return fail(WKV_ERR_INVALID_ARGUMENT, "tau must be positive");
  a = LifArgs{};
  a.decay = static_cast<float>(1.0 - 1.0 / static_cast<double>(tau));  // as the reference's decay
  a.threshold = threshold;
  a.reset = reset;
  a.slope = slope;
  a.B = (int)B;
  a.T = (int)T;
  a.C = (int)C;
  a.ncblk = (int)((C + kLanes - 1) / kLanes);
  a.ntiles = (int)((T + kSub - 1) / kSub);
  a.err = with_device ? device_err_ptr() : nullptr;
  return WKV_OK;
}

// The spike test can compare the membrane with the threshold directly when
// that gives the reference's slope * (v - threshold) >= 0 for every membrane:
// a finite slope >= 1 and a finite threshold (see lif.cuh).
bool lif_plain_test(const LifArgs& a) {
  return a.slope >= 1.f && std::isfinite(a.slope) && std::isfinite(a.threshold);
}

template <typename IO, bool kTma, bool kPlain>
void lif_fwd_go(const LifArgs& a, const CUtensorMap& mx, const CUtensorMap& ms, unsigned grid, size_t sm,
                cudaStream_t st) {
  lif_fwd_kernel<IO, kTma, kPlain><<<grid, 32 * kLifWarps, sm, st>>>(a, mx, ms);
}

// Segments of the time-segmented LIF forward (lif_fwd_seg_kernel), 1 for the
// sequential one: with the checkpoints requested, whole 16-step sub-tiles and
// whole 64-channel blocks on the aligned path, and decay <= 0.75 (tau <= 4:
// a membrane difference no spike removes falls below the rounding within
// about four sub-tiles, so the repair passes stay short; with a decay near 1
// segments often fail to converge and their repair runs in sequence), and
// at most 256 (block, row) units (the sequential forward then runs fewer
// than half a warp per scheduler; above that it is left as measured), as
// many segments (up to kLifSegMax, each at least 4 sub-tiles) as keep a
// launch within 2048 warps (about 3.5 a scheduler). force_segments of
// wkv_set_debug_overrides fixes the count whatever the decay (1: the
// sequential forward). `ls` = sub-tiles a segment (the last one shorter); no
// segment is empty.
int lif_fwd_segments(const LifArgs& a, bool tma, bool with_state, int& ls) {
  ls = 0;
  if (!tma || !with_state || a.C % kLanes != 0 || a.T % kSub != 0) return 1;
  if (g_force_segments.load() <= 0 && !(a.decay <= 0.75f)) return 1;
  const int ntiles = a.T / kSub;
  const int forced = g_force_segments.load();
  int n = kLifSegMax;
  if (forced > 0) {
    n = std::min(forced, kLifSegMax);
  } else {
    const int64_t units = (int64_t)a.ncblk * a.B;
    if (units > 256) return 1;
    while (n > 1 && units * n > 2048) n /= 2;
    n = std::min(n, ntiles / 4);
  }
  n = std::min(n, ntiles);
  if (n < 2) return 1;
  ls = (ntiles + n - 1) / n;
  return (ntiles + ls - 1) / ls;
}

template <typename IO>
int lif_launch_forward(LifArgs& a, bool tma, cudaStream_t st) {
  const int dt = sizeof(IO) == 4 ? WKV_DTYPE_F32
                 : std::is_same<IO, __nv_bfloat16>::value ? WKV_DTYPE_BF16
                                                         : WKV_DTYPE_F16;
  CUtensorMap mx, ms;
  std::memset(&mx, 0, sizeof(mx));
  std::memset(&ms, 0, sizeof(ms));
  int rc;
  if (tma && ((rc = make_map(&mx, dt, a.x, a.B, a.T, a.C, lif_rows<IO>())) ||
              (rc = make_map(&ms, dt, a.s, a.B, a.T, a.C, lif_rows<IO>()))))
    return rc;
  const bool plain = lif_plain_test(a);
  int ls = 0;
  const int fseg = lif_fwd_segments(a, tma, a.state != nullptr, ls);
  if (fseg > 1) {
    const unsigned grid = (unsigned)((int64_t)a.ncblk * a.B);
    launch(K_LIF_FWD, st, [&] {
      if (plain) lif_fwd_seg_kernel<IO, true><<<grid, 32 * fseg, 0, st>>>(a, fseg, ls);
      else lif_fwd_seg_kernel<IO, false><<<grid, 32 * fseg, 0, st>>>(a, fseg, ls);
    });
    const cudaError_t le = cudaGetLastError();
    return le == cudaSuccess ? WKV_OK : cuda_fail(le, "LIF forward launch");
  }
  const size_t sm = kLifWarps * lif_fwd_smem_bytes();
  cudaError_t e = tma ? (plain ? allow_smem(lif_fwd_kernel<IO, true, true>, sm)
                               : allow_smem(lif_fwd_kernel<IO, true, false>, sm))
                      : (plain ? allow_smem(lif_fwd_kernel<IO, false, true>, sm)
                               : allow_smem(lif_fwd_kernel<IO, false, false>, sm));
  if (e != cudaSuccess) return cuda_fail(e, "setting the LIF kernel's shared memory size");
  const unsigned grid = (unsigned)(((int64_t)a.ncblk * a.B + kLifWarps - 1) / kLifWarps);
  launch(K_LIF_FWD, st, [&] {
    if (tma && plain) lif_fwd_go<IO, true, true>(a, mx, ms, grid, sm, st);
    else if (tma) lif_fwd_go<IO, true, false>(a, mx, ms, grid, sm, st);
    else if (plain) lif_fwd_go<IO, false, true>(a, mx, ms, grid, sm, st);
    else lif_fwd_go<IO, false, false>(a, mx, ms, grid, sm, st);
  });
  const cudaError_t le = cudaGetLastError();
  return le == cudaSuccess ? WKV_OK : cuda_fail(le, "LIF forward launch");
}

template <typename IO, bool kTma, bool kPlain>
void lif_bwd_go(const LifArgs& a, const CUtensorMap& mx, const CUtensorMap& mg, const CUtensorMap& mst,
                const CUtensorMap& mo, unsigned grid, size_t sm, cudaStream_t st) {
  if constexpr (kTma)
    lif_bwd_ws_kernel<IO, kPlain><<<dim3(grid, (unsigned)a.nseg), kLifWsThreads, sm, st>>>(a, mx, mg, mst, mo);
  else lif_bwd_kernel<IO, kPlain><<<grid, 32 * kLifWarps, sm, st>>>(a);
}

template <typename IO>
int lif_launch_backward(LifArgs& a, bool tma, cudaStream_t st) {
  const int dt = sizeof(IO) == 4 ? WKV_DTYPE_F32
                 : std::is_same<IO, __nv_bfloat16>::value ? WKV_DTYPE_BF16
                                                         : WKV_DTYPE_F16;
  // TMA path: x, grad and grad_x in lif_ws_rows<IO>() x kLifWsCols boxes; the
  // checkpoints of a staged tile's sub-tiles in one [sub-tiles][kLifWsCols] float box
  CUtensorMap mx, mg, mst, mo;
  std::memset(&mx, 0, sizeof(mx));
  std::memset(&mg, 0, sizeof(mg));
  std::memset(&mst, 0, sizeof(mst));
  std::memset(&mo, 0, sizeof(mo));
  int rc;
  constexpr int WR = lif_ws_rows<IO>();
  if (tma && ((rc = make_map(&mx, dt, a.x, a.B, a.T, a.C, WR, kLifWsCols)) ||
              (rc = make_map(&mg, dt, a.gs, a.B, a.T, a.C, WR, kLifWsCols)) ||
              (rc = make_map(&mo, dt, a.gx, a.B, a.T, a.C, WR, kLifWsCols)) ||
              (rc = make_map(&mst, WKV_DTYPE_F32, a.state, a.B, a.ntiles, a.C, WR / kSub, kLifWsCols))))
    return rc;
  const bool plain = lif_plain_test(a);
  const size_t sm = tma ? lif_ws_bwd_smem_bytes<IO>() : kLifWarps * lif_bwd_smem_bytes<IO>();
  cudaError_t e = tma ? (plain ? allow_smem(lif_bwd_ws_kernel<IO, true>, sm)
                               : allow_smem(lif_bwd_ws_kernel<IO, false>, sm))
                      : (plain ? allow_smem(lif_bwd_kernel<IO, true>, sm)
                               : allow_smem(lif_bwd_kernel<IO, false>, sm));
  if (e != cudaSuccess) return cuda_fail(e, "setting the LIF kernel's shared memory size");
  // TMA path: one CTA per kLifWarps channel blocks of a batch row (channel
  // groups fastest); generic path: kLifWarps consecutive units per CTA
  const unsigned grid = tma ? (unsigned)((a.ncblk + kLifWarps - 1) / kLifWarps) * (unsigned)a.B
                            : (unsigned)(((int64_t)a.ncblk * a.B + kLifWarps - 1) / kLifWarps);
  a.nseg = 1;
  if (tma) {
    a.nseg = lif_bwd_segments(dt, a.B, a.T, a.C, &a.seg_tiles);
    a.seg_sum = reinterpret_cast<float*>(reinterpret_cast<char*>(a.state) + lif_ckpt_bytes(a.B, a.T, a.C));
  }
  if (a.nseg > 1) {
    const dim3 sg((unsigned)((int64_t)a.ncblk * a.B), (unsigned)(a.nseg - 1));  // CTA: block, sequence, segment
    launch(K_LIF_SUM, st, [&] {
      if (plain) lif_bwd_summary_kernel<IO, true><<<sg, 32 * kLifWarps, 0, st>>>(a);
      else lif_bwd_summary_kernel<IO, false><<<sg, 32 * kLifWarps, 0, st>>>(a);
    });
  }
  launch(K_LIF_BWD, st, [&] {
    if (tma && plain) lif_bwd_go<IO, true, true>(a, mx, mg, mst, mo, grid, sm, st);
    else if (tma) lif_bwd_go<IO, true, false>(a, mx, mg, mst, mo, grid, sm, st);
    else if (plain) lif_bwd_go<IO, false, true>(a, mx, mg, mst, mo, grid, sm, st);
    else lif_bwd_go<IO, false, false>(a, mx, mg, mst, mo, grid, sm, st);
  });
  const cudaError_t le = cudaGetLastError();
  return le == cudaSuccess ? WKV_OK : cuda_fail(le, "LIF backward launch");
}

}  // namespace

extern "C" {

int lif_forward(int dtype, const void* x, void* spikes, float* state, size_t state_bytes,
                int64_t B, int64_t T, int64_t C, float tau, float threshold, float reset,
                float slope, void* stream) {
  g_last_error[0] = '\0';
  LifArgs a;
  int rc = lif_prepare(dtype, B, T, C, tau, threshold, reset, slope, a);
  if (rc) return rc;
  if (B == 0 || T == 0 || C == 0) return WKV_OK;
  if (!x || !spikes) return fail(WKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (state != nullptr) {
    const size_t need = lif_state_size(dtype, B, T, C);
    if (state_bytes < need)
      return fail(WKV_ERR_WORKSPACE_TOO_SMALL, "LIF state needs %zu bytes, got %zu", need, state_bytes);
    if (!aligned16(state)) return fail(WKV_ERR_INVALID_ARGUMENT, "state must be 16-byte aligned");
  }
  a.x = x;
  a.s = spikes;
  a.state = state;
  const bool tma = g_force_generic.load() == 0 && aligned16(x) && aligned16(spikes) &&
                   (C * (int64_t)dtype_size(dtype)) % 16 == 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case WKV_DTYPE_F32: return lif_launch_forward<float>(a, tma, st);
    case WKV_DTYPE_BF16: return lif_launch_forward<__nv_bfloat16>(a, tma, st);
    default: return lif_launch_forward<__half>(a, tma, st);
  }
}

int lif_plan(int dtype, int64_t B, int64_t T, int64_t C, float tau, int with_state, int* forward_segments,
             int* backward_segments) {
  g_last_error[0] = '\0';
  LifArgs a;
  const int rc = lif_prepare(dtype, B, T, C, tau, 1.f, 0.f, 1.f, a, false);
  if (rc) return rc;
  const bool tma = (C * (int64_t)dtype_size(dtype)) % 16 == 0;  // aligned tensors assumed
  int ls = 0, per = 0;
  if (forward_segments)
    *forward_segments = (B == 0 || T == 0 || C == 0) ? 1 : lif_fwd_segments(a, tma, with_state != 0, ls);
  if (backward_segments) *backward_segments = lif_bwd_segments(dtype, B, T, C, &per);
  return WKV_OK;
}

int lif_backward(int dtype, const void* grad_spikes, const void* x, float* state,
                 size_t state_bytes, void* grad_x, int64_t B, int64_t T, int64_t C, float tau,
                 float threshold, float reset, float slope, void* stream) {
  g_last_error[0] = '\0';
  LifArgs a;
  int rc = lif_prepare(dtype, B, T, C, tau, threshold, reset, slope, a);
  if (rc) return rc;
  if (B == 0 || T == 0 || C == 0) return WKV_OK;
  if (!grad_spikes || !x || !grad_x || !state)
    return fail(WKV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  const size_t need = lif_state_size(dtype, B, T, C);
  if (state_bytes < need)
    return fail(WKV_ERR_WORKSPACE_TOO_SMALL, "LIF state needs %zu bytes, got %zu", need, state_bytes);
  if (!aligned16(state)) return fail(WKV_ERR_INVALID_ARGUMENT, "state must be 16-byte aligned");
  a.x = x;
  a.gs = grad_spikes;
  a.gx = grad_x;
  a.state = state;
  const bool tma = g_force_generic.load() == 0 && aligned16(x) && aligned16(grad_spikes) &&
                   aligned16(grad_x) && (C * (int64_t)dtype_size(dtype)) % 16 == 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case WKV_DTYPE_F32: return lif_launch_backward<float>(a, tma, st);
    case WKV_DTYPE_BF16: return lif_launch_backward<__nv_bfloat16>(a, tma, st);
    default: return lif_launch_backward<__half>(a, tma, st);
  }
}

}  // extern "C"

namespace {

int mix_check(int n, int64_t B, int64_t T, int64_t C) {
  if (n < 1 || n > kMixMax) return fail(WKV_ERR_INVALID_ARGUMENT, "n must be 1..%d, got %d", kMixMax, n);
  if (B < 0 || T < 0 || C <= 0) return fail(WKV_ERR_INVALID_ARGUMENT, "bad sizes B=%lld T=%lld C=%lld",
                                            (long long)B, (long long)T, (long long)C);
  if (C % 128 != 0 || C > kMixMaxC)
    return fail(WKV_ERR_INVALID_ARGUMENT, "C must be a multiple of 128 up to %d, got %lld", kMixMaxC,
                (long long)C);
  if (B * T > (1ll << 31) - 1) return fail(WKV_ERR_INVALID_ARGUMENT, "B*T out of range");
  return WKV_OK;
}

// Steps per CTA of the LayerNorm-mix kernels: the largest power of two in
// [kMixMinRows, kMixMaxRows] that still gives a launch about 8 CTAs per SM
// (148 SMs), so small batches fill the GPU too; and the CTAs per sequence that
// follow from it.
int mix_rows_per_cta(int64_t B, int64_t T) {
  int r = kMixMaxRows;
  while (r > kMixMinRows && B * ((T + r - 1) / r) < 8 * 148) r /= 2;
  return r;
}
int64_t mix_ctas_per_seq(int64_t B, int64_t T) {
  const int r = mix_rows_per_cta(B, T);
  return (T + r - 1) / r;
}

template <int N>
cudaError_t mix_bwd_go(const MixArgs& a, unsigned grid, cudaStream_t st) {
  const cudaError_t e = allow_smem(ln_mix_bwd_kernel<N>, kMixStages * mix_bwd_stage_bytes(N, kMixMaxC, true));
  if (e != cudaSuccess) return e;
  const size_t smem = kMixStages * mix_bwd_stage_bytes(N, a.C, a.gres != nullptr);
  launch(K_MIX_BWD, st, [&] { ln_mix_bwd_kernel<N><<<grid, a.C / 4, smem, st>>>(a); });
  return cudaSuccess;
}

}  // namespace

extern "C" {

size_t ln_mix_workspace_size(int n, int64_t B, int64_t T, int64_t C) {
  if (mix_check(n, B, T, C)) return 0;
  // one partial row set (dw, db, dm_i) per CTA
  return round_up((size_t)(B * mix_ctas_per_seq(B, T)) * (2 + n) * C * sizeof(float));
}

int ln_mix_forward(int n, const float* x, const float* w, const float* b, const float* mix, void* out0, void* out1,
                   void* out2, float* mean, float* rstd, int64_t B, int64_t T, int64_t C, float eps, void* stream) {
  g_last_error[0] = '\0';
  int rc = mix_check(n, B, T, C);
  if (rc) return rc;
  if (B == 0 || T == 0) return WKV_OK;
  void* outs[kMixMax] = {out0, out1, out2};
  if (!x || !w || !b || !mix || !mean || !rstd) return fail(WKV_ERR_INVALID_ARGUMENT, "null pointer");
  if (!aligned16(x) || !aligned16(w) || !aligned16(b) || !aligned16(mix))
    return fail(WKV_ERR_INVALID_ARGUMENT, "x, w, b and mix must be 16-byte aligned");
  MixArgs a{};
  for (int i = 0; i < n; ++i) {
    if (!outs[i] || (reinterpret_cast<uintptr_t>(outs[i]) & 7u))
      return fail(WKV_ERR_INVALID_ARGUMENT, "output %d must be non-null and 8-byte aligned", i);
    a.out[i] = static_cast<__nv_bfloat16*>(outs[i]);
  }
  a.x = x;
  a.w = w;
  a.b = b;
  a.mix = mix;
  a.mean = mean;
  a.rstd = rstd;
  a.n = n;
  a.B = (int)B;
  a.T = (int)T;
  a.C = (int)C;
  a.rows = mix_rows_per_cta(B, T);
  a.nct = (int)mix_ctas_per_seq(B, T);
  a.eps = eps;
  const unsigned grid = (unsigned)(B * a.nct);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  launch(K_MIX_FWD, st, [&] { ln_mix_fwd_kernel<<<grid, (unsigned)(C / 4), 0, st>>>(a); });
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? WKV_OK : cuda_fail(e, "ln_mix forward launch");
}

int ln_mix_backward(int n, const void* g0, const void* g1, const void* g2, const float* x, const float* w,
                    const float* b, const float* mix, const float* mean, const float* rstd,
                    const float* grad_residual, float* gx, void* gx_bf16, float* gw, float* gb, float* gmix,
                    void* workspace,
                    size_t workspace_bytes, int64_t B, int64_t T, int64_t C, void* stream) {
  g_last_error[0] = '\0';
  int rc = mix_check(n, B, T, C);
  if (rc) return rc;
  if (!gw || !gb || !gmix) return fail(WKV_ERR_INVALID_ARGUMENT, "null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B == 0 || T == 0) {  // empty batch: zero parameter gradients
    cudaMemsetAsync(gw, 0, C * sizeof(float), st);
    cudaMemsetAsync(gb, 0, C * sizeof(float), st);
    cudaMemsetAsync(gmix, 0, n * C * sizeof(float), st);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? WKV_OK : cuda_fail(e, "ln_mix backward");
  }
  const void* gs[kMixMax] = {g0, g1, g2};
  if (!x || !w || !b || !mix || !mean || !rstd || !gx) return fail(WKV_ERR_INVALID_ARGUMENT, "null pointer");
  if (!aligned16(x) || !aligned16(w) || !aligned16(b) || !aligned16(mix) || !aligned16(gx) ||
      !aligned16(grad_residual))
    return fail(WKV_ERR_INVALID_ARGUMENT, "x, w, b, mix, grad_residual and grad_x must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(gx_bf16) & 7u)
    return fail(WKV_ERR_INVALID_ARGUMENT, "grad_x_bf16 must be 8-byte aligned");
  const size_t need = ln_mix_workspace_size(n, B, T, C);
  if (workspace_bytes < need || !workspace)
    return fail(WKV_ERR_WORKSPACE_TOO_SMALL, "ln_mix backward needs %zu workspace bytes, got %zu", need,
                workspace_bytes);
  MixArgs a{};
  for (int i = 0; i < n; ++i) {
    if (!gs[i] || (reinterpret_cast<uintptr_t>(gs[i]) & 7u))
      return fail(WKV_ERR_INVALID_ARGUMENT, "gradient %d must be non-null and 8-byte aligned", i);
    a.gout[i] = static_cast<const __nv_bfloat16*>(gs[i]);
  }
  a.x = x;
  a.w = w;
  a.b = b;
  a.mix = mix;
  a.mean = const_cast<float*>(mean);
  a.rstd = const_cast<float*>(rstd);
  a.gx = gx;
  a.gx16 = static_cast<__nv_bfloat16*>(gx_bf16);
  a.gres = grad_residual;
  a.partial = static_cast<float*>(workspace);
  a.n = n;
  a.B = (int)B;
  a.T = (int)T;
  a.C = (int)C;
  a.rows = mix_rows_per_cta(B, T);
  a.nct = (int)mix_ctas_per_seq(B, T);
  const int chunks = (int)(B * a.nct);  // CTAs, each leaving one partial row set
  const unsigned grid = (unsigned)chunks;
  const cudaError_t ae = n == 1 ? mix_bwd_go<1>(a, grid, st) : n == 2 ? mix_bwd_go<2>(a, grid, st)
                                                                    : mix_bwd_go<3>(a, grid, st);
  if (ae != cudaSuccess) return cuda_fail(ae, "setting the ln_mix backward kernel's shared memory size");
  const int rows = 2 + n;
  launch(K_MIX_RED, st, [&] {
    ln_mix_reduce_kernel<<<dim3((unsigned)((C + 31) / 32), (unsigned)rows), dim3(32, 32), 0, st>>>(
        a.partial, chunks, rows, (int)C, gw, gb, gmix);
  });
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? WKV_OK : cuda_fail(e, "ln_mix backward launch");
}

}  // extern "C"

namespace {

// Grid of the elementwise gate kernels: one 8-element vector per thread per
// iteration, at most 8 CTAs per SM (grid-stride beyond that).
unsigned gate_grid(int64_t n) {
  const int64_t v = (n / 8 + kGateThreads - 1) / kGateThreads;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(v, 8 * 148));
}

int gate_check(int64_t n, std::initializer_list<const void*> ptrs) {
  if (n < 0) return fail(WKV_ERR_INVALID_ARGUMENT, "n must be >= 0, got %lld", (long long)n);
  if (n == 0) return WKV_OK;
  for (const void* p : ptrs) {
    if (!p) return fail(WKV_ERR_INVALID_ARGUMENT, "null pointer");
    if (!aligned16(p)) return fail(WKV_ERR_INVALID_ARGUMENT, "bf16 tensors must be 16-byte aligned");
  }
  return WKV_OK;
}

int launched(const char* what) {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? WKV_OK : cuda_fail(e, what);
}

}  // namespace

extern "C" {

int gate_forward(const void* r, const void* x, void* out, int64_t n, void* stream) {
  g_last_error[0] = '\0';
  const int rc = gate_check(n, {r, x, out});
  if (rc || n == 0) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  launch(K_GATE_FWD, st, [&] {
    gate_fwd_kernel<<<gate_grid(n), kGateThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(r),
                                                            static_cast<const __nv_bfloat16*>(x),
                                                            static_cast<__nv_bfloat16*>(out), n);
  });
  return launched("gate forward launch");
}

int gate_backward(const void* grad_out, const void* r, const void* x, void* grad_r, void* grad_x, int64_t n,
                  void* stream) {
  g_last_error[0] = '\0';
  const int rc = gate_check(n, {grad_out, r, x, grad_r, grad_x});
  if (rc || n == 0) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  launch(K_GATE_BWD, st, [&] {
    gate_bwd_kernel<<<gate_grid(n), kGateThreads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(grad_out), static_cast<const __nv_bfloat16*>(r),
        static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(grad_r),
        static_cast<__nv_bfloat16*>(grad_x), n);
  });
  return launched("gate backward launch");
}

int relu_square_forward(const void* k, void* out, int64_t n, void* stream) {
  g_last_error[0] = '\0';
  const int rc = gate_check(n, {k, out});
  if (rc || n == 0) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  launch(K_RSQ_FWD, st, [&] {
    relu_square_fwd_kernel<<<gate_grid(n), kGateThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(k),
                                                                   static_cast<__nv_bfloat16*>(out), n);
  });
  return launched("relu_square forward launch");
}

int relu_square_backward(const void* grad_out, const void* k, void* grad_k, int64_t n, void* stream) {
  g_last_error[0] = '\0';
  const int rc = gate_check(n, {grad_out, k, grad_k});
  if (rc || n == 0) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  launch(K_RSQ_BWD, st, [&] {
    relu_square_bwd_kernel<<<gate_grid(n), kGateThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(grad_out),
                                                                   static_cast<const __nv_bfloat16*>(k),
                                                                   static_cast<__nv_bfloat16*>(grad_k), n);
  });
  return launched("relu_square backward launch");
}

int residual_add_forward(const float* x, const void* spikes, float* out, int64_t n, void* stream) {
  g_last_error[0] = '\0';
  const int rc = gate_check(n, {x, spikes, out});
  if (rc || n == 0) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  launch(K_RESID, st, [&] {
    residual_add_kernel<<<gate_grid(n), kGateThreads, 0, st>>>(x, static_cast<const __nv_bfloat16*>(spikes), out,
                                                                n);
  });
  return launched("residual_add launch");
}

int rwkv7_forward(const float* r, const float* w, const float* k, const float* v, const float* a,
                  const float* b, const float* state_in, float* y, float* state_out, int64_t B, int64_t T,
                  int64_t H, int64_t N, void* stream) {
  g_last_error[0] = '\0';
  if (N != kR7N) return fail(WKV_ERR_INVALID_ARGUMENT, "head size must be %d, got %lld", kR7N, (long long)N);
  if (B < 0 || T < 0 || H < 0) return fail(WKV_ERR_INVALID_ARGUMENT, "negative size");
  if (B * H > (1ll << 31) - 1 || B * T * H * N > (1ll << 40))
    return fail(WKV_ERR_INVALID_ARGUMENT, "sizes out of range");
  if (B == 0 || H == 0) return WKV_OK;
  if (T > 0 && (!r || !w || !k || !v || !a || !b || !y))  // an empty sequence reads no step vectors
    return fail(WKV_ERR_INVALID_ARGUMENT, "null pointer");
  for (const void* q : {static_cast<const void*>(r), static_cast<const void*>(w), static_cast<const void*>(k),
                        static_cast<const void*>(v), static_cast<const void*>(a), static_cast<const void*>(b),
                        static_cast<const void*>(y)})
    if (!aligned16(q)) return fail(WKV_ERR_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  R7Args p{r, w, k, v, a, b, state_in, y, state_out, (int)B, (int)T, (int)H};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  launch(K_R7_FWD, st, [&] { rwkv7_fwd_kernel<<<(unsigned)(B * H), kR7Threads, 0, st>>>(p); });
  return launched("rwkv7 forward launch");
}

namespace {
int xent_check(const void* logits, int64_t ld, const int64_t* targets, int64_t rows, int64_t V) {
  if (rows < 0 || V < 1 || ld < V || ld % 8 != 0 || rows > (1ll << 31) - 1)
    return fail(WKV_ERR_INVALID_ARGUMENT, "bad sizes rows=%lld V=%lld ld=%lld (ld >= V, a multiple of 8)",
                (long long)rows, (long long)V, (long long)ld);
  if (rows > 0 && (!logits || !targets)) return fail(WKV_ERR_INVALID_ARGUMENT, "null pointer");
  if (!aligned16(logits)) return fail(WKV_ERR_INVALID_ARGUMENT, "logits must be 16-byte aligned");
  return WKV_OK;
}
}  // namespace

int cross_entropy_forward(const void* logits, int64_t ld, const int64_t* targets, int64_t rows, int64_t V,
                          float* loss, float* lse, void* stream) {
  g_last_error[0] = '\0';
  int rc = xent_check(logits, ld, targets, rows, V);
  if (rc || rows == 0) return rc;
  if (!loss || !lse) return fail(WKV_ERR_INVALID_ARGUMENT, "null pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  launch(K_XENT_FWD, st, [&] {
    xent_fwd_kernel<<<(unsigned)rows, kXentThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(logits), ld, targets,
                                                              V, loss, lse, device_err_ptr());
  });
  return launched("cross_entropy forward launch");
}

int cross_entropy_backward(const void* logits, int64_t ld, const int64_t* targets, const float* lse,
                           const float* grad_loss, void* grad_logits, int64_t rows, int64_t V, void* stream) {
  g_last_error[0] = '\0';
  int rc = xent_check(logits, ld, targets, rows, V);
  if (rc || rows == 0) return rc;
  if (!lse || !grad_loss || !grad_logits) return fail(WKV_ERR_INVALID_ARGUMENT, "null pointer");
  if (!aligned16(grad_logits)) return fail(WKV_ERR_INVALID_ARGUMENT, "grad_logits must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  launch(K_XENT_BWD, st, [&] {
    xent_bwd_kernel<<<(unsigned)rows, kXentThreads, 0, st>>>(static_cast<const __nv_bfloat16*>(logits), ld, targets,
                                                              lse, grad_loss,
                                                              static_cast<__nv_bfloat16*>(grad_logits), V);
  });
  return launched("cross_entropy backward launch");
}

int wkv_kernel_kinds(void) { return K_COUNT; }

const char* wkv_kernel_name(int kind) {
  return (kind >= 0 && kind < K_COUNT) ? kKindNames[kind] : "";
}

int wkv_launch_counts(long long* counts, int n) {
  if (!counts || n < 0) return fail(WKV_ERR_INVALID_ARGUMENT, "null counts");
  for (int i = 0; i < n && i < K_COUNT; ++i) counts[i] = g_launches[i].load();
  return WKV_OK;
}

int wkv_timing_enable(int on) {
  g_timing.store(on != 0);
  return WKV_OK;
}

int wkv_timing_collect(double* total_ms, long long* launches, int n) {
  g_last_error[0] = '\0';
  std::vector<TimedLaunch> recs;
  {
    std::lock_guard<std::mutex> lk(g_timing_mu);
    recs.swap(g_timed);
  }
  for (int i = 0; i < n; ++i) {
    if (total_ms) total_ms[i] = 0.0;
    if (launches) launches[i] = 0;
  }
  int rc = WKV_OK;
  for (const TimedLaunch& r : recs) {
    float ms = 0.f;
    cudaError_t e = cudaEventSynchronize(r.stop);
    if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, r.start, r.stop);
    if (e != cudaSuccess && rc == WKV_OK) rc = cuda_fail(e, "reading kernel timing events");
    if (r.kind < n) {
      if (total_ms) total_ms[r.kind] += ms;
      if (launches) launches[r.kind] += 1;
    }
  }
  std::lock_guard<std::mutex> lk(g_timing_mu);
  for (const TimedLaunch& r : recs) {
    g_event_pool.push_back(r.start);
    g_event_pool.push_back(r.stop);
  }
  return rc;
}

int wkv_device_error_flags(unsigned* flags, int clear) {
  g_last_error[0] = '\0';
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  unsigned v = 0;
  e = cudaMemcpyFromSymbol(&v, g_device_error_flags, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "reading device error flags");
  if (flags) *flags = v;
  if (clear) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(g_device_error_flags, &zero, sizeof(zero));
    if (e != cudaSuccess) return cuda_fail(e, "clearing device error flags");
  }
  return WKV_OK;
}

}  // extern "C"
