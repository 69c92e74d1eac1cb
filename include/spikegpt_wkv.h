/*
 * spikegpt_wkv.h -- C ABI of the B200 (sm_100a) WKV recurrence library
 * (libspikegpt_wkv.so).
 *
 * The library implements SpikeGPT's RWKV-4 WKV time-mix recurrence, forward and
 * backward, as hand-written CUDA kernels. The entry points take plain device
 * pointers, sizes and a cudaStream_t passed as void*; there are no torch types in
 * any signature. Every entry point is asynchronous on the given stream, performs
 * no host synchronisation and allocates no device memory: scratch ("workspace")
 * is sized by the *_workspace_size query and owned by the caller.
 *
 * Layout: key, value, y, grad_y, grad_key, grad_value are contiguous row-major
 * [B, T, C] (element (b, t, c) at b*T*C + t*C + c). time_decay, time_first, w, u,
 * grad_time_decay, grad_time_first are contiguous float32 [C].
 *
 * Arithmetic: the recurrence runs in float32 whatever the I/O dtype; I/O values
 * are widened in registers and results are rounded to the I/O dtype on store.
 *
 * Reference interfaces these entry points replace (paths relative to the
 * reference project djsaunde/spikegpt-myelin):
 *   wkv_forward   <- torch op myelin::wkv_forward, src/spikegpt/wkv_triton.py:147-158,
 *                    and its bf16 twin myelin::wkv_forward_bf16io, src/spikegpt/wkv_bf16.py:143-154
 *   wkv_backward  <- torch op myelin::wkv_backward, src/spikegpt/wkv_triton.py:164-194,
 *                    and myelin::wkv_backward_bf16io, src/spikegpt/wkv_bf16.py:160-191
 */
#ifndef SPIKEGPT_WKV_H_
#define SPIKEGPT_WKV_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define WKV_API __attribute__((visibility("default")))
#else
#define WKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* I/O element types of key, value, y, grad_y, grad_key, grad_value. */
#define WKV_DTYPE_F32 0
#define WKV_DTYPE_BF16 1
#define WKV_DTYPE_F16 2

/* Status codes returned by every int-valued entry point. */
#define WKV_OK 0
#define WKV_ERR_INVALID_ARGUMENT 1   /* bad dtype, negative size, null pointer, ...   */
#define WKV_ERR_WORKSPACE_TOO_SMALL 2 /* workspace_bytes < the *_workspace_size query */
#define WKV_ERR_CUDA 3               /* a CUDA runtime call or kernel launch failed   */
#define WKV_ERR_DRIVER 4             /* TMA descriptor encoding failed                 */

/* Sticky device-side error flags (see wkv_device_error_flags). */
#define WKV_DEVERR_PIPELINE_TIMEOUT 1u /* a bounded wait on a copy barrier expired */
#define WKV_DEVERR_BAD_TARGET 2u       /* cross_entropy_*: a target outside [0, V) other than -100 */

/* ABI version of this header; bumped on incompatible changes. */
#define WKV_ABI_VERSION 1
WKV_API int wkv_abi_version(void);

/* Human-readable text for a status code (static storage). */
WKV_API const char* wkv_status_string(int status);

/* Details of the last failure on the calling thread ("" if none). */
WKV_API const char* wkv_last_error(void);

/*
 * Forward: y = WKV(key, value; w = -exp(time_decay), u = time_first).
 * Replaces myelin::wkv_forward / myelin::wkv_forward_bf16io
 * (reference src/spikegpt/wkv_triton.py:147-158, src/spikegpt/wkv_bf16.py:143-154):
 * same arithmetic contract (float32 recurrence, y in the I/O dtype). Unlike the
 * reference wrapper, the I/O tensors are read in their native dtype; no float32
 * copies are made.
 * Sizes: B, T, C >= 0 (any zero size is a no-op).
 */
WKV_API size_t wkv_forward_workspace_size(int dtype, int64_t B, int64_t T, int64_t C);
WKV_API int wkv_forward(int dtype, const void* key, const void* value, const float* time_decay,
                const float* time_first, void* y, int64_t B, int64_t T, int64_t C,
                void* workspace, size_t workspace_bytes, void* stream);

/*
 * Backward of the forward above given grad_y = dL/dy.
 * Replaces myelin::wkv_backward / myelin::wkv_backward_bf16io
 * (reference src/spikegpt/wkv_triton.py:164-194, src/spikegpt/wkv_bf16.py:160-191):
 * inputs w = -exp(time_decay) and u = time_first (float32 [C]); outputs
 * grad_key, grad_value ([B,T,C], I/O dtype), grad_time_decay = dL/dw * w summed
 * over the batch (the reference folds the chain rule of w = -exp(time_decay) in,
 * wkv_triton.py:117,194) and grad_time_first = dL/du summed over the batch
 * (float32 [C]). The per-channel sums are reduced in a fixed order (no atomics),
 * so results are deterministic.
 */
WKV_API size_t wkv_backward_workspace_size(int dtype, int64_t B, int64_t T, int64_t C);
WKV_API int wkv_backward(int dtype, const void* grad_y, const float* w, const float* u,
                 const void* key, const void* value, void* grad_key, void* grad_value,
                 float* grad_time_decay, float* grad_time_first, int64_t B, int64_t T,
                 int64_t C, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Allocation-free backward (no counterpart in the reference: it is an extra
 * entry point for callers of this library that must not allocate device
 * memory). Same arguments and results as wkv_backward, minus the workspace:
 * the scratch it needs (checkpoints, per-lane partial sums, reduction
 * counters) lives in one static device array of WKV_NOALLOC_SCRATCH_BYTES
 * inside this library. The CUDA runtime reserves that array on every device
 * that loads the library and keeps it until the process exits.
 *
 * Who needs it: a host whose device memory is owned by another allocator (a
 * framework's caching allocator or a serving engine's arena that has already
 * reserved the HBM, where a raw cudaMalloc can fail or cudaFree would stall
 * every stream), and thin FFI bindings that have no allocator to hand and
 * cannot manage a workspace's lifetime.
 *
 * - Shapes whose scratch exceeds WKV_NOALLOC_SCRATCH_BYTES (roughly
 *   B*T*C above 44 million elements: the checkpoints take 0.75 bytes per
 *   element) fail with WKV_ERR_INVALID_ARGUMENT and a message naming the
 *   bytes needed; use wkv_backward for those.
 * - The first call on a device looks up the array's device address (once per
 *   device and CUDA context, with that device current); make that first call
 *   before any stream capture begins on the device. After a device reset the
 *   next call looks the address up again in the new context.
 * - Every call shares the one array and it keeps the previous call's
 *   contents; the call clears what must start at zero itself. Calls that
 *   overlap on the GPU (different streams, or different host threads on one
 *   device) race on the array and give wrong gradients: serialise them.
 * - Allocates nothing: no cudaMalloc, cudaFree or allocating library call.
 */
#define WKV_NOALLOC_SCRATCH_BYTES ((size_t)32 << 20)
WKV_API int wkv_backward_noalloc(int dtype, const void* grad_y, const float* w, const float* u,
                                 const void* key, const void* value, void* grad_key,
                                 void* grad_value, float* grad_time_decay,
                                 float* grad_time_first, int64_t B, int64_t T, int64_t C,
                                 void* stream);

/*
 * One recurrent (single-token) WKV step for generation. Replaces the WKV
 * arithmetic of SpikeTimeMix.step (reference src/spikegpt/language.py:977-1013,
 * the lines 993-1010 between the key/value projections and the receptance
 * gate), on the reference's state: numerator, denominator and log_scale
 * (natural-log scale), all [B, C]. key, value: [B, C] in `dtype`; the state
 * and y: [B, C] in `state_dtype`, which is either `dtype` (a module run
 * entirely in one dtype) or WKV_DTYPE_F32 (mixed precision: under autocast the
 * reference's state is float32 while the projections give bf16/fp16 keys, and
 * torch promotes the step's result to float32). The state is updated in
 * place; y receives the WKV output of the step. time_decay, time_first:
 * float32 [C] (w = -exp(time_decay) is formed inside). Arithmetic is float32.
 * The initial state is zeros with log_scale = the state dtype's most negative
 * finite value, as the reference's initial_state (language.py:957-975).
 */
WKV_API int wkv_step(int dtype, int state_dtype, const void* key, const void* value,
                     const float* time_decay, const float* time_first, void* numerator,
                     void* denominator, void* log_scale, void* y, int64_t B, int64_t C,
                     void* stream);

/*
 * LIF sequence op: the spiking activation of SpikeGPT blocks. Replaces the
 * fused LIF kernels the reference calls from SpikingSequenceLIF.forward
 * (src/spikegpt/language.py:849-906: myelin's surrogate_lif_bf16io and
 * triton_surrogate_lif_function) with the semantics of its per-step loop
 * (language.py:816-843, 907-918): per (b, c) over t,
 *   v = v * decay + x_t (decay = 1 - 1/tau);  s_t = slope * (v - threshold) >= 0;
 *   v = v * (1 - s_t) + reset * s_t,
 * membrane in float32, x and spikes [B, T, C] in `dtype`. lif_forward writes
 * the spikes and, when `state` is non-null (lif_state_size bytes, 16-byte
 * aligned), for every 16-step tile the membrane entering it times decay
 * ([B][ceil(T/16)][C] float32), which lif_backward recomputes the tile from.
 * lif_backward gives grad_x from grad_spikes through the loop with the
 * spike's surrogate derivative slope * 1 / (2 (1 + (pi/2 * centered)^2)) (the
 * published arc-tangent surrogate; the reference's own surrogate lives in
 * myelin@68b8ebb and is not available to pin against). tau > 0.
 * With few sequences for the GPU (the 256-channel groups times B under half
 * the SMs) lif_backward splits T into segments that run at once (each
 * segment's adjoint map composed first); the per-segment maps go into
 * scratch at the end of `state` (lif_state_size includes it), so backward
 * calls that share one state buffer concurrently race. The last segment's
 * gradients are bit-identical to the one-sweep ones, the others agree to
 * float32 rounding.
 */
WKV_API size_t lif_state_size(int dtype, int64_t B, int64_t T, int64_t C);
/*
 * The segment counts lif_forward and lif_backward pick for a shape (no
 * reference counterpart; like wkv_plan, it exposes a choice the reference
 * never makes), for 16-byte aligned tensors. forward_segments: 1 = the
 * sequential forward; > 1 = the time-segmented forward (few sequences, T a
 * multiple of 16, C a multiple of 64, with_state != 0 (the checkpoints
 * requested, as autograd does), tau <= 4), whose results equal the
 * sequential forward's bit for bit. backward_segments as described above.
 */
WKV_API int lif_plan(int dtype, int64_t B, int64_t T, int64_t C, float tau, int with_state,
                     int* forward_segments, int* backward_segments);
WKV_API int lif_forward(int dtype, const void* x, void* spikes, float* state, size_t state_bytes,
                        int64_t B, int64_t T, int64_t C, float tau, float threshold, float reset,
                        float slope, void* stream);
WKV_API int lif_backward(int dtype, const void* grad_spikes, const void* x, float* state,
                         size_t state_bytes, void* grad_x, int64_t B, int64_t T, int64_t C,
                         float tau, float threshold, float reset, float slope, void* stream);

/*
 * Fused LayerNorm + token-shift mixing: the GEMM inputs of the SpikeGPT
 * blocks under bf16 autocast. Replaces, per sublayer, the reference's
 * LayerNorm followed by `_mix_with_previous` once per projection
 * (src/spikegpt/language.py:344-353; time mixing 1009-1012 with n = 3,
 * channel mixing 1190-1192 with n = 2) and autocast's bf16 copy:
 *   out_i[b,t,:] = bf16(h[t] * m_i + h[t-1] * (1 - m_i)),  h = LayerNorm(x; w, b, eps),
 * h[-1] = 0, x [B,T,C] float32, w, b [C], mix [n][C] float32, outputs bf16.
 * ln_mix_forward also writes the row mean and 1/std ([B*T] float32) that
 * ln_mix_backward takes with the n bf16 output gradients to give grad_x
 * [B,T,C], grad_w, grad_b [C] and grad_mix [n][C] (parameter gradients
 * reduced in a fixed order through `workspace`, ln_mix_workspace_size
 * bytes). grad_residual, when non-null ([B,T,C] float32), is added to
 * grad_x (the gradient the sublayer's residual connection passes to x,
 * language.py:1353-1358), one rounded add as autograd's sum of the two.
 * grad_x_bf16, when non-null ([B,T,C] bf16), also receives grad_x rounded to
 * bf16 (to nearest even): when x is the residual stream after bf16 spikes
 * were added to it, that is the spikes' gradient, without a cast pass of its
 * own. n in 1..3, C a multiple of 128 up to 1024; x, w, b, mix, grad_x
 * 16-byte aligned, bf16 tensors 8-byte aligned; unused output pointers null.
 */
WKV_API size_t ln_mix_workspace_size(int n, int64_t B, int64_t T, int64_t C);
WKV_API int ln_mix_forward(int n, const float* x, const float* w, const float* b, const float* mix,
                           void* out0, void* out1, void* out2, float* mean, float* rstd, int64_t B,
                           int64_t T, int64_t C, float eps, void* stream);
WKV_API int ln_mix_backward(int n, const void* grad_out0, const void* grad_out1,
                            const void* grad_out2, const float* x, const float* w, const float* b,
                            const float* mix, const float* mean, const float* rstd,
                            const float* grad_residual, float* grad_x, void* grad_x_bf16,
                            float* grad_w, float* grad_b, float* grad_mix, void* workspace,
                            size_t workspace_bytes, int64_t B, int64_t T, int64_t C, void* stream);

/*
 * Elementwise gates of the SpikeGPT blocks under bf16 autocast, one pass each
 * way (no reference C interface; they replace the eager ops the reference's
 * modules run): the receptance gate `sigmoid(receptance(xr)) * x` of time and
 * channel mixing (src/spikegpt/language.py:1022 and 1035, 1195-1196) and the
 * channel-mixing activation `relu(k).square()` (language.py:1193), with the
 * eager bf16 roundings:
 *   gate_forward:         out = bf16(s * x),  s = bf16(1 / (1 + exp(-r)))
 *   gate_backward:        grad_x = bf16(g * s),
 *                         grad_r = bf16(bf16(bf16(g * x) * bf16(1 - s)) * s)
 *   relu_square_forward:  out = bf16(relu(k)^2)
 *   relu_square_backward: grad_k = k <= 0 ? 0 : bf16(g * 2k)
 * All tensors bf16, n elements, 16-byte aligned.
 */
WKV_API int gate_forward(const void* r, const void* x, void* out, int64_t n, void* stream);
WKV_API int gate_backward(const void* grad_out, const void* r, const void* x, void* grad_r, void* grad_x,
                          int64_t n, void* stream);
WKV_API int relu_square_forward(const void* k, void* out, int64_t n, void* stream);
WKV_API int relu_square_backward(const void* grad_out, const void* k, void* grad_k, int64_t n, void* stream);

/*
 * The residual connection around a LIF sublayer under bf16 autocast
 * (src/spikegpt/language.py:1353-1358, `residual + lif(...)`):
 * out = x + float(spikes), x and out float32, spikes bf16, n elements,
 * 16-byte aligned; the same values as PyTorch's type-promoting add. Its
 * backward is the identity for x and a cast to bf16 for the spikes.
 */
WKV_API int residual_add_forward(const float* x, const void* spikes, float* out, int64_t n, void* stream);

/*
 * RWKV-7 diagonal-plus-low-rank time mixing, forward (the optional op of the
 * 216M configuration; the reference has no code for it, only prose about an
 * external library's kernel, so the restatement is the published state update):
 * per sequence b and head h, with S [N][N] (rows value channels, columns key
 * channels), S_0 = state_in (or zero when null),
 *   S_t = S_{t-1} diag(w_t) + (S_{t-1} a_t) b_t^T + v_t k_t^T,   y_t = S_t r_t.
 * r, w, k, v, a, b, y: [B, T, H, N] float32, 16-byte aligned; N = 64;
 * state_in / state_out [B, H, N, N] float32 or null. Sequential over T
 * (one CTA per sequence and head, the state in registers).
 */
/*
 * Cross-entropy over bf16 logits (the language-model loss under bf16
 * autocast; replaces F.cross_entropy(logits.float(), targets) of
 * src/spikegpt/language.py:1475-1480 and its backward): per row i of a
 * [rows, ld] bf16 logits buffer whose first V columns are the classes,
 * loss[i] = logsumexp_j x_ij - x_i,t_i and lse[i] = logsumexp_j x_ij
 * (float32); rows whose target is -100 (PyTorch's ignore_index) are
 * ignored (loss 0, gradient 0); a target outside [0, V) other than -100
 * gives that row a NaN loss and NaN gradient and sets
 * WKV_DEVERR_BAD_TARGET (PyTorch raises for such a target).
 * cross_entropy_backward writes grad_logits [rows, ld] bf16:
 * grad_loss[i] * (softmax_ij - [j == t_i]) for j < V, zero beyond. ld a
 * multiple of 8, logits and grad_logits 16-byte aligned.
 */
WKV_API int cross_entropy_forward(const void* logits, int64_t ld, const int64_t* targets, int64_t rows,
                                  int64_t V, float* loss, float* lse, void* stream);
WKV_API int cross_entropy_backward(const void* logits, int64_t ld, const int64_t* targets, const float* lse,
                                   const float* grad_loss, void* grad_logits, int64_t rows, int64_t V,
                                   void* stream);

WKV_API int rwkv7_forward(const float* r, const float* w, const float* k, const float* v, const float* a,
                          const float* b, const float* state_in, float* y, float* state_out, int64_t B,
                          int64_t T, int64_t H, int64_t N, void* stream);

/*
 * Forward/backward with a saved forward state (no reference counterpart; an
 * optimisation of wkv_forward/wkv_backward). wkv_forward_with_state computes y exactly as
 * wkv_forward and also stores the recurrence state at every 16th step into
 * `state` (wkv_state_size bytes, 16-byte aligned, caller-owned).
 * wkv_backward_from_state returns the same gradients as wkv_backward for the
 * same inputs, reading that state instead of re-running the forward sweep, so it
 * reads key/value once instead of twice. The state must come from
 * wkv_forward_with_state on the same key, value and time_decay; it is reusable
 * by later backward calls, but calls that use one state buffer concurrently on
 * the GPU race.
 */
WKV_API size_t wkv_state_size(int dtype, int64_t B, int64_t T, int64_t C);
WKV_API int wkv_forward_with_state(int dtype, const void* key, const void* value,
                                   const float* time_decay, const float* time_first, void* y,
                                   float* state, size_t state_bytes, int64_t B, int64_t T,
                                   int64_t C, void* workspace, size_t workspace_bytes,
                                   void* stream);
WKV_API int wkv_backward_from_state(int dtype, const void* grad_y, const float* w, const float* u,
                                    const void* key, const void* value, const float* state,
                                    size_t state_bytes, void* grad_key, void* grad_value,
                                    float* grad_time_decay, float* grad_time_first, int64_t B,
                                    int64_t T, int64_t C, void* workspace,
                                    size_t workspace_bytes, void* stream);

/*
 * Execution plan the library picks for a shape (no reference counterpart; it
 * exposes the choice the reference never had to make). tma = 1 when tiles are
 * staged with TMA (needs C*sizeof(dtype) % 16 == 0 and 16-byte aligned
 * pointers), segments = number of time segments per (b, c) lane (1 = one
 * sequential sweep; > 1 = chunked two-level scan for small B*C).
 */
WKV_API int wkv_plan(int dtype, int64_t B, int64_t T, int64_t C, int* tma, int* segments);

/*
 * Test and benchmark hooks (process-wide; no reference counterpart).
 * force_segments > 0 fixes the segment count (of the WKV plan, the LIF
 * backward and the LIF forward; 1 = the sequential forms); force_generic != 0 disables the
 * TMA path; force_slow != 0 makes every sub-chunk take the exact per-step
 * rescaling path. Pass zeros to restore the defaults.
 */
WKV_API int wkv_set_debug_overrides(int force_segments, int force_generic, int force_slow);

/*
 * Failure-path test hook (process-wide; no reference counterpart). The
 * time-parallel forward kernels wait on copy barriers with a bounded wait;
 * wait_limit_cycles > 0 shortens the consumers' limit (0 restores the default,
 * about 2 s), and withhold_first_copies != 0 makes every CTA skip issuing its
 * first round's copies, so that wait runs out: the kernel then sets
 * WKV_DEVERR_PIPELINE_TIMEOUT, waits for the copies it did issue, and returns
 * without finishing its outputs. For tests of the error path only.
 */
WKV_API int wkv_set_debug_pipeline(long long wait_limit_cycles, int withhold_first_copies);


/*
 * Launch accounting and per-kernel device timing (no reference counterpart; the
 * benchmark uses them for its launch count and roofline figures).
 * Kernel kinds 0 .. wkv_kernel_kinds()-1, named by wkv_kernel_name().
 * wkv_launch_counts: cumulative launches per kind since the library loaded.
 * wkv_timing_enable(1): bracket every later launch with CUDA events on its stream.
 * wkv_timing_collect: waits for the recorded events and returns, per kind, the
 * summed device milliseconds and the number of timed launches since the last
 * collect.
 */
WKV_API int wkv_kernel_kinds(void);
WKV_API const char* wkv_kernel_name(int kind);
WKV_API int wkv_launch_counts(long long* counts, int n);
WKV_API int wkv_timing_enable(int on);
WKV_API int wkv_timing_collect(double* total_ms, long long* launches, int n);

/*
 * Reads (and with clear != 0 resets) the sticky device-side error flags of the
 * current device; synchronises the device. Returns a status code.
 */
WKV_API int wkv_device_error_flags(unsigned* flags, int clear);

#ifdef __cplusplus
}
#endif

#endif /* SPIKEGPT_WKV_H_ */
