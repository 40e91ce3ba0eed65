/*
 * vtq.h -- C ABI of the B200 (sm_100a) k-quant linear backend for vitni-tensor.
 *
 * Drop-in for the reference's quantized linear seam: every output is
 * bit-identical to the reference CPU path on the same inputs. Plain C types
 * only; every call returns a vtq_status. Citations are file:line in the
 * vitni-tensor project (Rust).
 *
 * Threading: one vtq_ctx per host thread. Calls on one context are
 * serialised on that context's CUDA stream.
 */
#ifndef VTQ_H
#define VTQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. They map 1:1 onto the reference's error enum
 * (src/error.rs:7-63) where one exists. */
typedef int32_t vtq_status;
#define VTQ_OK 0
#define VTQ_ERR_INTERNAL 1        /* Error::Internal(&str): shape / length checks (quant.rs:944-949) */
#define VTQ_ERR_NOT_IMPLEMENTED 2 /* Error::NotImplemented{op,why} (forward_quantized.rs:777-782) */
#define VTQ_ERR_GPU 3             /* Error::GpuError(&str): a CUDA call failed */
#define VTQ_ERR_OOM 4             /* Error::OutOfMemory: device allocation failed */
#define VTQ_ERR_TIMEOUT 5         /* a bounded device-side wait ran out (no reference counterpart) */
#define VTQ_ERR_INVALID_ARG 6     /* null pointer / bad handle (no reference counterpart: Rust slices) */
#define VTQ_ERR_MALFORMED 7       /* Error::Malformed(&str): GGUF parse */
#define VTQ_ERR_TRUNCATED 8       /* Error::Truncated(&str): GGUF parse */

/* GGML tensor type tags (src/model/gguf.rs:127-139). */
#define VTQ_F32 0
#define VTQ_Q4_0 2
#define VTQ_Q5_0 6
#define VTQ_Q8_0 8
#define VTQ_Q4_K 12
#define VTQ_Q6_K 14

/* vtq_linear flags. */
#define VTQ_PTR_HOST 1u  /* x and y are host pointers; the call copies x in and y out and returns
                            when y is written. Otherwise x/y are device pointers and the call is
                            asynchronous on the context stream. */
#define VTQ_GATHER_DEFER 4u /* vtq_linear_gather: do not signal arrival; a later gathered launch on
                              the same stream signals for this one too */
#define VTQ_Q4K_FLOAT 2u /* Q4_K in the reference's default-feature regime (float-fused canonical,
                            quant.rs:616-702) instead of the `std-parallel` integer regime. */

typedef struct vtq_ctx vtq_ctx;
typedef struct vtq_weight vtq_weight;

/* Context: one CUDA device, one stream, a device status word.
 * No reference counterpart (the reference's CPU path has no device state). */
vtq_status vtq_init(int device, vtq_ctx** out);
vtq_status vtq_destroy(vtq_ctx* ctx);
/* Message of the last failed call on this context ("" if none). */
const char* vtq_last_error(const vtq_ctx* ctx);
/* Use the caller's cudaStream_t (NULL = the context's own stream). */
vtq_status vtq_set_stream(vtq_ctx* ctx, void* cuda_stream);
/* Wait for the context stream; returns VTQ_ERR_TIMEOUT (and clears the flag)
 * if a bounded device-side wait of an asynchronous call ran out since the
 * last check. */
vtq_status vtq_synchronize(vtq_ctx* ctx);
/* Bound of the device-side gather arrival waits of this context (default
 * 2 s); a wait that runs out gives up, flags VTQ_ERR_TIMEOUT and leaves the
 * GPU and the context usable. No reference counterpart. */
vtq_status vtq_set_wait_limit(vtq_ctx* ctx, uint64_t ns);

/* Upload rows [row_begin, row_end) of a row-major GGUF weight matrix
 * (QuantTensor bytes, src/model/quant_weights.rs:47-52; shape [out][in] in
 * row-major terms) to device memory in the kernels' layout. `bytes` holds the
 * whole matrix (out_feat rows). row_end = -1 means out_feat.
 * Replaces the reference's zero-copy borrow of the GGUF blob
 * (quant_weights.rs:121-181): the weight is resident for the handle's life. */
vtq_status vtq_weight_upload(vtq_ctx* ctx, int32_t dtype, const uint8_t* bytes, size_t nbytes,
                             int64_t in_feat, int64_t out_feat, int64_t row_begin,
                             int64_t row_end, vtq_weight** out);
vtq_status vtq_weight_free(vtq_weight* w);
vtq_status vtq_weight_info(const vtq_weight* w, int32_t* dtype, int64_t* in_feat,
                           int64_t* rows, size_t* device_bytes);

/* y[b][r] = row r of the uploaded weight against x[b] for b < batch;
 * x is [batch][in_feat], y is [batch][rows]. Arithmetic by dtype exactly as
 * linear_dispatch (src/model/forward_quantized.rs:663-785):
 *   Q4_K  integer (linear_q4_k_integer(_parallel), quant.rs:936/:1149), or
 *         float-fused with VTQ_Q4K_FLOAT (linear_q4_k_fused, quant.rs:1433)
 *   Q6_K  integer (linear_q6_k_integer(_parallel), quant.rs:1060/:1099)
 *   Q8_0, Q5_0  dequantize row + canonical_dot (forward_quantized.rs:751-776)
 *   Q4_0  linear_q4_0_cpu (quant.rs:1529)
 *   F32   canonical_dot per row (forward_quantized.rs:674-697)
 * The reference's row-parallel variants are bit-identical to the serial ones,
 * so there is no thread-count argument. */
vtq_status vtq_linear(vtq_ctx* ctx, const vtq_weight* w, const float* x, float* y, int64_t batch,
                      uint32_t flags);

/* A list of integer k-quant linears (Q4_K / Q6_K weights, batch 1, device
 * pointers) run by ONE persistent kernel launch, in list order, async on the
 * context stream. Replaces a run of consecutive linear_dispatch calls
 * (src/model/forward_quantized.rs:663-785, made 7 times per layer) with one
 * launch: each item's y is bit-identical to vtq_linear on the same inputs,
 * but the next item's weights stream from HBM while the current one is still
 * being reduced, so no kernel boundary sits between the linears.
 * wait_for = j (an earlier item) makes item i read x only after every row of
 * item j's y has been stored -- use it when x is (or is computed from) y_j;
 * -1 means x is ready when the call is made. Calls on one context share its
 * completion counters: run them on one stream (the context's).
 * flags VTQ_PTR_HOST: x and y are host pointers (no wait_for); the call copies
 * every x in, runs the one launch, reads every y back with one copy and
 * returns when they are written. */
#define VTQ_LIST_MAX 32
typedef struct vtq_list_item {
  const vtq_weight* w;
  const float* x; /* device, in_feat floats */
  float* y;       /* device, rows floats */
  int32_t wait_for;
} vtq_list_item;
vtq_status vtq_linear_list(vtq_ctx* ctx, const vtq_list_item* items, int32_t n, uint32_t flags);

/* linear_dispatch with host slices (src/model/forward_quantized.rs:663-668,
 * batch 1): uploads `w` on every call. For parity tests and one-off calls;
 * resident weights go through vtq_weight_upload + vtq_linear. */
vtq_status vtq_linear_dispatch(vtq_ctx* ctx, int32_t dtype, const float* x, const uint8_t* w,
                               size_t wlen, size_t in_feat, size_t out_feat, float* y,
                               uint32_t flags);

/* The op-level signature the reference's linears share,
 * fn(x, w, y_out, batch, in_feat, out_feat) -> Result<()>, host slices:
 *   vtq_linear_q4_k_integer   replaces linear_q4_k_integer(_parallel) quant.rs:936 / :1149
 *   vtq_linear_q6_k_integer   replaces linear_q6_k_integer(_parallel) quant.rs:1060 / :1099
 *   vtq_linear_q4_k_fused     replaces linear_q4_k_fused(_parallel)   quant.rs:1433 / :1385
 *   vtq_linear_q4_0           replaces linear_q4_0_cpu                quant.rs:1529 */
vtq_status vtq_linear_q4_k_integer(vtq_ctx* ctx, const float* x, const uint8_t* w, size_t wlen,
                                   float* y, size_t batch, size_t in_feat, size_t out_feat);
vtq_status vtq_linear_q6_k_integer(vtq_ctx* ctx, const float* x, const uint8_t* w, size_t wlen,
                                   float* y, size_t batch, size_t in_feat, size_t out_feat);
vtq_status vtq_linear_q4_k_fused(vtq_ctx* ctx, const float* x, const uint8_t* w, size_t wlen,
                                 float* y, size_t batch, size_t in_feat, size_t out_feat);
vtq_status vtq_linear_q4_0(vtq_ctx* ctx, const float* x, const uint8_t* w, size_t wlen, float* y,
                           size_t batch, size_t in_feat, size_t out_feat);

/* ---- Context-free device API (for embedding in a host that owns memory and
 * streams). ---- */

/* Bytes of the device layout for `rows` rows (rows re-pitched to 16 B, plus
 * a 16-byte tail pad). -1 if in_feat is invalid for dtype. No reference
 * counterpart: the reference borrows GGUF bytes in place. */
int64_t vtq_device_layout_bytes(int32_t dtype, int64_t in_feat, int64_t rows);
/* Convert `rows` packed GGUF rows already in device memory (src_dev) into the
 * device layout at dst_dev (vtq_device_layout_bytes bytes). Async on stream. */
vtq_status vtq_device_repack(int32_t dtype, int64_t in_feat, int64_t rows, const uint8_t* src_dev,
                             uint8_t* dst_dev, void* cuda_stream);
/* Same arithmetic as vtq_linear on device pointers, async on `cuda_stream`.
 * w_dev: device layout from vtq_device_repack. status_dev: optional device
 * word; kernels OR in 1 if a bounded wait timed out.
 * Allocation: none, except for integer Q4_K at batch >= 16 (the tensor-core
 * path), whose quantised activations live in a library buffer cached per
 * (device, stream): allocated with cudaMalloc on first use, grown when a
 * larger batch comes, freed when the library is unloaded. Callers that must
 * not allocate use vtq_linear_device_ws. */
vtq_status vtq_linear_device(int32_t dtype, const uint8_t* w_dev, int64_t in_feat, int64_t rows,
                             const float* x_dev, int64_t ldx, float* y_dev, int64_t ldy,
                             int64_t batch, uint32_t flags, uint32_t* status_dev,
                             void* cuda_stream);
/* Bytes of caller workspace vtq_linear_device_ws needs for this linear (0 when
 * the kernel needs none: every dtype and batch except integer Q4_K at batch
 * >= 16). No reference counterpart. */
size_t vtq_linear_device_workspace_bytes(int32_t dtype, int64_t in_feat, int64_t batch,
                                         uint32_t flags);
/* vtq_linear_device with caller-owned scratch (256-byte aligned, at least
 * vtq_linear_device_workspace_bytes); allocates nothing. Work queued on one
 * workspace must be ordered (one stream, or the caller's events). */
vtq_status vtq_linear_device_ws(int32_t dtype, const uint8_t* w_dev, int64_t in_feat, int64_t rows,
                                const float* x_dev, int64_t ldx, float* y_dev, int64_t ldy,
                                int64_t batch, uint32_t flags, uint32_t* status_dev,
                                void* workspace, size_t workspace_bytes, void* cuda_stream);

/* Q4_K / Q6_K integer linear with host x and y that allocates nothing: for
 * callers that cannot call cudaMalloc (their device memory is owned by a pool
 * or budget they do not control, or allocation is not allowed on their path).
 * No counterpart in the reference. Same arithmetic and result as vtq_linear
 * with VTQ_PTR_HOST; w_dev is caller-owned device memory in the layout of
 * vtq_device_repack. x, y and the status word are staged in one static device
 * array of 1 MiB (256K floats, kept by every GPU that loads the library until
 * exit): 64 + batch*in_feat + batch*rows floats must fit, else VTQ_ERR_INTERNAL.
 * All calls on a device share that array, so calls that overlap on the GPU
 * race. The first call on a device looks the array's address up; make it
 * before any stream capture. The address is kept for the life of the process
 * (it belongs to the device's primary context): do not call this again after
 * a cudaDeviceReset in the same process. Synchronous: returns when y is
 * written. */
vtq_status vtq_linear_host_noalloc(int32_t dtype, const uint8_t* w_dev, int64_t in_feat,
                                   int64_t rows, const float* x, float* y, int64_t batch,
                                   void* cuda_stream);

/* ---- Quantized decode session (TinyLlama-shaped decode workload): a GGUF Llama or Qwen2 model resident on
 * one device; the decode step of src/model/forward_quantized.rs:329-649 and the
 * prompt + greedy loop of src/model/inference.rs:312-327 run as one CUDA graph
 * per step with the position and current token in device memory. ---- */
typedef struct vtq_decode vtq_decode;
/* Parse the GGUF blob (src/model/gguf.rs:305-422, config.rs:156-212,
 * quant_weights.rs:121-181) and upload every tensor. On failure *out still
 * receives a handle carrying the message (vtq_decode_last_error); close it. */
vtq_status vtq_decode_open(vtq_ctx* ctx, int device, const uint8_t* gguf, size_t len,
                           vtq_decode** out);
const char* vtq_decode_last_error(const vtq_decode* d);
/* dim, hidden, layers, heads, kv_heads, vocab, seq_len, shared_weights. */
vtq_status vtq_decode_config(const vtq_decode* d, int64_t* out8);
/* run_quantized's token loop (inference.rs:312-327): out_tokens receives the
 * n_new generated ids; logits (optional) receives (n_prompt + n_new) x vocab. */
vtq_status vtq_decode_run(vtq_decode* d, const uint32_t* prompt, size_t n_prompt, size_t n_new,
                          uint32_t* out_tokens, float* logits);
/* Device time of the last vtq_decode_run, CUDA events on the session stream:
 * ms2[0] = the decode steps alone, ms2[1] = the whole call including the prompt
 * upload and the token / logits read-back. No reference counterpart. */
vtq_status vtq_decode_timing(const vtq_decode* d, float* ms2);
/* Diagnostic: copy an activation buffer left by the last step (0 x, 1 xb, 2 q,
 * 3 k, 4 v, 5 xo, 6 xb2, 7 gate, 8 up, 9 SwiGLU, 10 logits); n elements. */
vtq_status vtq_decode_debug_buffer(vtq_decode* d, int which, float* out, size_t n);
/* How a step runs: 0 a graph of per-op kernels, 1 the same graph with the fused
 * norm / projection kernels, 2 one persistent cooperative kernel per step.
 * Environment at open: VTQ_DECODE_PERSISTENT=1 (the persistent kernel, when
 * the model fits it), VTQ_DECODE_UNFUSED (per-op kernels without the fused
 * norm). No reference counterpart. */
int vtq_decode_step_kind(const vtq_decode* d);
/* Kernels this library launched for the last vtq_decode_run's decode work (the
 * batched prompt's launches plus the step graph's kernel nodes per step, or one
 * per step for the persistent kernel). No reference counterpart. */
unsigned long long vtq_decode_launches(const vtq_decode* d);
vtq_status vtq_decode_close(vtq_decode* d);

/* ---- The left-to-right fp32 sum of non-negative terms (the sum of squares of
 * rms_norm_slice, src/ops/rms_norm.rs:97-100) as a CTA computes it: runs of
 * steps inside one ulp range composed by a parallel scan, crossing steps added
 * in order by one thread, every run verified (else the plain loop). Test
 * entry points; no reference counterpart. ---- */
/* The plan evaluated on the host, step by step; *fallback = 1 when it fell
 * back to the plain loop. */
float vtq_exact_sum_host(const float* a, size_t n, int* fallback);
/* nvec vectors of n terms from host memory, one CTA of nthr threads each
 * (nthr a multiple of 32, at most 1024); out receives nvec sums. */
vtq_status vtq_exact_sum_device(const float* host, int nvec, int n, int nthr, float* out);

/* ---- Software transcendentals shared by host and device. ----
 * Bit-for-bit the single-precision functions of the Rust `libm` crate the
 * reference calls (Cargo.toml:23): expf (forward_quantized.rs:559, :934),
 * sinf / cosf / powf (RoPE, forward_quantized.rs:453-456). */
float vtq_expf(float x);
float vtq_sinf(float x);
float vtq_cosf(float x);
float vtq_powf(float x, float y);
/* For each in[i], the 7 values the reference's determinism sweep hashes
 * (tests/transcendental_determinism.rs:36-44): expf, sqrtf(|v|), cosf, sinf,
 * powf(1e4, v/64), powf(1e6, v/64), 1/(1+expf(-v)); out holds 7*n floats. */
void vtq_libm_sweep(const float* in, size_t n, float* out);
/* The same sweep with expf, sqrtf and the sigmoid computed by device code
 * (the decode kernels' functions); sin / cos / pow are host-only (RoPE tables). */
int vtq_libm_sweep_device(const float* in, size_t n, float* out);

/* ---- Row-sharded linears with the all-gather fused into the kernel ----
 * No counterpart in the reference (it is single-process; its parallel
 * linears split output rows over threads, src/ops/quant.rs:1120-1143, which
 * is the same row split these calls spread over GPUs).
 * Each rank creates a gather buffer (full y + counters), exports its CUDA IPC
 * handle (64 bytes), and connects to every rank's handle. vtq_linear_gather
 * computes this rank's rows [row0, row0 + rows) of y = W x and stores them into
 * the full y of every rank over NVLink, then signals every rank once;
 * vtq_gather_wait holds the context's stream until `signals` more rank
 * launches have arrived (one per rank per signalling gathered linear; a launch
 * with VTQ_GATHER_DEFER does not signal, the next signalling one covers it).
 * Waits are bounded (vtq_set_wait_limit, 2 s by default) and report
 * VTQ_ERR_TIMEOUT through the context status (vtq_synchronize). */
typedef struct vtq_gather vtq_gather;
vtq_status vtq_gather_create(vtq_ctx* ctx, int32_t world, int32_t rank, size_t y_floats,
                             vtq_gather** out, uint8_t* ipc_handle /* 64 bytes */);
vtq_status vtq_gather_connect(vtq_gather* g, const uint8_t* handles /* world x 64 bytes */);
float* vtq_gather_y(vtq_gather* g);
vtq_status vtq_linear_gather(vtq_ctx* ctx, const vtq_weight* w, const float* x, int64_t batch,
                             vtq_gather* g, int64_t y_offset, int64_t ldy, int64_t row0,
                             uint32_t flags);
vtq_status vtq_gather_wait(vtq_ctx* ctx, vtq_gather* g, uint32_t signals);
/* vtq_linear_gather whose launch also ends with the wait for `wait_signals`
 * arrivals (no separate wait launch; use it for the last gathered linear
 * before y is read). */
vtq_status vtq_linear_gather_wait(vtq_ctx* ctx, const vtq_weight* w, const float* x,
                                  int64_t batch, vtq_gather* g, int64_t y_offset, int64_t ldy,
                                  int64_t row0, uint32_t flags, uint32_t wait_signals);
/* vtq_linear_list over row shards: every item's y must lie in this rank's
 * gather buffer (vtq_gather_y(g) + offset); one persistent launch computes the
 * items in order, stores each item's rows into every rank's buffer, and
 * signals every rank ONCE per launch. wait_signals > 0: the launch ends once
 * that many more rank arrivals have reached this rank (e.g. world, one launch
 * later, to let ranks run one launch apart). */
vtq_status vtq_linear_list_gather(vtq_ctx* ctx, const vtq_list_item* items, int32_t n,
                                  vtq_gather* g, uint32_t flags, uint32_t wait_signals);
vtq_status vtq_gather_destroy(vtq_gather* g);

#ifdef __cplusplus
}
#endif
#endif /* VTQ_H */
