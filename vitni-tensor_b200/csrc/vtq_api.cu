// vtq_api.cu -- the C ABI (include/vtq.h): contexts, resident weights,
// linear_dispatch-shaped entry points, and the context-free device API.
//
// Validation and error messages follow the reference functions each entry
// point replaces (vitni-tensor src/ops/quant.rs, src/model/forward_quantized.rs)
// so a caller sees the same failure for the same bad input. There is no CPU
// fallback: every arithmetic result comes from the sm_100a kernels.
#include <chrono>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/vtq.h"
#include "vtq_internal.h"

using namespace vtq;

struct vtq_ctx {
  int device = 0;
  cudaStream_t own = nullptr;
  cudaStream_t stream = nullptr;
  // io buffer: [status word | 252 B pad][y capacity][x capacity]
  uint8_t* io = nullptr;
  size_t io_cap = 0;
  // pinned host staging for host-pointer calls whose buffers are not pinned
  uint8_t* hio = nullptr;
  size_t hio_cap = 0;
  cudaEvent_t done = nullptr;  // end of a host-pointer call (polled, not blocked on)
  unsigned* list_cnt = nullptr;  // completion counters of vtq_linear_list (zeroed, left zeroed)
  uint8_t* list_rec = nullptr;   // vtq_linear_list's quantised activations (KQ_LIST_MAX records)
  unsigned* hstat = nullptr;     // page-locked completion word of in-place host-pointer lists
  uint64_t wait_limit_ns = 2000000000ull;  // bound of the gather arrival waits
  uint8_t* ws = nullptr;  // batched (tensor-core) linears' quantised activations
  size_t ws_cap = 0;
  std::string err;
};

struct vtq_weight {
  int device = 0;  // the owning context may be destroyed before the weight
  DevMatrix m{};
  uint8_t* buf = nullptr;
  size_t bytes = 0;
};

namespace {

constexpr size_t kStatusBytes = 256;

vtq_status fail(vtq_ctx* c, vtq_status s, const std::string& msg) {
  if (c) c->err = msg;
  return s;
}

vtq_status gpu_fail(vtq_ctx* c, cudaError_t e, const char* where) {
  const vtq_status s = (e == cudaErrorMemoryAllocation) ? VTQ_ERR_OOM : VTQ_ERR_GPU;
  char b[256];
  snprintf(b, sizeof b, "gpu error: %s: %s", where, cudaGetErrorString(e));
  return fail(c, s, b);
}

#define VTQ_CUDA(c, call)                                    \
  do {                                                       \
    cudaError_t e_ = (call);                                 \
    if (e_ != cudaSuccess) return gpu_fail((c), e_, #call);  \
  } while (0)

vtq_status ensure_io(vtq_ctx* c, size_t need) {
  if (need <= c->io_cap) return VTQ_OK;
  size_t cap = std::max(need, c->io_cap * 2);
  cap = (cap + 4095) / 4096 * 4096;
  if (c->io) {
    VTQ_CUDA(c, cudaStreamSynchronize(c->stream));
    cudaFree(c->io);
    c->io = nullptr;
    c->io_cap = 0;
  }
  VTQ_CUDA(c, cudaMalloc(&c->io, cap));
  VTQ_CUDA(c, cudaMemsetAsync(c->io, 0, kStatusBytes, c->stream));
  c->io_cap = cap;
  return VTQ_OK;
}

bool dtype_supported(int dtype) {
  return dtype == T_F32 || dtype == T_Q4_0 || dtype == T_Q5_0 || dtype == T_Q8_0 ||
         dtype == T_Q4_K || dtype == T_Q6_K;
}

// From this many activation rows on, integer Q4_K runs on the tensor-core
// GEMM (one weight pass for all rows) instead of the matvec (one weight pass
// per 4 rows). Overridable with VTQ_GEMM_MIN_BATCH.
const int64_t kGemmMinBatch = [] {
  const char* e = getenv("VTQ_GEMM_MIN_BATCH");
  return (e && *e) ? (int64_t)atoll(e) : (int64_t)16;
}();

// Launch the kernel that implements dtype's linear_dispatch arm.
bool uses_gemm(const DevMatrix& m, int64_t batch, uint32_t flags) {
  return m.dtype == T_Q4_K && !(flags & VTQ_Q4K_FLOAT) && batch >= kGemmMinBatch &&
         kq_gemm_supported(m, batch);
}

cudaError_t run_linear(const DevMatrix& m, const float* x, int64_t ldx, float* y, int64_t ldy,
                       int64_t batch, uint32_t flags, unsigned* status, cudaStream_t st,
                       uint8_t* ws = nullptr, size_t ws_bytes = 0) {
  if (uses_gemm(m, batch, flags))
    return launch_kq_gemm(m, x, ldx, batch, y, ldy, status, st, ws, ws_bytes);
  if (m.dtype == T_Q6_K || (m.dtype == T_Q4_K && !(flags & VTQ_Q4K_FLOAT)))
    return launch_kq_matvec(m, x, ldx, batch, y, ldy, status, st);
  return launch_canon_matvec(m, x, ldx, batch, y, ldy, status, st);
}

// The context's workspace for a batched linear, grown (after the stream has
// drained) when a larger batch arrives; freed with the context.
vtq_status ensure_ws(vtq_ctx* c, const DevMatrix& m, int64_t batch, uint32_t flags) {
  if (!uses_gemm(m, batch, flags)) return VTQ_OK;
  const size_t need = kq_gemm_workspace_bytes(m.in_feat, batch);
  if (need <= c->ws_cap) return VTQ_OK;
  const size_t cap = (std::max(need, c->ws_cap * 2) + 4095) / 4096 * 4096;
  if (c->ws) {
    VTQ_CUDA(c, cudaStreamSynchronize(c->stream));
    cudaFree(c->ws);
    c->ws = nullptr;
    c->ws_cap = 0;
  }
  VTQ_CUDA(c, cudaMalloc(&c->ws, cap));
  c->ws_cap = cap;
  return VTQ_OK;
}

// Kernel-side limits (shared-memory residency of one activation row set).
vtq_status check_kernel_limits(vtq_ctx* c, const DevMatrix& m, uint32_t flags) {
  const bool integer = m.dtype == T_Q6_K || (m.dtype == T_Q4_K && !(flags & VTQ_Q4K_FLOAT));
  if (m.in_feat > 32768)
    return fail(c, VTQ_ERR_NOT_IMPLEMENTED,
                std::string("vtq_linear: not implemented (in_feat > 32768 on the ") +
                    (integer ? "integer" : "canonical") + " kernel)");
  if (m.out_feat > INT32_MAX) return fail(c, VTQ_ERR_NOT_IMPLEMENTED, "vtq_linear: out_feat too large");
  return VTQ_OK;
}

// Host-pointer linear on a device-resident matrix: x in, kernel, y+status out.
// Page-locked (cudaHostAlloc'd or registered) host memory: copies to and from
// it run as asynchronous DMA; pageable memory goes through the context's
// pinned staging buffer instead.
bool host_pinned(const void* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

// The device address of page-locked host memory (nullptr if p is not
// page-locked and mapped).
void* host_mapped(const void* p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return a.type == cudaMemoryTypeHost ? a.devicePointer : nullptr;
}

vtq_status ensure_hio(vtq_ctx* c, size_t need) {
  if (need <= c->hio_cap) return VTQ_OK;
  const size_t cap = (std::max(need, c->hio_cap * 2) + 4095) / 4096 * 4096;
  if (c->hio) {
    VTQ_CUDA(c, cudaStreamSynchronize(c->stream));
    cudaFreeHost(c->hio);
    c->hio = nullptr;
    c->hio_cap = 0;
  }
  VTQ_CUDA(c, cudaHostAlloc(&c->hio, cap, cudaHostAllocDefault));
  c->hio_cap = cap;
  return VTQ_OK;
}

// Wait for everything enqueued on the context stream by polling an event: a
// host-pointer call is short and latency-bound, so the calling thread spins
// instead of sleeping in the driver.
vtq_status wait_call(vtq_ctx* c) {
  if (!c->done) VTQ_CUDA(c, cudaEventCreateWithFlags(&c->done, cudaEventDisableTiming));
  VTQ_CUDA(c, cudaEventRecord(c->done, c->stream));
  const auto t0 = std::chrono::steady_clock::now();
  for (unsigned i = 0;; i++) {
    const cudaError_t e = cudaEventQuery(c->done);
    if (e == cudaSuccess) return VTQ_OK;
    if (e != cudaErrorNotReady) VTQ_CUDA(c, e);
    // Device-side waits are bounded at 2 s; a call still running after a
    // minute means the device stopped answering.
    if ((i & 1023) == 1023 && std::chrono::steady_clock::now() - t0 > std::chrono::seconds(60))
      return fail(c, VTQ_ERR_TIMEOUT, "vtq_linear: the device did not finish the call in 60 s");
  }
}

vtq_status linear_host(vtq_ctx* c, const DevMatrix& m, const float* x, float* y, int64_t batch,
                       uint32_t flags) {
  if (vtq_status s = check_kernel_limits(c, m, flags)) return s;
  const size_t ybytes = (size_t)batch * m.out_feat * 4, xbytes = (size_t)batch * m.in_feat * 4;
  const size_t yoff = kStatusBytes, xoff = (yoff + ybytes + 255) / 256 * 256;
  if (vtq_status s = ensure_io(c, xoff + xbytes)) return s;
  float* dx = reinterpret_cast<float*>(c->io + xoff);
  float* dy = reinterpret_cast<float*>(c->io + yoff);
  unsigned* dstat = reinterpret_cast<unsigned*>(c->io);
  const bool x_pinned = host_pinned(x), y_pinned = host_pinned(y);
  // Staging layout: [status | y][x], the device io buffer's layout.
  if (vtq_status s = ensure_hio(c, (y_pinned ? kStatusBytes : yoff + ybytes) +
                                       (x_pinned ? 0 : xoff + xbytes)))
    return s;
  if (x_pinned) {
    VTQ_CUDA(c, cudaMemcpyAsync(dx, x, xbytes, cudaMemcpyHostToDevice, c->stream));
  } else {
    memcpy(c->hio + xoff, x, xbytes);
    VTQ_CUDA(c, cudaMemcpyAsync(dx, c->hio + xoff, xbytes, cudaMemcpyHostToDevice, c->stream));
  }
  if (vtq_status s = ensure_ws(c, m, batch, flags)) return s;
  VTQ_CUDA(c, run_linear(m, dx, m.in_feat, dy, m.out_feat, batch, flags, dstat, c->stream, c->ws,
                         c->ws_cap));
  uint32_t statbuf[kStatusBytes / 4];
  if (y_pinned) {
    VTQ_CUDA(c, cudaMemcpyAsync(c->hio, c->io, kStatusBytes, cudaMemcpyDeviceToHost, c->stream));
    VTQ_CUDA(c, cudaMemcpyAsync(y, dy, ybytes, cudaMemcpyDeviceToHost, c->stream));
  } else {
    // One D2H copy brings back the status word and y together.
    VTQ_CUDA(c, cudaMemcpyAsync(c->hio, c->io, yoff + ybytes, cudaMemcpyDeviceToHost, c->stream));
  }
  if (vtq_status s = wait_call(c)) return s;
  if (!y_pinned) memcpy(y, c->hio + yoff, ybytes);
  memcpy(statbuf, c->hio, kStatusBytes);
  if (statbuf[0] != 0) {
    VTQ_CUDA(c, cudaMemsetAsync(c->io, 0, 4, c->stream));
    return fail(c, VTQ_ERR_TIMEOUT, "vtq_linear: a device-side wait timed out");
  }
  return VTQ_OK;
}

// Upload `rows` packed rows from host bytes into a fresh device matrix.
vtq_status upload(vtq_ctx* c, int dtype, const uint8_t* bytes, int64_t in_feat, int64_t row0,
                  int64_t rows, vtq_weight** out) {
  auto* w = new vtq_weight();
  w->device = c->device;
  w->m.dtype = dtype;
  w->m.in_feat = in_feat;
  w->m.out_feat = rows;
  w->m.row_bytes = packed_row_bytes(dtype, in_feat);
  w->m.pitch = device_pitch(dtype, in_feat);
  w->bytes = (size_t)vtq_device_layout_bytes(dtype, in_feat, rows);
  cudaError_t e = cudaMalloc(&w->buf, std::max<size_t>(w->bytes, 256));
  if (e != cudaSuccess) {
    delete w;
    return gpu_fail(c, e, "cudaMalloc(weight)");
  }
  w->m.data = w->buf;
  const size_t raw = (size_t)rows * w->m.row_bytes;
  uint8_t* staging = nullptr;
  if (raw) {
    e = cudaMallocAsync(&staging, raw, c->stream);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(staging, bytes + row0 * w->m.row_bytes, raw, cudaMemcpyHostToDevice,
                          c->stream);
    if (e == cudaSuccess) e = launch_repack(staging, w->m, w->buf, c->stream);
    if (e == cudaSuccess)
      e = cudaMemsetAsync(w->buf + rows * w->m.pitch, 0, w->bytes - rows * w->m.pitch, c->stream);
    if (staging) cudaFreeAsync(staging, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  }
  if (e != cudaSuccess) {
    cudaFree(w->buf);
    delete w;
    return gpu_fail(c, e, "weight upload");
  }
  *out = w;
  return VTQ_OK;
}

// Shared body of the host-slice entry points: validate like the reference,
// upload, run, free.
vtq_status host_linear(vtq_ctx* c, int dtype, const float* x, const uint8_t* w, size_t wlen,
                       float* y, size_t batch, size_t in, size_t out, uint32_t flags) {
  if (!c || (!x && batch * in) || (!w && wlen) || (!y && batch * out))
    return fail(c, VTQ_ERR_INVALID_ARG, "null argument");
  if (out == 0 || batch == 0) return VTQ_OK;
  vtq_weight* wt = nullptr;
  if (vtq_status s = upload(c, dtype, w, (int64_t)in, 0, (int64_t)out, &wt)) return s;
  const vtq_status s = linear_host(c, wt->m, x, y, (int64_t)batch, flags | VTQ_PTR_HOST);
  cudaFree(wt->buf);
  delete wt;
  return s;
}

// Reference validation for the integer k-quant linears (quant.rs:944-949, :1068-1073).
vtq_status check_kquant(vtq_ctx* c, const char* fn, int bytes_per_sb, size_t wlen, size_t in,
                        size_t out) {
  if (in % 256) return fail(c, VTQ_ERR_INTERNAL, std::string(fn) + ": in_feat not a multiple of 256");
  if (wlen < out * (in / 256) * bytes_per_sb)
    return fail(c, VTQ_ERR_INTERNAL, std::string(fn) + ": weight shape mismatch");
  return VTQ_OK;
}

}  // namespace

namespace vtq {
unsigned long long& kernel_launch_count() {
  static thread_local unsigned long long n = 0;
  return n;
}

cudaError_t linear_any(const DevMatrix& m, const float* x, int64_t ldx, float* y, int64_t ldy,
                       int64_t batch, unsigned* status, cudaStream_t st) {
  return run_linear(m, x, ldx, y, ldy, batch, 0, status, st);
}
}  // namespace vtq

extern "C" {

vtq_status vtq_init(int device, vtq_ctx** out) {
  if (!out) return VTQ_ERR_INVALID_ARG;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return VTQ_ERR_GPU;
  auto* c = new vtq_ctx();
  c->device = device;
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&c->own, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    delete c;
    return VTQ_ERR_GPU;
  }
  c->stream = c->own;
  if (ensure_io(c, kStatusBytes + 64 * 1024) != VTQ_OK ||
      cudaMalloc(&c->list_cnt, (KQ_LIST_MAX + 2) * sizeof(unsigned)) != cudaSuccess ||
      cudaMemset(c->list_cnt, 0, (KQ_LIST_MAX + 2) * sizeof(unsigned)) != cudaSuccess ||
      cudaMalloc(&c->list_rec, KQ_LIST_MAX * KQ_LIST_REC) != cudaSuccess) {
    if (c->io) cudaFree(c->io);
    if (c->list_cnt) cudaFree(c->list_cnt);
    if (c->list_rec) cudaFree(c->list_rec);
    cudaStreamDestroy(c->own);
    delete c;
    return VTQ_ERR_OOM;
  }
  *out = c;
  return VTQ_OK;
}

vtq_status vtq_destroy(vtq_ctx* c) {
  if (!c) return VTQ_ERR_INVALID_ARG;
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  if (c->io) cudaFree(c->io);
  if (c->list_cnt) cudaFree(c->list_cnt);
  if (c->list_rec) cudaFree(c->list_rec);
  if (c->ws) cudaFree(c->ws);
  if (c->hstat) cudaFreeHost(c->hstat);
  if (c->hio) cudaFreeHost(c->hio);
  if (c->done) cudaEventDestroy(c->done);
  if (c->own) cudaStreamDestroy(c->own);
  delete c;
  return VTQ_OK;
}

const char* vtq_last_error(const vtq_ctx* c) { return c ? c->err.c_str() : "null context"; }

vtq_status vtq_set_stream(vtq_ctx* c, void* s) {
  if (!c) return VTQ_ERR_INVALID_ARG;
  c->stream = s ? static_cast<cudaStream_t>(s) : c->own;
  return VTQ_OK;
}

vtq_status vtq_synchronize(vtq_ctx* c) {
  if (!c) return VTQ_ERR_INVALID_ARG;
  VTQ_CUDA(c, cudaSetDevice(c->device));
  VTQ_CUDA(c, cudaStreamSynchronize(c->stream));
  // Errors of asynchronous calls surface here: a bounded device wait that ran
  // out left a flag in the context's status word.
  unsigned st = 0;
  VTQ_CUDA(c, cudaMemcpyAsync(&st, c->io, 4, cudaMemcpyDeviceToHost, c->stream));
  VTQ_CUDA(c, cudaStreamSynchronize(c->stream));
  if (st != 0) {
    VTQ_CUDA(c, cudaMemsetAsync(c->io, 0, 4, c->stream));
    VTQ_CUDA(c, cudaStreamSynchronize(c->stream));
    return fail(c, VTQ_ERR_TIMEOUT, "a device-side wait timed out");
  }
  return VTQ_OK;
}

vtq_status vtq_set_wait_limit(vtq_ctx* c, uint64_t ns) {
  if (!c || ns == 0) return fail(c, VTQ_ERR_INVALID_ARG, "vtq_set_wait_limit: limit must be > 0");
  c->wait_limit_ns = ns;
  return VTQ_OK;
}

vtq_status vtq_weight_upload(vtq_ctx* c, int32_t dtype, const uint8_t* bytes, size_t nbytes,
                             int64_t in_feat, int64_t out_feat, int64_t row_begin, int64_t row_end,
                             vtq_weight** out) {
  if (!c || !out || (!bytes && nbytes)) return fail(c, VTQ_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  if (!dtype_supported(dtype))
    return fail(c, VTQ_ERR_NOT_IMPLEMENTED,
                "vtq_weight_upload: not implemented (weight dtype not Q4_0 / Q4_K / Q5_0 / Q6_K / "
                "Q8_0 / F32)");
  if (in_feat <= 0 || out_feat < 0) return fail(c, VTQ_ERR_INTERNAL, "vtq_weight_upload: bad shape");
  const int64_t rb = packed_row_bytes(dtype, in_feat);
  if (rb < 0)
    return fail(c, VTQ_ERR_INTERNAL, "vtq_weight_upload: in_feat not a multiple of the block size");
  if (row_end < 0) row_end = out_feat;
  if (row_begin < 0 || row_begin > row_end || row_end > out_feat)
    return fail(c, VTQ_ERR_INTERNAL, "vtq_weight_upload: row range outside [0, out_feat]");
  if ((int64_t)nbytes < out_feat * rb)
    return fail(c, VTQ_ERR_INTERNAL, "vtq_weight_upload: weight blob too small");
  VTQ_CUDA(c, cudaSetDevice(c->device));
  return upload(c, dtype, bytes, in_feat, row_begin, row_end - row_begin, out);
}

vtq_status vtq_weight_free(vtq_weight* w) {
  if (!w) return VTQ_ERR_INVALID_ARG;
  cudaSetDevice(w->device);
  cudaFree(w->buf);  // cudaFree waits for work in flight on the device
  delete w;
  return VTQ_OK;
}

vtq_status vtq_weight_info(const vtq_weight* w, int32_t* dtype, int64_t* in_feat, int64_t* rows,
                           size_t* device_bytes) {
  if (!w) return VTQ_ERR_INVALID_ARG;
  if (dtype) *dtype = w->m.dtype;
  if (in_feat) *in_feat = w->m.in_feat;
  if (rows) *rows = w->m.out_feat;
  if (device_bytes) *device_bytes = w->bytes;
  return VTQ_OK;
}

vtq_status vtq_linear(vtq_ctx* c, const vtq_weight* w, const float* x, float* y, int64_t batch,
                      uint32_t flags) {
  if (!c || !w || !x || !y) return fail(c, VTQ_ERR_INVALID_ARG, "null argument");
  if (batch < 0) return fail(c, VTQ_ERR_INTERNAL, "vtq_linear: negative batch");
  if (batch == 0 || w->m.out_feat == 0) return VTQ_OK;
  VTQ_CUDA(c, cudaSetDevice(c->device));
  if (flags & VTQ_PTR_HOST) return linear_host(c, w->m, x, y, batch, flags);
  if (vtq_status s = check_kernel_limits(c, w->m, flags)) return s;
  if (vtq_status s = ensure_ws(c, w->m, batch, flags)) return s;
  VTQ_CUDA(c, run_linear(w->m, x, w->m.in_feat, y, w->m.out_feat, batch, flags,
                         reinterpret_cast<unsigned*>(c->io), c->stream, c->ws, c->ws_cap));
  return VTQ_OK;
}

vtq_status vtq_linear_list(vtq_ctx* c, const vtq_list_item* items, int32_t n, uint32_t flags) {
  if (!c || (!items && n)) return fail(c, VTQ_ERR_INVALID_ARG, "null argument");
  if (n == 0) return VTQ_OK;
  if (n < 0 || n > VTQ_LIST_MAX)
    return fail(c, VTQ_ERR_INVALID_ARG, "vtq_linear_list: 1..VTQ_LIST_MAX items");
  if (flags & VTQ_Q4K_FLOAT)
    return fail(c, VTQ_ERR_NOT_IMPLEMENTED, "vtq_linear_list: not implemented (integer regime only)");
  static_assert(VTQ_LIST_MAX == KQ_LIST_MAX, "list capacity");
  const bool host = (flags & VTQ_PTR_HOST) != 0;
  KqListItem it[KQ_LIST_MAX];
  size_t yoff[KQ_LIST_MAX], xoff[KQ_LIST_MAX], end = kStatusBytes;
  for (int i = 0; i < n; i++) {
    const vtq_list_item& s = items[i];
    if (!s.w || !s.x || !s.y) return fail(c, VTQ_ERR_INVALID_ARG, "vtq_linear_list: null item field");
    if (s.w->m.dtype != T_Q4_K && s.w->m.dtype != T_Q6_K)
      return fail(c, VTQ_ERR_NOT_IMPLEMENTED,
                  "vtq_linear_list: not implemented (weight dtype not Q4_K / Q6_K)");
    if (s.w->device != c->device)
      return fail(c, VTQ_ERR_INVALID_ARG, "vtq_linear_list: weight on another device");
    if (s.wait_for < -1 || s.wait_for >= i)
      return fail(c, VTQ_ERR_INVALID_ARG, "vtq_linear_list: wait_for must name an earlier item");
    if (host && s.wait_for >= 0)
      return fail(c, VTQ_ERR_INVALID_ARG,
                  "vtq_linear_list: wait_for needs device pointers (x would be a device y)");
    if (vtq_status st = check_kernel_limits(c, s.w->m, 0)) return st;
    it[i] = KqListItem{s.w->m, s.x, s.y, s.wait_for};
    yoff[i] = end;
    end = (end + (size_t)s.w->m.out_feat * 4 + 255) / 256 * 256;
  }
  VTQ_CUDA(c, cudaSetDevice(c->device));
  unsigned* dstat = reinterpret_cast<unsigned*>(c->io);
  if (!host) {
    VTQ_CUDA(c, launch_kq_list(it, n, c->list_cnt, c->list_rec, dstat, c->stream));
    return VTQ_OK;
  }
  // Host pointers, all page-locked: the kernel reads every x in place (once,
  // in its quantisation pass) and stores every y in place; the call is one
  // launch and a completion poll. The launch's last CTA writes the status
  // word to page-locked memory last; a sentinel there means it never ran.
  bool mapped = true;
  for (int i = 0; i < n && mapped; i++) {
    void* dx = host_mapped(items[i].x);
    void* dy = host_mapped(items[i].y);
    mapped = dx && dy;
    it[i].x = static_cast<const float*>(dx);
    it[i].y = static_cast<float*>(dy);
  }
  if (mapped) {
    if (!c->hstat) VTQ_CUDA(c, cudaHostAlloc(&c->hstat, 256, cudaHostAllocMapped));
    void* dh = host_mapped(c->hstat);
    if (!dh) return fail(c, VTQ_ERR_GPU, "vtq_linear_list: status word not mapped");
    *reinterpret_cast<volatile unsigned*>(c->hstat) = 0xFFFFFFFFu;
    VTQ_CUDA(c, launch_kq_list(it, n, c->list_cnt, c->list_rec, dstat, c->stream,
                               static_cast<unsigned*>(dh)));
    if (vtq_status s = wait_call(c)) return s;
    const unsigned st0 = *reinterpret_cast<volatile unsigned*>(c->hstat);
    if (st0 != 0) {
      VTQ_CUDA(c, cudaMemsetAsync(c->io, 0, 4, c->stream));
      return fail(c, VTQ_ERR_TIMEOUT, st0 == 0xFFFFFFFFu
                                          ? "vtq_linear_list: the launch did not complete"
                                          : "vtq_linear_list: a device-side wait timed out");
    }
    return VTQ_OK;
  }
  // Otherwise: device io buffer [status | y_0 | y_1 ... | x_0 | x_1 ...];
  // x's go in by DMA (straight from page-locked memory, else staged), one
  // D2H copy brings back the status word and every y.
  const size_t ybytes_end = end;
  for (int i = 0; i < n; i++) {
    xoff[i] = end;
    end = (end + (size_t)items[i].w->m.in_feat * 4 + 255) / 256 * 256;
  }
  if (vtq_status s = ensure_io(c, end)) return s;
  if (vtq_status s = ensure_hio(c, end)) return s;
  for (int i = 0; i < n; i++) {
    const size_t xb = (size_t)items[i].w->m.in_feat * 4;
    const void* src = items[i].x;
    if (!host_pinned(src)) {
      memcpy(c->hio + xoff[i], src, xb);
      src = c->hio + xoff[i];
    }
    VTQ_CUDA(c, cudaMemcpyAsync(c->io + xoff[i], src, xb, cudaMemcpyHostToDevice, c->stream));
    it[i].x = reinterpret_cast<const float*>(c->io + xoff[i]);
    it[i].y = reinterpret_cast<float*>(c->io + yoff[i]);
  }
  VTQ_CUDA(c, launch_kq_list(it, n, c->list_cnt, c->list_rec, dstat, c->stream));
  VTQ_CUDA(c, cudaMemcpyAsync(c->hio, c->io, ybytes_end, cudaMemcpyDeviceToHost, c->stream));
  if (vtq_status s = wait_call(c)) return s;
  for (int i = 0; i < n; i++)
    memcpy(items[i].y, c->hio + yoff[i], (size_t)items[i].w->m.out_feat * 4);
  uint32_t st0;
  memcpy(&st0, c->hio, 4);
  if (st0 != 0) {
    VTQ_CUDA(c, cudaMemsetAsync(c->io, 0, 4, c->stream));
    return fail(c, VTQ_ERR_TIMEOUT, "vtq_linear_list: a device-side wait timed out");
  }
  return VTQ_OK;
}

vtq_status vtq_linear_dispatch(vtq_ctx* c, int32_t dtype, const float* x, const uint8_t* w,
                               size_t wlen, size_t in, size_t out, float* y, uint32_t flags) {
  if (!c) return VTQ_ERR_INVALID_ARG;
  switch (dtype) {
    case T_Q4_0:
      return vtq_linear_q4_0(c, x, w, wlen, y, 1, in, out);
    case T_F32:
      if (wlen != out * in * 4)
        return fail(c, VTQ_ERR_INTERNAL, "linear_dispatch F32: weight size mismatch");
      return host_linear(c, dtype, x, w, wlen, y, 1, in, out, flags);
    case T_Q4_K:
      if (flags & VTQ_Q4K_FLOAT) return vtq_linear_q4_k_fused(c, x, w, wlen, y, 1, in, out);
      return vtq_linear_q4_k_integer(c, x, w, wlen, y, 1, in, out);
    case T_Q6_K:
      return vtq_linear_q6_k_integer(c, x, w, wlen, y, 1, in, out);
    case T_Q8_0:
    case T_Q5_0: {
      const char* nm = dtype == T_Q8_0 ? "Q8_0" : "Q5_0";
      if (in % 32)
        return fail(c, VTQ_ERR_INTERNAL, std::string(nm) + ": in_feat must be a multiple of 32");
      if (wlen < out * (in / 32) * (dtype == T_Q8_0 ? 34 : 22))
        return fail(c, VTQ_ERR_INTERNAL, std::string("linear_dispatch ") + nm + ": weight blob too small");
      return host_linear(c, dtype, x, w, wlen, y, 1, in, out, flags);
    }
    default:
      return fail(c, VTQ_ERR_NOT_IMPLEMENTED,
                  "forward_quantized::linear_dispatch: not implemented (weight dtype not Q4_0 / "
                  "Q4_K / Q5_0 / Q6_K / Q8_0 / F32)");
  }
}

vtq_status vtq_linear_q4_k_integer(vtq_ctx* c, const float* x, const uint8_t* w, size_t wlen,
                                   float* y, size_t batch, size_t in, size_t out) {
  if (!c) return VTQ_ERR_INVALID_ARG;
  if (vtq_status s = check_kquant(c, "linear_q4_k_integer", 144, wlen, in, out)) return s;
  return host_linear(c, T_Q4_K, x, w, wlen, y, batch, in, out, 0);
}

vtq_status vtq_linear_q6_k_integer(vtq_ctx* c, const float* x, const uint8_t* w, size_t wlen,
                                   float* y, size_t batch, size_t in, size_t out) {
  if (!c) return VTQ_ERR_INVALID_ARG;
  if (vtq_status s = check_kquant(c, "linear_q6_k_integer", 210, wlen, in, out)) return s;
  return host_linear(c, T_Q6_K, x, w, wlen, y, batch, in, out, 0);
}

vtq_status vtq_linear_q4_k_fused(vtq_ctx* c, const float* x, const uint8_t* w, size_t wlen,
                                 float* y, size_t batch, size_t in, size_t out) {
  if (!c) return VTQ_ERR_INVALID_ARG;
  if (in % 256) return fail(c, VTQ_ERR_INTERNAL, "linear_q4_k_fused: in_feat not a multiple of 256");
  if (wlen < out * (in / 256) * 144)
    return fail(c, VTQ_ERR_INTERNAL, "linear_q4_k_fused: weight shape mismatch");
  return host_linear(c, T_Q4_K, x, w, wlen, y, batch, in, out, VTQ_Q4K_FLOAT);
}

vtq_status vtq_linear_q4_0(vtq_ctx* c, const float* x, const uint8_t* w, size_t wlen, float* y,
                           size_t batch, size_t in, size_t out) {
  if (!c) return VTQ_ERR_INVALID_ARG;
  if (in % 32) return fail(c, VTQ_ERR_INTERNAL, "linear_q4_0: in_feat must be multiple of 32");
  if (wlen != out * (in / 32) * 18)
    return fail(c, VTQ_ERR_INTERNAL, "linear_q4_0: weight blob length mismatch");
  return host_linear(c, T_Q4_0, x, w, wlen, y, batch, in, out, 0);
}

int64_t vtq_device_layout_bytes(int32_t dtype, int64_t in_feat, int64_t rows) {
  const int64_t p = device_pitch(dtype, in_feat);
  if (p < 0 || rows < 0) return -1;
  return p * rows + 16;
}

vtq_status vtq_device_repack(int32_t dtype, int64_t in_feat, int64_t rows, const uint8_t* src_dev,
                             uint8_t* dst_dev, void* s) {
  if (!dtype_supported(dtype)) return VTQ_ERR_NOT_IMPLEMENTED;
  const int64_t rb = packed_row_bytes(dtype, in_feat);
  if (rb < 0 || rows < 0) return VTQ_ERR_INTERNAL;
  if ((!src_dev || !dst_dev) && rows) return VTQ_ERR_INVALID_ARG;
  DevMatrix m{dtype, in_feat, rows, rb, device_pitch(dtype, in_feat), dst_dev};
  cudaStream_t st = static_cast<cudaStream_t>(s);
  if (launch_repack(src_dev, m, dst_dev, st) != cudaSuccess) return VTQ_ERR_GPU;
  if (cudaMemsetAsync(dst_dev + rows * m.pitch, 0, 16, st) != cudaSuccess) return VTQ_ERR_GPU;
  return VTQ_OK;
}

size_t vtq_linear_device_workspace_bytes(int32_t dtype, int64_t in_feat, int64_t batch,
                                         uint32_t flags) {
  const int64_t rb = packed_row_bytes(dtype, in_feat);
  if (rb < 0 || batch < 0) return 0;
  DevMatrix m{dtype, in_feat, 1, rb, device_pitch(dtype, in_feat), nullptr};
  return uses_gemm(m, batch, flags) ? kq_gemm_workspace_bytes(in_feat, batch) : 0;
}

vtq_status vtq_linear_device_ws(int32_t dtype, const uint8_t* w_dev, int64_t in_feat, int64_t rows,
                                const float* x_dev, int64_t ldx, float* y_dev, int64_t ldy,
                                int64_t batch, uint32_t flags, uint32_t* status_dev,
                                void* workspace, size_t workspace_bytes, void* s) {
  if (!dtype_supported(dtype)) return VTQ_ERR_NOT_IMPLEMENTED;
  const int64_t rb = packed_row_bytes(dtype, in_feat);
  if (rb < 0 || rows < 0 || batch < 0 || ldx < in_feat || ldy < rows) return VTQ_ERR_INTERNAL;
  if (batch == 0 || rows == 0) return VTQ_OK;
  if (!w_dev || !x_dev || !y_dev) return VTQ_ERR_INVALID_ARG;
  if (in_feat > 32768) return VTQ_ERR_NOT_IMPLEMENTED;
  if (reinterpret_cast<uintptr_t>(w_dev) & 15u) return VTQ_ERR_INVALID_ARG;
  DevMatrix m{dtype, in_feat, rows, rb, device_pitch(dtype, in_feat), w_dev};
  const size_t need = uses_gemm(m, batch, flags) ? kq_gemm_workspace_bytes(in_feat, batch) : 0;
  if (need && (!workspace || workspace_bytes < need ||
               (reinterpret_cast<uintptr_t>(workspace) & 255u)))
    return VTQ_ERR_INVALID_ARG;
  if (run_linear(m, x_dev, ldx, y_dev, ldy, batch, flags, status_dev, static_cast<cudaStream_t>(s),
                 static_cast<uint8_t*>(workspace), workspace_bytes) != cudaSuccess)
    return VTQ_ERR_GPU;
  return VTQ_OK;
}

vtq_status vtq_linear_device(int32_t dtype, const uint8_t* w_dev, int64_t in_feat, int64_t rows,
                             const float* x_dev, int64_t ldx, float* y_dev, int64_t ldy,
                             int64_t batch, uint32_t flags, uint32_t* status_dev, void* s) {
  if (!dtype_supported(dtype)) return VTQ_ERR_NOT_IMPLEMENTED;
  const int64_t rb = packed_row_bytes(dtype, in_feat);
  if (rb < 0 || rows < 0 || batch < 0 || ldx < in_feat || ldy < rows) return VTQ_ERR_INTERNAL;
  if (batch == 0 || rows == 0) return VTQ_OK;
  if (!w_dev || !x_dev || !y_dev) return VTQ_ERR_INVALID_ARG;
  if (in_feat > 32768) return VTQ_ERR_NOT_IMPLEMENTED;
  if (reinterpret_cast<uintptr_t>(w_dev) & 15u) return VTQ_ERR_INVALID_ARG;
  DevMatrix m{dtype, in_feat, rows, rb, device_pitch(dtype, in_feat), w_dev};
  if (run_linear(m, x_dev, ldx, y_dev, ldy, batch, flags, status_dev, static_cast<cudaStream_t>(s)) !=
      cudaSuccess)
    return VTQ_ERR_GPU;
  return VTQ_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Row-sharded linears with the all-gather fused into the kernel (NVLink P2P).

struct vtq_gather {
  int device = 0, world = 0, rank = 0;
  uint8_t* base = nullptr;                    // [counters 256 B | y]
  uint8_t* peer[kMaxRanks] = {};              // every rank's base (own included)
  size_t y_floats = 0;
};

namespace {
constexpr size_t kGatherHdr = 256;  // cnt @0, expected @4, done @8
}

vtq_status vtq_gather_create(vtq_ctx* c, int32_t world, int32_t rank, size_t y_floats,
                             vtq_gather** out, uint8_t* ipc_handle) {
  if (!c || !out || !ipc_handle) return fail(c, VTQ_ERR_INVALID_ARG, "null argument");
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || y_floats == 0)
    return fail(c, VTQ_ERR_INVALID_ARG, "vtq_gather_create: bad world / rank / size");
  VTQ_CUDA(c, cudaSetDevice(c->device));
  auto* g = new vtq_gather;
  g->device = c->device;
  g->world = world;
  g->rank = rank;
  g->y_floats = y_floats;
  cudaError_t e = cudaMalloc(&g->base, kGatherHdr + y_floats * 4);
  if (e == cudaSuccess) e = cudaMemset(g->base, 0, kGatherHdr + y_floats * 4);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, g->base);
  if (e != cudaSuccess) {
    if (g->base) cudaFree(g->base);
    delete g;
    return fail(c, VTQ_ERR_GPU, std::string("vtq_gather_create: ") + cudaGetErrorString(e));
  }
  static_assert(sizeof(h) == 64, "IPC handle size");
  memcpy(ipc_handle, &h, 64);
  g->peer[rank] = g->base;
  *out = g;
  return VTQ_OK;
}

vtq_status vtq_gather_connect(vtq_gather* g, const uint8_t* handles) {
  if (!g || !handles) return VTQ_ERR_INVALID_ARG;
  if (cudaSetDevice(g->device) != cudaSuccess) return VTQ_ERR_GPU;
  for (int q = 0; q < g->world; q++) {
    if (q == g->rank || g->peer[q]) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, handles + 64 * q, 64);
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
      return VTQ_ERR_GPU;
    g->peer[q] = static_cast<uint8_t*>(p);
  }
  return VTQ_OK;
}

float* vtq_gather_y(vtq_gather* g) {
  return g ? reinterpret_cast<float*>(g->base + kGatherHdr) : nullptr;
}

vtq_status vtq_linear_gather_wait(vtq_ctx* c, const vtq_weight* w, const float* x,
                                  int64_t batch, vtq_gather* g, int64_t y_offset, int64_t ldy,
                                  int64_t row0, uint32_t flags, uint32_t wait_signals) {
  if (!c || !w || !x || !g) return fail(c, VTQ_ERR_INVALID_ARG, "null argument");
  for (int q = 0; q < g->world; q++)
    if (!g->peer[q]) return fail(c, VTQ_ERR_INVALID_ARG, "vtq_linear_gather: gather not connected");
  const DevMatrix& m = w->m;
  if (!(m.dtype == T_Q6_K || (m.dtype == T_Q4_K && !(flags & VTQ_Q4K_FLOAT))))
    return fail(c, VTQ_ERR_NOT_IMPLEMENTED,
                "vtq_linear_gather: not implemented (fused gather needs an integer k-quant weight)");
  if (batch < 1 || batch > 4)
    return fail(c, VTQ_ERR_NOT_IMPLEMENTED, "vtq_linear_gather: batch must be 1..4");
  if (row0 < 0 || row0 + m.out_feat > ldy || y_offset < 0 ||
      (size_t)(y_offset + batch * ldy) > g->y_floats)
    return fail(c, VTQ_ERR_INVALID_ARG, "vtq_linear_gather: rows outside the gather buffer");
  if (vtq_status s = check_kernel_limits(c, m, flags)) return s;
  VTQ_CUDA(c, cudaSetDevice(c->device));
  GatherTarget t{};
  t.world = g->world;
  t.row0 = row0;
  t.ldy = ldy;
  for (int q = 0; q < g->world; q++) {
    t.y[q] = reinterpret_cast<float*>(g->peer[q] + kGatherHdr) + y_offset;
    t.cnt[q] = reinterpret_cast<unsigned*>(g->peer[q]);
  }
  t.done = reinterpret_cast<unsigned*>(g->base + 8);
  t.my_cnt = reinterpret_cast<unsigned*>(g->base);
  t.expected = reinterpret_cast<unsigned*>(g->base + 4);
  t.wait_signals = wait_signals;
  t.signal = (flags & VTQ_GATHER_DEFER) ? 0 : 1;
  t.limit_ns = c->wait_limit_ns;
  if (!t.signal && wait_signals)
    return fail(c, VTQ_ERR_INVALID_ARG, "vtq_linear_gather: a deferred launch cannot wait");
  VTQ_CUDA(c, launch_kq_matvec(m, x, m.in_feat, batch, nullptr, 0,
                               reinterpret_cast<unsigned*>(c->io), c->stream, &t));
  return VTQ_OK;
}

vtq_status vtq_linear_gather(vtq_ctx* c, const vtq_weight* w, const float* x, int64_t batch,
                             vtq_gather* g, int64_t y_offset, int64_t ldy, int64_t row0,
                             uint32_t flags) {
  return vtq_linear_gather_wait(c, w, x, batch, g, y_offset, ldy, row0, flags, 0);
}

vtq_status vtq_gather_wait(vtq_ctx* c, vtq_gather* g, uint32_t signals) {
  if (!c || !g) return VTQ_ERR_INVALID_ARG;
  VTQ_CUDA(c, cudaSetDevice(c->device));
  VTQ_CUDA(c, launch_gather_wait(reinterpret_cast<unsigned*>(g->base),
                                 reinterpret_cast<unsigned*>(g->base + 4), signals,
                                 reinterpret_cast<unsigned*>(c->io), c->stream,
                                 c->wait_limit_ns));
  return VTQ_OK;
}

vtq_status vtq_linear_list_gather(vtq_ctx* c, const vtq_list_item* items, int32_t n,
                                  vtq_gather* g, uint32_t flags, uint32_t wait_signals) {
  if (!c || !g || (!items && n)) return fail(c, VTQ_ERR_INVALID_ARG, "null argument");
  if (n < 1 || n > VTQ_LIST_MAX)
    return fail(c, VTQ_ERR_INVALID_ARG, "vtq_linear_list_gather: 1..VTQ_LIST_MAX items");
  if (flags & (VTQ_PTR_HOST | VTQ_Q4K_FLOAT))
    return fail(c, VTQ_ERR_NOT_IMPLEMENTED,
                "vtq_linear_list_gather: not implemented (device pointers, integer regime only)");
  for (int q = 0; q < g->world; q++)
    if (!g->peer[q])
      return fail(c, VTQ_ERR_INVALID_ARG, "vtq_linear_list_gather: gather not connected");
  const float* ybeg = reinterpret_cast<const float*>(g->base + kGatherHdr);
  const float* yend = ybeg + g->y_floats;
  KqListItem it[KQ_LIST_MAX];
  for (int i = 0; i < n; i++) {
    const vtq_list_item& s = items[i];
    if (!s.w || !s.x || !s.y)
      return fail(c, VTQ_ERR_INVALID_ARG, "vtq_linear_list_gather: null item field");
    if (s.w->m.dtype != T_Q4_K && s.w->m.dtype != T_Q6_K)
      return fail(c, VTQ_ERR_NOT_IMPLEMENTED,
                  "vtq_linear_list_gather: not implemented (weight dtype not Q4_K / Q6_K)");
    if (s.wait_for < -1 || s.wait_for >= i)
      return fail(c, VTQ_ERR_INVALID_ARG, "vtq_linear_list_gather: wait_for must name an earlier item");
    if (s.y < ybeg || s.y + s.w->m.out_feat > yend)
      return fail(c, VTQ_ERR_INVALID_ARG,
                  "vtq_linear_list_gather: y must lie in this rank's gather buffer");
    if (vtq_status st = check_kernel_limits(c, s.w->m, 0)) return st;
    it[i] = KqListItem{s.w->m, s.x, s.y, s.wait_for};
  }
  KqListGather lg;
  lg.world = g->world;
  lg.rank = g->rank;
  for (int q = 0; q < g->world; q++) {
    lg.peer_off[q] = g->peer[q] - g->base;
    lg.cnt[q] = reinterpret_cast<unsigned*>(g->peer[q]);
  }
  lg.my_cnt = reinterpret_cast<unsigned*>(g->base);
  lg.expected = reinterpret_cast<unsigned*>(g->base + 4);
  lg.wait_signals = wait_signals;
  lg.limit_ns = c->wait_limit_ns;
  VTQ_CUDA(c, cudaSetDevice(c->device));
  VTQ_CUDA(c, launch_kq_list(it, n, c->list_cnt, c->list_rec, reinterpret_cast<unsigned*>(c->io),
                             c->stream, nullptr, &lg));
  return VTQ_OK;
}

vtq_status vtq_gather_destroy(vtq_gather* g) {
  if (!g) return VTQ_OK;
  cudaSetDevice(g->device);
  cudaDeviceSynchronize();
  for (int q = 0; q < g->world; q++)
    if (q != g->rank && g->peer[q]) cudaIpcCloseMemHandle(g->peer[q]);
  cudaFree(g->base);
  delete g;
  return VTQ_OK;
}
