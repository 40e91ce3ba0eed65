// noalloc.cu -- vtq_linear_host_noalloc: the integer k-quant linear with host
// inputs and outputs, for callers that cannot allocate device memory.
//
// Some hosts cannot call cudaMalloc at all: a caller that runs inside a memory
// pool it does not own (an allocator-owned runtime, a plugin loaded into a
// process whose device memory is budgeted by someone else), or a caller on a
// path where allocation is forbidden because it can block or fail. The normal
// host-pointer path (vtq_linear with VTQ_PTR_HOST) stages x, y and the kernel's
// status word in a context buffer obtained with cudaMalloc. This variant keeps
// that staging in one file-scope device array instead, so a call allocates
// nothing; the weights stay in caller-owned device memory.
//
// Limits and sharing rules:
//  * the array holds kNoAllocFloats floats (1 MiB): the status word plus
//    batch*in_feat x values plus batch*rows y values must fit, else the call
//    returns VTQ_ERR_INTERNAL without touching the device;
//  * every loaded GPU keeps the array until the process exits;
//  * all calls on a device share it and it keeps the last call's contents, so
//    calls whose work overlaps on the GPU race; the status word is cleared on
//    every call;
//  * the first call on a device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current); make that first call
//    before any stream capture;
//  * that address is kept for the life of the process: it belongs to the
//    device's primary context, so a process that resets the device
//    (cudaDeviceReset) must not call this entry point again afterwards.
#include <mutex>

#include "../../include/vtq.h"
#include "vtq_internal.h"

namespace {

constexpr size_t kNoAllocFloats = 256 * 1024;  // 1 MiB of staging
constexpr size_t kStatusFloats = 64;           // status word + padding (256 B)

static __device__ __align__(256) float g_noalloc_scratch[kNoAllocFloats];

constexpr int kMaxDevices = 64;
float* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// The device address of g_noalloc_scratch on `device` (looked up once, with
// that device current). In host code the array's name is only a host-side
// stand-in; kernels must be given this address.
cudaError_t scratch_on(int device, float** out) {
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_addr[device] = static_cast<float*>(p);
  }
  *out = g_scratch_addr[device];
  return cudaSuccess;
}

}  // namespace

extern "C" vtq_status vtq_linear_host_noalloc(int32_t dtype, const uint8_t* w_dev, int64_t in_feat,
                                              int64_t rows, const float* x, float* y,
                                              int64_t batch, void* cuda_stream) {
  using namespace vtq;
  if (dtype != T_Q4_K && dtype != T_Q6_K) return VTQ_ERR_NOT_IMPLEMENTED;
  if (in_feat <= 0 || in_feat % 256 || in_feat > 32768 || rows < 0 || batch < 0)
    return VTQ_ERR_INTERNAL;
  if (batch == 0 || rows == 0) return VTQ_OK;
  if (!w_dev || !x || !y) return VTQ_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(w_dev) & 15u) return VTQ_ERR_INVALID_ARG;
  const size_t xn = (size_t)batch * (size_t)in_feat, yn = (size_t)batch * (size_t)rows;
  if (kStatusFloats + xn + yn > kNoAllocFloats) return VTQ_ERR_INTERNAL;  // over the limit
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) return VTQ_ERR_GPU;
  float* base = nullptr;
  if (scratch_on(device, &base) != cudaSuccess) return VTQ_ERR_GPU;
  unsigned* status = reinterpret_cast<unsigned*>(base);
  float* dx = base + kStatusFloats;  // 256-byte aligned
  float* dy = dx + (xn + 63) / 64 * 64;
  cudaStream_t st = static_cast<cudaStream_t>(cuda_stream);
  const DevMatrix m{dtype, in_feat, rows, packed_row_bytes(dtype, in_feat),
                    device_pitch(dtype, in_feat), w_dev};
  unsigned stat = 0;
  if (cudaMemsetAsync(status, 0, sizeof(unsigned), st) != cudaSuccess ||
      cudaMemcpyAsync(dx, x, xn * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
      launch_kq_matvec(m, dx, in_feat, batch, dy, rows, status, st) != cudaSuccess ||
      cudaMemcpyAsync(y, dy, yn * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaMemcpyAsync(&stat, status, sizeof stat, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return VTQ_ERR_GPU;
  return stat ? VTQ_ERR_TIMEOUT : VTQ_OK;
}
