// exact_sum.cu -- entry points that exercise exact_sum.cuh: the run/crossing
// plan evaluated on the host (one step after another, the arithmetic the CTA
// uses), and the CTA version on the device, both for tests against the plain
// left-to-right loop.
#include <cuda_runtime.h>

#include <cstring>
#include <vector>

#include "exact_sum.cuh"
#include "../../include/vtq.h"
#include "vtq_internal.h"

namespace vtq {
namespace {

using namespace xsum;

__global__ void exact_sum_test_kernel(const float* a, int n, float* out) {
  __shared__ Scratch sc;
  const float s = exact_serial_sum<16>(a + (size_t)blockIdx.x * n, n, &sc, threadIdx.x, blockDim.x,
                                   [] { __syncthreads(); });
  if (threadIdx.x == 0) out[blockIdx.x] = s;
}

}  // namespace
}  // namespace vtq

using namespace vtq;
using namespace vtq::xsum;

// Host evaluation of the plan: *fallback = 1 when verification failed or the
// input was not finite (the result is then the plain loop's).
extern "C" float vtq_exact_sum_host(const float* a, size_t n, int* fallback) {
  float plain = 0.0f;
  for (size_t i = 0; i < n; i++) plain = plain + a[i];
  bool ok = true;
  for (size_t i = 0; i < n && ok; i++) ok = (fbits(a[i]) >> 23) != 0xff;
  float s = 0.0f;
  if (ok) {
    Seg r{0, Map{0, 0}, kNone};
    float p_prev = 0.0f;
    for (size_t j = 0; j < n && ok; j++) {
      const float p = p_prev + a[j];  // the fp32 prefix: here the states themselves
      const int us = classify(p_prev, p, margin((int)j, 24));
      if (us == kNone) {
        if (r.us != kNone) ok = apply_run(s, r.m, r.us);
        s = s + a[j];
        r = Seg{1, Map{0, 0}, kNone};
      } else {
        r = seg_combine(r, Seg{0, term_map(a[j], us), us});
      }
      p_prev = p;
    }
    if (ok && r.us != kNone) ok = apply_run(s, r.m, r.us);
  }
  if (fallback) *fallback = ok ? 0 : 1;
  return ok ? s : plain;
}

// Device: nvec vectors of n terms (host memory), one CTA of nthr threads each.
extern "C" int vtq_exact_sum_device(const float* host, int nvec, int n, int nthr, float* out) {
  if (nvec <= 0 || n <= 0 || nthr < 32 || nthr > 1024 || nthr % 32) return VTQ_ERR_INVALID_ARG;
  float *da = nullptr, *dout = nullptr;
  cudaError_t e = cudaMalloc(&da, (size_t)nvec * n * 4);
  if (e == cudaSuccess) e = cudaMalloc(&dout, (size_t)nvec * 4);
  if (e == cudaSuccess) e = cudaMemcpy(da, host, (size_t)nvec * n * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) {
    exact_sum_test_kernel<<<nvec, nthr>>>(da, n, dout);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpy(out, dout, (size_t)nvec * 4, cudaMemcpyDeviceToHost);
  cudaFree(da);
  cudaFree(dout);
  return e == cudaSuccess ? VTQ_OK : VTQ_ERR_GPU;
}
