// libm_api.cu -- C exports of the software transcendentals (vtq_libm.h) the
// decode path shares with the host: RoPE tables are built from vtq_powf,
// vtq_cosf and vtq_sinf; the device computes SiLU / softmax with the same expf.
#include "../../include/vtq.h"
#include "vtq_libm.h"

namespace {

// The sweep outputs that the decode kernels compute on the device: expf
// (softmax), the correctly rounded sqrt, and the SiLU sigmoid. sin / cos / pow
// are only used on the host (RoPE tables) and are filled in by the host.
__global__ void libm_sweep_kernel(const float* in, size_t n, float* out) {
  namespace L = vtq::libm;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const float v = in[i];
    float* o = out + 7 * i;
    o[0] = L::expf(v);
    o[1] = __fsqrt_rn(fabsf(v));
    o[6] = __fdiv_rn(1.0f, __fadd_rn(1.0f, L::expf(-v)));
  }
}

}  // namespace

extern "C" {

float vtq_expf(float x) { return vtq::libm::expf(x); }
float vtq_sinf(float x) { return vtq::libm::sinf(x); }
float vtq_cosf(float x) { return vtq::libm::cosf(x); }
float vtq_powf(float x, float y) { return vtq::libm::powf(x, y); }

void vtq_libm_sweep(const float* in, size_t n, float* out) {
  namespace L = vtq::libm;
  for (size_t i = 0; i < n; i++) {
    const float v = in[i];
    float* o = out + 7 * i;
    o[0] = L::expf(v);
    o[1] = std::sqrt(std::fabs(v));
    o[2] = L::cosf(v);
    o[3] = L::sinf(v);
    o[4] = L::powf(10000.0f, v / 64.0f);
    o[5] = L::powf(1000000.0f, v / 64.0f);
    o[6] = 1.0f / (1.0f + L::expf(-v));
  }
}

int vtq_libm_sweep_device(const float* in, size_t n, float* out) {
  float *din = nullptr, *dout = nullptr;
  int st = 0;
  if (cudaMalloc(&din, n * 4) != cudaSuccess || cudaMalloc(&dout, n * 7 * 4) != cudaSuccess ||
      cudaMemcpy(din, in, n * 4, cudaMemcpyHostToDevice) != cudaSuccess)
    st = VTQ_ERR_GPU;
  if (!st) {
    libm_sweep_kernel<<<296, 256>>>(din, n, dout);
    if (cudaMemcpy(out, dout, n * 7 * 4, cudaMemcpyDeviceToHost) != cudaSuccess) st = VTQ_ERR_GPU;
  }
  namespace L = vtq::libm;
  for (size_t i = 0; !st && i < n; i++) {
    const float v = in[i];
    float* o = out + 7 * i;
    o[2] = L::cosf(v);
    o[3] = L::sinf(v);
    o[4] = L::powf(10000.0f, v / 64.0f);
    o[5] = L::powf(1000000.0f, v / 64.0f);
  }
  cudaFree(din);
  cudaFree(dout);
  return st;
}

}  // extern "C"
