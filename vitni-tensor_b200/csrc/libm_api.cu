// libm_api.cu -- C exports of the software transcendentals (vtq_libm.h) the
// decode path shares with the host: RoPE tables are built from vtq_powf,
// vtq_cosf and vtq_sinf; the device computes SiLU / softmax with the same expf.
#include "../../include/vtq.h"
#include "vtq_libm.h"

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

}  // extern "C"
