// decode_mk.h -- the persistent decode-step kernel (decode_mk.cu): one
// cooperative launch per decode step instead of ~180 dependent launches.
#pragma once
#include <cstddef>
#include <cstdint>
#include <vector>

#include <cuda_runtime.h>

#include "vtq_internal.h"

namespace vtq {

struct StepState {  // device-resident per-run state
  int pos;          // position of the step about to run
  uint32_t cur;     // token fed at `pos`
  int n_prompt, total, n_gen;
};

// A Llama decode step whose linears are all integer k-quant (Q4_K / Q6_K):
// q|k and gate|up back to back in HBM, v, wo, down, head.
struct MkLayer {
  DevMatrix wqk, wv, wo, w13, w2;
  const float *rms_att, *rms_ffn;
  const float *bq, *bk, *bv;  // QKV biases or null
};

struct MkModel {
  int dim, hidden, n_layers, n_heads, n_kv_heads, vocab, seq_len;
  float eps;
  bool neox;  // NeoX RoPE (Qwen2)
  DevMatrix embd, head;
  const float* rms_final;
  std::vector<MkLayer> layers;
  // Device buffers owned by the session.
  float *x, *xr, *q, *v, *xo, *xb2, *g, *logits, *kc, *vc, *rcos, *rsin;
  StepState* st;
  const uint32_t* prompt;
  uint32_t* out_tokens;
  unsigned* status;
};

struct MkPlan;

// True when the model fits the persistent kernel (every linear integer
// k-quant with at most 32 superblocks per row, activations fit its shared
// memory, and the cooperative grid fits the device).
bool mk_supported(const MkModel& m);
cudaError_t mk_build(const MkModel& m, MkPlan** out);
// Enqueue one decode step (memset of the barrier counter + the kernel).
// log != nullptr: the step's logits are also copied to log[pos * vocab].
cudaError_t mk_launch(MkPlan* plan, float* log, cudaStream_t st);
void mk_free(MkPlan* plan);

}  // namespace vtq
