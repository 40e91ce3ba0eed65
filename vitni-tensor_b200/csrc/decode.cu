// decode.cu -- the reference's quantized Llama decode step on the device.
//
// Mirrors src/model/forward_quantized.rs:329-649 (step_with_recorders, Llama
// path) and the prompt + greedy loop of src/model/inference.rs:312-327, with
// the weights resident in HBM and every linear on the sm_100a kernels
// (kquant_matvec.cu / canon_matvec.cu). One decode step is captured once as a
// CUDA graph; the position and the current token live in device memory and the
// last kernel of a step selects the next token on the device, so a whole
// prompt + generation is a sequence of graph launches with no host round trip.
//
// Order-pinned pieces (each a single thread or an exact parallel map):
//   rms_norm       serial sum of squares over the row (rms_norm.rs:97-100)
//   attention      serial q.k over head_dim, serial softmax sum, serial P.V
//                  over positions (forward_quantized.rs:476-500, :925-941)
//   RoPE           host tables from the restated powf/cosf/sinf (vtq_libm.h)
//   SwiGLU/softmax expf restated on the device (vtq_libm.h)
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/vtq.h"
#include "vtq_device.cuh"
#include "vtq_internal.h"
#include "vtq_libm.h"
#include "decode_ops.cuh"
#include "exact_sum.cuh"
#include "decode_mk.h"

namespace vtq {

cudaError_t launch_kq_or_canon(const DevMatrix& m, const float* x, float* y, unsigned* status,
                               cudaStream_t st) {
  if (m.dtype == T_Q4_K || m.dtype == T_Q6_K)
    return launch_kq_matvec(m, x, m.in_feat, 1, y, m.out_feat, status, st);
  return launch_canon_matvec(m, x, m.in_feat, 1, y, m.out_feat, status, st);
}

namespace {

// Programmatic dependent launch: every kernel of a step waits for its
// predecessor before touching data, then lets its own successor start (the
// next matvec streams its weights while this kernel runs).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_release() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), unsigned grid, unsigned block, size_t smem,
                       cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------- GGUF ----
// Zero-copy parse of a GGUF v2/v3 blob (src/model/gguf.rs:305-422): metadata
// scalars and strings, tensor infos, alignment, tensor byte ranges.
struct GTensor {
  std::vector<uint64_t> shape;
  int dtype;
  const uint8_t* bytes;
  size_t len;
};
struct GMeta {
  int type;
  uint64_t u;  // unsigned / bool / signed as two's complement
  double f;
  std::string s;
  uint64_t arr_len;
};
struct Gguf {
  std::map<std::string, GMeta> meta;
  std::map<std::string, GTensor> tensors;
};

struct GgufError {
  vtq_status status;
  const char* msg;
};

struct Cur {
  const uint8_t* p;
  size_t n, pos = 0;
  const uint8_t* take(size_t k) {
    if (k > n - pos) throw GgufError{VTQ_ERR_TRUNCATED, "gguf: read past end"};
    const uint8_t* r = p + pos;
    pos += k;
    return r;
  }
  uint32_t u32() { uint32_t v; memcpy(&v, take(4), 4); return v; }
  uint64_t u64() { uint64_t v; memcpy(&v, take(8), 8); return v; }
  std::string str() {
    const uint64_t k = u64();
    if (k > (1u << 20)) throw GgufError{VTQ_ERR_MALFORMED, "gguf: string length > 1 MiB"};
    const uint8_t* s = take((size_t)k);
    return std::string(reinterpret_cast<const char*>(s), (size_t)k);
  }
};

size_t value_size(int t) {
  switch (t) {
    case 0: case 1: case 7: return 1;
    case 2: case 3: return 2;
    case 4: case 5: case 6: return 4;
    case 10: case 11: case 12: return 8;
    default: return 0;
  }
}

GMeta read_value(Cur& c, int t) {
  GMeta m{};
  m.type = t;
  switch (t) {
    case 0: m.u = *c.take(1); break;
    case 1: m.u = (uint64_t)(int64_t)(int8_t)*c.take(1); break;
    case 2: { uint16_t v; memcpy(&v, c.take(2), 2); m.u = v; break; }
    case 3: { int16_t v; memcpy(&v, c.take(2), 2); m.u = (uint64_t)(int64_t)v; break; }
    case 4: m.u = c.u32(); break;
    case 5: m.u = (uint64_t)(int64_t)(int32_t)c.u32(); break;
    case 6: { uint32_t b = c.u32(); float f; memcpy(&f, &b, 4); m.f = f; break; }
    case 7: m.u = *c.take(1) != 0; break;
    case 8: m.s = c.str(); break;
    case 9: {
      const int et = (int)c.u32();
      if (et == 9) throw GgufError{VTQ_ERR_MALFORMED, "gguf: nested arrays not supported"};
      if (et > 12) throw GgufError{VTQ_ERR_MALFORMED, "gguf: bad array elem type"};
      m.arr_len = c.u64();
      if (et == 8) {
        for (uint64_t i = 0; i < m.arr_len; i++) c.str();
      } else {
        const unsigned __int128 total = (unsigned __int128)m.arr_len * value_size(et);
        if (total > c.n) throw GgufError{VTQ_ERR_TRUNCATED, "gguf: array past end"};
        c.take((size_t)total);
      }
      break;
    }
    case 10: m.u = c.u64(); break;
    case 11: m.u = c.u64(); break;
    case 12: { uint64_t b = c.u64(); memcpy(&m.f, &b, 8); break; }
    default: throw GgufError{VTQ_ERR_MALFORMED, "gguf: unknown value type"};
  }
  return m;
}

Gguf parse_gguf(const uint8_t* blob, size_t len) {
  Cur c{blob, len};
  Gguf g;
  if (memcmp(c.take(4), "GGUF", 4) != 0)
    throw GgufError{VTQ_ERR_MALFORMED, "gguf: bad magic (not 'GGUF')"};
  const uint32_t version = c.u32();
  if (version != 2 && version != 3)
    throw GgufError{VTQ_ERR_MALFORMED, "gguf: unsupported version (only v2/v3 supported)"};
  const uint64_t nt = c.u64(), nm = c.u64();
  for (uint64_t i = 0; i < nm; i++) {
    std::string key = c.str();
    g.meta[key] = read_value(c, (int)c.u32());
  }
  struct Info { std::string name; std::vector<uint64_t> shape; int dtype; uint64_t off; };
  std::vector<Info> infos;
  for (uint64_t i = 0; i < nt; i++) {
    Info in;
    in.name = c.str();
    const uint32_t nd = c.u32();
    if (nd > 8) throw GgufError{VTQ_ERR_MALFORMED, "gguf: tensor rank > 8 (sanity bound)"};
    for (uint32_t d = 0; d < nd; d++) in.shape.push_back(c.u64());
    in.dtype = (int)c.u32();
    in.off = c.u64();
    infos.push_back(in);
  }
  uint64_t align = 32;
  auto it = g.meta.find("general.alignment");
  if (it != g.meta.end() && it->second.type == 4) align = it->second.u;
  if (align == 0) throw GgufError{VTQ_ERR_MALFORMED, "gguf: general.alignment is zero"};
  const uint64_t base = (c.pos + align - 1) / align * align;
  for (auto& in : infos) {
    unsigned __int128 numel = 1;
    for (uint64_t d : in.shape) {
      numel *= d;
      if (numel >> 64) throw GgufError{VTQ_ERR_MALFORMED, "gguf: shape product overflows u64"};
    }
    int64_t per, nb;
    switch (in.dtype) {
      case T_F32: per = 1; nb = 4; break;
      case T_F16: per = 1; nb = 2; break;
      case T_Q4_0: per = 32; nb = 18; break;
      case T_Q5_0: per = 32; nb = 22; break;
      case T_Q8_0: per = 32; nb = 34; break;
      case T_Q4_K: per = 256; nb = 144; break;
      case T_Q6_K: per = 256; nb = 210; break;
      default:
        throw GgufError{VTQ_ERR_MALFORMED, "gguf: byte size unknown for unsupported ggml_type"};
    }
    if ((uint64_t)numel % per)
      throw GgufError{VTQ_ERR_MALFORMED, "gguf: tensor numel not a multiple of the block size"};
    const unsigned __int128 bytes = (unsigned __int128)((uint64_t)numel / per) * nb;
    const unsigned __int128 end = (unsigned __int128)base + in.off + bytes;
    if (end > len) throw GgufError{VTQ_ERR_TRUNCATED, "gguf: tensor extends past end of file"};
    g.tensors[in.name] = GTensor{in.shape, in.dtype, blob + base + in.off, (size_t)bytes};
  }
  return g;
}

// ------------------------------------------------------------- kernels ----



// embedding_row (forward_quantized.rs:818-919): dequantise one row of the
// table into x. Device layouts as uploaded (Q6_K regrouped, see repack.cu).
__global__ void embed_kernel(const uint8_t* table, int dtype, int64_t pitch, int dim,
                             const StepState* st, float* x) {
  const uint32_t row = st->cur;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < dim; e += gridDim.x * blockDim.x)
    x[e] = embed_value(table, dtype, pitch, dim, row, e);
}

// x = x + delta (if delta), then xb = rms_norm(x) * w (rms_norm.rs:94-108):
// sumsq is the left-to-right fp32 sum (exact_serial_sum computes it with the CTA).
__global__ void __launch_bounds__(256) rmsnorm_kernel(float* x, const float* delta, const float* w, float eps, int n,
                               float* out) {
  extern __shared__ float sq[];
  __shared__ float s_scale;
  __shared__ xsum::Scratch scr;
  pdl_wait();
  pdl_release();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = x[i];
    if (delta) {
      v = __fadd_rn(v, delta[i]);
      x[i] = v;
    }
    sq[i] = __fmul_rn(v, v);
  }
  __syncthreads();
  const float s = xsum::exact_serial_sum<16>(sq, n, &scr, threadIdx.x, blockDim.x,
                                         [] { __syncthreads(); });  // rms_norm.rs:97-100
  if (threadIdx.x == 0) {
    const float mean = __fdiv_rn(s, (float)n);
    s_scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  }
  __syncthreads();
  const float scale = s_scale;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float v = x[i];
    out[i] = __fmul_rn(__fmul_rn(v, scale), w[i]);
  }
}

// RMSNorm with the residual add written to a separate buffer:
// v = x (+ delta) -> res; out = (v * scale) * w (rms_norm.rs:94-108).
// Row blockIdx.x of [rows][n] buffers (one row in the decode step).
__global__ void __launch_bounds__(256) rmsnorm_res_kernel(const float* x, const float* delta,
                                                          const float* w, float eps, int n,
                                                          float* out, float* res) {
  extern __shared__ float sq[];
  __shared__ float s_scale;
  __shared__ xsum::Scratch scr;
  pdl_wait();
  pdl_release();
  const size_t row = (size_t)blockIdx.x * n;
  x += row;
  if (delta) delta += row;
  out += row;
  res += row;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    float v = x[i];
    if (delta) v = __fadd_rn(v, delta[i]);
    res[i] = v;
    sq[i] = __fmul_rn(v, v);
  }
  __syncthreads();
  const float s = xsum::exact_serial_sum<16>(sq, n, &scr, threadIdx.x, blockDim.x,
                                         [] { __syncthreads(); });  // rms_norm.rs:97-100
  if (threadIdx.x == 0) {
    const float mean = __fdiv_rn(s, (float)n);
    s_scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
  }
  __syncthreads();
  const float scale = s_scale;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    out[i] = __fmul_rn(__fmul_rn(res[i], scale), w[i]);
}

// ---- batched prompt (positions 0 .. P-1 of the prompt at once) ----

// Embedding rows of the prompt tokens: row blockIdx.y.
__global__ void embed_rows_kernel(const uint8_t* table, int dtype, int64_t pitch, int dim,
                                  const uint32_t* tokens, float* x) {
  const uint32_t row = tokens[blockIdx.y];
  float* xr = x + (size_t)blockIdx.y * dim;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < dim; e += gridDim.x * blockDim.x)
    xr[e] = embed_value(table, dtype, pitch, dim, row, e);
}

// k (+ bias) rotated and v (+ bias) into the caches at position blockIdx.x, with
// the arithmetic of attention_head (decode_ops.cuh), for every kv head.
__global__ void cache_kv_rows_kernel(const float* k, int64_t ldk, const float* v, int64_t ldv,
                                     AttnExtras ex, float* kc, float* vc, int layer,
                                     int seq_len, int kv_dim, int hs, const float* rcos,
                                     const float* rsin) {
  const int pos = blockIdx.x, half = hs / 2;
  const float* kr = k + (size_t)pos * ldk;
  const float* vr = v + (size_t)pos * ldv;
  const size_t off = ((size_t)layer * seq_len + pos) * kv_dim;
  for (int idx = threadIdx.x; idx < kv_dim / 2; idx += blockDim.x) {
    const int g = idx / half, p = idx - g * half;
    const int e0 = ex.neox ? p : 2 * p, e1 = ex.neox ? p + half : 2 * p + 1;
    const float fcr = rcos[(size_t)pos * half + p], fci = rsin[(size_t)pos * half + p];
    float k0 = kr[g * hs + e0], k1 = kr[g * hs + e1];
    float v0 = vr[g * hs + e0], v1 = vr[g * hs + e1];
    if (ex.bk) {
      k0 = __fadd_rn(k0, ex.bk[g * hs + e0]);
      k1 = __fadd_rn(k1, ex.bk[g * hs + e1]);
    }
    if (ex.bv) {
      v0 = __fadd_rn(v0, ex.bv[g * hs + e0]);
      v1 = __fadd_rn(v1, ex.bv[g * hs + e1]);
    }
    kc[off + g * hs + e0] = __fsub_rn(__fmul_rn(k0, fcr), __fmul_rn(k1, fci));
    kc[off + g * hs + e1] = __fadd_rn(__fmul_rn(k0, fci), __fmul_rn(k1, fcr));
    vc[off + g * hs + e0] = v0;
    vc[off + g * hs + e1] = v1;
  }
}

// Attention of head blockIdx.x for prompt position blockIdx.y over the cache
// (every prompt position's k / v is cached before this launch).
__global__ void attention_rows_kernel(const float* q, int64_t ldq, const float* k, const float* v,
                                      int64_t ldv, float* kc, float* vc, int layer, int seq_len,
                                      int kv_dim, int hs, int kv_mul, const float* rcos,
                                      const float* rsin, float* out, int dim, AttnExtras ex) {
  extern __shared__ float sm[];
  __shared__ float red[2];
  const int t = blockIdx.y;
  ex.no_cache_write = 1;
  attention_head(blockIdx.x, q + (size_t)t * ldq, k + (size_t)t * ldq, v + (size_t)t * ldv, kc,
                 vc, layer, seq_len, kv_dim, hs, kv_mul, rcos, rsin, t, out + (size_t)t * dim, sm,
                 red, threadIdx.x, blockDim.x, [] { __syncthreads(); }, ex);
}

// SwiGLU of prompt row blockIdx.y: g / u read with stride st from rows of ld.
__global__ void swiglu_rows_kernel(const float* g, const float* u, int st, int64_t ld,
                                   float* out, int n) {
  const size_t r = blockIdx.y;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float gi = g[r * ld + (int64_t)i * st];
    const float silu = __fdiv_rn(gi, __fadd_rn(1.0f, libm::expf(-gi)));
    out[r * n + i] = __fmul_rn(silu, u[r * ld + (int64_t)i * st]);
  }
}

// One query head per CTA (attention_head, decode_ops.cuh).
__global__ void attention_rope_kernel(const float* q, const float* k, const float* v, float* kc,
                                      float* vc, int layer, int seq_len, int kv_dim, int hs,
                                      int kv_mul, const float* rcos, const float* rsin,
                                      const StepState* st, float* out, AttnExtras ex) {
  extern __shared__ float sm[];
  __shared__ float red[2];
  pdl_wait();
  pdl_release();
  attention_head(blockIdx.x, q, k, v, kc, vc, layer, seq_len, kv_dim, hs, kv_mul, rcos, rsin,
                 st->pos, out, sm, red, threadIdx.x, blockDim.x, [] { __syncthreads(); }, ex);
}

// SwiGLU: silu(g) * up with silu = g / (1 + expf(-g)) (forward_quantized.rs:556-561).
// g and u are read with stride `st` (2 for the interleaved gate|up output).
__global__ void swiglu_kernel(const float* g, const float* u, int st, float* out, int n) {
  pdl_wait();
  pdl_release();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float gi = g[(int64_t)i * st];
    const float silu = __fdiv_rn(gi, __fadd_rn(1.0f, libm::expf(-gi)));
    out[i] = __fmul_rn(silu, u[(int64_t)i * st]);
  }
}

// Next-token choice (argmax_next, decode_ops.cuh) in one CTA.
__global__ void argmax_next_kernel(const float* logits, int n, StepState* st,
                                   const uint32_t* prompt, uint32_t* out_tokens) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  pdl_wait();
  pdl_release();
  argmax_next(logits, n, st, prompt, out_tokens, bv, bi, threadIdx.x, blockDim.x,
              [] { __syncthreads(); });
}

// Copy the step's logits into the per-position log (optional output).
__global__ void log_logits_kernel(const float* logits, int vocab, const StepState* st,
                                  float* log) {
  pdl_wait();
  pdl_release();
  const int pos = st->pos;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < vocab; i += gridDim.x * blockDim.x)
    log[(size_t)pos * vocab + i] = logits[i];
}

}  // namespace
}  // namespace vtq

using namespace vtq;

struct vtq_decode {
  int device = 0;
  cudaStream_t stream = nullptr;
  int dim = 0, hidden = 0, n_layers = 0, n_heads = 0, n_kv_heads = 0, vocab = 0, seq_len = 0;
  bool shared = false;
  float rope_theta = 10000.0f, rms_eps = 1e-5f;
  bool neox = false;  // NeoX split-half RoPE (architecture "qwen2", quant_weights.rs:151)
  std::vector<void*> allocs;
  DevMatrix embd{}, head{};
  struct Layer {
    float *rms_att, *rms_ffn;
    float *bq = nullptr, *bk = nullptr, *bv = nullptr;  // Qwen2 QKV biases (-0.0 padded)
    DevMatrix wq, wk, wv, wo, w1, w2, w3;
    // q|k and gate|up share their input: when each pair has one dtype, the two
    // matrices sit back to back in HBM and run as one launch (wqk, w13).
    bool fused_qk = false, fused_13 = false;
    DevMatrix wqk{}, w13{};
  };
  std::vector<Layer> layers;
  float* rms_final = nullptr;
  float *rcos = nullptr, *rsin = nullptr, *kc = nullptr, *vc = nullptr;
  float *x, *xb, *q, *k, *v, *xo, *xb2, *g, *u, *inner, *logits;
  float* xr = nullptr;  // second residual buffer (fused path: the norms alternate x <-> xr)
  bool fused = false;   // every linear integer k-quant: norms/SwiGLU fused into the matvecs
  int fuse_mask = 2;    // RMSNorm into the consuming matvec: 1 attention, 2 FFN (2 measured fastest)
  MkPlan* mk = nullptr;  // persistent one-kernel step (decode_mk.cu), when the model fits
  float* logit_log = nullptr;
  size_t logit_log_cap = 0;
  StepState* st = nullptr;
  uint32_t* prompt = nullptr;
  uint32_t* out_tokens = nullptr;
  unsigned* status = nullptr;
  cudaGraphExec_t graph = nullptr;
  bool graph_logs = false;
  cudaEvent_t ev[4] = {};  // call start, first step, after last step, call end
  // v runs on a second stream, concurrently with q|k (captured as a graph branch).
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
  float ms_steps = 0.0f, ms_call = 0.0f;
  // Batched prompt: positions 0 .. n_prompt-2 run as batched linears before the
  // per-token loop (their next token is the prompt's, so only the KV cache and
  // the logged logits carry over). Row buffers for up to pf_cap positions.
  bool prefill = true;
  int pf_cap = 0;
  unsigned long long launches = 0;  // kernels of the last vtq_decode_run's decode work
  unsigned long long graph_kernels = 0;  // kernel nodes of the step graph
  float *pf_x = nullptr, *pf_xr = nullptr, *pf_xb = nullptr, *pf_q = nullptr, *pf_v = nullptr,
        *pf_xo = nullptr, *pf_xb2 = nullptr, *pf_g = nullptr, *pf_inner = nullptr;
  std::string err;
};

namespace {

vtq_status dfail(vtq_decode* d, vtq_status s, const std::string& m) {
  if (d) d->err = m;
  return s;
}

#define DCUDA(d, call)                                                                   \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess)                                                               \
      return dfail((d), e_ == cudaErrorMemoryAllocation ? VTQ_ERR_OOM : VTQ_ERR_GPU,     \
                   std::string("gpu error: ") + #call + ": " + cudaGetErrorString(e_)); \
  } while (0)

template <typename T>
vtq_status dalloc(vtq_decode* d, T** p, size_t bytes) {
  void* q = nullptr;
  DCUDA(d, cudaMalloc(&q, bytes ? bytes : 16));
  d->allocs.push_back(q);
  *p = static_cast<T*>(q);
  return VTQ_OK;
}

vtq_status upload_matrix(vtq_decode* d, const GTensor& t, int64_t in, int64_t out, DevMatrix* m,
                         uint8_t* into = nullptr) {
  if (t.shape.size() != 2 || (int64_t)t.shape[0] != in || (int64_t)t.shape[1] != out)
    return dfail(d, VTQ_ERR_INTERNAL, "gguf: weight shape mismatch");
  const int64_t rb = packed_row_bytes(t.dtype, in);
  if (rb < 0) return dfail(d, VTQ_ERR_NOT_IMPLEMENTED, "weight dtype not supported by the kernels");
  m->dtype = t.dtype;
  m->in_feat = in;
  m->out_feat = out;
  m->row_bytes = rb;
  m->pitch = device_pitch(t.dtype, in);
  uint8_t *dst = into, *stage;
  if (!dst)
    if (vtq_status s = dalloc(d, &dst, (size_t)(out * m->pitch + 16))) return s;
  DCUDA(d, cudaMalloc(&stage, t.len));
  DCUDA(d, cudaMemcpyAsync(stage, t.bytes, t.len, cudaMemcpyHostToDevice, d->stream));
  DCUDA(d, launch_repack(stage, *m, dst, d->stream));
  DCUDA(d, cudaMemsetAsync(dst + out * m->pitch, 0, 16, d->stream));
  DCUDA(d, cudaStreamSynchronize(d->stream));
  cudaFree(stage);
  m->data = dst;
  return VTQ_OK;
}

vtq_status upload_f32(vtq_decode* d, const Gguf& g, const std::string& name, int n, float** out) {
  auto it = g.tensors.find(name);
  if (it == g.tensors.end())
    return dfail(d, VTQ_ERR_INTERNAL, "gguf: required Llama tensor not found: " + name);
  if (it->second.dtype != T_F32)
    return dfail(d, VTQ_ERR_INTERNAL, "gguf: expected F32 norm-weight tensor, got something else");
  if ((int64_t)it->second.len != (int64_t)n * 4)
    return dfail(d, VTQ_ERR_INTERNAL, "gguf: norm length mismatch");
  if (vtq_status s = dalloc(d, out, (size_t)n * 4)) return s;
  DCUDA(d, cudaMemcpyAsync(*out, it->second.bytes, (size_t)n * 4, cudaMemcpyHostToDevice,
                           d->stream));
  DCUDA(d, cudaStreamSynchronize(d->stream));
  return VTQ_OK;
}

const GTensor* need(vtq_decode* d, const Gguf& g, const std::string& name) {
  auto it = g.tensors.find(name);
  if (it == g.tensors.end()) {
    d->err = "gguf: required Llama tensor not found: " + name;
    return nullptr;
  }
  return &it->second;
}

int64_t meta_uint(const Gguf& g, const std::string& key, bool* ok) {
  auto it = g.meta.find(key);
  if (it == g.meta.end()) {
    *ok = false;
    return 0;
  }
  const GMeta& m = it->second;
  switch (m.type) {
    case 4: case 10: return (int64_t)m.u;
    case 5: case 11: if ((int64_t)m.u >= 0) return (int64_t)m.u; break;
    default: break;
  }
  *ok = false;
  return 0;
}

// One decode step: every launch on d->stream; captured into the graph.
vtq_status enqueue_step(vtq_decode* d, bool log_logits) {
  cudaStream_t s = d->stream;
  const int dim = d->dim, hs = dim / d->n_heads, kv_dim = d->n_kv_heads * hs;
  const int kv_mul = d->n_heads / d->n_kv_heads;
  embed_kernel<<<(dim + 255) / 256, 256, 0, s>>>(d->embd.data, d->embd.dtype, d->embd.pitch, dim,
                                                  d->st, d->x);
  const size_t rms_smem = ((size_t)dim + 4) * 4;
  const size_t att_smem = ((size_t)3 * hs + d->seq_len) * 4;
  const float* delta = nullptr;
  if (d->fused) {
    // RMSNorm runs inside the matvecs that consume it (every CTA computes the
    // serial sum while its weights stream in; CTA 0 of one launch stores the
    // residual into the other buffer) and SwiGLU in the gate|up epilogue.
    auto mv = [&](const DevMatrix& m, const float* x, float* y, cudaStream_t st,
                  const KqXform* xf) {
      return launch_kq_matvec(m, x, m.in_feat, 1, y, m.out_feat, d->status, st, nullptr, xf);
    };
    const int fz = d->fuse_mask;
    for (int l = 0; l < d->n_layers; l++) {
      auto& L = d->layers[l];
      if (fz & 1) {
        KqXform att;
        att.kind = 2;
        att.delta = delta;
        att.nw = L.rms_att;
        att.eps = d->rms_eps;
        DCUDA(d, cudaEventRecord(d->fork, s));
        DCUDA(d, cudaStreamWaitEvent(d->side, d->fork, 0));
        DCUDA(d, mv(L.wv, d->x, d->v, d->side, &att));
        DCUDA(d, cudaEventRecord(d->join, d->side));
        att.res_out = d->xr;
        DCUDA(d, mv(L.wqk, d->x, d->q, s, &att));
        DCUDA(d, cudaStreamWaitEvent(s, d->join, 0));
      } else {
        // Norm kernel (residual x -> xr), then q|k and v side by side.
        DCUDA(d, launch_pdl(rmsnorm_res_kernel, 1, 256, rms_smem, s, d->x, delta, L.rms_att,
                            d->rms_eps, dim, d->xb, d->xr));
        DCUDA(d, cudaEventRecord(d->fork, s));
        DCUDA(d, cudaStreamWaitEvent(d->side, d->fork, 0));
        DCUDA(d, mv(L.wv, d->xb, d->v, d->side, nullptr));
        DCUDA(d, cudaEventRecord(d->join, d->side));
        DCUDA(d, mv(L.wqk, d->xb, d->q, s, nullptr));
        DCUDA(d, cudaStreamWaitEvent(s, d->join, 0));
      }
      DCUDA(d, launch_pdl(attention_rope_kernel, d->n_heads, 128, att_smem, s, d->q, d->k, d->v,
                          d->kc, d->vc, l, d->seq_len, kv_dim, hs, kv_mul, d->rcos, d->rsin,
                          d->st, d->xo, AttnExtras{d->neox ? 1 : 0, L.bq, L.bk, L.bv}));
      DCUDA(d, mv(L.wo, d->xo, d->xb2, s, nullptr));
      if (fz & 2) {
        KqXform ffn;
        ffn.kind = 2;
        ffn.delta = d->xb2;
        ffn.nw = L.rms_ffn;
        ffn.eps = d->rms_eps;
        ffn.res_out = d->x;
        ffn.swiglu_pairs = 1;
        DCUDA(d, mv(L.w13, d->xr, d->inner, s, &ffn));
      } else {
        DCUDA(d, launch_pdl(rmsnorm_res_kernel, 1, 256, rms_smem, s, d->xr, d->xb2, L.rms_ffn,
                            d->rms_eps, dim, d->xb, d->x));
        KqXform sw;
        sw.swiglu_pairs = 1;
        DCUDA(d, mv(L.w13, d->xb, d->inner, s, &sw));
      }
      DCUDA(d, mv(L.w2, d->inner, d->xb2, s, nullptr));
      delta = d->xb2;
    }
    KqXform fin;
    fin.kind = 2;
    fin.delta = delta;
    fin.nw = d->rms_final;
    fin.eps = d->rms_eps;
    DCUDA(d, mv(d->head, d->x, d->logits, s, &fin));
    if (log_logits)
      DCUDA(d, launch_pdl(log_logits_kernel, (d->vocab + 255) / 256, 256, 0, s, d->logits,
                          d->vocab, d->st, d->logit_log));
    DCUDA(d, launch_pdl(argmax_next_kernel, 1, 1024, 0, s, d->logits, d->vocab, d->st,
                        d->prompt, d->out_tokens));
    DCUDA(d, cudaGetLastError());
    return VTQ_OK;
  }
  for (int l = 0; l < d->n_layers; l++) {
    auto& L = d->layers[l];
    DCUDA(d, launch_pdl(rmsnorm_kernel, 1, 256, rms_smem, s, d->x, delta, L.rms_att,
                        d->rms_eps, dim, d->xb));
    // v depends only on the normed x: fork it onto the side stream so that it
    // runs next to q|k, and join before attention.
    DCUDA(d, cudaEventRecord(d->fork, s));
    DCUDA(d, cudaStreamWaitEvent(d->side, d->fork, 0));
    DCUDA(d, launch_kq_or_canon(L.wv, d->xb, d->v, d->status, d->side));
    DCUDA(d, cudaEventRecord(d->join, d->side));
    if (L.fused_qk) {
      DCUDA(d, launch_kq_or_canon(L.wqk, d->xb, d->q, d->status, s));
    } else {
      DCUDA(d, launch_kq_or_canon(L.wq, d->xb, d->q, d->status, s));
      DCUDA(d, launch_kq_or_canon(L.wk, d->xb, d->k, d->status, s));
    }
    DCUDA(d, cudaStreamWaitEvent(s, d->join, 0));
    DCUDA(d, launch_pdl(attention_rope_kernel, d->n_heads, 128, att_smem, s, d->q, d->k, d->v,
                        d->kc, d->vc, l, d->seq_len, kv_dim, hs, kv_mul, d->rcos, d->rsin, d->st,
                        d->xo, AttnExtras{d->neox ? 1 : 0, L.bq, L.bk, L.bv}));
    DCUDA(d, launch_kq_or_canon(L.wo, d->xo, d->xb2, d->status, s));
    DCUDA(d, launch_pdl(rmsnorm_kernel, 1, 256, rms_smem, s, d->x, d->xb2, L.rms_ffn,
                        d->rms_eps, dim, d->xb));
    if (L.fused_13) {
      DCUDA(d, launch_kq_or_canon(L.w13, d->xb, d->g, d->status, s));
    } else {
      DCUDA(d, launch_kq_or_canon(L.w1, d->xb, d->g, d->status, s));
      DCUDA(d, launch_kq_or_canon(L.w3, d->xb, d->u, d->status, s));
    }
    // The fused gate|up output is interleaved (gate_i, up_i).
    DCUDA(d, launch_pdl(swiglu_kernel, (d->hidden + 255) / 256, 256, 0, s, d->g,
                        L.fused_13 ? d->g + 1 : d->u, L.fused_13 ? 2 : 1, d->inner, d->hidden));
    DCUDA(d, launch_kq_or_canon(L.w2, d->inner, d->xb2, d->status, s));
    delta = d->xb2;
  }
  DCUDA(d, launch_pdl(rmsnorm_kernel, 1, 256, rms_smem, s, d->x, delta, d->rms_final,
                      d->rms_eps, dim, d->xb));
  DCUDA(d, launch_kq_or_canon(d->head, d->xb, d->logits, d->status, s));
  if (log_logits)
    DCUDA(d, launch_pdl(log_logits_kernel, (d->vocab + 255) / 256, 256, 0, s, d->logits,
                        d->vocab, d->st, d->logit_log));
  DCUDA(d, launch_pdl(argmax_next_kernel, 1, 1024, 0, s, d->logits, d->vocab, d->st, d->prompt,
                      d->out_tokens));
  DCUDA(d, cudaGetLastError());
  return VTQ_OK;
}

}  // namespace

extern "C" {

vtq_status vtq_decode_open(vtq_ctx* ctx, int device, const uint8_t* gguf, size_t len,
                           vtq_decode** out) {
  if (!out || !gguf) return VTQ_ERR_INVALID_ARG;
  *out = nullptr;
  (void)ctx;
  auto* d = new vtq_decode();
  d->device = device;
  vtq_status s = VTQ_OK;
  cudaError_t ce = cudaSetDevice(device);
  if (ce == cudaSuccess) ce = cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking);
  if (ce == cudaSuccess) ce = cudaStreamCreateWithFlags(&d->side, cudaStreamNonBlocking);
  if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&d->fork, cudaEventDisableTiming);
  if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&d->join, cudaEventDisableTiming);
  if (ce != cudaSuccess) {
    delete d;
    return VTQ_ERR_GPU;
  }
  *out = d;
  Gguf g;
  try {
    g = parse_gguf(gguf, len);
  } catch (const GgufError& e) {
    d->err = e.msg;
    return e.status;
  }
  // Config (src/model/config.rs:156-212) and Llama hyperparameters (quant_weights.rs:137-151).
  auto arch_it = g.meta.find("general.architecture");
  if (arch_it == g.meta.end() || arch_it->second.type != 8)
    return dfail(d, VTQ_ERR_INTERNAL, "gguf: missing 'general.architecture' metadata");
  const std::string arch = arch_it->second.s;
  // Any architecture string keys the metadata (config.rs:141-165); "qwen2"
  // selects NeoX RoPE below, every other one the Llama layout.
  bool ok = true;
  d->dim = (int)meta_uint(g, arch + ".embedding_length", &ok);
  d->hidden = (int)meta_uint(g, arch + ".feed_forward_length", &ok);
  d->n_layers = (int)meta_uint(g, arch + ".block_count", &ok);
  d->n_heads = (int)meta_uint(g, arch + ".attention.head_count", &ok);
  d->seq_len = (int)meta_uint(g, arch + ".context_length", &ok);
  bool ok_kv = true;
  d->n_kv_heads = (int)meta_uint(g, arch + ".attention.head_count_kv", &ok_kv);
  if (!ok_kv) d->n_kv_heads = d->n_heads;
  auto tok = g.meta.find("tokenizer.ggml.tokens");
  if (tok != g.meta.end() && tok->second.type == 9)
    d->vocab = (int)tok->second.arr_len;
  else
    d->vocab = (int)meta_uint(g, arch + ".vocab_size", &ok);
  if (!ok) return dfail(d, VTQ_ERR_INTERNAL, "gguf: numeric metadata missing or wrong type");
  auto f32meta = [&](const std::string& key, float def) {
    auto it = g.meta.find(key);
    return (it != g.meta.end() && it->second.type == 6) ? (float)it->second.f : def;
  };
  d->rope_theta = f32meta(arch + ".rope.freq_base", 10000.0f);
  d->rms_eps = f32meta(arch + ".attention.layer_norm_rms_epsilon", 1e-5f);
  d->neox = arch == "qwen2";
  if (d->dim <= 0 || d->n_heads <= 0 || d->dim % d->n_heads || d->n_kv_heads <= 0 ||
      d->n_heads % d->n_kv_heads || (d->dim / d->n_heads) % 2 || d->dim > 8192 ||
      d->seq_len <= 0 || d->vocab <= 0)
    return dfail(d, VTQ_ERR_INTERNAL, "decode session: unsupported model shape");
  const int dim = d->dim, hs = dim / d->n_heads, kv_dim = d->n_kv_heads * hs;
  const GTensor* te = need(d, g, "token_embd.weight");
  if (!te) return VTQ_ERR_INTERNAL;
  if ((s = upload_matrix(d, *te, dim, d->vocab, &d->embd))) return s;
  auto wcls = g.tensors.find("output.weight");
  d->shared = wcls == g.tensors.end();
  if (d->shared)
    d->head = d->embd;
  else if ((s = upload_matrix(d, wcls->second, dim, d->vocab, &d->head)))
    return s;
  if ((s = upload_f32(d, g, "output_norm.weight", dim, &d->rms_final))) return s;
  d->layers.resize(d->n_layers);
  for (int l = 0; l < d->n_layers; l++) {
    auto& L = d->layers[l];
    const std::string p = "blk." + std::to_string(l) + ".";
    if ((s = upload_f32(d, g, p + "attn_norm.weight", dim, &L.rms_att))) return s;
    if ((s = upload_f32(d, g, p + "ffn_norm.weight", dim, &L.rms_ffn))) return s;
    // Optional QKV biases (quant_weights.rs:172-174, F32). add_bias zips with the
    // shorter length (forward_quantized.rs:807-813): entries past the tensor are
    // padded with -0.0, which adds nothing to any value.
    struct {
      const char* name;
      int n;
      float** dst;
    } biases[] = {{"attn_q.bias", dim, &L.bq}, {"attn_k.bias", kv_dim, &L.bk},
                  {"attn_v.bias", kv_dim, &L.bv}};
    for (auto& b : biases) {
      auto it = g.tensors.find(p + b.name);
      if (it == g.tensors.end()) continue;
      if (it->second.dtype != T_F32)
        return dfail(d, VTQ_ERR_INTERNAL, "gguf: expected F32 bias tensor");
      if (it->second.len % 4)
        return dfail(d, VTQ_ERR_INTERNAL, "gguf: F32 bias byte length not a multiple of 4");
      std::vector<float> h(b.n, -0.0f);
      memcpy(h.data(), it->second.bytes, std::min<size_t>(it->second.len, (size_t)b.n * 4));
      if (vtq_status e = dalloc(d, b.dst, (size_t)b.n * 4)) return e;
      DCUDA(d, cudaMemcpy(*b.dst, h.data(), (size_t)b.n * 4, cudaMemcpyHostToDevice));
    }
    struct {
      const char* name;
      int64_t in, out;
      DevMatrix* m;
    } mats[] = {{"attn_q.weight", dim, dim, &L.wq},         {"attn_k.weight", dim, kv_dim, &L.wk},
                {"attn_v.weight", dim, kv_dim, &L.wv},      {"attn_output.weight", dim, dim, &L.wo},
                {"ffn_gate.weight", dim, d->hidden, &L.w1}, {"ffn_down.weight", d->hidden, dim, &L.w2},
                {"ffn_up.weight", dim, d->hidden, &L.w3}};
    const GTensor* tq = need(d, g, p + "attn_q.weight");
    const GTensor* tk = need(d, g, p + "attn_k.weight");
    const GTensor* t1 = need(d, g, p + "ffn_gate.weight");
    const GTensor* t3 = need(d, g, p + "ffn_up.weight");
    if (!tq || !tk || !t1 || !t3) return VTQ_ERR_INTERNAL;
    // interleave: rows (a_0, b_0, a_1, b_1, ...) for the gate|up pair epilogue
    // (ma / mb then do not describe separate matrices and stay unused).
    auto fuse = [&](const GTensor* ta, const GTensor* tb, int64_t in, int64_t ra, int64_t rb,
                    DevMatrix* ma, DevMatrix* mb, DevMatrix* both, bool* fused,
                    bool interleave) -> vtq_status {
      if (ta->dtype != tb->dtype || (ta->dtype != T_Q4_K && ta->dtype != T_Q6_K)) return VTQ_OK;
      const int64_t pitch = device_pitch(ta->dtype, in);
      if (pitch <= 0 || (interleave && ra != rb)) return VTQ_OK;
      uint8_t* buf;
      if (vtq_status e = dalloc(d, &buf, (size_t)((ra + rb) * pitch + 16))) return e;
      uint8_t* tmp = buf;
      if (interleave) DCUDA(d, cudaMalloc(&tmp, (size_t)((ra + rb) * pitch + 16)));
      vtq_status e = upload_matrix(d, *ta, in, ra, ma, tmp);
      if (!e) e = upload_matrix(d, *tb, in, rb, mb, tmp + ra * pitch);
      if (!e && interleave) {
        for (int h = 0; h < 2 && !e; h++)
          if (cudaMemcpy2D(buf + h * pitch, 2 * pitch, tmp + h * ra * pitch, pitch, pitch, ra,
                           cudaMemcpyDeviceToDevice) != cudaSuccess)
            e = dfail(d, VTQ_ERR_GPU, "decode session: interleaving gate|up failed");
        if (!e && cudaMemset(buf + (ra + rb) * pitch, 0, 16) != cudaSuccess)
          e = dfail(d, VTQ_ERR_GPU, "decode session: interleaving gate|up failed");
      }
      if (interleave) cudaFree(tmp);
      if (e) return e;
      *both = *ma;
      both->data = buf;
      both->out_feat = ra + rb;
      *fused = true;
      return VTQ_OK;
    };
    if ((s = fuse(tq, tk, dim, dim, kv_dim, &L.wq, &L.wk, &L.wqk, &L.fused_qk, false))) return s;
    if ((s = fuse(t1, t3, dim, d->hidden, d->hidden, &L.w1, &L.w3, &L.w13, &L.fused_13, true)))
      return s;
    for (auto& mm : mats) {
      if ((L.fused_qk && (mm.m == &L.wq || mm.m == &L.wk)) ||
          (L.fused_13 && (mm.m == &L.w1 || mm.m == &L.w3)))
        continue;
      const GTensor* t = need(d, g, p + mm.name);
      if (!t) return VTQ_ERR_INTERNAL;
      if ((s = upload_matrix(d, *t, mm.in, mm.out, mm.m))) return s;
    }
  }
  // RoPE tables from the restated libm (forward_quantized.rs:449-458).
  std::vector<float> hc((size_t)d->seq_len * (hs / 2)), hsn((size_t)d->seq_len * (hs / 2));
  for (int pos = 0; pos < d->seq_len; pos++)
    for (int j = 0; j < hs / 2; j++) {
      const int idx = 2 * j;
      const float freq = 1.0f / libm::powf(d->rope_theta, (float)idx / (float)hs);
      const float val = (float)pos * freq;
      hc[(size_t)pos * (hs / 2) + j] = libm::cosf(val);
      hsn[(size_t)pos * (hs / 2) + j] = libm::sinf(val);
    }
  if ((s = dalloc(d, &d->rcos, hc.size() * 4)) || (s = dalloc(d, &d->rsin, hsn.size() * 4)))
    return s;
  DCUDA(d, cudaMemcpyAsync(d->rcos, hc.data(), hc.size() * 4, cudaMemcpyHostToDevice, d->stream));
  DCUDA(d, cudaMemcpyAsync(d->rsin, hsn.data(), hsn.size() * 4, cudaMemcpyHostToDevice,
                           d->stream));
  DCUDA(d, cudaStreamSynchronize(d->stream));
  const size_t kvb = (size_t)d->n_layers * d->seq_len * kv_dim * 4;
  if ((s = dalloc(d, &d->kc, kvb)) || (s = dalloc(d, &d->vc, kvb))) return s;
  // All set-up work goes on the session stream: it is non-blocking, so work
  // on the legacy default stream (a plain cudaMemset) would not be ordered
  // before the first decode step.
  DCUDA(d, cudaMemsetAsync(d->kc, 0, kvb, d->stream));
  DCUDA(d, cudaMemsetAsync(d->vc, 0, kvb, d->stream));
  float** bufs[] = {&d->x, &d->xr, &d->xb, &d->xo, &d->xb2};
  for (float** b : bufs)
    if ((s = dalloc(d, b, (size_t)dim * 4))) return s;
  // q|k and gate|up are contiguous so that a fused launch writes both.
  if ((s = dalloc(d, &d->q, (size_t)(dim + kv_dim) * 4))) return s;
  d->k = d->q + dim;
  if ((s = dalloc(d, &d->g, (size_t)2 * d->hidden * 4))) return s;
  d->u = d->g + d->hidden;
  if ((s = dalloc(d, &d->v, (size_t)kv_dim * 4)) ||
      (s = dalloc(d, &d->inner, (size_t)d->hidden * 4)) ||
      (s = dalloc(d, &d->logits, (size_t)d->vocab * 4)) ||
      (s = dalloc(d, &d->st, sizeof(StepState))) ||
      (s = dalloc(d, &d->prompt, (size_t)d->seq_len * 4)) ||
      (s = dalloc(d, &d->out_tokens, (size_t)d->seq_len * 4)) || (s = dalloc(d, &d->status, 16)))
    return s;
  DCUDA(d, cudaMemsetAsync(d->status, 0, 16, d->stream));
  DCUDA(d, cudaStreamSynchronize(d->stream));
  // Fused step when every linear runs on the integer k-quant matvec and the
  // activation row fits the matvec's shared-memory staging.
  auto kq = [](const DevMatrix& m) { return m.dtype == T_Q4_K || m.dtype == T_Q6_K; };
  d->fused = kq(d->head) && dim % 256 == 0 && d->hidden % 256 == 0 && dim * 4 <= 65536 &&
             d->hidden * 4 <= 65536 && getenv("VTQ_DECODE_UNFUSED") == nullptr;
  if (const char* e = getenv("VTQ_DECODE_FUSE")) d->fuse_mask = atoi(e) & 3;
  d->prefill = getenv("VTQ_DECODE_NO_PREFILL") == nullptr;
  // Attention keeps 3 head vectors and one score per cached position in shared
  // memory: long contexts need the opt-in size.
  {
    const size_t att_smem = ((size_t)3 * hs + d->seq_len) * 4;
    int optin = 0;
    DCUDA(d, cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, d->device));
    if (att_smem > (size_t)optin)
      return dfail(d, VTQ_ERR_NOT_IMPLEMENTED,
                   "decode session: context_length too long for the attention kernel");
    if (att_smem > 48 * 1024)
      DCUDA(d, cudaFuncSetAttribute(attention_rope_kernel,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)att_smem));
  }
  for (auto& L : d->layers)
    d->fused = d->fused && L.fused_qk && L.fused_13 && kq(L.wqk) && kq(L.wv) && kq(L.wo) &&
               kq(L.w13) && kq(L.w2);
  if (d->fused) {
    MkModel mm;
    mm.dim = dim;
    mm.hidden = d->hidden;
    mm.n_layers = d->n_layers;
    mm.n_heads = d->n_heads;
    mm.n_kv_heads = d->n_kv_heads;
    mm.vocab = d->vocab;
    mm.seq_len = d->seq_len;
    mm.eps = d->rms_eps;
    mm.embd = d->embd;
    mm.head = d->head;
    mm.rms_final = d->rms_final;
    for (auto& L : d->layers)
      mm.layers.push_back({L.wqk, L.wv, L.wo, L.w13, L.w2, L.rms_att, L.rms_ffn, L.bq, L.bk, L.bv});
    mm.neox = d->neox;
    mm.x = d->x;
    mm.xr = d->xr;
    mm.q = d->q;
    mm.v = d->v;
    mm.xo = d->xo;
    mm.xb2 = d->xb2;
    mm.g = d->g;
    mm.logits = d->logits;
    mm.kc = d->kc;
    mm.vc = d->vc;
    mm.rcos = d->rcos;
    mm.rsin = d->rsin;
    mm.st = d->st;
    mm.prompt = d->prompt;
    mm.out_tokens = d->out_tokens;
    mm.status = d->status;
    if (mk_supported(mm) && mk_build(mm, &d->mk) != cudaSuccess) {
      d->mk = nullptr;
      cudaGetLastError();  // fall back to the per-op graph
    }
  }
  return VTQ_OK;
}

const char* vtq_decode_last_error(const vtq_decode* d) { return d ? d->err.c_str() : "null"; }

unsigned long long vtq_decode_launches(const vtq_decode* d) { return d ? d->launches : 0; }

int vtq_decode_step_kind(const vtq_decode* d) {
  if (!d) return -1;
  return d->mk ? 2 : d->fused ? 1 : 0;
}

vtq_status vtq_decode_config(const vtq_decode* d, int64_t* out8) {
  if (!d || !out8) return VTQ_ERR_INVALID_ARG;
  const int64_t v[8] = {d->dim,        d->hidden, d->n_layers, d->n_heads,
                        d->n_kv_heads, d->vocab,  d->seq_len,  d->shared ? 1 : 0};
  memcpy(out8, v, sizeof v);
  return VTQ_OK;
}

// Batched prompt positions 0 .. P-1 (forward_quantized.rs:329-649 per position,
// run as batched linears): every linear produces, row by row, the bits of the
// per-position call (the batch rows are independent: quant.rs:936-980), the
// norms and SwiGLU are per row, and each position's attention reads the cache
// exactly as the per-token step does once keys / values of positions <= it
// are cached. Fills the KV cache and, with want_logits, rows 0 .. P-1 of the
// logits log; the per-token loop then starts at position P.
vtq_status enqueue_prefill(vtq_decode* d, int P, bool want_logits) {
  cudaStream_t s = d->stream;
  const int dim = d->dim, hs = dim / d->n_heads, kv_dim = d->n_kv_heads * hs, H = d->hidden;
  const int kv_mul = d->n_heads / d->n_kv_heads;
  const int64_t ldqk = dim + kv_dim;
  if (P > d->pf_cap) {
    const int cap = std::min(d->seq_len, std::max(P, 2 * d->pf_cap));
    const size_t c = (size_t)cap;
    for (auto pr : {std::make_pair(&d->pf_x, c * dim), std::make_pair(&d->pf_xr, c * dim),
                    std::make_pair(&d->pf_xb, c * dim), std::make_pair(&d->pf_q, c * ldqk),
                    std::make_pair(&d->pf_v, c * kv_dim), std::make_pair(&d->pf_xo, c * dim),
                    std::make_pair(&d->pf_xb2, c * dim), std::make_pair(&d->pf_g, c * 2 * H),
                    std::make_pair(&d->pf_inner, c * H)})
      if (vtq_status e = dalloc(d, pr.first, pr.second * 4)) return e;
    d->pf_cap = cap;
  }
  const size_t rms_smem = ((size_t)dim + 4) * 4;
  const size_t att_smem = ((size_t)3 * hs + d->seq_len) * 4;
  if (att_smem > 48 * 1024)
    DCUDA(d, cudaFuncSetAttribute(attention_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)att_smem));
  auto lin = [&](const DevMatrix& m, const float* x, int64_t ldx, float* y, int64_t ldy) {
    return linear_any(m, x, ldx, y, ldy, P, d->status, s);
  };
  unsigned long long& count = kernel_launch_count();
  float *A = d->pf_x, *B = d->pf_xr;
  count++;
  embed_rows_kernel<<<dim3((dim + 255) / 256, P), 256, 0, s>>>(d->embd.data, d->embd.dtype,
                                                                d->embd.pitch, dim, d->prompt, A);
  const float* delta = nullptr;
  for (int l = 0; l < d->n_layers; l++) {
    auto& L = d->layers[l];
    count++;
    rmsnorm_res_kernel<<<P, 256, rms_smem, s>>>(A, delta, L.rms_att, d->rms_eps, dim, d->pf_xb, B);
    if (L.fused_qk) {
      DCUDA(d, lin(L.wqk, d->pf_xb, dim, d->pf_q, ldqk));
    } else {
      DCUDA(d, lin(L.wq, d->pf_xb, dim, d->pf_q, ldqk));
      DCUDA(d, lin(L.wk, d->pf_xb, dim, d->pf_q + dim, ldqk));
    }
    DCUDA(d, lin(L.wv, d->pf_xb, dim, d->pf_v, kv_dim));
    const AttnExtras ex{d->neox ? 1 : 0, L.bq, L.bk, L.bv};
    count++;
    cache_kv_rows_kernel<<<P, 128, 0, s>>>(d->pf_q + dim, ldqk, d->pf_v, kv_dim, ex, d->kc, d->vc,
                                           l, d->seq_len, kv_dim, hs, d->rcos, d->rsin);
    count++;
    attention_rows_kernel<<<dim3(d->n_heads, P), 128, att_smem, s>>>(
        d->pf_q, ldqk, d->pf_q + dim, d->pf_v, kv_dim, d->kc, d->vc, l, d->seq_len, kv_dim, hs,
        kv_mul, d->rcos, d->rsin, d->pf_xo, dim, ex);
    DCUDA(d, lin(L.wo, d->pf_xo, dim, d->pf_xb2, dim));
    count++;
    rmsnorm_res_kernel<<<P, 256, rms_smem, s>>>(B, d->pf_xb2, L.rms_ffn, d->rms_eps, dim,
                                                d->pf_xb, A);
    if (L.fused_13) {  // rows interleaved (gate_i, up_i)
      DCUDA(d, lin(L.w13, d->pf_xb, dim, d->pf_g, 2 * H));
      count++;
      swiglu_rows_kernel<<<dim3((H + 255) / 256, P), 256, 0, s>>>(d->pf_g, d->pf_g + 1, 2, 2 * H,
                                                                   d->pf_inner, H);
    } else {
      DCUDA(d, lin(L.w1, d->pf_xb, dim, d->pf_g, 2 * H));
      DCUDA(d, lin(L.w3, d->pf_xb, dim, d->pf_g + H, 2 * H));
      count++;
      swiglu_rows_kernel<<<dim3((H + 255) / 256, P), 256, 0, s>>>(d->pf_g, d->pf_g + H, 1, 2 * H,
                                                                   d->pf_inner, H);
    }
    DCUDA(d, lin(L.w2, d->pf_inner, H, d->pf_xb2, dim));
    delta = d->pf_xb2;
  }
  if (want_logits) {
    count++;
    rmsnorm_res_kernel<<<P, 256, rms_smem, s>>>(A, delta, d->rms_final, d->rms_eps, dim,
                                                d->pf_xb, B);
    DCUDA(d, lin(d->head, d->pf_xb, dim, d->logit_log, d->vocab));
  }
  DCUDA(d, cudaGetLastError());
  return VTQ_OK;
}

vtq_status vtq_decode_run(vtq_decode* d, const uint32_t* prompt, size_t n_prompt, size_t n_new,
                          uint32_t* out_tokens, float* logits) {
  if (!d || (!prompt && n_prompt) || (!out_tokens && n_new)) return VTQ_ERR_INVALID_ARG;
  if (n_prompt == 0)
    return dfail(d, VTQ_ERR_INTERNAL, "invalid shape: prompt_tokens must not be empty");
  const size_t total = n_prompt + n_new;
  if (total > (size_t)d->seq_len)
    return dfail(d, VTQ_ERR_INTERNAL, "invalid shape: prompt + n_new_tokens exceeds seq_len");
  for (size_t i = 0; i < n_prompt; i++)
    if (prompt[i] >= (uint32_t)d->vocab)
      return dfail(d, VTQ_ERR_INTERNAL, "embedding_row: table too small for token id");
  DCUDA(d, cudaSetDevice(d->device));
  const bool want_logits = logits != nullptr;
  if (want_logits && d->logit_log_cap < total * d->vocab) {
    float* p;
    if (vtq_status s = dalloc(d, &p, total * d->vocab * 4)) return s;
    d->logit_log = p;
    d->logit_log_cap = total * d->vocab;
    if (d->graph) {
      cudaGraphExecDestroy(d->graph);
      d->graph = nullptr;
    }
  }
  // Prompt positions whose next token is the prompt's own run batched.
  const size_t P0 = d->prefill && n_prompt >= 2 ? n_prompt - 1 : 0;
  if (d->mk) {
    // Persistent step kernel: one cooperative launch per position.
    if (!d->ev[0])
      for (auto& e : d->ev) DCUDA(d, cudaEventCreate(&e));
    DCUDA(d, cudaEventRecord(d->ev[0], d->stream));
    StepState hs0{(int)P0, prompt[P0], (int)n_prompt, (int)total, 0};
    DCUDA(d, cudaMemcpyAsync(d->st, &hs0, sizeof hs0, cudaMemcpyHostToDevice, d->stream));
    DCUDA(d, cudaMemcpyAsync(d->prompt, prompt, n_prompt * 4, cudaMemcpyHostToDevice, d->stream));
    DCUDA(d, cudaEventRecord(d->ev[1], d->stream));
    const unsigned long long c0 = kernel_launch_count();
    if (P0 > 0)
      if (vtq_status e = enqueue_prefill(d, (int)P0, want_logits)) return e;
    for (size_t pos = P0; pos < total; pos++)
      DCUDA(d, mk_launch(d->mk, want_logits ? d->logit_log : nullptr, d->stream));
    d->launches = kernel_launch_count() - c0 + (total - P0);
    DCUDA(d, cudaEventRecord(d->ev[2], d->stream));
    if (n_new)
      DCUDA(d, cudaMemcpyAsync(out_tokens, d->out_tokens, n_new * 4, cudaMemcpyDeviceToHost,
                               d->stream));
    if (want_logits)
      DCUDA(d, cudaMemcpyAsync(logits, d->logit_log, total * d->vocab * 4,
                               cudaMemcpyDeviceToHost, d->stream));
    unsigned stat = 0;
    DCUDA(d, cudaMemcpyAsync(&stat, d->status, 4, cudaMemcpyDeviceToHost, d->stream));
    DCUDA(d, cudaEventRecord(d->ev[3], d->stream));
    DCUDA(d, cudaStreamSynchronize(d->stream));
    DCUDA(d, cudaEventElapsedTime(&d->ms_steps, d->ev[1], d->ev[2]));
    DCUDA(d, cudaEventElapsedTime(&d->ms_call, d->ev[0], d->ev[3]));
    if (stat) return dfail(d, VTQ_ERR_TIMEOUT, "decode: a device-side wait timed out");
    return VTQ_OK;
  }
  if (!d->graph || d->graph_logs != want_logits) {
    if (d->graph) cudaGraphExecDestroy(d->graph);
    d->graph = nullptr;
    // One uncaptured step on a dummy state first: kernel attributes and tensor
    // maps are set up outside the capture. (It writes position 0 of the KV
    // cache, which every run rewrites before reading.)
    StepState warm{0, 0u, 1, 1, 0};
    DCUDA(d, cudaMemcpyAsync(d->st, &warm, sizeof warm, cudaMemcpyHostToDevice, d->stream));
    if (vtq_status s0 = enqueue_step(d, want_logits)) return s0;
    DCUDA(d, cudaStreamSynchronize(d->stream));
    cudaGraph_t graph;
    DCUDA(d, cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal));
    const vtq_status s = enqueue_step(d, want_logits);
    cudaError_t ce = cudaStreamEndCapture(d->stream, &graph);
    if (s) return s;
    DCUDA(d, ce);
    DCUDA(d, cudaGraphInstantiate(&d->graph, graph, 0));
    size_t nn = 0;
    DCUDA(d, cudaGraphGetNodes(graph, nullptr, &nn));
    std::vector<cudaGraphNode_t> nodes(nn);
    DCUDA(d, cudaGraphGetNodes(graph, nodes.data(), &nn));
    d->graph_kernels = 0;
    for (auto nd : nodes) {
      cudaGraphNodeType t;
      DCUDA(d, cudaGraphNodeGetType(nd, &t));
      d->graph_kernels += t == cudaGraphNodeTypeKernel;
    }
    cudaGraphDestroy(graph);
    d->graph_logs = want_logits;
  }
  if (!d->ev[0])
    for (auto& e : d->ev) DCUDA(d, cudaEventCreate(&e));
  DCUDA(d, cudaEventRecord(d->ev[0], d->stream));
  StepState hs{(int)P0, prompt[P0], (int)n_prompt, (int)total, 0};
  DCUDA(d, cudaMemcpyAsync(d->st, &hs, sizeof hs, cudaMemcpyHostToDevice, d->stream));
  DCUDA(d, cudaMemcpyAsync(d->prompt, prompt, n_prompt * 4, cudaMemcpyHostToDevice, d->stream));
  DCUDA(d, cudaEventRecord(d->ev[1], d->stream));
  const unsigned long long c0 = kernel_launch_count();
  if (P0 > 0)
    if (vtq_status e = enqueue_prefill(d, (int)P0, want_logits)) return e;
  for (size_t pos = P0; pos < total; pos++) DCUDA(d, cudaGraphLaunch(d->graph, d->stream));
  d->launches = kernel_launch_count() - c0 + d->graph_kernels * (total - P0);
  DCUDA(d, cudaEventRecord(d->ev[2], d->stream));
  if (n_new)
    DCUDA(d, cudaMemcpyAsync(out_tokens, d->out_tokens, n_new * 4, cudaMemcpyDeviceToHost,
                             d->stream));
  if (want_logits)
    DCUDA(d, cudaMemcpyAsync(logits, d->logit_log, total * d->vocab * 4, cudaMemcpyDeviceToHost,
                             d->stream));
  unsigned stat = 0;
  DCUDA(d, cudaMemcpyAsync(&stat, d->status, 4, cudaMemcpyDeviceToHost, d->stream));
  DCUDA(d, cudaEventRecord(d->ev[3], d->stream));
  DCUDA(d, cudaStreamSynchronize(d->stream));
  DCUDA(d, cudaEventElapsedTime(&d->ms_steps, d->ev[1], d->ev[2]));
  DCUDA(d, cudaEventElapsedTime(&d->ms_call, d->ev[0], d->ev[3]));
  if (stat) return dfail(d, VTQ_ERR_TIMEOUT, "decode: a device-side wait timed out");
  return VTQ_OK;
}

vtq_status vtq_decode_timing(const vtq_decode* d, float* ms2) {
  if (!d || !ms2) return VTQ_ERR_INVALID_ARG;
  ms2[0] = d->ms_steps;
  ms2[1] = d->ms_call;
  return VTQ_OK;
}

// Diagnostic: copy one of the session's activation buffers (as left by the
// last step) to host memory. 0 x, 1 xb, 2 q, 3 k, 4 v, 5 xo, 6 xb2, 7 g,
// 8 u, 9 inner, 10 logits; n is the element count to copy.
vtq_status vtq_decode_debug_buffer(vtq_decode* d, int which, float* out, size_t n) {
  if (!d || !out) return VTQ_ERR_INVALID_ARG;
  float* bufs[] = {d->x, d->xb, d->q, d->k, d->v, d->xo, d->xb2, d->g, d->u, d->inner, d->logits};
  if (which < 0 || which > 10) return VTQ_ERR_INVALID_ARG;
  DCUDA(d, cudaMemcpyAsync(out, bufs[which], n * 4, cudaMemcpyDeviceToHost, d->stream));
  DCUDA(d, cudaStreamSynchronize(d->stream));
  return VTQ_OK;
}

vtq_status vtq_decode_close(vtq_decode* d) {
  if (!d) return VTQ_ERR_INVALID_ARG;
  cudaSetDevice(d->device);
  if (d->stream) cudaStreamSynchronize(d->stream);
  if (d->graph) cudaGraphExecDestroy(d->graph);
  for (auto e : d->ev)
    if (e) cudaEventDestroy(e);
  if (d->side) cudaStreamSynchronize(d->side);
  mk_free(d->mk);
  if (d->fork) cudaEventDestroy(d->fork);
  if (d->join) cudaEventDestroy(d->join);
  for (void* p : d->allocs) cudaFree(p);
  if (d->stream) cudaStreamDestroy(d->stream);
  if (d->side) cudaStreamDestroy(d->side);
  delete d;
  return VTQ_OK;
}

}  // extern "C"
