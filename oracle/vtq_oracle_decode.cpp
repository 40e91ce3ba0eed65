// vtq_oracle_decode.cpp -- CPU restatement of the reference's quantized decode
// step and prompt+generate loop.
//
// TEST INFRASTRUCTURE ONLY: the checker for the device decode session.
//   step            src/model/forward_quantized.rs:329-649 (interleaved RoPE for
//                   Llama, NeoX split-half RoPE for Qwen2 (:414-448), optional
//                   QKV bias (add_bias :807-813), separate or shared LM head)
//   embedding_row   src/model/forward_quantized.rs:818-919
//   softmax_inplace src/model/forward_quantized.rs:925-941
//   rms_norm_slice  src/ops/rms_norm.rs:94-108
//   argmax          src/ops/argmax.rs:49-60
//   run loop        src/model/inference.rs:312-327
// Linears go through or_linear_dispatch (the std-parallel regime). The
// transcendentals come from the project's libm restatement (vtq_libm.h), which
// is pinned independently by the reference's sweep hash.
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "../vitni-tensor_b200/csrc/vtq_libm.h"
#include "vtq_oracle.h"

extern "C" {

typedef struct {
  int32_t dtype;
  const uint8_t* bytes;
  size_t len;
} or_tensor;

typedef struct {
  const float* rms_att;
  const float* rms_ffn;
  or_tensor wq, wk, wv, wo, w1, w2, w3;
  const float *bq, *bk, *bv;  // NULL when absent; else bq_len / bk_len / bv_len entries
  int32_t bq_len, bk_len, bv_len;
} or_layer;

typedef struct {
  int32_t dim, hidden, n_layers, n_heads, n_kv_heads, vocab, seq_len;
  float rope_theta, rms_eps;
  int32_t rope_neox;  // quant_weights.rs:151: architecture "qwen2"
  or_tensor embd;
  const float* rms_final;
  or_tensor wcls;  // bytes == NULL: the head shares token_embd
  const or_layer* layers;
} or_model;

}  // extern "C"

namespace {

struct State {
  const or_model* m;
  std::vector<float> key_cache, value_cache;  // [layers][seq_len][kv_dim]
  int threads;
};

int linear(const float* x, const or_tensor& w, int in, int out, float* y, int threads) {
  return or_linear_dispatch(w.dtype, x, w.bytes, w.len, (size_t)in, (size_t)out, y, 0,
                            (size_t)threads);
}

// embedding_row: dequantise row `row` of the table (forward_quantized.rs:818-919).
int embedding_row(const or_tensor& t, int row, int dim, float* out) {
  if (t.dtype == OR_F32) {
    memcpy(out, reinterpret_cast<const float*>(t.bytes) + (size_t)row * dim, dim * 4);
    return OR_OK;
  }
  size_t per = 0, nb = 0;
  switch (t.dtype) {
    case OR_Q4_0: per = 32; nb = 18; break;
    case OR_Q5_0: per = 32; nb = 22; break;
    case OR_Q8_0: per = 32; nb = 34; break;
    case OR_Q4_K: per = 256; nb = 144; break;
    case OR_Q6_K: per = 256; nb = 210; break;
    default: return OR_ERR_NOT_IMPLEMENTED;
  }
  const size_t rb = dim / per * nb;
  const uint8_t* p = t.bytes + (size_t)row * rb;
  switch (t.dtype) {
    case OR_Q4_0: return or_dequantize_q4_0(p, rb, out);
    case OR_Q5_0: return or_dequantize_q5_0(p, rb, out);
    case OR_Q8_0: return or_dequantize_q8_0(p, rb, out);
    case OR_Q4_K: return or_dequantize_q4_k(p, rb, out);
    default: return or_dequantize_q6_k(p, rb, out);
  }
}

void softmax_inplace(float* x, int n) {
  float mx = -INFINITY;
  for (int i = 0; i < n; i++)
    if (x[i] > mx) mx = x[i];
  float sum = 0.0f;
  for (int i = 0; i < n; i++) {
    x[i] = vtq::libm::expf(x[i] - mx);
    sum += x[i];
  }
  const float inv = 1.0f / sum;
  for (int i = 0; i < n; i++) x[i] *= inv;
}

// add_bias (forward_quantized.rs:807-813): v[i] += b[i] over the shorter length.
void add_bias(float* v, int n, const float* b, int blen) {
  if (!b) return;
  for (int i = 0; i < n && i < blen; i++) v[i] = v[i] + b[i];
}

int step(State& st, uint32_t token, int pos, float* logits) {
  const or_model& m = *st.m;
  const int dim = m.dim, hs = dim / m.n_heads, kv_dim = m.n_kv_heads * hs;
  const int kv_mul = m.n_heads / m.n_kv_heads, hidden = m.hidden;
  std::vector<float> x(dim), xb(dim), q(dim), k(kv_dim), v(kv_dim), xo(dim), xb2(dim);
  std::vector<float> g(hidden), u(hidden), inner(hidden), att(pos + 1);
  int s = embedding_row(m.embd, (int)token, dim, x.data());
  if (s) return s;
  for (int l = 0; l < m.n_layers; l++) {
    const or_layer& L = m.layers[l];
    or_rms_norm(x.data(), L.rms_att, dim, m.rms_eps, xb.data());
    if ((s = linear(xb.data(), L.wq, dim, dim, q.data(), st.threads))) return s;
    if ((s = linear(xb.data(), L.wk, dim, kv_dim, k.data(), st.threads))) return s;
    if ((s = linear(xb.data(), L.wv, dim, kv_dim, v.data(), st.threads))) return s;
    add_bias(q.data(), dim, L.bq, L.bq_len);
    add_bias(k.data(), kv_dim, L.bk, L.bk_len);
    add_bias(v.data(), kv_dim, L.bv, L.bv_len);
    const size_t off = ((size_t)l * m.seq_len + pos) * kv_dim;
    float* kc = st.key_cache.data();
    float* vc = st.value_cache.data();
    memcpy(kc + off, k.data(), kv_dim * 4);
    memcpy(vc + off, v.data(), kv_dim * 4);
    if (m.rope_neox) {
      // NeoX RoPE: pairs (j, j + hs/2) within each head, q heads then cached k heads.
      const int half = hs / 2;
      for (int pass = 0; pass < 2; pass++) {
        const int nh = pass == 0 ? m.n_heads : kv_dim / hs;
        float* base0 = pass == 0 ? q.data() : kc + off;
        for (int h = 0; h < nh; h++) {
          float* b = base0 + h * hs;
          for (int j = 0; j < half; j++) {
            const float freq = 1.0f / vtq::libm::powf(m.rope_theta, (float)(2 * j) / (float)hs);
            const float val = (float)pos * freq;
            const float fcr = vtq::libm::cosf(val), fci = vtq::libm::sinf(val);
            const float a = b[j], c = b[j + half];
            b[j] = a * fcr - c * fci;
            b[j + half] = a * fci + c * fcr;
          }
        }
      }
    }
    // Interleaved RoPE on q (all of dim) and on the cached k (i < kv_dim).
    for (int i = 0; i < dim && !m.rope_neox; i += 2) {
      const int idx = i % hs;
      const float freq = 1.0f / vtq::libm::powf(m.rope_theta, (float)idx / (float)hs);
      const float val = (float)pos * freq;
      const float fcr = vtq::libm::cosf(val), fci = vtq::libm::sinf(val);
      const float q0 = q[i], q1 = q[i + 1];
      q[i] = q0 * fcr - q1 * fci;
      q[i + 1] = q0 * fci + q1 * fcr;
      if (i < kv_dim) {
        const float k0 = kc[off + i], k1 = kc[off + i + 1];
        kc[off + i] = k0 * fcr - k1 * fci;
        kc[off + i + 1] = k0 * fci + k1 * fcr;
      }
    }
    // Attention (forward_quantized.rs:476-500).
    std::fill(xo.begin(), xo.end(), 0.0f);
    for (int h = 0; h < m.n_heads; h++) {
      for (int t = 0; t <= pos; t++) {
        const float* kt = kc + ((size_t)l * m.seq_len + t) * kv_dim + (h / kv_mul) * hs;
        float score = 0.0f;
        for (int d = 0; d < hs; d++) score += q[h * hs + d] * kt[d];
        score /= std::sqrt((float)hs);
        att[t] = score;
      }
      softmax_inplace(att.data(), pos + 1);
      for (int t = 0; t <= pos; t++) {
        const float* vt = vc + ((size_t)l * m.seq_len + t) * kv_dim + (h / kv_mul) * hs;
        const float a = att[t];
        for (int d = 0; d < hs; d++) xo[h * hs + d] += a * vt[d];
      }
    }
    if ((s = linear(xo.data(), L.wo, dim, dim, xb2.data(), st.threads))) return s;
    for (int i = 0; i < dim; i++) x[i] = x[i] + xb2[i];
    or_rms_norm(x.data(), L.rms_ffn, dim, m.rms_eps, xb.data());
    if ((s = linear(xb.data(), L.w1, dim, hidden, g.data(), st.threads))) return s;
    if ((s = linear(xb.data(), L.w3, dim, hidden, u.data(), st.threads))) return s;
    for (int i = 0; i < hidden; i++) {
      const float gi = g[i];
      const float silu = gi / (1.0f + vtq::libm::expf(-gi));
      inner[i] = silu * u[i];
    }
    if ((s = linear(inner.data(), L.w2, hidden, dim, xb2.data(), st.threads))) return s;
    for (int i = 0; i < dim; i++) x[i] = x[i] + xb2[i];
  }
  or_rms_norm(x.data(), m.rms_final, dim, m.rms_eps, xb.data());
  const or_tensor& head = m.wcls.bytes ? m.wcls : m.embd;
  return linear(xb.data(), head, dim, m.vocab, logits, st.threads);
}

}  // namespace

extern "C" {

// The prompt + greedy loop of run_quantized_with_sink (inference.rs:312-327).
// out_tokens receives n_new ids; logits (optional) (n_prompt + n_new) x vocab.
int or_decode_run(const or_model* m, const uint32_t* prompt, size_t n_prompt, size_t n_new,
                  uint32_t* out_tokens, float* logits, int threads) {
  if (n_prompt == 0) return OR_ERR_INTERNAL;
  const size_t total = n_prompt + n_new;
  if (total > (size_t)m->seq_len) return OR_ERR_INTERNAL;
  State st;
  st.m = m;
  st.threads = threads;
  const size_t kv_dim = (size_t)m->n_kv_heads * (m->dim / m->n_heads);
  st.key_cache.assign((size_t)m->n_layers * m->seq_len * kv_dim, 0.0f);
  st.value_cache.assign((size_t)m->n_layers * m->seq_len * kv_dim, 0.0f);
  std::vector<float> lg(m->vocab);
  uint32_t cur = prompt[0];
  size_t gen = 0;
  for (size_t pos = 0; pos < total; pos++) {
    const int s = step(st, cur, (int)pos, lg.data());
    if (s) return s;
    if (logits) memcpy(logits + pos * m->vocab, lg.data(), (size_t)m->vocab * 4);
    const uint32_t picked = or_argmax(lg.data(), m->vocab);
    const uint32_t next = (pos + 1 < n_prompt) ? prompt[pos + 1] : picked;
    if (pos >= n_prompt) out_tokens[gen++] = next;
    cur = next;
  }
  return OR_OK;
}

}  // extern "C"
