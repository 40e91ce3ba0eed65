// decode_ops.cuh -- per-step operations of the quantized Llama decode shared
// by the one-kernel-per-op step (decode.cu) and the persistent step kernel
// (decode_mk.cu). Each follows the reference's op order bit for bit.
#pragma once
#include <cuda_fp16.h>

#include "decode_mk.h"
#include "vtq_device.cuh"
#include "vtq_internal.h"
#include "vtq_libm.h"

namespace vtq {
namespace {

// Qwen2 additions to the attention step: NeoX RoPE and the QKV biases
// (device vectors of the q / kv widths, or null).
struct AttnExtras {
  int neox;
  const float *bq, *bk, *bv;
  int no_cache_write = 0;  // batched prompt: k / v already cached for every position
};

// embedding_row (forward_quantized.rs:818-919): element e of row `row` of the
// table in its device layout (Q6_K regrouped, see repack.cu).
__device__ __forceinline__ float embed_value(const uint8_t* table, int dtype, int64_t pitch,
                                             int dim, uint32_t row, int e) {
  const uint8_t* r = table + (int64_t)row * pitch;
  float v;
  if (dtype == T_F32) {
    v = reinterpret_cast<const float*>(r)[e];
  } else if (dtype == T_Q8_0) {
    const uint8_t* b = r + (e >> 5) * 34;
    v = __fmul_rn(f16_bits_to_f32(b[0] | (b[1] << 8)), (float)(int8_t)b[2 + (e & 31)]);
  } else if (dtype == T_Q4_K) {  // quant.rs:280-326
    const uint8_t* sb = r + (e >> 8) * 144;
    const int k = e & 255, half = k >> 6, hi = (k >> 5) & 1, l = k & 31, j = 2 * half + hi;
    const uint8_t* s = sb + 4;
    int sc, m;
    if (j < 4) {
      sc = s[j] & 63;
      m = s[j + 4] & 63;
    } else {
      sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
      m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
    const float d = f16_bits_to_f32(sb[0] | (sb[1] << 8));
    const float dmin = f16_bits_to_f32(sb[2] | (sb[3] << 8));
    const uint8_t byte = sb[16 + 32 * half + l];
    const int q = hi ? (byte >> 4) : (byte & 15);
    v = __fsub_rn(__fmul_rn(__fmul_rn(d, (float)sc), (float)q), __fmul_rn(dmin, (float)m));
  } else {  // Q6_K, device layout: group of G superblocks
    const int s = e >> 8, gi = s >> 3, i = s & 7;
    const int S = dim >> 8, G = min(8, S - 8 * gi);
    const uint8_t* gb = r + gi * 1680;
    const int k = e & 255, half = k >> 7, w = k & 127, t = w >> 5, l = w & 31;
    // ql byte (64 half + l + 32 (t & 1)), nibble t >> 1; qh byte (32 half + l), bits 2t.
    const int qlb = 64 * half + l + 32 * (t & 1), qhb = 32 * half + l;
    const uint8_t ql = gb[16 * (G * (qlb >> 4) + i) + (qlb & 15)];
    const uint8_t qh = gb[128 * G + 16 * (G * (qhb >> 4) + i) + (qhb & 15)];
    const int q = (int)(((t >> 1) ? (ql >> 4) : (ql & 15)) | (((qh >> (2 * t)) & 3) << 4)) - 32;
    const int sc = (int8_t)gb[192 * G + 16 * i + 8 * half + (l >> 4) + 2 * t];
    const float d = f16_bits_to_f32(gb[208 * G + 2 * i] | (gb[208 * G + 2 * i + 1] << 8));
    v = __fmul_rn(__fmul_rn(d, (float)sc), (float)q);  // d * s * q (quant.rs:378-381)
  }
  return v;
}

// Attention for one query head with the step's RoPE fused in
// (forward_quantized.rs:407-500): rotate this head's q and its kv head's new
// k (interleaved pairs, host cos/sin tables), store the rotated k and the raw
// v at `pos` of the cache (first query head of each kv group), then serial
// scores over head_dim, softmax with a serial sum, and a serial P.V sum over
// positions for every head dimension. Positions < pos come from the cache;
// position pos uses the k/v computed here (the same values the cache gets).
// Run by `nthr` threads (index tid); sync() is their barrier; sm holds
// 3 hs + seq_len floats, red two floats.
template <class Sync>
__device__ __forceinline__ void attention_head(int h, const float* q, const float* k,
                                               const float* v, float* kc, float* vc, int layer,
                                               int seq_len, int kv_dim, int hs, int kv_mul,
                                               const float* rcos, const float* rsin, int pos,
                                               float* out, float* sm, float* red, int tid,
                                               int nthr, Sync sync, const AttnExtras& ex) {
  float* qh = sm;            // [hs] rotated query head
  float* kh = sm + hs;       // [hs] rotated new key
  float* vh = sm + 2 * hs;   // [hs] new value
  float* att = sm + 3 * hs;  // [pos + 1]
  const int g = h / kv_mul, np = pos + 1;
  const size_t off = ((size_t)layer * seq_len + pos) * kv_dim;
  // Pair p of the head: elements (2p, 2p + 1) for Llama's interleaved RoPE,
  // (p, p + hs/2) for NeoX (Qwen2, forward_quantized.rs:417-448). Both use
  // freq = 1 / powf(theta, 2p / hs), so one cos/sin table serves both. The
  // optional QKV bias is added first (add_bias, :807-813; pad entries are
  // -0.0, which leaves every value unchanged).
  const int half = hs / 2;
  for (int p = tid; p < half; p += nthr) {
    const int e0 = ex.neox ? p : 2 * p, e1 = ex.neox ? p + half : 2 * p + 1;
    const float fcr = rcos[(size_t)pos * half + p], fci = rsin[(size_t)pos * half + p];
    float q0 = q[h * hs + e0], q1 = q[h * hs + e1];
    float k0 = k[g * hs + e0], k1 = k[g * hs + e1];
    float v0 = v[g * hs + e0], v1 = v[g * hs + e1];
    if (ex.bq) {
      q0 = __fadd_rn(q0, ex.bq[h * hs + e0]);
      q1 = __fadd_rn(q1, ex.bq[h * hs + e1]);
    }
    if (ex.bk) {
      k0 = __fadd_rn(k0, ex.bk[g * hs + e0]);
      k1 = __fadd_rn(k1, ex.bk[g * hs + e1]);
    }
    if (ex.bv) {
      v0 = __fadd_rn(v0, ex.bv[g * hs + e0]);
      v1 = __fadd_rn(v1, ex.bv[g * hs + e1]);
    }
    qh[e0] = __fsub_rn(__fmul_rn(q0, fcr), __fmul_rn(q1, fci));
    qh[e1] = __fadd_rn(__fmul_rn(q0, fci), __fmul_rn(q1, fcr));
    const float r0 = __fsub_rn(__fmul_rn(k0, fcr), __fmul_rn(k1, fci));
    const float r1 = __fadd_rn(__fmul_rn(k0, fci), __fmul_rn(k1, fcr));
    kh[e0] = r0;
    kh[e1] = r1;
    vh[e0] = v0;
    vh[e1] = v1;
    if (h % kv_mul == 0 && !ex.no_cache_write) {
      kc[off + g * hs + e0] = r0;
      kc[off + g * hs + e1] = r1;
      vc[off + g * hs + e0] = v0;
      vc[off + g * hs + e1] = v1;
    }
  }
  sync();
  const float* kbase = kc + (size_t)layer * seq_len * kv_dim + g * hs;
  const float* vbase = vc + (size_t)layer * seq_len * kv_dim + g * hs;
  const float root = __fsqrt_rn((float)hs);
  for (int t = tid; t < np; t += nthr) {
    const float* kt = (t == pos) ? kh : kbase + (size_t)t * kv_dim;
    float score = 0.0f;
    if ((hs & 15) == 0) {
      for (int d0 = 0; d0 < hs; d0 += 16) {
        float4 kv4[4], qv4[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
          kv4[u] = *reinterpret_cast<const float4*>(kt + d0 + 4 * u);
          qv4[u] = *reinterpret_cast<const float4*>(qh + d0 + 4 * u);
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
          score = __fadd_rn(score, __fmul_rn(qv4[u].x, kv4[u].x));
          score = __fadd_rn(score, __fmul_rn(qv4[u].y, kv4[u].y));
          score = __fadd_rn(score, __fmul_rn(qv4[u].z, kv4[u].z));
          score = __fadd_rn(score, __fmul_rn(qv4[u].w, kv4[u].w));
        }
      }
    } else {
      for (int d = 0; d < hs; d++) score = __fadd_rn(score, __fmul_rn(qh[d], kt[d]));
    }
    att[t] = __fdiv_rn(score, root);
  }
  sync();
  if (tid == 0) {
    float mx = -INFINITY;
    for (int t = 0; t < np; t++)
      if (att[t] > mx) mx = att[t];
    red[0] = mx;
  }
  sync();
  for (int t = tid; t < np; t += nthr) att[t] = libm::expf(__fsub_rn(att[t], red[0]));
  sync();
  if (tid == 0) {
    float sum = 0.0f;
    int t = 0;
    for (; t + 4 <= np; t += 4) {
      const float a0 = att[t], a1 = att[t + 1], a2 = att[t + 2], a3 = att[t + 3];
      sum = __fadd_rn(sum, a0);
      sum = __fadd_rn(sum, a1);
      sum = __fadd_rn(sum, a2);
      sum = __fadd_rn(sum, a3);
    }
    for (; t < np; t++) sum = __fadd_rn(sum, att[t]);
    red[1] = __fdiv_rn(1.0f, sum);
  }
  sync();
  for (int t = tid; t < np; t += nthr) att[t] = __fmul_rn(att[t], red[1]);
  sync();
  for (int d = tid; d < hs; d += nthr) {
    float acc = 0.0f;
    int t = 0;
    for (; t + 4 <= pos; t += 4) {
      const float v0 = vbase[(size_t)t * kv_dim + d], v1 = vbase[(size_t)(t + 1) * kv_dim + d];
      const float v2 = vbase[(size_t)(t + 2) * kv_dim + d], v3 = vbase[(size_t)(t + 3) * kv_dim + d];
      acc = __fadd_rn(acc, __fmul_rn(att[t], v0));
      acc = __fadd_rn(acc, __fmul_rn(att[t + 1], v1));
      acc = __fadd_rn(acc, __fmul_rn(att[t + 2], v2));
      acc = __fadd_rn(acc, __fmul_rn(att[t + 3], v3));
    }
    for (; t < pos; t++) acc = __fadd_rn(acc, __fmul_rn(att[t], vbase[(size_t)t * kv_dim + d]));
    acc = __fadd_rn(acc, __fmul_rn(att[pos], vh[d]));
    out[h * hs + d] = acc;
  }
}

// argmax (argmax.rs:49-60: first index of the maximum, strict >) and the
// token choice of the run loop (inference.rs:318-326), then pos += 1.
// Run by nthr threads (a multiple of 32, at most 1024); bv / bi hold 32
// entries each; sync() is their barrier.
template <class Sync>
__device__ __forceinline__ void argmax_next(const float* logits, int n, StepState* st,
                                            const uint32_t* prompt, uint32_t* out_tokens,
                                            float* bv, int* bi, int tid, int nthr, Sync sync) {
  float best = -INFINITY;
  int besti = 0x7fffffff;
  for (int i = tid; i < n; i += nthr) {
    const float v = logits[i];
    if (v > best || (v == best && i < besti)) {
      best = v;
      besti = i;
    }
  }
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_down_sync(0xffffffffu, best, o);
    const int oi = __shfl_down_sync(0xffffffffu, besti, o);
    if (ov > best || (ov == best && oi < besti)) {
      best = ov;
      besti = oi;
    }
  }
  const int w = tid >> 5, lane = tid & 31;
  if (lane == 0) {
    bv[w] = best;
    bi[w] = besti;
  }
  sync();
  if (tid == 0) {
    for (int k = 1; k < nthr / 32; k++)
      if (bv[k] > best || (bv[k] == best && bi[k] < besti)) {
        best = bv[k];
        besti = bi[k];
      }
    // NaN at index 0 is never beaten by a strict > (sequential rule).
    if (logits[0] != logits[0] || besti == 0x7fffffff) besti = 0;
    const int pos = st->pos;
    const uint32_t picked = (uint32_t)besti;
    const uint32_t next = (pos + 1 < st->n_prompt) ? prompt[pos + 1] : picked;
    if (pos >= st->n_prompt) out_tokens[st->n_gen++] = next;
    st->cur = next;
    st->pos = pos + 1;
  }
}

}  // namespace
}  // namespace vtq
