/*
 * vtq_oracle.c -- CPU restatement of vitni-tensor's k-quant linear arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path, never the product.
 * Build: -O2 -ffp-contract=off -fno-fast-math (see oracle/Makefile). On x86-64
 * float arithmetic is SSE single precision, so every C float operation below is
 * one IEEE binary32 operation rounded to nearest, as in Rust.
 *
 * Citations are file:line in the vitni-tensor project.
 */
#include "vtq_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* Rust `f as i32`: truncate toward zero, saturate, NaN -> 0. */
static inline int32_t rust_f32_to_i32(float f) {
  if (f != f) return 0;
  if (f >= 2147483648.0f) return INT32_MAX;
  if (f < -2147483648.0f) return INT32_MIN;
  return (int32_t)f;
}

static inline uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* src/ops/quant.rs:41-66 */
float or_f16_to_f32(uint16_t half) {
  uint32_t sign = (half >> 15) & 1u, exp = (half >> 10) & 0x1Fu, mant = half & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (mant == 0) {
      bits = sign << 31;
    } else {
      uint32_t m = mant;
      int32_t e = 1;
      while ((m & 0x400u) == 0) { m <<= 1; e -= 1; }
      m &= 0x3FFu;
      bits = (sign << 31) | ((uint32_t)(127 - 15 + e) << 23) | (m << 13);
    }
  } else if (exp == 0x1F) {
    bits = (sign << 31) | 0x7F800000u | (mant << 13);
  } else {
    bits = (sign << 31) | ((exp + 127 - 15) << 23) | (mant << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* src/ops/quant.rs:69-84 (truncating encoder used by the reference's tests). */
uint16_t or_f32_to_f16(float f) {
  uint32_t bits;
  memcpy(&bits, &f, 4);
  uint16_t sign = (uint16_t)((bits >> 31) & 1u);
  int32_t exp = (int32_t)((bits >> 23) & 0xFFu) - 127 + 15;
  uint32_t mant = (bits >> 13) & 0x3FFu;
  if (exp <= 0) return (uint16_t)(sign << 15);
  if (exp >= 0x1F) return (uint16_t)((sign << 15) | 0x7C00u);
  return (uint16_t)((sign << 15) | ((uint32_t)exp << 10) | mant);
}

/* src/ops/quant.rs:91-111 */
int or_dequantize_q4_0(const uint8_t* q, size_t nbytes, float* out) {
  if (nbytes % 18) return OR_ERR_INTERNAL;
  size_t nb = nbytes / 18;
  for (size_t b = 0; b < nb; b++) {
    const uint8_t* blk = q + b * 18;
    float scale = or_f16_to_f32(rd16(blk));
    for (int k = 0; k < 16; k++) {
      uint8_t byte = blk[2 + k];
      int32_t lo = (int32_t)(byte & 0x0F) - 8, hi = (int32_t)(byte >> 4) - 8;
      out[b * 32 + 2 * k] = scale * (float)lo;
      out[b * 32 + 2 * k + 1] = scale * (float)hi;
    }
  }
  return OR_OK;
}

/* src/ops/quant.rs:116-152 */
int or_quantize_q4_0(const float* data, size_t n, uint8_t* out) {
  if (n % 32) return OR_ERR_INTERNAL;
  for (size_t b = 0; b < n / 32; b++) {
    const float* blk = data + b * 32;
    float amax = 0.0f, max_val = 0.0f;
    for (int i = 0; i < 32; i++) {
      float a = fabsf(blk[i]);
      if (a > amax) { amax = a; max_val = blk[i]; }
    }
    float scale = max_val / -8.0f;
    float inv = scale != 0.0f ? 1.0f / scale : 0.0f;
    uint16_t h = or_f32_to_f16(scale);
    out[b * 18] = (uint8_t)(h & 0xFF);
    out[b * 18 + 1] = (uint8_t)(h >> 8);
    for (int k = 0; k < 16; k++) {
      float x0 = blk[2 * k] * inv + 8.5f;
      float x1 = blk[2 * k + 1] * inv + 8.5f;
      int32_t q0 = rust_f32_to_i32(x0), q1 = rust_f32_to_i32(x1);
      q0 = q0 < 0 ? 0 : (q0 > 15 ? 15 : q0);
      q1 = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
      out[b * 18 + 2 + k] = (uint8_t)(q0 | (q1 << 4));
    }
  }
  return OR_OK;
}

/* src/ops/quant.rs:160-186 */
int or_dequantize_q5_0(const uint8_t* q, size_t nbytes, float* out) {
  if (nbytes % 22) return OR_ERR_INTERNAL;
  size_t nb = nbytes / 22;
  for (size_t b = 0; b < nb; b++) {
    const uint8_t* blk = q + b * 22;
    float scale = or_f16_to_f32(rd16(blk));
    uint32_t qh = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8) | ((uint32_t)blk[4] << 16) |
                  ((uint32_t)blk[5] << 24);
    const uint8_t* qs = blk + 6;
    for (int j = 0; j < 16; j++) {
      uint8_t xh0 = (uint8_t)(((qh >> j) << 4) & 0x10u);
      uint8_t xh1 = (uint8_t)((qh >> (j + 12)) & 0x10u);
      int32_t x0 = (int32_t)((qs[j] & 0x0F) | xh0) - 16;
      int32_t x1 = (int32_t)((qs[j] >> 4) | xh1) - 16;
      out[b * 32 + j] = scale * (float)x0;
      out[b * 32 + j + 16] = scale * (float)x1;
    }
  }
  return OR_OK;
}

/* src/ops/quant.rs:193-210 */
int or_dequantize_q8_0(const uint8_t* q, size_t nbytes, float* out) {
  if (nbytes % 34) return OR_ERR_INTERNAL;
  size_t nb = nbytes / 34;
  for (size_t b = 0; b < nb; b++) {
    const uint8_t* blk = q + b * 34;
    float scale = or_f16_to_f32(rd16(blk));
    for (int k = 0; k < 32; k++) out[b * 32 + k] = scale * (float)(int8_t)blk[2 + k];
  }
  return OR_OK;
}

/* src/ops/quant.rs:214-241 */
int or_quantize_q8_0(const float* data, size_t n, uint8_t* out) {
  if (n % 32) return OR_ERR_INTERNAL;
  for (size_t b = 0; b < n / 32; b++) {
    const float* blk = data + b * 32;
    float amax = 0.0f;
    for (int i = 0; i < 32; i++) {
      float a = fabsf(blk[i]);
      if (a > amax) amax = a;
    }
    float scale = amax / 127.0f;
    float inv = scale != 0.0f ? 1.0f / scale : 0.0f;
    uint16_t h = or_f32_to_f16(scale);
    out[b * 34] = (uint8_t)(h & 0xFF);
    out[b * 34 + 1] = (uint8_t)(h >> 8);
    for (int k = 0; k < 32; k++) {
      float scaled = blk[k] * inv;
      float bias = scaled >= 0.0f ? 0.5f : -0.5f;
      int32_t q = rust_f32_to_i32(scaled + bias);
      q = q < -127 ? -127 : (q > 127 ? 127 : q);
      out[b * 34 + 2 + k] = (uint8_t)(int8_t)q;
    }
  }
  return OR_OK;
}

/* src/ops/quant.rs:268-276 */
static inline void get_scale_min_k4(int j, const uint8_t* s, int* sc, int* m) {
  if (j < 4) {
    *sc = s[j] & 63;
    *m = s[j + 4] & 63;
  } else {
    *sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
    *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

/* src/ops/quant.rs:280-326 */
int or_dequantize_q4_k(const uint8_t* q, size_t nbytes, float* out) {
  if (nbytes % 144) return OR_ERR_INTERNAL;
  size_t nb = nbytes / 144;
  for (size_t b = 0; b < nb; b++) {
    const uint8_t* blk = q + b * 144;
    float d = or_f16_to_f32(rd16(blk)), dmin = or_f16_to_f32(rd16(blk + 2));
    const uint8_t* sc = blk + 4;
    const uint8_t* qs = blk + 16;
    float* y = out + b * 256;
    for (int it = 0; it < 4; it++) {
      int sc1, m1, sc2, m2;
      get_scale_min_k4(2 * it, sc, &sc1, &m1);
      get_scale_min_k4(2 * it + 1, sc, &sc2, &m2);
      float d1 = d * (float)sc1, m1f = dmin * (float)m1;
      float d2 = d * (float)sc2, m2f = dmin * (float)m2;
      for (int l = 0; l < 32; l++) y[64 * it + l] = d1 * (float)(qs[32 * it + l] & 0x0F) - m1f;
      for (int l = 0; l < 32; l++) y[64 * it + 32 + l] = d2 * (float)(qs[32 * it + l] >> 4) - m2f;
    }
  }
  return OR_OK;
}

/* One Q6_K superblock to 256 floats (src/ops/quant.rs:337-386, same
 * arithmetic as the fused copy at :1245-1270): d * s * q, left to right. */
static void dequant_q6k_block(const uint8_t* blk, float* out) {
  const uint8_t* ql = blk;
  const uint8_t* qh = blk + 128;
  const uint8_t* sc = blk + 192;
  float d = or_f16_to_f32(rd16(blk + 208));
  for (int half = 0; half < 2; half++) {
    int ql_p = 64 * half, qh_p = 32 * half, sc_p = 8 * half, y = 128 * half;
    for (int l = 0; l < 32; l++) {
      int is = l / 16;
      uint8_t h = qh[qh_p + l];
      float q1 = (float)((int32_t)((ql[ql_p + l] & 0x0F) | ((h & 3) << 4)) - 32);
      float q2 = (float)((int32_t)((ql[ql_p + l + 32] & 0x0F) | (((h >> 2) & 3) << 4)) - 32);
      float q3 = (float)((int32_t)((ql[ql_p + l] >> 4) | (((h >> 4) & 3) << 4)) - 32);
      float q4 = (float)((int32_t)((ql[ql_p + l + 32] >> 4) | (((h >> 6) & 3) << 4)) - 32);
      float s1 = (float)(int8_t)sc[sc_p + is], s2 = (float)(int8_t)sc[sc_p + is + 2];
      float s3 = (float)(int8_t)sc[sc_p + is + 4], s4 = (float)(int8_t)sc[sc_p + is + 6];
      out[y + l] = d * s1 * q1;
      out[y + l + 32] = d * s2 * q2;
      out[y + l + 64] = d * s3 * q3;
      out[y + l + 96] = d * s4 * q4;
    }
  }
}

int or_dequantize_q6_k(const uint8_t* q, size_t nbytes, float* out) {
  if (nbytes % 210) return OR_ERR_INTERNAL;
  for (size_t b = 0; b < nbytes / 210; b++) dequant_q6k_block(q + b * 210, out + b * 256);
  return OR_OK;
}

/* src/ops/quant.rs:462-476 */
float or_fixed_tree(float* part, size_t len) {
  if (len == 0) return 0.0f;
  while (len > 1) {
    size_t half = (len + 1) / 2;
    for (size_t t = 0; t < half; t++) {
      size_t u = 2 * t;
      part[t] = (u + 1 < len) ? part[u] + part[u + 1] : part[u];
    }
    len = half;
  }
  return part[0];
}

#define CANON_LANES 8
#define CANON_CHUNK 8192

/* src/ops/quant.rs:482-505 */
float or_canonical_chunk(const float* x, const float* w, size_t n) {
  float lanes[CANON_LANES] = {0};
  size_t full = n - (n % CANON_LANES), i = 0;
  for (; i < full; i += CANON_LANES)
    for (int j = 0; j < CANON_LANES; j++) {
      float p = x[i + j] * w[i + j];
      lanes[j] += p;
    }
  for (; i < n; i++) {
    float p = x[i] * w[i];
    lanes[i % CANON_LANES] += p;
  }
  return or_fixed_tree(lanes, CANON_LANES);
}

/* src/ops/quant.rs:551-566 */
float or_canonical_dot(const float* x, const float* w, size_t n) {
  if (n == 0) return 0.0f;
  if (n <= CANON_CHUNK) return or_canonical_chunk(x, w, n);
  size_t nch = (n + CANON_CHUNK - 1) / CANON_CHUNK;
  float* sums = (float*)malloc(nch * sizeof(float));
  for (size_t c = 0; c < nch; c++) {
    size_t s = c * CANON_CHUNK, e = s + CANON_CHUNK < n ? s + CANON_CHUNK : n;
    sums[c] = or_canonical_chunk(x + s, w + s, e - s);
  }
  float r = or_fixed_tree(sums, nch);
  free(sums);
  return r;
}

/* src/ops/quant.rs:750-771 */
void or_quantize_block_q8(const float* x, size_t n, or_q8block* out) {
  float amax = 0.0f;
  for (size_t i = 0; i < n; i++) {
    float v = x[i];
    float a = v < 0.0f ? -v : v;
    if (a > amax) amax = a;
  }
  float d = amax / 127.0f;
  float inv = d != 0.0f ? 1.0f / d : 0.0f;
  memset(out->qs, 0, sizeof(out->qs));
  memset(out->bsums, 0, sizeof(out->bsums));
  for (size_t i = 0; i < n; i++) {
    float scaled = x[i] * inv;
    float bias = scaled >= 0.0f ? 0.5f : -0.5f;
    int32_t q = rust_f32_to_i32(scaled + bias);
    q = q < -127 ? -127 : (q > 127 ? 127 : q);
    out->qs[i] = (int8_t)q;
    out->bsums[i / 32] += q;
  }
  out->d = d;
}

/* src/ops/quant.rs:850-898 (dot32_pair_scalar :776-784 inlined). */
float or_dot_q4k_q8_block(const uint8_t* w, const or_q8block* xq, size_t n) {
  float d = or_f16_to_f32(rd16(w)), dmin = or_f16_to_f32(rd16(w + 2));
  const uint8_t* scales = w + 4;
  const uint8_t* qs = w + 16;
  int32_t acc = 0, acc_m = 0;
  for (int half = 0; half < 4; half++) {
    int sc_lo, m_lo, sc_hi, m_hi;
    get_scale_min_k4(half * 2, scales, &sc_lo, &m_lo);
    get_scale_min_k4(half * 2 + 1, scales, &sc_hi, &m_hi);
    int q_off = half * 32, base = half * 64;
    int32_t s_lo = 0, s_hi = 0;
    for (int l = 0; l < 32; l++) {
      size_t il = (size_t)base + l, ih = (size_t)base + 32 + l;
      if (il < n) s_lo += (int32_t)(qs[q_off + l] & 0x0F) * (int32_t)xq->qs[il];
      if (ih < n) s_hi += (int32_t)(qs[q_off + l] >> 4) * (int32_t)xq->qs[ih];
    }
    acc += sc_lo * s_lo + sc_hi * s_hi;
    acc_m += m_lo * xq->bsums[half * 2] + m_hi * xq->bsums[half * 2 + 1];
  }
  return d * xq->d * (float)acc - dmin * xq->d * (float)acc_m;
}

/* src/ops/quant.rs:996-1057 */
float or_dot_q6k_q8_block(const uint8_t* w, const or_q8block* xq, size_t n) {
  float d = or_f16_to_f32(rd16(w + 208));
  const uint8_t* ql = w;
  const uint8_t* qh = w + 128;
  const uint8_t* sc = w + 192;
  int32_t sums[16] = {0};
  for (int half = 0; half < 2; half++) {
    int ql_p = half * 64, qh_p = half * 32, sc_p = half * 8, y = half * 128;
    for (int l = 0; l < 32; l++) {
      int is = l / 16;
      uint8_t h = qh[qh_p + l], b0 = ql[ql_p + l], b1 = ql[ql_p + l + 32];
      int32_t q1 = (int32_t)((b0 & 0x0F) | ((h & 3) << 4)) - 32;
      int32_t q2 = (int32_t)((b1 & 0x0F) | (((h >> 2) & 3) << 4)) - 32;
      int32_t q3 = (int32_t)((b0 >> 4) | (((h >> 4) & 3) << 4)) - 32;
      int32_t q4 = (int32_t)((b1 >> 4) | (((h >> 6) & 3) << 4)) - 32;
      size_t i1 = (size_t)y + l, i2 = i1 + 32, i3 = i1 + 64, i4 = i1 + 96;
      if (i1 < n) sums[sc_p + is] += q1 * xq->qs[i1];
      if (i2 < n) sums[sc_p + is + 2] += q2 * xq->qs[i2];
      if (i3 < n) sums[sc_p + is + 4] += q3 * xq->qs[i3];
      if (i4 < n) sums[sc_p + is + 6] += q4 * xq->qs[i4];
    }
  }
  int32_t acc = 0;
  for (int j = 0; j < 16; j++) acc += (int32_t)(int8_t)sc[j] * sums[j];
  return d * xq->d * (float)acc;
}

/* src/ops/quant.rs:904-926 */
int or_integer_dot_q4k(const float* x, const uint8_t* w, size_t nbytes, size_t n, float* out) {
  if (nbytes % 144) return OR_ERR_INTERNAL;
  if (n == 0) { *out = 0.0f; return OR_OK; }
  size_t ns = nbytes / 144, np = 0;
  float* parts = (float*)malloc((ns ? ns : 1) * sizeof(float));
  or_q8block xq;
  for (size_t b = 0; b < ns; b++) {
    size_t base = b * 256;
    if (base >= n) break;
    size_t avail = n - base < 256 ? n - base : 256;
    or_quantize_block_q8(x + base, avail, &xq);
    parts[np++] = or_dot_q4k_q8_block(w + b * 144, &xq, avail);
  }
  *out = or_fixed_tree(parts, np);
  free(parts);
  return OR_OK;
}

/* Shared body of canonical_dot_q4k_fused (:616-702) and canonical_dot_q6k_fused
 * (:1212-1300): 8-lane chains continue across superblocks; a chunk closes every
 * 32 superblocks or at the row end. */
static int canonical_fused(const float* x, const uint8_t* w, size_t nbytes, size_t n,
                           int is_q6, float* out) {
  size_t bb = is_q6 ? 210 : 144;
  if (nbytes % bb) return OR_ERR_INTERNAL;
  if (n == 0) { *out = 0.0f; return OR_OK; }
  size_t ns = nbytes / bb;
  if (is_q6 && ns * 256 < n) return OR_ERR_INTERNAL;
  size_t spc = CANON_CHUNK / 256, nch = 0;
  float* chunk_sums = (float*)malloc((ns / spc + 2) * sizeof(float));
  float lanes[CANON_LANES] = {0};
  float buf[256];
  for (size_t b = 0; b < ns; b++) {
    size_t base = b * 256;
    if (base >= n) break;
    if (is_q6) dequant_q6k_block(w + b * bb, buf);
    else or_dequantize_q4_k(w + b * bb, 144, buf);
    size_t avail = n - base < 256 ? n - base : 256;
    size_t full = avail - avail % CANON_LANES;
    for (size_t i = 0; i < full; i += CANON_LANES)
      for (int j = 0; j < CANON_LANES; j++) {
        float p = x[base + i + j] * buf[i + j];
        lanes[j] += p;
      }
    for (size_t t = full; t < avail; t++) {
      float p = x[base + t] * buf[t];
      lanes[t % CANON_LANES] += p;
    }
    int is_last = base + avail >= n;
    if ((b + 1) % spc == 0 || is_last) {
      float l[CANON_LANES];
      memcpy(l, lanes, sizeof(l));
      chunk_sums[nch++] = or_fixed_tree(l, CANON_LANES);
      memset(lanes, 0, sizeof(lanes));
    }
  }
  *out = or_fixed_tree(chunk_sums, nch);
  free(chunk_sums);
  return OR_OK;
}

int or_canonical_dot_q4k_fused(const float* x, const uint8_t* w, size_t nbytes, size_t n,
                               float* out) {
  return canonical_fused(x, w, nbytes, n, 0, out);
}
int or_canonical_dot_q6k_fused(const float* x, const uint8_t* w, size_t nbytes, size_t n,
                               float* out) {
  return canonical_fused(x, w, nbytes, n, 1, out);
}

/* ------------------------------------------------------------------------ */
/* Row kernels shared by the serial and the row-parallel linears.           */

typedef struct {
  int kind; /* 0 q4k int, 1 q6k int, 2 q4k fused, 3 q6k fused, 4 f32 rows (canonical),
               5 q8_0 rows, 6 q5_0 rows */
  const float* x;
  const uint8_t* w;
  const or_q8block* xq;
  size_t in, row_bytes, n_super;
} row_job;

static float run_row(const row_job* j, size_t r, float* scratch) {
  const uint8_t* wr = j->w + r * j->row_bytes;
  float v = 0.0f;
  switch (j->kind) {
    case 0:
      for (size_t s = 0; s < j->n_super; s++)
        scratch[s] = or_dot_q4k_q8_block(wr + s * 144, &j->xq[s], 256);
      return or_fixed_tree(scratch, j->n_super);
    case 1:
      for (size_t s = 0; s < j->n_super; s++)
        scratch[s] = or_dot_q6k_q8_block(wr + s * 210, &j->xq[s], 256);
      return or_fixed_tree(scratch, j->n_super);
    case 2:
      canonical_fused(j->x, wr, j->row_bytes, j->in, 0, &v);
      return v;
    case 3:
      canonical_fused(j->x, wr, j->row_bytes, j->in, 1, &v);
      return v;
    case 4:
      return or_canonical_dot(j->x, (const float*)j->w + r * j->in, j->in);
    case 5:
      or_dequantize_q8_0(wr, j->row_bytes, scratch);
      return or_canonical_dot(j->x, scratch, j->in);
    case 6:
      or_dequantize_q5_0(wr, j->row_bytes, scratch);
      return or_canonical_dot(j->x, scratch, j->in);
  }
  return 0.0f;
}

typedef struct {
  const row_job* job;
  float* y;
  size_t out, grain, n_tasks;
  size_t next; /* atomically incremented task index */
  size_t scratch_len;
} pool_state;

static void* pool_worker(void* arg) {
  pool_state* ps = (pool_state*)arg;
  float* scratch = (float*)malloc(ps->scratch_len * sizeof(float));
  for (;;) {
    size_t t = __atomic_fetch_add(&ps->next, 1, __ATOMIC_RELAXED);
    if (t >= ps->n_tasks) break;
    size_t r0 = t * ps->grain, r1 = r0 + ps->grain < ps->out ? r0 + ps->grain : ps->out;
    for (size_t r = r0; r < r1; r++) ps->y[r] = run_row(ps->job, r, scratch);
  }
  free(scratch);
  return NULL;
}

/* One batch row of a linear: serial (threads<=1) or rayon-style chunks of
 * `grain` rows handed to a pool (src/ops/quant.rs:1121,1171). */
static void run_rows(const row_job* job, float* y, size_t out, size_t threads) {
  size_t scratch_len = job->in > job->n_super ? job->in : job->n_super;
  if (scratch_len == 0) scratch_len = 1;
  if (threads <= 1) {
    float* scratch = (float*)malloc(scratch_len * sizeof(float));
    for (size_t r = 0; r < out; r++) y[r] = run_row(job, r, scratch);
    free(scratch);
    return;
  }
  size_t grain = (out + threads * 4 - 1) / (threads * 4);
  if (grain < 1) grain = 1;
  pool_state ps = {job, y, out, grain, (out + grain - 1) / grain, 0, scratch_len};
  pthread_t th[256];
  size_t nt = threads > 256 ? 256 : threads;
  for (size_t i = 0; i < nt; i++) pthread_create(&th[i], NULL, pool_worker, &ps);
  for (size_t i = 0; i < nt; i++) pthread_join(th[i], NULL);
}

static int linear_int(int is_q6, const float* x, const uint8_t* w, size_t wlen, float* y,
                      size_t batch, size_t in, size_t out, size_t threads) {
  size_t bb = is_q6 ? 210 : 144;
  if (in % 256) return OR_ERR_INTERNAL;
  size_t row_bytes = (in / 256) * bb, ns = in / 256;
  if (wlen < out * row_bytes) return OR_ERR_INTERNAL;
  or_q8block* xq = (or_q8block*)malloc((ns ? ns : 1) * sizeof(or_q8block));
  for (size_t b = 0; b < batch; b++) {
    const float* xr = x + b * in;
    for (size_t s = 0; s < ns; s++) or_quantize_block_q8(xr + s * 256, 256, &xq[s]);
    row_job job = {is_q6 ? 1 : 0, xr, w, xq, in, row_bytes, ns};
    run_rows(&job, y + b * out, out, threads);
  }
  free(xq);
  return OR_OK;
}

int or_linear_q4_k_integer(const float* x, const uint8_t* w, size_t wlen, float* y,
                           size_t batch, size_t in, size_t out) {
  return linear_int(0, x, w, wlen, y, batch, in, out, 1);
}
int or_linear_q6_k_integer(const float* x, const uint8_t* w, size_t wlen, float* y,
                           size_t batch, size_t in, size_t out) {
  return linear_int(1, x, w, wlen, y, batch, in, out, 1);
}
int or_linear_q4_k_integer_parallel(const float* x, const uint8_t* w, size_t wlen, float* y,
                                    size_t batch, size_t in, size_t out, size_t threads) {
  return linear_int(0, x, w, wlen, y, batch, in, out, threads);
}
int or_linear_q6_k_integer_parallel(const float* x, const uint8_t* w, size_t wlen, float* y,
                                    size_t batch, size_t in, size_t out, size_t threads) {
  return linear_int(1, x, w, wlen, y, batch, in, out, threads);
}

static int linear_fused(int is_q6, const float* x, const uint8_t* w, size_t wlen, float* y,
                        size_t batch, size_t in, size_t out, size_t threads) {
  size_t bb = is_q6 ? 210 : 144;
  if (in % 256) return OR_ERR_INTERNAL;
  size_t row_bytes = (in / 256) * bb;
  if (is_q6 && wlen < out * row_bytes) return OR_ERR_INTERNAL;
  (void)wlen;
  for (size_t b = 0; b < batch; b++) {
    row_job job = {is_q6 ? 3 : 2, x + b * in, w, NULL, in, row_bytes, in / 256};
    run_rows(&job, y + b * out, out, threads);
  }
  return OR_OK;
}

int or_linear_q4_k_fused(const float* x, const uint8_t* w, size_t wlen, float* y, size_t batch,
                         size_t in, size_t out) {
  return linear_fused(0, x, w, wlen, y, batch, in, out, 1);
}
int or_linear_q4_k_fused_parallel(const float* x, const uint8_t* w, size_t wlen, float* y,
                                  size_t batch, size_t in, size_t out, size_t threads) {
  if (in % 256) return OR_ERR_INTERNAL;
  if (wlen < out * (in / 256) * 144) return OR_ERR_INTERNAL;
  return linear_fused(0, x, w, wlen, y, batch, in, out, threads);
}
int or_linear_q6_k_fused(const float* x, const uint8_t* w, size_t wlen, float* y, size_t batch,
                         size_t in, size_t out) {
  return linear_fused(1, x, w, wlen, y, batch, in, out, 1);
}

/* Dequantize the whole matrix, then canonical_dot per (b, o):
 * linear_q4_k_cpu :1456, linear_q6_k_cpu :1485, linear_q4_0_cpu :1529. */
static int linear_dequant_all(int dtype, const float* x, const uint8_t* w, size_t wlen,
                              float* y, size_t batch, size_t in, size_t out) {
  size_t nel = out * in;
  float* wf = (float*)malloc((nel ? nel : 1) * sizeof(float));
  int st;
  size_t expect;
  if (dtype == OR_Q4_0) {
    if (in % 32) { free(wf); return OR_ERR_INTERNAL; }
    expect = out * (in / 32) * 18;
    if (wlen != expect) { free(wf); return OR_ERR_INTERNAL; }
    st = or_dequantize_q4_0(w, wlen, wf);
  } else {
    size_t bb = dtype == OR_Q4_K ? 144 : 210;
    if (wlen % bb || (wlen / bb) * 256 != out * in) { free(wf); return OR_ERR_INTERNAL; }
    st = dtype == OR_Q4_K ? or_dequantize_q4_k(w, wlen, wf) : or_dequantize_q6_k(w, wlen, wf);
  }
  if (st) { free(wf); return st; }
  for (size_t b = 0; b < batch; b++)
    for (size_t o = 0; o < out; o++) y[b * out + o] = or_canonical_dot(x + b * in, wf + o * in, in);
  free(wf);
  return OR_OK;
}

int or_linear_q4_k_cpu(const float* x, const uint8_t* w, size_t wlen, float* y, size_t batch,
                       size_t in, size_t out) {
  return linear_dequant_all(OR_Q4_K, x, w, wlen, y, batch, in, out);
}
int or_linear_q6_k_cpu(const float* x, const uint8_t* w, size_t wlen, float* y, size_t batch,
                       size_t in, size_t out) {
  return linear_dequant_all(OR_Q6_K, x, w, wlen, y, batch, in, out);
}
int or_linear_q4_0_cpu(const float* x, const uint8_t* w, size_t wlen, float* y, size_t batch,
                       size_t in, size_t out) {
  return linear_dequant_all(OR_Q4_0, x, w, wlen, y, batch, in, out);
}

/* src/model/forward_quantized.rs:663-785 */
int or_linear_dispatch(int dtype, const float* x, const uint8_t* w, size_t wlen, size_t in,
                       size_t out, float* y, int q4k_float_mode, size_t threads) {
  const size_t PAR_MIN_ROWS = 512;
  size_t t = (out >= PAR_MIN_ROWS) ? threads : 1;
  switch (dtype) {
    case OR_Q4_0:
      return or_linear_q4_0_cpu(x, w, wlen, y, 1, in, out);
    case OR_F32: {
      if (wlen != out * in * 4) return OR_ERR_INTERNAL;
      row_job job = {4, x, w, NULL, in, in * 4, 0};
      run_rows(&job, y, out, threads);
      return OR_OK;
    }
    case OR_Q4_K:
      if (q4k_float_mode) return linear_fused(0, x, w, wlen, y, 1, in, out, 1);
      return linear_int(0, x, w, wlen, y, 1, in, out, t);
    case OR_Q6_K:
      return linear_int(1, x, w, wlen, y, 1, in, out, t);
    case OR_Q8_0:
    case OR_Q5_0: {
      size_t bb = dtype == OR_Q8_0 ? 34 : 22;
      if (in % 32) return OR_ERR_INTERNAL;
      size_t rb = (in / 32) * bb;
      if (wlen < out * rb) return OR_ERR_INTERNAL;
      row_job job = {dtype == OR_Q8_0 ? 5 : 6, x, w, NULL, in, rb, 0};
      run_rows(&job, y, out, threads);
      return OR_OK;
    }
    default:
      return OR_ERR_NOT_IMPLEMENTED;
  }
}

/* src/ops/rms_norm.rs:94-108 (sqrtf is correctly rounded in every IEEE libm). */
void or_rms_norm(const float* x, const float* w, size_t n, float eps, float* out) {
  float sumsq = 0.0f;
  for (size_t i = 0; i < n; i++) sumsq += x[i] * x[i];
  float mean = sumsq / (float)n;
  float scale = 1.0f / sqrtf(mean + eps);
  for (size_t i = 0; i < n; i++) out[i] = x[i] * scale * w[i];
}

/* src/ops/argmax.rs:49-60 */
uint32_t or_argmax(const float* x, size_t n) {
  size_t best = 0;
  float bv = x[0];
  for (size_t i = 1; i < n; i++)
    if (x[i] > bv) { bv = x[i]; best = i; }
  return (uint32_t)best;
}

/* src/ops/quant.rs:1856-1865: a then b from one LCG stream. */
void or_lcg_pair(size_t n, float* a, float* b) {
  uint64_t s = 0x1234;
  for (size_t k = 0; k < 2 * n; k++) {
    s = s * 6364136223846793005ULL + 1ULL;
    float v = ((float)(uint32_t)(s >> 33) / 2147483648.0f) * 2.0f - 1.0f;
    if (k < n) a[k] = v; else b[k - n] = v;
  }
}

/* src/ops/matmul.rs:159-195 (matmul :106-128 delegates to canonical_dot). */
uint64_t or_matmul_fnv_golden(void) {
  enum { M = 4, K = 64, N = 4 };
  float a[M * K], b[K * N], col[K], outv[M * N];
  uint64_t s = 0x1234;
  for (int k = 0; k < M * K + K * N; k++) {
    s = s * 6364136223846793005ULL + 1ULL;
    float v = ((float)(uint32_t)(s >> 33) / (float)(1u << 31)) * 2.0f - 1.0f;
    if (k < M * K) a[k] = v; else b[k - M * K] = v;
  }
  for (int j = 0; j < N; j++) {
    for (int kk = 0; kk < K; kk++) col[kk] = b[kk * N + j];
    for (int i = 0; i < M; i++) outv[i * N + j] = or_canonical_dot(a + i * K, col, K);
  }
  uint64_t h = 0xcbf29ce484222325ULL;
  for (int i = 0; i < M * N; i++) {
    uint32_t bits;
    memcpy(&bits, &outv[i], 4);
    for (int byte = 0; byte < 4; byte++) {
      h ^= (bits >> (8 * byte)) & 0xFFu;
      h *= 0x00000100000001b3ULL;
    }
  }
  return h;
}
