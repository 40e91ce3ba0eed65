// kq_core.cuh -- device building blocks of the exact-integer k-quant matvec,
// shared by the standalone matvec kernel (kquant_matvec.cu) and the
// persistent decode kernel (decode_mk.cu): the launch descriptor, activation
// quantisation (quantize_block_q8, src/ops/quant.rs:750-771), the Q4_K / Q6_K
// superblock dots (quant.rs:850-898, :996-1057), the cross-superblock
// fixed_tree (quant.rs:462-476) and one warp pass over a stage of rows.
#pragma once
#include <cuda_fp16.h>

#include "exact_sum.cuh"
#include "vtq_device.cuh"
#include "vtq_internal.h"
#include "vtq_libm.h"

namespace vtq {
namespace {

constexpr int KQ_NST_MAX = 16;                   // ring depth
constexpr int KQ_SMAX = 128;                     // superblocks per row (in_feat <= 32768)
constexpr int XQ_STRIDE = 272;                   // padded bytes per quantised activation block
// Activation-sum records per block, padded by 4 ints so that 8 lanes reading
// 8 consecutive blocks' records hit 8 different groups of 4 banks.
template <int NB> struct BsumStride { static constexpr int v = NB + 4; };
constexpr uint32_t FULL = 0xffffffffu;


constexpr uint32_t kScaleOff = 448;  // inside the 512-byte head, above the barriers

struct KqParams {
  const float* x;
  int64_t ldx;
  int batch, n, S;
  const uint8_t* W;
  int64_t pitch;
  int R;
  int rows_base, rows_rem;  // CTA b owns rows_base (+1 if b < rows_rem) rows
  float* y;
  int64_t ldy;
  int rps;                  // rows per stage (multiple of rows per warp pass)
  int nst;                  // ring depth
  uint32_t stage_bytes;     // rps * pitch
  int lpr;                  // lanes per row segment (power of two, <= 32)
  int x_smem;               // x rows fetched by TMA into off_xf
  uint32_t off_xd, off_bsum, off_xq, off_xf, off_stage;
  unsigned* status;
  GatherTarget g;           // g.world > 0: fused all-gather of y to every rank
  KqXform xf;               // activation transform (batch 1; kind 2 needs x_smem)
  uint32_t off_ystage;      // gather: this CTA's finished rows [batch][rows_base + 1]
  uint32_t off_xsq;         // kind 2: squares of v (n floats)
  int epi;                  // 1: rows come in (gate, up) pairs; y[b, r / 2] = silu(gate) * up
};

// quantize_block_q8 (quant.rs:750-771) of one 256-element block held by a
// warp (8 contiguous values per lane): the block's int8 codes (8 per lane) go
// to xqb, its scale d to *xdp (lane 0) and its activation sums -- NB = 8: one
// per 32 elements (Q4_K's bsums), NB = 16: one per 16 (the Q6_K -32 offset
// term) -- to bs[0..NB). Shared or global destinations.
template <int NB>
__device__ __forceinline__ void quant_block(const float (&v)[8], int lane, int8_t* xqb, int* bs,
                                            float* xdp) {
  // amax = max over non-NaN |v|, starting at +0.0 (quant.rs:752-758).
  uint32_t am = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const uint32_t bits = __float_as_uint(v[i]) & 0x7fffffffu;
    if (bits <= 0x7f800000u) am = max(am, bits);
  }
  am = __reduce_max_sync(FULL, am);
  const float d = __fdiv_rn(__uint_as_float(am), 127.0f);
  const float inv = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
  int sum = 0;
  uint32_t w0 = 0, w1 = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int q = q8_round(__fmul_rn(v[i], inv));
    sum += q;
    if (i < 4) w0 |= (uint32_t)(q & 0xff) << (8 * i);
    else w1 |= (uint32_t)(q & 0xff) << (8 * (i - 4));
  }
  const int s16 = sum + __shfl_xor_sync(FULL, sum, 1);
  const int s32 = s16 + __shfl_xor_sync(FULL, s16, 2);
  if (NB == 8) {
    if ((lane & 3) == 0) bs[lane >> 2] = s32;
  } else {
    if ((lane & 1) == 0) bs[lane >> 1] = s16;
  }
  *reinterpret_cast<uint2*>(xqb + lane * 8) = make_uint2(w0, w1);
  if (lane == 0) *xdp = d;
}

// quantize_block_q8 for every (batch row, superblock): one warp per block,
// 8 contiguous elements per lane. NB = 8 (sums per 32: Q4_K's bsums) or 16
// (sums per 16: the Q6_K -32 offset term). `xs` is the activation source:
// the TMA-staged rows in shared memory (row stride n) or global x (ldx).
// CG: load x at L2 (ld.global.cg), for rows written by other CTAs of the
// same launch (read after an acquire of their completion counter).
template <int NB, int CW, bool CG = false>
__device__ __forceinline__ void quantize_x(const KqParams& p, const float* xs, int64_t lds,
                                           int warp, int lane, float* xd, int* bsum, int8_t* xq,
                                           float xscale) {
  const int nblk = p.batch * p.S;
  for (int u = warp; u < nblk; u += CW) {
    const int b = u / p.S, s = u - b * p.S;
    const float* src = xs + (int64_t)b * lds + s * 256 + lane * 8;
    float v[8];
    if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
      const float4 a = CG ? __ldcg(reinterpret_cast<const float4*>(src))
                          : *reinterpret_cast<const float4*>(src);
      const float4 c = CG ? __ldcg(reinterpret_cast<const float4*>(src) + 1)
                          : *(reinterpret_cast<const float4*>(src) + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; i++) v[i] = CG ? __ldcg(src + i) : src[i];
    }
    if (p.xf.kind == 2) {  // RMSNorm output (v already holds x + delta)
      const float* nw = p.xf.nw + s * 256 + lane * 8;
#pragma unroll
      for (int i = 0; i < 8; i++) v[i] = __fmul_rn(__fmul_rn(v[i], xscale), nw[i]);
    }
    const int blk = b * p.S + s;
    quant_block<NB>(v, lane, xq + blk * XQ_STRIDE, bsum + blk * BsumStride<NB>::v, xd + blk);
  }
}

// dp4a, signed x signed bytes.
__device__ __forceinline__ int dot_ss(uint4 q, int4 x) {
  int a = __dp4a((int)q.x, x.x, 0);
  int b = __dp4a((int)q.y, x.y, 0);
  a = __dp4a((int)q.z, x.z, a);
  b = __dp4a((int)q.w, x.w, b);
  return a + b;
}

// dp4a, unsigned bytes of q x signed bytes of x.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dot_us(uint4 q, int4 x) {
  int a = dp4a_us(q.x, x.x, 0);
  int b = dp4a_us(q.y, x.y, 0);
  a = dp4a_us(q.z, x.z, a);
  b = dp4a_us(q.w, x.w, b);
  return a + b;
}

__device__ __forceinline__ uint4 mask4(uint4 v, uint32_t m) {
  return make_uint4(v.x & m, v.y & m, v.z & m, v.w & m);
}

__device__ __forceinline__ int4 lds_i4(const int8_t* p) { return *reinterpret_cast<const int4*>(p); }
__device__ __forceinline__ uint4 lds_u4(const uint8_t* p) {
  return *reinterpret_cast<const uint4*>(p);
}

// binary16 -> binary32 through the hardware convert: exact for every finite
// value and infinity (subnormal halves are normal floats). Only a NaN's
// payload may differ from the reference's bit-level decode; NaN payloads are
// outside the bit-identity contract (quant.rs:2033-2044).
__device__ __forceinline__ float h2f(uint32_t bits) {
  return __half2float(__ushort_as_half((unsigned short)bits));
}

// One Q4_K superblock (raw GGUF layout, 144 B, 16-byte aligned in shared
// memory) against the quantised activation block s of every batch row.
// part[b] = d * xd * acc - dmin * xd * acc_m   (quant.rs:850-898)
// High nibbles are dotted in place (q & 0xF0 = 16 * nibble) and the exact
// sum is divided by 16 afterwards.
template <int MAXB>
__device__ __forceinline__ void q4k_superblock(const uint8_t* sb, int s, const KqParams& p,
                                               const int8_t* xq, const float* xd, const int* bsum,
                                               float* part) {
  const uint4 hdr = lds_u4(sb);  // d | dmin, scales[0..12)
  // get_scale_min_k4 (quant.rs:268-276) for all 8 sub-blocks.
  int sc[8], mn[8];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    sc[j] = (hdr.y >> (8 * j)) & 63;
    mn[j] = (hdr.z >> (8 * j)) & 63;
    const uint32_t lo4 = (hdr.w >> (8 * j)) & 0xff;
    sc[j + 4] = (lo4 & 15) | (((hdr.y >> (8 * j + 6)) & 3) << 4);
    mn[j + 4] = (lo4 >> 4) | (((hdr.z >> (8 * j + 6)) & 3) << 4);
  }
  int acc[MAXB];
#pragma unroll
  for (int b = 0; b < MAXB; b++) acc[b] = 0;
#pragma unroll
  for (int it = 0; it < 4; it++) {
    const uint4 qa = lds_u4(sb + 16 + 32 * it), qb = lds_u4(sb + 32 + 32 * it);
    const uint4 la = mask4(qa, 0x0F0F0F0Fu), lb = mask4(qb, 0x0F0F0F0Fu);
    const uint4 ha = mask4(qa, 0xF0F0F0F0u), hb = mask4(qb, 0xF0F0F0F0u);
#pragma unroll
    for (int b = 0; b < MAXB; b++) {
      if (b < p.batch) {
        const int8_t* xb = xq + (b * p.S + s) * XQ_STRIDE + 64 * it;
        const int s_lo = dot_ss(la, lds_i4(xb)) + dot_ss(lb, lds_i4(xb + 16));
        const int s_hi16 = dot_us(ha, lds_i4(xb + 32)) + dot_us(hb, lds_i4(xb + 48));
        acc[b] += sc[2 * it] * s_lo + sc[2 * it + 1] * (s_hi16 >> 4);
      }
    }
  }
  const float d = h2f(hdr.x & 0xffffu), dmin = h2f(hdr.x >> 16);
#pragma unroll
  for (int b = 0; b < MAXB; b++) {
    if (b < p.batch) {
      const int blk = b * p.S + s;
      const int4 b0 = *reinterpret_cast<const int4*>(bsum + blk * BsumStride<8>::v);
      const int4 b1 = *reinterpret_cast<const int4*>(bsum + blk * BsumStride<8>::v + 4);
      const int accm = mn[0] * b0.x + mn[1] * b0.y + mn[2] * b0.z + mn[3] * b0.w +
                       mn[4] * b1.x + mn[5] * b1.y + mn[6] * b1.z + mn[7] * b1.w;
      const float xdv = xd[blk];
      const float t0 = __fmul_rn(__fmul_rn(d, xdv), __int2float_rn(acc[b]));
      const float t1 = __fmul_rn(__fmul_rn(dmin, xdv), __int2float_rn(accm));
      part[b] = __fsub_rn(t0, t1);
    }
  }
}

// Sign-extended byte k of w.
__device__ __forceinline__ int sbyte(uint32_t w, int k) {
  return ((int)(w << (24 - 8 * k))) >> 24;
}

// One Q6_K superblock in the device layout (repack.cu): within a group of G
// superblocks, ql chunk k (16 B) of superblock i is at 16 (G k + i), qh chunk k
// at 128 G + 16 (G k + i), scales at 192 G + 16 i, d at 208 G + 2 i.
// dp4a runs on the unsigned 6-bit codes; the -32 offset is applied exactly via
// the per-16 activation sums: sum((q - 32) x) = sum(q x) - 32 sum(x).
// part[b] = d * xd * acc   (quant.rs:996-1057)
template <int MAXB>
__device__ __forceinline__ void q6k_superblock(const uint8_t* gb, int G, int i, int s,
                                               const KqParams& p, const int8_t* xq,
                                               const float* xd, const int* bsum, float* part) {
  const uint4 scw = lds_u4(gb + 192 * G + 16 * i);
  const float d = h2f(*reinterpret_cast<const uint16_t*>(gb + 208 * G + 2 * i));
  const uint32_t scv[4] = {scw.x, scw.y, scw.z, scw.w};
  int sc[16];
#pragma unroll
  for (int j = 0; j < 16; j++) sc[j] = sbyte(scv[j >> 2], j & 3);
  int acc[MAXB];
#pragma unroll
  for (int b = 0; b < MAXB; b++) acc[b] = 0;
#pragma unroll
  for (int h = 0; h < 2; h++) {
#pragma unroll
    for (int hc = 0; hc < 2; hc++) {  // l in [16 hc, 16 hc + 16)
      const uint4 A = lds_u4(gb + 16 * (G * (4 * h + hc) + i));      // ql[64h + l]
      const uint4 B = lds_u4(gb + 16 * (G * (4 * h + 2 + hc) + i));  // ql[64h + 32 + l]
      const uint4 H = lds_u4(gb + 128 * G + 16 * (G * (2 * h + hc) + i));  // qh[32h + l]
      const uint4 q1 = make_uint4((A.x & 0x0F0F0F0Fu) | ((H.x & 0x03030303u) << 4),
                                  (A.y & 0x0F0F0F0Fu) | ((H.y & 0x03030303u) << 4),
                                  (A.z & 0x0F0F0F0Fu) | ((H.z & 0x03030303u) << 4),
                                  (A.w & 0x0F0F0F0Fu) | ((H.w & 0x03030303u) << 4));
      const uint4 q2 = make_uint4((B.x & 0x0F0F0F0Fu) | ((H.x & 0x0C0C0C0Cu) << 2),
                                  (B.y & 0x0F0F0F0Fu) | ((H.y & 0x0C0C0C0Cu) << 2),
                                  (B.z & 0x0F0F0F0Fu) | ((H.z & 0x0C0C0C0Cu) << 2),
                                  (B.w & 0x0F0F0F0Fu) | ((H.w & 0x0C0C0C0Cu) << 2));
      const uint4 q3 = make_uint4(((A.x >> 4) & 0x0F0F0F0Fu) | (H.x & 0x30303030u),
                                  ((A.y >> 4) & 0x0F0F0F0Fu) | (H.y & 0x30303030u),
                                  ((A.z >> 4) & 0x0F0F0F0Fu) | (H.z & 0x30303030u),
                                  ((A.w >> 4) & 0x0F0F0F0Fu) | (H.w & 0x30303030u));
      const uint4 q4 = make_uint4(((B.x >> 4) & 0x0F0F0F0Fu) | ((H.x >> 2) & 0x30303030u),
                                  ((B.y >> 4) & 0x0F0F0F0Fu) | ((H.y >> 2) & 0x30303030u),
                                  ((B.z >> 4) & 0x0F0F0F0Fu) | ((H.z >> 2) & 0x30303030u),
                                  ((B.w >> 4) & 0x0F0F0F0Fu) | ((H.w >> 2) & 0x30303030u));
      const int j = 8 * h + hc;  // scale bucket of q1; q2 +2, q3 +4, q4 +6
#pragma unroll
      for (int b = 0; b < MAXB; b++) {
        if (b < p.batch) {
          const int8_t* xb = xq + (b * p.S + s) * XQ_STRIDE + 128 * h + 16 * hc;
          acc[b] += sc[j] * dot_ss(q1, lds_i4(xb)) + sc[j + 2] * dot_ss(q2, lds_i4(xb + 32)) +
                    sc[j + 4] * dot_ss(q3, lds_i4(xb + 64)) +
                    sc[j + 6] * dot_ss(q4, lds_i4(xb + 96));
        }
      }
    }
  }
#pragma unroll
  for (int b = 0; b < MAXB; b++) {
    if (b < p.batch) {
      const int blk = b * p.S + s;
      int cor = 0;  // sum_j sc_j * (sum of the 16 activations of bucket j)
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const int4 bs = *reinterpret_cast<const int4*>(bsum + blk * BsumStride<16>::v + 4 * q);
        cor += sc[4 * q] * bs.x + sc[4 * q + 1] * bs.y + sc[4 * q + 2] * bs.z + sc[4 * q + 3] * bs.w;
      }
      const int total = acc[b] - 32 * cor;
      part[b] = __fmul_rn(__fmul_rn(d, xd[blk]), __int2float_rn(total));
    }
  }
}

// fixed_tree (quant.rs:462-476) over the `len` values of one row held by a
// segment of `lpr` lanes (value i on segment lane i % lpr, chunk i / lpr).
// Stride-doubling: index i (a multiple of 2^(k+1)) adds index i + 2^k when
// that index is < len -- the same additions as the reference's level-wise
// loop. Strides below lpr pair lanes of one chunk (shuffles); strides from
// lpr up pair whole chunks, whose sums sit on segment lane 0.
template <int NCH>
__device__ __forceinline__ float seg_fixed_tree(float (&v)[NCH], int sl, int lpr, int len) {
  for (int st = 1; st < lpr; st <<= 1) {
#pragma unroll
    for (int c = 0; c < NCH; c++) {
      const float o = __shfl_down_sync(FULL, v[c], st);
      if ((sl & (2 * st - 1)) == 0 && c * lpr + sl + st < len) v[c] = __fadd_rn(v[c], o);
    }
  }
#pragma unroll
  for (int st = 1; st < NCH; st <<= 1) {
#pragma unroll
    for (int c = 0; c + st < NCH; c += 2 * st)
      if ((c + st) * lpr < len) v[c] = __fadd_rn(v[c], v[c + st]);
  }
  return v[0];  // valid on segment lane 0
}

// One warp pass: rows rr0 + seg of the stage buffer.
template <int QT, int MAXB, int NCH>
__device__ __forceinline__ void consume_pass(const KqParams& p, const uint8_t* sbuf, int rr,
                                             bool row_ok, int sl, int64_t yrow,
                                             const int8_t* xq, const float* xd, const int* bsum,
                                             float* ystage, int64_t ycta0) {
  float part[NCH][MAXB];
#pragma unroll
  for (int c = 0; c < NCH; c++) {
    const int s = c * p.lpr + sl;
#pragma unroll
    for (int b = 0; b < MAXB; b++) part[c][b] = 0.0f;
    if (row_ok && s < p.S) {
      const uint8_t* row = sbuf + (int64_t)rr * p.pitch;
      if (QT == 0) {
        q4k_superblock<MAXB>(row + s * 144, s, p, xq, xd, bsum, part[c]);
      } else {
        const int gi = s >> 3;
        q6k_superblock<MAXB>(row + gi * 1680, min(8, p.S - 8 * gi), s & 7, s, p, xq, xd, bsum,
                             part[c]);
      }
    }
  }
#pragma unroll
  for (int b = 0; b < MAXB; b++) {
    if (b < p.batch) {
      float v[NCH];
#pragma unroll
      for (int c = 0; c < NCH; c++) v[c] = part[c][b];
      const float t = seg_fixed_tree<NCH>(v, sl, p.lpr, p.S);
      if (p.epi) {
        // SwiGLU of the pair, silu(g) * up with silu = g / (1 + expf(-g))
        // (forward_quantized.rs:556-561): the up row is the next segment of
        // this warp pass (pairs start on even rows; a pass holds an even
        // number of rows).
        const float up = __shfl_down_sync(0xffffffffu, t, p.lpr);
        if (row_ok && sl == 0 && (yrow & 1) == 0) {
          const float silu = __fdiv_rn(t, __fadd_rn(1.0f, libm::expf(-t)));
          p.y[(int64_t)b * p.ldy + (yrow >> 1)] = __fmul_rn(silu, up);
        }
      } else if (row_ok && sl == 0) {
        if (p.g.world == 0)
          p.y[(int64_t)b * p.ldy + yrow] = t;
        else  // row-sharded: stage; warp 0 sends the CTA's rows at the end
          ystage[b * (p.rows_base + 1) + (int)(yrow - ycta0)] = t;
      }
    }
  }
}

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}


}  // namespace
}  // namespace vtq
