// kquant_matvec.cu -- exact-integer Q4_K / Q6_K matvec for sm_100a.
//
// Computes, bit for bit, vitni-tensor's integer linears
//   linear_q4_k_integer(_parallel)  src/ops/quant.rs:936-980, :1149-1196
//   linear_q6_k_integer(_parallel)  src/ops/quant.rs:1060-1146
// y[b, r] = fixed_tree_s( blockdot(W[r, s], quantize_block_q8(x[b, 256s..])) ).
//
// Design (one persistent CTA per SM, 8 warps):
//  * Each CTA owns a contiguous range of output rows, i.e. one contiguous byte
//    range of the weight matrix in HBM. Thread 0 streams it into a shared-
//    memory ring with TMA bulk copies (cp.async.bulk + mbarrier complete_tx,
//    L2 evict-first) -- stages are whole rows, the ring is as deep as shared
//    memory allows, so small matrices are requested in full at kernel entry.
//  * While the first stages are in flight, every CTA quantises the activation
//    rows into shared memory (quantize_block_q8, quant.rs:750-771, restated
//    with __fdiv_rn/__fmul_rn/__fadd_rn and cvt.rzi; identical bits in every
//    CTA, so the reference's once-per-call quantisation is reproduced).
//  * 4 lanes cooperate on one superblock: each unpacks its quarter of the
//    packed quants with shifts/masks and forms exact int32 dots with dp4a.
//    Integer sums are exact, so the lane split and shuffle order are free.
//    Only the per-superblock fp combine (quant.rs:897 / :1056) and the
//    cross-superblock fixed_tree (quant.rs:462) are order-pinned; both run
//    with explicit round-to-nearest intrinsics (no FMA contraction) in the
//    reference's order.
//  * When a stage's rows are complete, one warp per (row, batch) reduces the
//    S superblock partials with a stride-doubling shuffle tree whose pairing
//    is identical to the reference's level-wise fixed_tree.
#include "vtq_device.cuh"
#include "vtq_internal.h"

namespace vtq {
namespace {

constexpr int KQ_WARPS = 8;
constexpr int KQ_THREADS = KQ_WARPS * 32;
constexpr int KQ_BMAX = 8;      // activation rows per launch
constexpr int KQ_NST_MAX = 8;   // ring depth
constexpr int KQ_SMAX = 128;    // superblocks per row (in_feat <= 32768)
constexpr uint32_t FULL = 0xffffffffu;

struct KqParams {
  const float* x;
  int64_t ldx;
  int batch, n, S;
  const uint8_t* W;
  int64_t pitch;
  int R;
  float* y;
  int64_t ldy;
  int rps;                 // rows per stage
  int nst;                 // ring depth
  uint32_t stage_bytes;    // rps * pitch
  uint32_t off_xd, off_bsum, off_part, off_xq, off_stage;
  unsigned* status;
};

// quantize_block_q8 for every (batch row, superblock): one warp per block,
// 8 contiguous elements per lane. NB = 8 (sums per 32, Q4_K's bsums) or 16
// (sums per 16, used for Q6_K's -32 offset).
template <int NB>
__device__ __forceinline__ void quantize_x(const KqParams& p, float* xd, int* bsum, int8_t* xq) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nblk = p.batch * p.S;
  for (int u = warp; u < nblk; u += KQ_WARPS) {
    const int b = u / p.S, s = u - b * p.S;
    const float* src = p.x + (int64_t)b * p.ldx + (int64_t)s * 256 + lane * 8;
    float v[8];
    if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(src));
      const float4 c = __ldg(reinterpret_cast<const float4*>(src) + 1);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
      v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; i++) v[i] = __ldg(src + i);
    }
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
    const int blk = b * p.S + s;
    if (NB == 8) {
      if ((lane & 3) == 0) bsum[blk * 8 + (lane >> 2)] = s32;
    } else {
      if ((lane & 1) == 0) bsum[blk * 16 + (lane >> 1)] = s16;
    }
    *reinterpret_cast<uint2*>(xq + (int64_t)b * p.n + s * 256 + lane * 8) = make_uint2(w0, w1);
    if (lane == 0) xd[blk] = d;
  }
}

// Q4_K: scales for sub-blocks 2h, 2h+1 (get_scale_min_k4, quant.rs:268-276).
__device__ __forceinline__ void q4k_scales(uint32_t w0, uint32_t w1, uint32_t w2, int h, int& sc0,
                                           int& sc1, int& m0, int& m1) {
  const int sh = (h & 1) * 16;
  const uint32_t a = w0 >> sh, m = w1 >> sh, hi = w2 >> sh;
  if (h < 2) {
    sc0 = a & 63; sc1 = (a >> 8) & 63;
    m0 = m & 63;  m1 = (m >> 8) & 63;
  } else {
    sc0 = (hi & 15) | (((a >> 6) & 3) << 4);
    sc1 = ((hi >> 8) & 15) | (((a >> 14) & 3) << 4);
    m0 = ((hi >> 4) & 15) | (((m >> 6) & 3) << 4);
    m1 = ((hi >> 12) & 15) | (((m >> 14) & 3) << 4);
  }
}

// One Q4_K superblock (raw GGUF layout, 144 B) against one activation block.
// Lane quarter h owns qs[32h..32h+32) = elements 64h..64h+64.
// Returns this lane's partial float (valid in the h == 0 lane only).
__device__ __forceinline__ void q4k_unit(const uint8_t* sb, int h, const KqParams& p,
                                         const int8_t* xq, const float* xd, const int* bsum,
                                         int s, float* out, int out_stride, bool valid) {
  const uint4 qa = *reinterpret_cast<const uint4*>(sb + 16 + 32 * h);
  const uint4 qb = *reinterpret_cast<const uint4*>(sb + 32 + 32 * h);
  const uint32_t qw[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
  const uint32_t sw0 = *reinterpret_cast<const uint32_t*>(sb + 4);
  const uint32_t sw1 = *reinterpret_cast<const uint32_t*>(sb + 8);
  const uint32_t sw2 = *reinterpret_cast<const uint32_t*>(sb + 12);
  const uint32_t dw = *reinterpret_cast<const uint32_t*>(sb);
  int sc0, sc1, m0, m1;
  q4k_scales(sw0, sw1, sw2, h, sc0, sc1, m0, m1);
  uint32_t lo[8], hi[8];
#pragma unroll
  for (int k = 0; k < 8; k++) {
    lo[k] = qw[k] & 0x0F0F0F0Fu;
    hi[k] = (qw[k] >> 4) & 0x0F0F0F0Fu;
  }
  const float d = f16_bits_to_f32(dw & 0xffffu), dmin = f16_bits_to_f32(dw >> 16);
  for (int b = 0; b < p.batch; b++) {
    const int8_t* xb = xq + (int64_t)b * p.n + s * 256 + 64 * h;
    const int4 x0 = *reinterpret_cast<const int4*>(xb);
    const int4 x1 = *reinterpret_cast<const int4*>(xb + 16);
    const int4 x2 = *reinterpret_cast<const int4*>(xb + 32);
    const int4 x3 = *reinterpret_cast<const int4*>(xb + 48);
    int s_lo = 0, s_hi = 0;
    s_lo = __dp4a((int)lo[0], x0.x, s_lo); s_lo = __dp4a((int)lo[1], x0.y, s_lo);
    s_lo = __dp4a((int)lo[2], x0.z, s_lo); s_lo = __dp4a((int)lo[3], x0.w, s_lo);
    s_lo = __dp4a((int)lo[4], x1.x, s_lo); s_lo = __dp4a((int)lo[5], x1.y, s_lo);
    s_lo = __dp4a((int)lo[6], x1.z, s_lo); s_lo = __dp4a((int)lo[7], x1.w, s_lo);
    s_hi = __dp4a((int)hi[0], x2.x, s_hi); s_hi = __dp4a((int)hi[1], x2.y, s_hi);
    s_hi = __dp4a((int)hi[2], x2.z, s_hi); s_hi = __dp4a((int)hi[3], x2.w, s_hi);
    s_hi = __dp4a((int)hi[4], x3.x, s_hi); s_hi = __dp4a((int)hi[5], x3.y, s_hi);
    s_hi = __dp4a((int)hi[6], x3.z, s_hi); s_hi = __dp4a((int)hi[7], x3.w, s_hi);
    const int blk = b * p.S + s;
    int acc = sc0 * s_lo + sc1 * s_hi;
    int accm = m0 * bsum[blk * 8 + 2 * h] + m1 * bsum[blk * 8 + 2 * h + 1];
    acc += __shfl_xor_sync(FULL, acc, 1);
    accm += __shfl_xor_sync(FULL, accm, 1);
    acc += __shfl_xor_sync(FULL, acc, 2);
    accm += __shfl_xor_sync(FULL, accm, 2);
    if (valid && h == 0) {
      // d * xq.d * acc as f32 - dmin * xq.d * acc_m as f32   (quant.rs:897)
      const float xdv = xd[blk];
      const float t0 = __fmul_rn(__fmul_rn(d, xdv), __int2float_rn(acc));
      const float t1 = __fmul_rn(__fmul_rn(dmin, xdv), __int2float_rn(accm));
      out[b * out_stride] = __fsub_rn(t0, t1);
    }
  }
}

__device__ __forceinline__ int sbyte(uint32_t w, int k) {  // sign-extended byte k
  return ((int)(w << (24 - 8 * k))) >> 24;
}

// One Q6_K superblock (device SoA-8 group layout, see repack.cu). Lane
// quarter j covers half h = j/2 and the 16-element runs l in [l0, l0+16),
// l0 = 16 (j & 1): scale buckets 8h + (j&1) + {0, 2, 4, 6} (quant.rs:996-1057).
// dp4a runs on the unsigned 6-bit codes; the -32 offset is applied exactly
// through the per-16 activation sums: sum((q-32) x) = sum(q x) - 32 sum(x).
__device__ __forceinline__ void q6k_unit(const uint8_t* row, int s, int j, const KqParams& p,
                                         const int8_t* xq, const float* xd, const int* bsum,
                                         float* out, int out_stride, bool valid) {
  const int h = j >> 1, odd = j & 1, l0 = odd * 16;
  const int gi = s >> 3, ii = s & 7;
  const int G = min(8, p.S - gi * 8);
  const uint8_t* gb = row + (int64_t)gi * 1680;
  const uint4 A = *reinterpret_cast<const uint4*>(gb + 128 * ii + 64 * h + l0);
  const uint4 B = *reinterpret_cast<const uint4*>(gb + 128 * ii + 64 * h + 32 + l0);
  const uint4 H = *reinterpret_cast<const uint4*>(gb + 128 * G + 64 * ii + 32 * h + l0);
  const uint2 SC = *reinterpret_cast<const uint2*>(gb + 192 * G + 16 * ii + 8 * h);
  const uint32_t dbits = *reinterpret_cast<const uint16_t*>(gb + 208 * G + 2 * ii);
  const int sc_t[4] = {sbyte(SC.x, odd), sbyte(SC.x, odd + 2), sbyte(SC.y, odd),
                       sbyte(SC.y, odd + 2)};
  const uint32_t a[4] = {A.x, A.y, A.z, A.w}, bb[4] = {B.x, B.y, B.z, B.w},
                 hh[4] = {H.x, H.y, H.z, H.w};
  uint32_t q[4][4];
#pragma unroll
  for (int k = 0; k < 4; k++) {
    q[0][k] = (a[k] & 0x0F0F0F0Fu) | ((hh[k] & 0x03030303u) << 4);
    q[1][k] = (bb[k] & 0x0F0F0F0Fu) | (((hh[k] >> 2) & 0x03030303u) << 4);
    q[2][k] = ((a[k] >> 4) & 0x0F0F0F0Fu) | (((hh[k] >> 4) & 0x03030303u) << 4);
    q[3][k] = ((bb[k] >> 4) & 0x0F0F0F0Fu) | (((hh[k] >> 6) & 0x03030303u) << 4);
  }
  const float d = f16_bits_to_f32(dbits);
  for (int b = 0; b < p.batch; b++) {
    const int blk = b * p.S + s;
    const int8_t* xb = xq + (int64_t)b * p.n + s * 256 + 128 * h + l0;
    int acc = 0;
#pragma unroll
    for (int t = 0; t < 4; t++) {
      const int4 xv = *reinterpret_cast<const int4*>(xb + 32 * t);
      int su = 0;
      su = __dp4a((int)q[t][0], xv.x, su);
      su = __dp4a((int)q[t][1], xv.y, su);
      su = __dp4a((int)q[t][2], xv.z, su);
      su = __dp4a((int)q[t][3], xv.w, su);
      const int bucket = 8 * h + odd + 2 * t;
      acc += sc_t[t] * (su - 32 * bsum[blk * 16 + bucket]);
    }
    acc += __shfl_xor_sync(FULL, acc, 1);
    acc += __shfl_xor_sync(FULL, acc, 2);
    if (valid && j == 0) {
      // d * xq.d * acc as f32   (quant.rs:1056)
      out[b * out_stride] = __fmul_rn(__fmul_rn(d, xd[blk]), __int2float_rn(acc));
    }
  }
}

// fixed_tree (quant.rs:462-476) over part[0..len), len <= 128, by one warp.
// Stride-doubling pairs index i with i + 2^k (i a multiple of 2^(k+1),
// i + 2^k < len) -- the same additions as the reference's level-wise loop.
__device__ __forceinline__ float warp_fixed_tree(const float* part, int stride, int len) {
  const int lane = threadIdx.x & 31;
  float v[4];
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const int i = c * 32 + lane;
    v[c] = (i < len) ? part[i * stride] : 0.0f;
  }
#pragma unroll
  for (int k = 0; k < 5; k++) {
    const int st = 1 << k;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const float o = __shfl_down_sync(FULL, v[c], st);
      if ((lane & (2 * st - 1)) == 0 && c * 32 + lane + st < len) v[c] = __fadd_rn(v[c], o);
    }
  }
  float r = v[0];
  if (lane == 0) {
    if (32 < len) r = __fadd_rn(r, v[1]);
    float r2 = v[2];
    if (96 < len) r2 = __fadd_rn(r2, v[3]);
    if (64 < len) r = __fadd_rn(r, r2);
  }
  return r;  // valid in lane 0
}

template <int QT>  // 0 = Q4_K, 1 = Q6_K
__global__ void __launch_bounds__(KQ_THREADS, 1) kq_matvec_kernel(const KqParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  float* xd = reinterpret_cast<float*>(smem + p.off_xd);
  int* bsum = reinterpret_cast<int*>(smem + p.off_bsum);
  float* part = reinterpret_cast<float*>(smem + p.off_part);
  int8_t* xq = reinterpret_cast<int8_t*>(smem + p.off_xq);
  uint8_t* stg = smem + p.off_stage;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r0 = (int)((int64_t)blockIdx.x * p.R / gridDim.x);
  const int r1 = (int)((int64_t)(blockIdx.x + 1) * p.R / gridDim.x);
  const int nstages = (r1 - r0 + p.rps - 1) / p.rps;

  if (tid == 0) {
    for (int i = 0; i < p.nst; i++) mbar_init(&full[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const uint64_t pol = policy_evict_first();
  auto issue = [&](int k) {
    const int ra = r0 + k * p.rps, rb = min(ra + p.rps, r1);
    const uint32_t bytes = (uint32_t)((rb - ra) * p.pitch);
    const int buf = k % p.nst;
    mbar_arrive_expect_tx(&full[buf], bytes);
    bulk_g2s_stream(stg + (size_t)buf * p.stage_bytes, p.W + (int64_t)ra * p.pitch, bytes,
                    &full[buf], pol);
  };
  if (tid == 0)
    for (int k = 0; k < min(p.nst, nstages); k++) issue(k);

  quantize_x<QT == 0 ? 8 : 16>(p, xd, bsum, xq);
  __syncthreads();

  const int part_sz = p.rps * p.S * p.batch;
  for (int k = 0; k < nstages; k++) {
    const int buf = k % p.nst;
    const bool ok = mbar_wait_bounded(&full[buf], (uint32_t)((k / p.nst) & 1));
    const int ra = r0 + k * p.rps, rows = min(p.rps, r1 - ra);
    float* pb = part + (k & 1) * part_sz;
    const uint8_t* sbuf = stg + (size_t)buf * p.stage_bytes;
    if (ok) {
      const int U = rows * p.S;
      for (int u0 = warp * 8; u0 < U; u0 += KQ_WARPS * 8) {
        int u = u0 + (lane >> 2);
        const bool valid = u < U;
        if (!valid) u = U - 1;
        const int rr = u / p.S, s = u - rr * p.S;
        float* out = pb + (rr * p.S + s) * p.batch;
        if (QT == 0)
          q4k_unit(sbuf + (int64_t)rr * p.pitch + s * 144, lane & 3, p, xq, xd, bsum, s, out, 1,
                   valid);
        else
          q6k_unit(sbuf + (int64_t)rr * p.pitch, s, lane & 3, p, xq, xd, bsum, out, 1, valid);
      }
    }
    if (__syncthreads_or(!ok)) {
      if (tid == 0) {
        record_error(p.status, KERR_TIMEOUT);
        for (int j = k; j < min(k + p.nst, nstages); j++)
          mbar_wait_bounded(&full[j % p.nst], (uint32_t)((j / p.nst) & 1));
      }
      return;
    }
    if (tid == 0 && k + p.nst < nstages) issue(k + p.nst);
    for (int t = warp; t < rows * p.batch; t += KQ_WARPS) {
      const int rr = t / p.batch, b = t - rr * p.batch;
      const float v = warp_fixed_tree(pb + rr * p.S * p.batch + b, p.batch, p.S);
      if (lane == 0) p.y[(int64_t)b * p.ldy + ra + rr] = v;
    }
  }
}

}  // namespace

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

int max_smem_optin() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  }
  return n;
}

static inline uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

cudaError_t launch_kq_matvec(const DevMatrix& m, const float* x, int64_t ldx, int64_t batch,
                             float* y, int64_t ldy, unsigned* status, cudaStream_t st) {
  if (m.dtype != T_Q4_K && m.dtype != T_Q6_K) return cudaErrorInvalidValue;
  const int S = (int)(m.in_feat / 256);
  if (S < 1 || S > KQ_SMAX || m.in_feat % 256) return cudaErrorInvalidValue;
  if (m.out_feat <= 0 || batch <= 0) return cudaSuccess;
  const int smem_max = max_smem_optin();
  const int nsm = num_sms();
  for (int64_t b0 = 0; b0 < batch; b0 += KQ_BMAX) {
    const int nb = (int)std::min<int64_t>(KQ_BMAX, batch - b0);
    KqParams p{};
    p.x = x + b0 * ldx;
    p.ldx = ldx;
    p.batch = nb;
    p.n = (int)m.in_feat;
    p.S = S;
    p.W = m.data;
    p.pitch = m.pitch;
    p.R = (int)m.out_feat;
    p.y = y + b0 * ldy;
    p.ldy = ldy;
    p.status = status;
    const int NB = m.dtype == T_Q4_K ? 8 : 16;
    uint32_t off = align_up(KQ_NST_MAX * 8, 16);
    p.off_xd = off;
    off = align_up(off + nb * S * 4, 16);
    p.off_bsum = off;
    off = align_up(off + nb * S * NB * 4, 16);
    p.off_xq = off;
    off = align_up(off + nb * p.n, 128);
    // Stage = whole rows, about 24 KB; part double buffer sized to match.
    int rps = std::max<int>(1, (int)(24576 / m.pitch));
    const int rows_per_cta = (int)((m.out_feat + nsm - 1) / nsm);
    rps = std::min(rps, rows_per_cta);
    int nst;
    for (;;) {
      const uint32_t part_bytes = align_up(2u * rps * S * nb * 4, 128);
      const uint32_t stage_bytes = (uint32_t)(rps * m.pitch);
      const int avail = smem_max - (int)off - (int)part_bytes;
      nst = std::min<int>(KQ_NST_MAX, avail > 0 ? avail / (int)stage_bytes : 0);
      const int need = (rows_per_cta + rps - 1) / rps;  // stages per CTA
      nst = std::min(nst, std::max(need, 1));
      if (nst >= 2 || (nst >= 1 && need <= 1)) {
        p.off_part = off;
        p.off_stage = off + part_bytes;
        p.stage_bytes = stage_bytes;
        break;
      }
      if (rps == 1) return cudaErrorInvalidValue;  // row too long for shared memory
      rps = std::max(1, rps / 2);
    }
    p.rps = rps;
    p.nst = nst;
    const uint32_t smem = p.off_stage + (uint32_t)nst * p.stage_bytes;
    const int grid = (int)std::min<int64_t>(m.out_feat, nsm);
    cudaError_t e;
    // The opt-in size is set once per kernel (per process) to the device maximum.
    static bool attr_set[2] = {false, false};
    const int qi = m.dtype == T_Q4_K ? 0 : 1;
    if (!attr_set[qi]) {
      e = cudaFuncSetAttribute(qi == 0 ? kq_matvec_kernel<0> : kq_matvec_kernel<1>,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, smem_max);
      if (e != cudaSuccess) return e;
      attr_set[qi] = true;
    }
    if (qi == 0) kq_matvec_kernel<0><<<grid, KQ_THREADS, smem, st>>>(p);
    else kq_matvec_kernel<1><<<grid, KQ_THREADS, smem, st>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace vtq
