// canon_matvec.cu -- the reference's pinned fp32 canonical linear on sm_100a.
//
// Bit-exact restatement of the linears that dequantise to fp32 and reduce
// through canonical_dot (vitni-tensor src/ops/quant.rs:482-566):
//   Q8_0 / Q5_0  linear_dispatch arms  src/model/forward_quantized.rs:751-776
//   Q4_0         linear_q4_0_cpu       src/ops/quant.rs:1529-1565
//   F32          linear_dispatch arm   src/model/forward_quantized.rs:674-697
//   Q4_K float   canonical_dot_q4k_fused / linear_q4_k_fused  quant.rs:616-702, :1433
//                (the reference's default-feature build)
// Contract: lane[j] accumulates x[i]*w[i] (each product rounded, then added)
// for i = j mod 8 in ascending i; every 8192 elements a chunk closes with
// fixed_tree over the 8 lanes; the row result is fixed_tree over chunks.
// Chunk starts are multiples of 8192, so lane = i mod 8 everywhere.
//
// Design (Q4_K float mode, F32): a CTA owns a tile of up to 32 output rows; 4
// threads per row, thread p running lanes 2p and 2p+1 (the block-32 formats
// use canon_lane_kernel below: one thread per lane). Products are formed two at a time with
// mul.rn.f32x2; every accumulation add is a scalar add.rn.f32. A packed add
// must never consume a packed product: ptxas contracts mul.rn.f32x2 followed
// by add/sub.rn.f32x2 into a fused multiply-add (observed with -fmad=false and
// --fmad=false), which rounds once instead of twice and breaks bit parity. Weights arrive as [rows x 512
// column] tiles by one 2D TMA tensor copy per stage into a shared-memory
// ring; x is staged once per CTA in shared memory. Each weight pair is
// dequantised in the thread that consumes it with the reference's fp32 op
// order (scale * q, or d1 * q - m1 for Q4_K); int -> fp32 goes through an
// exact magic-number conversion instead of the I2F unit.
#include <cuda.h>
#include <cuda_fp16.h>

#include <mutex>
#include <unordered_map>

#include "vtq_device.cuh"
#include "vtq_internal.h"

namespace vtq {
namespace {

constexpr int CN_THREADS = 128;  // 32 rows x 4 threads
constexpr int CN_RMAX = 32;
constexpr int CN_BMAX = 4;
constexpr int CN_NST_MAX = 8;
constexpr int CN_MAXCH = 4;  // chunks per row: in_feat <= 32768
constexpr uint32_t FULL = 0xffffffffu;

struct CnParams {
  const float* x;
  int64_t ldx;
  int batch, n;
  int R, rt;           // rows, rows per tile (CTA)
  float* y;
  int64_t ldy;
  int slab_e;          // elements per slab (a divisor of 8192)
  int slab_b;          // packed bytes per slab row (multiple of 16)
  uint32_t stage_b;    // rt * slab_b
  int nst;
  int xs_stride;       // x row stride in shared memory (n rounded up to 4)
  uint32_t stage_stride;  // stage_b rounded up to 128 (TMA destination alignment)
  uint32_t off_x, off_stage;
  unsigned* status;
};

typedef unsigned long long f2;  // two packed fp32 lanes: low word = even lane

__device__ __forceinline__ f2 pk(float lo, float hi) {
  return (f2)__float_as_uint(lo) | ((f2)__float_as_uint(hi) << 32);
}
__device__ __forceinline__ float lo_of(f2 v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi_of(f2 v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ f2 sub2(f2 a, f2 b) {
  f2 d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
  f2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ float h2f(uint32_t bits) {
  return __half2float(__ushort_as_half((unsigned short)bits));
}
__device__ __forceinline__ uint32_t lds16(const uint8_t* p) {
  return *reinterpret_cast<const uint16_t*>(p);
}

// Exact small-integer -> fp32 pair: bytes b0, b1 (0..255) placed under
// exponent 2^23 then minus (2^23 + bias): gives (b0 - bias, b1 - bias).
__device__ __forceinline__ f2 bytes_to_f2(uint32_t b0, uint32_t b1, float bias) {
  const float m = 8388608.0f + bias;
  return sub2(pk(__uint_as_float(0x4B000000u | b0), __uint_as_float(0x4B000000u | b1)), pk(m, m));
}

// The dequantised weights of elements (e, e + 1), e = 8 g + 2 p, of one slab row.
template <int FMT>
__device__ __forceinline__ f2 weight_pair(const uint8_t* row, int g, int p) {
  if (FMT == T_Q8_0) {  // quant.rs:193-210: scale * (qs[k] as i8 as f32)
    const uint8_t* blk = row + (g >> 2) * 34;
    const float scale = h2f(lds16(blk));
    const uint32_t u = lds16(blk + 2 + 8 * (g & 3) + 2 * p) ^ 0x8080u;  // q + 128
    return mul2(pk(scale, scale), bytes_to_f2(u & 0xff, u >> 8, 128.0f));
  } else if (FMT == T_Q4_0) {  // quant.rs:91-111: scale * (nibble - 8)
    const uint8_t* blk = row + (g >> 2) * 18;
    const float scale = h2f(lds16(blk));
    const uint32_t byte = blk[2 + 4 * (g & 3) + p];
    return mul2(pk(scale, scale), bytes_to_f2(byte & 15, byte >> 4, 8.0f));
  } else if (FMT == T_Q5_0) {  // quant.rs:160-186: scale * ((nib | hbit << 4) - 16)
    const uint8_t* blk = row + (g >> 2) * 22;
    const float scale = h2f(lds16(blk));
    const uint32_t qh = lds16(blk + 2) | (lds16(blk + 4) << 16);
    const int e = 8 * (g & 3) + 2 * p;  // element within the 32-block
    uint32_t n0, n1;
    if (e < 16) {
      n0 = blk[6 + e] & 15;
      n1 = blk[7 + e] & 15;
    } else {
      n0 = blk[6 + e - 16] >> 4;
      n1 = blk[7 + e - 16] >> 4;
    }
    n0 |= ((qh >> e) & 1u) << 4;
    n1 |= ((qh >> (e + 1)) & 1u) << 4;
    return mul2(pk(scale, scale), bytes_to_f2(n0, n1, 16.0f));
  } else if (FMT == T_Q4_K) {  // quant.rs:654-673: d1 * q - m1, d1 = d * sc, m1 = dmin * m
    const uint8_t* sb = row + (g >> 5) * 144;
    const int e = 8 * (g & 31) + 2 * p;  // element within the superblock
    const int half = e >> 6, hi = (e >> 5) & 1, l = e & 31;
    const int j = 2 * half + hi;
    const uint8_t* s = sb + 4;
    int sc, m;
    if (j < 4) {
      sc = s[j] & 63;
      m = s[j + 4] & 63;
    } else {
      sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
      m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
    const float d = h2f(lds16(sb)), dmin = h2f(lds16(sb + 2));
    const float d1 = __fmul_rn(d, __int2float_rn(sc));
    const float m1 = __fmul_rn(dmin, __int2float_rn(m));
    const uint32_t b2 = lds16(sb + 16 + 32 * half + l);
    const uint32_t q0 = hi ? ((b2 >> 4) & 15) : (b2 & 15);
    const uint32_t q1 = hi ? (b2 >> 12) : ((b2 >> 8) & 15);
    const f2 t = mul2(pk(d1, d1), bytes_to_f2(q0, q1, 0.0f));
    return pk(__fsub_rn(lo_of(t), m1), __fsub_rn(hi_of(t), m1));  // scalar: no contraction
  } else {  // F32
    return *reinterpret_cast<const f2*>(row + 4 * (8 * g + 2 * p));
  }
}

// Close a chunk: fixed_tree over the row's 8 lanes, held as 4 pairs on 4
// consecutive threads: ((l0+l1)+(l2+l3))+((l4+l5)+(l6+l7)). Valid on p == 0.
__device__ __forceinline__ float lane_tree(float lo, float hi, int p) {
  float t = __fadd_rn(lo, hi);
  float o = __shfl_down_sync(FULL, t, 1);
  if ((p & 1) == 0) t = __fadd_rn(t, o);
  o = __shfl_down_sync(FULL, t, 2);
  if (p == 0) t = __fadd_rn(t, o);
  return t;
}

// fixed_tree over up to 4 chunk sums.
__device__ __forceinline__ float chunk_tree(const float* c, int n) {
  if (n <= 1) return n == 1 ? c[0] : 0.0f;
  const float a = __fadd_rn(c[0], c[1]);
  if (n == 2) return a;
  const float b = (n == 4) ? __fadd_rn(c[2], c[3]) : c[2];
  return __fadd_rn(a, b);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

template <int FMT, int MAXB>
__global__ void __launch_bounds__(CN_THREADS)
    canon_matvec_kernel(const __grid_constant__ CUtensorMap tm, const CnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  float* xs = reinterpret_cast<float*>(smem + p.off_x);
  uint8_t* stg = smem + p.off_stage;

  const int tid = threadIdx.x, rr = tid >> 2, pp = tid & 3;
  const int row0 = blockIdx.x * p.rt;
  const int nrows = min(p.rt, p.R - row0);
  const int nslab = (p.n + p.slab_e - 1) / p.slab_e;

  if (tid == 0) {
    for (int i = 0; i < p.nst; i++) mbar_init(&full[i], 1);
    fence_mbar_init();
    for (int k = 0; k < min(p.nst, nslab); k++) {
      mbar_arrive_expect_tx(&full[k], p.stage_b);
      tma_load_2d(stg + (size_t)k * p.stage_stride, &tm, k * (p.slab_b / 4), row0, &full[k]);
    }
  }
  for (int b = 0; b < p.batch; b++)
    for (int i = tid; i < p.n; i += CN_THREADS) xs[b * p.xs_stride + i] = __ldg(p.x + b * p.ldx + i);
  __syncthreads();

  float acc_lo[MAXB], acc_hi[MAXB];
  float chs[MAXB][CN_MAXCH];
#pragma unroll
  for (int b = 0; b < MAXB; b++) {
    acc_lo[b] = 0.0f;
    acc_hi[b] = 0.0f;
#pragma unroll
    for (int c = 0; c < CN_MAXCH; c++) chs[b][c] = 0.0f;
  }
  int nch = 0;
  const bool row_ok = rr < nrows;

  for (int k = 0; k < nslab; k++) {
    const int buf = k % p.nst;
    const bool ok = mbar_wait_bounded(&full[buf], (uint32_t)((k / p.nst) & 1));
    const int e0 = k * p.slab_e;
    const int ecount = min(p.slab_e, p.n - e0);
    if (ok && row_ok) {
      const uint8_t* row = stg + (size_t)buf * p.stage_stride + (size_t)rr * p.slab_b;
      const int full_groups = ecount >> 3;
#pragma unroll 4
      for (int g = 0; g < full_groups; g++) {
        const f2 w = weight_pair<FMT>(row, g, pp);
        const int e = e0 + 8 * g + 2 * pp;
#pragma unroll
        for (int b = 0; b < MAXB; b++) {
          if (b < p.batch) {
            const f2 prod = mul2(*reinterpret_cast<const f2*>(xs + b * p.xs_stride + e), w);
            acc_lo[b] = __fadd_rn(acc_lo[b], lo_of(prod));
            acc_hi[b] = __fadd_rn(acc_hi[b], hi_of(prod));
          }
        }
      }
      if (FMT == T_F32 && (ecount & 7)) {  // ragged tail (F32 only): lane-exact scalar steps
        const int g = full_groups, e = e0 + 8 * g + 2 * pp;
        const float* wr = reinterpret_cast<const float*>(row) + 8 * g + 2 * pp;
#pragma unroll
        for (int b = 0; b < MAXB; b++) {
          if (b < p.batch) {
            if (e < p.n) acc_lo[b] = __fadd_rn(acc_lo[b], __fmul_rn(xs[b * p.xs_stride + e], wr[0]));
            if (e + 1 < p.n)
              acc_hi[b] = __fadd_rn(acc_hi[b], __fmul_rn(xs[b * p.xs_stride + e + 1], wr[1]));
          }
        }
      }
    }
    // Close a chunk every 8192 elements and at the row end (quant.rs:557-565).
    const int e_end = e0 + ecount;
    if (e_end % 8192 == 0 || e_end == p.n) {
#pragma unroll
      for (int b = 0; b < MAXB; b++) {
        const float t = lane_tree(acc_lo[b], acc_hi[b], pp);
#pragma unroll
        for (int c = 0; c < CN_MAXCH; c++)
          if (c == nch) chs[b][c] = t;
        acc_lo[b] = 0.0f;
        acc_hi[b] = 0.0f;
      }
      nch++;
    }
    if (__syncthreads_or(!ok)) {
      if (tid == 0) {
        record_error(p.status, KERR_TIMEOUT);
        for (int i = k; i < min(k + p.nst, nslab); i++)
          mbar_wait_bounded(&full[i % p.nst], (uint32_t)((i / p.nst) & 1));
      }
      return;
    }
    if (tid == 0 && k + p.nst < nslab) {
      mbar_arrive_expect_tx(&full[buf], p.stage_b);
      tma_load_2d(stg + (size_t)buf * p.stage_stride, &tm, (k + p.nst) * (p.slab_b / 4), row0,
                  &full[buf]);
    }
  }
  if (row_ok && pp == 0) {
#pragma unroll
    for (int b = 0; b < MAXB; b++)
      if (b < p.batch) p.y[(int64_t)b * p.ldy + row0 + rr] = chunk_tree(chs[b], nch);
  }
}

// ---- Block-32 formats (Q8_0 / Q4_0 / Q5_0): one thread per (row, lane) ----
// Thread (r, j) runs lane j of row r: within every 32-element block it owns
// elements j, j + 8, j + 16, j + 24, i.e. exactly the reference's lane
// i mod 8, in ascending i. Every thread forms its own products (dequantise
// in the reference's fp32 order, multiply, then one add.rn into the lane), so
// a CTA of 32 rows runs 256 independent chains instead of 64.
constexpr int CL_RMAX = 32;
constexpr int CL_THREADS = CL_RMAX * 8;

// The 4 dequantised weights of lane j in one block (block bytes at blk).
template <int FMT>
__device__ __forceinline__ void lane_weights(const uint8_t* blk, int j, float (&w)[4]) {
  const float scale = h2f(lds16(blk));
  if (FMT == T_Q8_0) {  // quant.rs:193-210: scale * (qs[k] as i8 as f32)
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint32_t u = (uint32_t)(blk[2 + j + 8 * k] ^ 0x80u);  // q + 128
      w[k] = __fmul_rn(scale, __fsub_rn(__uint_as_float(0x4B000000u | u), 8388736.0f));
    }
  } else if (FMT == T_Q4_0) {  // quant.rs:91-111: scale * (nibble - 8)
    // Nibbles interleave: element 2m is the low nibble of byte m, 2m + 1 the
    // high one, so element j + 8k sits in byte j / 2 + 4k.
    const int sh = (j & 1) * 4;
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint32_t q = (blk[2 + (j >> 1) + 4 * k] >> sh) & 15u;
      w[k] = __fmul_rn(scale, __fsub_rn(__uint_as_float(0x4B000000u | q), 8388616.0f));
    }
  } else {  // T_Q5_0, quant.rs:160-186: scale * ((nib | hbit << 4) - 16)
    const uint32_t qh = lds16(blk + 2) | (lds16(blk + 4) << 16);
    const uint32_t b0 = blk[6 + j], b1 = blk[6 + j + 8];
    const uint32_t n4[4] = {b0 & 15, b1 & 15, b0 >> 4, b1 >> 4};
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const int e = j + 8 * k;
      const uint32_t q = n4[k] | (((qh >> e) & 1u) << 4);
      w[k] = __fmul_rn(scale, __fsub_rn(__uint_as_float(0x4B000000u | q), 8388624.0f));
    }
  }
}

template <int FMT, int MAXB>
__global__ void __launch_bounds__(CL_THREADS)
    canon_lane_kernel(const __grid_constant__ CUtensorMap tm, const CnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  float* xs = reinterpret_cast<float*>(smem + p.off_x);
  uint8_t* stg = smem + p.off_stage;
  constexpr int BB = FMT == T_Q8_0 ? 34 : (FMT == T_Q4_0 ? 18 : 22);  // block bytes

  const int tid = threadIdx.x, rr = tid >> 3, j = tid & 7;
  const int row0 = blockIdx.x * p.rt;
  const int nrows = min(p.rt, p.R - row0);
  const int nslab = (p.n + p.slab_e - 1) / p.slab_e;

  if (tid == 0) {
    for (int i = 0; i < p.nst; i++) mbar_init(&full[i], 1);
    fence_mbar_init();
    for (int k = 0; k < min(p.nst, nslab); k++) {
      mbar_arrive_expect_tx(&full[k], p.stage_b);
      tma_load_2d(stg + (size_t)k * p.stage_stride, &tm, k * (p.slab_b / 4), row0, &full[k]);
    }
  }
  // Programmatic launch: the weights above never depend on the previous
  // kernel; x may, so read it only after the previous grid has completed.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  for (int b = 0; b < p.batch; b++)
    for (int i = tid; i < p.n; i += CL_THREADS) xs[b * p.xs_stride + i] = __ldg(p.x + b * p.ldx + i);
  __syncthreads();

  float acc[MAXB], chs[MAXB][CN_MAXCH];
#pragma unroll
  for (int b = 0; b < MAXB; b++) {
    acc[b] = 0.0f;
#pragma unroll
    for (int c = 0; c < CN_MAXCH; c++) chs[b][c] = 0.0f;
  }
  int nch = 0;
  const bool row_ok = rr < nrows;
  for (int k = 0; k < nslab; k++) {
    const int buf = k % p.nst;
    const bool ok = mbar_wait_bounded(&full[buf], (uint32_t)((k / p.nst) & 1));
    const int e0 = k * p.slab_e;
    const int ecount = min(p.slab_e, p.n - e0);
    if (ok && row_ok) {
      const uint8_t* row = stg + (size_t)buf * p.stage_stride + (size_t)rr * p.slab_b;
      const int nblk = ecount >> 5;
#pragma unroll 4
      for (int g = 0; g < nblk; g++) {
        float w[4];
        lane_weights<FMT>(row + g * BB, j, w);
        const int e = e0 + 32 * g + j;
#pragma unroll
        for (int b = 0; b < MAXB; b++) {
          if (b < p.batch) {
            const float* xb = xs + b * p.xs_stride + e;
#pragma unroll
            for (int q = 0; q < 4; q++) acc[b] = __fadd_rn(acc[b], __fmul_rn(xb[8 * q], w[q]));
          }
        }
      }
    }
    // Close a chunk every 8192 elements and at the row end (quant.rs:557-565):
    // fixed_tree over the row's 8 lanes, held by 8 consecutive threads.
    const int e_end = e0 + ecount;
    if (e_end % 8192 == 0 || e_end == p.n) {
#pragma unroll
      for (int b = 0; b < MAXB; b++) {
        float t = acc[b];
        float o = __shfl_down_sync(FULL, t, 1);
        if ((j & 1) == 0) t = __fadd_rn(t, o);
        o = __shfl_down_sync(FULL, t, 2);
        if ((j & 3) == 0) t = __fadd_rn(t, o);
        o = __shfl_down_sync(FULL, t, 4);
        if (j == 0) t = __fadd_rn(t, o);
#pragma unroll
        for (int c = 0; c < CN_MAXCH; c++)
          if (c == nch) chs[b][c] = t;
        acc[b] = 0.0f;
      }
      nch++;
    }
    if (__syncthreads_or(!ok)) {
      if (tid == 0) {
        record_error(p.status, KERR_TIMEOUT);
        for (int i = k; i < min(k + p.nst, nslab); i++)
          mbar_wait_bounded(&full[i % p.nst], (uint32_t)((i / p.nst) & 1));
      }
      return;
    }
    if (tid == 0 && k + p.nst < nslab) {
      mbar_arrive_expect_tx(&full[buf], p.stage_b);
      tma_load_2d(stg + (size_t)buf * p.stage_stride, &tm, (k + p.nst) * (p.slab_b / 4), row0,
                  &full[buf]);
    }
  }
  if (row_ok && j == 0) {
#pragma unroll
    for (int b = 0; b < MAXB; b++)
      if (b < p.batch) p.y[(int64_t)b * p.ldy + row0 + rr] = chunk_tree(chs[b], nch);
  }
}

// Tensor maps are cached per (pointer, rows, pitch, box).
struct TmKey {
  const void* ptr;
  int64_t rows, pitch;
  int box_x, box_y;
  bool operator==(const TmKey& o) const {
    return ptr == o.ptr && rows == o.rows && pitch == o.pitch && box_x == o.box_x &&
           box_y == o.box_y;
  }
};
struct TmHash {
  size_t operator()(const TmKey& k) const {
    return std::hash<const void*>()(k.ptr) ^ (size_t)(k.rows * 1315423911u) ^
           (size_t)(k.pitch << 7) ^ (size_t)(k.box_x << 3) ^ (size_t)k.box_y;
  }
};

cudaError_t get_tensor_map(const DevMatrix& m, int box_x_u32, int box_y, CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<TmKey, CUtensorMap, TmHash> cache;
  const TmKey key{m.data, m.out_feat, m.pitch, box_x_u32, box_y};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return cudaSuccess;
  }
  if (cache.size() > 4096) cache.clear();
  // The driver entry point is resolved at run time so that the library loads
  // (for ABI checks) on machines without a CUDA driver.
  typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                               const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                               const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                               CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static EncodeFn encode = nullptr;
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return cudaErrorInvalidValue;
    encode = reinterpret_cast<EncodeFn>(fn);
  }
  cuuint64_t gdim[2] = {(cuuint64_t)(m.pitch / 4), (cuuint64_t)m.out_feat};
  cuuint64_t gstride[1] = {(cuuint64_t)m.pitch};
  cuuint32_t box[2] = {(cuuint32_t)box_x_u32, (cuuint32_t)box_y};
  cuuint32_t estride[2] = {1, 1};
  const CUresult r = encode(out, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint8_t*>(m.data),
                            gdim, gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  cache.emplace(key, *out);
  return cudaSuccess;
}

template <int FMT, int MAXB>
cudaError_t launch_fmt(const CUtensorMap& tm, const CnParams& p, int grid, uint32_t smem,
                       cudaStream_t st) {
  static bool attr_set = false;  // once per instantiation
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(canon_matvec_kernel<FMT, MAXB>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         max_smem_optin());
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  kernel_launch_count()++;
  canon_matvec_kernel<FMT, MAXB><<<grid, CN_THREADS, smem, st>>>(tm, p);
  return cudaGetLastError();
}

template <int FMT, int MAXB>
cudaError_t launch_lane(const CUtensorMap& tm, const CnParams& p, int grid, uint32_t smem,
                        cudaStream_t st) {
  static bool attr_set = false;  // once per instantiation
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(canon_lane_kernel<FMT, MAXB>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         max_smem_optin());
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(CL_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  kernel_launch_count()++;
  return cudaLaunchKernelEx(&cfg, canon_lane_kernel<FMT, MAXB>, tm, p);
}

template <int FMT>
cudaError_t launch_batch(const CUtensorMap& tm, const CnParams& p, int grid, uint32_t smem,
                         cudaStream_t st) {
  if constexpr (FMT == T_Q8_0 || FMT == T_Q4_0 || FMT == T_Q5_0) {
    if (p.batch <= 1) return launch_lane<FMT, 1>(tm, p, grid, smem, st);
    if (p.batch <= 2) return launch_lane<FMT, 2>(tm, p, grid, smem, st);
    return launch_lane<FMT, 4>(tm, p, grid, smem, st);
  }
  if (p.batch <= 1) return launch_fmt<FMT, 1>(tm, p, grid, smem, st);
  if (p.batch <= 2) return launch_fmt<FMT, 2>(tm, p, grid, smem, st);
  return launch_fmt<FMT, 4>(tm, p, grid, smem, st);
}

}  // namespace

cudaError_t launch_canon_matvec(const DevMatrix& m, const float* x, int64_t ldx, int64_t batch,
                                float* y, int64_t ldy, unsigned* status, cudaStream_t st) {
  if (m.in_feat > CN_MAXCH * 8192) return cudaErrorInvalidValue;
  if (m.out_feat <= 0 || batch <= 0) return cudaSuccess;
  CnParams p{};
  p.n = (int)m.in_feat;
  p.R = (int)m.out_feat;
  p.status = status;
  switch (m.dtype) {
    case T_Q8_0: p.slab_e = 512; p.slab_b = 16 * 34; break;
    case T_Q5_0: p.slab_e = 512; p.slab_b = 16 * 22; break;
    case T_Q4_0: p.slab_e = 512; p.slab_b = 16 * 18; break;
    case T_Q4_K: p.slab_e = 512; p.slab_b = 2 * 144; break;
    case T_F32:  p.slab_e = 256; p.slab_b = 256 * 4; break;
    default: return cudaErrorInvalidValue;
  }
  const int nsm = num_sms();
  p.rt = (int)std::max<int64_t>(1, std::min<int64_t>(CN_RMAX, (m.out_feat + nsm - 1) / nsm));
  const int grid = (int)((m.out_feat + p.rt - 1) / p.rt);
  p.stage_b = (uint32_t)(p.rt * p.slab_b);
  CUtensorMap tm;
  cudaError_t e = get_tensor_map(m, p.slab_b / 4, p.rt, &tm);
  if (e != cudaSuccess) return e;
  const int smem_max = max_smem_optin();
  p.xs_stride = (p.n + 3) / 4 * 4;
  p.stage_stride = (p.stage_b + 127) / 128 * 128;
  const int nslab = (p.n + p.slab_e - 1) / p.slab_e;
  // Activation rows per launch: as many as fit beside a ring of >= 2 stages.
  const int64_t room = (int64_t)smem_max - 256 - 2 * (int64_t)p.stage_stride;
  const int bfit = (int)std::min<int64_t>(CN_BMAX, room / ((int64_t)p.xs_stride * 4));
  if (bfit < 1) return cudaErrorInvalidValue;
  for (int64_t b0 = 0; b0 < batch; b0 += bfit) {
    CnParams q = p;
    q.batch = (int)std::min<int64_t>(bfit, batch - b0);
    q.x = x + b0 * ldx;
    q.ldx = ldx;
    q.y = y + b0 * ldy;
    q.ldy = ldy;
    q.off_x = 128;
    q.off_stage = (uint32_t)((q.off_x + q.batch * q.xs_stride * 4 + 127) / 128 * 128);
    const int avail = smem_max - (int)q.off_stage;
    q.nst = std::min(std::min(CN_NST_MAX, nslab), avail / (int)q.stage_stride);
    if (q.nst < 1) return cudaErrorInvalidValue;
    const uint32_t smem = q.off_stage + (uint32_t)q.nst * q.stage_stride;
    switch (m.dtype) {
      case T_Q8_0: e = launch_batch<T_Q8_0>(tm, q, grid, smem, st); break;
      case T_Q5_0: e = launch_batch<T_Q5_0>(tm, q, grid, smem, st); break;
      case T_Q4_0: e = launch_batch<T_Q4_0>(tm, q, grid, smem, st); break;
      case T_Q4_K: e = launch_batch<T_Q4_K>(tm, q, grid, smem, st); break;
      default:     e = launch_batch<T_F32>(tm, q, grid, smem, st); break;
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace vtq
