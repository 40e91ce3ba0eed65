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
// Design: a CTA owns 16 output rows; thread (row, j) runs lane chain j of its
// row for every activation row in the launch. Weights stream through a
// shared-memory ring of column slabs (512 elements of 16 rows) filled by TMA
// bulk copies, one per row, completing on one mbarrier per stage. Each
// element's dequantisation is recomputed in the thread that consumes it with
// the reference's exact fp32 op order (scale * q, or d1 * q - m1 for Q4_K).
#include "vtq_device.cuh"
#include "vtq_internal.h"

namespace vtq {
namespace {

constexpr int CN_ROWS = 16;
constexpr int CN_THREADS = CN_ROWS * 8;
constexpr int CN_BMAX = 4;
constexpr int CN_NST = 4;
constexpr int CN_MAXCH = 4;  // chunks per row: in_feat <= 32768
constexpr uint32_t FULL = 0xffffffffu;

struct CnParams {
  const float* x;
  int64_t ldx;
  int batch, n;
  const uint8_t* W;
  int64_t pitch, row_bytes;
  int R;
  float* y;
  int64_t ldy;
  int slab_e;          // elements per slab
  int slab_b;          // packed bytes per full slab per row
  uint32_t stage_b;    // bytes per stage = CN_ROWS * slab_b
  unsigned* status;
};

__device__ __forceinline__ uint32_t ld16(const uint8_t* p) {
  return *reinterpret_cast<const uint16_t*>(p);
}

// Packed bytes of `e` elements of a row (e a multiple of the block size).
template <int FMT>
__device__ __forceinline__ int row_bytes_of(int e) {
  if (FMT == T_Q8_0) return e / 32 * 34;
  if (FMT == T_Q5_0) return e / 32 * 22;
  if (FMT == T_Q4_0) return e / 32 * 18;
  if (FMT == T_Q4_K) return e / 256 * 144;
  return e * 4;  // F32
}

// Dequantised weight for slab-local element index e (fp32 op order of the
// reference's dequantisers).
template <int FMT>
__device__ __forceinline__ float weight_at(const uint8_t* slab, int e) {
  if (FMT == T_Q8_0) {  // quant.rs:193-210: scale * (qs[k] as i8 as f32)
    const uint8_t* blk = slab + (e >> 5) * 34;
    const float scale = f16_bits_to_f32(ld16(blk));
    const int q = (int8_t)blk[2 + (e & 31)];
    return __fmul_rn(scale, __int2float_rn(q));
  } else if (FMT == T_Q5_0) {  // quant.rs:160-186
    const uint8_t* blk = slab + (e >> 5) * 22;
    const float scale = f16_bits_to_f32(ld16(blk));
    const uint32_t qh = ld16(blk + 2) | (ld16(blk + 4) << 16);
    const int k = e & 31;
    const int jj = k & 15;
    const uint32_t byte = blk[6 + jj];
    const uint32_t nib = k < 16 ? (byte & 0x0F) : (byte >> 4);
    const uint32_t hb = ((qh >> k) & 1u) << 4;
    return __fmul_rn(scale, __int2float_rn((int)(nib | hb) - 16));
  } else if (FMT == T_Q4_0) {  // quant.rs:91-111
    const uint8_t* blk = slab + (e >> 5) * 18;
    const float scale = f16_bits_to_f32(ld16(blk));
    const int k = e & 31;
    const uint32_t byte = blk[2 + (k >> 1)];
    const int nib = (k & 1) ? (int)(byte >> 4) : (int)(byte & 0x0F);
    return __fmul_rn(scale, __int2float_rn(nib - 8));
  } else if (FMT == T_Q4_K) {  // quant.rs:280-326 / :654-673
    const uint8_t* sb = slab + (e >> 8) * 144;
    const int k = e & 255, half = k >> 6, hi = (k >> 5) & 1, l = k & 31;
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
    const float d = f16_bits_to_f32(ld16(sb)), dmin = f16_bits_to_f32(ld16(sb + 2));
    const float d1 = __fmul_rn(d, __int2float_rn(sc));
    const float m1 = __fmul_rn(dmin, __int2float_rn(m));
    const uint32_t byte = sb[16 + 32 * half + l];
    const int q = hi ? (int)(byte >> 4) : (int)(byte & 0x0F);
    return __fsub_rn(__fmul_rn(d1, __int2float_rn(q)), m1);
  } else {  // F32
    return reinterpret_cast<const float*>(slab)[e];
  }
}

// fixed_tree over the 8 lanes of one row (8 consecutive threads), pairing
// ((l0+l1)+(l2+l3))+((l4+l5)+(l6+l7)). Result valid in lane j == 0.
__device__ __forceinline__ float lane_tree8(float v, int j) {
  float o = __shfl_down_sync(FULL, v, 1);
  if ((j & 1) == 0) v = __fadd_rn(v, o);
  o = __shfl_down_sync(FULL, v, 2);
  if ((j & 3) == 0) v = __fadd_rn(v, o);
  o = __shfl_down_sync(FULL, v, 4);
  if (j == 0) v = __fadd_rn(v, o);
  return v;
}

// fixed_tree over up to 4 chunk sums.
__device__ __forceinline__ float chunk_tree(const float* c, int n) {
  if (n <= 1) return n == 1 ? c[0] : 0.0f;
  const float a = __fadd_rn(c[0], c[1]);
  if (n == 2) return a;
  const float b = (n == 4) ? __fadd_rn(c[2], c[3]) : c[2];
  return __fadd_rn(a, b);
}

template <int FMT>
__global__ void __launch_bounds__(CN_THREADS) canon_matvec_kernel(const CnParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint8_t* stg = smem + 128;

  const int tid = threadIdx.x, lane = tid & 31, rr = tid >> 3, j = tid & 7;
  const int row0 = blockIdx.x * CN_ROWS;
  const int nrows = min(CN_ROWS, p.R - row0);
  const int nslab = (p.n + p.slab_e - 1) / p.slab_e;

  if (tid == 0) {
    for (int i = 0; i < CN_NST; i++) mbar_init(&full[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const uint64_t pol = policy_evict_first();
  // Warp 0 fills stage k: lane r copies row r's slab bytes.
  auto issue = [&](int k) {
    const int buf = k % CN_NST;
    const int e0 = k * p.slab_e;
    const int ecount = min(p.slab_e, p.n - e0);
    const uint32_t bytes = (uint32_t)((row_bytes_of<FMT>(ecount) + 15) & ~15);
    if (lane == 0) mbar_arrive_expect_tx(&full[buf], bytes * nrows);
    __syncwarp();
    if (lane < nrows)
      bulk_g2s_stream(stg + (size_t)buf * p.stage_b + (size_t)lane * p.slab_b,
                      p.W + (int64_t)(row0 + lane) * p.pitch + row_bytes_of<FMT>(e0), bytes,
                      &full[buf], pol);
  };
  if (tid < 32)
    for (int k = 0; k < min(CN_NST, nslab); k++) issue(k);

  float acc[CN_BMAX], chs[CN_BMAX][CN_MAXCH];
#pragma unroll
  for (int b = 0; b < CN_BMAX; b++) {
    acc[b] = 0.0f;
#pragma unroll
    for (int c = 0; c < CN_MAXCH; c++) chs[b][c] = 0.0f;
  }
  int nch = 0;
  const bool row_ok = rr < nrows;

  for (int k = 0; k < nslab; k++) {
    const int buf = k % CN_NST;
    const bool ok = mbar_wait_bounded(&full[buf], (uint32_t)((k / CN_NST) & 1));
    const int e0 = k * p.slab_e;
    const int ecount = min(p.slab_e, p.n - e0);
    if (ok && row_ok) {
      const uint8_t* slab = stg + (size_t)buf * p.stage_b + (size_t)rr * p.slab_b;
      for (int e = j; e < ecount; e += 8) {
        const float w = weight_at<FMT>(slab, e);
#pragma unroll
        for (int b = 0; b < CN_BMAX; b++) {
          if (b < p.batch) {
            const float xv = __ldg(p.x + (int64_t)b * p.ldx + e0 + e);
            acc[b] = __fadd_rn(acc[b], __fmul_rn(xv, w));
          }
        }
      }
    }
    // Close a chunk every 8192 elements and at the row end (quant.rs:557-565).
    const int e_end = e0 + ecount;
    if (e_end % 8192 == 0 || e_end == p.n) {
#pragma unroll
      for (int b = 0; b < CN_BMAX; b++) {
        const float t = lane_tree8(acc[b], j);
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
        for (int i = k; i < min(k + CN_NST, nslab); i++)
          mbar_wait_bounded(&full[i % CN_NST], (uint32_t)((i / CN_NST) & 1));
      }
      return;
    }
    if (tid < 32 && k + CN_NST < nslab) issue(k + CN_NST);
  }
  if (row_ok && j == 0) {
#pragma unroll
    for (int b = 0; b < CN_BMAX; b++)
      if (b < p.batch) p.y[(int64_t)b * p.ldy + row0 + rr] = chunk_tree(chs[b], nch);
  }
}

template <int FMT>
cudaError_t launch_fmt(const CnParams& p0, int64_t batch, cudaStream_t st) {
  const uint32_t smem = 128 + CN_NST * p0.stage_b;
  static bool attr_set = false;  // once per format instantiation
  cudaError_t e;
  if (!attr_set) {
    e = cudaFuncSetAttribute(canon_matvec_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             max_smem_optin());
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  const int grid = (p0.R + CN_ROWS - 1) / CN_ROWS;
  for (int64_t b0 = 0; b0 < batch; b0 += CN_BMAX) {
    CnParams p = p0;
    p.batch = (int)std::min<int64_t>(CN_BMAX, batch - b0);
    p.x = p0.x + b0 * p0.ldx;
    p.y = p0.y + b0 * p0.ldy;
    canon_matvec_kernel<FMT><<<grid, CN_THREADS, smem, st>>>(p);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace

cudaError_t launch_canon_matvec(const DevMatrix& m, const float* x, int64_t ldx, int64_t batch,
                                float* y, int64_t ldy, unsigned* status, cudaStream_t st) {
  if (m.in_feat > CN_MAXCH * 8192) return cudaErrorInvalidValue;
  if (m.out_feat <= 0 || batch <= 0) return cudaSuccess;
  CnParams p{};
  p.x = x;
  p.ldx = ldx;
  p.n = (int)m.in_feat;
  p.W = m.data;
  p.pitch = m.pitch;
  p.row_bytes = m.row_bytes;
  p.R = (int)m.out_feat;
  p.y = y;
  p.ldy = ldy;
  p.status = status;
  switch (m.dtype) {
    case T_Q8_0: p.slab_e = 512; p.slab_b = 16 * 34; break;
    case T_Q5_0: p.slab_e = 512; p.slab_b = 16 * 22; break;
    case T_Q4_0: p.slab_e = 512; p.slab_b = 16 * 18; break;
    case T_Q4_K: p.slab_e = 512; p.slab_b = 2 * 144; break;
    case T_F32:  p.slab_e = 256; p.slab_b = 256 * 4; break;
    default: return cudaErrorInvalidValue;
  }
  p.stage_b = (uint32_t)(CN_ROWS * p.slab_b);
  switch (m.dtype) {
    case T_Q8_0: return launch_fmt<T_Q8_0>(p, batch, st);
    case T_Q5_0: return launch_fmt<T_Q5_0>(p, batch, st);
    case T_Q4_0: return launch_fmt<T_Q4_0>(p, batch, st);
    case T_Q4_K: return launch_fmt<T_Q4_K>(p, batch, st);
    default:     return launch_fmt<T_F32>(p, batch, st);
  }
}

}  // namespace vtq
