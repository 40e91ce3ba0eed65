// kquant_gemm.cu -- batched (prefill-sized) exact-integer Q4_K linear on the
// sm_100a tensor cores (tcgen05.mma kind::i8, int32 accumulators in TMEM).
//
// Computes, bit for bit, vitni-tensor's integer Q4_K linear for many
// activation rows at once:
//   linear_q4_k_integer(_parallel)  src/ops/quant.rs:936-980, :1149-1196
// y[b, o] = fixed_tree_s( (d_os * xd_bs) * f32(acc) - (dmin_os * xd_bs) * f32(acc_m) )
//   acc   = sum_j sc_j * sum_l q_jl * xq_bjl      (dot_q4k_q8_block, quant.rs:850-898)
//   acc_m = sum_j mn_j * bsum_bj
// Each activation row is quantised per 256-block exactly like
// quantize_block_q8 (quant.rs:750-771), independently of the other rows.
//
// Tensor-core mapping. For one superblock s both integers are contractions
// over its 256 positions k, so they are computed as one MMA product of the
// activation tile (A: 128 tokens x 256 int8, K-major) with three unsigned
// byte planes of the weights (B: 96 "rows" x 256). With sc = 8 sh + sl
// (sh, sl in [0, 7]):
//   rows  0..31  lo_k = sl_j(k) * q_k                 (<= 105)
//   rows 32..63  hi_k = sh_j(k) * q_k                 (<= 105)
//   rows 64..95  mn_j(k)                              (the 6-bit min, repeated)
// so acc = D[:, r] + 8 * D[:, 32 + r] and acc_m = D[:, 64 + r] exactly
// (|acc| <= 256 * 127 * 945 < 2^31). Every byte product stays below 256, so
// one 32-bit multiply scales four packed quants at once. The planes are built
// in shared memory from the packed superblocks by four builder warps; the per-superblock fp
// combine and the cross-superblock fixed_tree stay on CUDA cores, in the
// reference's op order, with the tree kept per (token, row) in registers as a
// binary counter of complete subtrees (identical pairings to the level-wise
// loop of quant.rs:462-476).
//
// CTA = 128 tokens x 32 weight rows, looping over superblocks:
//   warp 0      TMA producer: activation tile (2 x 16 KB, 128B-swizzled) and
//               the 32 rows' superblock (32 x 144 B) per step
//   warp 1      TMEM owner; lane 0 issues 8 MMAs (K = 32 each) per step
//   warps 4-7   plane builders (128 threads: one row x one pair of sub-blocks)
//   warps 8-15  epilogue: TMEM -> registers, fp combine, fixed_tree
// Every wait is bounded (%globaltimer); a timeout sets the status word, stops
// the pipeline and still frees TMEM.
#include <cuda.h>
#include <cuda_fp16.h>

#include <map>
#include <mutex>
#include <vector>
#include <unordered_map>

#include "vtq_device.cuh"
#include "vtq_internal.h"

namespace vtq {
namespace {

constexpr int GM = 128;         // tokens per CTA = MMA M = TMEM lanes
constexpr int GR = 32;          // weight rows per CTA
constexpr int GN = 3 * GR;      // MMA N: lo | hi | mins
constexpr int NX = 4;           // activation stages
constexpr int NW = 4;           // packed-weight stages
constexpr int NP = 3;           // plane stages
constexpr int NA = 3;           // TMEM accumulator buffers (128 columns apart)
constexpr int NMETA = 4;        // d / dmin stages
constexpr uint32_t X_STAGE = GM * 256;  // 2 K-blocks x 16 KB
constexpr uint32_t P_STAGE = GN * 256;  // 2 K-blocks x 12 KB
constexpr uint32_t P_KBLK = GN * 128;
constexpr uint32_t W_STAGE = GR * 144;
constexpr uint32_t TMEM_COLS = 512;     // NA accumulator buffers of GN columns
constexpr int kBuildWarps = 4, kEpiWarps = 8;
// Warpgroups: 0 = producer, MMA issuer, two idle warps; 1 = builders;
// 2-3 = epilogue. Registers are re-split per warpgroup with setmaxnreg
// (sum 128*56 + 128*80 + 256*184 = 64512 <= 512 threads * 128 at launch).
constexpr int kThreads = 512;
constexpr int kBuildWarp0 = 4, kEpiWarp0 = 8;

// Shared-memory map (offsets from a 1024-aligned base).
constexpr uint32_t OFF_X = 0;
constexpr uint32_t OFF_P = OFF_X + NX * X_STAGE;
constexpr uint32_t OFF_W = OFF_P + NP * P_STAGE;
constexpr uint32_t OFF_META = OFF_W + NW * W_STAGE;
constexpr uint32_t OFF_BAR = OFF_META + NMETA * GR * 8;
constexpr int NBAR = 2 * (NX + NW + NP + NMETA + NA);
static_assert(NA * 128 <= (int)TMEM_COLS, "accumulator buffers exceed the TMEM allocation");
constexpr uint32_t OFF_SLOT = OFF_BAR + NBAR * 8;
constexpr uint32_t SMEM_BYTES = OFF_SLOT + 16 + 1024;  // + alignment slack

#ifdef VTQ_GEMM_TRACE
__device__ long long g_gemm_trace[64][8];
#define GT(slot, s_)                                                              \
  do {                                                                            \
    if (blockIdx.x == 0 && (s_) < 64) g_gemm_trace[s_][slot] = clock64(); \
  } while (0)
#else
#define GT(slot, s_) (void)0
#endif

struct GemmParams {
  int M, n, S, R;
  int tiles_m, ntiles;  // token tiles; work units (token tile fastest, then row tile)
  float* y;
  int64_t ldy;
  const float* xd;  // [S][M] activation block scales (token-major per superblock)
  unsigned* status;
};

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* tm, int x, int y,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%2, %3}], [%4];" ::"r"(dst),
      "l"(tm), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// UMMA shared-memory descriptor, K-major, 128-byte swizzle: 8-row groups
// 1024 B apart (SBO), version 1, layout type 2.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3fffu);
  d |= (uint64_t)1 << 16;               // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;     // SBO
  d |= (uint64_t)1 << 46;               // descriptor version
  d |= (uint64_t)2 << 61;               // SWIZZLE_128B
  return d;
}

// Instruction descriptor: D s32, A s8 (activations), B u8 (planes), both
// K-major, N = GN, M = GM.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (0u << 10) | ((uint32_t)(GN >> 3) << 17) |
                            ((uint32_t)(GM >> 4) << 24);

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(kIdesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, int (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr));
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool wait_u32(uint32_t bar, uint32_t parity) {
  return mbar_wait_bounded(reinterpret_cast<uint64_t*>(__cvta_shared_to_generic(bar)), parity);
}

// Byte offset of (plane row nr, position k in [0, 256)) in a plane stage:
// two K-blocks of 128 positions, 8-row atoms of 1024 B, 16-byte chunks
// XOR-swizzled by the row within the atom (the TMA/UMMA 128B pattern).
__device__ __forceinline__ uint32_t plane_off(int nr, int k) {
  const int kb = k >> 7, chunk = (k & 127) >> 4;
  return (uint32_t)(kb * P_KBLK + (nr >> 3) * 1024 + (nr & 7) * 128 + ((chunk ^ (nr & 7)) << 4));
}

__device__ __forceinline__ float h2f(uint32_t bits) {
  return __half2float(__ushort_as_half((unsigned short)bits));
}

// Push leaf values v into the per-pair binary counters: merge with levels
// 0..tz-1 (older subtree on the left), store at level tz.
template <int LV, int TZ>
__device__ __forceinline__ void tree_push_tz(float (&st)[LV][16], float (&v)[16]) {
#pragma unroll
  for (int i = 0; i < 16; i++) {
    float c = v[i];
#pragma unroll
    for (int L = 0; L < TZ; L++) c = __fadd_rn(st[L][i], c);
    st[TZ][i] = c;
  }
}

template <int LV>
__device__ __forceinline__ void tree_push(float (&st)[LV][16], float (&v)[16], int tz) {
  switch (tz) {
    case 0: tree_push_tz<LV, 0>(st, v); break;
    case 1: tree_push_tz<LV, 1>(st, v); break;
    case 2: tree_push_tz<LV, 2>(st, v); break;
    case 3: tree_push_tz<LV, (3 < LV ? 3 : LV - 1)>(st, v); break;
    case 4: tree_push_tz<LV, (4 < LV ? 4 : LV - 1)>(st, v); break;
    case 5: tree_push_tz<LV, (5 < LV ? 5 : LV - 1)>(st, v); break;
    default: tree_push_tz<LV, LV - 1>(st, v); break;
  }
}

template <int LV>
__global__ void __launch_bounds__(kThreads, 1)
    kq_gemm_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw,
                   const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  uint8_t* gbase = smem_raw + (base - smem_u32(smem_raw));
  const uint32_t bar0 = base + OFF_BAR;
  auto X_FULL = [&](int i) { return bar0 + 8u * i; };
  auto X_EMPTY = [&](int i) { return bar0 + 8u * (NX + i); };
  auto W_FULL = [&](int i) { return bar0 + 8u * (2 * NX + i); };
  auto W_EMPTY = [&](int i) { return bar0 + 8u * (2 * NX + NW + i); };
  auto P_FULL = [&](int i) { return bar0 + 8u * (2 * NX + 2 * NW + i); };
  auto P_EMPTY = [&](int i) { return bar0 + 8u * (2 * NX + 2 * NW + NP + i); };
  auto M_FULL = [&](int i) { return bar0 + 8u * (2 * NX + 2 * NW + 2 * NP + i); };
  auto M_EMPTY = [&](int i) { return bar0 + 8u * (2 * NX + 2 * NW + 2 * NP + NMETA + i); };
  auto A_FULL = [&](int i) { return bar0 + 8u * (2 * NX + 2 * NW + 2 * NP + 2 * NMETA + i); };
  auto A_EMPTY = [&](int i) { return bar0 + 8u * (2 * NX + 2 * NW + 2 * NP + 2 * NMETA + NA + i); };
  volatile uint32_t* slot = reinterpret_cast<volatile uint32_t*>(gbase + OFF_SLOT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(gbase + OFF_SLOT + 4);
  float2* meta = reinterpret_cast<float2*>(gbase + OFF_META);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = p.S;
  // Persistent CTAs: unit u covers tokens [GM (u mod tiles_m), +GM) and rows
  // [GR (u div tiles_m), +GR). Every role walks the same units and counts
  // superblock steps g across them, so the pipeline (stages, TMEM buffers,
  // barrier phases) runs on from one unit into the next.

  if (tid == 0) {
    auto init = [](uint32_t b, unsigned c) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(b), "r"(c));
    };
    for (int i = 0; i < NX; i++) { init(X_FULL(i), 1); init(X_EMPTY(i), 1); }
    for (int i = 0; i < NW; i++) { init(W_FULL(i), 1); init(W_EMPTY(i), 32 * kBuildWarps); }
    for (int i = 0; i < NP; i++) { init(P_FULL(i), 32 * kBuildWarps); init(P_EMPTY(i), 1); }
    for (int i = 0; i < NMETA; i++) { init(M_FULL(i), 32 * kBuildWarps); init(M_EMPTY(i), kEpiWarps); }
    for (int i = 0; i < NA; i++) { init(A_FULL(i), 1); init(A_EMPTY(i), kEpiWarps); }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(base + OFF_SLOT),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;

  auto fail = [&]() {
    record_error(p.status, KERR_TIMEOUT);
    *abort_flag = 1;
  };

  if (warp == 0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 56;");
    // ---- producer ----
    if (lane == 0) {
      int g = 0;
      for (int u = blockIdx.x; u < p.ntiles && !*abort_flag; u += gridDim.x) {
      const int tok0 = (u % p.tiles_m) * GM, row0 = (u / p.tiles_m) * GR;
      for (int s = 0; s < S && !*abort_flag; s++, g++) {
        const int sx = g % NX, sw = g % NW;
        if (!wait_u32(X_EMPTY(sx), ((g / NX) + 1) & 1)) { fail(); break; }
        mbar_arrive_expect_tx(reinterpret_cast<uint64_t*>(gbase + OFF_BAR + 8 * sx), X_STAGE);
        const uint32_t xs = base + OFF_X + sx * X_STAGE;
        tma_load_2d(xs, &tmx, 256 * s, tok0, X_FULL(sx));
        tma_load_2d(xs + X_STAGE / 2, &tmx, 256 * s + 128, tok0, X_FULL(sx));
        if (!wait_u32(W_EMPTY(sw), ((g / NW) + 1) & 1)) { fail(); break; }
        mbar_arrive_expect_tx(reinterpret_cast<uint64_t*>(gbase + OFF_BAR + 8 * (2 * NX + sw)),
                              W_STAGE);
        tma_load_2d(base + OFF_W + sw * W_STAGE, &tmw, 144 * s, row0, W_FULL(sw));
        GT(0, g);
      }
      }
    }
  } else if (warp == 1) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 56;");
    // ---- MMA issuer ----
    if (lane == 0) {
      const int nsteps = ((p.ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x) * S;
      for (int g = 0; g < nsteps && !*abort_flag; g++) {
        const int s = g % S;
        const int sx = g % NX, sp = g % NP, ab = g % NA;
        bool ok = wait_u32(X_FULL(sx), (g / NX) & 1);
        GT(6, g);
        ok = ok && wait_u32(P_FULL(sp), (g / NP) & 1);
        GT(7, g);
        if (!ok || !wait_u32(A_EMPTY(ab), ((g / NA) + 1) & 1)) {
          fail();
          break;
        }
        tc_fence_after();
        GT(2, g);
        const uint32_t xs = base + OFF_X + sx * X_STAGE, ps = base + OFF_P + sp * P_STAGE;
        const uint32_t d = tmem + (uint32_t)ab * 128u;
#pragma unroll
        for (int c = 0; c < 8; c++) {
          const uint32_t kb = (uint32_t)(c >> 2), ko = (uint32_t)(c & 3) * 32u;
          mma_i8(d, desc_sw128(xs + kb * (X_STAGE / 2) + ko), desc_sw128(ps + kb * P_KBLK + ko),
                 c > 0 ? 1u : 0u);
        }
        mma_commit(X_EMPTY(sx));
        mma_commit(P_EMPTY(sp));
        mma_commit(A_FULL(ab));
      }
    }
  } else if (warp < kBuildWarp0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 56;");  // idle
  } else if (warp < kEpiWarp0) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 80;");
    // ---- plane builders: thread = (row r, sub-block pair jp = 2 jp, 2 jp + 1);
    // 8 consecutive lanes take 8 consecutive rows so that their 16-byte plane
    // stores land in 8 different swizzled slots of a 128-byte line ----
    const int t = tid - 32 * kBuildWarp0, r = t & 31, jp = t >> 5;
    // This thread's 12 plane offsets (3 planes x 2 sub-blocks x 2 halves) are
    // the same for every superblock.
    uint32_t poff[2][2][3];
#pragma unroll
    for (int h16 = 0; h16 < 2; h16++)
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const int k = 32 * (2 * jp + e) + 16 * h16;
        poff[h16][e][0] = plane_off(r, k);
        poff[h16][e][1] = plane_off(GR + r, k);
        poff[h16][e][2] = plane_off(2 * GR + r, k);
      }
    const int nsteps = ((p.ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x) * S;
    for (int g = 0; g < nsteps && !*abort_flag; g++) {
      const int s = g % S;
      const int sw = g % NW, sp = g % NP, sm = g % NMETA;
      if (t == 0) GT(5, g);
      if (!wait_u32(W_FULL(sw), (g / NW) & 1) || !wait_u32(P_EMPTY(sp), ((g / NP) + 1) & 1) ||
          !wait_u32(M_EMPTY(sm), ((g / NMETA) + 1) & 1)) {
        fail();
        break;
      }
      const uint8_t* sb = gbase + OFF_W + sw * W_STAGE + r * 144;
      const uint4 hdr = *reinterpret_cast<const uint4*>(sb);
      uint8_t* pl = gbase + OFF_P + sp * P_STAGE;
      if (jp == 0) meta[sm * GR + r] = make_float2(h2f(hdr.x & 0xffffu), h2f(hdr.x >> 16));
      {
      // get_scale_min_k4 (quant.rs:268-276) for sub-blocks 2 jp (low nibbles)
      // and 2 jp + 1 (high nibbles of the same 32 bytes).
      uint32_t sc[2], mn[2];
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const int j = 2 * jp + e;
        if (j < 4) {
          sc[e] = (hdr.y >> (8 * j)) & 63;
          mn[e] = (hdr.z >> (8 * j)) & 63;
        } else {
          const int k4 = j - 4;
          const uint32_t lo4 = (hdr.w >> (8 * k4)) & 0xff;
          sc[e] = (lo4 & 15) | (((hdr.y >> (8 * k4 + 6)) & 3) << 4);
          mn[e] = (lo4 >> 4) | (((hdr.z >> (8 * k4 + 6)) & 3) << 4);
        }
      }
      const uint8_t* qs = sb + 16 + 32 * jp;
#pragma unroll
      for (int h16 = 0; h16 < 2; h16++) {
        const uint4 w = *reinterpret_cast<const uint4*>(qs + 16 * h16);
        const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 2; e++) {
          const uint32_t sl = sc[e] & 7, sh = sc[e] >> 3;
          uint32_t lo[4], hi[4];
#pragma unroll
          for (int u = 0; u < 4; u++) {
            const uint32_t nib = e ? ((wv[u] >> 4) & 0x0F0F0F0Fu) : (wv[u] & 0x0F0F0F0Fu);
            lo[u] = nib * sl;  // byte products <= 105: no carries between bytes
            hi[u] = nib * sh;
          }
          const uint32_t mrep = mn[e] * 0x01010101u;
          *reinterpret_cast<uint4*>(pl + poff[h16][e][0]) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
          *reinterpret_cast<uint4*>(pl + poff[h16][e][1]) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
          *reinterpret_cast<uint4*>(pl + poff[h16][e][2]) = make_uint4(mrep, mrep, mrep, mrep);
        }
      }
      }
      // Generic-proxy stores -> visible to the tensor core (async proxy).
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      if (t == 0) GT(1, g);
      mbar_arrive(P_FULL(sp));
      mbar_arrive(M_FULL(sm));
      mbar_arrive(W_EMPTY(sw));
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 184;");
    // ---- epilogue: thread = token (TMEM lane), 16 weight rows ----
    const int ew = warp - kEpiWarp0;
    const int q = warp & 3, half = ew >> 2;
    const int rbase = 16 * half;
    int g = 0;
    // Token of this thread in unit u; the first block scale of the CTA's first
    // unit, then of each next unit during the current unit's last step.
    auto token_of = [&](int u) { return (u % p.tiles_m) * GM + 32 * q + lane; };
    float xd_next = 0.0f;
    if ((int)blockIdx.x < p.ntiles && token_of(blockIdx.x) < p.M) xd_next = p.xd[token_of(blockIdx.x)];
    for (int u = blockIdx.x; u < p.ntiles && !*abort_flag; u += gridDim.x) {
    const int tok0 = (u % p.tiles_m) * GM, row0 = (u / p.tiles_m) * GR;
    const int b = tok0 + 32 * q + lane;
    const bool bvalid = b < p.M;
    const int un = u + gridDim.x, bn = un < p.ntiles ? token_of(un) : p.M;
    float st[LV][16];
#pragma unroll
    for (int L = 0; L < LV; L++)
#pragma unroll
      for (int i = 0; i < 16; i++) st[L][i] = 0.0f;
    for (int s = 0; s < S && !*abort_flag; s++, g++) {
      const int ab = g % NA, sm = g % NMETA;
      const float xdv = xd_next;
      if (s + 1 < S) xd_next = bvalid ? p.xd[(int64_t)(s + 1) * p.M + b] : 0.0f;
      else xd_next = bn < p.M ? p.xd[bn] : 0.0f;
      if (!wait_u32(A_FULL(ab), (g / NA) & 1) || !wait_u32(M_FULL(sm), (g / NMETA) & 1)) {
        if (lane == 0) fail();
        break;
      }
      tc_fence_after();
      if (ew == 0 && lane == 0) GT(3, g);
      float part[16];
#pragma unroll
      for (int hh = 0; hh < 2; hh++) {
        const int rr = rbase + 8 * hh;
        const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)ab * 128u + (uint32_t)rr;
        int vlo[8], vhi[8], vmn[8];
        tmem_ld8(ta, vlo);
        tmem_ld8(ta + GR, vhi);
        tmem_ld8(ta + 2 * GR, vmn);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const float2 dm = meta[sm * GR + rr + i];
          const int acc = vlo[i] + (vhi[i] << 3);
          const float t0 = __fmul_rn(__fmul_rn(dm.x, xdv), __int2float_rn(acc));
          const float t1 = __fmul_rn(__fmul_rn(dm.y, xdv), __int2float_rn(vmn[i]));
          part[8 * hh + i] = __fsub_rn(t0, t1);
        }
      }
      // Binary counter over superblocks: level L holds a complete subtree of
      // 2^L leaves while bit L of the number of leaves seen (s) is set. Leaf s
      // merges with the levels below the lowest clear bit of s (warp-uniform).
      tree_push<LV>(st, part, __ffs(~s) - 1);
      if (ew == 0 && lane == 0) GT(4, g);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(A_EMPTY(ab));
        mbar_arrive(M_EMPTY(sm));
      }
    }
    if (!*abort_flag && bvalid) {
      // Remaining subtrees sit at the set bits of S; fold them right to left.
      float out[16];
#pragma unroll
      for (int i = 0; i < 16; i++) {
        float acc = 0.0f;
        bool have = false;
#pragma unroll
        for (int L = 0; L < LV; L++) {
          if ((S >> L) & 1) {
            acc = have ? __fadd_rn(st[L][i], acc) : st[L][i];
            have = true;
          }
        }
        out[i] = acc;
      }
      // This thread's 16 consecutive outputs of token b: four 16-byte stores
      // when they are whole and aligned, else one by one.
      const int o0 = row0 + rbase;
      float* yr = p.y + (int64_t)b * p.ldy + o0;
      if (o0 + 16 <= p.R && (reinterpret_cast<uintptr_t>(yr) & 15u) == 0) {
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          *reinterpret_cast<float4*>(yr + i) = make_float4(out[i], out[i + 1], out[i + 2], out[i + 3]);
      } else {
#pragma unroll
        for (int i = 0; i < 16; i++)
          if (o0 + i < p.R) yr[i] = out[i];
      }
    }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

// quantize_block_q8 (quant.rs:750-771) for every (row, 256-block): one warp
// per block, 8 contiguous elements per lane; int8 codes to xq [M][n], block
// scales to xd [S][M].
__global__ void quantize_rows_kernel(const float* __restrict__ x, int64_t ldx, int M, int n,
                                     int8_t* __restrict__ xq, float* __restrict__ xd) {
  const int S = n / 256;
  const int64_t u = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (u >= (int64_t)M * S) return;
  const int lane = threadIdx.x & 31;
  const int b = (int)(u / S), s = (int)(u - (int64_t)b * S);
  const float* src = x + (int64_t)b * ldx + 256 * s + 8 * lane;
  float v[8];
#pragma unroll
  for (int i = 0; i < 8; i++) v[i] = src[i];
  uint32_t am = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const uint32_t bits = __float_as_uint(v[i]) & 0x7fffffffu;
    if (bits <= 0x7f800000u) am = max(am, bits);
  }
  am = __reduce_max_sync(0xffffffffu, am);
  const float d = __fdiv_rn(__uint_as_float(am), 127.0f);
  const float inv = (d != 0.0f) ? __fdiv_rn(1.0f, d) : 0.0f;
  uint32_t w0 = 0, w1 = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const int qv = q8_round(__fmul_rn(v[i], inv));
    if (i < 4) w0 |= (uint32_t)(qv & 0xff) << (8 * i);
    else w1 |= (uint32_t)(qv & 0xff) << (8 * (i - 4));
  }
  *reinterpret_cast<uint2*>(xq + (int64_t)b * n + 256 * s + 8 * lane) = make_uint2(w0, w1);
  if (lane == 0) xd[(int64_t)s * M + b] = d;
}

typedef CUresult (*EncodeFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                             const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                             CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                             CUtensorMapFloatOOBfill);

EncodeFn encoder() {
  static EncodeFn fn = nullptr;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(f);
  }
  return fn;
}

// 2D byte tensor map [rows][cols] with row stride `pitch`.
cudaError_t byte_map(CUtensorMap* tm, const void* ptr, int64_t rows, int64_t cols, int64_t pitch,
                     uint32_t box_x, uint32_t box_y, CUtensorMapSwizzle sw) {
  EncodeFn enc = encoder();
  if (!enc) return cudaErrorInvalidValue;
  cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t gstride[1] = {(cuuint64_t)pitch};
  cuuint32_t box[2] = {box_x, box_y};
  cuuint32_t es[2] = {1, 1};
  return enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), gdim, gstride, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS
             ? cudaSuccess
             : cudaErrorInvalidValue;
}

// Scratch for the quantised activations, one buffer per (device, stream): GEMMs
// on different streams never share it, and work on one stream is ordered. A
// buffer that is outgrown is retired, not freed: launches already queued, and
// CUDA graphs captured with it, keep a valid pointer (the retired buffers are
// released at process exit).
struct Scratch {
  uint8_t* ptr = nullptr;
  size_t cap = 0;
};
std::mutex g_scratch_mu;
std::map<std::pair<int, cudaStream_t>, Scratch> g_scratch;
std::vector<uint8_t*> g_scratch_retired;
// Release every cached buffer when the library is unloaded (errors ignored:
// the CUDA context may already be gone at that point).
struct ScratchReaper {
  ~ScratchReaper() {
    for (auto& kv : g_scratch)
      if (kv.second.ptr) cudaFree(kv.second.ptr);
    for (uint8_t* p : g_scratch_retired) cudaFree(p);
  }
} g_scratch_reaper;

cudaError_t scratch(size_t bytes, cudaStream_t st, uint8_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  Scratch& sc = g_scratch[{dev, st}];
  if (sc.cap < bytes) {
    const size_t cap = (bytes + (1u << 20) - 1) & ~(size_t)((1u << 20) - 1);
    uint8_t* p = nullptr;
    cudaError_t e = cudaMalloc(&p, cap);
    if (e != cudaSuccess) return e;
    if (sc.ptr) g_scratch_retired.push_back(sc.ptr);
    sc.ptr = p;
    sc.cap = cap;
  }
  *out = sc.ptr;
  return cudaSuccess;
}

template <int LV>
cudaError_t launch_lv(const CUtensorMap& tmx, const CUtensorMap& tmw, const GemmParams& p, dim3 grid,
                      cudaStream_t st) {
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(kq_gemm_kernel<LV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)SMEM_BYTES);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  kernel_launch_count()++;
  kq_gemm_kernel<LV><<<grid, kThreads, SMEM_BYTES, st>>>(tmx, tmw, p);
  return cudaGetLastError();
}

}  // namespace

#ifdef VTQ_GEMM_TRACE
// Diagnostic build only: the per-role clock64 stamps of CTA 0's first 64 steps.
extern "C" int vtq_gemm_trace(long long* out) {
  return (int)cudaMemcpyFromSymbol(out, g_gemm_trace, sizeof(long long) * 64 * 8);
}
#endif

bool kq_gemm_supported(const DevMatrix& m, int64_t batch) {
  return m.dtype == T_Q4_K && batch >= 1 && batch <= (int64_t)INT32_MAX / 2 && m.in_feat % 256 == 0 &&
         m.in_feat / 256 < 128 && m.in_feat >= 256 && m.out_feat <= INT32_MAX &&
         (int64_t)SMEM_BYTES <= max_smem_optin();
}

size_t kq_gemm_workspace_bytes(int64_t in_feat, int64_t batch) {
  const size_t xq_bytes = ((size_t)batch * in_feat + 1023) & ~(size_t)1023;
  return xq_bytes + (size_t)batch * (in_feat / 256) * 4;
}

cudaError_t launch_kq_gemm(const DevMatrix& m, const float* x, int64_t ldx, int64_t batch, float* y,
                           int64_t ldy, unsigned* status, cudaStream_t st, uint8_t* ws,
                           size_t ws_bytes) {
  if (!kq_gemm_supported(m, batch)) return cudaErrorInvalidValue;
  const int n = (int)m.in_feat, S = n / 256, M = (int)batch, R = (int)m.out_feat;
  const size_t xq_bytes = ((size_t)M * n + 1023) & ~(size_t)1023;
  const size_t need = kq_gemm_workspace_bytes(n, M);
  uint8_t* buf = ws;
  cudaError_t e = cudaSuccess;
  if (ws) {
    if (ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 255u)) return cudaErrorInvalidValue;
  } else if ((e = scratch(need, st, &buf)) != cudaSuccess) {
    return e;
  }
  int8_t* xq = reinterpret_cast<int8_t*>(buf);
  float* xd = reinterpret_cast<float*>(buf + xq_bytes);
  {
    const int64_t blocks = ((int64_t)M * S + 7) / 8;
    kernel_launch_count()++;
    quantize_rows_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, ldx, M, n, xq, xd);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  CUtensorMap tmx, tmw;
  if ((e = byte_map(&tmx, xq, M, n, n, 128, GM, CU_TENSOR_MAP_SWIZZLE_128B)) != cudaSuccess) return e;
  if ((e = byte_map(&tmw, m.data, R, m.pitch, m.pitch, 144, GR, CU_TENSOR_MAP_SWIZZLE_NONE)) !=
      cudaSuccess)
    return e;
  const int tiles_m = (M + GM - 1) / GM, ntiles = tiles_m * ((R + GR - 1) / GR);
  GemmParams p{M, n, S, R, tiles_m, ntiles, y, ldy, xd, status};
  // Persistent: at most one CTA per SM, each walking units gridDim.x apart.
  const dim3 grid((unsigned)std::min(ntiles, num_sms()));
  // Levels of the fixed-tree counter: floor(log2 S) + 1.
  int lv = 1;
  while ((1 << lv) <= S) lv++;
  if (lv <= 4) return launch_lv<4>(tmx, tmw, p, grid, st);
  if (lv == 5) return launch_lv<5>(tmx, tmw, p, grid, st);
  if (lv == 6) return launch_lv<6>(tmx, tmw, p, grid, st);
  return launch_lv<7>(tmx, tmw, p, grid, st);
}

}  // namespace vtq
