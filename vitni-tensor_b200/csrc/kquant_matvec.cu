// kquant_matvec.cu -- exact-integer Q4_K / Q6_K matvec for sm_100a.
//
// Computes, bit for bit, vitni-tensor's integer linears
//   linear_q4_k_integer(_parallel)  src/ops/quant.rs:936-980, :1149-1196
//   linear_q6_k_integer(_parallel)  src/ops/quant.rs:1060-1146
// y[b, r] = fixed_tree_s( blockdot(W[r, s], quantize_block_q8(x[b, 256s..])) ).
//
// Design (one persistent CTA per SM: 8 consumer warps + 1 TMA producer warp):
//  * Each CTA owns a contiguous range of output rows, i.e. one contiguous byte
//    range of the weight matrix in HBM. The producer warp streams it into a
//    shared-memory ring of whole-row stages with TMA bulk copies
//    (cp.async.bulk, mbarrier complete_tx, L2 evict-first). full/empty
//    mbarrier pairs decouple it from the consumers; small matrices are
//    requested in full at kernel entry.
//  * Meanwhile the consumer warps quantise the activation rows into shared
//    memory (quantize_block_q8, quant.rs:750-771, restated with __fdiv_rn /
//    __fmul_rn / __fadd_rn and cvt.rzi -- the same bits in every CTA, so the
//    reference's once-per-call quantisation is reproduced). Activation blocks
//    are padded to 272 B so that lanes reading different superblocks at the
//    same offset hit different shared-memory banks.
//  * One lane owns one whole superblock of one row: it unpacks the quants
//    with masks/shifts and forms exact int32 dots with dp4a, so scale decoding
//    happens once per superblock and no cross-lane integer reduction is
//    needed. A row's S superblocks sit on S consecutive lanes (a warp holds
//    32/S rows when S <= 16); S > 32 puts up to 4 superblocks on a lane.
//  * The per-superblock fp combine (quant.rs:897 / :1056) and the
//    cross-superblock fixed_tree (quant.rs:462) are the only order-pinned
//    steps; both use explicit round-to-nearest intrinsics (no contraction).
//    The tree is a stride-doubling shuffle tree over the row's lanes whose
//    pairing is identical to the reference's level-wise loop.
#include "kq_core.cuh"

namespace vtq {
namespace {

#ifdef VTQ_TRACE
// Diagnostic build only: per-CTA %globaltimer stamps for up to 8 launches,
// selected by their output pointer (set by a host-side probe).
__device__ unsigned long long g_kq_trace[8][1024][8];
__device__ const float* g_kq_trace_y[8];
__device__ unsigned long long g_kq_arrive[8][1024][16];  // stage k full (k < 15), 15: x ready
#define KQ_TRACE(slot)                                                      \
  do {                                                                      \
    for (int ti_ = 0; ti_ < 8; ti_++)                                       \
      if (g_kq_trace_y[ti_] == p.y) g_kq_trace[ti_][blockIdx.x][slot] = globaltimer(); \
  } while (0)
#define KQ_ARRIVE(k)                                                        \
  do {                                                                      \
    for (int ti_ = 0; ti_ < 8; ti_++)                                       \
      if (g_kq_trace_y[ti_] == p.y && (k) < 16) g_kq_arrive[ti_][blockIdx.x][k] = globaltimer(); \
  } while (0)
#else
#define KQ_TRACE(slot) (void)0
#define KQ_ARRIVE(k) (void)0
#endif

#ifndef VTQ_KQ_CTAS
#define VTQ_KQ_CTAS 1
#endif
#ifndef VTQ_KQ_XMAX
#define VTQ_KQ_XMAX 65536
#endif
#ifndef VTQ_KQ_CW1
#define VTQ_KQ_CW1 16
#endif

template <int QT, int MAXB, int NCH, int CW>
__global__ void __launch_bounds__((CW + 1) * 32, VTQ_KQ_CTAS) kq_matvec_kernel(const KqParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + KQ_NST_MAX;
  uint64_t* xbar = empty + KQ_NST_MAX;
  float* xd = reinterpret_cast<float*>(smem + p.off_xd);
  int* bsum = reinterpret_cast<int*>(smem + p.off_bsum);
  int8_t* xq = reinterpret_cast<int8_t*>(smem + p.off_xq);
  float* xf = reinterpret_cast<float*>(smem + p.off_xf);
  float* ystage = reinterpret_cast<float*>(smem + p.off_ystage);
  uint8_t* stg = smem + p.off_stage;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bid = blockIdx.x;
  const int unit = p.epi ? 2 : 1;  // rows are dealt to CTAs in (gate, up) pairs for the epilogue
  const int r0 = unit * (bid * p.rows_base + min(bid, p.rows_rem));
  const int nrows = unit * (p.rows_base + (bid < p.rows_rem ? 1 : 0));
  const int nstages = (nrows + p.rps - 1) / p.rps;

  if (tid == 0) {
    KQ_TRACE(0);
    for (int i = 0; i < p.nst; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], CW);
    }
    mbar_init(xbar, 1);
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == CW) {
    // ---- producer: one thread streams x, then the CTA's rows, through TMA ----
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      auto issue = [&](int k) {
        const int buf = k % p.nst;
        const int ra = k * p.rps, rb = min(ra + p.rps, nrows);
        const uint32_t bytes = (uint32_t)((rb - ra) * p.pitch);
        mbar_arrive_expect_tx(&full[buf], bytes);
        bulk_g2s_stream(stg + (size_t)buf * p.stage_bytes, p.W + (int64_t)(r0 + ra) * p.pitch,
                        bytes, &full[buf], pol);
      };
      // Weights are never written by a preceding kernel: stream the first
      // stages before waiting on the previous grid (programmatic launch).
      const int first = min(p.nst, nstages);
      if (first > 0) issue(0);
      KQ_TRACE(6);
      grid_dep_wait();
      KQ_TRACE(7);
      if (p.x_smem) {
        const uint32_t rowb = (uint32_t)p.n * 4u;
        mbar_arrive_expect_tx(xbar, rowb * p.batch);
        for (int b = 0; b < p.batch; b++) bulk_g2s(xf + (size_t)b * p.n, p.x + b * p.ldx, rowb, xbar);
      }
      for (int k = 1; k < first; k++) issue(k);
      KQ_TRACE(1);
      grid_dep_launch();
      for (int k = first; k < nstages; k++) {
        const int buf = k % p.nst;
        if (!mbar_wait_bounded(&empty[buf], (uint32_t)(((k / p.nst) - 1) & 1))) {
          record_error(p.status, KERR_TIMEOUT);
          for (int j = max(0, k - p.nst); j < k; j++)  // drain copies already issued
            mbar_wait_bounded(&full[j % p.nst], (uint32_t)((j / p.nst) & 1));
          if (p.x_smem) mbar_wait_bounded(xbar, 0);
          return;
        }
        issue(k);
      }
    }
    return;
  }

  // ---- consumers ----
  const float* xs = p.x;
  int64_t xstride = p.ldx;
  if (p.x_smem) {
    if (!mbar_wait_bounded(xbar, 0)) {
      if (lane == 0) record_error(p.status, KERR_TIMEOUT);
      return;
    }
    xs = xf;
    xstride = p.n;
    if (tid == 0) KQ_TRACE(4);
  } else {
    grid_dep_wait();
  }
  float xscale = 0.0f;
  if (p.xf.kind == 2) {
    // Fused RMSNorm: v = x (+ delta) in place, squares beside it, then the
    // left-to-right sum of the squares (exact_serial_sum: the CTA computes
    // the serial result) while the weight stages keep streaming in.
    float* xsq = reinterpret_cast<float*>(smem + p.off_xsq);
    // The scale lives in the reserved head of the dynamic block (after the
    // barriers): no static shared memory, so the dynamic size may use the
    // whole opt-in limit.
    float& s_scale = *reinterpret_cast<float*>(smem + kScaleOff);
    for (int i = tid; i < p.n; i += CW * 32) {
      float v = xf[i];
      if (p.xf.delta) v = __fadd_rn(v, p.xf.delta[i]);
      xf[i] = v;
      xsq[i] = __fmul_rn(v, v);
      if (p.xf.res_out && blockIdx.x == 0) p.xf.res_out[i] = v;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(CW * 32));
    auto* xs_scr = reinterpret_cast<xsum::Scratch*>(smem + p.off_xsq +
                                                    ((uint32_t)p.n * 4 + 127) / 128 * 128);
    const float sum = xsum::exact_serial_sum<8>(xsq, p.n, xs_scr, tid, CW * 32, [] {
      asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory");
    });
    if (tid == 0) {
      const float mean = __fdiv_rn(sum, (float)p.n);
      s_scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, p.xf.eps)));
    }
    asm volatile("bar.sync 1, %0;" ::"n"(CW * 32));
    xscale = s_scale;
  }
  quantize_x<QT == 0 ? 8 : 16, CW>(p, xs, xstride, warp, lane, xd, bsum, xq, xscale);
  asm volatile("bar.sync 1, %0;" ::"n"(CW * 32));
  if (tid == 0) KQ_TRACE(2);

  // Row groups of rpw rows (one warp pass) are dealt to warps round-robin
  // across the whole CTA range, so warps work on different stages at once.
  const int rpw = 32 / p.lpr;
  const int seg = lane / p.lpr, sl = lane - seg * p.lpr;
  const int gps = p.rps / rpw;  // groups per stage
  int g = warp;                 // next group of this warp
  for (int k = 0; k < nstages; k++) {
    const int buf = k % p.nst;
    const int gend = min((k + 1) * gps, (nrows + rpw - 1) / rpw);
    // Every warp waits for every stage in order, also for stages where it
    // has no rows: a parity wait is only unambiguous one phase ahead, so a
    // warp that first waited on stage k + nst (same buffer, other parity)
    // would pass on the barrier's initial state. The in-order waits also
    // keep the CTA alive until all of its bulk copies have landed.
    if (!mbar_wait_bounded(&full[buf], (uint32_t)((k / p.nst) & 1))) {
      if (lane == 0) record_error(p.status, KERR_TIMEOUT);
      return;
    }
    if (tid == 0 && k < 15) KQ_ARRIVE(k);
    if (g < gend) {
      if (tid == 0 && k == 0) KQ_TRACE(3);
      const uint8_t* sbuf = stg + (size_t)buf * p.stage_bytes;
      for (; g < gend; g += CW) {
        const int r = g * rpw + seg;  // CTA-local row
        consume_pass<QT, MAXB, NCH>(p, sbuf, r - k * p.rps, r < nrows, sl, r0 + r, xq, xd, bsum,
                                    ystage, r0);
      }
    }
    __syncwarp();
    if (lane == 0) {
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&empty[buf]))
                   : "memory");
    }
  }
  if (tid == 0) KQ_TRACE(5);
  if (p.g.world > 0) {
    // Send: after every consumer has staged its rows, warp 0 writes the CTA's
    // contiguous rows into every rank's y (coalesced, over NVLink for peers).
    // The launch's last CTA (completion counter in this rank's memory) then
    // fences at system scope, signals every rank once and, if asked, waits
    // for the other ranks.
    asm volatile("bar.sync 1, %0;" ::"n"(CW * 32));
    if (warp == 0) {
      for (int b = 0; b < p.batch; b++)
        for (int i = lane; i < nrows; i += 32) {
          const float v = ystage[b * (p.rows_base + 1) + i];
          const int64_t at = (int64_t)b * p.g.ldy + p.g.row0 + r0 + i;
#pragma unroll
          for (int q = 0; q < kMaxRanks; q++)
            if (q < p.g.world) p.g.y[q][at] = v;
        }
      // Ordering: each CTA's stores reach lane 0 through __syncwarp, lane 0's
      // acq_rel add on the completion counter (GPU scope) chains every CTA
      // into the last one, whose system-scope fence then covers all of them
      // before the arrival signals (causality order is transitive).
      __syncwarp();
      if (lane == 0 && p.g.signal) {
        unsigned prev;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(p.g.done)
                     : "memory");
        if (prev == gridDim.x - 1) {
          *p.g.done = 0;  // every CTA of this launch has counted
          __threadfence_system();
#pragma unroll
          for (int q = 0; q < kMaxRanks; q++)
            if (q < p.g.world) atomicAdd_system(p.g.cnt[q], 1u);
          if (p.g.wait_signals) {
            const unsigned target = *p.g.expected + p.g.wait_signals;
            const uint64_t t0 = globaltimer();
            bool ok = true;
            for (;;) {
              unsigned v;
              asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p.g.my_cnt)
                           : "memory");
              if ((int)(v - target) >= 0) break;
              if (globaltimer() - t0 > p.g.limit_ns) {
                record_error(p.status, KERR_TIMEOUT);
                ok = false;  // the missing arrivals are not counted as consumed
                break;
              }
            }
            if (ok) *p.g.expected = target;
            __threadfence_system();
          }
        }
      }
    }
  }
}

bool use_pdl() { return pdl_enabled(); }

template <int QT, int MAXB, int NCH, int CW>
cudaError_t launch_variant(const KqParams& p, int grid, uint32_t smem, cudaStream_t st) {
  static bool attr_set = false;  // opt-in shared memory, once per instantiation
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kq_matvec_kernel<QT, MAXB, NCH, CW>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         max_smem_optin());
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3((CW + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = use_pdl() ? 1 : 0;
  kernel_launch_count()++;
  return cudaLaunchKernelEx(&cfg, kq_matvec_kernel<QT, MAXB, NCH, CW>, p);
}

template <int QT, int MAXB>
cudaError_t launch_nch(const KqParams& p, int grid, uint32_t smem, cudaStream_t st) {
  const int nch = (p.S + 31) / 32;
  constexpr int CW = MAXB <= 1 ? VTQ_KQ_CW1 : (MAXB <= 2 ? 16 : 8);
  if (nch <= 1) return launch_variant<QT, MAXB, 1, CW>(p, grid, smem, st);
  if (nch == 2) return launch_variant<QT, MAXB, 2, CW>(p, grid, smem, st);
  return launch_variant<QT, MAXB, 4, CW>(p, grid, smem, st);
}

template <int QT>
cudaError_t launch_qt(const KqParams& p, int grid, uint32_t smem, cudaStream_t st) {
  if (p.batch <= 1) return launch_nch<QT, 1>(p, grid, smem, st);
  if (p.batch <= 2) return launch_nch<QT, 2>(p, grid, smem, st);
  return launch_nch<QT, 4>(p, grid, smem, st);
}

}  // namespace

bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = getenv("VTQ_NO_PDL");
    v = (e && *e && *e != '0') ? 0 : 1;
  }
  return v == 1;
}

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
                             float* y, int64_t ldy, unsigned* status, cudaStream_t st,
                             const GatherTarget* g, const KqXform* xform) {
  constexpr int KQ_BMAX = 4;  // activation rows per launch
  if (m.dtype != T_Q4_K && m.dtype != T_Q6_K) return cudaErrorInvalidValue;
  const int S = (int)(m.in_feat / 256);
  if (S < 1 || S > KQ_SMAX || m.in_feat % 256) return cudaErrorInvalidValue;
  if (m.out_feat <= 0 || batch <= 0) return cudaSuccess;
  int smem_max = max_smem_optin();
  if (VTQ_KQ_CTAS == 2) {
    int dev = 0, per_sm = 0, resv = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&resv, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    smem_max = std::min(smem_max, per_sm / 2 - resv);
  }
  const int nsm = num_sms();
  int lpr = 1;
  while (lpr < S && lpr < 32) lpr <<= 1;
  const int rpw = 32 / lpr;
  const int grid = (int)std::min<int64_t>(m.out_feat, nsm);
  for (int64_t b0 = 0; b0 < batch; b0 += KQ_BMAX) {
    int grid_l = grid;
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
    p.rows_base = p.R / grid;
    p.rows_rem = p.R % grid;
    p.y = y + b0 * ldy;
    p.ldy = ldy;
    p.status = status;
    if (g) {
      if (g->world < 1 || g->world > kMaxRanks || batch > KQ_BMAX) return cudaErrorInvalidValue;
      p.g = *g;
    }
    if (xform && xform->kind) {
      if (batch != 1 || xform->kind != 2 || !xform->nw) return cudaErrorInvalidValue;
      p.xf = *xform;
    }
    if (xform && xform->swiglu_pairs) {
      // Rows interleaved (gate_i, up_i): pairs dealt to CTAs, both rows of a
      // pair in one warp pass.
      if (g || p.R % 2 || rpw < 2) return cudaErrorInvalidValue;
      p.epi = 1;
      const int gp = std::min(p.R / 2, nsm);
      p.rows_base = (p.R / 2) / gp;
      p.rows_rem = (p.R / 2) % gp;
      grid_l = gp;
    }
    p.lpr = lpr;
    const int NB = m.dtype == T_Q4_K ? BsumStride<8>::v : BsumStride<16>::v;
    constexpr uint32_t kBarBytes = (2 * KQ_NST_MAX + 1) * 8;  // full[], empty[], xbar
    static_assert(kBarBytes <= kScaleOff && kScaleOff + 4 <= 512, "barrier area");
    uint32_t off = 512;  // mbarriers (kBarBytes) live below this offset
    p.off_xd = off;
    off = align_up(off + nb * S * 4, 16);
    p.off_bsum = off;
    off = align_up(off + nb * S * NB * 4, 16);
    p.off_xq = off;
    off = align_up(off + nb * S * XQ_STRIDE, 128);
    // Stage x through TMA when every row start is 16-byte aligned and it fits.
    const uint32_t xbytes = (uint32_t)(nb * p.n * 4);
    p.x_smem = ((reinterpret_cast<uintptr_t>(p.x) & 15u) == 0 && (ldx % 4) == 0 &&
                xbytes <= (uint32_t)VTQ_KQ_XMAX) ? 1 : 0;
    p.off_xf = off;
    if (p.x_smem) off = align_up(off + xbytes, 128);
    if (p.xf.kind == 2) {
      if (!p.x_smem) return cudaErrorInvalidValue;  // the fused norm works on the staged row
      p.off_xsq = off;  // squares, then the scratch of the CTA-wide exact sum
      off = align_up(off + align_up((uint32_t)p.n * 4, 128) + (uint32_t)sizeof(xsum::Scratch), 128);
    }
    if (p.g.world > 0) {
      p.off_ystage = off;
      off = align_up(off + (uint32_t)(nb * (p.rows_base + 1)) * 4, 128);
    }
    p.off_stage = off;
    // Stages of ~24 KB of whole warp passes (TMA streams at full rate from 16 KB).
    const int rows_per_cta = (p.epi ? 2 : 1) * (p.rows_base + (p.rows_rem ? 1 : 0));
    int rps = std::max(rpw, (int)(24576 / m.pitch) / rpw * rpw);
    rps = std::min(rps, (rows_per_cta + rpw - 1) / rpw * rpw);
    int nst;
    for (;;) {
      const uint32_t stage_bytes = (uint32_t)(rps * m.pitch);
      const int avail = smem_max - (int)off;
      nst = std::min<int>(KQ_NST_MAX, avail > 0 ? avail / (int)stage_bytes : 0);
      const int need = (rows_per_cta + rps - 1) / rps;  // stages per CTA
      nst = std::min(nst, std::max(need, 1));
      if (nst >= 2 || (nst >= 1 && need <= 1)) {
        p.stage_bytes = stage_bytes;
        break;
      }
      if (rps <= rpw) return cudaErrorInvalidValue;  // rows too long for shared memory
      rps = std::max(rpw, rps / 2 / rpw * rpw);
    }
    p.rps = rps;
    p.nst = nst;
    const uint32_t smem = p.off_stage + (uint32_t)nst * p.stage_bytes;
    const cudaError_t e = m.dtype == T_Q4_K ? launch_qt<0>(p, grid_l, smem, st)
                                            : launch_qt<1>(p, grid_l, smem, st);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace vtq
