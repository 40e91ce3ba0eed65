// kquant_list.cu -- one persistent launch over a list of integer k-quant
// linears (Q4_K / Q6_K, batch 1).
//
// Each item is exactly linear_q4_k_integer / linear_q6_k_integer
// (vitni-tensor src/ops/quant.rs:936-980, :1060-1146) on its own activation
// row; items run in list order, as consecutive linear_dispatch calls of a
// layer do (src/model/forward_quantized.rs:663-785). The arithmetic of every
// output row is the single matvec's (kq_core.cuh: quantize_x, the superblock
// dots, seg_fixed_tree), so every item's y is bit-identical to vtq_linear.
//
// Why a list kernel: a matvec launch on B200 loses ~2-3 us at every kernel
// boundary (CTA exit, next CTA start, first-byte latency of the weight
// stream), which is a third of a 25 MB matvec. Here one CTA per SM walks the
// items in order and its producer warp streams all of its weight rows,
// item after item, through one shared-memory ring: the next item's weights
// arrive while the consumers still work on the current one, so HBM never
// idles at an item boundary.
//
// Activation quantisation: the activations of the items that need no earlier
// item (x ready at launch) are quantised ONCE per launch, not once per CTA:
// the launch's consumer warps share those blocks out, write each block's
// int8 codes, scale and sums (quantize_block_q8, quant.rs:750-771) to a
// per-item record in global memory, and publish them through a counter; a
// CTA then copies an item's record (~1.2 bytes per input) into shared memory
// before its rows. Weight streaming runs on throughout.
//
// Dependencies: an item may name an earlier item (wait_for) whose y is its
// activation. Every CTA, after storing its rows of an item that others wait
// for, adds 1 to that item's completion counter (release, GPU scope); a
// consumer about to quantise a dependent item's x polls the counter until
// every CTA has arrived (acquire, bounded by VTQ_WAIT_LIMIT_NS) and then reads
// x at L2. The producer keeps streaming weights during that wait. The last CTA
// to leave resets the counters, so a list can be replayed (CUDA graphs) with
// no host work; the next launch on the stream touches them only after
// griddepcontrol.wait, i.e. after this launch has completed.
#include "kq_core.cuh"

namespace vtq {
namespace {

#ifndef VTQ_LIST_CW
#define VTQ_LIST_CW 16
#endif
#ifndef VTQ_LIST_SLOTS
#define VTQ_LIST_SLOTS 8
#endif
constexpr int CWL = VTQ_LIST_CW;        // consumer warps
constexpr int NSLOT = VTQ_LIST_SLOTS;   // ring slots; slot j is consumed by warp group j only
constexpr int WPG = CWL / NSLOT;        // warps per slot group
static_assert(CWL % NSLOT == 0 && NSLOT <= KQ_NST_MAX, "slot groups");

struct KqLItem {
  const uint8_t* W;
  const float* x;
  float* y;
  int pitch, R, S, qt, lpr, nch, rps, rows_base, rows_rem, wait_for, signal;
  int qbase;  // first global block index of this item's pre-quantisation (-1: dependent item)
  int send;   // gathered list: this item's rows go to the other ranks (last item writing its y)
};

// Global record of one item's quantised activation: [xd | bsum | xq], the
// same three arrays (and strides) as the shared-memory copy.
__host__ __device__ constexpr uint32_t rec_bsum_off(int S) { return ((uint32_t)S * 4 + 15) / 16 * 16; }
__host__ __device__ constexpr uint32_t rec_xq_off(int S, int nbs) {
  return rec_bsum_off(S) + (uint32_t)S * nbs * 4;
}

struct KqListParams {
  KqLItem it[KQ_LIST_MAX];
  int n;
  uint32_t slot;
  uint32_t off_x[2], off_stage;  // two activation buffers, then the ring
  unsigned* cnt;  // [KQ_LIST_MAX] completion counters, the exit counter, the x-ready counter
  unsigned* status;
  uint8_t* xrec;  // KQ_LIST_MAX records of KQ_LIST_REC bytes
  unsigned* hstatus;  // optional host-mapped word: the last CTA copies *status there
  int nq;         // blocks to pre-quantise (sum of S over independent items)
  KqListGather g;  // g.world > 0: every y row also goes to every other rank
};

__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(CWL * 32) : "memory");
}

// The warp passes (rpw rows each) of one ring stage of one item that fall to
// warp `wig` of the stage's slot group.
template <int QT, int NCH>
__device__ __forceinline__ void stage_passes(const KqParams& p, const uint8_t* sbuf, int st,
                                             int wig, int nrows, int r0, int sl, int seg,
                                             const int8_t* xq, const float* xd, const int* bsum) {
  const int rpw = 32 / p.lpr;
  const int rows = min(p.rps, nrows - st * p.rps);
  for (int pr = wig * rpw; pr < rows; pr += WPG * rpw) {
    const int r = st * p.rps + pr + seg;  // CTA-local row
    consume_pass<QT, 1, NCH>(p, sbuf, pr + seg, pr + seg < rows, sl, r0 + r, xq, xd, bsum,
                             nullptr, r0);
  }
}

// Byte size of an item's quantised-activation record (and of its copy in one
// of the two shared-memory activation buffers).
__host__ __device__ constexpr uint32_t rec_bytes(int S, int nbs) {
  return rec_xq_off(S, nbs) + (uint32_t)S * XQ_STRIDE;
}

__device__ __forceinline__ bool poll_count(const unsigned* c, unsigned target) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(c) : "memory");
  return v >= target;
}

// Bounded wait until *c >= target (acquire, GPU scope). False on timeout.
__device__ __forceinline__ bool wait_count(const unsigned* c, unsigned target) {
  if (poll_count(c, target)) return true;
  const uint64_t t0 = globaltimer();
  while (!poll_count(c, target))
    if (globaltimer() - t0 > VTQ_WAIT_LIMIT_NS) return false;
  return true;
}

__global__ void __launch_bounds__((CWL + 1) * 32, 1) kq_list_kernel(const __grid_constant__ KqListParams P) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);  // ring slots
  uint64_t* empty = full + KQ_NST_MAX;
  uint64_t* xfull = empty + KQ_NST_MAX;                // activation buffers
  uint64_t* xempty = xfull + 2;
  int* s_abort = reinterpret_cast<int*>(smem + kScaleOff);
  uint8_t* ring = smem + P.off_stage;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bid = blockIdx.x, grid = gridDim.x;
  unsigned* const qx_cnt = P.cnt + KQ_LIST_MAX + 1;

  if (tid == 0) {
    for (int i = 0; i < NSLOT; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], WPG);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&xfull[b], 1);
      mbar_init(&xempty[b], CWL);
    }
    *s_abort = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == CWL) {
    // ---- producer: for every item with rows here, in list order, the
    // item's quantised activation record (independent items) into activation
    // buffer i & 1, then the CTA's weight rows through the ring ----
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      bool qx_ready = P.nq == 0;
      int k = 0, uses[2] = {0, 0};
      bool failed = false;
      for (int i = 0; i < P.n && !failed; i++) {
        const KqLItem& it = P.it[i];
        const int r0 = bid * it.rows_base + min(bid, it.rows_rem);
        const int nrows = it.rows_base + (bid < it.rows_rem ? 1 : 0);
        if (nrows == 0) continue;
        const int b = i & 1;
        // The buffer's previous use must be finished by every consumer warp.
        if (uses[b] > 0 && !mbar_wait_bounded(&xempty[b], (uint32_t)((uses[b] - 1) & 1))) {
          failed = true;
          break;
        }
        uses[b]++;
        int pend = it.wait_for < 0 ? i : -1;
        auto issue_record = [&]() {
          const uint32_t bytes = rec_bytes(it.S, it.qt == 0 ? BsumStride<8>::v : BsumStride<16>::v);
          mbar_arrive_expect_tx(&xfull[b], bytes);
          bulk_g2s(smem + P.off_x[b], P.xrec + (size_t)i * KQ_LIST_REC, bytes, &xfull[b]);
          pend = -1;
        };
        for (int ra = 0; ra < nrows; ra += it.rps, k++) {
          const int buf = k % NSLOT;
          if (pend >= 0) {
            if (!qx_ready && poll_count(qx_cnt, (unsigned)grid)) {
              // Records were written by generic stores of other CTAs; order
              // them before this thread's bulk (async-proxy) reads.
              asm volatile("fence.proxy.async.global;" ::: "memory");
              qx_ready = true;
            }
            if (!qx_ready && k >= NSLOT && !mbar_try_wait(&empty[buf], (uint32_t)(((k / NSLOT) - 1) & 1))) {
              // The ring is full and its consumers need this record first.
              if (!wait_count(qx_cnt, (unsigned)grid)) {
                failed = true;
                break;
              }
              asm volatile("fence.proxy.async.global;" ::: "memory");
              qx_ready = true;
            }
            if (qx_ready) issue_record();
          }
          if (k >= NSLOT && !mbar_wait_bounded(&empty[buf], (uint32_t)(((k / NSLOT) - 1) & 1))) {
            failed = true;
            break;
          }
          const uint32_t bytes = (uint32_t)(min(it.rps, nrows - ra) * it.pitch);
          mbar_arrive_expect_tx(&full[buf], bytes);
          bulk_g2s_stream(ring + (size_t)buf * P.slot, it.W + (int64_t)(r0 + ra) * it.pitch,
                          bytes, &full[buf], pol);
          // Weights are never written by a preceding kernel, so they stream
          // before griddepcontrol.wait; the next launch may start early.
          if (k == 0) grid_dep_launch();
        }
        if (pend >= 0 && !failed) {
          // Every stage of the item is issued; its consumers need the record.
          if (!qx_ready) {
            if (!wait_count(qx_cnt, (unsigned)grid)) {
              failed = true;
              break;
            }
            asm volatile("fence.proxy.async.global;" ::: "memory");
            qx_ready = true;
          }
          issue_record();
        }
      }
      if (failed) {
        record_error(P.status, KERR_TIMEOUT);
        for (int j = max(0, k - NSLOT); j < k; j++)  // drain the weight copies in flight
          mbar_wait_bounded(&full[j % NSLOT], (uint32_t)((j / NSLOT) & 1));
      }
      if (k == 0) grid_dep_launch();
    }
    return;
  }

  // ---- consumers ----
  grid_dep_wait();  // x (and the counters) may be written by the previous kernel
  // Pre-quantisation of the independent items, shared out over every
  // consumer warp of the launch (one 256-element block per warp pass).
  if (P.nq > 0) {
    for (int u = bid * CWL + warp; u < P.nq; u += grid * CWL) {
      int i = 0;
      while (P.it[i].qbase < 0 || u >= P.it[i].qbase + P.it[i].S) i++;
      const KqLItem& it = P.it[i];
      const int s = u - it.qbase;
      const float* src = it.x + s * 256 + lane * 8;
      float v[8];
      if ((reinterpret_cast<uintptr_t>(it.x) & 15u) == 0) {
        const float4 a = *reinterpret_cast<const float4*>(src);
        const float4 c = *(reinterpret_cast<const float4*>(src) + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
      } else {
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = src[e];
      }
      uint8_t* rec = P.xrec + (size_t)i * KQ_LIST_REC;
      if (it.qt == 0)
        quant_block<8>(v, lane, reinterpret_cast<int8_t*>(rec + rec_xq_off(it.S, BsumStride<8>::v)) + s * XQ_STRIDE,
                       reinterpret_cast<int*>(rec + rec_bsum_off(it.S)) + s * BsumStride<8>::v,
                       reinterpret_cast<float*>(rec) + s);
      else
        quant_block<16>(v, lane, reinterpret_cast<int8_t*>(rec + rec_xq_off(it.S, BsumStride<16>::v)) + s * XQ_STRIDE,
                        reinterpret_cast<int*>(rec + rec_bsum_off(it.S)) + s * BsumStride<16>::v,
                        reinterpret_cast<float*>(rec) + s);
    }
    // The records are read by bulk copies (async proxy) of other CTAs.
    asm volatile("fence.proxy.async.global;" ::: "memory");
    consumer_sync();
    if (tid == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(qx_cnt) : "memory");
  }
  bool abort = false;
  const int grp = warp / WPG, wig = warp - grp * WPG;
  int k = 0;               // launch-wide index of the current item's first stage
  int loads[2] = {0, 0};   // record loads seen per activation buffer
  for (int i = 0; i < P.n; i++) {
    const KqLItem& it = P.it[i];
    const int r0 = bid * it.rows_base + min(bid, it.rows_rem);
    const int nrows = it.rows_base + (bid < it.rows_rem ? 1 : 0);
    if (nrows > 0) {
      const int b = i & 1;
      const int nbs = it.qt == 0 ? BsumStride<8>::v : BsumStride<16>::v;
      uint8_t* xb = smem + P.off_x[b];
      float* xd = reinterpret_cast<float*>(xb);
      int* bsum = reinterpret_cast<int*>(xb + rec_bsum_off(it.S));
      int8_t* xq = reinterpret_cast<int8_t*>(xb + rec_xq_off(it.S, nbs));
      KqParams p{};
      p.batch = 1;
      p.n = it.S * 256;
      p.S = it.S;
      p.pitch = it.pitch;
      p.R = it.R;
      p.rows_base = it.rows_base;
      p.rows_rem = it.rows_rem;
      p.y = it.y;
      p.ldy = it.R;
      p.rps = it.rps;
      p.lpr = it.lpr;
      p.status = P.status;
      if (it.wait_for >= 0) {
        // x is an earlier item's y: every CTA must have stored its rows. The
        // CTA quantises x itself (read at L2) once every warp is done with
        // this buffer's previous use.
        if (tid == 0 && !abort && !wait_count(P.cnt + it.wait_for, (unsigned)grid)) {
          record_error(P.status, KERR_TIMEOUT);
          *s_abort = 1;
        }
        consumer_sync();
        abort = *s_abort != 0;
        if (!abort) {
          if (it.qt == 0) quantize_x<8, CWL, true>(p, it.x, p.n, warp, lane, xd, bsum, xq, 0.0f);
          else quantize_x<16, CWL, true>(p, it.x, p.n, warp, lane, xd, bsum, xq, 0.0f);
        }
        consumer_sync();
      } else {
        if (!mbar_wait_bounded(&xfull[b], (uint32_t)(loads[b] & 1))) {
          if (lane == 0) record_error(P.status, KERR_TIMEOUT);
          return;
        }
        loads[b]++;
      }
      const int seg = lane / it.lpr, sl = lane - seg * it.lpr;
      const int nst_i = (nrows + it.rps - 1) / it.rps;
      // Stage k of the launch sits in slot k % NSLOT and is consumed by that
      // slot's warp group alone, which waits for the slot's phases in order.
      int st = (grp - k) % NSLOT;
      if (st < 0) st += NSLOT;
      for (; st < nst_i; st += NSLOT) {
        const int kk = k + st;
        if (!mbar_wait_bounded(&full[grp], (uint32_t)((kk / NSLOT) & 1))) {
          if (lane == 0) record_error(P.status, KERR_TIMEOUT);
          return;
        }
#ifdef VTQ_LIST_NOCOMPUTE
        if (false) {
#else
        if (!abort) {
#endif
          const uint8_t* sbuf = ring + (size_t)grp * P.slot;
          const int sel = it.qt * 4 + it.nch;  // nch in 1..4
          switch (sel) {
            case 1: stage_passes<0, 1>(p, sbuf, st, wig, nrows, r0, sl, seg, xq, xd, bsum); break;
            case 2: stage_passes<0, 2>(p, sbuf, st, wig, nrows, r0, sl, seg, xq, xd, bsum); break;
            case 3: stage_passes<0, 3>(p, sbuf, st, wig, nrows, r0, sl, seg, xq, xd, bsum); break;
            case 4: stage_passes<0, 4>(p, sbuf, st, wig, nrows, r0, sl, seg, xq, xd, bsum); break;
            case 5: stage_passes<1, 1>(p, sbuf, st, wig, nrows, r0, sl, seg, xq, xd, bsum); break;
            case 6: stage_passes<1, 2>(p, sbuf, st, wig, nrows, r0, sl, seg, xq, xd, bsum); break;
            case 7: stage_passes<1, 3>(p, sbuf, st, wig, nrows, r0, sl, seg, xq, xd, bsum); break;
            default: stage_passes<1, 4>(p, sbuf, st, wig, nrows, r0, sl, seg, xq, xd, bsum); break;
          }
        }
        __syncwarp();
        if (lane == 0)
          asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&empty[grp]))
                       : "memory");
      }
      k += nst_i;
      // This warp is done with the activation buffer.
      __syncwarp();
      if (lane == 0)
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&xempty[b]))
                     : "memory");
    }
    if (it.signal) {
      // Every warp has stored its rows of y: publish them.
      consumer_sync();
      if (tid == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(P.cnt + i) : "memory");
    }
  }
  consumer_sync();
  if (P.g.world > 0) {
    // Row-sharded list: this CTA's finished rows of every item go to every
    // other rank's copy of y (contiguous rows, coalesced stores over NVLink;
    // no multicast). Rows were stored to this rank's y by other warps of the
    // CTA before the barrier above.
    for (int job = warp; job < P.n * P.g.world; job += CWL) {
      const int i = job / P.g.world, q = job - i * P.g.world;
      const KqLItem& it = P.it[i];
      if (q == P.g.rank || !it.send) continue;
      const int r0 = bid * it.rows_base + min(bid, it.rows_rem);
      const int nrows = it.rows_base + (bid < it.rows_rem ? 1 : 0);
      const float* src = it.y + r0;
      float* dst = reinterpret_cast<float*>(reinterpret_cast<char*>(it.y + r0) + P.g.peer_off[q]);
      for (int e = lane; e < nrows; e += 32) dst[e] = src[e];
    }
    consumer_sync();
  }
  if (tid == 0) {
    unsigned prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                 : "=r"(prev)
                 : "l"(P.cnt + KQ_LIST_MAX)
                 : "memory");
    if (prev == (unsigned)grid - 1) {  // every CTA has finished every wait
      for (int i = 0; i < P.n; i++) P.cnt[i] = 0;
      P.cnt[KQ_LIST_MAX] = 0;
      P.cnt[KQ_LIST_MAX + 1] = 0;
      if (P.g.world > 0) {
        // Every CTA's stores reached this thread through the acq_rel chain
        // on the exit counter; one system-scope fence covers them all before
        // the arrival signals. Then, if asked, wait for the other ranks.
        __threadfence_system();
        for (int q = 0; q < P.g.world; q++)
          asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(P.g.cnt[q]) : "memory");
        if (P.g.wait_signals) {
          const unsigned target = *P.g.expected + P.g.wait_signals;
          const uint64_t t0 = globaltimer();
          bool ok = true;
          for (;;) {
            unsigned v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(P.g.my_cnt)
                         : "memory");
            if ((int)(v - target) >= 0) break;
            if (globaltimer() - t0 > P.g.limit_ns) {
              record_error(P.status, KERR_TIMEOUT);
              ok = false;  // the missing arrivals are not counted as consumed
              break;
            }
          }
          if (ok) *P.g.expected = target;
          __threadfence_system();
        }
      }
      // Completion word for a host that reads y in place: it holds a sentinel
      // until this store, so a launch that never got here reads as failed.
      if (P.hstatus) *reinterpret_cast<volatile unsigned*>(P.hstatus) = P.status ? *P.status : 0u;
    }
  }
}

static inline uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

}  // namespace

cudaError_t launch_kq_list(const KqListItem* items, int n, unsigned* counters, uint8_t* xrec,
                           unsigned* status, cudaStream_t st, unsigned* hstatus,
                           const KqListGather* g) {
  if (n < 1 || n > KQ_LIST_MAX || !counters || !xrec) return cudaErrorInvalidValue;
  KqListParams P{};
  P.n = n;
  P.hstatus = hstatus;
  if (g) {
    if (g->world < 1 || g->world > kMaxRanks || g->rank < 0 || g->rank >= g->world)
      return cudaErrorInvalidValue;
    P.g = *g;
  }
  P.cnt = counters;
  P.xrec = xrec;
  P.status = status;
  const int grid = num_sms();
  for (int i = 0; i < n; i++) {
    const DevMatrix& m = items[i].m;
    if (m.dtype != T_Q4_K && m.dtype != T_Q6_K) return cudaErrorInvalidValue;
    const int S = (int)(m.in_feat / 256);
    if (S < 1 || S > KQ_SMAX || m.in_feat % 256 || m.out_feat < 1 || m.out_feat > INT32_MAX)
      return cudaErrorInvalidValue;
    if (items[i].wait_for >= i || items[i].wait_for < -1) return cudaErrorInvalidValue;
    if (!items[i].x || !items[i].y || !m.data) return cudaErrorInvalidValue;
  }
  // Ring: NSLOT equal slots filling the shared memory left after the
  // activation arrays; an item's stage is as many whole warp passes (rpw
  // rows each) as fit in a slot.
  int nq = 0;
  for (int i = 0; i < n; i++) {
    const DevMatrix& m = items[i].m;
    KqLItem& it = P.it[i];
    it.W = m.data;
    it.x = items[i].x;
    it.y = items[i].y;
    it.pitch = (int)m.pitch;
    it.R = (int)m.out_feat;
    it.S = (int)(m.in_feat / 256);
    it.qt = m.dtype == T_Q4_K ? 0 : 1;
    // Lanes per row: the power of two covering S when S <= 32; above, the
    // segment width (8, 16 or 32 lanes, at most 4 superblocks per lane) that
    // leaves the fewest lane slots idle (S = 43: 16 lanes x 3 = 48 slots, not
    // 32 x 2 = 64), ties to the wider segment.
    int lpr = 1;
    while (lpr < it.S && lpr < 32) lpr <<= 1;
    if (it.S > 32) {
      int best = 32;
      for (int l = 16; l >= 8; l >>= 1)
        if ((it.S + l - 1) / l <= 4 && l * ((it.S + l - 1) / l) < best * ((it.S + best - 1) / best))
          best = l;
      lpr = best;
    }
    it.lpr = lpr;
    it.nch = (it.S + lpr - 1) / lpr;
    it.rows_base = it.R / grid;
    it.rows_rem = it.R % grid;
    it.wait_for = items[i].wait_for;
    it.signal = 0;
    it.qbase = it.wait_for < 0 ? nq : -1;
    if (it.wait_for < 0) nq += it.S;
  }
  for (int i = 0; i < n; i++) {
    if (P.it[i].wait_for >= 0) P.it[P.it[i].wait_for].signal = 1;
    // Only the last item that writes a given y sends it to the other ranks.
    P.it[i].send = 1;
    for (int j = i + 1; j < n; j++)
      if (items[j].y == items[i].y && items[j].m.out_feat == items[i].m.out_feat) P.it[i].send = 0;
  }
  P.nq = nq;
  uint32_t xbytes = 0;  // one activation buffer: the largest record of the list
  for (int i = 0; i < n; i++)
    xbytes = std::max(xbytes, rec_bytes(P.it[i].S, P.it[i].qt == 0 ? BsumStride<8>::v
                                                                   : BsumStride<16>::v));
  xbytes = align_up(xbytes, 128);
  uint32_t off = 512;
  P.off_x[0] = off;
  P.off_x[1] = off + xbytes;
  off += 2 * xbytes;
  P.off_stage = off;
  const int smem_max = max_smem_optin();
  const uint32_t slot = (uint32_t)((smem_max - (int)off) / NSLOT) / 128 * 128;
  for (int i = 0; i < n; i++) {
    KqLItem& it = P.it[i];
    const int rpw = 32 / it.lpr;
    it.rps = (int)(slot / (uint32_t)it.pitch) / rpw * rpw;
    if (it.rps < rpw) return cudaErrorInvalidValue;  // one warp pass of rows must fit a slot
  }
  P.slot = slot;
  const uint32_t smem = off + (uint32_t)NSLOT * slot;

  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kq_list_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         smem_max);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3((CWL + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  kernel_launch_count()++;
  return cudaLaunchKernelEx(&cfg, kq_list_kernel, P);
}

}  // namespace vtq
