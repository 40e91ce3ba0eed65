// decode_mk.cu -- one decode step of a quantized Llama model as a single
// persistent, cooperative kernel.
//
// The step is the reference's step_with_recorders (src/model/
// forward_quantized.rs:329-649) with every linear on the integer k-quant path;
// the arithmetic of every piece is shared with the one-kernel-per-op step
// (kq_core.cuh for the linears, decode_ops.cuh for embedding, attention and
// the token choice), so both produce the same bits.
//
// Structure. One CTA per SM (16 consumer warps + 1 TMA producer warp) walks a
// host-built list of phases: EMBED, NORM (the RMSNorm with its left-to-right sum, computed by
// every CTA into shared memory), MATVEC (this CTA's rows of one matrix),
// ATTN (one query head per CTA) and ARGMAX. Dependent phases are separated by
// a grid barrier (one global counter, bounded wait). The producer warp walks
// the same list and streams the weight rows of every MATVEC phase through one
// shared-memory ring, so the next matrices' bytes are already arriving while
// the CTAs wait at a barrier, run a serial norm chain or attend. Every wait is
// bounded (2 s, %globaltimer) and reports through the status word.
#include <cuda.h>

#include <vector>

#include "decode_mk.h"
#include "decode_ops.cuh"
#include "kq_core.cuh"

namespace vtq {
namespace {

#ifdef VTQ_MK_TRACE
// Phase timeline of the launch at position VTQ_MK_TRACE: [0] CTA 0 enters the
// phase, [1] latest CTA to finish its share, [2] CTA 0 leaves the barrier.
__device__ unsigned long long g_mk_trace[5][1024];
#define MKT(i, v, cond)                                                        \
  do {                                                                         \
    if ((cond) && tid == 0 && a.st->pos == VTQ_MK_TRACE && pi < 1024)          \
      atomicMax(&g_mk_trace[i][pi], (unsigned long long)globaltimer());        \
  } while (0)
#else
#define MKT(i, v, cond) \
  do {                  \
  } while (0)
#endif

constexpr int MK_CW = 15;  // consumer warps (16 warps in all: 128 registers a thread)
constexpr int MK_THREADS = (MK_CW + 1) * 32;
constexpr int MK_NST_MAX = 16;          // barrier array size
constexpr int MK_NSLOT = 5;             // ring slots; slot j is consumed by warp group j only
constexpr int MK_WPG = MK_CW / MK_NSLOT;  // warps per slot group
static_assert(MK_CW % MK_NSLOT == 0, "slot groups");

enum : int { PH_EMBED = 0, PH_NORM = 1, PH_MATVEC = 2, PH_ATTN = 3, PH_ARGMAX = 4 };
enum : int { XS_GLOBAL = 0, XS_NORMED = 1 };

struct MkPhase {
  int kind;
  int barrier;  // grid barrier after the phase
  // NORM: v = x (+ delta) -> res_out (CTA 0); xn = (v * scale) * nw in shared memory.
  const float* x;
  const float* delta;
  const float* nw;
  float* res_out;
  int n;
  // MATVEC
  KqParams kp;
  int qt;    // 0 Q4_K, 1 Q6_K
  int xsrc;  // XS_GLOBAL: kp.x, XS_NORMED: the NORM result
  // ATTN
  int layer;
  const float *bq, *bk, *bv;
};

struct MkArgs {
  const MkPhase* ph;
  int nph;
  unsigned* gbar;  // grid-barrier counter (zeroed before each launch)
  unsigned* status;
  StepState* st;
  // model
  int dim, hs, kv_dim, kv_mul, n_heads, seq_len, vocab, neox;
  float eps;
  const uint8_t* embd;
  int embd_dtype;
  int64_t embd_pitch;
  float *x0, *q, *k, *v, *xo, *kc, *vc, *logits, *log;
  const float *rcos, *rsin;
  const uint32_t* prompt;
  uint32_t* out_tokens;
  // shared-memory layout
  int nst;
  uint32_t slot_bytes;
  uint32_t off_xn, off_xsq, off_xscr, off_xd, off_bsum, off_xq, off_ring;
};

__device__ __forceinline__ void cons_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(MK_CW * 32) : "memory");
}

// This CTA's rows of a MATVEC phase (dealt in (gate, up) pairs for the
// SwiGLU epilogue).
__device__ __forceinline__ int mv_rows(const KqParams& p, int bid, int* r0) {
  const int unit = p.epi ? 2 : 1;
  *r0 = unit * (bid * p.rows_base + min(bid, p.rows_rem));
  return unit * (p.rows_base + (bid < p.rows_rem ? 1 : 0));
}

__global__ void __launch_bounds__(MK_THREADS, 1) decode_mk_kernel(const MkArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + MK_NST_MAX;
  float* red = reinterpret_cast<float*>(smem + 2 * MK_NST_MAX * 8);  // 64 floats of scratch
  int* redi = reinterpret_cast<int*>(red + 32);
  float* xn = reinterpret_cast<float*>(smem + a.off_xn);
  float* xsq = reinterpret_cast<float*>(smem + a.off_xsq);  // also the attention scratch
  auto* xscr = reinterpret_cast<xsum::Scratch*>(smem + a.off_xscr);
  float* xd = reinterpret_cast<float*>(smem + a.off_xd);
  int* bsum = reinterpret_cast<int*>(smem + a.off_bsum);
  int8_t* xq = reinterpret_cast<int8_t*>(smem + a.off_xq);
  uint8_t* ring = smem + a.off_ring;
  // No static shared memory: the dynamic block may use the whole opt-in size.
  volatile int& s_abort = *reinterpret_cast<volatile int*>(smem + 768);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, bid = blockIdx.x;
  if (tid == 0) {
    for (int i = 0; i < a.nst; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], MK_WPG);
    }
    fence_mbar_init();
    s_abort = 0;
  }
  __syncthreads();

  if (warp == MK_CW) {
    // ---- producer: the weight rows of every MATVEC phase, in phase order ----
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      uint32_t gs = 0;  // global stage counter (same sequence as the consumers)
      for (int pi = 0; pi < a.nph; pi++) {
        const MkPhase& ph = a.ph[pi];
        if (ph.kind != PH_MATVEC) continue;
        const KqParams& p = ph.kp;
        int r0;
        const int nrows = mv_rows(p, bid, &r0);
        const int nstages = (nrows + p.rps - 1) / p.rps;
        for (int k = 0; k < nstages; k++, gs++) {
          const int slot = gs % a.nst, use = gs / a.nst;
          if (use > 0 && !mbar_wait_bounded(&empty[slot], (uint32_t)((use - 1) & 1))) {
            record_error(a.status, KERR_TIMEOUT);
            // Drain the copies already issued before leaving.
            for (uint32_t j = (gs >= (uint32_t)a.nst ? gs - a.nst : 0); j < gs; j++)
              mbar_wait_bounded(&full[j % a.nst], (uint32_t)((j / a.nst) & 1));
            return;
          }
          const int ra = k * p.rps, rb = min(ra + p.rps, nrows);
          const uint32_t bytes = (uint32_t)((rb - ra) * p.pitch);
          mbar_arrive_expect_tx(&full[slot], bytes);
          bulk_g2s_stream(ring + (size_t)slot * a.slot_bytes, p.W + (int64_t)(r0 + ra) * p.pitch, bytes,
                          &full[slot], pol);
        }
      }
    }
    return;
  }

  // ---- consumers ----
  uint32_t gs = 0;
  unsigned bar_target = 0;
  for (int pi = 0; pi < a.nph; pi++) {
    const MkPhase& ph = a.ph[pi];
    MKT(0, 0, bid == 0);
    if (ph.kind == PH_EMBED) {
      if (bid == 0) {
        const uint32_t row = a.st->cur;
        for (int e = tid; e < a.dim; e += MK_CW * 32)
          a.x0[e] = embed_value(a.embd, a.embd_dtype, a.embd_pitch, a.dim, row, e);
      }
    } else if (ph.kind == PH_NORM) {
      // rms_norm_slice (rms_norm.rs:94-108) with the residual add, in every CTA.
      // 16-byte loads (n is a multiple of 256): one L2 round trip per thread
      // for the first 4 * 480 elements instead of one per element.
      for (int i = 4 * tid; i < ph.n; i += 4 * MK_CW * 32) {
        float4 v = *reinterpret_cast<const float4*>(ph.x + i);
        if (ph.delta) {
          const float4 dl = *reinterpret_cast<const float4*>(ph.delta + i);
          v = make_float4(__fadd_rn(v.x, dl.x), __fadd_rn(v.y, dl.y), __fadd_rn(v.z, dl.z),
                          __fadd_rn(v.w, dl.w));
        }
        *reinterpret_cast<float4*>(xn + i) = v;
        *reinterpret_cast<float4*>(xsq + i) = make_float4(__fmul_rn(v.x, v.x), __fmul_rn(v.y, v.y),
                                                          __fmul_rn(v.z, v.z), __fmul_rn(v.w, v.w));
        if (ph.res_out && bid == 0) *reinterpret_cast<float4*>(ph.res_out + i) = v;
      }
      // The norm weights do not depend on the step: fetch this thread's share
      // now, while the sum runs.
      float4 nwv[2];
#pragma unroll
      for (int c = 0; c < 2; c++) {
        const int i = 4 * tid + c * 4 * MK_CW * 32;
        if (i < ph.n) nwv[c] = *reinterpret_cast<const float4*>(ph.nw + i);
      }
      cons_sync();
      MKT(3, 0, bid == 0);
      const float sum = xsum::exact_serial_sum<8>(xsq, ph.n, xscr, tid, MK_CW * 32,
                                               [] { cons_sync(); });
      if (tid == 0) {
        const float mean = __fdiv_rn(sum, (float)ph.n);
        red[0] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
      }
      cons_sync();
      MKT(4, 0, bid == 0);
      const float scale = red[0];
      for (int i = 4 * tid, c = 0; i < ph.n; i += 4 * MK_CW * 32, c++) {
        const float4 w = c < 2 ? nwv[c & 1] : *reinterpret_cast<const float4*>(ph.nw + i);
        float4 v = *reinterpret_cast<const float4*>(xn + i);
        v = make_float4(__fmul_rn(__fmul_rn(v.x, scale), w.x), __fmul_rn(__fmul_rn(v.y, scale), w.y),
                        __fmul_rn(__fmul_rn(v.z, scale), w.z), __fmul_rn(__fmul_rn(v.w, scale), w.w));
        *reinterpret_cast<float4*>(xn + i) = v;
      }
      cons_sync();
    } else if (ph.kind == PH_MATVEC) {
      const KqParams& p = ph.kp;
      // Quantise this phase's activation row (quantize_block_q8) into shared memory.
      const float* xs = ph.xsrc == XS_NORMED ? xn : p.x;
      if (ph.qt == 0)
        quantize_x<8, MK_CW>(p, xs, p.n, warp, lane, xd, bsum, xq, 0.0f);
      else
        quantize_x<16, MK_CW>(p, xs, p.n, warp, lane, xd, bsum, xq, 0.0f);
      cons_sync();
      int r0;
      const int nrows = mv_rows(p, bid, &r0);
      const int nstages = (nrows + p.rps - 1) / p.rps;
      const int rpw = 32 / p.lpr;
      const int seg = lane / p.lpr, sl = lane - seg * p.lpr;
      const int grp = warp / MK_WPG, wig = warp - grp * MK_WPG;
      // Stage gs + k sits in slot (gs + k) % nst and is consumed by that slot's
      // warp group alone, which waits for the slot's phases in order.
      int k = (grp - (int)(gs % a.nst)) % a.nst;
      if (k < 0) k += a.nst;
      for (; k < nstages; k += a.nst) {
        const uint32_t kk = gs + k;
        if (!mbar_wait_bounded(&full[grp], (uint32_t)((kk / a.nst) & 1))) {
          if (lane == 0) record_error(a.status, KERR_TIMEOUT);
          s_abort = 1;
        }
        const uint8_t* sbuf = ring + (size_t)grp * a.slot_bytes;
        if (!s_abort) {
          const int rows = min(p.rps, nrows - k * p.rps);
          for (int pr = wig * rpw; pr < rows; pr += MK_WPG * rpw) {
            const int r = k * p.rps + pr + seg;
            if (ph.qt == 0)
              consume_pass<0, 1, 1>(p, sbuf, pr + seg, pr + seg < rows, sl, r0 + r, xq, xd, bsum,
                                    nullptr, 0);
            else
              consume_pass<1, 1, 1>(p, sbuf, pr + seg, pr + seg < rows, sl, r0 + r, xq, xd, bsum,
                                    nullptr, 0);
          }
        }
        __syncwarp();
        if (lane == 0)
          asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&empty[grp]))
                       : "memory");
      }
      gs += nstages;
      cons_sync();  // the next phase reuses xq / xd / bsum
    } else if (ph.kind == PH_ATTN) {
      if (bid < a.n_heads)
        attention_head(bid, a.q, a.k, a.v, a.kc, a.vc, ph.layer, a.seq_len, a.kv_dim, a.hs,
                       a.kv_mul, a.rcos, a.rsin, a.st->pos, a.xo, xsq, red, tid, MK_CW * 32,
                       [] { cons_sync(); }, AttnExtras{a.neox, ph.bq, ph.bk, ph.bv});
    } else if (ph.kind == PH_ARGMAX) {
      if (a.log)  // every CTA copies a slice of the step's logits to the log
        for (int i = bid * MK_CW * 32 + tid; i < a.vocab; i += gridDim.x * MK_CW * 32)
          a.log[(size_t)a.st->pos * a.vocab + i] = a.logits[i];
      if (a.log) {
        // the token choice below advances pos: every CTA must have read it
        cons_sync();
        if (tid == 0) {
          __threadfence();
          atomicAdd(a.gbar, 1u);
        }
        bar_target += gridDim.x;
        if (tid == 0) {
          const uint64_t t0 = globaltimer();
          for (;;) {
            unsigned v;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a.gbar) : "memory");
            if (v >= bar_target) break;
            if (globaltimer() - t0 > VTQ_WAIT_LIMIT_NS) {
              record_error(a.status, KERR_TIMEOUT);
              break;
            }
          }
        }
        cons_sync();
      }
      if (bid == 0)
        argmax_next(a.logits, a.vocab, a.st, a.prompt, a.out_tokens, red, redi, tid, MK_CW * 32,
                    [] { cons_sync(); });
    }
#ifdef VTQ_MK_TRACE
    cons_sync();
    MKT(1, 0, true);
#endif
    if (ph.barrier) {
      // Grid barrier of the consumer threads: CTA-local barrier, then thread 0
      // publishes (GPU-scope fence + add) and waits (acquire) for every CTA.
      cons_sync();
      bar_target += gridDim.x;
      if (tid == 0) {
        __threadfence();
        atomicAdd(a.gbar, 1u);
        const uint64_t t0 = globaltimer();
        // After a timeout the step's result is void: stop waiting at barriers.
        for (; !s_abort;) {
          unsigned v;
          asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(a.gbar) : "memory");
          if (v >= bar_target) break;
          if (globaltimer() - t0 > VTQ_WAIT_LIMIT_NS) {
            record_error(a.status, KERR_TIMEOUT);
            s_abort = 1;
            break;
          }
        }
        __threadfence();
      }
      cons_sync();
    }
    MKT(2, 0, bid == 0);
  }
}

int sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

}  // namespace

struct MkPlan {
  MkArgs args{};
  MkPhase* dph = nullptr;
  unsigned* gbar = nullptr;
  uint32_t smem = 0;
  int grid = 0;
};

bool mk_supported(const MkModel& m) {
  auto kq = [](const DevMatrix& d) { return d.dtype == T_Q4_K || d.dtype == T_Q6_K; };
  auto s_ok = [](const DevMatrix& d) { return d.in_feat % 256 == 0 && d.in_feat / 256 <= 32; };
  if (!kq(m.head) || !s_ok(m.head)) return false;
  for (const auto& L : m.layers)
    for (const DevMatrix* d : {&L.wqk, &L.wv, &L.wo, &L.w13, &L.w2})
      if (!kq(*d) || !s_ok(*d)) return false;
  const int hs = m.dim / m.n_heads;
  if (hs % 2 || m.dim % 256 || m.hidden % 256) return false;
  if (m.n_heads > sms()) return false;
  // Opt-in: the per-op graph measured faster on TinyLlama shapes.
  const char* e = getenv("VTQ_DECODE_PERSISTENT");
  return e != nullptr && e[0] == '1';
}

cudaError_t mk_build(const MkModel& m, MkPlan** out) {
  auto* plan = new MkPlan;
  const int grid = sms();
  const int hs = m.dim / m.n_heads, kv_dim = m.n_kv_heads * hs;
  const int xmax = std::max(m.dim, m.hidden);
  // Shared memory: barriers + scratch, xn, xsq (also attention scratch),
  // quantised activation (xd, bsum, xq), then the ring.
  const int smax = xmax / 256;
  uint32_t off = 1024;  // barriers (256 B), scratch (256 B), abort flag
  const uint32_t off_xn = off;
  off = align_up(off + (uint32_t)xmax * 4, 128);
  const uint32_t off_xsq = off;
  off = align_up(off + (uint32_t)std::max(m.dim, 3 * hs + m.seq_len) * 4, 128);
  const uint32_t off_xscr = off;
  off = align_up(off + (uint32_t)sizeof(xsum::Scratch), 128);
  const uint32_t off_xd = off;
  off = align_up(off + (uint32_t)smax * 4, 16);
  const uint32_t off_bsum = off;
  off = align_up(off + (uint32_t)smax * BsumStride<16>::v * 4, 16);
  const uint32_t off_xq = off;
  off = align_up(off + (uint32_t)smax * XQ_STRIDE, 128);
  const uint32_t off_ring = off;
  int optin = 0, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const int nst = MK_NSLOT;
  const uint32_t MK_SLOT = (uint32_t)((optin - (int)off_ring) / nst) / 128 * 128;
  if (MK_SLOT < 8192) {
    delete plan;
    return cudaErrorInvalidValue;
  }
  plan->smem = off_ring + nst * MK_SLOT;

  std::vector<MkPhase> ph;
  auto matvec = [&](const DevMatrix& d, const float* x, float* y, int xsrc, bool pairs,
                    int barrier) {
    MkPhase P{};
    P.kind = PH_MATVEC;
    P.barrier = barrier;
    P.qt = d.dtype == T_Q4_K ? 0 : 1;
    P.xsrc = xsrc;
    KqParams& p = P.kp;
    const int S = (int)(d.in_feat / 256);
    int lpr = 1;
    while (lpr < S && lpr < 32) lpr <<= 1;
    const int rpw = 32 / lpr;
    p.x = x;
    p.ldx = d.in_feat;
    p.batch = 1;
    p.n = (int)d.in_feat;
    p.S = S;
    p.W = d.data;
    p.pitch = d.pitch;
    p.R = (int)d.out_feat;
    p.epi = pairs ? 1 : 0;  // gate|up rows interleaved: y = silu(gate) * up
    const int unit = pairs ? 2 : 1;
    p.rows_base = p.R / unit / grid;
    p.rows_rem = p.R / unit % grid;
    p.y = y;
    p.ldy = d.out_feat / unit;
    p.lpr = lpr;
    p.status = m.status;
    const int rows_per_cta = unit * (p.rows_base + (p.rows_rem ? 1 : 0));
    int rps = std::max(rpw, (int)(MK_SLOT / d.pitch) / rpw * rpw);
    rps = std::min(rps, std::max(rpw, (rows_per_cta + rpw - 1) / rpw * rpw));
    p.rps = rps;
    if ((uint32_t)(rps * d.pitch) > MK_SLOT) p.rps = 0;   // rows too long for a slot
    if (pairs && (rpw < 2 || p.R % 2)) p.rps = 0;         // a pair must share a warp pass
    ph.push_back(P);
  };
  auto norm = [&](const float* x, const float* delta, const float* nw, float* res) {
    MkPhase P{};
    P.kind = PH_NORM;
    P.x = x;
    P.delta = delta;
    P.nw = nw;
    P.res_out = res;
    P.n = m.dim;
    ph.push_back(P);
  };
  {
    MkPhase E{};
    E.kind = PH_EMBED;
    E.barrier = 1;
    ph.push_back(E);
  }
  const float* delta = nullptr;
  float* A = m.x;
  float* B = m.xr;
  for (int l = 0; l < m.n_layers; l++) {
    const MkLayer& L = m.layers[l];
    norm(A, delta, L.rms_att, B);
    matvec(L.wqk, nullptr, m.q, XS_NORMED, false, 0);
    matvec(L.wv, nullptr, m.v, XS_NORMED, false, 1);
    MkPhase At{};
    At.kind = PH_ATTN;
    At.barrier = 1;
    At.layer = l;
    At.bq = L.bq;
    At.bk = L.bk;
    At.bv = L.bv;
    ph.push_back(At);
    matvec(L.wo, m.xo, m.xb2, XS_GLOBAL, false, 1);
    norm(B, m.xb2, L.rms_ffn, A);
    matvec(L.w13, nullptr, m.g, XS_NORMED, true, 1);  // m.g receives silu(gate) * up
    matvec(L.w2, m.g, m.xb2, XS_GLOBAL, false, 1);
    delta = m.xb2;
  }
  norm(A, delta, m.rms_final, nullptr);
  matvec(m.head, nullptr, m.logits, XS_NORMED, false, 1);
  {
    MkPhase G{};
    G.kind = PH_ARGMAX;
    ph.push_back(G);
  }
  for (const auto& P : ph)
    if (P.kind == PH_MATVEC && P.kp.rps == 0) {
      delete plan;
      return cudaErrorInvalidValue;
    }

  cudaError_t e = cudaMalloc(&plan->dph, ph.size() * sizeof(MkPhase));
  if (e == cudaSuccess)
    e = cudaMemcpy(plan->dph, ph.data(), ph.size() * sizeof(MkPhase), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&plan->gbar, 256);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(decode_mk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)plan->smem);
  int per_sm = 0;
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_mk_kernel, MK_THREADS,
                                                      plan->smem);
  if (e == cudaSuccess && per_sm < 1) e = cudaErrorInvalidValue;
  if (e != cudaSuccess) {
    mk_free(plan);
    return e;
  }
  MkArgs& a = plan->args;
  a.ph = plan->dph;
  a.nph = (int)ph.size();
  a.gbar = plan->gbar;
  a.status = m.status;
  a.st = m.st;
  a.dim = m.dim;
  a.hs = hs;
  a.kv_dim = kv_dim;
  a.kv_mul = m.n_heads / m.n_kv_heads;
  a.n_heads = m.n_heads;
  a.seq_len = m.seq_len;
  a.vocab = m.vocab;
  a.eps = m.eps;
  a.neox = m.neox ? 1 : 0;
  a.embd = m.embd.data;
  a.embd_dtype = m.embd.dtype;
  a.embd_pitch = m.embd.pitch;
  a.x0 = m.x;
  a.q = m.q;
  a.k = m.q + m.dim;
  a.v = m.v;
  a.xo = m.xo;
  a.kc = m.kc;
  a.vc = m.vc;
  a.logits = m.logits;
  a.rcos = m.rcos;
  a.rsin = m.rsin;
  a.prompt = m.prompt;
  a.out_tokens = m.out_tokens;
  a.nst = nst;
  a.slot_bytes = MK_SLOT;
  a.off_xn = off_xn;
  a.off_xsq = off_xsq;
  a.off_xscr = off_xscr;
  a.off_xd = off_xd;
  a.off_bsum = off_bsum;
  a.off_xq = off_xq;
  a.off_ring = off_ring;
  plan->grid = grid;
  *out = plan;
  return cudaSuccess;
}

cudaError_t mk_launch(MkPlan* plan, float* log, cudaStream_t st) {
  MkArgs a = plan->args;
  a.log = log;
  cudaError_t e = cudaMemsetAsync(plan->gbar, 0, 4, st);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan->grid);
  cfg.blockDim = dim3(MK_THREADS);
  cfg.dynamicSmemBytes = plan->smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_mk_kernel, a);
}

#ifdef VTQ_MK_TRACE
extern "C" int vtq_mk_trace(unsigned long long* out, int nph) {
  return (int)cudaMemcpyFromSymbol(out, g_mk_trace, sizeof(unsigned long long) * 5 * 1024);
}
#endif

void mk_free(MkPlan* plan) {
  if (!plan) return;
  if (plan->dph) cudaFree(plan->dph);
  if (plan->gbar) cudaFree(plan->gbar);
  delete plan;
}

}  // namespace vtq
