// vtq_internal.h -- launchers shared between the kernel files and the C ABI.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace vtq {

// GGML type tags (vitni-tensor src/model/gguf.rs:127-139).
enum GgmlType : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q5_0 = 6, T_Q8_0 = 8, T_Q4_K = 12, T_Q6_K = 14 };

// Device layout of a weight matrix. Rows are re-pitched to a multiple of 16
// bytes so every row starts on a bulk-copy boundary. Q6_K superblocks are
// additionally regrouped in runs of 8 (see repack.cu) so that each field of
// each superblock is 16-byte aligned in shared memory. All other formats keep
// their GGUF byte order within a row.
struct DevMatrix {
  int dtype;
  int64_t in_feat, out_feat;  // n, R
  int64_t row_bytes;          // packed GGUF bytes per row
  int64_t pitch;              // device bytes per row (multiple of 16)
  const uint8_t* data;        // device pointer, 256-byte aligned, + 16 B tail pad
};

int64_t packed_row_bytes(int dtype, int64_t in_feat);  // -1 if in_feat invalid
int64_t device_pitch(int dtype, int64_t in_feat);

// Raw GGUF rows (host or device bytes already on device in `staging`) to the
// device layout. `staging` holds out_feat*row_bytes packed bytes.
cudaError_t launch_repack(const uint8_t* staging, const DevMatrix& m, uint8_t* dst,
                          cudaStream_t st);

// Fused all-gather target of a row-sharded linear: the kernel stores its rows
// into the full-y buffer of every rank (peer pointers over NVLink, rows
// [row0, row0 + R) of a [batch][ldy] array at y[q]) and, once every CTA of
// the launch has stored, adds 1 to every rank's arrival counter cnt[q].
// `done` is a launch-completion counter in this rank's memory (starts at 0,
// left at 0).
constexpr int kMaxRanks = 8;
struct GatherTarget {
  int world;
  int64_t row0, ldy;
  float* y[kMaxRanks];
  unsigned* cnt[kMaxRanks];
  unsigned* done;
  // wait_signals > 0: the launch's last CTA also waits until this rank's
  // counter (my_cnt) has `wait_signals` more arrivals than *expected, then
  // advances *expected, so the launch ends with the whole y gathered.
  unsigned* my_cnt;
  unsigned* expected;
  unsigned wait_signals;
  // 0: this launch does not signal; a later gathered launch on the same
  // stream signals for it (its system fence covers every earlier launch's
  // stores, which precede it in stream order).
  int signal = 1;
  uint64_t limit_ns = 2000000000ull;  // bound of the arrival wait
};

// Transform applied to a batch-1 activation row while the matvec quantises it
// (decode fusion; each is the reference's op order):
//   kind 1 SwiGLU  x_i = silu(x_i) * x2_i, silu(g) = g / (1 + expf(-g))
//                  (forward_quantized.rs:556-561)
//   kind 2 RMSNorm v_i = x_i (+ delta_i); x_i = (v_i * scale) * nw_i with
//                  scale = 1 / sqrtf(sum(v^2) / n + eps), the sum serial
//                  (rms_norm.rs:94-108); CTA 0 stores v to res_out if set.
// Activation transform of a k-quant matvec (batch 1): kind 2 = RMSNorm of
// v = x + delta (written to res_out) scaled by nw, computed in the prologue.
// swiglu_pairs: the matrix rows are (gate_i, up_i) pairs and y receives
// silu(gate_i) * up_i (R / 2 values) from the epilogue.
struct KqXform {
  int kind = 0;
  int swiglu_pairs = 0;
  const float* delta = nullptr;
  const float* nw = nullptr;
  float eps = 0.0f;
  float* res_out = nullptr;
};

// Integer k-quant matvec (Q4_K / Q6_K against int8-quantised activations):
// y[b, r] for r in [0, R), b in [0, batch). x row stride ldx, y row stride ldy.
// With `g`, y/ldy are ignored and the rows go to every rank of g instead.
cudaError_t launch_kq_matvec(const DevMatrix& m, const float* x, int64_t ldx, int64_t batch,
                             float* y, int64_t ldy, unsigned* status, cudaStream_t st,
                             const GatherTarget* g = nullptr, const KqXform* xf = nullptr);

// One persistent launch over a list of integer k-quant linears (batch 1), in
// list order; item i's y is bit-identical to launch_kq_matvec on the same
// inputs. wait_for = j (< i) makes item i read its x only after every row of
// item j's y is stored (x may be y_j); -1 = x is ready at launch. `counters`
// is a zeroed device array of KQ_LIST_MAX + 2 words owned by the caller; the
// kernel leaves it zeroed. `xrec` is caller-owned scratch of KQ_LIST_MAX *
// KQ_LIST_REC bytes (the quantised activations). Launches sharing counters
// or scratch must be ordered on one stream.
constexpr int KQ_LIST_MAX = 32;
constexpr size_t KQ_LIST_REC = 45568;  // 128 superblocks: xd 512 + bsum 128*80 + xq 128*272
struct KqListItem {
  DevMatrix m;
  const float* x;
  float* y;
  int wait_for;
};
// Row-sharded list: every item's y lies in this rank's gather buffer; the
// launch also stores its rows into every other rank's buffer (at byte offset
// peer_off[q] from this rank's) and, once all CTAs have, signals every
// rank's arrival counter once; wait_signals > 0 makes it then wait (bounded
// by limit_ns) until that many more arrivals have reached this rank.
struct KqListGather {
  int world = 0, rank = 0;
  int64_t peer_off[kMaxRanks] = {};
  unsigned* cnt[kMaxRanks] = {};
  unsigned* my_cnt = nullptr;
  unsigned* expected = nullptr;
  unsigned wait_signals = 0;
  uint64_t limit_ns = 2000000000ull;
};
// `hstatus` (optional, host-mapped): receives the status word once the whole
// launch has finished (for callers that read y straight from host memory).
cudaError_t launch_kq_list(const KqListItem* items, int n, unsigned* counters, uint8_t* xrec,
                           unsigned* status, cudaStream_t st, unsigned* hstatus = nullptr,
                           const KqListGather* g = nullptr);

// Waits on `st` until this rank's arrival counter has received `signals` more
// arrivals than before (`expected` is a device counter of arrivals consumed).
// Bounded: after limit_ns the status word gets KERR_TIMEOUT and the consumed
// count is left unchanged (the missing arrivals are not counted as seen).
cudaError_t launch_gather_wait(unsigned* cnt, unsigned* expected, unsigned signals,
                               unsigned* status, cudaStream_t st,
                               uint64_t limit_ns = 2000000000ull);

// Batched integer Q4_K linear on the tensor cores (tcgen05 kind::i8): same
// results as launch_kq_matvec for any batch; used for prefill-sized batches.
// Scratch: the quantised activations (kq_gemm_workspace_bytes). With ws ==
// nullptr the launcher uses a buffer cached per (device, stream), allocated
// on first use and grown with cudaMalloc, freed when the library unloads.
bool kq_gemm_supported(const DevMatrix& m, int64_t batch);
size_t kq_gemm_workspace_bytes(int64_t in_feat, int64_t batch);
cudaError_t launch_kq_gemm(const DevMatrix& m, const float* x, int64_t ldx, int64_t batch,
                           float* y, int64_t ldy, unsigned* status, cudaStream_t st,
                           uint8_t* ws = nullptr, size_t ws_bytes = 0);

// Canonical fp32 matvec (8 pinned lanes, 8192-element chunks, fixed trees)
// for Q8_0 / Q5_0 / Q4_0 / F32 rows and the float-fused Q4_K mode.
cudaError_t launch_canon_matvec(const DevMatrix& m, const float* x, int64_t ldx, int64_t batch,
                                float* y, int64_t ldy, unsigned* status, cudaStream_t st);

// The linear_dispatch arm for m's dtype (integer k-quant or canonical), batch 1.
// Kernel launches issued by this library's linear launchers since load
// (graph replays are not launches of the launcher; callers count those).
unsigned long long& kernel_launch_count();

// A linear of any device format over `batch` activation rows, dispatched like
// vtq_linear: the tcgen05 GEMM for Q4_K at batch >= 16, the integer matvec for
// Q4_K / Q6_K, the canonical fp32 kernel otherwise.
cudaError_t linear_any(const DevMatrix& m, const float* x, int64_t ldx, float* y, int64_t ldy,
                       int64_t batch, unsigned* status, cudaStream_t st);
cudaError_t launch_kq_or_canon(const DevMatrix& m, const float* x, float* y, unsigned* status,
                               cudaStream_t st);

int num_sms();
int max_smem_optin();

// Programmatic dependent launch for the kernels of a dependent chain (off
// with VTQ_NO_PDL=1). A kernel launched this way may start while its
// predecessor runs; it must execute griddepcontrol.wait before reading the
// predecessor's outputs or writing anything the predecessor reads.
bool pdl_enabled();

}  // namespace vtq
