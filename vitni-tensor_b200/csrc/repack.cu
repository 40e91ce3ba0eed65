// repack.cu -- GGUF row bytes to the device weight layout.
//
// Every format: rows re-pitched to a multiple of 16 bytes (bulk-copy boundary),
// zero padding after the packed row bytes.
// Q6_K additionally: within a row, superblocks are grouped in runs of 8
// (the last run may be shorter, G = min(8, S - 8g)) and each run is stored
// field by field: ql as 8 chunks of 16 bytes per superblock with chunk k of
// superblock i at slot G k + i, then qh the same way (4 chunks each), then
// the 16 scale bytes of each superblock, then the 2-byte d values. Every
// field starts on a 16-byte boundary (210 * 8 = 1680 = 105 * 16), and lanes
// that read chunk k of consecutive superblocks touch consecutive 16-byte
// slots (no shared-memory bank conflicts). The bytes are a permutation of the
// GGUF bytes: nothing is converted, so the kernel reads the reference's values.
#include "vtq_device.cuh"
#include "vtq_internal.h"

namespace vtq {

int64_t packed_row_bytes(int dtype, int64_t n) {
  switch (dtype) {
    case T_F32: return n * 4;
    case T_Q4_0: return n % 32 ? -1 : n / 32 * 18;
    case T_Q5_0: return n % 32 ? -1 : n / 32 * 22;
    case T_Q8_0: return n % 32 ? -1 : n / 32 * 34;
    case T_Q4_K: return n % 256 ? -1 : n / 256 * 144;
    case T_Q6_K: return n % 256 ? -1 : n / 256 * 210;
    default: return -1;
  }
}

int64_t device_pitch(int dtype, int64_t n) {
  const int64_t rb = packed_row_bytes(dtype, n);
  return rb < 0 ? -1 : (rb + 15) / 16 * 16;
}

namespace {

__global__ void repack_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst,
                              int64_t rows, int64_t row_bytes, int64_t pitch, int q6k, int S) {
  const int64_t total = rows * pitch;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = t / pitch;
    const int64_t o = t - r * pitch;
    uint8_t v = 0;
    if (o < row_bytes) {
      int64_t so = o;
      if (q6k) {
        const int gi = (int)(o / 1680), w = (int)(o - (int64_t)gi * 1680);
        const int G = min(8, S - 8 * gi);
        int ii, f;
        if (w < 128 * G) {  // ql: 16-byte chunk k of superblock i at slot G k + i
          const int slot = w / 16;
          ii = slot % G;
          f = 16 * (slot / G) + w % 16;
        } else if (w < 192 * G) {  // qh: same interleave, 4 chunks per superblock
          const int v = w - 128 * G, slot = v / 16;
          ii = slot % G;
          f = 128 + 16 * (slot / G) + v % 16;
        } else if (w < 208 * G) {  // scales: 16 bytes per superblock
          ii = (w - 192 * G) / 16;
          f = 192 + (w - 192 * G) % 16;
        } else {  // d: 2 bytes per superblock
          ii = (w - 208 * G) / 2;
          f = 208 + (w - 208 * G) % 2;
        }
        so = (int64_t)(8 * gi + ii) * 210 + f;
      }
      v = src[r * row_bytes + so];
    }
    dst[t] = v;
  }
}

}  // namespace

cudaError_t launch_repack(const uint8_t* staging, const DevMatrix& m, uint8_t* dst,
                          cudaStream_t st) {
  const int64_t total = m.out_feat * m.pitch;
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const int64_t blocks = std::min<int64_t>((total + threads - 1) / threads, (int64_t)num_sms() * 16);
  repack_kernel<<<(int)blocks, threads, 0, st>>>(staging, dst, m.out_feat, m.row_bytes, m.pitch,
                                                 m.dtype == T_Q6_K, (int)(m.in_feat / 256));
  return cudaGetLastError();
}

}  // namespace vtq
