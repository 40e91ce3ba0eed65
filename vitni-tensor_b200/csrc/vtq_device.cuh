// vtq_device.cuh -- sm_100a device helpers shared by the vtq kernels.
//
// Bulk-copy (TMA, non-tensor mode) + mbarrier pipeline primitives written as
// inline PTX, the exact-rounding fp32 helpers the bit-parity contract needs,
// and the reference's f16 decode restated in integer operations.
//
// Every spin-wait is bounded by %globaltimer: after VTQ_WAIT_LIMIT_NS the
// waiting thread records an error code in the caller's status word and the
// kernel drains its own copies in flight (again bounded) before returning.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#ifndef VTQ_WAIT_LIMIT_NS
#define VTQ_WAIT_LIMIT_NS 2000000000ull  // 2 s: far above any legitimate wait
#endif

namespace vtq {

// Status bits written by kernels into the caller's device status word.
enum : unsigned { KERR_TIMEOUT = 1u, KERR_SHAPE = 2u };

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Arrive once and add `bytes` to the transaction count of the current phase.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for phase `parity` of `bar`. Returns false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > VTQ_WAIT_LIMIT_NS) return false;
  }
  return true;
}

// Global -> shared bulk copy through the TMA unit, completing on `bar`.
// dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Same, with an L2 evict-first hint: weights are streamed exactly once.
__device__ __forceinline__ void bulk_g2s_stream(void* dst_smem, const void* src_gmem,
                                                uint32_t bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], "
      "%2, [%3], %4;" ::"r"(smem_u32(dst_smem)),
      "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void record_error(unsigned* status, unsigned code) {
  if (status) atomicOr(status, code);
}

// binary16 -> binary32 exactly as the reference decodes it (vitni-tensor
// src/ops/quant.rs:41-66), including subnormals and NaN payload (mant << 13).
__device__ __forceinline__ float f16_bits_to_f32(uint32_t h) {
  const uint32_t sign = (h >> 15) & 1u, ex = (h >> 10) & 0x1Fu, mant = h & 0x3FFu;
  uint32_t bits;
  if (ex == 0) {
    if (mant == 0) {
      bits = sign << 31;
    } else {
      const int p = 31 - __clz(mant);  // highest set bit, 0..9
      const int shifts = 10 - p;
      const int e = 1 - shifts;
      const uint32_t m = (mant << shifts) & 0x3FFu;
      bits = (sign << 31) | ((uint32_t)(127 - 15 + e) << 23) | (m << 13);
    }
  } else if (ex == 0x1F) {
    bits = (sign << 31) | 0x7F800000u | (mant << 13);
  } else {
    bits = (sign << 31) | ((ex + 127 - 15) << 23) | (mant << 13);
  }
  return __uint_as_float(bits);
}

// Exact int8 -> fp32 without the I2F unit: byte k of `w` (pre-XORed with
// 0x80808080 so it holds q+128) placed under exponent 2^23, minus 2^23+128.
__device__ __forceinline__ float i8_byte_to_f32(uint32_t w_xor80, uint32_t k) {
  const uint32_t bits = __byte_perm(w_xor80, 0x4B000000u, 0x7650u | k);
  return __fsub_rn(__uint_as_float(bits), 8388736.0f);
}

// Rust `f32 as i32` then clamp(-127, 127): cvt.rzi saturates and maps NaN to 0.
__device__ __forceinline__ int q8_round(float scaled) {
  const float bias = scaled >= 0.0f ? 0.5f : -0.5f;
  int q = __float2int_rz(__fadd_rn(scaled, bias));
  return max(-127, min(127, q));
}

// The reference's serial fp32 sum of n values in shared memory (rms_norm.rs:
// 97-100: one dependent add per element, left to right). Two register batches
// of 32 in ping-pong keep the next loads in flight while the current batch is
// added, so the chain runs at add latency. `v` must be 16-byte aligned.
__device__ __forceinline__ float serial_sum(const float* v, int n) {
  float s = 0.0f;
  const float4* q4 = reinterpret_cast<const float4*>(v);
  const int nb = n / 32;
  float4 a[8], b[8];
  auto add8 = [&](const float4 (&w)[8]) {
#pragma unroll
    for (int u = 0; u < 8; u++) {
      s = __fadd_rn(s, w[u].x);
      s = __fadd_rn(s, w[u].y);
      s = __fadd_rn(s, w[u].z);
      s = __fadd_rn(s, w[u].w);
    }
  };
  if (nb > 0) {
#pragma unroll
    for (int u = 0; u < 8; u++) a[u] = q4[u];
  }
  for (int c = 0; c < nb; c += 2) {
    if (c + 1 < nb) {
#pragma unroll
      for (int u = 0; u < 8; u++) b[u] = q4[8 * (c + 1) + u];
    }
    add8(a);
    if (c + 2 < nb) {
#pragma unroll
      for (int u = 0; u < 8; u++) a[u] = q4[8 * (c + 2) + u];
    }
    if (c + 1 < nb) add8(b);
  }
  for (int i = 32 * nb; i < n; i++) s = __fadd_rn(s, v[i]);
  return s;
}

}  // namespace vtq
