/*
 * vtq_oracle.h -- CPU restatement of vitni-tensor's k-quant linear arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA path is
 * compared against (tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg). No product code links or calls it.
 *
 * Every function restates one function of the Rust reference (paths relative
 * to the vitni-tensor project root) and keeps its operation order exactly:
 * fp32 IEEE with no FMA contraction (build with -ffp-contract=off), Rust
 * `f32 as i32` = truncate + saturate + NaN->0, `i32 as f32` = round to nearest.
 *
 * Pinning: canonical_dot is checked against the reference's published
 * bit goldens (src/ops/quant.rs:1571 0x40ce39e1 at n=4096, :1975 0xc1a3bf11 at
 * n=14336) and the matmul FNV-1a hash (src/ops/matmul.rs:135). The integer
 * Q4_K/Q6_K kernels have no numeric golden in the reference; they are pinned
 * by the reference's property tests restated in tests/test_oracle.py
 * (single-superblock bit equality with the float path, order independence,
 * parallel == serial).
 */
#ifndef VTQ_ORACLE_H
#define VTQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes: same numbering as the product C ABI (include/vtq.h). */
enum {
  OR_OK = 0,
  OR_ERR_INTERNAL = 1,        /* Error::Internal(&str) */
  OR_ERR_NOT_IMPLEMENTED = 2, /* Error::NotImplemented{op,why} */
};

/* GGML type tags (src/model/gguf.rs:127-139). */
enum {
  OR_F32 = 0, OR_F16 = 1, OR_Q4_0 = 2, OR_Q5_0 = 6, OR_Q8_0 = 8,
  OR_Q4_K = 12, OR_Q6_K = 14
};

/* Q4_K activation block (src/ops/quant.rs:738-745). */
typedef struct {
  float d;
  int8_t qs[256];
  int32_t bsums[8];
} or_q8block;

float or_f16_to_f32(uint16_t h);                                  /* quant.rs:41 */
uint16_t or_f32_to_f16(float f);                                  /* quant.rs:69 */
int or_dequantize_q4_0(const uint8_t* w, size_t nbytes, float* out); /* :91  */
int or_dequantize_q5_0(const uint8_t* w, size_t nbytes, float* out); /* :160 */
int or_dequantize_q8_0(const uint8_t* w, size_t nbytes, float* out); /* :193 */
int or_dequantize_q4_k(const uint8_t* w, size_t nbytes, float* out); /* :280 */
int or_dequantize_q6_k(const uint8_t* w, size_t nbytes, float* out); /* :337 */
int or_quantize_q8_0(const float* x, size_t n, uint8_t* out);        /* :214 */
int or_quantize_q4_0(const float* x, size_t n, uint8_t* out);        /* :116 */

float or_fixed_tree(float* part, size_t len);                     /* quant.rs:462 */
float or_canonical_chunk(const float* x, const float* w, size_t n); /* :482 */
float or_canonical_dot(const float* x, const float* w, size_t n);   /* :551 */

void or_quantize_block_q8(const float* x, size_t n, or_q8block* out); /* :750 */
float or_dot_q4k_q8_block(const uint8_t* w, const or_q8block* xq, size_t n); /* :850 */
float or_dot_q6k_q8_block(const uint8_t* w, const or_q8block* xq, size_t n); /* :996 */
int or_integer_dot_q4k(const float* x, const uint8_t* w, size_t nbytes, size_t n,
                       float* out);                               /* :904 */
int or_canonical_dot_q4k_fused(const float* x, const uint8_t* w, size_t nbytes,
                               size_t n, float* out);             /* :616 */
int or_canonical_dot_q6k_fused(const float* x, const uint8_t* w, size_t nbytes,
                               size_t n, float* out);             /* :1212 */

/* Linears: x [batch][in], W row-major [out][row_bytes], y [batch][out]. */
int or_linear_q4_k_integer(const float* x, const uint8_t* w, size_t wlen, float* y,
                           size_t batch, size_t in, size_t out); /* :936 */
int or_linear_q6_k_integer(const float* x, const uint8_t* w, size_t wlen, float* y,
                           size_t batch, size_t in, size_t out); /* :1060 */
int or_linear_q4_k_fused(const float* x, const uint8_t* w, size_t wlen, float* y,
                         size_t batch, size_t in, size_t out);   /* :1433 */
int or_linear_q6_k_fused(const float* x, const uint8_t* w, size_t wlen, float* y,
                         size_t batch, size_t in, size_t out);   /* :1304 */
int or_linear_q4_k_cpu(const float* x, const uint8_t* w, size_t wlen, float* y,
                       size_t batch, size_t in, size_t out);     /* :1456 */
int or_linear_q6_k_cpu(const float* x, const uint8_t* w, size_t wlen, float* y,
                       size_t batch, size_t in, size_t out);     /* :1485 */
int or_linear_q4_0_cpu(const float* x, const uint8_t* w, size_t wlen, float* y,
                       size_t batch, size_t in, size_t out);     /* :1529 */
/* Row-parallel twins (:1099, :1149, :1330, :1385): rayon's grain rule
 * max(1, ceil(out/(4*threads))) with a pthread pool; bit-identical to serial. */
int or_linear_q4_k_integer_parallel(const float* x, const uint8_t* w, size_t wlen,
                                    float* y, size_t batch, size_t in, size_t out,
                                    size_t threads);
int or_linear_q6_k_integer_parallel(const float* x, const uint8_t* w, size_t wlen,
                                    float* y, size_t batch, size_t in, size_t out,
                                    size_t threads);
int or_linear_q4_k_fused_parallel(const float* x, const uint8_t* w, size_t wlen,
                                  float* y, size_t batch, size_t in, size_t out,
                                  size_t threads);

/* linear_dispatch (src/model/forward_quantized.rs:663-785), batch 1.
 * q4k_float_mode=0: `std-parallel` build (integer Q4_K); 1: default build
 * (float-fused Q4_K). threads: 0/1 = serial; >1 uses the row-parallel twins
 * where the reference does (out >= 512, Q4_K/Q6_K only). Q8_0/Q5_0 arms are
 * always serial in the reference; threads>1 on them runs the same per-row
 * arithmetic on a pool (bit-identical) and is used only for CPU timing. */
int or_linear_dispatch(int dtype, const float* x, const uint8_t* w, size_t wlen,
                       size_t in, size_t out, float* y, int q4k_float_mode,
                       size_t threads);

/* Decode glue (src/ops/rms_norm.rs:94-108, src/ops/argmax.rs:49-60,
 * src/model/forward_quantized.rs:925-941). */
void or_rms_norm(const float* x, const float* w, size_t n, float eps, float* out);
uint32_t or_argmax(const float* x, size_t n);

/* Published-vector helpers used by the goldens. */
void or_lcg_pair(size_t n, float* a, float* b);                  /* quant.rs:1856 */
uint64_t or_matmul_fnv_golden(void);                             /* matmul.rs:159 */

#ifdef __cplusplus
}
#endif
#endif
