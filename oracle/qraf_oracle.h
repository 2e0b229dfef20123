/*
 * qraf_oracle.h — CPU restatement of QRAF's quantized matvec path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * kernels in qraf_b200/.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py may load it; the product path never does.
 *
 * Every function restates one function of the reference (simonpierreboucher02/
 * qraf) and cites the file:line it follows.  The restatement keeps the
 * reference's exact floating-point operation order (separate fp32 multiply and
 * add roundings, sequential accumulation) so that its results are bit-identical
 * to the reference's Linux scalar path.  Build with -ffp-contract=off.
 *
 * Parity of this restatement is pinned by tests/test_oracle.py against golden
 * vectors produced by the reference's own compiled sources (oracle/_ref) and
 * committed under tests/golden/.
 */
#ifndef QRAF_ORACLE_H
#define QRAF_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* DType values of the reference (include/core/types.h:27-39). */
#define QO_DTYPE_Q8_0 10u
#define QO_DTYPE_Q4_0 20u

/* fp16 helpers — src/tensor/dtype.cpp:9-37 and :39-59 (truncating encode). */
float    qo_fp16_to_fp32(uint16_t h);
uint16_t qo_fp32_to_fp16(float f);

/* Bytes one quantized block occupies: Q8 4+bs (quantize.cpp:107), Q4 2+bs/2
 * (quantize.cpp:146).  0 for an unknown dtype. */
size_t qo_block_bytes(uint32_t dtype, int block_size);
/* Bytes of one row of K elements: ceil(K/bs) blocks (backend.cpp:138-139,
 * 167-168). */
size_t qo_row_bytes(uint32_t dtype, int block_size, uint32_t K);

/* quantize_q8_0 / quantize_q4_0 — src/tensor/quantize.cpp:105-140, 144-183.
 * Writes qo_row_bytes(dtype, bs, count) bytes to out (zero padding included)
 * and returns that size. */
size_t qo_quantize_q8_0(const float* data, size_t count, int block_size, uint8_t* out);
size_t qo_quantize_q4_0(const float* data, size_t count, int block_size, uint8_t* out);

/* dequantize_block_q8_0 / _q4_0 — quantize.cpp:17-28, 35-51. */
void qo_dequantize_block_q8_0(const void* block, float* out, int block_size);
void qo_dequantize_block_q4_0(const void* block, float* out, int block_size);

/* dot_q8_0_f32 / dot_q4_0_f32 — quantize.cpp:187-210, 212-239. */
float qo_dot_q8_0_f32(const void* q8, const float* x, size_t count, int block_size);
float qo_dot_q4_0_f32(const void* q4, const float* x, size_t count, int block_size);

/* dispatch_matvec_q, Linux scalar branch — src/nn/backend.cpp:131-199.
 * Unknown dtype zero-fills y (backend.cpp:195-198). */
void qo_matvec_q(const void* w, uint32_t dtype, int block_size, uint32_t N, uint32_t K,
                 const float* x, float* y);

/* M independent matvecs: the reference's continuous batching runs one batch-1
 * forward per request (include/runtime/batch_scheduler.h:187-228), so row m of
 * Y is dispatch_matvec_q(W, X[m]).  X is [M][K], Y is [M][N]. */
void qo_matmul_q(const void* w, uint32_t dtype, int block_size, uint32_t N, uint32_t K,
                 uint32_t M, const float* x, float* y);

/* Per-block partial products p[n][b] = block_sum * scale, exactly as the
 * reference forms them inside dot_q*_0_f32 before `total += ...`
 * (quantize.cpp:201-205, 226-234).  p is [N][ceil(K/bs)]. */
void qo_block_partials(const void* w, uint32_t dtype, int block_size, uint32_t N, uint32_t K,
                       const float* x, float* p);

/* fp64 evaluation of the same dequantized product (for error analysis only):
 * y64[n] = sum_b scale_b * sum_i q_i * x_i in double. */
void qo_matvec_q_f64(const void* w, uint32_t dtype, int block_size, uint32_t N, uint32_t K,
                     const float* x, double* y);

/* Per-block integer partial sums of the batch-1 FAST arithmetic (a restatement
 * of the GPU kernels' integer path, for bit-exact checks; block size 32, K a
 * multiple of 32).  For every 32-element block b of x: t = fl(max|x| * (1 + 2^-8))
 * and e_b with t < 2^e_b (t in [2^(e_b-1), 2^e_b)); X_i = rint(x_i * 2^(30 - e_b))
 * (round half to even); X_i = L0*2^24 + L1*2^16 + L2*2^8 + L3 with balanced
 * digits -128 <= L_j <= 127; D[n][b][j] = sum_i q_i * L_j,i with the true codes q
 * (Q8: int8, Q4: nibble - 8); c[b] = 2^(e_b - 30) (0 for an all-zero block).  A
 * block that holds a NaN or an infinity gets zero digits and c = NaN. */
/* RMSNorm in place (src/nn/ops.cpp:107-118). */
void qo_rms_norm(float* x, const float* w, int size, float eps);

void qo_limb_partials(const void* w, uint32_t dtype, uint32_t N, uint32_t K, const float* x, int32_t* D,
                      float* c);

#ifdef __cplusplus
}
#endif
#endif /* QRAF_ORACLE_H */
