/* trc_oracle.h -- TEST INFRASTRUCTURE: CPU restatement of train.cpp's quantized-weight hot path.
 *
 * This library is the parity checker for the CUDA path. It is never linked into, called by, or
 * shipped with the product (libtrc_cuda.so). Only tests/, __graft_entry__.smoke() and bench.py's
 * CPU-baseline leg load it.
 *
 * Every function restates one reference function (paths relative to the train.cpp source tree):
 *   oracle_fp16_to_fp32   src/core/trc_float.h:23-40      (written from the IEEE-754 binary16
 *                                                          definition, pinned bit-for-bit against
 *                                                          the reference over all 65536 inputs)
 *   oracle_fp32_to_fp16   src/core/trc_float.h:42-63      (round-to-nearest-even encoder)
 *   oracle_dequant        src/io/trc_gguf.cpp:320-417     (dequantize_q4_0 .. dequantize_q8_0)
 *   oracle_mul_mat        src/backends/cpu/trc_cpu_ops.cpp:182-216 (compute_mul_mat)
 *   oracle_cont           src/backends/cpu/trc_cpu_ops.cpp:219-236 (compute_dup)
 *   oracle_repeat_back    src/backends/cpu/trc_cpu_ops.cpp:932-951
 *   oracle_acc            src/backends/cpu/trc_cpu_ops.cpp:954-998
 *   oracle_unary          src/backends/cpu/trc_cpu_ops.cpp:84-94, 119-149 (fn_sqr .. fn_step, compute_scale)
 *   oracle_sum_rows       src/backends/cpu/trc_cpu_ops.cpp:284-300, 317-333 (row_sum_f32, compute_sum_rows_or_mean)
 *   oracle_adamw          src/backends/cpu/trc_cpu_ops.cpp:1506-1538 (compute_opt_step_adamw)
 *   oracle_sgd            src/backends/cpu/trc_cpu_ops.cpp:1540-1573 (compute_opt_step_sgd)
 *   oracle_sum_sqr_acc    src/backends/cpu/trc_cpu_ops.cpp:1578-1591 (compute_sum_sqr_acc)
 *   oracle_clip_scale     src/backends/cpu/trc_cpu_ops.cpp:1594-1611 (compute_clip_scale_inplace)
 *
 * Parity status: pinned. tests/test_oracle.py checks this library against the reference's own
 * known-answer tests (tests/test_gguf.cpp:355-444 of the reference) and against the reference
 * compiled from its sources (oracle/_ref/libtrc_ref.so), bit-for-bit.
 */
#ifndef TRC_ORACLE_H
#define TRC_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (the values are the GGUF on-disk type ids). */
enum { ORACLE_Q4_0 = 2, ORACLE_Q4_1 = 3, ORACLE_Q5_0 = 6, ORACLE_Q5_1 = 7, ORACLE_Q8_0 = 8 };

float    oracle_fp16_to_fp32(uint16_t h);
uint16_t oracle_fp32_to_fp16(float f);

/* Bytes per 32-weight block (18/20/22/24/34), 0 for an unknown type. */
size_t oracle_block_bytes(int type);

/* Dequantize n_blocks consecutive blocks into 32*n_blocks floats. 0 = ok, -1 = unknown type. */
int oracle_dequant(int type, const uint8_t* src, int64_t n_blocks, float* out);

/* ggml mul_mat over byte-strided views: d[i,j,p2,p3] = sum_k a[k,i,p2%a2,p3%a3] * b[k,j,p2,p3],
 * one float accumulator, k ascending (the reference's order, so results are bit-identical).
 * ne/nb follow ggml: ne[0] innermost, nb[] in bytes. n_threads > 1 splits output columns. */
int oracle_mul_mat(const void* a, const int64_t a_ne[4], const size_t a_nb[4],
                   const void* b, const int64_t b_ne[4], const size_t b_nb[4],
                   void* d, const int64_t d_ne[4], const size_t d_nb[4], int n_threads);

/* dst (contiguous, ne = a_ne) = a (any strides). */
void oracle_cont(const void* a, const int64_t a_ne[4], const size_t a_nb[4], float* dst);

/* dst (contiguous, shape dst_ne) = sum of a over the dims it repeats (index i -> i % dst_ne). */
void oracle_repeat_back(const void* a, const int64_t a_ne[4], const size_t a_nb[4],
                        float* dst, const int64_t dst_ne[4]);

/* In-place acc: for every element of b (any strides), dst_bytes[offset + i0*4 + i1*nb1 + i2*nb2
 * + i3*nb3] += b[i]. dst is the byte base of the contiguous destination tensor. */
void oracle_acc(void* dst, const void* b, const int64_t b_ne[4], const size_t b_nb[4],
                size_t nb1, size_t nb2, size_t nb3, size_t offset);

/* Element-wise unary over n contiguous floats; op: 0 sqr, 1 sqrt, 2 abs, 3 neg, 4 sgn, 5 step,
 * 6 scale by param. */
void oracle_unary(int op, const float* x, int64_t n, float param, float* out);

/* out[r] = sum (take_mean: mean) of row r of a contiguous [ne0, rows] array, in double, in order. */
void oracle_sum_rows(const float* x, int64_t ne0, int64_t rows, int take_mean, float* out);

/* In-place optimizer steps over n floats; params6 as the reference optimizer writes them. */
void oracle_adamw(float* p, const float* g, float* m, float* v, int64_t n, const float params6[6]);
void oracle_sgd(float* p, const float* g, float* mom, int64_t n, const float params6[6]);

/* acc[0] += (float) sum (double) x^2, sequential. */
void oracle_sum_sqr_acc(float* acc, const float* x, int64_t n);

/* x *= min(1, max_norm / (sqrt(norm) + eps)). */
void oracle_clip_scale(float* x, int64_t n, float norm, float max_norm, float eps);

#ifdef __cplusplus
}
#endif

#endif
