/*
 * odi_oracle.h -- CPU restatement of ODIEngine's quantized matrix product.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA
 * backend: tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg
 * may call it; the product path (odiengine_b200) never does.
 *
 * What it restates (reference paths are relative to the ODIEngine tree):
 *   - fp16 -> fp32 conversion, both IEEE and the reference's own converter
 *     (src/compute/cpu/cpu_backend.cpp:660-684), which is wrong for subnormals;
 *   - Q4_0 / Q8_0 dequantisation (cpu_backend.cpp:686-702, 769-780);
 *   - the fp32 quantized matmul loops matmul_q4_0 / matmul_q8_0
 *     (cpu_backend.cpp:786-826, 828-854), in their exact operation order;
 *   - the same loop order applied to Q4_K / Q5_K / Q6_K, for which the
 *     reference has no kernel (its matmul throws, cpu_backend.cpp:211-216,646):
 *     blocks are decoded per the GGML K-quant format and dotted sequentially;
 *   - Q4_0 / Q8_0 quantisers and the Q8_0 activation quantiser, following the
 *     published algorithm of the `gguf` Python package 0.19.0
 *     (gguf/quants.py Q4_0.quantize_blocks, Q8_0.quantize_blocks) and pinned
 *     byte-for-byte against it by tests/test_oracle.py;
 *   - K-quant quantisers of this project's own design (gguf 0.19.0 has none):
 *     their output is pinned only through decode, i.e. gguf's dequantize of
 *     the produced bytes must equal this library's dequantize bit-exactly;
 *   - the Q8-activation integer dot that the CUDA kernels compute, together
 *     with the analytic error bounds used by the parity tests;
 *   - the tiled device layout ("units" of 64 rows x 256 columns) that the
 *     CUDA loader repacks GGUF blocks into, and its inverse.
 *
 * Build with -ffp-contract=off: the reference compiled for baseline x86-64
 * has no fused multiply-add in these scalar loops.
 */
#ifndef ODI_ORACLE_H
#define ODI_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype ids are odi_dtype_t values (include/odi/odi_types.h:32-49). */
enum {
  ORC_Q8_0 = 6,
  ORC_Q4_0 = 7,
  ORC_Q4_1 = 8,
  ORC_Q5_0 = 9,
  ORC_Q5_1 = 10,
  ORC_Q4_K = 11,
  ORC_Q5_K = 12,
  ORC_Q6_K = 13
};

/* Tiled layout constants (shared with the CUDA loader). */
enum { ORC_UNIT_ROWS = 64, ORC_UNIT_COLS = 256 };

float orc_fp16_to_fp32(uint16_t h);
float orc_fp16_to_fp32_ref(uint16_t h);
uint16_t orc_fp32_to_fp16(float f);

int orc_block_elems(int dtype);
int orc_block_bytes(int dtype);
int64_t orc_row_bytes(int dtype, int64_t K);

/* fp32 weights [N][K] -> GGUF blocks, row-major by output row. 0 = ok. */
int orc_quantize(int dtype, const float* w, int64_t N, int64_t K, void* out);
/* GGUF blocks [N][ceil(K/blk)] -> fp32 [N][K].  ref_fp16 != 0 uses the
 * reference's fp16 converter. */
int orc_dequantize(int dtype, const void* blocks, int64_t N, int64_t K, float* out, int ref_fp16);

/* out[M][N] = a[M][K] . dequant(b)^T in the reference's loop order, using the
 * reference's fp16 converter for Q4_0/Q8_0 (the reference's own kernels) and
 * IEEE decode for the K-quants (no reference code; gguf semantics).  nthreads > 1 splits output rows N across
 * threads (each output element keeps its sequential sum). */
int orc_matmul_ref(int dtype, float* out, const float* a, const void* b,
                   int64_t M, int64_t K, int64_t N, int nthreads);

/* Q8_0 activation quantiser.  x [M][K] -> blocks [M][ceil(K/32)] of 34 bytes
 * (the last block zero-padded). */
void orc_quantize_q8_0_act(const float* x, int64_t M, int64_t K, void* blocks);
/* Same quantisation in the device plane form: xq int8 [M][Kp], xs 8-byte
 * records {float d; int16 s_lo16; int16 s_hi16} [M][Kp/32], Kp = K rounded up
 * to 256, padding zero. */
void orc_quantize_act_planes(const float* x, int64_t M, int64_t K, int8_t* xq, void* xs);

/* Q8-activation product: y = sum over blocks of the exact integer block dot
 * times the fp32 block scales (the CUDA kernels' arithmetic, sequential
 * order).  If bound != NULL, bound[m*N+n] receives a rigorous bound on
 * |y_q8 - y_exact| where y_exact is the real-number product of fp32 x and the
 * dequantised weights: sum_b 0.5625*d_x,b*sum|w| plus fp32 rounding terms.
 * If mag != NULL, mag[m*N+n] receives sum of |scaled block terms|, the
 * magnitude that bounds fp32 reordering error of the Q8 product itself. */
/* |A_g*q| + |B_g| per element ([N][K]): scale of fp16 decoding errors. */
int orc_term_magnitude(int dtype, const void* blocks, int64_t N, int64_t K, float* out);

/* value = A*q - B per element ([N][K] each). */
int orc_block_factors(int dtype, const void* blocks, int64_t N, int64_t K, float* A, float* B, int32_t* q);

int orc_matmul_q8act(int dtype, float* out, const float* a, const void* b,
                     int64_t M, int64_t K, int64_t N, float* bound, float* mag);
/* The same on nthreads host threads (rows split evenly; identical results). */
int orc_matmul_q8act_mt(int dtype, float* out, const float* a, const void* b, int64_t M, int64_t K,
                        int64_t N, float* bound, float* mag, int nthreads);

/* Rigorous bound on |y_fp32 - y_exact| for any fp32 summation order of the
 * reference product: 2*(K+8)*2^-24 * sum_k |a_k| * |w_k|  (plus tiny). */
int orc_fp32_bound(int dtype, const float* a, const void* b, int64_t M, int64_t K, int64_t N, float* bound);
int orc_fp32_bound_mt(int dtype, const float* a, const void* b, int64_t M, int64_t K, int64_t N, float* bound,
                      int nthreads);

/* Tiled device layout. */
int64_t orc_tiled_bytes(int dtype, int64_t N, int64_t K);
int64_t orc_unit_bytes(int dtype);
int orc_repack(int dtype, const void* gguf, void* tiled, int64_t N, int64_t K);
int orc_unpack(int dtype, const void* tiled, void* gguf, int64_t N, int64_t K);

#ifdef __cplusplus
}
#endif
#endif
