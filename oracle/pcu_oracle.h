/*
 * pcu_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of Fusion-PCU's strict checked-arithmetic path, used as the
 * checker for the CUDA provider in fusion-pcu_b200/.  Only tests/, the smoke()
 * entry of __graft_entry__.py and the cpu_baseline / reference legs of bench.py
 * may load this library.  The product never links or calls it.
 *
 * Parity pin: the reference (a Rust workspace) cannot be compiled in this image
 * (no cargo/rustc), so this restatement is pinned against the reference's own
 * known-answer tests, transcribed into tests/golden/reference_kats.json with a
 * file:line citation per case, and against host IEEE arithmetic on the same
 * randomized xorshift streams the reference tests use.
 *
 * Encodings follow the reference's CUDA status ABI
 * (Crates/backends/cuda/owned_dispatch/owned_dispatch.rs:20-22,70-109):
 *   kind tags 1 DivideByZero, 2 SignedDivisionOverflow, 3 ArithmeticOverflow,
 *   4 ArithmeticUnderflow, 5 InvalidFloatingOperand; a status word is
 *   (event << 3) | kind, and UINT64_MAX means "no fault".
 * Underflow policies (Crates/core/scalar_float_underflow.rs:47-56):
 *   0 IeeeAfterRounding, 1 RejectSubnormalResult, 2 AllowGradualUnderflow.
 * Binary op tags (Crates/backends/cuda/codegen/lower/checked_float/checked_float.rs:230-235):
 *   0 Add, 1 Sub, 2 Mul, 3 Div.
 */
#ifndef PCU_ORACLE_H
#define PCU_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PCU_ORACLE_OK 0
#define PCU_ORACLE_DIVIDE_BY_ZERO 1
#define PCU_ORACLE_SIGNED_DIVISION_OVERFLOW 2
#define PCU_ORACLE_OVERFLOW 3
#define PCU_ORACLE_UNDERFLOW 4
#define PCU_ORACLE_INVALID 5

/* ---- scalar law (checked_float.c) ---- returns the fault kind, 0 on success */
int pcu_oracle_f32_binary(uint32_t left, uint32_t right, int op, int policy, uint32_t *out);
int pcu_oracle_f64_binary(uint64_t left, uint64_t right, int op, int policy, uint64_t *out);
int pcu_oracle_f32_relu(uint32_t x, int policy, uint32_t *out);
int pcu_oracle_f64_relu(uint64_t x, int policy, uint64_t *out);
int pcu_oracle_f32_relu_backward(uint32_t x, uint32_t upstream, int policy, uint32_t *out);
int pcu_oracle_f64_relu_backward(uint64_t x, uint64_t upstream, int policy, uint64_t *out);
int pcu_oracle_f32_neg(uint32_t x, int policy, uint32_t *out);
int pcu_oracle_f64_neg(uint64_t x, int policy, uint64_t *out);
uint32_t pcu_oracle_count_f32(uint64_t count);
uint64_t pcu_oracle_count_f64(uint64_t count);
uint64_t pcu_oracle_f32_bits_to_f64_bits(uint32_t bits);

/* ---- ordered tensor primitives (strict_ops.c): reference order, soft-float,
 * single-threaded.  Each returns a status word: UINT64_MAX on success, else
 * (first event << 3) | kind.  `elem` is 4 (binary32) or 8 (binary64); data are
 * raw little-endian bit patterns. ---- */
uint64_t pcu_oracle_matmul(int elem, const void *left, const void *right, void *out,
                           uint64_t rows, uint64_t inner, uint64_t columns,
                           uint64_t left_stride, uint64_t right_stride,
                           int transpose_left, int transpose_right, int policy,
                           uint64_t row_begin, uint64_t row_end);
uint64_t pcu_oracle_matmul_cells(int elem, const void *left, const void *right, void *out,
                                 uint64_t rows, uint64_t inner, uint64_t columns,
                                 uint64_t left_stride, uint64_t right_stride,
                                 int transpose_left, int transpose_right, int policy,
                                 const uint64_t *cells, uint64_t cell_count);
uint64_t pcu_oracle_mse(int elem, const void *prediction, const void *target, uint64_t count,
                        int policy, void *out);
uint64_t pcu_oracle_mse_segment(int elem, const void *prediction, const void *target, uint64_t count,
                                uint64_t first_index, uint64_t total_count, int policy, uint64_t *carry,
                                void *out);
uint64_t pcu_oracle_sgd(int elem, const void *weights, const void *gradient, uint32_t rate_bits_f32,
                        uint64_t count, int policy, void *out);
uint64_t pcu_oracle_binary(int elem, int op, const void *left, const void *right, uint64_t count,
                           int left_uniform, int right_uniform, int policy, void *out);
uint64_t pcu_oracle_relu(int elem, const void *input, uint64_t count, int policy, void *out);
uint64_t pcu_oracle_relu_backward(int elem, const void *input, const void *upstream, uint64_t count,
                                  int policy, void *out);

/* ---- fast oracle (fast_ops.c): host IEEE binary32/binary64 arithmetic with
 * FMA contraction disabled, multi-threaded over output rows.  Any cell whose
 * hardware trajectory could hide a fault is recomputed with the soft-float law,
 * so the results and status are identical to pcu_oracle_matmul. ---- */
uint64_t pcu_oracle_fast_matmul(int elem, const void *left, const void *right, void *out,
                                uint64_t rows, uint64_t inner, uint64_t columns,
                                uint64_t left_stride, uint64_t right_stride,
                                int transpose_left, int transpose_right, int policy,
                                uint64_t row_begin, uint64_t row_end, int threads);
uint64_t pcu_oracle_soft_matmul_threads(int elem, const void *left, const void *right, void *out,
                                        uint64_t rows, uint64_t inner, uint64_t columns,
                                        uint64_t left_stride, uint64_t right_stride,
                                        int transpose_left, int transpose_right, int policy,
                                        uint64_t row_begin, uint64_t row_end, int threads);

#ifdef __cplusplus
}
#endif
#endif
