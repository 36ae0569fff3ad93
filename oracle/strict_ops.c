/*
 * strict_ops.c -- TEST INFRASTRUCTURE ONLY (see pcu_oracle.h).
 *
 * Ordered strict tensor primitives on top of the soft-float law, in the exact
 * loop order of the reference's strict CPU provider (the path the north star
 * names as the parity target and the timed CPU baseline):
 *   elementwise Add/Sub/Mul/Div  Crates/backends/cpu/prepared_tensor/execution/execution.rs:192-211
 *   ReLU                         execution.rs:212-219
 *   ReLU backward                execution.rs:220-230
 *   SGD  (rate*g, then w-p)      execution.rs:231-242 (core: reference/strict_sgd/strict_sgd.rs:20-46)
 *   MatMul (ordered K from +0)   execution.rs:243-281 (core: reference/strict_matmul/strict_matmul.rs:22-73)
 *   MSE  (sub, mul, add; div)    execution.rs:282-302 (core: reference/strict_mse/strict_mse.rs:22-59)
 * Fault positions use the reference's ordinal domains
 * (Crates/core/dialect/tensor/fault_domain/fault_domain.rs:122-171):
 *   MatMul (cell*K + k)*2 + {Multiply 0, Add 1};  SGD i*2 + {Multiply 0, Subtract 1};
 *   MSE i*3 + {Subtract 0, Multiply 1, Add 2}, Divide = 3n;  elementwise: element index.
 * The first fault in loop order stops the primitive, exactly as the `?` in the
 * reference loops does; the status word is (event << 3) | kind.
 */
#include <stdint.h>
#include <string.h>

#include "pcu_oracle.h"

#define STATUS_OK UINT64_MAX

static inline uint64_t status_of(uint64_t event, int kind) { return (event << 3) | (uint64_t)kind; }

static inline int binop(int elem, uint64_t a, uint64_t b, int op, int policy, uint64_t *out)
{
    if (elem == 4) {
        uint32_t r = 0;
        int kind = pcu_oracle_f32_binary((uint32_t)a, (uint32_t)b, op, policy, &r);
        *out = r;
        return kind;
    }
    return pcu_oracle_f64_binary(a, b, op, policy, out);
}

static inline uint64_t load(int elem, const void *base, uint64_t index)
{
    if (elem == 4) return ((const uint32_t *)base)[index];
    return ((const uint64_t *)base)[index];
}

static inline void store(int elem, void *base, uint64_t index, uint64_t value)
{
    if (elem == 4) ((uint32_t *)base)[index] = (uint32_t)value;
    else ((uint64_t *)base)[index] = value;
}

/* One output cell of the ordered dot product.  Returns 0 or the fault kind and
 * the failing (k, step) through *k_out / *step_out. */
static int matmul_cell(int elem, const void *left, const void *right,
                       uint64_t row, uint64_t column, uint64_t inner,
                       uint64_t left_stride, uint64_t right_stride,
                       int transpose_left, int transpose_right, int policy,
                       uint64_t *value, uint64_t *k_out, int *step_out)
{
    uint64_t total = 0; /* +0 */
    for (uint64_t k = 0; k < inner; ++k) {
        uint64_t li = transpose_left ? k * left_stride + row : row * left_stride + k;
        uint64_t ri = transpose_right ? column * right_stride + k : k * right_stride + column;
        uint64_t product = 0;
        int kind = binop(elem, load(elem, left, li), load(elem, right, ri), 2, policy, &product);
        if (kind) { *k_out = k; *step_out = 0; return kind; }
        kind = binop(elem, total, product, 0, policy, &total);
        if (kind) { *k_out = k; *step_out = 1; return kind; }
    }
    *value = total;
    return 0;
}

uint64_t pcu_oracle_matmul(int elem, const void *left, const void *right, void *out,
                           uint64_t rows, uint64_t inner, uint64_t columns,
                           uint64_t left_stride, uint64_t right_stride,
                           int transpose_left, int transpose_right, int policy,
                           uint64_t row_begin, uint64_t row_end)
{
    if (row_end > rows) row_end = rows;
    for (uint64_t row = row_begin; row < row_end; ++row) {
        for (uint64_t column = 0; column < columns; ++column) {
            uint64_t cell = row * columns + column;
            uint64_t value = 0, k = 0;
            int step = 0;
            int kind = matmul_cell(elem, left, right, row, column, inner, left_stride, right_stride,
                                   transpose_left, transpose_right, policy, &value, &k, &step);
            if (kind) return status_of((cell * inner + k) * 2 + (uint64_t)step, kind);
            store(elem, out, cell, value);
        }
    }
    return STATUS_OK;
}

/* Same arithmetic for an explicit list of cells (ascending order not required);
 * returns the minimum status over the listed cells, which is what the full
 * primitive reports when only these cells can fault. */
uint64_t pcu_oracle_matmul_cells(int elem, const void *left, const void *right, void *out,
                                 uint64_t rows, uint64_t inner, uint64_t columns,
                                 uint64_t left_stride, uint64_t right_stride,
                                 int transpose_left, int transpose_right, int policy,
                                 const uint64_t *cells, uint64_t cell_count)
{
    uint64_t status = STATUS_OK;
    (void)rows;
    for (uint64_t i = 0; i < cell_count; ++i) {
        uint64_t cell = cells[i];
        uint64_t value = 0, k = 0;
        int step = 0;
        int kind = matmul_cell(elem, left, right, cell / columns, cell % columns, inner, left_stride,
                               right_stride, transpose_left, transpose_right, policy, &value, &k, &step);
        if (kind) {
            uint64_t s = status_of((cell * inner + k) * 2 + (uint64_t)step, kind);
            if (s < status) status = s;
        } else {
            store(elem, out, i, value);
        }
    }
    return status;
}

/* One segment [first_index, first_index + count) of the ordered MSE reduction over
 * total_count elements: the loop of pcu_oracle_mse started from the running sum *carry
 * (bits) instead of +0, with global event ordinals.  *carry receives the running sum after
 * the segment; the last segment (out != NULL) also divides by count(total_count).  Splitting
 * the reduction this way is exactly the one-pass loop, since each step only reads the sum. */
uint64_t pcu_oracle_mse_segment(int elem, const void *prediction, const void *target, uint64_t count,
                                uint64_t first_index, uint64_t total_count, int policy, uint64_t *carry,
                                void *out)
{
    uint64_t total = *carry;
    for (uint64_t i = 0; i < count; ++i) {
        const uint64_t g = first_index + i;
        uint64_t difference = 0, square = 0;
        int kind = binop(elem, load(elem, prediction, i), load(elem, target, i), 1, policy, &difference);
        if (kind) return status_of(g * 3, kind);
        kind = binop(elem, difference, difference, 2, policy, &square);
        if (kind) return status_of(g * 3 + 1, kind);
        kind = binop(elem, total, square, 0, policy, &total);
        if (kind) return status_of(g * 3 + 2, kind);
    }
    *carry = total;
    if (!out) return STATUS_OK;
    uint64_t denominator = elem == 4 ? pcu_oracle_count_f32(total_count) : pcu_oracle_count_f64(total_count);
    uint64_t mean = 0;
    int kind = binop(elem, total, denominator, 3, policy, &mean);
    if (kind) return status_of(total_count * 3, kind);
    store(elem, out, 0, mean);
    return STATUS_OK;
}

uint64_t pcu_oracle_mse(int elem, const void *prediction, const void *target, uint64_t count,
                        int policy, void *out)
{
    uint64_t carry = 0;
    return pcu_oracle_mse_segment(elem, prediction, target, count, 0, count, policy, &carry, out);
}

uint64_t pcu_oracle_sgd(int elem, const void *weights, const void *gradient, uint32_t rate_bits_f32,
                        uint64_t count, int policy, void *out)
{
    uint64_t rate = elem == 4 ? rate_bits_f32 : pcu_oracle_f32_bits_to_f64_bits(rate_bits_f32);
    for (uint64_t i = 0; i < count; ++i) {
        uint64_t product = 0, updated = 0;
        int kind = binop(elem, rate, load(elem, gradient, i), 2, policy, &product);
        if (kind) return status_of(i * 2, kind);
        kind = binop(elem, load(elem, weights, i), product, 1, policy, &updated);
        if (kind) return status_of(i * 2 + 1, kind);
        store(elem, out, i, updated);
    }
    return STATUS_OK;
}

uint64_t pcu_oracle_binary(int elem, int op, const void *left, const void *right, uint64_t count,
                           int left_uniform, int right_uniform, int policy, void *out)
{
    for (uint64_t i = 0; i < count; ++i) {
        uint64_t value = 0;
        int kind = binop(elem, load(elem, left, left_uniform ? 0 : i), load(elem, right, right_uniform ? 0 : i),
                         op, policy, &value);
        if (kind) return status_of(i, kind);
        store(elem, out, i, value);
    }
    return STATUS_OK;
}

uint64_t pcu_oracle_relu(int elem, const void *input, uint64_t count, int policy, void *out)
{
    for (uint64_t i = 0; i < count; ++i) {
        int kind;
        if (elem == 4) {
            uint32_t r = 0;
            kind = pcu_oracle_f32_relu(((const uint32_t *)input)[i], policy, &r);
            if (!kind) ((uint32_t *)out)[i] = r;
        } else {
            uint64_t r = 0;
            kind = pcu_oracle_f64_relu(((const uint64_t *)input)[i], policy, &r);
            if (!kind) ((uint64_t *)out)[i] = r;
        }
        if (kind) return status_of(i, kind);
    }
    return STATUS_OK;
}

uint64_t pcu_oracle_relu_backward(int elem, const void *input, const void *upstream, uint64_t count,
                                  int policy, void *out)
{
    for (uint64_t i = 0; i < count; ++i) {
        int kind;
        if (elem == 4) {
            uint32_t r = 0;
            kind = pcu_oracle_f32_relu_backward(((const uint32_t *)input)[i], ((const uint32_t *)upstream)[i],
                                                policy, &r);
            if (!kind) ((uint32_t *)out)[i] = r;
        } else {
            uint64_t r = 0;
            kind = pcu_oracle_f64_relu_backward(((const uint64_t *)input)[i], ((const uint64_t *)upstream)[i],
                                                policy, &r);
            if (!kind) ((uint64_t *)out)[i] = r;
        }
        if (kind) return status_of(i, kind);
    }
    return STATUS_OK;
}
