/*
 * fast_ops.c -- TEST INFRASTRUCTURE ONLY (see pcu_oracle.h).
 *
 * A faster CPU checker for the ordered strict MatMul, used for parity at sizes
 * the soft-float loop cannot finish in seconds.  It is NOT the reference path;
 * its results are defined to equal pcu_oracle_matmul bit for bit:
 *
 *  - Each cell walks k in increasing order with separately rounded host IEEE
 *    multiply and add (the file is compiled with -ffp-contract=off, no fast-math,
 *    with the default SSE environment: no flush-to-zero, no denormals-are-zero).
 *    When no step faults under the checked law, these are exactly the law's
 *    results (the reference pins this equality for random finite pairs,
 *    Crates/core/scalar_checked_float/tests.rs:306-353).
 *  - A cell is re-run with the soft-float law when its trajectory could hide a
 *    fault: the final sum is not finite (overflow and invalid operands are
 *    sticky through IEEE add/multiply), a product of nonzero operands has
 *    magnitude <= the smallest normal (possible tiny-inexact product, including
 *    the round-up-to-MIN_NORMAL case of tests.rs:228-241), or, under
 *    RejectSubnormalResult, a nonzero sum is subnormal.
 *
 * pcu_oracle_soft_matmul_threads is the soft-float law itself, split across
 * threads by rows, for the all-core CPU reference timing.
 */
#include <float.h>
#include <math.h>
#include <pthread.h>
#include <stdbool.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "pcu_oracle.h"

#define STATUS_OK UINT64_MAX
#define COLUMN_BLOCK 512

typedef struct {
    int elem;
    const void *left, *right;
    void *out;
    uint64_t rows, inner, columns, left_stride, right_stride;
    int transpose_left, transpose_right, policy;
    const void *right_kn; /* op(right) densely as inner x columns */
    uint64_t row_begin, row_end;
    int thread_index, thread_count;
    int soft;
    uint64_t status;
} job;

static void soft_cell(job *j, uint64_t row, uint64_t column)
{
    uint64_t cell = row * j->columns + column;
    uint64_t value = 0;
    /* Reuse the public per-cell path: one listed cell. */
    uint64_t status = pcu_oracle_matmul_cells(j->elem, j->left, j->right, &value, j->rows, j->inner,
                                              j->columns, j->left_stride, j->right_stride,
                                              j->transpose_left, j->transpose_right, j->policy, &cell, 1);
    if (status != STATUS_OK) {
        if (status < j->status) j->status = status;
    } else if (j->elem == 4) {
        ((uint32_t *)j->out)[cell] = (uint32_t)value;
    } else {
        ((uint64_t *)j->out)[cell] = value;
    }
}

static void fast_row_f32(job *j, uint64_t row)
{
    float acc[COLUMN_BLOCK];
    unsigned char flag[COLUMN_BLOCK];
    const float *left = (const float *)j->left;
    const float *bkn = (const float *)j->right_kn;
    float *out = (float *)j->out;
    for (uint64_t c0 = 0; c0 < j->columns; c0 += COLUMN_BLOCK) {
        uint64_t width = j->columns - c0 < COLUMN_BLOCK ? j->columns - c0 : COLUMN_BLOCK;
        for (uint64_t c = 0; c < width; ++c) { acc[c] = 0.0f; flag[c] = 0; }
        for (uint64_t k = 0; k < j->inner; ++k) {
            float a = j->transpose_left ? left[k * j->left_stride + row] : left[row * j->left_stride + k];
            const float *b = bkn + k * j->columns + c0;
            bool check_tiny = j->policy != 2 && a != 0.0f;
            for (uint64_t c = 0; c < width; ++c) {
                float p = a * b[c];
                float s = acc[c] + p;
                unsigned char f = 0;
                if (check_tiny) f |= (unsigned char)((fabsf(p) <= FLT_MIN) & (b[c] != 0.0f));
                if (j->policy == 1) f |= (unsigned char)((s != 0.0f) & (fabsf(s) < FLT_MIN));
                flag[c] |= f;
                acc[c] = s;
            }
        }
        for (uint64_t c = 0; c < width; ++c) {
            if (flag[c] || !isfinite(acc[c])) soft_cell(j, row, c0 + c);
            else out[row * j->columns + c0 + c] = acc[c];
        }
    }
}

static void fast_row_f64(job *j, uint64_t row)
{
    double acc[COLUMN_BLOCK];
    unsigned char flag[COLUMN_BLOCK];
    const double *left = (const double *)j->left;
    const double *bkn = (const double *)j->right_kn;
    double *out = (double *)j->out;
    for (uint64_t c0 = 0; c0 < j->columns; c0 += COLUMN_BLOCK) {
        uint64_t width = j->columns - c0 < COLUMN_BLOCK ? j->columns - c0 : COLUMN_BLOCK;
        for (uint64_t c = 0; c < width; ++c) { acc[c] = 0.0; flag[c] = 0; }
        for (uint64_t k = 0; k < j->inner; ++k) {
            double a = j->transpose_left ? left[k * j->left_stride + row] : left[row * j->left_stride + k];
            const double *b = bkn + k * j->columns + c0;
            bool check_tiny = j->policy != 2 && a != 0.0;
            for (uint64_t c = 0; c < width; ++c) {
                double p = a * b[c];
                double s = acc[c] + p;
                unsigned char f = 0;
                if (check_tiny) f |= (unsigned char)((fabs(p) <= DBL_MIN) & (b[c] != 0.0));
                if (j->policy == 1) f |= (unsigned char)((s != 0.0) & (fabs(s) < DBL_MIN));
                flag[c] |= f;
                acc[c] = s;
            }
        }
        for (uint64_t c = 0; c < width; ++c) {
            if (flag[c] || !isfinite(acc[c])) soft_cell(j, row, c0 + c);
            else out[row * j->columns + c0 + c] = acc[c];
        }
    }
}

static void *run_job(void *arg)
{
    job *j = (job *)arg;
    for (uint64_t row = j->row_begin + (uint64_t)j->thread_index; row < j->row_end;
         row += (uint64_t)j->thread_count) {
        if (j->soft) {
            for (uint64_t c = 0; c < j->columns; ++c) soft_cell(j, row, c);
        } else if (j->elem == 4) {
            fast_row_f32(j, row);
        } else {
            fast_row_f64(j, row);
        }
    }
    return NULL;
}

static uint64_t run_threads(job *proto, int threads)
{
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    job jobs[256];
    pthread_t ids[256];
    for (int t = 0; t < threads; ++t) {
        jobs[t] = *proto;
        jobs[t].thread_index = t;
        jobs[t].thread_count = threads;
        jobs[t].status = STATUS_OK;
    }
    for (int t = 1; t < threads; ++t) pthread_create(&ids[t], NULL, run_job, &jobs[t]);
    run_job(&jobs[0]);
    uint64_t status = jobs[0].status;
    for (int t = 1; t < threads; ++t) {
        pthread_join(ids[t], NULL);
        if (jobs[t].status < status) status = jobs[t].status;
    }
    return status;
}

uint64_t pcu_oracle_fast_matmul(int elem, const void *left, const void *right, void *out,
                                uint64_t rows, uint64_t inner, uint64_t columns,
                                uint64_t left_stride, uint64_t right_stride,
                                int transpose_left, int transpose_right, int policy,
                                uint64_t row_begin, uint64_t row_end, int threads)
{
    if (row_end > rows) row_end = rows;
    size_t bytes = (size_t)inner * (size_t)columns * (size_t)elem;
    void *kn = malloc(bytes ? bytes : 1);
    if (!kn) return STATUS_OK - 1; /* impossible status: caller treats as error */
    for (uint64_t k = 0; k < inner; ++k) {
        for (uint64_t c = 0; c < columns; ++c) {
            uint64_t src = transpose_right ? c * right_stride + k : k * right_stride + c;
            if (elem == 4) ((uint32_t *)kn)[k * columns + c] = ((const uint32_t *)right)[src];
            else ((uint64_t *)kn)[k * columns + c] = ((const uint64_t *)right)[src];
        }
    }
    job proto;
    memset(&proto, 0, sizeof proto);
    proto.elem = elem;
    proto.left = left;
    proto.right = right;
    proto.out = out;
    proto.rows = rows;
    proto.inner = inner;
    proto.columns = columns;
    proto.left_stride = left_stride;
    proto.right_stride = right_stride;
    proto.transpose_left = transpose_left;
    proto.transpose_right = transpose_right;
    proto.policy = policy;
    proto.right_kn = kn;
    proto.row_begin = row_begin;
    proto.row_end = row_end;
    proto.soft = 0;
    uint64_t status = run_threads(&proto, threads);
    free(kn);
    return status;
}

uint64_t pcu_oracle_soft_matmul_threads(int elem, const void *left, const void *right, void *out,
                                        uint64_t rows, uint64_t inner, uint64_t columns,
                                        uint64_t left_stride, uint64_t right_stride,
                                        int transpose_left, int transpose_right, int policy,
                                        uint64_t row_begin, uint64_t row_end, int threads)
{
    if (row_end > rows) row_end = rows;
    job proto;
    memset(&proto, 0, sizeof proto);
    proto.elem = elem;
    proto.left = left;
    proto.right = right;
    proto.out = out;
    proto.rows = rows;
    proto.inner = inner;
    proto.columns = columns;
    proto.left_stride = left_stride;
    proto.right_stride = right_stride;
    proto.transpose_left = transpose_left;
    proto.transpose_right = transpose_right;
    proto.policy = policy;
    proto.row_begin = row_begin;
    proto.row_end = row_end;
    proto.soft = 1;
    return run_threads(&proto, threads);
}
