// provider.h -- the C++ entry points behind the node calls of pcu_b200.h.  Each takes the same
// arguments as its C function plus the guard of the guarded stage chain (common.cuh); the C
// functions pass an empty guard, the graph layer (tensor_graph.cu) passes a real one.
#pragma once

#include <cstddef>
#include <cstdint>

#include "common.cuh"
#include "pcu_b200.h"

namespace pcu {

int strict_matmul(int dtype, int policy, const void *left, const void *right, void *out, uint64_t rows,
                  uint64_t inner, uint64_t columns, uint64_t left_stride, uint64_t right_stride, int transpose_left,
                  int transpose_right, void *workspace, size_t workspace_bytes, uint64_t *status, void *stream,
                  const ChainGuard &guard, const pcu_b200_epilogue_stage *stages = nullptr, int stage_count = 0);
int strict_sgd(int dtype, int policy, const void *weights, const void *gradient, void *out, uint64_t count,
               uint32_t rate_bits_f32, uint64_t *status, void *stream, const ChainGuard &guard);
int strict_mse(int dtype, int policy, const void *prediction, const void *target, void *out, uint64_t count,
               void *workspace, size_t workspace_bytes, uint64_t *status, void *stream, const ChainGuard &guard);
int checked_binary(int dtype, int policy, int op, const void *left, const void *right, void *out, uint64_t count,
                   int left_uniform, int right_uniform, uint64_t *status, void *stream, const ChainGuard &guard);
int checked_relu(int dtype, int policy, const void *input, void *out, uint64_t count, uint64_t *status,
                 void *stream, const ChainGuard &guard);
int checked_relu_backward(int dtype, int policy, const void *input, const void *upstream, void *out,
                          uint64_t count, uint64_t *status, void *stream, const ChainGuard &guard);

// For a stage that launches no kernel (an empty tensor): records its disposition alone.
int chain_decide_only(const ChainGuard &guard, cudaStream_t stream);

}  // namespace pcu
