/*
 * pcu_b200_graph.h -- strict tensor graph host layer over the pcu_b200.h kernels.
 *
 * Mirrors, in C++ behind a C ABI, the part of the reference that drives the strict path
 * (paths relative to the Fusion-PCU checkout):
 *   capture builders        Crates/core/dialect/tensor.rs:3925-4345 (Graph::add/sub/mul/div,
 *                           relu, relu_backward, matmul_transposed, mean_squared_error, sgd_update)
 *   reverse mode            Crates/core/dialect/tensor/gradients/gradients.rs:31-444
 *                           (Graph::backward_mse_for, tensor.rs:4359)
 *   plan selection          Crates/core/dialect/tensor.rs:3234-3285 (dependency closure of the
 *                           outputs plus every checked node with its dependencies)
 *   strict execution        Crates/backends/cuda/tensor/tensor.rs:4406-5360 (nodes in graph order,
 *                           one status word per node, the first faulting node wins) and the
 *                           per-node fault decoders (strict_matmul.rs:191-215, strict_sgd.rs:198-219,
 *                           strict_mse.rs:189-222, element faults (index << 3) | kind)
 * A graph has one element type and one underflow policy (the captured function's flags).
 * Capture is pure host code and never touches a GPU; prepare/execute run on one device.
 */
#ifndef PCU_B200_GRAPH_H
#define PCU_B200_GRAPH_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* TensorError variants (Crates/core/dialect/tensor.rs:234-304) that this layer produces */
#define PCU_B200_TENSOR_OK 0
#define PCU_B200_TENSOR_ARITHMETIC_FAULT 1          /* value, element_index, kind */
#define PCU_B200_TENSOR_COMPOUND_ARITHMETIC_FAULT 2 /* value, element_index, reduction_index, step, kind */
#define PCU_B200_TENSOR_SHAPE_MISMATCH 3
#define PCU_B200_TENSOR_MATMUL_SHAPE 4
#define PCU_B200_TENSOR_UNKNOWN_VALUE 5
#define PCU_B200_TENSOR_INVALID_LEARNING_RATE 6
#define PCU_B200_TENSOR_GRADIENT_ROOT_NOT_MSE 7
#define PCU_B200_TENSOR_UNSUPPORTED_GRADIENT 8
#define PCU_B200_TENSOR_EMPTY_OUTPUTS 9
#define PCU_B200_TENSOR_DATA_LENGTH 10
#define PCU_B200_TENSOR_BACKEND 11                  /* CUDA failure or malformed/watchdog status */
#define PCU_B200_TENSOR_FAILED_COMPLETION 12        /* guarded-chain records violate the protocol
                                                       (CudaTensorExecutionError::FailedCompletion) */

/* TensorArithmeticStep (Crates/core/dialect/tensor.rs:425-430) */
#define PCU_B200_STEP_MULTIPLY 0
#define PCU_B200_STEP_ADD 1
#define PCU_B200_STEP_SUBTRACT 2
#define PCU_B200_STEP_DIVIDE 3

/* node operations (OpDescriptor, Crates/core/dialect/tensor.rs:375-421) */
#define PCU_B200_NODE_INPUT 0
#define PCU_B200_NODE_UNIFORM 1
#define PCU_B200_NODE_ADD 2
#define PCU_B200_NODE_SUB 3
#define PCU_B200_NODE_MUL 4
#define PCU_B200_NODE_DIV 5
#define PCU_B200_NODE_RELU 6
#define PCU_B200_NODE_RELU_BACKWARD 7
#define PCU_B200_NODE_MATMUL 8
#define PCU_B200_NODE_MEAN_SQUARED_ERROR 9
#define PCU_B200_NODE_SGD_UPDATE 10

typedef struct {
    int32_t code;             /* PCU_B200_TENSOR_* */
    int32_t value;            /* node id the error belongs to (-1 if none) */
    uint64_t element_index;
    uint64_t reduction_index;
    int32_t step;             /* PCU_B200_STEP_* for compound faults */
    int32_t kind;             /* fault kind 1..5 (pcu_b200.h) */
    int32_t backend;          /* pcu_b200 return code or cudaError_t for PCU_B200_TENSOR_BACKEND */
} pcu_b200_tensor_error;

typedef struct pcu_b200_graph pcu_b200_graph;
typedef struct pcu_b200_prepared pcu_b200_prepared;

/* ---- capture (host only) ------------------------------------------------------------ */
pcu_b200_graph *pcu_b200_graph_new(int dtype, int policy);
void pcu_b200_graph_free(pcu_b200_graph *graph);
/* Every builder returns the new value id, or -1 with *error filled. shape: rank 0..2. */
int32_t pcu_b200_graph_input(pcu_b200_graph *graph, const uint64_t *shape, int rank, pcu_b200_tensor_error *error);
int32_t pcu_b200_graph_uniform(pcu_b200_graph *graph, const uint64_t *shape, int rank, uint64_t value_bits,
                               pcu_b200_tensor_error *error);
int32_t pcu_b200_graph_binary(pcu_b200_graph *graph, int op, int32_t left, int32_t right,
                              pcu_b200_tensor_error *error); /* op: PCU_B200_ADD..PCU_B200_DIV */
int32_t pcu_b200_graph_relu(pcu_b200_graph *graph, int32_t input, pcu_b200_tensor_error *error);
int32_t pcu_b200_graph_relu_backward(pcu_b200_graph *graph, int32_t input, int32_t upstream,
                                     pcu_b200_tensor_error *error);
int32_t pcu_b200_graph_matmul(pcu_b200_graph *graph, int32_t left, int32_t right, int transpose_left,
                              int transpose_right, pcu_b200_tensor_error *error);
int32_t pcu_b200_graph_mean_squared_error(pcu_b200_graph *graph, int32_t prediction, int32_t target,
                                          pcu_b200_tensor_error *error);
int32_t pcu_b200_graph_sgd_update(pcu_b200_graph *graph, int32_t weights, int32_t gradient, uint32_t rate_bits_f32,
                                  pcu_b200_tensor_error *error);
/* Graph::backward_mse_for(loss, target): appends the reverse-mode nodes and returns the value
 * holding d loss / d target. */
int32_t pcu_b200_graph_gradient(pcu_b200_graph *graph, int32_t loss, int32_t target, pcu_b200_tensor_error *error);
/* Graph::backward_mse_for_targets(loss, targets) (gradients.rs:289-303): one shared reverse pass;
 * gradients[j] receives d loss / d targets[j].  Returns 0 or a PCU_B200_TENSOR_* code. */
int pcu_b200_graph_gradients(pcu_b200_graph *graph, int32_t loss, const int32_t *targets, int count,
                             int32_t *gradients, pcu_b200_tensor_error *error);

/* Introspection (tests): node count and one node's description. */
int32_t pcu_b200_graph_node_count(const pcu_b200_graph *graph);
int pcu_b200_graph_describe(const pcu_b200_graph *graph, int32_t value, int32_t *op, int32_t *left, int32_t *right,
                            int32_t *transpose_left, int32_t *transpose_right, uint64_t *shape, int32_t *rank,
                            uint64_t *scalar_bits);

/* ---- prepared execution on one device ----------------------------------------------- */
/* Plans the outputs' dependency closure plus every checked node, allocates one device buffer
 * per planned value, one status word per node and the largest workspace, and uploads uniform
 * constants.  The current CUDA device is used. */
pcu_b200_prepared *pcu_b200_graph_prepare(const pcu_b200_graph *graph, const int32_t *outputs, int count,
                                          pcu_b200_tensor_error *error);
void pcu_b200_prepared_free(pcu_b200_prepared *prepared);
/* Number of graph inputs the plan binds, in capture order, and the value id of input i. */
int32_t pcu_b200_prepared_input_count(const pcu_b200_prepared *prepared);
int32_t pcu_b200_prepared_input_value(const pcu_b200_prepared *prepared, int32_t index);
/* How many of the nodes planned right after MatMul node `value` run in its epilogue in the
 * chained mode (pcu_b200_strict_matmul_epilogue): elementwise nodes of the same shape (checked
 * Add/Sub/Mul/Div, ReLU, ReLU-backward) that take the previous node's result as one operand, at
 * most PCU_B200_EPILOGUE_MAX.  0 for every other node and in the other modes' sense: the
 * each-node and guarded modes run one kernel per node. */
int pcu_b200_prepared_fused(const pcu_b200_prepared *p, int32_t value);

/* Device buffer of a planned value (inputs can be written there directly). */
void *pcu_b200_prepared_buffer(const pcu_b200_prepared *prepared, int32_t value);

/* Execution modes of pcu_b200_prepared_execute */
#define PCU_B200_EXEC_CHAINED 0   /* every node launched back to back; one status read at the end */
#define PCU_B200_EXEC_EACH_NODE 1 /* the reference's protocol: one host wait and status read per node */
#define PCU_B200_EXEC_GRAPH 2     /* the guarded chain replayed as one CUDA graph; one read at the end */
#define PCU_B200_EXEC_GUARDED 3   /* the guarded chain launched back to back; one read at the end */

/* Guarded stage chain (Crates/backends/cuda/owned_dispatch/guarded/guarded.rs:15-38,
 * Crates/core/runtime/execution/guarded/guarded.rs:30-147).  Every planned node that launches
 * work is a stage with a fault word and a disposition.  A stage runs only when its predecessor
 * executed with a clear fault word; otherwise it is skipped and touches no user data: no loads,
 * no arithmetic and no output writes after the first fault.  The single observation at the
 * end reads every record and validates the chain as the reference does.  The stages in front of
 * the first fault must have executed cleanly, and the stages after it must be skipped with a
 * clear word.  A violation returns PCU_B200_TENSOR_FAILED_COMPLETION. */
#define PCU_B200_DISPOSITION_PENDING 0
#define PCU_B200_DISPOSITION_EXECUTED 1
#define PCU_B200_DISPOSITION_SKIPPED 2

/* Execute: copies `host_inputs` (one host pointer per planned input, NULL = already on the
 * device buffer) to the device, runs every planned node in graph order on `stream`, and
 * reports the first faulting node exactly as the reference does (every mode gives the same
 * answer: the lowest faulting node, and in it the lowest event).  PCU_B200_EXEC_GRAPH records
 * the plan's launches as a CUDA graph on the first call on a stream (that call runs the plan
 * normally) and replays it afterwards; with the legacy stream (NULL) the prepared graph uses a
 * stream of its own.  Returns 0 on success or a PCU_B200_TENSOR_* code (details in *error). */
int pcu_b200_prepared_execute(pcu_b200_prepared *prepared, const void *const *host_inputs, int mode,
                              void *stream, pcu_b200_tensor_error *error);
/* The last execution's record of a planned node: its fault word and, for the guarded modes,
 * its disposition (PCU_B200_DISPOSITION_*). */
int pcu_b200_prepared_stage(const pcu_b200_prepared *prepared, int32_t value, uint64_t *fault_word,
                            uint64_t *disposition, void *stream);
/* Copy a planned value back to host memory (bytes must cover the value). */
int pcu_b200_prepared_read(const pcu_b200_prepared *prepared, int32_t value, void *host, size_t bytes, void *stream);

#ifdef __cplusplus
}
#endif
#endif
