/*
 * pcu_b200.h -- C ABI of the B200 (sm_100a) strict-tensor CUDA provider for Fusion-PCU.
 *
 * Each entry point replaces one per-node executor of the reference's CUDA provider
 * (paths relative to the Fusion-PCU checkout):
 *
 *   pcu_b200_strict_matmul          CudaTensorAssessor::execute_strict_matmul
 *                                   Crates/backends/cuda/tensor/strict_matmul/strict_matmul.rs:278-332
 *   pcu_b200_strict_sgd             execute_strict_sgd        tensor/strict_sgd/strict_sgd.rs:234-289
 *   pcu_b200_strict_mse             execute_strict_mse        tensor/strict_mse/strict_mse.rs:234-291
 *   pcu_b200_checked_binary         execute_elementwise       tensor/tensor.rs:5657 (checked Add/Sub/Mul/Div,
 *                                   uniform operands as in the scalar mask of tensor.rs:4813-4826)
 *   pcu_b200_checked_relu           ReLU node                 tensor/tensor.rs:4944 (helper
 *                                   codegen/lower/checked_float/checked_float.rs:606-626)
 *   pcu_b200_checked_relu_backward  execute_admitted_relu_backward tensor/relu_backward/relu_backward.rs:298
 *
 * Contract shared by all entry points (the reference's fusion_kernel ABI,
 * strict_matmul.rs:335-343, owned_dispatch/owned_dispatch.rs:20-22,70-109):
 *   - Every data pointer is DEVICE memory owned by the caller; the library never frees it.
 *   - `status` points to one device uint64 that the caller initialised to UINT64_MAX
 *     (pcu_b200_status_reset).  A checked arithmetic fault is reported ONLY there, as
 *     (event << 3) | kind with kinds 1 DivideByZero, 2 SignedDivisionOverflow,
 *     3 ArithmeticOverflow, 4 ArithmeticUnderflow, 5 InvalidFloatingOperand; the lowest
 *     event wins (atomicMin).  Event ordinals are the reference's fault domains
 *     (Crates/core/dialect/tensor/fault_domain/fault_domain.rs:122-171):
 *       matmul  (cell * inner + k) * 2 + {0 Multiply, 1 Add},   cell = row * columns + column
 *       sgd     index * 2 + {0 Multiply, 1 Subtract}
 *       mse     index * 3 + {0 Subtract, 1 Multiply, 2 Add};  3 * count = Divide
 *       elementwise / relu / relu_backward: the element index
 *     Kind 7 (PCU_B200_STATUS_WATCHDOG) means a device wait gave up; it is a provider
 *     failure, never an arithmetic fault, and the reference decoder rejects it as malformed.
 *   - Outputs are written even when a fault is recorded; a caller publishes them only
 *     after reading the sentinel back (nothing is published on fault).
 *   - The int return is PCU_B200_OK or a host-side error (argument validation, shape or
 *     event-domain overflow, CUDA launch failure).  Calls are asynchronous on `stream`
 *     (a cudaStream_t, NULL = legacy default stream), never synchronise the host, and are
 *     reentrant per (device, stream).
 *   - dtype: PCU_B200_F32 or PCU_B200_F64.  policy: the checked-float underflow policy
 *     (Crates/core/scalar_float_underflow.rs:47-56).
 */
#ifndef PCU_B200_H
#define PCU_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PCU_B200_ABI_VERSION 2

/* element types (PcuScalarType::F32 / F64) */
#define PCU_B200_F32 0
#define PCU_B200_F64 1

/* PcuFloatUnderflowPolicy */
#define PCU_B200_IEEE_AFTER_ROUNDING 0
#define PCU_B200_REJECT_SUBNORMAL_RESULT 1
#define PCU_B200_ALLOW_GRADUAL_UNDERFLOW 2

/* checked binary op tags (PcuDispatchFloatBinaryOp, checked_float.rs:230-235) */
#define PCU_B200_ADD 0
#define PCU_B200_SUB 1
#define PCU_B200_MUL 2
#define PCU_B200_DIV 3

/* status word */
#define PCU_B200_STATUS_OK UINT64_MAX
#define PCU_B200_KIND_DIVIDE_BY_ZERO 1
#define PCU_B200_KIND_SIGNED_DIVISION_OVERFLOW 2
#define PCU_B200_KIND_OVERFLOW 3
#define PCU_B200_KIND_UNDERFLOW 4
#define PCU_B200_KIND_INVALID 5
#define PCU_B200_STATUS_WATCHDOG 7

/* host return codes */
#define PCU_B200_OK 0
#define PCU_B200_ERROR_INVALID_ARGUMENT 1
#define PCU_B200_ERROR_SIZE_OVERFLOW 2
#define PCU_B200_ERROR_WORKSPACE 3
#define PCU_B200_ERROR_CUDA 4
#define PCU_B200_ERROR_UNSUPPORTED 5
#define PCU_B200_ERROR_TIMEOUT 6

/* ------------------------------------------------------------------ library */

/* PCU_B200_ABI_VERSION of the loaded library. */
int pcu_b200_abi_version(void);

/* Static description of a host return code. */
const char *pcu_b200_error_string(int code);

/* The cudaError_t behind the calling thread's last PCU_B200_ERROR_CUDA (0 if none). */
int pcu_b200_last_cuda_error(void);

/* Fill `count` status words with UINT64_MAX (owned_scratch::submit's reset,
 * Crates/backends/cuda/owned_dispatch/fault_word.rs:17-31). */
int pcu_b200_status_reset(uint64_t *status, uint64_t count, void *stream);

/* ------------------------------------------------------------------ strict MatMul */

/* Device workspace bytes pcu_b200_strict_matmul needs for this shape (row/column
 * operand-exponent minima used to prove that no product can underflow). */
size_t pcu_b200_strict_matmul_workspace_size(uint64_t rows, uint64_t inner, uint64_t columns);

/* out[rows x columns] (dense, row-major) = op(left) . op(right), each cell folding k = 0..inner-1
 * in increasing order from +0 with a separately rounded, checked multiply then add
 * (reference: Crates/core/dialect/tensor/reference/strict_matmul/strict_matmul.rs:22-73).
 * left is stored row-major as rows x inner (or inner x rows when transpose_left) with row
 * stride left_stride elements; right as inner x columns (or columns x inner when
 * transpose_right) with row stride right_stride.  inner may be 0 (out = +0).
 * Rejects rows*columns*inner*2 > 2^60 (the reference's packed event bound,
 * strict_matmul.rs:121-127) with PCU_B200_ERROR_SIZE_OVERFLOW. */
int pcu_b200_strict_matmul(int dtype, int policy, const void *left, const void *right, void *out,
                           uint64_t rows, uint64_t inner, uint64_t columns, uint64_t left_stride,
                           uint64_t right_stride, int transpose_left, int transpose_right, void *workspace,
                           size_t workspace_bytes, uint64_t *status, void *stream);

/* Strict MatMul with up to PCU_B200_EPILOGUE_MAX elementwise nodes fused into its epilogue: the
 * graph's MatMul -> bias Add -> ReLU of a layer, or MatMul -> ReLU-backward of the backward
 * pass, computed by one kernel.  Stage s applies a checked node to the previous value (the
 * MatMul's result for stage 0): a checked binary op (PCU_B200_ADD..DIV) with `operand` as its
 * other argument (an array laid out like out, rows x columns dense, or one element when
 * operand_uniform; operand_left puts it on the left: op(operand, value)),
 * PCU_B200_EPILOGUE_RELU, or PCU_B200_EPILOGUE_RELU_BACKWARD (relu_backward(x, dy), see below).
 * Each stage writes
 * its own output and records its first fault in its own status word, with the element-index
 * events of the unfused node (tensor.rs:5657, relu_backward.rs:259-281), so the lowest faulting
 * node in graph order and its event are exactly those of the unfused sequence: a cell whose
 * MatMul (or earlier stage) faulted runs no later stage, and an earlier node's fault is always
 * reported first.  out (the MatMul's own result) is written too.  For
 * PCU_B200_EPILOGUE_RELU_BACKWARD, operand_left = 1 means operand is the forward input x and the
 * value is the upstream gradient dy; operand_left = 0 the opposite.  Not for guarded chains.
 * No counterpart call in the reference, which runs these nodes one by one
 * (tensor/tensor.rs:4714-4727, 4891-4943). */
#define PCU_B200_EPILOGUE_MAX 2
#define PCU_B200_EPILOGUE_RELU 4
#define PCU_B200_EPILOGUE_RELU_BACKWARD 5
typedef struct pcu_b200_epilogue_stage {
    int op;
    const void *operand;
    int operand_uniform;
    int operand_left;
    void *out;
    uint64_t *status;
} pcu_b200_epilogue_stage;
int pcu_b200_strict_matmul_epilogue(int dtype, int policy, const void *left, const void *right, void *out,
                                    uint64_t rows, uint64_t inner, uint64_t columns, uint64_t left_stride,
                                    uint64_t right_stride, int transpose_left, int transpose_right,
                                    const pcu_b200_epilogue_stage *stages, int stage_count, void *workspace,
                                    size_t workspace_bytes, uint64_t *status, void *stream);

/* pcu_b200_strict_matmul for callers that cannot allocate device memory.  It has no
 * counterpart in the reference.
 *
 * Some callers are handed only the operand, output and status buffers and have no way to get
 * more device memory for the call: a plain C or FFI caller that does not own the process's
 * device allocator (in Fusion-PCU every device allocation belongs to the Rust memory-resource
 * pool), or a caller that must keep the call itself free of allocation.  This variant takes no
 * workspace.  Its scratch is a fixed array of device memory inside this library (about 257 KB,
 * held on every GPU that loads the library until the process exits).  A call that uses it (a
 * non-empty product under IeeeAfterRounding or RejectSubnormalResult) is limited to
 * rows + columns <= 65536; larger ones return PCU_B200_ERROR_WORKSPACE.  Calls that need no
 * scratch (empty shapes, inner == 0, AllowGradualUnderflow) have no limit.  It calls no
 * cudaMalloc or cudaFree.  The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) and later calls reuse it while the device's context stays the same (a
 * new context after a device reset gets a new lookup); make that first call before any stream
 * capture.  All calls share the one array: each call re-initialises what it reads, but calls
 * whose executions overlap on the GPU (other streams, other host threads) race on it and must be
 * serialised by the caller.  Everything else -- arguments, results, status word, errors -- is
 * exactly pcu_b200_strict_matmul. */
int pcu_b200_strict_matmul_static_scratch(int dtype, int policy, const void *left, const void *right, void *out,
                                          uint64_t rows, uint64_t inner, uint64_t columns, uint64_t left_stride,
                                          uint64_t right_stride, int transpose_left, int transpose_right,
                                          uint64_t *status, void *stream);

/* Strict MatMul with its operands and result in HOST memory: the host-boundary form of the node
 * (the reference's pending upload, tensor/pending_upload/pending_upload.rs:115-190, the node's
 * kernel and the read of its output).  Row-major, untransposed operands with dense rows:
 * left is rows x inner, right is inner x columns, out is rows x columns.  The rows of out are
 * computed in blocks so that the uploads of A and the read-backs of C overlap the arithmetic
 * (two copy streams of this library, ordered after the work already on `stream`, and joined
 * back into it); with page-locked host memory they run concurrently, with pageable memory they
 * serialise.  Results and the status word are exactly those of pcu_b200_strict_matmul on the
 * same operands; the status word goes to *status_host (host memory).  All writes to host memory
 * are asynchronous: synchronise `stream` before reading out or *status_host.  The device scratch
 * holds B, two row blocks of A and C, and the workspace:
 * pcu_b200_strict_matmul_host_scratch_size bytes. */
size_t pcu_b200_strict_matmul_host_scratch_size(int dtype, uint64_t rows, uint64_t inner, uint64_t columns);
int pcu_b200_strict_matmul_host(int dtype, int policy, const void *left, const void *right, void *out, uint64_t rows,
                                uint64_t inner, uint64_t columns, void *device_scratch, size_t scratch_bytes,
                                uint64_t *status_host, void *stream);

/* The host-boundary form with B already on the device: left (rows x inner, dense rows) and out
 * (rows x columns) in host memory, right on the device (inner x columns, row stride right_stride
 * elements).  The rows of A go up and the rows of C come back by row blocks, overlapped with the
 * arithmetic as in pcu_b200_strict_matmul_host; results and status word are exactly those of
 * pcu_b200_strict_matmul.  The row-sharded end-to-end step uses it: each rank uploads its rows of
 * A and a slice of B's rows, the slices are all-gathered over NVLink into a device B, and this
 * call computes the rank's rows.  Device scratch: pcu_b200_strict_matmul_host_left_scratch_size
 * bytes (two row blocks of A and C, the workspace and the status words).  No counterpart in the
 * reference. */
size_t pcu_b200_strict_matmul_host_left_scratch_size(int dtype, uint64_t rows, uint64_t inner, uint64_t columns);
int pcu_b200_strict_matmul_host_left(int dtype, int policy, const void *left, const void *right, uint64_t right_stride,
                                     void *out, uint64_t rows, uint64_t inner, uint64_t columns, void *device_scratch,
                                     size_t scratch_bytes, uint64_t *status_host, void *stream);

/* Row-sharded strict MatMul with the all-gather of C in the same kernel.  This rank computes rows
 * [row0, row0 + rows) of the rows_total x columns product C = A . op(B) (left_rows: this rank's
 * rows of A, rows x inner with row stride left_stride; right: B as in pcu_b200_strict_matmul,
 * transpose_right allowed) with the full ordered K loop.  Each finished output tile is written
 * into out_full (this rank's buffer: its whole C, rows_total x columns, dense) and into every
 * peer's buffer at the same place: peer_outs holds npeers (<= 7) device pointers of the peers'
 * buffers, in rank order without this rank, mapped into this process with pcu_b200_peer_open.
 * So the transfer overlaps the arithmetic tile by tile, with plain NVLink stores (no TMA or bulk
 * copy touches peer memory).  The status word holds the whole product's event ordinals (cells
 * offset by row0 * columns); the global first fault is the MIN of all ranks' words.
 *
 * Buffers: every rank's buffer is pcu_b200_peer_rows_bytes(dtype, rows_total, columns) bytes
 * from pcu_b200_peer_alloc (zero-filled): C, then a flag block with one word per rank.
 *
 * Ordering, both directions:
 *   - read side: a peer's rows are complete in this rank's C once every rank's call has
 *     finished (a kernel's peer stores are visible to whatever is ordered after its completion),
 *     which the caller establishes with a collective after the call (the status MIN);
 *   - write side: `epoch` numbers the calls on this set of buffers (1, 2, 3, ..., the same on
 *     every rank) and `rank` is this rank's index (0..npeers).  The kernel records its entry in
 *     each peer's flag block and stores into a peer's C only after that peer's kernel of the
 *     same call has started, i.e. after everything the peer queued before it on its stream --
 *     its readers of the previous call's C -- has finished.  Readers of C on another stream must
 *     be joined into the calling stream before the next call.  A peer that has not entered the
 *     call within 10 s gets no stores and the status word records PCU_B200_STATUS_WATCHDOG.
 *
 * No counterpart in the reference (its strict MatMul runs on one device). */
size_t pcu_b200_peer_rows_bytes(int dtype, uint64_t rows_total, uint64_t columns);
int pcu_b200_strict_matmul_rows_allgather(int dtype, int policy, const void *left_rows, const void *right,
                                          void *out_full, uint64_t row0, uint64_t rows, uint64_t rows_total,
                                          uint64_t inner, uint64_t columns, uint64_t left_stride,
                                          uint64_t right_stride, int transpose_right, void *const *peer_outs,
                                          int npeers, int rank, uint64_t epoch, void *workspace,
                                          size_t workspace_bytes, uint64_t *status, void *stream);

/* CUDA IPC for the buffers peers write into: allocate `bytes` of zero-filled device memory and
 * its 64-byte IPC handle; map a peer's buffer from its handle (into this process, on the current device);
 * unmap; free. */
int pcu_b200_peer_alloc(size_t bytes, void **ptr, void *handle);
int pcu_b200_peer_open(const void *handle, void **ptr);
int pcu_b200_peer_close(void *ptr);
int pcu_b200_peer_free(void *ptr);

/* Measured roofline denominator of the strict MatMul (no counterpart in the reference): the
 * FP32 or FP64 non-FMA issue rate of this GPU.  pcu_b200_issue_probe launches `iterations`
 * rounds of independent, separately rounded multiplies and adds on every SM at full occupancy;
 * time it with CUDA events on `stream`.  pcu_b200_issue_probe_ops is the number of multiplies
 * plus adds that launch executes on the current device. */
uint64_t pcu_b200_issue_probe_ops(int dtype, uint64_t iterations);
int pcu_b200_issue_probe(int dtype, uint64_t iterations, void *stream);

/* ------------------------------------------------------------------ strict SGD */

/* out[i] = weights[i] - rate * gradient[i] with the multiply and the subtract separately
 * rounded and checked (reference/strict_sgd/strict_sgd.rs:20-46).  The rate is a finite
 * binary32 pattern; for F64 it is widened exactly (reference.rs:507-517).  out may alias
 * weights (in-place update). */
int pcu_b200_strict_sgd(int dtype, int policy, const void *weights, const void *gradient, void *out,
                        uint64_t count, uint32_t rate_bits_f32, uint64_t *status, void *stream);

/* ------------------------------------------------------------------ strict MSE */

/* Device workspace bytes pcu_b200_strict_mse needs for `count` elements. */
size_t pcu_b200_strict_mse_workspace_size(int dtype, uint64_t count);

/* out[0] = (sum over i ascending of (prediction[i] - target[i])^2) / count, every subtract,
 * square, accumulate and the final divide separately rounded and checked, the running sum
 * starting at +0 (reference/strict_mse/strict_mse.rs:22-59; the divisor is count rounded to
 * nearest-even, constants/constants.rs:18-27).  count must be >= 1. */
int pcu_b200_strict_mse(int dtype, int policy, const void *prediction, const void *target, void *out,
                        uint64_t count, void *workspace, size_t workspace_bytes, uint64_t *status,
                        void *stream);

/* Segment form of pcu_b200_strict_mse for a reduction split across devices (one tensor's
 * elements sharded over GPUs) with an ordered hand-off of the running sum.  It has no
 * counterpart in the reference, whose strict MSE runs on one device; the results are those of
 * the one-device reduction over the concatenated segments.
 *
 * The segment holds the global elements [first_index, first_index + count) of a reduction
 * over total_count elements; its fault events are global (element i -> i*3 + step, Divide
 * -> total_count*3).  Call prepare (all of the segment's bandwidth-bound work; it does not
 * depend on the running sum, so every device runs it at once), then walk with the running
 * sum that enters the segment (carry_in, a device scalar, NULL = +0).  Walk writes the running
 * sum after the segment to *carry_out (if not NULL; it may equal carry_in) and, for the last
 * segment (first_index + count == total_count) with out not NULL, the checked mean to out[0].
 * A fault already recorded in `status` in front of the segment stops the walk at once.  Both
 * take the workspace of pcu_b200_strict_mse_workspace_size(dtype, count); count may be 0. */
int pcu_b200_strict_mse_segment_prepare(int dtype, int policy, const void *prediction, const void *target,
                                        uint64_t count, uint64_t first_index, void *workspace,
                                        size_t workspace_bytes, uint64_t *status, void *stream);
int pcu_b200_strict_mse_segment_walk(int dtype, int policy, const void *prediction, const void *target,
                                     uint64_t count, uint64_t first_index, uint64_t total_count,
                                     const void *carry_in, void *carry_out, void *out, void *workspace,
                                     size_t workspace_bytes, uint64_t *status, void *stream);

/* ------------------------------------------------------------------ MSE and SGD in one pass */

/* One strict MSE node and one strict SGD node that do not depend on each other, as the loss and
 * a weight update of a training step are (the MSE gradient reads prediction and target, never
 * the loss), run in one pass.  The MSE's chunk pass is bound by integer work and its final walk
 * by latency, so the SGD's HBM traffic is streamed inside those launches instead of after them.
 * There is no single counterpart in the reference; the call replaces its two executor calls
 * (execute_strict_mse and execute_strict_sgd, tensor/tensor.rs:5144-5166 and 5077-5103).
 * Results, events and status words are exactly those of pcu_b200_strict_mse (prediction,
 * target, loss, mse_count, mse_status) and pcu_b200_strict_sgd (weights, gradient, updated,
 * sgd_count, rate, sgd_status) run one after the other; each node keeps its own status word.
 * The workspace is pcu_b200_strict_mse_workspace_size(dtype, mse_count).  updated may alias
 * weights; no other buffer may overlap updated.  sgd_count may be 0. */
int pcu_b200_strict_mse_sgd(int dtype, int policy, const void *prediction, const void *target, void *loss,
                            uint64_t mse_count, void *workspace, size_t workspace_bytes, uint64_t *mse_status,
                            const void *weights, const void *gradient, void *updated, uint64_t sgd_count,
                            uint32_t rate_bits_f32, uint64_t *sgd_status, void *stream);

/* pcu_b200_strict_mse_segment_prepare with an SGD share carried by the same launch: the SGD
 * elements [0, sgd_count) given are the global elements [sgd_first_index, sgd_first_index +
 * sgd_count) of their node (events (sgd_first_index + i) * 2 + step).  No counterpart in the
 * reference (see pcu_b200_strict_mse_segment_prepare). */
int pcu_b200_strict_mse_sgd_segment_prepare(int dtype, int policy, const void *prediction, const void *target,
                                            uint64_t mse_count, uint64_t mse_first_index, void *workspace,
                                            size_t workspace_bytes, uint64_t *mse_status, const void *weights,
                                            const void *gradient, void *updated, uint64_t sgd_count,
                                            uint64_t sgd_first_index, uint32_t rate_bits_f32,
                                            uint64_t *sgd_status, void *stream);

/* A whole segment in one call: pcu_b200_strict_mse_sgd_segment_prepare followed by
 * pcu_b200_strict_mse_segment_walk (same arguments and results), in one launch for binary32, so
 * the walk runs beside the segment's bandwidth-bound work.  Useful for the first segment of a
 * split reduction, whose running sum starts at carry_in = NULL (+0): it needs no hand-off before
 * it can walk.  sgd_count may be 0 (weights, gradient, updated then unused; sgd_status still
 * required).  No counterpart in the reference. */
int pcu_b200_strict_mse_sgd_segment(int dtype, int policy, const void *prediction, const void *target,
                                    uint64_t mse_count, uint64_t mse_first_index, uint64_t total_count,
                                    const void *carry_in, void *carry_out, void *out, void *workspace,
                                    size_t workspace_bytes, uint64_t *mse_status, const void *weights,
                                    const void *gradient, void *updated, uint64_t sgd_count, uint64_t sgd_first_index,
                                    uint32_t rate_bits_f32, uint64_t *sgd_status, void *stream);

/* The split strict MSE (with an optional independent strict SGD node riding along) with every
 * exchange on the device: one process per GPU of one node, nranks <= 8, rank r holding the
 * global elements [mse_first_index, mse_first_index + mse_count) of a total_count-element
 * reduction, the segments in rank order (rank nranks - 1 holds the last one).
 *   - blocks: nranks device pointers in rank order, each rank's hand-off block
 *     (pcu_b200_mse_handoff_bytes bytes from pcu_b200_peer_alloc, mapped here with
 *     pcu_b200_peer_open; blocks[rank] is this rank's own);
 *   - epoch numbers the calls on this set of blocks (1, 2, 3, ..., the same on every rank).
 * The segment's maps and walk run as one launch (binary32; three for binary64).  The walker of
 * rank r > 0 waits until rank r - 1 has stored its running sum into this rank's block, and
 * rank r < nranks - 1 stores its own into rank r + 1's (plain NVLink stores and a release flag:
 * no NCCL, no host round trip).  Then a one-warp exchange stores this rank's words into every
 * peer's block and waits for theirs.  When the work on `stream` is done, on every rank:
 * *mse_status and *sgd_status hold the MIN over ranks (the global first faults; words carry
 * global events), *mean_out holds the mean (binary32/64 as dtype).  A device wait that gives up
 * (10 s) leaves PCU_B200_STATUS_WATCHDOG in *mse_status.  The SGD node ([sgd_first_index,
 * sgd_first_index + sgd_count) of its own tensor) is as in pcu_b200_strict_mse_sgd_segment.
 * No counterpart in the reference (its strict MSE runs on one lane of one device). */
size_t pcu_b200_mse_handoff_bytes(void);
int pcu_b200_strict_mse_sgd_split(int dtype, int policy, const void *prediction, const void *target,
                                  uint64_t mse_count, uint64_t mse_first_index, uint64_t total_count, void *mean_out,
                                  void *workspace, size_t workspace_bytes, uint64_t *mse_status, const void *weights,
                                  const void *gradient, void *updated, uint64_t sgd_count, uint64_t sgd_first_index,
                                  uint32_t rate_bits_f32, uint64_t *sgd_status, void *const *blocks, int rank,
                                  int nranks, uint64_t epoch, void *stream);

/* ------------------------------------------------------------------ checked elementwise */

/* out[i] = op(left[i], right[i]); a nonzero *_uniform flag broadcasts element 0 of that
 * operand (the reference's UniformScalar representation).  out may alias a non-uniform input. */
int pcu_b200_checked_binary(int dtype, int policy, int op, const void *left, const void *right, void *out,
                            uint64_t count, int left_uniform, int right_uniform, uint64_t *status,
                            void *stream);

/* out[i] = checked ReLU(input[i]): non-finite -> Invalid, negative or signed zero -> +0,
 * RejectSubnormalResult rejects a subnormal result (scalar_checked_float.rs:273-309). */
int pcu_b200_checked_relu(int dtype, int policy, const void *input, void *out, uint64_t count,
                          uint64_t *status, void *stream);

/* out[i] = input[i] > 0 ? upstream[i] : +0, both operands required finite
 * (scalar_checked_float.rs:634-652). */
int pcu_b200_checked_relu_backward(int dtype, int policy, const void *input, const void *upstream, void *out,
                                   uint64_t count, uint64_t *status, void *stream);

/* ------------------------------------------------------------------ guarded chains
 *
 * An ordered, stop-on-fault chain of node calls on one stream, without a host wait between them.
 * This replaces the guarded kernel ABI of the reference's owned dispatch, where the status
 * argument `u64* fault_word` becomes `(u64* chain_records, u32 chain_stage)`
 * (Crates/backends/cuda/owned_dispatch/guarded/guarded.rs, guarded_source).  It also replaces the
 * record slab that Crates/backends/cuda/tensor/guarded/guarded.rs:355-400 initialises, submits and
 * reads back.
 *
 * Records: one slab of 2 x stages u64 words.  Record s is [fault word, disposition].
 *   * The fault word is stage s's status word (sentinel PCU_B200_STATUS_OK).
 *   * The disposition is PENDING until stage s's first kernel decides it.  Stage s is admitted
 *     (EXECUTED) when s == 0, or when record s-1 is EXECUTED with a clear fault word.  Otherwise
 *     it is SKIPPED, and none of its kernels writes anything.
 *
 * pcu_b200_guarded_* take the arguments of the unguarded call of the same name, with `status`
 * replaced by (chain_records, chain_stage).  Stage numbers are the order of submission on the
 * stream, from 0.  The chain's calls must all be on one stream (or ordered by events).
 * The host reads the slab back once, after the last stage, and checks it with
 * pcu_b200_chain_validate. */
#define PCU_B200_CHAIN_PENDING 0
#define PCU_B200_CHAIN_EXECUTED 1
#define PCU_B200_CHAIN_SKIPPED 2

/* Every record to [PCU_B200_STATUS_OK, PENDING], ordered on `stream`. */
int pcu_b200_chain_reset(uint64_t *chain_records, uint32_t stages, void *stream);

int pcu_b200_guarded_strict_matmul(int dtype, int policy, const void *left, const void *right, void *out,
                                   uint64_t rows, uint64_t inner, uint64_t columns, uint64_t left_stride,
                                   uint64_t right_stride, int transpose_left, int transpose_right, void *workspace,
                                   size_t workspace_bytes, uint64_t *chain_records, uint32_t chain_stage,
                                   void *stream);
int pcu_b200_guarded_strict_sgd(int dtype, int policy, const void *weights, const void *gradient, void *out,
                                uint64_t count, uint32_t rate_bits_f32, uint64_t *chain_records, uint32_t chain_stage,
                                void *stream);
int pcu_b200_guarded_strict_mse(int dtype, int policy, const void *prediction, const void *target, void *out,
                                uint64_t count, void *workspace, size_t workspace_bytes, uint64_t *chain_records,
                                uint32_t chain_stage, void *stream);
int pcu_b200_guarded_checked_binary(int dtype, int policy, int op, const void *left, const void *right, void *out,
                                    uint64_t count, int left_uniform, int right_uniform, uint64_t *chain_records,
                                    uint32_t chain_stage, void *stream);
int pcu_b200_guarded_checked_relu(int dtype, int policy, const void *input, void *out, uint64_t count,
                                  uint64_t *chain_records, uint32_t chain_stage, void *stream);
int pcu_b200_guarded_checked_relu_backward(int dtype, int policy, const void *input, const void *upstream,
                                           void *out, uint64_t count, uint64_t *chain_records, uint32_t chain_stage,
                                           void *stream);

/* Outcomes of pcu_b200_chain_validate (Crates/core/runtime/execution/guarded/guarded.rs:84-140). */
#define PCU_B200_CHAIN_SUCCEEDED 0           /* every stage executed without a fault */
#define PCU_B200_CHAIN_FAULT 1               /* *stage: the first faulting stage; every later one skipped */
#define PCU_B200_CHAIN_STAGE_DECODE 2        /* *stage: a pending or unknown disposition, a fault word on a
                                                skipped stage, or a fault word no node call writes */
#define PCU_B200_CHAIN_UNEXPECTED_SKIP 3     /* *stage: skipped although no earlier stage faulted */
#define PCU_B200_CHAIN_EXECUTED_AFTER_FAULT 4 /* *stage: executed after an earlier fault */

/* Checks a record slab that was read back to HOST memory after the chain completed.  Host
 * code only; it makes no CUDA call.  Stages are decoded in order, and the first decode error
 * or order violation is reported, so an earlier fault cannot hide a later bad record.  Only
 * PCU_B200_CHAIN_SUCCEEDED and PCU_B200_CHAIN_FAULT mean that the outputs may be published.
 *
 * A fault word decodes when its kind is one that node calls write: DIVIDE_BY_ZERO, OVERFLOW,
 * UNDERFLOW or INVALID.  SIGNED_DIVISION_OVERFLOW and a watchdog word are decode errors.
 * `event_extents` is optional.  When it is given, stage s's event must also be below
 * event_extents[s]: rows*columns*inner*2 for MatMul, 2n for SGD, 3n+1 for MSE, n for the
 * elementwise calls.
 * The return value is PCU_B200_OK or PCU_B200_ERROR_INVALID_ARGUMENT; the outcome goes to
 * *outcome, and *stage is the stage it names (0 for SUCCEEDED). */
int pcu_b200_chain_validate(const uint64_t *chain_records, uint32_t stages, const uint64_t *event_extents,
                            int *outcome, uint32_t *stage);

/* ------------------------------------------------------------------ waiting */

/* Waits until all work submitted to `stream` has completed, for at most timeout_ms
 * milliseconds.  The other calls of this library never block the host; this one does,
 * by polling.  Returns PCU_B200_OK when the work has completed, PCU_B200_ERROR_TIMEOUT when
 * it has not, and PCU_B200_ERROR_CUDA for an error that the stream reports. */
int pcu_b200_wait(void *stream, uint32_t timeout_ms);

/* ------------------------------------------------------------------ multi-GPU exchange steps
 *
 * A communicator over the ranks of one job, one process per GPU (at most 8, one node), for a
 * host that has none of its own.  It carries the exchange steps of the split paths:
 *   * the global first fault, an unsigned MIN of the ranks' status words;
 *   * the running-sum hand-off of a split MSE;
 *   * the exchange of peer-buffer handles for the row-sharded MatMul.
 * The all-gather of that MatMul's C happens inside the MatMul kernel.  None of this has a
 * counterpart in the reference, whose strict path runs on one device.
 *
 * NCCL is loaded at run time (dlopen of libnccl.so.2) by the first call here.  The library has
 * no load-time dependency on it, and a process that already loaded NCCL reuses that copy.
 *   * PCU_B200_ERROR_UNSUPPORTED: NCCL could not be loaded.
 *   * PCU_B200_ERROR_COMM: NCCL returned an error; pcu_b200_last_comm_error gives its code.
 *
 * Every rank makes the same collective calls in the same order.  The calls enqueue work on
 * `stream` and return without waiting, except pcu_b200_comm_init (which waits for every rank to
 * join) and the two peer-buffer calls.  A call that fails on one rank returns before its
 * collective and leaves the other ranks waiting in theirs.  The host then bounds its wait with
 * pcu_b200_wait and aborts the communicator on every rank with pcu_b200_comm_abort. */
#define PCU_B200_ERROR_COMM 7
#define PCU_B200_COMM_ID_BYTES 128
typedef struct pcu_b200_comm pcu_b200_comm;

int pcu_b200_last_comm_error(void);

/* Rank 0 makes the id (PCU_B200_COMM_ID_BYTES bytes); the host hands it to every rank, which
 * then calls init on its own GPU (the current device) with the job's rank count and its rank. */
int pcu_b200_comm_unique_id(void *id);
int pcu_b200_comm_init(const void *id, int nranks, int rank, pcu_b200_comm **comm);
int pcu_b200_comm_free(pcu_b200_comm *comm);
int pcu_b200_comm_abort(pcu_b200_comm *comm);

/* status[0..count) becomes the unsigned MIN over ranks, on every rank (all-reduce).  The status
 * words must carry global events, as every split call here writes them. */
int pcu_b200_comm_status_min(pcu_b200_comm *comm, uint64_t *status, uint64_t count, void *stream);

/* Device bytes to or from one peer (a matching send and recv), and a broadcast from `root`. */
int pcu_b200_comm_send(pcu_b200_comm *comm, const void *buffer, size_t bytes, int peer, void *stream);
int pcu_b200_comm_recv(pcu_b200_comm *comm, void *buffer, size_t bytes, int peer, void *stream);
int pcu_b200_comm_broadcast(pcu_b200_comm *comm, void *buffer, size_t bytes, int root, void *stream);

/* Collective.  Every rank allocates `bytes` of zero-filled device memory that the others map
 * with CUDA IPC (for a row-sharded MatMul: pcu_b200_peer_rows_bytes(dtype, rows_total, columns)).
 * buffers[r] (nranks entries) is rank r's buffer as this process sees it; buffers[rank] is this
 * rank's own.  Returns once this rank has mapped every peer.  Collective when it fails too: if
 * any rank cannot allocate its buffer or map a peer's, every rank releases what it holds, leaves
 * buffers[] null and returns the same error.  _free unmaps the peers, waits for every rank to do
 * the same, and frees this rank's buffer. */
int pcu_b200_comm_peer_buffers(pcu_b200_comm *comm, size_t bytes, void **buffers, void *stream);
int pcu_b200_comm_peer_buffers_free(pcu_b200_comm *comm, void **buffers, void *stream);

/* The row-sharded strict MatMul in one call.  It runs pcu_b200_strict_matmul_rows_allgather for
 * rows [row0, row0 + rows) into buffers[rank] and every peer's buffer (buffers from
 * pcu_b200_comm_peer_buffers, pcu_b200_peer_rows_bytes each), then the status MIN.  When the
 * work on `stream` is done, every rank's buffers[rank] holds all of C and `status` holds the
 * global first fault.  The communicator numbers the calls on each buffer set, so the next
 * call's stores into a rank's C wait until that rank's stream has reached the call: readers of C
 * queued on `stream` before the next call are never overwritten. */
int pcu_b200_comm_strict_matmul_rows(pcu_b200_comm *comm, int dtype, int policy, const void *left_rows,
                                     const void *right, void *const *buffers, uint64_t row0, uint64_t rows,
                                     uint64_t rows_total, uint64_t inner, uint64_t columns, uint64_t left_stride,
                                     uint64_t right_stride, int transpose_right, void *workspace,
                                     size_t workspace_bytes, uint64_t *status, void *stream);

/* The split strict MSE in one call: rank r holds the global elements [first_index, first_index +
 * count) of a total_count-element reduction, the segments in rank order.  It runs
 * pcu_b200_strict_mse_sgd_split: the running sum goes from rank to rank on the device through
 * IPC-mapped hand-off blocks that the first call makes (collectively, like every call here, and
 * kept until the communicator is freed), and a one-warp exchange leaves the mean in *out and the
 * global first fault in *status on every rank.  No NCCL call after the first.  A segment may be
 * empty (count 0: the rank passes the running sum on); the last rank's ends at total_count; the
 * result equals pcu_b200_strict_mse over the whole tensor.  The workspace is
 * pcu_b200_strict_mse_workspace_size(dtype, count) (at least one byte). */
int pcu_b200_comm_strict_mse(pcu_b200_comm *comm, int dtype, int policy, const void *prediction, const void *target,
                             uint64_t count, uint64_t first_index, uint64_t total_count, void *out, void *workspace,
                             size_t workspace_bytes, uint64_t *status, void *stream);

#ifdef __cplusplus
}
#endif
#endif
