// abi.cu -- library-level entry points and host helpers of the B200 strict-tensor provider.
#include <algorithm>
#include <chrono>
#include <cstring>
#include <mutex>
#include <thread>

#include "common.cuh"
#include "pcu_b200.h"
#include "provider.h"

namespace {

thread_local int g_last_cuda_error = 0;

__global__ void fill_status_kernel(unsigned long long *status, uint64_t count) {
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (; i < count; i += stride) status[i] = pcu::kStatusOk;
}

__global__ void chain_decide_kernel(pcu::ChainGuard guard) { (void)pcu::chain_admits(guard); }

// record s of a chain slab = [fault word, disposition]
__global__ void chain_reset_kernel(unsigned long long *records, uint32_t stages) {
    for (uint64_t s = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; s < stages; s += (uint64_t)gridDim.x * blockDim.x) {
        records[2 * s] = pcu::kStatusOk;
        records[2 * s + 1] = pcu::kDispPending;
    }
}

// The guard of stage `stage` of a record slab: admitted by record stage-1, deciding record
// stage's disposition in its first kernel.
pcu::ChainGuard slab_guard(uint64_t *records, uint32_t stage) {
    auto *r = reinterpret_cast<unsigned long long *>(records);
    pcu::ChainGuard g{};
    g.disp = r + 2ull * stage + 1;
    g.decide = 1;
    if (stage > 0) {
        g.prev_status = r + 2ull * (stage - 1);
        g.prev_disp = r + 2ull * (stage - 1) + 1;
    }
    return g;
}

}  // namespace

namespace pcu {

int chain_decide_only(const ChainGuard &guard, cudaStream_t stream) {
    if (!guard.disp || !guard.decide) return PCU_B200_OK;
    chain_decide_kernel<<<1, 1, 0, stream>>>(guard);
    return pcu_host::launch_status();
}

}  // namespace pcu

namespace pcu_host {

int set_cuda_error(cudaError_t err) {
    g_last_cuda_error = (int)err;
    return PCU_B200_ERROR_CUDA;
}

int launch_status(void) {
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return set_cuda_error(err);
    return PCU_B200_OK;
}

int sm_count(void) {
    static std::mutex lock;
    static int cached[64] = {0};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return 148;
    std::lock_guard<std::mutex> guard(lock);
    if (!cached[device]) {
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || sms <= 0)
            sms = 148;
        cached[device] = sms;
    }
    return cached[device];
}

}  // namespace pcu_host

extern "C" int pcu_b200_abi_version(void) { return PCU_B200_ABI_VERSION; }

extern "C" const char *pcu_b200_error_string(int code) {
    switch (code) {
    case PCU_B200_OK: return "ok";
    case PCU_B200_ERROR_INVALID_ARGUMENT: return "invalid argument";
    case PCU_B200_ERROR_SIZE_OVERFLOW: return "shape or fault-event domain exceeds the supported range";
    case PCU_B200_ERROR_WORKSPACE: return "workspace missing or too small";
    case PCU_B200_ERROR_CUDA: return "CUDA launch or configuration failure (see pcu_b200_last_cuda_error)";
    case PCU_B200_ERROR_UNSUPPORTED: return "unsupported on this device";
    case PCU_B200_ERROR_TIMEOUT: return "the stream's work did not complete within the timeout";
    case PCU_B200_ERROR_COMM: return "communicator failure (NCCL; see pcu_b200_last_comm_error)";
    default: return "unknown error";
    }
}

extern "C" int pcu_b200_last_cuda_error(void) { return g_last_cuda_error; }

extern "C" int pcu_b200_status_reset(uint64_t *status, uint64_t count, void *stream) {
    if (count == 0) return PCU_B200_OK;
    if (!status) return PCU_B200_ERROR_INVALID_ARGUMENT;
    unsigned blocks = (unsigned)((count + 255) / 256 < 1024 ? (count + 255) / 256 : 1024);
    fill_status_kernel<<<blocks, 256, 0, pcu_host::as_stream(stream)>>>(
        reinterpret_cast<unsigned long long *>(status), count);
    return pcu_host::launch_status();
}

// ---------------------------------------------------------------------------- guarded chains

extern "C" int pcu_b200_chain_reset(uint64_t *chain_records, uint32_t stages, void *stream) {
    if (stages == 0) return PCU_B200_OK;
    if (!chain_records) return PCU_B200_ERROR_INVALID_ARGUMENT;
    const unsigned blocks = (unsigned)((stages + 255) / 256 < 1024 ? (stages + 255) / 256 : 1024);
    chain_reset_kernel<<<blocks, 256, 0, pcu_host::as_stream(stream)>>>(
        reinterpret_cast<unsigned long long *>(chain_records), stages);
    return pcu_host::launch_status();
}

extern "C" int pcu_b200_guarded_strict_matmul(int dtype, int policy, const void *left, const void *right, void *out,
                                              uint64_t rows, uint64_t inner, uint64_t columns, uint64_t left_stride,
                                              uint64_t right_stride, int transpose_left, int transpose_right,
                                              void *workspace, size_t workspace_bytes, uint64_t *chain_records,
                                              uint32_t chain_stage, void *stream) {
    if (!chain_records) return PCU_B200_ERROR_INVALID_ARGUMENT;
    return pcu::strict_matmul(dtype, policy, left, right, out, rows, inner, columns, left_stride, right_stride,
                              transpose_left, transpose_right, workspace, workspace_bytes,
                              chain_records + 2ull * chain_stage, stream, slab_guard(chain_records, chain_stage));
}

extern "C" int pcu_b200_guarded_strict_sgd(int dtype, int policy, const void *weights, const void *gradient, void *out,
                                           uint64_t count, uint32_t rate_bits_f32, uint64_t *chain_records,
                                           uint32_t chain_stage, void *stream) {
    if (!chain_records) return PCU_B200_ERROR_INVALID_ARGUMENT;
    return pcu::strict_sgd(dtype, policy, weights, gradient, out, count, rate_bits_f32,
                           chain_records + 2ull * chain_stage, stream, slab_guard(chain_records, chain_stage));
}

extern "C" int pcu_b200_guarded_strict_mse(int dtype, int policy, const void *prediction, const void *target,
                                           void *out, uint64_t count, void *workspace, size_t workspace_bytes,
                                           uint64_t *chain_records, uint32_t chain_stage, void *stream) {
    if (!chain_records) return PCU_B200_ERROR_INVALID_ARGUMENT;
    return pcu::strict_mse(dtype, policy, prediction, target, out, count, workspace, workspace_bytes,
                           chain_records + 2ull * chain_stage, stream, slab_guard(chain_records, chain_stage));
}

extern "C" int pcu_b200_guarded_checked_binary(int dtype, int policy, int op, const void *left, const void *right,
                                               void *out, uint64_t count, int left_uniform, int right_uniform,
                                               uint64_t *chain_records, uint32_t chain_stage, void *stream) {
    if (!chain_records) return PCU_B200_ERROR_INVALID_ARGUMENT;
    return pcu::checked_binary(dtype, policy, op, left, right, out, count, left_uniform, right_uniform,
                               chain_records + 2ull * chain_stage, stream, slab_guard(chain_records, chain_stage));
}

extern "C" int pcu_b200_guarded_checked_relu(int dtype, int policy, const void *input, void *out, uint64_t count,
                                             uint64_t *chain_records, uint32_t chain_stage, void *stream) {
    if (!chain_records) return PCU_B200_ERROR_INVALID_ARGUMENT;
    return pcu::checked_relu(dtype, policy, input, out, count, chain_records + 2ull * chain_stage, stream,
                             slab_guard(chain_records, chain_stage));
}

extern "C" int pcu_b200_guarded_checked_relu_backward(int dtype, int policy, const void *input, const void *upstream,
                                                      void *out, uint64_t count, uint64_t *chain_records,
                                                      uint32_t chain_stage, void *stream) {
    if (!chain_records) return PCU_B200_ERROR_INVALID_ARGUMENT;
    return pcu::checked_relu_backward(dtype, policy, input, upstream, out, count, chain_records + 2ull * chain_stage,
                                      stream, slab_guard(chain_records, chain_stage));
}

namespace {

// One record (Crates/backends/cuda/owned_dispatch/guarded/guarded.rs, decode_record): 0 succeeded,
// 1 fault, 2 skipped, -1 malformed.  A fault needs an executed stage, a kind that node calls write
// and (when an extent is given) an event inside the stage's fault domain; a skipped stage needs a
// clear word; a pending or unknown disposition never decodes.
int decode_record(uint64_t word, uint64_t disposition, const uint64_t *extent) {
    if (disposition == PCU_B200_CHAIN_SKIPPED) return word == PCU_B200_STATUS_OK ? 2 : -1;
    if (disposition != PCU_B200_CHAIN_EXECUTED) return -1;
    if (word == PCU_B200_STATUS_OK) return 0;
    const uint64_t kind = word & 7u, event = word >> 3;
    const bool known = kind == PCU_B200_KIND_DIVIDE_BY_ZERO || kind == PCU_B200_KIND_OVERFLOW ||
                       kind == PCU_B200_KIND_UNDERFLOW || kind == PCU_B200_KIND_INVALID;
    if (!known || (extent && event >= *extent)) return -1;
    return 1;
}

}  // namespace

// Crates/core/runtime/execution/guarded/guarded.rs:107-140 (validate_guarded_execution): every
// stage before the first fault succeeded, every stage after it was skipped.
extern "C" int pcu_b200_chain_validate(const uint64_t *chain_records, uint32_t stages, const uint64_t *event_extents,
                                       int *outcome, uint32_t *stage) {
    if (!outcome || !stage || (stages > 0 && !chain_records)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    int64_t first = -1;
    for (uint32_t s = 0; s < stages; ++s) {
        const int r = decode_record(chain_records[2ull * s], chain_records[2ull * s + 1],
                                    event_extents ? event_extents + s : nullptr);
        int bad = -1;
        if (r < 0) bad = PCU_B200_CHAIN_STAGE_DECODE;
        else if (first < 0 && r == 2) bad = PCU_B200_CHAIN_UNEXPECTED_SKIP;
        else if (first >= 0 && r != 2) bad = PCU_B200_CHAIN_EXECUTED_AFTER_FAULT;
        if (bad >= 0) {
            *outcome = bad;
            *stage = s;
            return PCU_B200_OK;
        }
        if (first < 0 && r == 1) first = s;
    }
    *outcome = first < 0 ? PCU_B200_CHAIN_SUCCEEDED : PCU_B200_CHAIN_FAULT;
    *stage = first < 0 ? 0u : (uint32_t)first;
    return PCU_B200_OK;
}

// ---------------------------------------------------------------------------- waiting

extern "C" int pcu_b200_wait(void *stream, uint32_t timeout_ms) {
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
    auto pause = std::chrono::microseconds(20);
    for (;;) {
        const cudaError_t err = cudaStreamQuery(pcu_host::as_stream(stream));
        if (err == cudaSuccess) return PCU_B200_OK;
        if (err != cudaErrorNotReady) return pcu_host::set_cuda_error(err);
        const auto now = std::chrono::steady_clock::now();
        if (now >= deadline) return PCU_B200_ERROR_TIMEOUT;
        std::this_thread::sleep_for(std::min<std::chrono::steady_clock::duration>(pause, deadline - now));
        if (pause < std::chrono::milliseconds(1)) pause *= 2;
    }
}
