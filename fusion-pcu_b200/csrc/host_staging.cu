// host_staging.cu -- strict MatMul with its operands and result in host memory: the host-boundary
// form of a node (upload, execute, read back), pipelined by row blocks of the result.
//
// The reference runs a host-fed node as three steps on one stream: the pending upload of the
// inputs (Crates/backends/cuda/tensor/pending_upload/pending_upload.rs:115-190: a private host
// copy, then cudaMemcpyAsync on the execution stream), the node's kernel, and the read of the
// output.  Here the rows of C are split into blocks.  B goes up once; then, while block i is
// computed on the caller's stream, block i + 1's rows of A go up on one copy stream and block
// i - 1's rows of C come back on another, so the PCIe transfers hide behind the ordered-K
// arithmetic.  Every block is computed by the same strict MatMul as the device call, with a
// status word of its own; a last kernel shifts each block's events to the ordinals of the whole
// product (row offset x columns x inner x 2) and keeps the lowest, which is the first fault of
// the one-call form.  Then that word is copied to the host.
#include <mutex>

#include "common.cuh"
#include "pcu_b200.h"
#include "provider.h"

namespace {

constexpr int kMaxBlocks = 8;
constexpr uint64_t kRowsPerBlockMin = 2048;  // smaller blocks lose compute to their last wave

__global__ void combine_block_status(const unsigned long long *words, int blocks, uint64_t block_rows,
                                     uint64_t columns, uint64_t inner, unsigned long long *out) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    unsigned long long best = pcu::kStatusOk;
    for (int i = 0; i < blocks; ++i) {
        const unsigned long long w = words[i];
        if (w == pcu::kStatusOk) continue;
        const unsigned long long kind = w & 7;
        // a wait that gave up (kind 7) is not an event of the product: kept as it is
        const unsigned long long shifted =
            kind == pcu::kWatchdog ? w
                                   : ((((w >> 3) + (unsigned long long)i * block_rows * columns * (inner ? inner : 1) * 2)
                                       << 3) |
                                      kind);
        best = shifted < best ? shifted : best;
    }
    *out = best;
}

struct Staging {  // per device: the two copy streams and a pool of events
    cudaStream_t up = nullptr, down = nullptr;
    cudaEvent_t ev[2 + 3 * kMaxBlocks] = {};
    bool ready = false;
};

std::mutex g_staging_lock;
Staging g_staging[64];

int staging_for_device(Staging **out) {
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return pcu_host::set_cuda_error(err);
    if (device < 0 || device >= 64) return PCU_B200_ERROR_UNSUPPORTED;
    Staging &st = g_staging[device];
    if (!st.ready) {
        err = cudaStreamCreateWithFlags(&st.up, cudaStreamNonBlocking);
        if (err == cudaSuccess) err = cudaStreamCreateWithFlags(&st.down, cudaStreamNonBlocking);
        for (int i = 0; i < 2 + 3 * kMaxBlocks && err == cudaSuccess; ++i)
            err = cudaEventCreateWithFlags(&st.ev[i], cudaEventDisableTiming);
        if (err != cudaSuccess) return pcu_host::set_cuda_error(err);
        st.ready = true;
    }
    *out = &st;
    return PCU_B200_OK;
}

struct HostLayout {
    int blocks;
    uint64_t block_rows;
    size_t b_off, a_off[2], c_off[2], ws_off, st_off, ws_bytes, bytes;
    HostLayout(size_t elem, uint64_t rows, uint64_t inner, uint64_t columns) {
        auto up = [](size_t v) { return (v + 255) / 256 * 256; };
        blocks = (int)(rows / kRowsPerBlockMin);
        blocks = blocks < 1 ? 1 : (blocks > 4 ? 4 : blocks);
        block_rows = (rows + blocks - 1) / blocks;
        size_t off = 0;
        b_off = off;
        off += up(inner * columns * elem);
        const int buffers = blocks > 1 ? 2 : 1;
        for (int i = 0; i < 2; ++i) {
            a_off[i] = off;
            if (i < buffers) off += up(block_rows * inner * elem);
        }
        for (int i = 0; i < 2; ++i) {
            c_off[i] = off;
            if (i < buffers) off += up(block_rows * columns * elem);
        }
        if (buffers == 1) {
            a_off[1] = a_off[0];
            c_off[1] = c_off[0];
        }
        ws_off = off;
        ws_bytes = pcu_b200_strict_matmul_workspace_size(block_rows, inner, columns);
        off += up(ws_bytes ? ws_bytes : 1);
        st_off = off;
        off += up((kMaxBlocks + 1) * sizeof(uint64_t));
        bytes = off;
    }
};

}  // namespace

extern "C" size_t pcu_b200_strict_matmul_host_scratch_size(int dtype, uint64_t rows, uint64_t inner,
                                                           uint64_t columns) {
    return HostLayout(dtype == PCU_B200_F64 ? 8 : 4, rows, inner, columns).bytes;
}

extern "C" int pcu_b200_strict_matmul_host(int dtype, int policy, const void *left, const void *right, void *out,
                                           uint64_t rows, uint64_t inner, uint64_t columns, void *device_scratch,
                                           size_t scratch_bytes, uint64_t *status_host, void *stream) {
    if ((dtype != PCU_B200_F32 && dtype != PCU_B200_F64) || policy < 0 || policy > 2 || !status_host)
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (rows == 0 || columns == 0) {
        *status_host = PCU_B200_STATUS_OK;
        return PCU_B200_OK;
    }
    if (!out || (inner > 0 && (!left || !right))) return PCU_B200_ERROR_INVALID_ARGUMENT;
    unsigned __int128 events = (unsigned __int128)rows * columns;
    events *= (inner ? inner : 1);
    events *= 2;
    if (events > ((unsigned __int128)1 << 60)) return PCU_B200_ERROR_SIZE_OVERFLOW;
    const size_t elem = dtype == PCU_B200_F64 ? 8 : 4;
    const HostLayout lay(elem, rows, inner, columns);
    if (!device_scratch || scratch_bytes < lay.bytes) return PCU_B200_ERROR_WORKSPACE;
    std::lock_guard<std::mutex> guard(g_staging_lock);  // the event pool is shared per device
    Staging *stg = nullptr;
    int rc = staging_for_device(&stg);
    if (rc) return rc;
    cudaStream_t s = pcu_host::as_stream(stream);
    char *base = reinterpret_cast<char *>(device_scratch);
    uint64_t *st = reinterpret_cast<uint64_t *>(base + lay.st_off);
    const char *a_host = reinterpret_cast<const char *>(left);
    char *c_host = reinterpret_cast<char *>(out);
    cudaEvent_t *ev = stg->ev;
    cudaEvent_t ev_begin = ev[0], ev_b = ev[1];
    auto ev_a = [&](int i) { return ev[2 + i]; };
    auto ev_c = [&](int i) { return ev[2 + kMaxBlocks + i]; };
    auto ev_d = [&](int i) { return ev[2 + 2 * kMaxBlocks + i]; };
    auto check = [&](cudaError_t e) { return e == cudaSuccess ? 0 : pcu_host::set_cuda_error(e); };

    // everything the copy streams do comes after the work already queued on the caller's stream
    if ((rc = check(cudaEventRecord(ev_begin, s)))) return rc;
    if ((rc = check(cudaStreamWaitEvent(stg->up, ev_begin, 0)))) return rc;
    if ((rc = check(cudaStreamWaitEvent(stg->down, ev_begin, 0)))) return rc;
    if (inner > 0) {
        if ((rc = check(cudaMemcpyAsync(base + lay.b_off, right, inner * columns * elem, cudaMemcpyHostToDevice,
                                        stg->up))))
            return rc;
    }
    if ((rc = check(cudaEventRecord(ev_b, stg->up)))) return rc;
    for (int i = 0; i < lay.blocks; ++i) {
        const int buf = i & 1;
        const uint64_t r0 = (uint64_t)i * lay.block_rows;
        const uint64_t nr = r0 + lay.block_rows < rows ? lay.block_rows : rows - r0;
        char *da = base + lay.a_off[buf], *dc = base + lay.c_off[buf];
        // rows of A: after the product two blocks back has stopped reading this buffer
        if (i >= 2 && (rc = check(cudaStreamWaitEvent(stg->up, ev_c(i - 2), 0)))) return rc;
        if (inner > 0 && (rc = check(cudaMemcpyAsync(da, a_host + r0 * inner * elem, nr * inner * elem,
                                                     cudaMemcpyHostToDevice, stg->up))))
            return rc;
        if ((rc = check(cudaEventRecord(ev_a(i), stg->up)))) return rc;
        // the block's product: after its rows of A, B, and the read-back of this C buffer
        if ((rc = check(cudaStreamWaitEvent(s, ev_a(i), 0)))) return rc;
        if (i == 0 && (rc = check(cudaStreamWaitEvent(s, ev_b, 0)))) return rc;
        if (i >= 2 && (rc = check(cudaStreamWaitEvent(s, ev_d(i - 2), 0)))) return rc;
        if ((rc = pcu_b200_status_reset(st + i, 1, s))) return rc;
        rc = pcu::strict_matmul(dtype, policy, da, base + lay.b_off, dc, nr, inner, columns, inner, columns, 0, 0,
                                base + lay.ws_off, lay.ws_bytes, st + i, s, pcu::ChainGuard{});
        if (rc) return rc;
        if ((rc = check(cudaEventRecord(ev_c(i), s)))) return rc;
        // rows of C back to the host
        if ((rc = check(cudaStreamWaitEvent(stg->down, ev_c(i), 0)))) return rc;
        if ((rc = check(cudaMemcpyAsync(c_host + r0 * columns * elem, dc, nr * columns * elem, cudaMemcpyDeviceToHost,
                                        stg->down))))
            return rc;
        if ((rc = check(cudaEventRecord(ev_d(i), stg->down)))) return rc;
    }
    // the caller's stream completes only after every read-back (the copy streams run in order)
    if ((rc = check(cudaStreamWaitEvent(s, ev_d(lay.blocks - 1), 0)))) return rc;
    combine_block_status<<<1, 32, 0, s>>>(reinterpret_cast<const unsigned long long *>(st), lay.blocks,
                                          lay.block_rows, columns, inner,
                                          reinterpret_cast<unsigned long long *>(st + kMaxBlocks));
    if ((rc = pcu_host::launch_status())) return rc;
    return check(cudaMemcpyAsync(status_host, st + kMaxBlocks, sizeof(uint64_t), cudaMemcpyDeviceToHost, s));
}
