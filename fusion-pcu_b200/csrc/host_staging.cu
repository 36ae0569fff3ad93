// host_staging.cu -- strict MatMul with its operands and result in host memory: the host-boundary
// form of a node (upload, execute, read back), pipelined by row blocks of the result.
//
// The reference runs a host-fed node as three steps on one stream: the pending upload of the
// inputs (Crates/backends/cuda/tensor/pending_upload/pending_upload.rs:115-190: a private host
// copy, then cudaMemcpyAsync on the execution stream), the node's kernel, and the read of the
// output.  Here the rows of C are split into blocks.  B goes up once, in column pieces, and the
// first block is computed piece by piece as B's columns arrive; then, while block i is computed
// on the caller's stream, block i + 1's rows of A go up on one copy stream and block i - 1's rows
// of C come back on another, so the PCIe transfers hide behind the ordered-K arithmetic.  Every
// partial product is computed by the same strict MatMul as the device call, with a status word of
// its own; a last kernel maps each partial product's events to the ordinals of the whole product
// and keeps the lowest, which is the first fault of the one-call form.  Then that word is copied
// to the host.
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "pcu_b200.h"
#include "provider.h"

namespace {

constexpr int kMaxBlocks = 8;
constexpr int kFirstSplit = 4;               // column sub-blocks of the first row block
constexpr int kMaxWords = kMaxBlocks + kFirstSplit;
constexpr uint64_t kRowsPerBlockMin = 2048;  // smaller blocks lose compute to their last wave

// Where each partial product's cells sit in the whole product: rows [row0, ...), columns
// [col0, col0 + cols) of C.
struct Pieces {
    uint64_t row0[kMaxWords], col0[kMaxWords], cols[kMaxWords];
};

// The lowest first fault of the partial products, in the whole product's event ordinals: a
// partial product's cell (r, c) is the product's cell (row0 + r, col0 + c), and its event
// (cell * inner + k) * 2 + step keeps k and the step.
__global__ void combine_block_status(const unsigned long long *words, int count, Pieces pieces, uint64_t columns,
                                     uint64_t inner, unsigned long long *out) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    unsigned long long best = pcu::kStatusOk;
    const uint64_t per_cell = 2 * (inner ? inner : 1);
    for (int i = 0; i < count; ++i) {
        const unsigned long long w = words[i];
        if (w == pcu::kStatusOk) continue;
        const unsigned long long kind = w & 7;
        unsigned long long shifted = w;  // a wait that gave up (kind 7) is not an event of the product
        if (kind != pcu::kWatchdog) {
            const uint64_t ev = w >> 3, cell = ev / per_cell, rest = ev % per_cell;
            const uint64_t r = cell / pieces.cols[i], c = cell % pieces.cols[i];
            const uint64_t global = ((pieces.row0[i] + r) * columns + pieces.col0[i] + c) * per_cell + rest;
            shifted = (global << 3) | kind;
        }
        best = shifted < best ? shifted : best;
    }
    *out = best;
}

struct Staging {  // per device: the two copy streams and a pool of events
    cudaStream_t up = nullptr, down = nullptr;
    cudaEvent_t ev[2 + 3 * kMaxBlocks + 2 * kFirstSplit] = {};
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
        for (int i = 0; i < 2 + 3 * kMaxBlocks + 2 * kFirstSplit && err == cudaSuccess; ++i)
            err = cudaEventCreateWithFlags(&st.ev[i], cudaEventDisableTiming);
        if (err != cudaSuccess) return pcu_host::set_cuda_error(err);
        st.ready = true;
    }
    *out = &st;
    return PCU_B200_OK;
}

// Device scratch of a host-boundary call: B (unless it is already on the device), two row blocks
// of A and of C, the MatMul workspace and the status words.
struct HostLayout {
    int blocks;
    uint64_t block_rows;
    size_t b_off, a_off[2], c_off[2], ws_off, st_off, ws_bytes, bytes;
    HostLayout(size_t elem, uint64_t rows, uint64_t inner, uint64_t columns, bool right_on_device = false) {
        auto up = [](size_t v) { return (v + 255) / 256 * 256; };
        blocks = (int)(rows / kRowsPerBlockMin);
        blocks = blocks < 1 ? 1 : (blocks > 4 ? 4 : blocks);
        block_rows = (rows + blocks - 1) / blocks;
        size_t off = 0;
        b_off = off;
        if (!right_on_device) off += up(inner * columns * elem);
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
        off += up((kMaxWords + 1) * sizeof(uint64_t));
        bytes = off;
    }
};

}  // namespace

extern "C" size_t pcu_b200_strict_matmul_host_scratch_size(int dtype, uint64_t rows, uint64_t inner,
                                                           uint64_t columns) {
    return HostLayout(dtype == PCU_B200_F64 ? 8 : 4, rows, inner, columns).bytes;
}

extern "C" size_t pcu_b200_strict_matmul_host_left_scratch_size(int dtype, uint64_t rows, uint64_t inner,
                                                                uint64_t columns) {
    return HostLayout(dtype == PCU_B200_F64 ? 8 : 4, rows, inner, columns, true).bytes;
}

namespace {

// Both host-boundary forms: `right` in host memory (dense rows, uploaded here) or, with
// right_on_device, already on the device with row stride right_stride.
int run_host(int dtype, int policy, const void *left, const void *right, bool right_on_device, uint64_t right_stride,
             void *out, uint64_t rows, uint64_t inner, uint64_t columns, void *device_scratch, size_t scratch_bytes,
             uint64_t *status_host, void *stream) {
    if ((dtype != PCU_B200_F32 && dtype != PCU_B200_F64) || policy < 0 || policy > 2 || !status_host)
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (rows == 0 || columns == 0) {
        *status_host = PCU_B200_STATUS_OK;
        return PCU_B200_OK;
    }
    if (!out || (inner > 0 && (!left || !right))) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (right_on_device && inner > 0 && right_stride < columns) return PCU_B200_ERROR_INVALID_ARGUMENT;
    unsigned __int128 events = (unsigned __int128)rows * columns;
    events *= (inner ? inner : 1);
    events *= 2;
    if (events > ((unsigned __int128)1 << 60)) return PCU_B200_ERROR_SIZE_OVERFLOW;
    const size_t elem = dtype == PCU_B200_F64 ? 8 : 4;
    const HostLayout lay(elem, rows, inner, columns, right_on_device);
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
    cudaEvent_t ev_begin = ev[0];
    auto ev_a = [&](int i) { return ev[2 + i]; };
    auto ev_c = [&](int i) { return ev[2 + kMaxBlocks + i]; };
    auto ev_d = [&](int i) { return ev[2 + 2 * kMaxBlocks + i]; };
    auto ev_bj = [&](int j) { return ev[2 + 3 * kMaxBlocks + j]; };  // columns j of B are up
    auto ev_cj = [&](int j) { return ev[2 + 3 * kMaxBlocks + kFirstSplit + j]; };  // sub-product j done
    auto check = [&](cudaError_t e) { return e == cudaSuccess ? 0 : pcu_host::set_cuda_error(e); };
    const size_t pitch = columns * elem;
    // The first row block is computed in column sub-blocks, each as soon as its columns of B are
    // up, so B's upload overlaps the arithmetic too.  A sub-block's columns start 16-byte aligned
    // (a TMA requirement) and it needs enough columns to fill the GPU.
    const uint64_t align = 16 / elem;
    uint64_t sub_cols = (columns + kFirstSplit - 1) / kFirstSplit;
    sub_cols = (sub_cols + align - 1) / align * align;
    const int split = (!right_on_device && lay.blocks > 1 && inner > 0 && sub_cols >= 512)
                          ? (int)((columns + sub_cols - 1) / sub_cols)
                          : 1;
    const char *b_dev = right_on_device ? reinterpret_cast<const char *>(right) : base + lay.b_off;
    const uint64_t ldb = right_on_device ? right_stride : columns;
    Pieces pieces{};
    int words = 0;

    // everything the copy streams do comes after the work already queued on the caller's stream
    if ((rc = check(cudaEventRecord(ev_begin, s)))) return rc;
    if ((rc = check(cudaStreamWaitEvent(stg->up, ev_begin, 0)))) return rc;
    if ((rc = check(cudaStreamWaitEvent(stg->down, ev_begin, 0)))) return rc;
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
        if (i == 0) {  // B, in column blocks of `sub_cols` (the whole of B at once when split == 1)
            for (int j = 0; j < split && inner > 0 && !right_on_device; ++j) {
                const uint64_t c0 = (uint64_t)j * sub_cols, nc = split == 1 ? columns : std::min(sub_cols, columns - c0);
                if ((rc = check(cudaMemcpy2DAsync(base + lay.b_off + c0 * elem, pitch,
                                                  reinterpret_cast<const char *>(right) + c0 * elem, pitch, nc * elem,
                                                  inner, cudaMemcpyHostToDevice, stg->up))))
                    return rc;
                if ((rc = check(cudaEventRecord(ev_bj(j), stg->up)))) return rc;
            }
            if ((inner == 0 || right_on_device) && (rc = check(cudaEventRecord(ev_bj(0), stg->up)))) return rc;
        }
        // the block's product: after its rows of A, B (or its columns), and the read-back of this
        // C buffer two blocks back
        if ((rc = check(cudaStreamWaitEvent(s, ev_a(i), 0)))) return rc;
        if (i >= 2 && (rc = check(cudaStreamWaitEvent(s, ev_d(i - 2), 0)))) return rc;
        const int parts = i == 0 ? split : 1;
        for (int j = 0; j < parts; ++j) {
            const uint64_t c0 = (uint64_t)j * sub_cols, nc = parts == 1 ? columns : std::min(sub_cols, columns - c0);
            if (i == 0 && (rc = check(cudaStreamWaitEvent(s, ev_bj(parts == 1 ? 0 : j), 0)))) return rc;
            char *dcj = dc + (size_t)j * lay.block_rows * sub_cols * elem;  // dense nr x nc
            if ((rc = pcu_b200_status_reset(st + words, 1, s))) return rc;
            rc = pcu::strict_matmul(dtype, policy, da, b_dev + c0 * elem, dcj, nr, inner, nc, inner, ldb, 0, 0,
                                    base + lay.ws_off, lay.ws_bytes, st + words, s, pcu::ChainGuard{});
            if (rc) return rc;
            pieces.row0[words] = r0;
            pieces.col0[words] = c0;
            pieces.cols[words] = nc;
            ++words;
            cudaEvent_t done = parts == 1 ? ev_c(i) : ev_cj(j);
            if ((rc = check(cudaEventRecord(done, s)))) return rc;
            // rows of C (these columns) back to the host
            if ((rc = check(cudaStreamWaitEvent(stg->down, done, 0)))) return rc;
            if ((rc = check(cudaMemcpy2DAsync(c_host + (r0 * columns + c0) * elem, pitch, dcj, nc * elem, nc * elem, nr,
                                              cudaMemcpyDeviceToHost, stg->down))))
                return rc;
        }
        if (parts > 1 && (rc = check(cudaEventRecord(ev_c(i), s)))) return rc;
        if ((rc = check(cudaEventRecord(ev_d(i), stg->down)))) return rc;
    }
    // the caller's stream completes only after every read-back (the copy streams run in order)
    if ((rc = check(cudaStreamWaitEvent(s, ev_d(lay.blocks - 1), 0)))) return rc;
    combine_block_status<<<1, 32, 0, s>>>(reinterpret_cast<const unsigned long long *>(st), words, pieces, columns,
                                          inner, reinterpret_cast<unsigned long long *>(st + kMaxWords));
    if ((rc = pcu_host::launch_status())) return rc;
    return check(cudaMemcpyAsync(status_host, st + kMaxWords, sizeof(uint64_t), cudaMemcpyDeviceToHost, s));
}

}  // namespace

extern "C" int pcu_b200_strict_matmul_host(int dtype, int policy, const void *left, const void *right, void *out,
                                           uint64_t rows, uint64_t inner, uint64_t columns, void *device_scratch,
                                           size_t scratch_bytes, uint64_t *status_host, void *stream) {
    return run_host(dtype, policy, left, right, false, columns, out, rows, inner, columns, device_scratch,
                    scratch_bytes, status_host, stream);
}

extern "C" int pcu_b200_strict_matmul_host_left(int dtype, int policy, const void *left, const void *right,
                                                uint64_t right_stride, void *out, uint64_t rows, uint64_t inner,
                                                uint64_t columns, void *device_scratch, size_t scratch_bytes,
                                                uint64_t *status_host, void *stream) {
    return run_host(dtype, policy, left, right, true, right_stride, out, rows, inner, columns, device_scratch,
                    scratch_bytes, status_host, stream);
}
