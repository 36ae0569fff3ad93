// comm.cu -- the exchange steps of the multi-GPU paths behind the C ABI, for a host that has no
// communicator of its own (one process per GPU):
//   * the global first fault: an unsigned MIN of the ranks' status words (NCCL's Uint64 MIN is
//     unsigned, so the no-fault sentinel, all ones, stays the largest word);
//   * point-to-point hand-offs and broadcasts of device scalars (the running sum of a split MSE);
//   * the exchange of peer-buffer IPC handles for the row-sharded MatMul whose all-gather is
//     inside the kernel, and that MatMul with its fault MIN as one call;
//   * the split strict MSE with its ordered hand-off as one call.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2) when the first communicator is made, so the
// library has no load-time dependency on it.  A process that has already loaded NCCL (through
// torch.distributed, say) gets that same copy back from dlopen.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <new>
#include <type_traits>
#include <utility>
#include <vector>

#include "common.cuh"
#include "pcu_b200.h"

struct pcu_b200_comm {
    ncclComm_t comm;
    int nranks, rank;
    // device memory made with the communicator: words [0] the unused SGD status of a segment
    // call, [1] barrier, [2] the peer-buffer set-up's agreement; then one staging slot per rank for
    // the set-up's exchange of IPC handles (a status word, then the handle)
    uint64_t *scratch;
    // Calls made so far on each set of peer buffers (keyed by this rank's buffer): the call
    // number of the row-sharded MatMul's write-side order.  Every rank makes the same calls, so
    // the counts agree across ranks.
    std::vector<std::pair<void *, uint64_t>> calls;
    // The split strict MSE's hand-off blocks (every rank's, mapped here), made by the first
    // pcu_b200_comm_strict_mse call, and the number of such calls.
    void *handoff[8];
    uint64_t mse_calls;
};

namespace {

constexpr int kMaxRanks = 8;  // one rank per GPU of one node: the row-sharded MatMul takes <= 7 peers
constexpr size_t kHandleBytes = 64;
constexpr size_t kScratchWords = 3;
constexpr size_t kSlotBytes = 8 + kHandleBytes;
constexpr size_t kScratchBytes = kScratchWords * 8 + kMaxRanks * kSlotBytes;

struct Nccl {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) init_rank = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclCommAbort) abort = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclBroadcast) broadcast = nullptr;
    decltype(&ncclSend) send = nullptr;
    decltype(&ncclRecv) recv = nullptr;
    bool ok = false;
};

const Nccl &nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) return;
        bool all = true;
        auto bind = [&](auto &fn, const char *name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            all = all && fn != nullptr;
        };
        bind(n.get_unique_id, "ncclGetUniqueId");
        bind(n.init_rank, "ncclCommInitRank");
        bind(n.destroy, "ncclCommDestroy");
        bind(n.abort, "ncclCommAbort");
        bind(n.all_reduce, "ncclAllReduce");
        bind(n.all_gather, "ncclAllGather");
        bind(n.broadcast, "ncclBroadcast");
        bind(n.send, "ncclSend");
        bind(n.recv, "ncclRecv");
        n.ok = all;
    });
    return n;
}

thread_local int g_last_comm_error = 0;

int comm_status(ncclResult_t r) {
    if (r == ncclSuccess) return PCU_B200_OK;
    g_last_comm_error = (int)r;
    return PCU_B200_ERROR_COMM;
}

int cuda_status(cudaError_t e) { return e == cudaSuccess ? PCU_B200_OK : pcu_host::set_cuda_error(e); }

bool usable(const pcu_b200_comm *c) { return c && c->comm; }

// Every rank reaches this point before any goes on (host and device): a one-word all-reduce,
// then a wait for it.
int barrier(pcu_b200_comm *c, cudaStream_t s) {
    int rc = comm_status(nccl().all_reduce(c->scratch + 1, c->scratch + 1, 1, ncclUint64, ncclMin, c->comm, s));
    if (rc) return rc;
    return cuda_status(cudaStreamSynchronize(s));
}

}  // namespace

extern "C" int pcu_b200_last_comm_error(void) { return g_last_comm_error; }

extern "C" int pcu_b200_comm_unique_id(void *id) {
    if (!id) return PCU_B200_ERROR_INVALID_ARGUMENT;
    const Nccl &n = nccl();
    if (!n.ok) return PCU_B200_ERROR_UNSUPPORTED;
    ncclUniqueId u;
    if (int rc = comm_status(n.get_unique_id(&u))) return rc;
    static_assert(sizeof(u) == PCU_B200_COMM_ID_BYTES, "NCCL unique id size");
    memcpy(id, &u, sizeof(u));
    return PCU_B200_OK;
}

extern "C" int pcu_b200_comm_init(const void *id, int nranks, int rank, pcu_b200_comm **comm) {
    if (!comm) return PCU_B200_ERROR_INVALID_ARGUMENT;
    *comm = nullptr;
    if (!id || nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks) return PCU_B200_ERROR_INVALID_ARGUMENT;
    const Nccl &n = nccl();
    if (!n.ok) return PCU_B200_ERROR_UNSUPPORTED;
    auto *c = new (std::nothrow) pcu_b200_comm{};
    if (!c) return PCU_B200_ERROR_INVALID_ARGUMENT;
    c->nranks = nranks;
    c->rank = rank;
    int rc = cuda_status(cudaMalloc(reinterpret_cast<void **>(&c->scratch), kScratchBytes));
    if (!rc) rc = cuda_status(cudaMemset(c->scratch, 0xff, kScratchBytes));
    ncclUniqueId u;
    memcpy(&u, id, sizeof(u));
    if (!rc) rc = comm_status(n.init_rank(&c->comm, nranks, u, rank));
    if (rc) {
        if (c->scratch) cudaFree(c->scratch);
        delete c;
        return rc;
    }
    *comm = c;
    return PCU_B200_OK;
}

// The hand-off blocks without a collective (free and abort): unmap the peers', free this rank's.
static void drop_handoff(pcu_b200_comm *c) {
    if (!c->handoff[c->rank]) return;
    for (int r = 0; r < c->nranks; ++r)
        if (r != c->rank && c->handoff[r]) pcu_b200_peer_close(c->handoff[r]);
    pcu_b200_peer_free(c->handoff[c->rank]);
    for (int r = 0; r < c->nranks; ++r) c->handoff[r] = nullptr;
}

extern "C" int pcu_b200_comm_free(pcu_b200_comm *comm) {
    if (!comm) return PCU_B200_OK;
    if (comm->handoff[comm->rank]) {
        // every rank unmaps before any frees: the barrier of the peer-buffer release
        const int rc = pcu_b200_comm_peer_buffers_free(comm, comm->handoff, nullptr);
        if (rc) drop_handoff(comm);
    }
    int rc = comm->comm ? comm_status(nccl().destroy(comm->comm)) : PCU_B200_OK;
    if (comm->scratch) cudaFree(comm->scratch);
    delete comm;
    return rc;
}

extern "C" int pcu_b200_comm_abort(pcu_b200_comm *comm) {
    if (!comm) return PCU_B200_OK;
    int rc = comm->comm ? comm_status(nccl().abort(comm->comm)) : PCU_B200_OK;
    drop_handoff(comm);
    if (comm->scratch) cudaFree(comm->scratch);
    delete comm;
    return rc;
}

extern "C" int pcu_b200_comm_status_min(pcu_b200_comm *comm, uint64_t *status, uint64_t count, void *stream) {
    if (!usable(comm) || (count && !status)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (count == 0) return PCU_B200_OK;
    return comm_status(nccl().all_reduce(status, status, count, ncclUint64, ncclMin, comm->comm,
                                         pcu_host::as_stream(stream)));
}

extern "C" int pcu_b200_comm_send(pcu_b200_comm *comm, const void *buffer, size_t bytes, int peer, void *stream) {
    if (!usable(comm) || peer < 0 || peer >= comm->nranks || peer == comm->rank || (bytes && !buffer))
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    return comm_status(nccl().send(buffer, bytes, ncclUint8, peer, comm->comm, pcu_host::as_stream(stream)));
}

extern "C" int pcu_b200_comm_recv(pcu_b200_comm *comm, void *buffer, size_t bytes, int peer, void *stream) {
    if (!usable(comm) || peer < 0 || peer >= comm->nranks || peer == comm->rank || (bytes && !buffer))
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    return comm_status(nccl().recv(buffer, bytes, ncclUint8, peer, comm->comm, pcu_host::as_stream(stream)));
}

extern "C" int pcu_b200_comm_broadcast(pcu_b200_comm *comm, void *buffer, size_t bytes, int root, void *stream) {
    if (!usable(comm) || root < 0 || root >= comm->nranks || (bytes && !buffer))
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    return comm_status(
        nccl().broadcast(buffer, buffer, bytes, ncclUint8, root, comm->comm, pcu_host::as_stream(stream)));
}

// Each rank allocates its buffer with an IPC handle; the handles are all-gathered through the
// communicator's staging slots; each rank maps the others'.  Blocks until every rank has its
// mappings.  Collective even when it fails: every rank takes part in the exchange with its
// allocation's status and in a MAX of the mapping results, so when one rank cannot allocate or map,
// every rank releases what it holds and returns the same error, and none is left waiting in a
// later collective.
extern "C" int pcu_b200_comm_peer_buffers(pcu_b200_comm *comm, size_t bytes, void **buffers, void *stream) {
    if (!usable(comm) || !bytes || !buffers) return PCU_B200_ERROR_INVALID_ARGUMENT;
    const int n = comm->nranks, me = comm->rank;
    cudaStream_t s = pcu_host::as_stream(stream);
    for (int r = 0; r < n; ++r) buffers[r] = nullptr;
    unsigned char slot[kSlotBytes] = {};  // this rank's status word, then its handle
    const uint64_t alloc_rc = (uint64_t)pcu_b200_peer_alloc(bytes, &buffers[me], slot + 8);
    memcpy(slot, &alloc_rc, 8);
    unsigned char *staging = reinterpret_cast<unsigned char *>(comm->scratch + kScratchWords);
    std::vector<unsigned char> all(n * kSlotBytes);
    int rc = cuda_status(cudaMemcpyAsync(staging + me * kSlotBytes, slot, kSlotBytes, cudaMemcpyHostToDevice, s));
    const int ex = comm_status(
        nccl().all_gather(staging + me * kSlotBytes, staging, kSlotBytes, ncclUint8, comm->comm, s));
    rc = rc ? rc : ex;
    if (!rc) rc = cuda_status(cudaMemcpyAsync(all.data(), staging, all.size(), cudaMemcpyDeviceToHost, s));
    if (!rc) rc = cuda_status(cudaStreamSynchronize(s));
    for (int r = 0; r < n && !rc; ++r) {  // the first rank that could not allocate, as every rank sees it
        uint64_t st;
        memcpy(&st, all.data() + r * kSlotBytes, 8);
        if (st) rc = (int)st;
    }
    if (rc) {
        if (buffers[me]) pcu_b200_peer_free(buffers[me]);  // no peer has mapped it
        buffers[me] = nullptr;
        return rc;
    }
    int open_rc = 0;
    for (int r = 0; r < n && !open_rc; ++r)
        if (r != me) open_rc = pcu_b200_peer_open(all.data() + r * kSlotBytes + 8, &buffers[r]);
    uint64_t agreed = (uint64_t)open_rc;
    rc = cuda_status(cudaMemcpyAsync(comm->scratch + 2, &agreed, 8, cudaMemcpyHostToDevice, s));
    const int mx = comm_status(nccl().all_reduce(comm->scratch + 2, comm->scratch + 2, 1, ncclUint64, ncclMax,
                                                 comm->comm, s));
    rc = rc ? rc : mx;
    if (!rc) rc = cuda_status(cudaMemcpyAsync(&agreed, comm->scratch + 2, 8, cudaMemcpyDeviceToHost, s));
    if (!rc) rc = cuda_status(cudaStreamSynchronize(s));
    // every rank read the same non-zero word: every rank takes the barrier below.  Only a failure of
    // the exchange itself (a broken context or communicator) is left to this rank alone.
    const bool together = !rc && agreed;
    if (together) rc = open_rc ? open_rc : (int)agreed;
    if (rc) {
        for (int r = 0; r < n; ++r)
            if (r != me && buffers[r]) pcu_b200_peer_close(buffers[r]);
        if (together) barrier(comm, s);  // no rank still maps this rank's buffer when it is freed
        pcu_b200_peer_free(buffers[me]);
        for (int r = 0; r < n; ++r) buffers[r] = nullptr;
        return rc;
    }
    comm->calls.emplace_back(buffers[me], 0);
    return rc;
}

// Unmap the peers' buffers, wait until every rank has done so, then free this rank's own.
extern "C" int pcu_b200_comm_peer_buffers_free(pcu_b200_comm *comm, void **buffers, void *stream) {
    if (!usable(comm) || !buffers) return PCU_B200_ERROR_INVALID_ARGUMENT;
    const int me = comm->rank;
    cudaStream_t s = pcu_host::as_stream(stream);
    int rc = cuda_status(cudaStreamSynchronize(s));
    for (int r = 0; r < comm->nranks; ++r)
        if (r != me && buffers[r]) {
            const int e = pcu_b200_peer_close(buffers[r]);
            rc = rc ? rc : e;
            buffers[r] = nullptr;
        }
    const int b = barrier(comm, s);
    rc = rc ? rc : b;
    for (size_t i = 0; i < comm->calls.size(); ++i)
        if (comm->calls[i].first == buffers[me]) {
            comm->calls.erase(comm->calls.begin() + i);
            break;
        }
    if (buffers[me]) {
        const int e = pcu_b200_peer_free(buffers[me]);
        rc = rc ? rc : e;
        buffers[me] = nullptr;
    }
    return rc;
}

// Rows [row0, row0 + rows) of C = A . op(B) with the all-gather of C in the kernel
// (pcu_b200_strict_matmul_rows_allgather into buffers[rank] and every peer's buffer), then the
// status MIN that orders every rank's stores before C is read.  The call number on this buffer
// set orders the stores after the peers' reads of the previous call's C.
extern "C" int pcu_b200_comm_strict_matmul_rows(pcu_b200_comm *comm, int dtype, int policy, const void *left_rows,
                                                const void *right, void *const *buffers, uint64_t row0, uint64_t rows,
                                                uint64_t rows_total, uint64_t inner, uint64_t columns,
                                                uint64_t left_stride, uint64_t right_stride, int transpose_right,
                                                void *workspace, size_t workspace_bytes, uint64_t *status,
                                                void *stream) {
    if (!usable(comm) || !buffers || !status) return PCU_B200_ERROR_INVALID_ARGUMENT;
    uint64_t *calls = nullptr;
    for (auto &entry : comm->calls)
        if (entry.first == buffers[comm->rank]) calls = &entry.second;
    if (!calls) return PCU_B200_ERROR_INVALID_ARGUMENT;  // not a buffer set of this communicator
    void *peers[kMaxRanks - 1];
    int np = 0;
    for (int r = 0; r < comm->nranks; ++r)
        if (r != comm->rank) peers[np++] = buffers[r];
    int rc = pcu_b200_strict_matmul_rows_allgather(dtype, policy, left_rows, right, buffers[comm->rank], row0, rows,
                                                   rows_total, inner, columns, left_stride, right_stride,
                                                   transpose_right, peers, np, comm->rank, *calls + 1, workspace,
                                                   workspace_bytes, status, stream);
    if (rc) return rc;
    ++*calls;
    return pcu_b200_comm_status_min(comm, status, 1, stream);
}

// A strict MSE over total_count elements split into contiguous segments, rank r holding the
// global elements [first_index, first_index + count), through pcu_b200_strict_mse_sgd_split: the
// running sum goes from rank to rank on the device (IPC-mapped hand-off blocks, made by the
// first call, which is collective like every call here), and a one-warp exchange leaves the
// mean and the MIN of the status words on every rank.  No NCCL call after the first.
extern "C" int pcu_b200_comm_strict_mse(pcu_b200_comm *comm, int dtype, int policy, const void *prediction,
                                        const void *target, uint64_t count, uint64_t first_index, uint64_t total_count,
                                        void *out, void *workspace, size_t workspace_bytes, uint64_t *status,
                                        void *stream) {
    if (!usable(comm) || !out || !status || (dtype != PCU_B200_F32 && dtype != PCU_B200_F64))
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    // a rank's segment may be empty (its walk passes the running sum on unchanged)
    if (total_count == 0 || first_index > total_count || count > total_count - first_index)
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (!comm->handoff[comm->rank]) {
        const int rc = pcu_b200_comm_peer_buffers(comm, pcu_b200_mse_handoff_bytes(), comm->handoff, stream);
        if (rc) return rc;
    }
    const int rc = pcu_b200_strict_mse_sgd_split(dtype, policy, prediction, target, count, first_index, total_count,
                                                 out, workspace, workspace_bytes, status, nullptr, nullptr, nullptr, 0,
                                                 0, 0x3f800000u, nullptr, comm->handoff, comm->rank, comm->nranks,
                                                 comm->mse_calls + 1, stream);
    if (!rc) ++comm->mse_calls;
    return rc;
}
