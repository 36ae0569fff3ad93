// common.cuh -- shared device/host helpers of the B200 strict-tensor provider.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "checked_law.cuh"

namespace pcu {

// Record a fault (event, kind) in the node's status word; the lowest word wins
// (the reference's atomicMin contract, strict_matmul.rs:253-256).
__device__ __forceinline__ void record_fault(unsigned long long *status, unsigned long long event, unsigned kind) {
    atomicMin(status, (event << 3) | (unsigned long long)kind);
}

__device__ __forceinline__ unsigned long long read_status(const unsigned long long *status) {
    return *(volatile const unsigned long long *)status;
}

// True when an event strictly below `event` has already been recorded, so work whose
// first possible event is `event` can no longer change the reported fault.
__device__ __forceinline__ bool fault_precedes(const unsigned long long *status, unsigned long long event) {
    unsigned long long s = read_status(status);
    return s != kStatusOk && (s >> 3) < event;
}

// ---- guarded stage chain (Crates/backends/cuda/owned_dispatch/guarded/guarded.rs:15-38,
// Crates/core/runtime/execution/guarded/guarded.rs:30-55).  Every stage has a fault word and a
// disposition (pending 0, executed 1, skipped 2).  A stage is admitted when it has no
// predecessor, or when its predecessor executed and its fault word is still clear; otherwise
// it is skipped and touches no user data (no loads, no arithmetic, no output writes).  The
// stage's first kernel decides and records the disposition; its later kernels run only when
// it recorded "executed".  Kernels on one stream run in order, so the predecessor's record is
// final when a stage's first kernel reads it.
enum : unsigned long long { kDispPending = 0, kDispExecuted = 1, kDispSkipped = 2 };

struct ChainGuard {
    const unsigned long long *prev_status;  // predecessor's fault word (null: first stage)
    const unsigned long long *prev_disp;    // predecessor's disposition
    unsigned long long *disp;               // this stage's disposition (null: not guarded)
    int decide;                             // this launch is the stage's first kernel
};

// Out of line, so that unguarded launches (the common case) pay one compare and no registers.
static __device__ __noinline__ bool chain_decide(const unsigned long long *prev_status, const unsigned long long *prev_disp,
                                          unsigned long long *disp, int decide) {
    if (!decide) return read_status(disp) == kDispExecuted;
    const bool ok = !prev_disp || (read_status(prev_disp) == kDispExecuted && read_status(prev_status) == kStatusOk);
    if ((blockIdx.x | blockIdx.y | blockIdx.z | threadIdx.x | threadIdx.y | threadIdx.z) == 0)
        *disp = ok ? kDispExecuted : kDispSkipped;
    return ok;
}

__device__ __forceinline__ bool chain_admits(const ChainGuard &g) {
    return !g.disp || chain_decide(g.prev_status, g.prev_disp, g.disp, g.decide);
}

// The guard for a stage's later kernels.
inline ChainGuard chain_follow(ChainGuard g) {
    g.decide = 0;
    return g;
}

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Every device-side wait in this library gives up after this long and reports
// kWatchdog in the status word instead of spinning forever.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;
// Waits on another GPU's progress (a peer process entering the same call) allow for host-side
// skew between the ranks' processes as well, so they give up later.
constexpr unsigned long long kPeerWaitLimitNs = 10000000000ull;

}  // namespace pcu

// ---------------------------------------------------------------------------- host side
namespace pcu_host {

int set_cuda_error(cudaError_t err);  // records err for pcu_b200_last_cuda_error; returns PCU_B200_ERROR_CUDA
int launch_status(void);              // checks cudaGetLastError after a launch
int sm_count(void);                   // SMs of the current device (cached per device)

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// the SGD learning rate: a binary32 pattern, used as is (binary32) or widened (binary64)
inline float rate_f32(uint32_t bits) {
    float r;
    memcpy(&r, &bits, 4);
    return r;
}

// exact binary32 -> binary64 widening of a finite pattern (Crates/core/scalar_widen.rs:9-33)
inline double rate_f64(uint32_t bits) {
    uint64_t sign = (uint64_t)(bits >> 31) << 63;
    uint32_t field = (bits >> 23) & 0xffu, frac = bits & 0x7fffffu;
    uint64_t out;
    if (field != 0) {
        out = sign | ((uint64_t)(field + 1023 - 127) << 52) | ((uint64_t)frac << 29);
    } else if (frac == 0) {
        out = sign;
    } else {
        int lead = 31 - __builtin_clz(frac);
        uint64_t sig = (uint64_t)frac << (52 - lead);
        out = sign | ((uint64_t)(lead + 874) << 52) | (sig & 0x000fffffffffffffull);
    }
    double r;
    memcpy(&r, &out, 8);
    return r;
}

}  // namespace pcu_host
