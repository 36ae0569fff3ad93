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

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Every device-side wait in this library gives up after this long and reports
// kWatchdog in the status word instead of spinning forever.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

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
