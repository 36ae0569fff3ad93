// calibrate.cu -- the measured roofline denominator of the strict MatMul: this GPU's FP32 and
// FP64 non-FMA issue rate.
//
// The strict contract forbids FMA, so the MatMul's peak is one separately rounded multiply or
// add per FP lane per cycle, not the FMA-counted figure.  The probe runs exactly that
// instruction mix with nothing to wait on: every thread keeps 8 independent multiply chains and
// 8 independent add chains (x = x * m and y = y + a, separately rounded), at full occupancy on
// every SM.  The multiplier and the addend are kernel arguments (1 and 0 in practice), so the
// compiler cannot fold the chains away and the values stay finite however long it runs.  The
// caller times the launch with CUDA events; pcu_b200_issue_probe_ops gives the operation count.
// Not part of the reference's path: a measurement aid for the bench's roofline.
#include <cstdint>

#include "common.cuh"
#include "pcu_b200.h"

namespace {

constexpr int kProbeThreads = 256;
constexpr int kProbeCtasPerSm = 8;  // 2048 threads per SM
constexpr int kChains = 8;          // independent multiply chains (and as many add chains) per thread
constexpr int kUnroll = 8;          // iterations per loop trip

__device__ double g_probe_sink;

template <typename T>
__global__ void __launch_bounds__(kProbeThreads) issue_probe_kernel(T m, T a, uint64_t trips) {
    using F = pcu::Fmt<T>;
    T x[kChains], y[kChains];
#pragma unroll
    for (int i = 0; i < kChains; ++i) {
        x[i] = T(1) + T(i) * T(0.125);
        y[i] = T(threadIdx.x) + T(i);
    }
    for (uint64_t t = 0; t < trips; ++t) {
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
#pragma unroll
            for (int i = 0; i < kChains; ++i) {
                x[i] = F::mul(x[i], m);
                y[i] = F::add(y[i], a);
            }
    }
    T s = T(0);
#pragma unroll
    for (int i = 0; i < kChains; ++i) s = F::add(s, F::add(x[i], y[i]));
    if (s == T(-1)) g_probe_sink = (double)s;  // never true for m = 1, a = 0; keeps every chain live
}

}  // namespace

extern "C" uint64_t pcu_b200_issue_probe_ops(int dtype, uint64_t iterations) {
    (void)dtype;
    const uint64_t trips = (iterations + kUnroll - 1) / kUnroll;
    return (uint64_t)pcu_host::sm_count() * kProbeCtasPerSm * kProbeThreads * trips * kUnroll * kChains * 2;
}

extern "C" int pcu_b200_issue_probe(int dtype, uint64_t iterations, void *stream) {
    if (dtype != PCU_B200_F32 && dtype != PCU_B200_F64) return PCU_B200_ERROR_INVALID_ARGUMENT;
    const uint64_t trips = (iterations + kUnroll - 1) / kUnroll;
    const unsigned ctas = (unsigned)pcu_host::sm_count() * kProbeCtasPerSm;
    cudaStream_t s = pcu_host::as_stream(stream);
    if (dtype == PCU_B200_F32) issue_probe_kernel<float><<<ctas, kProbeThreads, 0, s>>>(1.0f, 0.0f, trips);
    else issue_probe_kernel<double><<<ctas, kProbeThreads, 0, s>>>(1.0, 0.0, trips);
    return pcu_host::launch_status();
}
