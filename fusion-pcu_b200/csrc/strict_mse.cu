// strict_mse.cu -- ordered strict mean squared error.
//
// Semantics (paths relative to the Fusion-PCU checkout): for i ascending, d = sub(p, t),
// q = mul(d, d), s = add(s, q) from s = +0, then mean = div(s, count rounded to nearest-even);
// each step separately rounded and checked; events i*3 + {Subtract 0, Multiply 1, Add 2} and
// 3n for Divide (Crates/core/dialect/tensor/reference/strict_mse/strict_mse.rs:22-59,
// Crates/core/dialect/tensor/fault_domain/fault_domain.rs:148-158).  The reference CUDA
// provider runs this on one lane (Crates/backends/cuda/tensor/strict_mse/strict_mse.rs:144-188).
//
// This provider splits the work:
//   phase 1 (all SMs, HBM-bound): every element's subtract and square with their checks,
//            writing the squares q[i] to the workspace plus a per-block maximum;
//   phase 2 (one warp): the ordered running sum.  The running sum of squares is monotone,
//            so a block whose largest square is below half an ulp of the current sum cannot
//            change it and is skipped whole; overflow (the only fault an Add of nonnegative
//            finite squares can raise, fault_domain.rs:207-214) is sticky, so it is checked per
//            block and located exactly only when it happened.
#include <cstring>

#include "common.cuh"
#include "pcu_b200.h"

namespace pcu {

constexpr int kMseBlock = 1024;  // elements per phase-2 skip block

template <typename T>
__global__ void __launch_bounds__(256) mse_squares_kernel(const T *prediction, const T *target, uint64_t n,
                                                          T *squares, T *block_max, int policy,
                                                          unsigned long long *status) {
    // one CTA of 256 threads covers kMseBlock elements per iteration
    __shared__ T warp_max[8];
    for (uint64_t blk = blockIdx.x; blk * kMseBlock < n; blk += gridDim.x) {
        T local = T(0);
        bool stop = false;
        for (int e = threadIdx.x; e < kMseBlock; e += 256) {
            const uint64_t i = blk * kMseBlock + e;
            if (i >= n || stop) break;
            T d, q;
            unsigned kind = checked_sub<T>(prediction[i], target[i], policy, d);
            if (kind) { record_fault(status, i * 3, kind); stop = true; break; }
            kind = checked_mul<T>(d, d, policy, q);
            if (kind) { record_fault(status, i * 3 + 1, kind); stop = true; break; }
            squares[i] = q;
            local = local > q ? local : q;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            T other = __shfl_xor_sync(0xffffffffu, local, o);
            local = local > other ? local : other;
        }
        if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = local;
        __syncthreads();
        if (threadIdx.x == 0) {
            T m = warp_max[0];
            for (int w = 1; w < 8; ++w) m = m > warp_max[w] ? m : warp_max[w];
            block_max[blk] = m;
        }
        __syncthreads();
    }
}

template <typename T>
__device__ __forceinline__ T half_ulp(T s) {
    using F = Fmt<T>;
    typename F::Bits b = F::bits(s);
    const int64_t field = (int64_t)((b & F::kExpMask) >> F::kFrac);
    // half an ulp of a normal s is 2^(field - bias - frac - 1), i.e. biased field - frac - 1;
    // near the bottom of the range (or for subnormal s) never skip
    if (field - F::kFrac - 1 <= 0) return T(0);
    return F::value((typename F::Bits)(field - F::kFrac - 1) << F::kFrac);
}

template <typename T>
__global__ void mse_sum_kernel(const T *squares, const T *block_max, uint64_t n, T denominator, int policy, T *out,
                               unsigned long long *status) {
    if (threadIdx.x != 0) return;
    using F = Fmt<T>;
    T s = T(0);
    const uint64_t blocks = (n + kMseBlock - 1) / kMseBlock;
    for (uint64_t blk = 0; blk < blocks; ++blk) {
        const uint64_t i0 = blk * kMseBlock;
        const uint64_t i1 = i0 + kMseBlock < n ? i0 + kMseBlock : n;
        // a subtract/multiply fault at or before this block ends the ordered walk
        if (fault_precedes(status, i1 * 3)) {
            // the walk may still own an earlier Add overflow inside [i0, i1)
            const unsigned long long st = read_status(status);
            const uint64_t first = (st >> 3) / 3;  // element of the earlier fault
            for (uint64_t i = i0; i < first && i < i1; ++i) {
                T t = F::add(s, squares[i]);
                if (nonfinite_bits<T>(F::bits(t))) { record_fault(status, i * 3 + 2, kOverflow); return; }
                s = t;
            }
            return;
        }
        if (block_max[blk] < half_ulp<T>(s)) continue;  // every step rounds back to s
        T t = s;
#pragma unroll 8
        for (uint64_t i = i0; i < i1; ++i) t = F::add(t, squares[i]);
        if (nonfinite_bits<T>(F::bits(t))) {
            for (uint64_t i = i0; i < i1; ++i) {
                T u = F::add(s, squares[i]);
                if (nonfinite_bits<T>(F::bits(u))) { record_fault(status, i * 3 + 2, kOverflow); return; }
                s = u;
            }
        }
        s = t;
    }
    if (fault_precedes(status, n * 3)) return;
    T mean;
    unsigned kind = checked_div<T>(s, denominator, policy, mean);
    if (kind) { record_fault(status, n * 3, kind); return; }
    out[0] = mean;
}

// binary32/binary64 encoding of an element count, nearest-even (constants/constants.rs:18-27)
template <typename T> T count_value(uint64_t n) {
    const int frac = sizeof(T) == 4 ? 23 : 52;
    const int bias = sizeof(T) == 4 ? 127 : 1023;
    uint64_t bits = 0;
    if (n) {
        int e = 63 - __builtin_clzll(n);
        uint64_t sig;
        if (e <= frac) {
            sig = n << (frac - e);
        } else {
            int sh = e - frac;
            uint64_t q = n >> sh, rem = n & ((1ull << sh) - 1), half = 1ull << (sh - 1);
            sig = q + (uint64_t)(rem > half || (rem == half && (q & 1)));
        }
        if (sig == (1ull << (frac + 1))) { sig >>= 1; e += 1; }
        bits = ((uint64_t)(e + bias) << frac) | (sig & ((1ull << frac) - 1));
    }
    T v;
    if (sizeof(T) == 4) {
        uint32_t b32 = (uint32_t)bits;
        memcpy(&v, &b32, 4);
    } else {
        memcpy(&v, &bits, 8);
    }
    return v;
}

template <typename T>
int run_mse(int policy, const T *p, const T *t, T *out, uint64_t n, void *workspace, size_t workspace_bytes,
            unsigned long long *status, cudaStream_t stream) {
    const uint64_t blocks = (n + kMseBlock - 1) / kMseBlock;
    size_t need = pcu_b200_strict_mse_workspace_size(sizeof(T) == 4 ? PCU_B200_F32 : PCU_B200_F64, n);
    if (!workspace || workspace_bytes < need) return PCU_B200_ERROR_WORKSPACE;
    T *squares = reinterpret_cast<T *>(workspace);
    T *block_max = reinterpret_cast<T *>(reinterpret_cast<char *>(workspace) + ((n * sizeof(T) + 255) / 256) * 256);
    uint64_t grid = blocks < (uint64_t)pcu_host::sm_count() * 8 ? blocks : (uint64_t)pcu_host::sm_count() * 8;
    mse_squares_kernel<T><<<(unsigned)grid, 256, 0, stream>>>(p, t, n, squares, block_max, policy, status);
    int rc = pcu_host::launch_status();
    if (rc) return rc;
    mse_sum_kernel<T><<<1, 32, 0, stream>>>(squares, block_max, n, count_value<T>(n), policy, out, status);
    return pcu_host::launch_status();
}

}  // namespace pcu

extern "C" size_t pcu_b200_strict_mse_workspace_size(int dtype, uint64_t count) {
    const size_t elem = dtype == PCU_B200_F64 ? 8 : 4;
    const uint64_t blocks = (count + pcu::kMseBlock - 1) / pcu::kMseBlock;
    return ((count * elem + 255) / 256) * 256 + ((blocks * elem + 255) / 256) * 256;
}

extern "C" int pcu_b200_strict_mse(int dtype, int policy, const void *prediction, const void *target, void *out,
                                   uint64_t count, void *workspace, size_t workspace_bytes, uint64_t *status,
                                   void *stream) {
    if ((dtype != PCU_B200_F32 && dtype != PCU_B200_F64) || policy < 0 || policy > 2 || !status)
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (count == 0 || !prediction || !target || !out) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (count > (1ull << 58)) return PCU_B200_ERROR_SIZE_OVERFLOW;
    auto *st = reinterpret_cast<unsigned long long *>(status);
    cudaStream_t s = pcu_host::as_stream(stream);
    if (dtype == PCU_B200_F32)
        return pcu::run_mse<float>(policy, (const float *)prediction, (const float *)target, (float *)out, count,
                                   workspace, workspace_bytes, st, s);
    return pcu::run_mse<double>(policy, (const double *)prediction, (const double *)target, (double *)out, count,
                                workspace, workspace_bytes, st, s);
}
