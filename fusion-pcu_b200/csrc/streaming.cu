// streaming.cu -- HBM-streaming checked elementwise kernels: strict SGD, checked
// Add/Sub/Mul/Div (with uniform operands), checked ReLU and ReLU backward.
//
// Reference semantics (paths relative to the Fusion-PCU checkout):
//   SGD            Crates/core/dialect/tensor/reference/strict_sgd/strict_sgd.rs:20-46,
//                  CPU order execution.rs:231-242, CUDA event law tensor/strict_sgd/strict_sgd.rs:184-196
//   elementwise    Crates/backends/cpu/prepared_tensor/execution/execution.rs:192-211,
//                  CUDA status (index << 3) | kind, codegen/lower/checked_float/checked_float.rs:392-395
//   ReLU           execution.rs:212-219 / scalar_checked_float.rs:273-309
//   ReLU backward  execution.rs:220-230 / scalar_checked_float.rs:634-652,
//                  CUDA kernel tensor/relu_backward/relu_backward.rs:136-233
//
// Design: one thread walks 16-byte vectors of its elements in increasing order with a
// grid-stride loop (coalesced LDG.128/STG.128 with streaming cache hints), evaluates each
// element with the hardware-exact checked ops of checked_law.cuh and, at its first fault,
// records (event << 3) | kind with atomicMin and stops: later events of the same thread
// cannot be the minimum.  Every element in front of the first fault is still written, as in
// the reference's element-by-element loop.  Unaligned or uniform operands use the same loop
// with V = 1.
#include <cstring>

#include "common.cuh"
#include "pcu_b200.h"
#include "provider.h"

namespace pcu {

template <typename T, int V> struct Vec;
template <> struct Vec<float, 4> { using type = float4; };
template <> struct Vec<double, 2> { using type = double2; };

template <typename T, int V>
__device__ __forceinline__ void load_vec(const T *p, T (&v)[V]) {
    if constexpr (V == 1) {
        v[0] = __ldcs(p);
    } else {
        typename Vec<T, V>::type x = __ldcs(reinterpret_cast<const typename Vec<T, V>::type *>(p));
        const T *e = reinterpret_cast<const T *>(&x);
#pragma unroll
        for (int i = 0; i < V; ++i) v[i] = e[i];
    }
}

template <typename T, int V>
__device__ __forceinline__ void store_vec(T *p, const T (&v)[V]) {
    if constexpr (V == 1) {
        __stcs(p, v[0]);
    } else {
        typename Vec<T, V>::type x;
        T *e = reinterpret_cast<T *>(&x);
#pragma unroll
        for (int i = 0; i < V; ++i) e[i] = v[i];
        __stcs(reinterpret_cast<typename Vec<T, V>::type *>(p), x);
    }
}

// ---- per-element operations: return kOk or a kind, set `step` (event = index * kSteps + step)
// kFast: fast(a, b, out) evaluates a whole vector when no element can fault (false: run the
// elements one at a time)
template <typename T> struct SgdOp {
    static constexpr unsigned kSteps = 2;
    static constexpr bool kFast = true;
    T rate;
    int policy;
    __device__ __forceinline__ unsigned operator()(T w, T g, T &out, unsigned &step) const {
        return checked_sgd<T>(w, g, rate, policy, out, step);
    }
    template <int V> __device__ __forceinline__ bool fast(const T *w, const T *g, T *out) const {
        return sgd_fast<T, V>(w, g, rate, policy, out);
    }
};

template <typename T> struct BinaryOp {
    static constexpr unsigned kSteps = 1;
    static constexpr bool kFast = false;
    int op, policy;
    __device__ __forceinline__ unsigned operator()(T a, T b, T &out, unsigned &step) const {
        step = 0;
        return checked_binary<T>(op, a, b, policy, out);
    }
};

template <typename T> struct ReluOp {
    static constexpr unsigned kSteps = 1;
    static constexpr bool kFast = false;
    int policy;
    __device__ __forceinline__ unsigned operator()(T a, T, T &out, unsigned &step) const {
        step = 0;
        return checked_relu<T>(a, policy, out);
    }
};

template <typename T> struct ReluBackwardOp {
    static constexpr unsigned kSteps = 1;
    static constexpr bool kFast = false;
    int policy;
    __device__ __forceinline__ unsigned operator()(T x, T dy, T &out, unsigned &step) const {
        step = 0;
        return checked_relu_backward<T>(x, dy, policy, out);
    }
};

// a and b are element streams; a uniform stream (or a missing b) reads element 0 only.
#ifndef PCU_STREAM_UNROLL
#define PCU_STREAM_UNROLL 2
#endif

template <typename T, int V, class Op, int U = (V > 1 ? PCU_STREAM_UNROLL : 1)>
__global__ void __launch_bounds__(256) streaming_kernel(const T *a, const T *b,
                                                         T *out, uint64_t n, int a_uniform, int b_uniform,
                                                         Op op, unsigned long long *status, ChainGuard guard) {
    if (!chain_admits(guard)) return;  // a skipped stage of a guarded chain touches nothing
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t nvec = n / V;
    const T a0 = a_uniform ? a[0] : T(0);
    const T b0 = (b_uniform && b) ? b[0] : T(0);
    // U vectors per trip (the thread's vectors v, v + stride, ...: still in increasing order), all
    // loads issued before any is used, so every thread keeps U * 32 bytes in flight
    for (uint64_t v0 = tid; v0 < nvec; v0 += stride * U) {
        T av[U][V], bv[U][V];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint64_t v = v0 + (uint64_t)u * stride;
            if (v >= nvec) break;
            if (a_uniform) {
#pragma unroll
                for (int i = 0; i < V; ++i) av[u][i] = a0;
            } else {
                load_vec<T, V>(a + v * V, av[u]);
            }
            if (b_uniform || !b) {
#pragma unroll
                for (int i = 0; i < V; ++i) bv[u][i] = b0;
            } else {
                load_vec<T, V>(b + v * V, bv[u]);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const uint64_t v = v0 + (uint64_t)u * stride;
            if (v >= nvec) break;
            const uint64_t base = v * V;
            T ov[V];
            bool done = false;
            if constexpr (Op::kFast && V > 1) done = op.template fast<V>(av[u], bv[u], ov);
#pragma unroll
            for (int i = 0; i < V && !done; ++i) {
                unsigned step;
                unsigned kind = op(av[u][i], bv[u][i], ov[i], step);
                if (kind) {  // the elements in front of it are still written, as one at a time would
#pragma unroll
                    for (int q = 0; q < i; ++q) out[base + q] = ov[q];
                    record_fault(status, (unsigned long long)(base + i) * Op::kSteps + step, kind);
                    return;
                }
            }
            store_vec<T, V>(out + base, ov);
        }
    }
    for (uint64_t i = nvec * V + tid; i < n; i += stride) {
        T x = a_uniform ? a0 : a[i];
        T y = (b_uniform || !b) ? b0 : b[i];
        T r;
        unsigned step;
        unsigned kind = op(x, y, r, step);
        if (kind) {
            record_fault(status, (unsigned long long)i * Op::kSteps + step, kind);
            return;
        }
        out[i] = r;
    }
}

template <typename T, class Op>
int launch_streaming(const T *a, const T *b, T *out, uint64_t n, int a_uniform, int b_uniform, Op op,
                     unsigned long long *status, cudaStream_t stream, const ChainGuard &guard) {
    if (n == 0) return chain_decide_only(guard, stream);
    constexpr int V = 16 / sizeof(T);
    bool vec = pcu_host::aligned(out, 16) && (a_uniform || pcu_host::aligned(a, 16)) &&
               (b_uniform || !b || pcu_host::aligned(b, 16));
    const int threads = 256;
    uint64_t units = vec ? (n + V - 1) / V : n;
    uint64_t want = (units + threads - 1) / threads;
#ifndef PCU_STREAM_CTAS_PER_SM
#define PCU_STREAM_CTAS_PER_SM 8
#endif
    uint64_t cap = (uint64_t)pcu_host::sm_count() * PCU_STREAM_CTAS_PER_SM;
    unsigned blocks = (unsigned)(want < cap ? (want ? want : 1) : cap);
    if (vec)
        streaming_kernel<T, V, Op><<<blocks, threads, 0, stream>>>(a, b, out, n, a_uniform, b_uniform, op, status,
                                                                    guard);
    else
        streaming_kernel<T, 1, Op><<<blocks, threads, 0, stream>>>(a, b, out, n, a_uniform, b_uniform, op, status,
                                                                    guard);
    return pcu_host::launch_status();
}

}  // namespace pcu

using namespace pcu;

static bool valid_common(int dtype, int policy, const uint64_t *status) {
    return (dtype == PCU_B200_F32 || dtype == PCU_B200_F64) && policy >= 0 && policy <= 2 && status != nullptr;
}

int pcu::strict_sgd(int dtype, int policy, const void *weights, const void *gradient, void *out, uint64_t count,
                    uint32_t rate_bits_f32, uint64_t *status, void *stream, const ChainGuard &guard) {
    if (!valid_common(dtype, policy, status)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if ((rate_bits_f32 & 0x7f800000u) == 0x7f800000u) return PCU_B200_ERROR_INVALID_ARGUMENT;  // capture rejects
    if (count && (!weights || !gradient || !out)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (count > (1ull << 59)) return PCU_B200_ERROR_SIZE_OVERFLOW;
    auto *st = reinterpret_cast<unsigned long long *>(status);
    cudaStream_t s = pcu_host::as_stream(stream);
    if (dtype == PCU_B200_F32) {
        SgdOp<float> op{pcu_host::rate_f32(rate_bits_f32), policy};
        return launch_streaming<float>((const float *)weights, (const float *)gradient, (float *)out, count, 0, 0,
                                       op, st, s, guard);
    }
    SgdOp<double> op{pcu_host::rate_f64(rate_bits_f32), policy};
    return launch_streaming<double>((const double *)weights, (const double *)gradient, (double *)out, count, 0, 0,
                                    op, st, s, guard);
}

int pcu::checked_binary(int dtype, int policy, int op, const void *left, const void *right, void *out,
                        uint64_t count, int left_uniform, int right_uniform, uint64_t *status, void *stream,
                        const ChainGuard &guard) {
    if (!valid_common(dtype, policy, status) || op < 0 || op > 3) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (count && (!left || !right || !out)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (count > (1ull << 60)) return PCU_B200_ERROR_SIZE_OVERFLOW;
    auto *st = reinterpret_cast<unsigned long long *>(status);
    cudaStream_t s = pcu_host::as_stream(stream);
    if (dtype == PCU_B200_F32)
        return launch_streaming<float>((const float *)left, (const float *)right, (float *)out, count,
                                       left_uniform != 0, right_uniform != 0, BinaryOp<float>{op, policy}, st, s, guard);
    return launch_streaming<double>((const double *)left, (const double *)right, (double *)out, count,
                                    left_uniform != 0, right_uniform != 0, BinaryOp<double>{op, policy}, st, s, guard);
}

int pcu::checked_relu(int dtype, int policy, const void *input, void *out, uint64_t count, uint64_t *status,
                      void *stream, const ChainGuard &guard) {
    if (!valid_common(dtype, policy, status)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (count && (!input || !out)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (count > (1ull << 60)) return PCU_B200_ERROR_SIZE_OVERFLOW;
    auto *st = reinterpret_cast<unsigned long long *>(status);
    cudaStream_t s = pcu_host::as_stream(stream);
    if (dtype == PCU_B200_F32)
        return launch_streaming<float>((const float *)input, nullptr, (float *)out, count, 0, 0,
                                       ReluOp<float>{policy}, st, s, guard);
    return launch_streaming<double>((const double *)input, nullptr, (double *)out, count, 0, 0,
                                    ReluOp<double>{policy}, st, s, guard);
}

int pcu::checked_relu_backward(int dtype, int policy, const void *input, const void *upstream, void *out,
                               uint64_t count, uint64_t *status, void *stream, const ChainGuard &guard) {
    if (!valid_common(dtype, policy, status)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (count && (!input || !upstream || !out)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (count > (1ull << 60)) return PCU_B200_ERROR_SIZE_OVERFLOW;
    auto *st = reinterpret_cast<unsigned long long *>(status);
    cudaStream_t s = pcu_host::as_stream(stream);
    if (dtype == PCU_B200_F32)
        return launch_streaming<float>((const float *)input, (const float *)upstream, (float *)out, count, 0, 0,
                                       ReluBackwardOp<float>{policy}, st, s, guard);
    return launch_streaming<double>((const double *)input, (const double *)upstream, (double *)out, count, 0, 0,
                                    ReluBackwardOp<double>{policy}, st, s, guard);
}

extern "C" int pcu_b200_strict_sgd(int dtype, int policy, const void *weights, const void *gradient, void *out,
                                   uint64_t count, uint32_t rate_bits_f32, uint64_t *status, void *stream) {
    return pcu::strict_sgd(dtype, policy, weights, gradient, out, count, rate_bits_f32, status, stream, ChainGuard{});
}

extern "C" int pcu_b200_checked_binary(int dtype, int policy, int op, const void *left, const void *right,
                                       void *out, uint64_t count, int left_uniform, int right_uniform,
                                       uint64_t *status, void *stream) {
    return pcu::checked_binary(dtype, policy, op, left, right, out, count, left_uniform, right_uniform, status, stream,
                               ChainGuard{});
}

extern "C" int pcu_b200_checked_relu(int dtype, int policy, const void *input, void *out, uint64_t count,
                                     uint64_t *status, void *stream) {
    return pcu::checked_relu(dtype, policy, input, out, count, status, stream, ChainGuard{});
}

extern "C" int pcu_b200_checked_relu_backward(int dtype, int policy, const void *input, const void *upstream,
                                              void *out, uint64_t count, uint64_t *status, void *stream) {
    return pcu::checked_relu_backward(dtype, policy, input, upstream, out, count, status, stream, ChainGuard{});
}
