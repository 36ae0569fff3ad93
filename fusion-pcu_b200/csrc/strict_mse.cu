// strict_mse.cu -- ordered strict mean squared error at HBM speed, bit-exact.
//
// Semantics (paths relative to the Fusion-PCU checkout): for i ascending, d = sub(p, t),
// q = mul(d, d), s = add(s, q) from s = +0, then mean = div(s, count rounded to nearest-even);
// each step separately rounded and checked; events i*3 + {Subtract 0, Multiply 1, Add 2} and 3n
// for Divide (Crates/core/dialect/tensor/reference/strict_mse/strict_mse.rs:22-59,
// Crates/core/dialect/tensor/fault_domain/fault_domain.rs:148-158).  The reference CUDA
// provider runs the whole reduction on one lane (tensor/strict_mse/strict_mse.rs:144-188).
//
// Exact parallel algorithm.  Write the running sum as s = x * u with u = 2^k its ulp (k = e - P
// for s in the binade [2^e, 2^(e+1)), P = 23 or 52 fraction bits; below the top of the
// smallest normal binade the spacing is the minimum, k = KMIN).  While s stays inside its
// binade, one step is x' = x + y rounded to the nearest integer, ties to even, y = q / u.  That
// equals x + RN_half_up(y) unless y is an exact half-integer (a tie), where the result is the
// even neighbour and so depends on x's parity.  A run of squares therefore acts on the state as
//                     x  ->  x + D[x mod 2]
// for two integers D[0], D[1] (they differ only through ties), valid while the final state stays
// below 2^(P+1) (every intermediate exact sum is then inside the binade).  Such maps compose:
// D12[p] = D1[p] + D2[(p + D1[p]) mod 2].  Squares are >= 0, so s is monotone and only ever
// moves up through the binades.
//
//   phase 1 (mse_chunk_kernel, all SMs, HBM bound): one warp per CHUNK elements computes the
//     subtract and the square (a cheap test selects the exact checked path for rare suspects),
//     then D for every binade k of the window [k_hi - W + 1, k_hi], k_hi = exponent(max q) + 1
//     (above it every y < 1/2: identity):
//       * q in fixed point Q = floor(q / 2^(k_lo - 1)); the half-up increment at binade k is
//         (Q + 2^(j-1)) >> j, j = k - k_lo + 1, so its chunk sum is W_j + cnt[j-1] with
//         W_j = sum over b >= j of cnt[b] 2^(b-j), from the per-bit population counts cnt[b]
//         (Harley-Seal vertical counters per lane, a warp bit-transpose per counter plane);
//       * the parity of a half-up increment is bit j of R = Q ^ (Q << 1), so one exclusive
//         prefix-XOR of R gives, for every binade at once, the parity of the half-up running
//         increment in front of each element;
//       * a tie at binade k is a square whose lowest set bit of Q is bit j-1, with nothing of q
//         below 2^(k_lo - 1).  Only binades where the chunk's half-up sum stays below 2^P are
//         kept (below them the map could never be applied); their ties (rare for rounded squares, common
//         for exact ones) are found from the largest lowest set bit, confirmed exactly, listed
//         in element order and give the corrections for an even and an odd start.
//   phase 2 (mse_compose_kernel, twice): compose the maps of kFanout chunks into block maps,
//     and of kFanout blocks into superblock maps.
//   phase 3 (mse_walk_kernel, one CTA): from the carried running sum, warp 0 applies up to 32
//     superblock, block or chunk maps at a time (a prefix scan of the map composition over the
//     lanes; the leading maps whose state stays inside the binade are taken), descending a
//     level where a map cannot be applied.  A chunk whose map cannot be applied (the state
//     crosses a binade inside it, or a Subtract/Multiply fault lies in it) is resolved with one
//     thread per element: the half-up increments at the current
//     binade are prefix-summed, every element before the first tie or binade crossing is
//     applied at once, and that one element is added exactly with the IEEE add.  The only
//     fault an Add of nonnegative finite squares can raise is overflow (fault_domain.rs:207-214);
//     a map is never applied when its result would leave the binade, so overflow is always met
//     by the exact add.  Then the checked divide.
#include <algorithm>
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "mse_walk_plan.h"
#include "pcu_b200.h"
#include "provider.h"

#ifndef PCU_MSE_MIN_BLOCKS_F32
#define PCU_MSE_MIN_BLOCKS_F32 4
#endif

namespace pcu {

template <typename T> struct MseTraits;
template <> struct MseTraits<float> {
    using Fix = uint32_t;     // fixed-point square (W bits) under the bits of 2^P
    using D = uint32_t;       // map increment: a valid one is below 2^24
    static constexpr int EPT = 32;               // elements per lane
    static constexpr int CHUNK = 32 * EPT;       // 1024: one warp
    static constexpr int W = 23;                 // binades per window: Q < 2^W fits a significand
    static constexpr int P = 23;                 // fraction bits
    static constexpr int KMIN = -149;            // smallest ulp exponent
    static constexpr int PLANES = 6;             // vertical counter planes: counts up to 63
    static constexpr uint64_t SAT = 1ull << 40;  // no valid increment comes near this
    static constexpr int MIN_BLOCKS = PCU_MSE_MIN_BLOCKS_F32;  // chunk kernel residency target per SM
};
template <> struct MseTraits<double> {
    using Fix = uint64_t;
    using D = uint64_t;       // a valid increment is below 2^53
    static constexpr int EPT = 16;
    static constexpr int CHUNK = 32 * EPT;       // 512
    static constexpr int W = 52;
    static constexpr int P = 52;
    static constexpr int KMIN = -1074;
    static constexpr int PLANES = 5;
    static constexpr uint64_t SAT = 1ull << 62;
    static constexpr int MIN_BLOCKS = 2;
};

constexpr int kFanout = 64;      // child maps per parent map: chunk -> block -> superblock
constexpr int kLevels = 3;       // chunk, block, superblock
constexpr int kChunkWarps = 8;   // chunks (warps) per CTA of the chunk kernel

enum : int { kHeadZero = 1, kHeadFault = 4 };

struct MseHead {
    int32_t k_lo;      // window [k_lo, k_lo + W - 1]
    int32_t flags;     // kHeadZero: every square is +0; kHeadFault: a Subtract/Multiply fault
    uint32_t fault;    // first Subtract/Multiply fault (relative to the map's first element)
    uint32_t pad;
};

template <typename T> __device__ __forceinline__ typename MseTraits<T>::D no_map() {
    return (typename MseTraits<T>::D)~0ull;
}

template <typename T> __device__ __forceinline__ typename MseTraits<T>::D sat_d(uint64_t v) {
    return v >= MseTraits<T>::SAT ? no_map<T>() : (typename MseTraits<T>::D)v;
}

template <typename T> __device__ __forceinline__ int exponent_of(typename Fmt<T>::Bits b) {
    using F = Fmt<T>;
    const int field = (int)((b & F::kExpMask) >> F::kFrac);
    if (field) return field - F::kBias;
    typename F::Bits f = b & F::kFracMask;
    const int top = sizeof(T) == 4 ? 31 - __clz((int)f) : 63 - __clzll((long long)f);
    return top + F::kMinExp - F::kFrac;
}

// x (state in ulps) and k (ulp exponent) of a running sum s >= 0.
template <typename T>
__device__ __forceinline__ void state_of(T s, uint64_t &x, int &k) {
    using F = Fmt<T>;
    using Tr = MseTraits<T>;
    typename F::Bits b = F::bits(s);
    const int field = (int)((b & F::kExpMask) >> F::kFrac);
    const uint64_t frac = (uint64_t)(b & F::kFracMask);
    if (field <= 1) {  // subnormal or smallest normal binade: spacing is the minimum ulp
        k = Tr::KMIN;
        x = field ? (frac | (1ull << Tr::P)) : frac;
    } else {
        k = field - F::kBias - Tr::P;
        x = frac | (1ull << Tr::P);
    }
}

template <typename T>
__device__ __forceinline__ T value_of(uint64_t x, int k) {
    using F = Fmt<T>;
    using Tr = MseTraits<T>;
    if (k == Tr::KMIN) return F::value((typename F::Bits)x);  // field 0 or 1 encodes x directly
    return F::value(((typename F::Bits)(k + Tr::P + F::kBias) << F::kFrac) |
                    ((typename F::Bits)x & F::kFracMask));
}

struct Tie {
    uint16_t index;   // chunk-relative element
    uint8_t j;        // binade offset: k = k_lo + j - 1
    uint8_t bits;     // bit 0: parity of floor(q / 2^k); bit 1: parity of the half-up increments in front
};

template <typename T> __device__ __forceinline__ typename Fmt<T>::Bits warp_max_bits(typename Fmt<T>::Bits v) {
    if constexpr (sizeof(T) == 4) {
        return __reduce_max_sync(0xffffffffu, (unsigned)v);
    } else {
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            unsigned long long other = __shfl_xor_sync(0xffffffffu, (unsigned long long)v, o);
            v = other > v ? other : v;
        }
        return v;
    }
}

template <typename X> __device__ __forceinline__ X shfl_up_x(X v, int o) {
    if constexpr (sizeof(X) == 4) return __shfl_up_sync(0xffffffffu, (unsigned)v, o);
    else return __shfl_up_sync(0xffffffffu, (unsigned long long)v, o);
}

template <typename X> __device__ __forceinline__ X shfl_down_x(X v, int o) {
    if constexpr (sizeof(X) == 4) return __shfl_down_sync(0xffffffffu, (unsigned)v, o);
    else return __shfl_down_sync(0xffffffffu, (unsigned long long)v, o);
}

template <typename X> __device__ __forceinline__ X shfl_xor_x(X v, int o) {
    if constexpr (sizeof(X) == 4) return __shfl_xor_sync(0xffffffffu, (unsigned)v, o);
    else return __shfl_xor_sync(0xffffffffu, (unsigned long long)v, o);
}

template <typename X> __device__ __forceinline__ X shfl_x(X v, int src) {
    if constexpr (sizeof(X) == 4) return __shfl_sync(0xffffffffu, (unsigned)v, src);
    else return __shfl_sync(0xffffffffu, (unsigned long long)v, src);
}

// Element layout of a chunk (one warp): in row r lane l owns the V consecutive elements from
// r * 32 * V + l * V (32 bytes per lane and row, coalesced across the warp).
template <typename T> struct ChunkMap {
    static constexpr int V = 32 / sizeof(T);
    static constexpr int ROWS = MseTraits<T>::EPT / V;
    __device__ static __forceinline__ int index(int row, int lane, int e) { return row * 32 * V + lane * V + e; }
};

// a[idx] for a register array and a run-time index, without demoting the array to memory
template <typename X, int N> __device__ __forceinline__ X get_at(const X (&a)[N], int idx) {
    X v = a[0];
#pragma unroll
    for (int i = 1; i < N; ++i)
        if (i == idx) v = a[i];
    return v;
}

// a[idx] = v for a register array and a run-time index, without demoting the array to memory
template <typename X, int N> __device__ __forceinline__ void set_at(X (&a)[N], int idx, X v) {
#pragma unroll
    for (int i = 0; i < N; ++i)
        if (i == idx) a[i] = v;
}

// The square of one element with the reference's checked subtract and multiply (first fault
// recorded); used only for the rare elements the fast test flags.
template <typename T>
__device__ __noinline__ bool checked_square(T p, T t, uint64_t i, int policy, unsigned long long *status, T &q) {
    T d;
    unsigned kind = checked_sub<T>(p, t, policy, d);
    if (kind) { record_fault(status, i * 3, kind); return false; }
    kind = checked_mul<T>(d, d, policy, q);
    if (kind) { record_fault(status, i * 3 + 1, kind); return false; }
    return true;
}

// carry-save adder on bit vectors: a + b + c = 2 * hi + lo in every bit position
template <typename X> __device__ __forceinline__ void csa(X &hi, X &lo, X a, X b, X c) {
    const X u = a ^ b;
    hi = (a & b) | (u & c);
    lo = u ^ c;
}

// Harley-Seal tree: adds the 2^L words q[BASE .. BASE + 2^L) into the vertical bit counters
// acc[0 .. L-1] (acc[i] holds bit i of every column's count) and returns the carry word of
// weight 2^L.  2^L - 1 carry-save adders in all.
template <int L, int BASE> struct SealTree {
    template <typename X, int N, int P>
    __device__ static __forceinline__ X run(const X (&q)[N], X (&acc)[P]) {
        const X a = SealTree<L - 1, BASE>::run(q, acc);
        const X b = SealTree<L - 1, BASE + (1 << (L - 1))>::run(q, acc);
        X h;
        csa(h, acc[L - 1], acc[L - 1], a, b);
        return h;
    }
};
template <int BASE> struct SealTree<1, BASE> {
    template <typename X, int N, int P>
    __device__ static __forceinline__ X run(const X (&q)[N], X (&acc)[P]) {
        X h;
        csa(h, acc[0], acc[0], q[BASE], q[BASE + 1]);
        return h;
    }
};

// 32 x 32 bit-matrix transpose across a warp: on return lane b holds, in bit l, bit b of lane
// l's input word.  Five butterfly stages swap the off-diagonal blocks: the 16- and 8-bit
// stages are byte permutes, the 4-, 2- and 1-bit stages a rotation and a masked merge (the
// rotated-in bits always land in positions the mask drops).
__device__ __forceinline__ unsigned warp_transpose32(unsigned x, int lane) {
    unsigned y = __shfl_xor_sync(0xffffffffu, x, 16);
    x = __byte_perm(x, y, (lane & 16) ? 0x3276 : 0x5410);
    y = __shfl_xor_sync(0xffffffffu, x, 8);
    x = __byte_perm(x, y, (lane & 8) ? 0x3715 : 0x6240);
#pragma unroll
    for (int h = 4; h; h >>= 1) {
        const unsigned m = h == 4 ? 0x0f0f0f0fu : h == 2 ? 0x33333333u : 0x55555555u;  // (index & h) == 0
        const bool hi = lane & h;
        y = __shfl_xor_sync(0xffffffffu, x, h);
        const unsigned t = __funnelshift_r(y, y, hi ? h : 32 - h);  // hi: y >> h, lo: y << h (rotations)
        const unsigned keep = hi ? ~m : m;
        x = (x & keep) | (t & ~keep);
    }
    return x;
}

// Fixed-point form of one square (bits qb, finite, >= +0): Q = floor(q / 2^L0) given
// C = bias + frac + 3 + L0 and K = (1 - C) * 2^(frac + 3).  q = m * 2^(e1 - bias - frac) with
// e1 = max(field, 1) and m its significand; Q = (8 m) >> (C - e1) (C - e1 >= 0 for q <= qmax).
// `mm` receives 8 m and `dn` the shift (for the exact remainder test of the rare tie path).
template <typename T>
__device__ __forceinline__ typename MseTraits<T>::Fix fixed_point(typename MseTraits<T>::Fix qb, int C,
                                                                  typename MseTraits<T>::Fix K, int &dn,
                                                                  typename MseTraits<T>::Fix &mm) {
    using F = Fmt<T>;
    using Fix = typename MseTraits<T>::Fix;
    const int field = (int)(qb >> F::kFrac);
    dn = min(C - field, C - 1);                                        // C - e1
    mm = qb * (Fix)8 + K + (Fix)dn * ((Fix)1 << (F::kFrac + 3));       // 8 m, exact modulo 2^bits
    if constexpr (sizeof(Fix) == 4) return __funnelshift_rc(mm, 0u, dn);  // 0 once dn >= 32
    else return dn < 64 ? mm >> dn : 0;
}

// a + b rounded toward zero (for a >= 0 and b = 2^P: 2^P + floor(a) while a < 2^P)
__device__ __forceinline__ float add_rz(float a, float b) { return __fadd_rz(a, b); }
__device__ __forceinline__ double add_rz(double a, double b) { return __dadd_rz(a, b); }

// Ask the L2 to fetch [p, p + bytes) ahead of its use (a hint: no destination, no completion).
__device__ __forceinline__ void prefetch_l2(const void *p, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// x << s clamped at `sat` (x <= sat), for 0 <= s
__device__ __forceinline__ uint64_t sat_shl(uint64_t x, int s, uint64_t sat) {
    if (!x) return 0;
    if (s >= 63) return sat;
    return x >= (sat >> s) ? sat : x << s;
}

// ---- an independent strict SGD node riding along (pcu_b200_strict_mse_sgd).  Its HBM traffic
// overlaps the chunk kernel's integer work (and, for an SGD node far larger than the MSE, the
// single-CTA walker); its elements, events and status word are its own, so the result is that
// of the SGD node run alone.
template <typename T> struct SgdRider {
    const T *weights, *gradient;
    T *out;
    uint64_t n;         // elements [0, n) of this launch's share
    uint64_t base;      // global index of element 0: events (base + i) * 2 + step
    uint64_t per_unit;  // chunk kernel: elements per SGD CTA (a multiple of sgd_unit<T>())
    T rate;
    int policy;
    bool vec;  // weights, gradient and out 16-byte aligned
    unsigned long long *status;
};

// The chunk kernel carries its SGD share in dedicated CTAs: every kSgdPeriod-th CTA of the launch
// streams a block of SGD elements, the others are chunk CTAs.  The chunk warps are bound by
// integer issue and the SGD CTAs by HBM, so an SM holding both keeps both busy (an SGD slice
// inside every chunk warp instead stalls that warp's integer work on memory).
#ifndef PCU_SGD_PERIOD
#define PCU_SGD_PERIOD 4
#endif
constexpr int kSgdPeriod = PCU_SGD_PERIOD;
constexpr int kSgdTrip = 2;  // 16-byte vectors per thread in flight
#ifndef PCU_SGD_CTA_TRIP
#define PCU_SGD_CTA_TRIP 2
#endif
constexpr int kSgdCtaTrip = PCU_SGD_CTA_TRIP;  // in the SGD CTAs of a chunk launch
// elements of one SGD CTA trip: the per-CTA share is a multiple of it
template <typename T> constexpr uint64_t sgd_unit() { return 32ull * kChunkWarps * (16 / sizeof(T)) * kSgdCtaTrip; }

// Elements [s0, s1) of a rider over `lanes` threads (this one is `lane`), s0 a multiple of the
// vector width.  Every thread takes its elements in increasing order and stops at its first
// fault: its later events cannot be the minimum.
template <typename T, int kTrip = kSgdTrip>
__device__ __forceinline__ void sgd_range(const SgdRider<T> &r, uint64_t s0, uint64_t s1, uint64_t lane,
                                          uint64_t lanes) {
    using VT = typename std::conditional<sizeof(T) == 4, float4, double2>::type;
    constexpr int VW = 16 / sizeof(T);
    const uint64_t vend = r.vec ? s0 + (s1 - s0) / VW * VW : s0;
    const uint64_t nv = (vend - s0) / VW;
    for (uint64_t j0 = lane; j0 < nv; j0 += lanes * kTrip) {
        VT a[kTrip], b[kTrip];
#pragma unroll
        for (int u = 0; u < kTrip; ++u) {
            const uint64_t j = j0 + u * lanes;
            if (j < nv) {
                a[u] = __ldcs(reinterpret_cast<const VT *>(r.weights + s0) + j);
                b[u] = __ldcs(reinterpret_cast<const VT *>(r.gradient + s0) + j);
            }
        }
#pragma unroll
        for (int u = 0; u < kTrip; ++u) {
            const uint64_t j = j0 + u * lanes;
            if (j >= nv) break;
            VT o;
            const bool done = sgd_fast<T, VW>(reinterpret_cast<const T *>(&a[u]), reinterpret_cast<const T *>(&b[u]),
                                              r.rate, r.policy, reinterpret_cast<T *>(&o));
#pragma unroll
            for (int e = 0; e < VW && !done; ++e) {
                unsigned step;
                const unsigned kind = checked_sgd<T>(reinterpret_cast<const T *>(&a[u])[e],
                                                     reinterpret_cast<const T *>(&b[u])[e], r.rate, r.policy,
                                                     reinterpret_cast<T *>(&o)[e], step);
                if (kind) {  // the elements in front of it are still written, as one at a time would
#pragma unroll
                    for (int q = 0; q < e; ++q) r.out[s0 + j * VW + q] = reinterpret_cast<const T *>(&o)[q];
                    record_fault(r.status, (r.base + s0 + j * VW + e) * 2 + step, kind);
                    return;
                }
            }
            __stcs(reinterpret_cast<VT *>(r.out + s0) + j, o);
        }
    }
    for (uint64_t i = vend + lane; i < s1; i += lanes) {
        T o;
        unsigned step;
        const unsigned kind = checked_sgd<T>(r.weights[i], r.gradient[i], r.rate, r.policy, o, step);
        if (kind) {
            record_fault(r.status, (r.base + i) * 2 + step, kind);
            return;
        }
        r.out[i] = o;
    }
}

// A chunk warp's shared-memory slot: its fixed-point squares, later its ties.
template <typename T> constexpr size_t kSlotBytes = (size_t)MseTraits<T>::CHUNK * sizeof(typename MseTraits<T>::Fix);

// The maps of one chunk, one warp (chunk `cta * kChunkWarps + warp`); returns early per warp.
template <typename T>
__device__ __forceinline__ void chunk_maps(uint64_t cta, const T *prediction, const T *target, uint64_t n,
                                           uint64_t base, bool vec, int policy, uint64_t chunks, uint64_t ahead,
                                           MseHead *heads, typename MseTraits<T>::D *deltas,
                                           unsigned long long *status, unsigned char *slots) {
    using Tr = MseTraits<T>;
    using F = Fmt<T>;
    using B = typename F::Bits;
    using Fix = typename Tr::Fix;
    using CM = ChunkMap<T>;
    constexpr int EPT = Tr::EPT, W = Tr::W, V = CM::V, ROWS = CM::ROWS;
    constexpr int LOG_EPT = EPT == 32 ? 5 : 4;
    constexpr int NW = (W + 31) / 32;  // 32-bit words of a fixed-point square
    static_assert((1 << LOG_EPT) == EPT && LOG_EPT + 1 == Tr::PLANES, "counter planes");
    // |d| below 2^-62 (binary32) / 2^-510 (binary64) may square to <= the smallest normal
    constexpr B kTinyDiff = sizeof(T) == 4 ? (B)(127 - 62) << 23 : (B)(1023 - 510) << 52;
    using VT = typename std::conditional<sizeof(T) == 4, float4, double2>::type;
    constexpr int VW = 16 / sizeof(T);  // elements per 16-byte load
    constexpr unsigned FULL = 0xffffffffu;

    // per warp, in `slots` (kChunkWarps x kSlotBytes<T> bytes of shared memory): the chunk's
    // fixed-point squares, then (in place) its ties in element order
    __shared__ Fix s_lane_ex[kChunkWarps][ROWS][32];  // per (row, lane): the XOR of its Q words

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t chunk = cta * kChunkWarps + warp;
    if (chunk >= chunks) return;  // the whole warp: nothing below synchronises beyond it
    const uint64_t chunk0 = chunk * Tr::CHUNK;
    if (lane == 0) {
        // the chunk that will run `ahead` chunks later (one wave of resident warps): its operands
        // come from L2 instead of HBM when it starts
        const uint64_t next = chunk0 + ahead * Tr::CHUNK;
        if (vec && ahead && next < n) {
            const unsigned bytes = (unsigned)(min((uint64_t)Tr::CHUNK, n - next) * sizeof(T)) & ~15u;
            if (bytes) {
                prefetch_l2(prediction + next, bytes);
                prefetch_l2(target + next, bytes);
            }
        }
    }

    // ---- squares.  A lane is suspect when one of its squares is non-finite (an invalid operand
    // or an overflow in either step) or, unless the policy allows gradual underflow, one of its
    // differences is nonzero and below 2^-62 / 2^-510 (only such a difference can square to <=
    // the smallest normal, and a subnormal difference is one of them).  Suspect lanes redo their
    // elements with the checked law, in order, and stop at their first fault (their later events
    // cannot win).
    Fix qf[EPT];  // q's bits first, its fixed-point form later; qf[row * V + e]
    B qmax_t = 0, dmin = ~(B)0;  // the lane's largest square (bits), smallest nonzero |d| (below)
    const uint64_t t0 = chunk0 + CM::index(0, lane, 0);  // this lane's first element
    if (vec && chunk0 + Tr::CHUNK <= n) {  // whole chunk in range, 16-byte aligned operands
        const T *pp = prediction + t0;
        const T *tp = target + t0;
#pragma unroll
        for (int r = 0; r < ROWS; ++r)
#pragma unroll
            for (int v = 0; v < V / VW; ++v) {
                const VT a = __ldcs(reinterpret_cast<const VT *>(pp + r * 32 * V + v * VW));
                const VT b = __ldcs(reinterpret_cast<const VT *>(tp + r * 32 * V + v * VW));
#pragma unroll
                for (int e = 0; e < VW; ++e) {
                    const T d = F::sub(reinterpret_cast<const T *>(&a)[e], reinterpret_cast<const T *>(&b)[e]);
                    const B qb = F::bits(F::mul(d, d));
                    qmax_t = qb > qmax_t ? qb : qmax_t;
                    const B dd = F::bits(d) * 2 - 1;  // |d| doubled minus one: +-0 becomes all ones
                    dmin = dd < dmin ? dd : dmin;
                    qf[r * V + v * VW + e] = (Fix)qb;
                }
            }
    } else {
#pragma unroll
        for (int r = 0; r < ROWS; ++r)
#pragma unroll
            for (int e = 0; e < V; ++e) {
                const uint64_t i = t0 + r * 32 * V + e;
                const T d = i < n ? F::sub(prediction[i], target[i]) : T(0);
                const B qb = F::bits(F::mul(d, d));
                qmax_t = qb > qmax_t ? qb : qmax_t;
                const B dd = F::bits(d) * 2 - 1;
                dmin = dd < dmin ? dd : dmin;
                qf[r * V + e] = (Fix)qb;
            }
    }
    unsigned my_fault = 0xffffffffu;
    if (qmax_t >= F::kExpMask || (policy != kPolicyGradual && dmin < kTinyDiff * 2 - 1)) {
        // rare: reload and redo this lane's elements with the checked law
        bool stopped = false;
#pragma unroll 1
        for (int r = 0; r < ROWS; ++r)
#pragma unroll 1
            for (int e = 0; e < V; ++e) {
                const int c = CM::index(r, lane, e);
                const uint64_t i = chunk0 + c;
                T q = T(0);
                if (!stopped && i < n && !checked_square<T>(prediction[i], target[i], base + i, policy, status, q)) {
                    my_fault = (unsigned)c;
                    stopped = true;
                }
                if (i < n) set_at(qf, r * V + e, stopped ? (Fix)0 : (Fix)F::bits(q));
            }
        qmax_t = 0;
#pragma unroll
        for (int e = 0; e < EPT; ++e) qmax_t = (B)qf[e] > qmax_t ? (B)qf[e] : qmax_t;
    }
    const unsigned chunk_fault = __reduce_min_sync(FULL, my_fault);
    const B qmax = warp_max_bits<T>(qmax_t);

    MseHead head;
    head.pad = 0;
    head.fault = chunk_fault;
    head.flags = chunk_fault != 0xffffffffu ? kHeadFault : 0;
    head.k_lo = 0;
    if (qmax == 0) {  // every square is +0 (or faulted): the identity at every binade
        if (lane == 0) {
            head.flags |= kHeadZero;
            heads[chunk] = head;
        }
        return;
    }
    const int k_hi = exponent_of<T>(qmax) + 1;  // every square is below 2^k_hi
    const int k_lo = max(k_hi - (W - 1), Tr::KMIN);
    const int L0 = k_lo - 1;  // fixed-point unit 2^L0
    const int C = F::kBias + F::kFrac + 3 + L0;
    const Fix K = (Fix)(1 - C) * ((Fix)1 << (F::kFrac + 3));
    head.k_lo = k_lo;

    // ---- fixed point Q = floor(q / 2^L0) < 2^W, carried as the bits of 2^P + Q (MARK | Q), with a
    // sticky flag in the (otherwise clear) sign bit when q has bits below 2^L0.  While
    // 2^-L0 is a normal number, q * 2^-L0 is exact and the round-toward-zero add of 2^P floors it,
    // both on the FP pipe; otherwise the integer form (rare; rolled, through the shared-memory
    // slot, to keep the kernel's code small).  Per row: the XOR of the words.  The words also go
    // to this warp's shared-memory slot, where the tie pass reads them.
    constexpr Fix MARK = sizeof(T) == 4 ? (Fix)0x4b000000u : (Fix)0x4330000000000000ull;  // bits of 2^P
    constexpr Fix LOW = ((Fix)1 << W) - 1;
    constexpr Fix STICKY = (Fix)1 << (sizeof(Fix) * 8 - 1);  // the sign bit: set when q has bits below 2^L0
    Fix X[ROWS];
    Fix *qs = reinterpret_cast<Fix *>(slots + (size_t)warp * kSlotBytes<T>);
    if (L0 >= -F::kBias) {
        const T scale = F::value((B)(F::kBias - L0) << F::kFrac);  // 2^-L0
        const T magic = F::value((B)MARK);                         // 2^P
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
            X[r] = 0;
#pragma unroll
            for (int e = 0; e < V; ++e) {
                const T qs_ = F::mul(F::value((B)qf[r * V + e]), scale);  // q / 2^L0, exact
                const T t = add_rz(qs_, magic);                          // 2^P + floor(q / 2^L0)
                // floor(q / 2^L0) - q / 2^L0, exact: +0 when nothing of q lies below 2^L0, negative
                // otherwise, so its sign bit is the sticky flag (FP pipe, no compare or select)
                const T frac = F::sub(F::sub(t, magic), qs_);
                const Fix tb = (Fix)F::bits(t) | ((Fix)F::bits(frac) & STICKY);
                qf[r * V + e] = tb;
                X[r] ^= tb;
            }
        }
    } else {  // rare (squares far below 1): the integer form, one element at a time through the slot
#pragma unroll
        for (int r = 0; r < ROWS; ++r)
#pragma unroll
            for (int v = 0; v < (int)(V * sizeof(Fix) / 16); ++v)
                reinterpret_cast<uint4 *>(qs + CM::index(r, lane, 0))[v] = reinterpret_cast<const uint4 *>(&qf[r * V])[v];
#pragma unroll 1
        for (int r = 0; r < ROWS; ++r) {
            Fix x = 0;
#pragma unroll 1
            for (int e = 0; e < V; ++e) {
                Fix *slot = qs + CM::index(r, lane, 0) + e;
                int dn;
                Fix mm;
                const Fix Q = fixed_point<T>(*slot, C, K, dn, mm);
                const bool exact = dn >= (int)(sizeof(Fix) * 8) ? mm == 0 : (mm & (((Fix)1 << dn) - 1)) == 0;
                const Fix tb = Q | MARK | (exact ? (Fix)0 : STICKY);
                *slot = tb;
                x ^= tb;
            }
            set_at(X, r, x);
        }
#pragma unroll
        for (int r = 0; r < ROWS; ++r)
#pragma unroll
            for (int v = 0; v < (int)(V * sizeof(Fix) / 16); ++v)
                reinterpret_cast<uint4 *>(&qf[r * V])[v] = reinterpret_cast<const uint4 *>(qs + CM::index(r, lane, 0))[v];
    }
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
        for (int v = 0; v < (int)(V * sizeof(Fix) / 16); ++v)
            reinterpret_cast<uint4 *>(qs + CM::index(r, lane, 0))[v] = reinterpret_cast<const uint4 *>(&qf[r * V])[v];
    // ---- the XOR of each row's Q words per lane: the prefix XOR of R = Q ^ (Q << 1) that the tie
    // listing needs is formed from it only for rows that hold a tie (XOR is linear: R of a XOR is
    // the XOR of the Rs)
#pragma unroll
    for (int r = 0; r < ROWS; ++r) s_lane_ex[warp][r][lane] = X[r] & LOW;
    // ---- per-bit population counts of the chunk: Harley-Seal vertical counters per lane, then
    // a warp bit-transpose per counter plane leaves the count of bit 32 w + b in lane b, word w
    uint64_t cnt[NW];
    {
        Fix acc[LOG_EPT + 1];
#pragma unroll
        for (int i = 0; i <= LOG_EPT; ++i) acc[i] = 0;
        acc[LOG_EPT] = SealTree<LOG_EPT, 0>::run(qf, acc);
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            unsigned c = 0;
#pragma unroll
            for (int pl = 0; pl <= LOG_EPT; ++pl)
                c += (unsigned)__popc(warp_transpose32((unsigned)(acc[pl] >> (32 * w)), lane)) << pl;
            cnt[w] = 32 * w + lane < W ? c : 0;
        }
    }
    // ---- S_b = sum over bits b' >= b of cnt[b'] 2^(b'-b) (saturated) for b = 32 w + lane: a
    // suffix scan over the lanes per word, the upper word's total carried into the lower one.
    // W_j = S_j.  jmin: the lowest j from which on every half-up sum W_j + cnt[j-1] is below 2^P
    // (a state in a normal binade is at least 2^P ulps, so a larger sum always leaves it); the
    // sums only grow as j falls, so the failing j form a prefix.
    uint64_t S[NW];
    if constexpr (NW == 1) {
        // one word (binary32): a 32-bit scan saturated at 2^30, far above the 2^P that decides
        // usability, so no saturated sum is ever taken for a usable one
        constexpr unsigned SAT32 = 1u << 30;
        unsigned s = (unsigned)cnt[0];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned v = __shfl_down_sync(FULL, s, o);
            const unsigned sh = v >= (SAT32 >> o) ? SAT32 : v << o;
            if (lane + o < 32) s = min(s + sh, SAT32);
        }
        S[0] = s >= SAT32 ? Tr::SAT : s;
    } else {
#pragma unroll
        for (int w = NW - 1; w >= 0; --w) {
            uint64_t s = cnt[w];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint64_t v = shfl_down_x(s, o);
                if (lane + o < 32) s = min(s + sat_shl(v, o, Tr::SAT), (uint64_t)Tr::SAT);
            }
            if (w + 1 < NW)
                s = min(s + sat_shl(shfl_x(S[w + 1 < NW ? w + 1 : w], 0), 32 - lane, Tr::SAT), (uint64_t)Tr::SAT);
            S[w] = s;
        }
    }
    uint64_t cprev[NW];  // cnt[b - 1] for b = 32 w + lane
    int fail_max = 0;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        const uint64_t below = shfl_up_x(cnt[w], 1);
        const uint64_t carry = shfl_x(cnt[w > 0 ? w - 1 : 0], 31);
        cprev[w] = lane > 0 ? below : (w > 0 ? carry : 0);
        const int j = 32 * w + lane;
        if (j >= 1 && j <= W && (S[w] >= Tr::SAT || S[w] + cprev[w] >= (1ull << Tr::P))) fail_max = j;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) fail_max = max(fail_max, __shfl_xor_sync(FULL, fail_max, o));
    const int jmin = fail_max + 1;

    // ---- ties at the usable binades: a Q whose lowest set bit is at or above jmin - 1 with
    // nothing of q below 2^L0.  Rare for rounded squares, common for exactly representable
    // ones.  The rows are read back from the slot one at a time (a rolled loop: the kernel is
    // issue bound and its unrolled code no longer fit the instruction cache), and only rows
    // holding a candidate go on to the listing.  The ties are listed
    // in element order, with the parity of the half-up increments in front of each, in place of
    // the Q already read (a row's ties never outnumber its elements).  (A chunk with a
    // Subtract/Multiply fault is never mapped, only resolved up to the fault.)
    unsigned ties = 0;
    Tie *tl = reinterpret_cast<Tie *>(slots + (size_t)warp * kSlotBytes<T>);
    if (!(head.flags & kHeadFault) && jmin <= W) {
        const Fix threshold = (Fix)1 << (jmin - 1), lowmask = threshold - 1;
        // a word (MARK | Q, STICKY when q has bits below 2^L0) can be a tie iff it has neither the
        // sticky flag nor a set bit under 2^(jmin - 1): one AND per element (MARK lies above the
        // mask).  A zero Q passes too; such rare rows are re-checked exactly below.
        const Fix may_mask = STICKY | lowmask;
#pragma unroll 1
        for (int r = 0; r < ROWS; ++r) {
            Fix Q[V];
#pragma unroll
            for (int v = 0; v < (int)(V * sizeof(Fix) / 16); ++v)
                reinterpret_cast<uint4 *>(Q)[v] = reinterpret_cast<const uint4 *>(qs + CM::index(r, lane, 0))[v];
            bool row_may = false;
#pragma unroll
            for (int e = 0; e < V; ++e) row_may |= (Q[e] & may_mask) == 0;
            if (!__any_sync(FULL, row_may)) continue;
            row_may = false;  // the exact test: a nonzero Q, not sticky, lowest set bit >= jmin - 1
#pragma unroll
            for (int e = 0; e < V; ++e) {
                const Fix q = Q[e] & LOW;
                row_may |= q != 0 && (q & lowmask) == 0 && !(Q[e] & STICKY);
            }
            if (!__any_sync(FULL, row_may)) continue;
            // exclusive prefix XOR of R in front of (r, lane): R of every lane's words of the rows
            // before r, then an exclusive scan over the lanes of this row
            Fix earlier = 0;
#pragma unroll 1
            for (int r2 = 0; r2 < r; ++r2) earlier ^= s_lane_ex[warp][r2][lane];
#pragma unroll
            for (int o = 16; o; o >>= 1) earlier ^= shfl_xor_x(earlier, o);
            const Fix xr = s_lane_ex[warp][r][lane];
            const Fix rrow = xr ^ (xr << 1);
            Fix incl = rrow;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const Fix v = shfl_up_x(incl, o);
                if (lane >= o) incl ^= v;
            }
            unsigned mask = 0;   // bit e: element (r, lane, e) is a tie
            uint64_t code = 0;   // byte e: its j (6 bits) and parities (2 bits)
            if (row_may) {
                Fix prefix = (earlier ^ (earlier << 1)) ^ incl ^ rrow;
#pragma unroll
                for (int e = 0; e < V; ++e) {
                    const Fix q = Q[e] & LOW;
                    if (q != 0 && (q & lowmask) == 0 && !(Q[e] & STICKY)) {
                        const int j = sizeof(Fix) == 4 ? __ffs((int)q) : __ffsll((long long)q);  // lowest bit + 1
                        mask |= 1u << e;
                        code |= (uint64_t)(j | (int)((q >> j) & 1) << 6 | (int)((prefix >> j) & 1) << 7) << (8 * e);
                    }
                    prefix ^= q ^ (q << 1);
                }
            }
            // lanes in order, each lane's elements in order: an exclusive prefix of the counts
            const unsigned here = __popc(mask);
            unsigned before = here;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned v = __shfl_up_sync(FULL, before, o);
                if (lane >= o) before += v;
            }
            const unsigned row_total = __shfl_sync(FULL, before, 31);
            unsigned slot = ties + before - here;  // <= this row's first element: already read
#pragma unroll
            for (int e = 0; e < V; ++e) {
                if (mask >> e & 1) {
                    const unsigned b = (unsigned)(code >> (8 * e)) & 0xffu;
                    Tie t;
                    t.index = (uint16_t)CM::index(r, lane, e);
                    t.j = (uint8_t)(b & 63);
                    t.bits = (uint8_t)(b >> 6);
                    tl[slot++] = t;
                }
            }
            ties += row_total;
            __syncwarp();
        }
    }
    if (lane == 0) heads[chunk] = head;
    // ---- one lane per binade offset j (binade k = k_lo + j - 1): the half-up sum
    // W_j + cnt[j-1] = S_j + cnt[j-1] (both held by lane j - 32 w of word w), then the ties of
    // that binade in element order
#pragma unroll
    for (int w = 0; w < NW; ++w) {
        const int j = 32 * w + lane;
        if (j < 1 || j > W) continue;
        const bool usable = j >= jmin;
        const uint64_t half_up = usable ? S[w] + cprev[w] : Tr::SAT;
        int64_t corr[2] = {0, 0};
        if (usable) {
            for (unsigned i = 0; i < ties; ++i) {
                const Tie t = tl[i];
                if (t.j != j) continue;
#pragma unroll
                for (int p0 = 0; p0 < 2; ++p0) {
                    // state parity in front of the tie: start + half-up prefix + corrections so far
                    const int parity = (p0 + ((t.bits >> 1) & 1) + (int)(corr[p0] & 1)) & 1;
                    // round to even: up iff (state + floor(q/u)) is odd; half-up assumed up
                    if (((parity + (t.bits & 1)) & 1) == 0) corr[p0] -= 1;
                }
            }
        }
        typename Tr::D *d = deltas + ((size_t)chunk * W + (j - 1)) * 2;
        d[0] = usable ? sat_d<T>((uint64_t)((int64_t)half_up + corr[0])) : no_map<T>();
        d[1] = usable ? sat_d<T>((uint64_t)((int64_t)half_up + corr[1])) : no_map<T>();
    }
}

// Which CTAs of a chunk launch carry the SGD node (every kSgdPeriod-th when it rides along), and
// the chunk-CTA number of the others.
// Within every period of P CTAs of a launch that carries SGD, the last S are SGD CTAs.
template <bool RIDE, int P, int S> __device__ __forceinline__ bool sgd_cta(uint64_t b) {
    return RIDE && b % P >= (uint64_t)(P - S);
}
template <bool RIDE, int P, int S> __device__ __forceinline__ uint64_t chunk_cta(uint64_t b) {
    return RIDE ? (b / P) * (P - S) + b % P : b;
}

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((unsigned)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// An SGD CTA's block [s0, s1): like sgd_range over the CTA's threads, but the operands come in
// through cp.async copies into `smem` (kSgdStages stages of kSgdTrip vectors of each operand per
// thread) instead of registers, so twice the bytes are in flight without costing the chunk
// code's register budget.  Each thread reads back only its own copies (cp.async.wait_group makes
// them visible to it), so no barrier is needed; every copy is drained before the thread leaves.
constexpr int kSgdStages = 2;
static_assert(kSgdStages * 2 * kSgdTrip * 32 * kChunkWarps * 16 <= kChunkWarps * 1024 * 4, "SGD stages fit the slots");
template <typename T>
__device__ __forceinline__ void sgd_range_async(const SgdRider<T> &r, uint64_t s0, uint64_t s1, unsigned char *smem) {
    using VT = typename std::conditional<sizeof(T) == 4, float4, double2>::type;
    constexpr int VW = 16 / sizeof(T);
    const unsigned tid = threadIdx.x, nt = blockDim.x;
    if (!r.vec) {
        sgd_range<T>(r, s0, s1, tid, nt);
        return;
    }
    const uint64_t vend = s0 + (s1 - s0) / VW * VW;
    const uint64_t nv = (vend - s0) / VW;
    VT *buf = reinterpret_cast<VT *>(smem);  // [stage][operand][u][thread]
    auto slot = [&](int st, int op, int u) { return buf + ((size_t)(st * 2 + op) * kSgdTrip + u) * nt + tid; };
    const VT *wv = reinterpret_cast<const VT *>(r.weights + s0), *gv = reinterpret_cast<const VT *>(r.gradient + s0);
    const uint64_t step = (uint64_t)nt * kSgdTrip;  // vectors per stage of the CTA
    auto issue = [&](int st, uint64_t j0) {
#pragma unroll
        for (int u = 0; u < kSgdTrip; ++u) {
            const uint64_t j = j0 + (uint64_t)u * nt;
            if (j < nv) {
                cp_async16(slot(st, 0, u), wv + j);
                cp_async16(slot(st, 1, u), gv + j);
            }
        }
        cp_async_commit();  // (an empty group keeps the counting uniform)
    };
#pragma unroll
    for (int st = 0; st < kSgdStages; ++st) issue(st, tid + (uint64_t)st * step);
    bool stopped = false;
    int st = 0;
    for (uint64_t j0 = tid; j0 < nv && !stopped; j0 += step) {
        cp_async_wait<kSgdStages - 1>();  // the oldest stage has landed
#pragma unroll
        for (int u = 0; u < kSgdTrip; ++u) {
            const uint64_t j = j0 + (uint64_t)u * nt;
            if (j >= nv || stopped) break;
            const VT a = *slot(st, 0, u), b = *slot(st, 1, u);
            VT o;
            const bool done = sgd_fast<T, VW>(reinterpret_cast<const T *>(&a), reinterpret_cast<const T *>(&b),
                                              r.rate, r.policy, reinterpret_cast<T *>(&o));
#pragma unroll
            for (int e = 0; e < VW && !done; ++e) {
                unsigned step_k;
                const unsigned kind = checked_sgd<T>(reinterpret_cast<const T *>(&a)[e],
                                                     reinterpret_cast<const T *>(&b)[e], r.rate, r.policy,
                                                     reinterpret_cast<T *>(&o)[e], step_k);
                if (kind) {  // the elements in front of it are still written, as one at a time would
#pragma unroll
                    for (int q = 0; q < e; ++q) r.out[s0 + j * VW + q] = reinterpret_cast<const T *>(&o)[q];
                    record_fault(r.status, (r.base + s0 + j * VW + e) * 2 + step_k, kind);
                    stopped = true;
                    break;
                }
            }
            if (!stopped) __stcs(reinterpret_cast<VT *>(r.out + s0) + j, o);
        }
        if (!stopped) issue(st, j0 + (uint64_t)kSgdStages * step);  // refill this stage
        st ^= 1;
    }
    cp_async_wait<0>();  // nothing may land in shared memory after the thread has gone
    if (stopped) return;
    for (uint64_t i = vend + tid; i < s1; i += nt) {
        T o;
        unsigned step_k;
        const unsigned kind = checked_sgd<T>(r.weights[i], r.gradient[i], r.rate, r.policy, o, step_k);
        if (kind) {
            record_fault(r.status, (r.base + i) * 2 + step_k, kind);
            return;
        }
        r.out[i] = o;
    }
}

// ASYNC: the operands through cp.async (the one-launch kernel: 1.07 -> 1.01 ms for 2^28 F32 MSE +
// SGD); otherwise through registers (measured faster in the three-launch chunk kernel).
template <typename T, int P, int S, bool ASYNC>
__device__ __forceinline__ void sgd_cta_work(uint64_t b, const SgdRider<T> &rider, unsigned char *smem) {
    const uint64_t s0 = ((b / P) * S + (b % P - (P - S))) * rider.per_unit;
    if (s0 >= rider.n) return;
    if (ASYNC)
        sgd_range_async<T>(rider, s0, min(s0 + rider.per_unit, rider.n), smem);
    else
        sgd_range<T, kSgdCtaTrip>(rider, s0, min(s0 + rider.per_unit, rider.n), threadIdx.x, blockDim.x);
}

// Phase 1 of the three-launch form: chunk maps (and the riding SGD CTAs).
template <typename T, bool RIDE>
__global__ void __launch_bounds__(32 * kChunkWarps, MseTraits<T>::MIN_BLOCKS)
mse_chunk_kernel(const T *prediction, const T *target, uint64_t n, uint64_t base, bool vec, int policy,
                 uint64_t chunks, uint64_t ahead, MseHead *heads, typename MseTraits<T>::D *deltas,
                 unsigned long long *status, SgdRider<T> rider, ChainGuard guard) {
    // a skipped stage of a guarded chain touches nothing (the SGD-carrying form is never guarded)
    if constexpr (!RIDE)
        if (!chain_admits(guard)) return;
    __shared__ __align__(16) unsigned char s_slots[kChunkWarps * kSlotBytes<T>];
    if (sgd_cta<RIDE, kSgdPeriod, 1>(blockIdx.x)) {  // an SGD CTA (its own status word)
        sgd_cta_work<T, kSgdPeriod, 1, false>(blockIdx.x, rider, s_slots);
        return;
    }
    chunk_maps<T>(chunk_cta<RIDE, kSgdPeriod, 1>(blockIdx.x), prediction, target, n, base, vec, policy, chunks, ahead,
                  heads, deltas,
                  status, s_slots);
}

// Compose the maps of kFanout consecutive children (chunks or blocks, each spanning `span`
// elements) into one parent map per binade.  The children's heads and increment rows are
// staged in shared memory, kStageMaps at a time, with coalesced loads; then one thread per
// binade folds them in order.
constexpr int kStageMaps = 16;
// One CTA of 256 threads composes parent `group`.  The children are read through L2 (__ldcg): in
// the one-launch form other CTAs wrote them, and they are published by a fence and a counter.
// `s_rows` holds STAGE maps' increment rows; the children are staged STAGE at a time.
template <typename T, int STAGE>
__device__ __forceinline__ void compose_group(const MseHead *heads, const typename MseTraits<T>::D *deltas,
                                              uint64_t children, uint64_t span, uint64_t group, MseHead *pheads,
                                              typename MseTraits<T>::D *pdeltas, typename MseTraits<T>::D *s_rows) {
    using Tr = MseTraits<T>;
    using D = typename Tr::D;
    constexpr int W = Tr::W;
    constexpr int ROW = W * 2;  // increment words per map
    const uint64_t c0 = group * kFanout;
    const int count = (int)(c0 + kFanout < children ? kFanout : children - c0);
    __shared__ MseHead s_heads[kFanout];
    __shared__ int s_khi, s_flags;
    __shared__ unsigned s_fault;
    const int tid = threadIdx.x, lane = tid & 31;
    if (tid < count) {
        const uint4 hv = __ldcg(reinterpret_cast<const uint4 *>(heads + c0 + tid));
        memcpy(&s_heads[tid], &hv, sizeof(MseHead));
    }
    __syncthreads();
    if (tid < 32) {  // parent head: union of the flags, highest window top, earliest fault
        int khi = INT_MIN, flags = kHeadZero;
        unsigned fault = 0xffffffffu;
        for (int c = lane; c < count; c += 32) {
            const MseHead h = s_heads[c];
            if (h.flags & kHeadFault) {
                flags |= kHeadFault;
                fault = min(fault, (unsigned)((uint64_t)c * span + h.fault));
            }
            if (!(h.flags & kHeadZero)) {
                flags &= ~kHeadZero;
                khi = max(khi, h.k_lo + W - 1);
            }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            khi = max(khi, __shfl_xor_sync(0xffffffffu, khi, o));
            fault = min(fault, __shfl_xor_sync(0xffffffffu, fault, o));
            const int f = __shfl_xor_sync(0xffffffffu, flags, o);
            flags = ((flags | f) & ~kHeadZero) | (flags & f & kHeadZero);
        }
        if (lane == 0) {
            s_khi = khi;
            s_flags = flags;
            s_fault = fault;
        }
    }
    __syncthreads();
    const int flags = s_flags;
    MseHead bh;
    bh.pad = 0;
    bh.flags = flags;
    bh.fault = s_fault;
    bh.k_lo = (flags & kHeadZero) ? 0 : max(s_khi - (W - 1), Tr::KMIN);
    if (tid == 0) pheads[group] = bh;
    if (flags & kHeadZero) return;  // uniform across the CTA
    const int k = bh.k_lo + tid;
    uint64_t acc[2] = {0, 0};
    bool valid = !(flags & kHeadFault);
    for (int g = 0; g < count; g += STAGE) {
        const int in_stage = min(STAGE, count - g);
        __syncthreads();  // the previous stage has been consumed
#pragma unroll 4
        for (int i = tid; i < in_stage * ROW; i += 256) s_rows[i] = __ldcg(deltas + (c0 + g) * ROW + i);
        __syncthreads();
        if (tid < W && valid) {
            for (int c = 0; c < in_stage; ++c) {
                const MseHead h = s_heads[g + c];
                if (h.flags & kHeadZero) continue;
                if (k > h.k_lo + W - 1) continue;  // every square of the child is below half an ulp
                if (k < h.k_lo) { valid = false; break; }
                const D d0 = s_rows[c * ROW + (k - h.k_lo) * 2], d1 = s_rows[c * ROW + (k - h.k_lo) * 2 + 1];
                if (d0 == no_map<T>() || d1 == no_map<T>()) { valid = false; break; }
                const uint64_t n0 = acc[0] + ((acc[0] & 1) ? d1 : d0);
                const uint64_t n1 = acc[1] + (((1 + acc[1]) & 1) ? d1 : d0);
                acc[0] = n0;
                acc[1] = n1;
                if (acc[0] >= (2ull << Tr::P) || acc[1] >= (2ull << Tr::P)) { valid = false; break; }  // cannot fit a binade
            }
        }
    }
    if (tid < W) {
        D *out = pdeltas + ((size_t)group * W + tid) * 2;
        out[0] = valid ? sat_d<T>(acc[0]) : no_map<T>();
        out[1] = valid ? sat_d<T>(acc[1]) : no_map<T>();
    }
}

// Phase 2 of the three-launch form: one CTA per parent.
template <typename T>
__global__ void __launch_bounds__(256) mse_compose_kernel(const MseHead *heads, const typename MseTraits<T>::D *deltas,
                                                          uint64_t children, uint64_t span, MseHead *pheads,
                                                          typename MseTraits<T>::D *pdeltas, ChainGuard guard) {
    if (!chain_admits(guard)) return;
    __shared__ typename MseTraits<T>::D s_rows[kStageMaps * MseTraits<T>::W * 2];
    compose_group<T, kStageMaps>(heads, deltas, children, span, blockIdx.x, pheads, pdeltas, s_rows);
}

// One map at the binade of the state: x -> x + D[x mod 2].  `ok` is false when the map cannot
// be used there (its window does not reach down to k, its sum does not fit a binade there, or a
// Subtract/Multiply fault lies in it).
struct MapStep {
    uint64_t d0, d1;
    bool ok;
};

template <typename T>
__device__ __forceinline__ MapStep map_at(const MseHead &h, const typename MseTraits<T>::D *row, int k) {
    using Tr = MseTraits<T>;
    MapStep m{0, 0, true};
    if (h.flags & kHeadFault) { m.ok = false; return m; }
    if ((h.flags & kHeadZero) || k > h.k_lo + Tr::W - 1) return m;  // identity: every square < half an ulp
    if (k < h.k_lo) { m.ok = false; return m; }
    const typename Tr::D a = __ldcg(row + (size_t)(k - h.k_lo) * 2), b = __ldcg(row + (size_t)(k - h.k_lo) * 2 + 1);
    if (a == no_map<T>() || b == no_map<T>()) { m.ok = false; return m; }
    m.d0 = a;
    m.d1 = b;
    return m;
}

// A map as the walk composes it: the increments (d0, d1) for an even and an odd state.  A map
// that cannot be used (a fault, a binade outside its window, not published yet, or a thread with
// no map) carries POISON = 2^(P+2) on both parities, and every composition saturates there: a
// chain through it ends above the binade, so no separate flag is needed, and a chain of any
// length stays in 32 bits for binary32.
template <typename T> struct WalkMap {
    using V = typename std::conditional<sizeof(T) == 4, uint32_t, uint64_t>::type;
    static constexpr V POISON = (V)1 << (MseTraits<T>::P + 2);
    V d0, d1;
};

// First l, then r: D[p] = l[p] + r[(p + l[p]) mod 2], saturated at POISON (a valid map is below
// 2^(P+1), so the sum of two is below 2^(P+3)).
template <typename T> __device__ __forceinline__ WalkMap<T> compose_maps(WalkMap<T> l, WalkMap<T> r) {
    using V = typename WalkMap<T>::V;
    const V n0 = l.d0 + ((l.d0 & 1) ? r.d1 : r.d0);
    const V n1 = l.d1 + ((l.d1 & 1) ? r.d0 : r.d1);
    return WalkMap<T>{n0 < WalkMap<T>::POISON ? n0 : WalkMap<T>::POISON,
                      n1 < WalkMap<T>::POISON ? n1 : WalkMap<T>::POISON};
}

static_assert(kLevels == kPlanLevels, "the walk plan's levels");

// Prefix sums of half-up increments inside one binade: 32-bit for binary32 (a state is below
// 2^24 and everything is clamped at 2^30), 64-bit for binary64.
template <typename T> struct WalkAcc;
template <> struct WalkAcc<float> {
    using U = uint32_t;
    static constexpr U SAT = 1u << 30;
};
template <> struct WalkAcc<double> {
    using U = uint64_t;
    static constexpr U SAT = 1ull << 62;
};

template <typename U> __device__ __forceinline__ U sat_add(U a, U b, U sat) {
    const U s = a + b;  // a, b <= sat, so no wrap-around
    return s < sat ? s : sat;
}

// Half-up increment of a square (bits qb) at ulp 2^k, clamped at WalkAcc<T>::SAT, and whether
// it is a tie there (q / 2^k an exact half-integer).
template <typename T>
__device__ __forceinline__ typename WalkAcc<T>::U walk_increment(typename Fmt<T>::Bits qb, int k, bool &tie) {
    using F = Fmt<T>;
    using U = typename WalkAcc<T>::U;
    constexpr U SAT = WalkAcc<T>::SAT;
    constexpr int UB = sizeof(U) * 8;
    const int field = (int)(qb >> F::kFrac);
    const int e1 = field > 1 ? field : 1;
    const U m = (U)(qb - ((typename F::Bits)(e1 - 1) << F::kFrac));  // significand, implicit bit included
    const int sh = e1 - F::kBias - F::kFrac - k;                      // q = m * 2^(k + sh)
    tie = false;
    if (sh >= 0) return (sh >= UB - F::kFrac - 2 || m >= (SAT >> sh)) ? (m ? SAT : (U)0) : m << sh;
    const int d = -sh;
    if (d > F::kFrac + 2) return 0;  // q < 2^(k-1): below half an ulp
    const U half = (U)1 << (d - 1);
    tie = (m & ((half << 1) - 1)) == half;
    return (m + half) >> d;
}

// Readiness of the maps in the one-launch form (strict_mse_onepass_kernel); a null block_ctas
// means the three-launch form, where every map is complete before the walk starts.  The
// counters live in the workspace and are zeroed before each launch.
struct MseSync {
    unsigned *block_ctas;    // per block: chunk CTAs that have published their chunk maps
    unsigned *block_ready;   // per block: its composed map is published
    unsigned *super_blocks;  // per superblock: blocks whose composed map is published
    unsigned *super_ready;   // per superblock: its composed map is published
    unsigned chunks_per_cta; // chunks a publishing CTA covers
};

// Publication primitives of the one-launch form: a counter add that releases everything the CTA
// wrote before it (ordered by a preceding barrier) and acquires what earlier adders released; a
// flag store that releases; a flag load that acquires.
__device__ __forceinline__ unsigned add_acq_rel(unsigned *p, unsigned v) {
    unsigned old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void store_release(unsigned *p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned load_flag(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Chunk CTAs of the one-launch form take several groups of kChunkWarps chunks each (all in one
// block) and publish once: a publication (a fence and a counter round trip) holds the CTA's slot
// for about a microsecond, too long to pay once per group.  With an SGD node riding along, one
// group per CTA keeps the SGD CTAs short and well interleaved.
constexpr int kGroupsPerCta = 4;  // when there are at least kManyWaves waves of such CTAs (else 1)
constexpr int kManyWaves = 6;
#ifndef PCU_MSE_RIDE_GROUPS
#define PCU_MSE_RIDE_GROUPS 1
#endif
constexpr int kRideGroupsPerCta = PCU_MSE_RIDE_GROUPS;  // with an SGD node riding along
#ifndef PCU_MSE_RIDE_PERIOD
#define PCU_MSE_RIDE_PERIOD 4
#endif
#ifndef PCU_MSE_RIDE_SGD
#define PCU_MSE_RIDE_SGD 1
#endif
constexpr int kRidePeriod = PCU_MSE_RIDE_PERIOD, kRideSgd = PCU_MSE_RIDE_SGD;  // S SGD CTAs in every P
static_assert((kFanout / kChunkWarps) % kGroupsPerCta == 0, "a chunk CTA's groups lie in one block");

// publishing chunk CTAs of block b in the one-launch form
__device__ __forceinline__ unsigned block_ctas_onepass(uint64_t chunks, uint64_t b, unsigned per_cta) {
    const uint64_t c = min((uint64_t)kFanout, chunks - b * kFanout);
    return (unsigned)((c + per_cta - 1) / per_cta);
}

// The device-side hand-off of a split reduction's running sum between ranks (one GPU each):
// the walker of rank r > 0 waits (bounded) until rank r - 1 has stored the call's carry into this
// rank's hand-off block (in_flag reaches `epoch`), and the walker of rank r < last stores its own
// into rank r + 1's block (the value, then out_flag = epoch, a system-scope release over
// NVLink).  Both null: a carry from, and to, this device's own memory in stream order.
struct CarryLink {
    const unsigned long long *in_flag;
    unsigned long long *out_flag;
    unsigned long long epoch;
};

__device__ __forceinline__ unsigned long long load_acquire_sys_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void store_release_sys_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// The ordered walk of a segment, one CTA of NT threads; a chunk is resolved with CHUNK / NT
// consecutive elements per thread.  In the one-launch form it runs beside the CTAs that build
// the maps: it reads a map only after its publication flag (a bounded wait at the chunk level;
// a coarser map that is not published yet is passed over for a finer one), and it learns of a
// Subtract/Multiply fault from the faulting chunk's head when it reaches it.
template <typename T, int NT>
__device__ __forceinline__ void mse_walk(
    const T *prediction, const T *target, uint64_t n, const MseHead *heads0, const typename MseTraits<T>::D *deltas0,
    const MseHead *heads1, const typename MseTraits<T>::D *deltas1, const MseHead *heads2,
    const typename MseTraits<T>::D *deltas2, uint64_t chunks, uint64_t blocks, uint64_t supers, uint64_t base,
    uint64_t total, T denominator, int policy, const T *carry_in, T *carry_out, T *out, unsigned long long *status,
    const MseSync &sync, const CarryLink &link) {
    using Tr = MseTraits<T>;
    using F = Fmt<T>;
    using U = typename WalkAcc<T>::U;
    constexpr U SAT = WalkAcc<T>::SAT;
    constexpr int E = Tr::CHUNK / NT, WARPS = NT / 32;
    static_assert(E * NT == Tr::CHUNK && WARPS * 32 == NT, "walker shape");
    constexpr U TOP = (U)2 << Tr::P;  // a state at or above this has left its binade
    constexpr unsigned FULL = 0xffffffffu;
    __shared__ typename F::Bits sq[Tr::CHUNK];
    __shared__ T s_sum;
    __shared__ uint64_t s_g;    // elements [0, s_g) of the segment are summed into s_sum
    __shared__ uint64_t s_arg;  // chunk to resolve, or ~0 when the walk is done
    __shared__ uint64_t s_end;  // the walk stops in front of this element (the first Subtract/Multiply fault)
    __shared__ int s_done;      // 2: overflow recorded, 3: a wait gave up
    __shared__ unsigned s_stop[2];
    __shared__ U s_warp_sum[32];
    __shared__ U s_front[Tr::CHUNK];  // the state in front of each element of the chunk resolved
    __shared__ U s_after;             // the state after all of them

    // The walk stops in front of the earliest Subtract/Multiply fault, so only earlier Adds can
    // still report (their events are smaller).  The segment holds global elements
    // [base, base + n); a fault already recorded in front of it stops it at once.
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        s_done = 0;
        if (link.in_flag) {  // the previous rank's running sum, over NVLink (bounded wait)
            const unsigned long long t0 = global_ns();
            while (load_acquire_sys_u64(link.in_flag) < link.epoch) {
                if (global_ns() - t0 > kPeerWaitLimitNs) {
                    record_fault(status, 0, kWatchdog);
                    s_done = 3;
                    break;
                }
                __nanosleep(512);
            }
        }
        const unsigned long long st0 = read_status(status);
        uint64_t stop = s_done == 3 ? 0 : n;
        if (st0 != kStatusOk && (st0 & 7) != kWatchdog) {
            const uint64_t first = (st0 >> 3) / 3;
            stop = first < base ? 0 : (first - base < n ? first - base : n);
        }
        s_end = stop;
        s_sum = carry_in ? *(volatile const T *)carry_in : T(0);
        s_g = 0;
    }
    if (tid < 32) s_warp_sum[tid] = 0;
    __syncthreads();
    const bool onepass = sync.block_ctas != nullptr;
    using WM = WalkMap<T>;
    using V = typename WM::V;
    __shared__ WalkPlan s_plan;
    __shared__ uint64_t s_fail_c;  // the map at this chunk position failed at level s_fail_level:
    __shared__ int s_fail_level;   // the next round goes down to its children
    __shared__ V s_wmap[WARPS][2];
    __shared__ unsigned s_wbad[WARPS];
    __shared__ int s_cut_late, s_cut_level;
    __shared__ MseHead s_cut_head;  // the head of the map at the cut, when it was loaded
    __shared__ uint64_t s_known_c;  // the chunk to resolve whose head a round loaded (after its flag)
    __shared__ MseHead s_known_head;
    if (tid == 0) {
        s_fail_c = ~0ull;
        s_fail_level = kLevels;
        s_known_c = ~0ull;
    }
    // one-launch form: wait (bounded) until the chunk maps of block b are published
    auto wait_block = [&](uint64_t b) {
        const unsigned need = block_ctas_onepass(chunks, b, sync.chunks_per_cta);
        const unsigned long long t0 = global_ns();
        while (load_flag(sync.block_ctas + b) < need) {
            if (global_ns() - t0 > kWaitLimitNs) return false;
            __nanosleep(256);
        }
        return true;
    };
    for (;;) {
        // ---- thread 0: the next round's maps, or the chunk to resolve element by element
        if (tid == 0) {
            uint64_t arg = ~0ull;
            s_plan.runs = 0;
            s_plan.start[0] = 0;
            const uint64_t g = s_g, stop = s_end;
            if (s_done == 0 && g < stop) {
                const uint64_t c = g / Tr::CHUNK;
                if (c == s_fail_c && s_fail_level == 0) {
                    arg = c;
                } else {
                    const uint64_t lim[kLevels] = {stop == n ? chunks : stop / Tr::CHUNK,
                                                   stop == n ? blocks : stop / ((uint64_t)Tr::CHUNK << 6),
                                                   stop == n ? supers : stop / ((uint64_t)Tr::CHUNK << 12)};
                    plan_walk_round(c, lim, s_fail_c, s_fail_level, NT, s_plan);
                    if (!s_plan.runs) arg = c;  // the stop lies inside this chunk
                }
                // its head: from the round that found its map unusable, or read here (in the
                // one-launch form after its publication)
                const bool known = arg != ~0ull && arg == s_known_c;
                if (arg != ~0ull && !known && onepass && !wait_block(arg / kFanout)) {
                    record_fault(status, 0, kWatchdog);
                    s_done = 3;
                    arg = ~0ull;
                }
                if (arg != ~0ull) {  // a fault in the chunk to resolve ends the walk there
                    MseHead h = s_known_head;
                    if (!known) {
                        const uint4 hv = __ldcg(reinterpret_cast<const uint4 *>(heads0 + arg));
                        memcpy(&h, &hv, sizeof(h));
                    }
                    if (h.flags & kHeadFault) s_end = min(s_end, arg * Tr::CHUNK + h.fault);
                }
            }
            s_arg = arg;
        }
        __syncthreads();
        if (s_arg == ~0ull && !s_plan.runs) break;  // the walk is done (or a wait gave up)
        if (s_arg == ~0ull) {
            // ---- a round of maps: thread j loads map j of the plan at the state's binade (in the
            // one-launch form only a published one), a CTA-wide inclusive scan composes them in
            // walk order, and the leading maps whose state stays below 2^(P+1) are applied
            uint64_t x;
            int k;
            state_of<T>(s_sum, x, k);
            const unsigned count = s_plan.start[s_plan.runs];
            int l = 0;
            uint64_t idx = 0;
            bool late = false;
            MseHead h{};
            WM m{WM::POISON, WM::POISON};
            if ((unsigned)tid < count) {
                int e = 0;
                while (e + 1 < s_plan.runs && s_plan.start[e + 1] <= (unsigned)tid) ++e;
                l = s_plan.level[e];
                idx = s_plan.first[e] + (tid - s_plan.start[e]);
                if (onepass)  // the flag's acquire orders this thread's map loads below
                    late = !(l == 0   ? load_flag(sync.block_ctas + idx / kFanout) >=
                                          block_ctas_onepass(chunks, idx / kFanout, sync.chunks_per_cta)
                             : l == 1 ? load_flag(sync.block_ready + idx) != 0
                                      : load_flag(sync.super_ready + idx) != 0);
                if (!late) {  // through L2: in the one-launch form other CTAs wrote the maps
                    const MseHead *heads = l == 0 ? heads0 : l == 1 ? heads1 : heads2;
                    const typename Tr::D *deltas = l == 0 ? deltas0 : l == 1 ? deltas1 : deltas2;
                    const uint4 hv = __ldcg(reinterpret_cast<const uint4 *>(heads + idx));
                    memcpy(&h, &hv, sizeof(h));
                    const MapStep ms = map_at<T>(h, deltas + idx * (size_t)Tr::W * 2, k);
                    if (ms.ok) m = WM{(V)ms.d0, (V)ms.d1};
                }
            }
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const WM left{shfl_up_x(m.d0, o), shfl_up_x(m.d1, o)};
                if (lane >= o) m = compose_maps<T>(left, m);
            }
            if (lane == 31) {
                s_wmap[warp][0] = m.d0;
                s_wmap[warp][1] = m.d1;
            }
            __syncthreads();
            if (warp) {
                WM front{s_wmap[0][0], s_wmap[0][1]};
                for (int w = 1; w < warp; ++w) front = compose_maps<T>(front, WM{s_wmap[w][0], s_wmap[w][1]});
                m = compose_maps<T>(front, m);
            }
            const uint64_t nx = x + ((x & 1) ? m.d1 : m.d0);
            const bool good = (unsigned)tid < count && nx < TOP;  // the state only grows
            const unsigned bad = __ballot_sync(FULL, !good);
            if (lane == 0) s_wbad[warp] = bad ? (unsigned)(warp * 32 + __ffs((int)bad) - 1) : (unsigned)NT;
            __syncthreads();
            unsigned cut = NT;
#pragma unroll
            for (int w = 0; w < WARPS; ++w) cut = min(cut, s_wbad[w]);
            if (cut && (unsigned)tid == cut - 1) {
                s_sum = value_of<T>(nx, k);
                s_g = min((idx + 1) * ((uint64_t)Tr::CHUNK << (6 * l)), n);
            }
            if ((unsigned)tid == cut && cut < count) {
                s_cut_late = late;
                s_cut_level = l;
                s_cut_head = h;
            }
            __syncthreads();
            if (tid == 0 && cut < count) {
                // the map at the cut leaves the binade or cannot be used: its children next (a
                // chunk's is resolved element by element); not published yet: go on from there,
                // with its children if it is the first (a finer level may be published already),
                // or after waiting for a chunk's
                const uint64_t c = s_g / Tr::CHUNK;
                if (!s_cut_late || (cut == 0 && s_cut_level > 0)) {
                    s_fail_c = c;
                    s_fail_level = s_cut_level;
                    if (!s_cut_late && s_cut_level == 0) {
                        s_known_c = c;
                        s_known_head = s_cut_head;
                    }
                } else if (cut == 0 && !wait_block(c / kFanout)) {
                    record_fault(status, 0, kWatchdog);
                    s_done = 3;
                }
            }
            continue;  // thread 0 plans the next round; the others wait for it at the barrier
        }

        // ---- resolve one chunk: thread t owns elements [t E, t E + E) (all fault-free in front
        // of the stop)
        const uint64_t stop = s_end;
        const uint64_t i0 = s_arg * Tr::CHUNK;
        const unsigned len = (unsigned)((i0 + Tr::CHUNK < stop ? i0 + Tr::CHUNK : stop) - i0);
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const unsigned c = tid + e * NT;
            if (c < len) {
                const T d = F::sub(prediction[i0 + c], target[i0 + c]);
                sq[c] = F::bits(F::mul(d, d));
            }
        }
        if (tid == 0) s_stop[0] = s_stop[1] = len;
        __syncthreads();
        // Apply every element in front of the first tie or binade crossing at once (a prefix sum
        // of half-up increments), then add that element exactly; repeat.  Every thread follows
        // the running sum itself: the states in front of all elements go to shared memory, so
        // after the cut is known each thread computes the same exact step (two barriers a round).
        T cur = s_sum;
        unsigned pos = 0;
        for (int it = 0; pos < len; it ^= 1) {
            uint64_t x64;
            int k;
            state_of<T>(cur, x64, k);
            const U x = (U)x64;  // below 2^(P+1)
            U c[E];              // inclusive prefix of this thread's increments
            bool tie[E];
            U run = 0;
#pragma unroll
            for (int e = 0; e < E; ++e) {
                const unsigned idx = tid * E + e;
                const bool active = idx >= pos && idx < len;
                bool t = false;
                const U inc = active ? walk_increment<T>(sq[idx], k, t) : (U)0;
                tie[e] = active && t;
                run = sat_add<U>(run, inc, SAT);
                c[e] = run;
            }
            // exclusive prefix of the thread totals (element order)
            U incl = run;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const U v = shfl_up_x(incl, o);
                if (lane >= o) incl = sat_add<U>(incl, v, SAT);
            }
            if (lane == 31) s_warp_sum[warp] = incl;
            __syncthreads();
            if (tid == 0) s_stop[it ^ 1] = len;  // armed for the next round (its last readers are past)
            U wsum = lane < WARPS ? s_warp_sum[lane] : (U)0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const U v = shfl_up_x(wsum, o);
                if (lane >= o) wsum = sat_add<U>(wsum, v, SAT);
            }
            const U warp_before = warp ? shfl_x(wsum, warp - 1) : (U)0;
            U before = shfl_up_x(incl, 1);
            if (lane == 0) before = 0;
            before = sat_add<U>(before, warp_before, SAT);
            const U start = sat_add<U>(x, before, SAT);  // the state in front of this thread's elements
            // the first element that reaches TOP, or the first tie, stops the run
            unsigned mine = len;
#pragma unroll
            for (int e = E - 1; e >= 0; --e) {
                const unsigned idx = tid * E + e;
                s_front[idx] = e ? sat_add<U>(start, c[e - 1], SAT) : start;
                if (idx >= pos && idx < len && (tie[e] || sat_add<U>(start, c[e], SAT) >= TOP)) mine = idx;
            }
            if (tid == NT - 1) s_after = sat_add<U>(start, run, SAT);
            if (mine < len) atomicMin(&s_stop[it], mine);
            __syncthreads();
            const unsigned cut = s_stop[it];
            // below TOP: nothing in front of `cut` left the binade
            const T sv = value_of<T>((uint64_t)(cut < len ? s_front[cut] : s_after), k);
            if (cut < len) {
                const T t = F::add(sv, F::value(sq[cut]));
                if (nonfinite_bits<T>(F::bits(t))) {
                    if (tid == 0) {
                        record_fault(status, (base + i0 + cut) * 3 + 2, kOverflow);
                        s_done = 2;
                    }
                    pos = len;
                } else {
                    cur = t;
                    pos = cut + 1;
                }
            } else {
                cur = sv;
                pos = len;
            }
        }
        if (tid == 0) s_sum = cur;
        if (tid == 0) s_g = s_done == 2 ? stop : i0 + len;
        __syncthreads();
        if (s_done == 2) break;
    }
    if (tid == 0) {
        if (s_done != 3 && carry_out) *carry_out = s_sum;  // the running sum handed to the next segment
        if (link.out_flag)  // published even after a give-up: the next rank must not wait for it; the
            // release orders this thread's store of the sum before the flag
            store_release_sys_u64(link.out_flag, link.epoch);
        if (s_done == 3) return;  // a wait gave up: the status word says so
        if (!out || s_done == 2 || s_end < n || fault_precedes(status, total * 3)) return;
        T mean;
        const unsigned kind = checked_div<T>(s_sum, denominator, policy, mean);
        if (kind) {
            record_fault(status, total * 3, kind);
            return;
        }
        out[0] = mean;
    }
}

#define PCU_MSE_WALK_PARAMS                                                                                        \
    const T *prediction, const T *target, uint64_t n, const MseHead *heads0, const typename MseTraits<T>::D *deltas0, \
        const MseHead *heads1, const typename MseTraits<T>::D *deltas1, const MseHead *heads2,                   \
        const typename MseTraits<T>::D *deltas2, uint64_t chunks, uint64_t blocks, uint64_t supers, uint64_t base, \
        uint64_t total, T denominator, int policy, const T *carry_in, T *carry_out, T *out,                       \
        unsigned long long *status
#define PCU_MSE_WALK_ARGS                                                                                     \
    prediction, target, n, heads0, deltas0, heads1, deltas1, heads2, deltas2, chunks, blocks, supers, base, total, \
        denominator, policy, carry_in, carry_out, out, status

constexpr int kWalkThreads = 32 * kChunkWarps;  // the walker's CTA (also a chunk CTA's shape)

template <typename T>
__global__ void __launch_bounds__(kWalkThreads) mse_walk_kernel(PCU_MSE_WALK_PARAMS, ChainGuard guard, CarryLink link) {
    if (chain_admits(guard)) mse_walk<T, kWalkThreads>(PCU_MSE_WALK_ARGS, MseSync{}, link);
}

// CTA 0 walks; the other CTAs stream an SGD node's elements meanwhile (the walker is latency
// bound and holds one SM).
template <typename T>
__global__ void __launch_bounds__(kWalkThreads) mse_walk_sgd_kernel(PCU_MSE_WALK_PARAMS, SgdRider<T> rider,
                                                                      CarryLink link) {
    if (blockIdx.x == 0) {
        mse_walk<T, kWalkThreads>(PCU_MSE_WALK_ARGS, MseSync{}, link);
        return;
    }
    sgd_range<T>(rider, 0, rider.n, (uint64_t)(blockIdx.x - 1) * blockDim.x + threadIdx.x,
                 (uint64_t)(gridDim.x - 1) * blockDim.x);
}

// An SGD share on its own (the part a segment's chunk warps do not carry).
template <typename T> __global__ void __launch_bounds__(256) sgd_share_kernel(SgdRider<T> rider) {
    sgd_range<T>(rider, 0, rider.n, (uint64_t)blockIdx.x * blockDim.x + threadIdx.x, (uint64_t)gridDim.x * blockDim.x);
}

// ---- the one-launch form (binary32): CTA 0 walks while the other CTAs build the chunk maps.
// The last chunk CTA of a block composes the block map, and the last block of a superblock the
// superblock map; each publication is a fence followed by a counter or a flag.  Only CTA 0 ever
// waits (bounded), and only on CTAs that wait for nothing, so the launch always completes: CTA 0
// is dispatched first and holds one slot, and every other CTA runs to completion.  The walk
// trails the chunk CTAs by about a block, so it ends shortly after the last chunk instead of
// running alone for ~0.1 ms after them.
template <typename T, bool RIDE, int G>
__global__ void __launch_bounds__(32 * kChunkWarps, MseTraits<T>::MIN_BLOCKS)
mse_onepass_kernel(const T *prediction, const T *target, uint64_t n, bool vec, int policy, uint64_t chunks,
                   uint64_t blocks, uint64_t supers, uint64_t ahead, MseHead *h0, typename MseTraits<T>::D *d0,
                   MseHead *h1, typename MseTraits<T>::D *d1, MseHead *h2, typename MseTraits<T>::D *d2,
                   MseSync sync, T denominator, T *out, unsigned long long *status, SgdRider<T> rider,
                   ChainGuard guard, uint64_t base, uint64_t total, const T *carry_in, T *carry_out, CarryLink link) {
    using Tr = MseTraits<T>;
    if constexpr (!RIDE)
        if (!chain_admits(guard)) return;  // the whole launch, walker included
    if (blockIdx.x == 0) {
        mse_walk<T, kWalkThreads>(prediction, target, n, h0, d0, h1, d1, h2, d2, chunks, blocks, supers, base, total,
                                  denominator, policy, carry_in, carry_out, out, status, sync, link);
        return;
    }
    // the chunk warps' slots; once the chunks are done, the staging area of a composition (all
    // kFanout children at once); in an SGD CTA, its copy stages
    __shared__ __align__(16) unsigned char s_slots[kChunkWarps * kSlotBytes<T>];
    const uint64_t b = blockIdx.x - 1;
    if (sgd_cta<RIDE, kRidePeriod, kRideSgd>(b)) {
        sgd_cta_work<T, kRidePeriod, kRideSgd, true>(b, rider, s_slots);
        return;
    }
    constexpr uint64_t kPerCta = (uint64_t)kChunkWarps * G;
    const uint64_t cta = chunk_cta<RIDE, kRidePeriod, kRideSgd>(b);
    if (cta * kPerCta >= chunks) return;  // past the last chunk: part of no block
    static_assert(kChunkWarps * kSlotBytes<T> >= (size_t)kFanout * Tr::W * 2 * sizeof(typename Tr::D), "staging");
#pragma unroll 1
    for (int q = 0; q < G; ++q)  // a group prefetches the next one into L2; the last group, the first
        // group of the CTA that takes this slot one wave later (`ahead` chunks on)
        chunk_maps<T>(cta * G + q, prediction, target, n, base, vec, policy, chunks,
                      q + 1 < G ? (uint64_t)kChunkWarps : ahead, h0, d0, status, s_slots);
    // Publish this CTA's chunk maps: the barrier orders every thread's writes before thread 0,
    // whose acquire-release count releases them (cumulatively); the last CTA of a block acquires
    // the others' maps with the same count, and its threads read them after the barrier.
    __shared__ unsigned s_last;
    __syncthreads();
    const uint64_t blk = cta / (kFanout / kPerCta);
    if (threadIdx.x == 0)
        s_last = add_acq_rel(sync.block_ctas + blk, 1u) + 1 == block_ctas_onepass(chunks, blk, (unsigned)kPerCta);
    __syncthreads();
    if (!s_last) return;
    compose_group<T, kFanout>(h0, d0, chunks, Tr::CHUNK, blk, h1, d1, reinterpret_cast<typename Tr::D *>(s_slots));
    __syncthreads();
    const uint64_t sb = blk / kFanout;
    if (threadIdx.x == 0) {
        store_release(sync.block_ready + blk, 1u);
        s_last = add_acq_rel(sync.super_blocks + sb, 1u) + 1 == min((uint64_t)kFanout, blocks - sb * kFanout);
    }
    __syncthreads();
    if (!s_last) return;
    compose_group<T, kFanout>(h1, d1, blocks, (uint64_t)Tr::CHUNK << 6, sb, h2, d2,
                              reinterpret_cast<typename Tr::D *>(s_slots));
    __syncthreads();
    if (threadIdx.x == 0) store_release(sync.super_ready + sb, 1u);
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

// Workspace: per level (chunk, block, superblock) the map heads, then the increment rows.
template <typename T> struct MseLayout {
    uint64_t count[kLevels];
    size_t heads_off[kLevels], deltas_off[kLevels], sync_off, sync_bytes, bytes;
    explicit MseLayout(uint64_t n) {
        using Tr = MseTraits<T>;
        auto up = [](size_t v) { return (v + 255) / 256 * 256; };
        const size_t row = Tr::W * 2 * sizeof(typename Tr::D);
        count[0] = (n + Tr::CHUNK - 1) / Tr::CHUNK;
        for (int l = 1; l < kLevels; ++l) count[l] = (count[l - 1] + kFanout - 1) / kFanout;
        size_t off = 0;
        for (int l = 0; l < kLevels; ++l) {
            heads_off[l] = off;
            off += up(count[l] * sizeof(MseHead));
            deltas_off[l] = off;
            off += up(count[l] * row);
        }
        // the one-launch form's publication counters: per block two words, per superblock two
        sync_off = off;
        sync_bytes = up((2 * count[1] + 2 * count[2]) * sizeof(unsigned));
        off += sync_bytes;
        bytes = off;
    }
};

// The chunk kernel's grid when it carries SGD, and how many units (chunk warps or SGD CTAs)
// carry it.
// (chunks_per_cta: kChunkWarps, or more for the one-launch form without SGD)
inline uint64_t chunk_grid(uint64_t chunks, bool ride, uint64_t chunks_per_cta = kChunkWarps, int P = kSgdPeriod,
                           int S = 1) {
    const uint64_t ctas = (chunks + chunks_per_cta - 1) / chunks_per_cta;
    return ride ? (ctas + (P - S) - 1) / (P - S) * P : ctas;
}
inline uint64_t sgd_units(uint64_t chunks, uint64_t chunks_per_cta = kChunkWarps, int P = kSgdPeriod, int S = 1) {
    return chunk_grid(chunks, true, chunks_per_cta, P, S) / P * S;
}

// Phases 1 and 2 of a segment (global elements [base, base + n)): chunk maps, then block and
// superblock maps.  `sgd` (if not null and not empty) rides on the chunk kernel, per_unit
// elements per SGD CTA.
template <typename T>
int prepare_mse(int policy, const T *p, const T *t, uint64_t n, uint64_t base, void *workspace, size_t workspace_bytes,
                unsigned long long *status, cudaStream_t stream, const SgdRider<T> *sgd = nullptr,
                const ChainGuard &guard = ChainGuard{}) {
    using D = typename MseTraits<T>::D;
    MseLayout<T> lay(n);
    if (!workspace || workspace_bytes < lay.bytes) return PCU_B200_ERROR_WORKSPACE;
    if (lay.count[0] > 0x7fffffffull * kChunkWarps) return PCU_B200_ERROR_SIZE_OVERFLOW;
    if (!n) return PCU_B200_OK;
    const bool ride = sgd && sgd->n;
    char *ws = reinterpret_cast<char *>(workspace);
    const bool vec = pcu_host::aligned(p, 16) && pcu_host::aligned(t, 16);
    static int resident[2][64] = {};  // chunk-kernel warps resident at once, per variant and device
    int device = 0;
    cudaGetDevice(&device);
    const bool cached = device >= 0 && device < 64;
    int ahead = cached ? resident[ride][device] : 0;
    if (!ahead) {
        int per_sm = 0;
        cudaError_t e = ride ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mse_chunk_kernel<T, true>,
                                                                           32 * kChunkWarps, 0)
                             : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mse_chunk_kernel<T, false>,
                                                                           32 * kChunkWarps, 0);
        if (e != cudaSuccess) return pcu_host::set_cuda_error(e);
        ahead = per_sm * kChunkWarps * pcu_host::sm_count();
        if (cached) resident[ride][device] = ahead;
    }
    const unsigned grid = (unsigned)chunk_grid(lay.count[0], ride);
    MseHead *h0 = reinterpret_cast<MseHead *>(ws + lay.heads_off[0]);
    D *d0 = reinterpret_cast<D *>(ws + lay.deltas_off[0]);
    if (ride)
        mse_chunk_kernel<T, true><<<grid, 32 * kChunkWarps, 0, stream>>>(p, t, n, base, vec, policy, lay.count[0],
                                                                         (uint64_t)ahead, h0, d0, status, *sgd, guard);
    else
        mse_chunk_kernel<T, false><<<grid, 32 * kChunkWarps, 0, stream>>>(p, t, n, base, vec, policy, lay.count[0],
                                                                          (uint64_t)ahead, h0, d0, status,
                                                                          SgdRider<T>{}, guard);
    int rc = pcu_host::launch_status();
    for (int l = 1; l < kLevels && !rc; ++l) {
        mse_compose_kernel<T><<<(unsigned)lay.count[l], 256, 0, stream>>>(
            reinterpret_cast<const MseHead *>(ws + lay.heads_off[l - 1]),
            reinterpret_cast<const D *>(ws + lay.deltas_off[l - 1]), lay.count[l - 1],
            (uint64_t)MseTraits<T>::CHUNK << (6 * (l - 1)), reinterpret_cast<MseHead *>(ws + lay.heads_off[l]),
            reinterpret_cast<D *>(ws + lay.deltas_off[l]), chain_follow(guard));
        rc = pcu_host::launch_status();
    }
    return rc;
}

// Phase 3 of a segment: the ordered walk from *carry_in (+0 if null); the running sum goes to
// *carry_out (if not null) and, when out is not null, the checked mean over `total` elements.
// `sgd` (if not null and not empty) is streamed by extra CTAs of the same launch.
template <typename T>
int walk_mse(int policy, const T *p, const T *t, uint64_t n, uint64_t base, uint64_t total, const T *carry_in,
             T *carry_out, T *out, void *workspace, size_t workspace_bytes, unsigned long long *status,
             cudaStream_t stream, const SgdRider<T> *sgd = nullptr, const ChainGuard &guard = ChainGuard{},
             const CarryLink &link = CarryLink{}) {
    using D = typename MseTraits<T>::D;
    constexpr unsigned THREADS = kWalkThreads;
    MseLayout<T> lay(n);
    if (n && (!workspace || workspace_bytes < lay.bytes)) return PCU_B200_ERROR_WORKSPACE;
    char *ws = reinterpret_cast<char *>(workspace);
    auto H = [&](int l) { return reinterpret_cast<const MseHead *>(ws + lay.heads_off[l]); };
    auto R = [&](int l) { return reinterpret_cast<const D *>(ws + lay.deltas_off[l]); };
    if (sgd && sgd->n) {
        const uint64_t per_cta = (uint64_t)THREADS * (16 / sizeof(T)) * kSgdTrip;
        const uint64_t cap = (uint64_t)(2048 / THREADS) * pcu_host::sm_count() - 1;
        const uint64_t want = (sgd->n + per_cta - 1) / per_cta;
        const unsigned extra = (unsigned)(want < cap ? want : cap);
        mse_walk_sgd_kernel<T><<<1 + extra, THREADS, 0, stream>>>(
            p, t, n, H(0), R(0), H(1), R(1), H(2), R(2), lay.count[0], lay.count[1], lay.count[2], base, total,
            count_value<T>(total), policy, carry_in, carry_out, out, status, *sgd, link);
    } else {
        mse_walk_kernel<T><<<1, THREADS, 0, stream>>>(p, t, n, H(0), R(0), H(1), R(1), H(2), R(2), lay.count[0],
                                                      lay.count[1], lay.count[2], base, total, count_value<T>(total),
                                                      policy, carry_in, carry_out, out, status, guard, link);
    }
    return pcu_host::launch_status();
}

// The one-launch form of a whole reduction (binary32): the publication counters are zeroed, then
// one launch builds the maps and walks them.  `sgd` (if not null and not empty) rides along.
template <typename T>
int onepass_mse(int policy, const T *p, const T *t, T *out, uint64_t n, void *workspace, size_t workspace_bytes,
                unsigned long long *status, cudaStream_t stream, const SgdRider<T> *sgd, const ChainGuard &guard,
                uint64_t base = 0, uint64_t total = 0, const T *carry_in = nullptr, T *carry_out = nullptr,
                const CarryLink &link = CarryLink{}) {
    if (!total) total = n;  // a whole reduction unless a segment [base, base + n) of `total`
    MseLayout<T> lay(n);
    if (!workspace || workspace_bytes < lay.bytes) return PCU_B200_ERROR_WORKSPACE;
    if (lay.count[0] > 0x7fffffffull * kChunkWarps) return PCU_B200_ERROR_SIZE_OVERFLOW;
    const bool ride = sgd && sgd->n;
    char *ws = reinterpret_cast<char *>(workspace);
    cudaError_t e = cudaMemsetAsync(ws + lay.sync_off, 0, lay.sync_bytes, stream);
    if (e != cudaSuccess) return pcu_host::set_cuda_error(e);
    const bool vec = pcu_host::aligned(p, 16) && pcu_host::aligned(t, 16);
    static int resident[64] = {};  // CTAs of the one-launch kernel resident at once, per device
    int device = 0;
    cudaGetDevice(&device);
    const bool cached = device >= 0 && device < 64;
    int slots = cached ? resident[device] : 0;
    if (!slots) {  // every variant has the same footprint: 64 registers and the same shared memory
        int per_sm = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, mse_onepass_kernel<T, false, kGroupsPerCta>,
                                                          kWalkThreads, 0);
        if (e != cudaSuccess) return pcu_host::set_cuda_error(e);
        slots = std::max(2, per_sm * pcu_host::sm_count());
        if (cached) resident[device] = slots;
    }
    // chunk CTAs resident at once (the walker holds one slot; SGD CTAs hold S in every P)
    int64_t ctas = slots - 1;
    if (ride) ctas = ctas * (kRidePeriod - kRideSgd) / kRidePeriod;
    // several groups per chunk CTA only when there are enough waves of them (the last wave runs
    // partly empty), never with an SGD node riding along
    const int g = ride ? kRideGroupsPerCta
                       : (lay.count[0] >= (uint64_t)kManyWaves * ctas * kChunkWarps * kGroupsPerCta ? kGroupsPerCta : 1);
    // the first group of the CTA that takes this slot one wave later
    const uint64_t ahead = (uint64_t)std::max<int64_t>(1, ctas * g * kChunkWarps - (int64_t)(g - 1) * kChunkWarps);
    using D = typename MseTraits<T>::D;
    auto H = [&](int l) { return reinterpret_cast<MseHead *>(ws + lay.heads_off[l]); };
    auto R = [&](int l) { return reinterpret_cast<D *>(ws + lay.deltas_off[l]); };
    unsigned *u = reinterpret_cast<unsigned *>(ws + lay.sync_off);
    const unsigned per_cta = kChunkWarps * g;
    MseSync sync{u, u + lay.count[1], u + 2 * lay.count[1], u + 2 * lay.count[1] + lay.count[2], per_cta};
    const unsigned grid = (unsigned)(1 + chunk_grid(lay.count[0], ride, per_cta, kRidePeriod, kRideSgd));
    if (ride)
        mse_onepass_kernel<T, true, kRideGroupsPerCta><<<grid, kWalkThreads, 0, stream>>>(
            p, t, n, vec, policy, lay.count[0], lay.count[1], lay.count[2], ahead, H(0), R(0), H(1), R(1), H(2), R(2),
            sync, count_value<T>(total), out, status, *sgd, guard, base, total, carry_in, carry_out, link);
    else if (g == kGroupsPerCta)
        mse_onepass_kernel<T, false, kGroupsPerCta><<<grid, kWalkThreads, 0, stream>>>(
            p, t, n, vec, policy, lay.count[0], lay.count[1], lay.count[2], ahead, H(0), R(0), H(1), R(1), H(2), R(2),
            sync, count_value<T>(total), out, status, SgdRider<T>{}, guard, base, total, carry_in, carry_out,
            link);
    else
        mse_onepass_kernel<T, false, 1><<<grid, kWalkThreads, 0, stream>>>(
            p, t, n, vec, policy, lay.count[0], lay.count[1], lay.count[2], ahead, H(0), R(0), H(1), R(1), H(2), R(2),
            sync, count_value<T>(total), out, status, SgdRider<T>{}, guard, base, total, carry_in, carry_out,
            link);
    return pcu_host::launch_status();
}

template <typename T>
int run_mse(int policy, const T *p, const T *t, T *out, uint64_t n, void *workspace, size_t workspace_bytes,
            unsigned long long *status, cudaStream_t stream, const ChainGuard &guard) {
    if constexpr (sizeof(T) == 4) {
        return onepass_mse<T>(policy, p, t, out, n, workspace, workspace_bytes, status, stream, nullptr, guard);
    } else {  // binary64: three launches (its chunk maps and composition stage do not fit one CTA's memory)
        int rc = prepare_mse<T>(policy, p, t, n, 0, workspace, workspace_bytes, status, stream, nullptr, guard);
        if (rc) return rc;
        return walk_mse<T>(policy, p, t, n, 0, n, nullptr, nullptr, out, workspace, workspace_bytes, status, stream,
                           nullptr, chain_follow(guard));
    }
}

// ---- MSE + SGD in one pass.  The SGD node's elements go to the chunk kernel's SGD CTAs, up to
// kMaxSgdPerCta each; what is left (an SGD node far larger than the MSE) is streamed by extra
// CTAs of the walker's launch.
constexpr uint64_t kMaxSgdPerCta = 131072;

template <typename T>
SgdRider<T> make_rider(int policy, const void *weights, const void *gradient, void *out, uint64_t n, uint64_t base,
                       uint32_t rate_bits, unsigned long long *status) {
    SgdRider<T> r{};
    r.weights = reinterpret_cast<const T *>(weights);
    r.gradient = reinterpret_cast<const T *>(gradient);
    r.out = reinterpret_cast<T *>(out);
    r.n = n;
    r.base = base;
    r.per_unit = 0;
    if constexpr (sizeof(T) == 4)
        r.rate = pcu_host::rate_f32(rate_bits);
    else
        r.rate = pcu_host::rate_f64(rate_bits);
    r.policy = policy;
    r.vec = pcu_host::aligned(weights, 16) && pcu_host::aligned(gradient, 16) && pcu_host::aligned(out, 16);
    r.status = status;
    return r;
}

// head: elements [0, h) carried by `units` SGD CTAs of the chunk kernel; tail: the rest
template <typename T>
void split_sgd(const SgdRider<T> &all, uint64_t units, SgdRider<T> &head, SgdRider<T> &tail) {
    uint64_t per = units ? (all.n + units - 1) / units : 0;
    per = (per + sgd_unit<T>() - 1) / sgd_unit<T>() * sgd_unit<T>();
    if (per > kMaxSgdPerCta) per = kMaxSgdPerCta;
    const uint64_t h = per * units < all.n ? per * units : all.n;
    head = all;
    head.n = h;
    head.per_unit = per;
    tail = all;
    tail.weights += h;
    tail.gradient += h;
    tail.out += h;
    tail.n = all.n - h;
    tail.base = all.base + h;
}

template <typename T>
int run_mse_sgd(int policy, const T *p, const T *t, T *loss, uint64_t n, void *workspace, size_t workspace_bytes,
                unsigned long long *mse_status, const SgdRider<T> &sgd, cudaStream_t stream) {
    MseLayout<T> lay(n);
    SgdRider<T> head, tail;
    split_sgd<T>(sgd,
                 sizeof(T) == 4 ? sgd_units(lay.count[0], kChunkWarps * kRideGroupsPerCta, kRidePeriod, kRideSgd)
                                : sgd_units(lay.count[0]),
                 head, tail);
    if constexpr (sizeof(T) == 4) {
        int rc = onepass_mse<T>(policy, p, t, loss, n, workspace, workspace_bytes, mse_status, stream, &head,
                                ChainGuard{});
        if (rc || !tail.n) return rc;
        const uint64_t per_cta = 256ull * (16 / sizeof(T)) * kSgdTrip;
        const uint64_t cap = 8ull * pcu_host::sm_count();
        const uint64_t want = (tail.n + per_cta - 1) / per_cta;
        sgd_share_kernel<T><<<(unsigned)(want < cap ? want : cap), 256, 0, stream>>>(tail);
        return pcu_host::launch_status();
    } else {
        int rc = prepare_mse<T>(policy, p, t, n, 0, workspace, workspace_bytes, mse_status, stream, &head);
        if (rc) return rc;
        return walk_mse<T>(policy, p, t, n, 0, n, nullptr, nullptr, loss, workspace, workspace_bytes, mse_status,
                           stream, &tail);
    }
}

// A segment's phases 1 and 2 with an SGD share on the chunk warps; what they cannot carry runs
// in a launch of its own.
template <typename T>
int prepare_mse_sgd(int policy, const T *p, const T *t, uint64_t n, uint64_t base, void *workspace,
                    size_t workspace_bytes, unsigned long long *mse_status, const SgdRider<T> &sgd,
                    cudaStream_t stream) {
    MseLayout<T> lay(n);
    if (!workspace || workspace_bytes < lay.bytes) return PCU_B200_ERROR_WORKSPACE;
    SgdRider<T> head, tail;
    split_sgd<T>(sgd, n ? sgd_units(lay.count[0]) : 0, head, tail);
    int rc = prepare_mse<T>(policy, p, t, n, base, workspace, workspace_bytes, mse_status, stream, &head);
    if (rc || !tail.n) return rc;
    const uint64_t per_cta = 256ull * (16 / sizeof(T)) * kSgdTrip;
    const uint64_t cap = 8ull * pcu_host::sm_count();
    const uint64_t want = (tail.n + per_cta - 1) / per_cta;
    sgd_share_kernel<T><<<(unsigned)(want < cap ? want : cap), 256, 0, stream>>>(tail);
    return pcu_host::launch_status();
}

}  // namespace pcu

extern "C" size_t pcu_b200_strict_mse_workspace_size(int dtype, uint64_t count) {
    if (dtype == PCU_B200_F64) return pcu::MseLayout<double>(count).bytes;
    return pcu::MseLayout<float>(count).bytes;
}

extern "C" int pcu_b200_strict_mse(int dtype, int policy, const void *prediction, const void *target, void *out,
                                   uint64_t count, void *workspace, size_t workspace_bytes, uint64_t *status,
                                   void *stream) {
    return pcu::strict_mse(dtype, policy, prediction, target, out, count, workspace, workspace_bytes, status, stream,
                           pcu::ChainGuard{});
}

int pcu::strict_mse(int dtype, int policy, const void *prediction, const void *target, void *out, uint64_t count,
                    void *workspace, size_t workspace_bytes, uint64_t *status, void *stream, const ChainGuard &guard) {
    if ((dtype != PCU_B200_F32 && dtype != PCU_B200_F64) || policy < 0 || policy > 2 || !status)
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (count == 0 || !prediction || !target || !out) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (count > (1ull << 58)) return PCU_B200_ERROR_SIZE_OVERFLOW;
    auto *st = reinterpret_cast<unsigned long long *>(status);
    cudaStream_t s = pcu_host::as_stream(stream);
    if (dtype == PCU_B200_F32)
        return pcu::run_mse<float>(policy, (const float *)prediction, (const float *)target, (float *)out, count,
                                   workspace, workspace_bytes, st, s, guard);
    return pcu::run_mse<double>(policy, (const double *)prediction, (const double *)target, (double *)out, count,
                                workspace, workspace_bytes, st, s, guard);
}

extern "C" int pcu_b200_strict_mse_segment_prepare(int dtype, int policy, const void *prediction, const void *target,
                                                   uint64_t count, uint64_t first_index, void *workspace,
                                                   size_t workspace_bytes, uint64_t *status, void *stream) {
    if ((dtype != PCU_B200_F32 && dtype != PCU_B200_F64) || policy < 0 || policy > 2 || !status)
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (count && (!prediction || !target)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (count > (1ull << 58) || first_index > (1ull << 58) - count) return PCU_B200_ERROR_SIZE_OVERFLOW;
    auto *st = reinterpret_cast<unsigned long long *>(status);
    cudaStream_t s = pcu_host::as_stream(stream);
    if (dtype == PCU_B200_F32)
        return pcu::prepare_mse<float>(policy, (const float *)prediction, (const float *)target, count, first_index,
                                       workspace, workspace_bytes, st, s);
    return pcu::prepare_mse<double>(policy, (const double *)prediction, (const double *)target, count, first_index,
                                    workspace, workspace_bytes, st, s);
}

extern "C" int pcu_b200_strict_mse_segment_walk(int dtype, int policy, const void *prediction, const void *target,
                                                uint64_t count, uint64_t first_index, uint64_t total_count,
                                                const void *carry_in, void *carry_out, void *out, void *workspace,
                                                size_t workspace_bytes, uint64_t *status, void *stream) {
    if ((dtype != PCU_B200_F32 && dtype != PCU_B200_F64) || policy < 0 || policy > 2 || !status)
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (count && (!prediction || !target)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (total_count > (1ull << 58) || first_index > total_count || count > total_count - first_index)
        return PCU_B200_ERROR_SIZE_OVERFLOW;
    if (out && (total_count == 0 || first_index + count != total_count)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    auto *st = reinterpret_cast<unsigned long long *>(status);
    cudaStream_t s = pcu_host::as_stream(stream);
    if (dtype == PCU_B200_F32)
        return pcu::walk_mse<float>(policy, (const float *)prediction, (const float *)target, count, first_index,
                                    total_count, (const float *)carry_in, (float *)carry_out, (float *)out, workspace,
                                    workspace_bytes, st, s);
    return pcu::walk_mse<double>(policy, (const double *)prediction, (const double *)target, count, first_index,
                                 total_count, (const double *)carry_in, (double *)carry_out, (double *)out, workspace,
                                 workspace_bytes, st, s);
}

static bool valid_sgd_args(int dtype, uint64_t count, const void *weights, const void *gradient, const void *updated,
                           uint32_t rate_bits_f32, const uint64_t *status) {
    if (!status || (rate_bits_f32 & 0x7f800000u) == 0x7f800000u) return false;  // capture rejects
    (void)dtype;
    return !count || (weights && gradient && updated);
}

extern "C" int pcu_b200_strict_mse_sgd(int dtype, int policy, const void *prediction, const void *target, void *loss,
                                       uint64_t mse_count, void *workspace, size_t workspace_bytes,
                                       uint64_t *mse_status, const void *weights, const void *gradient,
                                       void *updated, uint64_t sgd_count, uint32_t rate_bits_f32,
                                       uint64_t *sgd_status, void *stream) {
    if ((dtype != PCU_B200_F32 && dtype != PCU_B200_F64) || policy < 0 || policy > 2 || !mse_status)
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (mse_count == 0 || !prediction || !target || !loss) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (!valid_sgd_args(dtype, sgd_count, weights, gradient, updated, rate_bits_f32, sgd_status))
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (mse_count > (1ull << 58) || sgd_count > (1ull << 59)) return PCU_B200_ERROR_SIZE_OVERFLOW;
    auto *ms = reinterpret_cast<unsigned long long *>(mse_status);
    auto *ss = reinterpret_cast<unsigned long long *>(sgd_status);
    cudaStream_t s = pcu_host::as_stream(stream);
    if (dtype == PCU_B200_F32)
        return pcu::run_mse_sgd<float>(policy, (const float *)prediction, (const float *)target, (float *)loss,
                                       mse_count, workspace, workspace_bytes, ms,
                                       pcu::make_rider<float>(policy, weights, gradient, updated, sgd_count, 0,
                                                              rate_bits_f32, ss),
                                       s);
    return pcu::run_mse_sgd<double>(policy, (const double *)prediction, (const double *)target, (double *)loss,
                                    mse_count, workspace, workspace_bytes, ms,
                                    pcu::make_rider<double>(policy, weights, gradient, updated, sgd_count, 0,
                                                            rate_bits_f32, ss),
                                    s);
}

extern "C" int pcu_b200_strict_mse_sgd_segment_prepare(int dtype, int policy, const void *prediction,
                                                       const void *target, uint64_t mse_count,
                                                       uint64_t mse_first_index, void *workspace,
                                                       size_t workspace_bytes, uint64_t *mse_status,
                                                       const void *weights, const void *gradient, void *updated,
                                                       uint64_t sgd_count, uint64_t sgd_first_index,
                                                       uint32_t rate_bits_f32, uint64_t *sgd_status, void *stream) {
    if ((dtype != PCU_B200_F32 && dtype != PCU_B200_F64) || policy < 0 || policy > 2 || !mse_status)
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (mse_count && (!prediction || !target)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (!valid_sgd_args(dtype, sgd_count, weights, gradient, updated, rate_bits_f32, sgd_status))
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (mse_count > (1ull << 58) || mse_first_index > (1ull << 58) - mse_count) return PCU_B200_ERROR_SIZE_OVERFLOW;
    if (sgd_count > (1ull << 59) || sgd_first_index > (1ull << 59) - sgd_count) return PCU_B200_ERROR_SIZE_OVERFLOW;
    auto *ms = reinterpret_cast<unsigned long long *>(mse_status);
    auto *ss = reinterpret_cast<unsigned long long *>(sgd_status);
    cudaStream_t s = pcu_host::as_stream(stream);
    if (dtype == PCU_B200_F32)
        return pcu::prepare_mse_sgd<float>(policy, (const float *)prediction, (const float *)target, mse_count,
                                           mse_first_index, workspace, workspace_bytes, ms,
                                           pcu::make_rider<float>(policy, weights, gradient, updated, sgd_count,
                                                                  sgd_first_index, rate_bits_f32, ss),
                                           s);
    return pcu::prepare_mse_sgd<double>(policy, (const double *)prediction, (const double *)target, mse_count,
                                        mse_first_index, workspace, workspace_bytes, ms,
                                        pcu::make_rider<double>(policy, weights, gradient, updated, sgd_count,
                                                                sgd_first_index, rate_bits_f32, ss),
                                        s);
}

// A whole segment in one call: its maps, and the walk from *carry_in, in one launch for binary32
// (three for binary64).  `sgd` as in pcu_b200_strict_mse_sgd_segment_prepare.
namespace pcu {
template <typename T>
int run_mse_sgd_segment(int policy, const T *p, const T *t, uint64_t n, uint64_t base, uint64_t total, const T *carry_in,
                        T *carry_out, T *out, void *workspace, size_t workspace_bytes, unsigned long long *mse_status,
                        const SgdRider<T> &sgd, cudaStream_t stream, const CarryLink &link = CarryLink{}) {
    MseLayout<T> lay(n);
    if (!workspace || workspace_bytes < lay.bytes) return PCU_B200_ERROR_WORKSPACE;
    if constexpr (sizeof(T) == 4) {
        if (n) {
            SgdRider<T> head, tail;
            split_sgd<T>(sgd, sgd_units(lay.count[0], kChunkWarps * kRideGroupsPerCta, kRidePeriod, kRideSgd), head,
                         tail);
            int rc = onepass_mse<T>(policy, p, t, out, n, workspace, workspace_bytes, mse_status, stream, &head,
                                    ChainGuard{}, base, total, carry_in, carry_out, link);
            if (rc || !tail.n) return rc;
            const uint64_t per_cta = 256ull * (16 / sizeof(T)) * kSgdTrip;
            const uint64_t cap = 8ull * pcu_host::sm_count();
            const uint64_t want = (tail.n + per_cta - 1) / per_cta;
            sgd_share_kernel<T><<<(unsigned)(want < cap ? want : cap), 256, 0, stream>>>(tail);
            return pcu_host::launch_status();
        }
    }
    int rc = prepare_mse_sgd<T>(policy, p, t, n, base, workspace, workspace_bytes, mse_status, sgd, stream);
    if (rc) return rc;
    return walk_mse<T>(policy, p, t, n, base, total, carry_in, carry_out, out, workspace, workspace_bytes, mse_status,
                       stream, nullptr, ChainGuard{}, link);
}
}  // namespace pcu

extern "C" int pcu_b200_strict_mse_sgd_segment(int dtype, int policy, const void *prediction, const void *target,
                                               uint64_t mse_count, uint64_t mse_first_index, uint64_t total_count,
                                               const void *carry_in, void *carry_out, void *out, void *workspace,
                                               size_t workspace_bytes, uint64_t *mse_status, const void *weights,
                                               const void *gradient, void *updated, uint64_t sgd_count,
                                               uint64_t sgd_first_index, uint32_t rate_bits_f32, uint64_t *sgd_status,
                                               void *stream) {
    if ((dtype != PCU_B200_F32 && dtype != PCU_B200_F64) || policy < 0 || policy > 2 || !mse_status)
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (mse_count && (!prediction || !target)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (!valid_sgd_args(dtype, sgd_count, weights, gradient, updated, rate_bits_f32, sgd_status))
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (total_count > (1ull << 58) || mse_first_index > total_count || mse_count > total_count - mse_first_index)
        return PCU_B200_ERROR_SIZE_OVERFLOW;
    if (out && (total_count == 0 || mse_first_index + mse_count != total_count)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (sgd_count > (1ull << 59) || sgd_first_index > (1ull << 59) - sgd_count) return PCU_B200_ERROR_SIZE_OVERFLOW;
    auto *ms = reinterpret_cast<unsigned long long *>(mse_status);
    auto *ss = reinterpret_cast<unsigned long long *>(sgd_status);
    cudaStream_t s = pcu_host::as_stream(stream);
    if (dtype == PCU_B200_F32)
        return pcu::run_mse_sgd_segment<float>(
            policy, (const float *)prediction, (const float *)target, mse_count, mse_first_index, total_count,
            (const float *)carry_in, (float *)carry_out, (float *)out, workspace, workspace_bytes, ms,
            pcu::make_rider<float>(policy, weights, gradient, updated, sgd_count, sgd_first_index, rate_bits_f32, ss),
            s);
    return pcu::run_mse_sgd_segment<double>(
        policy, (const double *)prediction, (const double *)target, mse_count, mse_first_index, total_count,
        (const double *)carry_in, (double *)carry_out, (double *)out, workspace, workspace_bytes, ms,
        pcu::make_rider<double>(policy, weights, gradient, updated, sgd_count, sgd_first_index, rate_bits_f32, ss), s);
}

// ============================================================================
// The split strict MSE with every exchange on the device (one process per GPU).
//
// Every rank's hand-off block (pcu_b200_peer_alloc, zero-filled, mapped into every peer with
// pcu_b200_peer_open) holds the carry slot its predecessor stores into, and two banks of
// exchange slots, one per rank, selected by the call number's parity.  A call is one launch of
// the segment (maps and walk together for binary32) whose walker waits for the carry from rank
// r - 1 and stores its own into rank r + 1's block, then mse_exchange_kernel: it stores this
// rank's MSE and SGD words (and, on the last rank, the mean) into every peer's slot, waits for
// every peer's slot of the same call, and leaves the MIN of all ranks' words and the mean on
// this rank.  A rank's store of call e + 2 into a peer's bank can only follow that peer's exit
// from call e (it needs the peer's call e + 1 slot first), so two banks never mix calls.
// ============================================================================
namespace {

constexpr int kHandoffRanks = 8;

struct HandoffSlot {
    unsigned long long mse, sgd, mean, epoch;
};

struct HandoffBlock {
    unsigned long long carry;        // the running sum's bits (binary32 in the low half)
    unsigned long long carry_epoch;  // call number of `carry`
    unsigned long long pad[6];
    HandoffSlot slot[2][kHandoffRanks];
};

struct ExchangeArgs {
    HandoffBlock *blocks[kHandoffRanks];  // as this process sees them; blocks[rank] is its own
    unsigned long long *mse_status, *sgd_status;  // sgd_status may be null
    void *mean;                                   // this rank's mean output
    unsigned long long epoch;
    int rank, nranks, mean_bytes;
};

__global__ void __launch_bounds__(32) mse_exchange_kernel(const __grid_constant__ ExchangeArgs a) {
    using pcu::load_acquire_sys_u64;
    using pcu::store_release_sys_u64;
    const int q = threadIdx.x, last = a.nranks - 1;
    const int bank = (int)(a.epoch & 1);
    const unsigned long long mse = *(volatile unsigned long long *)a.mse_status;
    const unsigned long long sgd = a.sgd_status ? *(volatile unsigned long long *)a.sgd_status : ~0ull;
    unsigned long long mean = 0;
    if (a.rank == last)
        mean = a.mean_bytes == 8 ? *(volatile unsigned long long *)a.mean : *(volatile unsigned *)a.mean;
    const bool peer = q < a.nranks && q != a.rank;
    if (peer) {
        HandoffSlot *dst = &a.blocks[q]->slot[bank][a.rank];
        dst->mse = mse;
        dst->sgd = sgd;
        dst->mean = mean;
        store_release_sys_u64(&dst->epoch, a.epoch);  // the release orders the three stores before it
    }
    bool ok = true;
    unsigned long long m_mse = mse, m_sgd = sgd, peer_mean = 0;
    if (peer) {
        const HandoffSlot *src = &a.blocks[a.rank]->slot[bank][q];
        const unsigned long long t0 = pcu::global_ns();
        while (load_acquire_sys_u64(&src->epoch) < a.epoch) {
            if (pcu::global_ns() - t0 > pcu::kPeerWaitLimitNs) {
                ok = false;
                break;
            }
            __nanosleep(256);
        }
        if (ok) {
            const unsigned long long pm = *(volatile const unsigned long long *)&src->mse;
            const unsigned long long ps = *(volatile const unsigned long long *)&src->sgd;
            m_mse = pm < m_mse ? pm : m_mse;
            m_sgd = ps < m_sgd ? ps : m_sgd;
            peer_mean = *(volatile const unsigned long long *)&src->mean;
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const unsigned long long om = __shfl_xor_sync(0xffffffffu, m_mse, o);
        const unsigned long long os = __shfl_xor_sync(0xffffffffu, m_sgd, o);
        m_mse = om < m_mse ? om : m_mse;
        m_sgd = os < m_sgd ? os : m_sgd;
    }
    const bool all_ok = __all_sync(0xffffffffu, ok);
    if (q == 0) {
        constexpr unsigned long long kGaveUp = (0ull << 3) | pcu::kWatchdog;
        *a.mse_status = all_ok ? m_mse : kGaveUp;
        if (a.sgd_status) *a.sgd_status = m_sgd;
    }
    if (q == last && peer && ok) {  // the mean comes from the last rank
        if (a.mean_bytes == 8) *(unsigned long long *)a.mean = peer_mean;
        else *(unsigned *)a.mean = (unsigned)peer_mean;
    }
}

}  // namespace

extern "C" size_t pcu_b200_mse_handoff_bytes(void) { return (sizeof(HandoffBlock) + 255) / 256 * 256; }

extern "C" int pcu_b200_strict_mse_sgd_split(int dtype, int policy, const void *prediction, const void *target,
                                             uint64_t mse_count, uint64_t mse_first_index, uint64_t total_count,
                                             void *mean_out, void *workspace, size_t workspace_bytes,
                                             uint64_t *mse_status, const void *weights, const void *gradient,
                                             void *updated, uint64_t sgd_count, uint64_t sgd_first_index,
                                             uint32_t rate_bits_f32, uint64_t *sgd_status, void *const *blocks,
                                             int rank, int nranks, uint64_t epoch, void *stream) {
    if ((dtype != PCU_B200_F32 && dtype != PCU_B200_F64) || policy < 0 || policy > 2 || !mse_status || !mean_out)
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (nranks < 1 || nranks > kHandoffRanks || rank < 0 || rank >= nranks || !blocks || epoch == 0)
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    for (int r = 0; r < nranks; ++r)
        if (!blocks[r]) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (mse_count && (!prediction || !target)) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (sgd_count && !sgd_status) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (sgd_count && !valid_sgd_args(dtype, sgd_count, weights, gradient, updated, rate_bits_f32, sgd_status))
        return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (total_count == 0 || total_count > (1ull << 58) || mse_first_index > total_count ||
        mse_count > total_count - mse_first_index)
        return PCU_B200_ERROR_SIZE_OVERFLOW;
    // the last rank's segment ends the reduction (it divides); earlier ones may end there too when
    // the segments after them are empty
    if (rank == nranks - 1 && mse_first_index + mse_count != total_count) return PCU_B200_ERROR_INVALID_ARGUMENT;
    if (sgd_count > (1ull << 59) || sgd_first_index > (1ull << 59) - sgd_count) return PCU_B200_ERROR_SIZE_OVERFLOW;
    auto *ms = reinterpret_cast<unsigned long long *>(mse_status);
    auto *ss = reinterpret_cast<unsigned long long *>(sgd_status);
    cudaStream_t s = pcu_host::as_stream(stream);
    auto *mine = static_cast<HandoffBlock *>(blocks[rank]);
    pcu::CarryLink link{};
    link.epoch = epoch;
    const void *carry_in = nullptr;
    void *carry_out = nullptr;
    if (rank > 0) {
        carry_in = &mine->carry;
        link.in_flag = &mine->carry_epoch;
    }
    if (rank < nranks - 1) {
        auto *next = static_cast<HandoffBlock *>(blocks[rank + 1]);
        carry_out = &next->carry;
        link.out_flag = &next->carry_epoch;
    }
    void *out = rank == nranks - 1 ? mean_out : nullptr;
    int rc;
    if (dtype == PCU_B200_F32)
        rc = pcu::run_mse_sgd_segment<float>(
            policy, (const float *)prediction, (const float *)target, mse_count, mse_first_index, total_count,
            (const float *)carry_in, (float *)carry_out, (float *)out, workspace, workspace_bytes, ms,
            pcu::make_rider<float>(policy, weights, gradient, updated, sgd_count, sgd_first_index, rate_bits_f32, ss),
            s, link);
    else
        rc = pcu::run_mse_sgd_segment<double>(
            policy, (const double *)prediction, (const double *)target, mse_count, mse_first_index, total_count,
            (const double *)carry_in, (double *)carry_out, (double *)out, workspace, workspace_bytes, ms,
            pcu::make_rider<double>(policy, weights, gradient, updated, sgd_count, sgd_first_index, rate_bits_f32,
                                    ss),
            s, link);
    if (rc || nranks == 1) return rc;
    ExchangeArgs a{};
    for (int r = 0; r < nranks; ++r) a.blocks[r] = static_cast<HandoffBlock *>(blocks[r]);
    a.mse_status = ms;
    a.sgd_status = ss;
    a.mean = mean_out;
    a.epoch = epoch;
    a.rank = rank;
    a.nranks = nranks;
    a.mean_bytes = dtype == PCU_B200_F64 ? 8 : 4;
    mse_exchange_kernel<<<1, 32, 0, s>>>(a);
    return pcu_host::launch_status();
}
