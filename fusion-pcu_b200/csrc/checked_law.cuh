// checked_law.cuh -- the reference's checked binary32/binary64 scalar law on the device.
//
// Two layers:
//  * exact_*  : integer-significand evaluation of one checked operation (round to nearest,
//               ties to even, tininess after rounding at unbounded exponent, policy decision).
//               Restates Crates/core/scalar_checked_float.rs:312-631 and
//               Crates/core/scalar_checked_float/f64.rs:98-421.  Used only on rare paths.
//  * checked_*: the hot path.  The IEEE hardware operation (__fmul_rn/__fadd_rn/...; the
//               library is built with -fmad=false -ftz=false -prec-div=true) gives the law's
//               result bit for bit whenever the law does not fault (the reference pins this
//               equality, scalar_checked_float/tests.rs:306-353).  Faults are recognised from
//               the operands and the rounded result: a non-finite operand is Invalid, a
//               non-finite result of finite operands is Overflow, and only a result whose
//               magnitude is <= the smallest normal can carry an underflow decision, which is
//               then delegated to exact_*.  Under RejectSubnormalResult a nonzero subnormal
//               sum is rejected directly (sums of floats are exact in the subnormal range).
#pragma once

#include <cstdint>

namespace pcu {

enum : unsigned {
    kOk = 0,
    kDivideByZero = 1,
    kSignedDivisionOverflow = 2,
    kOverflow = 3,
    kUnderflow = 4,
    kInvalid = 5,
    kWatchdog = 7,
};

enum : int { kPolicyIeee = 0, kPolicyRejectSubnormal = 1, kPolicyGradual = 2 };
enum : int { kOpAdd = 0, kOpSub = 1, kOpMul = 2, kOpDiv = 3 };

constexpr unsigned long long kStatusOk = ~0ull;

struct UnderflowClass {
    bool tiny, inexact, subnormal;
};

__host__ __device__ __forceinline__ bool policy_rejects(int policy, UnderflowClass c) {
    return policy == kPolicyIeee ? (c.tiny && c.inexact)
         : policy == kPolicyRejectSubnormal ? (c.subnormal || (c.tiny && c.inexact))
         : false;
}

__device__ __forceinline__ uint64_t shift_jam(uint64_t v, uint32_t d) {
    if (d == 0) return v;
    if (d < 64) return (v >> d) | (uint64_t)((v & ((1ull << d) - 1)) != 0);
    return (uint64_t)(v != 0);
}

__device__ __forceinline__ bool rne_up(uint64_t sig, uint64_t guard) {
    return guard > 4 || (guard == 4 && (sig & 1));
}

// ------------------------------------------------------------------------- layout traits
template <typename T> struct Fmt;

template <> struct Fmt<float> {
    using Bits = uint32_t;
    static constexpr int kFrac = 23;          // stored fraction bits
    static constexpr int kMinExp = -126;      // exponent of the smallest normal
    static constexpr int kMaxExp = 127;
    static constexpr int kBias = 127;
    static constexpr Bits kSign = 0x80000000u;
    static constexpr Bits kExpMask = 0x7f800000u;
    static constexpr Bits kFracMask = 0x007fffffu;
    static constexpr Bits kMinNormalBits = 0x00800000u;
    __device__ static __forceinline__ Bits bits(float x) { return __float_as_uint(x); }
    __device__ static __forceinline__ float value(Bits b) { return __uint_as_float(b); }
    __device__ static __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }
    __device__ static __forceinline__ float add(float a, float b) { return __fadd_rn(a, b); }
    __device__ static __forceinline__ float sub(float a, float b) { return __fsub_rn(a, b); }
    __device__ static __forceinline__ float div(float a, float b) { return __fdiv_rn(a, b); }
    __device__ static __forceinline__ float abs(float x) { return fabsf(x); }
};

template <> struct Fmt<double> {
    using Bits = uint64_t;
    static constexpr int kFrac = 52;
    static constexpr int kMinExp = -1022;
    static constexpr int kMaxExp = 1023;
    static constexpr int kBias = 1023;
    static constexpr Bits kSign = 0x8000000000000000ull;
    static constexpr Bits kExpMask = 0x7ff0000000000000ull;
    static constexpr Bits kFracMask = 0x000fffffffffffffull;
    static constexpr Bits kMinNormalBits = 0x0010000000000000ull;
    __device__ static __forceinline__ Bits bits(double x) { return (Bits)__double_as_longlong(x); }
    __device__ static __forceinline__ double value(Bits b) { return __longlong_as_double((long long)b); }
    __device__ static __forceinline__ double mul(double a, double b) { return __dmul_rn(a, b); }
    __device__ static __forceinline__ double add(double a, double b) { return __dadd_rn(a, b); }
    __device__ static __forceinline__ double sub(double a, double b) { return __dsub_rn(a, b); }
    __device__ static __forceinline__ double div(double a, double b) { return __ddiv_rn(a, b); }
    __device__ static __forceinline__ double abs(double x) { return fabs(x); }
};

template <typename T>
__device__ __forceinline__ bool nonfinite_bits(typename Fmt<T>::Bits b) {
    return (b & Fmt<T>::kExpMask) == Fmt<T>::kExpMask;
}

// magnitude <= smallest normal (includes zero and subnormals)
template <typename T>
__device__ __forceinline__ bool at_or_below_min_normal(typename Fmt<T>::Bits b) {
    return (b & ~Fmt<T>::kSign) <= Fmt<T>::kMinNormalBits;
}

template <typename T>
__device__ __forceinline__ bool nonzero_subnormal(typename Fmt<T>::Bits b) {
    typename Fmt<T>::Bits m = b & ~Fmt<T>::kSign;
    return m != 0 && m < Fmt<T>::kMinNormalBits;
}

// ------------------------------------------------------------------------- exact law
// A decoded finite nonzero operand: value = sig * 2^(exp - kFrac).
struct Decoded {
    uint32_t sign;
    int32_t exp;
    uint64_t sig;
};

// 1 finite nonzero, 0 zero, -1 NaN/infinity
template <typename T>
__device__ __forceinline__ int decode(typename Fmt<T>::Bits bits, Decoded &d) {
    using F = Fmt<T>;
    uint64_t field = (uint64_t)((bits & F::kExpMask) >> F::kFrac);
    uint64_t frac = (uint64_t)(bits & F::kFracMask);
    d.sign = (uint32_t)(bits >> (sizeof(T) * 8 - 1));
    if (field == (uint64_t)(F::kExpMask >> F::kFrac)) return -1;
    if (field == 0 && frac == 0) return 0;
    if (field == 0) {
        d.exp = F::kMinExp;
        d.sig = frac;
    } else {
        d.exp = (int32_t)field - F::kBias;
        d.sig = frac | (1ull << F::kFrac);
    }
    return 1;
}

// Round and pack ext (kFrac+1 significand bits and 3 guard bits once normalised; value
// ext * 2^(exp - kFrac - 3)) into the destination format, classifying underflow.
template <typename T>
__device__ unsigned pack(uint32_t sign, uint64_t ext, int32_t exp, typename Fmt<T>::Bits &out,
                         UnderflowClass &c) {
    using F = Fmt<T>;
    constexpr int kTop = F::kFrac + 3;  // normalised ext lies in [2^kTop, 2^(kTop+1))
    while (ext >= (1ull << (kTop + 1))) { ext = shift_jam(ext, 1); exp += 1; }
    while (ext < (1ull << kTop)) { ext <<= 1; exp -= 1; }
    {
        uint64_t s = ext >> 3;
        int32_t e = exp;
        if (rne_up(s, ext & 7)) s += 1;
        if (s == (1ull << (F::kFrac + 1))) e += 1;
        c.tiny = e < F::kMinExp;
    }
    if (exp < F::kMinExp) {
        ext = shift_jam(ext, (uint32_t)(F::kMinExp - exp));
        exp = F::kMinExp;
    }
    uint64_t guard = ext & 7, sig = ext >> 3;
    c.inexact = guard != 0;
    if (rne_up(sig, guard)) sig += 1;
    using B = typename F::Bits;
    B sbits = (B)sign << (sizeof(T) * 8 - 1);
    if (exp == F::kMinExp && sig < (1ull << F::kFrac)) {
        out = sbits | (B)sig;
        c.subnormal = sig != 0;
        return kOk;
    }
    if (sig >= (1ull << (F::kFrac + 1))) { sig >>= 1; exp += 1; }
    if (exp > F::kMaxExp) return kOverflow;
    out = sbits | ((B)(exp + F::kBias) << F::kFrac) | ((B)sig & F::kFracMask);
    c.subnormal = false;
    return kOk;
}

template <typename T>
__device__ unsigned exact_passthrough(typename Fmt<T>::Bits v, int policy, typename Fmt<T>::Bits &out) {
    UnderflowClass c;
    c.subnormal = nonzero_subnormal<T>(v);
    c.tiny = c.subnormal;
    c.inexact = false;
    if (policy_rejects(policy, c)) return kUnderflow;
    out = v;
    return kOk;
}

template <typename T>
__device__ __noinline__ unsigned exact_addsub(typename Fmt<T>::Bits l, typename Fmt<T>::Bits r, bool subtract,
                                              int policy, typename Fmt<T>::Bits &out) {
    using B = typename Fmt<T>::Bits;
    constexpr int kSignShift = sizeof(T) * 8 - 1;
    Decoded a, b;
    int ka = decode<T>(l, a);
    if (ka < 0) return kInvalid;
    int kb = decode<T>(r, b);
    if (kb < 0) return kInvalid;
    if (kb) b.sign ^= (uint32_t)subtract;
    if (!ka) {
        if (kb) return exact_passthrough<T>(((B)b.sign << kSignShift) | (r & ~Fmt<T>::kSign), policy, out);
        B ls = l >> kSignShift, rs = (r >> kSignShift) ^ (B)subtract;
        out = ls == rs ? (ls << kSignShift) : (B)0;
        return kOk;
    }
    if (!kb) return exact_passthrough<T>(l, policy, out);
    if (a.exp < b.exp) { Decoded t = a; a = b; b = t; }
    uint64_t ae = a.sig << 3;
    uint64_t be = shift_jam(b.sig << 3, (uint32_t)(a.exp - b.exp));
    uint32_t sign;
    uint64_t ext;
    if (a.sign == b.sign) { sign = a.sign; ext = ae + be; }
    else if (ae >= be) { sign = a.sign; ext = ae - be; }
    else { sign = b.sign; ext = be - ae; }
    if (ext == 0) { out = 0; return kOk; }
    UnderflowClass c;
    unsigned k = pack<T>(sign, ext, a.exp, out, c);
    if (k) return k;
    return policy_rejects(policy, c) ? kUnderflow : kOk;
}

// Full-width product of two significands, normalised with sticky into ext.
__device__ __forceinline__ void wide_product(uint64_t x, uint64_t y, int frac, uint64_t &ext, int32_t &top_shift) {
    // value = x*y; find its top bit and reduce to frac+4 significant bits with sticky
    uint64_t lo = x * y;
    uint64_t hi = __umul64hi(x, y);
    int top = hi ? 127 - __clzll(hi) : 63 - __clzll(lo);
    int keep = frac + 3;  // ext top bit position
    if (top > keep) {
        uint32_t d = (uint32_t)(top - keep);
        // shift the 128-bit value right by d with sticky
        uint64_t r, sticky;
        if (d >= 64) {
            uint32_t e = d - 64;
            r = e ? (hi >> e) : hi;
            sticky = lo != 0 || (e && (hi & ((1ull << e) - 1)) != 0);
        } else {
            r = (lo >> d) | (d ? (hi << (64 - d)) : 0);
            sticky = (lo & ((1ull << d) - 1)) != 0;
        }
        ext = r | (uint64_t)sticky;
    } else {
        ext = lo << (keep - top);
    }
    top_shift = top;
}

template <typename T>
__device__ __noinline__ unsigned exact_mul(typename Fmt<T>::Bits l, typename Fmt<T>::Bits r, int policy,
                                           typename Fmt<T>::Bits &out) {
    using F = Fmt<T>;
    using B = typename F::Bits;
    constexpr int kSignShift = sizeof(T) * 8 - 1;
    Decoded a, b;
    int ka = decode<T>(l, a);
    if (ka < 0) return kInvalid;
    int kb = decode<T>(r, b);
    if (kb < 0) return kInvalid;
    if (!ka || !kb) { out = ((l ^ r) >> kSignShift) << kSignShift; return kOk; }
    uint64_t ext;
    int32_t top;
    wide_product(a.sig, b.sig, F::kFrac, ext, top);
    int32_t exp = a.exp + b.exp + top - 2 * F::kFrac;
    UnderflowClass c;
    unsigned k = pack<T>(a.sign ^ b.sign, ext, exp, out, c);
    (void)sizeof(B);
    if (k) return k;
    return policy_rejects(policy, c) ? kUnderflow : kOk;
}

// 128/64 restoring division of (num << shift) by den for the quotient's ext bits.
__device__ __forceinline__ uint64_t quotient_with_sticky(uint64_t num, uint64_t den, int shift) {
    // num < 2*den, den < 2^(frac+1), shift = frac + 3 ... computed bitwise to stay exact
    uint64_t q = 0, rem = num;
    // integer part
    if (rem >= den) { q = 1; rem -= den; }
    for (int i = 0; i < shift; ++i) {
        rem <<= 1;
        q <<= 1;
        if (rem >= den) { rem -= den; q |= 1; }
    }
    return q | (uint64_t)(rem != 0);
}

template <typename T>
__device__ __noinline__ unsigned exact_div(typename Fmt<T>::Bits l, typename Fmt<T>::Bits r, int policy,
                                           typename Fmt<T>::Bits &out) {
    using F = Fmt<T>;
    using B = typename F::Bits;
    constexpr int kSignShift = sizeof(T) * 8 - 1;
    Decoded a, b;
    int ka = decode<T>(l, a);
    if (ka < 0) return kInvalid;
    int kb = decode<T>(r, b);
    if (kb < 0) return kInvalid;
    B sign = ((l ^ r) >> kSignShift);
    if (!kb) return kDivideByZero;
    if (!ka) { out = sign << kSignShift; return kOk; }
    int s = F::kFrac - (63 - __clzll(a.sig));
    a.sig <<= s; a.exp -= s;
    s = F::kFrac - (63 - __clzll(b.sig));
    b.sig <<= s; b.exp -= s;
    uint64_t num = a.sig;
    int32_t exp = a.exp - b.exp;
    if (num < b.sig) { num <<= 1; exp -= 1; }
    uint64_t ext = quotient_with_sticky(num, b.sig, F::kFrac + 3);
    UnderflowClass c;
    unsigned k = pack<T>((uint32_t)sign, ext, exp, out, c);
    if (k) return k;
    return policy_rejects(policy, c) ? kUnderflow : kOk;
}

template <typename T>
__device__ __forceinline__ unsigned exact_binary(int op, typename Fmt<T>::Bits l, typename Fmt<T>::Bits r,
                                                 int policy, typename Fmt<T>::Bits &out) {
    switch (op) {
    case kOpAdd: return exact_addsub<T>(l, r, false, policy, out);
    case kOpSub: return exact_addsub<T>(l, r, true, policy, out);
    case kOpMul: return exact_mul<T>(l, r, policy, out);
    default: return exact_div<T>(l, r, policy, out);
    }
}

// ------------------------------------------------------------------------- hot checked ops
// Each returns kOk or the fault kind; `out` holds the law's result on kOk.

template <typename T>
__device__ __forceinline__ unsigned checked_mul(T a, T b, int policy, T &out) {
    using F = Fmt<T>;
    typename F::Bits ab = F::bits(a), bb = F::bits(b);
    if (nonfinite_bits<T>(ab) || nonfinite_bits<T>(bb)) return kInvalid;
    T p = F::mul(a, b);
    typename F::Bits pb = F::bits(p);
    if (nonfinite_bits<T>(pb)) return kOverflow;
    if (policy != kPolicyGradual && at_or_below_min_normal<T>(pb) && (ab << 1) != 0 && (bb << 1) != 0) {
        typename F::Bits r;
        unsigned k = exact_mul<T>(ab, bb, policy, r);
        if (k) return k;
        out = F::value(r);
        return kOk;
    }
    out = p;
    return kOk;
}

template <typename T>
__device__ __forceinline__ unsigned checked_add(T a, T b, int policy, T &out) {
    using F = Fmt<T>;
    typename F::Bits ab = F::bits(a), bb = F::bits(b);
    if (nonfinite_bits<T>(ab) || nonfinite_bits<T>(bb)) return kInvalid;
    T s = F::add(a, b);
    typename F::Bits sb = F::bits(s);
    if (nonfinite_bits<T>(sb)) return kOverflow;
    if (policy == kPolicyRejectSubnormal && nonzero_subnormal<T>(sb)) return kUnderflow;
    out = s;
    return kOk;
}

template <typename T>
__device__ __forceinline__ unsigned checked_sub(T a, T b, int policy, T &out) {
    using F = Fmt<T>;
    typename F::Bits ab = F::bits(a), bb = F::bits(b);
    if (nonfinite_bits<T>(ab) || nonfinite_bits<T>(bb)) return kInvalid;
    T s = F::sub(a, b);
    typename F::Bits sb = F::bits(s);
    if (nonfinite_bits<T>(sb)) return kOverflow;
    if (policy == kPolicyRejectSubnormal && nonzero_subnormal<T>(sb)) return kUnderflow;
    out = s;
    return kOk;
}

template <typename T>
__device__ __forceinline__ unsigned checked_div(T a, T b, int policy, T &out) {
    using F = Fmt<T>;
    typename F::Bits ab = F::bits(a), bb = F::bits(b);
    if (nonfinite_bits<T>(ab) || nonfinite_bits<T>(bb)) return kInvalid;
    if ((bb << 1) == 0) return kDivideByZero;
    T q = F::div(a, b);
    typename F::Bits qb = F::bits(q);
    if (nonfinite_bits<T>(qb)) return kOverflow;
    if (policy != kPolicyGradual && at_or_below_min_normal<T>(qb) && (ab << 1) != 0) {
        typename F::Bits r;
        unsigned k = exact_div<T>(ab, bb, policy, r);
        if (k) return k;
        out = F::value(r);
        return kOk;
    }
    out = q;
    return kOk;
}

template <typename T>
__device__ __forceinline__ unsigned checked_binary(int op, T a, T b, int policy, T &out) {
    switch (op) {
    case kOpAdd: return checked_add<T>(a, b, policy, out);
    case kOpSub: return checked_sub<T>(a, b, policy, out);
    case kOpMul: return checked_mul<T>(a, b, policy, out);
    default: return checked_div<T>(a, b, policy, out);
    }
}

// Strict SGD of one element (Crates/core/dialect/tensor/reference/strict_sgd/strict_sgd.rs:20-46):
// p = rate * g, then w - p, each step checked; `step` is 0 for the multiply and 1 for the
// subtract (event = index * 2 + step, tensor/strict_sgd/strict_sgd.rs:184-196).
template <typename T>
__device__ __forceinline__ unsigned checked_sgd(T w, T g, T rate, int policy, T &out, unsigned &step) {
    T p;
    const unsigned k = checked_mul<T>(rate, g, policy, p);
    if (k) {
        step = 0;
        return k;
    }
    step = 1;
    return checked_sub<T>(w, p, policy, out);
}

// The strict SGD law on V elements at once, for the common case.  Suppose every product
// rate * g is finite and either above the smallest normal or the product of a zero gradient, and
// every difference w - p is finite (and, under RejectSubnormalResult, zero or at least the
// smallest normal).  Then no step of any element faults and the hardware results are the
// law's: `out` holds them and the call returns true.  Otherwise it returns false, `out` is
// meaningless, and the caller runs checked_sgd element by element.  A non-finite w or g always
// shows as a non-finite product or difference, because the rate is finite.  A few compares
// per element and one branch per vector replace the per-step branches of checked_sgd.
template <typename T, int V>
__device__ __forceinline__ bool sgd_fast(const T *w, const T *g, T rate, int policy, T *out) {
    using F = Fmt<T>;
    const T inf = F::value(F::kExpMask), tiny = F::value(F::kMinNormalBits);
    const bool lax = policy != kPolicyRejectSubnormal;
    bool ok = true;
#pragma unroll
    for (int e = 0; e < V; ++e) {
        const T p = F::mul(rate, g[e]);
        const T r = F::sub(w[e], p);
        const T ap = F::abs(p), ar = F::abs(r);
        ok = ok & (ap < inf) & ((ap > tiny) | (g[e] == T(0))) & (ar < inf) & (lax | (ar >= tiny) | (r == T(0)));
        out[e] = r;
    }
    return ok;
}

// ReLU selection (scalar_checked_float.rs:273-309): non-finite -> Invalid; negative or either
// signed zero -> +0; RejectSubnormalResult rejects a subnormal result.
template <typename T>
__device__ __forceinline__ unsigned checked_relu(T x, int policy, T &out) {
    using F = Fmt<T>;
    typename F::Bits xb = F::bits(x);
    if (nonfinite_bits<T>(xb)) return kInvalid;
    typename F::Bits r = ((xb & F::kSign) || (xb << 1) == 0) ? (typename F::Bits)0 : xb;
    if (policy == kPolicyRejectSubnormal && nonzero_subnormal<T>(r)) return kUnderflow;
    out = F::value(r);
    return kOk;
}

// ReLU backward (scalar_checked_float.rs:634-652): both operands finite; select upstream when
// the input is strictly positive (by encoding), else +0; RejectSubnormalResult rejects a
// selected subnormal.
template <typename T>
__device__ __forceinline__ unsigned checked_relu_backward(T x, T dy, int policy, T &out) {
    using F = Fmt<T>;
    typename F::Bits xb = F::bits(x), yb = F::bits(dy);
    if (nonfinite_bits<T>(xb) || nonfinite_bits<T>(yb)) return kInvalid;
    bool positive = !(xb & F::kSign) && (xb << 1) != 0;
    typename F::Bits r = positive ? yb : (typename F::Bits)0;
    if (policy == kPolicyRejectSubnormal && nonzero_subnormal<T>(r)) return kUnderflow;
    out = F::value(r);
    return kOk;
}

}  // namespace pcu
