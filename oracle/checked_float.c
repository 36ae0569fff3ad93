/*
 * checked_float.c -- TEST INFRASTRUCTURE ONLY (see pcu_oracle.h).
 *
 * Integer-significand restatement of the reference's checked binary32/binary64
 * law.  Every operation rounds to nearest, ties to even, on an integer
 * significand carried with three guard bits (two extra plus a sticky bit);
 * tininess is judged after rounding to the destination precision with an
 * unbounded exponent, inexactness on the final exponent-limited result.
 *
 * Followed, step for step:
 *   binary32  Crates/core/scalar_checked_float.rs:312-631
 *             (decode :312-336, shift_right_jam :338-347, round_increment :349-352,
 *              round_to_precision :357-370, pack :372-446, add :448-506,
 *              passthrough :508-532, multiply :534-579, divide :581-631,
 *              relu :273-309, neg :235-271, relu_backward :634-652)
 *   binary64  Crates/core/scalar_checked_float/f64.rs:25-421
 *   policy    Crates/core/scalar_float_underflow.rs:58-73
 *   counts    Crates/core/scalar_checked_conversion/integer/integer.rs:13-44
 *   widening  Crates/core/scalar_widen.rs:9-33
 * No host floating-point arithmetic is used in this file.
 */
#include <stdbool.h>
#include <stdint.h>

#include "pcu_oracle.h"

typedef struct {
    bool tiny;      /* tiny after rounding at unbounded exponent (IEEE 754-2019 7.5(a)) */
    bool inexact;   /* final, exponent-limited rounding discarded information */
    bool subnormal; /* final result is a nonzero subnormal */
} underflow_class;

static bool policy_rejects(int policy, underflow_class c)
{
    switch (policy) {
    case 0: return c.tiny && c.inexact;
    case 1: return c.subnormal || (c.tiny && c.inexact);
    default: return false;
    }
}

static uint64_t jam64(uint64_t value, uint32_t distance)
{
    if (distance == 0) return value;
    if (distance < 64) return (value >> distance) | (uint64_t)((value & ((1ull << distance) - 1)) != 0);
    return (uint64_t)(value != 0);
}

static uint64_t jam128(unsigned __int128 value, uint32_t distance)
{
    if (distance == 0) return (uint64_t)value;
    if (distance < 128) {
        unsigned __int128 mask = (((unsigned __int128)1) << distance) - 1;
        return (uint64_t)((value >> distance) | (unsigned __int128)((value & mask) != 0));
    }
    return (uint64_t)(value != 0);
}

static bool round_up(uint64_t significand, uint64_t discarded)
{
    return discarded > 4 || (discarded == 4 && (significand & 1) != 0);
}

static int top_bit64(uint64_t v) { return 63 - __builtin_clzll(v); }

static int top_bit128(unsigned __int128 v)
{
    uint64_t hi = (uint64_t)(v >> 64);
    return hi ? 64 + top_bit64(hi) : top_bit64((uint64_t)v);
}

/* ===================================================================== binary32 */

typedef struct {
    uint32_t sign;
    int32_t exponent;
    uint64_t significand;
} parts;

/* 1 = nonzero finite, 0 = signed zero, -1 = NaN or infinity */
static int unpack32(uint32_t bits, parts *p)
{
    uint32_t field = (bits >> 23) & 0xffu;
    uint32_t fraction = bits & 0x7fffffu;
    if (field == 0xffu) return -1;
    p->sign = bits >> 31;
    if (field == 0 && fraction == 0) return 0;
    if (field == 0) {
        p->exponent = -126;
        p->significand = fraction;
    } else {
        p->exponent = (int32_t)field - 127;
        p->significand = fraction | 0x800000u;
    }
    return 1;
}

/* ext carries 24 significand bits plus 3 guard bits once normalized to
 * [2^26, 2^27); its value is ext * 2^(exponent - 26). */
static int pack32(uint32_t sign, uint64_t ext, int32_t exponent, uint32_t *out, underflow_class *c)
{
    while (ext >= (1ull << 27)) { ext = jam64(ext, 1); exponent += 1; }
    while (ext < (1ull << 26)) { ext <<= 1; exponent -= 1; }

    {   /* destination precision at unbounded exponent */
        uint64_t s = ext >> 3;
        int32_t e = exponent;
        if (round_up(s, ext & 7)) s += 1;
        if (s == (1ull << 24)) e += 1;
        c->tiny = e < -126;
    }
    if (exponent < -126) {
        ext = jam64(ext, (uint32_t)(-126 - exponent));
        exponent = -126;
    }
    uint64_t discarded = ext & 7;
    uint64_t significand = ext >> 3;
    c->inexact = discarded != 0;
    if (round_up(significand, discarded)) significand += 1;

    if (exponent == -126 && significand < 0x800000u) {
        *out = (sign << 31) | (uint32_t)significand;
        c->subnormal = significand != 0;
        return 0;
    }
    if (significand >= (1ull << 24)) { significand >>= 1; exponent += 1; }
    if (exponent > 127) return PCU_ORACLE_OVERFLOW;
    *out = (sign << 31) | ((uint32_t)(exponent + 127) << 23) | ((uint32_t)significand & 0x7fffffu);
    c->subnormal = false;
    return 0;
}

static int passthrough32(uint32_t value, int policy, uint32_t *out)
{
    uint32_t magnitude = value & 0x7fffffffu;
    underflow_class c;
    c.subnormal = magnitude != 0 && magnitude < 0x800000u;
    c.tiny = c.subnormal;
    c.inexact = false;
    if (policy_rejects(policy, c)) return PCU_ORACLE_UNDERFLOW;
    *out = value;
    return 0;
}

static int finish32(int kind, int policy, underflow_class c)
{
    if (kind) return kind;
    return policy_rejects(policy, c) ? PCU_ORACLE_UNDERFLOW : 0;
}

static int add32(uint32_t left, uint32_t right, bool subtract, int policy, uint32_t *out)
{
    parts a, b;
    int ka = unpack32(left, &a);
    if (ka < 0) return PCU_ORACLE_INVALID;
    int kb = unpack32(right, &b);
    if (kb < 0) return PCU_ORACLE_INVALID;
    if (kb) b.sign ^= (uint32_t)subtract;
    if (!ka) {
        if (kb) return passthrough32((b.sign << 31) | (right & 0x7fffffffu), policy, out);
        uint32_t ls = left >> 31, rs = (right >> 31) ^ (uint32_t)subtract;
        *out = ls == rs ? (ls << 31) : 0u;
        return 0;
    }
    if (!kb) return passthrough32(left, policy, out);
    if (a.exponent < b.exponent) { parts t = a; a = b; b = t; }
    uint64_t a_ext = a.significand << 3;
    uint64_t b_ext = jam64(b.significand << 3, (uint32_t)(a.exponent - b.exponent));
    uint32_t sign;
    uint64_t ext;
    if (a.sign == b.sign) { sign = a.sign; ext = a_ext + b_ext; }
    else if (a_ext >= b_ext) { sign = a.sign; ext = a_ext - b_ext; }
    else { sign = b.sign; ext = b_ext - a_ext; }
    if (ext == 0) { *out = 0u; return 0; }
    underflow_class c;
    return finish32(pack32(sign, ext, a.exponent, out, &c), policy, c);
}

static int mul32(uint32_t left, uint32_t right, int policy, uint32_t *out)
{
    parts a, b;
    int ka = unpack32(left, &a);
    if (ka < 0) return PCU_ORACLE_INVALID;
    int kb = unpack32(right, &b);
    if (kb < 0) return PCU_ORACLE_INVALID;
    if (!ka || !kb) { *out = ((left ^ right) >> 31) << 31; return 0; }
    uint64_t product = a.significand * b.significand;
    int top = top_bit64(product);
    int32_t exponent = a.exponent + b.exponent + top - 46;
    uint64_t ext = top > 26 ? jam64(product, (uint32_t)(top - 26)) : product << (26 - top);
    underflow_class c;
    return finish32(pack32(a.sign ^ b.sign, ext, exponent, out, &c), policy, c);
}

static int div32(uint32_t left, uint32_t right, int policy, uint32_t *out)
{
    parts a, b;
    int ka = unpack32(left, &a);
    if (ka < 0) return PCU_ORACLE_INVALID;
    int kb = unpack32(right, &b);
    if (kb < 0) return PCU_ORACLE_INVALID;
    uint32_t sign = (left ^ right) >> 31;
    if (!kb) return PCU_ORACLE_DIVIDE_BY_ZERO;
    if (!ka) { *out = sign << 31; return 0; }
    int shift = 23 - top_bit64(a.significand);
    a.significand <<= shift; a.exponent -= shift;
    shift = 23 - top_bit64(b.significand);
    b.significand <<= shift; b.exponent -= shift;
    uint64_t numerator = a.significand;
    int32_t exponent = a.exponent - b.exponent;
    if (numerator < b.significand) { numerator <<= 1; exponent -= 1; }
    uint64_t scaled = numerator << 26;
    uint64_t ext = scaled / b.significand;
    if (scaled % b.significand) ext |= 1;
    underflow_class c;
    return finish32(pack32(sign, ext, exponent, out, &c), policy, c);
}

int pcu_oracle_f32_binary(uint32_t left, uint32_t right, int op, int policy, uint32_t *out)
{
    switch (op) {
    case 0: return add32(left, right, false, policy, out);
    case 1: return add32(left, right, true, policy, out);
    case 2: return mul32(left, right, policy, out);
    default: return div32(left, right, policy, out);
    }
}

static int exact_select32(uint32_t result, int policy, uint32_t *out)
{
    underflow_class c;
    c.subnormal = result != 0 && (result & 0x7f800000u) == 0 && (result & 0x7fffffffu) != 0;
    c.tiny = c.subnormal;
    c.inexact = false;
    if (policy_rejects(policy, c)) return PCU_ORACLE_UNDERFLOW;
    *out = result;
    return 0;
}

int pcu_oracle_f32_relu(uint32_t x, int policy, uint32_t *out)
{
    if ((x & 0x7f800000u) == 0x7f800000u) return PCU_ORACLE_INVALID;
    uint32_t result = ((x & 0x80000000u) || (x << 1) == 0) ? 0u : x;
    return exact_select32(result, policy, out);
}

int pcu_oracle_f32_neg(uint32_t x, int policy, uint32_t *out)
{
    if ((x & 0x7f800000u) == 0x7f800000u) return PCU_ORACLE_INVALID;
    return exact_select32(x ^ 0x80000000u, policy, out);
}

int pcu_oracle_f32_relu_backward(uint32_t x, uint32_t upstream, int policy, uint32_t *out)
{
    if ((x & 0x7f800000u) == 0x7f800000u || (upstream & 0x7f800000u) == 0x7f800000u)
        return PCU_ORACLE_INVALID;
    bool positive = (x & 0x80000000u) == 0 && (x & 0x7fffffffu) != 0;
    uint32_t selected = positive ? upstream : 0u;
    uint32_t negated;
    int kind = pcu_oracle_f32_neg(selected, policy, &negated);
    if (kind) return kind;
    return pcu_oracle_f32_neg(negated, 0, out);
}

/* ===================================================================== binary64 */

static int unpack64(uint64_t bits, parts *p)
{
    uint64_t field = (bits >> 52) & 0x7ffu;
    uint64_t fraction = bits & ((1ull << 52) - 1);
    if (field == 0x7ffu) return -1;
    p->sign = (uint32_t)(bits >> 63);
    if (field == 0 && fraction == 0) return 0;
    if (field == 0) {
        p->exponent = -1022;
        p->significand = fraction;
    } else {
        p->exponent = (int32_t)field - 1023;
        p->significand = fraction | (1ull << 52);
    }
    return 1;
}

/* ext normalized to [2^55, 2^56): 53 significand bits plus 3 guard bits. */
static int pack64(uint32_t sign, uint64_t ext, int32_t exponent, uint64_t *out, underflow_class *c)
{
    while (ext >= (1ull << 56)) { ext = jam64(ext, 1); exponent += 1; }
    while (ext < (1ull << 55)) { ext <<= 1; exponent -= 1; }
    {
        uint64_t s = ext >> 3;
        int32_t e = exponent;
        if (round_up(s, ext & 7)) s += 1;
        if (s == (1ull << 53)) e += 1;
        c->tiny = e < -1022;
    }
    if (exponent < -1022) {
        ext = jam64(ext, (uint32_t)(-1022 - exponent));
        exponent = -1022;
    }
    uint64_t discarded = ext & 7;
    uint64_t significand = ext >> 3;
    c->inexact = discarded != 0;
    if (round_up(significand, discarded)) significand += 1;
    uint64_t sign_bits = (uint64_t)sign << 63;
    if (exponent == -1022 && significand < (1ull << 52)) {
        *out = sign_bits | significand;
        c->subnormal = significand != 0;
        return 0;
    }
    if (significand >= (1ull << 53)) { significand >>= 1; exponent += 1; }
    if (exponent > 1023) return PCU_ORACLE_OVERFLOW;
    *out = sign_bits | ((uint64_t)(exponent + 1023) << 52) | (significand & ((1ull << 52) - 1));
    c->subnormal = false;
    return 0;
}

static int passthrough64(uint64_t value, int policy, uint64_t *out)
{
    uint64_t magnitude = value & ~(1ull << 63);
    underflow_class c;
    c.subnormal = magnitude != 0 && magnitude < (1ull << 52);
    c.tiny = c.subnormal;
    c.inexact = false;
    if (policy_rejects(policy, c)) return PCU_ORACLE_UNDERFLOW;
    *out = value;
    return 0;
}

static int add64(uint64_t left, uint64_t right, bool subtract, int policy, uint64_t *out)
{
    parts a, b;
    int ka = unpack64(left, &a);
    if (ka < 0) return PCU_ORACLE_INVALID;
    int kb = unpack64(right, &b);
    if (kb < 0) return PCU_ORACLE_INVALID;
    if (kb) b.sign ^= (uint32_t)subtract;
    if (!ka) {
        if (kb) return passthrough64(((uint64_t)b.sign << 63) | (right & ~(1ull << 63)), policy, out);
        uint64_t ls = left >> 63, rs = (right >> 63) ^ (uint64_t)subtract;
        *out = ls == rs ? (ls << 63) : 0u;
        return 0;
    }
    if (!kb) return passthrough64(left, policy, out);
    if (a.exponent < b.exponent) { parts t = a; a = b; b = t; }
    uint64_t a_ext = a.significand << 3;
    uint64_t b_ext = jam64(b.significand << 3, (uint32_t)(a.exponent - b.exponent));
    uint32_t sign;
    uint64_t ext;
    if (a.sign == b.sign) { sign = a.sign; ext = a_ext + b_ext; }
    else if (a_ext >= b_ext) { sign = a.sign; ext = a_ext - b_ext; }
    else { sign = b.sign; ext = b_ext - a_ext; }
    if (ext == 0) { *out = 0u; return 0; }
    underflow_class c;
    int kind = pack64(sign, ext, a.exponent, out, &c);
    if (kind) return kind;
    return policy_rejects(policy, c) ? PCU_ORACLE_UNDERFLOW : 0;
}

static int mul64(uint64_t left, uint64_t right, int policy, uint64_t *out)
{
    parts a, b;
    int ka = unpack64(left, &a);
    if (ka < 0) return PCU_ORACLE_INVALID;
    int kb = unpack64(right, &b);
    if (kb < 0) return PCU_ORACLE_INVALID;
    if (!ka || !kb) { *out = ((left ^ right) >> 63) << 63; return 0; }
    unsigned __int128 product = (unsigned __int128)a.significand * b.significand;
    int top = top_bit128(product);
    int32_t exponent = a.exponent + b.exponent + top - 104;
    uint64_t ext = top > 55 ? jam128(product, (uint32_t)(top - 55)) : (uint64_t)(product << (55 - top));
    underflow_class c;
    int kind = pack64(a.sign ^ b.sign, ext, exponent, out, &c);
    if (kind) return kind;
    return policy_rejects(policy, c) ? PCU_ORACLE_UNDERFLOW : 0;
}

static int div64(uint64_t left, uint64_t right, int policy, uint64_t *out)
{
    parts a, b;
    int ka = unpack64(left, &a);
    if (ka < 0) return PCU_ORACLE_INVALID;
    int kb = unpack64(right, &b);
    if (kb < 0) return PCU_ORACLE_INVALID;
    uint32_t sign = (uint32_t)((left ^ right) >> 63);
    if (!kb) return PCU_ORACLE_DIVIDE_BY_ZERO;
    if (!ka) { *out = (uint64_t)sign << 63; return 0; }
    int shift = 52 - top_bit64(a.significand);
    a.significand <<= shift; a.exponent -= shift;
    shift = 52 - top_bit64(b.significand);
    b.significand <<= shift; b.exponent -= shift;
    unsigned __int128 numerator = a.significand;
    unsigned __int128 denominator = b.significand;
    int32_t exponent = a.exponent - b.exponent;
    if (numerator < denominator) { numerator <<= 1; exponent -= 1; }
    unsigned __int128 scaled = numerator << 55;
    uint64_t ext = (uint64_t)(scaled / denominator);
    if (scaled % denominator) ext |= 1;
    underflow_class c;
    int kind = pack64(sign, ext, exponent, out, &c);
    if (kind) return kind;
    return policy_rejects(policy, c) ? PCU_ORACLE_UNDERFLOW : 0;
}

int pcu_oracle_f64_binary(uint64_t left, uint64_t right, int op, int policy, uint64_t *out)
{
    switch (op) {
    case 0: return add64(left, right, false, policy, out);
    case 1: return add64(left, right, true, policy, out);
    case 2: return mul64(left, right, policy, out);
    default: return div64(left, right, policy, out);
    }
}

static int exact_select64(uint64_t result, int policy, uint64_t *out)
{
    underflow_class c;
    uint64_t magnitude = result & ~(1ull << 63);
    c.subnormal = magnitude != 0 && (result & 0x7ff0000000000000ull) == 0;
    c.tiny = c.subnormal;
    c.inexact = false;
    if (policy_rejects(policy, c)) return PCU_ORACLE_UNDERFLOW;
    *out = result;
    return 0;
}

int pcu_oracle_f64_relu(uint64_t x, int policy, uint64_t *out)
{
    if ((x & 0x7ff0000000000000ull) == 0x7ff0000000000000ull) return PCU_ORACLE_INVALID;
    uint64_t result = ((x >> 63) || (x << 1) == 0) ? 0u : x;
    return exact_select64(result, policy, out);
}

int pcu_oracle_f64_neg(uint64_t x, int policy, uint64_t *out)
{
    if ((x & 0x7ff0000000000000ull) == 0x7ff0000000000000ull) return PCU_ORACLE_INVALID;
    return exact_select64(x ^ (1ull << 63), policy, out);
}

int pcu_oracle_f64_relu_backward(uint64_t x, uint64_t upstream, int policy, uint64_t *out)
{
    if ((x & 0x7ff0000000000000ull) == 0x7ff0000000000000ull ||
        (upstream & 0x7ff0000000000000ull) == 0x7ff0000000000000ull)
        return PCU_ORACLE_INVALID;
    bool positive = (x >> 63) == 0 && (x << 1) != 0;
    uint64_t selected = positive ? upstream : 0u;
    uint64_t negated;
    int kind = pcu_oracle_f64_neg(selected, policy, &negated);
    if (kind) return kind;
    return pcu_oracle_f64_neg(negated, 0, out);
}

/* ===================================================================== conversions */

static uint64_t pack_count(uint64_t count, uint32_t fraction_bits, uint32_t bias)
{
    if (count == 0) return 0;
    uint32_t exponent = (uint32_t)top_bit64(count);
    uint64_t significand;
    if (exponent <= fraction_bits) {
        significand = count << (fraction_bits - exponent);
    } else {
        uint32_t shift = exponent - fraction_bits;
        uint64_t quotient = count >> shift;
        uint64_t remainder = count & ((1ull << shift) - 1);
        uint64_t halfway = 1ull << (shift - 1);
        bool up = remainder > halfway || (remainder == halfway && (quotient & 1));
        significand = quotient + (uint64_t)up;
    }
    if (significand == (1ull << (fraction_bits + 1))) { significand >>= 1; exponent += 1; }
    return ((uint64_t)(exponent + bias) << fraction_bits) | (significand & ((1ull << fraction_bits) - 1));
}

uint32_t pcu_oracle_count_f32(uint64_t count) { return (uint32_t)pack_count(count, 23, 127); }
uint64_t pcu_oracle_count_f64(uint64_t count) { return pack_count(count, 52, 1023); }

uint64_t pcu_oracle_f32_bits_to_f64_bits(uint32_t bits)
{
    uint64_t sign = (uint64_t)(bits >> 31) << 63;
    uint32_t exponent = (bits >> 23) & 0xffu;
    uint32_t fraction = bits & 0x7fffffu;
    if (exponent == 0xffu) return sign | (0x7ffull << 52) | ((uint64_t)fraction << 29);
    if (exponent != 0) return sign | ((uint64_t)(exponent + 1023 - 127) << 52) | ((uint64_t)fraction << 29);
    if (fraction == 0) return sign;
    uint32_t leading = (uint32_t)top_bit64(fraction);
    uint64_t significand = (uint64_t)fraction << (52 - leading);
    return sign | ((uint64_t)(leading + 874) << 52) | (significand & ((1ull << 52) - 1));
}
