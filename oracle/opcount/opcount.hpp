// Executed-operation counter for the CPU oracle — TEST INFRASTRUCTURE.
//
// opcount.cpp compiles shoehorn_oracle.c as C++ with `float` replaced by
// sh_cf, a 4-byte wrapper whose operators perform the same IEEE f32
// arithmetic as the C code (same operand order, same promotions: f32 op
// integer stays f32, f32 op f64 widens to f64) and count each executed
// operation.  The counting build's encoded bytes are checked equal to the
// plain oracle's, which shows that the substitution changed no result.
//
// Counting convention (one unit each): f32 add, sub, mul, div, sqrt,
// compare, min/max (f32::max/min), and round-to-integer (nearest_int).
// Not counted: negation and fabsf (operand modifiers on the GPU), integer
// arithmetic, integer <-> float conversions, f64 arithmetic (counted apart).
#pragma once
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <cmath>
#include <type_traits>

namespace shoc {
struct Counts {
    uint64_t arith, cmp, sqrt, round, minmax, f64;
};
extern thread_local Counts counts;
}  // namespace shoc

struct sh_cf {
    float v;
    sh_cf() = default;
    template <class T, std::enable_if_t<std::is_arithmetic_v<T>, int> = 0>
    constexpr sh_cf(T x) : v((float)x) {}
    template <class T, std::enable_if_t<std::is_arithmetic_v<T>, int> = 0>
    explicit constexpr operator T() const { return (T)v; }
    static sh_cf raw(float x) { sh_cf r; r.v = x; return r; }
    sh_cf operator-() const { return raw(-v); }
    sh_cf operator+() const { return *this; }
};
static_assert(sizeof(sh_cf) == 4 && std::is_trivially_copyable_v<sh_cf>, "sh_cf must be layout-equal to float");

namespace shoc {
template <class T>
using narrow_t = std::enable_if_t<std::is_arithmetic_v<T> && !std::is_floating_point_v<T>, int>;
template <class T>
using f32_t = std::enable_if_t<std::is_same_v<T, float>, int>;
}  // namespace shoc

// f32 op f32 / f32 op integer / f32 op float literal -> f32, counted;
// f32 op f64 -> f64 (C's usual arithmetic conversions), counted as f64.
#define SHOC_BINOP(op)                                                                                   \
    inline sh_cf operator op(sh_cf a, sh_cf b) { shoc::counts.arith++; return sh_cf::raw(a.v op b.v); }  \
    template <class T, shoc::narrow_t<T> = 0>                                                            \
    inline sh_cf operator op(sh_cf a, T b) { shoc::counts.arith++; return sh_cf::raw(a.v op (float)b); } \
    template <class T, shoc::narrow_t<T> = 0>                                                            \
    inline sh_cf operator op(T a, sh_cf b) { shoc::counts.arith++; return sh_cf::raw((float)a op b.v); } \
    inline sh_cf operator op(sh_cf a, float b) { shoc::counts.arith++; return sh_cf::raw(a.v op b); }    \
    inline sh_cf operator op(float a, sh_cf b) { shoc::counts.arith++; return sh_cf::raw(a op b.v); }    \
    inline double operator op(sh_cf a, double b) { shoc::counts.f64++; return (double)a.v op b; }        \
    inline double operator op(double a, sh_cf b) { shoc::counts.f64++; return a op (double)b.v; }        \
    template <class T>                                                                                   \
    inline sh_cf &operator op##=(sh_cf &a, T b) { a = a op b; return a; }
SHOC_BINOP(+)
SHOC_BINOP(-)
SHOC_BINOP(*)
SHOC_BINOP(/)
#undef SHOC_BINOP

#define SHOC_CMP(op)                                                                                   \
    inline bool operator op(sh_cf a, sh_cf b) { shoc::counts.cmp++; return a.v op b.v; }               \
    template <class T, shoc::narrow_t<T> = 0>                                                          \
    inline bool operator op(sh_cf a, T b) { shoc::counts.cmp++; return a.v op (float)b; }              \
    template <class T, shoc::narrow_t<T> = 0>                                                          \
    inline bool operator op(T a, sh_cf b) { shoc::counts.cmp++; return (float)a op b.v; }              \
    inline bool operator op(sh_cf a, float b) { shoc::counts.cmp++; return a.v op b; }                 \
    inline bool operator op(float a, sh_cf b) { shoc::counts.cmp++; return a op b.v; }                 \
    inline bool operator op(sh_cf a, double b) { shoc::counts.cmp++; return (double)a.v op b; }        \
    inline bool operator op(double a, sh_cf b) { shoc::counts.cmp++; return a op (double)b.v; }
SHOC_CMP(<)
SHOC_CMP(>)
SHOC_CMP(<=)
SHOC_CMP(>=)
SHOC_CMP(==)
SHOC_CMP(!=)
#undef SHOC_CMP

inline sh_cf sqrtf(sh_cf a) { shoc::counts.sqrt++; return sh_cf::raw(::sqrtf(a.v)); }
inline sh_cf fabsf(sh_cf a) { return sh_cf::raw(::fabsf(a.v)); }
inline sh_cf roundf(sh_cf a) { shoc::counts.round++; return sh_cf::raw(::roundf(a.v)); }
inline bool signbit(sh_cf a) { return std::signbit(a.v); }

// The oracle's scalar helpers, with the oracle's semantics, counted as one
// operation each (the oracle leaves them out under SH_OPCOUNT).
extern "C" inline int32_t oq_nearest_int(sh_cf x) {
    shoc::counts.round++;
    float r = ::roundf(x.v);
    if (r != r) return 0;
    if (r >= 2147483648.0f) return INT32_MAX;
    if (r <= -2147483648.0f) return INT32_MIN;
    return (int32_t)r;
}
static inline sh_cf rmaxf(sh_cf a, sh_cf b) {
    shoc::counts.minmax++;
    float x = a.v, y = b.v;
    if (x != x) return b;
    if (y != y) return a;
    if (x > y) return a;
    if (y > x) return b;
    return std::signbit(x) ? b : a;
}
static inline sh_cf rminf(sh_cf a, sh_cf b) {
    shoc::counts.minmax++;
    float x = a.v, y = b.v;
    if (x != x) return b;
    if (y != y) return a;
    if (x < y) return a;
    if (y < x) return b;
    return std::signbit(x) ? a : b;
}

#define float sh_cf
