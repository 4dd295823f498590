// oracle/opcount.hpp - TEST/MEASUREMENT INFRASTRUCTURE. Compiles oracle/oracle.c as C++ with every `float` replaced
// by a counting type, so running the restatement counts the FP32 operations ggml's algorithm executes, in two kinds:
// arithmetic (each float add, subtract, multiply, divide, square root, round - what the FADD/FMUL issue rate of the
// roofline's denominator measures) and comparisons (each float <, >, <=, >=, ==, != - which issue as FSETP, another
// instruction class). Negation and fabs are sign-bit modifiers, int<->float conversions are not arithmetic: not
// counted. Used by oracle/count_ops.py to define the algorithmic work per weight of each quantizer.
#pragma once
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <type_traits>

extern thread_local unsigned long long g_fops, g_fcmp;

struct cf {
    float v;
    cf() = default;
    constexpr cf(float x) : v(x) {}
    constexpr cf(double x) : v((float) x) {}
    template <typename I, typename std::enable_if<std::is_integral<I>::value, int>::type = 0>
    constexpr cf(I x) : v((float) x) {}
    explicit operator float() const { return v; }
    template <typename I, typename std::enable_if<std::is_integral<I>::value, int>::type = 0>
    explicit operator I() const { return (I) v; }
    explicit operator bool() const { return v != 0; }
    cf operator-() const { return cf(-v); }
    cf & operator+=(cf o) { ++g_fops; v += o.v; return *this; }
    cf & operator-=(cf o) { ++g_fops; v -= o.v; return *this; }
    cf & operator*=(cf o) { ++g_fops; v *= o.v; return *this; }
    cf & operator/=(cf o) { ++g_fops; v /= o.v; return *this; }
};
inline cf operator+(cf a, cf b) { ++g_fops; return cf(a.v + b.v); }
inline cf operator-(cf a, cf b) { ++g_fops; return cf(a.v - b.v); }
inline cf operator*(cf a, cf b) { ++g_fops; return cf(a.v * b.v); }
inline cf operator/(cf a, cf b) { ++g_fops; return cf(a.v / b.v); }
inline bool operator<(cf a, cf b) { ++g_fcmp; return a.v < b.v; }
inline bool operator>(cf a, cf b) { ++g_fcmp; return a.v > b.v; }
inline bool operator<=(cf a, cf b) { ++g_fcmp; return a.v <= b.v; }
inline bool operator>=(cf a, cf b) { ++g_fcmp; return a.v >= b.v; }
inline bool operator==(cf a, cf b) { ++g_fcmp; return a.v == b.v; }
inline bool operator!=(cf a, cf b) { ++g_fcmp; return a.v != b.v; }
inline cf sqrtf(cf a) { ++g_fops; return cf(std::sqrt(a.v)); }
inline cf fabsf(cf a) { return cf(std::fabs(a.v)); }
inline cf roundf(cf a) { ++g_fops; return cf(std::round(a.v)); }
#define float cf
