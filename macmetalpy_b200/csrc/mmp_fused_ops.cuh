// Scalar element functions used by the kernels the fusion engine emits.
//
// The reference builds each fused op from an MSL template
// (src/macmetalpy/_fusion.py:86-264) and its eager shaders
// (_kernels.py:21-404).  Its Metal results are not those of its own CPU
// path in several places (integer floor_divide truncates, _kernels.py:44;
// float floor_divide is floor(a/b), _kernels.py:32).  The functions here
// reproduce the CPU path (numpy calls), bit for bit on the integer and
// division ops:
//   * float floor_divide: numpy's fmod-based divmod with sign and rounding
//     fix-ups (numpy npy_math: npy_divmod / npy_floor_divide, the same steps
//     as CPython's float_divmod); f_remainder is numpy's remainder;
//   * `%` / mod / remainder: the reference's composite
//     x1 - floor_divide(x1, x2) * x2 (math_ops.py:540-548), see ref_mod_f;
//   * integer floor_divide / remainder: floor semantics, division by zero
//     gives 0, INT_MIN // -1 gives INT_MIN;
//   * maximum/minimum propagate NaN, fmax/fmin ignore it, with numpy's
//     comparison order (so signed zeros come out as numpy's do);
//   * logaddexp / logaddexp2: numpy's max + log1p(exp(-|d|)) form.
// Float math calls CUDA's libdevice functions (not reproduced here).
#pragma once
#include "mmp_device.cuh"

namespace mmpf {
using mmpd::isnan_;

// ---- separately rounded + - * of the generated code.  The compiler never
// contracts these into an fma, whatever --fmad says, so a fused expression
// rounds every user-level operation as numpy does; expressions whose other
// ops are all library calls can then be compiled with --fmad=true.
__device__ __forceinline__ float rn_add(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ double rn_add(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ float rn_sub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ double rn_sub(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ float rn_mul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ double rn_mul(double a, double b) { return __dmul_rn(a, b); }

// ---- math dispatch on float / double.  float32 functions whose CUDA
// error bound is above 2 ulp (tan, sinh, cosh, asinh, acosh, atanh, pow,
// atan2, hypot) are evaluated in double and rounded once.
__device__ __forceinline__ float m_sqrt(float x) { return sqrtf(x); }
__device__ __forceinline__ double m_sqrt(double x) { return sqrt(x); }
__device__ __forceinline__ float m_exp(float x) { return expf(x); }
__device__ __forceinline__ double m_exp(double x) { return exp(x); }
__device__ __forceinline__ float m_log(float x) { return logf(x); }
__device__ __forceinline__ double m_log(double x) { return log(x); }
__device__ __forceinline__ float m_sin(float x) { return sinf(x); }
__device__ __forceinline__ double m_sin(double x) { return sin(x); }
__device__ __forceinline__ float m_cos(float x) { return cosf(x); }
__device__ __forceinline__ double m_cos(double x) { return cos(x); }
__device__ __forceinline__ float m_tan(float x) { return (float)tan((double)x); }
__device__ __forceinline__ double m_tan(double x) { return tan(x); }
__device__ __forceinline__ float m_asin(float x) { return asinf(x); }
__device__ __forceinline__ double m_asin(double x) { return asin(x); }
__device__ __forceinline__ float m_acos(float x) { return acosf(x); }
__device__ __forceinline__ double m_acos(double x) { return acos(x); }
__device__ __forceinline__ float m_atan(float x) { return atanf(x); }
__device__ __forceinline__ double m_atan(double x) { return atan(x); }
__device__ __forceinline__ float m_sinh(float x) { return (float)sinh((double)x); }
__device__ __forceinline__ double m_sinh(double x) { return sinh(x); }
__device__ __forceinline__ float m_cosh(float x) { return (float)cosh((double)x); }
__device__ __forceinline__ double m_cosh(double x) { return cosh(x); }
__device__ __forceinline__ float m_tanh(float x) { return tanhf(x); }
__device__ __forceinline__ double m_tanh(double x) { return tanh(x); }
__device__ __forceinline__ float m_log2(float x) { return log2f(x); }
__device__ __forceinline__ double m_log2(double x) { return log2(x); }
__device__ __forceinline__ float m_log10(float x) { return log10f(x); }
__device__ __forceinline__ double m_log10(double x) { return log10(x); }
__device__ __forceinline__ float m_exp2(float x) { return exp2f(x); }
__device__ __forceinline__ double m_exp2(double x) { return exp2(x); }
__device__ __forceinline__ float m_expm1(float x) { return expm1f(x); }
__device__ __forceinline__ double m_expm1(double x) { return expm1(x); }
__device__ __forceinline__ float m_log1p(float x) { return log1pf(x); }
__device__ __forceinline__ double m_log1p(double x) { return log1p(x); }
__device__ __forceinline__ float m_cbrt(float x) { return cbrtf(x); }
__device__ __forceinline__ double m_cbrt(double x) { return cbrt(x); }
__device__ __forceinline__ float m_asinh(float x) { return (float)asinh((double)x); }
__device__ __forceinline__ double m_asinh(double x) { return asinh(x); }
__device__ __forceinline__ float m_acosh(float x) { return (float)acosh((double)x); }
__device__ __forceinline__ double m_acosh(double x) { return acosh(x); }
__device__ __forceinline__ float m_atanh(float x) { return (float)atanh((double)x); }
__device__ __forceinline__ double m_atanh(double x) { return atanh(x); }
__device__ __forceinline__ float m_floor(float x) { return floorf(x); }
__device__ __forceinline__ double m_floor(double x) { return floor(x); }
__device__ __forceinline__ float m_ceil(float x) { return ceilf(x); }
__device__ __forceinline__ double m_ceil(double x) { return ceil(x); }
__device__ __forceinline__ float m_trunc(float x) { return truncf(x); }
__device__ __forceinline__ double m_trunc(double x) { return trunc(x); }
__device__ __forceinline__ float m_rint(float x) { return rintf(x); }
__device__ __forceinline__ double m_rint(double x) { return rint(x); }
__device__ __forceinline__ float m_fabs(float x) { return fabsf(x); }
__device__ __forceinline__ double m_fabs(double x) { return fabs(x); }
// Exact fmod.  The remainder a - n*b (n = trunc(a/b)) is always
// representable, so when the quotient is below 2^24 (2^53 for double) it is
// computed directly: q = trunc(|a|/|b|) is the true quotient or one above
// it (rounding of the division can only carry up to the next integer), and
// fma(-q, |b|, |a|) is then exactly the remainder, or negative, in which case
// q - 1 gives it.  Larger quotients, infinities, NaN and b == 0 take the
// library fmod.  Bit-identical to fmodf/fmod, several times cheaper.
__device__ __forceinline__ float m_fmod(float a, float b) {
  float ab = fabsf(a), bb = fabsf(b);
  if (ab < bb * 16777216.0f && bb > 0.0f && bb <= 3.402823466e38f) {
    float q = truncf(ab / bb);
    float r = fmaf(-q, bb, ab);
    if (r < 0.0f) r = fmaf(-(q - 1.0f), bb, ab);
    return copysignf(r, a);
  }
  return fmodf(a, b);
}
__device__ __forceinline__ double m_fmod(double a, double b) {
  double ab = fabs(a), bb = fabs(b);
  if (ab < bb * 9007199254740992.0 && bb > 0.0 && bb <= 1.7976931348623157e308) {
    double q = trunc(ab / bb);
    double r = fma(-q, bb, ab);
    if (r < 0.0) r = fma(-(q - 1.0), bb, ab);
    return copysign(r, a);
  }
  return fmod(a, b);
}
__device__ __forceinline__ float m_pow(float a, float b) { return (float)pow((double)a, (double)b); }
__device__ __forceinline__ double m_pow(double a, double b) { return pow(a, b); }
__device__ __forceinline__ float m_atan2(float a, float b) { return (float)atan2((double)a, (double)b); }
__device__ __forceinline__ double m_atan2(double a, double b) { return atan2(a, b); }
__device__ __forceinline__ float m_hypot(float a, float b) { return (float)hypot((double)a, (double)b); }
__device__ __forceinline__ double m_hypot(double a, double b) { return hypot(a, b); }
__device__ __forceinline__ float m_copysign(float a, float b) { return copysignf(a, b); }
__device__ __forceinline__ double m_copysign(double a, double b) { return copysign(a, b); }
__device__ __forceinline__ float m_nextafter(float a, float b) { return nextafterf(a, b); }
__device__ __forceinline__ double m_nextafter(double a, double b) { return nextafter(a, b); }

template <class R> struct Consts;
template <> struct Consts<float> {
  __device__ static float loge2() { return 0.693147180559945309417232121458176568f; }
  __device__ static float log2e() { return 1.442695040888963407359924681001892137f; }
  __device__ static float nan() { return __int_as_float(0x7fc00000); }
};
template <> struct Consts<double> {
  __device__ static double loge2() { return 0.693147180559945309417232121458176568; }
  __device__ static double log2e() { return 1.442695040888963407359924681001892137; }
  __device__ static double nan() { return __longlong_as_double(0x7ff8000000000000ll); }
};

// ---- float divmod (numpy npy_divmod)
template <class R>
__device__ __forceinline__ R f_floor_divide(R a, R b) {
  if (b == R(0)) return a / b;  // inf or nan, as numpy
  R mod = m_fmod(a, b);
  R div = (a - mod) / b;
  if (mod != R(0)) {
    if ((b < R(0)) != (mod < R(0))) {
      mod += b;
      div -= R(1);
    }
  }
  R floordiv;
  if (div != R(0)) {
    floordiv = m_floor(div);
    if (div - floordiv > R(0.5)) floordiv += R(1);
  } else {
    floordiv = m_copysign(R(0), a / b);
  }
  return floordiv;
}

// float32 floor_divide with the same result as numpy's algorithm above,
// cheaper: for |a/b| < 2^20 with a normal, finite b, the truncated quotient q
// and remainder r of |a| / |b| are found exactly (approximate division, then
// an exact fma remainder that corrects q by one either way), and numpy's
// result is then s*q, minus one when r != 0 and the signs differ (s < 0),
// with numpy's signed zero when q == 0.  In that range numpy's own f32
// steps (fmod, (a - mod) / b, floor, snap) land exactly on that integer: the
// rounding of (a - mod) / b stays within q * 2^-23 < 1/8 of it.  Everything
// else takes f_floor_divide.
__device__ __forceinline__ float f_floor_divide_fast(float a, float b) {
  const float ab = fabsf(a), bb = fabsf(b);
  if (ab < bb * 1048576.0f && bb >= 1.17549435e-38f && bb < 8.50705917e37f) {
    float q = truncf(__fdividef(ab, bb));
    float r = fmaf(-q, bb, ab);
    if (r < 0.0f) {
      q -= 1.0f;
      r = fmaf(-q, bb, ab);
    } else if (r >= bb) {
      q += 1.0f;
      r = fmaf(-q, bb, ab);
    }
    const bool neg = (__float_as_uint(a) ^ __float_as_uint(b)) >> 31;
    if (q == 0.0f) {
      if (r == 0.0f) return neg ? -0.0f : 0.0f;
      return neg ? -1.0f : 0.0f;
    }
    return neg ? -(q + (r != 0.0f ? 1.0f : 0.0f)) : q;
  }
  return f_floor_divide<float>(a, b);
}
template <class R> __device__ __forceinline__ R floor_divide_f(R a, R b) { return f_floor_divide<R>(a, b); }
template <> __device__ __forceinline__ float floor_divide_f<float>(float a, float b) {
  return f_floor_divide_fast(a, b);
}

template <class R>
__device__ __forceinline__ R f_remainder(R a, R b) {
  R mod = m_fmod(a, b);
  if (b == R(0)) return mod;  // nan
  if (mod != R(0)) {
    if ((b < R(0)) != (mod < R(0))) mod += b;
  } else {
    mod = m_copysign(R(0), b);
  }
  return mod;
}

// ---- integer floor division / remainder (numpy semantics)
template <class I>
__device__ __forceinline__ I i_floor_divide(I a, I b) {
  if (b == I(0)) return I(0);
  if (mmpd::IsSigned<I>::value) {
    if (b == I(-1)) return (I)(I(0) - a);  // wraps INT_MIN to INT_MIN
    I q = a / b;
    I r = (I)(a - q * b);  // one division: the remainder from the quotient
    if (r != I(0) && ((r < I(0)) != (b < I(0)))) q -= I(1);
    return q;
  }
  return a / b;
}

// int32 floor division for |a| < 2^21, |b| < 2^24 through float: both
// convert exactly, |a/b| < 2^21 so the 2-ulp approximate quotient is within
// 1/2 of a/b, its truncation q0 is within {-1, 0, +1, +2} of the floor, and
// the exact integer remainder a - q*b steers q onto the floor quotient in
// at most two steps.  Everything else takes the integer division.
__device__ __forceinline__ int i32_floor_divide(int a, int b) {
  const unsigned ua = (unsigned)(a < 0 ? -a : a), ub = (unsigned)(b < 0 ? -b : b);
  if (b != 0 && ua < (1u << 21) && ub < (1u << 24)) {
    // corrections as selects (no divergent branches inside the fast path)
    int q = (int)truncf(__fdividef((float)a, (float)b));
    int r = a - q * b;
    const bool pos = b > 0;
    bool c = pos ? (r < 0) : (r > 0);
    q -= c ? 1 : 0;
    r += c ? b : 0;
    c = pos ? (r < 0) : (r > 0);
    q -= c ? 1 : 0;
    r += c ? b : 0;
    q += (pos ? (r >= b) : (r <= b)) ? 1 : 0;
    return q;
  }
  return i_floor_divide<int>(a, b);
}
template <class I> __device__ __forceinline__ I floor_divide_i(I a, I b) { return i_floor_divide<I>(a, b); }
template <> __device__ __forceinline__ int floor_divide_i<int>(int a, int b) { return i32_floor_divide(a, b); }

template <class I>
__device__ __forceinline__ I i_remainder(I a, I b) {
  if (b == I(0)) return I(0);
  if (mmpd::IsSigned<I>::value) {
    if (b == I(-1)) return I(0);
    I r = a % b;
    if (r != I(0) && ((r < I(0)) != (b < I(0)))) r += b;
    return r;
  }
  return a % b;
}

// The reference's mod / remainder / `%` is the composite
// x1 - floor_divide(x1, x2) * x2 (src/macmetalpy/math_ops.py:540-548), each
// step rounded to the array dtype T as its CPU path (numpy) evaluates it.
// This is not np.remainder for floats; it is what the reference returns.
template <class T, class R>
__device__ __forceinline__ R ref_mod_f(R a, R b) {
  R fd = mmpd::cvt<R>(mmpd::cvt<T>(floor_divide_f<R>(a, b)));
  R t = mmpd::cvt<R>(mmpd::cvt<T>(fd * b));
  return a - t;
}
template <class I>
__device__ __forceinline__ I ref_mod_i(I a, I b) {
  I fd = floor_divide_i<I>(a, b);
  I t = (I)(fd * b);
  return (I)(a - t);
}

template <class I>
__device__ __forceinline__ I i_fmod(I a, I b) {
  if (b == I(0)) return I(0);
  if (mmpd::IsSigned<I>::value && b == I(-1)) return I(0);
  return a % b;
}

// integer power by squaring; negative exponents give 0 (numpy raises)
template <class I>
__device__ __forceinline__ I i_power(I a, I b) {
  if (mmpd::IsSigned<I>::value && b < I(0)) return I(0);
  I r = I(1);
  I base = a;
  unsigned long long e = (unsigned long long)b;
  while (e) {
    if (e & 1ull) r = (I)(r * base);
    base = (I)(base * base);
    e >>= 1;
  }
  return r;
}

// ---- max/min with numpy's NaN rules
// isinf / isfinite / signbit on the bit pattern (not folded under
// fast-math); integers and bool are finite, and signbit of an integer is
// its sign (numpy computes it through a float loop, same answer).
template <class R>
__device__ __forceinline__ bool isinf_(R) { return false; }
__device__ __forceinline__ bool isinf_(float x) { return (__float_as_uint(x) & 0x7fffffffu) == 0x7f800000u; }
__device__ __forceinline__ bool isinf_(double x) {
  return ((unsigned long long)__double_as_longlong(x) & 0x7fffffffffffffffull) == 0x7ff0000000000000ull;
}
template <class R>
__device__ __forceinline__ bool isfinite_(R) { return true; }
__device__ __forceinline__ bool isfinite_(float x) { return (__float_as_uint(x) & 0x7fffffffu) < 0x7f800000u; }
__device__ __forceinline__ bool isfinite_(double x) {
  return ((unsigned long long)__double_as_longlong(x) & 0x7fffffffffffffffull) < 0x7ff0000000000000ull;
}
template <class R>
__device__ __forceinline__ bool signbit_(R x) { return x < R(0); }
__device__ __forceinline__ bool signbit_(float x) { return (__float_as_uint(x) >> 31) != 0u; }
__device__ __forceinline__ bool signbit_(double x) {
  return ((unsigned long long)__double_as_longlong(x) >> 63) != 0ull;
}

// numpy's shifts (npy_lshift / npy_rshift): a shift count outside
// [0, bits) gives 0 (left) or the sign fill (right); the count is compared
// as an unsigned value, so a negative count is out of range.
template <class R>
__device__ __forceinline__ R shl_(R a, R b) {
  return ((unsigned long long)(long long)b < sizeof(R) * 8ull) ? (R)((unsigned long long)(long long)a << (int)b)
                                                              : R(0);
}
template <class R>
__device__ __forceinline__ R shr_(R a, R b) {
  if ((unsigned long long)(long long)b < sizeof(R) * 8ull) return (R)(a >> (int)b);
  return (a < R(0)) ? (R)(~R(0)) : R(0);
}

template <class R>
__device__ __forceinline__ R maximum(R a, R b) { return (a >= b || isnan_(a)) ? a : b; }
template <class R>
__device__ __forceinline__ R minimum(R a, R b) { return (a <= b || isnan_(a)) ? a : b; }
template <class R>
__device__ __forceinline__ R fmax_(R a, R b) { return (a >= b || isnan_(b)) ? a : b; }
template <class R>
__device__ __forceinline__ R fmin_(R a, R b) { return (a <= b || isnan_(b)) ? a : b; }

// ---- logaddexp (numpy npy_logaddexp / npy_logaddexp2)
// log1p(t) for t = exp(-|x - y|) in (0, 1].  Below 2^-12 the series
// t - t^2/2 is exact to t^3/3 < t * 2^-24 / 3 (under a sixth of an ulp of
// t), so the library log1p is only needed for |x - y| < 12 ln 2.
template <class R>
__device__ __forceinline__ R log1p_of_exp(R t) {
  return (t < R(2.44140625e-4)) ? (t - R(0.5) * t * t) : m_log1p(t);
}
// numpy's npy_logaddexp: x == y -> x + ln 2 (equal infinities without nan);
// otherwise max(x, y) + log1p(exp(-|x - y|)); nan in, nan out.  Written
// with one divergent branch (inside log1p_of_exp) and selects for the
// special cases, so a warp runs the exp once and the library log1p only
// when one of its lanes needs it.
template <class R>
__device__ __forceinline__ R logaddexp(R x, R y) {
  const R tmp = x - y;
  const R mx = (tmp > R(0)) ? x : y;
  const R r = mx + log1p_of_exp(m_exp(-fabs(tmp)));
  return (x == y) ? x + Consts<R>::loge2() : ((tmp != tmp) ? tmp : r);
}
template <class R>
__device__ __forceinline__ R log2_1p(R x) { return Consts<R>::log2e() * m_log1p(x); }
template <class R>
__device__ __forceinline__ R logaddexp2(R x, R y) {  // numpy's npy_logaddexp2, same structure as logaddexp
  const R tmp = x - y;
  const R mx = (tmp > R(0)) ? x : y;
  const R r = mx + log2_1p(m_exp2(-fabs(tmp)));
  return (x == y) ? x + R(1) : ((tmp != tmp) ? tmp : r);
}

template <class R>
__device__ __forceinline__ R sign_(R a) {
  return a > R(0) ? R(1) : (a < R(0) ? R(-1) : (a == R(0) ? R(0) : a));
}

template <class R>
__device__ __forceinline__ R heaviside(R a, R h) {
  if (isnan_(a)) return a;
  if (a == R(0)) return h;
  return a < R(0) ? R(0) : R(1);
}

template <class I>
__device__ __forceinline__ I i_abs(I a) {
  return (mmpd::IsSigned<I>::value && a < I(0)) ? (I)(I(0) - a) : a;
}

}  // namespace mmpf
