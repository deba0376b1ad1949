// Device-side helpers shared by the precompiled kernels (nvcc) and the
// kernels the fusion engine generates at run time (NVRTC): fixed-width
// types, the dtype-code switch, NaN tests that survive fast-math, aligned
// vector loads/stores and 32-bit magic-number division.
#pragma once

#ifdef __CUDACC_RTC__
typedef signed char int8_t;
typedef unsigned char uint8_t;
typedef short int16_t;
typedef unsigned short uint16_t;
typedef int int32_t;
typedef unsigned int uint32_t;
typedef long long int64_t;
typedef unsigned long long uint64_t;
typedef unsigned long long uintptr_t;
#else
#include <stdint.h>
#endif
#include <cuda_fp16.h>

#define MMP_DT_BOOL 0
#define MMP_DT_INT8 1
#define MMP_DT_UINT8 2
#define MMP_DT_INT16 3
#define MMP_DT_UINT16 4
#define MMP_DT_INT32 5
#define MMP_DT_UINT32 6
#define MMP_DT_INT64 7
#define MMP_DT_UINT64 8
#define MMP_DT_FLOAT16 9
#define MMP_DT_FLOAT32 10
#define MMP_DT_FLOAT64 11

namespace mmpd {

// NaN test on the bit pattern, so it is not folded away under fast-math.
__device__ __forceinline__ bool isnan_(float x) {
  return (__float_as_uint(x) & 0x7fffffffu) > 0x7f800000u;
}
__device__ __forceinline__ bool isnan_(double x) {
  return ((unsigned long long)__double_as_longlong(x) & 0x7fffffffffffffffull) >
         0x7ff0000000000000ull;
}
__device__ __forceinline__ bool isnan_(__half x) { return isnan_(__half2float(x)); }
template <class T>
__device__ __forceinline__ bool isnan_(T) { return false; }

// Promotion of a stored element to its arithmetic type: f16 computes in f32
// (the reference casts through float, _fusion.py:86-172), everything else in
// its own type.
template <class T> struct Arith { typedef T type; };
template <> struct Arith<__half> { typedef float type; };
template <> struct Arith<bool> { typedef bool type; };

template <class T> struct IsFloat { static const bool value = false; };
template <> struct IsFloat<float> { static const bool value = true; };
template <> struct IsFloat<double> { static const bool value = true; };
template <> struct IsFloat<__half> { static const bool value = true; };

template <class T> struct IsSigned { static const bool value = T(-1) < T(0); };
template <> struct IsSigned<__half> { static const bool value = true; };

// Conversions between stored types.  bool follows numpy's `!= 0` rule.
template <class D, class S>
struct Cvt { __device__ __forceinline__ static D f(S s) { return (D)s; } };
template <class S> struct Cvt<bool, S> {
  __device__ __forceinline__ static bool f(S s) { return s != S(0); }
};
template <> struct Cvt<bool, bool> { __device__ __forceinline__ static bool f(bool s) { return s; } };
template <> struct Cvt<bool, __half> {
  __device__ __forceinline__ static bool f(__half s) { return __half2float(s) != 0.0f; }
};
template <class S> struct Cvt<__half, S> {
  __device__ __forceinline__ static __half f(S s) { return __float2half_rn((float)s); }
};
template <> struct Cvt<__half, double> {
  __device__ __forceinline__ static __half f(double s) { return __double2half(s); }
};
template <> struct Cvt<__half, __half> { __device__ __forceinline__ static __half f(__half s) { return s; } };
template <class D> struct Cvt<D, __half> {
  __device__ __forceinline__ static D f(__half s) { return (D)__half2float(s); }
};
// float -> integer casts: C++ leaves out-of-range values undefined; numpy on
// x86 yields the "integer indefinite" value.  Match it for NaN/inf/overflow.
template <class D> struct FloatToInt {
  template <class F>
  __device__ __forceinline__ static D f(F s) {
    if (isnan_(s)) return (D)(IsSigned<D>::value ? (D)((unsigned long long)1 << (sizeof(D) * 8 - 1)) : (D)0);
    return (D)s;
  }
};
template <> struct Cvt<int64_t, float> { __device__ __forceinline__ static int64_t f(float s) {
  if (isnan_(s) || !(s > -9.2233720368547758e18f && s < 9.2233720368547758e18f)) return (int64_t)0x8000000000000000ll;
  return (int64_t)s; } };
template <> struct Cvt<int64_t, double> { __device__ __forceinline__ static int64_t f(double s) {
  if (isnan_(s) || !(s > -9.2233720368547758e18 && s < 9.2233720368547758e18)) return (int64_t)0x8000000000000000ll;
  return (int64_t)s; } };
template <> struct Cvt<int32_t, float> { __device__ __forceinline__ static int32_t f(float s) {
  if (isnan_(s) || !(s > -2147483904.0f && s < 2147483648.0f)) return (int32_t)0x80000000;
  return (int32_t)s; } };
template <> struct Cvt<int32_t, double> { __device__ __forceinline__ static int32_t f(double s) {
  if (isnan_(s) || !(s > -2147483649.0 && s < 2147483648.0)) return (int32_t)0x80000000;
  return (int32_t)s; } };

template <class D, class S>
__device__ __forceinline__ D cvt(S s) { return Cvt<D, S>::f(s); }

// Store one scalar into `out[idx]` of runtime dtype `dt`, from either an
// exact integer (is_int) or a double.
__device__ __forceinline__ void store_scalar(void *out, long long idx, int dt, bool is_int,
                                             long long iv, unsigned long long uv, double dv,
                                             bool is_unsigned) {
  switch (dt) {
    case MMP_DT_BOOL: ((bool *)out)[idx] = is_int ? (is_unsigned ? uv != 0 : iv != 0) : dv != 0.0; break;
    case MMP_DT_INT8: ((int8_t *)out)[idx] = is_int ? (int8_t)(is_unsigned ? (long long)uv : iv) : cvt<int8_t>(dv); break;
    case MMP_DT_UINT8: ((uint8_t *)out)[idx] = is_int ? (uint8_t)(is_unsigned ? uv : (unsigned long long)iv) : (uint8_t)cvt<int64_t>(dv); break;
    case MMP_DT_INT16: ((int16_t *)out)[idx] = is_int ? (int16_t)(is_unsigned ? (long long)uv : iv) : (int16_t)cvt<int32_t>(dv); break;
    case MMP_DT_UINT16: ((uint16_t *)out)[idx] = is_int ? (uint16_t)(is_unsigned ? uv : (unsigned long long)iv) : (uint16_t)cvt<int32_t>(dv); break;
    case MMP_DT_INT32: ((int32_t *)out)[idx] = is_int ? (int32_t)(is_unsigned ? (long long)uv : iv) : cvt<int32_t>(dv); break;
    case MMP_DT_UINT32: ((uint32_t *)out)[idx] = is_int ? (uint32_t)(is_unsigned ? uv : (unsigned long long)iv) : (uint32_t)cvt<int64_t>(dv); break;
    case MMP_DT_INT64: ((int64_t *)out)[idx] = is_int ? (is_unsigned ? (long long)uv : iv) : cvt<int64_t>(dv); break;
    case MMP_DT_UINT64: ((uint64_t *)out)[idx] = is_int ? (is_unsigned ? uv : (unsigned long long)iv) : (uint64_t)cvt<int64_t>(dv); break;
    case MMP_DT_FLOAT16: ((__half *)out)[idx] = is_int ? (is_unsigned ? __double2half((double)uv) : __double2half((double)iv)) : __double2half(dv); break;
    case MMP_DT_FLOAT32: ((float *)out)[idx] = is_int ? (is_unsigned ? (float)uv : (float)iv) : (float)dv; break;
    case MMP_DT_FLOAT64: ((double *)out)[idx] = is_int ? (is_unsigned ? (double)uv : (double)iv) : dv; break;
    default: break;
  }
}

// Aligned vector of N elements of T; loads/stores of 4, 8, 16 and 32 bytes
// compile to single vector instructions (two for 32 bytes).
template <class T, int N>
struct __align__(sizeof(T) * N) Vec { T v[N]; };

template <class T, int N>
__device__ __forceinline__ Vec<T, N> ldvec(const T *p) {
  return *reinterpret_cast<const Vec<T, N> *>(p);
}
template <class T, int N>
__device__ __forceinline__ Vec<T, N> ldvec_stream(const T *p) {
  // read-once data: evict-first so it does not push reused lines out of L2
  Vec<T, N> r;
  if (sizeof(Vec<T, N>) == 16) {
    int4 t = __ldcs(reinterpret_cast<const int4 *>(p));
    r = *reinterpret_cast<Vec<T, N> *>(&t);
  } else {
    r = *reinterpret_cast<const Vec<T, N> *>(p);
  }
  return r;
}
template <class T, int N>
__device__ __forceinline__ void stvec(T *p, const Vec<T, N> &v) {
  *reinterpret_cast<Vec<T, N> *>(p) = v;
}
template <class T, int N>
__device__ __forceinline__ void stvec_stream(T *p, const Vec<T, N> &v) {
  if (sizeof(Vec<T, N>) == 16) {
    __stcs(reinterpret_cast<int4 *>(p), *reinterpret_cast<const int4 *>(&v));
  } else {
    *reinterpret_cast<Vec<T, N> *>(p) = v;
  }
}

// Unsigned 32-bit division by a run-time constant d >= 1 with a multiply and
// a shift (Granlund & Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994): q = (umulhi(n, m) + n) >> s, exact for all
// 32-bit n.  The host computes (m, s); d == 1 uses m = 0, s = 0.
struct FastDiv {
  unsigned d, m, s;
  __device__ __forceinline__ unsigned div(unsigned n) const {
    unsigned long long t = (unsigned long long)__umulhi(n, m) + n;
    return (unsigned)(t >> s);
  }
};

}  // namespace mmpd
