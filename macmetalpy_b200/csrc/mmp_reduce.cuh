// Reduction kernels for sm_100a: full (one launch, last block finishes),
// per-row (axis over contiguous elements) and per-column (axis with a
// contiguous inner extent, split along the reduced axis when the column
// count alone cannot fill the GPU).
//
// Reference kernels these replace: reduce_sum/max/min/prod and reduce_dot
// (src/macmetalpy/_kernels.py:422-594, a multi-launch tree driven from
// ndarray._reduce at ndarray.py:1927-1946), nan_reduce_* (_kernels.py:612-730,
// partials finished on the CPU at nan_ops.py:89-98), the one-thread-per-row
// axis kernels (_kernels.py:1062-1146, after a transpose copy at
// ndarray.py:2039-2047) and the two-pass argmax (_kernels.py:1189-1257).
// Results follow numpy (the reference's CPU path): int sums accumulate in
// 64 bits, argmax/argmin take the first index of the extreme value and the
// first NaN wins, mean/var are computed in double.
//
// The element loader `L` is a template parameter: the precompiled kernels
// read a contiguous array, the fusion engine passes a loader that evaluates
// an elementwise expression, so `sum(f(x))` reads x once and never writes
// f(x) to memory.
#pragma once
#include "mmp_device.cuh"

#define MMP_R_SUM 0
#define MMP_R_PROD 1
#define MMP_R_MAX 2
#define MMP_R_MIN 3
#define MMP_R_MEAN 4
#define MMP_R_VAR 5
#define MMP_R_STD 6
#define MMP_R_ARGMAX 7
#define MMP_R_ARGMIN 8
#define MMP_R_NANSUM 9
#define MMP_R_NANMEAN 10
#define MMP_R_NANMAX 11
#define MMP_R_NANMIN 12
#define MMP_R_ANY 13
#define MMP_R_ALL 14
#define MMP_R_NANVAR 15
#define MMP_R_NANSTD 16

namespace mmpd {

// Device mirror of mmp_partial (include/mmp_cuda.h).
struct PartialOut {
  double s1, s2, shift;
  long long count, ival, index;
};

constexpr int RBLOCK = 256;

// ---------------------------------------------------------------- shuffles
template <class A>
__device__ __forceinline__ A shfl_down(const A &a, int delta) {
  static_assert(sizeof(A) % 4 == 0, "accumulator must be a multiple of 4 bytes");
  A r;
  const unsigned *src = reinterpret_cast<const unsigned *>(&a);
  unsigned *dst = reinterpret_cast<unsigned *>(&r);
#pragma unroll
  for (int i = 0; i < (int)(sizeof(A) / 4); ++i) dst[i] = __shfl_down_sync(0xffffffffu, src[i], delta);
  return r;
}

template <class A>
__device__ __forceinline__ A load_cg(const A *p) {
  A r;
  const unsigned *src = reinterpret_cast<const unsigned *>(p);
  unsigned *dst = reinterpret_cast<unsigned *>(&r);
#pragma unroll
  for (int i = 0; i < (int)(sizeof(A) / 4); ++i) dst[i] = __ldcg(src + i);
  return r;
}

// ---------------------------------------------------------------- type maps
template <class T> struct SumAcc { typedef long long type; };
template <> struct SumAcc<unsigned char> { typedef unsigned long long type; };
template <> struct SumAcc<unsigned short> { typedef unsigned long long type; };
template <> struct SumAcc<unsigned int> { typedef unsigned long long type; };
template <> struct SumAcc<unsigned long long> { typedef unsigned long long type; };
template <> struct SumAcc<float> { typedef double type; };
template <> struct SumAcc<__half> { typedef double type; };
template <> struct SumAcc<double> { typedef double type; };

template <class T> struct AsF { __device__ __forceinline__ static float f(T v) { return (float)v; } };
template <> struct AsF<__half> { __device__ __forceinline__ static float f(__half v) { return __half2float(v); } };
template <class T> __device__ __forceinline__ double as_d(T v) { return (double)v; }
template <> __device__ __forceinline__ double as_d<__half>(__half v) { return (double)__half2float(v); }
template <class T> __device__ __forceinline__ typename Arith<T>::type ar(T v) { return (typename Arith<T>::type)v; }
template <> __device__ __forceinline__ float ar<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ bool ar<bool>(bool v) { return v; }

template <class A>
__device__ __forceinline__ void store_acc_value(void *out, long long idx, int dt, A v) {
  store_scalar(out, idx, dt, true, (long long)v, (unsigned long long)v, 0.0, !IsSigned<A>::value);
}
__device__ __forceinline__ void store_acc_value(void *out, long long idx, int dt, double v) {
  store_scalar(out, idx, dt, false, 0, 0, v, false);
}
__device__ __forceinline__ void store_acc_value(void *out, long long idx, int dt, float v) {
  store_scalar(out, idx, dt, false, 0, 0, (double)v, false);
}

__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float min_nan(float a, float b) {
  float r;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// ---------------------------------------------------------------- ops
// four(acc, v0..v3, idx) folds four successive values of one reduction
// (consecutive rows of the column kernel); ops without a cheaper form
// apply one() four times.
// Every op provides: Acc, init(), start(first_value), one(acc, v, idx),
// vec<V>(acc, v[], base), combine(a, b), finish(acc, n, out, idx, dt, ddof, part).

template <int OPC, class T> struct RedOp;

// sum / mean: float inputs add vectors in f32 and carry the total in f64;
// integers add exactly in 64 bits (numpy's int32 sum gives int64).
template <class T, bool MEAN>
struct SumLike {
  typedef typename SumAcc<T>::type Acc;
  __device__ static Acc init() { return Acc(0); }
  __device__ static Acc start(Acc a, T) { return a; }
  __device__ static void one(Acc &a, T v, long long) {
    if (IsFloat<T>::value && sizeof(T) < 8) a += (Acc)AsF<T>::f(v);
    else a += (Acc)ar(v);
  }
  template <int V>
  __device__ static void vec(Acc &a, const T (&v)[V], long long) {
    if (IsFloat<T>::value && sizeof(T) < 8) {
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < V; ++j) s += AsF<T>::f(v[j]);
      a += (Acc)s;
    } else if (!IsFloat<T>::value && sizeof(T) <= 2 && V <= 8) {
      // bool / 8- and 16-bit integers: a vector's sum fits 32 bits, one
      // 64-bit add per vector instead of one per element
      int s = 0;
#pragma unroll
      for (int j = 0; j < V; ++j) s += (int)ar(v[j]);
      a += (Acc)s;
    } else {
#pragma unroll
      for (int j = 0; j < V; ++j) a += (Acc)ar(v[j]);
    }
  }
  __device__ static void four(Acc &a, T v0, T v1, T v2, T v3, long long) {
    if (IsFloat<T>::value && sizeof(T) < 8) {
      a += (Acc)((AsF<T>::f(v0) + AsF<T>::f(v1)) + (AsF<T>::f(v2) + AsF<T>::f(v3)));
    } else {
      a += (Acc)ar(v0);
      a += (Acc)ar(v1);
      a += (Acc)ar(v2);
      a += (Acc)ar(v3);
    }
  }
  __device__ static Acc combine(Acc a, Acc b) { return a + b; }
  __device__ static void finish(Acc a, long long n, void *out, long long idx, int dt, double,
                                PartialOut *p) {
    if (MEAN) {
      store_acc_value(out, idx, dt, (double)a / (double)n);
    } else {
      store_acc_value(out, idx, dt, a);
    }
    if (p) {
      p->s1 = (double)a;
      p->count = n;
      p->ival = (long long)a;
    }
  }
};
template <class T> struct RedOp<MMP_R_SUM, T> : SumLike<T, false> {};
template <class T> struct RedOp<MMP_R_MEAN, T> : SumLike<T, true> {};

template <class T> struct ProdAcc { typedef typename SumAcc<T>::type type; };
template <class T>
struct RedOp<MMP_R_PROD, T> {
  typedef typename ProdAcc<T>::type Acc;
  __device__ static Acc init() { return Acc(1); }
  __device__ static Acc start(Acc a, T) { return a; }
  __device__ static void one(Acc &a, T v, long long) { a *= (Acc)ar(v); }
  template <int V>
  __device__ static void vec(Acc &a, const T (&v)[V], long long) {
#pragma unroll
    for (int j = 0; j < V; ++j) a *= (Acc)ar(v[j]);
  }
  __device__ static void four(Acc &a, T v0, T v1, T v2, T v3, long long i) {
    one(a, v0, i);
    one(a, v1, i);
    one(a, v2, i);
    one(a, v3, i);
  }
  __device__ static Acc combine(Acc a, Acc b) { return a * b; }
  __device__ static void finish(Acc a, long long n, void *out, long long idx, int dt, double,
                                PartialOut *p) {
    store_acc_value(out, idx, dt, a);
    if (p) {
      p->s1 = (double)a;
      p->ival = (long long)a;
      p->count = n;
    }
  }
};

// max / min (NaN propagates, numpy.maximum.reduce) and nanmax / nanmin
// (NaN ignored; all-NaN gives NaN).
template <class T, bool MAX, bool IGNORE_NAN>
struct ExtremeOp {
  typedef typename Arith<T>::type V_;
  struct Acc {
    V_ v;
    int has;
  };
  __device__ static Acc init() {
    Acc a;
    a.v = V_(0);
    a.has = 0;
    return a;
  }
  __device__ static Acc start(Acc a, T) { return a; }
  __device__ static Acc pick(Acc a, Acc b) {
    if (!a.has) return b;
    if (!b.has) return a;
    bool an = isnan_(a.v), bn = isnan_(b.v);
    if (IGNORE_NAN) {
      if (an) return b;
      if (bn) return a;
    } else {
      if (an) return a;
      if (bn) return b;
    }
    if (MAX) return (b.v > a.v) ? b : a;
    return (b.v < a.v) ? b : a;
  }
  __device__ static void one(Acc &a, T v, long long) {
    Acc b;
    b.v = ar(v);
    b.has = 1;
    a = pick(a, b);
  }
  template <int V>
  __device__ static void vec(Acc &a, const T (&v)[V], long long) {
#pragma unroll
    for (int j = 0; j < V; ++j) one(a, v[j], 0);
  }
  __device__ static void four(Acc &a, T v0, T v1, T v2, T v3, long long i) {
    one(a, v0, i);
    one(a, v1, i);
    one(a, v2, i);
    one(a, v3, i);
  }
  __device__ static Acc combine(Acc a, Acc b) { return pick(a, b); }
  __device__ static void finish(Acc a, long long n, void *out, long long idx, int dt, double,
                                PartialOut *p) {
    store_acc_value(out, idx, dt, a.v);
    if (p) {
      p->s1 = as_d(a.v);
      p->ival = IsFloat<T>::value ? 0 : (long long)a.v;
      p->count = a.has ? n : 0;
    }
  }
};
template <class T> struct RedOp<MMP_R_MAX, T> : ExtremeOp<T, true, false> {};
template <class T> struct RedOp<MMP_R_MIN, T> : ExtremeOp<T, false, false> {};
template <class T> struct RedOp<MMP_R_NANMAX, T> : ExtremeOp<T, true, true> {};
template <class T> struct RedOp<MMP_R_NANMIN, T> : ExtremeOp<T, false, true> {};

// var / std in one pass: every element is shifted by the first element K of
// its reduction, S1 = sum(x-K) and S2 = sum((x-K)^2) are additive across
// threads, blocks and GPUs, and var = (S2 - S1^2/n) / (n - ddof).  The shift
// removes the cancellation of the textbook E[x^2]-E[x]^2 formula.
template <class T, bool STD>
struct VarOp {
  struct Acc {
    double s1, s2, k;
  };
  __device__ static Acc init() {
    Acc a;
    a.s1 = 0.0;
    a.s2 = 0.0;
    a.k = 0.0;
    return a;
  }
  __device__ static Acc start(Acc a, T first) {
    a.k = as_d(first);
    return a;
  }
  __device__ static void one(Acc &a, T v, long long) {
    double d = as_d(v) - a.k;
    a.s1 += d;
    a.s2 += d * d;
  }
  template <int V>
  __device__ static void vec(Acc &a, const T (&v)[V], long long) {
    if (IsFloat<T>::value && sizeof(T) < 8) {
      float kf = (float)a.k, f1 = 0.f, f2 = 0.f;
#pragma unroll
      for (int j = 0; j < V; ++j) {
        float d = AsF<T>::f(v[j]) - kf;
        f1 += d;
        f2 += d * d;
      }
      a.s1 += (double)f1;
      a.s2 += (double)f2;
    } else {
#pragma unroll
      for (int j = 0; j < V; ++j) one(a, v[j], 0);
    }
  }
  __device__ static void four(Acc &a, T v0, T v1, T v2, T v3, long long i) {
    if (IsFloat<T>::value && sizeof(T) < 8) {
      const float kf = (float)a.k;
      const float d0 = AsF<T>::f(v0) - kf, d1 = AsF<T>::f(v1) - kf, d2 = AsF<T>::f(v2) - kf,
                  d3 = AsF<T>::f(v3) - kf;
      a.s1 += (double)((d0 + d1) + (d2 + d3));
      a.s2 += (double)((d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3));
    } else {
      one(a, v0, i);
      one(a, v1, i);
      one(a, v2, i);
      one(a, v3, i);
    }
  }
  __device__ static Acc combine(Acc a, Acc b) {
    a.s1 += b.s1;
    a.s2 += b.s2;
    return a;
  }
  __device__ static void finish(Acc a, long long n, void *out, long long idx, int dt, double ddof,
                                PartialOut *p) {
    double dn = (double)n;
    double m2 = a.s2 - a.s1 * a.s1 / dn;
    if (m2 < 0.0) m2 = 0.0;
    double denom = dn - ddof;
    if (denom < 0.0) denom = 0.0;
    double var = m2 / denom;
    store_acc_value(out, idx, dt, STD ? sqrt(var) : var);
    if (p) {
      p->s1 = a.s1;
      p->s2 = a.s2;
      p->shift = a.k;
      p->count = n;
    }
  }
};
template <class T> struct RedOp<MMP_R_VAR, T> : VarOp<T, false> {};
template <class T> struct RedOp<MMP_R_STD, T> : VarOp<T, true> {};

// argmax / argmin: (value, index) pairs; the larger (smaller) value wins,
// equal values keep the lower index, and NaN beats every number (numpy
// returns the index of the first NaN).
template <class T, bool MAX>
struct ArgOp {
  typedef typename Arith<T>::type V_;
  struct Acc {
    V_ v;
    long long i;
  };
  __device__ static Acc init() {
    Acc a;
    a.v = V_(0);
    a.i = -1;
    return a;
  }
  __device__ static Acc start(Acc a, T) { return a; }
  __device__ static Acc pick(const Acc &a, const Acc &b) {
    if (b.i < 0) return a;
    if (a.i < 0) return b;
    bool an = isnan_(a.v), bn = isnan_(b.v);
    if (an || bn) {
      if (an && bn) return (b.i < a.i) ? b : a;
      return an ? a : b;
    }
    if (MAX) {
      if (b.v > a.v) return b;
      if (a.v > b.v) return a;
    } else {
      if (b.v < a.v) return b;
      if (a.v < b.v) return a;
    }
    return (b.i < a.i) ? b : a;
  }
  // One accumulator sees its indices in increasing order in every kernel
  // here, so a strict comparison keeps the first occurrence, and a NaN,
  // once held, is never replaced (the first NaN wins).
  __device__ static void one(Acc &a, T v, long long idx) {
    const V_ x = ar(v);
    const bool take = (a.i < 0) || (!isnan_(a.v) && (isnan_(x) || (MAX ? (x > a.v) : (x < a.v))));
    if (take) {
      a.v = x;
      a.i = idx;
    }
  }
  // float / half vectors: the NaN-propagating vector extreme first; the
  // position of its first occurrence is only searched when it beats the
  // running value (rare once a few vectors are in).
  template <int V>
  __device__ static void vec(Acc &a, const T (&v)[V], long long base) {
    if constexpr (IsFloat<T>::value && sizeof(T) <= 4) {
      float m = AsF<T>::f(v[0]);
#pragma unroll
      for (int j = 1; j < V; ++j) m = MAX ? max_nan(m, AsF<T>::f(v[j])) : min_nan(m, AsF<T>::f(v[j]));
      const bool mn = isnan_(m);
      const bool take = (a.i < 0) || (!isnan_(a.v) && (mn || (MAX ? (m > a.v) : (m < a.v))));
      if (take) {
        int jj = V - 1;
#pragma unroll
        for (int j = V - 1; j >= 0; --j) {
          const float x = AsF<T>::f(v[j]);
          if (mn ? isnan_(x) : (x == m)) jj = j;
        }
        a.v = m;
        a.i = base + jj;
      }
    } else {
#pragma unroll
      for (int j = 0; j < V; ++j) one(a, v[j], base + j);
    }
  }
  // Deferred first-occurrence search (float / half): the loop keeps the
  // running extreme pm, the first of its step's four vectors that holds it
  // (values in pv, first element index pg), branch-free; the index inside
  // that vector is searched once after the loop.  Searching inside the loop
  // cost the whole warp a divergent search whenever any one lane found a
  // new extreme -- nearly every step early on; reloading the step after the
  // loop instead of keeping pv cost a DRAM burst per 16-byte vector (27 %
  // more DRAM reads at 2^26 float32).
  static constexpr bool kGroupDeferred = IsFloat<T>::value && sizeof(T) <= 4;
  template <int V>
  __device__ static void group_step(float &pm, long long &pg, T (&pv)[V], const T (&v0)[V], const T (&v1)[V],
                                    const T (&v2)[V], const T (&v3)[V], long long g0, long long step) {
    float m0 = AsF<T>::f(v0[0]), m1 = AsF<T>::f(v1[0]), m2 = AsF<T>::f(v2[0]), m3 = AsF<T>::f(v3[0]);
#pragma unroll
    for (int j = 1; j < V; ++j) {
      m0 = MAX ? max_nan(m0, AsF<T>::f(v0[j])) : min_nan(m0, AsF<T>::f(v0[j]));
      m1 = MAX ? max_nan(m1, AsF<T>::f(v1[j])) : min_nan(m1, AsF<T>::f(v1[j]));
      m2 = MAX ? max_nan(m2, AsF<T>::f(v2[j])) : min_nan(m2, AsF<T>::f(v2[j]));
      m3 = MAX ? max_nan(m3, AsF<T>::f(v3[j])) : min_nan(m3, AsF<T>::f(v3[j]));
    }
    const float m = MAX ? max_nan(max_nan(m0, m1), max_nan(m2, m3)) : min_nan(min_nan(m0, m1), min_nan(m2, m3));
    const bool mn = isnan_(m);
    // the same rule as vec4: a strictly better value or the first NaN
    const bool take = (pg < 0) || (!isnan_(pm) && (mn || (MAX ? (m > pm) : (m < pm))));
    // the first of the four vectors whose extreme is m
    const bool h0 = mn ? isnan_(m0) : (m0 == m), h1 = mn ? isnan_(m1) : (m1 == m),
               h2 = mn ? isnan_(m2) : (m2 == m);
    const int jv = h0 ? 0 : h1 ? 1 : h2 ? 2 : 3;
#pragma unroll
    for (int e = 0; e < V; ++e) {
      const T x = jv == 0 ? v0[e] : jv == 1 ? v1[e] : jv == 2 ? v2[e] : v3[e];
      pv[e] = take ? x : pv[e];
    }
    pm = take ? m : pm;
    pg = take ? g0 + (long long)jv * step : pg;
  }
  // the same for one vector per step (the row kernels)
  template <int V>
  __device__ static void vec_step(float &pm, long long &pg, const T (&v)[V], long long g) {
    float m = AsF<T>::f(v[0]);
#pragma unroll
    for (int j = 1; j < V; ++j) m = MAX ? max_nan(m, AsF<T>::f(v[j])) : min_nan(m, AsF<T>::f(v[j]));
    const bool take = (pg < 0) || (!isnan_(pm) && (isnan_(m) || (MAX ? (m > pm) : (m < pm))));
    pm = take ? m : pm;
    pg = take ? g : pg;
  }
  // four vectors at element offsets b0, b0 + step, b0 + 2 step, b0 + 3 step
  // (increasing): one NaN-propagating extreme of all of them, one compare
  // with the running value, and the first-occurrence search only when it wins
  template <int V>
  __device__ static void vec4(Acc &a, const T (&v0)[V], const T (&v1)[V], const T (&v2)[V], const T (&v3)[V],
                              long long b0, long long step) {
    if constexpr (IsFloat<T>::value && sizeof(T) <= 4) {
      float m0 = AsF<T>::f(v0[0]), m1 = AsF<T>::f(v1[0]), m2 = AsF<T>::f(v2[0]), m3 = AsF<T>::f(v3[0]);
#pragma unroll
      for (int j = 1; j < V; ++j) {
        m0 = MAX ? max_nan(m0, AsF<T>::f(v0[j])) : min_nan(m0, AsF<T>::f(v0[j]));
        m1 = MAX ? max_nan(m1, AsF<T>::f(v1[j])) : min_nan(m1, AsF<T>::f(v1[j]));
        m2 = MAX ? max_nan(m2, AsF<T>::f(v2[j])) : min_nan(m2, AsF<T>::f(v2[j]));
        m3 = MAX ? max_nan(m3, AsF<T>::f(v3[j])) : min_nan(m3, AsF<T>::f(v3[j]));
      }
      const float m = MAX ? max_nan(max_nan(m0, m1), max_nan(m2, m3)) : min_nan(min_nan(m0, m1), min_nan(m2, m3));
      const bool mn = isnan_(m);
      const bool take = (a.i < 0) || (!isnan_(a.v) && (mn || (MAX ? (m > a.v) : (m < a.v))));
      if (take) {
        long long idx = b0;
#pragma unroll
        for (int j = V - 1; j >= 0; --j) {  // last match in reverse order = first occurrence
          const float x = AsF<T>::f(v3[j]);
          if (mn ? isnan_(x) : (x == m)) idx = b0 + 3 * step + j;
        }
#pragma unroll
        for (int j = V - 1; j >= 0; --j) {
          const float x = AsF<T>::f(v2[j]);
          if (mn ? isnan_(x) : (x == m)) idx = b0 + 2 * step + j;
        }
#pragma unroll
        for (int j = V - 1; j >= 0; --j) {
          const float x = AsF<T>::f(v1[j]);
          if (mn ? isnan_(x) : (x == m)) idx = b0 + step + j;
        }
#pragma unroll
        for (int j = V - 1; j >= 0; --j) {
          const float x = AsF<T>::f(v0[j]);
          if (mn ? isnan_(x) : (x == m)) idx = b0 + j;
        }
        a.v = m;
        a.i = idx;
      }
    } else {
      vec<V>(a, v0, b0);
      vec<V>(a, v1, b0 + step);
      vec<V>(a, v2, b0 + 2 * step);
      vec<V>(a, v3, b0 + 3 * step);
    }
  }
  // rows i, i + 8, i + 16, i + 24 of one column: for float / half, the
  // NaN-propagating extreme of the four first, then one compare with the
  // running value and selects (the same result as one() four times in row
  // order: a strictly better value or the first NaN, first occurrence kept)
  __device__ static void four(Acc &a, T v0, T v1, T v2, T v3, long long i) {
    if constexpr (IsFloat<T>::value && sizeof(T) <= 4) {
      const float x0 = AsF<T>::f(v0), x1 = AsF<T>::f(v1), x2 = AsF<T>::f(v2), x3 = AsF<T>::f(v3);
      const float m = MAX ? max_nan(max_nan(x0, x1), max_nan(x2, x3)) : min_nan(min_nan(x0, x1), min_nan(x2, x3));
      const bool mn = isnan_(m);
      const bool take = (a.i < 0) || (!isnan_(a.v) && (mn || (MAX ? (m > a.v) : (m < a.v))));
      const int j = (mn ? isnan_(x0) : (x0 == m)) ? 0 : (mn ? isnan_(x1) : (x1 == m)) ? 8
                  : (mn ? isnan_(x2) : (x2 == m)) ? 16 : 24;
      a.v = take ? (V_)m : a.v;
      a.i = take ? i + j : a.i;
    } else {
      one(a, v0, i);
      one(a, v1, i + 8);
      one(a, v2, i + 16);
      one(a, v3, i + 24);
    }
  }
  __device__ static Acc combine(Acc a, Acc b) { return pick(a, b); }
  __device__ static void finish(Acc a, long long n, void *out, long long idx, int dt, double,
                                PartialOut *p) {
    store_scalar(out, idx, dt, true, a.i, (unsigned long long)a.i, 0.0, false);
    if (p) {
      p->s1 = as_d(a.v);
      p->ival = IsFloat<T>::value ? 0 : (long long)a.v;
      p->index = a.i;
      p->count = n;
    }
  }
};
template <class T> struct RedOp<MMP_R_ARGMAX, T> : ArgOp<T, true> {};
template <class T> struct RedOp<MMP_R_ARGMIN, T> : ArgOp<T, false> {};

// nansum / nanmean: NaNs count as absent; the count of present values is
// carried for nanmean (count 0 gives NaN, as numpy does).
template <class T, bool MEAN>
struct NanSumOp {
  struct Acc {
    double s;
    long long c;
  };
  __device__ static Acc init() {
    Acc a;
    a.s = 0.0;
    a.c = 0;
    return a;
  }
  __device__ static Acc start(Acc a, T) { return a; }
  __device__ static void one(Acc &a, T v, long long) {
    if (!isnan_(v)) {
      a.s += as_d(v);
      a.c += 1;
    }
  }
  template <int V>
  __device__ static void vec(Acc &a, const T (&v)[V], long long) {
    if (IsFloat<T>::value && sizeof(T) < 8) {
      float s = 0.f;
      int c = 0;
#pragma unroll
      for (int j = 0; j < V; ++j) {
        float f = AsF<T>::f(v[j]);
        bool ok = !isnan_(f);
        s += ok ? f : 0.f;
        c += ok ? 1 : 0;
      }
      a.s += (double)s;
      a.c += c;
    } else {
#pragma unroll
      for (int j = 0; j < V; ++j) one(a, v[j], 0);
    }
  }
  // four vectors: one float partial and one count, then one double add
  template <int V>
  __device__ static void vec4(Acc &a, const T (&v0)[V], const T (&v1)[V], const T (&v2)[V], const T (&v3)[V],
                              long long, long long) {
    if constexpr (IsFloat<T>::value && sizeof(T) < 8) {
      float s0 = 0.f, s1 = 0.f;
      int c = 0;
#pragma unroll
      for (int j = 0; j < V; ++j) {
        const float f0 = AsF<T>::f(v0[j]), f1 = AsF<T>::f(v1[j]), f2 = AsF<T>::f(v2[j]), f3 = AsF<T>::f(v3[j]);
        const bool k0 = !isnan_(f0), k1 = !isnan_(f1), k2 = !isnan_(f2), k3 = !isnan_(f3);
        s0 += (k0 ? f0 : 0.f) + (k1 ? f1 : 0.f);
        s1 += (k2 ? f2 : 0.f) + (k3 ? f3 : 0.f);
        c += (int)k0 + (int)k1 + (int)k2 + (int)k3;
      }
      a.s += (double)s0 + (double)s1;
      a.c += c;
    } else {
      vec<V>(a, v0, 0);
      vec<V>(a, v1, 0);
      vec<V>(a, v2, 0);
      vec<V>(a, v3, 0);
    }
  }
  __device__ static void four(Acc &a, T v0, T v1, T v2, T v3, long long i) {
    one(a, v0, i);
    one(a, v1, i);
    one(a, v2, i);
    one(a, v3, i);
  }
  __device__ static Acc combine(Acc a, Acc b) {
    a.s += b.s;
    a.c += b.c;
    return a;
  }
  __device__ static void finish(Acc a, long long n, void *out, long long idx, int dt, double,
                                PartialOut *p) {
    double r = MEAN ? (a.c > 0 ? a.s / (double)a.c : __longlong_as_double(0x7ff8000000000000ll)) : a.s;
    store_acc_value(out, idx, dt, r);
    if (p) {
      p->s1 = a.s;
      p->count = a.c;
    }
  }
};
template <class T> struct RedOp<MMP_R_NANSUM, T> : NanSumOp<T, false> {};
template <class T> struct RedOp<MMP_R_NANMEAN, T> : NanSumOp<T, true> {};

// nanvar / nanstd in one pass.  An accumulator holds the count n of the
// non-NaN values it has seen and their sums S1 = sum(x - k), S2 =
// sum((x - k)^2) around its own shift k: the first non-NaN value it saw (the
// array's first element may be NaN, so there is no common shift as in
// VarOp).  Per element that is a subtract, an add and an fma, with the f32
// partial of a loop step added to f64.  Two accumulators merge without a
// division by moving b's sums to a's shift, d = kb - ka:
//   S1 = S1a + S1b + nb d,  S2 = S2a + S2b + d (2 S1b + nb d)
// (exact algebra; in f64 the d^2 terms cost precision only when the shifts,
// two values of the data, lie ~1e5 standard deviations apart).
// var = (S2 - S1^2/n) / (n - ddof), NaN when n - ddof <= 0 (numpy's nanvar).
template <class T, bool STD>
struct NanVarOp {
  struct Acc {
    double n, k, s1, s2;
  };
  __device__ static Acc init() {
    Acc a;
    a.n = 0.0;
    a.k = 0.0;
    a.s1 = 0.0;
    a.s2 = 0.0;
    return a;
  }
  __device__ static Acc start(Acc a, T) { return a; }
  __device__ static void one(Acc &a, T v, long long) {
    if (isnan_(v)) return;
    const double x = as_d(v);
    if (a.n == 0.0) a.k = x;
    const double d = x - a.k;
    a.s1 += d;
    a.s2 += d * d;
    a.n += 1.0;
  }
  // the non-NaN values of f[0..K): f32 partial sums around the shift
  template <int K>
  __device__ static void group(Acc &a, const float (&f)[K]) {
    if (a.n == 0.0) {  // the first values this accumulator sees
      float g = 0.f;
      bool any = false;
#pragma unroll
      for (int j = K - 1; j >= 0; --j) {
        const bool ok = !isnan_(f[j]);
        g = ok ? f[j] : g;
        any = any || ok;
      }
      if (!any) return;
      a.k = (double)g;
    }
    const float kf = (float)a.k;  // exact: k is one of the f32 inputs
    float s1 = 0.f, s2 = 0.f;
    int c = 0;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const bool ok = !isnan_(f[j]);
      const float d = ok ? f[j] - kf : 0.f;
      s1 += d;
      s2 += d * d;
      c += ok ? 1 : 0;
    }
    a.s1 += (double)s1;
    a.s2 += (double)s2;
    a.n += (double)c;
  }
  template <int V>
  __device__ static void vec(Acc &a, const T (&v)[V], long long) {
    if constexpr (IsFloat<T>::value && sizeof(T) < 8) {
      float f[V];
#pragma unroll
      for (int j = 0; j < V; ++j) f[j] = AsF<T>::f(v[j]);
      group<V>(a, f);
    } else {
#pragma unroll
      for (int j = 0; j < V; ++j) one(a, v[j], 0);
    }
  }
  template <int V>
  __device__ static void vec4(Acc &a, const T (&v0)[V], const T (&v1)[V], const T (&v2)[V], const T (&v3)[V],
                              long long, long long) {
    if constexpr (IsFloat<T>::value && sizeof(T) < 8) {
      float f[4 * V];
#pragma unroll
      for (int j = 0; j < V; ++j) {
        f[j] = AsF<T>::f(v0[j]);
        f[V + j] = AsF<T>::f(v1[j]);
        f[2 * V + j] = AsF<T>::f(v2[j]);
        f[3 * V + j] = AsF<T>::f(v3[j]);
      }
      group<4 * V>(a, f);
    } else {
      vec<V>(a, v0, 0);
      vec<V>(a, v1, 0);
      vec<V>(a, v2, 0);
      vec<V>(a, v3, 0);
    }
  }
  __device__ static void four(Acc &a, T v0, T v1, T v2, T v3, long long i) {
    if constexpr (IsFloat<T>::value && sizeof(T) < 8) {
      const float f[4] = {AsF<T>::f(v0), AsF<T>::f(v1), AsF<T>::f(v2), AsF<T>::f(v3)};
      group<4>(a, f);
    } else {
      one(a, v0, i);
      one(a, v1, i);
      one(a, v2, i);
      one(a, v3, i);
    }
  }
  __device__ static Acc combine(Acc a, Acc b) {
    if (b.n == 0.0) return a;
    if (a.n == 0.0) return b;
    const double d = b.k - a.k;
    a.s2 += b.s2 + d * (2.0 * b.s1 + b.n * d);
    a.s1 += b.s1 + b.n * d;
    a.n += b.n;
    return a;
  }
  __device__ static void finish(Acc a, long long, void *out, long long idx, int dt, double ddof,
                                PartialOut *p) {
    double m2 = a.n > 0.0 ? a.s2 - a.s1 * a.s1 / a.n : 0.0;
    if (m2 < 0.0) m2 = 0.0;
    const double dof = a.n - ddof;
    const double var = dof > 0.0 ? m2 / dof : __longlong_as_double(0x7ff8000000000000ll);
    store_acc_value(out, idx, dt, STD ? sqrt(var) : var);
    if (p) {  // the shifted form of VarOp's partial
      p->s1 = a.s1;
      p->s2 = a.s2;
      p->shift = a.k;
      p->count = (long long)a.n;
    }
  }
};
template <class T> struct RedOp<MMP_R_NANVAR, T> : NanVarOp<T, false> {};
template <class T> struct RedOp<MMP_R_NANSTD, T> : NanVarOp<T, true> {};

template <class T, bool ANY>
struct BoolOp {
  typedef int Acc;
  __device__ static Acc init() { return ANY ? 0 : 1; }
  __device__ static Acc start(Acc a, T) { return a; }
  __device__ static void one(Acc &a, T v, long long) {
    bool nz = cvt<bool>(v);
    if (ANY) a |= nz ? 1 : 0;
    else a &= nz ? 1 : 0;
  }
  template <int V>
  __device__ static void vec(Acc &a, const T (&v)[V], long long) {
#pragma unroll
    for (int j = 0; j < V; ++j) one(a, v[j], 0);
  }
  __device__ static void four(Acc &a, T v0, T v1, T v2, T v3, long long i) {
    one(a, v0, i);
    one(a, v1, i);
    one(a, v2, i);
    one(a, v3, i);
  }
  __device__ static Acc combine(Acc a, Acc b) { return ANY ? (a | b) : (a & b); }
  __device__ static void finish(Acc a, long long n, void *out, long long idx, int dt, double,
                                PartialOut *p) {
    store_scalar(out, idx, dt, true, a, (unsigned long long)a, 0.0, false);
    if (p) {
      p->ival = a;
      p->count = n;
    }
  }
};
template <class T> struct RedOp<MMP_R_ANY, T> : BoolOp<T, true> {};
template <class T> struct RedOp<MMP_R_ALL, T> : BoolOp<T, false> {};

// ---------------------------------------------------------------- loaders
// Contiguous array loader; `aligned` says whether x is aligned to a vector.
template <class T>
struct ContigLoader {
  typedef T value_type;
  const T *x;
  int aligned;
  __device__ __forceinline__ T operator()(long long i) const { return x[i]; }
  template <int V>
  using Raw = Vec<T, V>;
  template <int V>
  __device__ __forceinline__ void load(long long i, Raw<V> &r) const {
    r = ldvec_stream<T, V>(x + i);
  }
  template <int V>
  __device__ __forceinline__ void apply(const Raw<V> &r, T (&v)[V]) const {
#pragma unroll
    for (int j = 0; j < V; ++j) v[j] = r.v[j];
  }
  template <int V>
  __device__ __forceinline__ void vec(long long i, T (&v)[V]) const {
    Raw<V> r;
    load<V>(i, r);
    apply<V>(r, v);
  }
};

// Elements per vector load: 16 bytes, at most 8 elements.
template <class T> struct VW { static const int value = (16 / sizeof(T)) > 8 ? 8 : (16 / sizeof(T)); };

// ---------------------------------------------------------------- block reduce
template <class Op>
__device__ __forceinline__ typename Op::Acc warp_reduce(typename Op::Acc a) {
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) a = Op::combine(a, shfl_down(a, d));
  return a;
}

// Reduce across the block; the result is valid in thread 0.
template <class Op, int NT>
__device__ __forceinline__ typename Op::Acc block_reduce(typename Op::Acc a) {
  typedef typename Op::Acc Acc;
  __shared__ Acc sm[NT / 32];
  int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  a = warp_reduce<Op>(a);
  __syncthreads();  // sm may still be read by a previous call
  if (lane == 0) sm[w] = a;
  __syncthreads();
  if (w == 0) {
    a = (lane < NT / 32) ? sm[lane] : Op::init();
    a = warp_reduce<Op>(a);
  }
  return a;
}

// ---------------------------------------------------------------- full reduce
// One launch for any n: every block reduces a grid-strided share (four
// vectors in flight per thread), writes its partial to scratch, and the last
// block to take a ticket merges the partials in block order (deterministic)
// and writes the result.  The ticket is returned to zero for the next call.
// Ops may process the four vectors of one loop step together (vec4);
// the others take them one by one.
template <class Op, class = void>
struct HasVec4 {
  static constexpr bool value = false;
};
template <class Op>
struct HasVec4<Op, decltype((void)&Op::template vec4<4>)> {
  static constexpr bool value = true;
};

// Ops that defer the first-occurrence search of their vector loop steps
// (ArgOp on float / half).
template <class Op, class = void>
struct HasGroupDeferred {
  static constexpr bool value = false;
};
template <class Op>
struct HasGroupDeferred<Op, decltype((void)Op::kGroupDeferred)> {
  static constexpr bool value = Op::kGroupDeferred;
};

template <int OPC, class T, class L>
__device__ __forceinline__ bool reduce_full_body(const L &ld, long long n, void *out, int out_dt,
                                                 double ddof, void *scratch, unsigned *ticket,
                                                 PartialOut *part) {
  typedef RedOp<OPC, T> Op;
  typedef typename Op::Acc Acc;
  constexpr int V = VW<T>::value;
  Acc acc = Op::init();
  if (n > 0) acc = Op::start(acc, ld(0));
  const Acc acc0 = acc;
  long long tid = (long long)blockIdx.x * RBLOCK + threadIdx.x;
  long long nth = (long long)gridDim.x * RBLOCK;
  long long done = 0;
  if (ld.aligned) {
    long long nv = n / V;
    long long i = tid;
    if constexpr (HasGroupDeferred<Op>::value) {
      float pm = 0.0f;
      long long pg = -1;  // first element index of the vector holding the best value so far
      T pv[V];
#pragma unroll
      for (int e = 0; e < V; ++e) pv[e] = T(0);
      for (; i + 3 * nth < nv; i += 4 * nth) {
        typename L::template Raw<V> r0, r1, r2, r3;
        ld.template load<V>(i * V, r0);
        ld.template load<V>((i + nth) * V, r1);
        ld.template load<V>((i + 2 * nth) * V, r2);
        ld.template load<V>((i + 3 * nth) * V, r3);
        T a0[V], a1[V], a2[V], a3[V];
        ld.template apply<V>(r0, a0);
        ld.template apply<V>(r1, a1);
        ld.template apply<V>(r2, a2);
        ld.template apply<V>(r3, a3);
        Op::template group_step<V>(pm, pg, pv, a0, a1, a2, a3, i * V, nth * V);
      }
      if (pg >= 0) Op::template vec<V>(acc, pv, pg);  // the exact first index inside the vector
    }
    for (; i + 3 * nth < nv; i += 4 * nth) {
      typename L::template Raw<V> r0, r1, r2, r3;
      ld.template load<V>(i * V, r0);
      ld.template load<V>((i + nth) * V, r1);
      ld.template load<V>((i + 2 * nth) * V, r2);
      ld.template load<V>((i + 3 * nth) * V, r3);
      T a0[V], a1[V], a2[V], a3[V];
      ld.template apply<V>(r0, a0);
      ld.template apply<V>(r1, a1);
      ld.template apply<V>(r2, a2);
      ld.template apply<V>(r3, a3);
      if constexpr (HasVec4<Op>::value) {
        Op::template vec4<V>(acc, a0, a1, a2, a3, i * V, nth * V);
      } else {
        Op::template vec<V>(acc, a0, i * V);
        Op::template vec<V>(acc, a1, (i + nth) * V);
        Op::template vec<V>(acc, a2, (i + 2 * nth) * V);
        Op::template vec<V>(acc, a3, (i + 3 * nth) * V);
      }
    }
    for (; i < nv; i += nth) {
      T a0[V];
      ld.template vec<V>(i * V, a0);
      Op::template vec<V>(acc, a0, i * V);
    }
    done = nv * V;
  }
  for (long long j = done + tid; j < n; j += nth) Op::one(acc, ld(j), j);
  acc = block_reduce<Op, RBLOCK>(acc);
  if (gridDim.x == 1) {
    if (threadIdx.x == 0) Op::finish(acc, n, out, 0, out_dt, ddof, part);
    return true;
  }
  __shared__ int is_last;
  if (threadIdx.x == 0) {
    reinterpret_cast<Acc *>(scratch)[blockIdx.x] = acc;
    __threadfence();
    unsigned t = atomicAdd(ticket, 1u);
    is_last = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (!is_last) return false;
  __threadfence();
  Acc m = acc0;
  bool first = true;
  for (int b = threadIdx.x; b < (int)gridDim.x; b += RBLOCK) {
    Acc pb = load_cg(reinterpret_cast<const Acc *>(scratch) + b);
    m = first ? pb : Op::combine(m, pb);
    first = false;
  }
  if (first) m = acc0;
  m = block_reduce<Op, RBLOCK>(m);
  if (threadIdx.x == 0) {
    Op::finish(m, n, out, 0, out_dt, ddof, part);
    *ticket = 0u;
  }
  return true;
}

template <int OPC, class T, class L>
__global__ void __launch_bounds__(RBLOCK) reduce_full_kernel(L ld, long long n, void *out, int out_dt,
                                                             double ddof, void *scratch,
                                                             unsigned *ticket, PartialOut *part) {
  reduce_full_body<OPC, T, L>(ld, n, out, out_dt, ddof, scratch, ticket, part);
}

// ---------------------------------------------------------------- row reduce
// out[r] = reduce(x[r*k : r*k+k]) with one block per row (k large) ...
template <int OPC, class T, class L>
__device__ __forceinline__ void reduce_rows_block_body(const L &ld, long long rows, long long k, void *out,
                                                       int out_dt, double ddof) {
  typedef RedOp<OPC, T> Op;
  typedef typename Op::Acc Acc;
  constexpr int V = VW<T>::value;
  const bool vec_ok = ld.aligned && (k % V == 0);
  for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
    long long base = r * k;
    Acc acc = Op::start(Op::init(), ld(base));
    long long done = 0;
    if (vec_ok) {
      long long nv = k / V;
      long long i = threadIdx.x;
      if constexpr (HasGroupDeferred<Op>::value) {
        // extreme and its vector first, the index inside the vector after
        // the loop (see ArgOp::group_step)
        float pm = 0.0f;
        long long pg = -1;
        for (; i + RBLOCK < nv; i += 2 * RBLOCK) {
          T a0[V], a1[V];
          ld.template vec<V>(base + i * V, a0);
          ld.template vec<V>(base + (i + RBLOCK) * V, a1);
          Op::template vec_step<V>(pm, pg, a0, i);
          Op::template vec_step<V>(pm, pg, a1, i + RBLOCK);
        }
        if (pg >= 0) {
          T a0[V];
          ld.template vec<V>(base + pg * V, a0);
          Op::template vec<V>(acc, a0, pg * V);
        }
      }
      for (; i + RBLOCK < nv; i += 2 * RBLOCK) {
        T a0[V], a1[V];
        ld.template vec<V>(base + i * V, a0);
        ld.template vec<V>(base + (i + RBLOCK) * V, a1);
        Op::template vec<V>(acc, a0, i * V);
        Op::template vec<V>(acc, a1, (i + RBLOCK) * V);
      }
      for (; i < nv; i += RBLOCK) {
        T a0[V];
        ld.template vec<V>(base + i * V, a0);
        Op::template vec<V>(acc, a0, i * V);
      }
      done = nv * V;
    }
    for (long long j = done + threadIdx.x; j < k; j += RBLOCK) Op::one(acc, ld(base + j), j);
    acc = block_reduce<Op, RBLOCK>(acc);
    if (threadIdx.x == 0) Op::finish(acc, k, out, r, out_dt, ddof, nullptr);
  }
}
template <int OPC, class T, class L>
__global__ void __launch_bounds__(RBLOCK) reduce_rows_block_kernel(L ld, long long rows, long long k,
                                                                   void *out, int out_dt, double ddof) {
  reduce_rows_block_body<OPC, T, L>(ld, rows, k, out, out_dt, ddof);
}

// ... or one warp per row (k small).
template <int OPC, class T, class L>
__device__ __forceinline__ void reduce_rows_warp_body(const L &ld, long long rows, long long k, void *out,
                                                      int out_dt, double ddof) {
  typedef RedOp<OPC, T> Op;
  typedef typename Op::Acc Acc;
  int lane = threadIdx.x & 31;
  long long w = ((long long)blockIdx.x * RBLOCK + threadIdx.x) >> 5;
  long long nw = ((long long)gridDim.x * RBLOCK) >> 5;
  for (long long r = w; r < rows; r += nw) {
    long long base = r * k;
    Acc acc = Op::start(Op::init(), ld(base));
    for (long long j = lane; j < k; j += 32) Op::one(acc, ld(base + j), j);
    acc = warp_reduce<Op>(acc);
    if (lane == 0) Op::finish(acc, k, out, r, out_dt, ddof, nullptr);
  }
}
template <int OPC, class T, class L>
__global__ void __launch_bounds__(RBLOCK) reduce_rows_warp_kernel(L ld, long long rows, long long k,
                                                                  void *out, int out_dt, double ddof) {
  reduce_rows_warp_body<OPC, T, L>(ld, rows, k, out, out_dt, ddof);
}

// ---------------------------------------------------------------- column reduce
// x is (outer, k, inner); out[o*inner + c] = reduce_r x[(o*k + r)*inner + c].
// Block = 32 x 8 threads covering 32*CV adjacent columns; the 8 thread rows
// split the reduced axis, gridDim.y further splits it into chunks whose
// partials are merged in chunk order by the last block of each column tile.
template <int OPC, class T, class L, int CV>
__device__ __forceinline__ void reduce_cols_body(const L &ld, long long outer, long long k, long long inner,
                                                 long long kchunk, void *out, int out_dt, double ddof,
                                                 void *scratch, unsigned *tickets) {
  typedef RedOp<OPC, T> Op;
  typedef typename Op::Acc Acc;
  const long long ctiles = (inner + 32 * CV - 1) / (32 * CV);
  const long long o = blockIdx.x / ctiles;
  const long long ct = blockIdx.x % ctiles;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const long long c0 = ct * 32 * CV + (long long)tx * CV;
  const long long r0 = (long long)blockIdx.y * kchunk;
  long long r1 = r0 + kchunk;
  if (r1 > k) r1 = k;
  const long long obase = o * k * inner;
  Acc acc[CV];
#pragma unroll
  for (int j = 0; j < CV; ++j) {
    long long c = c0 + j;
    acc[j] = Op::init();
    if (c < inner) acc[j] = Op::start(acc[j], ld(obase + c));
  }
  Acc acc0[CV];
#pragma unroll
  for (int j = 0; j < CV; ++j) acc0[j] = acc[j];
  const bool full = (c0 + CV <= inner);
  long long r = r0 + ty;
  if (CV > 1 && full) {
    // four rows of loads in flight per thread, consumed in row order
    for (; r + 24 < r1; r += 32) {
      T v0[CV], v1[CV], v2[CV], v3[CV];
      const long long off = obase + r * inner + c0;
      ld.template vec<CV>(off, v0);
      ld.template vec<CV>(off + 8 * inner, v1);
      ld.template vec<CV>(off + 16 * inner, v2);
      ld.template vec<CV>(off + 24 * inner, v3);
#pragma unroll
      for (int j = 0; j < CV; ++j) Op::four(acc[j], v0[j], v1[j], v2[j], v3[j], r);
    }
  }
  for (; r < r1; r += 8) {
    long long off = obase + r * inner + c0;
    if (CV > 1 && full) {
      T v[CV];
      ld.template vec<CV>(off, v);
#pragma unroll
      for (int j = 0; j < CV; ++j) Op::one(acc[j], v[j], r);
    } else {
#pragma unroll
      for (int j = 0; j < CV; ++j)
        if (c0 + j < inner) Op::one(acc[j], ld(off + j), r);
    }
  }
  __shared__ Acc sm[8][32 * CV];
#pragma unroll
  for (int j = 0; j < CV; ++j) sm[ty][tx * CV + j] = acc[j];
  __syncthreads();
  if (ty == 0) {
#pragma unroll
    for (int j = 0; j < CV; ++j) {
      Acc a = sm[0][tx * CV + j];
      for (int y = 1; y < 8; ++y) a = Op::combine(a, sm[y][tx * CV + j]);
      acc[j] = a;
    }
  }
  if (gridDim.y == 1) {
    if (ty == 0) {
#pragma unroll
      for (int j = 0; j < CV; ++j)
        if (c0 + j < inner) Op::finish(acc[j], k, out, o * inner + c0 + j, out_dt, ddof, nullptr);
    }
    return;
  }
  Acc *part = reinterpret_cast<Acc *>(scratch);
  if (ty == 0) {
#pragma unroll
    for (int j = 0; j < CV; ++j)
      if (c0 + j < inner) part[((long long)blockIdx.y * outer + o) * inner + c0 + j] = acc[j];
    __threadfence();
  }
  __syncthreads();
  __shared__ int is_last;
  if (threadIdx.x == 0) {
    unsigned t = atomicAdd(tickets + blockIdx.x, 1u);
    is_last = (t == gridDim.y - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if (ty == 0) {
#pragma unroll
    for (int j = 0; j < CV; ++j) {
      long long c = c0 + j;
      if (c >= inner) continue;
      Acc a = acc0[j];
      for (unsigned s = 0; s < gridDim.y; ++s) {
        Acc ps = load_cg(part + ((long long)s * outer + o) * inner + c);
        a = (s == 0) ? ps : Op::combine(a, ps);
      }
      Op::finish(a, k, out, o * inner + c, out_dt, ddof, nullptr);
    }
  }
  if (threadIdx.x == 0) tickets[blockIdx.x] = 0u;
}
template <int OPC, class T, class L, int CV>
__global__ void __launch_bounds__(RBLOCK) reduce_cols_kernel(L ld, long long outer, long long k,
                                                             long long inner, long long kchunk,
                                                             void *out, int out_dt, double ddof,
                                                             void *scratch, unsigned *tickets) {
  reduce_cols_body<OPC, T, L, CV>(ld, outer, k, inner, kchunk, out, out_dt, ddof, scratch, tickets);
}

}  // namespace mmpd
