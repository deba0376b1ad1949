// Compile-time dispatch helpers: dtype code -> C++ type, reduction op code
// -> template argument, and which (op, dtype) pairs are precompiled.
#pragma once
#include <cuda_fp16.h>

#include "mmp_internal.h"
#include "mmp_reduce.cuh"

namespace mmp {

template <class T> struct IsFloatT { static constexpr bool value = false; };
template <> struct IsFloatT<float> { static constexpr bool value = true; };
template <> struct IsFloatT<double> { static constexpr bool value = true; };
template <> struct IsFloatT<__half> { static constexpr bool value = true; };

template <class T> struct DtypeCode;
template <> struct DtypeCode<bool> { static constexpr int value = MMP_BOOL; };
template <> struct DtypeCode<short> { static constexpr int value = MMP_INT16; };
template <> struct DtypeCode<unsigned short> { static constexpr int value = MMP_UINT16; };
template <> struct DtypeCode<int> { static constexpr int value = MMP_INT32; };
template <> struct DtypeCode<unsigned int> { static constexpr int value = MMP_UINT32; };
template <> struct DtypeCode<long long> { static constexpr int value = MMP_INT64; };
template <> struct DtypeCode<unsigned long long> { static constexpr int value = MMP_UINT64; };
template <> struct DtypeCode<__half> { static constexpr int value = MMP_FLOAT16; };
template <> struct DtypeCode<float> { static constexpr int value = MMP_FLOAT32; };
template <> struct DtypeCode<double> { static constexpr int value = MMP_FLOAT64; };

// nan-ops exist for float types only (the host maps integer nan-ops to the
// plain op, as nan_ops.nansum does at nan_ops.py:132-134).
template <int OPC, class T> struct RedSupported {
  static constexpr bool value =
      !(OPC == MMP_R_NANSUM || OPC == MMP_R_NANMEAN || OPC == MMP_R_NANMAX || OPC == MMP_R_NANMIN ||
        OPC == MMP_R_NANVAR || OPC == MMP_R_NANSTD) ||
      IsFloatT<T>::value;
};

// F<OPC, T>::run(args...) for the dtype code.  int8/uint8 never reach the
// kernels: the host resolves them to int16/uint16 (_dtypes.py:126-129).
template <template <int, class> class F, int OPC, class... Args>
int dispatch_dtype(int dt, Args... args) {
  switch (dt) {
    case MMP_BOOL: return F<OPC, bool>::run(args...);
    case MMP_INT16: return F<OPC, short>::run(args...);
    case MMP_UINT16: return F<OPC, unsigned short>::run(args...);
    case MMP_INT32: return F<OPC, int>::run(args...);
    case MMP_UINT32: return F<OPC, unsigned int>::run(args...);
    case MMP_INT64: return F<OPC, long long>::run(args...);
    case MMP_UINT64: return F<OPC, unsigned long long>::run(args...);
    case MMP_FLOAT16: return F<OPC, __half>::run(args...);
    case MMP_FLOAT32: return F<OPC, float>::run(args...);
    case MMP_FLOAT64: return F<OPC, double>::run(args...);
    default: return set_error(MMP_E_ARG, "unsupported dtype code");
  }
}

template <template <int, class> class F, class... Args>
int dispatch_op(int op, int dt, Args... args) {
  switch (op) {
    case MMP_R_SUM: return dispatch_dtype<F, MMP_R_SUM>(dt, args...);
    case MMP_R_PROD: return dispatch_dtype<F, MMP_R_PROD>(dt, args...);
    case MMP_R_MAX: return dispatch_dtype<F, MMP_R_MAX>(dt, args...);
    case MMP_R_MIN: return dispatch_dtype<F, MMP_R_MIN>(dt, args...);
    case MMP_R_MEAN: return dispatch_dtype<F, MMP_R_MEAN>(dt, args...);
    case MMP_R_VAR: return dispatch_dtype<F, MMP_R_VAR>(dt, args...);
    case MMP_R_STD: return dispatch_dtype<F, MMP_R_STD>(dt, args...);
    case MMP_R_ARGMAX: return dispatch_dtype<F, MMP_R_ARGMAX>(dt, args...);
    case MMP_R_ARGMIN: return dispatch_dtype<F, MMP_R_ARGMIN>(dt, args...);
    case MMP_R_NANSUM: return dispatch_dtype<F, MMP_R_NANSUM>(dt, args...);
    case MMP_R_NANMEAN: return dispatch_dtype<F, MMP_R_NANMEAN>(dt, args...);
    case MMP_R_NANMAX: return dispatch_dtype<F, MMP_R_NANMAX>(dt, args...);
    case MMP_R_NANMIN: return dispatch_dtype<F, MMP_R_NANMIN>(dt, args...);
    case MMP_R_ANY: return dispatch_dtype<F, MMP_R_ANY>(dt, args...);
    case MMP_R_ALL: return dispatch_dtype<F, MMP_R_ALL>(dt, args...);
    case MMP_R_NANVAR: return dispatch_dtype<F, MMP_R_NANVAR>(dt, args...);
    case MMP_R_NANSTD: return dispatch_dtype<F, MMP_R_NANSTD>(dt, args...);
    default: return set_error(MMP_E_ARG, "unsupported reduction op");
  }
}

}  // namespace mmp
