// CUDA-core GEMM used for the shapes, strides and dtypes the tensor-core
// path does not take (integers, float64, unaligned leading dimensions,
// tiny problems).  Row-major C[b] = A[b] @ B[b]; 64x64 output tile per
// block, 16x16 threads with 4x4 outputs each, K staged through shared memory.
// Accumulates in double for float32/float64, float for float16 and in 64-bit
// integers for integer types (wrapping to the output type, as numpy does).
#pragma once
#include "mmp_device.cuh"

namespace mmpd {

template <class T> struct GemmAcc { typedef long long type; };
template <> struct GemmAcc<unsigned short> { typedef unsigned long long type; };
template <> struct GemmAcc<unsigned int> { typedef unsigned long long type; };
template <> struct GemmAcc<unsigned long long> { typedef unsigned long long type; };
template <> struct GemmAcc<float> { typedef double type; };
template <> struct GemmAcc<double> { typedef double type; };
template <> struct GemmAcc<__half> { typedef float type; };

template <class Acc, class T> __device__ __forceinline__ Acc gacc(T v) { return (Acc)v; }
template <> __device__ __forceinline__ float gacc<float, __half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ long long gacc<long long, bool>(bool v) { return v ? 1 : 0; }

template <class T>
__global__ void __launch_bounds__(256) gemm_simt_kernel(long long M, long long N, long long K, const T *A,
                                                        long long lda, long long sA, const T *B,
                                                        long long ldb, long long sB, T *C, long long ldc,
                                                        long long sC) {
  typedef typename GemmAcc<T>::type Acc;
  __shared__ Acc As[16][65];
  __shared__ Acc Bs[16][65];
  const long long b = blockIdx.z;
  A += b * sA;
  B += b * sB;
  C += b * sC;
  const long long m0 = (long long)blockIdx.y * 64, n0 = (long long)blockIdx.x * 64;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  Acc acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = Acc(0);
  for (long long k0 = 0; k0 < K; k0 += 16) {
    for (int e = threadIdx.x; e < 16 * 64; e += 256) {
      int kk = e & 15, mm = e >> 4;
      long long gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < M && gk < K) ? gacc<Acc, T>(A[gm * lda + gk]) : Acc(0);
      int nn = e & 63, kb = e >> 6;
      long long gn = n0 + nn, gk2 = k0 + kb;
      Bs[kb][nn] = (gn < N && gk2 < K) ? gacc<Acc, T>(B[gk2 * ldb + gn]) : Acc(0);
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      Acc a[4], bb[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bb[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] += a[i] * bb[j];
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      long long gm = m0 + ty * 4 + i, gn = n0 + tx * 4 + j;
      if (gm < M && gn < N) C[gm * ldc + gn] = cvt<T>(acc[i][j]);
    }
}

}  // namespace mmpd
