// mmp_gemm: row-major batched matmul.  float32 and float16 go to the
// tcgen05/TMEM tensor-core kernels (mmp_gemm_tc.cu) when the layout allows
// it; everything else takes the CUDA-core kernel in mmp_gemm_simt.cuh.
#include <cuda_runtime.h>

#include "mmp_dispatch.h"
#include "mmp_gemm_simt.cuh"

using namespace mmpd;

namespace mmp {

// Implemented in mmp_gemm_tc.cu; returns MMP_E_UNSUPPORTED when the
// tensor-core path cannot take the problem.
int gemm_tc(int dtype, int mode, long long batch, long long m, long long n, long long k, const void *a,
            long long lda, long long sa, const void *b, long long ldb, long long sb, void *c, long long ldc,
            long long sc);

template <int UNUSED, class T>
struct GemmSimtRun {
  static int run(long long batch, long long m, long long n, long long k, const void *a, long long lda,
                 long long sa, const void *b, long long ldb, long long sb, void *c, long long ldc,
                 long long sc) {
    cudaStream_t st = stream();
    if (!st) return set_error(MMP_E_CUDA, "no stream");
    if (batch > 65535) return set_error(MMP_E_ARG, "batch too large for the CUDA-core path");
    dim3 grid((unsigned)((n + 63) / 64), (unsigned)((m + 63) / 64), (unsigned)batch);
    if (grid.y > 65535) return set_error(MMP_E_ARG, "M too large for the CUDA-core path");
    gemm_simt_kernel<T><<<grid, 256, 0, st>>>(m, n, k, (const T *)a, lda, sa, (const T *)b, ldb, sb, (T *)c,
                                              ldc, sc);
    MMP_LAUNCH_CHECK("gemm_simt_kernel");
    return MMP_OK;
  }
};

}  // namespace mmp

extern "C" int mmp_gemm(int dtype, int mode, int64_t batch, int64_t m, int64_t n, int64_t k, const void *a,
                        int64_t lda, int64_t stride_a, const void *b, int64_t ldb, int64_t stride_b, void *c,
                        int64_t ldc, int64_t stride_c) {
  if (batch < 0 || m < 0 || n < 0 || k < 0) return mmp::set_error(MMP_E_ARG, "negative extent");
  if (batch == 0 || m == 0 || n == 0) return MMP_OK;
  if (!a || !b || !c) return mmp::set_error(MMP_E_ARG, "null pointer");
  if (k == 0) {
    size_t es = mmp_dtype_size(dtype);
    if (!es) return mmp::set_error(MMP_E_ARG, "bad dtype");
    if (ldc == n && (stride_c == m * n || batch == 1))
      return mmp_memset(c, 0, (size_t)batch * m * n * es);
  }
  if (mode != MMP_GEMM_SIMT && (dtype == MMP_FLOAT32 || dtype == MMP_FLOAT16)) {
    int rc = mmp::gemm_tc(dtype, mode, batch, m, n, k, a, lda, stride_a, b, ldb, stride_b, c, ldc, stride_c);
    if (rc != MMP_E_UNSUPPORTED) return rc;
    if (mode != MMP_GEMM_AUTO) return rc;
  }
  return mmp::dispatch_dtype<mmp::GemmSimtRun, 0>(dtype, (long long)batch, (long long)m, (long long)n,
                                                  (long long)k, a, (long long)lda, (long long)stride_a, b,
                                                  (long long)ldb, (long long)stride_b, c, (long long)ldc,
                                                  (long long)stride_c);
}
