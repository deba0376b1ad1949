// mmp_gather / mmp_scatter / mmp_compact_indices: the device side of
// advanced (integer- and boolean-array) indexing.
//
// Reference: ndarray.__getitem__ / __setitem__ take numpy on the host for
// every advanced key (src/macmetalpy/ndarray.py:874-957, "CPU fallback for
// advanced indexing"), and indexing.py's take / put / nonzero / compress /
// extract run numpy too (indexing.py:24-410).  Here the Python layer turns
// any advanced key into one int64 array of element offsets (numpy's
// broadcasting and axis-placement rules, built by the fusion engine), and
// these kernels move the elements: out[i] = src[off[i]] and
// dst[off[i]] = val[i].  Elements are moved as raw 1/2/4/8-byte words.
// Offsets were range-checked on the host side (IndexError); each kernel
// still checks 0 <= off < limit and sets the device error word (5) instead
// of touching memory outside the buffer.
//
// mmp_compact_indices writes the positions of the true entries of a bool
// mask, in order, given the inclusive scan of the mask (numpy's nonzero on
// the flattened mask).
#include <cuda_runtime.h>

#include "mmp_dispatch.h"

namespace mmpd {

template <class W>
__global__ void gather_kernel(const W *__restrict__ src, long long limit, const long long *__restrict__ off,
                              long long n, W *__restrict__ out, int *err) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const long long o = off[i];
    if (o < 0 || o >= limit) {
      atomicExch(err, 5);
      continue;
    }
    out[i] = src[o];
  }
}

template <class W>
__global__ void scatter_kernel(W *__restrict__ dst, long long limit, const long long *__restrict__ off, long long n,
                               const W *__restrict__ val, int *err) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const long long o = off[i];
    if (o < 0 || o >= limit) {
      atomicExch(err, 5);
      continue;
    }
    dst[o] = val[i];
  }
}

__global__ void compact_kernel(const bool *__restrict__ mask, const long long *__restrict__ incl, long long n,
                               long long count, long long *__restrict__ out, int *err) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    if (!mask[i]) continue;
    const long long p = incl[i] - 1;
    if (p < 0 || p >= count) {
      atomicExch(err, 5);
      continue;
    }
    out[p] = i;
  }
}

}  // namespace mmpd

namespace {

int grid_for(long long n) {
  long long b = (n + 255) / 256;
  const long long cap = (long long)mmp::sm_count() * 16;
  return (int)(b < cap ? (b ? b : 1) : cap);
}

template <class W>
int gather_w(const void *src, long long limit, const int64_t *off, long long n, void *out) {
  mmpd::gather_kernel<W><<<grid_for(n), 256, 0, mmp::stream()>>>((const W *)src, limit, (const long long *)off, n,
                                                                  (W *)out, mmp::device_error_word());
  MMP_LAUNCH_CHECK("gather_kernel");
  return MMP_OK;
}

template <class W>
int scatter_w(void *dst, long long limit, const int64_t *off, long long n, const void *val) {
  mmpd::scatter_kernel<W><<<grid_for(n), 256, 0, mmp::stream()>>>((W *)dst, limit, (const long long *)off, n,
                                                                   (const W *)val, mmp::device_error_word());
  MMP_LAUNCH_CHECK("scatter_kernel");
  return MMP_OK;
}

}  // namespace

extern "C" int mmp_gather(int dtype, const void *src, int64_t limit, const int64_t *offsets, int64_t n, void *out) {
  if (n < 0 || limit < 0) return mmp::set_error(MMP_E_ARG, "negative extent");
  if (n == 0) return MMP_OK;
  if (!src || !offsets || !out) return mmp::set_error(MMP_E_ARG, "null pointer");
  switch (mmp_dtype_size(dtype)) {
    case 1: return gather_w<unsigned char>(src, limit, offsets, n, out);
    case 2: return gather_w<unsigned short>(src, limit, offsets, n, out);
    case 4: return gather_w<unsigned>(src, limit, offsets, n, out);
    case 8: return gather_w<unsigned long long>(src, limit, offsets, n, out);
    default: return mmp::set_error(MMP_E_ARG, "unsupported dtype code");
  }
}

extern "C" int mmp_scatter(int dtype, void *dst, int64_t limit, const int64_t *offsets, int64_t n,
                           const void *values) {
  if (n < 0 || limit < 0) return mmp::set_error(MMP_E_ARG, "negative extent");
  if (n == 0) return MMP_OK;
  if (!dst || !offsets || !values) return mmp::set_error(MMP_E_ARG, "null pointer");
  switch (mmp_dtype_size(dtype)) {
    case 1: return scatter_w<unsigned char>(dst, limit, offsets, n, values);
    case 2: return scatter_w<unsigned short>(dst, limit, offsets, n, values);
    case 4: return scatter_w<unsigned>(dst, limit, offsets, n, values);
    case 8: return scatter_w<unsigned long long>(dst, limit, offsets, n, values);
    default: return mmp::set_error(MMP_E_ARG, "unsupported dtype code");
  }
}

extern "C" int mmp_compact_indices(const void *mask, const int64_t *incl, int64_t n, int64_t count, int64_t *out) {
  if (n < 0 || count < 0) return mmp::set_error(MMP_E_ARG, "negative extent");
  if (n == 0 || count == 0) return MMP_OK;
  if (!mask || !incl || !out) return mmp::set_error(MMP_E_ARG, "null pointer");
  mmpd::compact_kernel<<<grid_for(n), 256, 0, mmp::stream()>>>((const bool *)mask, (const long long *)incl, n,
                                                                count, (long long *)out, mmp::device_error_word());
  MMP_LAUNCH_CHECK("compact_kernel");
  return MMP_OK;
}
