// mmp_merge_partials: the merge step of a block-distributed full reduction,
// on the device.  Each shard's mmp_reduce_partial writes one partial; the
// exchange (mmp_allgather) puts all of them, in rank order, into one device
// array on every rank; this kernel folds them in that order with the same
// accumulator arithmetic and the same finish as the single-GPU reduction
// (mmp_reduce.cuh), so a distributed result is computed exactly like a
// single-GPU result whose blocks happen to be the shards.
//
// Per op family:
//   sum / mean / prod / nansum / nanmean / any / all: the exact partials add
//     (multiply) in rank order (float sums in float64, integers in 64 bits);
//   var / std: the shifted moments of shard b move to the first shard's
//     shift, d = k_b - k_a:  S1 += S1_b + n_b d,  S2 += S2_b + d (2 S1_b + n_b d)
//     (the algebra of Chan, Golub & LeVeque's pairwise update written for
//     shifted sums, so no division happens before the finish);
//   nanvar / nanstd: the same move, inside NanVarOp::combine;
//   max / min / nan-variants: the NaN rule of the op; absent shards skipped;
//   argmax / argmin: (value, global index) pairs, numpy's first occurrence,
//     NaN first.
// nparts == 0 gives the op's identity (the carry of rank 0 in a scan).
//
// Reference: the single-device reductions this distributes are
// ndarray._reduce (src/macmetalpy/ndarray.py:1895-1963), reductions.var
// (reductions.py:525-584) and reductions.argmax (reductions.py:381-418).
#include <cuda_runtime.h>

#include "mmp_dispatch.h"

using namespace mmpd;

namespace mmpd {

template <int OPC, class T>
struct MergeFold {
  typedef RedOp<OPC, T> Op;
  typedef typename Op::Acc Acc;
  // fold partial p into a; `first` is true for the first present partial
  __device__ static void fold(Acc &a, const PartialOut &p, bool &seen) {
    constexpr bool kFloat = IsFloat<T>::value;
    if constexpr (OPC == MMP_R_SUM || OPC == MMP_R_MEAN) {
      Acc v = kFloat ? (Acc)p.s1 : (Acc)p.ival;
      a = Op::combine(a, v);
    } else if constexpr (OPC == MMP_R_PROD) {
      Acc v = kFloat ? (Acc)p.s1 : (Acc)p.ival;
      a = Op::combine(a, v);
    } else if constexpr (OPC == MMP_R_MAX || OPC == MMP_R_MIN || OPC == MMP_R_NANMAX || OPC == MMP_R_NANMIN) {
      Acc b;
      b.has = p.count > 0 ? 1 : 0;
      b.v = kFloat ? (decltype(b.v))p.s1 : (decltype(b.v))p.ival;
      a = Op::combine(a, b);
    } else if constexpr (OPC == MMP_R_ARGMAX || OPC == MMP_R_ARGMIN) {
      Acc b;
      b.i = p.index;
      b.v = kFloat ? (decltype(b.v))p.s1 : (decltype(b.v))p.ival;
      a = Op::combine(a, b);
    } else if constexpr (OPC == MMP_R_VAR || OPC == MMP_R_STD) {
      if (p.count <= 0) return;
      if (!seen) {
        a.s1 = p.s1;
        a.s2 = p.s2;
        a.k = p.shift;
      } else {
        const double nb = (double)p.count, d = p.shift - a.k;
        a.s2 += p.s2 + d * (2.0 * p.s1 + nb * d);
        a.s1 += p.s1 + nb * d;
      }
      seen = true;
    } else if constexpr (OPC == MMP_R_NANVAR || OPC == MMP_R_NANSTD) {
      Acc b;
      b.n = (double)p.count;
      b.k = p.shift;
      b.s1 = p.s1;
      b.s2 = p.s2;
      a = Op::combine(a, b);
    } else if constexpr (OPC == MMP_R_NANSUM || OPC == MMP_R_NANMEAN) {
      Acc b;
      b.s = p.s1;
      b.c = p.count;
      a = Op::combine(a, b);
    } else {  // any / all
      a = Op::combine(a, (Acc)(p.ival != 0 ? 1 : 0));
    }
  }
};

template <int OPC, class T>
__global__ void merge_partials_kernel(const PartialOut *parts, int nparts, void *out, int out_dt, double ddof,
                                      PartialOut *merged) {
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  typedef RedOp<OPC, T> Op;
  typename Op::Acc a = Op::init();
  long long n = 0;
  bool seen = false;
  for (int i = 0; i < nparts; ++i) {
    const PartialOut p = parts[i];
    MergeFold<OPC, T>::fold(a, p, seen);
    // nan-ops carry the count of non-NaN values; the rest the element count
    n += p.count;
  }
  if (merged) {
    merged->s1 = merged->s2 = merged->shift = 0.0;
    merged->count = 0;
    merged->ival = 0;
    merged->index = -1;
  }
  Op::finish(a, n, out, 0, out_dt, ddof, merged);
}

}  // namespace mmpd

namespace mmp {

template <int OPC, class T>
struct MergeRun {
  static int run(const PartialOut *parts, int nparts, int out_dt, void *out, double ddof, PartialOut *merged) {
    if constexpr (!RedSupported<OPC, T>::value) {
      return set_error(MMP_E_UNSUPPORTED, "nan-reduction of a non-float dtype");
    } else {
      cudaStream_t st = stream();
      if (!st) return set_error(MMP_E_CUDA, "no stream");
      merge_partials_kernel<OPC, T><<<1, 32, 0, st>>>(parts, nparts, out, out_dt, ddof, merged);
      MMP_LAUNCH_CHECK("merge_partials_kernel");
      return MMP_OK;
    }
  }
};

}  // namespace mmp

extern "C" int mmp_merge_partials(int op, int dtype, const mmp_partial *dev_parts, int nparts, int out_dtype,
                                  void *out, double ddof, mmp_partial *dev_merged) {
  if (nparts < 0) return mmp::set_error(MMP_E_ARG, "negative partial count");
  if ((nparts > 0 && !dev_parts) || !out) return mmp::set_error(MMP_E_ARG, "null pointer");
  if (mmp_dtype_size(out_dtype) == 0) return mmp::set_error(MMP_E_ARG, "bad out dtype");
  if (((uintptr_t)dev_parts) % 8 || ((uintptr_t)dev_merged) % 8)
    return mmp::set_error(MMP_E_ARG, "partials not 8-byte aligned");
  if (!mmp::is_ready()) return mmp::set_error(MMP_E_ARG, "call mmp_init first");
  return mmp::dispatch_op<mmp::MergeRun>(op, dtype, (const PartialOut *)dev_parts, nparts, out_dtype, out, ddof,
                                         (PartialOut *)dev_merged);
}
