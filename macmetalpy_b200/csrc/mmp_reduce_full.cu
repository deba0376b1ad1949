// mmp_reduce: full reductions of contiguous arrays (one launch each).
#include <cuda_runtime.h>

#include "mmp_dispatch.h"

using namespace mmpd;

namespace mmp {

template <int OPC, class T>
struct FullRun {
  // `part` (host) receives the merged partial after a synchronisation;
  // `dev_part` (device), when set, receives it on the stream instead, and
  // `out` may then be NULL (the scalar result goes to scratch).
  static int run(const void *x, long long n, int out_dt, void *out, double ddof, mmp_partial *part,
                 PartialOut *dev_part) {
    if constexpr (!RedSupported<OPC, T>::value) {
      return set_error(MMP_E_UNSUPPORTED, "nan-reduction of a non-float dtype");
    } else {
      typedef typename RedOp<OPC, T>::Acc Acc;
      typedef ContigLoader<T> L;
      constexpr int V = VW<T>::value;
      cudaStream_t st = stream();
      if (!st) return set_error(MMP_E_CUDA, "no stream");
      static int occ = 0;
      if (!occ) {
        MMP_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, reduce_full_kernel<OPC, T, L>,
                                                                   RBLOCK, 0));
        if (occ < 1) occ = 1;
      }
      long long per_block = (long long)RBLOCK * V * 4;
      long long want = (n + per_block - 1) / per_block;
      long long maxb = (long long)sm_count() * occ;
      long long grid = want < 1 ? 1 : (want > maxb ? maxb : want);
      size_t acc_bytes = ((size_t)grid * sizeof(Acc) + 255) & ~size_t(255);
      void *scr = nullptr;
      unsigned *tickets = nullptr;
      int rc = scratch(acc_bytes + sizeof(PartialOut), &scr, &tickets);
      if (rc) return rc;
      PartialOut *slot = (PartialOut *)((char *)scr + acc_bytes);
      PartialOut *dpart = dev_part ? dev_part : (part ? slot : nullptr);
      if (!out) out = slot;  // result unused: any 8 bytes of scratch
      L ld;
      ld.x = (const T *)x;
      ld.aligned = ((uintptr_t)x % 16) == 0;
      reduce_full_kernel<OPC, T, L><<<(unsigned)grid, RBLOCK, 0, st>>>(ld, n, out, out_dt, ddof, scr,
                                                                      tickets, dpart);
      MMP_LAUNCH_CHECK("reduce_full_kernel");
      if (part) {
        PartialOut hp;
        MMP_CUDA_TRY(cudaMemcpyAsync(&hp, dpart, sizeof hp, cudaMemcpyDeviceToHost, st));
        MMP_CUDA_TRY(cudaStreamSynchronize(st));
        part->s1 = hp.s1;
        part->s2 = hp.s2;
        part->shift = hp.shift;
        part->count = hp.count;
        part->ival = hp.ival;
        part->index = hp.index;
      }
      return MMP_OK;
    }
  }
};

}  // namespace mmp

extern "C" int mmp_reduce(int op, int dtype, const void *x, int64_t n, int out_dtype, void *out,
                          double ddof, mmp_partial *partial) {
  if (n < 0) return mmp::set_error(MMP_E_ARG, "negative element count");
  if ((n > 0 && !x) || !out) return mmp::set_error(MMP_E_ARG, "null pointer");
  if (mmp_dtype_size(out_dtype) == 0) return mmp::set_error(MMP_E_ARG, "bad out dtype");
  if (partial) {
    partial->s1 = partial->s2 = partial->shift = 0.0;
    partial->count = 0;
    partial->ival = 0;
    partial->index = -1;
  }
  return mmp::dispatch_op<mmp::FullRun>(op, dtype, x, (long long)n, out_dtype, out, ddof, partial,
                                        (PartialOut *)nullptr);
}

namespace mmpd {
// A shard's argmax / argmin index is local to the shard: move it to the
// global flat index (absent results, index -1, stay -1).
__global__ void partial_index_base_kernel(PartialOut *p, long long base) {
  if (threadIdx.x == 0 && p->index >= 0) p->index += base;
}
}  // namespace mmpd

extern "C" int mmp_reduce_partial(int op, int dtype, const void *x, int64_t n, int64_t index_base,
                                  mmp_partial *dev_partial) {
  if (n < 0) return mmp::set_error(MMP_E_ARG, "negative element count");
  if ((n > 0 && !x) || !dev_partial) return mmp::set_error(MMP_E_ARG, "null pointer");
  if (((uintptr_t)dev_partial) % 8) return mmp::set_error(MMP_E_ARG, "partial not 8-byte aligned");
  if (!mmp::is_ready()) return mmp::set_error(MMP_E_ARG, "call mmp_init first");
  PartialOut *dp = (PartialOut *)dev_partial;
  int rc = mmp::dispatch_op<mmp::FullRun>(op, dtype, x, (long long)n, (int)MMP_FLOAT64, (void *)nullptr, 0.0,
                                          (mmp_partial *)nullptr, dp);
  if (rc) return rc;
  if ((op == MMP_R_ARGMAX || op == MMP_R_ARGMIN) && index_base != 0) {
    partial_index_base_kernel<<<1, 32, 0, mmp::stream()>>>(dp, (long long)index_base);
    MMP_LAUNCH_CHECK("partial_index_base_kernel");
  }
  return MMP_OK;
}
