// mmp_reduce_axis: reductions over the middle axis of (outer, k, inner).
#include <cuda_runtime.h>

#include "mmp_dispatch.h"

using namespace mmpd;

namespace mmp {

// Reduce row r of a (rows, k) array with the full-GPU kernel.
template <class T>
static int FullDispatchT(int op, const void *x, long long r, long long k, int out_dt, void *out,
                         double ddof) {
  return mmp_reduce(op, DtypeCode<T>::value, (const T *)x + r * k, k, out_dt, out, ddof, nullptr);
}
#define FullDispatch(OPC_, x_, r_, k_, dt_, out_, ddof_) FullDispatchT<T>(OPC_, x_, r_, k_, dt_, out_, ddof_)

template <int OPC, class T>
struct AxisRun {
  static int run(const void *x, long long outer, long long k, long long inner, int out_dt, void *out,
                 double ddof) {
    if constexpr (!RedSupported<OPC, T>::value) {
      return set_error(MMP_E_UNSUPPORTED, "nan-reduction of a non-float dtype");
    } else {
      typedef typename RedOp<OPC, T>::Acc Acc;
      typedef ContigLoader<T> L;
      constexpr int V = VW<T>::value;
      cudaStream_t st = stream();
      if (!st) return set_error(MMP_E_CUDA, "no stream");
      const int sms = sm_count();
      L ld;
      ld.x = (const T *)x;
      ld.aligned = ((uintptr_t)x % 16) == 0;
      const size_t osz = mmp_dtype_size(out_dt);
      if (inner == 1) {
        const long long rows = outer;
        if (rows < 32 && k >= (1ll << 16)) {
          // few long rows: one full-GPU reduction per row
          for (long long r = 0; r < rows; ++r) {
            int rc = FullDispatch(OPC, x, r, k, out_dt, (char *)out + r * osz, ddof);
            if (rc) return rc;
          }
          return MMP_OK;
        }
        if (k >= 2048 || rows < (long long)sms * 4) {
          static int occ = 0;
          if (!occ) {
            MMP_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                &occ, reduce_rows_block_kernel<OPC, T, L>, RBLOCK, 0));
            if (occ < 1) occ = 1;
          }
          long long maxb = (long long)sms * occ;
          long long grid = rows < maxb ? rows : maxb;
          if (grid < 1) grid = 1;
          reduce_rows_block_kernel<OPC, T, L><<<(unsigned)grid, RBLOCK, 0, st>>>(ld, rows, k, out, out_dt,
                                                                               ddof);
          MMP_LAUNCH_CHECK("reduce_rows_block_kernel");
        } else {
          long long blocks = (rows + 7) / 8;
          long long maxb = (long long)sms * 8;
          long long grid = blocks < maxb ? blocks : maxb;
          if (grid < 1) grid = 1;
          reduce_rows_warp_kernel<OPC, T, L><<<(unsigned)grid, RBLOCK, 0, st>>>(ld, rows, k, out, out_dt,
                                                                              ddof);
          MMP_LAUNCH_CHECK("reduce_rows_warp_kernel");
        }
        (void)osz;
        return MMP_OK;
      }
      // column reduction
      constexpr int CV = V < 4 ? V : 4;  // columns per thread (shared memory bound)
      const bool vec = ld.aligned && (inner % CV == 0);
      const int cv = vec ? CV : 1;
      const long long ctiles = (inner + 32 * cv - 1) / (32 * cv);
      const long long gx = outer * ctiles;
      if (gx > 0x7fffffffll) return set_error(MMP_E_ARG, "reduction too large");
      // split the reduced axis so that the grid is one full wave
      int occ = 0;
      if (vec) {
        MMP_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, reduce_cols_kernel<OPC, T, L, CV>, RBLOCK, 0));
      } else {
        MMP_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, reduce_cols_kernel<OPC, T, L, 1>, RBLOCK, 0));
      }
      if (occ < 1) occ = 1;
      long long target = (long long)sms * occ;
      long long S = 1;
      if (gx <= 4096 && gx < target) {
        S = target / gx;
        long long maxS = (k + 63) / 64;  // at least 64 rows per chunk
        if (S > maxS) S = maxS;
        if (S > 65535) S = 65535;
        if (S < 1) S = 1;
      }
      long long kchunk = (k + S - 1) / S;
      if (kchunk < 1) kchunk = 1;
      S = (k + kchunk - 1) / kchunk;
      if (S < 1) S = 1;
      void *scr = nullptr;
      unsigned *tickets = nullptr;
      if (S > 1) {
        int rc = scratch((size_t)S * outer * inner * sizeof(Acc), &scr, &tickets);
        if (rc) return rc;
      }
      dim3 grid((unsigned)gx, (unsigned)S, 1);
      if (vec) {
        reduce_cols_kernel<OPC, T, L, CV><<<grid, RBLOCK, 0, st>>>(ld, outer, k, inner, kchunk, out, out_dt,
                                                                  ddof, scr, tickets);
      } else {
        reduce_cols_kernel<OPC, T, L, 1><<<grid, RBLOCK, 0, st>>>(ld, outer, k, inner, kchunk, out, out_dt,
                                                                  ddof, scr, tickets);
      }
      MMP_LAUNCH_CHECK("reduce_cols_kernel");
      return MMP_OK;
    }
  }
};

}  // namespace mmp

extern "C" int mmp_reduce_axis(int op, int dtype, const void *x, int64_t outer, int64_t k, int64_t inner,
                               int out_dtype, void *out, double ddof) {
  if (outer < 0 || k < 0 || inner < 0) return mmp::set_error(MMP_E_ARG, "negative extent");
  if (outer == 0 || inner == 0) return MMP_OK;
  if (!out || (k > 0 && !x)) return mmp::set_error(MMP_E_ARG, "null pointer");
  if (k == 0) return mmp::set_error(MMP_E_ARG, "reduction over an empty axis");
  if (mmp_dtype_size(out_dtype) == 0) return mmp::set_error(MMP_E_ARG, "bad out dtype");
  return mmp::dispatch_op<mmp::AxisRun>(op, dtype, x, (long long)outer, (long long)k, (long long)inner,
                                        out_dtype, out, ddof);
}
