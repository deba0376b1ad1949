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
#include "mmp_scan.cuh"

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

// ---- fused reduce + exchange (mmp_reduce_allranks).  Exchange block of a
// rank: slots [2 parities][64 ranks] of 64 bytes (a partial), then flags
// [2 parities][64 ranks] of 8 bytes (the epoch of the last store).  Calls
// alternate parities: a rank can only overwrite parity p again after every
// rank has finished the call before (their flags of the other parity were
// needed to get there), so a slot is never rewritten while it is read.
constexpr int XSLOT = 64;
constexpr int XFLAG_OFF = 2 * 64 * XSLOT;
static_assert(XFLAG_OFF + 2 * 64 * 8 <= MMP_XBLOCK_BYTES, "exchange block layout");

struct XPeers {
  unsigned char *blk[64];
};

__device__ __forceinline__ void st_sys_v2(void *p, unsigned long long a, unsigned long long b) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_sys_v2(const void *p, unsigned long long &a, unsigned long long &b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ unsigned long long ld_sys_u64(const void *p) {
  unsigned long long v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// The exchange and merge, run by one full warp of one block.  `p` (valid in
// lane 0) is this rank's partial; it goes into slot [par][rank] of every
// rank's block, then the epoch into flag [par][rank]; the warp waits for
// every rank's flag in its own block (bounded: 2 s, then device error 8 and
// the missing ranks count as empty) and lane 0 folds the partials of ranks
// 0 .. upto-1 in rank order and finishes into out (out_dt) -- upto = nranks
// for a reduction, rank for the carry of a scan.
template <int OPC, class T>
__device__ __forceinline__ void exchange_merge_warp(const PartialOut &p, const XPeers &peers, int rank, int nranks,
                                                    int upto, unsigned long long epoch, void *out, int out_dt,
                                                    double ddof, int *err) {
  const int lane = threadIdx.x & 31;
  unsigned long long f[6];
  if (lane == 0) {
    memcpy(&f[0], &p.s1, 8);
    memcpy(&f[1], &p.s2, 8);
    memcpy(&f[2], &p.shift, 8);
    f[3] = (unsigned long long)p.count;
    f[4] = (unsigned long long)p.ival;
    f[5] = (unsigned long long)p.index;
  }
#pragma unroll
  for (int q = 0; q < 6; ++q) f[q] = __shfl_sync(0xffffffffu, f[q], 0);
  const int par = (int)(epoch & 1ull);
  const long long slot_off = (long long)(par * 64 + rank) * XSLOT;
  const long long flag_off = XFLAG_OFF + (long long)(par * 64 + rank) * 8;
  // ---- the partial into slot [par][rank] of every rank's block, then the flag
  for (int r = lane; r < nranks; r += 32) {
    unsigned char *b = peers.blk[r];
    st_sys_v2(b + slot_off, f[0], f[1]);
    st_sys_v2(b + slot_off + 16, f[2], f[3]);
    st_sys_v2(b + slot_off + 32, f[4], f[5]);
  }
  __threadfence_system();  // the slots before any flag, on every peer
  for (int r = lane; r < nranks; r += 32) {
    unsigned char *b = peers.blk[r];
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(b + flag_off), "l"(epoch) : "memory");
  }
  // ---- wait for every rank's flag in this rank's own block (bounded)
  unsigned char *own = peers.blk[rank];
  bool missing = false;
  for (int r = lane; r < nranks; r += 32) {
    const void *fp = own + XFLAG_OFF + (long long)(par * 64 + r) * 8;
    const unsigned long long t0 = now_ns();
    unsigned ns = 32;
    while (ld_sys_u64(fp) != epoch) {
      if (now_ns() - t0 > 2000000000ull) {
        missing = true;
        break;
      }
      __nanosleep(ns);
      if (ns < 1024) ns <<= 1;
    }
  }
  // each lane saw some ranks' flags: fence after its observations, then the
  // warp barrier orders them before lane 0 reads every slot
  __threadfence_system();
  __syncwarp();
  if (__any_sync(0xffffffffu, missing) && lane == 0) atomicExch(err, 8);
  if (lane != 0) return;
  // ---- merge in rank order, as mmp_merge_partials
  typedef RedOp<OPC, T> Op;
  typename Op::Acc a = Op::init();
  long long cnt = 0;
  bool seen = false;
  for (int r = 0; r < upto; ++r) {
    const unsigned char *sp = own + (long long)(par * 64 + r) * XSLOT;
    unsigned long long g[6];
    ld_sys_v2(sp, g[0], g[1]);
    ld_sys_v2(sp + 16, g[2], g[3]);
    ld_sys_v2(sp + 32, g[4], g[5]);
    if (ld_sys_u64(own + XFLAG_OFF + (long long)(par * 64 + r) * 8) != epoch) continue;  // never arrived
    PartialOut q;
    memcpy(&q.s1, &g[0], 8);
    memcpy(&q.s2, &g[1], 8);
    memcpy(&q.shift, &g[2], 8);
    q.count = (long long)g[3];
    q.ival = (long long)g[4];
    q.index = (long long)g[5];
    MergeFold<OPC, T>::fold(a, q, seen);
    cnt += q.count;
  }
  Op::finish(a, cnt, out, 0, out_dt, ddof, nullptr);
}

template <int OPC, class T>
__global__ void __launch_bounds__(RBLOCK) reduce_exchange_kernel(ContigLoader<T> ld, long long n,
                                                                 long long index_base, void *out, int out_dt,
                                                                 double ddof, void *scratch, unsigned *ticket,
                                                                 PartialOut *mine, XPeers peers, int rank,
                                                                 int nranks, int upto, unsigned long long epoch,
                                                                 int *err) {
  // this rank's partial, by the single-GPU reduction (its finishing block
  // goes on below; every other block returns)
  if (!reduce_full_body<OPC, T, ContigLoader<T>>(ld, n, (void *)&mine->shift, MMP_DT_FLOAT64, ddof, scratch,
                                                 ticket, mine))
    return;
  if (threadIdx.x >= 32) return;
  __syncwarp();
  PartialOut p;
  if (threadIdx.x == 0) {  // lane 0 wrote the partial (Op::finish)
    p = *mine;
    if ((OPC == MMP_R_ARGMAX || OPC == MMP_R_ARGMIN) && p.index >= 0) p.index += index_base;
  }
  exchange_merge_warp<OPC, T>(p, peers, rank, nranks, upto, epoch, out, out_dt, ddof, err);
}

// ---- column all-reduce over peer memory (mmp_allreduce_sum_peer).  The
// exchange block's column area follows its first 16 KB: one MMP_XCOL_BYTES
// region per call parity.  Every block copies its share of `send` into this
// rank's region; the last block to finish (ticket) raises this rank's flag
// in every rank's block; every block waits (bounded) for every rank's flag
// and sums its share of the columns over the ranks, in rank order, into
// out (out_dt).  All blocks of a launch are resident at once (the grid is
// at most one block per SM), so the last block always arrives.
constexpr long long XCOL_OFF = 16384;
static_assert(XCOL_OFF >= XFLAG_OFF + 2 * 64 * 8, "column area after the flags");
static_assert(XCOL_OFF + 2ll * MMP_XCOL_BYTES <= MMP_XBLOCK_BYTES, "exchange block layout");

template <class W>
__global__ void __launch_bounds__(RBLOCK) allreduce_cols_kernel(const W *__restrict__ send, long long count,
                                                                void *out, int out_dt, XPeers peers, int rank,
                                                                int nranks, unsigned long long epoch,
                                                                unsigned *ticket, int *err) {
  const int par = (int)(epoch & 1ull);
  const long long area = XCOL_OFF + (long long)par * MMP_XCOL_BYTES;
  W *mine = reinterpret_cast<W *>(peers.blk[rank] + area);
  const long long stride = (long long)gridDim.x * RBLOCK;
  const long long t0 = (long long)blockIdx.x * RBLOCK + threadIdx.x;
  for (long long i = t0; i < count; i += stride) mine[i] = send[i];
  __threadfence_system();  // this thread's copies before the block's ticket
  __syncthreads();
  __shared__ int s_last;
  __shared__ unsigned long long s_seen;
  if (threadIdx.x == 0) s_last = atomicAdd(ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (s_last) {
    // every block's copies are fenced and counted: raise this rank's flag
    if (threadIdx.x == 0) *ticket = 0u;  // for the next launch
    __threadfence_system();
    for (int r = threadIdx.x; r < nranks; r += RBLOCK) {
      unsigned char *b = peers.blk[r];
      asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(b + XFLAG_OFF + (long long)(par * 64 + rank) * 8),
                   "l"(epoch)
                   : "memory");
    }
  }
  // ---- every rank's flag in this rank's block (bounded: 2 s)
  if (threadIdx.x == 0) {
    unsigned long long seen = 0;
    const unsigned char *own = peers.blk[rank];
    for (int r = 0; r < nranks; ++r) {
      const void *fp = own + XFLAG_OFF + (long long)(par * 64 + r) * 8;
      const unsigned long long ts = now_ns();
      unsigned ns = 32;
      bool ok = true;
      while (ld_sys_u64(fp) != epoch) {
        if (now_ns() - ts > 2000000000ull) {
          ok = false;
          break;
        }
        __nanosleep(ns);
        if (ns < 1024) ns <<= 1;
      }
      if (ok) seen |= 1ull << r;
      else atomicExch(err, 8);
    }
    s_seen = seen;
  }
  __threadfence_system();
  __syncthreads();
  const unsigned long long seen = s_seen;
  constexpr bool kFloat = IsFloat<W>::value;
  constexpr bool kUnsigned = !kFloat && W(-1) > W(0);
  for (long long i = t0; i < count; i += stride) {
    W acc = W(0);
    for (int r = 0; r < nranks; ++r) {
      if (!((seen >> r) & 1ull)) continue;  // never arrived: counts as empty
      const unsigned long long bits =
          ld_sys_u64(peers.blk[r] + area + (unsigned long long)i * sizeof(W));
      W v;
      memcpy(&v, &bits, sizeof(W));
      acc += v;
    }
    if constexpr (kFloat) store_scalar(out, i, out_dt, false, 0, 0, (double)acc, false);
    else if constexpr (kUnsigned) store_scalar(out, i, out_dt, true, 0, (unsigned long long)acc, 0.0, true);
    else store_scalar(out, i, out_dt, true, (long long)acc, 0, 0.0, false);
  }
}

// The carry of a distributed scan from the shard's tile aggregates (the
// first launch of the long-row scan): one block sums (multiplies) the
// aggregates in the carry type, then its first warp exchanges the shard
// total and folds the lower ranks' totals into carry_out.
template <class T, bool PROD>
__global__ void __launch_bounds__(RBLOCK) scan_total_exchange_kernel(const typename ScanTypes<T>::carry_t *agg,
                                                                     long long ntiles, void *carry_out,
                                                                     int carry_dt, XPeers peers, int rank,
                                                                     int nranks, unsigned long long epoch,
                                                                     int *err) {
  typedef typename ScanTypes<T>::carry_t C;
  typedef ScanOp<PROD> SOp;
  __shared__ C s_part[RBLOCK / 32];
  C a = SOp::template id<C>();
  for (long long i = threadIdx.x; i < ntiles; i += RBLOCK) a = SOp::op(a, agg[i]);
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) a = SOp::op(a, __shfl_xor_sync(0xffffffffu, a, d));
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = a;
  __syncthreads();
  if (threadIdx.x >= 32) return;
  PartialOut p;
  if (threadIdx.x == 0) {
    C t = s_part[0];
#pragma unroll
    for (int w = 1; w < RBLOCK / 32; ++w) t = SOp::op(t, s_part[w]);  // fixed order
    p.s1 = (double)t;
    p.s2 = 0.0;
    p.shift = 0.0;
    p.ival = (long long)t;
    p.count = ntiles;
    p.index = -1;
  }
  exchange_merge_warp<PROD ? MMP_R_PROD : MMP_R_SUM, T>(p, peers, rank, nranks, rank, epoch, carry_out, carry_dt,
                                                       0.0, err);
}

}  // namespace mmpd

namespace mmp {

template <int OPC, class T>
struct XRun {
  // upto < 0: merge every rank (a reduction); otherwise the ranks below
  // this one (the carry of a scan)
  static int run(const void *x, long long n, long long index_base, int out_dt, void *out, double ddof, int upto) {
    if constexpr (!RedSupported<OPC, T>::value) {
      return set_error(MMP_E_UNSUPPORTED, "nan-reduction of a non-float dtype");
    } else {
      void *blk[64];
      int rank = 0, nranks = 0;
      unsigned long long epoch = 0;
      if (!peer_table(blk, &rank, &nranks, &epoch))
        return set_error(MMP_E_COMM, "no peer exchange on this device: call mmp_comm_peer_init");
      cudaStream_t st = stream();
      if (!st) return set_error(MMP_E_CUDA, "no stream");
      typedef typename RedOp<OPC, T>::Acc Acc;
      constexpr int V = VW<T>::value;
      static int occ = 0;
      if (!occ) {
        MMP_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, reduce_exchange_kernel<OPC, T>, RBLOCK, 0));
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
      PartialOut *mine = (PartialOut *)((char *)scr + acc_bytes);
      ContigLoader<T> ld;
      ld.x = (const T *)x;
      ld.aligned = ((uintptr_t)x % 16) == 0;
      XPeers xp;
      for (int q = 0; q < 64; ++q) xp.blk[q] = q < nranks ? (unsigned char *)blk[q] : nullptr;
      reduce_exchange_kernel<OPC, T><<<(unsigned)grid, RBLOCK, 0, st>>>(ld, n, (long long)index_base, out, out_dt,
                                                                       ddof, scr, tickets, mine, xp, rank, nranks,
                                                                       upto < 0 ? nranks : rank, epoch,
                                                                       device_error_word());
      MMP_LAUNCH_CHECK("reduce_exchange_kernel");
      return MMP_OK;
    }
  }
};

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

extern "C" int mmp_reduce_allranks(int op, int dtype, const void *x, int64_t n, int64_t index_base, int out_dtype,
                                   void *out, double ddof) {
  if (n < 0) return mmp::set_error(MMP_E_ARG, "negative element count");
  if ((n > 0 && !x) || !out) return mmp::set_error(MMP_E_ARG, "null pointer");
  if (mmp_dtype_size(out_dtype) == 0) return mmp::set_error(MMP_E_ARG, "bad out dtype");
  if (!mmp::is_ready()) return mmp::set_error(MMP_E_ARG, "call mmp_init first");
  return mmp::dispatch_op<mmp::XRun>(op, dtype, x, (long long)n, (long long)index_base, out_dtype, out, ddof, -1);
}

namespace mmp {

template <int PRODI, class T>
struct ScanCarryRun {
  static int run(const void *agg, long long ntiles, void *carry_out) {
    typedef typename ScanTypes<T>::carry_t C;
    void *blk[64];
    int rank = 0, nranks = 0;
    unsigned long long epoch = 0;
    if (!peer_table(blk, &rank, &nranks, &epoch))
      return set_error(MMP_E_COMM, "no peer exchange on this device: call mmp_comm_peer_init");
    XPeers xp;
    for (int q = 0; q < 64; ++q) xp.blk[q] = q < nranks ? (unsigned char *)blk[q] : nullptr;
    const int cdt = IsFloatT<C>::value ? MMP_FLOAT64 : (IsSigned<C>::value ? MMP_INT64 : MMP_UINT64);
    scan_total_exchange_kernel<T, PRODI != 0><<<1, RBLOCK, 0, stream()>>>((const C *)agg, ntiles, carry_out, cdt, xp,
                                                                        rank, nranks, epoch, device_error_word());
    MMP_LAUNCH_CHECK("scan_total_exchange_kernel");
    return MMP_OK;
  }
};

template <class W>
int allreduce_cols_run(const void *send, void *recv, long long count, int out_dt) {
  void *blk[64];
  int rank = 0, nranks = 0;
  unsigned long long epoch = 0;
  if (!peer_table(blk, &rank, &nranks, &epoch))
    return set_error(MMP_E_UNSUPPORTED, "no peer exchange on this device: call mmp_comm_peer_init");
  cudaStream_t st = stream();
  if (!st) return set_error(MMP_E_CUDA, "no stream");
  void *scr = nullptr;
  unsigned *tickets = nullptr;
  int rc = scratch(256, &scr, &tickets);
  if (rc) return rc;
  XPeers xp;
  for (int q = 0; q < 64; ++q) xp.blk[q] = q < nranks ? (unsigned char *)blk[q] : nullptr;
  long long grid = (count + RBLOCK - 1) / RBLOCK;
  if (grid > sm_count()) grid = sm_count();  // one block per SM at most: all resident
  if (grid < 1) grid = 1;
  allreduce_cols_kernel<W><<<(unsigned)grid, RBLOCK, 0, st>>>((const W *)send, count, recv, out_dt, xp, rank,
                                                                nranks, epoch, tickets, device_error_word());
  MMP_LAUNCH_CHECK("allreduce_cols_kernel");
  return MMP_OK;
}

// The carry of a distributed scan (the combination of the lower ranks'
// shard totals), by the exchange: from the shard's tile aggregates (`agg`,
// ntiles values of the carry type) when given, else from a full reduction
// of x[0..n).  One exchange epoch either way, so ranks whose shards take
// different paths still meet.
int scan_carry_allranks(int prod, int dtype, const void *agg, long long ntiles, const void *x, long long n,
                        void *carry_out) {
  if (agg) {
    if (prod) return dispatch_dtype<ScanCarryRun, 1>(dtype, agg, ntiles, carry_out);
    return dispatch_dtype<ScanCarryRun, 0>(dtype, agg, ntiles, carry_out);
  }
  int cdt;
  switch (dtype) {
    case MMP_FLOAT16: case MMP_FLOAT32: case MMP_FLOAT64: cdt = MMP_FLOAT64; break;
    case MMP_UINT16: case MMP_UINT32: case MMP_UINT64: cdt = MMP_UINT64; break;
    default: cdt = MMP_INT64;
  }
  return dispatch_op<XRun>(prod ? MMP_R_PROD : MMP_R_SUM, dtype, x, n, 0ll, cdt, carry_out, 0.0, 0);
}

}  // namespace mmp


extern "C" int mmp_allreduce_sum_peer(const void *send, void *recv, size_t count, int dtype, int out_dtype) {
  if ((count > 0 && (!send || !recv)) || mmp_dtype_size(out_dtype) == 0)
    return mmp::set_error(MMP_E_ARG, "bad argument to mmp_allreduce_sum_peer");
  if (count * 8 > (size_t)MMP_XCOL_BYTES)
    return mmp::set_error(MMP_E_UNSUPPORTED, "column buffer larger than the exchange area");
  if (!mmp::is_ready()) return mmp::set_error(MMP_E_ARG, "call mmp_init first");
  switch (dtype) {
    case MMP_FLOAT64: return mmp::allreduce_cols_run<double>(send, recv, (long long)count, out_dtype);
    case MMP_INT64: return mmp::allreduce_cols_run<long long>(send, recv, (long long)count, out_dtype);
    case MMP_UINT64: return mmp::allreduce_cols_run<unsigned long long>(send, recv, (long long)count, out_dtype);
    default: return mmp::set_error(MMP_E_ARG, "mmp_allreduce_sum_peer sums int64, uint64 or float64");
  }
}
