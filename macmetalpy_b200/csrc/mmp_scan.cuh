// Inclusive scans (cumsum / cumprod) for sm_100a.
//
// Reference: parallel_scan_shader (src/macmetalpy/_kernels.py:1263-1358) runs
// three launches -- a serial scan of 1024 elements per thread, a scan of the
// block totals on ONE thread, and a propagate pass -- and keeps the input
// dtype (int32 stays int32); the axis variant (prefix_sum, _kernels.py:1148)
// scans one row per thread after a transpose copy (ndarray.py:2068-2152).
// Results here follow numpy (the reference's CPU path): integer cumsum
// accumulates and returns 64-bit integers, float cumsum returns the input
// float type.
//
// Rows of a (rows, k) view are cut into tiles of STILE = 4096 elements
// (256 threads x 16).  Each block
// takes the next tile id from a global counter (so every lower tile is
// already running), reduces its tile (one barrier) and publishes the tile
// aggregate at once, then looks back over its predecessors within the same row
// (decoupled look-back, warp 0, while the other warps compute their
// tile-local prefixes) until it meets a published inclusive prefix, then
// publishes its own inclusive prefix and writes its outputs: one read and
// one write of the data, one launch.  Every wait is bounded; a wait that
// runs out sets the device error word and the block carries on, so a fault
// shows up as an error from mmp_check_device_error, never as a hang.
//
// Float and half inputs are summed in f64 throughout: a thread's own 16
// consecutive elements, every total across threads, tile aggregate and
// carry.  Each output is then one rounding of the f64 prefix.  (With f32
// sums over a thread's 16 elements, their rounding errors add up along the
// row like a random walk: on signed data the error at a zero crossing
// reached 2.4e-4 to 8.7e-3 of eps * sum|x| at 2^20 to 2^25 elements, above
// the 1e-4 bar; f64 sums give 6e-8.)
#pragma once
#include "mmp_device.cuh"

namespace mmpd {

constexpr int SBLOCK = 256;
constexpr int SITEMS = 16;
constexpr int STILE = SBLOCK * SITEMS;

template <class T> struct ScanTypes {  // signed integers and bool
  typedef long long local_t;
  typedef long long carry_t;
};
template <> struct ScanTypes<unsigned short> { typedef unsigned long long local_t; typedef unsigned long long carry_t; };
template <> struct ScanTypes<unsigned int> { typedef unsigned long long local_t; typedef unsigned long long carry_t; };
template <> struct ScanTypes<unsigned long long> { typedef unsigned long long local_t; typedef unsigned long long carry_t; };
template <> struct ScanTypes<float> { typedef double local_t; typedef double carry_t; };
template <> struct ScanTypes<__half> { typedef double local_t; typedef double carry_t; };
template <> struct ScanTypes<double> { typedef double local_t; typedef double carry_t; };

template <bool PROD> struct ScanOp {
  template <class A> __device__ __forceinline__ static A id() { return PROD ? A(1) : A(0); }
  template <class A> __device__ __forceinline__ static A op(A a, A b) { return PROD ? a * b : a + b; }
};

template <class L, class T>
__device__ __forceinline__ L to_local(T v) { return (L)v; }
template <>
__device__ __forceinline__ double to_local<double, __half>(__half v) { return (double)__half2float(v); }
template <>
__device__ __forceinline__ long long to_local<long long, bool>(bool v) { return v ? 1 : 0; }

// Per-tile state: the value and its flag in one 16-byte descriptor, written
// and read with single 16-byte accesses, so a reader never sees a flag
// without its value and no memory fence is needed between them.  flag =
// (epoch << 2) | state, state 1 = aggregate, 2 = inclusive prefix; a flag
// from an older launch reads as "not ready", so descriptors are never
// cleared between launches.
template <class C>
struct __align__(16) TileDesc {
  C value;
  unsigned long long flag;
};
template <class C>
struct TileState {
  TileDesc<C> *desc;
};

template <class C>
__device__ __forceinline__ void desc_store(TileDesc<C> *d, C v, unsigned long long flag) {
  unsigned long long bits;
  memcpy(&bits, &v, 8);
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(d), "l"(bits), "l"(flag) : "memory");
}
template <class C>
__device__ __forceinline__ void desc_load(const TileDesc<C> *d, C &v, unsigned long long &flag) {
  unsigned long long bits;
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(bits), "=l"(flag) : "l"(d) : "memory");
  memcpy(&v, &bits, 8);
}

__device__ __forceinline__ bool desc_ready(unsigned long long f, unsigned epoch) {
  return (unsigned)(f >> 2) == (epoch & 0x3fffffffu) && (f & 3ull);
}

// Wait for tile `t`'s descriptor of this launch (given its first read);
// spins, then backs off; bounded.  Returns the state (1 or 2), or 0 when
// the wait ran out (the device error word is set).
template <class C>
__device__ __forceinline__ unsigned wait_desc(const TileDesc<C> *desc, long long t, unsigned epoch, int *err,
                                              C &val, unsigned long long f) {
  unsigned ns = 32;
  for (long long it = 0; !desc_ready(f, epoch); ++it) {
    if (it >= (1ll << 22)) {
      atomicExch(err, 2);  // look-back wait ran out
      return 0;
    }
    if (it >= 64) {
      __nanosleep(ns);
      if (ns < 512) ns <<= 1;
    }
    desc_load(desc + t, val, f);
  }
  return (unsigned)(f & 3ull);
}

// Decoupled look-back by one full warp: the exclusive prefix of `tile`
// (its row starts at tile row_first) from the descriptors of its
// predecessors, 32 * LB_PER_LANE per round (lane 0 the nearest),
// folding aggregates back to the nearest inclusive prefix.  Measured on
// B200, one descriptor per lane (a 32-tile window) beats four (128) by
// 15-20 % on scans of 2^22 - 2^24 elements.  `carry` (one row only) stands
// as an inclusive prefix before the row's first tile.  A wait that runs out
// sets device error 2 and ends the look-back there.  Every lane returns the
// prefix.
template <class C, bool PROD, int LB_PER_LANE = 1>
__device__ __forceinline__ C lookback_warp(const TileDesc<C> *desc, long long tile, long long row_first, unsigned ep,
                                           int *err, const C *carry) {
  typedef ScanOp<PROD> Op;
  constexpr int LB_WINDOW = 32 * LB_PER_LANE;
  const int lane = threadIdx.x & 31;
  C excl = Op::template id<C>();
  long long look = tile - 1;  // the nearest tile not folded in yet
#pragma unroll 1
  for (;;) {
    C val[LB_PER_LANE];
    unsigned long long f[LB_PER_LANE];
    // issue every read of the round first (one round trip), then wait
#pragma unroll
    for (int q = 0; q < LB_PER_LANE; ++q) {
      const long long t = look - LB_PER_LANE * lane - q;
      val[q] = Op::template id<C>();
      f[q] = 0;
      if (t >= row_first) desc_load(desc + t, val[q], f[q]);
      else if (carry && t == row_first - 1) val[q] = *carry;
    }
    int stop = LB_PER_LANE;  // this lane's nearest inclusive prefix (or end)
#pragma unroll
    for (int q = 0; q < LB_PER_LANE; ++q) {
      const long long t = look - LB_PER_LANE * lane - q;
      unsigned state = 2;  // before the row: an inclusive prefix
      if (t >= row_first) {
        state = wait_desc(desc, t, ep, err, val[q], f[q]);
        if (state == 0) val[q] = Op::template id<C>();  // ran out: stop here
      }
      if (state != 1 && stop == LB_PER_LANE) stop = q;
    }
    const unsigned m = __ballot_sync(0xffffffffu, stop < LB_PER_LANE);
    const int first = m ? __ffs(m) - 1 : 32;  // the lane holding the nearest one
    C part = Op::template id<C>();
#pragma unroll
    for (int q = 0; q < LB_PER_LANE; ++q)
      if (lane < first || (lane == first && q <= stop)) part = Op::op(part, val[q]);
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) part = Op::op(part, __shfl_xor_sync(0xffffffffu, part, d));
    excl = Op::op(excl, part);
    if (m) return excl;
    look -= LB_WINDOW;
  }
}

// Tile staging through shared memory in 16-byte chunks.  Chunk c of a tile
// (elements c*16/sizeof(E) ...) is kept at chunk c ^ ((c >> 3) & 7): the
// coalesced global side (consecutive threads, consecutive chunks) and the
// per-thread side (a thread's SITEMS consecutive elements, 1 to 8 chunks)
// both reach eight different bank groups per quarter warp, with one 16-byte
// shared-memory access per chunk instead of one per element.
__device__ __forceinline__ int chunk_swz(int c) { return c ^ ((c >> 3) & 7); }

template <class T, class O>
constexpr int StageSize() {
  return STILE * (int)(sizeof(T) > sizeof(O) ? sizeof(T) : sizeof(O));
}

// the whole tile (STILE elements from src, 16-byte aligned) into the stage
template <class T>
__device__ __forceinline__ void stage_load_tile(unsigned char *stage, const T *__restrict__ src) {
  constexpr int VE = 16 / (int)sizeof(T);
#pragma unroll
  for (int q = 0; q < SITEMS / VE; ++q) {
    const int c = q * SBLOCK + (int)threadIdx.x;
    *reinterpret_cast<Vec<T, VE> *>(stage + chunk_swz(c) * 16) = ldvec_stream<T, VE>(src + (long long)c * VE);
  }
}
// this thread's SITEMS consecutive elements out of the stage
template <class T, class A>
__device__ __forceinline__ void stage_read_thread(const unsigned char *stage, A (&v)[SITEMS]) {
  constexpr int VE = 16 / (int)sizeof(T);
#pragma unroll
  for (int q = 0; q < SITEMS / VE; ++q) {
    const Vec<T, VE> t =
        *reinterpret_cast<const Vec<T, VE> *>(stage + chunk_swz((int)threadIdx.x * (SITEMS / VE) + q) * 16);
#pragma unroll
    for (int e = 0; e < VE; ++e) v[q * VE + e] = to_local<A, T>(t.v[e]);
  }
}
// this thread's SITEMS consecutive outputs into the stage
template <class O>
__device__ __forceinline__ void stage_write_thread(unsigned char *stage, const O (&r)[SITEMS]) {
  constexpr int VO = 16 / (int)sizeof(O);
#pragma unroll
  for (int q = 0; q < SITEMS / VO; ++q) {
    Vec<O, VO> t;
#pragma unroll
    for (int e = 0; e < VO; ++e) t.v[e] = r[q * VO + e];
    *reinterpret_cast<Vec<O, VO> *>(stage + chunk_swz((int)threadIdx.x * (SITEMS / VO) + q) * 16) = t;
  }
}
// the whole staged tile out to dst (16-byte aligned), coalesced
template <class O>
__device__ __forceinline__ void stage_store_tile(const unsigned char *stage, O *__restrict__ dst) {
  constexpr int VO = 16 / (int)sizeof(O);
#pragma unroll
  for (int q = 0; q < SITEMS / VO; ++q) {
    const int c = q * SBLOCK + (int)threadIdx.x;
    stvec_stream<O, VO>(dst + (long long)c * VO, *reinterpret_cast<const Vec<O, VO> *>(stage + chunk_swz(c) * 16));
  }
}

// Resident blocks per SM the tile kernels are compiled for: the look-back
// kernel's speed follows the number of tiles in flight (each waits on its
// look-back); with 64-bit locals, 4-byte and smaller inputs keep 4 blocks
// per SM, 8-byte inputs 2.
template <class T> struct LookbackMinBlocks { static constexpr int value = sizeof(T) >= 8 ? 2 : 4; };

template <class T, class O, bool PROD>
__global__ void __launch_bounds__(SBLOCK, LookbackMinBlocks<T>::value) scan_tiles_kernel(
    const T *__restrict__ x, O *__restrict__ y, long long rows, long long k, long long tiles_per_row,
    long long total_tiles, TileState<typename ScanTypes<T>::carry_t> st, unsigned *tile_counter,
    unsigned epoch, int *err, const typename ScanTypes<T>::carry_t *carry_in, int vec_ok) {
  typedef typename ScanTypes<T>::local_t A;
  typedef typename ScanTypes<T>::carry_t C;
  typedef ScanOp<PROD> Op;
  __shared__ long long s_tile;
  __shared__ C s_warp[SBLOCK / 32];
  __shared__ C s_excl;
  extern __shared__ __align__(16) unsigned char s_stage[];  // StageSize<T, O>() bytes
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  if (tid == 0) s_tile = (long long)atomicAdd(tile_counter, 1u);
  __syncthreads();
  const long long tile = s_tile;
  if (tid == 0 && tile == total_tiles - 1) *tile_counter = 0u;  // every id is handed out
  if (tile >= total_tiles) return;
  const long long row = tile / tiles_per_row;
  const long long j = tile - row * tiles_per_row;
  const long long start = row * k + j * STILE;
  long long count = k - j * STILE;
  if (count > STILE) count = STILE;
  const unsigned ep = epoch & 0x3fffffffu;

  // ---- load the tile: coalesced 16-byte vectors into shared memory
  // (swizzled 16-byte chunks, see chunk_swz), then SITEMS consecutive
  // elements per thread
  A v[SITEMS];
  const long long my0 = (long long)tid * SITEMS;
  const bool full_vec = vec_ok && count == STILE;
  if (full_vec) {
    stage_load_tile<T>(s_stage, x + start);
    __syncthreads();
    stage_read_thread<T, A>(s_stage, v);
  } else {
#pragma unroll
    for (int e = 0; e < SITEMS; ++e) {
      long long i = my0 + e;
      v[e] = (i < count) ? to_local<A, T>(x[start + i]) : Op::template id<A>();
    }
  }
  // ---- the tile aggregate first, so that it is published as early as
  // possible: thread totals, their warp-inclusive prefixes, one barrier.
  // Everything across threads is in the carry type C (float64 for float
  // inputs): only a thread's own SITEMS elements are summed in A.
#pragma unroll
  for (int e = 1; e < SITEMS; ++e) v[e] = Op::op(v[e - 1], v[e]);  // thread-local prefixes
  C inc = (C)v[SITEMS - 1];
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    C o = __shfl_up_sync(0xffffffffu, inc, d);
    if (lane >= d) inc = Op::op(o, inc);
  }
  if (lane == 31) s_warp[w] = inc;  // warp totals
  __syncthreads();
  // every warp folds the warp totals itself: its exclusive prefix and the
  // tile aggregate (no second barrier)
  C warp_excl = Op::template id<C>();
  C tile_agg = Op::template id<C>();
#pragma unroll
  for (int q = 0; q < SBLOCK / 32; ++q) {
    const C t = s_warp[q];
    if (q < w) warp_excl = Op::op(warp_excl, t);
    tile_agg = Op::op(tile_agg, t);
  }
  // inc is the inclusive prefix of thread totals within the warp; the
  // exclusive prefix is the neighbour's inclusive one.
  C thread_excl;
  {
    C o = __shfl_up_sync(0xffffffffu, inc, 1);
    C wexcl_in_warp = (lane == 0) ? Op::template id<C>() : o;
    thread_excl = Op::op(warp_excl, wexcl_in_warp);
  }

  // ---- decoupled look-back over earlier tiles of the same row
  if (w == 0) {
    C excl = Op::template id<C>();
    const unsigned long long ep2 = (unsigned long long)ep << 2;
    if (j == 0) {
      if (carry_in && rows == 1) excl = (C)(*carry_in);
      if (lane == 0) desc_store(st.desc + tile, Op::op(excl, tile_agg), ep2 | 2ull);
    } else {
      if (lane == 0) desc_store(st.desc + tile, tile_agg, ep2 | 1ull);
      excl = lookback_warp<C, PROD>(st.desc, tile, row * tiles_per_row, ep, err,
                                    (carry_in && rows == 1) ? carry_in : nullptr);
      if (lane == 0) desc_store(st.desc + tile, Op::op(excl, tile_agg), ep2 | 2ull);
    }
    if (lane == 0) s_excl = excl;
  }
  __syncthreads();
  const C base = Op::op(s_excl, thread_excl);

  // ---- outputs: carry and thread prefix (C) + thread-local prefix (A)
  O res[SITEMS];
#pragma unroll
  for (int e = 0; e < SITEMS; ++e) res[e] = cvt<O>(Op::op(base, (C)v[e]));
  if (full_vec) {
    // stage the outputs through shared memory, write 16-byte vectors
    __syncthreads();  // every thread has finished reading its inputs
    stage_write_thread<O>(s_stage, res);
    __syncthreads();
    stage_store_tile<O>(s_stage, y + start);
  } else {
#pragma unroll
    for (int e = 0; e < SITEMS; ++e) {
      long long i = my0 + e;
      if (i < count) y[start + i] = res[e];
    }
  }
}

// ---------------------------------------------------------------------------
// Reduce-then-scan for long rows.  The look-back chain makes every tile wait
// for the slowest aggregate published before it (a tile whose loads came
// back late holds up all later tiles), which caps the look-back kernel near
// half of HBM bandwidth once a row has hundreds of tiles.  Long rows
// therefore take three launches without any wait between tiles:
//   1. tile_aggregates_kernel: one warp per tile sums (or multiplies) its
//      STILE elements into the tile aggregate (no barriers);
//   2. the library's own scan of the aggregates, per row, with the carry;
//   3. scan_tiles_carry_kernel: every tile scans itself with its exclusive
//      prefix (the inclusive aggregate prefix of the tile before it), in
//      reverse tile order so that the tail of the input, the part the first
//      launch read last, is still in L2.
// Bytes moved: 2 reads and 1 write of the data (16 per int32 element
// instead of 12), all at streaming speed.

template <class T, bool PROD>
__global__ void __launch_bounds__(SBLOCK) tile_aggregates_kernel(const T *__restrict__ x, long long k,
                                                                 long long tiles_per_row, long long total_tiles,
                                                                 typename ScanTypes<T>::carry_t *__restrict__ agg,
                                                                 int vec_ok) {
  typedef typename ScanTypes<T>::local_t A;
  typedef typename ScanTypes<T>::carry_t C;
  typedef ScanOp<PROD> Op;
  constexpr int VE = 16 / sizeof(T);          // elements per 16-byte load
  constexpr int NVT = STILE / (32 * VE);      // loads per lane per tile
  constexpr int BATCH = 8;                    // loads in flight per lane
  static_assert(NVT % BATCH == 0, "whole batches per tile");
  const int lane = threadIdx.x & 31;
  const long long nwarps = ((long long)gridDim.x * SBLOCK) >> 5;
  for (long long t = ((long long)blockIdx.x * SBLOCK + threadIdx.x) >> 5; t < total_tiles; t += nwarps) {
    const long long row = t / tiles_per_row;
    const long long j = t - row * tiles_per_row;
    const long long start = row * k + j * STILE;
    long long count = k - j * STILE;
    if (count > STILE) count = STILE;
    C acc = Op::template id<C>();  // float64 for float inputs
    if (vec_ok && count == STILE) {
      const T *p = x + start + lane * VE;
#pragma unroll 1
      for (int q = 0; q < NVT; q += BATCH) {
        Vec<T, VE> b[BATCH];
#pragma unroll
        for (int u = 0; u < BATCH; ++u) b[u] = ldvec<T, VE>(p + (long long)(q + u) * 32 * VE);
#pragma unroll
        for (int u = 0; u < BATCH; ++u)
#pragma unroll
          for (int e = 0; e < VE; ++e) acc = Op::op(acc, (C)to_local<A, T>(b[u].v[e]));
      }
    } else {
      for (long long i = lane; i < count; i += 32) acc = Op::op(acc, (C)to_local<A, T>(x[start + i]));
    }
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) acc = Op::op(acc, __shfl_xor_sync(0xffffffffu, acc, d));
    if (lane == 0) agg[t] = acc;
  }
}

// Tile scan with a known exclusive prefix: incl holds, per row, the
// inclusive scan of the tile aggregates (carry included), so tile j > 0 of
// a row starts from incl[tile - 1].  One block per tile, highest tile first.
template <class T, class O, bool PROD>
__global__ void __launch_bounds__(SBLOCK, LookbackMinBlocks<T>::value) scan_tiles_carry_kernel(
    const T *__restrict__ x, O *__restrict__ y, long long rows, long long k, long long tiles_per_row,
    long long total_tiles, const typename ScanTypes<T>::carry_t *__restrict__ incl,
    const typename ScanTypes<T>::carry_t *carry_in, int vec_ok) {
  typedef typename ScanTypes<T>::local_t A;
  typedef typename ScanTypes<T>::carry_t C;
  typedef ScanOp<PROD> Op;
  __shared__ C s_warp[SBLOCK / 32];
  extern __shared__ __align__(16) unsigned char s_stage[];  // StageSize<T, O>() bytes
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const long long tile = total_tiles - 1 - (long long)blockIdx.x;
  const long long row = tile / tiles_per_row;
  const long long j = tile - row * tiles_per_row;
  const long long start = row * k + j * STILE;
  long long count = k - j * STILE;
  if (count > STILE) count = STILE;
  C excl = Op::template id<C>();
  if (j > 0) excl = incl[tile - 1];
  else if (carry_in && rows == 1) excl = (C)(*carry_in);

  // ---- load: coalesced 16-byte vectors through padded shared memory to
  // SITEMS consecutive elements per thread (as in scan_tiles_kernel)
  A v[SITEMS];
  const long long my0 = (long long)tid * SITEMS;
  const bool full_vec = vec_ok && count == STILE;
  if (full_vec) {
    stage_load_tile<T>(s_stage, x + start);
    __syncthreads();
    stage_read_thread<T, A>(s_stage, v);
  } else {
#pragma unroll
    for (int e = 0; e < SITEMS; ++e) {
      long long i = my0 + e;
      v[e] = (i < count) ? to_local<A, T>(x[start + i]) : Op::template id<A>();
    }
  }
  // ---- thread-local prefixes (A), then thread totals scanned across the
  // tile in C (float64 for float inputs), one barrier
#pragma unroll
  for (int e = 1; e < SITEMS; ++e) v[e] = Op::op(v[e - 1], v[e]);
  C inc = (C)v[SITEMS - 1];
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    C o = __shfl_up_sync(0xffffffffu, inc, d);
    if (lane >= d) inc = Op::op(o, inc);
  }
  if (lane == 31) s_warp[w] = inc;
  __syncthreads();  // also: every thread has read its staged inputs
  C warp_excl = Op::template id<C>();
#pragma unroll
  for (int q = 0; q < SBLOCK / 32; ++q)
    if (q < w) warp_excl = Op::op(warp_excl, s_warp[q]);
  {
    C o = __shfl_up_sync(0xffffffffu, inc, 1);
    excl = Op::op(excl, Op::op(warp_excl, (lane == 0) ? Op::template id<C>() : o));
  }

  // ---- outputs: carry and thread prefix (C) + thread-local prefix (A)
  if (full_vec) {
    O res[SITEMS];
#pragma unroll
    for (int e = 0; e < SITEMS; ++e) res[e] = cvt<O>(Op::op(excl, (C)v[e]));
    stage_write_thread<O>(s_stage, res);
    __syncthreads();
    stage_store_tile<O>(s_stage, y + start);
  } else {
#pragma unroll
    for (int e = 0; e < SITEMS; ++e) {
      long long i = my0 + e;
      if (i < count) y[start + i] = cvt<O>(Op::op(excl, (C)v[e]));
    }
  }
}

// Streaming variant of scan_tiles_carry_kernel for aligned scans (rows a
// multiple of 16 elements, 16-byte aligned input and output): a persistent
// grid, block b taking tiles total-1-b, total-1-b-G, ... (highest first, as
// scan_tiles_carry_kernel), with the next tile's input copied into shared
// memory by cp.async while the current tile is scanned and stored.  Tiles
// depend on nothing but their known prefix, so no block waits on another;
// each block keeps a tile's load in flight at all times instead of loading,
// scanning and storing in turn.
__device__ __forceinline__ void cp_async16(unsigned dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Shared memory of scan_carry_stream_kernel: two input tiles, then the output stage.
template <class T, class O>
constexpr int StreamSmem() {
  return 2 * STILE * (int)sizeof(T) + STILE * (int)sizeof(O);
}

// Start the copy of tile `tile` (skipped when negative) into buf, as
// swizzled 16-byte chunks; one commit group either way.
template <class T>
__device__ __forceinline__ void stream_issue(unsigned char *buf, const T *__restrict__ x, long long tile, long long k,
                                             long long tiles_per_row) {
  constexpr int VE = 16 / (int)sizeof(T);
  if (tile >= 0) {
    const long long row = tile / tiles_per_row, j = tile - row * tiles_per_row;
    long long count = k - j * STILE;
    if (count > STILE) count = STILE;
    const int nch = (int)(count / VE);
    const unsigned base = (unsigned)__cvta_generic_to_shared(buf);
    const char *src = reinterpret_cast<const char *>(x + row * k + j * STILE);
#pragma unroll
    for (int q = 0; q < SITEMS / VE; ++q) {
      const int c = q * SBLOCK + (int)threadIdx.x;
      if (c < nch) cp_async16(base + (unsigned)chunk_swz(c) * 16u, src + (long long)c * 16);
    }
  }
  cp_async_commit();
}

// Scan one tile whose input is staged in shared memory `buf` (swizzled
// 16-byte chunks, `count` elements) from the exclusive prefix `excl`, and
// store the outputs to y + start through the stage s_out (coalesced 16-byte
// streaming stores); returns the tile's total (every thread).  Called by all
// SBLOCK threads after the tile's copy has landed and a barrier; ends with a
// barrier after which buf, s_out and s_warp are free again.
template <class T, class O, bool PROD>
__device__ __forceinline__ typename ScanTypes<T>::carry_t scan_staged_tile(const unsigned char *buf, unsigned char *s_out,
                                                 typename ScanTypes<T>::carry_t *s_warp, long long start,
                                                 long long count, typename ScanTypes<T>::carry_t excl,
                                                 O *__restrict__ y) {
  typedef typename ScanTypes<T>::local_t A;
  typedef typename ScanTypes<T>::carry_t C;
  typedef ScanOp<PROD> Op;
  constexpr int VE = 16 / (int)sizeof(T);
  constexpr int VO = 16 / (int)sizeof(O);
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  // ---- this thread's SITEMS consecutive elements (past count: identity)
  A v[SITEMS];
  const bool full = count == STILE;  // every tile but a row's last: no masks
  if (full) {
    stage_read_thread<T, A>(buf, v);
  } else {
    const int cnt = (int)count;
#pragma unroll
    for (int q = 0; q < SITEMS / VE; ++q) {
      const int c = tid * (SITEMS / VE) + q;
      const Vec<T, VE> t = *reinterpret_cast<const Vec<T, VE> *>(buf + chunk_swz(c) * 16);
#pragma unroll
      for (int e = 0; e < VE; ++e) v[q * VE + e] = (c * VE + e < cnt) ? to_local<A, T>(t.v[e]) : Op::template id<A>();
    }
  }
  // ---- thread-local prefixes (A), thread totals scanned in C
#pragma unroll
  for (int e = 1; e < SITEMS; ++e) v[e] = Op::op(v[e - 1], v[e]);
  C inc = (C)v[SITEMS - 1];
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    C o = __shfl_up_sync(0xffffffffu, inc, d);
    if (lane >= d) inc = Op::op(o, inc);
  }
  if (lane == 31) s_warp[w] = inc;
  __syncthreads();
  C warp_excl = Op::template id<C>();
  C total = Op::template id<C>();
#pragma unroll
  for (int q = 0; q < SBLOCK / 32; ++q) {
    const C t = s_warp[q];
    if (q < w) warp_excl = Op::op(warp_excl, t);
    total = Op::op(total, t);
  }
  {
    C o = __shfl_up_sync(0xffffffffu, inc, 1);
    excl = Op::op(excl, Op::op(warp_excl, (lane == 0) ? Op::template id<C>() : o));
  }
  // ---- outputs through the stage, 16-byte coalesced stores
  O res[SITEMS];
#pragma unroll
  for (int e = 0; e < SITEMS; ++e) res[e] = cvt<O>(Op::op(excl, (C)v[e]));
  stage_write_thread<O>(s_out, res);
  __syncthreads();
  if (full) {
    stage_store_tile<O>(s_out, y + start);
  } else {
    const int nch = (int)(count / VO);
#pragma unroll
    for (int q = 0; q < SITEMS / VO; ++q) {
      const int c = q * SBLOCK + tid;
      if (c < nch)
        stvec_stream<O, VO>(y + start + (long long)c * VO,
                            *reinterpret_cast<const Vec<O, VO> *>(s_out + chunk_swz(c) * 16));
    }
  }
  __syncthreads();  // the stage, s_warp and the tile's buffer are free
  return total;
}

template <class T, class O, bool PROD>
__global__ void __launch_bounds__(SBLOCK, LookbackMinBlocks<T>::value) scan_carry_stream_kernel(
    const T *__restrict__ x, O *__restrict__ y, long long rows, long long k, long long tiles_per_row,
    long long total_tiles, const typename ScanTypes<T>::carry_t *__restrict__ incl,
    const typename ScanTypes<T>::carry_t *carry_in) {
  typedef typename ScanTypes<T>::carry_t C;
  typedef ScanOp<PROD> Op;
  constexpr int TB = STILE * (int)sizeof(T);
  __shared__ C s_warp[SBLOCK / 32];
  extern __shared__ __align__(128) unsigned char s_mem[];  // StreamSmem<T, O>() bytes
  unsigned char *s_out = s_mem + 2 * TB;
  const long long G = gridDim.x;
  const long long first = total_tiles - 1 - (long long)blockIdx.x;

  stream_issue<T>(s_mem, x, first, k, tiles_per_row);
#pragma unroll 1
  for (long long i = 0;; ++i) {
    const long long tile = first - i * G;
    if (tile < 0) break;
    const long long next = tile - G;
    // the other buffer was last read before the previous iteration's final barrier
    stream_issue<T>(s_mem + (int)((i + 1) & 1) * TB, x, next, k, tiles_per_row);
    const long long row = tile / tiles_per_row;
    const long long j = tile - row * tiles_per_row;
    const long long start = row * k + j * STILE;
    long long count = k - j * STILE;
    if (count > STILE) count = STILE;
    C excl = Op::template id<C>();
    if (j > 0) excl = incl[tile - 1];
    else if (carry_in && rows == 1) excl = (C)(*carry_in);
    cp_async_wait1();  // this tile's group has landed (the next one may still be in flight)
    __syncthreads();
    scan_staged_tile<T, O, PROD>(s_mem + (int)(i & 1) * TB, s_out, s_warp, start, count, excl, y);
  }
  cp_async_wait_all();
}

// One warp per row for short rows (k < STILE / 4).
template <class T, class O, bool PROD>
__global__ void __launch_bounds__(SBLOCK) scan_rows_warp_kernel(const T *__restrict__ x,
                                                                O *__restrict__ y, long long rows,
                                                                long long k, const typename ScanTypes<T>::carry_t *carry_in) {
  typedef typename ScanTypes<T>::local_t A;
  typedef typename ScanTypes<T>::carry_t C;
  typedef ScanOp<PROD> Op;
  const int lane = threadIdx.x & 31;
  long long wid = ((long long)blockIdx.x * SBLOCK + threadIdx.x) >> 5;
  long long nw = ((long long)gridDim.x * SBLOCK) >> 5;
  for (long long r = wid; r < rows; r += nw) {
    C carry = Op::template id<C>();
    if (carry_in && rows == 1) carry = (C)(*carry_in);
    for (long long c0 = 0; c0 < k; c0 += 32) {
      long long i = c0 + lane;
      C v = (i < k) ? (C)to_local<A, T>(x[r * k + i]) : Op::template id<C>();
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        C o = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v = Op::op(o, v);
      }
      if (i < k) y[r * k + i] = cvt<O>(Op::op(carry, v));
      carry = Op::op(carry, __shfl_sync(0xffffffffu, v, 31));
    }
  }
}

// Scan along a strided axis of an (outer, k, inner) view, inner > 1: one
// thread per column walks down the k rows (coalesced across columns).
template <class T, class O, bool PROD>
__global__ void __launch_bounds__(SBLOCK) scan_cols_kernel(const T *__restrict__ x,
                                                           O *__restrict__ y, long long outer,
                                                           long long k, long long inner) {
  typedef typename ScanTypes<T>::carry_t C;
  typedef ScanOp<PROD> Op;
  long long g = (long long)blockIdx.x * SBLOCK + threadIdx.x;
  long long total = outer * inner;
  for (; g < total; g += (long long)gridDim.x * SBLOCK) {
    long long o = g / inner, c = g - o * inner;
    long long base = o * k * inner + c;
    C carry = Op::template id<C>();
    for (long long r = 0; r < k; ++r) {
      carry = Op::op(carry, (C)to_local<typename ScanTypes<T>::local_t, T>(x[base + r * inner]));
      y[base + r * inner] = cvt<O>(carry);
    }
  }
}

}  // namespace mmpd
