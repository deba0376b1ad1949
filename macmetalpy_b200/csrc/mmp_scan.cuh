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
// Float inputs are scanned inside a tile in f32 and carried between tiles in
// f64, so the error stays near the f32 rounding of each output instead of
// growing with the prefix length.
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
template <> struct ScanTypes<float> { typedef float local_t; typedef double carry_t; };
template <> struct ScanTypes<__half> { typedef float local_t; typedef double carry_t; };
template <> struct ScanTypes<double> { typedef double local_t; typedef double carry_t; };

template <bool PROD> struct ScanOp {
  template <class A> __device__ __forceinline__ static A id() { return PROD ? A(1) : A(0); }
  template <class A> __device__ __forceinline__ static A op(A a, A b) { return PROD ? a * b : a + b; }
};

template <class L, class T>
__device__ __forceinline__ L to_local(T v) { return (L)v; }
template <>
__device__ __forceinline__ float to_local<float, __half>(__half v) { return __half2float(v); }
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

// Shared-memory index with one padding element per 128 bytes.
template <class E>
__device__ __forceinline__ int spad(int i) {
  return i + i / (int)(128 / sizeof(E));
}
template <class E>
struct StageBytes {
  static constexpr int value = (STILE + STILE / (128 / sizeof(E))) * sizeof(E);
};

template <class T, class O>
constexpr int StageSize() {
  return StageBytes<T>::value > StageBytes<O>::value ? StageBytes<T>::value : StageBytes<O>::value;
}

template <class T, class O, bool PROD>
__global__ void __launch_bounds__(SBLOCK) scan_tiles_kernel(
    const T *__restrict__ x, O *__restrict__ y, long long rows, long long k, long long tiles_per_row,
    long long total_tiles, TileState<typename ScanTypes<T>::carry_t> st, unsigned *tile_counter,
    unsigned epoch, int *err, const typename ScanTypes<T>::carry_t *carry_in, int vec_ok) {
  typedef typename ScanTypes<T>::local_t A;
  typedef typename ScanTypes<T>::carry_t C;
  typedef ScanOp<PROD> Op;
  __shared__ long long s_tile;
  __shared__ A s_warp[SBLOCK / 32];
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

  // ---- load the tile: coalesced 16-byte vectors into shared memory (one
  // padding element per 128 bytes keeps both access patterns free of bank
  // conflicts), then SITEMS consecutive elements per thread
  A v[SITEMS];
  const long long my0 = (long long)tid * SITEMS;
  const bool full_vec = vec_ok && count == STILE;
  if (full_vec) {
    T *smT = reinterpret_cast<T *>(s_stage);
    constexpr int VE = (16 / sizeof(T)) < SITEMS ? (16 / sizeof(T)) : SITEMS;
#pragma unroll
    for (int q = 0; q < SITEMS / VE; ++q) {
      const int i0 = (q * SBLOCK + tid) * VE;
      Vec<T, VE> t = ldvec_stream<T, VE>(x + start + i0);
#pragma unroll
      for (int e = 0; e < VE; ++e) smT[spad<T>(i0 + e)] = t.v[e];
    }
    __syncthreads();
#pragma unroll
    for (int e = 0; e < SITEMS; ++e) v[e] = to_local<A, T>(smT[spad<T>(tid * SITEMS + e)]);
  } else {
#pragma unroll
    for (int e = 0; e < SITEMS; ++e) {
      long long i = my0 + e;
      v[e] = (i < count) ? to_local<A, T>(x[start + i]) : Op::template id<A>();
    }
  }
  // ---- the tile aggregate first, so that it is published as early as
  // possible: thread totals, their warp-inclusive prefixes, one barrier
  A tot = v[0];
#pragma unroll
  for (int e = 1; e < SITEMS; ++e) tot = Op::op(tot, v[e]);
  A inc = tot;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    A o = __shfl_up_sync(0xffffffffu, inc, d);
    if (lane >= d) inc = Op::op(o, inc);
  }
  if (lane == 31) s_warp[w] = inc;  // warp totals
  __syncthreads();
  // every warp folds the warp totals itself: its exclusive prefix and the
  // tile aggregate (no second barrier)
  A warp_excl = Op::template id<A>();
  A tile_agg = Op::template id<A>();
#pragma unroll
  for (int q = 0; q < SBLOCK / 32; ++q) {
    const A t = s_warp[q];
    if (q < w) warp_excl = Op::op(warp_excl, t);
    tile_agg = Op::op(tile_agg, t);
  }
  // inc is the inclusive prefix of thread totals within the warp; the
  // exclusive prefix is the neighbour's inclusive one.
  A thread_excl;
  {
    A o = __shfl_up_sync(0xffffffffu, inc, 1);
    A wexcl_in_warp = (lane == 0) ? Op::template id<A>() : o;
    thread_excl = Op::op(warp_excl, wexcl_in_warp);
  }

  // ---- decoupled look-back over earlier tiles of the same row
  if (w == 0) {
    C excl = Op::template id<C>();
    const unsigned long long ep2 = (unsigned long long)ep << 2;
    if (j == 0) {
      if (carry_in && rows == 1) excl = (C)(*carry_in);
      if (lane == 0) desc_store(st.desc + tile, Op::op(excl, (C)tile_agg), ep2 | 2ull);
    } else {
      if (lane == 0) desc_store(st.desc + tile, (C)tile_agg, ep2 | 1ull);
      const long long row_first = row * tiles_per_row;
      long long look = tile - 1;  // highest tile id still to fold in
      bool done = false;
      // each round looks at 32 predecessors: lane l at tile look - l
      while (!done) {
        const long long t = look - lane;
        C val = Op::template id<C>();
        unsigned state = 2;  // before the row start: an inclusive prefix of identity
        if (t >= row_first) {
          unsigned long long f;
          desc_load(st.desc + t, val, f);
          state = wait_desc(st.desc, t, ep, err, val, f);
          if (state == 0) val = Op::template id<C>();
        } else if (carry_in && rows == 1 && t == row_first - 1) {
          val = (C)(*carry_in);
        }
        const unsigned m = __ballot_sync(0xffffffffu, state == 2);
        const int stop = m ? (__ffs(m) - 1) : 31;
        // fold lanes 0..stop (tile-1, tile-2, ..., the nearest inclusive prefix)
        C part = (lane <= stop) ? val : Op::template id<C>();
#pragma unroll
        for (int d = 16; d >= 1; d >>= 1) part = Op::op(part, __shfl_down_sync(0xffffffffu, part, d));
        excl = Op::op(excl, __shfl_sync(0xffffffffu, part, 0));
        if (m) done = true;
        else look -= 32;
      }
      if (lane == 0) desc_store(st.desc + tile, Op::op(excl, (C)tile_agg), ep2 | 2ull);
    }
    if (lane == 0) s_excl = excl;
  }
  // ---- tile-local inclusive prefixes; warps 1.. do this while warp 0 is
  // still looking back
  v[0] = Op::op(thread_excl, v[0]);
#pragma unroll
  for (int e = 1; e < SITEMS; ++e) v[e] = Op::op(v[e - 1], v[e]);
  __syncthreads();
  const C excl = s_excl;

  // ---- outputs: carry (C) + tile-local prefix (A)
  O res[SITEMS];
#pragma unroll
  for (int e = 0; e < SITEMS; ++e) res[e] = cvt<O>(Op::op(excl, (C)v[e]));
  if (full_vec) {
    // stage the outputs through shared memory, write 16-byte vectors
    O *smO = reinterpret_cast<O *>(s_stage);
    __syncthreads();  // every thread has finished reading its inputs
#pragma unroll
    for (int e = 0; e < SITEMS; ++e) smO[spad<O>(tid * SITEMS + e)] = res[e];
    __syncthreads();
    constexpr int VO = (16 / sizeof(O)) < SITEMS ? (16 / sizeof(O)) : SITEMS;
#pragma unroll
    for (int q = 0; q < SITEMS / VO; ++q) {
      const int i0 = (q * SBLOCK + tid) * VO;
      Vec<O, VO> t;
#pragma unroll
      for (int e = 0; e < VO; ++e) t.v[e] = smO[spad<O>(i0 + e)];
      stvec_stream<O, VO>(y + start + i0, t);
    }
  } else {
#pragma unroll
    for (int e = 0; e < SITEMS; ++e) {
      long long i = my0 + e;
      if (i < count) y[start + i] = res[e];
    }
  }
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
      A v = (i < k) ? to_local<A, T>(x[r * k + i]) : Op::template id<A>();
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        A o = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v = Op::op(o, v);
      }
      if (i < k) y[r * k + i] = cvt<O>(Op::op(carry, (C)v));
      A last = __shfl_sync(0xffffffffu, v, 31);
      carry = Op::op(carry, (C)last);
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
