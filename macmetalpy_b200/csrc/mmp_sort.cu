// mmp_sort / mmp_searchsorted: stable LSD radix sort of the rows of a
// (rows, cols) array, and binary-search insertion points.
//
// Reference: sorting.sort / argsort (src/macmetalpy/sorting.py:22-54) take
// numpy's np.sort / np.argsort below 262,144 elements and a bitonic network
// (one launch per (k, j) step, padded to a power of two, :57-190) above it,
// for 1-D float32/int32/uint32/int16/uint16 only; searchsorted (:218-272)
// runs one plain binary search per query.  Results here follow numpy (the
// reference's CPU path) for every size and dtype: NaN sorts last, argsort is
// stable (numpy kind="stable"; -0.0 and +0.0 tie), indices are int64.
//
// Algorithm.  Each key is mapped to an unsigned integer of the same width
// whose order is the numpy order (sign bit flipped for signed integers;
// floats: every NaN -> all ones, negatives bit-inverted, positives with the
// sign bit set).  Rows are sorted together: an element's row id travels
// with it and is sorted last, so the final order is by row, then by key.
// One radix pass per byte (8-bit digits), least significant first:
//   rs_hist     per-tile digit histogram, digit-major counts[d][tile]
//   mmp_scan    inclusive scan of the counts -> (digit, tile) offsets
//   rs_scatter  stable placement: a tile is cut into one contiguous segment
//               per warp, each warp walks its keys in memory order, ranking
//               each key among equal digits with __match_any_sync and
//               per-warp digit counters in shared memory.
// rs_prep maps the keys and builds the histograms of every pass in one read;
// the host reads them (one small copy) and skips passes whose digit is the
// same for every key.  Temporary buffers come from the stream-ordered pool.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <vector>

#include "mmp_dispatch.h"
#include "mmp_device.cuh"

namespace mmpd {

constexpr int RS_THREADS = 256;
constexpr int RS_ITEMS = 16;
constexpr int RS_TILE = RS_THREADS * RS_ITEMS;
constexpr int RS_WARPS = RS_THREADS / 32;
constexpr int RS_SEG = 32 * RS_ITEMS;  // keys per warp segment

// ---- order-preserving unsigned keys
template <class T> struct RKey;
template <> struct RKey<bool> {
  typedef unsigned char K;
  __device__ static K key(bool v, bool) { return v ? 1 : 0; }
  __device__ static bool val(K k) { return k != 0; }
};
template <> struct RKey<short> {
  typedef unsigned short K;
  __device__ static K key(short v, bool) { return (K)((unsigned short)v ^ 0x8000u); }
  __device__ static short val(K k) { return (short)(unsigned short)(k ^ 0x8000u); }
};
template <> struct RKey<unsigned short> {
  typedef unsigned short K;
  __device__ static K key(unsigned short v, bool) { return v; }
  __device__ static unsigned short val(K k) { return k; }
};
template <> struct RKey<int> {
  typedef unsigned K;
  __device__ static K key(int v, bool) { return (unsigned)v ^ 0x80000000u; }
  __device__ static int val(K k) { return (int)(k ^ 0x80000000u); }
};
template <> struct RKey<unsigned> {
  typedef unsigned K;
  __device__ static K key(unsigned v, bool) { return v; }
  __device__ static unsigned val(K k) { return k; }
};
template <> struct RKey<long long> {
  typedef unsigned long long K;
  __device__ static K key(long long v, bool) { return (unsigned long long)v ^ 0x8000000000000000ull; }
  __device__ static long long val(K k) { return (long long)(k ^ 0x8000000000000000ull); }
};
template <> struct RKey<unsigned long long> {
  typedef unsigned long long K;
  __device__ static K key(unsigned long long v, bool) { return v; }
  __device__ static unsigned long long val(K k) { return k; }
};
// floats: NaN -> all ones (last); with `tie_zero`, -0.0 keys as +0.0 so the
// two tie (argsort); without it the bit pattern of every value is kept.
template <class U>
__device__ __forceinline__ U fkey(U b, bool nan, bool tie_zero) {
  constexpr U sign = (U)1 << (sizeof(U) * 8 - 1);
  if (nan) return (U)~(U)0;
  if (tie_zero && b == sign) b = 0;
  return (b & sign) ? (U)~b : (U)(b | sign);
}
template <class U>
__device__ __forceinline__ U funkey(U k) {
  constexpr U sign = (U)1 << (sizeof(U) * 8 - 1);
  return (k & sign) ? (U)(k ^ sign) : (U)~k;
}
template <> struct RKey<__half> {
  typedef unsigned short K;
  __device__ static K key(__half v, bool tz) {
    const unsigned short b = __half_as_ushort(v);
    return fkey<unsigned short>(b, (b & 0x7fffu) > 0x7c00u, tz);
  }
  __device__ static __half val(K k) { return __ushort_as_half(funkey<unsigned short>(k)); }
};
template <> struct RKey<float> {
  typedef unsigned K;
  __device__ static K key(float v, bool tz) {
    const unsigned b = __float_as_uint(v);
    return fkey<unsigned>(b, (b & 0x7fffffffu) > 0x7f800000u, tz);
  }
  __device__ static float val(K k) { return __uint_as_float(funkey<unsigned>(k)); }
};
template <> struct RKey<double> {
  typedef unsigned long long K;
  __device__ static K key(double v, bool tz) {
    const unsigned long long b = (unsigned long long)__double_as_longlong(v);
    return fkey<unsigned long long>(b, (b & 0x7fffffffffffffffull) > 0x7ff0000000000000ull, tz);
  }
  __device__ static double val(K k) { return __longlong_as_double((long long)funkey<unsigned long long>(k)); }
};

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// Map keys, write row / column ids, and histogram every pass's digit.
// ghist: [kbytes + rbytes][256].
template <class T, bool HI, bool HR>
__global__ void __launch_bounds__(RS_THREADS) rs_prep(const T *__restrict__ x, typename RKey<T>::K *__restrict__ kout,
                                                      unsigned *__restrict__ iout, unsigned *__restrict__ rout,
                                                      unsigned long long n, FastDiv cols, int rbytes, int tie_zero,
                                                      unsigned *__restrict__ ghist) {
  typedef typename RKey<T>::K K;
  constexpr int KB = (int)sizeof(K);
  extern __shared__ unsigned sh[];  // (KB + rbytes) * 256
  const int lane = threadIdx.x & 31;
  const int nh = (KB + rbytes) * 256;
  for (int j = threadIdx.x; j < nh; j += blockDim.x) sh[j] = 0;
  __syncthreads();
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  for (unsigned long long base = (unsigned long long)blockIdx.x * blockDim.x + (threadIdx.x & ~31u); base < n;
       base += stride) {
    const unsigned long long i = base + lane;
    const bool valid = i < n;
    const unsigned act = __ballot_sync(0xffffffffu, valid);
    if (!valid) continue;
    const K k = RKey<T>::key(x[i], tie_zero != 0);
    kout[i] = k;
    unsigned r = 0;
    if (HI || HR) {
      r = cols.div((unsigned)i);
      if (HI) iout[i] = (unsigned)i - r * cols.d;
      if (HR) rout[i] = r;
    }
#pragma unroll
    for (int b = 0; b < KB; ++b) {
      const unsigned d = (unsigned)(k >> (8 * b)) & 255u;
      const unsigned peers = __match_any_sync(act, d);
      if ((peers & lanemask_lt()) == 0) atomicAdd(&sh[b * 256 + d], (unsigned)__popc(peers));
    }
    for (int b = 0; b < rbytes; ++b) {
      const unsigned d = (r >> (8 * b)) & 255u;
      const unsigned peers = __match_any_sync(act, d);
      if ((peers & lanemask_lt()) == 0) atomicAdd(&sh[(KB + b) * 256 + d], (unsigned)__popc(peers));
    }
  }
  __syncthreads();
  for (int j = threadIdx.x; j < nh; j += blockDim.x)
    if (sh[j]) atomicAdd(&ghist[j], sh[j]);
}

template <class K, bool FR>
__device__ __forceinline__ unsigned digit_of(K k, unsigned r, int shift) {
  return FR ? ((r >> shift) & 255u) : ((unsigned)(k >> shift) & 255u);
}

// Digit histogram of one tile; counts are digit-major: counts[d * tiles + t].
template <class K, bool FR>
__global__ void __launch_bounds__(RS_THREADS) rs_hist(const K *__restrict__ kin, const unsigned *__restrict__ rin,
                                                      unsigned long long n, int shift, unsigned *__restrict__ counts,
                                                      unsigned tiles) {
  __shared__ unsigned h[256];
  h[threadIdx.x] = 0;
  __syncthreads();
  const unsigned long long t0 = (unsigned long long)blockIdx.x * RS_TILE;
#pragma unroll 4
  for (int e = 0; e < RS_ITEMS; ++e) {
    const unsigned long long i = t0 + (unsigned long long)e * RS_THREADS + threadIdx.x;
    if (i < n) atomicAdd(&h[digit_of<K, FR>(FR ? K(0) : kin[i], FR ? rin[i] : 0u, shift)], 1u);
  }
  __syncthreads();
  counts[(unsigned long long)threadIdx.x * tiles + blockIdx.x] = h[threadIdx.x];
}

// Stable scatter of one tile (see the file comment).  incl is the inclusive
// scan of counts.
template <class K, bool HI, bool HR, bool FR>
__global__ void __launch_bounds__(RS_THREADS) rs_scatter(
    const K *__restrict__ kin, K *__restrict__ kout, const unsigned *__restrict__ iin, unsigned *__restrict__ iout,
    const unsigned *__restrict__ rin, unsigned *__restrict__ rout, unsigned long long n, int shift,
    const unsigned *__restrict__ counts, const unsigned long long *__restrict__ incl, unsigned tiles, int *err) {
  __shared__ unsigned s_cnt[RS_WARPS][256];
  __shared__ unsigned long long s_off[256];
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  for (int j = tid; j < RS_WARPS * 256; j += RS_THREADS) (&s_cnt[0][0])[j] = 0;
  {
    const unsigned long long c = (unsigned long long)tid * tiles + blockIdx.x;
    s_off[tid] = incl[c] - counts[c];
  }
  __syncthreads();
  const unsigned long long seg = (unsigned long long)blockIdx.x * RS_TILE + (unsigned long long)w * RS_SEG;
  K k[RS_ITEMS];
  unsigned iv[RS_ITEMS], rv[RS_ITEMS], rank[RS_ITEMS];
#pragma unroll
  for (int e = 0; e < RS_ITEMS; ++e) {
    const unsigned long long i = seg + e * 32 + lane;
    k[e] = 0;
    iv[e] = rv[e] = 0;
    if (i < n) {
      k[e] = kin[i];
      if (HI) iv[e] = iin[i];
      if (HR) rv[e] = rin[i];
    }
  }
  const unsigned lt = lanemask_lt();
#pragma unroll
  for (int e = 0; e < RS_ITEMS; ++e) {
    const bool valid = seg + e * 32 + lane < n;
    const unsigned vm = __ballot_sync(0xffffffffu, valid);
    rank[e] = 0;
    if (valid) {
      const unsigned d = digit_of<K, FR>(k[e], rv[e], shift);
      const unsigned peers = __match_any_sync(vm, d);
      const unsigned before = (unsigned)__popc(peers & lt);
      const unsigned c = s_cnt[w][d];
      __syncwarp(vm);
      if (before == 0) s_cnt[w][d] = c + (unsigned)__popc(peers);
      __syncwarp(vm);
      rank[e] = c + before;
    }
  }
  __syncthreads();
  {  // exclusive prefix of the warp counters, per digit (thread = digit)
    unsigned run = 0;
#pragma unroll
    for (int v = 0; v < RS_WARPS; ++v) {
      const unsigned c = s_cnt[v][tid];
      s_cnt[v][tid] = run;
      run += c;
    }
  }
  __syncthreads();
#pragma unroll
  for (int e = 0; e < RS_ITEMS; ++e) {
    if (seg + e * 32 + lane < n) {
      const unsigned d = digit_of<K, FR>(k[e], rv[e], shift);
      const unsigned long long dst = s_off[d] + s_cnt[w][d] + rank[e];
      if (dst >= n) {  // inconsistent offsets: report, never write out of bounds
        atomicExch(err, 4);
        continue;
      }
      kout[dst] = k[e];
      if (HI) iout[dst] = iv[e];
      if (HR) rout[dst] = rv[e];
    }
  }
}

// Sorted values (inverse key map) and/or int64 indices.
template <class T>
__global__ void rs_finish(const typename RKey<T>::K *__restrict__ kin, const unsigned *__restrict__ iin,
                          T *__restrict__ y, long long *__restrict__ idx, unsigned long long n) {
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  for (unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    if (y) y[i] = RKey<T>::val(kin[i]);
    if (idx) idx[i] = (long long)iin[i];
  }
}

// ---- searchsorted: numpy's order (NaN last) for the comparisons
template <class T> __device__ __forceinline__ bool s_lt(T a, T b) { return a < b; }
__device__ __forceinline__ bool s_lt(float a, float b) { return a < b || (b != b && a == a); }
__device__ __forceinline__ bool s_lt(double a, double b) { return a < b || (b != b && a == a); }
__device__ __forceinline__ bool s_lt(__half a, __half b) { return s_lt(__half2float(a), __half2float(b)); }

template <class T>
__global__ void searchsorted_kernel(const T *__restrict__ a, long long n, const T *__restrict__ v, long long m,
                                    int right, const long long *__restrict__ sorter, long long *__restrict__ out) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x; q < m; q += stride) {
    const T val = v[q];
    long long lo = 0, hi = n;
    while (lo < hi) {
      const long long mid = lo + ((hi - lo) >> 1);
      const T am = sorter ? a[sorter[mid]] : a[mid];
      const bool go = right ? !s_lt(val, am) : s_lt(am, val);
      if (go) lo = mid + 1;
      else hi = mid;
    }
    out[q] = lo;
  }
}

}  // namespace mmpd

namespace mmp {
namespace {

using namespace mmpd;

FastDiv make_fastdiv(unsigned d) {
  unsigned l = 0;
  while (l < 32 && (1ull << l) < d) ++l;
  const unsigned long long m = ((1ull << 32) * ((1ull << l) - d)) / d + 1;
  FastDiv f;
  f.d = d;
  f.m = (unsigned)m;
  f.s = l;
  return f;
}

struct PoolBuf {
  void *p = nullptr;
  ~PoolBuf() {
    if (p) cudaFreeAsync(p, stream());
  }
  int alloc(size_t bytes) {
    MMP_CUDA_TRY(cudaMallocAsync(&p, bytes ? bytes : 16, stream()));
    return MMP_OK;
  }
};

int grid_for(unsigned long long n, int threads) {
  unsigned long long b = (n + threads - 1) / threads;
  const unsigned long long cap = (unsigned long long)sm_count() * 8;
  return (int)(b < cap ? (b ? b : 1) : cap);
}

template <class T, bool HI, bool HR>
int run_passes(const T *x, T *y, long long *idx, unsigned long long rows, unsigned long long cols) {
  typedef typename RKey<T>::K K;
  constexpr int KB = (int)sizeof(K);
  cudaStream_t st = stream();
  const unsigned long long n = rows * cols;
  int rbytes = 0;
  if (HR)
    for (unsigned long long r = rows - 1; r; r >>= 8) ++rbytes;
  const unsigned tiles = (unsigned)((n + RS_TILE - 1) / RS_TILE);
  PoolBuf kb[2], ib[2], rb[2], cnt, inc, gh;
  for (int b = 0; b < 2; ++b) {
    int rc = kb[b].alloc(n * sizeof(K));
    if (!rc && HI) rc = ib[b].alloc(n * 4);
    if (!rc && HR) rc = rb[b].alloc(n * 4);
    if (rc) return rc;
  }
  const size_t nc = (size_t)tiles * 256;
  int rc = cnt.alloc(nc * 4);
  if (!rc) rc = inc.alloc(nc * 8);
  if (!rc) rc = gh.alloc((size_t)(KB + rbytes) * 256 * 4);
  if (rc) return rc;
  MMP_CUDA_TRY(cudaMemsetAsync(gh.p, 0, (size_t)(KB + rbytes) * 256 * 4, st));
  const FastDiv fd = make_fastdiv((unsigned)cols);
  const int smem = (KB + rbytes) * 256 * 4;
  rs_prep<T, HI, HR><<<grid_for(n, RS_THREADS), RS_THREADS, smem, st>>>(
      x, (K *)kb[0].p, (unsigned *)ib[0].p, (unsigned *)rb[0].p, n, fd, rbytes, HI ? 1 : 0, (unsigned *)gh.p);
  MMP_LAUNCH_CHECK("rs_prep");
  std::vector<unsigned> hist((size_t)(KB + rbytes) * 256);
  MMP_CUDA_TRY(cudaMemcpyAsync(hist.data(), gh.p, hist.size() * 4, cudaMemcpyDeviceToHost, st));
  MMP_CUDA_TRY(cudaStreamSynchronize(st));
  int cur = 0;
  for (int p = 0; p < KB + rbytes; ++p) {
    bool trivial = false;
    for (int d = 0; d < 256; ++d)
      if (hist[(size_t)p * 256 + d] == n) trivial = true;
    if (trivial) continue;  // every key has the same digit: the pass keeps the order
    const bool fr = p >= KB;
    const int shift = 8 * (fr ? p - KB : p);
    const K *kin = (const K *)kb[cur].p;
    const unsigned *rin = (const unsigned *)rb[cur].p;
    if (fr) rs_hist<K, true><<<tiles, RS_THREADS, 0, st>>>(kin, rin, n, shift, (unsigned *)cnt.p, tiles);
    else rs_hist<K, false><<<tiles, RS_THREADS, 0, st>>>(kin, rin, n, shift, (unsigned *)cnt.p, tiles);
    MMP_LAUNCH_CHECK("rs_hist");
    rc = mmp_scan(MMP_S_SUM, MMP_UINT32, cnt.p, MMP_UINT64, inc.p, 1, (int64_t)nc, 1, nullptr);
    if (rc) return rc;
    K *kout = (K *)kb[cur ^ 1].p;
    const unsigned *iin = (const unsigned *)ib[cur].p;
    unsigned *iout = (unsigned *)ib[cur ^ 1].p, *rout = (unsigned *)rb[cur ^ 1].p;
    if (fr)
      rs_scatter<K, HI, HR, true><<<tiles, RS_THREADS, 0, st>>>(kin, kout, iin, iout, rin, rout, n, shift,
                                                                 (const unsigned *)cnt.p,
                                                                 (const unsigned long long *)inc.p, tiles,
                                                                 device_error_word());
    else
      rs_scatter<K, HI, HR, false><<<tiles, RS_THREADS, 0, st>>>(kin, kout, iin, iout, rin, rout, n, shift,
                                                                  (const unsigned *)cnt.p,
                                                                  (const unsigned long long *)inc.p, tiles,
                                                                  device_error_word());
    MMP_LAUNCH_CHECK("rs_scatter");
    cur ^= 1;
  }
  rs_finish<T><<<grid_for(n, 256), 256, 0, st>>>((const K *)kb[cur].p, (const unsigned *)ib[cur].p, y, idx, n);
  MMP_LAUNCH_CHECK("rs_finish");
  return MMP_OK;
}

}  // namespace

template <int UNUSED, class T>
struct SortRun {
  static int run(const void *x, void *y, void *idx, long long rows, long long cols) {
    const bool hi = idx != nullptr, hr = rows > 1;
    if (hi && hr) return run_passes<T, true, true>((const T *)x, (T *)y, (long long *)idx, rows, cols);
    if (hi) return run_passes<T, true, false>((const T *)x, (T *)y, (long long *)idx, rows, cols);
    if (hr) return run_passes<T, false, true>((const T *)x, (T *)y, (long long *)idx, rows, cols);
    return run_passes<T, false, false>((const T *)x, (T *)y, (long long *)idx, rows, cols);
  }
};

template <int UNUSED, class T>
struct SearchRun {
  static int run(const void *a, long long n, const void *v, long long m, int right, const long long *sorter,
                 long long *out) {
    searchsorted_kernel<T><<<grid_for((unsigned long long)m, 256), 256, 0, stream()>>>(
        (const T *)a, n, (const T *)v, m, right, sorter, out);
    MMP_LAUNCH_CHECK("searchsorted_kernel");
    return MMP_OK;
  }
};

}  // namespace mmp

extern "C" int mmp_sort(int dtype, const void *x, void *y, int64_t *indices, int64_t rows, int64_t cols) {
  if (rows < 0 || cols < 0) return mmp::set_error(MMP_E_ARG, "negative extent");
  if (rows == 0 || cols == 0) return MMP_OK;
  if (!x || (!y && !indices)) return mmp::set_error(MMP_E_ARG, "null pointer");
  if (cols > 0xffffffffll || rows > 0xffffffffll || rows * cols > 0xffffffffll)
    return mmp::set_error(MMP_E_ARG, "sort: more than 2^32 - 1 elements");
  if (dtype == MMP_INT8 || dtype == MMP_UINT8) return mmp::set_error(MMP_E_ARG, "sort: int8/uint8 are stored as 16-bit");
  return mmp::dispatch_dtype<mmp::SortRun, 0>(dtype, x, y, (void *)indices, (long long)rows, (long long)cols);
}

extern "C" int mmp_searchsorted(int dtype, const void *a, int64_t n, const void *v, int64_t m, int side,
                                const int64_t *sorter, int64_t *out) {
  if (n < 0 || m < 0) return mmp::set_error(MMP_E_ARG, "negative extent");
  if (m == 0) return MMP_OK;
  if (!v || !out || (n > 0 && !a)) return mmp::set_error(MMP_E_ARG, "null pointer");
  if (side != 0 && side != 1) return mmp::set_error(MMP_E_ARG, "side must be 0 (left) or 1 (right)");
  return mmp::dispatch_dtype<mmp::SearchRun, 0>(dtype, a, (long long)n, v, (long long)m, side,
                                                (const long long *)sorter, (long long *)out);
}
