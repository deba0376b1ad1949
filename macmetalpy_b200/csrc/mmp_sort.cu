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
//   rs_hist     per-tile digit histogram (16-byte loads, per-warp counters),
//               digit-major counts[d][tile]
//   mmp_scan    inclusive scan of the counts -> (digit, tile) offsets
//   rs_trivial  flags a pass whose digit is the same for every key; the host
//               reads the flag (4 bytes) and skips that pass's scatter
//   rs_scatter  stable placement: a tile is cut into one contiguous segment
//               per warp, each warp walks its keys in memory order, ranking
//               each key among equal digits (one ballot per digit bit) and
//               per-warp digit counters; the tile is first placed in digit
//               order in shared memory, then written out by consecutive
//               threads to consecutive addresses of each digit's range.
// rs_prep maps the keys (and writes row / column ids) in one pass.
// Temporary buffers come from the stream-ordered pool.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

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

// Map keys and write row / column ids.
template <class T, bool HI, bool HR>
__global__ void __launch_bounds__(RS_THREADS) rs_prep(const T *__restrict__ x, typename RKey<T>::K *__restrict__ kout,
                                                      unsigned *__restrict__ iout, unsigned *__restrict__ rout,
                                                      unsigned long long n, FastDiv cols, int tie_zero) {
  const unsigned long long stride = (unsigned long long)gridDim.x * blockDim.x;
  for (unsigned long long i = (unsigned long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    kout[i] = RKey<T>::key(x[i], tie_zero != 0);
    if (HI || HR) {
      const unsigned r = cols.div((unsigned)i);
      if (HI) iout[i] = (unsigned)i - r * cols.d;
      if (HR) rout[i] = r;
    }
  }
}

template <class K, bool FR>
__device__ __forceinline__ unsigned digit_of(K k, unsigned r, int shift) {
  return FR ? ((r >> shift) & 255u) : ((unsigned)(k >> shift) & 255u);
}

// Digit histogram of one tile; counts are digit-major: counts[d * tiles + t].
// Full tiles are read with 16-byte loads (tiles start 16-byte aligned); the
// last, partial tile element by element.
template <class K, bool FR>
__global__ void __launch_bounds__(RS_THREADS) rs_hist(const K *__restrict__ kin, const unsigned *__restrict__ rin,
                                                      unsigned long long n, int shift, unsigned *__restrict__ counts,
                                                      unsigned tiles) {
  __shared__ unsigned h[RS_WARPS][256];
  const int tid = threadIdx.x, w = tid >> 5;
  for (int j = tid; j < RS_WARPS * 256; j += RS_THREADS) (&h[0][0])[j] = 0;
  __syncthreads();
  const unsigned long long t0 = (unsigned long long)blockIdx.x * RS_TILE;
  if (t0 + RS_TILE <= n) {
    if (FR) {
      const uint4 *v = reinterpret_cast<const uint4 *>(rin + t0);
#pragma unroll
      for (int q = 0; q < RS_TILE / 4 / RS_THREADS; ++q) {
        const uint4 c = v[q * RS_THREADS + tid];
        atomicAdd(&h[w][(c.x >> shift) & 255u], 1u);
        atomicAdd(&h[w][(c.y >> shift) & 255u], 1u);
        atomicAdd(&h[w][(c.z >> shift) & 255u], 1u);
        atomicAdd(&h[w][(c.w >> shift) & 255u], 1u);
      }
    } else {
      constexpr int PER = 16 / (int)sizeof(K);
      const uint4 *v = reinterpret_cast<const uint4 *>(kin + t0);
#pragma unroll
      for (int q = 0; q < RS_TILE / PER / RS_THREADS; ++q) {
        uint4 c = v[q * RS_THREADS + tid];
        const K *e = reinterpret_cast<const K *>(&c);
#pragma unroll
        for (int u = 0; u < PER; ++u) atomicAdd(&h[w][(unsigned)(e[u] >> shift) & 255u], 1u);
      }
    }
  } else {
    for (int e = 0; e < RS_ITEMS; ++e) {
      const unsigned long long i = t0 + (unsigned long long)e * RS_THREADS + tid;
      if (i < n) atomicAdd(&h[w][digit_of<K, FR>(FR ? K(0) : kin[i], FR ? rin[i] : 0u, shift)], 1u);
    }
  }
  __syncthreads();
  unsigned c = 0;
#pragma unroll
  for (int v = 0; v < RS_WARPS; ++v) c += h[v][tid];
  counts[(unsigned long long)tid * tiles + blockIdx.x] = c;
}

// Flags (sets *trivial) a pass whose digit is the same for every key: the
// total of some digit equals n.  incl is the inclusive scan of counts.
__global__ void rs_trivial(const unsigned long long *__restrict__ incl, unsigned tiles, unsigned long long n,
                           unsigned *trivial) {
  const unsigned d = threadIdx.x;
  const unsigned long long end = incl[(unsigned long long)(d + 1) * tiles - 1];
  const unsigned long long beg = d ? incl[(unsigned long long)d * tiles - 1] : 0ull;
  if (end - beg == n) *trivial = 1u;
}

// Stable scatter of one tile (see the file comment).  incl is the inclusive
// scan of counts.  Dynamic shared memory: the tile's keys, then its column
// ids (HI), then its row ids (HR), in digit order.
template <class K, bool HI, bool HR>
constexpr int ScatterSmem() {
  return RS_TILE * ((int)sizeof(K) + (HI ? 4 : 0) + (HR ? 4 : 0));
}

// Resident blocks per SM asked of the register allocator: each key slot of
// the 16 per thread costs sizeof(K) / 4 registers plus one per payload.
template <class K, bool HI, bool HR>
constexpr int ScatterMinBlocks() {
  return ((int)sizeof(K) + (HI ? 4 : 0) + (HR ? 4 : 0)) <= 4 ? 4 : 3;
}

template <class K, bool HI, bool HR, bool FR>
__global__ void __launch_bounds__(RS_THREADS, (ScatterMinBlocks<K, HI, HR>())) rs_scatter(
    const K *__restrict__ kin, K *__restrict__ kout, const unsigned *__restrict__ iin, unsigned *__restrict__ iout,
    const unsigned *__restrict__ rin, unsigned *__restrict__ rout, unsigned long long n, int shift,
    const unsigned *__restrict__ counts, const unsigned long long *__restrict__ incl, unsigned tiles, int *err) {
  __shared__ unsigned s_cnt[RS_WARPS][256];
  __shared__ unsigned long long s_off[256];  // global offset of (digit, this tile)
  __shared__ unsigned s_bex[256];            // offset of each digit inside the tile
  __shared__ unsigned s_wsum[RS_WARPS];
  extern __shared__ __align__(16) unsigned char s_stage[];
  K *sk = reinterpret_cast<K *>(s_stage);
  unsigned *si = reinterpret_cast<unsigned *>(s_stage + RS_TILE * sizeof(K));
  unsigned *sr = si + (HI ? RS_TILE : 0);
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const unsigned long long t0 = (unsigned long long)blockIdx.x * RS_TILE;
  const unsigned long long seg = t0 + (unsigned long long)w * RS_SEG;
  K k[RS_ITEMS];
  unsigned iv[RS_ITEMS], rv[RS_ITEMS], rank[RS_ITEMS];
#pragma unroll
  for (int e = 0; e < RS_ITEMS; ++e) {  // the tile's loads go out first
    const unsigned long long i = seg + e * 32 + lane;
    k[e] = 0;
    iv[e] = rv[e] = 0;
    if (i < n) {
      k[e] = kin[i];
      if (HI) iv[e] = iin[i];
      if (HR) rv[e] = rin[i];
    }
  }
  for (int j = tid; j < RS_WARPS * 256; j += RS_THREADS) (&s_cnt[0][0])[j] = 0;
  {
    const unsigned long long c = (unsigned long long)tid * tiles + blockIdx.x;
    s_off[tid] = incl[c] - counts[c];
  }
  __syncthreads();
  const unsigned lt = lanemask_lt();
#pragma unroll
  for (int e = 0; e < RS_ITEMS; ++e) {
    const bool valid = seg + e * 32 + lane < n;
    const unsigned d = valid ? digit_of<K, FR>(k[e], rv[e], shift) : 0u;
    // lanes holding the same digit: one ballot per digit bit (warp-level
    // multisplit; a fixed cost, unlike __match_any_sync, whose cost grows
    // with the number of distinct digits in the warp)
    unsigned peers = __ballot_sync(0xffffffffu, valid);
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const bool bit = (d >> b) & 1u;
      const unsigned bal = __ballot_sync(0xffffffffu, bit);
      peers &= bit ? bal : ~bal;
    }
    const unsigned before = (unsigned)__popc(peers & lt);
    const unsigned c = valid ? s_cnt[w][d] : 0u;
    __syncwarp();
    if (valid && before == 0) s_cnt[w][d] = c + (unsigned)__popc(peers);
    __syncwarp();
    rank[e] = c + before;
  }
  __syncthreads();
  {  // thread = digit: warp-exclusive counters, then the digit's offset in the tile
    unsigned tot = 0;
#pragma unroll
    for (int v = 0; v < RS_WARPS; ++v) {
      const unsigned c = s_cnt[v][tid];
      s_cnt[v][tid] = tot;
      tot += c;
    }
    unsigned inc = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const unsigned t = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += t;
    }
    if (lane == 31) s_wsum[w] = inc;
    __syncthreads();
    unsigned pre = 0;
    for (int v = 0; v < w; ++v) pre += s_wsum[v];
    s_bex[tid] = pre + inc - tot;
  }
  __syncthreads();
#pragma unroll
  for (int e = 0; e < RS_ITEMS; ++e) {
    if (seg + e * 32 + lane < n) {
      const unsigned d = digit_of<K, FR>(k[e], rv[e], shift);
      const unsigned lp = s_bex[d] + s_cnt[w][d] + rank[e];
      if (lp >= (unsigned)RS_TILE) {  // inconsistent ranks: report, never write out of bounds
        atomicExch(err, 4);
        continue;
      }
      sk[lp] = k[e];
      if (HI) si[lp] = iv[e];
      if (HR) sr[lp] = rv[e];
    }
  }
  __syncthreads();
  const unsigned count = (unsigned)((n - t0) < (unsigned long long)RS_TILE ? (n - t0) : (unsigned long long)RS_TILE);
  for (unsigned j = tid; j < count; j += RS_THREADS) {
    const K key = sk[j];
    const unsigned r = HR ? sr[j] : 0u;
    const unsigned d = digit_of<K, FR>(key, r, shift);
    const unsigned long long dst = s_off[d] + (j - s_bex[d]);
    if (dst >= n) {  // inconsistent offsets: report, never write out of bounds
      atomicExch(err, 4);
      continue;
    }
    kout[dst] = key;
    if (HI) iout[dst] = si[j];
    if (HR) rout[dst] = r;
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

template <class K, bool HI, bool HR, bool FR>
int launch_scatter(const K *kin, K *kout, const unsigned *iin, unsigned *iout, const unsigned *rin, unsigned *rout,
                   unsigned long long n, int shift, const unsigned *cnt, const unsigned long long *inc,
                   unsigned tiles) {
  constexpr int SM = ScatterSmem<K, HI, HR>();
  static bool attr[64];  // per device: function attributes are set per device
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return set_error(MMP_E_ARG, "device out of range");
  if (!attr[dev]) {
    MMP_CUDA_TRY(cudaFuncSetAttribute(rs_scatter<K, HI, HR, FR>, cudaFuncAttributeMaxDynamicSharedMemorySize, SM));
    attr[dev] = true;
  }
  rs_scatter<K, HI, HR, FR><<<tiles, RS_THREADS, SM, stream()>>>(kin, kout, iin, iout, rin, rout, n, shift, cnt,
                                                                inc, tiles, device_error_word());
  MMP_LAUNCH_CHECK("rs_scatter");
  return MMP_OK;
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
  PoolBuf kb[2], ib[2], rb[2], cnt, inc, flag;
  for (int b = 0; b < 2; ++b) {
    int rc = kb[b].alloc(n * sizeof(K));
    if (!rc && HI) rc = ib[b].alloc(n * 4);
    if (!rc && HR) rc = rb[b].alloc(n * 4);
    if (rc) return rc;
  }
  const size_t nc = (size_t)tiles * 256;
  int rc = cnt.alloc(nc * 4);
  if (!rc) rc = inc.alloc(nc * 8);
  if (!rc) rc = flag.alloc(16);
  if (rc) return rc;
  rs_prep<T, HI, HR><<<grid_for(n, RS_THREADS), RS_THREADS, 0, st>>>(
      x, (K *)kb[0].p, (unsigned *)ib[0].p, (unsigned *)rb[0].p, n, make_fastdiv((unsigned)cols), HI ? 1 : 0);
  MMP_LAUNCH_CHECK("rs_prep");
  int cur = 0;
  for (int p = 0; p < KB + rbytes; ++p) {
    const bool fr = p >= KB;
    const int shift = 8 * (fr ? p - KB : p);
    const K *kin = (const K *)kb[cur].p;
    const unsigned *rin = (const unsigned *)rb[cur].p;
    if (fr) rs_hist<K, true><<<tiles, RS_THREADS, 0, st>>>(kin, rin, n, shift, (unsigned *)cnt.p, tiles);
    else rs_hist<K, false><<<tiles, RS_THREADS, 0, st>>>(kin, rin, n, shift, (unsigned *)cnt.p, tiles);
    MMP_LAUNCH_CHECK("rs_hist");
    rc = mmp_scan(MMP_S_SUM, MMP_UINT32, cnt.p, MMP_UINT64, inc.p, 1, (int64_t)nc, 1, nullptr);
    if (rc) return rc;
    // a pass whose digit is the same for every key keeps the order: skip it
    MMP_CUDA_TRY(cudaMemsetAsync(flag.p, 0, 4, st));
    rs_trivial<<<1, 256, 0, st>>>((const unsigned long long *)inc.p, tiles, n, (unsigned *)flag.p);
    MMP_LAUNCH_CHECK("rs_trivial");
    unsigned trivial = 0;
    MMP_CUDA_TRY(cudaMemcpyAsync(&trivial, flag.p, 4, cudaMemcpyDeviceToHost, st));
    MMP_CUDA_TRY(cudaStreamSynchronize(st));
    if (trivial) continue;
    K *kout = (K *)kb[cur ^ 1].p;
    const unsigned *iin = (const unsigned *)ib[cur].p;
    unsigned *iout = (unsigned *)ib[cur ^ 1].p, *rout = (unsigned *)rb[cur ^ 1].p;
    const unsigned *cp = (const unsigned *)cnt.p;
    const unsigned long long *ip = (const unsigned long long *)inc.p;
    rc = fr ? launch_scatter<K, HI, HR, true>(kin, kout, iin, iout, rin, rout, n, shift, cp, ip, tiles)
            : launch_scatter<K, HI, HR, false>(kin, kout, iin, iout, rin, rout, n, shift, cp, ip, tiles);
    if (rc) return rc;
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
