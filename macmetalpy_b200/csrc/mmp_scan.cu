// mmp_scan: inclusive cumsum / cumprod along the middle axis of
// (outer, k, inner).  See mmp_scan.cuh for the algorithm.
#include <cuda_runtime.h>

#include "mmp_dispatch.h"
#include "mmp_scan.cuh"

#include <cstdio>

using namespace mmpd;

namespace mmp {
namespace {

// Look-back state of the current device: tile aggregates, inclusive
// prefixes, flags and the tile counter.  Zeroed when (re)allocated; flags
// carry a launch epoch so they never need clearing between launches.
struct ScanState {
  void *buf = nullptr;
  size_t tiles = 0;
  unsigned epoch = 0;
};
ScanState g_scan[64];

int scan_state(long long tiles, void **desc, unsigned **counter, unsigned *epoch) {
  int dev = current_device();
  if (dev < 0 || dev >= 64) return set_error(MMP_E_ARG, "device out of range");
  ScanState &s = g_scan[dev];
  cudaStream_t st = stream();
  if ((size_t)tiles > s.tiles) {
    size_t want = (size_t)tiles < 4096 ? 4096 : (size_t)tiles;
    if (s.buf) MMP_CUDA_TRY(cudaFreeAsync(s.buf, st));
    s.buf = nullptr;
    s.tiles = 0;
    size_t bytes = want * 16 + 256;
    MMP_CUDA_TRY(cudaMallocAsync(&s.buf, bytes, st));
    MMP_CUDA_TRY(cudaMemsetAsync(s.buf, 0, bytes, st));
    s.tiles = want;
    s.epoch = 0;
  }
  s.epoch = (s.epoch + 1) & 0x3fffffffu;
  if (s.epoch == 0) {  // wrapped: clear stale flags once
    MMP_CUDA_TRY(cudaMemsetAsync(s.buf, 0, s.tiles * 16 + 256, st));
    s.epoch = 1;
  }
  char *b = (char *)s.buf;
  *desc = b;
  *counter = (unsigned *)(b + s.tiles * 16);
  *epoch = s.epoch;
  return MMP_OK;
}

template <class T> struct ScanOut { typedef long long type; static constexpr int code = MMP_INT64; };
template <> struct ScanOut<unsigned short> { typedef unsigned long long type; static constexpr int code = MMP_UINT64; };
template <> struct ScanOut<unsigned int> { typedef unsigned long long type; static constexpr int code = MMP_UINT64; };
template <> struct ScanOut<unsigned long long> { typedef unsigned long long type; static constexpr int code = MMP_UINT64; };
template <> struct ScanOut<__half> { typedef __half type; static constexpr int code = MMP_FLOAT16; };
template <> struct ScanOut<float> { typedef float type; static constexpr int code = MMP_FLOAT32; };
template <> struct ScanOut<double> { typedef double type; static constexpr int code = MMP_FLOAT64; };

// The tile kernel stages a tile through dynamic shared memory (more than
// the 48 KB default for 8-byte outputs); raise the limit once per kernel
// and device (function attributes are set per device).
template <class T, class O, bool PROD>
int set_stage_smem() {
  static bool done[64];
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return set_error(MMP_E_ARG, "device out of range");
  if (!done[dev]) {
    MMP_CUDA_TRY(cudaFuncSetAttribute(scan_tiles_kernel<T, O, PROD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      StageSize<T, O>()));
    MMP_CUDA_TRY(cudaFuncSetAttribute(scan_tiles_carry_kernel<T, O, PROD>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, StageSize<T, O>()));
    done[dev] = true;
  }
  return MMP_OK;
}

// Resident blocks per SM of a persistent streaming scan kernel (its shared
// memory raised past the 48 KB default once per device), for its grid.
template <class K>
int persistent_blocks_per_sm(K kernel, int smem, int *per_sm, const char *name, int *out) {
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return set_error(MMP_E_ARG, "device out of range");
  if (!per_sm[dev]) {
    MMP_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    int n = 0;
    MMP_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, SBLOCK, smem));
    if (n < 1) return set_error(MMP_E_CUDA, name);
    per_sm[dev] = n;
  }
  *out = per_sm[dev];
  return MMP_OK;
}
template <class T, class O, bool PROD>
int stream_blocks_per_sm(int *out) {
  static int per_sm[64];
  return persistent_blocks_per_sm(scan_carry_stream_kernel<T, O, PROD>, StreamSmem<T, O>(), per_sm,
                                  "scan_carry_stream_kernel does not fit on an SM", out);
}

}  // namespace

// Rows of at least kLongRowTiles tiles, in scans of at least
// kLongRowElements elements, take the reduce-then-scan path
// (tile_aggregates_kernel, a scan of the aggregates, scan_tiles_carry_kernel)
// instead of the look-back kernel, whose chain of waits grows with the row.
// Measured on B200: int32 -> int64 over 2^30 elements 4.6 TB/s against
// 3.5 TB/s; float32 (f64 sums) 3.84; rows of 16 tiles (4096 x 65536
// float32) 3.71 against 3.35 on the look-back kernel.  Scans below ~2^24
// elements (three launches, a pool allocation) stay on the look-back
// kernel.
constexpr long long kLongRowTiles = 16;
constexpr long long kLongRowElements = 1ll << 24;

template <int PRODI, class T>
struct ScanRun {
  typedef typename ScanOut<T>::type O;
  typedef typename ScanTypes<T>::carry_t CT;

  // exch_dtype >= 0 (one row, the shard of a distributed scan of that
  // input dtype): the carry is the lower ranks' combined totals, exchanged
  // over peer memory from this shard's tile aggregates between the first
  // launch and the aggregate scan (cin is ignored).
  static int long_rows(const T *x, O *y, long long rows, long long k, long long tpr, long long total,
                       const CT *cin, int vec_ok, int exch_dtype = -1) {
    constexpr bool PROD = PRODI != 0;
    cudaStream_t st = stream();
    CT *agg = nullptr;
    MMP_CUDA_TRY(cudaMallocAsync((void **)&agg, ((size_t)total * 2 + 1) * sizeof(CT), st));
    CT *incl = agg + total;
    long long blocks = (total * 32 + SBLOCK - 1) / SBLOCK;
    const long long maxb = (long long)sm_count() * 8;
    tile_aggregates_kernel<T, PROD><<<(unsigned)(blocks < maxb ? blocks : maxb), SBLOCK, 0, st>>>(
        x, k, tpr, total, agg, vec_ok);
    cudaError_t e = cudaGetLastError();
    int rc = e == cudaSuccess ? MMP_OK : cuda_error(e, "tile_aggregates_kernel");
    if (exch_dtype >= 0) {
      CT *carry = agg + 2 * total;
      if (!rc) rc = scan_carry_allranks(PRODI, exch_dtype, agg, total, nullptr, 0, carry);
      cin = carry;
    }
    // the aggregates are scanned per row by this same library (CT is its
    // own accumulation type), with the caller's carry
    if (!rc) rc = ScanRun<PRODI, CT>::run(agg, ScanOut<CT>::code, incl, rows, tpr, 1, cin);
    if (!rc && vec_ok) {
      // aligned: the persistent streaming carry scan, as many blocks as fit
      int per_sm = 0;
      rc = stream_blocks_per_sm<T, O, PROD>(&per_sm);
      if (!rc) {
        long long g = (long long)sm_count() * per_sm;
        if (g > total) g = total;
        scan_carry_stream_kernel<T, O, PROD><<<(unsigned)g, SBLOCK, StreamSmem<T, O>(), st>>>(
            x, y, rows, k, tpr, total, incl, cin);
        e = cudaGetLastError();
        if (e != cudaSuccess) rc = cuda_error(e, "scan_carry_stream_kernel");
      }
    } else {
      if (!rc) rc = set_stage_smem<T, O, PROD>();
      if (!rc) {
        scan_tiles_carry_kernel<T, O, PROD><<<(unsigned)total, SBLOCK, StageSize<T, O>(), st>>>(
            x, y, rows, k, tpr, total, incl, cin, vec_ok);
        e = cudaGetLastError();
        if (e != cudaSuccess) rc = cuda_error(e, "scan_tiles_carry_kernel");
      }
    }
    cudaFreeAsync(agg, st);
    return rc;
  }

  // A 1-D shard of a distributed scan (collective over the peer exchange).
  static int allranks(int dtype, const void *xv, int out_dt, void *yv, long long n) {
    if (out_dt != ScanOut<T>::code)
      return set_error(MMP_E_ARG, "scan output dtype must be the numpy accumulation type");
    cudaStream_t st = stream();
    if (!st) return set_error(MMP_E_CUDA, "no stream");
    const long long tpr = (n + STILE - 1) / STILE;
    if (tpr > 0x7fffffffll) return set_error(MMP_E_ARG, "scan too large");
    const int vec_ok = ((uintptr_t)xv % 16 == 0) && ((uintptr_t)yv % 16 == 0) && (n % 16 == 0);
    if (vec_ok && tpr >= kLongRowTiles && n >= kLongRowElements)
      return long_rows((const T *)xv, (O *)yv, 1, n, tpr, tpr, nullptr, vec_ok, dtype);
    // otherwise: the carry by a full reduce + exchange, then the local scan
    CT *carry = nullptr;
    MMP_CUDA_TRY(cudaMallocAsync((void **)&carry, sizeof(CT), st));
    int rc = scan_carry_allranks(PRODI, dtype, nullptr, 0, xv, n, carry);
    if (!rc && n > 0) rc = run(xv, out_dt, yv, 1, n, 1, carry);
    cudaFreeAsync(carry, st);
    return rc;
  }

  static int run(const void *xv, int out_dt, void *yv, long long outer, long long k, long long inner,
                 const void *carry) {
    constexpr bool PROD = PRODI != 0;
    if (out_dt != ScanOut<T>::code)
      return set_error(MMP_E_ARG, "scan output dtype must be the numpy accumulation type");
    cudaStream_t st = stream();
    if (!st) return set_error(MMP_E_CUDA, "no stream");
    const T *x = (const T *)xv;
    O *y = (O *)yv;
    const CT *cin = (const CT *)carry;
    const int sms = sm_count();
    if (inner > 1) {
      long long total = outer * inner;
      long long blocks = (total + SBLOCK - 1) / SBLOCK;
      long long maxb = (long long)sms * 8;
      scan_cols_kernel<T, O, PROD><<<(unsigned)(blocks < maxb ? blocks : maxb), SBLOCK, 0, st>>>(x, y, outer,
                                                                                              k, inner);
      MMP_LAUNCH_CHECK("scan_cols_kernel");
      return MMP_OK;
    }
    const long long rows = outer;
    if (k < STILE / 4) {
      long long blocks = (rows + 7) / 8;
      long long maxb = (long long)sms * 8;
      scan_rows_warp_kernel<T, O, PROD><<<(unsigned)(blocks < maxb ? blocks : maxb), SBLOCK, 0, st>>>(
          x, y, rows, k, cin);
      MMP_LAUNCH_CHECK("scan_rows_warp_kernel");
      return MMP_OK;
    }
    long long tpr = (k + STILE - 1) / STILE;
    if (rows > 0x7fffffffll / tpr) return set_error(MMP_E_ARG, "scan too large");  // before rows * tpr can wrap
    long long total = rows * tpr;
    int vec_ok = ((uintptr_t)x % 16 == 0) && ((uintptr_t)y % 16 == 0) && (k % 16 == 0);
    if (tpr >= kLongRowTiles && rows * k >= kLongRowElements) return long_rows(x, y, rows, k, tpr, total, cin, vec_ok);
    void *desc;
    unsigned *counter, epoch;
    int rc = scan_state(total, &desc, &counter, &epoch);
    if (rc) return rc;
    typedef typename ScanTypes<T>::carry_t C;
    TileState<C> ts;
    ts.desc = (TileDesc<C> *)desc;
    rc = set_stage_smem<T, O, PROD>();
    if (rc) return rc;
    scan_tiles_kernel<T, O, PROD><<<(unsigned)total, SBLOCK, StageSize<T, O>(), st>>>(
        x, y, rows, k, tpr, total, ts, counter, epoch, device_error_word(), cin, vec_ok);
    MMP_LAUNCH_CHECK("scan_tiles_kernel");
    return MMP_OK;
  }
};

}  // namespace mmp

extern "C" int mmp_scan(int op, int dtype, const void *x, int out_dtype, void *y, int64_t outer, int64_t k,
                        int64_t inner, const void *carry_in) {
  if (outer < 0 || k < 0 || inner < 0) return mmp::set_error(MMP_E_ARG, "negative extent");
  if (outer == 0 || k == 0 || inner == 0) return MMP_OK;
  if (!x || !y) return mmp::set_error(MMP_E_ARG, "null pointer");
  if (op == MMP_S_SUM) return mmp::dispatch_dtype<mmp::ScanRun, 0>(dtype, x, out_dtype, y, (long long)outer,
                                                                  (long long)k, (long long)inner, carry_in);
  if (op == MMP_S_PROD) return mmp::dispatch_dtype<mmp::ScanRun, 1>(dtype, x, out_dtype, y, (long long)outer,
                                                                   (long long)k, (long long)inner, carry_in);
  return mmp::set_error(MMP_E_ARG, "unsupported scan op");
}

namespace mmp {

template <int PRODI, class T>
struct ScanAllRun {
  static int run(int dtype, const void *x, int out_dt, void *y, long long n) {
    return ScanRun<PRODI, T>::allranks(dtype, x, out_dt, y, n);
  }
};

}  // namespace mmp

extern "C" int mmp_scan_allranks(int op, int dtype, const void *x, int out_dtype, void *y, int64_t n) {
  if (n < 0) return mmp::set_error(MMP_E_ARG, "negative element count");
  if (n > 0 && (!x || !y)) return mmp::set_error(MMP_E_ARG, "null pointer");
  if (!mmp::is_ready()) return mmp::set_error(MMP_E_ARG, "call mmp_init first");
  if (op == MMP_S_SUM) return mmp::dispatch_dtype<mmp::ScanAllRun, 0>(dtype, dtype, x, out_dtype, y, (long long)n);
  if (op == MMP_S_PROD) return mmp::dispatch_dtype<mmp::ScanAllRun, 1>(dtype, dtype, x, out_dtype, y, (long long)n);
  return mmp::set_error(MMP_E_ARG, "unsupported scan op");
}

// ---------------------------------------------------------------------------
// Allocation-free scan.
//
// Some callers cannot let this library allocate device memory during a
// call: a host framework that owns the GPU's memory (it reserves almost all
// of HBM for its own pool and hands us only its input and output buffers,
// so a hidden cudaMalloc could fail or fragment its pool), or code that
// runs while that framework holds its allocator lock, where re-entering an
// allocator would deadlock.  mmp_scan_noalloc gives them the same scan as
// mmp_scan with its look-back state in a fixed device array that is part of
// this library, so the call itself allocates nothing.
//
// The array holds the state of at most MMP_NOALLOC_SCAN_TILES tiles of
// 4096 elements; larger scans are rejected with MMP_E_ARG.  Every GPU that
// loads the library keeps the array (about 3.2 MiB) until the process exits.
// All calls share it: calls that can overlap on the GPU (different streams
// or devices sharing nothing else) race on it and must be serialised by the
// caller.  The first call on each device looks up the array's address with
// cudaGetSymbolAddress; make that first call before any stream capture.
// The caller must have called mmp_init on the device.
// ---------------------------------------------------------------------------
// Look-back state of mmp_scan_noalloc: one 16-byte descriptor per tile
// (TileDesc: an 8-byte value and an 8-byte flag), then the 4-byte tile
// counter in the 256-byte tail.
static __device__ __align__(256) unsigned char g_noalloc_scan[(size_t)MMP_NOALLOC_SCAN_TILES * 16 + 256];

namespace mmp {
namespace {

constexpr size_t kNoallocTiles = MMP_NOALLOC_SCAN_TILES;

unsigned char *g_noalloc_addr[64];  // device address of g_noalloc_scan, per device

int noalloc_state(unsigned char **base) {
  int dev = current_device();
  if (dev < 0 || dev >= 64) return set_error(MMP_E_ARG, "device out of range");
  if (!g_noalloc_addr[dev]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scan);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(g_noalloc_scan)");
    g_noalloc_addr[dev] = (unsigned char *)p;
  }
  *base = g_noalloc_addr[dev];
  return MMP_OK;
}

template <int PRODI, class T>
struct ScanNoallocRun {
  static int run(const void *xv, int out_dt, void *yv, long long outer, long long k, long long inner,
                 const void *carry) {
    typedef typename ScanOut<T>::type O;
    typedef typename ScanTypes<T>::carry_t C;
    constexpr bool PROD = PRODI != 0;
    if (out_dt != ScanOut<T>::code)
      return set_error(MMP_E_ARG, "scan output dtype must be the numpy accumulation type");
    if (inner > 1 || k < STILE / 4)  // these shapes need no scratch at all
      return ScanRun<PRODI, T>::run(xv, out_dt, yv, outer, k, inner, carry);
    static_assert(sizeof(TileDesc<C>) == 16, "the counter sits after kNoallocTiles 16-byte descriptors");
    const long long tpr = (k + STILE - 1) / STILE;
    // compare before multiplying: outer * tpr could wrap for absurd extents
    if (outer > (long long)kNoallocTiles / tpr) {
      char msg[200];
      snprintf(msg, sizeof msg,
               "mmp_scan_noalloc: %lld rows of %lld tiles of %d elements exceed the fixed scratch of %zu "
               "tiles; use mmp_scan",
               outer, tpr, STILE, kNoallocTiles);
      return set_error(MMP_E_ARG, msg);
    }
    const long long total = outer * tpr;
    unsigned char *base = nullptr;
    int rc = noalloc_state(&base);
    if (rc) return rc;
    cudaStream_t st = stream();
    TileDesc<C> *desc = (TileDesc<C> *)base;
    unsigned *counter = (unsigned *)(base + kNoallocTiles * 16);
    // the previous call's descriptors and counter must not be read as this call's
    MMP_CUDA_TRY(cudaMemsetAsync(desc, 0, (size_t)total * sizeof(TileDesc<C>), st));
    MMP_CUDA_TRY(cudaMemsetAsync(counter, 0, sizeof(unsigned), st));
    TileState<C> ts;
    ts.desc = desc;
    const T *x = (const T *)xv;
    O *y = (O *)yv;
    int vec_ok = ((uintptr_t)x % 16 == 0) && ((uintptr_t)y % 16 == 0) && (k % 16 == 0);
    rc = set_stage_smem<T, O, PROD>();
    if (rc) return rc;
    scan_tiles_kernel<T, O, PROD><<<(unsigned)total, SBLOCK, StageSize<T, O>(), st>>>(
        x, y, outer, k, tpr, total, ts, counter, 1u, device_error_word(), (const C *)carry, vec_ok);
    MMP_LAUNCH_CHECK("scan_tiles_kernel (noalloc)");
    return MMP_OK;
  }
};

}  // namespace
}  // namespace mmp

extern "C" int mmp_scan_noalloc(int op, int dtype, const void *x, int out_dtype, void *y, int64_t outer,
                                int64_t k, int64_t inner, const void *carry_in) {
  if (outer < 0 || k < 0 || inner < 0) return mmp::set_error(MMP_E_ARG, "negative extent");
  if (outer == 0 || k == 0 || inner == 0) return MMP_OK;
  if (!x || !y) return mmp::set_error(MMP_E_ARG, "null pointer");
  if (!mmp::is_ready()) return mmp::set_error(MMP_E_ARG, "mmp_scan_noalloc: call mmp_init on this device first");
  if (op == MMP_S_SUM)
    return mmp::dispatch_dtype<mmp::ScanNoallocRun, 0>(dtype, x, out_dtype, y, (long long)outer, (long long)k,
                                                      (long long)inner, carry_in);
  if (op == MMP_S_PROD)
    return mmp::dispatch_dtype<mmp::ScanNoallocRun, 1>(dtype, x, out_dtype, y, (long long)outer, (long long)k,
                                                      (long long)inner, carry_in);
  return mmp::set_error(MMP_E_ARG, "unsupported scan op");
}
