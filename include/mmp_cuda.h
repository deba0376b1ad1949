/*
 * mmp_cuda.h -- C ABI of libmmp_cuda.so, the B200 (sm_100a) backend of the
 * macmetalpy_b200 array hot path.
 *
 * The reference reaches its GPU through the un-vendored metalgpu bridge,
 * whose ctypes declarations are at src/macmetalpy/_metal_backend.py:221-263
 * (init, createBuffer, releaseBuffer, getBufferPointer,
 * createLibraryFromString, setFunction, runFunction, ...).  Each entry point
 * below names the reference interface it replaces.  Every function returns 0
 * on success or a negative MMP_E_* code; the message of the last failure on
 * the calling thread is available from mmp_last_error().  All work is
 * enqueued on one stream per device (stream-ordered, asynchronous unless the
 * function says it synchronises).  Pointers are plain device addresses;
 * sizes are bytes unless named otherwise.  No torch types cross this ABI.
 */
#ifndef MMP_CUDA_H
#define MMP_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MMP_ABI_VERSION 1

/* status codes */
#define MMP_OK 0
#define MMP_E_CUDA (-1)      /* a CUDA runtime / driver call failed          */
#define MMP_E_ARG (-2)       /* invalid argument (shape, dtype, pointer)     */
#define MMP_E_NVRTC (-3)     /* NVRTC compile failed; log in the log buffer  */
#define MMP_E_UNSUPPORTED (-4)
#define MMP_E_DEVICE (-5)    /* a kernel reported an error (bounded wait)    */
#define MMP_E_COMM (-6)      /* NCCL missing or failed, or a collective timed
                                out (the communicator is then aborted)      */

/* dtype codes (numpy kinds the reference supports, _dtypes.py:21-31, plus
 * int8/uint8 and float64 which B200 computes natively) */
enum mmp_dtype {
  MMP_BOOL = 0, MMP_INT8 = 1, MMP_UINT8 = 2, MMP_INT16 = 3, MMP_UINT16 = 4,
  MMP_INT32 = 5, MMP_UINT32 = 6, MMP_INT64 = 7, MMP_UINT64 = 8,
  MMP_FLOAT16 = 9, MMP_FLOAT32 = 10, MMP_FLOAT64 = 11
};

/* reduction ops: the reference's reduce_sum/max/min/prod (_kernels.py:422-565),
 * mean/var/std (ndarray.py:1779-1834), argmax/argmin (_kernels.py:1189-1257),
 * nan reductions (_kernels.py:612-730, nan_ops.py:112-432; nanvar/nanstd:
 * nan_ops.py:444-530, float inputs only) */
enum mmp_reduce_op {
  MMP_R_SUM = 0, MMP_R_PROD = 1, MMP_R_MAX = 2, MMP_R_MIN = 3,
  MMP_R_MEAN = 4, MMP_R_VAR = 5, MMP_R_STD = 6,
  MMP_R_ARGMAX = 7, MMP_R_ARGMIN = 8,
  MMP_R_NANSUM = 9, MMP_R_NANMEAN = 10, MMP_R_NANMAX = 11, MMP_R_NANMIN = 12,
  MMP_R_ANY = 13, MMP_R_ALL = 14, MMP_R_NANVAR = 15, MMP_R_NANSTD = 16
};

/* scan ops: prefix_sum / prefix_prod (_kernels.py:1148-1170, 1263-1358) */
enum mmp_scan_op { MMP_S_SUM = 0, MMP_S_PROD = 1 };

/* gemm modes (matmul_op, _kernels.py:735-759) */
enum mmp_gemm_mode {
  MMP_GEMM_AUTO = 0,    /* f32 -> 3xTF32 tensor cores, f16 -> f16 tensor cores */
  MMP_GEMM_3XTF32 = 1,  /* f32 split into big+small TF32 parts, 3 MMAs/tile   */
  MMP_GEMM_TF32 = 2,    /* f32 rounded to TF32, 1 MMA/tile (fast, ~1e-3)      */
  MMP_GEMM_F16 = 3,     /* f16 inputs, f32 accumulation in TMEM               */
  MMP_GEMM_SIMT = 4     /* CUDA-core fallback (any dtype, any stride)         */
};

/* Merged partial of a full reduction, written when `partial` is non-NULL so
 * that block-distributed arrays can combine shards across GPUs.  Field use
 * depends on the op (see mmp_reduce). */
typedef struct mmp_partial {
  double s1;       /* sum / shifted first moment / value (as double)          */
  double s2;       /* shifted second moment (var/std)                          */
  double shift;    /* shift K used for the moments (var/std)                   */
  int64_t count;   /* element count (nan ops: non-NaN count)                   */
  int64_t ival;    /* exact integer sum/prod, or the int value (max/min/arg)   */
  int64_t index;   /* argmax/argmin flat index, -1 if none                     */
} mmp_partial;

/* ---- library / device (replaces init/deleteInstance, _metal_backend.py:221-226) */
int mmp_abi_version(void);
const char *mmp_last_error(void);
int mmp_device_count(int *count);
/* Make `device` current on this thread, create its stream and configure its
 * stream-ordered memory pool (MetalBackend._setup, _metal_backend.py:197-219). */
int mmp_init(int device);
int mmp_get_device(int *device);
int mmp_sm_count(int *sms);
/* The stream all work of the current device is enqueued on. */
int mmp_get_stream(void **stream);
/* Replace the current device's stream (e.g. with a torch/NCCL stream). */
int mmp_set_stream(void *stream);

/* ---- memory (createBuffer/releaseBuffer/getBufferPointer, _metal_backend.py:227-240) */
int mmp_malloc(size_t bytes, void **ptr);     /* stream-ordered cudaMallocAsync  */
int mmp_free(void *ptr);                      /* stream-ordered cudaFreeAsync    */
int mmp_memset(void *ptr, int value, size_t bytes);
int mmp_h2d(void *dst, const void *src, size_t bytes);  /* async on the stream  */
int mmp_d2h(void *dst, const void *src, size_t bytes);  /* synchronises         */
int mmp_d2d(void *dst, const void *src, size_t bytes);
int mmp_host_alloc(size_t bytes, void **ptr);  /* pinned host memory           */
int mmp_host_free(void *ptr);
/* Per-device scratch region for multi-block kernels (partials + tickets).
 * Returned memory is reused by every call on the device (stream-ordered). */
int mmp_scratch(size_t bytes, void **ptr, void **tickets);

/* ---- synchronisation (synchronize, _metal_backend.py:359-372) */
int mmp_synchronize(void);
/* Synchronise, then read and clear the device-side error word that kernels
 * set instead of hanging or writing out of bounds: 0 = no error, 2 = scan
 * look-back wait ran out, 3 = GEMM pipeline wait ran out, 4 = sort scatter
 * offset out of range, 5 = gather / scatter / compaction offset out of
 * range, 6 = the self-test wait ran out (mmp_selftest_bounded_wait),
 * 8 = a peer's flag did not arrive in mmp_reduce_allranks,
 * mmp_scan_allranks or mmp_allreduce_sum_peer. */
int mmp_check_device_error(int *code);

/* ---- timing */
int mmp_event_create(void **event);
int mmp_event_destroy(void *event);
int mmp_event_record(void *event);
int mmp_event_elapsed_ms(void *start, void *end, float *ms);

/* ---- side streams and asynchronous copies (no counterpart in the
 * reference: MetalBackend has one implicit queue, _metal_backend.py:341-372).
 * They let a caller overlap host<->device copies with kernels and with
 * each other (the copy engines of the two directions run concurrently).
 * A NULL stream means the current device's library stream; order work
 * across streams with events.  Memory used by work on a side stream must
 * stay allocated until that work has finished.  Copies from / to pageable
 * host memory are staged by the driver; pinned memory (mmp_host_alloc)
 * runs at the full link rate. */
int mmp_stream_create(void **stream);          /* non-blocking stream */
int mmp_stream_destroy(void *stream);
int mmp_stream_synchronize(void *stream);
/* *busy = 1 while work enqueued on the stream has not finished, else 0 (the
 * reference's MetalBackend._has_pending, _metal_backend.py:341-372). */
int mmp_stream_query(void *stream, int *busy);
int mmp_stream_wait_event(void *stream, void *event);
int mmp_event_record_on(void *event, void *stream);
int mmp_h2d_async(void *dst, const void *src, size_t bytes, void *stream);
int mmp_d2h_async(void *dst, const void *src, size_t bytes, void *stream);

/* ---- runtime compilation (createLibraryFromString/setFunction/runFunction,
 *      _metal_backend.py:241-257): NVRTC for sm_100a, cached by source+options.
 * `options` is a '\n'-separated list.  `func` receives a launchable handle. */
int mmp_compile(const char *source, const char *name, const char *options,
                void **func, char *log, size_t log_size);
int mmp_launch(void *func, const unsigned grid[3], const unsigned block[3],
               unsigned shared_bytes, void **args);
/* mmp_launch of a kernel that takes this library's per-device scratch (as
 * mmp_scratch returns it) in two of its arguments: takes a region of at
 * least scratch_bytes, writes its address into the void * that
 * args[scr_slot] points to and the ticket array's into args[tick_slot]'s,
 * then launches -- one call where mmp_scratch + mmp_launch take two.  The
 * slots must index `args`. */
int mmp_launch_scratch(void *func, const unsigned grid[3], const unsigned block[3],
                       unsigned shared_bytes, void **args, size_t scratch_bytes,
                       int scr_slot, int tick_slot);
/* Blocks of `block_threads` threads that fit on one SM at once (grid sizing
 * for the compiled function; runFunction picks its own in the reference). */
int mmp_occupancy(void *func, int block_threads, unsigned shared_bytes, int *blocks_per_sm);

/* ---- typed hot-path kernels */

/* Full reduction of n contiguous elements (ndarray._reduce, ndarray.py:1895-1963;
 * reductions.argmax, reductions.py:381-418; nan_ops._nan_reduce, nan_ops.py:72-100).
 * Writes one element of out_dtype to `out` (argmax/argmin: int64 index).
 * ddof is used by VAR/STD only.  `partial` may be NULL. */
int mmp_reduce(int op, int dtype, const void *x, int64_t n, int out_dtype,
               void *out, double ddof, mmp_partial *partial);

/* Reduction over the middle axis of a C-contiguous (outer, k, inner) view
 * (ndarray._reduce_axis, ndarray.py:2015-2066); out is (outer, inner). */
int mmp_reduce_axis(int op, int dtype, const void *x, int64_t outer, int64_t k,
                    int64_t inner, int out_dtype, void *out, double ddof);

/* Inclusive scan along the middle axis of a C-contiguous (outer, k, inner)
 * view (ndarray._prefix_scan, ndarray.py:2068-2152); y has the same shape in
 * out_dtype, which must be numpy's accumulation type (int64 for signed ints
 * and bool, uint64 for unsigned, the input type for floats).  For a 1-D scan
 * (outer == 1, inner == 1) carry_in, when non-NULL, points to one value in
 * device memory of the carry type (float64 for float inputs, int64/uint64
 * for integers) that is combined into every output (distributed scans). */
int mmp_scan(int op, int dtype, const void *x, int out_dtype, void *y,
             int64_t outer, int64_t k, int64_t inner, const void *carry_in);

/* Allocation-free form of mmp_scan, for callers that cannot have this
 * library allocate device memory during a call -- a host framework that owns
 * nearly all of HBM through its own pool and passes only its input and output
 * buffers, or code holding that framework's allocator lock.  Same arguments
 * and results as mmp_scan.  No counterpart in the reference (it has no such
 * callers).  The look-back state lives in a fixed device array of this
 * library (16 bytes per tile: about 3.2 MiB per GPU that loads it, kept
 * until exit), so scans
 * longer than MMP_NOALLOC_SCAN_TILES tiles of 4096 elements per row-set
 * (outer * ceil(k / 4096)) are rejected with MMP_E_ARG.  Calls share the
 * array: calls that may overlap on the GPU race and must be serialised by
 * the caller.  Requires mmp_init on the device; the first call on a device
 * looks up the array's address (make it before any stream capture). */
#define MMP_NOALLOC_SCAN_TILES 209715
int mmp_scan_noalloc(int op, int dtype, const void *x, int out_dtype, void *y,
                     int64_t outer, int64_t k, int64_t inner, const void *carry_in);

/* Row-major C[b] = A[b] @ B[b] for b < batch (ndarray.__matmul__,
 * ndarray.py:1398-1450; linalg_top.matmul, linalg_top.py:94-111).
 * Leading dimensions and batch strides are in elements. */
int mmp_gemm(int dtype, int mode, int64_t batch, int64_t m, int64_t n,
             int64_t k, const void *a, int64_t lda, int64_t stride_a,
             const void *b, int64_t ldb, int64_t stride_b, void *c,
             int64_t ldc, int64_t stride_c);

/* Stable ascending sort of each row of a C-contiguous (rows, cols) array
 * (sorting.sort / argsort, sorting.py:22-54, whose GPU branch is the bitonic
 * network of :57-190).  Writes the sorted values to `y` and/or, when
 * `indices` is not NULL, each sorted element's column index (int64, numpy's
 * argsort).  numpy order: NaN last; with indices, -0.0 and +0.0 tie (and a
 * -0.0 comes back as +0.0 in `y`).  rows * cols < 2^32.  Synchronises the
 * stream once (to skip radix passes that would not move anything). */
int mmp_sort(int dtype, const void *x, void *y, int64_t *indices, int64_t rows,
             int64_t cols);

/* out[q] = insertion point of v[q] in the ascending array a[0..n)
 * (sorting.searchsorted, sorting.py:218-272).  side 0 = left, 1 = right;
 * `sorter` (NULL or n int64 indices, already validated) reads a[sorter[i]].
 * numpy's order: NaN sorts last.  a and v share `dtype`; out is int64. */
int mmp_searchsorted(int dtype, const void *a, int64_t n, const void *v,
                     int64_t m, int side, const int64_t *sorter, int64_t *out);

/* ---- advanced indexing (ndarray.__getitem__/__setitem__ advanced keys,
 * ndarray.py:874-957; indexing.take/put/nonzero/compress/extract,
 * indexing.py:24-410 -- numpy on the host in the reference).  Offsets are in
 * elements from `src` / `dst`; entries outside [0, limit) are skipped and
 * set device error 5.  Elements move as raw 1/2/4/8-byte words. */
int mmp_gather(int dtype, const void *src, int64_t limit, const int64_t *offsets,
               int64_t n, void *out);
int mmp_scatter(int dtype, void *dst, int64_t limit, const int64_t *offsets,
                int64_t n, const void *values);
/* out[k] = position of the k-th true entry of the bool mask[0..n), given
 * incl = the inclusive scan of the mask and count = incl[n-1] (numpy's
 * flatnonzero). */
int mmp_compact_indices(const void *mask, const int64_t *incl, int64_t n,
                        int64_t count, int64_t *out);

/* ---- block-distributed arrays: partials and their merge on the device.
 * The reference is single-device (MetalBackend, _metal_backend.py:186-204);
 * these split its full reductions (ndarray._reduce, ndarray.py:1895-1963;
 * reductions.var, reductions.py:525-584; reductions.argmax,
 * reductions.py:381-418) into a per-shard step and a merge step, with no
 * host round trip in between. */

/* Write the merged partial of a full reduction of x[0..n) to device memory
 * `dev_partial` (8-byte aligned; layout mmp_partial), on the stream, without
 * synchronising.  For argmax/argmin the index is offset by index_base (the
 * shard's first global flat index); an empty shard gives index -1. */
int mmp_reduce_partial(int op, int dtype, const void *x, int64_t n, int64_t index_base,
                       mmp_partial *dev_partial);

/* Fold nparts device partials (rank order) with the op's own arithmetic and
 * write the result as mmp_reduce would (one out_dtype element at `out`, a
 * device pointer); `dev_merged` (device, may be NULL) receives the merged
 * partial.  nparts == 0 gives the op's identity, e.g. the zero carry of
 * rank 0 in a distributed scan (op MMP_R_SUM, out_dtype int64/float64). */
int mmp_merge_partials(int op, int dtype, const mmp_partial *dev_parts, int nparts, int out_dtype,
                       void *out, double ddof, mmp_partial *dev_merged);

/* ---- collectives over NCCL (one process per GPU; no counterpart in the
 * reference, which is single-device -- these extend its ctypes ABI table,
 * _metal_backend.py:221-263, with the exchange steps of block-distributed
 * arrays).  NCCL is opened at run time (dlopen of libnccl.so.2, or the
 * path in MMP_NCCL_LIB).  One communicator per device; every collective is
 * enqueued on the current device's library stream, so kernels and
 * collectives are ordered without host synchronisation.  Buffers are device
 * pointers; count is in elements of dtype (bool is sent as 1-byte words).
 * A call that does not complete within the communicator's timeout aborts
 * it and returns MMP_E_COMM. */
#define MMP_COMM_ID_BYTES 256
enum mmp_comm_op { MMP_COMM_SUM = 0, MMP_COMM_PROD = 1, MMP_COMM_MAX = 2, MMP_COMM_MIN = 3 };
int mmp_nccl_version(int *version);
/* Rank 0 creates the id (MMP_COMM_ID_BYTES: two NCCL ids, one for a
 * bounded bootstrap, one for the data-plane communicator) and hands the
 * bytes to every rank out of band. */
int mmp_comm_unique_id(void *id);
/* Join the communicator of nranks ranks as `rank`, on the current device
 * (after mmp_init).  Blocks until every rank joined or timeout_s passed. */
int mmp_comm_init(int nranks, int rank, const void *id, double timeout_s);
int mmp_comm_rank(int *rank, int *nranks);
int mmp_comm_destroy(void);   /* synchronises the stream first */
int mmp_comm_abort(void);     /* no synchronisation: for error paths */
int mmp_allreduce(const void *send, void *recv, size_t count, int dtype, int op);
/* recv holds nranks * count elements, rank r's at offset r * count. */
int mmp_allgather(const void *send, void *recv, size_t count, int dtype);
/* send is read on `root` only; every rank receives into recv (in place
 * when send == recv on the root). */
int mmp_broadcast(const void *send, void *recv, size_t count, int dtype, int root);
int mmp_group_start(void);
int mmp_group_end(void);
/* ---- fused reduce + exchange over peer memory (no NCCL kernel on the
 * path).  mmp_comm_peer_init (collective, after mmp_comm_init) makes an
 * exchange block of MMP_XBLOCK_BYTES on every rank and maps every other
 * rank's block into this process over CUDA IPC; MMP_E_UNSUPPORTED on every
 * rank when any rank cannot map its peers (keep the NCCL path then).
 * mmp_reduce_allranks (collective: every rank calls it with the same op and
 * dtype, in the same order) reduces this rank's x[0..n) and, in the same
 * launch, stores the partial into every rank's block over NVLink, raises
 * its flag there, waits for every rank's flag (bounded: 2 s of device time,
 * then device error 8 and the missing ranks count as empty) and merges the
 * partials in rank order, exactly as mmp_merge_partials does, into `out`
 * (one out_dtype element, device memory) on every rank.  index_base is the
 * shard's first global flat index (argmax / argmin). */
#define MMP_XCOL_BYTES (1 << 20)
#define MMP_XBLOCK_BYTES (16384 + 2 * MMP_XCOL_BYTES)
int mmp_comm_peer_init(void);
int mmp_reduce_allranks(int op, int dtype, const void *x, int64_t n, int64_t index_base, int out_dtype,
                        void *out, double ddof);
/* Inclusive scan (op MMP_S_SUM / MMP_S_PROD) of a 1-D array block-
 * distributed over the ranks in rank order: this rank's shard x[0..n) into
 * y[0..n), with the combined totals of the lower ranks' shards as the carry
 * (the global cumsum / cumprod, reductions.py:661-705, of the concatenated
 * shards).  Collective over the peer exchange like mmp_reduce_allranks, and
 * with its bounded wait.  A long aligned shard (n >= 2^24, x and y 16-byte
 * aligned, n a multiple of 16) exchanges its total from the scan's own tile
 * aggregates between its launches, so the shard's data is read twice and
 * written once as in mmp_scan; any other shard reduces and exchanges first.
 * Shards may be empty (n = 0: x and y unused, the call still takes part). */
int mmp_scan_allranks(int op, int dtype, const void *x, int out_dtype, void *y, int64_t n);
/* Sum of `count` elements of `dtype` (int64, uint64 or float64: column
 * partials in their accumulation type) over every rank, in rank order, into
 * `recv` (count elements of out_dtype, every rank) -- one launch: the
 * send buffer goes into this rank's exchange area (MMP_XCOL_BYTES per call
 * parity), flags as mmp_reduce_allranks, then every rank reads every
 * rank's area over NVLink.  Collective, bounded wait (device error 8).
 * MMP_E_UNSUPPORTED when count * 8 > MMP_XCOL_BYTES or there is no peer
 * exchange (use mmp_allreduce). */
int mmp_allreduce_sum_peer(const void *send, void *recv, size_t count, int dtype, int out_dtype);

/* Wait for this device's stream, giving up after timeout_s seconds (<= 0:
 * the communicator's timeout): then the communicator is aborted and
 * MMP_E_COMM returned, so a lost rank ends in an error, not a hang. */
int mmp_comm_synchronize(double timeout_s);

/* Self-test of the failure behaviour of waiting kernels (no counterpart in
 * the reference): one kernel waits on a device flag that nothing sets, gives
 * up after timeout_us of device time, sets device error 6 and returns; the
 * next mmp_check_device_error reports 6 and the context stays usable.
 * `polls` (may be NULL) receives the number of polls made. */
int mmp_selftest_bounded_wait(int timeout_us, unsigned *polls);

#ifdef __cplusplus
}
#endif
#endif /* MMP_CUDA_H */
