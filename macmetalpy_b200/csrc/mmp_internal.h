// Internal helpers shared by the translation units of libmmp_cuda.so.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>
#include <string>

#include "../../include/mmp_cuda.h"

namespace mmp {

// Record `msg` as this thread's last error and return `code`.
int set_error(int code, const std::string &msg);
int cuda_error(cudaError_t e, const char *what);

// Stream of the current device (created by mmp_init on first use).
cudaStream_t stream();
int current_device();
int sm_count();
// Per-device scratch: at least `bytes` of reusable device memory plus an
// array of 4096 zero-initialised 32-bit tickets.  Kernels that take a
// ticket leave it at zero when they finish.
int scratch(size_t bytes, void **ptr, unsigned **tickets);
// Device-side error word (bounded waits set it instead of hanging).
int *device_error_word();
// True once mmp_init has set up the current device (no side effects).
bool is_ready();
// The current device's peer exchange blocks (blk[0..nranks), this rank's
// included) and a fresh exchange epoch; false when mmp_comm_peer_init has
// not set them up.
bool peer_table(void **blk, int *rank, int *nranks, unsigned long long *epoch);
// Collective: the carry of a distributed scan (the lower ranks' combined
// shard totals, carry type: float64 / int64 / uint64) into device memory,
// from the shard's tile aggregates when `agg` is given, else from a full
// reduction of x[0..n) (mmp_merge.cu).
int scan_carry_allranks(int prod, int dtype, const void *agg, long long ntiles, const void *x, long long n,
                        void *carry_out);

}  // namespace mmp

#define MMP_CUDA_TRY(call)                                   \
  do {                                                       \
    cudaError_t _e = (call);                                 \
    if (_e != cudaSuccess) return mmp::cuda_error(_e, #call); \
  } while (0)

#define MMP_LAUNCH_CHECK(what)                                  \
  do {                                                          \
    cudaError_t _e = cudaGetLastError();                        \
    if (_e != cudaSuccess) return mmp::cuda_error(_e, what);    \
  } while (0)

// Size in bytes of an mmp_dtype code (0 for an unknown code).
static inline size_t mmp_dtype_size(int dt) {
  switch (dt) {
    case MMP_BOOL: case MMP_INT8: case MMP_UINT8: return 1;
    case MMP_INT16: case MMP_UINT16: case MMP_FLOAT16: return 2;
    case MMP_INT32: case MMP_UINT32: case MMP_FLOAT32: return 4;
    case MMP_INT64: case MMP_UINT64: case MMP_FLOAT64: return 8;
    default: return 0;
  }
}
