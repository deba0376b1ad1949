// mmp_comm: the collective exchange steps of block-distributed arrays, as
// C-ABI entry points over NCCL (one process per GPU, one communicator per
// device, every collective enqueued on the device's library stream).
//
// The reference is single-device (MetalBackend, src/macmetalpy/
// _metal_backend.py:186-204); these exports extend its ctypes ABI table
// (_metal_backend.py:221-263) with the exchange steps that the block
// distribution needs: all-gather of per-shard partials, all-reduce of
// per-column partials and the broadcast of a replicated matmul operand.
//
// NCCL is opened with dlopen on the first mmp_comm_* call ("libnccl.so.2",
// or the path in MMP_NCCL_LIB), so the library still loads -- and its CPU
// tests run -- on a host without NCCL or a GPU.  In a process that already
// loaded NCCL (e.g. through torch), dlopen returns that copy.  nccl.h is
// used for its types only.
//
// Joining is bounded: a non-blocking bootstrap communicator is polled on the
// host with a deadline (the timeout passed to mmp_comm_init) and aborted if
// it is not ready in time (MMP_E_COMM), so a rank that never joins ends in an
// error instead of a hang.  The data plane then uses a blocking communicator
// split from it; mmp_comm_synchronize bounds the wait for its collectives and
// aborts both communicators when a peer is gone.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include <mutex>
#include <string>

#include "mmp_internal.h"

namespace {

struct NcclApi {
  bool loaded = false;
  void *handle = nullptr;
  ncclResult_t (*GetVersion)(int *) = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
  ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Broadcast)(const void *, void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char *(*GetErrorString)(ncclResult_t) = nullptr;
};

NcclApi g_api;
std::mutex g_api_mu;

// `comm` carries the data plane and is blocking: a collective call returns
// once its kernel is enqueued.  (In NCCL's non-blocking mode every call is
// handed to a new host thread and returns ncclInProgress, which cost
// ~150 us per collective here.)  `boot` is a non-blocking communicator made
// first from the first of the two ids: creating it can be polled with a
// deadline, so a rank that never joins ends init with an error; the
// blocking one is then created (second id) among ranks that are all
// present, and `boot` is released.
struct CommState {
  ncclComm_t comm = nullptr;
  ncclComm_t boot = nullptr;
  int rank = -1;
  int nranks = 0;
  double timeout_s = 120.0;
  // peer exchange (mmp_comm_peer_init): this rank's exchange block and every
  // rank's, mapped into this process (own one included)
  void *xblk = nullptr;
  void *peer[64] = {};
  bool peer_ok = false;
  unsigned long long epoch = 0;
};
constexpr int kMaxDev = 64;
CommState g_comm[kMaxDev];
std::mutex g_comm_mu;

void drop_peers(CommState *c) {
  if (!c->peer_ok) return;
  for (int r = 0; r < c->nranks && r < 64; ++r)
    if (r != c->rank && c->peer[r]) cudaIpcCloseMemHandle(c->peer[r]);
  if (c->xblk) cudaFree(c->xblk);
  for (int r = 0; r < 64; ++r) c->peer[r] = nullptr;
  c->xblk = nullptr;
  c->peer_ok = false;
}

void drop(CommState *c, bool abort) {
  drop_peers(c);
  if (c->comm) (abort ? g_api.CommAbort : g_api.CommDestroy)(c->comm);
  if (c->boot) g_api.CommAbort(c->boot);
  c->comm = nullptr;
  c->boot = nullptr;
  c->rank = -1;
  c->nranks = 0;
}

double now_s() {
  timespec ts;
  clock_gettime(CLOCK_MONOTONIC, &ts);
  return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

template <class F>
bool sym(void *h, const char *name, F &out) {
  out = reinterpret_cast<F>(dlsym(h, name));
  return out != nullptr;
}

int load_api() {
  std::lock_guard<std::mutex> lk(g_api_mu);
  if (g_api.loaded) return MMP_OK;
  const char *env = getenv("MMP_NCCL_LIB");
  const char *cands[] = {env, "libnccl.so.2", "libnccl.so"};
  void *h = nullptr;
  std::string tried;
  for (const char *c : cands) {
    if (!c || !*c) continue;
    h = dlopen(c, RTLD_NOW | RTLD_GLOBAL);
    if (h) break;
    tried += std::string(" ") + c;
  }
  if (!h) return mmp::set_error(MMP_E_COMM, "NCCL not found (tried" + tried + "); set MMP_NCCL_LIB");
  bool ok = sym(h, "ncclGetVersion", g_api.GetVersion) && sym(h, "ncclGetUniqueId", g_api.GetUniqueId) &&
            sym(h, "ncclCommInitRankConfig", g_api.CommInitRankConfig) &&
            sym(h, "ncclCommDestroy", g_api.CommDestroy) && sym(h, "ncclCommAbort", g_api.CommAbort) &&
            sym(h, "ncclCommGetAsyncError", g_api.CommGetAsyncError) &&
            sym(h, "ncclAllReduce", g_api.AllReduce) && sym(h, "ncclAllGather", g_api.AllGather) &&
            sym(h, "ncclBroadcast", g_api.Broadcast) && sym(h, "ncclGroupStart", g_api.GroupStart) &&
            sym(h, "ncclGroupEnd", g_api.GroupEnd) && sym(h, "ncclGetErrorString", g_api.GetErrorString);
  if (!ok) {
    dlclose(h);
    return mmp::set_error(MMP_E_COMM, "the NCCL library lacks a required symbol (NCCL >= 2.14 needed)");
  }
  g_api.handle = h;
  g_api.loaded = true;
  return MMP_OK;
}

int nccl_error(ncclResult_t r, const char *what) {
  std::string m = std::string(what) + ": " + (g_api.GetErrorString ? g_api.GetErrorString(r) : "NCCL error");
  return mmp::set_error(MMP_E_COMM, m);
}

CommState *cur_comm(int *rc) {
  int dev = mmp::current_device();
  if (dev < 0 || dev >= kMaxDev) {
    *rc = mmp::set_error(MMP_E_ARG, "device out of range");
    return nullptr;
  }
  CommState *c = &g_comm[dev];
  if (!c->comm) {
    *rc = mmp::set_error(MMP_E_COMM, "no communicator on this device: call mmp_comm_init first");
    return nullptr;
  }
  *rc = MMP_OK;
  return c;
}

// Poll a non-blocking communicator until NCCL reports it ready, an error, or
// the deadline passes (then abort everything: pending NCCL kernels stop).
int wait_comm(CommState *c, ncclComm_t comm, ncclResult_t r, const char *what) {
  if (r == ncclSuccess) return MMP_OK;
  if (r != ncclInProgress) return nccl_error(r, what);
  const double t0 = now_s();
  for (int it = 0;; ++it) {
    ncclResult_t st = ncclSuccess;
    ncclResult_t q = g_api.CommGetAsyncError(comm, &st);
    if (q != ncclSuccess) return nccl_error(q, what);
    if (st == ncclSuccess) return MMP_OK;
    if (st != ncclInProgress) {
      drop(c, true);
      return nccl_error(st, what);
    }
    if (now_s() - t0 > c->timeout_s) {
      drop(c, true);
      return mmp::set_error(MMP_E_COMM, std::string(what) + ": timed out; communicator aborted");
    }
    if (it > 1000) usleep(100);
  }
}

// A blocking call's status (the data-plane communicator is blocking).
int check_call(ncclResult_t r, const char *what) {
  if (r == ncclSuccess) return MMP_OK;
  return nccl_error(r, what);
}

bool nccl_type(int dt, ncclDataType_t *t) {
  switch (dt) {
    case MMP_BOOL: case MMP_INT8: *t = ncclInt8; return true;
    case MMP_UINT8: *t = ncclUint8; return true;
    case MMP_INT32: *t = ncclInt32; return true;
    case MMP_UINT32: *t = ncclUint32; return true;
    case MMP_INT64: *t = ncclInt64; return true;
    case MMP_UINT64: *t = ncclUint64; return true;
    case MMP_FLOAT16: *t = ncclFloat16; return true;
    case MMP_FLOAT32: *t = ncclFloat32; return true;
    case MMP_FLOAT64: *t = ncclFloat64; return true;
    default: return false;
  }
}

bool nccl_op(int op, ncclRedOp_t *o) {
  switch (op) {
    case MMP_COMM_SUM: *o = ncclSum; return true;
    case MMP_COMM_PROD: *o = ncclProd; return true;
    case MMP_COMM_MAX: *o = ncclMax; return true;
    case MMP_COMM_MIN: *o = ncclMin; return true;
    default: return false;
  }
}

}  // namespace

extern "C" int mmp_comm_unique_id(void *id) {
  if (!id) return mmp::set_error(MMP_E_ARG, "null id buffer");
  int rc = load_api();
  if (rc) return rc;
  static_assert(2 * sizeof(ncclUniqueId) == MMP_COMM_ID_BYTES, "ncclUniqueId size");
  for (int k = 0; k < 2; ++k) {  // bootstrap id, data-plane id
    ncclUniqueId u;
    ncclResult_t r = g_api.GetUniqueId(&u);
    if (r != ncclSuccess) return nccl_error(r, "ncclGetUniqueId");
    memcpy((char *)id + k * sizeof u, &u, sizeof u);
  }
  return MMP_OK;
}

extern "C" int mmp_comm_init(int nranks, int rank, const void *id, double timeout_s) {
  if (nranks < 1 || rank < 0 || rank >= nranks) return mmp::set_error(MMP_E_ARG, "bad rank / nranks");
  if (!id) return mmp::set_error(MMP_E_ARG, "null unique id");
  if (!mmp::is_ready()) return mmp::set_error(MMP_E_ARG, "call mmp_init on this device first");
  int rc = load_api();
  if (rc) return rc;
  int dev = mmp::current_device();
  if (dev < 0 || dev >= kMaxDev) return mmp::set_error(MMP_E_ARG, "device out of range");
  std::lock_guard<std::mutex> lk(g_comm_mu);
  CommState *c = &g_comm[dev];
  if (c->comm) return mmp::set_error(MMP_E_ARG, "a communicator already exists on this device");
  ncclUniqueId u;
  memcpy(&u, id, sizeof u);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  c->timeout_s = timeout_s > 0 ? timeout_s : 120.0;
  c->rank = rank;
  c->nranks = nranks;
  ncclComm_t boot = nullptr;
  ncclResult_t r = g_api.CommInitRankConfig(&boot, nranks, u, rank, &cfg);
  if (r != ncclSuccess && r != ncclInProgress) {
    c->rank = -1;
    c->nranks = 0;
    return nccl_error(r, "ncclCommInitRankConfig");
  }
  c->boot = boot;
  rc = wait_comm(c, boot, r, "ncclCommInitRankConfig");
  if (rc) return rc;
  // every rank is present: create the blocking data-plane communicator
  ncclUniqueId u2;
  memcpy(&u2, (const char *)id + sizeof(ncclUniqueId), sizeof u2);
  ncclConfig_t cfg2 = NCCL_CONFIG_INITIALIZER;
  cfg2.blocking = 1;
  ncclComm_t data = nullptr;
  r = g_api.CommInitRankConfig(&data, nranks, u2, rank, &cfg2);
  if (r != ncclSuccess || !data) {
    drop(c, true);
    return nccl_error(r, "ncclCommInitRankConfig (data plane)");
  }
  g_api.CommAbort(boot);  // no work was ever enqueued on it
  c->boot = nullptr;
  c->comm = data;
  return MMP_OK;
}

extern "C" int mmp_comm_rank(int *rank, int *nranks) {
  int rc;
  CommState *c = cur_comm(&rc);
  if (!c) return rc;
  if (rank) *rank = c->rank;
  if (nranks) *nranks = c->nranks;
  return MMP_OK;
}

extern "C" int mmp_comm_destroy(void) {
  int dev = mmp::current_device();
  if (dev < 0 || dev >= kMaxDev) return mmp::set_error(MMP_E_ARG, "device out of range");
  std::lock_guard<std::mutex> lk(g_comm_mu);
  CommState *c = &g_comm[dev];
  if (!c->comm) return MMP_OK;
  // the stream's collectives must be done before the communicator goes
  cudaStream_t st = mmp::stream();
  if (st) MMP_CUDA_TRY(cudaStreamSynchronize(st));
  // every peer's stores into this rank's exchange block happened before this
  // rank's last exchange saw their flags, so the block can go once the stream
  // is done
  drop_peers(c);
  ncclResult_t r = g_api.CommDestroy(c->comm);
  c->comm = nullptr;
  drop(c, true);  // the boot communicator has no work in flight
  if (r != ncclSuccess) return nccl_error(r, "ncclCommDestroy");
  return MMP_OK;
}

extern "C" int mmp_comm_abort(void) {
  int dev = mmp::current_device();
  if (dev < 0 || dev >= kMaxDev) return mmp::set_error(MMP_E_ARG, "device out of range");
  std::lock_guard<std::mutex> lk(g_comm_mu);
  CommState *c = &g_comm[dev];
  if (!c->comm) return MMP_OK;
  drop(c, true);
  return MMP_OK;
}

extern "C" int mmp_allreduce(const void *send, void *recv, size_t count, int dtype, int op) {
  int rc;
  CommState *c = cur_comm(&rc);
  if (!c) return rc;
  ncclDataType_t t;
  ncclRedOp_t o;
  if (!nccl_type(dtype, &t)) return mmp::set_error(MMP_E_ARG, "dtype not supported by the collective");
  if (!nccl_op(op, &o)) return mmp::set_error(MMP_E_ARG, "bad collective op");
  if (count && (!send || !recv)) return mmp::set_error(MMP_E_ARG, "null pointer");
  return check_call(g_api.AllReduce(send, recv, count, t, o, c->comm, mmp::stream()), "ncclAllReduce");
}

extern "C" int mmp_allgather(const void *send, void *recv, size_t count, int dtype) {
  int rc;
  CommState *c = cur_comm(&rc);
  if (!c) return rc;
  ncclDataType_t t;
  if (!nccl_type(dtype, &t)) return mmp::set_error(MMP_E_ARG, "dtype not supported by the collective");
  if (count && (!send || !recv)) return mmp::set_error(MMP_E_ARG, "null pointer");
  return check_call(g_api.AllGather(send, recv, count, t, c->comm, mmp::stream()), "ncclAllGather");
}

extern "C" int mmp_broadcast(const void *send, void *recv, size_t count, int dtype, int root) {
  int rc;
  CommState *c = cur_comm(&rc);
  if (!c) return rc;
  ncclDataType_t t;
  if (!nccl_type(dtype, &t)) return mmp::set_error(MMP_E_ARG, "dtype not supported by the collective");
  if (root < 0 || root >= c->nranks) return mmp::set_error(MMP_E_ARG, "bad root rank");
  if (count && !recv) return mmp::set_error(MMP_E_ARG, "null pointer");
  return check_call(g_api.Broadcast(send, recv, count, t, root, c->comm, mmp::stream()), "ncclBroadcast");
}

extern "C" int mmp_group_start(void) {
  int rc = load_api();
  if (rc) return rc;
  ncclResult_t r = g_api.GroupStart();
  if (r != ncclSuccess) return nccl_error(r, "ncclGroupStart");
  return MMP_OK;
}

extern "C" int mmp_group_end(void) {
  int rc = load_api();
  if (rc) return rc;
  ncclResult_t r = g_api.GroupEnd();
  if (r != ncclSuccess) return nccl_error(r, "ncclGroupEnd");
  return MMP_OK;
}

// Wait until every collective and kernel enqueued on this device's stream
// has finished, but give up after timeout_s seconds: then abort the
// communicator (NCCL stops its kernels that wait on a dead peer) and
// return MMP_E_COMM.  A synchronise that cannot hang on a lost rank.
extern "C" int mmp_comm_synchronize(double timeout_s) {
  int rc;
  CommState *c = cur_comm(&rc);
  if (!c) return rc;
  cudaStream_t st = mmp::stream();
  const double t0 = now_s();
  const double limit = timeout_s > 0 ? timeout_s : c->timeout_s;
  for (;;) {
    cudaError_t e = cudaStreamQuery(st);
    if (e == cudaSuccess) return MMP_OK;
    if (e != cudaErrorNotReady) return mmp::cuda_error(e, "cudaStreamQuery");
    ncclResult_t as = ncclSuccess;
    g_api.CommGetAsyncError(c->comm, &as);
    if (as != ncclSuccess && as != ncclInProgress) {
      drop(c, true);
      return nccl_error(as, "communicator failed; aborted");
    }
    if (now_s() - t0 > limit) {
      drop(c, true);
      return mmp::set_error(MMP_E_COMM, "collectives did not finish in time (a rank is gone?); communicator aborted");
    }
    usleep(50);
  }
}

extern "C" int mmp_nccl_version(int *version) {
  if (!version) return mmp::set_error(MMP_E_ARG, "null pointer");
  int rc = load_api();
  if (rc) return rc;
  ncclResult_t r = g_api.GetVersion(version);
  if (r != ncclSuccess) return nccl_error(r, "ncclGetVersion");
  return MMP_OK;
}

// ---------------------------------------------------------------------------
// Peer exchange blocks: the partials of a distributed reduction cross NVLink
// as plain stores from the reducing kernel into every rank's block (see
// mmp_reduce_allranks), instead of an NCCL collective and a merge launch.
// Each rank cudaMallocs MMP_XBLOCK_BYTES, the IPC handles are all-gathered
// over the communicator, and every rank maps the others' blocks.  Collective:
// if any rank cannot map a peer, every rank gets MMP_E_UNSUPPORTED and the
// exchange stays off (callers keep the NCCL path).
extern "C" int mmp_comm_peer_init(void) {
  int rc;
  CommState *c = cur_comm(&rc);
  if (!c) return rc;
  if (c->peer_ok) return MMP_OK;
  if (c->nranks > 64) return mmp::set_error(MMP_E_UNSUPPORTED, "peer exchange supports at most 64 ranks");
  cudaStream_t st = mmp::stream();
  void *blk = nullptr;
  MMP_CUDA_TRY(cudaMalloc(&blk, MMP_XBLOCK_BYTES));
  cudaError_t e = cudaMemset(blk, 0, MMP_XBLOCK_BYTES);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, blk);
  char *dev = nullptr;
  if (e == cudaSuccess) e = cudaMalloc((void **)&dev, sizeof(h) * (size_t)(c->nranks + 1) + 16);
  if (e != cudaSuccess) {
    if (dev) cudaFree(dev);
    cudaFree(blk);
    return mmp::cuda_error(e, "peer exchange block");
  }
  // all-gather the handles on the device
  char *hosth = new char[sizeof(h) * (size_t)c->nranks];
  int ok = 1;
  e = cudaMemcpyAsync(dev, &h, sizeof h, cudaMemcpyHostToDevice, st);
  ncclResult_t r = ncclSuccess;
  if (e == cudaSuccess) r = g_api.AllGather(dev, dev + sizeof h, sizeof h, ncclChar, c->comm, st);
  if (e == cudaSuccess && r == ncclSuccess)
    e = cudaMemcpyAsync(hosth, dev + sizeof h, sizeof(h) * (size_t)c->nranks, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess && r == ncclSuccess) e = cudaStreamSynchronize(st);
  void *peer[64] = {};
  if (e != cudaSuccess || r != ncclSuccess) ok = 0;
  for (int q = 0; ok && q < c->nranks; ++q) {
    if (q == c->rank) {
      peer[q] = blk;
      continue;
    }
    cudaIpcMemHandle_t hq;
    memcpy(&hq, hosth + sizeof(h) * (size_t)q, sizeof hq);
    if (cudaIpcOpenMemHandle(&peer[q], hq, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      peer[q] = nullptr;
      ok = 0;
    }
  }
  delete[] hosth;
  // every rank learns whether all of them mapped all peers (MIN of the flags)
  int *dok = (int *)(dev + sizeof(h) * (size_t)(c->nranks + 1));
  int all_ok = 0;
  cudaError_t e2 = cudaMemcpyAsync(dok, &ok, sizeof ok, cudaMemcpyHostToDevice, st);
  ncclResult_t r2 = ncclSuccess;
  if (e2 == cudaSuccess) r2 = g_api.AllReduce(dok, dok, 1, ncclInt32, ncclMin, c->comm, st);
  if (e2 == cudaSuccess && r2 == ncclSuccess) e2 = cudaMemcpyAsync(&all_ok, dok, sizeof all_ok, cudaMemcpyDeviceToHost, st);
  if (e2 == cudaSuccess && r2 == ncclSuccess) e2 = cudaStreamSynchronize(st);
  cudaFree(dev);
  if (e2 != cudaSuccess || r2 != ncclSuccess || !all_ok) {
    for (int q = 0; q < c->nranks; ++q)
      if (q != c->rank && peer[q]) cudaIpcCloseMemHandle(peer[q]);
    cudaFree(blk);
    if (r2 != ncclSuccess) return nccl_error(r2, "peer exchange agreement");
    if (e2 != cudaSuccess) return mmp::cuda_error(e2, "peer exchange agreement");
    return mmp::set_error(MMP_E_UNSUPPORTED, "a rank could not map its peers' exchange blocks");
  }
  for (int q = 0; q < c->nranks; ++q) c->peer[q] = peer[q];
  c->xblk = blk;
  c->epoch = 0;
  c->peer_ok = true;
  return MMP_OK;
}

namespace mmp {
// The current device's exchange blocks and the next exchange epoch (every
// call takes a new one; all ranks make the same sequence of calls).
bool peer_table(void **blk, int *rank, int *nranks, unsigned long long *epoch) {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDev) return false;
  CommState *c = &g_comm[dev];
  if (!c->comm || !c->peer_ok) return false;
  for (int q = 0; q < c->nranks; ++q) blk[q] = c->peer[q];
  *rank = c->rank;
  *nranks = c->nranks;
  *epoch = ++c->epoch;
  return true;
}
}  // namespace mmp

