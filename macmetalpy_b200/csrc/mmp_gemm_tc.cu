// Tensor-core GEMM for sm_100a: TMA -> shared-memory ring -> tcgen05.mma
// with the accumulator in TMEM -> tcgen05.ld epilogue.
//
// Replaces the reference's matmul_op (src/macmetalpy/_kernels.py:735-759),
// a naive one-thread-per-output kernel that accumulates in the element type.
//
// float32 uses the 3xTF32 split: every operand x is written once as
// big = tf32_round(x) and small = x - big (both exactly representable), and
// each k-step issues small*big + big*small + big*big into the same float32
// TMEM accumulator, which keeps float32-level accuracy on the TF32 tensor
// pipe.  float16 runs kind::f16 with float32 accumulation.
//
// A pre-pass writes both operands K-major, zero-padded to whole tiles
// (A -> [batch][Mp][Kp], B -> B^T [batch][Np][Kp]); that is the only layout
// the kernel reads, so any M, N, K, leading dimension and alignment works,
// and every TMA box is fully in bounds.
//
// Kernel: each CTA walks 128 x 256 output tiles round-robin (grouped
// rasterisation for L2 reuse; float16 launches one persistent CTA per SM,
// the TF32 modes one CTA per tile, see run()): warp 0 issues TMA loads
// (one elected lane) and runs straight on into the next tile's K loop, warp 1
// allocates TMEM and issues MMAs (one elected lane), the epilogue warps drain
// TMEM and store C (8 warps accumulating every CHUNK k-tiles for the TF32
// modes, see Cfg::FLUSH; 4 warps for float16).  Two TMEM accumulators
// alternate over the sequence of chunks (float16: one chunk per tile), so
// the MMAs of the next chunk or tile run while the epilogue drains and
// stores the previous one.  Stages and accumulators are handed over with
// mbarriers; tcgen05.commit frees a stage when the MMAs reading it have
// completed.  Every wait is bounded (2 s on %globaltimer): a wait that runs
// out sets the device error word and a CTA-wide abort flag, every role
// leaves its loop, and the CTA finishes (draining its own TMA loads,
// freeing TMEM) instead of hanging.  No TMA multicast is used.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "mmp_device.cuh"
#include "mmp_internal.h"

namespace mmp {
void *driver_fn(const char *name);
}

namespace tc {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int GROUP_M = 16;  // m-blocks per rasterisation group

enum { MODE_3XTF32 = 0, MODE_TF32 = 1, MODE_F16 = 2 };

template <int MODE> struct Cfg {
  static constexpr int ELEM = (MODE == MODE_F16) ? 2 : 4;
  // bytes of K per tile row (128: 128-byte swizzle; 64-byte rows with the
  // 64-byte swizzle are supported too).  3xTF32 keeps 128-byte rows and two
  // stages: measured faster than 64-byte rows with four stages, as the
  // kernel is bound by L2->SM operand bandwidth, not by TMA latency
  static constexpr int ROW_BYTES = 128;
  static constexpr int BK = ROW_BYTES / ELEM;
  static constexpr int NOPS = (MODE == MODE_3XTF32) ? 2 : 1;  // tiles per operand
  static constexpr int A_BYTES = BM * ROW_BYTES;
  static constexpr int B_BYTES = BN * ROW_BYTES;
  static constexpr int STAGE_BYTES = NOPS * (A_BYTES + B_BYTES);
  static constexpr int STAGES = (MODE == MODE_3XTF32) ? 2 : 4;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  static constexpr int UMMA_K_BYTES = 32;  // K of one MMA: 8 tf32 or 16 f16
  static constexpr int KSTEPS = ROW_BYTES / UMMA_K_BYTES;
  static constexpr uint32_t SWIZZLE = (ROW_BYTES == 128) ? 2u : 4u;  // descriptor layout type
  // TF32 modes drain the TMEM accumulator every CHUNK k-tiles into
  // round-to-nearest float32 registers (two TMEM buffers alternate, so the
  // MMAs never wait): the tensor core's float32 accumulation then only spans
  // CHUNK * BK terms, which keeps the 3xTF32 result at float32 accuracy for
  // any K.  float16 keeps one accumulator per tile (its chunk is the tile).
  static constexpr bool FLUSH = (MODE != MODE_F16);
  static constexpr int CHUNK = 512 / ROW_BYTES;  // k-tiles per TMEM chunk: K = 128
  static constexpr int EPI_WARPS = FLUSH ? 8 : 4;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int TMEM_COLS = 2 * BN;  // two accumulators (512 columns, one CTA per SM)
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for the phase of parity `parity`; gives up after ~2 s.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > 2000000000ull) {
      atomicExch(err, 3);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Shared-memory matrix descriptor: K-major tile written by TMA with a
// ROW-byte swizzle (8-row x ROW-byte atoms, 8*ROW bytes apart; layout type 2
// = 128-byte swizzle, 4 = 64-byte swizzle), sm100 version field.
template <int ROW>
__device__ __forceinline__ uint64_t sw_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)1 << 16;                   // leading byte offset (unused with swizzle)
  d |= (uint64_t)((8 * ROW) >> 4) << 32;    // stride byte offset between 8-row groups
  d |= (uint64_t)1 << 46;                   // descriptor version
  d |= (uint64_t)(ROW == 128 ? 2 : 4) << 61;
  return d;
}

// Shared-memory descriptor of an MN-major operand that TMA wrote in boxes of
// 64 MN-elements (128 bytes) x K-rows with the 128-byte swizzle: 8 K-rows
// form a 1024-byte atom, the next 8 K-rows follow at +1024 (stride byte
// offset) and the next 64 MN-elements at +mn_stride (leading byte offset).
__device__ __forceinline__ uint64_t sw_desc_mn(uint32_t saddr, uint32_t mn_stride) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)(mn_stride >> 4) << 16;  // leading byte offset
  d |= (uint64_t)(1024u >> 4) << 32;      // stride byte offset
  d |= (uint64_t)1 << 46;  // descriptor version
  d |= (uint64_t)2 << 61;  // 128-byte swizzle
  return d;
}

// Instruction descriptor: D = f32, A/B format, both K-major, N and M.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t ab_fmt, int M, int N) {
  return (1u << 4) | (ab_fmt << 7) | (ab_fmt << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

template <int MODE>
__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  if constexpr (MODE == MODE_F16) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(acc)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(acc)
        : "memory");
  }
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <int MODE>
__device__ __forceinline__ void store_chunk32(char *crow, long long col0, long long N, const float *v) {
  if (MODE == MODE_F16) {
    __half *p = (__half *)crow + col0;
    if (col0 + 32 <= N && ((uintptr_t)p & 15) == 0) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        __half2 h0 = __floats2half2_rn(v[q * 8 + 0], v[q * 8 + 1]);
        __half2 h1 = __floats2half2_rn(v[q * 8 + 2], v[q * 8 + 3]);
        __half2 h2 = __floats2half2_rn(v[q * 8 + 4], v[q * 8 + 5]);
        __half2 h3 = __floats2half2_rn(v[q * 8 + 6], v[q * 8 + 7]);
        w.x = *reinterpret_cast<uint32_t *>(&h0);
        w.y = *reinterpret_cast<uint32_t *>(&h1);
        w.z = *reinterpret_cast<uint32_t *>(&h2);
        w.w = *reinterpret_cast<uint32_t *>(&h3);
        reinterpret_cast<uint4 *>(p)[q] = w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) p[j] = __float2half_rn(v[j]);
    }
  } else {
    float *p = (float *)crow + col0;
    if (col0 + 32 <= N && ((uintptr_t)p & 15) == 0) {
#pragma unroll
      for (int q = 0; q < 8; ++q)
        reinterpret_cast<float4 *>(p)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + j < N) p[j] = v[j];
    }
  }
}

// B_MN: B is read straight from the caller's row-major (K x N) matrix,
// MN-major in shared memory (four 64-column boxes per stage), instead of
// from the pre-pass's K-major copy.
template <int MODE, bool B_MN>
__global__ void __launch_bounds__(Cfg<MODE>::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmA1,
                   const __grid_constant__ CUtensorMap tmB0, const __grid_constant__ CUtensorMap tmB1, void *C,
                   long long M, long long N, long long ldc, long long sC, int m_blocks, int n_blocks,
                   int k_tiles, int batch, int a_bcast, int b_bcast, int *err) {
  typedef Cfg<MODE> G;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t *full = (uint64_t *)(smem + G::STAGES * G::STAGE_BYTES);
  uint64_t *empty = full + G::STAGES;
  uint64_t *acc_full = empty + G::STAGES;  // [2]
  uint64_t *acc_empty = acc_full + 2;      // [2]
  uint32_t *tmem_holder = (uint32_t *)(acc_empty + 2);
  volatile int *abort_flag = (volatile int *)(tmem_holder + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int per_batch = m_blocks * n_blocks;
  const long long total = (long long)per_batch * batch;
  const int chunk_kt = G::FLUSH ? G::CHUNK : k_tiles;
  const int nchunks = (k_tiles + chunk_kt - 1) / chunk_kt;
  // tile t -> (batch, m-block, n-block); grouped rasterisation: GROUP_M
  // m-blocks share the n sweep (L2 reuse)
  auto coords = [&](long long t, int &bz, int &m_blk, int &n_blk) {
    bz = (int)(t / per_batch);
    const int pid = (int)(t - (long long)bz * per_batch);
    const int per_group = GROUP_M * n_blocks;
    const int first_m = (pid / per_group) * GROUP_M;
    const int gsize = min(m_blocks - first_m, GROUP_M);
    m_blk = first_m + (pid % per_group) % gsize;
    n_blk = (pid % per_group) / gsize;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < G::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], G::EPI_WARPS);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_holder)),
                 "r"(G::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      long long g = 0;  // k-tiles issued by this CTA (stage and phase)
      for (long long t = blockIdx.x; t < total && !*abort_flag; t += gridDim.x) {
        int bz, m_blk, n_blk;
        coords(t, bz, m_blk, n_blk);
        const int ca = a_bcast ? 0 : bz, cb = b_bcast ? 0 : bz;
        for (int kt = 0; kt < k_tiles; ++kt, ++g) {
          const int s = (int)(g % G::STAGES);
          const uint32_t ph = (uint32_t)(g / G::STAGES) & 1u;
          if (*abort_flag || !mbar_wait(&empty[s], ph ^ 1u, err)) {
            *abort_flag = 1;
            break;
          }
          uint8_t *st = smem + s * G::STAGE_BYTES;
          mbar_expect_tx(&full[s], G::STAGE_BYTES);
          const int kc = kt * G::BK;
          tma_load_3d(st, &tmA0, &full[s], kc, m_blk * BM, ca);
          if (G::NOPS == 2) tma_load_3d(st + G::A_BYTES, &tmA1, &full[s], kc, m_blk * BM, ca);
          if (B_MN) {
#pragma unroll
            for (int q = 0; q < BN / 64; ++q)
              tma_load_3d(st + G::A_BYTES + q * (G::BK * 128), &tmB0, &full[s], n_blk * BN + 64 * q, kc, cb);
          } else {
            tma_load_3d(st + G::NOPS * G::A_BYTES, &tmB0, &full[s], kc, n_blk * BN, cb);
            if (G::NOPS == 2)
              tma_load_3d(st + G::NOPS * G::A_BYTES + G::B_BYTES, &tmB1, &full[s], kc, n_blk * BN, cb);
          }
        }
      }
      // drain: every load this CTA issued has landed before it may exit
      for (long long gg = (g > G::STAGES ? g - G::STAGES : 0); gg < g; ++gg)
        mbar_wait(&full[gg % G::STAGES], (uint32_t)(gg / G::STAGES) & 1u, err);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // bit 16: B is MN-major
      constexpr uint32_t ID = make_idesc(MODE == MODE_F16 ? 0u : 2u, BM, BN) | (B_MN ? (1u << 16) : 0u);
      long long g = 0, cg = 0;  // k-tiles and accumulator chunks consumed by this CTA
      bool ok = true;
      for (long long t = blockIdx.x; t < total && ok; t += gridDim.x) {
        for (int kt = 0; kt < k_tiles && ok; ++kt, ++g) {
          const int buf = (int)(cg & 1);
          const bool first_of_chunk = (kt % chunk_kt) == 0;
          if (first_of_chunk && cg >= 2) {  // buffer drained by the epilogue?
            if (*abort_flag || !mbar_wait(&acc_empty[buf], (uint32_t)((cg >> 1) - 1) & 1u, err)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          const int s = (int)(g % G::STAGES);
          const uint32_t ph = (uint32_t)(g / G::STAGES) & 1u;
          if (*abort_flag || !mbar_wait(&full[s], ph, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + (uint32_t)(buf * BN);
          const uint32_t base = smem_u32(smem + s * G::STAGE_BYTES);
          const uint32_t b0 = base + G::NOPS * G::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < G::KSTEPS; ++kk) {
            const uint32_t off = kk * G::UMMA_K_BYTES;
            const uint64_t da0 = sw_desc<G::ROW_BYTES>(base + off);
            // MN-major B: one MMA's K (16 rows of 128 bytes) is 2048 bytes
            const uint64_t db0 = B_MN ? sw_desc_mn(b0 + kk * 2048, G::BK * 128) : sw_desc<G::ROW_BYTES>(b0 + off);
            const uint32_t acc = (!first_of_chunk || kk > 0) ? 1u : 0u;
            if (MODE == MODE_3XTF32) {
              const uint64_t da1 = sw_desc<G::ROW_BYTES>(base + G::A_BYTES + off);
              const uint64_t db1 = sw_desc<G::ROW_BYTES>(b0 + G::B_BYTES + off);
              umma<MODE>(d, da1, db0, ID, acc);  // small * big
              umma<MODE>(d, da0, db1, ID, 1u);   // big * small
              umma<MODE>(d, da0, db0, ID, 1u);   // big * big
            } else {
              umma<MODE>(d, da0, db0, ID, acc);
            }
          }
          umma_commit(&empty[s]);  // stage reusable once these MMAs are done
          if ((kt % chunk_kt) == chunk_kt - 1 || kt == k_tiles - 1) {
            umma_commit(&acc_full[buf]);
            ++cg;
          }
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // epilogue warps: lane quadrant q = warp % 4 (TMEM access rule), column
    // half h when there are 8 of them
    const int ew = warp - 2;
    const int q = warp & 3;
    const int h = (G::EPI_WARPS == 8) ? (ew >> 2) : 0;
    constexpr int COLS = BN / (G::EPI_WARPS / 4);  // columns per warp
    const int row = q * 32 + lane;
    long long cg = 0;  // accumulator chunks drained by this CTA
    bool ok = true;
    for (long long t = blockIdx.x; t < total && ok; t += gridDim.x) {
      int bz, m_blk, n_blk;
      coords(t, bz, m_blk, n_blk);
      const long long gm = (long long)m_blk * BM + row;
      const long long n0 = (long long)n_blk * BN + h * COLS;
      char *crow = (char *)C + ((long long)bz * sC + gm * ldc) * (MODE == MODE_F16 ? 2 : 4);
      if (G::FLUSH) {
        float acc[COLS];
#pragma unroll
        for (int j = 0; j < COLS; ++j) acc[j] = 0.f;
        for (int chunk = 0; chunk < nchunks; ++chunk, ++cg) {
          const int buf = (int)(cg & 1);
          if (ok && (*abort_flag || !mbar_wait(&acc_full[buf], (uint32_t)(cg >> 1) & 1u, err))) ok = false;
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < COLS / 32; ++c) {
            uint32_t r[32];
            tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN + h * COLS + c * 32), r);
#pragma unroll
            for (int j = 0; j < 32; ++j) acc[c * 32 + j] += __uint_as_float(r[j]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&acc_empty[buf]))
                                      : "memory");
        }
        if (ok && gm < M) {
#pragma unroll
          for (int c = 0; c < COLS / 32; ++c) {
            const long long col0 = n0 + c * 32;
            if (col0 < N) store_chunk32<MODE>(crow, col0, N, acc + c * 32);
          }
        }
      } else {
        const int buf = (int)(cg & 1);
        if (*abort_flag || !mbar_wait(&acc_full[buf], (uint32_t)(cg >> 1) & 1u, err)) ok = false;
        if (!ok) break;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < COLS / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * BN + h * COLS + c * 32), r);
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
          const long long col0 = n0 + c * 32;
          if (gm < M && col0 < N) store_chunk32<MODE>(crow, col0, N, v);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&acc_empty[buf]))
                                    : "memory");
        ++cg;
      }
    }
    if (!ok) *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(G::TMEM_COLS) : "memory");
  }
}

// ---------------------------------------------------------------- pre-pass
__device__ __forceinline__ float tf32_round(float v) {
  uint32_t u = __float_as_uint(v);
  if ((u & 0x7f800000u) == 0x7f800000u) return v;  // inf / nan unchanged
  u = (u + 0x1000u) & 0xffffe000u;
  return __uint_as_float(u);
}

// One element of an operand in the pre-pass's output form(s).
template <class T, int MODE>
__device__ __forceinline__ void prep_split(T v, T &o0, T &o1) {
  if constexpr (MODE == MODE_3XTF32) {
    const float big = tf32_round((float)v);
    o0 = big;
    o1 = (float)v - big;
  } else if constexpr (MODE == MODE_TF32) {
    o0 = tf32_round((float)v);
  } else {
    o0 = v;
  }
}

// A[b] (M x K, row stride lda) -> out0/out1 [b][Mp][Kp], zero padded: rows
// of Kp over blockIdx.y (grid-stride), 4 consecutive k per thread (one
// vector load when the source row allows, `vec_src`), vector stores.
template <class T, int MODE>
__global__ void __launch_bounds__(256) prep_rows_kernel(const T *__restrict__ A, long long lda, long long sA,
                                                        long long M, long long K, long long Mp, long long Kp,
                                                        long long batch, T *__restrict__ out0,
                                                        T *__restrict__ out1, int vec_src) {
  const long long rows = batch * Mp;
  for (long long r = blockIdx.y; r < rows; r += gridDim.y) {
    const long long b = r / Mp, m = r - b * Mp;
    const T *src = A + b * sA + m * lda;
    T *d0 = out0 + r * Kp;
    T *d1 = out1 + r * Kp;
    for (long long k0 = ((long long)blockIdx.x * 256 + threadIdx.x) * 4; k0 < Kp;
         k0 += (long long)gridDim.x * 256 * 4) {
      T v[4];
      if (m < M && vec_src && k0 + 3 < K) {
        const mmpd::Vec<T, 4> t = mmpd::ldvec_stream<T, 4>(src + k0);
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = t.v[e];
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = (m < M && k0 + e < K) ? src[k0 + e] : T(0);
      }
      mmpd::Vec<T, 4> o0, o1;
#pragma unroll
      for (int e = 0; e < 4; ++e) prep_split<T, MODE>(v[e], o0.v[e], o1.v[e]);
      mmpd::stvec<T, 4>(d0 + k0, o0);
      if (MODE == MODE_3XTF32) mmpd::stvec<T, 4>(d1 + k0, o1);
    }
  }
}

// B[b] (K x N, row stride ldb) -> out[b][Np][Kp] = B^T, through a 32 (k) x
// 128 (n) shared tile: 4 consecutive n per thread on the way in (one vector
// load when the source row allows), 4 consecutive k per thread on the way
// out (vector stores); the one-word row padding keeps the column reads free
// of bank conflicts.
template <class T, int MODE>
__global__ void __launch_bounds__(256) prep_cols_kernel(const T *__restrict__ B, long long ldb, long long sB,
                                                        long long K, long long N, long long Np, long long Kp,
                                                        long long batch, T *__restrict__ out0,
                                                        T *__restrict__ out1, int vec_src) {
  __shared__ T tile[32][129];
  const long long n0 = (long long)blockIdx.x * 128, k0 = (long long)blockIdx.y * 32;
  const int t = threadIdx.x;
  for (long long b = blockIdx.z; b < batch; b += gridDim.z) {
    const T *src = B + b * sB;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int kr = (t >> 5) + 8 * i, nl = (t & 31) * 4;
      const long long k = k0 + kr, n = n0 + nl;
      T v[4];
      if (k < K && vec_src && n + 3 < N) {
        const mmpd::Vec<T, 4> q = mmpd::ldvec_stream<T, 4>(src + k * ldb + n);
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = q.v[e];
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = (k < K && n + e < N) ? src[k * ldb + n + e] : T(0);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) tile[kr][nl + e] = v[e];
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int nl = (t >> 3) + 32 * i, kl = (t & 7) * 4;
      const long long o = (b * Np + n0 + nl) * Kp + k0 + kl;
      mmpd::Vec<T, 4> o0, o1;
#pragma unroll
      for (int e = 0; e < 4; ++e) prep_split<T, MODE>(tile[kl + e][nl], o0.v[e], o1.v[e]);
      mmpd::stvec<T, 4>(out0 + o, o0);
      if (MODE == MODE_3XTF32) mmpd::stvec<T, 4>(out1 + o, o1);
    }
    __syncthreads();
  }
}

typedef CUresult (*PFN_Encode)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                               const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                               CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static int make_map(CUtensorMap *map, const void *base, bool f16, long long kp, long long rows, long long batch,
                    int box_k, int box_rows, int row_bytes) {
  static PFN_Encode enc = nullptr;
  if (!enc) enc = (PFN_Encode)mmp::driver_fn("cuTensorMapEncodeTiled");
  if (!enc) return mmp::set_error(MMP_E_CUDA, "cuTensorMapEncodeTiled unavailable");
  const int es = f16 ? 2 : 4;
  cuuint64_t dims[3] = {(cuuint64_t)kp, (cuuint64_t)rows, (cuuint64_t)batch};
  cuuint64_t strides[2] = {(cuuint64_t)(kp * es), (cuuint64_t)(kp * rows * es)};
  cuuint32_t box[3] = {(cuuint32_t)box_k, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                   const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return mmp::set_error(MMP_E_CUDA, "cuTensorMapEncodeTiled failed");
  return MMP_OK;
}

// Tensor map over a caller's matrix: dims {d0 (contiguous), d1, d2}, byte
// strides of d1 and d2, box {box0, box1}, 128-byte swizzle; loads past the
// edges read zeros.
static int make_map_user(CUtensorMap *map, const void *base, long long d0, long long d1, long long d2,
                         long long s1_bytes, long long s2_bytes, int box0, int box1) {
  static PFN_Encode enc = nullptr;
  if (!enc) enc = (PFN_Encode)mmp::driver_fn("cuTensorMapEncodeTiled");
  if (!enc) return mmp::set_error(MMP_E_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
  cuuint64_t strides[2] = {(cuuint64_t)s1_bytes, (cuuint64_t)s2_bytes};
  cuuint32_t box[3] = {(cuuint32_t)box0, (cuuint32_t)box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return mmp::set_error(MMP_E_CUDA, "cuTensorMapEncodeTiled failed");
  return MMP_OK;
}

template <int MODE, bool B_MN>
static int launch(const CUtensorMap &mA0, const CUtensorMap &mA1, const CUtensorMap &mB0, const CUtensorMap &mB1,
                  void *c, long long m, long long n, long long ldc, long long sc, long long m_blocks,
                  long long n_blocks, long long k_tiles, long long batch, int a_bc, int b_bc, cudaStream_t st) {
  typedef Cfg<MODE> G;
  static bool attr[64];  // per device: function attributes are set per device
  const int dev = mmp::current_device();
  if (dev < 0 || dev >= 64) return mmp::set_error(MMP_E_ARG, "device out of range");
  if (!attr[dev]) {
    MMP_CUDA_TRY(
        cudaFuncSetAttribute(gemm_tc_kernel<MODE, B_MN>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM));
    attr[dev] = true;
  }
  // float16: persistent, one CTA per SM (the stage ring fills shared
  // memory), tiles handed out round-robin -- the next tile's MMAs overlap
  // this tile's epilogue (measured 2-8 % faster than a CTA per tile).  The
  // TF32 modes are persistent too while K <= 8192 (a tile's fill and drain
  // are then a visible share of it: batched 64 x 1024^3 3xTF32 139.5 ->
  // 147.1 TFLOP/s, 4096^3 and 8192^3 +1 %); longer K launches one CTA per
  // tile, whose dynamic hardware order kept L2 reuse better (16384^3
  // 3xTF32 measured 11 % slower with the static round-robin order).
  const long long tiles = m_blocks * n_blocks * batch;
  const long long sms = (long long)mmp::sm_count();
  const bool persistent = MODE == MODE_F16 || k_tiles * G::BK <= 8192;
  const long long ctas = (persistent && tiles > sms) ? sms : tiles;
  if (ctas > 0x7fffffffll) return mmp::set_error(MMP_E_UNSUPPORTED, "GEMM too large for one launch");
  gemm_tc_kernel<MODE, B_MN><<<(unsigned)ctas, G::THREADS, G::SMEM, st>>>(
      mA0, mA1, mB0, mB1, c, m, n, ldc, sc, (int)m_blocks, (int)n_blocks, (int)k_tiles, (int)batch, a_bc, b_bc,
      mmp::device_error_word());
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return mmp::cuda_error(e, "gemm_tc_kernel");
  return MMP_OK;
}

template <int MODE, class T>
static int run(long long batch, long long m, long long n, long long k, const void *a, long long lda, long long sa,
               const void *b, long long ldb, long long sb, void *c, long long ldc, long long sc) {
  typedef Cfg<MODE> G;
  cudaStream_t st = mmp::stream();
  if (!st) return mmp::set_error(MMP_E_CUDA, "no stream");
  const long long Mp = (m + BM - 1) / BM * BM;
  const long long Np = (n + BN - 1) / BN * BN;
  const long long Kp = (k + G::BK - 1) / G::BK * G::BK;
  const int a_bc = (sa == 0 && batch > 1) ? 1 : 0;
  const int b_bc = (sb == 0 && batch > 1) ? 1 : 0;
  const long long ba = a_bc ? 1 : batch, bb = b_bc ? 1 : batch;
  const long long m_blocks = Mp / BM, n_blocks = Np / BN, k_tiles = Kp / G::BK;
  if (m_blocks * n_blocks > 0x7fffffffll || m_blocks * n_blocks * batch > (1ll << 40) || k_tiles > 0x7fffffffll)
    return mmp::set_error(MMP_E_UNSUPPORTED, "GEMM too large for one launch");
  if constexpr (MODE == MODE_F16) {
    // No pre-pass: TMA reads A (row-major, K-major tiles) and B (row-major,
    // MN-major tiles) from the caller's buffers, zero-filling past the
    // edges, when every row and batch pitch is a multiple of 16 bytes.
    const bool aligned = (uintptr_t)a % 16 == 0 && (uintptr_t)b % 16 == 0 && lda % 8 == 0 && ldb % 8 == 0 &&
                         (a_bc || batch == 1 || sa % 8 == 0) && (b_bc || batch == 1 || sb % 8 == 0);
    if (aligned) {
      CUtensorMap mA, mB;
      const long long sa_b = (a_bc || batch == 1) ? lda * m * 2 : sa * 2;
      const long long sb_b = (b_bc || batch == 1) ? ldb * k * 2 : sb * 2;
      int rc = make_map_user(&mA, a, k, m, ba, lda * 2, sa_b > 0 ? sa_b : 16, G::BK, BM);
      if (!rc) rc = make_map_user(&mB, b, n, k, bb, ldb * 2, sb_b > 0 ? sb_b : 16, 64, G::BK);
      if (rc) return rc;
      return launch<MODE, true>(mA, mA, mB, mB, c, m, n, ldc, sc, m_blocks, n_blocks, k_tiles, batch, a_bc, b_bc,
                                st);
    }
  }
  const size_t es = G::ELEM;
  const size_t a_el = (size_t)ba * Mp * Kp, b_el = (size_t)bb * Np * Kp;
  const size_t ws_bytes = G::NOPS * (a_el + b_el) * es + 1024;
  char *ws = nullptr;
  MMP_CUDA_TRY(cudaMallocAsync((void **)&ws, ws_bytes, st));
  T *A0 = (T *)ws;
  T *A1 = A0 + a_el;                       // used by 3xTF32 only
  T *B0 = A0 + (G::NOPS == 2 ? 2 * a_el : a_el);
  T *B1 = B0 + b_el;
  {
    const size_t vb = 4 * sizeof(T);  // one vector of 4 elements
    const int va = (uintptr_t)a % vb == 0 && lda % 4 == 0 && (ba == 1 || sa % 4 == 0);
    const int vbb = (uintptr_t)b % vb == 0 && ldb % 4 == 0 && (bb == 1 || sb % 4 == 0);
    const long long rows = ba * Mp, gx = (Kp + 1023) / 1024;
    dim3 g1((unsigned)gx, (unsigned)(rows < 65535 ? rows : 65535), 1);
    prep_rows_kernel<T, MODE><<<g1, 256, 0, st>>>((const T *)a, lda, sa, m, k, Mp, Kp, ba, A0, A1, va);
    dim3 g2((unsigned)(Np / 128), (unsigned)(Kp / 32), (unsigned)(bb < 65535 ? bb : 65535));
    prep_cols_kernel<T, MODE><<<g2, 256, 0, st>>>((const T *)b, ldb, sb, k, n, Np, Kp, bb, B0, B1, vbb);
  }
  CUtensorMap mA0, mA1, mB0, mB1;
  const bool f16 = MODE == MODE_F16;
  const int RB = G::ROW_BYTES;
  int rc = make_map(&mA0, A0, f16, Kp, Mp, ba, G::BK, BM, RB);
  if (!rc) rc = make_map(&mA1, G::NOPS == 2 ? (const void *)A1 : (const void *)A0, f16, Kp, Mp, ba, G::BK, BM, RB);
  if (!rc) rc = make_map(&mB0, B0, f16, Kp, Np, bb, G::BK, BN, RB);
  if (!rc) rc = make_map(&mB1, G::NOPS == 2 ? (const void *)B1 : (const void *)B0, f16, Kp, Np, bb, G::BK, BN, RB);
  if (rc) {
    cudaFreeAsync(ws, st);
    return rc;
  }
  rc = launch<MODE, false>(mA0, mA1, mB0, mB1, c, m, n, ldc, sc, m_blocks, n_blocks, k_tiles, batch, a_bc, b_bc,
                           st);
  cudaFreeAsync(ws, st);
  return rc;
}

}  // namespace tc

namespace mmp {

int gemm_tc(int dtype, int mode, long long batch, long long m, long long n, long long k, const void *a, long long lda,
            long long sa, const void *b, long long ldb, long long sb, void *c, long long ldc, long long sc) {
  if (mode == MMP_GEMM_AUTO && m * n * k < (1ll << 21))
    return set_error(MMP_E_UNSUPPORTED, "small problem: CUDA-core path");
  if (dtype == MMP_FLOAT32) {
    if (mode == MMP_GEMM_AUTO || mode == MMP_GEMM_3XTF32)
      return tc::run<tc::MODE_3XTF32, float>(batch, m, n, k, a, lda, sa, b, ldb, sb, c, ldc, sc);
    if (mode == MMP_GEMM_TF32)
      return tc::run<tc::MODE_TF32, float>(batch, m, n, k, a, lda, sa, b, ldb, sb, c, ldc, sc);
  }
  if (dtype == MMP_FLOAT16 && (mode == MMP_GEMM_AUTO || mode == MMP_GEMM_F16))
    return tc::run<tc::MODE_F16, __half>(batch, m, n, k, a, lda, sa, b, ldb, sb, c, ldc, sc);
  return set_error(MMP_E_UNSUPPORTED, "no tensor-core path for this dtype/mode");
}

}  // namespace mmp
