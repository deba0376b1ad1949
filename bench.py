"""Benchmark of the macmetalpy_b200 hot path (driver contract: one JSON line).

Headline workload ("C2"): binary ufuncs at 2^28
elements -- float32 add / floor_divide / mod / logaddexp and int32 add /
floor_divide / mod, with a ~ U(-1000, 1000) and b ~ U(1, 50) * (+-1), plus
the broadcast add (8192, 1) + (1, 32768) float32 ~ N(0, 1).  One step is one
pass over that op set through the public API (``cp.add(A, B, out=C)`` ...),
inputs resident in HBM.  ``value`` = algorithmic HBM bytes of the step
(12 bytes per element per binary op: two 4-byte reads, one 4-byte write;
the broadcast add counts its output and both inputs) / device time, summed
over ranks (weak scaling: every rank owns its own 2^28-element operands;
the elementwise path has no exchange step, so no collective).  Inputs are
1 GiB per operand, far above the 126 MB L2, so no flush is needed.

Extra keys: ``roofline`` (the dominant kernel timed live with CUDA events;
peak from MEASURED_PEAKS.json), ``cpu_baseline`` (the numpy oracle port on
a bounded sample, 1 thread), ``e2e`` (same op set with pinned host inputs
copied in and results copied out every step), ``clocks`` (nvidia-smi sampled
during the timed region), ``gpu_launches`` and ``suite`` (per-config GB/s or
TFLOP/s for C1, C3, C4, C5, each timed with CUDA events after the main run).

``--impl reference`` times the reference's CPU path for the same ops: the
numpy oracle port (the reference is Python; its Metal path cannot run on
Linux) over all host threads, on a bounded sample per step.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
# stdout carries the one JSON line: NCCL's log (its version line, printed
# when NCCL_DEBUG is set in the environment) goes to stderr instead
os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")

N_C2 = 1 << 28
BC_ROWS, BC_COLS = 8192, 32768
METRIC = "fused elementwise/reduce/scan HBM GB/s (% of 8 TB/s); fp32 matmul TFLOP/s"
F32_OPS = ("add", "floor_divide", "mod", "logaddexp")
I32_OPS = ("add", "floor_divide", "mod")


def _peaks():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def _env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (SM clock, throttle reasons) while running."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, local_rank: int):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        idx = local_rank
        if vis and all(v.strip().isdigit() for v in vis.split(",")):
            idx = int(vis.split(",")[local_rank])
        self.idx = idx
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-i",
                 str(self.idx), "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                rows.append((float(parts[0]), float(parts[1]), float(parts[2]), parts[3:]))
            except ValueError:
                continue
        if not rows:
            return None
        loaded = [r for r in rows if r[2] > 200.0] or rows
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in loaded:
            for nm, v in zip(names, r[3][1:]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": sorted(reasons), "samples": len(loaded)}


# --------------------------------------------------------------------------- device inputs
RNG_SRC = r'''
// SplitMix64 (Steele, Lea, Flood 2014) of (seed, index): seeded synthetic data
__device__ __forceinline__ unsigned long long sm64(unsigned long long z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}
__device__ __forceinline__ double u01(unsigned long long h) { return ((h >> 11) + 0.5) * (1.0 / 9007199254740992.0); }
extern "C" __global__ void gen_f32(float* out, long long n, unsigned long long seed, int kind, float lo, float hi) {
  long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  long long st = (long long)gridDim.x * blockDim.x;
  for (; i < n; i += st) {
    unsigned long long h = sm64(seed * 0x100000001b3ull + (unsigned long long)i);
    double u = u01(h);
    float v;
    if (kind == 0) v = (float)(lo + (hi - lo) * u);                          // uniform
    else if (kind == 1) {                                                     // normal (Box-Muller)
      double u2 = u01(sm64(h));
      v = (float)(sqrt(-2.0 * log(u)) * cospi(2.0 * u2));
    } else {                                                                  // +-U(lo, hi)
      double s = (sm64(h ^ 0x5555ull) & 1ull) ? 1.0 : -1.0;
      v = (float)(s * (lo + (hi - lo) * u));
    }
    out[i] = v;
  }
}
extern "C" __global__ void gen_i32(int* out, long long n, unsigned long long seed, int lo, int hi, int signed_) {
  long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  long long st = (long long)gridDim.x * blockDim.x;
  for (; i < n; i += st) {
    unsigned long long h = sm64(seed * 0x100000001b3ull + (unsigned long long)i);
    int v = lo + (int)(h % (unsigned long long)(hi - lo));
    if (signed_ && (sm64(h ^ 0x5555ull) & 1ull)) v = -v;
    out[i] = v;
  }
}
'''


class Gen:
    def __init__(self, cp):
        self.cp = cp
        self.kf = cp.RawKernel(RNG_SRC, "gen_f32")
        self.ki = cp.RawKernel(RNG_SRC, "gen_i32")

    def _launch(self, k, out, args):
        n = out.size
        threads = min(n, 148 * 2048)
        k(max(threads, 1), (out, np.int64(n)) + args)

    def uniform(self, shape, lo, hi, seed):
        a = self.cp.empty(shape, dtype=np.float32)
        self._launch(self.kf, a, (np.uint64(seed), np.int32(0), np.float32(lo), np.float32(hi)))
        return a

    def normal(self, shape, seed):
        a = self.cp.empty(shape, dtype=np.float32)
        self._launch(self.kf, a, (np.uint64(seed), np.int32(1), np.float32(0), np.float32(1)))
        return a

    def signed_uniform(self, shape, lo, hi, seed):
        a = self.cp.empty(shape, dtype=np.float32)
        self._launch(self.kf, a, (np.uint64(seed), np.int32(2), np.float32(lo), np.float32(hi)))
        return a

    def integers(self, shape, lo, hi, seed, signed=False):
        a = self.cp.empty(shape, dtype=np.int32)
        self._launch(self.ki, a, (np.uint64(seed), np.int32(lo), np.int32(hi), np.int32(1 if signed else 0)))
        return a


# --------------------------------------------------------------------------- C2 workload
def c2_inputs(cp, gen, n=N_C2):
    d = {}
    d["af"] = gen.uniform((n,), -1000, 1000, 1)
    d["bf"] = gen.signed_uniform((n,), 1, 50, 2)
    d["ai"] = gen.integers((n,), -1000, 1000, 3)
    d["bi"] = gen.integers((n,), 1, 50, 4, signed=True)
    d["r"] = gen.normal((BC_ROWS, 1), 5)
    d["c"] = gen.normal((1, BC_COLS), 6)
    d["of"] = cp.empty((n,), dtype=np.float32)
    d["oi"] = cp.empty((n,), dtype=np.int32)
    d["ob"] = cp.empty((BC_ROWS, BC_COLS), dtype=np.float32)
    return d


def c2_ops(cp, d):
    """[(name, thunk, algorithmic bytes)] of one step."""
    n = d["af"].size
    ops = []
    for nm in F32_OPS:
        fn = getattr(cp, nm)
        ops.append((f"{nm}_f32", (lambda fn=fn: fn(d["af"], d["bf"], out=d["of"])), 12 * n))
    for nm in I32_OPS:
        fn = getattr(cp, nm)
        ops.append((f"{nm}_i32", (lambda fn=fn: fn(d["ai"], d["bi"], out=d["oi"])), 12 * n))
    bcb = 4 * BC_ROWS * BC_COLS + 4 * (BC_ROWS + BC_COLS)
    ops.append(("bcast_add_f32", lambda: cp.add(d["r"], d["c"], out=d["ob"]), bcb))
    return ops


def step_bytes(n=N_C2):
    return (len(F32_OPS) + len(I32_OPS)) * 12 * n + 4 * BC_ROWS * BC_COLS + 4 * (BC_ROWS + BC_COLS)


# --------------------------------------------------------------------------- CPU legs (oracle port)
def cpu_c2_inputs(n, seed=0):
    rng = np.random.default_rng(seed)
    af = rng.uniform(-1000, 1000, n).astype(np.float32)
    bf = (rng.uniform(1, 50, n) * rng.choice([-1, 1], n)).astype(np.float32)
    ai = rng.integers(-1000, 1000, n).astype(np.int32)
    bi = (rng.integers(1, 50, n) * rng.choice([-1, 1], n)).astype(np.int32)
    rows = max(1, int(BC_ROWS * n / N_C2))
    r = rng.standard_normal((rows, 1)).astype(np.float32)
    c = rng.standard_normal((1, BC_COLS)).astype(np.float32)
    return (af, bf, ai, bi, r, c)


def cpu_c2_pass(n, threads=1, seed=0, inputs=None):
    """The reference's CPU path for the C2 op set on n elements (numpy port),
    split over `threads` host threads (numpy releases the GIL in ufuncs).
    Returns (algorithmic bytes, seconds); input generation is not timed."""
    from oracle import oracle as O

    af, bf, ai, bi, r, c = inputs if inputs is not None else cpu_c2_inputs(n, seed)
    rows = r.shape[0]
    fns = [(O.add, af, bf), (O.floor_divide, af, bf), (O.mod, af, bf), (O.logaddexp, af, bf),
           (O.add, ai, bi), (O.floor_divide, ai, bi), (O.mod, ai, bi)]
    nbytes = 7 * 12 * n + 4 * rows * BC_COLS + 4 * (rows + BC_COLS)

    def run_chunk(lo, hi):
        for f, a, b in fns:
            f(a[lo:hi], b[lo:hi])
        rl, rh = lo * rows // n, hi * rows // n
        O.broadcast_add(r[rl:rh], c)

    t0 = time.perf_counter()
    if threads <= 1:
        run_chunk(0, n)
    else:
        bounds = [n * i // threads for i in range(threads + 1)]
        ts = [threading.Thread(target=run_chunk, args=(bounds[i], bounds[i + 1])) for i in range(threads)]
        for t in ts:
            t.start()
        for t in ts:
            t.join()
    dt = time.perf_counter() - t0
    return nbytes, dt


def cpu_baseline(sample_n=1 << 24, reps=2):
    best = None
    nbytes = 0
    inputs = cpu_c2_inputs(sample_n, 0)
    for _ in range(reps):
        nbytes, dt = cpu_c2_pass(sample_n, threads=1, inputs=inputs)
        best = dt if best is None else min(best, dt)
    return {"value": round(nbytes / best / 1e9, 3), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"C2 op set on {sample_n} elements per operand (broadcast add scaled to "
                      f"{max(1, int(BC_ROWS * sample_n / N_C2))} rows), numpy oracle, 1 thread, best of {reps}"}


def run_reference(args):
    """The reference's CPU path (the numpy oracle port) on the GPU arm's own
    configuration: the C2 op set on 2^28 elements per operand, inputs made
    once (seed 0, not timed), every step a full pass over all host threads
    (numpy releases the GIL inside ufuncs, so the pass is split into one
    contiguous chunk per thread)."""
    rank, world, _ = _env()
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    n = N_C2
    inputs = cpu_c2_inputs(n, 0)
    for _ in range(args.warmup):
        cpu_c2_pass(n, threads=threads, inputs=inputs)
    times, nbytes = [], 0
    for _ in range(args.steps):
        nbytes, dt = cpu_c2_pass(n, threads=threads, inputs=inputs)
        times.append(dt)
    tot = sum(times)
    val = nbytes * args.steps / tot / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(val, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * tot / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32+i32",
        "data": "synthetic (numpy default_rng, seeded)",
        "config": {"workload": "C2: binary ufuncs at 2^28 (add/floor_divide/mod/logaddexp f32, "
                               "add/floor_divide/mod i32) + broadcast add (8192,1)+(1,32768) f32",
                   "elements_per_operand": n},
        "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"the full workload: {n} elements per operand per step, {threads} threads"},
        "e2e": {"value": round(val, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


# --------------------------------------------------------------------------- GPU arm
def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-suite", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--case", default=None, help="time one op only (for profiling): " + ", ".join(CASES))
    ap.add_argument("--elements", type=int, default=1 << 26, help="--case size (matmul: n of n^3)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.case:
        return run_case(args)
    rank, world, local = _env()
    import macmetalpy_b200 as cp
    from macmetalpy_b200._cuda_backend import CudaBackend, Event

    dist = None
    if world > 1:
        # the library's own communicator (NCCL through the C ABI), bound to
        # the library stream; no torch process group
        from macmetalpy_b200 import distributed as dist

        dist.init(timeout_s=120)
    be = CudaBackend()
    gen = Gen(cp)
    d = c2_inputs(cp, gen)
    ops = c2_ops(cp, d)

    def barrier():
        be.synchronize()
        if dist is not None:
            dist.barrier()

    for _ in range(max(args.warmup, 3)):
        for _, f, _ in ops:
            f()
    barrier()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    evs = [[Event() for _ in range(len(ops) + 1)] for _ in range(args.steps)]
    barrier()
    t_start = Event()
    t_end = Event()
    t_start.record()
    for s in range(args.steps):
        evs[s][0].record()
        for j, (_, f, _) in enumerate(ops):
            f()
            evs[s][j + 1].record()
    t_end.record()
    barrier()
    clocks = sampler.stop() if sampler else None
    ms = t_start.elapsed_ms(t_end)
    per_op = [0.0] * len(ops)
    for s in range(args.steps):
        for j in range(len(ops)):
            per_op[j] += evs[s][j].elapsed_ms(evs[s][j + 1])
    if dist is not None:
        ms = dist.max_over_ranks(ms)
    sb = step_bytes()
    value = world * sb * args.steps / (ms / 1e3) / 1e9
    peaks, peak_kind = _peaks()
    hbm = float(peaks["hbm_gbs"])
    dom = max(range(len(ops)), key=lambda j: per_op[j])
    dom_ms = per_op[dom] / args.steps
    dom_gbs = ops[dom][2] / (dom_ms / 1e3) / 1e9
    op_table = {ops[j][0]: round(ops[j][2] / (per_op[j] / args.steps / 1e3) / 1e9, 1) for j in range(len(ops))}
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32+i32",
        "data": "synthetic, device-generated SplitMix64 streams (seeded), BASELINE distributions",
        "config": {"workload": "C2: binary ufuncs at 2^28 (add/floor_divide/mod/logaddexp f32, "
                               "add/floor_divide/mod i32) + broadcast add (8192,1)+(1,32768) f32",
                   "elements_per_operand_per_gpu": N_C2, "l2": "inputs 1 GiB per operand > 126 MB L2, no flush",
                   "parallelism": f"shard-local x{world}", "api": "cp.<ufunc>(a, b, out=c)"},
        "frac_of_hbm_peak": round(value / world / hbm, 4),
        "per_op_gbs": op_table,
        "roofline": {"bound": "hbm", "kernel": f"mmp_fused_ew ({ops[dom][0]})", "achieved": round(dom_gbs, 1),
                     "peak": hbm, "unit": "GB/s", "frac": round(dom_gbs / hbm, 4),
                     "peak_source": f"{peak_kind} hbm_gbs", "traffic": _traffic(ops[dom][0]),
                     "algorithmic_bytes_per_launch": ops[dom][2], "avg_launch_ms": round(dom_ms, 4)},
        "clocks": clocks,
        "gpu_launches": args.steps * len(ops),
    }
    if not args.no_e2e:
        # 8 steps: the pipeline's one-time fill (the first step's uploads,
        # ~80 ms at N = 1) is amortised over them
        line["e2e"] = e2e_c2(cp, d, steps=8, dist=dist)
    if rank == 0 and not args.no_cpu and world == 1:
        line["cpu_baseline"] = cpu_baseline()
    if not args.no_suite:
        del d, ops
        import gc

        gc.collect()
        if world == 1:
            if rank == 0:
                line["suite"] = run_suite(cp, gen)
        else:
            line["dist_suite"] = dist_suite(cp, gen)
            line["dist_parity"] = line["dist_suite"].pop("parity")
    if rank == 0:
        print(json.dumps(line))
    if dist is not None:
        dist.barrier()
        dist.finalize()
    return 0


CASES = ("add_f32", "floor_divide_f32", "mod_f32", "logaddexp_f32", "add_i32", "floor_divide_i32", "mod_i32",
         "bcast_add_f32", "c1_fused_sum", "sum_f32", "var_f32", "argmax_f32", "argmin_f32", "nansum_f32",
         "sum_axis0_f32", "sum_axis1_f32",
         "var_axis0_f32", "argmax_axis0_f32",
         "cumsum_i32", "cumsum_f32", "cumsum_axis1_f32", "matmul_f32", "matmul_f16", "sort_f32", "argsort_f32",
         "searchsorted_f32", "count_nonzero_gt_f32")


def run_case(args):
    """One op at one size, `--steps` timed launches after `--warmup` (for ncu)."""
    import macmetalpy_b200 as cp

    gen = Gen(cp)
    n = args.elements
    c = args.case
    if c.endswith("_i32") and c[:-4] in I32_OPS:
        a, b = gen.integers((n,), -1000, 1000, 3), gen.integers((n,), 1, 50, 4, signed=True)
        o = cp.empty((n,), dtype=np.int32)
        f = getattr(cp, c[:-4])
        fn, nb = (lambda: f(a, b, out=o)), 12 * n
    elif c.endswith("_f32") and c[:-4] in F32_OPS:
        a, b = gen.uniform((n,), -1000, 1000, 1), gen.signed_uniform((n,), 1, 50, 2)
        o = cp.empty((n,), dtype=np.float32)
        f = getattr(cp, c[:-4])
        fn, nb = (lambda: f(a, b, out=o)), 12 * n
    elif c == "bcast_add_f32":
        rows = max(1, n // BC_COLS)
        r, cc = gen.normal((rows, 1), 5), gen.normal((1, BC_COLS), 6)
        o = cp.empty((rows, BC_COLS), dtype=np.float32)
        fn, nb = (lambda: cp.add(r, cc, out=o)), 4 * rows * BC_COLS + 4 * (rows + BC_COLS)
    elif c == "c1_fused_sum":
        x = gen.normal((n,), 11)
        fn, nb = (lambda: cp.sum(cp.sqrt(cp.abs(x)) + cp.exp(-x ** 2))), 4 * n
    elif c in ("sum_f32", "var_f32", "argmax_f32", "nansum_f32", "argmin_f32"):
        x = gen.normal((n,), 21)
        f = {"sum_f32": cp.sum, "var_f32": cp.var, "argmax_f32": cp.argmax, "nansum_f32": cp.nansum,
             "argmin_f32": cp.argmin}[c]
        # arg-reductions keep the index on the device (keepdims) so the timed
        # loop holds the kernels only, not a host read per call
        kw = {"keepdims": True} if c.startswith("arg") else {}
        fn, nb = (lambda: f(x, **kw)), 4 * n
    elif c in ("sum_axis0_f32", "sum_axis1_f32", "var_axis0_f32", "argmax_axis0_f32"):
        side = int(math.isqrt(n))
        x = gen.normal((side, side), 21)
        ax = 1 if c == "sum_axis1_f32" else 0
        f = cp.var if c.startswith("var") else cp.argmax if c.startswith("argmax") else cp.sum
        fn, nb = (lambda: f(x, axis=ax)), 4 * side * side
    elif c == "cumsum_i32":
        x = gen.integers((n,), -100, 101, 31)
        fn, nb = (lambda: cp.cumsum(x)), 12 * n
    elif c == "cumsum_f32":
        x = gen.uniform((n,), 0, 1, 32)
        fn, nb = (lambda: cp.cumsum(x)), 8 * n
    elif c == "cumsum_axis1_f32":
        x = gen.normal((max(1, n // 65536), 65536), 33)
        fn, nb = (lambda: cp.cumsum(x, axis=1)), 8 * x.size
    elif c in ("matmul_f32", "matmul_f16"):
        x = gen.normal((n, n), 41) * np.float32(1 / math.sqrt(n))
        y = gen.normal((n, n), 42) * np.float32(1 / math.sqrt(n))
        if c == "matmul_f16":
            x, y = x.astype(np.float16), y.astype(np.float16)
        x, y = x.copy(), y.copy()
        fn, nb = (lambda: cp.matmul(x, y)), 2 * n ** 3
    elif c in ("sort_f32", "argsort_f32"):
        x = gen.normal((n,), 21)
        f = cp.sort if c == "sort_f32" else cp.argsort
        fn, nb = (lambda: f(x)), n
    elif c == "count_nonzero_gt_f32":
        x = gen.normal((n,), 21)
        fn, nb = (lambda: cp.count_nonzero(x > 0)), 4 * n
    elif c == "searchsorted_f32":
        a = cp.sort(gen.normal((1 << 20,), 22))
        x = gen.normal((n,), 21)
        fn, nb = (lambda: cp.searchsorted(a, x)), n
    else:
        raise SystemExit(f"unknown case {c}; one of {CASES}")
    ms = _time(cp, fn, iters=max(args.steps, 1), warm=max(args.warmup, 1))
    unit = "TFLOP/s" if c.startswith("matmul") else "Gkeys/s" if "sort" in c else "GB/s"
    val = nb / (ms / 1e3) / (1e12 if unit == "TFLOP/s" else 1e9)
    print(json.dumps({"case": c, "elements": n, "ms": round(ms, 4), "value": round(val, 2), "unit": unit}))
    return 0


def _traffic(opname):
    """DRAM bytes per launch from the committed ncu summary, if present."""
    p = os.path.join(REPO, "profiles", "c2_elementwise_ncu.md")
    if not os.path.exists(p):
        return None
    for ln in open(p):
        if ln.startswith(f"| {opname} |"):
            parts = [x.strip() for x in ln.strip().strip("|").split("|")]
            try:
                return int(float(parts[1]))
            except (IndexError, ValueError):
                return None
    return None


def dist_parity(cp):
    """The exchange steps at N ranks, checked against numpy on the whole
    array: every rank builds the same global arrays from one seed (2^22
    elements per rank), holds its row block, runs the distributed op and
    compares the result with numpy's on the global array (int32 sums and
    scans and argmax exact; float32 within 1e-4 of the float64 value;
    matmul within 1e-5 relative Frobenius).  Returns "ok" or the first
    mismatch (identical on every rank: every rank checks the same values)."""
    from macmetalpy_b200 import distributed as D

    W = D.world()
    rng = np.random.default_rng(2024)
    n = W << 22
    x = (rng.standard_normal(n) + 0.25).astype(np.float32)
    x[[5, n - 7]] = x.max() + 1  # a tie across the first and last shard
    xi = rng.integers(-100, 101, n).astype(np.int32)
    X, XI = D.DistArray.from_global(x), D.DistArray.from_global(xi)
    x64 = x.astype(np.float64)
    bad = []

    def rel(got, ref):
        return abs(float(got) - ref) / max(abs(ref), 1e-30)

    if rel(X.sum(), x64.sum()) > 1e-4 * np.abs(x64).sum() / abs(x64.sum()):
        bad.append("sum")
    if rel(X.var(), x64.var()) > 1e-4:
        bad.append("var")
    if X.argmax() != int(np.argmax(x)):
        bad.append("argmax")
    if int(XI.sum()) != int(xi.sum(dtype=np.int64)):
        bad.append("sum_i32")
    if not np.array_equal(XI.cumsum().gather(), np.cumsum(xi, dtype=np.int64)):
        bad.append("cumsum_i32")
    m = x.reshape(-1, 1024)
    M = D.DistArray.from_global(m)
    s0 = M.sum(axis=0).get()
    if np.max(np.abs(s0 - m.astype(np.float64).sum(axis=0))) > 1e-4 * np.abs(m).sum(axis=0).max():
        bad.append("sum_axis0")
    a = (rng.standard_normal((256 * W, 512)) / 20).astype(np.float32)
    b = (rng.standard_normal((512, 384)) / 20).astype(np.float32)
    A = D.DistArray.from_global(a)
    B = cp.array(b) if D.rank() == 0 else cp.zeros(b.shape, dtype=np.float32)
    C = A.matmul(B).gather()
    r = a.astype(np.float64) @ b.astype(np.float64)
    if np.linalg.norm(C - r) / np.linalg.norm(r) > 1e-5:
        bad.append("matmul")
    return "ok" if not bad else "mismatch: " + ",".join(bad)


def dist_suite(cp, gen):
    """Block-distributed ops over all ranks (the exchange steps included),
    weak-scaled: every rank holds the single-GPU C3 / C4 operand, so the
    global array is world x that.  Matmul is strong-scaled: A (16384,16384)
    row-sharded, B broadcast from rank 0; the broadcast alone and the local
    GEMM alone are timed too.  Device time (events on the library stream,
    where the collectives also run) over 10 back-to-back calls after a
    barrier (the ranks' start skew is paid once), max over ranks; values
    count every rank's bytes / FLOPs.  ``parity``: see dist_parity."""
    from macmetalpy_b200 import distributed as D
    from macmetalpy_b200 import linalg_top
    from macmetalpy_b200._cuda_backend import Event

    W, R = D.world(), D.rank()

    def timed(fn, iters=10, warm=2):
        for _ in range(warm):
            fn()
        D.barrier()
        s, e = Event(), Event()
        s.record()
        for _ in range(iters):
            fn()
        e.record()
        D.synchronize()
        ms = s.elapsed_ms(e) / iters
        return D.max_over_ranks(ms)

    out = {"parity": dist_parity(cp), "exchange": "peer" if D._state.get("peer") else "nccl"}
    n = 1 << 28
    x = gen.normal((n,), 21 + 100 * R)
    X = D.DistArray.from_local(x, W * n)
    for name, f in (("sum_f32", X.sum), ("var_f32", X.var), ("argmax_f32", X.argmax)):
        ms = timed(f)
        out[f"dist_{name}"] = {"gbs": round(W * 4 * n / ms / 1e6, 1), "ms": round(ms, 4)}
        if D._state.get("peer"):
            # the same op through the NCCL all-gather + device-merge path
            D._state["peer"] = False
            try:
                ms2 = timed(f)
            finally:
                D._state["peer"] = True
            out[f"dist_{name}"]["nccl_path_gbs"] = round(W * 4 * n / ms2 / 1e6, 1)
    M = D.DistArray.from_local(x.reshape(16384, 16384), W * 16384)
    ms = timed(lambda: M.sum(axis=0))
    out["dist_sum_axis0_f32"] = {"gbs": round(W * 4 * n / ms / 1e6, 1), "ms": round(ms, 4)}
    del X, M, x
    xi = gen.integers((n,), -100, 101, 31 + 100 * R)
    XI = D.DistArray.from_local(xi, W * n)
    ms = timed(lambda: XI.cumsum())
    out["dist_cumsum_i32"] = {"gbs": round(W * 12 * n / ms / 1e6, 1), "ms": round(ms, 4)}
    if D._state.get("peer"):
        # the carry through the NCCL all-gather + device merge, then the scan
        D._state["peer"] = False
        try:
            ms2 = timed(lambda: XI.cumsum())
        finally:
            D._state["peer"] = True
        out["dist_cumsum_i32"]["nccl_path_gbs"] = round(W * 12 * n / ms2 / 1e6, 1)
    del XI, xi
    m = 16384
    s0, e0 = D.row_partition(m, W)[R]
    a = gen.normal((e0 - s0, m), 41 + 100 * R) * np.float32(1 / 128)
    b = gen.normal((m, m), 42) * np.float32(1 / 128)
    A = D.DistArray.from_local(a, m)
    ms = timed(lambda: A.matmul(b), iters=2, warm=1)
    ms_gemm = timed(lambda: linalg_top.matmul(a, b), iters=2, warm=1)
    from macmetalpy_b200 import _cuda_backend as cb

    def bcast():
        cb.check(cb.lib.mmp_broadcast(ctypes.c_void_p(b._ptr), ctypes.c_void_p(b._ptr), 4 * m * m,
                                      cb.dtype_code(np.uint8), 0), "broadcast")

    ms_b = timed(bcast, iters=3, warm=1)
    out["dist_matmul_f32_16384_bcastB"] = {"tflops": round(2 * m ** 3 / ms / 1e9, 2), "ms": round(ms, 3),
                                           "broadcast_B_ms": round(ms_b, 3),
                                           "broadcast_B_gbs": round(4 * m * m / ms_b / 1e6, 1),
                                           "local_gemm_ms": round(ms_gemm, 3)}
    out["world"] = W
    return out


def e2e_c2(cp, d, steps=2, dist=None):
    """Same op set through the public API with host buffers: every step
    uploads its six inputs from pinned host memory and reads its eight
    results back into pinned host memory.  The copies go through
    ``macmetalpy_b200.cuda`` streams (``set(arr, stream=)``,
    ``get(stream=, out=)``): the next step's uploads and this step's
    downloads run on the two copy engines while the kernels run, with inputs
    and outputs double-buffered on the device.  The time runs from an event
    before the first upload to an event after the last download.  With
    several ranks every rank runs it on its own GPU and shard; the time is
    the maximum over ranks and the value counts every rank's bytes."""
    from macmetalpy_b200.cuda import Event, Stream, empty_pinned

    names = ("af", "bf", "ai", "bi", "r", "c")
    host_in = {k: empty_pinned(d[k].shape, d[k].dtype) for k in names}
    for k in names:
        d[k].get(out=host_in[k])
    n = d["af"].size
    out_specs = [((n,), np.float32)] * len(F32_OPS) + [((n,), np.int32)] * len(I32_OPS) + \
                [((BC_ROWS, BC_COLS), np.float32)]
    sets = []
    for _ in range(2):
        dev = {k: cp.empty(d[k].shape, dtype=d[k].dtype) for k in names}
        outs = [cp.empty(shp, dtype=dt) for shp, dt in out_specs]
        ops = []
        for j, nm in enumerate(F32_OPS):
            ops.append(lambda fn=getattr(cp, nm), dev=dev, o=outs[j]: fn(dev["af"], dev["bf"], out=o))
        for j, nm in enumerate(I32_OPS):
            ops.append(lambda fn=getattr(cp, nm), dev=dev, o=outs[len(F32_OPS) + j]:
                       fn(dev["ai"], dev["bi"], out=o))
        ops.append(lambda dev=dev, o=outs[-1]: cp.add(dev["r"], dev["c"], out=o))
        sets.append((dev, outs, ops))
    host_out = [empty_pinned(shp, dt) for shp, dt in out_specs]
    h2d = sum(host_in[k].nbytes for k in names)
    d2h = sum(h.nbytes for h in host_out)
    s_in, s_out = Stream(), Stream()
    ev_comp = [Event(), Event()]
    ev_d2h = [Event(), Event()]

    def one_step(k):
        b = k % 2
        dev, outs, ops = sets[b]
        if k >= 2:
            s_in.wait_event(ev_comp[b])  # the kernels of step k-2 have read input set b
        for kn in names:
            dev[kn].set(host_in[kn], stream=s_in)
        if k >= 2:
            Stream.null.wait_event(ev_d2h[b])  # the results of step k-2 are on the host
        for f, o, h in zip(ops, outs, host_out):
            f()
            o.get(stream=s_out, out=h)
        ev_comp[b].record(None)
        ev_d2h[b].record(s_out)

    one_step(0)
    one_step(1)
    s_in.synchronize()
    s_out.synchronize()
    cp.synchronize()
    world = 1
    if dist is not None:
        dist.barrier()
        world = dist.world()
    t0 = Event().record(None)
    s_in.wait_event(t0)
    s_out.wait_event(t0)
    for k in range(2, 2 + steps):
        one_step(k)
    Stream.null.wait_event(ev_d2h[(1 + steps) % 2])
    t1 = Event().record(None)
    ms = t0.elapsed_time(t1)
    s_in.synchronize()
    s_out.synchronize()
    if dist is not None:
        ms = dist.max_over_ranks(ms)
    del sets, host_in, host_out
    return {"value": round(world * step_bytes() * steps / (ms / 1e3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h), "steps": steps,
            "ms_per_step": round(ms / steps, 2),
            "copies": "pinned host, async on two copy streams, double-buffered (macmetalpy_b200.cuda)"}


def _time(cp, fn, iters=5, warm=2):
    from macmetalpy_b200._cuda_backend import Event

    for _ in range(warm):
        fn()
    cp.synchronize()
    s, e = Event(), Event()
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    return s.elapsed_ms(e) / iters


def _time_median(cp, fn, iters=50, reps=21, warm=20):
    """Median over ``reps`` event-timed batches of ``iters`` back-to-back
    calls (ms per call): for latency-bound calls, where one host hiccup
    would move a single short batch."""
    from macmetalpy_b200._cuda_backend import Event

    for _ in range(warm):
        fn()
    cp.synchronize()
    per = []
    for _ in range(reps):
        s, e = Event(), Event()
        s.record()
        for _ in range(iters):
            fn()
        e.record()
        per.append(s.elapsed_ms(e) / iters)
    per.sort()
    return per[len(per) // 2]


def library_gemm_ceiling():
    """The library GEMM on this box, in this run: torch.matmul (cuBLAS) at
    the C5 shapes, TFLOP/s of 2MNK, CUDA events on torch's stream after
    warm-up.  TF32 (allow_tf32: one TF32 pass, about 1e-3 relative error) is
    the measured ceiling of the tensor pipe in that format, the denominator
    of the 3xTF32 kernel's issued-MMA fraction; FP32 (allow_tf32 off) is the
    library's float32-accurate GEMM; float16 the f16 dense rate.  Inputs are
    made on the device; nothing here is part of the measured product."""
    try:
        import torch
    except Exception as e:  # pragma: no cover
        return {"unavailable": f"torch: {e}"}
    dev = torch.device("cuda", torch.cuda.current_device())

    def rate(a, b, flops, iters):
        for _ in range(2):
            torch.matmul(a, b)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(iters):
            torch.matmul(a, b)
        e.record()
        torch.cuda.synchronize()
        return round(flops / (s.elapsed_time(e) / iters / 1e3) / 1e12, 2)

    out = {"how": "torch.matmul (cuBLAS), CUDA events; tf32 = allow_tf32 on, fp32 = off"}
    old = torch.backends.cuda.matmul.allow_tf32
    try:
        g = torch.Generator(device=dev).manual_seed(0)
        a = torch.randn(16384, 16384, device=dev, generator=g) / 128
        b = torch.randn(16384, 16384, device=dev, generator=g) / 128
        torch.backends.cuda.matmul.allow_tf32 = True
        out["f32_16384_tf32"] = rate(a, b, 2 * 16384 ** 3, 3)
        torch.backends.cuda.matmul.allow_tf32 = False
        out["f32_16384_fp32"] = rate(a, b, 2 * 16384 ** 3, 2)
        del a, b
        a = torch.randn(64, 1024, 1024, device=dev, generator=g) / 32
        b = torch.randn(64, 1024, 1024, device=dev, generator=g) / 32
        torch.backends.cuda.matmul.allow_tf32 = True
        out["f32_batched_tf32"] = rate(a, b, 2 * 64 * 1024 ** 3, 5)
        torch.backends.cuda.matmul.allow_tf32 = False
        out["f32_batched_fp32"] = rate(a, b, 2 * 64 * 1024 ** 3, 3)
        del a, b
        a = (torch.randn(8192, 8192, device=dev, generator=g) / 90.5).half()
        b = (torch.randn(8192, 8192, device=dev, generator=g) / 90.5).half()
        out["f16_8192"] = rate(a, b, 2 * 8192 ** 3, 5)
        del a, b
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old
        torch.cuda.empty_cache()
    return out


def run_suite(cp, gen):
    """Per-config throughput (device time, CUDA events) for C1, C3, C4, C5."""
    hbm = float(_peaks()[0]["hbm_gbs"])
    out = {}

    def gbs(nbytes, ms):
        return {"gbs": round(nbytes / (ms / 1e3) / 1e9, 1), "ms": round(ms, 4),
                "frac": round(nbytes / (ms / 1e3) / 1e9 / hbm, 3)}

    # C1 (2^20, latency-bound) and the same expression at 2^28 (HBM claim)
    for n, tag in ((1 << 20, "c1_2^20"), (1 << 28, "c1_2^28")):
        x = gen.normal((n,), 11)
        y = lambda: cp.sqrt(cp.abs(x)) + cp.exp(-x ** 2)
        # 2^20 is latency-bound: the median of 21 batches of 50 calls
        t = (lambda f: _time_median(cp, f)) if n < (1 << 24) else (lambda f: _time(cp, f, iters=10))
        out[f"{tag}_fused_sum"] = gbs(4 * n, t(lambda: cp.sum(y())))
        out[f"{tag}_fused_mean"] = gbs(4 * n, t(lambda: cp.mean(y())))
        del x
    # C3 reductions on (16384, 16384)
    A = gen.normal((16384, 16384), 21)
    nb = A.nbytes
    for nm, fn in (("sum", cp.sum), ("mean", cp.mean), ("var", cp.var), ("argmax", cp.argmax)):
        # full argmax with keepdims: the index stays on the device like the
        # other full reductions' 0-d results; the plain call returns a Python
        # int (as the reference's does), so each call also waits for its read
        # back -- timed separately as c3_argmax_pyint
        full = (lambda fn=fn: fn(A, keepdims=True)) if nm == "argmax" else (lambda fn=fn: fn(A))
        out[f"c3_{nm}"] = gbs(nb, _time(cp, full))
        for ax in (0, 1):
            out[f"c3_{nm}_axis{ax}"] = gbs(nb, _time(cp, lambda fn=fn, ax=ax: fn(A, axis=ax)))
    out["c3_argmax_pyint"] = gbs(nb, _time(cp, lambda: cp.argmax(A)))
    B = gen.integers((16384, 16384), -100, 101, 22)
    out["c3_int32_sum"] = gbs(nb, _time(cp, lambda: cp.sum(B)))
    del B
    An = A.copy()
    gen_mask = gen.uniform((16384, 16384), 0, 1, 23)
    An[...] = cp.where(gen_mask < 0.01, np.float32(np.nan), An)
    del gen_mask
    out["c3_nansum"] = gbs(nb, _time(cp, lambda: cp.nansum(An)))
    out["c3_nanmean"] = gbs(nb, _time(cp, lambda: cp.nanmean(An)))
    del A, An
    # C4 scans
    n = 1 << 30
    xi = gen.integers((n,), -100, 101, 31)
    out["c4_cumsum_int32_2^30"] = gbs(12 * n, _time(cp, lambda: cp.cumsum(xi), iters=3))
    del xi
    xf = gen.uniform((n,), 0, 1, 32)
    out["c4_cumsum_f32_2^30"] = gbs(8 * n, _time(cp, lambda: cp.cumsum(xf), iters=3))
    del xf
    X2 = gen.normal((4096, 65536), 33)
    out["c4_cumsum_axis1_4096x65536"] = gbs(8 * X2.size, _time(cp, lambda: cp.cumsum(X2, axis=1), iters=3))
    del X2
    # C5 matmul.  float32 runs 3xTF32: three TF32 MMAs per multiply-add, so
    # besides the algorithmic rate (2MNK / t) the issued rate (3 x 2MNK / t)
    # is given against the nominal dense TF32 peak (no measured TF32 figure
    # exists; 1.1 PFLOP/s = half the 2.25 PFLOP/s dense bf16 figure), and
    # float16 against the measured dense bf16 peak (the same tensor rate).
    tf32_nominal = 1100.0
    bf16_meas = float(_peaks()[0].get("bf16_tflops", 0.0)) or None

    lib = library_gemm_ceiling()
    out["c5_library_ceiling"] = lib

    def tflops(flops, ms, tf32=False, f16=False, lib_key=None):
        t = flops / (ms / 1e3) / 1e12
        d = {"tflops": round(t, 2), "ms": round(ms, 3)}
        if tf32:
            d["issued_tflops"] = round(3 * t, 2)
            d["issued_frac_of_tf32_nominal"] = round(3 * t / tf32_nominal, 3)
            ceil = lib.get(lib_key + "_tf32") if lib_key else None
            if ceil:
                d["issued_frac_of_measured_library_tf32"] = round(3 * t / ceil, 3)
            acc = lib.get(lib_key + "_fp32") if lib_key else None
            if acc:
                d["speedup_vs_library_fp32"] = round(t / acc, 2)
        if f16 and bf16_meas:
            d["frac_of_measured_dense"] = round(t / bf16_meas, 3)
        if f16 and lib.get("f16_8192"):
            d["frac_of_library_f16"] = round(t / lib["f16_8192"], 3)
        return d

    Ma = gen.normal((16384, 16384), 41) * np.float32(1 / 128)
    Mb = gen.normal((16384, 16384), 42) * np.float32(1 / 128)
    Ma, Mb = Ma.copy(), Mb.copy()
    out["c5_f32_16384"] = tflops(2 * 16384 ** 3, _time(cp, lambda: cp.matmul(Ma, Mb), iters=2, warm=1), tf32=True,
                                 lib_key="f32_16384")
    del Ma, Mb
    Ba = (gen.normal((64, 1024, 1024), 43) * np.float32(1 / 32)).copy()
    Bb = (gen.normal((64, 1024, 1024), 44) * np.float32(1 / 32)).copy()
    out["c5_f32_batched_64x1024"] = tflops(2 * 64 * 1024 ** 3, _time(cp, lambda: cp.matmul(Ba, Bb), iters=3),
                                           tf32=True, lib_key="f32_batched")
    del Ba, Bb
    Ha = (gen.normal((8192, 8192), 45) * np.float32(1 / 90.5)).astype(np.float16)
    Hb = (gen.normal((8192, 8192), 46) * np.float32(1 / 90.5)).astype(np.float16)
    out["c5_f16_8192"] = tflops(2 * 8192 ** 3, _time(cp, lambda: cp.matmul(Ha, Hb), iters=3), f16=True)
    del Ha, Hb
    # next rows: logic (fused predicate + reduction), nan-ops, sort / searchsorted
    x = gen.normal((1 << 28,), 21)
    y = (x + np.float32(1e-7)).copy()
    # the device forms keep the result on the GPU; allclose / count_nonzero
    # themselves return Python scalars (a read back per call): the *_pyscalar lines
    out["f1_allclose_2^28"] = gbs(8 * x.size, _time(cp, lambda: cp.isclose(x, y).all(), iters=5))
    out["f1_count_nonzero_gt_2^28"] = gbs(4 * x.size, _time(cp, lambda: cp.count_nonzero(x > 0, keepdims=True),
                                                            iters=5))
    out["f1_allclose_2^28_pyscalar"] = gbs(8 * x.size, _time(cp, lambda: cp.allclose(x, y), iters=3))
    out["f1_count_nonzero_gt_2^28_pyscalar"] = gbs(4 * x.size, _time(cp, lambda: cp.count_nonzero(x > 0), iters=3))
    out["f4_nanvar_2^28"] = gbs(4 * x.size, _time(cp, lambda: cp.nanvar(x), iters=3))
    del y
    for n, tag in ((1 << 24, "2^24"), (1 << 28, "2^28")):
        xs = x[:n].copy()
        ms = _time(cp, lambda: cp.sort(xs), iters=3, warm=1)
        out[f"f3_sort_f32_{tag}"] = {"gkeys_s": round(n / ms / 1e6, 3), "ms": round(ms, 3)}
        ms = _time(cp, lambda: cp.argsort(xs), iters=3, warm=1)
        out[f"f3_argsort_f32_{tag}"] = {"gkeys_s": round(n / ms / 1e6, 3), "ms": round(ms, 3)}
        del xs
    srt = cp.sort(x[: 1 << 20].copy())
    q = x[: 1 << 24].copy()
    ms = _time(cp, lambda: cp.searchsorted(srt, q), iters=3)
    out["f3_searchsorted_2^20_x_2^24q"] = {"gq_s": round((1 << 24) / ms / 1e6, 3), "ms": round(ms, 3)}
    return out


if __name__ == "__main__":
    sys.exit(main())
