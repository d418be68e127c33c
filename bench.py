"""Batched GEMM throughput of libgemm_sm100.so on B200 (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload config5a|config2|config3|config4|config5b]
                    [--blocks config2,config3,config4,config5b|none]
                    [--precision fp32-strict|tf32] [--operand-dtype float32|bfloat16]

One step = one pass of a workload through the library's launchers:
  config5a (default, the headline) BASELINE config 5a: bf16
           A[512,2048,2048] x B[512,2048,2048], N(0,1), FP32 accumulation,
           bf16 output, the batch axis split over the N ranks (512/N batches
           each, one launch per step; strong scaling, no data-path
           collective).  It is the "large batched BF16 GEMM" of the 70 %
           target and the configuration the 1/2/4/8-GPU metric is quoted on.
  config2  BASELINE config 2: bf16 A[64,1024,1024] x B[64,1024,1024]; every
           rank runs its own 64-batch product (weak scaling).
  config3  BASELINE config 3: float16 A[8192,4096] . X^T (X [4096,4096]
           row-major, so B is a transposed view) with the fused +bias[4096],
           tanh epilogue (cuda_matmul_epilogue_nd_launcher); one per rank (weak).
  config4  BASELINE config 4: the float32 MLP GEMM set, batch 4096,
           784->1024->1024->10: per layer the forward product
           (cuda_matmul_launcher) and the autograd node's dA = dC.W^T and
           dW = h^T.dC on transposed views (pt_tensor_matmul_backward, dW on a
           forked side stream), nine products in strict float32 (3xTF32 /
           few-column kernels); one per rank (weak).
  config5b BASELINE config 5b: float64 [8192,8192]^2 split along N over the
           ranks.  Timed three ways: the fused N-split (the column block's
           epilogue stores into every rank's result over NVLink), the NCCL
           all-gather + permute, and the local column-block product alone
           (so exchange cost = exchange path - compute).  Strong scaling.
The JSON line is the headline workload; the others ride along under
"blocks" (by default with config5a: config2, config3, config4, config5b).

value     whole-job TFLOP/s (2*M*N*K per product, summed over the step and all
          ranks / max-over-ranks device time), inputs resident in HBM.
          config2/3/5 inputs (>= 167 MB per step) exceed the 126 MB L2;
          config4's per-GEMM operands are smaller, so every config4 step is
          timed alone after a 256 MB write that flushes L2.
e2e       the headline metric through the public API with pinned HOST buffers:
          config2/5a via phptensors.host_matmul -> pt_host_matmul (H2D of A
          and B, the product, D2H of C, pipelined over batch chunks); config3
          and config4 copy the step's inputs in and results out on the stream.
roofline  achieved = algorithmic FLOP per launch / mean launch time (CUDA events
          on the launching stream) against MEASURED_PEAKS.json: bf16 burst
          for the 16-bit kernels, bf16 / 6 for strict float32 (three TF32
          passes at half the bf16 rate); float64 against the nominal DMMA peak.
checks    after the timed region every block compares sampled rows of its
          result with an independent float64 product (torch on the same
          device) and, for config5b, across ranks bit for bit; any mismatch
          on any rank makes every rank exit non-zero without a bench line.
cpu_baseline  the reference's HostArray::matmul loop (the C oracle port,
          oracle/liboracle.so) over a bounded row sample, on all host cores
          and on one core (the reference's loop is single-threaded).
--impl reference  times only that CPU implementation (rank 0; other ranks exit).
"""
import argparse
import ctypes
import datetime
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "php-gpu-tensors_b200")
sys.path.insert(0, PKG)

WORKLOADS = {
    "config2": {"batches": 64, "M": 1024, "N": 1024, "K": 1024, "split": False},
    "config3": {"batches": 1, "M": 8192, "N": 4096, "K": 4096, "split": False,
                "dtype": "float16", "b_transposed": True},
    "config4": {"batches": 1, "M": 4096, "N": 1024, "K": 1024, "split": False,
                "dtype": "float32", "mlp": [784, 1024, 1024, 10]},
    "config5a": {"batches": 512, "M": 2048, "N": 2048, "K": 2048, "split": True},
    "config5b": {"batches": 1, "M": 8192, "N": 8192, "K": 8192, "split": True, "nsplit": True,
                 "dtype": "float64"},
}
HEADLINE = "config5a"
DEFAULT_BLOCKS = ["config2", "config3", "config4", "config5b"]
METRIC = "batched GEMM TFLOP/s (bf16/fp32/fp64) at 1/2/4/8 B200, % of dense TC peak"
FALLBACK_PEAK_TFLOPS = 1590.0
FALLBACK_SUSTAINED_TFLOPS = 1400.0
# No FP64 figure is measured on this pool; B200's nominal dense FP64 tensor
# (DMMA) rate is the denominator of the float64 roofline.
NOMINAL_FP64_TFLOPS = 40.0
# normwise tolerances of the self-checks (BASELINE's parity bounds)
CHECK_TOL = {"bf16": 1e-2, "f16": 1e-2, "f32": 1e-5, "f64": 1e-12}


def parse(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=30)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--workload", default=HEADLINE, choices=sorted(WORKLOADS))
    p.add_argument("--blocks", default=None,
                   help="comma-separated extra workloads measured after the headline, or "
                        "'none' (default: %s with config5a, none otherwise)"
                        % ",".join(DEFAULT_BLOCKS))
    p.add_argument("--batches", type=int, default=None,
                   help="override the batch count of config2/config5a (profiling a "
                        "smaller case of the same kernel)")
    p.add_argument("--nsplit", default="fused", choices=["fused", "nccl"],
                   help="config5b as the headline: the exchange path it reports")
    p.add_argument("--precision", default="fp32-strict", choices=["fp32-strict", "tf32"],
                   help="float32 precision mode for config4 (cuda_blas_set_precision)")
    p.add_argument("--operand-dtype", default="float32", choices=["float32", "bfloat16"],
                   help="config4: weights and activations in bfloat16 (forward in bf16, "
                        "float32 gradients from pt_tensor_matmul_backward without cast copies)")
    p.add_argument("--e2e-steps", type=int, default=5)
    p.add_argument("--cpu-seconds", type=float, default=8.0,
                   help="target duration of the bounded all-core CPU baseline sample "
                        "(the one-core sample takes half of it)")
    args = p.parse_args(argv)
    if args.blocks is None:
        args.blocks = list(DEFAULT_BLOCKS) if args.workload == HEADLINE else []
    elif args.blocks.strip() in ("", "none"):
        args.blocks = []
    else:
        args.blocks = [b.strip() for b in args.blocks.split(",") if b.strip()]
        for b in args.blocks:
            if b not in WORKLOADS:
                p.error("unknown block %r" % b)
    args.blocks = [b for b in args.blocks if b != args.workload]
    return args


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def shard(w, rank, world):
    """Batches this rank computes: the batch axis is partitioned for the
    strong-scaling workloads, replicated per rank for config2 (weak)."""
    if not w["split"] or w.get("nsplit"):
        return w["batches"]
    base, extra = divmod(w["batches"], world)
    return base + (1 if rank < extra else 0)


def max_over_ranks(x, world, device=None):
    """Max of a host float over all ranks (the bench's timing rule)."""
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def peaks():
    """(burst, sustained, source) bf16 TFLOP/s."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return (float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained") or 0.0) or None,
                "measured burst cuBLAS bf16 (MEASURED_PEAKS.json)")
    except (OSError, KeyError, ValueError):
        return FALLBACK_PEAK_TFLOPS, FALLBACK_SUSTAINED_TFLOPS, "fallback 1.59 PFLOP/s"


def traffic_for(workload, kernel):
    """DRAM bytes per launch from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            d = json.load(f)
    except (OSError, ValueError):
        return None
    v = d.get(workload, {})
    return v.get(kernel) if isinstance(v, dict) else None


def kernel_divisor(name):
    """Tensor-rate divisor of a kernel against the measured bf16 peak: three
    TF32 passes (strict float32) 6, one TF32 pass 2, three bf16 passes 3,
    16-bit 1; None for the CUDA-core kernels."""
    if "3xtf32" in name:
        return 6.0
    if "tf32" in name:
        return 2.0
    if "bf16x3" in name:
        return 3.0
    if name.startswith("tc"):
        return 1.0
    return None


def kernel_roofline(per_kernel, peak_info, step_achieved, step_peak):
    """Roofline of the kernel with the largest share of a multi-launch step:
    its algorithmic FLOP over its own CUDA-event time; the whole step's
    figures ride along under "step"."""
    dom = max(per_kernel, key=lambda k: per_kernel[k]["ms"])
    d = per_kernel[dom]
    total_ms = sum(v["ms"] for v in per_kernel.values())
    achieved = d["flop"] / (d["ms"] / 1e3) / 1e12
    div = kernel_divisor(dom)
    peak, src = peak_info
    out = {"bound": "tensor" if div else "issue", "kernel": dom, "achieved": achieved,
           "unit": "TFLOP/s", "share": d["ms"] / total_ms, "launches": d["launches"],
           "ms_per_launch": d["ms"] / d["launches"],
           "step": {"achieved": step_achieved, "peak": step_peak,
                    "frac": step_achieved / step_peak}}
    if div:
        out["peak"] = peak / div
        out["frac"] = achieved / out["peak"]
        out["peak_source"] = "%s / %g" % (src, div)
    out["per_kernel"] = {k: {"launches": v["launches"], "ms": v["ms"],
                             "tflops": v["flop"] / (v["ms"] / 1e3) / 1e12}
                         for k, v in sorted(per_kernel.items(), key=lambda kv: -kv[1]["ms"])}
    return out


def normwise_err(got, ref):
    """max|got - ref| / max(1, max|ref|) of two float64 tensors."""
    return float((got - ref).abs().max() / max(1.0, float(ref.abs().max())))


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Polls NVML (read-only) for SM clock and throttle reasons while running."""

    REASONS = {
        0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
        0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting",
        0x1: "gpu_idle", 0x10: "sync_boost", 0x100: "display_clocks_setting",
    }

    def __init__(self, device):
        self.device = device
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.nv:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


# ------------------------------------------------------------------ CPU side
def cpu_sample(w, seconds, cores=None):
    """Times the oracle port of HostArray::matmul over a bounded number of
    output rows of one product of the workload (batch 0; config4: its
    4096x1024x1024 layer) on `cores` threads (default: all host cores);
    returns (TFLOP/s, cores, s, text)."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib as O
    M, N, K = w["M"], w["N"], w["K"]
    dt_name = {"float16": "float16", "float32": "float32"}.get(w.get("dtype"), "bfloat16")
    if w.get("dtype") == "float64":
        dt_name = "float32"   # the reference has no float64 host matmul
    rng = np.random.default_rng(0)
    a = O.to_storage(rng.standard_normal(M * K).astype(np.float32), dt_name)
    b = O.to_storage(rng.standard_normal(K * N).astype(np.float32), dt_name)
    A = (a, [M, K], [K, 1], 0)
    B = (b, [K, N], [1, K], 0) if w.get("b_transposed") else (b, [K, N], [N, 1], 0)
    if cores is None:
        cores = O.oracle().orc_host_threads()
    t0 = time.perf_counter()
    rows = max(1, cores)
    O.host_matmul_range(A, B, dt_name, 0, rows * N, cores)
    dt = time.perf_counter() - t0
    rows = int(min(M, max(rows, rows * seconds / max(dt, 1e-6))))
    t0 = time.perf_counter()
    O.host_matmul_range(A, B, dt_name, 0, rows * N, cores)
    dt = time.perf_counter() - t0
    tflops = 2.0 * rows * N * K / dt / 1e12
    return tflops, cores, dt, "%d of %d output rows of one %dx%dx%d %s product%s on %d thread%s (%.1f s)" % (
        rows, M, M, N, K, dt_name, " with a transposed B" if w.get("b_transposed") else "",
        cores, "" if cores == 1 else "s", dt)


def cpu_baseline(w, seconds):
    """All-core and one-core timings of the oracle port (one line)."""
    v, cores, _, text = cpu_sample(w, seconds)
    v1, _, _, text1 = cpu_sample(w, seconds / 2, cores=1)
    return {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": text,
            "value_1core": v1, "sample_1core": text1}


def run_reference(args, w):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    values, values1 = [], []
    detail = None
    per = max(0.5, args.cpu_seconds / max(1, args.steps + args.warmup))
    for i in range(args.warmup + args.steps):
        v, cores, dt, text = cpu_sample(w, per)
        if i >= args.warmup:
            values.append(v)
            detail = (cores, text)
    # the reference's loop itself is single-threaded: one bounded sample of it
    v1, _, _, text1 = cpu_sample(w, max(1.0, args.cpu_seconds / 4), cores=1)
    value = statistics.median(values)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "strong" if w["split"] else "weak",
        "vs_baseline": None,
        "dtype": {"float16": "f16", "float32": "f32", "float64": "f64"}.get(w.get("dtype"), "bf16"),
        "data": "synthetic N(0,1)",
        "config": {"workload": args.workload, "batches": w["batches"], "M": w["M"],
                   "N": w["N"], "K": w["K"], "parallelism": "none (host CPU)"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": detail[0], "kind": "port",
                         "sample": detail[1], "value_1core": v1, "sample_1core": text1},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU side
class Ctx:
    """Per-process GPU context: rank, device, library, stream, collectives."""

    def __init__(self, args):
        import torch
        import phptensors as P
        self.torch, self.P = torch, P
        self.args = args
        self.rank, self.world, self.local = dist_env()
        torch.cuda.set_device(self.local)
        self.dist = None
        if self.world > 1:
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", self.local))
            self.dist = dist
        torch.backends.cuda.matmul.allow_tf32 = False
        self.lib = P.library()
        self.stream = torch.cuda.current_stream()
        self.sptr = ctypes.c_void_p(self.stream.cuda_stream)
        self.checks = {}
        self.failures = []

    def barrier(self):
        if self.dist:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def max(self, x):
        return max_over_ranks(x, self.world, "cuda")

    def check(self, name, err, tol, extra=None):
        ok = err <= tol
        rec = {"max_normwise_err": err, "tol": tol, "ok": ok}
        if extra:
            rec.update(extra)
        worst = self.max(err / tol) if self.world > 1 else err / tol
        rec["ok_all_ranks"] = worst <= 1.0
        self.checks[name] = rec
        if worst > 1.0:
            self.failures.append(name)

    def time_region(self, step, steps, flush=None):
        """Device time (ms) of `steps` calls of step(): CUDA events on the
        launching stream, barrier + synchronize on both sides; with `flush`
        every step is timed alone after an untimed write larger than L2.
        Returns (local ms, max-over-ranks ms, clock summary)."""
        torch = self.torch
        self.barrier()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        sampler = ClockSampler(self.local)
        with sampler:
            self.barrier()
            if flush is None:
                start.record(self.stream)
                for _ in range(steps):
                    step()
                stop.record(self.stream)
                torch.cuda.synchronize()
                ms_local = start.elapsed_time(stop)
            else:
                evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                       for _ in range(steps)]
                for e0, e1 in evs:
                    flush.add_(1)
                    e0.record(self.stream)
                    step()
                    e1.record(self.stream)
                torch.cuda.synchronize()
                ms_local = sum(e0.elapsed_time(e1) for e0, e1 in evs)
        self.barrier()
        return ms_local, self.max(ms_local), sampler.summary()

    def device_status(self):
        status = self.lib.gemm_sm100_device_status(self.local, 1)
        if status != 0:
            raise RuntimeError("device status %d after the timed region" % status)


def setup_batched(ctx, w, batches, name):
    """config2 / config5a: one bf16 batched product per step."""
    torch, P, lib = ctx.torch, ctx.P, ctx.lib
    M, N, K = w["M"], w["N"], w["K"]
    gen = torch.Generator(device="cuda").manual_seed(1000 + ctx.rank)
    a = torch.randn(batches, M, K, device="cuda", generator=gen).to(torch.bfloat16)
    b = torch.randn(batches, K, N, device="cuda", generator=gen).to(torch.bfloat16)
    c = torch.empty(batches, M, N, device="cuda", dtype=torch.bfloat16)
    sa = (ctypes.c_int * 10)(batches, M, K)
    sb = (ctypes.c_int * 10)(batches, K, N)
    sc = (ctypes.c_int * 10)(batches, M, N)
    ta = (ctypes.c_size_t * 10)(M * K, K, 1)
    tb = (ctypes.c_size_t * 10)(K * N, N, 1)
    tc = (ctypes.c_size_t * 10)(M * N, N, 1)
    bf16 = P.DTYPE_CODES["bfloat16"]
    sptr = ctx.sptr

    def step():
        ok = lib.cuda_low_precision_matmul_nd_launcher(
            a.data_ptr(), b.data_ptr(), c.data_ptr(), bf16, sa, ta, 3, sb, tb, 3, sc, tc, 3, sptr)
        if not ok:
            raise RuntimeError("launcher failed: %s" % P.cuda_get_backend_info())

    def check():
        # sampled batches and rows against a float64 product on the device
        errs = []
        for bi in sorted({0, batches // 2, batches - 1}):
            rows = [0, M // 2 + 1, M - 1]
            ref = a[bi, rows].double() @ b[bi].double()
            errs.append(normwise_err(c[bi, rows].double(), ref))
        return max(errs)

    state = {}

    def e2e_setup():
        # e2e: pt_host_matmul streams batch chunks so that both PCIe
        # directions and the tensor cores overlap; every step copies A and B
        # in and C out.
        state["ha"], state["hb"] = a.cpu().pin_memory(), b.cpu().pin_memory()
        state["hc"] = torch.empty(c.shape, dtype=c.dtype).pin_memory()

    def e2e_step():
        P.host_matmul(state["ha"], state["hb"], state["hc"], chunks=8)

    return {
        "step": step, "check": check, "e2e_setup": e2e_setup, "e2e_step": e2e_step,
        "flop": 2.0 * batches * M * N * K, "launches": 1, "dtype": "bf16", "flush": False,
        "peak_div": 1.0, "data": "synthetic N(0,1) on device",
        "config": {"batches_per_rank": batches, "M": M, "N": N, "K": K,
                   "l2": "inputs larger than L2 (%.0f MB per step)" %
                         ((a.numel() + b.numel() + c.numel()) * 2 / 1e6)},
        "h2d": (a.numel() + b.numel()) * 2, "d2h": c.numel() * 2,
        "api": "phptensors.host_matmul (pt_host_matmul: pinned host in, host out)",
    }


def setup_config3(ctx, w):
    """config3: float16 A . X^T with the fused +bias, tanh epilogue."""
    torch, P, lib = ctx.torch, ctx.P, ctx.lib
    M, N, K = w["M"], w["N"], w["K"]
    gen = torch.Generator(device="cuda").manual_seed(3000 + ctx.rank)
    a = (torch.rand(M, K, device="cuda", generator=gen) - 0.5).half()
    x = (torch.rand(N, K, device="cuda", generator=gen) - 0.5).half()
    bias = (torch.randn(N, device="cuda", generator=gen) * 0.1).half()
    c = torch.empty(M, N, device="cuda", dtype=torch.float16)
    sa = (ctypes.c_int * 10)(M, K)
    sb = (ctypes.c_int * 10)(K, N)
    sc = (ctypes.c_int * 10)(M, N)
    ta = (ctypes.c_size_t * 10)(K, 1)
    tb = (ctypes.c_size_t * 10)(1, K)      # X.transpose(): a strided view
    tc = (ctypes.c_size_t * 10)(N, 1)
    f16 = P.DTYPE_CODES["float16"]
    tanh = P.EPILOGUES["tanh"]
    sptr = ctx.sptr

    def step():
        ok = lib.cuda_matmul_epilogue_nd_launcher(
            a.data_ptr(), x.data_ptr(), c.data_ptr(), f16, sa, ta, 2, sb, tb, 2, sc, tc, 2,
            ctypes.c_void_p(bias.data_ptr()), tanh, sptr)
        if not ok:
            raise RuntimeError("launcher failed: %s" % P.cuda_get_backend_info())

    def check():
        # the unfused plan's arithmetic: product rounded to fp16, + bias, tanh
        rows = [0, M // 2 + 1, M - 1]
        prod = (a[rows].double() @ x.double().t()).half()
        ref = torch.tanh(prod.double() + bias.double())
        return normwise_err(c[rows].double(), ref)

    state = {}

    def e2e_setup():
        state["h"] = (a.cpu().pin_memory(), x.cpu().pin_memory(), bias.cpu().pin_memory())
        state["hc"] = torch.empty(c.shape, dtype=c.dtype).pin_memory()

    def e2e_step():
        ha, hx, hbias = state["h"]
        a.copy_(ha, non_blocking=True)
        x.copy_(hx, non_blocking=True)
        bias.copy_(hbias, non_blocking=True)
        step()
        state["hc"].copy_(c, non_blocking=True)

    return {
        "step": step, "check": check, "e2e_setup": e2e_setup, "e2e_step": e2e_step,
        "flop": 2.0 * M * N * K, "launches": 1, "dtype": "f16", "flush": False, "peak_div": 1.0,
        "data": "synthetic U[-0.5,0.5) / bias N(0,0.1) on device",
        "config": {"M": M, "N": N, "K": K, "b": "X.transpose() of row-major X[4096,4096]",
                   "epilogue": "+bias[4096], tanh (fused)",
                   "l2": "inputs larger than L2 (%.0f MB per step)" %
                         ((a.numel() + x.numel() + c.numel()) * 2 / 1e6)},
        "h2d": (a.numel() + x.numel() + bias.numel()) * 2, "d2h": c.numel() * 2,
        "api": "cuda_matmul_epilogue_nd_launcher with pinned-host copies on the stream",
    }


def setup_config4_bf16(ctx, w):
    """config4 with bfloat16 weights and activations: forward products in
    bf16 (cuda_low_precision_matmul_nd_launcher), and per layer one
    pt_tensor_matmul_backward call giving float32 dA and dW from the bf16
    operands and a float32 upstream gradient, without cast copies."""
    torch, P, lib = ctx.torch, ctx.P, ctx.lib
    dims = w["mlp"]
    batch = w["M"]
    gen = torch.Generator(device="cuda").manual_seed(4100 + ctx.rank)
    x = torch.rand(batch, dims[0], device="cuda", generator=gen).bfloat16()
    Ws = [(torch.randn(dims[i], dims[i + 1], device="cuda", generator=gen) / dims[i] ** 0.5)
          .bfloat16() for i in range(3)]
    dCs = [torch.randn(batch, dims[i + 1], device="cuda", generator=gen) for i in range(3)]
    hs = [x] + [torch.empty(batch, dims[i + 1], device="cuda", dtype=torch.bfloat16)
                for i in range(3)]
    dAs = [torch.empty(batch, dims[i], device="cuda") for i in range(3)]
    dWs = [torch.empty(dims[i], dims[i + 1], device="cuda") for i in range(3)]
    bf16 = P.DTYPE_CODES["bfloat16"]
    sptr = ctx.sptr
    fwd = []
    for l in range(3):
        fi, fo = dims[l], dims[l + 1]
        fwd.append((hs[l], Ws[l], hs[l + 1], (ctypes.c_int * 10)(batch, fi),
                    (ctypes.c_size_t * 10)(fi, 1), (ctypes.c_int * 10)(fi, fo),
                    (ctypes.c_size_t * 10)(fo, 1), (ctypes.c_int * 10)(batch, fo),
                    (ctypes.c_size_t * 10)(fo, 1)))
    wrap = [P.CudaArray.from_torch(t) for t in hs + Ws + dCs + dAs + dWs]
    pts = [t._pt() for t in wrap]
    H, W, DC, DA, DW = pts[0:4], pts[4:7], pts[7:10], pts[10:13], pts[13:16]
    flop = sum(6.0 * batch * dims[l] * dims[l + 1] for l in range(3))

    def step():
        for (a, b, c, sa, ta, sb, tb, sc, tc) in fwd:
            if not lib.cuda_low_precision_matmul_nd_launcher(
                    a.data_ptr(), b.data_ptr(), c.data_ptr(), bf16, sa, ta, 2, sb, tb, 2, sc, tc,
                    2, sptr):
                raise RuntimeError("launcher failed: %s" % P.cuda_get_backend_info())
        for l in range(3):
            rc = lib.pt_tensor_matmul_backward(ctypes.byref(H[l]), ctypes.byref(W[l]),
                                               ctypes.byref(DC[l]), ctypes.byref(DA[l]),
                                               ctypes.byref(DW[l]), sptr)
            if rc != P.PT_OK:
                raise RuntimeError(lib.pt_last_error())

    def check():
        # layer 1's float32 gradients against float64 products of the bf16 operands
        ref_da = dCs[1][:64].double() @ Ws[1].double().t()
        ref_dw = hs[1][:, :64].double().t() @ dCs[1].double()
        return max(normwise_err(dAs[1][:64].double(), ref_da),
                   normwise_err(dWs[1][:64].double(), ref_dw))

    inputs = [x] + Ws + dCs
    outputs = dWs + [hs[3]]
    state = {}

    def e2e_setup():
        state["in"] = [t.cpu().pin_memory() for t in inputs]
        state["out"] = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in outputs]

    def e2e_step():
        for d, h in zip(inputs, state["in"]):
            d.copy_(h, non_blocking=True)
        step()
        for h, d in zip(state["out"], outputs):
            h.copy_(d, non_blocking=True)

    return {
        "step": step, "check": check, "check_dtype": "f32", "e2e_setup": e2e_setup,
        "e2e_step": e2e_step, "flop": flop, "launches": 9,
        "dtype": "bf16 (float32 gradients)", "flush": True, "peak_div": 1.0,
        "data": "synthetic x U[0,1), W N(0,1/fan_in) in bf16, dC N(0,1) float32 on device",
        "config": {"batch": batch, "layers": "784->1024->1024->10", "gemms_per_step": 9,
                   "operands": "bfloat16 (forward bf16; dA, dW float32 via "
                               "pt_tensor_matmul_backward, no cast copies)",
                   "l2": "L2 flushed before every step (256 MB write, outside the timing)"},
        "h2d": sum(t.numel() * t.element_size() for t in inputs),
        "d2h": sum(t.numel() * t.element_size() for t in outputs),
        "api": "cuda_low_precision_matmul_nd_launcher x3 + pt_tensor_matmul_backward x3 "
               "with pinned-host copies on the stream",
    }


def setup_config4(ctx, w):
    """config4: the float32 MLP GEMM set: per layer the forward product
    through cuda_matmul_launcher (CudaArray::matmul's 2-D float32 entry) and
    the backward node's two products through pt_tensor_matmul_backward (the
    autograd matmul node, src/autograd.c:1539-1585: dA = dC.W^T on the
    caller's stream, dW = h^T.dC on a side stream forked from and joined back
    into it)."""
    torch, P, lib = ctx.torch, ctx.P, ctx.lib
    dims = w["mlp"]
    batch = w["M"]
    gen = torch.Generator(device="cuda").manual_seed(4000 + ctx.rank)
    x = torch.rand(batch, dims[0], device="cuda", generator=gen)
    Ws = [torch.randn(dims[i], dims[i + 1], device="cuda", generator=gen) / dims[i] ** 0.5
          for i in range(3)]
    dCs = [torch.randn(batch, dims[i + 1], device="cuda", generator=gen) for i in range(3)]
    hs = [x] + [torch.empty(batch, dims[i + 1], device="cuda") for i in range(3)]
    dAs = [torch.empty(batch, dims[i], device="cuda") for i in range(3)]
    dWs = [torch.empty(dims[i], dims[i + 1], device="cuda") for i in range(3)]
    sptr = ctx.sptr
    calls = []
    for l in range(3):
        fi, fo = dims[l], dims[l + 1]
        # forward h[l+1] = h[l] . W[l]
        calls.append((hs[l], Ws[l], hs[l + 1], batch, fi, fo, fi, 1, fo, 1, fo, 1))
    for l in range(3):
        fi, fo = dims[l], dims[l + 1]
        # dA = dC . W^T (W^T: strides (1, fo)); dW = h^T . dC (h^T: strides (1, fi))
        calls.append((dCs[l], Ws[l], dAs[l], batch, fo, fi, fo, 1, 1, fo, fi, 1))
        calls.append((hs[l], dCs[l], dWs[l], fi, batch, fo, 1, fi, fo, 1, fo, 1))
    flop = sum(2.0 * c[3] * c[4] * c[5] for c in calls)
    wrap = [P.CudaArray.from_torch(t) for t in hs + Ws + dCs + dAs + dWs]
    pts = [t._pt() for t in wrap]
    H, W, DC, DA, DW = pts[0:4], pts[4:7], pts[7:10], pts[10:13], pts[13:16]

    def launch(call):
        (a, b, c, m, n, k, a0, a1, b0, b1, c0, c1) = call
        if not lib.cuda_matmul_launcher(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k,
                                        a0, a1, b0, b1, c0, c1, sptr):
            raise RuntimeError("launcher failed: %s" % P.cuda_get_backend_info())

    def step():
        for call in calls[:3]:
            launch(call)
        for l in range(3):
            rc = lib.pt_tensor_matmul_backward(ctypes.byref(H[l]), ctypes.byref(W[l]),
                                               ctypes.byref(DC[l]), ctypes.byref(DA[l]),
                                               ctypes.byref(DW[l]), sptr)
            if rc != P.PT_OK:
                raise RuntimeError(lib.pt_last_error())

    def profile_step():
        """The step's nine products one by one on the caller's stream, with
        CUDA events around every launch (outside the timed region: events
        between launches stop their programmatic overlap, and the backward
        node's side stream is not used), to attribute time to kernels."""
        out = []
        for call in calls:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(ctx.stream)
            launch(call)
            e1.record(ctx.stream)
            out.append((P.cuda_get_backend_info()["kernel"], 2.0 * call[3] * call[4] * call[5],
                        e0, e1))
        return out

    def check():
        # one product of each kind against float64 on the same operands:
        # forward layer 1, dA of layer 1 (W^T view), dW of layers 1 and 2
        # (h^T view; layer 2 on the few-column kernel)
        errs = [normwise_err(hs[2][:64].double(), hs[1][:64].double() @ Ws[1].double()),
                normwise_err(dAs[1][:64].double(), dCs[1][:64].double() @ Ws[1].double().t()),
                normwise_err(dWs[1][:64].double(),
                             hs[1][:, :64].double().t() @ dCs[1].double()),
                normwise_err(dWs[2][:64].double(),
                             hs[2][:, :64].double().t() @ dCs[2].double())]
        return max(errs)

    inputs = [x] + Ws + dCs
    outputs = dWs + [hs[3]]
    state = {}

    def e2e_setup():
        state["in"] = [t.cpu().pin_memory() for t in inputs]
        state["out"] = [torch.empty(t.shape).pin_memory() for t in outputs]

    def e2e_step():
        for d, h in zip(inputs, state["in"]):
            d.copy_(h, non_blocking=True)
        step()
        for h, d in zip(state["out"], outputs):
            h.copy_(d, non_blocking=True)

    return {
        "step": step, "check": check, "e2e_setup": e2e_setup, "e2e_step": e2e_step,
        "profile_step": profile_step, "flop": flop, "launches": len(calls), "dtype": "f32",
        "flush": True, "peak_div": 6.0,
        "data": "synthetic x U[0,1), W N(0,1/fan_in), dC N(0,1) on device",
        "config": {"batch": batch, "layers": "784->1024->1024->10",
                   "gemms_per_step": len(calls), "precision": "fp32-strict",
                   "calls": "forward: cuda_matmul_launcher; backward: pt_tensor_matmul_backward "
                            "(dW on a forked side stream)",
                   "l2": "L2 flushed before every step (256 MB write, outside the timing)"},
        "h2d": sum(t.numel() for t in inputs) * 4, "d2h": sum(t.numel() for t in outputs) * 4,
        "api": "cuda_matmul_launcher x3 + pt_tensor_matmul_backward x3 with pinned-host "
               "copies on the stream",
    }


def setup_workload(ctx, name, args):
    w = WORKLOADS[name]
    P = ctx.P
    if name == "config3":
        return setup_config3(ctx, w)
    if name == "config4" and args.operand_dtype == "bfloat16":
        return setup_config4_bf16(ctx, w)
    if name == "config4":
        P.cuda_set_matmul_precision(args.precision)
        wl = setup_config4(ctx, w)
        wl["config"]["precision"] = args.precision
        if args.precision == "tf32":
            wl["peak_div"] = 2.0
        return wl
    batches = shard(w, ctx.rank, ctx.world)
    if args.batches is not None:
        batches = args.batches if not w["split"] else max(1, args.batches // ctx.world)
    return setup_batched(ctx, w, batches, name)


def measure_workload(ctx, name, args, with_e2e):
    """Runs one single-GPU-kernel workload: warm-up, timed region, check,
    optional e2e and per-kernel profile.  Returns a block dict (every rank)."""
    torch, P = ctx.torch, ctx.P
    w = WORKLOADS[name]
    wl = setup_workload(ctx, name, args)
    step = wl["step"]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda") if wl["flush"] else None
    for _ in range(args.warmup):
        step()
    kernel = P.cuda_get_backend_info()["kernel"]
    ms_local, ms, clocks = ctx.time_region(step, args.steps, flush)
    ctx.device_status()
    flop_rank = wl["flop"]
    value = flop_rank * ctx.world * args.steps / (ms / 1e3) / 1e12
    achieved = flop_rank / (ms_local / args.steps / 1e3) / 1e12
    ctx.check(name, wl["check"](), CHECK_TOL[wl.get("check_dtype", wl["dtype"])],
              {"what": "sampled rows vs a float64 product on the device"})

    e2e = None
    if with_e2e:
        wl["e2e_setup"]()
        e2e_steps = max(3, args.e2e_steps)
        for _ in range(min(args.warmup, 2)):
            wl["e2e_step"]()
        ctx.barrier()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(ctx.stream)
        for _ in range(e2e_steps):
            wl["e2e_step"]()
        stop.record(ctx.stream)
        torch.cuda.synchronize()
        e2e_ms = ctx.max(start.elapsed_time(stop))
        e2e = {"value": flop_rank * ctx.world * e2e_steps / (e2e_ms / 1e3) / 1e12,
               "unit": "TFLOP/s", "h2d_bytes_per_step": wl["h2d"] * ctx.world,
               "d2h_bytes_per_step": wl["d2h"] * ctx.world,
               "h2d_bytes_per_rank": wl["h2d"], "d2h_bytes_per_rank": wl["d2h"],
               "steps": e2e_steps, "api": wl["api"]}

    # Multi-launch steps: every launch timed on its own (CUDA events on the
    # launching stream, L2 flushed before each step as in the timed region);
    # the kernel with the largest share is the one the roofline describes.
    per_kernel, prof_steps = None, 0
    if "profile_step" in wl:
        recs = []
        prof_steps = max(3, min(args.steps, 10))
        for _ in range(prof_steps):
            if flush is not None:
                flush.add_(1)
            recs.extend(wl["profile_step"]())
        torch.cuda.synchronize()
        per_kernel = {}
        for kname, fl, e0, e1 in recs:
            d = per_kernel.setdefault(kname, {"launches": 0, "ms": 0.0, "flop": 0.0})
            d["launches"] += 1
            d["ms"] += e0.elapsed_time(e1)
            d["flop"] += fl

    burst, sustained, src = peaks()
    peak, peak_src = burst, src
    if wl["peak_div"] != 1.0:
        peak /= wl["peak_div"]
        peak_src += " / %g (%s)" % (wl["peak_div"], "TF32 runs at half the bf16 rate"
                                     if wl["peak_div"] == 2.0 else
                                     "strict float32: three TF32 passes at half the bf16 rate")
    cfg = {"workload": name}
    cfg.update(wl["config"])
    if name in ("config2", "config5a"):
        if w["split"]:
            cfg["global_batches"] = w["batches"] if args.batches is None else args.batches
        else:
            cfg["global_batches"] = wl["config"]["batches_per_rank"] * ctx.world
    cfg["parallelism"] = ("batch-sharded x%d (no collective)" % ctx.world if w["split"] else
                          "replicated per rank x%d (no collective)" % ctx.world)
    cfg["kernel"] = kernel
    roof = {"bound": "tensor", "kernel": kernel, "achieved": achieved, "peak": peak,
            "unit": "TFLOP/s", "frac": achieved / peak, "peak_source": peak_src,
            "traffic": traffic_for(name, kernel) if wl["launches"] == 1 else None,
            "algorithmic_flop_per_launch": flop_rank / wl["launches"]}
    if sustained and wl["peak_div"] == 1.0:
        roof["peak_sustained"] = sustained
        roof["frac_of_sustained"] = achieved / sustained
    if per_kernel:
        roof = kernel_roofline(per_kernel, (burst, src), achieved, peak)
        roof["traffic"] = traffic_for(name, roof["kernel"])
        cfg["kernels"] = {k: v["launches"] // prof_steps for k, v in per_kernel.items()}
    return {
        "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": ctx.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "strong" if w["split"] else "weak",
        "vs_baseline": None, "dtype": wl["dtype"], "data": wl["data"], "config": cfg,
        "roofline": roof, "e2e": e2e, "gpu_launches": args.steps * wl["launches"],
        "clocks": clocks, "check": ctx.checks.get(name),
    }


def measure_nsplit(ctx, args):
    """config5b: the float64 N-split product three ways (fused exchange, NCCL
    all-gather + permute, local column block alone).  Returns a block dict."""
    torch, P, lib = ctx.torch, ctx.P, ctx.lib
    w = WORKLOADS["config5b"]
    M, N, K = w["M"], w["N"], w["K"]
    rank, world = ctx.rank, ctx.world
    lo, hi = P.nsplit_columns(N, rank, world)
    gen = torch.Generator(device="cuda").manual_seed(77)   # the same A, B on every rank
    a = torch.rand(M, K, device="cuda", generator=gen, dtype=torch.float64) * 2 - 1
    b = torch.rand(K, N, device="cuda", generator=gen, dtype=torch.float64) * 2 - 1
    rows = [0, 4097, M - 1]
    ref_rows = a[rows] @ b            # the checker: cuBLAS float64 on the same device
    b_local = b[:, lo:hi].contiguous()
    del b
    comm = P.MgpuComm(rank, world)
    A = P.CudaArray.from_torch(a)
    Bl = P.CudaArray.from_torch(b_local)
    win = P.MgpuWindow(comm, M, N)
    ws = torch.empty(M * N * 8, dtype=torch.uint8, device="cuda")
    c_local = torch.empty(M, hi - lo, device="cuda", dtype=torch.float64)
    sa = (ctypes.c_int * 10)(M, K)
    sb = (ctypes.c_int * 10)(K, hi - lo)
    sc = (ctypes.c_int * 10)(M, hi - lo)
    ta = (ctypes.c_size_t * 10)(K, 1)
    tb = (ctypes.c_size_t * 10)(hi - lo, 1)
    tc = (ctypes.c_size_t * 10)(hi - lo, 1)
    out = {}

    def compute_only():
        if not lib.cuda_f64_matmul_nd_launcher(a.data_ptr(), b_local.data_ptr(),
                                               c_local.data_ptr(), sa, ta, 2, sb, tb, 2, sc, tc,
                                               2, ctx.sptr):
            raise RuntimeError("launcher failed: %s" % P.cuda_get_backend_info())

    results = {}

    def fused(mode):
        def run():
            win.set_exchange(mode)
            results["fused_" + mode] = P.nsplit_matmul_fused(win, A, Bl)
        return run

    # the fused entry point's two exchanges (auto: epilogue stores), NCCL,
    # and the compute alone
    variants = [("store", fused("store")), ("overlap", fused("overlap")),
                ("nccl", lambda: results.__setitem__("nccl", P.nsplit_matmul(comm, A, Bl, N, ws))),
                ("compute", compute_only)]
    flop = 2.0 * M * N * K
    kernel = None
    compute_kernel = None
    auto = "store"
    for vname, fn in variants:
        for _ in range(args.warmup):
            fn()
        if vname == auto:
            kernel = P.cuda_get_backend_info()["kernel"]
        elif vname == "compute":
            compute_kernel = P.cuda_get_backend_info()["kernel"]
        ms_local, ms, clocks = ctx.time_region(fn, args.steps)
        ctx.device_status()
        if vname in ("store", "overlap"):
            # both write the same window: keep this exchange's result
            results["fused_" + vname] = results["fused_" + vname].clone()
        out[vname] = {"value": flop * args.steps / (ms / 1e3) / 1e12,
                      "ms_per_step": ms / args.steps, "clocks": clocks}
    win.set_exchange("auto")
    for vname in ("fused_store", "fused_overlap", "nccl"):
        c = results[vname]
        c = c if isinstance(c, torch.Tensor) else c.to_torch()
        got = c[rows]
        err = normwise_err(got, ref_rows)
        same = True
        if world > 1:
            gathered = [torch.empty_like(got) for _ in range(world)]
            ctx.dist.all_gather(gathered, got.contiguous())
            same = all(torch.equal(gathered[0], g) for g in gathered)
        ctx.check("config5b_" + vname, err if same else float("inf"), CHECK_TOL["f64"],
                  {"what": "sampled rows vs cuBLAS float64; identical on every rank",
                   "identical_across_ranks": same})
    for k in ("store", "overlap", "nccl"):
        out[k]["exchange_ms_per_step"] = out[k]["ms_per_step"] - out["compute"]["ms_per_step"]
    out["fused"] = dict(out[auto], exchange=auto)
    head = out[args.nsplit] if args.workload == "config5b" else out["fused"]
    ctx.barrier()
    win.close()
    comm.close()
    achieved_c = flop / world / (out["compute"]["ms_per_step"] / 1e3) / 1e12
    return {
        "metric": METRIC, "value": head["value"], "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic U[-1,1) on device",
        "config": {"workload": "config5b", "M": M, "N": N, "K": K, "kernel": kernel,
                   "parallelism": "N-split x%d: fused = column-block epilogue stores into every "
                                  "rank's result over NVLink; nccl = all-gather + permute" % world,
                   "allgather_bytes_received_per_rank": M * (N - (hi - lo)) * 8,
                   "l2": "inputs larger than L2 (%.0f MB)" % ((M * K + K * N + M * N) * 8 / 1e6)},
        "paths": out,
        "roofline": {"bound": "tensor (DMMA)", "kernel": compute_kernel, "achieved": achieved_c,
                     "peak": NOMINAL_FP64_TFLOPS, "unit": "TFLOP/s",
                     "frac": achieved_c / NOMINAL_FP64_TFLOPS,
                     "peak_source": "nominal B200 dense FP64 tensor rate (no measured FP64 peak)",
                     "of": "the local column-block product (compute path)",
                     "traffic": traffic_for("config5b%s" % ("" if world == 1 else "_x%d" % world),
                                            compute_kernel)},
        "gpu_launches": args.steps * (1 if args.nsplit == "fused" else 2),
        "exchange": "fused = %s (gemm_mgpu_window_set_exchange AUTO: epilogue stores)" % auto,
        "clocks": head["clocks"],
        "check": {k: v for k, v in ctx.checks.items() if k.startswith("config5b")},
    }


def run_ours(args):
    ctx = Ctx(args)
    if args.workload == "config5b":
        line = measure_nsplit(ctx, args)
    else:
        line = measure_workload(ctx, args.workload, args, with_e2e=True)
    blocks = {}
    for b in args.blocks:
        if b == "config5b":
            blk = measure_nsplit(ctx, args)
        else:
            blk = measure_workload(ctx, b, args, with_e2e=False)
        blocks[b] = {k: blk[k] for k in ("value", "unit", "ms_per_step", "scaling", "dtype",
                                         "config", "roofline", "gpu_launches", "clocks",
                                         "check", "paths") if k in blk}
        ctx.torch.cuda.empty_cache()
    if ctx.rank == 0 and ctx.world == 1:
        line["cpu_baseline"] = cpu_baseline(WORKLOADS[args.workload], args.cpu_seconds)
    else:
        line["cpu_baseline"] = None
    if blocks:
        line["blocks"] = blocks
    line["checks"] = ctx.checks
    failed = bool(ctx.failures)
    if ctx.rank == 0:
        if failed:
            print("self-check failed: %s" % json.dumps(ctx.checks), file=sys.stderr, flush=True)
        else:
            print(json.dumps(line), flush=True)
    if ctx.dist:
        ctx.dist.barrier()
        ctx.dist.destroy_process_group()
    if failed:
        sys.exit(1)


def main():
    args = parse()
    w = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, w)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
