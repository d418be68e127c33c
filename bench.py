"""Batched GEMM throughput of libgemm_sm100.so on B200 (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload config2|config3|config4|config5a|config5b]
                    [--precision fp32-strict|tf32] [--operand-dtype float32|bfloat16]

One step = one pass of the workload through the library's launchers:
  config2  (default) BASELINE config 2: bf16 A[64,1024,1024] x B[64,1024,1024],
           N(0,1) entries, FP32 accumulation, bf16 output, one launch.  With
           N > 1 ranks (torchrun, one process per GPU) every rank runs its own
           64-batch shard: the batch axis is partitioned, there is no
           data-path collective, scaling is weak.
  config3  BASELINE config 3: float16 A[8192,4096] . X^T (X [4096,4096]
           row-major, so B is a transposed view) with the fused +bias[4096],
           tanh epilogue (cuda_matmul_epilogue_nd_launcher), one launch;
           every rank runs its own copy (weak).
  config4  BASELINE config 4: the float32 MLP GEMM set, batch 4096,
           784->1024->1024->10: per layer the forward product, dA = dC.W^T and
           dW = h^T.dC on transposed views, nine cuda_matmul_launcher calls
           in strict float32 (3xTF32 / few-column kernels); every rank runs its
           own batch (weak, data parallel without the gradient exchange).
  config5a BASELINE config 5a: bf16 [512,2048,2048]^2 split along the batch
           axis over the N ranks (strong scaling, 512/N batches per rank).
  config5b BASELINE config 5b: float64 [8192,8192]^2 split along N over the
           ranks; every step ends with the NCCL all-gather of the column
           blocks and the permute into the row-major result on every rank
           (strong scaling).
value     whole-job TFLOP/s (2*M*N*K per product, summed over the step and all
          ranks / max-over-ranks device time), inputs resident in HBM.
          config2/3/5 inputs (>= 167 MB per step) exceed the 126 MB L2;
          config4's per-GEMM operands are smaller, so its steps flush L2
          (a 256 MB write, timed separately and subtracted).
e2e       the same metric through the public API with pinned HOST buffers:
          config2/5a via phptensors.host_matmul -> pt_host_matmul (H2D of A
          and B, the product, D2H of C, pipelined over batch chunks); config3
          and config4 copy the step's inputs in and its results out on the
          stream around the same launcher calls.
roofline  achieved = algorithmic FLOP per step / mean step time (CUDA events
          on the launching stream) against MEASURED_PEAKS.json: bf16 burst
          for the 16-bit kernels, bf16 / 6 for strict float32 (three TF32
          passes at half the bf16 rate).
cpu_baseline  the reference's HostArray::matmul loop (the C oracle port,
          oracle/liboracle.so) on all host cores, over a bounded row sample.
--impl reference  times only that CPU implementation (rank 0; other ranks exit).
"""
import argparse
import ctypes
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
METRIC = "batched GEMM TFLOP/s (bf16/fp32/fp64) at 1/2/4/8 B200, % of dense TC peak"
FALLBACK_PEAK_TFLOPS = 1590.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--workload", default="config2", choices=sorted(WORKLOADS))
    p.add_argument("--nsplit", default="fused", choices=["fused", "nccl"],
                   help="config5b exchange: fused peer stores, or NCCL all-gather + permute")
    p.add_argument("--precision", default="fp32-strict", choices=["fp32-strict", "tf32"],
                   help="float32 precision mode for config4 (cuda_blas_set_precision)")
    p.add_argument("--operand-dtype", default="float32", choices=["float32", "bfloat16"],
                   help="config4: weights and activations in bfloat16 (forward in bf16, "
                        "float32 gradients from pt_tensor_matmul_backward without cast copies)")
    p.add_argument("--cpu-seconds", type=float, default=8.0,
                   help="target duration of the bounded CPU baseline sample")
    return p.parse_args()


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
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), "measured burst cuBLAS bf16 (MEASURED_PEAKS.json)"
    except (OSError, KeyError, ValueError):
        return FALLBACK_PEAK_TFLOPS, "fallback 1.59 PFLOP/s"


def traffic_for(kernel):
    """DRAM bytes per launch from the committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(kernel)
    except (OSError, ValueError):
        return None


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
           "ms_per_launch": d["ms"] / d["launches"], "traffic": traffic_for(dom),
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
def cpu_sample(w, seconds):
    """Times the oracle port of HostArray::matmul on all host cores over a
    bounded number of output rows of one product of the workload (batch 0;
    config4: its 4096x1024x1024 layer); returns (TFLOP/s, cores, s, text)."""
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
    return tflops, cores, dt, "%d of %d output rows of one %dx%dx%d %s product%s (%.1f s)" % (
        rows, M, M, N, K, dt_name, " with a transposed B" if w.get("b_transposed") else "", dt)


def run_reference(args, w):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    values = []
    detail = None
    for i in range(args.warmup + args.steps):
        per = max(0.5, args.cpu_seconds / max(1, args.steps + args.warmup))
        v, cores, dt, text = cpu_sample(w, per)
        if i >= args.warmup:
            values.append(v)
            detail = (cores, text)
    value = statistics.median(values)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": {"float16": "f16", "float32": "f32"}.get(w.get("dtype"), "bf16"),
        "data": "synthetic N(0,1)",
        "config": {"workload": args.workload, "batches": w["batches"], "M": w["M"],
                   "N": w["N"], "K": w["K"], "parallelism": "none (host CPU)"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": detail[0], "kind": "port",
                         "sample": detail[1]},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU side
def run_nsplit(args, w):
    """config5b: float64 N-split product + all-gather + permute per step."""
    import torch
    import phptensors as P

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    lib = P.library()
    M, N, K = w["M"], w["N"], w["K"]
    lo, hi = P.nsplit_columns(N, rank, world)
    gen = torch.Generator(device="cuda").manual_seed(77)
    a = torch.rand(M, K, device="cuda", generator=gen, dtype=torch.float64) * 2 - 1
    b = torch.rand(K, N, device="cuda", generator=gen, dtype=torch.float64) * 2 - 1
    b_local = b[:, lo:hi].contiguous()
    del b
    comm = P.MgpuComm(rank, world)
    A = P.CudaArray.from_torch(a)
    Bl = P.CudaArray.from_torch(b_local)
    fused = args.nsplit == "fused"
    if fused:
        win = P.MgpuWindow(comm, M, N)
        step = lambda: P.nsplit_matmul_fused(win, A, Bl)
    else:
        ws = torch.empty(M * N * 8, dtype=torch.uint8, device="cuda")
        step = lambda: P.nsplit_matmul(comm, A, Bl, N, ws)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    kernel = P.cuda_get_backend_info()["kernel"]
    barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    with sampler:
        barrier()
        start.record(stream)
        for _ in range(args.steps):
            step()
        stop.record(stream)
        torch.cuda.synchronize()
    ms_local = start.elapsed_time(stop)
    barrier()
    ms = max_over_ranks(ms_local, world, "cuda")
    if lib.gemm_sm100_device_status(local, 1) != 0:
        raise RuntimeError("device status after the timed region")
    flop = 2.0 * M * N * K
    value = flop * args.steps / (ms / 1e3) / 1e12
    if rank == 0:
        peak, peak_src = peaks()
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f64", "data": "synthetic U[-1,1) on device",
            "config": {"workload": "config5b", "M": M, "N": N, "K": K,
                       "parallelism": ("N-split x%d, exchange fused into the GEMM epilogue "
                                       "(peer stores over NVLink)" % world) if fused else
                                      ("N-split x%d + NCCL all-gather + permute" % world),
                       "kernel": kernel,
                       "allgather_bytes_received_per_rank": M * (N - (hi - lo)) * 8},
            "cpu_baseline": None, "e2e": None,
            "gpu_launches": args.steps * (1 if fused else 2),
            "clocks": sampler.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    if fused:
        win.close()
    comm.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def setup_batched(w, batches, rank, torch, P, lib, stream):
    """config2 / config5a: one bf16 batched product per step."""
    M, N, K = w["M"], w["N"], w["K"]
    gen = torch.Generator(device="cuda").manual_seed(1000 + rank)
    a = torch.randn(batches, M, K, device="cuda", generator=gen).to(torch.bfloat16)
    b = torch.randn(batches, K, N, device="cuda", generator=gen).to(torch.bfloat16)
    c = torch.empty(batches, M, N, device="cuda", dtype=torch.bfloat16)
    sa = (ctypes.c_int * 10)(batches, M, K)
    sb = (ctypes.c_int * 10)(batches, K, N)
    sc = (ctypes.c_int * 10)(batches, M, N)
    ta = (ctypes.c_size_t * 10)(M * K, K, 1)
    tb = (ctypes.c_size_t * 10)(K * N, N, 1)
    tc = (ctypes.c_size_t * 10)(M * N, N, 1)
    sptr = ctypes.c_void_p(stream.cuda_stream)
    bf16 = P.DTYPE_CODES["bfloat16"]

    def step():
        ok = lib.cuda_low_precision_matmul_nd_launcher(
            a.data_ptr(), b.data_ptr(), c.data_ptr(), bf16, sa, ta, 3, sb, tb, 3, sc, tc, 3, sptr)
        if not ok:
            raise RuntimeError("launcher failed: %s" % P.cuda_get_backend_info())

    # e2e: pt_host_matmul streams batch chunks so that both PCIe directions
    # and the tensor cores overlap; every step copies A and B in and C out.
    ha, hb = a.cpu().pin_memory(), b.cpu().pin_memory()
    hc = torch.empty(c.shape, dtype=c.dtype).pin_memory()

    def e2e_step():
        P.host_matmul(ha, hb, hc, chunks=8)

    return {
        "step": step, "e2e_step": e2e_step, "flop": 2.0 * batches * M * N * K, "launches": 1,
        "dtype": "bf16", "flush": False, "peak_div": 1.0, "data": "synthetic N(0,1) on device",
        "config": {"batches_per_rank": batches, "M": M, "N": N, "K": K,
                   "l2": "inputs larger than L2 (%.0f MB per step)" %
                         ((a.numel() + b.numel() + c.numel()) * 2 / 1e6)},
        "h2d": (a.numel() + b.numel()) * 2, "d2h": c.numel() * 2,
        "api": "phptensors.host_matmul (pt_host_matmul: pinned host in, host out)",
    }


def setup_config3(w, rank, torch, P, lib, stream):
    """config3: float16 A . X^T with the fused +bias, tanh epilogue."""
    M, N, K = w["M"], w["N"], w["K"]
    gen = torch.Generator(device="cuda").manual_seed(3000 + rank)
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
    sptr = ctypes.c_void_p(stream.cuda_stream)
    f16 = P.DTYPE_CODES["float16"]
    tanh = P.EPILOGUES["tanh"]

    def step():
        ok = lib.cuda_matmul_epilogue_nd_launcher(
            a.data_ptr(), x.data_ptr(), c.data_ptr(), f16, sa, ta, 2, sb, tb, 2, sc, tc, 2,
            ctypes.c_void_p(bias.data_ptr()), tanh, sptr)
        if not ok:
            raise RuntimeError("launcher failed: %s" % P.cuda_get_backend_info())

    ha, hx, hbias = a.cpu().pin_memory(), x.cpu().pin_memory(), bias.cpu().pin_memory()
    hc = torch.empty(c.shape, dtype=c.dtype).pin_memory()

    def e2e_step():
        a.copy_(ha, non_blocking=True)
        x.copy_(hx, non_blocking=True)
        bias.copy_(hbias, non_blocking=True)
        step()
        hc.copy_(c, non_blocking=True)

    return {
        "step": step, "e2e_step": e2e_step, "flop": 2.0 * M * N * K, "launches": 1,
        "dtype": "f16", "flush": False, "peak_div": 1.0,
        "data": "synthetic U[-0.5,0.5) / bias N(0,0.1) on device",
        "config": {"M": M, "N": N, "K": K, "b": "X.transpose() of row-major X[4096,4096]",
                   "epilogue": "+bias[4096], tanh (fused)",
                   "l2": "inputs larger than L2 (%.0f MB per step)" %
                         ((a.numel() + x.numel() + c.numel()) * 2 / 1e6)},
        "h2d": (a.numel() + x.numel() + bias.numel()) * 2, "d2h": c.numel() * 2,
        "api": "cuda_matmul_epilogue_nd_launcher with pinned-host copies on the stream",
    }


def setup_config4_bf16(w, rank, torch, P, lib, stream):
    """config4 with bfloat16 weights and activations: forward products in
    bf16 (cuda_low_precision_matmul_nd_launcher), and per layer one
    pt_tensor_matmul_backward call giving float32 dA and dW from the bf16
    operands and a float32 upstream gradient, without cast copies."""
    dims = w["mlp"]
    batch = w["M"]
    gen = torch.Generator(device="cuda").manual_seed(4100 + rank)
    x = torch.rand(batch, dims[0], device="cuda", generator=gen).bfloat16()
    Ws = [(torch.randn(dims[i], dims[i + 1], device="cuda", generator=gen) / dims[i] ** 0.5)
          .bfloat16() for i in range(3)]
    dCs = [torch.randn(batch, dims[i + 1], device="cuda", generator=gen) for i in range(3)]
    hs = [x] + [torch.empty(batch, dims[i + 1], device="cuda", dtype=torch.bfloat16)
                for i in range(3)]
    dAs = [torch.empty(batch, dims[i], device="cuda") for i in range(3)]
    dWs = [torch.empty(dims[i], dims[i + 1], device="cuda") for i in range(3)]
    bf16 = P.DTYPE_CODES["bfloat16"]
    sptr = ctypes.c_void_p(stream.cuda_stream)
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

    inputs = [x] + Ws + dCs
    outputs = dWs + [hs[3]]
    h_in = [t.cpu().pin_memory() for t in inputs]
    h_out = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in outputs]

    def e2e_step():
        for d, h in zip(inputs, h_in):
            d.copy_(h, non_blocking=True)
        step()
        for h, d in zip(h_out, outputs):
            h.copy_(d, non_blocking=True)

    return {
        "step": step, "e2e_step": e2e_step, "flop": flop, "launches": 9,
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


def setup_config4(w, rank, torch, P, lib, stream):
    """config4: the float32 MLP GEMM set (forward, dA, dW per layer)."""
    dims = w["mlp"]
    batch = w["M"]
    gen = torch.Generator(device="cuda").manual_seed(4000 + rank)
    x = torch.rand(batch, dims[0], device="cuda", generator=gen)
    Ws = [torch.randn(dims[i], dims[i + 1], device="cuda", generator=gen) / dims[i] ** 0.5
          for i in range(3)]
    dCs = [torch.randn(batch, dims[i + 1], device="cuda", generator=gen) for i in range(3)]
    hs = [x] + [torch.empty(batch, dims[i + 1], device="cuda") for i in range(3)]
    dAs = [torch.empty(batch, dims[i], device="cuda") for i in range(3)]
    dWs = [torch.empty(dims[i], dims[i + 1], device="cuda") for i in range(3)]
    sptr = ctypes.c_void_p(stream.cuda_stream)
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

    def launch(call):
        (a, b, c, m, n, k, a0, a1, b0, b1, c0, c1) = call
        if not lib.cuda_matmul_launcher(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k,
                                        a0, a1, b0, b1, c0, c1, sptr):
            raise RuntimeError("launcher failed: %s" % P.cuda_get_backend_info())

    def step():
        for call in calls:
            launch(call)

    def profile_step():
        """One step with CUDA events around every launch (outside the timed
        region: events between launches stop their programmatic overlap)."""
        out = []
        for call in calls:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            launch(call)
            e1.record(stream)
            out.append((P.cuda_get_backend_info()["kernel"], 2.0 * call[3] * call[4] * call[5], e0, e1))
        return out

    inputs = [x] + Ws + dCs
    outputs = dWs + [hs[3]]
    h_in = [t.cpu().pin_memory() for t in inputs]
    h_out = [torch.empty(t.shape).pin_memory() for t in outputs]

    def e2e_step():
        for d, h in zip(inputs, h_in):
            d.copy_(h, non_blocking=True)
        step()
        for h, d in zip(h_out, outputs):
            h.copy_(d, non_blocking=True)

    return {
        "step": step, "e2e_step": e2e_step, "profile_step": profile_step, "flop": flop,
        "launches": len(calls), "dtype": "f32", "flush": True, "peak_div": 6.0,
        "data": "synthetic x U[0,1), W N(0,1/fan_in), dC N(0,1) on device",
        "config": {"batch": batch, "layers": "784->1024->1024->10",
                   "gemms_per_step": len(calls), "precision": "fp32-strict",
                   "l2": "L2 flushed before every step (256 MB write, outside the timing)"},
        "h2d": sum(t.numel() for t in inputs) * 4, "d2h": sum(t.numel() for t in outputs) * 4,
        "api": "cuda_matmul_launcher x9 with pinned-host copies on the stream",
    }


def run_ours(args, w):
    import torch
    import phptensors as P

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    lib = P.library()
    stream = torch.cuda.current_stream()
    if args.workload == "config3":
        wl = setup_config3(w, rank, torch, P, lib, stream)
    elif args.workload == "config4" and args.operand_dtype == "bfloat16":
        wl = setup_config4_bf16(w, rank, torch, P, lib, stream)
    elif args.workload == "config4":
        P.cuda_set_matmul_precision(args.precision)
        wl = setup_config4(w, rank, torch, P, lib, stream)
        wl["config"]["precision"] = args.precision
        if args.precision == "tf32":
            wl["peak_div"] = 2.0
    else:
        wl = setup_batched(w, shard(w, rank, world), rank, torch, P, lib, stream)
    step = wl["step"]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda") if wl["flush"] else None

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    kernel = P.cuda_get_backend_info()["kernel"]
    barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    with sampler:
        barrier()
        if flush is None:
            start.record(stream)
            for _ in range(args.steps):
                step()
            stop.record(stream)
            torch.cuda.synchronize()
            ms_local = start.elapsed_time(stop)
        else:
            # time each step alone, after an untimed write larger than L2
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(args.steps)]
            for e0, e1 in evs:
                flush.add_(1)
                e0.record(stream)
                step()
                e1.record(stream)
            torch.cuda.synchronize()
            ms_local = sum(e0.elapsed_time(e1) for e0, e1 in evs)
    barrier()
    ms = max_over_ranks(ms_local, world, "cuda")
    status = lib.gemm_sm100_device_status(local, 1)
    if status != 0:
        raise RuntimeError("device status %d after the timed region" % status)
    flop_rank = wl["flop"]
    value = flop_rank * world * args.steps / (ms / 1e3) / 1e12
    achieved = flop_rank / (ms_local / args.steps / 1e3) / 1e12

    e2e_steps = max(3, min(args.steps, 20))
    for _ in range(min(args.warmup, 3)):
        wl["e2e_step"]()
    barrier()
    start.record(stream)
    for _ in range(e2e_steps):
        wl["e2e_step"]()
    stop.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(start.elapsed_time(stop), world, "cuda")
    e2e_value = flop_rank * world * e2e_steps / (e2e_ms / 1e3) / 1e12

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
        for name, fl, e0, e1 in recs:
            d = per_kernel.setdefault(name, {"launches": 0, "ms": 0.0, "flop": 0.0})
            d["launches"] += 1
            d["ms"] += e0.elapsed_time(e1)
            d["flop"] += fl

    cpu = None
    if rank == 0 and world == 1:
        v, cores, dt, text = cpu_sample(w, args.cpu_seconds)
        cpu = {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": text}

    if rank == 0:
        peak, peak_src = peaks()
        if wl["peak_div"] != 1.0:
            peak /= wl["peak_div"]
            peak_src += " / %g (%s)" % (wl["peak_div"], "TF32 runs at half the bf16 rate"
                                         if wl["peak_div"] == 2.0 else
                                         "strict float32: three TF32 passes at half the bf16 rate")
        cfg = {"workload": args.workload}
        cfg.update(wl["config"])
        if args.workload in ("config2", "config5a"):
            cfg["global_batches"] = wl["config"]["batches_per_rank"] * world
        cfg["parallelism"] = ("batch-sharded x%d (no collective)" % world if w["split"] else
                              "replicated per rank x%d (no collective)" % world)
        cfg["kernel"] = kernel
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True,
            "scaling": "strong" if w["split"] else "weak",
            "vs_baseline": None, "dtype": wl["dtype"], "data": wl["data"],
            "config": cfg,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "peak_source": peak_src,
                         "traffic": traffic_for(kernel) if wl["launches"] == 1 else None,
                         "algorithmic_flop_per_step": flop_rank},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": wl["h2d"], "d2h_bytes_per_step": wl["d2h"],
                    "api": wl["api"]},
            "gpu_launches": args.steps * wl["launches"],
            "clocks": sampler.summary(),
        }
        if per_kernel:
            line["roofline"] = kernel_roofline(per_kernel, peaks(), achieved, peak)
            line["config"]["kernels"] = {k: v["launches"] // prof_steps
                                         for k, v in per_kernel.items()}
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    w = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, w)
    elif w.get("nsplit"):
        run_nsplit(args, w)
    else:
        run_ours(args, w)


if __name__ == "__main__":
    main()
