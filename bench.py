"""Batched GEMM throughput of libgemm_sm100.so on B200 (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload config2|config5a|config5b]

One step = one batched product of the workload, one launch of the
library's kernel:
  config2  (default) BASELINE config 2: bf16 A[64,1024,1024] x B[64,1024,1024],
           N(0,1) entries, FP32 accumulation, bf16 output.  With N > 1 ranks
           (torchrun, one process per GPU) every rank runs its own 64-batch
           shard: the batch axis is partitioned, there is no data-path
           collective, scaling is weak.
  config5a BASELINE config 5a: bf16 [512,2048,2048]^2 split along the batch
           axis over the N ranks (strong scaling, 512/N batches per rank).
  config5b BASELINE config 5b: float64 [8192,8192]^2 split along N over the
           ranks; every step ends with the NCCL all-gather of the column
           blocks and the permute into the row-major result on every rank
           (strong scaling).
value     whole-job TFLOP/s (2*M*N*K*batches over all ranks / max-over-ranks
          device time), inputs resident in HBM; inputs (>= 384 MB per step)
          exceed the 126 MB L2, so no flush is needed between steps.
e2e       the same metric through the public API (phptensors.host_matmul ->
          pt_host_matmul) with pinned HOST buffers: H2D of A and B, the
          product, D2H of C in the timed region every step, pipelined over
          batch chunks.
roofline  achieved = algorithmic FLOP per launch / mean launch time (CUDA
          events on the launching stream) against MEASURED_PEAKS.json.
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
    bounded number of output rows of batch 0; returns (TFLOP/s, cores, text)."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib as O
    M, N, K = w["M"], w["N"], w["K"]
    rng = np.random.default_rng(0)
    a = O.to_storage(rng.standard_normal(M * K).astype(np.float32), "bfloat16")
    b = O.to_storage(rng.standard_normal(K * N).astype(np.float32), "bfloat16")
    A = (a, [M, K], [K, 1], 0)
    B = (b, [K, N], [N, 1], 0)
    cores = O.oracle().orc_host_threads()
    t0 = time.perf_counter()
    rows = max(1, cores)
    O.host_matmul_range(A, B, "bfloat16", 0, rows * N, cores)
    dt = time.perf_counter() - t0
    rows = int(min(M, max(rows, rows * seconds / max(dt, 1e-6))))
    t0 = time.perf_counter()
    O.host_matmul_range(A, B, "bfloat16", 0, rows * N, cores)
    dt = time.perf_counter() - t0
    tflops = 2.0 * rows * N * K / dt / 1e12
    return tflops, cores, dt, "%d of %d output rows of one %dx%dx%d bf16 batch (%.1f s)" % (
        rows, M, M, N, K, dt)


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
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
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
    batches, M, N, K = shard(w, rank, world), w["M"], w["N"], w["K"]
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
    stream = torch.cuda.current_stream()
    sptr = ctypes.c_void_p(stream.cuda_stream)
    bf16 = P.DTYPE_CODES["bfloat16"]

    def step():
        ok = lib.cuda_low_precision_matmul_nd_launcher(
            a.data_ptr(), b.data_ptr(), c.data_ptr(), bf16, sa, ta, 3, sb, tb, 3, sc, tc, 3, sptr)
        if not ok:
            raise RuntimeError("launcher failed: %s" % P.cuda_get_backend_info())

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
    status = lib.gemm_sm100_device_status(local, 1)
    if status != 0:
        raise RuntimeError("device status %d after the timed region" % status)
    flop_rank = 2.0 * batches * M * N * K
    total_flop = flop_rank * world * args.steps
    value = total_flop / (ms / 1e3) / 1e12
    launch_ms = ms_local / args.steps
    achieved = flop_rank / (launch_ms / 1e3) / 1e12

    # e2e through the public API with pinned host buffers: pt_host_matmul
    # streams batch chunks so that both PCIe directions and the tensor cores
    # overlap; every step copies A and B in and C out.
    ha = a.cpu().pin_memory()
    hb = b.cpu().pin_memory()
    hc = torch.empty(c.shape, dtype=c.dtype).pin_memory()

    def e2e_step():
        P.host_matmul(ha, hb, hc, chunks=8)

    e2e_steps = max(3, min(args.steps, 20))
    for _ in range(min(args.warmup, 3)):
        e2e_step()
    barrier()
    start.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    stop.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(start.elapsed_time(stop), world, "cuda")
    e2e_value = flop_rank * world * e2e_steps / (e2e_ms / 1e3) / 1e12

    cpu = None
    if rank == 0 and world == 1:
        v, cores, dt, text = cpu_sample(w, args.cpu_seconds)
        cpu = {"value": v, "unit": "TFLOP/s", "cores": cores, "kind": "port", "sample": text}

    if rank == 0:
        peak, peak_src = peaks()
        clocks = sampler.summary()
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True,
            "scaling": "strong" if w["split"] else "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic N(0,1) on device",
            "config": {"workload": args.workload, "batches_per_rank": batches, "M": M, "N": N,
                       "K": K, "global_batches": batches * world,
                       "parallelism": "batch-sharded x%d (no collective)" % world,
                       "l2": "inputs larger than L2 (%.0f MB per step)" %
                             ((a.numel() + b.numel() + c.numel()) * 2 / 1e6),
                       "kernel": kernel},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "peak_source": peak_src,
                         "traffic": traffic_for(kernel),
                         "algorithmic_flop_per_launch": flop_rank},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "TFLOP/s",
                    "h2d_bytes_per_step": (a.numel() + b.numel()) * 2,
                    "d2h_bytes_per_step": c.numel() * 2,
                    "api": "phptensors.host_matmul (pt_host_matmul: pinned host in, host out)"},
            "gpu_launches": args.steps,
            "clocks": clocks,
        }
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
