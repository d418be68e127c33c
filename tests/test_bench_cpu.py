"""bench.py's host-side helpers (no GPU): the per-kernel roofline of
multi-launch steps and the pass-count divisors it uses."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_kernel_divisor_by_pass_count():
    assert bench.kernel_divisor("tc2-3xtf32-256x256") == 6.0
    assert bench.kernel_divisor("tc-3xtf32-128x128") == 6.0
    assert bench.kernel_divisor("tc2-tf32-256x256") == 2.0
    assert bench.kernel_divisor("tc-tf32-128x256") == 2.0
    assert bench.kernel_divisor("tc2-f32xbf16-bf16x3-256x256") == 3.0
    assert bench.kernel_divisor("tc2-bf16-256x256") == 1.0
    assert bench.kernel_divisor("tc2-3xtf32-tmem-256x256") == 6.0
    assert bench.kernel_divisor("tc2-bf16-256x512") == 1.0
    assert bench.kernel_divisor("tc2-f16-256x512") == 1.0
    assert bench.kernel_divisor("skinny-f32") is None


def test_traffic_entries_for_the_bench_kernels():
    """Every kernel the default bench runs on its workloads has a committed
    DRAM traffic figure (the roofline's traffic field)."""
    for workload, kernel in (("config5a", "tc2-bf16-256x512"), ("config2", "tc2-bf16-256x512"),
                             ("config3", "tc2-f16-256x512"),
                             ("config4", "tc2-3xtf32-tmem-256x256"),
                             ("config5b", "dmma-f64-128x128")):
        t = bench.traffic_for(workload, kernel)
        assert isinstance(t, int) and t > 0, (workload, kernel)
    assert bench.kernel_divisor("simt-f32") is None


def test_kernel_roofline_picks_the_largest_share():
    per = {
        "tc2-3xtf32-256x256": {"launches": 8, "ms": 0.5, "flop": 8 * 8.6e9},
        "tc-3xtf32-128x128": {"launches": 4, "ms": 0.3, "flop": 4 * 8.6e9},
        "skinny-f32": {"launches": 4, "ms": 0.05, "flop": 4 * 8.4e7},
    }
    r = bench.kernel_roofline(per, (1635.7, "measured"), 100.0, 272.6)
    assert r["kernel"] == "tc2-3xtf32-256x256"
    assert abs(r["achieved"] - 8 * 8.6e9 / 0.5e-3 / 1e12) < 1e-9
    assert abs(r["peak"] - 1635.7 / 6) < 1e-9
    assert abs(r["frac"] - r["achieved"] / r["peak"]) < 1e-12
    assert abs(r["share"] - 0.5 / 0.85) < 1e-12
    assert r["launches"] == 8 and r["bound"] == "tensor"
    assert r["step"] == {"achieved": 100.0, "peak": 272.6, "frac": 100.0 / 272.6}
    assert list(r["per_kernel"]) == ["tc2-3xtf32-256x256", "tc-3xtf32-128x128", "skinny-f32"]


def test_kernel_roofline_cuda_core_kernel_has_no_tensor_peak():
    per = {"simt-f32": {"launches": 2, "ms": 0.2, "flop": 2e6}}
    r = bench.kernel_roofline(per, (1635.7, "measured"), 1.0, 272.6)
    assert r["bound"] == "issue" and "peak" not in r and "frac" not in r


def test_default_run_is_config5a_with_the_other_configs_as_blocks():
    args = bench.parse([])
    assert args.workload == "config5a"
    assert args.blocks == ["config2", "config3", "config4", "config5b"]
    assert bench.parse(["--workload", "config2"]).blocks == []
    assert bench.parse(["--blocks", "none"]).blocks == []
    assert bench.parse(["--workload", "config2", "--blocks", "config2,config4"]).blocks == \
        ["config4"]


def test_traffic_is_looked_up_per_workload_and_kernel():
    assert bench.traffic_for("config2", "tc2-bf16-256x256") > 0
    assert bench.traffic_for("config2", "no-such-kernel") is None
    assert bench.traffic_for("no-such-workload", "tc2-bf16-256x256") is None
