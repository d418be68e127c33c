"""Multi-GPU paths (one process per GPU).

CPU (gloo, world size 2, no GPU calls): batch sharding and N-split column
ranges tile the work exactly once, the library's N-split workspace size is
consistent across ranks, and the bench's max-over-ranks timing rule.

GPU: the N-split entry points (NCCL all-gather + permute, and the fused
kernel whose epilogue stores into every rank's window) with one rank equal
the plain product bit for bit; with two ranks every rank receives the full
product, again bit-identical to the single-GPU product.
"""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, out):
    import torch.distributed as dist
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "php-gpu-tensors_b200"))
    import bench
    import phptensors as P
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        res = {}
        for name, w in bench.WORKLOADS.items():
            res[name] = bench.shard(w, rank, world)
        res["cols"] = P.nsplit_columns(8192, rank, world)
        res["ws"] = P.library().gemm_mgpu_nsplit_workspace_bytes(world, 1, 8192, 8192)
        res["max"] = bench.max_over_ranks(float(rank + 1) * 1.5, world, "cpu")
        gathered = [None] * world
        dist.all_gather_object(gathered, res)
        if rank == 0:
            out.put(gathered)
    finally:
        dist.destroy_process_group()


def test_sharding_and_timing_plumbing_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # config2 is weak scaling (each rank a full 64-batch shard); config5a
    # partitions 512 batches exactly once
    assert [r["config2"] for r in res] == [64, 64]
    assert sum(r["config5a"] for r in res) == 512
    # N-split column blocks tile [0, N)
    cols = sorted(r["cols"] for r in res)
    assert cols[0][0] == 0 and cols[-1][1] == 8192 and cols[0][1] == cols[1][0]
    assert {r["ws"] for r in res} == {8192 * 8192 * 8}
    assert all(r["max"] == 3.0 for r in res)


@pytest.mark.gpu
def test_fused_nsplit_single_rank_equals_plain_product():
    sys.path.insert(0, os.path.join(ROOT, "php-gpu-tensors_b200"))
    import phptensors as P
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(5)
    M, N, K = 1000, 640, 776
    a = torch.rand(M, K, device="cuda", generator=g, dtype=torch.float64) - 0.5
    b = torch.rand(K, N, device="cuda", generator=g, dtype=torch.float64) - 0.5
    comm = P.MgpuComm(0, 1)
    win = P.MgpuWindow(comm, M, N)
    try:
        for _ in range(2):
            c = P.nsplit_matmul_fused(win, P.CudaArray.from_torch(a), P.CudaArray.from_torch(b))
            ref = P.CudaArray.from_torch(a).matmul(P.CudaArray.from_torch(b), allow_float64=True)
            torch.cuda.synchronize()
            assert torch.equal(c, ref.to_torch())
    finally:
        win.close()
        comm.close()


@pytest.mark.gpu
def test_nsplit_single_rank_equals_plain_product():
    sys.path.insert(0, os.path.join(ROOT, "php-gpu-tensors_b200"))
    import phptensors as P
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(3)
    for dt, tdt in (("float64", torch.float64), ("bfloat16", torch.bfloat16)):
        a = (torch.rand(1024, 768, device="cuda", generator=g, dtype=torch.float64) - 0.5).to(tdt)
        b = (torch.rand(768, 512, device="cuda", generator=g, dtype=torch.float64) - 0.5).to(tdt)
        comm = P.MgpuComm(0, 1)
        try:
            c = P.nsplit_matmul(comm, P.CudaArray.from_torch(a), P.CudaArray.from_torch(b), 512)
            ref = P.CudaArray.from_torch(a).matmul(P.CudaArray.from_torch(b), allow_float64=True)
            assert torch.equal(c.to_torch(), ref.to_torch()), dt
        finally:
            comm.close()


def _nccl_worker(rank, world, port, q):
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(ROOT, "php-gpu-tensors_b200"))
    import phptensors as P
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    comm = None
    try:
        M, N, K = 1024, 2048, 1536
        g = torch.Generator(device="cuda").manual_seed(11)
        a = torch.rand(M, K, device="cuda", generator=g, dtype=torch.float64) - 0.5
        b = torch.rand(K, N, device="cuda", generator=g, dtype=torch.float64) - 0.5
        lo, hi = P.nsplit_columns(N, rank, world)
        comm = P.MgpuComm(rank, world)
        bl = P.CudaArray.from_torch(b[:, lo:hi].contiguous())
        c = P.nsplit_matmul(comm, P.CudaArray.from_torch(a), bl, N)
        full = P.CudaArray.from_torch(a).matmul(P.CudaArray.from_torch(b), allow_float64=True)
        win = P.MgpuWindow(comm, M, N)
        fused_ok = True
        for _ in range(2):
            f = P.nsplit_matmul_fused(win, P.CudaArray.from_torch(a), bl)
            torch.cuda.synchronize()
            fused_ok = fused_ok and bool(torch.equal(f, full.to_torch()))
        dist.barrier()
        win.close()
        q.put((rank, bool(torch.equal(c.to_torch(), full.to_torch())) and fused_ok))
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


@pytest.mark.gpu
def test_nsplit_two_ranks_all_gather():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert got == {0: True, 1: True}
