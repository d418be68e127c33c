"""Multi-GPU paths (one process per GPU).

CPU (gloo, world size 2, no GPU calls): batch sharding and N-split column
ranges tile the work exactly once, the library's N-split workspace size is
consistent across ranks, and the bench's max-over-ranks timing rule.

GPU: the N-split entry points (NCCL all-gather + permute, the fused kernel
whose epilogue stores into every rank's window, and the allocation-free
variant) with one rank equal the plain product bit for bit; with two ranks
every rank receives the full product, bit-identical to the single-GPU
product, on two calls in a row with different inputs.
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
        for mode in ("auto", "store", "overlap"):
            win.set_exchange(mode)
            for _ in range(2):
                c = P.nsplit_matmul_fused(win, P.CudaArray.from_torch(a),
                                          P.CudaArray.from_torch(b))
                ref = P.CudaArray.from_torch(a).matmul(P.CudaArray.from_torch(b),
                                                       allow_float64=True)
                torch.cuda.synchronize()
                assert torch.equal(c, ref.to_torch()), mode
        with pytest.raises(P.InvalidArgumentException):
            win.set_exchange("sideways")
    finally:
        win.close()
        comm.close()


@pytest.mark.gpu
def test_fused_nsplit_full_and_half_tiles_single_rank():
    """A column block of 512 tiles (8192 x 1024: one rank's block of an
    8-way N-split) runs three waves of full tiles and its last 68 tiles as
    half tiles; every tile must come out once and equal the plain product."""
    sys.path.insert(0, os.path.join(ROOT, "php-gpu-tensors_b200"))
    import phptensors as P
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda").manual_seed(7)
    M, N, K = 8192, 1024, 256
    a = torch.rand(M, K, device="cuda", generator=g, dtype=torch.float64) - 0.5
    b = torch.rand(K, N, device="cuda", generator=g, dtype=torch.float64) - 0.5
    comm = P.MgpuComm(0, 1)
    win = P.MgpuWindow(comm, M, N)
    try:
        ref = P.CudaArray.from_torch(a).matmul(P.CudaArray.from_torch(b), allow_float64=True)
        for mode in ("store", "overlap"):
            win.set_exchange(mode)
            for _ in range(2):
                c = P.nsplit_matmul_fused(win, P.CudaArray.from_torch(a),
                                          P.CudaArray.from_torch(b))
                torch.cuda.synchronize()
                assert torch.equal(c, ref.to_torch()), mode
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
    """One rank of the 2-rank N-split test.  Each entry point is called twice
    with different inputs, so a result that kept data of the previous call
    (or a peer's stores into this rank's window that raced ahead of this
    rank's reads) shows up as a mismatch.  The reference for every call is
    the single-GPU product of the full operands; rank 0 also checks sampled
    rows of it against the oracle's double twin of HostArray::matmul."""
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(ROOT, "php-gpu-tensors_b200"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle_lib as O
    import phptensors as P
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    comm = None
    results = {}
    try:
        M, N, K = 1024, 2048, 1536
        lo, hi = P.nsplit_columns(N, rank, world)
        comm = P.MgpuComm(rank, world)
        win = P.MgpuWindow(comm, M, N)
        lib = P.library()
        for call in range(2):
            # the same seed on every rank: all ranks hold the same A and B
            g = torch.Generator(device="cuda").manual_seed(11 + call)
            a = torch.rand(M, K, device="cuda", generator=g, dtype=torch.float64) - 0.5
            b = torch.rand(K, N, device="cuda", generator=g, dtype=torch.float64) - 0.5
            bl = b[:, lo:hi].contiguous()
            full = P.CudaArray.from_torch(a).matmul(P.CudaArray.from_torch(b),
                                                    allow_float64=True).to_torch()
            c = P.nsplit_matmul(comm, P.CudaArray.from_torch(a), P.CudaArray.from_torch(bl), N)
            results[("nccl", call)] = bool(torch.equal(c.to_torch(), full))
            for mode in ("store", "overlap"):
                win.set_exchange(mode)
                f = P.nsplit_matmul_fused(win, P.CudaArray.from_torch(a),
                                          P.CudaArray.from_torch(bl))
                torch.cuda.synchronize()
                results[("fused_" + mode, call)] = bool(torch.equal(f, full))
            # the allocation-free entry point: its gather runs in the
            # library's own device buffer at rank offsets
            na = torch.full((M, N), float("nan"), device="cuda", dtype=torch.float64)
            ok = lib.gemm_mgpu_nsplit_matmul_noalloc(
                comm.handle, P.DTYPE_CODES["float64"], a.data_ptr(), a.stride(0), a.stride(1),
                bl.data_ptr(), bl.stride(0), bl.stride(1), na.data_ptr(), M, N, K,
                P.current_stream())
            torch.cuda.synchronize()
            results[("noalloc", call)] = ok == 1 and bool(torch.equal(na, full))
            if rank == 0:
                rows = [0, 517, M - 1]
                ao = O.dense(a.cpu().numpy(), [M, K])
                bo = O.dense(b.cpu().numpy(), [K, N])
                th = O.oracle().orc_host_threads()
                got = full.cpu().numpy()
                good = True
                for r in rows:
                    ref = O.host_matmul_f64_range(ao, bo, "float64", r * N, N, th)
                    err = np.max(np.abs(got[r] - ref)) / max(1.0, float(np.max(np.abs(ref))))
                    good = good and err <= 1e-12
                results[("oracle", call)] = good
            dist.barrier()
        win.close()
        # ragged edges: partial row and column tiles in every rank's block
        Mr, Nr, Kr = 1000, 1200, 776
        g = torch.Generator(device="cuda").manual_seed(21)
        a = torch.rand(Mr, Kr, device="cuda", generator=g, dtype=torch.float64) - 0.5
        b = torch.rand(Kr, Nr, device="cuda", generator=g, dtype=torch.float64) - 0.5
        lo, hi = P.nsplit_columns(Nr, rank, world)
        bl = b[:, lo:hi].contiguous()
        full = P.CudaArray.from_torch(a).matmul(P.CudaArray.from_torch(b),
                                                allow_float64=True).to_torch()
        win = P.MgpuWindow(comm, Mr, Nr)
        for mode in ("store", "overlap"):
            win.set_exchange(mode)
            f = P.nsplit_matmul_fused(win, P.CudaArray.from_torch(a), P.CudaArray.from_torch(bl))
            torch.cuda.synchronize()
            results[("fused_ragged_" + mode, 0)] = bool(torch.equal(f, full))
        dist.barrier()
        win.close()
        q.put((rank, results))
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
    for rank in range(world):
        for key, good in got[rank].items():
            assert good, (rank, key)
    assert ("oracle", 1) in got[0] and ("noalloc", 1) in got[1]
