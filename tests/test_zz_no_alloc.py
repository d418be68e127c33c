"""The allocation-free N-split entry point (gemm_mgpu_nsplit_matmul_noalloc).

It serves callers that cannot allocate device memory at the time they
multiply: a thread that is capturing a CUDA graph, where cudaMalloc is not
allowed, or a program whose device memory all belongs to its own pool and
that must not call cudaMalloc/cudaFree (cudaFree also synchronises the whole
device).  Instead of a gather buffer from the caller it uses a fixed buffer
inside the library.

This file is collected last, so a run that stops at the first failure has
already run every other test; it passes on its own in a fresh process as well.
"""
import ctypes
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "php-gpu-tensors_b200"))

import phptensors as P  # noqa: E402

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 32 << 20          # GEMM_MGPU_NSPLIT_SCRATCH_BYTES
STATUS_SCRATCH_LIMIT = 9005       # GEMM_SM100_STATUS_SCRATCH_LIMIT
STATUS_INVALID_ARGUMENT = 9006    # GEMM_SM100_STATUS_INVALID_ARGUMENT


def _call_noalloc(lib, comm, a, b, c, M, N, K, dtype):
    return lib.gemm_mgpu_nsplit_matmul_noalloc(
        comm.handle, P.DTYPE_CODES[dtype], a.data_ptr(), a.stride(0), a.stride(1),
        b.data_ptr(), b.stride(0), b.stride(1), c.data_ptr(), M, N, K,
        P.current_stream())


def _call_with_workspace(lib, comm, a, b, c, M, N, K, dtype, ws):
    return lib.gemm_mgpu_nsplit_matmul(
        comm.handle, P.DTYPE_CODES[dtype], a.data_ptr(), a.stride(0), a.stride(1),
        b.data_ptr(), b.stride(0), b.stride(1), c.data_ptr(), M, N, K, ws.data_ptr(),
        ws.numel(), P.current_stream())


@pytest.mark.parametrize("dtype,tdt", [("float64", torch.float64), ("bfloat16", torch.bfloat16)])
def test_noalloc_matches_workspace_entry_point_twice(dtype, tdt):
    """Two calls in a row, different inputs each time, through the C ABI:
    each result equals the workspace entry point's result (the tolerance of
    these tests for a product computed by the same kernels is exact
    equality), so what the shared buffer kept from the first call does not
    leak into the second."""
    torch.cuda.set_device(0)
    lib = P.library()
    comm = P.MgpuComm(0, 1)
    try:
        M, N, K = 640, 768, 520
        g = torch.Generator(device="cuda").manual_seed(101)
        ws = torch.empty(M * N * 8, dtype=torch.uint8, device="cuda")
        for call in range(2):
            a = (torch.rand(M, K, device="cuda", generator=g, dtype=torch.float64) - 0.5).to(tdt)
            b = (torch.rand(K, N, device="cuda", generator=g, dtype=torch.float64) - 0.5).to(tdt)
            got = torch.full((M, N), float("nan"), device="cuda", dtype=tdt)
            want = torch.full((M, N), float("nan"), device="cuda", dtype=tdt)
            assert _call_noalloc(lib, comm, a, b, got, M, N, K, dtype) == 1, call
            assert _call_with_workspace(lib, comm, a, b, want, M, N, K, dtype, ws) == 1, call
            torch.cuda.synchronize()
            assert torch.equal(got, want), (dtype, call)
            assert not torch.isnan(got).any(), (dtype, call)
        assert lib.gemm_sm100_device_status(0, 1) == 0
    finally:
        comm.close()


def test_noalloc_rejects_products_larger_than_its_buffer():
    torch.cuda.set_device(0)
    lib = P.library()
    comm = P.MgpuComm(0, 1)
    try:
        M, N, K = 4096, 2048, 8           # 64 MiB of float64: twice the buffer
        a = torch.zeros(M, K, device="cuda", dtype=torch.float64)
        b = torch.zeros(K, N, device="cuda", dtype=torch.float64)
        c = torch.full((M, N), 7.0, device="cuda", dtype=torch.float64)
        assert M * N * 8 > SCRATCH_BYTES
        assert _call_noalloc(lib, comm, a, b, c, M, N, K, "float64") == 0
        assert P.cuda_get_backend_info()["lastBlasStatus"] == STATUS_SCRATCH_LIMIT
        torch.cuda.synchronize()
        assert bool((c == 7.0).all())      # nothing was enqueued
        # an argument the N-split rejects sets its own status, not a stale one
        assert _call_noalloc(lib, comm, a, b, c, 64, 64, -1, "float64") == 0
        assert P.cuda_get_backend_info()["lastBlasStatus"] == STATUS_INVALID_ARGUMENT
    finally:
        comm.close()
