"""C ABI checks that need no GPU.

  * libgemm_sm100.so loads and exports exactly the functions include/*.h
    declares (no CUDA runtime or internal symbol leaks);
  * the host-side logic that runs before any CUDA call behaves like the
    reference: argument validation and degenerate extents of the launchers
    (src/backends/cuda/matmul_kernels.cu:680-710,856-875,912-914), precision
    state (:31-43), backend info (:45-59), and the tensor-level errors of
    src/cuda_array/ca_private.c:1097-1213 / cuda_array_ce.c:1568-1607.
"""
import ctypes
import os
import re
import subprocess

import pytest

import phptensors as P

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_functions():
    names = set()
    inc = os.path.join(ROOT, "include")
    for fn in sorted(os.listdir(inc)):
        if not fn.endswith(".h"):
            continue
        text = open(os.path.join(inc, fn)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        text = "\n".join(l for l in text.splitlines() if not l.lstrip().startswith("#"))
        for m in re.finditer(r"([A-Za-z_]\w*)\s*\(([^;{}]*)\)\s*;", text):
            names.add(m.group(1))
    return names


def _exported():
    out = subprocess.run(["nm", "-D", "--defined-only", P.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_library_exports_exactly_the_headers():
    declared = _declared_functions()
    assert "cuda_matmul_launcher" in declared and "pt_tensor_matmul_into" in declared
    lib = P.library()
    for name in declared:
        assert hasattr(lib, name), name
    assert _exported() == declared
    assert set(P.exported_symbols()) == declared


def _shape(vals):
    return (ctypes.c_int * 10)(*vals)


def _strides(vals):
    return (ctypes.c_size_t * 10)(*vals)


def test_launcher_validation_without_gpu():
    lib = P.library()
    s = ctypes.c_void_p(0)
    # cuda_matmul_launcher: negative extent -> 0; m == 0 or cols == 0 -> 1 (no launch)
    assert lib.cuda_matmul_launcher(None, None, None, -1, 2, 2, 2, 1, 2, 1, 2, 1, s) == 0
    assert lib.cuda_matmul_launcher(None, None, None, 0, 5, 3, 5, 1, 3, 1, 3, 1, s) == 1
    assert lib.cuda_matmul_launcher(None, None, None, 4, 5, 0, 5, 1, 0, 1, 0, 1, s) == 1
    nd = lib.cuda_batched_matmul_nd_launcher
    # rank < 2, rank > 10, inner mismatch, result mismatch -> 0
    assert nd(None, None, None, _shape([3]), _strides([1]), 1, _shape([3, 2]), _strides([2, 1]),
              2, _shape([1, 2]), _strides([2, 1]), 2, s) == 0
    assert nd(None, None, None, _shape([1] * 10), _strides([1] * 10), 11, _shape([1, 1]),
              _strides([1, 1]), 2, _shape([1, 1]), _strides([1, 1]), 2, s) == 0
    assert nd(None, None, None, _shape([2, 3]), _strides([3, 1]), 2, _shape([4, 2]),
              _strides([2, 1]), 2, _shape([2, 2]), _strides([2, 1]), 2, s) == 0
    assert nd(None, None, None, _shape([2, 3]), _strides([3, 1]), 2, _shape([3, 2]),
              _strides([2, 1]), 2, _shape([2, 3]), _strides([3, 1]), 2, s) == 0
    # incompatible batch extents -> 0 (the shape rule would have rejected them)
    assert nd(None, None, None, _shape([2, 1, 1]), _strides([1, 1, 1]), 3, _shape([3, 1, 1]),
              _strides([1, 1, 1]), 3, _shape([3, 1, 1]), _strides([1, 1, 1]), 3, s) == 0
    # empty batch / empty rows -> 1 without touching the device
    assert nd(None, None, None, _shape([0, 2, 3]), _strides([6, 3, 1]), 3, _shape([3, 2]),
              _strides([2, 1]), 2, _shape([0, 2, 2]), _strides([4, 2, 1]), 3, s) == 1
    lp = lib.cuda_low_precision_matmul_nd_launcher
    assert lp(None, None, None, 0, _shape([2, 2]), _strides([2, 1]), 2, _shape([2, 2]),
              _strides([2, 1]), 2, _shape([2, 2]), _strides([2, 1]), 2, s) == 0   # float32
    assert lp(None, None, None, 12, _shape([2, 0]), _strides([0, 1]), 2, _shape([0, 0]),
              _strides([0, 1]), 2, _shape([2, 0]), _strides([0, 1]), 2, s) == 1
    ep = lib.cuda_matmul_epilogue_nd_launcher
    assert ep(None, None, None, 11, _shape([2, 2]), _strides([2, 1]), 2, _shape([2, 2]),
              _strides([2, 1]), 2, _shape([2, 2]), _strides([2, 1]), 2, None, 9, s) == 0


def test_precision_state_and_info():
    lib = P.library()
    info = P.cuda_get_backend_info()
    assert info["cublas"] == 0 and info["cublasLt"] == 0
    assert info["precision"] == "fp32-strict"
    assert lib.cuda_blas_set_precision(7) == 0
    assert lib.cuda_blas_precision_name() == b"fp32-strict"
    assert lib.cuda_blas_set_precision(1) == 1
    assert P.cuda_get_backend_info()["precision"] == "tf32"
    with pytest.raises(P.InvalidArgumentException):
        P.cuda_set_matmul_precision("unknown")
    assert P.cuda_get_backend_info()["precision"] == "tf32"
    P.cuda_set_matmul_precision("fp32-strict")
    assert lib.cuda_blas_precision_name() == b"fp32-strict"
    lib.cuda_blas_shutdown()
    info = P.cuda_get_backend_info()
    assert info["builtinMatmulCalls"] == 0 and info["lastMatmul"] == "none"
    assert lib.gemm_sm100_version() >= 100
    assert lib.gemm_sm100_algorithm_name(1) == b"tc-3xtf32-128x128"
    assert lib.gemm_sm100_algorithm_name(99) == b"unknown"


def test_path_selector():
    lib = P.library()
    prev = lib.gemm_sm100_set_path(2)
    assert lib.gemm_sm100_set_path(1) == 2
    assert lib.gemm_sm100_set_path(6) == 1
    assert lib.gemm_sm100_set_path(7) == 6       # invalid values leave it unchanged
    assert lib.gemm_sm100_set_path(-1) == 6
    assert lib.gemm_sm100_set_path(prev) == 6


def _pt(shape, dtype, strides=None):
    t = P.PtTensor()
    t.data = 16
    t.dtype = P.DTYPE_CODES[dtype]
    t.ndims = len(shape)
    strides = strides or P._contiguous_strides(shape)
    for i, (d, s) in enumerate(zip(shape, strides)):
        t.shape[i] = d
        t.strides[i] = s
    return t


def test_tensor_layer_errors_without_gpu(golden):
    lib = P.library()
    sh = (ctypes.c_int * 10)()
    nd = ctypes.c_int()
    for s in golden["shapes"]:
        a, b = _pt(s["a"], "float32"), _pt(s["b"], "float32")
        rc = lib.pt_matmul_result_shape(ctypes.byref(a), ctypes.byref(b), sh, ctypes.byref(nd))
        if s["ok"]:
            assert rc == P.PT_OK and [sh[i] for i in range(nd.value)] == s["out"]
        else:
            assert rc == P.PT_INVALID_ARGUMENT
            assert lib.pt_last_error() == b"Matrix multiplication failed - incompatible dimensions"
    a, b, r = _pt([2, 2], "float32"), _pt([2, 2], "float16"), _pt([2, 2], "float32")
    s = ctypes.c_void_p(0)
    assert lib.pt_tensor_matmul_into(ctypes.byref(a), ctypes.byref(b), ctypes.byref(r), 0,
                                     s) == P.PT_INVALID_ARGUMENT
    assert lib.pt_last_error() == b"matmul requires matching float32, float16 or bfloat16 operands"
    # float64 is rejected like the reference unless explicitly allowed
    a, b, r = _pt([1, 1], "float64"), _pt([1, 1], "float64"), _pt([1, 1], "float64")
    assert lib.pt_tensor_matmul_into(ctypes.byref(a), ctypes.byref(b), ctypes.byref(r), 0,
                                     s) == P.PT_INVALID_ARGUMENT
    # result of the wrong shape
    a, b, r = _pt([2, 3], "float32"), _pt([3, 4], "float32"), _pt([2, 5], "float32")
    assert lib.pt_tensor_matmul_into(ctypes.byref(a), ctypes.byref(b), ctypes.byref(r), 0,
                                     s) == P.PT_INVALID_ARGUMENT
    # a degenerate product succeeds without a launch
    a, b, r = _pt([0, 3], "float32"), _pt([3, 4], "float32"), _pt([0, 4], "float32")
    assert lib.pt_tensor_matmul_into(ctypes.byref(a), ctypes.byref(b), ctypes.byref(r), 0,
                                     s) == P.PT_OK


def test_gradient_and_host_staging_errors_without_gpu():
    """Argument errors of pt_tensor_matmul_backward and pt_host_matmul_sharded
    are reported before any CUDA call."""
    lib = P.library()
    s = ctypes.c_void_p(0)
    # operands of different types
    a, b, g = _pt([3, 4], "float32"), _pt([4, 5], "bfloat16"), _pt([3, 5], "float32")
    ga = _pt([3, 4], "float32")
    assert lib.pt_tensor_matmul_backward(ctypes.byref(a), ctypes.byref(b), ctypes.byref(g),
                                         ctypes.byref(ga), None, s) == P.PT_INVALID_ARGUMENT
    assert b"matmul backward requires" in lib.pt_last_error()
    # a gradient of a 16-bit operand must be float32
    a, b = _pt([3, 4], "bfloat16"), _pt([4, 5], "bfloat16")
    ga = _pt([3, 4], "bfloat16")
    assert lib.pt_tensor_matmul_backward(ctypes.byref(a), ctypes.byref(b), ctypes.byref(g),
                                         ctypes.byref(ga), None, s) == P.PT_INVALID_ARGUMENT
    assert lib.pt_last_error() == b"matmul gradients are float32 tensors"
    # a gradient shape that is not a reduction of the product's batch shape
    a, b, g = _pt([2, 3, 4], "float32"), _pt([4, 5], "float32"), _pt([2, 3, 5], "float32")
    gb = _pt([3, 4, 5], "float32")
    assert lib.pt_tensor_matmul_backward(ctypes.byref(a), ctypes.byref(b), ctypes.byref(g),
                                         None, ctypes.byref(gb), s) == P.PT_INVALID_ARGUMENT
    assert lib.pt_last_error().startswith(b"Gradient shape cannot be reduced")
    # sharded host staging: the device list is checked first
    devs = (ctypes.c_int * 2)(0, 0)
    assert lib.pt_host_matmul_sharded(16, 16, 16, P.DTYPE_CODES["float32"], 4, 2, 2, 2, 0, devs,
                                      2, 2, 0) == P.PT_INVALID_ARGUMENT
    assert lib.pt_host_matmul_sharded(16, 16, 16, P.DTYPE_CODES["float32"], 4, 2, 2, 2, 0, devs,
                                      0, 2, 0) == P.PT_INVALID_ARGUMENT


def test_window_exchange_mode_rejects_a_null_window():
    """Argument checks of gemm_mgpu_window_set_exchange run before any CUDA call."""
    lib = P.library()
    assert lib.gemm_mgpu_window_set_exchange(None, 0) == 0
    assert P.cuda_get_backend_info()["lastBlasStatus"] == 9006
