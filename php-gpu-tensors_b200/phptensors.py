"""Python mirror of the php-gpu-tensors matmul API over libgemm_sm100.so.

The PHP extension cannot be built here (no PHP toolchain), so this module
stands in for its user-facing surface on the matmul path, with the reference's
names, argument meaning and exceptions:

    CudaArray::matmul                stubs/cuda.stub.php:472
    CudaArray::transpose / fromFlatArray / fromBuffer / ones / full / toArray
    cuda_get_backend_info            src/cuda.c:131-153
    cuda_set_matmul_precision        src/cuda.c:155-209
    cuda_tune_matmul                 src/cuda.c:211-290
    PhpTensors\\InvalidArgumentException / RuntimeException

Every product computed here runs on the GPU through the C ABI of
include/gemm_sm100.h and include/pt_tensor.h (the C++ host layer
pt_tensor_matmul_into dispatches to the launchers).  PyTorch is used only for
device memory, host<->device copies and the current CUDA stream.  There is no
CPU fallback: if the library is missing, or no CUDA device is present, the
calls raise.
"""
import ctypes
import math
import os
import struct

import numpy as np

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libgemm_sm100.so")

MAX_DIMS = 10
DTYPE_CODES = {"float32": 0, "float64": 1, "float16": 11, "bfloat16": 12}
ELEMENT_BYTES = {"float32": 4, "float64": 8, "float16": 2, "bfloat16": 2}
PT_OK, PT_INVALID_ARGUMENT, PT_RUNTIME = 0, 1, 2
PT_MATMUL_ALLOW_FLOAT64 = 1
EPILOGUES = {"none": 0, "tanh": 1, "relu": 2, "sigmoid": 3}


class InvalidArgumentException(ValueError):
    """PhpTensors\\InvalidArgumentException."""


class RuntimeException(RuntimeError):
    """PhpTensors\\RuntimeException."""


class CudaBackendInfo(ctypes.Structure):
    """cuda_backend_info (src/backends/cuda/backend_info.h:7-14)."""
    _fields_ = [
        ("cublas", ctypes.c_int), ("cublas_lt", ctypes.c_int), ("cudnn", ctypes.c_int),
        ("blas_calls", ctypes.c_ulonglong), ("lt_calls", ctypes.c_ulonglong),
        ("builtin_matmul_calls", ctypes.c_ulonglong),
        ("cub_calls", ctypes.c_ulonglong), ("axis_calls", ctypes.c_ulonglong),
        ("generic_reduce_calls", ctypes.c_ulonglong),
        ("last_matmul", ctypes.c_char_p), ("precision", ctypes.c_char_p),
        ("last_blas_status", ctypes.c_int),
    ]


class TuningCandidate(ctypes.Structure):
    _fields_ = [("algorithm_id", ctypes.c_int), ("workspace_bytes", ctypes.c_size_t),
                ("median_ms", ctypes.c_double)]


class TuningResult(ctypes.Structure):
    _fields_ = [("candidate_count", ctypes.c_int), ("selected_candidate", ctypes.c_int),
                ("candidates", TuningCandidate * 8)]


class PtTensor(ctypes.Structure):
    """pt_tensor (include/pt_tensor.h)."""
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int), ("ndims", ctypes.c_int),
                ("shape", ctypes.c_int * MAX_DIMS), ("strides", ctypes.c_size_t * MAX_DIMS)]


_LIB = None

_SIGNATURES = {
    "cuda_blas_shutdown": (None, []),
    "cuda_blas_set_precision": (ctypes.c_int, [ctypes.c_int]),
    "cuda_blas_precision_name": (ctypes.c_char_p, []),
    "cuda_blas_info": (None, [ctypes.POINTER(CudaBackendInfo)]),
    "cuda_blas_tune_matmul": (ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 +
                              [ctypes.c_size_t] * 4 + [ctypes.c_void_p,
                                                       ctypes.POINTER(TuningResult)]),
    "cuda_matmul_launcher": (ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3 +
                             [ctypes.c_size_t] * 6 + [ctypes.c_void_p]),
    "cuda_batched_matmul_nd_launcher": (
        ctypes.c_int, [ctypes.c_void_p] * 3 +
        [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_size_t), ctypes.c_int] * 3 +
        [ctypes.c_void_p]),
    "cuda_low_precision_matmul_nd_launcher": (
        ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_int] +
        [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_size_t), ctypes.c_int] * 3 +
        [ctypes.c_void_p]),
    "cuda_f64_matmul_nd_launcher": (
        ctypes.c_int, [ctypes.c_void_p] * 3 +
        [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_size_t), ctypes.c_int] * 3 +
        [ctypes.c_void_p]),
    "cuda_matmul_epilogue_nd_launcher": (
        ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_int] +
        [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_size_t), ctypes.c_int] * 3 +
        [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "cuda_mixed_matmul_nd_launcher": (
        ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                       ctypes.c_void_p] +
        [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_size_t), ctypes.c_int] * 3 +
        [ctypes.c_void_p]),
    "gemm_sm100_last_kernel": (ctypes.c_char_p, []),
    "gemm_sm100_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_void_p]),
    "gemm_sm100_set_path": (ctypes.c_int, [ctypes.c_int]),
    "gemm_sm100_last_launch": (None, [ctypes.POINTER(ctypes.c_int)] * 3),
    "gemm_sm100_device_status": (ctypes.c_int, [ctypes.c_int, ctypes.c_int]),
    "gemm_sm100_algorithm_name": (ctypes.c_char_p, [ctypes.c_int]),
    "gemm_sm100_version": (ctypes.c_int, []),
    "gemm_mgpu_unique_id": (ctypes.c_int, [ctypes.c_void_p]),
    "gemm_mgpu_comm_init": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                           ctypes.POINTER(ctypes.c_void_p)]),
    "gemm_mgpu_comm_destroy": (None, [ctypes.c_void_p]),
    "gemm_mgpu_nsplit_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int, ctypes.c_int,
                                                           ctypes.c_int, ctypes.c_int]),
    "gemm_mgpu_nsplit_matmul": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                               ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p,
                                               ctypes.c_size_t, ctypes.c_size_t, ctypes.c_void_p,
                                               ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                               ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "gemm_mgpu_nsplit_matmul_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int,
                                                       ctypes.c_void_p, ctypes.c_size_t,
                                                       ctypes.c_size_t, ctypes.c_void_p,
                                                       ctypes.c_size_t, ctypes.c_size_t,
                                                       ctypes.c_void_p, ctypes.c_int,
                                                       ctypes.c_int, ctypes.c_int,
                                                       ctypes.c_void_p]),
    "gemm_mgpu_window_create": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t,
                                               ctypes.POINTER(ctypes.c_void_p),
                                               ctypes.POINTER(ctypes.c_void_p)]),
    "gemm_mgpu_window_destroy": (None, [ctypes.c_void_p]),
    "gemm_mgpu_window_set_exchange": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "gemm_mgpu_nsplit_matmul_fused": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int,
                                                     ctypes.c_void_p, ctypes.c_size_t,
                                                     ctypes.c_size_t, ctypes.c_void_p,
                                                     ctypes.c_size_t, ctypes.c_size_t,
                                                     ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                                     ctypes.c_void_p]),
    "pt_host_matmul": (ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_int] * 8),
    "pt_host_matmul_sharded": (ctypes.c_int, [ctypes.c_void_p] * 3 + [ctypes.c_int] * 6 +
                               [ctypes.POINTER(ctypes.c_int)] + [ctypes.c_int] * 3),
    "pt_host_release": (None, []),
    "pt_last_error": (ctypes.c_char_p, []),
    "pt_matmul_result_shape": (ctypes.c_int, [ctypes.POINTER(PtTensor)] * 2 +
                               [ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
    "pt_tensor_matmul_into": (ctypes.c_int, [ctypes.POINTER(PtTensor)] * 3 +
                              [ctypes.c_int, ctypes.c_void_p]),
    "pt_tensor_matmul": (ctypes.c_int, [ctypes.POINTER(PtTensor)] * 3 +
                         [ctypes.c_int, ctypes.c_void_p]),
    "pt_tensor_release": (None, [ctypes.POINTER(PtTensor), ctypes.c_void_p]),
    "pt_tensor_matmul_backward": (ctypes.c_int, [ctypes.POINTER(PtTensor)] * 5 +
                                  [ctypes.c_void_p]),
}


def exported_symbols():
    """Names the C ABI headers declare (checked against the library by tests)."""
    return sorted(_SIGNATURES)


def library():
    """Loads libgemm_sm100.so (built in-tree); raises if it is missing."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeException(
                "libgemm_sm100.so is not built (%s); run php-gpu-tensors_b200/build.py" % LIB_PATH)
        lib = ctypes.CDLL(LIB_PATH)
        for name, (restype, argtypes) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _LIB = lib
    return _LIB


def _torch():
    import torch
    if not torch.cuda.is_available():
        raise RuntimeException("CUDA device unavailable: CudaArray needs a B200 (sm_100a)")
    return torch


def _torch_dtype(dtype):
    torch = _torch()
    return {"float32": torch.float32, "float64": torch.float64, "float16": torch.float16,
            "bfloat16": torch.bfloat16}[dtype]


def _check_dtype(dtype):
    if dtype not in DTYPE_CODES:
        raise InvalidArgumentException("Unsupported dtype '%s' for the matmul path" % dtype)


def _contiguous_strides(shape):
    strides, s = [], 1
    for d in reversed(shape):
        strides.insert(0, s)
        s *= d
    return strides


def current_stream():
    """Raw cudaStream_t of torch's current stream on the current device."""
    return ctypes.c_void_p(_torch().cuda.current_stream().cuda_stream)


def _raise_for(status):
    if status == PT_OK:
        return
    msg = library().pt_last_error().decode()
    if status == PT_INVALID_ARGUMENT:
        raise InvalidArgumentException(msg)
    raise RuntimeException(msg)


class CudaArray:
    """A device tensor view: flat storage + element offset, shape, strides.

    Mirrors the reference's tensor_t view model (src/tensor.h:49-79): strides
    are in elements, transpose() swaps the last two axes without copying.
    """

    def __init__(self, storage, shape, strides=None, offset=0, dtype="float32"):
        _check_dtype(dtype)
        self._storage = storage            # 1-D torch tensor of the dtype
        self._shape = [int(d) for d in shape]
        self._strides = [int(s) for s in (strides if strides is not None
                                          else _contiguous_strides(self._shape))]
        self._offset = int(offset)
        self._dtype = dtype

    # ---------------------------------------------------------- constructors
    @classmethod
    def fromFlatArray(cls, values, shape, dtype="float32"):
        """Values are converted like the reference: double -> float -> dtype (RNE)."""
        torch = _torch()
        host = torch.tensor(np.asarray(values, dtype=np.float64).astype(
            np.float64 if dtype == "float64" else np.float32), dtype=torch.float64
            if dtype == "float64" else torch.float32)
        storage = host.to(_torch_dtype(dtype)).cuda().reshape(-1)
        return cls(storage, shape, dtype=dtype)

    @classmethod
    def fromBuffer(cls, buffer, shape, dtype="float32"):
        """Raw little-endian element bytes (PHP pack('g*'/'e*'...) / toBuffer())."""
        torch = _torch()
        raw = torch.frombuffer(bytearray(buffer), dtype=torch.uint8)
        storage = raw.view(_torch_dtype(dtype)).cuda()
        return cls(storage, shape, dtype=dtype)

    @classmethod
    def from_torch(cls, tensor, dtype=None):
        """Wraps a CUDA torch tensor view without copying (storage offset kept)."""
        torch = _torch()
        rev = {torch.float32: "float32", torch.float64: "float64", torch.float16: "float16",
               torch.bfloat16: "bfloat16"}
        dtype = dtype or rev[tensor.dtype]
        n = tensor.untyped_storage().nbytes() // tensor.element_size()
        storage = torch.as_strided(tensor, (n,), (1,), 0)
        return cls(storage, list(tensor.shape), list(tensor.stride()),
                   tensor.storage_offset(), dtype)

    @classmethod
    def full(cls, shape, value, dtype="float32"):
        n = int(np.prod(shape)) if len(shape) else 1
        storage = _torch().full((n,), float(value), dtype=_torch_dtype(dtype), device="cuda")
        return cls(storage, shape, dtype=dtype)

    @classmethod
    def ones(cls, shape, dtype="float32"):
        return cls.full(shape, 1.0, dtype)

    @classmethod
    def zeros(cls, shape, dtype="float32"):
        return cls.full(shape, 0.0, dtype)

    # ---------------------------------------------------------- views
    def transpose(self):
        if len(self._shape) < 2:
            raise InvalidArgumentException("transpose requires rank >= 2")
        shape, strides = list(self._shape), list(self._strides)
        shape[-2], shape[-1] = shape[-1], shape[-2]
        strides[-2], strides[-1] = strides[-1], strides[-2]
        return CudaArray(self._storage, shape, strides, self._offset, self._dtype)

    def view(self, shape, strides, offset):
        """An arbitrary strided view of the same storage (slices, broadcasts)."""
        return CudaArray(self._storage, shape, strides, offset, self._dtype)

    # ---------------------------------------------------------- metadata
    def dtype(self):
        return self._dtype

    def getShape(self):
        return list(self._shape)

    def getStrides(self):
        return list(self._strides)

    def _pt(self):
        t = PtTensor()
        es = ELEMENT_BYTES[self._dtype]
        t.data = self._storage.data_ptr() + self._offset * es
        t.dtype = DTYPE_CODES[self._dtype]
        t.ndims = len(self._shape)
        for i, (d, s) in enumerate(zip(self._shape, self._strides)):
            t.shape[i] = d
            t.strides[i] = s
        return t

    # ---------------------------------------------------------- matmul
    def matmul(self, other, allow_float64=False):
        """C = self . other on the GPU (CudaArray::matmul)."""
        if not isinstance(other, CudaArray):
            raise InvalidArgumentException("Matrix multiplication operand must be a CudaArray")
        lib = library()
        a, b = self._pt(), other._pt()
        shape = (ctypes.c_int * MAX_DIMS)()
        nd = ctypes.c_int(0)
        if self._dtype != other._dtype or self._dtype not in DTYPE_CODES:
            raise InvalidArgumentException(
                "matmul requires matching float32, float16 or bfloat16 operands")
        _raise_for(lib.pt_matmul_result_shape(ctypes.byref(a), ctypes.byref(b), shape,
                                              ctypes.byref(nd)))
        out_shape = [shape[i] for i in range(nd.value)]
        n = int(np.prod(out_shape)) if out_shape else 1
        storage = _torch().empty(max(n, 1), dtype=_torch_dtype(self._dtype), device="cuda")
        result = CudaArray(storage, out_shape, dtype=self._dtype)
        r = result._pt()
        flags = PT_MATMUL_ALLOW_FLOAT64 if allow_float64 else 0
        _raise_for(lib.pt_tensor_matmul_into(ctypes.byref(a), ctypes.byref(b), ctypes.byref(r),
                                             flags, current_stream()))
        return result

    def matmul_epilogue(self, other, bias=None, activation="none"):
        """Fused native-matmul step: act(round(self . other) + bias)."""
        lib = library()
        if other._dtype != self._dtype:
            raise InvalidArgumentException(
                "matmul requires matching float32, float16 or bfloat16 operands")
        a, b = self._pt(), other._pt()
        shape = (ctypes.c_int * MAX_DIMS)()
        nd = ctypes.c_int(0)
        _raise_for(lib.pt_matmul_result_shape(ctypes.byref(a), ctypes.byref(b), shape,
                                              ctypes.byref(nd)))
        out_shape = [shape[i] for i in range(nd.value)]
        n = int(np.prod(out_shape)) if out_shape else 1
        storage = _torch().empty(max(n, 1), dtype=_torch_dtype(self._dtype), device="cuda")
        result = CudaArray(storage, out_shape, dtype=self._dtype)
        bias_ptr = None
        if bias is not None:
            if bias._dtype != self._dtype or bias.getShape() != [out_shape[-1]]:
                raise InvalidArgumentException("bias must be a [N] vector of the operand dtype")
            bias_ptr = ctypes.c_void_p(bias._storage.data_ptr() +
                                       bias._offset * ELEMENT_BYTES[self._dtype])
        arrays = [_shape_args(x) for x in (self, other, result)]
        ok = lib.cuda_matmul_epilogue_nd_launcher(
            a.data, b.data, result._pt().data, DTYPE_CODES[self._dtype],
            *arrays[0], *arrays[1], *arrays[2], bias_ptr, EPILOGUES[activation],
            current_stream())
        if not ok:
            info = cuda_get_backend_info()
            raise RuntimeException("Matmul backend submission failed (cuBLAS status %d)"
                                   % info["lastBlasStatus"])
        return result

    # ---------------------------------------------------------- export
    def to_torch(self):
        """A torch view of this array (no copy)."""
        return self._storage.as_strided(self._shape, self._strides, self._offset)

    def toArray(self):
        t = self.to_torch().float() if self._dtype in ("float16", "bfloat16") else self.to_torch()
        return t.cpu().tolist()

    def toBuffer(self):
        return self.to_torch().contiguous().cpu().view(-1).view(
            _torch().uint8).numpy().tobytes()

    def to_numpy(self):
        t = self.to_torch().contiguous().cpu()
        if self._dtype in ("float16", "bfloat16"):
            return t.view(_torch().int16).numpy().view(np.uint16)
        return t.numpy()


def host_matmul(a, b, c, chunks=8, allow_float64=False, devices=None):
    """Batched product between HOST torch tensors (pinned for overlap):
    a [batches, M, K], b [batches, K, N] or [K, N] (shared), c [batches, M, N]
    are filled through pt_host_matmul, whose copies and products overlap.
    devices=[d0, d1, ...] shards the batch over those GPUs of this process
    (pt_host_matmul_sharded), `chunks` pieces per device."""
    torch = _torch()
    rev = {torch.float32: "float32", torch.float64: "float64", torch.float16: "float16",
           torch.bfloat16: "bfloat16"}
    dt = rev[a.dtype]
    if not (a.is_contiguous() and b.is_contiguous() and c.is_contiguous()):
        raise InvalidArgumentException("host_matmul needs contiguous row-major host tensors")
    batches, M, K = a.shape
    shared = b.dim() == 2
    N = b.shape[-1]
    if (b.shape[-2] != K or list(c.shape) != [batches, M, N]
            or (not shared and b.shape[0] != batches)):
        raise InvalidArgumentException("Matrix multiplication failed - incompatible dimensions")
    flags = PT_MATMUL_ALLOW_FLOAT64 if allow_float64 else 0
    if devices is None:
        _raise_for(library().pt_host_matmul(
            a.data_ptr(), b.data_ptr(), c.data_ptr(), DTYPE_CODES[dt], batches, M, N, K,
            1 if shared else 0, chunks, flags))
    else:
        devs = (ctypes.c_int * len(devices))(*devices)
        _raise_for(library().pt_host_matmul_sharded(
            a.data_ptr(), b.data_ptr(), c.data_ptr(), DTYPE_CODES[dt], batches, M, N, K,
            1 if shared else 0, devs, len(devices), chunks, flags))
    return c


def _shape_args(x):
    nd = len(x._shape)
    shape = (ctypes.c_int * MAX_DIMS)(*x._shape)
    strides = (ctypes.c_size_t * MAX_DIMS)(*x._strides)
    return shape, strides, nd


def cuda_get_backend_info():
    """cuda_get_backend_info() matmul keys (src/cuda.c:131-153) + 'kernel'."""
    lib = library()
    info = CudaBackendInfo()
    lib.cuda_blas_info(ctypes.byref(info))
    return {
        "cublas": info.cublas, "cublasLt": info.cublas_lt,
        "blasCalls": info.blas_calls, "ltCalls": info.lt_calls,
        "builtinMatmulCalls": info.builtin_matmul_calls,
        "lastMatmul": info.last_matmul.decode(), "precision": info.precision.decode(),
        "lastBlasStatus": info.last_blas_status,
        "kernel": lib.gemm_sm100_last_kernel().decode(),
    }


def cuda_set_matmul_precision(precision):
    """src/cuda.c:155-209 (TF32 is supported by this backend)."""
    modes = {"fp32-strict": 0, "tf32": 1}
    if precision not in modes:
        raise InvalidArgumentException("Matmul precision must be 'fp32-strict' or 'tf32'")
    if not library().cuda_blas_set_precision(modes[precision]):
        raise RuntimeException("Failed to set matmul precision")


def cuda_tune_matmul(left, right):
    """src/cuda.c:211-290 over this library's own tile configurations."""
    if left.dtype() != "float32" or right.dtype() != "float32":
        raise InvalidArgumentException("Matmul autotuning currently requires valid float32 tensors")
    ls, rs = left.getShape(), right.getShape()
    if len(ls) != 2 or len(rs) != 2 or ls[1] != rs[0]:
        raise InvalidArgumentException("Matmul autotuning currently requires compatible 2D tensors")
    torch = _torch()
    out = torch.empty(ls[0] * rs[1], dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    result = TuningResult()
    a, b = left._pt(), right._pt()
    status = library().cuda_blas_tune_matmul(
        a.data, b.data, out.data_ptr(), ls[0], ls[1], rs[1], left._strides[0], left._strides[1],
        right._strides[0], right._strides[1], current_stream(), ctypes.byref(result))
    if status < 0:
        raise RuntimeException("Matmul autotuning failed (cuBLAS status %d)"
                               % cuda_get_backend_info()["lastBlasStatus"])
    if status == 0:
        raise InvalidArgumentException(
            "Matmul autotuning requires compatible strides and at least 10 million operations")
    cands = []
    for i in range(result.candidate_count):
        c = result.candidates[i]
        cands.append({"algorithmId": c.algorithm_id, "workspaceBytes": c.workspace_bytes,
                      "medianMs": c.median_ms, "selected": i == result.selected_candidate,
                      "name": library().gemm_sm100_algorithm_name(c.algorithm_id).decode()})
    return {"backend": "builtin", "precision": library().cuda_blas_precision_name().decode(),
            "selectedCandidate": result.selected_candidate,
            "candidateCount": result.candidate_count, "candidates": cands,
            "product": CudaArray(out, [ls[0], rs[1]])}


def set_kernel_path(path):
    """0 automatic, 1 single-CTA tensor-core kernel whenever the layout allows,
    2 CUDA cores only, 3 2-CTA tensor-core kernel whenever allowed (16-bit,
    tf32, strict float32, float32 x bf16), 4 few-column split-K kernel
    whenever N <= 32 and K >= 128, 5 the 2-CTA 256 x 512 kernel for 16-bit
    products with a 16-bit result (other products as 3), 6 the same kernel
    running every tile as two 256-column halves."""
    return library().gemm_sm100_set_path(
        {"auto": 0, "tensor-core": 1, "simt": 2, "tensor-core-pair": 3, "skinny": 4,
         "tensor-core-wide": 5, "tensor-core-wide-halves": 6}[path])


def last_launch():
    """(grid, block, cluster) of the last tensor-core or few-column launch on
    this thread."""
    g, b, c = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    library().gemm_sm100_last_launch(ctypes.byref(g), ctypes.byref(b), ctypes.byref(c))
    return g.value, b.value, c.value


def device_status(device=0, clear=True):
    return library().gemm_sm100_device_status(device, 1 if clear else 0)


# ---------------------------------------------------------------- multi-GPU
class MgpuComm:
    """NCCL communicator of the library for one process per GPU.

    Rank 0 creates the id with gemm_mgpu_unique_id; it reaches the other ranks
    through the already-initialised torch.distributed process group (host
    plumbing only), and every rank joins on its current device.
    """

    def __init__(self, rank, world):
        import torch.distributed as dist
        lib = library()
        idbuf = (ctypes.c_ubyte * 128)()
        if rank == 0 and not lib.gemm_mgpu_unique_id(idbuf):
            raise RuntimeException("NCCL is unavailable for the multi-GPU entry points")
        obj = [bytes(idbuf)]
        if world > 1:
            dist.broadcast_object_list(obj, src=0)
        idbuf = (ctypes.c_ubyte * 128).from_buffer_copy(obj[0])
        handle = ctypes.c_void_p()
        if not lib.gemm_mgpu_comm_init(idbuf, world, rank, ctypes.byref(handle)):
            raise RuntimeException("gemm_mgpu_comm_init failed (status %d)"
                                   % cuda_get_backend_info()["lastBlasStatus"])
        self.handle, self.rank, self.world = handle, rank, world

    def close(self):
        if self.handle:
            library().gemm_mgpu_comm_destroy(self.handle)
            self.handle = None


def nsplit_columns(N, rank, world):
    """Column block [lo, hi) of rank `rank` in an N-split product."""
    if N % world:
        raise InvalidArgumentException("N-split needs N divisible by the number of ranks")
    nb = N // world
    return rank * nb, (rank + 1) * nb


def nsplit_matmul(comm, a, b_local, N, workspace=None):
    """C = A . B with B split along N: `b_local` is this rank's column block;
    every rank receives the whole row-major C (gemm_mgpu_nsplit_matmul)."""
    lib = library()
    torch = _torch()
    M, K = a.getShape()
    if b_local.getShape() != [K, N // comm.world] or a.dtype() != b_local.dtype():
        raise InvalidArgumentException("b_local must be this rank's [K, N / ranks] block")
    dt = a.dtype()
    need = lib.gemm_mgpu_nsplit_workspace_bytes(comm.world, DTYPE_CODES[dt], M, N)
    if need == 0 and M * N > 0:
        raise InvalidArgumentException("N-split needs N divisible by the number of ranks")
    if workspace is None:
        workspace = torch.empty(max(need, 16), dtype=torch.uint8, device="cuda")
    c = CudaArray(torch.empty(max(M * N, 1), dtype=_torch_dtype(dt), device="cuda"), [M, N],
                  dtype=dt)
    es = ELEMENT_BYTES[dt]
    ok = lib.gemm_mgpu_nsplit_matmul(
        comm.handle, DTYPE_CODES[dt], a._storage.data_ptr() + a._offset * es, a._strides[0],
        a._strides[1], b_local._storage.data_ptr() + b_local._offset * es, b_local._strides[0],
        b_local._strides[1], c._storage.data_ptr(), M, N, K, workspace.data_ptr(),
        workspace.numel(), current_stream())
    if not ok:
        raise RuntimeException("N-split matmul failed (status %d)"
                               % cuda_get_backend_info()["lastBlasStatus"])
    return c


class MgpuWindow:
    """An [M, N] float64 result buffer mapped into every rank (the fused
    N-split product writes into all of them)."""

    def __init__(self, comm, M, N):
        lib = library()
        h, local = ctypes.c_void_p(), ctypes.c_void_p()
        if not lib.gemm_mgpu_window_create(comm.handle, M * N * 8, ctypes.byref(h),
                                           ctypes.byref(local)):
            raise RuntimeException("gemm_mgpu_window_create failed (status %d)"
                                   % cuda_get_backend_info()["lastBlasStatus"])
        self.handle, self.local, self.comm, self.M, self.N = h, local.value, comm, M, N

    EXCHANGE = {"auto": 0, "store": 1, "overlap": 2}

    def set_exchange(self, mode):
        """'auto', 'store' (epilogue stores into every window) or 'overlap'
        (persistent kernel, copies under the next tile's math)."""
        if mode not in self.EXCHANGE or not library().gemm_mgpu_window_set_exchange(
                self.handle, self.EXCHANGE[mode]):
            raise InvalidArgumentException("unknown exchange mode %r" % (mode,))

    def result(self):
        """The window as a torch view (float64 [M, N]); valid after a fused call."""
        torch = _torch()
        n = self.M * self.N
        holder = _CudaPointer(self.local, n * 8)
        return torch.as_tensor(holder, device="cuda").view(torch.float64)[:n].view(self.M, self.N)

    def close(self):
        if self.handle:
            library().gemm_mgpu_window_destroy(self.handle)
            self.handle = None


class _CudaPointer:
    """__cuda_array_interface__ over raw device memory (bytes)."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1",
                                         "data": (ptr, False), "version": 3}


def nsplit_matmul_fused(window, a, b_local):
    """Fused N-split float64 product into `window` (every rank's copy)."""
    lib = library()
    M, K = a.getShape()
    es = 8
    ok = lib.gemm_mgpu_nsplit_matmul_fused(
        window.handle, DTYPE_CODES["float64"], a._storage.data_ptr() + a._offset * es,
        a._strides[0], a._strides[1], b_local._storage.data_ptr() + b_local._offset * es,
        b_local._strides[0], b_local._strides[1], M, window.N, K, current_stream())
    if not ok:
        raise RuntimeException("fused N-split matmul failed (status %d)"
                               % cuda_get_backend_info()["lastBlasStatus"])
    return window.result()
