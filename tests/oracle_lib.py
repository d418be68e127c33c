"""ctypes binding of the CPU oracle (oracle/liboracle.so) -- test infrastructure.

Used only by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg,
as the checker (and as the timed CPU baseline); never by the product path.
Also binds oracle/_ref/libref.so (the reference's own converters and shape
rule) when it has been built in this container.

Operands are (storage, shape, strides, offset) with storage a numpy array:
float32 / float64 values, or uint16 bit patterns for float16 / bfloat16.
"""
import ctypes
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE_SO = os.path.join(ROOT, "oracle", "liboracle.so")
REF_SO = os.path.join(ROOT, "oracle", "_ref", "libref.so")

MAX_DIMS = 10
CODES = {"float32": 0, "float64": 1, "float16": 11, "bfloat16": 12}
STORAGE = {"float32": np.float32, "float64": np.float64, "float16": np.uint16,
           "bfloat16": np.uint16}


class OrcTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int), ("ndims", ctypes.c_int),
                ("shape", ctypes.c_int * MAX_DIMS), ("strides", ctypes.c_size_t * MAX_DIMS)]


_ORC = None
_REF = None


def oracle():
    global _ORC
    if _ORC is None:
        if not os.path.exists(ORACLE_SO):
            import subprocess
            subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "oracle"],
                           check=True)
        lib = ctypes.CDLL(ORACLE_SO)
        P = ctypes.POINTER
        lib.orc_float_to_float16_bits.restype = ctypes.c_uint16
        lib.orc_float_to_float16_bits.argtypes = [ctypes.c_float]
        lib.orc_float16_bits_to_float.restype = ctypes.c_float
        lib.orc_float16_bits_to_float.argtypes = [ctypes.c_uint16]
        lib.orc_float_to_bfloat16_bits.restype = ctypes.c_uint16
        lib.orc_float_to_bfloat16_bits.argtypes = [ctypes.c_float]
        lib.orc_bfloat16_bits_to_float.restype = ctypes.c_float
        lib.orc_bfloat16_bits_to_float.argtypes = [ctypes.c_uint16]
        for name in ("orc_floats_to_float16", "orc_floats_to_bfloat16"):
            getattr(lib, name).argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
        for name in ("orc_float16_to_floats", "orc_bfloat16_to_floats"):
            getattr(lib, name).argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
        lib.orc_matmul_shape.argtypes = [P(ctypes.c_int), ctypes.c_int, P(ctypes.c_int),
                                         ctypes.c_int, P(ctypes.c_int), P(ctypes.c_int)]
        lib.orc_host_matmul.argtypes = [P(OrcTensor), P(OrcTensor), ctypes.c_void_p,
                                        P(ctypes.c_int), P(ctypes.c_int), ctypes.c_int]
        lib.orc_host_matmul_f64.argtypes = [P(OrcTensor), P(OrcTensor), ctypes.c_void_p,
                                            P(ctypes.c_int), P(ctypes.c_int), ctypes.c_int]
        lib.orc_host_matmul_range.argtypes = [P(OrcTensor), P(OrcTensor), ctypes.c_void_p,
                                              ctypes.c_size_t, ctypes.c_size_t, ctypes.c_int]
        lib.orc_host_matmul_f64_range.argtypes = [P(OrcTensor), P(OrcTensor), ctypes.c_void_p,
                                                  ctypes.c_size_t, ctypes.c_size_t, ctypes.c_int]
        lib.orc_host_threads.restype = ctypes.c_int
        _ORC = lib
    return _ORC


def reference():
    """The reference's own data_types.c + tensor_shape.h, or None if not built."""
    global _REF
    if _REF is None and os.path.exists(REF_SO):
        lib = ctypes.CDLL(REF_SO)
        P = ctypes.POINTER
        lib.float_to_float16_bits.restype = ctypes.c_uint16
        lib.float_to_float16_bits.argtypes = [ctypes.c_float]
        lib.float16_bits_to_float.restype = ctypes.c_float
        lib.float16_bits_to_float.argtypes = [ctypes.c_uint16]
        lib.float_to_bfloat16_bits.restype = ctypes.c_uint16
        lib.float_to_bfloat16_bits.argtypes = [ctypes.c_float]
        lib.bfloat16_bits_to_float.restype = ctypes.c_float
        lib.bfloat16_bits_to_float.argtypes = [ctypes.c_uint16]
        lib.ref_bulk_half_to_float_bits.argtypes = [ctypes.c_void_p, ctypes.c_void_p,
                                                    ctypes.c_size_t, ctypes.c_int]
        lib.ref_bulk_float_bits_to_half.argtypes = [ctypes.c_void_p, ctypes.c_void_p,
                                                    ctypes.c_size_t, ctypes.c_int]
        lib.ref_tensor_matmul_shape.argtypes = [P(ctypes.c_int), ctypes.c_int, P(ctypes.c_int),
                                                ctypes.c_int, P(ctypes.c_int), P(ctypes.c_int)]
        _REF = lib
    return _REF


# ------------------------------------------------------------------ converters
def ref_widen(bits, dtype):
    """Reference converter, half/bfloat16 bits -> float32 (raw bits kept)."""
    b = np.ascontiguousarray(bits, dtype=np.uint16)
    out = np.empty(b.shape, dtype=np.uint32)
    reference().ref_bulk_half_to_float_bits(b.ctypes.data, out.ctypes.data, b.size,
                                            1 if dtype == "bfloat16" else 0)
    return out.view(np.float32)


def ref_narrow(values, dtype):
    """Reference converter, float32 -> half/bfloat16 bits."""
    v = np.ascontiguousarray(values, dtype=np.float32)
    out = np.empty(v.shape, dtype=np.uint16)
    reference().ref_bulk_float_bits_to_half(v.ctypes.data, out.ctypes.data, v.size,
                                            1 if dtype == "bfloat16" else 0)
    return out


def to_storage(values_f32, dtype):
    """float32 values -> storage of `dtype` (RNE bits for float16/bfloat16)."""
    v = np.ascontiguousarray(values_f32, dtype=np.float32)
    if dtype == "float32":
        return v.copy()
    if dtype == "float64":
        return v.astype(np.float64)
    out = np.empty(v.shape, dtype=np.uint16)
    fn = oracle().orc_floats_to_float16 if dtype == "float16" else oracle().orc_floats_to_bfloat16
    fn(v.ctypes.data, out.ctypes.data, v.size)
    return out


def to_float32(storage, dtype):
    s = np.ascontiguousarray(storage)
    if dtype in ("float32", "float64"):
        return s.astype(np.float32) if dtype == "float32" else s
    out = np.empty(s.shape, dtype=np.float32)
    fn = oracle().orc_float16_to_floats if dtype == "float16" else oracle().orc_bfloat16_to_floats
    fn(s.ctypes.data, out.ctypes.data, s.size)
    return out


# ------------------------------------------------------------------ matmul
def _tensor(storage, shape, strides, offset, dtype):
    t = OrcTensor()
    t.data = storage.ctypes.data + offset * storage.itemsize
    t.dtype = CODES[dtype]
    t.ndims = len(shape)
    for i, (d, s) in enumerate(zip(shape, strides)):
        t.shape[i] = d
        t.strides[i] = s
    return t


def matmul_shape(a_shape, b_shape, lib=None):
    lib = lib or oracle()
    fn = lib.orc_matmul_shape if lib is oracle() else lib.ref_tensor_matmul_shape
    a = (ctypes.c_int * max(len(a_shape), 1))(*a_shape)
    b = (ctypes.c_int * max(len(b_shape), 1))(*b_shape)
    out = (ctypes.c_int * MAX_DIMS)()
    nd = ctypes.c_int(0)
    if not fn(a, len(a_shape), b, len(b_shape), out, ctypes.byref(nd)):
        return None
    return [out[i] for i in range(nd.value)]


def host_matmul(a, b, dtype, threads=1):
    """HostArray::matmul restated.  a, b: (storage, shape, strides, offset).
    Returns the result storage (shape from the shape rule) or None if the
    reference would throw."""
    ta = _tensor(*a, dtype)
    tb = _tensor(*b, dtype)
    shape = matmul_shape(a[1], b[1])
    if shape is None or dtype not in ("float32", "float16", "bfloat16"):
        return None
    out = np.zeros(int(np.prod(shape)), dtype=STORAGE[dtype])
    sh = (ctypes.c_int * MAX_DIMS)()
    nd = ctypes.c_int(0)
    ok = oracle().orc_host_matmul(ctypes.byref(ta), ctypes.byref(tb), out.ctypes.data, sh,
                                  ctypes.byref(nd), threads)
    if not ok:
        return None
    return out.reshape(shape)


def host_matmul_f64(a, b, dtype, threads=1):
    """Double-precision twin: float64 result of the same loop."""
    ta = _tensor(*a, dtype)
    tb = _tensor(*b, dtype)
    shape = matmul_shape(a[1], b[1])
    if shape is None:
        return None
    out = np.zeros(int(np.prod(shape)), dtype=np.float64)
    sh = (ctypes.c_int * MAX_DIMS)()
    nd = ctypes.c_int(0)
    if not oracle().orc_host_matmul_f64(ctypes.byref(ta), ctypes.byref(tb), out.ctypes.data, sh,
                                        ctypes.byref(nd), threads):
        return None
    return out.reshape(shape)


def host_matmul_range(a, b, dtype, first, count, threads):
    ta = _tensor(*a, dtype)
    tb = _tensor(*b, dtype)
    out = np.zeros(count, dtype=STORAGE[dtype])
    if not oracle().orc_host_matmul_range(ctypes.byref(ta), ctypes.byref(tb), out.ctypes.data,
                                          first, count, threads):
        raise ValueError("range outside the product")
    return out


def host_matmul_f64_range(a, b, dtype, first, count, threads):
    ta = _tensor(*a, dtype)
    tb = _tensor(*b, dtype)
    out = np.zeros(count, dtype=np.float64)
    if not oracle().orc_host_matmul_f64_range(ctypes.byref(ta), ctypes.byref(tb),
                                              out.ctypes.data, first, count, threads):
        raise ValueError("range outside the product")
    return out


def absolute(op, dtype):
    """The operand with every element replaced by its magnitude."""
    storage, shape, strides, offset = op
    if dtype in ("float16", "bfloat16"):
        s = storage & np.uint16(0x7fff)
    else:
        s = np.abs(storage)
    return (s, shape, strides, offset)


def dense(storage, shape):
    strides, s = [], 1
    for d in reversed(shape):
        strides.insert(0, s)
        s *= d
    return (np.ascontiguousarray(storage).reshape(-1), list(shape), strides, 0)


# ------------------------------------------------------------------ golden
def golden_storage(op, dtype):
    st = op["storage"]
    if isinstance(st, dict):
        vals = np.full(st["n"], st["fill"], dtype=np.float32)
    else:
        vals = np.asarray(st, dtype=np.float64).astype(np.float32)
    return to_storage(vals, dtype)


def golden_operand(op, dtype):
    return (golden_storage(op, dtype), list(op["shape"]), list(op["strides"]), int(op["offset"]))


def golden_expected(case):
    n = int(np.prod(case["expect_shape"])) if case["expect_shape"] else 1
    e = case["expect"]
    if isinstance(e, dict) and "fill" in e:
        return np.full(n, e["fill"], dtype=np.float64)
    if isinstance(e, dict) and "fill_pattern" in e:
        pat = np.asarray(e["fill_pattern"], dtype=np.float64)
        return np.tile(pat, n // len(pat))
    return np.asarray(e, dtype=np.float64)


# ------------------------------------------------------------------ seeded inputs
def seeded(shape, seed, dist="uniform", lo=-1.0, hi=1.0, std=1.0):
    """Documented generator: numpy PCG64 (np.random.default_rng(seed)), float64
    draws rounded to float32.  uniform[lo, hi) or normal(0, std)."""
    rng = np.random.default_rng(seed)
    n = int(np.prod(shape))
    if dist == "uniform":
        v = rng.uniform(lo, hi, n)
    else:
        v = rng.standard_normal(n) * std
    return v.astype(np.float32)
