"""GPU parity of libgemm_sm100.so against the CPU oracle (marked gpu).

Every product goes through the C ABI (phptensors.CudaArray.matmul ->
pt_tensor_matmul_into -> cuda_*_launcher).  Checks:
  * golden vectors of the reference's matmul tests, on the automatic kernel
    choice, with the tensor-core kernel forced, and with the CUDA-core kernel
    forced -- exact wherever the reference asserts exact values;
  * seeded random parity with the oracle at sizes it finishes in seconds:
    odd M/N/K, padded (TMA-aligned) and unaligned views, transposed operands,
    broadcast and rank-4 batches, for float16/bfloat16 (tolerance of the
    reference harness, tests/host_array_core_cuda.phpt:33, and normwise 1e-2),
    float32 (normwise 1e-5) and float64 (bit-exact: same fma order);
  * BASELINE config sizes through size-independent properties: integer-valued
    inputs make every summation order exact, so the full-size products must
    match bit for bit; random inputs are compared with the oracle on sampled
    output rows.
"""
import numpy as np
import pytest

import oracle_lib as O
import phptensors as P

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

TOL_ELEM = {"float64": 2e-12, "float16": 5e-3, "bfloat16": 3e-2, "float32": 3e-5}
TOL_NORM = {"float64": 1e-12, "float16": 1e-2, "bfloat16": 1e-2, "float32": 1e-5}
TORCH_DT = {"float32": torch.float32, "float64": torch.float64, "float16": torch.float16,
            "bfloat16": torch.bfloat16}


@pytest.fixture(autouse=True)
def _reset_path():
    prev = P.set_kernel_path("auto")
    P.cuda_set_matmul_precision("fp32-strict")
    yield
    P.library().gemm_sm100_set_path(prev)
    P.cuda_set_matmul_precision("fp32-strict")


def to_device(op, dtype):
    storage, shape, strides, offset = op
    s = np.ascontiguousarray(storage)
    if dtype in ("float16", "bfloat16"):
        t = torch.from_numpy(s.view(np.int16).copy()).view(TORCH_DT[dtype])
    else:
        t = torch.from_numpy(s.copy())
    return P.CudaArray(t.cuda(), shape, strides, offset, dtype)


def as_f64(storage, dtype):
    return O.to_float32(storage, dtype).astype(np.float64) if dtype != "float64" else storage


def check_close(gpu, ref, dtype, what):
    g = as_f64(gpu.reshape(-1), dtype)
    r = as_f64(ref.reshape(-1), dtype)
    assert g.shape == r.shape, what
    if g.size == 0:
        return
    assert np.all(np.abs(g - r) <= TOL_ELEM[dtype] * np.maximum(1.0, np.abs(r))), what
    norm = np.max(np.abs(g - r)) / max(1.0, np.max(np.abs(r)))
    assert norm <= TOL_NORM[dtype], (what, norm)


def check_fp32(gpu, a, b, what, first=None, count=None):
    """float32 acceptance: normwise rel-err <= 1e-5 against the oracle (the
    BASELINE bound) and, per element, |C - C_fp64| <= K * 2^-24 * (|A|.|B|)_ij,
    the classical error bound of a float32 dot product of length K, against
    the double twin of the oracle loop."""
    K = a[1][-1]
    th = O.oracle().orc_host_threads()
    aa, ab = O.absolute(a, "float32"), O.absolute(b, "float32")
    if first is None:
        ref = O.host_matmul(a, b, "float32", th).reshape(-1)
        c64 = O.host_matmul_f64(a, b, "float32", th).reshape(-1)
        absp = O.host_matmul_f64(aa, ab, "float32", th).reshape(-1)
    else:
        ref = O.host_matmul_range(a, b, "float32", first, count, th)
        c64 = O.host_matmul_f64_range(a, b, "float32", first, count, th)
        absp = O.host_matmul_f64_range(aa, ab, "float32", first, count, th)
    g = np.asarray(gpu, dtype=np.float64).reshape(-1)
    bound = K * 2.0 ** -24 * absp
    excess = np.abs(g - c64) - bound
    assert np.all(excess <= 1e-30), (what, float(np.max(np.abs(g - c64) / np.maximum(absp, 1e-30))))
    norm = np.max(np.abs(g - ref)) / max(1.0, np.max(np.abs(ref))) if ref.size else 0.0
    assert norm <= TOL_NORM["float32"], (what, norm)


# ------------------------------------------------------------------ golden
@pytest.mark.parametrize("path", ["auto", "tensor-core", "tensor-core-pair", "tensor-core-wide",
                                  "tensor-core-wide-halves", "simt"])
def test_golden_vectors(golden, path):
    P.set_kernel_path(path)
    for case in golden["cases"]:
        for dt in case["dtypes"]:
            a = to_device(O.golden_operand(case["a"], dt), dt)
            b = to_device(O.golden_operand(case["b"], dt), dt)
            c = a.matmul(b)
            assert c.getShape() == case["expect_shape"], case["name"]
            got = as_f64(c.to_numpy().reshape(-1), dt)
            exp = O.golden_expected(case)
            if case["tol"] is None:
                assert np.array_equal(got, exp), (case["name"], dt, path)
            else:
                assert np.max(np.abs(got - exp)) < case["tol"], (case["name"], dt, path)
            info = P.cuda_get_backend_info()
            if got.size:
                family = "builtin" if dt == "float32" else "builtin-low-precision"
                assert info["lastMatmul"] == family
                if path == "simt":
                    assert info["kernel"].startswith("simt-")
    assert P.device_status() == 0


def test_golden_tensor_core_kernel_is_used(golden):
    """Cases whose layouts TMA can describe really run on tcgen05."""
    P.set_kernel_path("tensor-core")
    names = {"accel_batched": "float32", "accel_broadcast": "float32", "accel_rank4": "float32",
             "accel_transposed_view": "float32", "lowp_identity": "bfloat16",
             "fusion_workspace_parallel_x2": "float32"}
    for case in golden["cases"]:
        if case["name"] in names:
            dt = names[case["name"]]
            a = to_device(O.golden_operand(case["a"], dt), dt)
            b = to_device(O.golden_operand(case["b"], dt), dt)
            got = as_f64(a.matmul(b).to_numpy().reshape(-1), dt)
            assert np.array_equal(got, O.golden_expected(case)), case["name"]
            assert P.cuda_get_backend_info()["kernel"].startswith("tc-"), case["name"]


def test_reference_rejections(golden):
    for r in golden["rejects"]:
        dt = r["dtype"]
        a = P.CudaArray.ones(r["a_shape"], dt)
        b = P.CudaArray.ones(r["b_shape"], dt)
        with pytest.raises(P.InvalidArgumentException) as e:
            a.matmul(b)
        assert "matmul" in str(e.value) or "Matrix multiplication" in str(e.value)


# ------------------------------------------------------------------ seeded parity
def padded(values, shape, row_pad, dtype, transpose=False):
    """A [.., R, C] operand stored with a padded row stride (TMA-aligned), or
    its transposed view when transpose=True (storage is [.., C, R])."""
    *batch, R, C = shape
    if transpose:
        R, C = C, R
    ld = C + row_pad
    nb = int(np.prod(batch)) if batch else 1
    buf = np.zeros((nb, R, ld), dtype=np.float32)
    buf[:, :, :C] = values.reshape(nb, R, C)
    storage = O.to_storage(buf.reshape(-1), dtype)
    strides = []
    s = R * ld
    for d in reversed(batch):
        strides.insert(0, s)
        s *= d
    if transpose:
        return (storage, list(batch) + [C, R], strides + [1, ld], 0)
    return (storage, list(batch) + [R, C], strides + [ld, 1], 0)


CASES = [
    # (name, a_shape, b_shape, a_transposed, b_transposed, row padding)
    ("square", [256, 256], [256, 256], False, False, 0),
    ("odd_mnk", [131, 77], [77, 263], False, False, 0),
    ("odd_padded", [131, 77], [77, 263], False, False, 11),
    ("tiny", [1, 7], [7, 1], False, False, 0),
    ("skinny_k", [300, 8], [8, 520], False, False, 0),
    ("a_transposed", [200, 136], [136, 312], True, False, 0),
    ("b_transposed", [129, 264], [264, 257], False, True, 0),
    ("both_transposed", [96, 200], [200, 136], True, True, 0),
    ("batched", [5, 130, 72], [5, 72, 96], False, False, 0),
    ("broadcast_a", [1, 64, 136], [6, 136, 64], False, False, 0),
    ("broadcast_b", [3, 2, 136, 40], [2, 40, 264], False, False, 0),
    ("rank4_transposed", [2, 3, 72, 64], [2, 3, 64, 80], True, True, 0),
    ("long_k", [64, 4104], [4104, 48], False, False, 0),
    # few columns (N <= 32): the split-K kernel's layouts and ragged chunks
    ("few_cols", [300, 1000], [1000, 10], False, False, 0),
    ("few_cols_a_transposed", [200, 2050], [2050, 3], True, False, 0),
    ("few_cols_b_transposed", [65, 777], [777, 17], False, True, 3),
    ("few_cols_broadcast", [4, 70, 520], [1, 520, 6], True, False, 0),
    # M-contiguous A with a padded (16-byte) stride and M % 4 = 3: the vector
    # copies' partial row groups
    ("few_cols_a_t_ragged_m", [203, 600], [600, 12], True, False, 5),
]

SKINNY_CASES = [c for c in CASES if c[2][-1] <= 32 and c[2][-2] >= 128]


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("path", ["auto", "tensor-core", "tensor-core-pair", "tensor-core-wide",
                                  "tensor-core-wide-halves", "skinny"])
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_seeded_parity(case, path, dtype):
    name, ashape, bshape, at, bt, pad = case
    P.set_kernel_path(path)
    seed = sum(map(ord, name))
    av = O.seeded(ashape, seed, "normal")
    bv = O.seeded(bshape, seed + 1, "normal")
    a = padded(av, ashape, pad, dtype, at)
    b = padded(bv, bshape, pad, dtype, bt)
    c = to_device(a, dtype).matmul(to_device(b, dtype))
    what = (name, path, P.cuda_get_backend_info()["kernel"])
    if path.startswith(("tensor-core-pair", "tensor-core-wide")) and what[2].startswith("tc"):
        assert what[2].startswith("tc2-"), what
    if path.startswith("tensor-core-wide") and what[2].startswith("tc") and dtype != "float32":
        assert what[2].endswith("256x512"), what
    if path == "skinny" and case in SKINNY_CASES:
        assert what[2].startswith("skinny-"), what
    if dtype == "float32":
        check_fp32(c.to_numpy(), a, b, what)
    else:
        ref = O.host_matmul(a, b, dtype, threads=O.oracle().orc_host_threads())
        check_close(c.to_numpy(), ref, dtype, what)


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_float64_cuda_cores_bit_exact(case):
    """The CUDA-core kernel runs the oracle's fma sequence: identical bits."""
    name, ashape, bshape, at, bt, pad = case
    P.set_kernel_path("simt")
    av = O.seeded(ashape, 5, "uniform")
    bv = O.seeded(bshape, 6, "uniform")
    a = padded(av, ashape, pad, "float64", at)
    b = padded(bv, bshape, pad, "float64", bt)
    ref = O.host_matmul_f64(a, b, "float64", threads=O.oracle().orc_host_threads())
    c = to_device(a, "float64").matmul(to_device(b, "float64"), allow_float64=True)
    assert np.array_equal(c.to_numpy().reshape(-1), ref.reshape(-1)), name
    assert P.cuda_get_backend_info()["lastMatmul"] == "builtin-f64"
    assert P.cuda_get_backend_info()["kernel"] == "simt-f64"


def check_fp64(gpu, a, b, what, first=None, count=None):
    """float64 acceptance: normwise rel-err <= 1e-12 against the double twin of
    the oracle loop (BASELINE), and per element within 2*K*2^-53*(|A|.|B|)_ij,
    twice the classical float64 dot-product bound (both sides round)."""
    K = a[1][-1]
    th = O.oracle().orc_host_threads()
    aa, ab = O.absolute(a, "float64"), O.absolute(b, "float64")
    if first is None:
        ref = O.host_matmul_f64(a, b, "float64", th).reshape(-1)
        absp = O.host_matmul_f64(aa, ab, "float64", th).reshape(-1)
    else:
        ref = O.host_matmul_f64_range(a, b, "float64", first, count, th)
        absp = O.host_matmul_f64_range(aa, ab, "float64", first, count, th)
    g = np.asarray(gpu, dtype=np.float64).reshape(-1)
    assert np.all(np.abs(g - ref) <= 2 * K * 2.0 ** -53 * absp + 1e-300), what
    if ref.size:
        assert np.max(np.abs(g - ref)) / max(1.0, np.max(np.abs(ref))) <= TOL_NORM["float64"], what


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_float64_dmma(case):
    name, ashape, bshape, at, bt, pad = case
    P.set_kernel_path("tensor-core")
    av = O.seeded(ashape, 7, "uniform")
    bv = O.seeded(bshape, 8, "uniform")
    a = padded(av, ashape, pad, "float64", at)
    b = padded(bv, bshape, pad, "float64", bt)
    c = to_device(a, "float64").matmul(to_device(b, "float64"), allow_float64=True)
    assert P.cuda_get_backend_info()["kernel"] == "dmma-f64-128x128"
    check_fp64(c.to_numpy(), a, b, name)


def test_float64_half_tile_tail_is_bit_identical():
    """A launch whose last wave would be at most half full runs that wave's
    tiles as 128 x 64 halves.  Every output element sees the same k order in
    either width, so one 8192 x 1024 product (512 tiles: 444 full, 68 as
    halves on 148 SMs) equals, bit for bit, the same product as batch 0 of a
    2-batch launch (1024 tiles, no halves), and matches the oracle."""
    M, N, K = 8192, 1024, 512
    av = O.seeded([M, K], 60, "uniform").astype(np.float64)
    bv = O.seeded([K, N], 61, "uniform").astype(np.float64)
    a, b = O.dense(av, [M, K]), O.dense(bv, [K, N])
    single = to_device(a, "float64").matmul(to_device(b, "float64"), allow_float64=True)
    assert P.cuda_get_backend_info()["kernel"] == "dmma-f64-128x128"
    a2 = O.dense(np.concatenate([av, av]), [2, M, K])
    b2 = O.dense(np.concatenate([bv, bv]), [2, K, N])
    pair = to_device(a2, "float64").matmul(to_device(b2, "float64"), allow_float64=True)
    s_out = single.to_numpy().reshape(-1)
    p_out = pair.to_numpy().reshape(2, -1)
    assert np.array_equal(s_out, p_out[0]) and np.array_equal(s_out, p_out[1])
    for row in (0, 5000, M - 1):
        check_fp64(s_out[row * N:(row + 1) * N], a, b, row, row * N, N)


def test_config5b_fp64_full_size_sampled():
    """float64 [8192,8192] x [8192,8192], U[-1,1): the single-GPU product (each
    rank's N-split column block is a slice of it) on sampled rows."""
    n = 8192
    a = O.dense(O.seeded([n, n], 50, "uniform").astype(np.float64), [n, n])
    b = O.dense(O.seeded([n, n], 51, "uniform").astype(np.float64), [n, n])
    c = to_device(a, "float64").matmul(to_device(b, "float64"), allow_float64=True)
    assert P.cuda_get_backend_info()["kernel"] == "dmma-f64-128x128"
    out = c.to_numpy().reshape(-1)
    for row in (0, 4097, n - 1):
        check_fp64(out[row * n:(row + 1) * n], a, b, row, row * n, n)
    assert P.device_status() == 0


def test_fp32_strict_against_fp64_config1():
    """BASELINE config 1 on the GPU path: compared to the FP64 twin."""
    a = O.dense(O.seeded([512, 1024], 0), [512, 1024])
    b = O.dense(O.seeded([1024, 768], 1), [1024, 768])
    c64 = O.host_matmul_f64(a, b, "float32", threads=O.oracle().orc_host_threads())
    g = to_device(a, "float32").matmul(to_device(b, "float32")).to_numpy().astype(np.float64)
    assert P.cuda_get_backend_info()["kernel"] == "tc-3xtf32-128x128"
    assert np.max(np.abs(g - c64)) / max(1.0, np.max(np.abs(c64))) <= 1e-5
    check_fp32(g, a, b, "config1")


def test_tf32_mode_differs_but_stays_close():
    """tests/matmul_precision.phpt:26-53: TF32 != strict, within 2% of the
    max magnitude, and strict is bit-identical after switching back."""
    i = np.arange(65536, dtype=np.float64)
    left = (np.sin(i * 0.013) + 0.000123).astype(np.float32)
    right = (np.cos(i * 0.017) - 0.000321).astype(np.float32)
    a = P.CudaArray.fromFlatArray(left, [256, 256])
    b = P.CudaArray.fromFlatArray(right, [256, 256])
    P.set_kernel_path("tensor-core")
    strict = a.matmul(b).toBuffer()
    P.cuda_set_matmul_precision("tf32")
    assert P.cuda_get_backend_info()["precision"] == "tf32"
    fast = a.matmul(b).toBuffer()
    assert P.cuda_get_backend_info()["kernel"].startswith("tc-tf32")
    s = np.frombuffer(strict, np.float32).astype(np.float64)
    f = np.frombuffer(fast, np.float32).astype(np.float64)
    diff = np.max(np.abs(s - f))
    assert diff > 0.0 and diff <= 0.02 * max(1.0, np.max(np.abs(s)))
    P.cuda_set_matmul_precision("fp32-strict")
    assert a.matmul(b).toBuffer() == strict


def test_autotuning_schema():
    """tests/matmul_tuning.phpt:18-49 on this library's own configurations."""
    left, right = P.CudaArray.ones([256, 256]), P.CudaArray.ones([256, 256])
    t = P.cuda_tune_matmul(left, right)
    assert t["backend"] == "builtin" and t["precision"] == "fp32-strict"
    assert t["candidateCount"] > 0 and 0 <= t["selectedCandidate"] < t["candidateCount"]
    assert sum(c["selected"] for c in t["candidates"]) == 1
    for c in t["candidates"]:
        assert c["workspaceBytes"] == 0 and np.isfinite(c["medianMs"]) and c["medianMs"] > 0
    vals = np.frombuffer(t["product"].toBuffer(), np.float32)
    assert vals[0] == 256.0 and vals[-1] == 256.0
    prod = np.frombuffer(left.matmul(right).toBuffer(), np.float32)
    assert prod[0] == 256.0 and prod[-1] == 256.0
    assert P.cuda_get_backend_info()["lastMatmul"] == "builtin"
    with pytest.raises(P.InvalidArgumentException):
        P.cuda_tune_matmul(P.CudaArray.ones([32, 32]), P.CudaArray.ones([32, 32]))
    P.cuda_set_matmul_precision("tf32")
    t = P.cuda_tune_matmul(left, right)
    assert t["precision"] == "tf32" and t["candidateCount"] == 2


@pytest.mark.parametrize("case", SKINNY_CASES, ids=[c[0] for c in SKINNY_CASES])
def test_float64_skinny(case):
    name, ashape, bshape, at, bt, pad = case
    P.set_kernel_path("skinny")
    av = O.seeded(ashape, 9, "uniform")
    bv = O.seeded(bshape, 10, "uniform")
    a = padded(av, ashape, pad, "float64", at)
    b = padded(bv, bshape, pad, "float64", bt)
    c = to_device(a, "float64").matmul(to_device(b, "float64"), allow_float64=True)
    assert P.cuda_get_backend_info()["kernel"] == "skinny-f64"
    check_fp64(c.to_numpy(), a, b, name)


@pytest.mark.parametrize("dtype", ["bfloat16", "float32", "float64"])
def test_skinny_split_k_is_deterministic(dtype):
    """The split-K kernel adds its partial sums in a fixed order: repeated
    products are bit-identical, whatever the cluster size the launch picks."""
    P.set_kernel_path("skinny")
    g = torch.Generator(device="cuda").manual_seed(17)
    for M, N, K in ((1024, 10, 4096), (4096, 10, 1024), (33, 32, 40000), (5000, 1, 300),
                    (300, 14, 5000)):
        a = torch.randn(K, M, device="cuda", generator=g, dtype=torch.float64).to(TORCH_DT[dtype])
        b = torch.randn(K, N, device="cuda", generator=g, dtype=torch.float64).to(TORCH_DT[dtype])
        A = P.CudaArray.from_torch(a).transpose()
        B = P.CudaArray.from_torch(b)
        first = A.matmul(B, allow_float64=True).to_torch()
        assert P.cuda_get_backend_info()["kernel"].startswith("skinny-")
        for _ in range(3):
            assert torch.equal(A.matmul(B, allow_float64=True).to_torch(), first), (M, N, K)
        ref = a.double().t() @ b.double()
        err = ((first.double() - ref).abs().max() / ref.abs().max()).item()
        assert err <= {"bfloat16": 1e-2, "float32": 1e-5, "float64": 1e-12}[dtype], (M, N, K, err)
    assert P.device_status() == 0


PAIR_3X_CASES = [
    # (name, a_shape, b_shape, a_transposed, b_transposed): strict float32 on
    # the 2-CTA 3xTF32 kernel -- more tiles than co-resident clusters, ragged
    # K chunks, every operand layout, batches with broadcast
    ("more_tiles_than_clusters", [2048, 256], [256, 2560], False, False),
    ("ragged_chunks", [600, 520], [520, 700], False, False),
    ("a_transposed", [2048, 1000], [1000, 2048], True, False),
    ("b_transposed", [300, 392], [392, 520], False, True),
    ("both_transposed", [2048, 200], [200, 2048], True, True),
    ("batched_broadcast", [3, 1, 260, 136], [2, 136, 264], False, False),
]


@pytest.mark.parametrize("case", PAIR_3X_CASES, ids=[c[0] for c in PAIR_3X_CASES])
def test_pair_3xtf32(case):
    """The 2-CTA 3xTF32 kernel against the oracle's float64 twin (per-element
    K-ulp bound and normwise 1e-5), bit-identical on repetition."""
    name, ashape, bshape, at, bt = case
    P.set_kernel_path("tensor-core-pair")
    seed = sum(map(ord, name))
    a = padded(O.seeded(ashape, seed, "normal"), ashape, 0, "float32", at)
    b = padded(O.seeded(bshape, seed + 1, "normal"), bshape, 0, "float32", bt)
    ad, bd = to_device(a, "float32"), to_device(b, "float32")
    c = ad.matmul(bd)
    # few tiles split K over clusters of 2 or 4 pairs, 64 tiles and more do not
    cluster = P.last_launch()[2]
    assert cluster in (2, 4, 8)
    # K-major A without split-K: A's hi and lo in tensor memory
    expect = "tc2-3xtf32-tmem-256x256" if not at and cluster == 2 else "tc2-3xtf32-256x256"
    assert P.cuda_get_backend_info()["kernel"] == expect, name
    first = c.to_numpy()
    check_fp32(first, a, b, name)
    for _ in range(2):
        assert np.array_equal(ad.matmul(bd).to_numpy(), first), name
    assert P.device_status() == 0


@pytest.mark.parametrize("case", PAIR_3X_CASES, ids=[c[0] for c in PAIR_3X_CASES])
def test_pair_tf32_mode(case):
    """The tf32 precision mode on the 2-CTA kernel: within the TF32 error
    bound of the float64 product (operands truncated to 10 mantissa bits,
    float32 accumulation) and bit-identical on repetition."""
    name, ashape, bshape, at, bt = case
    seed = sum(map(ord, name))
    a = padded(O.seeded(ashape, seed, "normal"), ashape, 0, "float32", at)
    b = padded(O.seeded(bshape, seed + 1, "normal"), bshape, 0, "float32", bt)
    ad, bd = to_device(a, "float32"), to_device(b, "float32")
    P.cuda_set_matmul_precision("tf32")
    P.set_kernel_path("tensor-core-pair")
    first = ad.matmul(bd).to_numpy().astype(np.float64).reshape(-1)
    assert P.cuda_get_backend_info()["kernel"] == "tc2-tf32-256x256", name
    assert np.array_equal(ad.matmul(bd).to_numpy().astype(np.float64).reshape(-1), first), name
    P.cuda_set_matmul_precision("fp32-strict")
    th = O.oracle().orc_host_threads()
    c64 = O.host_matmul_f64(a, b, "float32", th).reshape(-1)
    absp = O.host_matmul_f64(O.absolute(a, "float32"), O.absolute(b, "float32"), "float32",
                             th).reshape(-1)
    K = a[1][-1]
    bound = (2.0 ** -9 + K * 2.0 ** -23) * absp
    assert np.all(np.abs(first - c64) <= bound + 1e-30), name
    assert P.device_status() == 0


PAIR_SPLIT_CASES = [
    # (name, a_shape, b_shape, a_transposed, b_transposed, a dtype, b dtype,
    # expected cluster size = 2 x pairs splitting K)
    ("f32_dw_g4", [1024, 4096], [4096, 1024], True, False, "float32", "float32", 8),
    ("f32_ragged_g4", [300, 3000], [3000, 264], False, True, "float32", "float32", 8),
    ("f32_g2", [1280, 1024], [1024, 1536], False, False, "float32", "float32", 4),
    ("bf16xf32_dw_g4", [784, 4096], [4096, 1024], True, False, "bfloat16", "float32", 8),
    ("f32xbf16_g2", [1280, 1024], [1024, 1536], False, True, "float32", "bfloat16", 4),
]


@pytest.mark.parametrize("case", PAIR_SPLIT_CASES, ids=[c[0] for c in PAIR_SPLIT_CASES])
def test_pair_split_k(case):
    """Split-K on the 2-CTA split kernels: clusters of G pairs share a tile,
    the partial blocks are added over DSMEM in a fixed order -- within the
    float32 bound of the oracle and bit-identical from call to call."""
    name, ashape, bshape, at, bt, adt, bdt, cluster = case
    seed = sum(map(ord, name))
    a = padded(O.seeded(ashape, seed, "normal"), ashape, 0, adt, at)
    b = padded(O.seeded(bshape, seed + 1, "normal"), bshape, 0, bdt, bt)
    P.set_kernel_path("tensor-core-pair")
    if adt == bdt:
        ad, bd = to_device(a, adt), to_device(b, bdt)
        run = lambda: ad.matmul(bd).to_numpy()
    else:
        run = lambda: mixed_product(a, adt, b, bdt).to_numpy()
    first = run()
    what = (name, P.cuda_get_backend_info()["kernel"], P.last_launch())
    assert what[1].startswith("tc2-") and what[2][2] == cluster, what
    check_fp32(first, as_f32_op(a, adt), as_f32_op(b, bdt), what)
    for _ in range(2):
        assert np.array_equal(run(), first), name
    assert P.device_status() == 0


SPLIT_K_CASES = [
    # (name, a_shape, b_shape, a_transposed, b_transposed, dtype, expected cluster)
    ("splitk_fp32_g4", [256, 4096], [4096, 384], False, False, "float32", 4),
    ("splitk_fp32_batched_t", [3, 200, 2048], [3, 2048, 136], True, True, "float32", 4),
    ("splitk_fp32_g2", [784, 4096], [4096, 1024], True, False, "float32", 2),
    ("splitk_bf16_g2", [512, 8192], [8192, 512], False, False, "bfloat16", 2),
    ("splitk_f16_ragged", [300, 3000], [3000, 200], False, True, "float16", 2),
]


@pytest.mark.parametrize("case", SPLIT_K_CASES, ids=[c[0] for c in SPLIT_K_CASES])
def test_split_k_tensor_core(case):
    """Few tiles, long K: a cluster of CTAs splits K and adds the partial
    tiles over DSMEM in a fixed order -- within the dtype's bound of the
    oracle, and bit-identical from call to call."""
    name, ashape, bshape, at, bt, dtype, cluster = case
    P.set_kernel_path("tensor-core")
    seed = sum(map(ord, name))
    a = padded(O.seeded(ashape, seed, "normal"), ashape, 0, dtype, at)
    b = padded(O.seeded(bshape, seed + 1, "normal"), bshape, 0, dtype, bt)
    ad, bd = to_device(a, dtype), to_device(b, dtype)
    c = ad.matmul(bd)
    what = (name, P.cuda_get_backend_info()["kernel"], P.last_launch())
    assert what[1].startswith("tc-") and what[2][2] == cluster, what
    first = c.to_torch().clone()
    for _ in range(2):
        assert torch.equal(ad.matmul(bd).to_torch(), first), name
    M, N = ashape[-2], bshape[-1]
    rows = [0, M // 2, M - 1]
    nb = int(np.prod(ashape[:-2])) if len(ashape) > 2 else 1
    flat = c.to_numpy().reshape(nb, M, N)
    for bi in range(nb):
        for r in rows:
            first_i = (bi * M + r) * N
            if dtype == "float32":
                check_fp32(flat[bi, r], a, b, what, first_i, N)
            else:
                ref = O.host_matmul_range(a, b, dtype, first_i, N, O.oracle().orc_host_threads())
                check_close(flat[bi, r], ref, dtype, what)
    assert P.device_status() == 0


def test_split_k_fused_epilogue():
    """Bias and activation run once, on the reduced tile."""
    P.set_kernel_path("tensor-core")
    M, K, N = 256, 4096, 384
    av = O.seeded([M, K], 31, "uniform", -0.5, 0.5)
    xv = O.seeded([N, K], 32, "uniform", -0.5, 0.5)
    bias = O.seeded([N], 33, "normal", std=0.1)
    a = to_device(O.dense(O.to_storage(av, "float32"), [M, K]), "float32")
    x = to_device(O.dense(O.to_storage(xv, "float32"), [N, K]), "float32")
    bdev = to_device(O.dense(O.to_storage(bias, "float32"), [N]), "float32")
    fused = a.matmul_epilogue(x.transpose(), bdev, "tanh").to_torch()
    assert P.last_launch()[2] == 4
    plain = a.matmul(x.transpose()).to_torch()
    unfused = torch.tanh(plain + bdev.to_torch())
    assert torch.all((fused - unfused).abs() <= 2.0 ** -22 * unfused.abs().clamp(min=1.0))


# ------------------------------------------------------------------ epilogue
@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("act", ["tanh", "relu", "sigmoid", "none"])
@pytest.mark.parametrize("N", [328, 24])
def test_fused_epilogue_matches_unfused_plan(dtype, act, N):
    """act(round(A.B) + bias) equals the unfused matmul step followed by the
    elementwise step computed in float (src/fusion_codegen.c:3-27)."""
    M, K = 300, 264
    av = O.seeded([M, K], 21, "uniform", -0.5, 0.5)
    xv = O.seeded([N, K], 22, "uniform", -0.5, 0.5)
    bias = O.seeded([N], 23, "normal", std=0.1)
    a = to_device(O.dense(O.to_storage(av, dtype), [M, K]), dtype)
    x = to_device(O.dense(O.to_storage(xv, dtype), [N, K]), dtype)
    bdev = to_device(O.dense(O.to_storage(bias, dtype), [N]), dtype)
    for path in ("tensor-core", "tensor-core-pair", "tensor-core-wide", "tensor-core-wide-halves",
                 "simt") + (
            ("skinny",) if N <= 32 else ()):
        P.set_kernel_path(path)
        fused = a.matmul_epilogue(x.transpose(), bdev, act).to_torch().float()
        plain = a.matmul(x.transpose()).to_torch().float()
        t = plain + bdev.to_torch().float()
        t = {"tanh": torch.tanh, "relu": torch.relu, "sigmoid": torch.sigmoid,
             "none": lambda v: v}[act](t)
        unfused = t.to(TORCH_DT[dtype]).float()
        ulp = {"float16": 2.0 ** -10, "bfloat16": 2.0 ** -7, "float32": 2.0 ** -22}[dtype]
        assert torch.all((fused - unfused).abs() <= ulp * unfused.abs().clamp(min=1.0)), path


# ------------------------------------------------------------------ configs
@pytest.mark.parametrize("shape", [(640, 520, 300), (3, 1024, 1024, 1000), (2048, 2048, 4096)],
                         ids=["ragged", "batched", "long_k"])
def test_strict_pair_tmem_a_matches_smem_a(shape):
    """Strict float32 on the 2-CTA kernels: with K-major A the split puts A's
    hi and lo in tensor memory (tc2-3xtf32-tmem), with an M-major A view it
    stays in shared memory (tc2-3xtf32); both issue the same MMAs and add the
    K chunks in the same order, so the products are bit-identical, and within
    the float32 bound of the oracle.  (The shapes have enough tiles, or too
    short a K, for the forced pair path not to split K, which only the
    shared-memory kernel does.)"""
    *batch, M, N, K = shape
    P.set_kernel_path("tensor-core-pair")
    av = O.seeded(list(batch) + [M, K], 51, "normal")
    bv = O.seeded(list(batch) + [K, N], 52, "normal")
    a_k = padded(av, list(batch) + [M, K], 0, "float32")
    # the same matrix stored M-contiguous: storage [.., K, M] holds A^T
    av_t = np.swapaxes(np.asarray(av).reshape(list(batch) + [M, K]), -1, -2).reshape(-1)
    a_m = padded(av_t, list(batch) + [M, K], 0, "float32", transpose=True)
    b = padded(bv, list(batch) + [K, N], 0, "float32")
    bd = to_device(b, "float32")
    c_k = to_device(a_k, "float32").matmul(bd)
    k_kernel = P.cuda_get_backend_info()["kernel"]
    c_m = to_device(a_m, "float32").matmul(bd)
    m_kernel = P.cuda_get_backend_info()["kernel"]
    assert k_kernel == "tc2-3xtf32-tmem-256x256", k_kernel
    assert m_kernel == "tc2-3xtf32-256x256", m_kernel
    assert np.array_equal(c_k.to_numpy().view(np.uint32), c_m.to_numpy().view(np.uint32))
    if len(batch) == 0 and K <= 1024:
        check_fp32(c_k.to_numpy(), a_k, b, ("tmem-a", shape))
    assert P.device_status() == 0


def test_config2_full_size_integer_exact():
    """bf16 [64,1024,1024] x [64,1024,1024]: with small-integer inputs every
    partial sum is exact in float32, so the product must be bit-identical to
    the exact product rounded once to bfloat16 (what the oracle computes)."""
    g = torch.Generator().manual_seed(2)
    a = torch.randint(-3, 4, (64, 1024, 1024), generator=g).to(torch.bfloat16)
    b = torch.randint(-3, 4, (64, 1024, 1024), generator=g).to(torch.bfloat16)
    exact = torch.bmm(a.double().cuda(), b.double().cuda()).float().to(torch.bfloat16)
    for path, prefix in (("auto", "tc"), ("tensor-core", "tc-bf16"), ("tensor-core-pair", "tc2-bf16"),
                         ("tensor-core-wide", "tc2-bf16-256x512"),
                         ("tensor-core-wide-halves", "tc2-bf16-256x512")):
        P.set_kernel_path(path)
        c = P.CudaArray.from_torch(a.cuda()).matmul(P.CudaArray.from_torch(b.cuda()))
        assert P.cuda_get_backend_info()["kernel"].startswith(prefix), path
        assert torch.equal(c.to_torch().view(torch.int16), exact.view(torch.int16)), path
    assert P.device_status() == 0


def test_config2_random_sampled_rows():
    """bf16 N(0,1) [64,1024,1024]^2 against the oracle on sampled rows."""
    M = N = K = 1024
    batches = 64
    av = O.seeded([batches, M, K], 0, "normal")
    bv = O.seeded([batches, K, N], 1, "normal")
    a = O.dense(O.to_storage(av, "bfloat16"), [batches, M, K])
    b = O.dense(O.to_storage(bv, "bfloat16"), [batches, K, N])
    c = to_device(a, "bfloat16").matmul(to_device(b, "bfloat16")).to_numpy().reshape(-1)
    threads = O.oracle().orc_host_threads()
    for batch in (0, 17, 63):
        for row in (0, 511, 1023):
            first = (batch * M + row) * N
            ref = O.host_matmul_range(a, b, "bfloat16", first, N, threads)
            check_close(c[first:first + N], ref, "bfloat16", (batch, row))


@pytest.mark.parametrize("path", ["auto", "tensor-core-pair", "tensor-core-wide"])
def test_config3_fp16_transposed_bias_tanh(path):
    """fp16 A[8192,4096] . X^T (X [4096,4096] row-major) + bias[4096], tanh:
    fused epilogue vs the unfused plan over the whole output, and the product
    vs the oracle on sampled rows."""
    P.set_kernel_path(path)
    M, K, N = 8192, 4096, 4096
    av = O.seeded([M, K], 30, "uniform", -0.5, 0.5)
    xv = O.seeded([N, K], 31, "uniform", -0.5, 0.5)
    bias = O.seeded([N], 32, "normal", std=0.1)
    a_op = O.dense(O.to_storage(av, "float16"), [M, K])
    x_op = O.dense(O.to_storage(xv, "float16"), [N, K])
    a, x = to_device(a_op, "float16"), to_device(x_op, "float16")
    bdev = to_device(O.dense(O.to_storage(bias, "float16"), [N]), "float16")
    fused = a.matmul_epilogue(x.transpose(), bdev, "tanh")
    kernel = P.cuda_get_backend_info()["kernel"]
    assert kernel.startswith(("tc-f16", "tc2-f16")), kernel
    # automatic choice: 256 x 4096 / 512 = 256 wide tiles are 3.5 rounds of
    # the 74 co-resident clusters, so the wide kernel runs 3 rounds of whole
    # tiles and the rest as 256-column halves
    assert kernel == {"auto": "tc2-f16-256x512", "tensor-core-pair": "tc2-f16-256x256",
                      "tensor-core-wide": "tc2-f16-256x512"}[path], kernel
    plain = a.matmul(x.transpose())
    assert P.cuda_get_backend_info()["kernel"] == kernel
    unfused = torch.tanh(plain.to_torch().float() + bdev.to_torch().float()).half().float()
    assert torch.all((fused.to_torch().float() - unfused).abs() <= 2.0 ** -10)
    c = plain.to_numpy().reshape(-1)
    xt = (x_op[0], [K, N], [1, K], 0)
    threads = O.oracle().orc_host_threads()
    for row in (0, 4095, 8191):
        ref = O.host_matmul_range(a_op, xt, "float16", row * N, N, threads)
        check_close(c[row * N:(row + 1) * N], ref, "float16", row)


# ------------------------------------------------------------------ gradients
def as_f32_op(op, dtype):
    """The same view over an exact float32 copy of the storage (what the
    reference's gradient_cast produces, src/autograd.c:683-712)."""
    storage, shape, strides, offset = op
    return (O.to_float32(storage, dtype).astype(np.float32), shape, strides, offset)


def mixed_product(a_op, a_dt, b_op, b_dt):
    """C (float32) = A . B through cuda_mixed_matmul_nd_launcher."""
    import ctypes
    ad, bd = to_device(a_op, a_dt), to_device(b_op, b_dt)
    M, N = a_op[1][-2], b_op[1][-1]
    batch = []
    for x, y in zip([1] * (max(len(a_op[1]), len(b_op[1])) - len(a_op[1])) + list(a_op[1][:-2]),
                    [1] * (max(len(a_op[1]), len(b_op[1])) - len(b_op[1])) + list(b_op[1][:-2])):
        batch.append(max(x, y))
    c = P.CudaArray.zeros(batch + [M, N])
    pa, pb, pc = ad._pt(), bd._pt(), c._pt()
    ok = P.library().cuda_mixed_matmul_nd_launcher(
        pa.data, P.DTYPE_CODES[a_dt], pb.data, P.DTYPE_CODES[b_dt], pc.data,
        pa.shape, pa.strides, pa.ndims, pb.shape, pb.strides, pb.ndims,
        pc.shape, pc.strides, pc.ndims, P.current_stream())
    assert ok, P.cuda_get_backend_info()
    return c


MIXED_CASES = [
    # (name, a_shape, b_shape, a_transposed, b_transposed, a dtype, b dtype, tensor-core kernel)
    ("f32_bf16_kk", [300, 520], [520, 264], False, True, "float32", "bfloat16", "tc-f32xbf16"),
    ("f32_bf16_mn", [300, 520], [520, 264], True, False, "float32", "bfloat16", "tc-f32xbf16"),
    ("f32_bf16_km", [257, 1000], [1000, 136], False, False, "float32", "bfloat16", "tc-f32xbf16"),
    ("bf16_f32_mm", [264, 704], [704, 392], True, False, "bfloat16", "float32", "tc-bf16xf32"),
    ("bf16_f32_kk", [264, 704], [704, 392], False, True, "bfloat16", "float32", "tc-bf16xf32"),
    ("bf16_f32_batched", [3, 200, 136], [136, 264], True, False, "bfloat16", "float32", "tc-bf16xf32"),
    ("bf16_bf16", [256, 512], [512, 384], False, False, "bfloat16", "bfloat16", "tc-bf16-f32out"),
    ("f16_f16", [256, 512], [512, 384], False, True, "float16", "float16", "tc-f16-f32out"),
    ("f32_f16_simt", [130, 300], [300, 70], False, False, "float32", "float16", "simt-"),
    ("f32_bf16_short_k", [200, 8], [8, 136], False, True, "float32", "bfloat16", "simt-"),
    ("bf16_f32_few_cols", [1024, 4096], [4096, 10], True, False, "bfloat16", "float32", "skinny-"),
    ("f32_f16_few_cols", [300, 1000], [1000, 6], False, False, "float32", "float16", "skinny-"),
]


@pytest.mark.parametrize("case", MIXED_CASES, ids=[c[0] for c in MIXED_CASES])
def test_mixed_precision_products(case):
    """float32 result from a float32 and a 16-bit operand (or two 16-bit
    operands) without a float32 copy: within the float32 bound of the oracle
    run on the exact float32 upcast."""
    name, ashape, bshape, at, bt, adt, bdt, kernel = case
    seed = sum(map(ord, name))
    a = padded(O.seeded(ashape, seed, "normal"), ashape, 0, adt, at)
    b = padded(O.seeded(bshape, seed + 1, "normal"), bshape, 0, bdt, bt)
    c = mixed_product(a, adt, b, bdt)
    got = P.cuda_get_backend_info()["kernel"]
    assert got.startswith(kernel), (name, got)
    check_fp32(c.to_numpy(), as_f32_op(a, adt), as_f32_op(b, bdt), (name, got))
    assert P.device_status() == 0


MIXED_PAIR_CASES = [c[:7] for c in MIXED_CASES[:6]] + [
    ("f32_bf16_ragged_chunks", [1100, 1300], [1300, 2104], False, False, "float32", "bfloat16"),
    ("bf16_f32_more_tiles_than_clusters", [2560, 520], [520, 2048], True, False, "bfloat16",
     "float32"),
]


@pytest.mark.parametrize("case", MIXED_PAIR_CASES, ids=[c[0] for c in MIXED_PAIR_CASES])
def test_mixed_precision_pair(case):
    """The mixed float32 x bf16 kinds on the 2-CTA bf16x3 kernel: within the
    float32 bound of the oracle on the exact float32 upcast, bit-identical on
    repetition."""
    name, ashape, bshape, at, bt, adt, bdt = case
    seed = sum(map(ord, name))
    a = padded(O.seeded(ashape, seed, "normal"), ashape, 0, adt, at)
    b = padded(O.seeded(bshape, seed + 1, "normal"), bshape, 0, bdt, bt)
    P.set_kernel_path("tensor-core-pair")
    c = mixed_product(a, adt, b, bdt)
    got = P.cuda_get_backend_info()["kernel"]
    assert got == ("tc2-f32xbf16-bf16x3-256x256" if adt == "float32"
                   else "tc2-bf16xf32-bf16x3-256x256"), (name, got)
    first = c.to_numpy()
    check_fp32(first, as_f32_op(a, adt), as_f32_op(b, bdt), (name, got))
    assert np.array_equal(mixed_product(a, adt, b, bdt).to_numpy(), first), name
    assert P.device_status() == 0


def _backward(a, b, gc, ga, gb):
    import ctypes
    rc = P.library().pt_tensor_matmul_backward(
        ctypes.byref(a._pt()), ctypes.byref(b._pt()), ctypes.byref(gc._pt()),
        ctypes.byref(ga._pt()) if ga is not None else None,
        ctypes.byref(gb._pt()) if gb is not None else None, P.current_stream())
    assert rc == P.PT_OK, P.library().pt_last_error()


def test_backward_under_graph_capture():
    """Both gradients run on a side stream forked from the caller's stream and
    joined back; a CUDA graph captures the fork and join and its replay
    equals the eager result."""
    ashape, bshape = [3, 200, 136], [136, 264]
    a = O.dense(O.to_storage(O.seeded(ashape, 91, "normal"), "bfloat16"), ashape)
    b = O.dense(O.to_storage(O.seeded(bshape, 92, "normal"), "bfloat16"), bshape)
    g = O.dense(O.seeded([3, 200, 264], 93, "normal"), [3, 200, 264])
    ad, bd, gd = to_device(a, "bfloat16"), to_device(b, "bfloat16"), to_device(g, "float32")
    ga0, gb0 = P.CudaArray.zeros(ashape), P.CudaArray.zeros(bshape)
    _backward(ad, bd, gd, ga0, gb0)
    ga, gb = P.CudaArray.zeros(ashape), P.CudaArray.zeros(bshape)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _backward(ad, bd, gd, ga, gb)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        _backward(ad, bd, gd, ga, gb)
    ga.to_torch().zero_()
    gb.to_torch().zero_()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(ga.to_torch(), ga0.to_torch())
    assert torch.equal(gb.to_torch(), gb0.to_torch())
    del graph
    assert P.device_status() == 0


@pytest.mark.parametrize("dt,gdt", [("bfloat16", "float32"), ("bfloat16", "bfloat16"),
                                    ("float16", "float32")])
def test_backward_low_precision_operands(dt, gdt):
    """src/autograd.c:1547-1577 for 16-bit operands: float32 gradients of the
    float32-cast operands, here computed without the casts."""
    M, K, N = 384, 520, 264
    a = O.dense(O.to_storage(O.seeded([M, K], 51, "normal"), dt), [M, K])
    b = O.dense(O.to_storage(O.seeded([K, N], 52, "normal"), dt), [K, N])
    gc = O.dense(O.to_storage(O.seeded([M, N], 53, "normal"), gdt), [M, N])
    ga, gb = P.CudaArray.zeros([M, K]), P.CudaArray.zeros([K, N])
    _backward(to_device(a, dt), to_device(b, dt), to_device(gc, gdt), ga, gb)
    af, bf, gf = as_f32_op(a, dt), as_f32_op(b, dt), as_f32_op(gc, gdt)
    bt = (bf[0], [N, K], [1, N], 0)
    at = (af[0], [K, M], [1, K], 0)
    check_fp32(ga.to_numpy(), gf, bt, ("dA", dt, gdt))
    check_fp32(gb.to_numpy(), at, gf, ("dB", dt, gdt))


@pytest.mark.parametrize("dt", ["float32", "bfloat16"])
def test_backward_broadcast_reduction_fused(dt):
    """A shared weight (rank 2) under a batched input: its gradient, requested
    in the weight's own shape, is the product summed over the batch
    (src/autograd.c:714-760).  dB folds the batch into one GEMM's inner axis;
    dA of a broadcast A goes through the scratch product and the fixed-order
    reduction."""
    Bt, M, K, N = 3, 200, 136, 264
    # dB fused by folding: A [Bt, M, K] contiguous, B [K, N] broadcast
    a = O.dense(O.to_storage(O.seeded([Bt, M, K], 61, "normal"), dt), [Bt, M, K])
    b = O.dense(O.to_storage(O.seeded([K, N], 62, "normal"), dt), [K, N])
    gc = O.dense(O.seeded([Bt, M, N], 63, "normal"), [Bt, M, N])
    gb = P.CudaArray.zeros([K, N])
    ga = P.CudaArray.zeros([Bt, M, K])
    _backward(to_device(a, dt), to_device(b, dt), to_device(gc, "float32"), ga, gb)
    af, bf = as_f32_op(a, dt), as_f32_op(b, dt)
    # reference dB: the same sum as one product over the folded (batch, M) axis
    a_fold_t = (af[0], [K, Bt * M], [1, K], 0)
    gc_fold = (gc[0], [Bt * M, N], [N, 1], 0)
    check_fp32(gb.to_numpy(), a_fold_t, gc_fold, ("dB folded", dt))
    check_fp32(ga.to_numpy(), gc, (bf[0], [N, K], [1, N], 0), ("dA batched", dt))

    # dA of a broadcast A: A [M, K], B [Bt, K, N]
    a2 = O.dense(O.to_storage(O.seeded([M, K], 64, "normal"), dt), [M, K])
    b2 = O.dense(O.to_storage(O.seeded([Bt, K, N], 65, "normal"), dt), [Bt, K, N])
    ga2 = P.CudaArray.zeros([M, K])
    _backward(to_device(a2, dt), to_device(b2, dt), to_device(gc, "float32"), ga2, None)
    b2f = as_f32_op(b2, dt)
    th = O.oracle().orc_host_threads()
    ref = np.zeros(M * K)
    absp = np.zeros(M * K)
    for i in range(Bt):
        gci = (gc[0][i * M * N:(i + 1) * M * N].copy(), [M, N], [N, 1], 0)
        bti = (b2f[0][i * K * N:(i + 1) * K * N].copy(), [N, K], [1, N], 0)
        ref += O.host_matmul_f64(gci, bti, "float32", th).reshape(-1)
        absp += O.host_matmul_f64(O.absolute(gci, "float32"), O.absolute(bti, "float32"),
                                  "float32", th).reshape(-1)
    got = ga2.to_numpy().reshape(-1).astype(np.float64)
    ratio = np.abs(got - ref) / (Bt * N * 2.0 ** -24 * absp + 1e-30)
    assert np.all(ratio <= 1.0), (dt, P.cuda_get_backend_info()["kernel"], float(ratio.max()),
                                  int(np.argmax(ratio)), int(np.sum(ratio > 0.1)))
    assert np.max(np.abs(got - ref)) / max(1.0, np.max(np.abs(ref))) <= 1e-5
    assert P.device_status() == 0


FOLD_CASES = [
    # (name, a_shape, b_shape, gradient of, dtype): the gradient tensor has the
    # operand's own shape, the product's batch axes where it has extent 1 are summed
    ("keep1_sum0", [2, 3, 96, 136], [1, 3, 136, 80], "b", "float32"),
    ("sum_all_dA", [200, 136], [3, 136, 264], "a", "bfloat16"),
    ("odd_n_cuda_cores", [4, 70, 33], [1, 33, 29], "b", "float32"),
    ("split_k_fold", [8, 512, 256], [256, 128], "b", "float32"),
    ("f16_sum", [5, 64, 72], [72, 48], "b", "float16"),
]


@pytest.mark.parametrize("path", ["auto", "tensor-core-pair"])
@pytest.mark.parametrize("case", FOLD_CASES, ids=[c[0] for c in FOLD_CASES])
def test_backward_gradient_folded_into_the_product(case, path):
    """A gradient requested in its operand's shape when the product broadcast
    that operand: the summed batch axes run inside the product kernel.
    Checked against the exact float64 sum of the per-batch products, and
    bit-identical on repetition."""
    name, ashape, bshape, which, dt = case
    seed = sum(map(ord, name))
    a = O.dense(O.to_storage(O.seeded(ashape, seed, "normal"), dt), ashape)
    b = O.dense(O.to_storage(O.seeded(bshape, seed + 1, "normal"), dt), bshape)
    nb = max(len(ashape), len(bshape)) - 2
    full = [max(x, y) for x, y in zip([1] * (nb - len(ashape) + 2) + ashape[:-2],
                                      [1] * (nb - len(bshape) + 2) + bshape[:-2])]
    M, K, N = ashape[-2], ashape[-1], bshape[-1]
    gshape = full + [M, N]
    gc = O.dense(O.seeded(gshape, seed + 2, "normal"), gshape)
    target = ashape if which == "a" else bshape
    P.set_kernel_path(path)
    out = [P.CudaArray.zeros(target) for _ in range(3)]
    ad, bd, gd = to_device(a, dt), to_device(b, dt), to_device(gc, "float32")
    for o in out:
        _backward(ad, bd, gd, o if which == "a" else None, o if which == "b" else None)
    first = out[0].to_torch()
    assert all(torch.equal(o.to_torch(), first) for o in out[1:]), name
    # exact reference: float64 per-batch products summed over the reduced axes
    A = torch.from_numpy(O.to_float32(a[0], dt).astype(np.float64)).reshape(ashape)
    B = torch.from_numpy(O.to_float32(b[0], dt).astype(np.float64)).reshape(bshape)
    G = torch.from_numpy(gc[0].astype(np.float64)).reshape(gshape)
    if which == "a":
        prod, absp = G @ B.transpose(-1, -2), G.abs() @ B.abs().transpose(-1, -2)
        inner = N
    else:
        prod, absp = A.transpose(-1, -2) @ G, A.abs().transpose(-1, -2) @ G.abs()
        inner = M
    lead = len(gshape) - len(target)
    dims = tuple(range(lead)) + tuple(lead + i for i, e in enumerate(target[:-2]) if e == 1)
    ref = prod.sum(dim=dims, keepdim=False).reshape(target)
    refabs = absp.sum(dim=dims, keepdim=False).reshape(target)
    folds = int(np.prod(gshape[:-2])) // max(1, int(np.prod(target[:-2])))
    got = first.double().cpu()
    bound = folds * inner * 2.0 ** -24 * refabs
    assert torch.all((got - ref).abs() <= bound + 1e-30), (name, P.cuda_get_backend_info()["kernel"])
    assert float((got - ref).abs().max() / max(1.0, float(ref.abs().max()))) <= 1e-5, name
    assert P.device_status() == 0


def test_config4_mlp_forward_backward_fp32():
    """float32 MLP 784->1024->1024->10, batch 4096: forward GEMMs and the
    backward pair dA = dC.B^T, dB = A^T.dC of every layer (transposed views),
    each against the oracle (sampled rows for the large ones)."""
    batch, dims = 4096, [784, 1024, 1024, 10]
    rng_seed = 40
    x = O.seeded([batch, dims[0]], rng_seed, "uniform", 0.0, 1.0)
    h = O.dense(x, [batch, dims[0]])
    threads = O.oracle().orc_host_threads()
    lib = P.library()
    for layer in range(3):
        fan_in, fan_out = dims[layer], dims[layer + 1]
        w = O.dense(O.seeded([fan_in, fan_out], rng_seed + 1 + layer, "normal",
                             std=1.0 / np.sqrt(fan_in)), [fan_in, fan_out])
        dc = O.dense(O.seeded([batch, fan_out], rng_seed + 10 + layer, "normal"),
                     [batch, fan_out])
        hd, wd, dcd = to_device(h, "float32"), to_device(w, "float32"), to_device(dc, "float32")
        out = hd.matmul(wd).to_numpy().reshape(batch, fan_out)
        for row in (0, batch - 1):
            check_fp32(out[row], h, w, ("fwd", layer), row * fan_out, fan_out)
        ga = P.CudaArray.zeros([batch, fan_in])
        gb = P.CudaArray.zeros([fan_in, fan_out])
        import ctypes
        rc = lib.pt_tensor_matmul_backward(ctypes.byref(hd._pt()), ctypes.byref(wd._pt()),
                                           ctypes.byref(dcd._pt()), ctypes.byref(ga._pt()),
                                           ctypes.byref(gb._pt()), P.current_stream())
        assert rc == P.PT_OK
        wt = (w[0], [fan_out, fan_in], [1, fan_out], 0)
        ht = (h[0], [fan_in, batch], [1, fan_in], 0)
        ga_h = ga.to_numpy().reshape(batch, fan_in)
        for row in (0, batch - 1):
            check_fp32(ga_h[row], dc, wt, ("dA", layer), row * fan_in, fan_in)
        gb_h = gb.to_numpy().reshape(fan_in, fan_out)
        for row in (0, fan_in - 1):
            check_fp32(gb_h[row], ht, dc, ("dB", layer), row * fan_out, fan_out)
        h = O.dense(out.reshape(-1).copy(), [batch, fan_out])
    assert P.device_status() == 0


def test_k_zero_and_empty_batch_on_device():
    a = P.CudaArray.zeros([2, 0])
    b = P.CudaArray.zeros([0, 3])
    assert a.matmul(b).toArray() == [[0.0, 0.0, 0.0], [0.0, 0.0, 0.0]]
    e = P.CudaArray.zeros([0, 2, 3]).matmul(P.CudaArray.ones([3, 2]))
    assert e.getShape() == [0, 2, 2]


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
@pytest.mark.parametrize("shared", [False, True])
def test_host_matmul_streams_equal_device_product(dtype, shared):
    """pt_host_matmul (host buffers in and out, chunked and overlapped) gives
    the same bits as the product of the same operands on the device."""
    tdt = TORCH_DT[dtype]
    g = torch.Generator().manual_seed(9)
    batches, M, N, K = 7, 200, 136, 264
    a = torch.randn(batches, M, K, generator=g).to(tdt).pin_memory()
    b = (torch.randn(K, N, generator=g) if shared
         else torch.randn(batches, K, N, generator=g)).to(tdt).pin_memory()
    c = torch.empty(batches, M, N, dtype=tdt).pin_memory()
    P.host_matmul(a, b, c, chunks=3)
    ref = P.CudaArray.from_torch(a.cuda()).matmul(P.CudaArray.from_torch(b.cuda())).to_torch()
    assert torch.equal(c, ref.cpu())
    with pytest.raises(P.InvalidArgumentException):
        P.host_matmul(a, b, torch.empty(batches, M, N + 1, dtype=tdt))


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_host_matmul_sharded_over_devices(dtype):
    """pt_host_matmul_sharded: the batch cut over every GPU of this process
    (one on a single-GPU box), chunks pipelined per device, against the CPU
    oracle (HostArray::matmul restated) on the same operands, every batch;
    a shared B reaches every device."""
    tdt = TORCH_DT[dtype]
    devices = list(range(torch.cuda.device_count()))
    batches, M, N, K = 9, 256, 264, 320

    def host(storage, shape):
        s = np.ascontiguousarray(storage)
        t = torch.from_numpy(s.view(np.int16).copy()).view(tdt) if dtype == "bfloat16" \
            else torch.from_numpy(s.copy())
        return t.reshape(shape).pin_memory()

    av = O.to_storage(O.seeded([batches, M, K], 12, "normal"), dtype)
    a = host(av, [batches, M, K])
    th = O.oracle().orc_host_threads()
    for shared in (False, True):
        bshape = [K, N] if shared else [batches, K, N]
        bv = O.to_storage(O.seeded(bshape, 13 + shared, "normal"), dtype)
        b = host(bv, bshape)
        c = torch.full((batches, M, N), float("nan"), dtype=tdt).pin_memory()
        P.host_matmul(a, b, c, chunks=2, devices=devices)
        torch.cuda.set_device(0)
        oa, ob = O.dense(av, [batches, M, K]), O.dense(bv, bshape)
        if dtype == "bfloat16":
            ref = O.host_matmul(oa, ob, dtype, th)
            check_close(c.view(torch.int16).numpy().view(np.uint16), ref, dtype,
                        ("sharded", shared))
        else:
            # float32: the K-ulp dot-product bound against the oracle's double twin
            check_fp32(c.numpy(), oa, ob, ("sharded", shared))
        assert torch.cuda.current_device() == 0


def test_bounded_wait_reports_timeout_and_context_survives():
    """Failure detection without a GPU fault: a warp waits, with the bounded
    mbarrier wait every tensor-core kernel uses, on a barrier nothing
    completes; after the 2 s limit the kernel records status 5 and returns,
    and the next product on the same context is correct."""
    P.device_status()   # clear
    assert P.library().gemm_sm100_selftest_wait_timeout(P.current_stream()) == 1
    assert P.device_status() == 5
    a = P.CudaArray.ones([256, 256])
    c = np.frombuffer(a.matmul(a).toBuffer(), np.float32)
    assert c[0] == 256.0 and c[-1] == 256.0
    assert P.device_status() == 0


# ------------------------------------------------------------------ randomized sweep
def _random_case(rng):
    """Random operand shapes with NumPy broadcasting, transposes and padding."""
    M, N, K = (int(rng.integers(1, 300)) for _ in range(3))
    nb = int(rng.integers(0, 3))
    batch = [int(rng.integers(1, 4)) for _ in range(nb)]
    a_batch = [d if rng.random() < 0.7 else 1 for d in batch]
    b_batch = [d if rng.random() < 0.7 else 1 for d in batch]
    if rng.random() < 0.3 and nb:
        b_batch = b_batch[int(rng.integers(0, nb + 1)):]   # B with fewer batch axes
    return (a_batch + [M, K], b_batch + [K, N], bool(rng.random() < 0.4),
            bool(rng.random() < 0.4), int(rng.choice([0, 0, 3, 8])))


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
@pytest.mark.parametrize("path", ["auto", "tensor-core", "tensor-core-pair", "tensor-core-wide",
                                  "tensor-core-wide-halves", "skinny"])
def test_randomized_products(dtype, path):
    """40 seeded random products per dtype and kernel path against the oracle."""
    rng = np.random.default_rng(sum(map(ord, dtype + path)))
    P.set_kernel_path(path)
    for i in range(40):
        ashape, bshape, at, bt, pad = _random_case(rng)
        a = padded(O.seeded(ashape, 1000 + i, "normal"), ashape, pad, dtype, at)
        b = padded(O.seeded(bshape, 2000 + i, "normal"), bshape, pad, dtype, bt)
        c = to_device(a, dtype).matmul(to_device(b, dtype))
        what = (dtype, path, i, ashape, bshape, at, bt, pad, P.cuda_get_backend_info()["kernel"])
        if dtype == "float32":
            check_fp32(c.to_numpy(), a, b, what)
        else:
            ref = O.host_matmul(a, b, dtype, threads=O.oracle().orc_host_threads())
            check_close(c.to_numpy(), ref, dtype, what)
    assert P.device_status() == 0


def test_randomized_gradients():
    """Seeded random backward nodes (float32 / bfloat16 operands, float32 or
    same-typed upstream, broadcast operands whose gradients are reduced)
    against exact float64 sums."""
    rng = np.random.default_rng(77)
    for i in range(30):
        dt = "bfloat16" if rng.random() < 0.5 else "float32"
        gdt = dt if rng.random() < 0.3 else "float32"
        ashape, bshape, _, _, _ = _random_case(rng)
        a = O.dense(O.to_storage(O.seeded(ashape, 3000 + i, "normal"), dt), ashape)
        b = O.dense(O.to_storage(O.seeded(bshape, 4000 + i, "normal"), dt), bshape)
        nb = max(len(ashape), len(bshape)) - 2
        full = [max(x, y) for x, y in zip([1] * (nb - len(ashape) + 2) + ashape[:-2],
                                          [1] * (nb - len(bshape) + 2) + bshape[:-2])]
        M, K, N = ashape[-2], ashape[-1], bshape[-1]
        gshape = full + [M, N]
        gc = O.dense(O.to_storage(O.seeded(gshape, 5000 + i, "normal"), gdt), gshape)
        ga, gb = P.CudaArray.zeros(ashape), P.CudaArray.zeros(bshape)
        _backward(to_device(a, dt), to_device(b, dt), to_device(gc, gdt), ga, gb)
        A = torch.from_numpy(O.to_float32(a[0], dt).astype(np.float64)).reshape(ashape)
        B = torch.from_numpy(O.to_float32(b[0], dt).astype(np.float64)).reshape(bshape)
        G = torch.from_numpy(O.to_float32(gc[0], gdt).astype(np.float64)).reshape(gshape)
        for got, prod, absp, target, inner in (
                (ga, G @ B.transpose(-1, -2), G.abs() @ B.abs().transpose(-1, -2), ashape, N),
                (gb, A.transpose(-1, -2) @ G, A.abs().transpose(-1, -2) @ G.abs(), bshape, M)):
            lead = len(gshape) - len(target)
            dims = tuple(range(lead)) + tuple(lead + j for j, e in enumerate(target[:-2])
                                              if e == 1 and gshape[lead + j] != 1)
            ref = (prod.sum(dim=dims) if dims else prod).reshape(target)
            refabs = (absp.sum(dim=dims) if dims else absp).reshape(target)
            folds = int(np.prod(gshape[:-2])) // max(1, int(np.prod(target[:-2])))
            g = got.to_torch().double().cpu()
            what = (i, dt, gdt, ashape, bshape, P.cuda_get_backend_info()["kernel"])
            assert torch.all((g - ref).abs() <= folds * inner * 2.0 ** -24 * refabs + 1e-30), what
    assert P.device_status() == 0
