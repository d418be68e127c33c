"""Generate tests/golden/matmul_golden.json from the reference's matmul tests.

The cases below restate, one by one, the matmul known-answer checks of
lcmialichi/php-gpu-tensors' own test files (cited per case as file:line).
Inputs are rebuilt from the literals or formulas those tests use; expected
values are the literals the tests assert (or, where a test computes its
expectation with its own PHP double loop, the same loop in Python floats).
The script reads nothing from the reference tree, so the fixture it writes is
self-contained and travels to the GPU box; rerun it after editing a case:

    python tests/golden/make_golden.py
"""
import json
import os

HERE = os.path.dirname(os.path.abspath(__file__))


def dense(shape, values, offset=0, storage=None):
    """A contiguous row-major operand (optionally an offset view of storage)."""
    strides, s = [], 1
    for d in reversed(shape):
        strides.insert(0, s)
        s *= d
    return {"shape": list(shape), "strides": strides, "offset": offset,
            "storage": list(storage if storage is not None else values)}


def fill(shape, value):
    n = 1
    for d in shape:
        n *= d
    op = dense(shape, [])
    op["storage"] = {"fill": value, "n": n}
    return op


def transposed(op):
    """The reference's zero-copy transpose() view: swap the last two axes."""
    t = dict(op)
    t["shape"] = op["shape"][:-2] + [op["shape"][-1], op["shape"][-2]]
    t["strides"] = op["strides"][:-2] + [op["strides"][-1], op["strides"][-2]]
    return t


def broadcast_to(op, shape):
    """HostArray::broadcastTo view: new leading axes and extent-1 axes get stride 0."""
    lead = len(shape) - len(op["shape"])
    strides = [0] * lead
    for d, (have, want) in enumerate(zip(op["shape"], shape[lead:])):
        strides.append(op["strides"][d] if have == want else 0)
    b = dict(op)
    b["shape"] = list(shape)
    b["strides"] = strides
    return b


def matmul_f64(a, b):
    """Plain float64 product of small dense nested lists (expectations only)."""
    return [[sum(a[i][k] * b[k][j] for k in range(len(b))) for j in range(len(b[0]))]
            for i in range(len(a))]


def flat(x):
    if isinstance(x, list):
        out = []
        for v in x:
            out.extend(flat(v))
        return out
    return [x]


CASES = []


def case(name, source, dtypes, a, b, expect_shape, expect=None, points=None,
         tol=None, gradient=None):
    CASES.append({
        "name": name, "source": source, "dtypes": dtypes, "a": a, "b": b,
        "expect_shape": expect_shape,
        "expect": expect,            # full flat expected values (exact unless tol)
        "points": points,            # [[index tuple], value] spot checks
        "tol": tol,                  # absolute tolerance, None = exact
        "gradient": gradient,        # autograd cases: which GEMM of the backward
    })


F32 = ["float32"]
LOW = ["float16", "bfloat16"]
ALL3 = ["float32", "float16", "bfloat16"]

# --- tests/ca_matmul.phpt -------------------------------------------------
case("ca_matmul_2d", "tests/ca_matmul.phpt:10-12", F32,
     dense([2, 2], [1, 2, 3, 4]), dense([2, 2], [5, 6, 7, 8]), [2, 2],
     expect=[19, 22, 43, 50])
case("ca_matmul_batched", "tests/ca_matmul.phpt:14-16", F32,
     dense([2, 2, 2], [1, 2, 3, 4, 2, 0, 1, 2]), dense([2, 2, 2], [5, 6, 7, 8, 1, 2, 3, 4]),
     [2, 2, 2], expect=[19, 22, 43, 50, 2, 4, 7, 10])

# --- tests/ca_matmul_accelerated.phpt -------------------------------------
case("accel_dot", "tests/ca_matmul_accelerated.phpt:10-12", F32,
     fill([1, 100000], 1.0), fill([100000, 1], 1.0), [1, 1], expect=[100000.0])
case("accel_transposed_view", "tests/ca_matmul_accelerated.phpt:14-17", F32,
     transposed(fill([64, 128], 1.0)), fill([64, 128], 1.0), [128, 128],
     expect={"fill": 64.0})
case("accel_batched", "tests/ca_matmul_accelerated.phpt:19-21", F32,
     fill([8, 64, 64], 1.0), fill([8, 64, 64], 1.0), [8, 64, 64], expect={"fill": 64.0})
case("accel_broadcast", "tests/ca_matmul_accelerated.phpt:23-25", F32,
     fill([1, 64, 64], 1.0), fill([8, 64, 64], 1.0), [8, 64, 64], expect={"fill": 64.0})
case("accel_rank4", "tests/ca_matmul_accelerated.phpt:27-29", F32,
     fill([2, 4, 64, 64], 1.0), fill([2, 4, 64, 64], 1.0), [2, 4, 64, 64],
     expect={"fill": 64.0})
left = [float((r + c * 2) % 7) for r in range(64) for c in range(128)]
right = [float((r * 3 + c) % 5) for r in range(64) for c in range(128)]
full = [[sum(left[i * 128 + r] * right[i * 128 + c] for i in range(64)) for c in range(128)]
        for r in range(128)]
case("accel_transposed_formula", "tests/ca_matmul_accelerated.phpt:31-48", F32,
     transposed(dense([64, 128], left)), dense([64, 128], right), [128, 128],
     expect=flat(full),
     points=[[[r, c], full[r][c]] for r, c in [(0, 0), (0, 127), (127, 0), (127, 127), (19, 73)]])

# --- tests/matmul_low_precision.phpt --------------------------------------
case("lowp_batched", "tests/matmul_low_precision.phpt:57-63", LOW,
     dense([2, 2, 2], [1, 2, 3, 4, 2, 0, 0, 2]), dense([2, 2, 1], [5, 6, 1, 2]), [2, 2, 1],
     expect=[17, 39, 2, 4])
case("lowp_broadcast", "tests/matmul_low_precision.phpt:65-73", LOW,
     dense([2, 1, 2, 2], [1, 2, 3, 4, 2, 0, 0, 2]), dense([1, 3, 2, 1], [5, 6, 1, 2, 2, 1]),
     [2, 3, 2, 1], expect=[17, 39, 5, 11, 4, 10, 10, 12, 2, 4, 4, 2])
ident = [1.0 if i == j else 0.0 for i in range(64) for j in range(64)]
case("lowp_identity", "tests/matmul_low_precision.phpt:80-84", LOW,
     fill([64, 64], 1.0), dense([64, 64], ident), [64, 64], expect={"fill": 1.0})
case("lowp_approximate", "tests/matmul_low_precision.phpt:86-93", LOW,
     dense([2, 2], [0.1, 0.2, 0.3, 0.4]), dense([2, 2], [0.5, 0.6, 0.7, 0.8]), [2, 2],
     expect=[0.19, 0.22, 0.43, 0.50], tol=0.005)
case("lowp_tracked_forward", "tests/matmul_low_precision.phpt:95-100", LOW,
     dense([1, 2], [1, 2]), dense([2, 1], [3, 4]), [1, 1], expect=[11])

# Backward GEMMs of matmul_low_precision.phpt run in float32 after the cast
# (src/autograd.c:1547-1551): dA = dC . B^T and dB = A^T . dC on views.
A1, B1 = dense([1, 2], [1, 2]), dense([2, 1], [3, 4])
dC1 = fill([1, 1], 1.0)
case("grad_scalar_dA", "tests/matmul_low_precision.phpt:101-103", F32,
     dC1, transposed(B1), [1, 2], expect=[3, 4], gradient="dA")
case("grad_scalar_dB", "tests/matmul_low_precision.phpt:104-106", F32,
     transposed(A1), dC1, [2, 1], expect=[1, 2], gradient="dB")
A2, B2 = dense([2, 2], [1, 2, 3, 4]), dense([2, 2], [5, 6, 7, 8])
dC2 = dense([2, 2], [1, 0, 0, 1])
case("grad_seeded_dA", "tests/matmul_low_precision.phpt:108-114", F32,
     dC2, transposed(B2), [2, 2], expect=[5, 7, 6, 8], gradient="dA")
case("grad_seeded_dB", "tests/matmul_low_precision.phpt:115-116", F32,
     transposed(A2), dC2, [2, 2], expect=[1, 3, 2, 4], gradient="dB")
A3 = dense([2, 1, 2, 2], [1, 2, 3, 4, 2, 0, 0, 2])
B3 = dense([1, 3, 2, 1], [5, 6, 1, 2, 2, 1])
dC3 = fill([2, 3, 2, 1], 1.0)
# un-reduced batch gradients; the test's expectations are these summed over
# the broadcast axes (src/autograd.c:714-760), checked in the test file
case("grad_broadcast_dA", "tests/matmul_low_precision.phpt:118-128", F32,
     dC3, transposed(B3), [2, 3, 2, 2], gradient="dA",
     expect=flat([[[[5, 6], [5, 6]], [[1, 2], [1, 2]], [[2, 1], [2, 1]]]] * 2))
case("grad_broadcast_dB", "tests/matmul_low_precision.phpt:129-132", F32,
     transposed(A3), dC3, [2, 3, 2, 1], gradient="dB",
     expect=flat([[[[4], [6]]] * 3, [[[2], [2]]] * 3]))

# --- tests/host_array_math.phpt -------------------------------------------
a23 = dense([2, 3], [1, 2, 3, 4, 5, 6])
b32 = dense([3, 2], [1, 4, 2, 5, 3, 6])
case("host_matrix", "tests/host_array_math.phpt:78-79", ALL3, a23, b32, [2, 2],
     expect=[14, 32, 32, 77])
case("host_strided", "tests/host_array_math.phpt:80", ALL3, a23, transposed(a23), [2, 2],
     expect=[14, 32, 32, 77])
case("host_batched_broadcast", "tests/host_array_math.phpt:81-82", ALL3,
     broadcast_to(a23, [2, 1, 2, 3]), broadcast_to(b32, [3, 3, 2]), [2, 3, 2, 2],
     expect={"fill_pattern": [14, 32, 32, 77]}, points=[[[1, 2, 1, 1], 77.0]])
case("host_empty_inner", "tests/host_array_math.phpt:83-84", ALL3,
     dense([2, 0], []), dense([0, 3], []), [2, 3], expect=[0, 0, 0, 0, 0, 0])
case("host_empty_batch", "tests/host_array_math.phpt:85", ALL3,
     dense([0, 2, 3], []), b32, [0, 2, 2], expect=[])

# --- tests/cpu_backend.phpt -----------------------------------------------
case("cpu_backend_product", "tests/cpu_backend.phpt:68-69", F32,
     dense([2, 2], [1, 2, 3, 4]), dense([2, 2], [10, 20, 30, 40]), [2, 2],
     expect=[70, 100, 150, 220])

# --- tests/autograd.phpt --------------------------------------------------
L4 = dense([2, 2, 2], [1, 2, 3, 4, 5, 6, 7, 8])
R4 = dense([2, 2], [1, 0, 0, 1])
dC4 = fill([2, 2, 2], 1.0)
case("autograd_batched_dA", "tests/autograd.phpt:145-148", F32,
     dC4, transposed(R4), [2, 2, 2], expect={"fill": 1.0}, gradient="dA")
case("autograd_batched_dB", "tests/autograd.phpt:149", F32,
     transposed(L4), dC4, [2, 2, 2], gradient="dB",
     # per-batch A^T . ones; their sum over the batch is [[16,16],[20,20]]
     expect=[4, 4, 6, 6, 12, 12, 14, 14])

# --- tests/backend_dispatch.phpt ------------------------------------------
flat130 = [float((i * 7) % 13 - 6) for i in range(64 * 130)]
sl = {"shape": [64, 128], "strides": [130, 1], "offset": 1, "storage": flat130}
prod = [[sum(flat130[r * 130 + k] * flat130[c * 130 + k] for k in range(1, 129))
         for c in range(64)] for r in range(64)]
case("dispatch_padded_slice", "tests/backend_dispatch.phpt:48-57", F32,
     sl, transposed(sl), [64, 64], expect=flat(prod),
     points=[[[r, c], prod[r][c]] for r, c in [(0, 0), (0, 63), (37, 15), (63, 63)]])
case("dispatch_aligned_transpose", "tests/backend_dispatch.phpt:61-62", F32,
     fill([64, 128], 1.0), transposed(fill([64, 128], 1.0)), [64, 64],
     expect={"fill": 128.0})
case("dispatch_dot", "tests/backend_dispatch.phpt:64-65", F32,
     fill([1, 100000], 1.0), fill([100000, 1], 1.0), [1, 1], expect=[100000.0])
case("dispatch_skinny", "tests/backend_dispatch.phpt:67-68", F32,
     fill([16, 1024], 1.0), fill([1024, 16], 1.0), [16, 16], expect={"fill": 1024.0})

# --- Fusion plans: the native matmul step's own product -------------------
case("fusion_boundaries_step", "tests/fusion_boundaries.phpt:14-17", F32,
     dense([2, 2], [3, 5, 7, 9]), dense([2, 2], [5, 6, 7, 8]), [2, 2],
     expect=[50, 58, 98, 114])
y = dense([2, 2], [2, 3, 4, 5])
case("fusion_workspace_view_alias", "tests/fusion_workspace.phpt:17-24", F32,
     transposed(y), y, [2, 2], expect=[20, 26, 26, 34])
sliced = {"shape": [2, 2], "strides": [2, 1], "offset": 4,
          "storage": [1, 2, 3, 4, 5, 6, 7, 8]}
case("fusion_workspace_offset_alias", "tests/fusion_workspace.phpt:46-49", F32,
     transposed(sliced), sliced, [2, 2], expect=[74, 86, 86, 100])
case("fusion_workspace_batched", "tests/fusion_workspace.phpt:55-57", F32,
     fill([2, 4, 4], 2.0), fill([2, 4, 4], 1.0), [2, 4, 4], expect={"fill": 8.0})
for v, total in ((1.0, 8193.0), (2.0, 32769.0), (3.0, 73729.0)):
    case("fusion_workspace_parallel_x%d" % v, "tests/fusion_workspace.phpt:71-79", F32,
         transposed(fill([64, 128], v)), fill([64, 128], v), [128, 128],
         expect={"fill": 64.0 * v * v})
case("fusion_cuda_graph_first", "tests/fusion_cuda_graph.phpt:43-52", F32,
     fill([64, 64], 1.0), fill([64, 64], 1.0), [64, 64], expect={"fill": 64.0})
case("fusion_cuda_graph_pointer_update", "tests/fusion_cuda_graph.phpt:50-53", F32,
     fill([64, 64], 2.0), fill([64, 64], 3.0), [64, 64], expect={"fill": 384.0})
LA, RA = dense([2, 2], [1, 2, 3, 4]), dense([2, 2], [1, 0, 0, 1])
case("fusion_cuda_graph_grad_dA", "tests/fusion_cuda_graph.phpt:63-77", F32,
     fill([2, 2], 1.0), transposed(RA), [2, 2], expect=[1, 1, 1, 1], gradient="dA")
case("fusion_cuda_graph_grad_dB", "tests/fusion_cuda_graph.phpt:63-77", F32,
     transposed(LA), fill([2, 2], 1.0), [2, 2], expect=[4, 4, 6, 6], gradient="dB")

# Calls the reference must reject (InvalidArgumentException in
# src/contiguous_array_ce.c:1305-1316 and src/cuda_array/ca_private.c:1099-1106).
REJECTS = [
    {"name": "rank1", "source": "tests/host_array_math.phpt:93",
     "a_shape": [1], "b_shape": [1], "dtype": "float32"},
    {"name": "float64", "source": "tests/host_array_math.phpt:94; tests/cpu_backend.phpt:70-75",
     "a_shape": [1, 1], "b_shape": [1, 1], "dtype": "float64"},
    {"name": "inner_mismatch", "source": "tests/host_array_math.phpt:95",
     "a_shape": [1, 2], "b_shape": [1, 2], "dtype": "float32"},
    {"name": "batch_mismatch", "source": "tests/host_array_math.phpt:96",
     "a_shape": [2, 1, 1], "b_shape": [3, 1, 1], "dtype": "float32"},
]

# tests/tensor_shape_test.c:154-162: the shape rule.
SHAPES = [
    {"a": [2, 1, 3, 4], "b": [5, 4, 6], "ok": True, "out": [2, 5, 3, 6]},
    {"a": [2, 0], "b": [0, 3], "ok": True, "out": [2, 3]},
    {"a": [2], "b": [0, 3], "ok": False},
    {"a": [2, 1, 3, 4], "b": [2, 2], "ok": False},
]


def main():
    out = {"generator": "tests/golden/make_golden.py", "cases": CASES,
           "rejects": REJECTS, "shapes": SHAPES}
    with open(os.path.join(HERE, "matmul_golden.json"), "w") as f:
        json.dump(out, f, separators=(",", ":"))
        f.write("\n")
    print("wrote %d cases, %d rejects, %d shape cases" % (len(CASES), len(REJECTS), len(SHAPES)))


if __name__ == "__main__":
    main()
