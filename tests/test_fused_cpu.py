"""FusedElem groups without a GPU: the oracle's step semantics pinned to the
reference's fixtures, the reduction orders cross-checked against the pinned
row / column trees, the host-side chain form, and the ABI's argument checks."""
import ctypes
import os

import numpy as np
import pytest

from chelis_b200 import fused as F
from chelis_b200 import lib as L

HERE = os.path.dirname(os.path.abspath(__file__))
UINT = {"f32": np.uint32, "f64": np.uint64}
FLOAT = {"f32": np.float32, "f64": np.float64}


def fixture_rows():
    """tests/golden/fused_steps.txt: (op, width, expected bits, operand bits)."""
    out = []
    with open(os.path.join(HERE, "golden", "fused_steps.txt")) as f:
        for line in f:
            line = line.split("#", 1)[0].split()
            if line:
                out.append((line[0], line[1], int(line[2], 16), [int(v, 16) for v in line[3:]]))
    return out


def grouped_rows():
    groups = {}
    for op, width, exp, operands in fixture_rows():
        groups.setdefault((op, width), []).append((exp, operands))
    return groups


def as_arrays(width, rows):
    n_ops = len(rows[0][1])
    ins = [np.array([r[1][k] for r in rows], dtype=UINT[width]).view(FLOAT[width])
           for k in range(n_ops)]
    exp = np.array([r[0] for r in rows], dtype=UINT[width])
    return ins, exp


@pytest.mark.parametrize("key", sorted(grouped_rows()))
def test_oracle_single_step_matches_reference_fixture(orc, key):
    """Each fixture row as a one-step chain (External operands), and the
    transcendental rows also behind neg(neg(x)) as the reference's
    `{name}_fused` canary route does (correctly_rounded_kernels.rs:300-312)."""
    op, width = key
    ins, exp = as_arrays(width, grouped_rows()[key])
    chain = [F.FusedStep(op, *[F.External(k) for k in range(len(ins))])]
    got = orc.fused_elementwise(F.triplets(chain), ins)
    assert (got.view(UINT[width]) == exp).all(), (op, width)
    if op not in F.BINARY:
        chain = F.parse(f"neg x0; neg v0; {op} v1")
        got = orc.fused_elementwise(F.triplets(chain), ins)
        assert (got.view(UINT[width]) == exp).all()


# hip gpu_correctness.rs:2461-2585: the fused GPU lane against the unfused
# evaluator on the tests' own inputs (values exact in binary)
GOLDEN_CASES = [
    ("add x0 x1; neg v0",
     [[1.0, -2.0, 3.5, -4.25], [0.5, 4.0, -1.5, 2.25]], [-1.5, -2.0, -2.0, 2.0]),
    ("add x0 x1; max_elem v0 x3; mul v1 x2",
     [[1.0, -2.0, 3.0, -4.0], [-0.5, 0.5, 2.0, 1.0], [2.0, 3.0, -1.5, 4.0], 0.0],
     [1.0, 0.0, -7.5, 0.0]),
    ("sub x0 x1; min_elem v0 x2",
     [[1.0, -2.0, 3.0, -4.0], [-0.5, 0.5, 2.0, 1.0], [0.0, -3.0, 0.5, -4.0]],
     [0.0, -3.0, 0.5, -5.0]),
]


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("case", range(len(GOLDEN_CASES)))
def test_oracle_reference_fused_cases(orc, case, dtype):
    text, ins, want = GOLDEN_CASES[case]
    got = orc.fused_elementwise(F.triplets(F.parse(text)), [np.asarray(v, dtype) for v in ins])
    assert (got == np.asarray(want, dtype)).all()


def test_oracle_step_nan_rules(orc):
    """fp_env.rs:213-241: arithmetic steps give the canonical NaN; MaxElem /
    MinElem select an operand with its bits (first operand when NaN, else a
    NaN second operand, else the first on ties)."""
    payload = np.array([0x7fc12345], np.uint32).view(np.float32)[0]
    x = np.array([payload, 1.0, 0.0, -0.0, 2.0], np.float32)
    y = np.array([3.0, payload, -0.0, 0.0, 2.0], np.float32)
    bits = lambda a: a.view(np.uint32).tolist()
    mx = orc.fused_elementwise(F.triplets(F.parse("max_elem x0 x1")), [x, y])
    assert bits(mx) == [0x7fc12345, 0x7fc12345, 0x00000000, 0x80000000, 0x40000000]
    mn = orc.fused_elementwise(F.triplets(F.parse("min_elem x0 x1")), [x, y])
    assert bits(mn) == [0x7fc12345, 0x7fc12345, 0x00000000, 0x80000000, 0x40000000]
    ad = orc.fused_elementwise(F.triplets(F.parse("add x0 x1")), [x, y])
    assert bits(ad)[:2] == [0x7fc00000, 0x7fc00000]
    ng = orc.fused_elementwise(F.triplets(F.parse("neg x0")), [x])
    assert bits(ng)[0] == 0x7fc00000 and bits(ng)[2] == 0x80000000
    # round is rint (ties to even); floor_div is floor(a / b)
    r = orc.fused_elementwise(F.triplets(F.parse("round x0")),
                              [np.array([0.5, 1.5, 2.5, -0.5, -2.5], np.float32)])
    assert r.tolist() == [0.0, 2.0, 2.0, -0.0, -2.0] and np.signbit(r[3])
    fd = orc.fused_elementwise(F.triplets(F.parse("floor_div x0 x1")),
                               [np.array([7.0, -7.0, 7.0], np.float32),
                                np.array([2.0, 2.0, -2.0], np.float32)])
    assert fd.tolist() == [3.0, -4.0, -4.0]


def test_oracle_reduce_orders_match_pinned_trees(orc):
    """Sum along the last / first axis is the canonical tree the pinned
    row_sum / col_sum use; Max is chelis_fmax_propnan folded from -inf."""
    rng = np.random.default_rng(5)
    rows, cols = 37, 1000
    ins = [rng.standard_normal((rows, cols)).astype(np.float32),
           rng.standard_normal(cols).astype(np.float32)]
    chain = F.parse("mul x0 x1; add v0 x0; abs v1; sqrt v2")
    t = F.triplets(chain)
    val = orc.fused_elementwise(t, ins)
    assert (orc.fused_reduce(t, ins, axis=1).view(np.uint32) ==
            orc.row_sum(val).view(np.uint32)).all()
    assert (orc.fused_reduce(t, ins, axis=0).view(np.uint32) ==
            orc.col_sum(val).view(np.uint32)).all()
    assert (orc.fused_reduce(t, ins, axis=1, kind="max") == val.max(axis=1)).all()
    # NaN anywhere gives the canonical NaN; among equal maxima the later wins
    x = np.array([[-0.0, 0.0, -1.0], [0.0, -0.0, -1.0], [1.0, np.nan, 2.0]], np.float32)
    m = orc.fused_reduce(F.triplets(F.parse("abs x0; neg v0; neg v1")), [x], axis=1, kind="max")
    m2 = orc.fused_reduce(F.triplets(F.parse("max_elem x0 x0")), [x], axis=1, kind="max")
    assert m2.view(np.uint32).tolist() == [0x00000000, 0x80000000, 0x7fc00000]
    assert m.view(np.uint32).tolist()[2] == 0x7fc00000


def test_oracle_broadcast_strides(orc):
    rng = np.random.default_rng(1)
    a = rng.standard_normal((3, 1, 5))
    b = rng.standard_normal((4, 1))
    c = np.float64(0.5)
    got = orc.fused_elementwise(F.triplets(F.parse("mul x0 x1; sub v0 x2")), [a, b, c])
    assert got.shape == (3, 4, 5)
    assert (got == a * b - c).all()
    # a transposed (non-contiguous) input
    at = rng.standard_normal((6, 7)).T
    got = orc.fused_elementwise(F.triplets(F.parse("add x0 x0")), [at])
    assert (got == at + at).all()


def test_host_chain_form():
    steps = F.parse("mul x0 x1; add v0 x2; tanh v1")
    assert F.triplets(steps) == [(2, 0, 1), (0, -1, 2), (18, -2, -2)]
    arr = F.encode(steps)
    assert ctypes.sizeof(arr) == 3 * 12 and (arr[2].op, arr[2].a) == (18, -2)
    assert F.OPS[F.OP_CODE["round"]] == "round" and len(F.OPS) == 25
    with pytest.raises(ValueError):
        F.FusedStep("add", F.External(0))
    with pytest.raises(ValueError):
        F.FusedStep("cbrt", F.External(0))
    with pytest.raises(ValueError):
        F.parse("add x0 y1")


def test_fused_abi_rejects_bad_programs_without_device():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    lib = L.load()
    shape = (ctypes.c_int64 * 1)(4)
    strides = (ctypes.c_int64 * 1)(1)
    ptrs = (ctypes.c_void_p * 1)(16)

    def call(text, dtype=L.DTYPE_F32, fn="chelis_cuda_fused_elementwise", extra=()):
        steps = F.encode(F.parse(text))
        return getattr(lib, fn)(dtype, steps, len(F.parse(text)), ptrs, strides, 1, shape, 1,
                                *extra, None)

    assert call("trunc_div x0 x0") == 4 and "integer-only" in L.last_error()
    assert call("add x0 x1") == 1 and "operand" in L.last_error()
    assert call("neg v0") == 1  # a step may only read earlier steps
    assert call("neg x0", dtype=L.DTYPE_I32) == 4
    assert call("neg x0") == 1 and "output" in L.last_error()  # null output
    assert call("neg x0", fn="chelis_cuda_fused_reduce", extra=(1, 0)) == 1  # axis out of range
    # an empty max axis is the Domain trap, whatever else the call holds
    zero = (ctypes.c_int64 * 1)(0)
    steps = F.encode(F.parse("neg x0"))
    assert lib.chelis_cuda_fused_reduce(L.DTYPE_F32, steps, 1, ptrs, strides, 1, zero, 1, 0, 1,
                                        None) == 1
    assert "max_reduce" in L.last_error()
    # empty elementwise work is a successful no-op
    assert lib.chelis_cuda_fused_elementwise(L.DTYPE_F32, steps, 1, ptrs, strides, 1, zero, 1,
                                             None) == 0


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_oracle_inlined_product_equals_matmul_tree(orc, dtype):
    """fuse.rs:483-560: a Sum over k of Mul(Expand(a), Expand(b)) keeps the
    materialised graph's bits -- the C lane's matmul tree (emit.rs:8431-8640)."""
    rng = np.random.default_rng(9)
    a = rng.standard_normal((19, 77)).astype(dtype)
    b = rng.standard_normal((77, 23)).astype(dtype)
    got = orc.fused_reduce(F.triplets(F.parse("mul x0 x1")), [a[:, :, None], b[None, :, :]],
                           axis=1, shape=(19, 77, 23))
    ref = orc.gemm(a, b)
    assert (got == ref).all()
