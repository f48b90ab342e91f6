"""FusedElem groups on the GPU against the oracle: bit for bit for chains of
IEEE arithmetic, selection and rounding steps (and their Sum / Max
reductions, which follow the same tree); within a few ulp per step for
transcendental steps, where CUDA's libm stands in for CORE-MATH."""
import numpy as np
import pytest

from chelis_b200 import fused as F
from chelis_b200 import lib as L

from test_fused_cpu import GOLDEN_CASES, UINT, as_arrays, grouped_rows

pytestmark = pytest.mark.gpu

EXACT_OPS = ["add", "sub", "mul", "div", "floor_div", "max_elem", "min_elem", "neg", "recip",
             "sqrt", "abs", "floor", "ceil", "round"]
# per-step bound for the transcendental steps: CUDA's documented maximum
# error (<= 4 ulp for f32 tanf / erfcf / powf; <= 5 ulp for f64 erfc) plus
# one for CORE-MATH's own half ulp
ULP_BOUND = 6


def t(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def ulp_distance(a, b, width):
    """Distance in representable values between same-width floats; NaN vs
    NaN is 0 (both canonical by then), NaN vs number is huge."""
    ui = UINT[width]
    top = np.array(1 << (31 if width == "f32" else 63), dtype=np.uint64)

    def ordered(x):
        u = x.view(ui).astype(np.uint64)
        neg = (u & top) != 0
        mag = (u & (top - 1)).astype(np.int64)
        return np.where(neg, -mag, mag)
    d = np.abs(ordered(a) - ordered(b))
    na, nb = np.isnan(a), np.isnan(b)
    d = np.where(na & nb, 0, d)
    return np.where(na ^ nb, np.iinfo(np.int64).max, d)


@pytest.mark.parametrize("key", sorted(grouped_rows()))
def test_single_step_fixture(cuda, key):
    op, width = key
    ins, exp = as_arrays(width, grouped_rows()[key])
    chain = [F.FusedStep(op, *[F.External(k) for k in range(len(ins))])]
    got = cuda.fused_elementwise(chain, [t(v) for v in ins]).cpu().numpy()
    if op in F.TRANSCENDENTAL:
        d = ulp_distance(got, exp.view(got.dtype), width)
        assert int(d.max()) <= ULP_BOUND, (op, width, int(np.argmax(d)))
    else:
        assert (got.view(UINT[width]) == exp).all(), (op, width)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("case", range(len(GOLDEN_CASES)))
def test_reference_fused_cases(cuda, case, dtype):
    text, ins, want = GOLDEN_CASES[case]
    got = cuda.fused_elementwise(F.parse(text), [t(np.asarray(v, dtype)) for v in ins])
    assert (got.cpu().numpy() == np.asarray(want, dtype)).all()


def special_values(rng, shape, dtype):
    n = int(np.prod(shape))
    flat = (rng.standard_normal(n) * 4).astype(dtype)
    specials = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1.5, -2.5, 0.5,
                         np.finfo(dtype).tiny / 4, -np.finfo(dtype).tiny / 8,
                         np.finfo(dtype).max], dtype=dtype)
    idx = rng.choice(n, size=min(n, max(1, n // 8)), replace=False)
    flat[idx] = specials[rng.integers(len(specials), size=idx.size)]
    # a NaN with a payload, which MaxElem / MinElem must carry through
    if n > 3:
        flat[3] = np.array([0x7fc01234 if dtype == np.float32 else 0x7ff8000000001234],
                           dtype=np.uint32 if dtype == np.float32 else np.uint64).view(dtype)[0]
    return flat.reshape(shape)


def random_chain(rng, n_inputs, n_steps, ops):
    steps = []
    for s in range(n_steps):
        op = ops[rng.integers(len(ops))]

        def pick():
            if s == 0 or rng.random() < 0.35:
                return F.External(int(rng.integers(n_inputs)))
            return F.PreviousStep(int(rng.integers(s)))
        steps.append(F.FusedStep(op, pick(), pick()) if op in F.BINARY else F.FusedStep(op, pick()))
    return steps


SHAPES = [
    # (iteration shape, input shapes): dense, broadcast rows / columns / scalars
    ((1000,), [(1000,), (1000,), ()]),
    ((33, 65), [(33, 65), (1, 65), (33, 1)]),
    ((4, 7, 129), [(4, 7, 129), (7, 1), (4, 1, 129), ()]),
    ((2, 3, 4, 5, 6, 7), [(2, 3, 4, 5, 6, 7), (6, 7), (3, 1, 1, 1, 1)]),
    ((0, 5), [(0, 5), (5,)]),
    ((), [(), ()]),
    # chunks of 8 / 4 consecutive elements per thread: dense with a ragged
    # end, strided rows of a multiple of 8 and of 4 only
    ((1003,), [(1003,), (1003,)]),
    ((16, 96), [(16, 96), (96,), (16, 1)]),
    ((3, 12), [(3, 12), (12,), ()]),
]


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("case", range(len(SHAPES)))
def test_random_exact_chains(cuda, orc, case, dtype):
    shape, in_shapes = SHAPES[case]
    rng = np.random.default_rng(100 + case)
    ins = [special_values(rng, s, dtype) for s in in_shapes]
    width = "f32" if dtype == np.float32 else "f64"
    for trial in range(6):
        chain = random_chain(rng, len(ins), int(rng.integers(1, 12)), EXACT_OPS)
        got = cuda.fused_elementwise(chain, [t(v) for v in ins], shape=shape).cpu().numpy()
        ref = orc.fused_elementwise(F.triplets(chain), ins, shape=shape)
        assert got.shape == ref.shape
        assert (got.view(UINT[width]) == ref.view(UINT[width])).all(), (trial, F.triplets(chain))


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_strided_inputs(cuda, orc, dtype):
    """Permuted and sliced inputs are read through their strides."""
    rng = np.random.default_rng(7)
    a = rng.standard_normal((64, 48)).astype(dtype)
    b = rng.standard_normal((48, 64)).astype(dtype)
    A, B = t(a), t(b)
    chain = F.parse("mul x0 x1; add v0 x0; min_elem v1 x1")
    got = cuda.fused_elementwise(chain, [A, B.T]).cpu().numpy()
    ref = orc.fused_elementwise(F.triplets(chain), [a, b.T])
    assert (got == ref).all()
    got = cuda.fused_elementwise(chain, [A[::2, 5:21], B.T[1::2, :16]]).cpu().numpy()
    ref = orc.fused_elementwise(F.triplets(chain), [a[::2, 5:21], b.T[1::2, :16]])
    assert (got == ref).all()


TRANS_OPS = ["exp", "log", "sin", "cos", "tan", "atan", "tanh", "erf", "erfc"]


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("op", TRANS_OPS + ["pow"])
def test_transcendental_steps(cuda, orc, op, dtype):
    rng = np.random.default_rng(sum(map(ord, op)))
    x = (rng.standard_normal(20000) * 3).astype(dtype)
    if op == "log":
        x = np.abs(x) + dtype(1e-3)
    y = (rng.standard_normal(20000)).astype(dtype)
    width = "f32" if dtype == np.float32 else "f64"
    chain = [F.FusedStep(op, F.External(0), F.External(1)) if op == "pow"
             else F.FusedStep(op, F.External(0))]
    ins = [np.abs(x) if op == "pow" else x, y] if op == "pow" else [x]
    got = cuda.fused_elementwise(chain, [t(v) for v in ins]).cpu().numpy()
    ref = orc.fused_elementwise(F.triplets(chain), ins)
    assert int(ulp_distance(got, ref, width).max()) <= ULP_BOUND


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_mixed_chain_within_tolerance(cuda, orc, dtype):
    """A GELU-like chain (tanh of a cubic): relative error 1e-5 (f32) /
    1e-12 (f64) against the CORE-MATH oracle, normwise."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal((256, 1024)).astype(dtype)
    c = [np.asarray(v, dtype) for v in (0.044715, 0.7978845608, 0.5, 1.0)]
    chain = F.parse("mul x0 x0; mul v0 x0; mul v1 x1; add v2 x0; mul v3 x2; tanh v4; "
                    "add v5 x4; mul v6 x0; mul v7 x3")
    ins = [x, *c]
    got = cuda.fused_elementwise(chain, [t(v) for v in ins]).cpu().numpy()
    ref = orc.fused_elementwise(F.triplets(chain), ins)
    tol = 1e-5 if dtype == np.float32 else 1e-12
    assert np.abs(got - ref).max() <= tol * np.abs(ref).max()


REDUCE_CASES = [
    # (shape, axis): last axis (warp per output), leading axes (thread per
    # output), few outputs over a long axis (segmented), ragged lengths
    ((64, 1000), 1),
    ((64, 1000), 0),
    ((5, 33, 17), 1),
    ((3, 200003), 1),
    ((300001, 3), 0),
    ((1, 1 << 20), 1),
    ((7,), 0),
    ((2, 0, 3), 2),
]


@pytest.mark.parametrize("kind", ["sum", "max"])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("case", range(len(REDUCE_CASES)))
def test_reduce_exact(cuda, orc, case, dtype, kind):
    shape, axis = REDUCE_CASES[case]
    rng = np.random.default_rng(case)
    x = rng.standard_normal(shape).astype(dtype)
    bias = rng.standard_normal(shape[-1:]).astype(dtype)
    chain = F.parse("mul x0 x0; add v0 x1; abs v1; sqrt v2; sub v3 x1")
    width = "f32" if dtype == np.float32 else "f64"
    got = cuda.fused_reduce(chain, [t(x), t(bias)], axis=axis, kind=kind).cpu().numpy()
    ref = orc.fused_reduce(F.triplets(chain), [x, bias], axis=axis, kind=kind)
    assert got.shape == ref.shape
    assert (got.view(UINT[width]) == ref.view(UINT[width])).all()


@pytest.mark.parametrize("axis", [0, 1])
def test_reduce_specials(cuda, orc, axis):
    """NaN anywhere on the axis is the canonical NaN; a zero maximum takes
    the sign of the last zero; infinities sum to NaN."""
    x = np.array([[-0.0, 0.0, -1.0, np.inf], [0.0, -0.0, -1.0, -np.inf],
                  [1.0, np.nan, 2.0, np.inf]], np.float32)
    for kind in ("sum", "max"):
        chain = F.parse("max_elem x0 x0")
        got = cuda.fused_reduce(chain, [t(x)], axis=axis, kind=kind).cpu().numpy()
        ref = orc.fused_reduce(F.triplets(chain), [x], axis=axis, kind=kind)
        assert (got.view(np.uint32) == ref.view(np.uint32)).all(), kind


def test_errors(cuda):
    import torch
    x = t(np.ones((4, 0), np.float32))
    with pytest.raises(L.ChelisCudaError, match="max_reduce"):
        cuda.fused_reduce(F.parse("neg x0"), [x], axis=1, kind="max")
    s = cuda.fused_reduce(F.parse("neg x0"), [x], axis=1, kind="sum")
    assert (s.cpu().numpy() == 0).all() and s.shape == (4,)
    with pytest.raises(L.ChelisCudaError, match="integer-only"):
        cuda.fused_elementwise(F.parse("trunc_div x0 x0"), [t(np.ones(3, np.float32))])
    with pytest.raises(ValueError):
        cuda.fused_elementwise(F.parse("add x0 x1"), [t(np.ones(3, np.float32)),
                                                      t(np.ones(3, np.float64))])
    torch.cuda.synchronize()


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("mkn", [(33, 70, 17), (8, 1000, 64)])
def test_inlined_product_is_the_c_lane_matmul(cuda, orc, mkn, dtype):
    """Sum(Mul(Expand(a), Expand(b))) along k -- the reduction-inlined product
    of fuse.rs:483-560 (an einsum contraction) -- as one fused reduction over
    the broadcast [m, k, n] iteration shape: bit for bit the C lane's matmul
    (fl(a*b) leaves, canonical tree over k, emit.rs:8431-8640)."""
    m, k, n = mkn
    rng = np.random.default_rng(m * k + n)
    a = rng.standard_normal((m, k)).astype(dtype)
    b = rng.standard_normal((k, n)).astype(dtype)
    A, B = t(a), t(b)
    got = cuda.fused_reduce(F.parse("mul x0 x1"), [A[:, :, None], B[None, :, :]], axis=1,
                            shape=(m, k, n)).cpu().numpy()
    ref = orc.gemm(a, b)
    width = "f32" if dtype == np.float32 else "f64"
    assert (got.view(UINT[width]) == ref.view(UINT[width])).all()


def _special_mix(rng, shape, dtype):
    x = (rng.standard_normal(shape) * 3).astype(dtype)
    flat = x.reshape(-1)
    specials = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-40, -1e-40, 0.5, -2.5, 1e30],
                        dtype=dtype)
    flat[: len(specials)] = specials
    return x


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("op", [o for o in F.OPS if o != "trunc_div"])
def test_compiled_chain_matches_interpreter(cuda, op, dtype):
    """Every step op through the per-chain compiled kernel (NVRTC) and through
    the interpreter gives the same bits, with a full-size operand, a row
    vector broadcast along the rows and a column broadcast along the
    innermost axis; and the compiled path is the one that ran."""
    import torch
    rng = np.random.default_rng(F.OP_CODE[op] + (0 if dtype == np.float32 else 100))
    rows, cols = 37, 96
    x = _special_mix(rng, (rows, cols), dtype)
    row = _special_mix(rng, (1, cols), dtype)        # broadcast over rows, unit inner stride
    col = (rng.standard_normal((rows, 1)) * 2).astype(dtype)  # broadcast along the inner axis
    second = "x1" if op in F.BINARY else ""
    chain = F.parse(f"{op} x0 {second}".strip() + "; mul v0 x2; " + (f"{op} v1 x1" if op in F.BINARY else f"{op} v1"))
    ins = [t(x), t(row), t(col)]
    before = L.load().chelis_cuda_fused_jit_launches()
    with cuda.fused_jit(True):
        jit = cuda.fused_elementwise(chain, ins).cpu().numpy()
    after = L.load().chelis_cuda_fused_jit_launches()
    with cuda.fused_jit(False):
        ref = cuda.fused_elementwise(chain, ins).cpu().numpy()
    torch.cuda.synchronize()
    assert after == before + 1
    w = UINT["f32" if dtype == np.float32 else "f64"]
    assert (jit.view(w) == ref.view(w)).all(), op


def test_compiled_chain_affine_large(cuda, orc):
    """The affine chain x * gamma + beta at 4096 x 4096 through the compiled
    kernel matches the oracle bit for bit."""
    rng = np.random.default_rng(11)
    x = rng.standard_normal((4096, 4096)).astype(np.float32)
    g = rng.uniform(0.5, 1.5, (1, 4096)).astype(np.float32)
    b = (rng.standard_normal((1, 4096)) * 0.1).astype(np.float32)
    chain = F.parse("mul x0 x1; add v0 x2")
    before = L.load().chelis_cuda_fused_jit_launches()
    got = cuda.fused_elementwise(chain, [t(x), t(g), t(b)]).cpu().numpy()
    assert L.load().chelis_cuda_fused_jit_launches() == before + 1
    ref = (x * g).astype(np.float32) + b
    assert (got.view(np.uint32) == ref.astype(np.float32).view(np.uint32)).all()


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("kind", ["sum", "max"])
@pytest.mark.parametrize("chain_text", ["mul x0 x0", "mul x0 x1; add v0 x2", "abs x0; neg v0", "exp x0"])
def test_compiled_last_axis_reduction_matches_interpreter(cuda, dtype, kind, chain_text):
    """Sum (canonical pair tree) and Max (first-NaN rule, later zero wins)
    over the last axis through the compiled kernel and through the
    interpreter give the same bits; rows of 1, 5 and 32 passes, specials
    and signed-zero ties included."""
    import torch
    rng = np.random.default_rng(len(chain_text) * 7 + (kind == "max"))
    v = 4 if dtype == np.float32 else 2
    # one warp per output: the compiled form takes row counts that fill the
    # GPU (>= 8 warps per SM)
    for rows, passes in ((1250, 1), (1250, 5), (1250, 7), (1250, 11), (1250, 32), (1250, 45)):
        cols = 32 * v * passes
        x = _special_mix(rng, (rows, cols), dtype)
        x[1, :] = 0.0
        x[1, cols // 2] = -0.0
        x[2, :] = -0.0
        x[2, 3] = 0.0
        row = _special_mix(rng, (1, cols), dtype)
        col = (rng.standard_normal((rows, 1)) * 2).astype(dtype)
        chain = F.parse(chain_text)
        n_in = 1 + max((int(tok[1:]) for tok in chain_text.replace(";", " ").split() if tok.startswith("x")), default=0)
        ins = [t(x), t(row), t(col)][:max(n_in, 1)]
        before = L.load().chelis_cuda_fused_jit_launches()
        with cuda.fused_jit(True):
            jit = cuda.fused_reduce(chain, ins, axis=1, kind=kind).cpu().numpy()
        after = L.load().chelis_cuda_fused_jit_launches()
        with cuda.fused_jit(False):
            ref = cuda.fused_reduce(chain, ins, axis=1, kind=kind).cpu().numpy()
        torch.cuda.synchronize()
        assert after == before + 1
        w = UINT["f32" if dtype == np.float32 else "f64"]
        assert (jit.view(w) == ref.view(w)).all(), (rows, passes)


@pytest.mark.parametrize("kind", ["sum", "max"])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_few_long_rows_reduce_in_segments(cuda, kind, dtype):
    """A whole-tensor reduction (one output) runs as aligned segments, one
    warp each through the compiled kernel, then the segment partials in
    order; the bits equal the interpreter's single canonical tree (Sum) and
    first-NaN / later-zero rule (Max)."""
    import torch
    rng = np.random.default_rng(3)
    for n, finite in ((1 << 20, True), (3 << 18, True), (1 << 20, False)):
        x = _special_mix(rng, (n,), dtype)
        if finite:
            x = np.nan_to_num(x, nan=0.5, posinf=2.0, neginf=-2.0)
        x[n // 3] = 0.0
        x[n // 2] = -0.0
        for chain_text in ("mul x0 x0", "abs x0; neg v0"):
            chain = F.parse(chain_text)
            before = L.load().chelis_cuda_fused_jit_launches()
            with cuda.fused_jit(True):
                jit = cuda.fused_reduce(chain, [t(x)], axis=0, kind=kind).cpu().numpy()
            after = L.load().chelis_cuda_fused_jit_launches()
            with cuda.fused_jit(False):
                ref = cuda.fused_reduce(chain, [t(x)], axis=0, kind=kind).cpu().numpy()
            torch.cuda.synchronize()
            assert after == before + 1
            w = UINT["f32" if dtype == np.float32 else "f64"]
            assert (jit.view(w) == ref.view(w)).all(), (n, chain_text)
