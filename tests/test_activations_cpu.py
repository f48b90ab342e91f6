"""Relu / ReluAdjoint, gelu, the layer_norm adjoint and the cross-entropy
without a GPU: the oracle against the reference's own test vectors
(crates/chelis-ir/tests/issue_1313_relu_adjoint.rs), against float64
evaluations of the same mathematics (torch autograd for the adjoints)."""
import numpy as np
import pytest

from chelis_b200 import lib as L

BITS = {np.float32: np.uint32, np.float64: np.uint64}


def bits(a):
    return a.view(BITS[a.dtype.type]).tolist()


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_relu_reference_vectors(orc, dtype):
    """issue_1313_relu_adjoint.rs:146-232: the forward keeps NaN and -0; the
    adjoint is +0 wherever 0 < x fails (zeros, negatives, NaN) and the
    cotangent's own bits elsewhere."""
    tiny = np.finfo(dtype).smallest_subnormal
    x = np.array([np.nan, -0.0, 0.0, -1.0, 1.0, tiny], dtype)
    g = np.array([np.nan, np.inf, -0.0, np.nan, -0.0, np.inf], dtype)
    y = orc.relu(x)
    assert np.isnan(y[0]) and np.signbit(y[1]) and y[1] == 0
    assert bits(y[2:3]) == [0] and bits(y[3:4]) == [0] and y[4] == 1 and y[5] == tiny
    dx = orc.relu_adjoint(x, g)
    assert bits(dx[:4]) == [0, 0, 0, 0]
    assert np.signbit(dx[4]) and dx[4] == 0 and dx[5] == np.inf
    # ReluAdjoint's own adjoint in g (second order): ReluAdjoint(x, 1)
    x2 = np.array([0.0, np.nan, 1.0, -1.0], dtype)
    assert orc.relu_adjoint(x2, np.ones(4, dtype)).tolist() == [0.0, 0.0, 1.0, 0.0]
    # a NaN input's payload survives the forward
    nan = np.array([0xfff8123456789abc if dtype == np.float64 else 0xffc12345],
                   dtype=BITS[dtype]).view(dtype)
    assert bits(orc.relu(nan)) == bits(nan)


def test_gelu_phi_graph_accuracy(orc):
    """The compensated Phi graph makes x * Phi(x) accurate to a few ulp
    against a float64 evaluation of 0.5 * x * erfc(-x / sqrt(2))."""
    from scipy.special import erfc
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000) * 3,
                        np.linspace(-12, 12, 5001), [0.0, -0.0, 1e-30, -1e-30, 64, -64, 100]]
                       ).astype(np.float32)
    got = orc.gelu(x)
    ref = 0.5 * x.astype(np.float64) * erfc(-x.astype(np.float64) / np.sqrt(2.0))
    ulp = np.spacing(np.abs(ref).astype(np.float32)).astype(np.float64)
    err = np.abs(got.astype(np.float64) - ref) / np.maximum(ulp, np.finfo(np.float32).smallest_subnormal)
    assert float(err.max()) <= 3.0
    special = orc.gelu(np.array([np.inf, -np.inf, np.nan], np.float32))
    assert special[0] == np.inf and special[1] == 0 and np.signbit(special[1])
    assert bits(special[2:]) == [0x7fc00000]


def test_layer_norm_bwd_matches_float64_autograd(orc):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(4)
    rows, hidden = 24, 300
    x = rng.standard_normal((rows, hidden)).astype(np.float32)
    g = rng.uniform(0.5, 1.5, hidden).astype(np.float32)
    b = (rng.standard_normal(hidden) * 0.1).astype(np.float32)
    dy = rng.standard_normal((rows, hidden)).astype(np.float32)
    dx, dg, db = orc.layer_norm_bwd(x, g, 1e-5, dy)
    X = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    G = torch.tensor(g, dtype=torch.float64, requires_grad=True)
    B = torch.tensor(b, dtype=torch.float64, requires_grad=True)
    y = torch.nn.functional.layer_norm(X, (hidden,), G, B, 1e-5)
    y.backward(torch.tensor(dy, dtype=torch.float64))
    for got, ref in ((dx, X.grad), (dg, G.grad), (db, B.grad)):
        ref = ref.numpy()
        assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()


def test_cross_entropy_matches_mlp_head_and_autograd(orc):
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(5)
    rows, classes = 64, 10
    z = (rng.standard_normal((rows, classes)) * 3).astype(np.float32)
    labels = rng.integers(0, classes, rows).astype(np.int64)
    loss, dz = orc.cross_entropy(z, labels)
    Z = torch.tensor(z, dtype=torch.float64, requires_grad=True)
    ref = torch.nn.functional.cross_entropy(Z, torch.tensor(labels))
    ref.backward()
    ref = float(ref.detach())
    assert abs(float(loss) - ref) <= 1e-5 * abs(ref)
    assert np.abs(dz - Z.grad.numpy()).max() <= 1e-5 * np.abs(Z.grad.numpy()).max()
    with pytest.raises(ValueError):
        orc.cross_entropy(z, np.full(rows, classes, np.int64))
    # a probability that underflows to 0 makes the log adjoint 0/0: the row's
    # gradient is NaN, as the AD graph computes it
    z2 = np.zeros((2, 3), np.float32)
    z2[0, 2] = -200.0
    _, dz2 = orc.cross_entropy(z2, np.array([0, 1], np.int64))
    assert np.isnan(dz2[0]).all() and np.isfinite(dz2[1]).all()


def test_new_entries_reject_bad_arguments_without_device():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    lib = L.load()
    assert lib.chelis_cuda_relu(L.DTYPE_I32, None, None, 4) == 4
    assert lib.chelis_cuda_relu(L.DTYPE_F32, None, None, -1) == 1
    assert lib.chelis_cuda_relu(L.DTYPE_F32, None, None, 0) == 0
    assert lib.chelis_cuda_relu_adjoint(L.DTYPE_F64, None, None, None, 3) == 1
    assert lib.chelis_cuda_gelu_f32(None, None, 0) == 0
    assert lib.chelis_cuda_layer_norm_bwd_f32(None, None, 1e-5, None, 4, 9000, None, None, None) == 4
    assert lib.chelis_cuda_cross_entropy_f32(None, None, 0, 10, None, None) == 1
    assert "cross_entropy" in L.last_error()
