"""Relu / ReluAdjoint, gelu and its adjoint, the layer_norm adjoint and the
cross-entropy on the GPU against the oracle."""
import numpy as np
import pytest

from chelis_b200 import lib as L

pytestmark = pytest.mark.gpu

BITS = {np.float32: np.uint32, np.float64: np.uint64}


def t(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def specials(rng, n, dtype):
    x = (rng.standard_normal(n) * 3).astype(dtype)
    pool = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, np.finfo(dtype).smallest_subnormal,
                     -np.finfo(dtype).smallest_subnormal], dtype)
    idx = rng.choice(n, n // 5, replace=False)
    x[idx] = pool[rng.integers(len(pool), size=idx.size)]
    x[1] = np.array([0xfff8123456789abc if dtype == np.float64 else 0xffc12345],
                    dtype=BITS[dtype]).view(dtype)[0]
    return x


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("n", [1, 1000, 1 << 20])
def test_relu_and_adjoint_bit_exact(cuda, orc, dtype, n):
    rng = np.random.default_rng(n)
    x = specials(rng, max(n, 2), dtype)[:n]
    g = specials(rng, max(n, 2), dtype)[:n]
    X, G = t(x), t(g)
    y = cuda.relu(X).cpu().numpy()
    dx = cuda.relu_adjoint(X, G).cpu().numpy()
    assert (y.view(BITS[dtype]) == orc.relu(x).view(BITS[dtype])).all()
    assert (dx.view(BITS[dtype]) == orc.relu_adjoint(x, g).view(BITS[dtype])).all()


def test_gelu_against_oracle(cuda, orc):
    """CUDA erfcf / expf for CORE-MATH's inside the same Phi graph: a few ulp."""
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.standard_normal(1 << 20) * 4, np.linspace(-70, 70, 10001),
                        [np.inf, -np.inf, np.nan, 0.0, -0.0]]).astype(np.float32)
    got = cuda.gelu(t(x)).cpu().numpy()
    ref = orc.gelu(x)
    fin = np.isfinite(ref)
    assert (np.isnan(got) == np.isnan(ref)).all()
    assert (got[~fin & ~np.isnan(ref)] == ref[~fin & ~np.isnan(ref)]).all()
    scale = np.maximum(np.abs(ref[fin]), 1e-30)
    assert float((np.abs(got[fin] - ref[fin]) / scale).max()) <= 2e-6 or \
        float(np.abs(got[fin] - ref[fin]).max()) <= 1e-6


def test_gelu_adjoint_against_float64(cuda):
    from scipy.special import erfc
    rng = np.random.default_rng(2)
    x = (rng.standard_normal(1 << 18) * 3).astype(np.float32)
    g = rng.standard_normal(1 << 18).astype(np.float32)
    got = cuda.gelu_adjoint(t(x), t(g)).cpu().numpy()
    xd = x.astype(np.float64)
    der = 0.5 * erfc(-xd / np.sqrt(2.0)) + xd * np.exp(-0.5 * xd * xd) / np.sqrt(2 * np.pi)
    ref = g.astype(np.float64) * der
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()


@pytest.mark.parametrize("shape", [(64, 1024), (37, 300), (8, 8192), (2048, 4096)])
def test_layer_norm_bwd(cuda, orc, shape):
    rows, hidden = shape
    rng = np.random.default_rng(rows)
    x = rng.standard_normal(shape).astype(np.float32)
    gm = rng.uniform(0.5, 1.5, hidden).astype(np.float32)
    dy = rng.standard_normal(shape).astype(np.float32)
    ref = orc.layer_norm_bwd(x, gm, 1e-5, dy)
    got = [v.cpu().numpy() for v in cuda.layer_norm_bwd(t(x), t(gm), 1e-5, t(dy))]
    for a, r in zip(got, ref):
        assert np.abs(a - r).max() <= 1e-5 * np.abs(r).max()
    # EXACT rows mode: dx is the oracle's, bit for bit (same operations and
    # trees); dgamma / dbeta fold rows per CTA before the tree over CTAs
    with cuda.rows_mode(0):
        dx = cuda.layer_norm_bwd(t(x), t(gm), 1e-5, t(dy))[0].cpu().numpy()
    assert (dx.view(np.uint32) == ref[0].view(np.uint32)).all()


@pytest.mark.parametrize("shape", [(128, 10), (64, 1000), (16, 32000)])
def test_cross_entropy(cuda, orc, shape):
    rows, classes = shape
    rng = np.random.default_rng(classes)
    z = (rng.standard_normal(shape) * 3).astype(np.float32)
    labels = rng.integers(0, classes, rows).astype(np.int64)
    loss, dz = cuda.cross_entropy(t(z), t(labels))
    ref_loss, ref_dz = orc.cross_entropy(z, labels)
    assert abs(float(loss) - float(ref_loss)) <= 1e-5 * abs(float(ref_loss))
    dz = dz.cpu().numpy()
    assert np.abs(dz - ref_dz).max() <= 1e-5 * np.abs(ref_dz).max()
    cuda.device_status()


def test_cross_entropy_underflow_and_bad_label(cuda, orc):
    z = np.zeros((2, 3), np.float32)
    z[0, 2] = -200.0  # its probability underflows to 0: the row's adjoint is NaN
    labels = np.array([0, 1], np.int64)
    _, dz = cuda.cross_entropy(t(z), t(labels))
    _, ref = orc.cross_entropy(z, labels)
    dz = dz.cpu().numpy()
    assert (np.isnan(dz) == np.isnan(ref)).all() and np.isnan(dz[0]).all()
    cuda.cross_entropy(t(z), t(np.array([0, 3], np.int64)))
    with pytest.raises(L.ChelisCudaError, match="gather"):
        cuda.device_status()
    cuda.device_status()


def test_softmax_rows_wider_than_the_row_kernels(cuda, orc):
    """Rows past 8192 go through FusedElem groups (max, shifted exp, sum,
    divide) -- the softmax lowering itself -- and the same for the adjoint."""
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((6, 20000)) * 2).astype(np.float32)
    g = rng.standard_normal((6, 20000)).astype(np.float32)
    y = cuda.softmax_rows(t(x))
    ref = orc.softmax_rows(x)
    assert np.abs(y.cpu().numpy() - ref).max() <= 1e-5 * np.abs(ref).max()
    dx = cuda.softmax_rows_bwd(t(ref), t(g)).cpu().numpy()
    ref_dx = orc.softmax_rows_bwd(ref, g)
    assert (dx.view(np.uint32) == ref_dx.view(np.uint32)).all()  # same tree, same operations
