"""Fused elementwise / reduction kernels on the GPU against the oracle.

Bit-exact (integer, index, bool-count and keyed-RNG work, and float work
whose every operation matches the C lane's: canonical-tree sums, IEEE
div / sqrt, no contraction): row/col sums, row max, count, dropout mask and
values, cumsum, softmax adjoint, layer_norm in EXACT mode.

Tolerance (f32 rel <= 1e-5 after reductions) where CUDA's expf stands in for
CORE-MATH's correctly rounded exp, or where the FAST mode rewrites divisions
as reciprocal multiplies: elementwise |y - y_ref| <= 1e-5 * max(|y_ref|,
row scale) with the row scale the largest |y_ref| of that row (normwise per
row), and for the column reductions dgamma / dbeta normwise over the vector.
"""
import numpy as np
import pytest

from chelis_b200 import lib as L
from chelis_b200 import workloads as W

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def t(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def bits_equal(a, b):
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    return a.shape == b.shape and (a.view(np.uint8) == b.view(np.uint8)).all()


def rowwise_ok(got, ref, rtol=RTOL):
    got = np.asarray(got, np.float64).reshape(ref.shape[0], -1)
    ref = np.asarray(ref, np.float64).reshape(ref.shape[0], -1)
    scale = np.abs(ref).max(axis=1, keepdims=True)
    err = np.abs(got - ref) / np.maximum(scale, 1e-30)
    return float(err.max())


def normwise(got, ref):
    return float(np.abs(np.asarray(got, np.float64) - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.mark.parametrize("rows,cols", [(1, 1), (3, 7), (64, 1024), (37, 4096), (5, 5000),
                                       (2, 100000), (129, 8192)])
def test_row_sum_bit_exact(cuda, orc, rows, cols):
    x = (np.random.default_rng(rows * cols).standard_normal((rows, cols)) * 3).astype(np.float32)
    assert bits_equal(cuda.row_sum(t(x)).cpu().numpy(), orc.row_sum(x))


@pytest.mark.parametrize("rows,cols", [(1, 3), (64, 5), (65, 130), (4097, 33), (16384, 64),
                                       (1000, 4096), (4129, 128), (96, 8)])
def test_col_sum_bit_exact(cuda, orc, rows, cols):
    x = np.random.default_rng(rows + cols).standard_normal((rows, cols)).astype(np.float32)
    assert bits_equal(cuda.col_sum(t(x)).cpu().numpy(), orc.col_sum(x))


def test_row_max_first_nan_and_ties(cuda, orc):
    x = np.random.default_rng(3).standard_normal((40, 300)).astype(np.float32)
    x[3, 10] = np.float32("nan")
    x[3, 200] = -np.float32("nan")
    x[5, :] = 0.0
    x[5, 7] = -0.0
    assert bits_equal(cuda.row_max(t(x)).cpu().numpy(), orc.row_max(x))


@pytest.mark.parametrize("rows,cols", [(9, 4), (9, 5), (12, 128), (12, 644), (10, 4096), (9, 4099)])
def test_row_max_selection_rules(cuda, orc, rows, cols):
    """First NaN (payload kept) wins, else the first of equal maxima (+0 / -0
    order kept); vectorised rows (width % 4 == 0) and ragged ones."""
    rng = np.random.default_rng(cols)
    x = rng.standard_normal((rows, cols)).astype(np.float32)
    nan1 = np.array([0x7fc00123], np.uint32).view(np.float32)[0]
    nan2 = np.array([0xffc00456], np.uint32).view(np.float32)[0]
    x[0, cols - 1] = nan1
    x[1, :] = -np.inf
    x[2, :] = 0.0
    x[2, cols // 2] = -0.0
    x[3, :] = -0.0
    x[3, cols - 1] = 0.0
    x[4, cols // 3] = nan2
    x[4, cols - 1] = nan1
    x[5, :] = nan2
    x[6, :] = 7.0
    x[7, 0] = np.inf
    x[7, cols - 1] = np.inf
    x[8, cols - 1] = 1e30
    assert bits_equal(cuda.row_max(t(x)).cpu().numpy(), orc.row_max(x))


def test_count_exact(cuda, orc):
    x = (np.random.default_rng(4).random(1_000_003) < 0.37).astype(np.uint8)
    assert cuda.count(t(x)) == orc.count(x)
    assert cuda.count(t(np.zeros(0, np.uint8))) == 0


@pytest.mark.parametrize("rate", [0.1, 0.5, 0.0])
def test_dropout_mask_bit_exact(cuda, orc, rate):
    n, base = 1 << 20, 12345
    got = cuda.dropout_mask(n, W.CHAIN_KEY, rate, base).cpu().numpy()
    assert bits_equal(got, orc.dropout_mask(n, W.CHAIN_KEY, np.float32(rate), base))


def test_dropout_mask_full_config_size(cuda, orc):
    """Every element of the config-3 draw (16384 x 4096, key 42, rate 0.1)."""
    n = 16384 * 4096
    got = cuda.dropout_mask(n, W.CHAIN_KEY, 0.1).cpu().numpy()
    ref = orc.dropout_mask(n, W.CHAIN_KEY, np.float32(0.1))
    assert bits_equal(got, ref)
    assert cuda.count(t(got)) == orc.count(ref)


def test_dropout_values_bit_exact(cuda, orc):
    x = np.random.default_rng(5).standard_normal(300001).astype(np.float32)
    x[:4] = [-0.0, 0.0, np.inf, -np.inf]
    got = cuda.dropout(t(x), 7, 0.25, 99).cpu().numpy()
    assert bits_equal(got, orc.dropout(x, 7, np.float32(0.25), 99))


@pytest.mark.parametrize("rows,hidden", [(1, 1), (7, 100), (64, 1024), (33, 4096), (8, 5000),
                                         (4, 8192)])
def test_layer_norm_exact_mode_bit_exact(cuda, orc, rows, hidden):
    x, g, b = W.chain_inputs(rows, hidden, seed=hidden)
    with cuda.rows_mode(L.ROWS_EXACT):
        y = cuda.layer_norm(t(x), t(g), t(b), 1e-5).cpu().numpy()
    assert bits_equal(y, orc.layer_norm(x, g, b, np.float32(1e-5)))


def test_layer_norm_fast_mode_tolerance(cuda, orc):
    x, g, b = W.chain_inputs(64, 4096, seed=1)
    y = cuda.layer_norm(t(x), t(g), t(b), 1e-5).cpu().numpy()
    assert rowwise_ok(y, orc.layer_norm(x, g, b, np.float32(1e-5))) <= RTOL


@pytest.mark.parametrize("rows,cols", [(1, 1), (16, 10), (64, 4096), (9, 3000)])
def test_softmax_tolerance(cuda, orc, rows, cols):
    x = (np.random.default_rng(cols).standard_normal((rows, cols)) * 4).astype(np.float32)
    for mode in (L.ROWS_EXACT, L.ROWS_FAST):
        with cuda.rows_mode(mode):
            y = cuda.softmax_rows(t(x)).cpu().numpy()
        ref = orc.softmax_rows(x)
        err = np.abs(y.astype(np.float64) - ref) / np.maximum(np.abs(ref), 1e-30)
        assert float(err.max()) <= RTOL


def test_softmax_bwd_bit_exact(cuda, orc):
    rng = np.random.default_rng(6)
    y = orc.softmax_rows(rng.standard_normal((50, 777)).astype(np.float32))
    g = rng.standard_normal((50, 777)).astype(np.float32)
    assert bits_equal(cuda.softmax_rows_bwd(t(y), t(g)).cpu().numpy(), orc.softmax_rows_bwd(y, g))


@pytest.mark.parametrize("rows,hidden", [(3, 1), (5, 100), (64, 4096), (17, 4095), (6, 8192)])
@pytest.mark.parametrize("mode", [L.ROWS_EXACT, L.ROWS_FAST])
def test_chain_fwd_bwd_small(cuda, orc, rows, hidden, mode):
    x, g, b = W.chain_inputs(rows, hidden, seed=rows + hidden)
    eps, key, rate = W.CHAIN_EPS, W.CHAIN_KEY, W.CHAIN_RATE
    base = 4096 * 7
    with cuda.rows_mode(mode):
        rs, stats = cuda.chain_fwd(t(x), t(g), t(b), float(eps), key, float(rate), base, want_stats=True)
        dx, dg, db = cuda.chain_bwd(t(x), t(g), t(b), float(eps), key, float(rate), base)
        dx2, dg2, db2 = cuda.chain_bwd(t(x), t(g), t(b), float(eps), key, float(rate), base, stats)
    rs_ref = orc.chain_fwd(x, g, b, eps, key, rate, base)
    dx_ref, dg_ref, db_ref = orc.chain_bwd(x, g, b, eps, key, rate, base)
    rs = rs.cpu().numpy()
    assert float((np.abs(rs - rs_ref) / np.maximum(np.abs(rs_ref), 1e-30)).max()) <= RTOL
    assert rowwise_ok(dx.cpu().numpy(), dx_ref) <= RTOL
    assert normwise(dg.cpu().numpy(), dg_ref) <= RTOL
    assert normwise(db.cpu().numpy(), db_ref) <= RTOL
    # saved statistics give the same adjoint as recomputing them
    assert bits_equal(dx2.cpu().numpy(), dx.cpu().numpy())
    assert bits_equal(dg2.cpu().numpy(), dg.cpu().numpy())


@pytest.mark.parametrize("rows,hidden", [(3, 1), (9, 333), (64, 4096), (5, 8192)])
@pytest.mark.parametrize("mode", [L.ROWS_EXACT, L.ROWS_FAST])
def test_chain_saved_state_matches_recompute(cuda, orc, rows, hidden, mode):
    """Forward with saved statistics + keep bits, adjoint from them: the keep
    bits equal the oracle's mask and the adjoint equals the recomputing one."""
    x, g, b = W.chain_inputs(rows, hidden, seed=rows * 7 + hidden)
    eps, key, rate = W.CHAIN_EPS, W.CHAIN_KEY, W.CHAIN_RATE
    X, G, B = t(x), t(g), t(b)
    with cuda.rows_mode(mode):
        rs, saved = cuda.chain_fwd_save(X, G, B, float(eps), key, float(rate))
        rs2 = cuda.chain_fwd(X, G, B, float(eps), key, float(rate))
        dx, dg, db = cuda.chain_bwd_saved(X, G, B, float(eps), float(rate), saved)
        dx2, dg2, db2 = cuda.chain_bwd(X, G, B, float(eps), key, float(rate))
    assert bits_equal(rs.cpu().numpy(), rs2.cpu().numpy())
    assert bits_equal(dx.cpu().numpy(), dx2.cpu().numpy())
    assert bits_equal(dg.cpu().numpy(), dg2.cpu().numpy())
    dx_ref, dg_ref, db_ref = orc.chain_bwd(x, g, b, eps, key, rate)
    assert rowwise_ok(dx.cpu().numpy(), dx_ref) <= RTOL
    assert normwise(db.cpu().numpy(), db_ref) <= RTOL


def test_chain_full_config_size(cuda, orc):
    """Config 3 at full size (16384 x 4096): forward and adjoint on the GPU
    against the oracle on the same seeded inputs."""
    import torch
    x, g, b = W.chain_inputs()
    eps, key, rate = W.CHAIN_EPS, W.CHAIN_KEY, W.CHAIN_RATE
    X, G, B = t(x), t(g), t(b)
    rs, stats = cuda.chain_fwd(X, G, B, float(eps), key, float(rate), want_stats=True)
    dx, dg, db = cuda.chain_bwd(X, G, B, float(eps), key, float(rate), 0, stats)
    torch.cuda.synchronize()
    cuda.device_status()
    rs_ref = orc.chain_fwd(x, g, b, eps, key, rate)
    dx_ref, dg_ref, db_ref = orc.chain_bwd(x, g, b, eps, key, rate)
    rs = rs.cpu().numpy()
    assert float((np.abs(rs - rs_ref) / np.abs(rs_ref)).max()) <= RTOL
    assert rowwise_ok(dx.cpu().numpy(), dx_ref) <= RTOL
    assert normwise(dg.cpu().numpy(), dg_ref) <= RTOL
    assert normwise(db.cpu().numpy(), db_ref) <= RTOL
    # size-independent property: the row sums of the kept, rescaled softmax
    # are 1/(1-rate) times the kept probability mass, all finite and in range
    assert np.isfinite(rs).all() and (rs > 0).all() and (rs < 1.0 / (1 - 0.1) + 1e-5).all()


@pytest.mark.parametrize("dtype", [np.float64, np.float32])
@pytest.mark.parametrize("lanes,length", [(1, 1), (5, 252), (300, 77), (1000, 1)])
def test_cumsum_bit_exact(cuda, orc, dtype, lanes, length):
    x = np.random.default_rng(lanes).standard_normal((lanes, length)).astype(dtype)
    x[0, 0] = -0.0
    for rev in (False, True):
        assert bits_equal(cuda.cumsum(t(x), rev).cpu().numpy(), orc.cumsum(x, rev))
