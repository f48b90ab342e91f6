"""EXACT rows mode with the correctly rounded device exp / log: the kernels
that evaluate exp / log now give the C lane's results bit for bit (CORE-MATH
on the oracle's side), where before they differed by CUDA's few ulp."""
import numpy as np
import pytest
import torch

from chelis_b200 import fused as F
from chelis_b200 import lib as L
from chelis_b200 import workloads as W

pytestmark = pytest.mark.gpu


def t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def bits_equal(a, b):
    a = np.asarray(a)
    b = np.asarray(b)
    ia = a.view(np.uint32 if a.dtype == np.float32 else np.uint64)
    ib = b.view(np.uint32 if b.dtype == np.float32 else np.uint64)
    return bool(((ia == ib) | (np.isnan(a) & np.isnan(b))).all())


@pytest.mark.parametrize("rows,cols", [(1, 1), (16, 10), (64, 4096), (9, 3000), (3, 8192)])
def test_softmax_exact_mode_bit_exact(cuda, orc, rows, cols):
    x = (np.random.default_rng(cols).standard_normal((rows, cols)) * 4).astype(np.float32)
    with cuda.rows_mode(L.ROWS_EXACT):
        y = cuda.softmax_rows(t(x)).cpu().numpy()
    assert bits_equal(y, orc.softmax_rows(x))


@pytest.mark.parametrize("jit", [True, False])
@pytest.mark.parametrize("chain", ["exp x0", "log x0", "sub x0 x1; exp v0; mul v1 x1; log v2"])
def test_fused_exp_log_exact_mode_bit_exact(cuda, orc, jit, chain):
    rng = np.random.default_rng(11)
    a = (rng.standard_normal((64, 512)) * 3).astype(np.float32)
    a[0, :8] = [0.0, -0.0, np.inf, -np.inf, np.nan, 1e-40, -1e-40, 88.7]
    b = np.abs(rng.standard_normal((64, 512))).astype(np.float32) + 0.5
    prog = F.parse(chain)
    with cuda.rows_mode(L.ROWS_EXACT), cuda.fused_jit(jit):
        got = cuda.fused_elementwise(prog, [t(a), t(b)]).cpu().numpy()
    want = orc.fused_elementwise(F.triplets(prog), [a, b])
    assert bits_equal(got, want)


def test_cross_entropy_exact_mode_loss_bit_exact(cuda, orc):
    rng = np.random.default_rng(3)
    z = (rng.standard_normal((128, 10)) * 3).astype(np.float32)
    labels = rng.integers(0, 10, 128).astype(np.int64)
    with cuda.rows_mode(L.ROWS_EXACT):
        loss, dz = cuda.cross_entropy(t(z), t(labels))
    ref_loss, ref_dz = orc.cross_entropy(z, labels)
    assert bits_equal(np.float32(float(loss)), np.float32(ref_loss))
    assert bits_equal(dz.cpu().numpy(), ref_dz)


def test_mlp_step_bit_exact(cuda, orc):
    x, labels, w1, b1, w2, b2 = W.mlp_inputs()
    b1 = (np.random.default_rng(2).standard_normal(b1.shape) * 0.05).astype(np.float32)
    got = [v.cpu().numpy() for v in cuda.mlp_step(t(x), t(labels), t(w1), t(b1), t(w2), t(b2))]
    ref = orc.mlp_step(x, labels, w1, b1, w2, b2)
    assert bits_equal(np.float32(got[0][0]), np.float32(ref[0]))
    for g, r in zip(got[1:], ref[1:]):
        assert bits_equal(g, r)


@pytest.mark.parametrize("rows,hidden", [(5, 100), (64, 4096), (17, 4095)])
def test_chain_forward_exact_mode_bit_exact(cuda, orc, rows, hidden):
    x, g, b = W.chain_inputs(rows, hidden, seed=rows + hidden)
    eps, key, rate = W.CHAIN_EPS, W.CHAIN_KEY, W.CHAIN_RATE
    with cuda.rows_mode(L.ROWS_EXACT):
        rs = cuda.chain_fwd(t(x), t(g), t(b), float(eps), key, float(rate), 0).cpu().numpy()
    assert bits_equal(rs, orc.chain_fwd(x, g, b, eps, key, rate, 0))


def test_mlp_step_graph_replays_read_current_inputs(cuda, orc):
    """A repeated chelis_cuda_mlp_step call (same buffers and stream) runs as
    a captured CUDA graph from the second call on; every call, the direct
    first one, the capturing second one and the replays, must see the
    inputs as they are at that call and stay bit-identical to the oracle."""
    import torch
    from chelis_b200 import lib as L
    x, labels, w1, b1, w2, b2 = W.mlp_inputs()
    batch, din = x.shape
    dh, dout = w1.shape[1], w2.shape[1]
    dev = [t(v) for v in (x, labels, w1, b1, w2, b2)]
    outs = [torch.empty(1, dtype=torch.float32, device="cuda"),
            torch.empty_like(dev[2]), torch.empty_like(dev[3]),
            torch.empty_like(dev[4]), torch.empty_like(dev[5])]
    rng = np.random.default_rng(11)
    launches = []
    for step in range(4):
        x_now = (x + np.float32(0.01 * step) * rng.standard_normal(x.shape).astype(np.float32))
        b1_now = (rng.standard_normal(b1.shape) * 0.05).astype(np.float32)
        dev[0].copy_(torch.from_numpy(x_now))
        dev[3].copy_(torch.from_numpy(b1_now))
        before = L.load().chelis_cuda_launch_count()
        L.call("chelis_cuda_mlp_step", *(v.data_ptr() for v in dev), batch, din, dh, dout,
               *(o.data_ptr() for o in outs))
        torch.cuda.synchronize()
        launches.append(L.load().chelis_cuda_launch_count() - before)
        cuda.device_status()
        ref = orc.mlp_step(x_now, labels, w1, b1_now, w2, b2)
        got = [o.cpu().numpy() for o in outs]
        assert bits_equal(np.float32(got[0][0]), np.float32(ref[0])), step
        for g, r in zip(got[1:], ref[1:]):
            assert bits_equal(g, r), step
    # the graph runs the same kernels the direct path launches
    assert len(set(launches)) == 1 and launches[0] >= 10, launches
