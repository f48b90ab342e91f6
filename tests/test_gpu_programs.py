"""Whole programs on the GPU: the vmap'd covariance / risk (config 5), the MLP
training step (config 1), and the generated-entry device ABI (`*_device`
entries with chelis_device_tensor_owner inputs and outputs)."""
import ctypes

import numpy as np
import pytest

from chelis_b200 import lib as L
from chelis_b200 import workloads as W

pytestmark = pytest.mark.gpu


def t(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


@pytest.mark.parametrize("count", [1, 3, 300])
def test_portfolio_matches_oracle(cuda, orc, count):
    r, w = W.portfolio_inputs(count=count, seed=count)
    sigma, risk, cum = cuda.portfolio(t(r), t(w))
    s_ref, risk_ref, cum_ref = orc.portfolio(r, w)
    sigma, risk, cum = sigma.cpu().numpy(), risk.cpu().numpy(), cum.cpu().numpy()
    # componentwise bound of the t-length dot products of the centred returns
    c = r - r.mean(axis=1, keepdims=True)
    bound = np.einsum("pti,ptj->pij", np.abs(c), np.abs(c)) / 251.0
    assert float((np.abs(sigma - s_ref) / bound).max()) <= 1e-12
    assert float((np.abs(risk - risk_ref) / risk_ref).max()) <= 1e-12
    # R.w and its sequential prefix follow the C lane's order exactly
    assert (cum.view(np.uint64) == cum_ref.view(np.uint64)).all()


def test_portfolio_full_count_property(cuda, orc):
    """Config 5 at its full batch (65536 portfolios): every portfolio on the
    GPU; a sample checked against the oracle and size-independent properties
    (symmetric PSD diagonal, risk^2 = w.Sigma.w) on all of them."""
    import torch
    r, w = W.torch_portfolio_inputs()
    sigma, risk, cum = cuda.portfolio(r, w)
    torch.cuda.synchronize()
    assert torch.isfinite(sigma).all() and (risk > 0).all()
    assert torch.allclose(sigma, sigma.transpose(1, 2), rtol=1e-13, atol=0)
    q = torch.einsum("pi,pij,pj->p", w, sigma, w)
    assert torch.allclose(risk * risk, q, rtol=1e-12, atol=0)
    idx = [0, 1, 777, 65535]
    rs, ws = r[idx].cpu().numpy(), w[idx].cpu().numpy()
    s_ref, risk_ref, cum_ref = orc.portfolio(rs, ws)
    assert np.allclose(sigma[idx].cpu().numpy(), s_ref, rtol=1e-11, atol=1e-18)
    assert (cum[idx].cpu().numpy().view(np.uint64) == cum_ref.view(np.uint64)).all()


@pytest.mark.parametrize("shape", [dict(batch=128, din=784, dh=256, dout=10),
                                   dict(batch=7, din=33, dh=19, dout=3)])
def test_mlp_step_matches_oracle(cuda, orc, shape):
    x, labels, w1, b1, w2, b2 = W.mlp_inputs(**shape)
    b1 = (np.random.default_rng(2).standard_normal(shape["dh"]) * 0.05).astype(np.float32)
    got = [v.cpu().numpy() for v in cuda.mlp_step(t(x), t(labels), t(w1), t(b1), t(w2), t(b2))]
    ref = orc.mlp_step(x, labels, w1, b1, w2, b2)
    assert abs(got[0][0] - ref[0]) <= 1e-5 * abs(ref[0])
    for g, r in zip(got[1:], ref[1:]):
        assert np.abs(g - r).max() <= 1e-5 * np.abs(r).max()


def test_mlp_rejects_out_of_range_label(cuda):
    x, labels, w1, b1, w2, b2 = W.mlp_inputs(batch=4, din=8, dh=8, dout=3)
    labels[2] = 3
    cuda.mlp_step(t(x), t(labels), t(w1), t(b1), t(w2), t(b2))  # asynchronous
    with pytest.raises(L.ChelisCudaError, match="gather"):
        cuda.device_status()
    cuda.device_status()  # read-and-clear: the next check is clean


def _owner_from(tensor, keep):
    shape = (ctypes.c_int64 * tensor.dim())(*tensor.shape)
    keep.append(shape)
    dt = {np.float32: L.DTYPE_F32, np.float64: L.DTYPE_F64}[
        {4: np.float32, 8: np.float64}[tensor.element_size()]]
    o = L.load().chelis_device_tensor_borrow_shape(dt, tensor.dim(), shape, tensor.data_ptr(),
                                                   tensor.numel() * tensor.element_size())
    assert o, L.last_error()
    return o


def _owner_array(lib, owner):
    v = lib.chelis_device_tensor_view(owner).contents
    shape = tuple(v.shape[i] for i in range(v.rank))
    nbytes = v.count * (4 if v.dtype == L.DTYPE_F32 else 8)
    host = np.empty(shape, np.float32 if v.dtype == L.DTYPE_F32 else np.float64)
    L.call("chelis_device_tensor_copy_to_host_bytes", host.ctypes.data, nbytes, owner)
    L.call("chelis_cuda_synchronize")
    return host


def test_generated_entry_device_abi(cuda, orc):
    import torch
    lib = L.load()
    keep = []
    x, g, b = W.chain_inputs(32, 1024, seed=3)
    X, G, B = t(x), t(g), t(b)
    cuda._prepare(X)
    ins = (ctypes.c_void_p * 3)(*[_owner_from(v, keep) for v in (X, G, B)])
    outs = (ctypes.c_void_p * 3)()
    L.call("chelis_chain_fwd_device", ins, 3, outs, 1)
    rs = _owner_array(lib, outs[0])
    ref = orc.chain_fwd(x, g, b, np.float32(1e-5), 42, np.float32(0.1))
    assert np.abs(rs - ref).max() <= 1e-5 * np.abs(ref).max()
    lib.chelis_device_tensor_release(outs[0])
    L.call("chelis_chain_grad_device", ins, 3, outs, 3)
    dx_ref, dg_ref, db_ref = orc.chain_bwd(x, g, b, np.float32(1e-5), 42, np.float32(0.1))
    for o, r in zip(outs, (dx_ref, dg_ref, db_ref)):
        got = _owner_array(lib, o)
        assert np.abs(got - r).max() <= 1e-5 * np.abs(r).max()
        lib.chelis_device_tensor_release(o)
    # matmul program: rank-3 batched f64
    a, bm = W.gemm_inputs(40, 30, 20, np.float64, seed=1, batch=2)
    A, Bm = t(a), t(bm)
    ins2 = (ctypes.c_void_p * 2)(_owner_from(A, keep), _owner_from(Bm, keep))
    out2 = (ctypes.c_void_p * 1)()
    L.call("chelis_matmul_device", ins2, 2, out2, 1)
    c = _owner_array(lib, out2[0])
    for i in range(2):
        assert np.abs(c[i] - orc.gemm(a[i], bm[i])).max() <= 1e-12 * 20
    # clone of a borrowed owner is an owned canonical copy
    cl = lib.chelis_device_tensor_clone(ins2[0])
    assert lib.chelis_device_tensor_view(cl).contents.ownership == 1
    assert (_owner_array(lib, cl) == a).all()
    for o in (cl, out2[0], *ins, *ins2):
        lib.chelis_device_tensor_release(o)
    # wrong arity is a domain error, outputs untouched
    assert lib.chelis_chain_fwd_device(ins, 2, outs, 1) == 1
    torch.cuda.synchronize()
