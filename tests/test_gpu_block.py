"""Transformer block (config 4) forward + vector-Jacobian product on the GPU
against a float64 autograd evaluation of the same graph (pre-LN, causal
softmax attention with scale 1/sqrt(head_dim), exact-erf GELU MLP, no
biases).  The block is a composition of kernels whose parts are pinned to
the oracle elsewhere (GEMM, layer norm, softmax and its adjoint).  The
whole graph chains up to twelve matmuls and row reductions (each within
f32 rel 1e-5 of its own exact value), so the rounding compounds: each output
tensor must be within normwise rel 2e-5 of the float64 evaluation, or no
further from it than three times a plain float32 evaluation of the same
graph (torch, CPU) is.
"""
import numpy as np
import pytest

from chelis_b200 import workloads as W
from _block_ref import normwise, reference

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [
    dict(batch=2, seq=64, d_model=128, heads=2, d_ff=512),
    dict(batch=1, seq=256, d_model=256, heads=4, d_ff=1024),
    dict(batch=1, seq=100, d_model=64, heads=4, d_ff=96),
])
def test_block_fwd_vjp_matches_float64_autograd(cuda, shape):
    import torch
    x, dy, w = W.block_inputs(seed=7, **shape)
    heads = shape["heads"]
    wt = {k: torch.from_numpy(v).cuda() for k, v in w.items()}
    out = cuda.block_step(torch.from_numpy(x).cuda(), wt, heads, 1e-5, torch.from_numpy(dy).cuda())
    torch.cuda.synchronize()
    cuda.device_status()
    y_ref, g_ref = reference(x, dy, w, heads, 1e-5)
    y32, g32 = reference(x, dy, w, heads, 1e-5, torch.float32)
    bound = lambda f32, ref: max(2e-5, 3.0 * normwise(f32, ref))  # noqa: E731
    assert normwise(out["y"].cpu().numpy(), y_ref) <= bound(y32, y_ref)
    for name, ref in g_ref.items():
        got = normwise(out[name].cpu().numpy(), ref)
        assert got <= bound(g32[name], ref), (name, got, normwise(g32[name], ref))


def test_block_workspace_entry_matches_pool_entry(cuda):
    import torch
    shape = dict(batch=1, seq=128, d_model=128, heads=2, d_ff=256)
    x, dy, w = W.block_inputs(seed=9, **shape)
    X, DY = torch.from_numpy(x).cuda(), torch.from_numpy(dy).cuda()
    wt = {k: torch.from_numpy(v).cuda() for k, v in w.items()}
    a = cuda.block_step(X, wt, 2, 1e-5, DY)
    ws = cuda.block_workspace(X, wt, 2)
    b = cuda.block_step(X, wt, 2, 1e-5, DY, workspace=ws)
    for k in a:
        assert torch.equal(a[k], b[k]), k


def _oracle_bound_check(out, y_ref, g_ref, tol):
    errs = {"y": normwise(out["y"].cpu().numpy(), y_ref)}
    errs.update({k: normwise(out[k].cpu().numpy(), v) for k, v in g_ref.items()})
    bad = {k: e for k, e in errs.items() if not e <= tol}
    assert not bad, (bad, errs)
    return errs


@pytest.mark.parametrize("shape", [
    dict(batch=2, seq=64, d_model=128, heads=2, d_ff=512),
    dict(batch=1, seq=300, d_model=256, heads=4, d_ff=1024),
])
def test_block_matches_oracle_small(cuda, orc, shape):
    """The CUDA block against the oracle's restatement of the reference graph
    (orc_block_step): every output within normwise f32 rel 1e-5."""
    import torch
    x, dy, w = W.block_inputs(seed=11, **shape)
    wt = {k: torch.from_numpy(v).cuda() for k, v in w.items()}
    out = cuda.block_step(torch.from_numpy(x).cuda(), wt, shape["heads"], 1e-5,
                          torch.from_numpy(dy).cuda())
    torch.cuda.synchronize()
    cuda.device_status()
    y_ref, g_ref = orc.block_step(x, w, shape["heads"], 1e-5, dy)
    _oracle_bound_check(out, y_ref, g_ref, 1e-5)


def test_block_config4_shape_matches_oracle(cuda, orc):
    """Config 4 at its own shape (S 2048, d_model 1024, 16 heads of 64, d_ff
    4096; one sample of the batch of 8, seed 3) against the oracle: y, dx and
    all eight parameter gradients within normwise f32 rel 1e-5."""
    import torch
    shape = dict(W.BLOCK_SHAPE, batch=1)
    x, dy, w = W.block_inputs(seed=3, **shape)
    wt = {k: torch.from_numpy(v).cuda() for k, v in w.items()}
    out = cuda.block_step(torch.from_numpy(x).cuda(), wt, shape["heads"], 1e-5,
                          torch.from_numpy(dy).cuda())
    torch.cuda.synchronize()
    cuda.device_status()
    y_ref, g_ref = orc.block_step(x, w, shape["heads"], 1e-5, dy)
    errs = _oracle_bound_check(out, y_ref, g_ref, 1e-5)
    print("config-4 normwise errors vs oracle:", {k: f"{v:.2e}" for k, v in errs.items()})


def test_block_step_dp_is_block_step_on_one_rank(cuda):
    """Without a multi-rank communicator the data-parallel entry runs the
    same step: bit-identical outputs."""
    import torch
    shape = dict(batch=2, seq=128, d_model=128, heads=2, d_ff=256)
    x, dy, w = W.block_inputs(seed=13, **shape)
    X, DY = torch.from_numpy(x).cuda(), torch.from_numpy(dy).cuda()
    wt = {k: torch.from_numpy(v).cuda() for k, v in w.items()}
    a = cuda.block_step(X, wt, 2, 1e-5, DY)
    b = cuda.block_step(X, wt, 2, 1e-5, DY, reduce_grads=True)
    for k in a:
        assert torch.equal(a[k], b[k]), k
