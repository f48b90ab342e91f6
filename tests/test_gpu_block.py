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

pytestmark = pytest.mark.gpu


def reference(x, dy, w, heads, eps, dtype=None):
    import torch
    dtype = dtype or torch.float64
    T = {k: torch.tensor(v, dtype=dtype, requires_grad=True) for k, v in w.items()}
    X = torch.tensor(x, dtype=dtype, requires_grad=True)
    B, S, D = x.shape
    Dh = D // heads

    def ln(v, g, b):
        m = v.mean(-1, keepdim=True)
        c = v - m
        var = (c * c).mean(-1, keepdim=True)
        return c / torch.sqrt(var + eps) * g + b

    h1 = ln(X, T["ln1_gamma"], T["ln1_beta"])
    qkv = h1 @ T["w_qkv"]
    q, k, v = qkv.split(D, dim=-1)
    q = q.view(B, S, heads, Dh).transpose(1, 2)
    k = k.view(B, S, heads, Dh).transpose(1, 2)
    v = v.view(B, S, heads, Dh).transpose(1, 2)
    s = (q @ k.transpose(-1, -2)) * (1.0 / np.sqrt(Dh))
    mask = torch.ones(S, S, dtype=torch.bool).tril()
    s = torch.where(mask, s, torch.tensor(-float("inf"), dtype=dtype))
    o = (torch.softmax(s, -1) @ v).transpose(1, 2).reshape(B, S, D)
    x2 = X + o @ T["w_o"]
    h2 = ln(x2, T["ln2_gamma"], T["ln2_beta"])
    y = x2 + torch.nn.functional.gelu(h2 @ T["w_1"]) @ T["w_2"]
    y.backward(torch.tensor(dy, dtype=dtype))
    grads = {"d" + k: t.grad.double().numpy() for k, t in T.items()}
    grads["dx"] = X.grad.double().numpy()
    return y.detach().double().numpy(), grads


def normwise(got, ref):
    return float(np.abs(got.astype(np.float64) - ref).max() / np.abs(ref).max())


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
