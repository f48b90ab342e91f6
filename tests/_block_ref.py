"""float64 (and float32) autograd evaluation of the transformer block graph
in torch on the CPU: pre-LN, causal softmax attention with scale
1/sqrt(head_dim), exact-erf GELU MLP, no biases.  An independent check of
both the oracle's block restatement and the CUDA block."""
import numpy as np


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
