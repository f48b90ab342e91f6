"""Seeded synthetic inputs for the five benchmark configurations.

The reference publishes no datasets for these configurations (its MNIST
capture read local IDX files that are not available); every input here is
synthetic with the shapes and distributions the configurations name.
`numpy` generators feed the parity tests (the oracle reads the same arrays);
`torch_*` generators build the full-size inputs directly in device memory for
the benchmark.
"""
from __future__ import annotations

import numpy as np

# ---- config 1: 2-layer MLP, batch 128, 784 -> 256 (relu) -> 10, seed 0
MLP_SHAPE = dict(batch=128, din=784, dh=256, dout=10)


def mlp_inputs(batch=128, din=784, dh=256, dout=10, seed=0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((batch, din), dtype=np.float32)
    labels = rng.integers(0, dout, size=batch, dtype=np.int64)
    w1 = (rng.standard_normal((din, dh)) * np.sqrt(2.0 / din)).astype(np.float32)
    w2 = (rng.standard_normal((dh, dout)) * np.sqrt(2.0 / dh)).astype(np.float32)
    b1 = np.zeros(dh, np.float32)
    b2 = np.zeros(dout, np.float32)
    return x, labels, w1, b1, w2, b2


# ---- config 2: GEMM sweep, U(-1, 1), seed 1
GEMM_SIZES = (512, 1024, 2048, 4096, 8192)
BATCHED_GEMM = dict(batch=256, n=512)


def gemm_inputs(m, n, k, dtype=np.float32, seed=1, batch=None):
    rng = np.random.default_rng(seed)
    sa = (m, k) if batch is None else (batch, m, k)
    sb = (k, n) if batch is None else (batch, k, n)
    a = rng.uniform(-1.0, 1.0, size=sa).astype(dtype)
    b = rng.uniform(-1.0, 1.0, size=sb).astype(dtype)
    return a, b


# ---- config 3: fused chain on X [16384, 4096], seed 2
CHAIN_SHAPE = dict(rows=16384, hidden=4096)
CHAIN_EPS = np.float32(1e-5)
CHAIN_KEY = 42          # key_from_seed(42): the raw i64 bits ([05-OP-69])
CHAIN_RATE = np.float32(0.1)


def chain_inputs(rows=16384, hidden=4096, seed=2):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, hidden), dtype=np.float32)
    gamma = rng.uniform(0.5, 1.5, size=hidden).astype(np.float32)
    beta = (rng.standard_normal(hidden) * 0.1).astype(np.float32)
    return x, gamma, beta


# ---- config 5: vmap'd covariance / risk, 65536 x [252 x 64] f64, seed 4
PORTFOLIO_SHAPE = dict(count=65536, t=252, a=64)


def portfolio_inputs(count=65536, t=252, a=64, seed=4):
    rng = np.random.default_rng(seed)
    r = rng.normal(0.0005, 0.02, size=(count, t, a))
    e = rng.exponential(1.0, size=(count, a))
    w = e / e.sum(axis=1, keepdims=True)  # Dirichlet(1, ..., 1)
    return r, w


# ---------------------------------------------------------------- device-side

def torch_gemm_inputs(m, n, k, dtype, seed=1, batch=None, device="cuda"):
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    sa = (m, k) if batch is None else (batch, m, k)
    sb = (k, n) if batch is None else (batch, k, n)
    a = torch.rand(sa, generator=g, device=device, dtype=dtype) * 2 - 1
    b = torch.rand(sb, generator=g, device=device, dtype=dtype) * 2 - 1
    return a, b


def torch_chain_inputs(rows=16384, hidden=4096, seed=2, device="cuda"):
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn((rows, hidden), generator=g, device=device, dtype=torch.float32)
    gamma = torch.rand(hidden, generator=g, device=device, dtype=torch.float32) + 0.5
    beta = torch.randn(hidden, generator=g, device=device, dtype=torch.float32) * 0.1
    return x, gamma, beta


def torch_portfolio_inputs(count=65536, t=252, a=64, seed=4, device="cuda"):
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    r = torch.randn((count, t, a), generator=g, device=device, dtype=torch.float64) * 0.02 + 0.0005
    e = -torch.log(torch.rand((count, a), generator=g, device=device, dtype=torch.float64))
    w = e / e.sum(dim=1, keepdim=True)
    return r, w


def torch_mlp_inputs(seed=0, device="cuda", **shape):
    import torch
    arrs = mlp_inputs(seed=seed, **shape)
    return tuple(torch.from_numpy(np.ascontiguousarray(a)).to(device) for a in arrs)


# ---- config 4: transformer block, B=8, S=2048, d=1024, 16 heads x 64, ff 4096, seed 3
BLOCK_SHAPE = dict(batch=8, seq=2048, d_model=1024, heads=16, d_ff=4096)


def block_inputs(batch=8, seq=2048, d_model=1024, heads=16, d_ff=4096, seed=3):
    """x ~ N(0,1), upstream cotangent dy ~ N(0,1), Xavier-uniform weights
    (bound sqrt(6 / (fan_in + fan_out)) per matrix; the q, k, v blocks of
    w_qkv are three d x d matrices), layer-norm gamma = 1, beta = 0."""
    rng = np.random.default_rng(seed)
    d, f = d_model, d_ff

    def xavier(fi, fo, shape):
        a = np.sqrt(6.0 / (fi + fo))
        return rng.uniform(-a, a, size=shape).astype(np.float32)

    x = rng.standard_normal((batch, seq, d), dtype=np.float32)
    dy = rng.standard_normal((batch, seq, d), dtype=np.float32)
    w = {
        "w_qkv": np.concatenate([xavier(d, d, (d, d)) for _ in range(3)], axis=1),
        "w_o": xavier(d, d, (d, d)),
        "w_1": xavier(d, f, (d, f)),
        "w_2": xavier(f, d, (f, d)),
        "ln1_gamma": np.ones(d, np.float32), "ln1_beta": np.zeros(d, np.float32),
        "ln2_gamma": np.ones(d, np.float32), "ln2_beta": np.zeros(d, np.float32),
    }
    return x, dy, w


def torch_block_inputs(batch=8, seq=2048, d_model=1024, heads=16, d_ff=4096, seed=3, device="cuda"):
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    d, f = d_model, d_ff

    def xavier(fi, fo, shape):
        a = float(np.sqrt(6.0 / (fi + fo)))
        return (torch.rand(shape, generator=g, device=device) * 2 - 1) * a

    x = torch.randn((batch, seq, d), generator=g, device=device)
    dy = torch.randn((batch, seq, d), generator=g, device=device)
    w = {
        "w_qkv": torch.cat([xavier(d, d, (d, d)) for _ in range(3)], dim=1).contiguous(),
        "w_o": xavier(d, d, (d, d)), "w_1": xavier(d, f, (d, f)), "w_2": xavier(f, d, (f, d)),
        "ln1_gamma": torch.ones(d, device=device), "ln1_beta": torch.zeros(d, device=device),
        "ln2_gamma": torch.ones(d, device=device), "ln2_beta": torch.zeros(d, device=device),
    }
    return x, dy, w
