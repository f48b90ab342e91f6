"""Small single-launch cases of each hot kernel, for profiler captures.

    python -m chelis_b200.profile_cases gemm        # 8192^3 f32 3xTF32 (split + main kernel)
    python -m chelis_b200.profile_cases dgemm       # 4096^3 f64 DMMA
    python -m chelis_b200.profile_cases chain       # config 3 forward (saving state) + adjoint
    python -m chelis_b200.profile_cases portfolio   # config 5, 4096 portfolios
    python -m chelis_b200.profile_cases block       # config 4 step, batch 1
    python -m chelis_b200.profile_cases block8      # config 4 step at the headline batch of 8
                                                    # (launch lists only: one metric, one pass)
    python -m chelis_b200.profile_cases attention   # config 4 attention, 8 x 16 heads x 2048 x 64,
                                                    # fused forward + reverse mode
    python -m chelis_b200.profile_cases attention16 # the same kernels on 16 heads (one batch item)
    python -m chelis_b200.profile_cases fused       # generic FusedElem groups on 16384 x 4096 f32:
                                                    # x*gamma+beta, then sum of squares per row
    python -m chelis_b200.profile_cases batched     # config 2b: 256 products of 512^3 f32 in one
                                                    # batched call (persistent CTA-pair kernel)
    python -m chelis_b200.profile_cases mlp         # config 1 step, called 4 times: a direct run,
                                                    # the capture, then two replays of its CUDA graph

Each case builds its inputs on the device, runs the hot path once and
synchronises; inputs exceed the 126 MB L2 except where the case is smaller
by construction (the MLP step and the batched 512^3 products).
"""
from __future__ import annotations

import sys

import torch

from . import ops
from . import workloads as W


def run(case: str) -> None:
    torch.cuda.set_device(0)
    if case == "gemm":
        a, b = W.torch_gemm_inputs(8192, 8192, 8192, torch.float32, seed=1)
        ops.matmul(a, b)
    elif case == "dgemm":
        a, b = W.torch_gemm_inputs(4096, 4096, 4096, torch.float64, seed=1)
        ops.matmul(a, b)
    elif case == "chain":
        x, g, be = W.torch_chain_inputs()
        _, saved = ops.chain_fwd_save(x, g, be, 1e-5, 42, 0.1)
        ops.chain_bwd_saved(x, g, be, 1e-5, 0.1, saved)
    elif case == "portfolio":
        r, w = W.torch_portfolio_inputs(count=4096)
        ops.portfolio(r, w)
    elif case == "block":
        x, dy, w = W.torch_block_inputs(**dict(W.BLOCK_SHAPE, batch=1))
        ops.block_step(x, w, W.BLOCK_SHAPE["heads"], 1e-5, dy)
    elif case == "block8":
        x, dy, w = W.torch_block_inputs(**W.BLOCK_SHAPE)
        ops.block_step(x, w, W.BLOCK_SHAPE["heads"], 1e-5, dy)
    elif case in ("attention", "attention16"):
        bh = 128 if case == "attention" else 16
        g = torch.Generator(device="cuda").manual_seed(3)
        q, k, v, do = (torch.randn(bh, 2048, 64, device="cuda", generator=g) for _ in range(4))
        o, lse = ops.attention_causal(q, k, v, 0.125, with_lse=True)
        ops.attention_causal_bwd(q, k, v, o, lse, do, 0.125)
    elif case == "fused":
        from . import fused as F
        x, g, be = W.torch_chain_inputs()
        ops.fused_elementwise(F.parse("mul x0 x1; add v0 x2"), [x, g, be])
        ops.fused_reduce(F.parse("mul x0 x0"), [x], axis=1)
    elif case == "batched":
        a, b = W.torch_gemm_inputs(512, 512, 512, torch.float32, seed=1, batch=256)
        ops.matmul(a, b)
    elif case == "mlp":
        x, labels, w1, b1, w2, b2 = W.torch_mlp_inputs()
        for _ in range(4):  # outputs dropped at once: the next call reuses their memory
            ops.mlp_step(x, labels, w1, b1, w2, b2)
    else:
        raise SystemExit(f"unknown case {case!r}")
    torch.cuda.synchronize()
    ops.device_status()
    print("done", case)


if __name__ == "__main__":
    run(sys.argv[1] if len(sys.argv) > 1 else "gemm")
