"""Host-side calls of the CUDA backend on torch-owned device memory.

torch provides device memory and streams only; every computation is one of
libchelis_cuda.so's kernels, reached through the C ABI (chelis_b200.lib).
Each wrapper enqueues on torch's current CUDA stream and returns torch
tensors.  Names and argument meanings follow the reference's operations
(matmul, layer_norm, softmax, dropout, sum, max_reduce, count, cumsum).
"""
from __future__ import annotations

import contextlib
import ctypes

import torch

from . import lib as L

_initialised: set[int] = set()


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _prepare(*tensors: torch.Tensor) -> None:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("chelis_b200 ops take CUDA tensors (device memory)")
        if not t.is_contiguous():
            raise ValueError("chelis_b200 ops take contiguous tensors")
        dev = t.device.index
    if dev is None:
        dev = torch.cuda.current_device()
    if dev not in _initialised:
        L.call("chelis_cuda_init", dev)
        _initialised.add(dev)
    L.load().chelis_cuda_set_stream(torch.cuda.current_stream(dev).cuda_stream)


@contextlib.contextmanager
def gemm_mode(mode: int):
    lib = L.load()
    old = lib.chelis_cuda_get_gemm_mode()
    L.call("chelis_cuda_set_gemm_mode", mode)
    try:
        yield
    finally:
        L.call("chelis_cuda_set_gemm_mode", old)


@contextlib.contextmanager
def dgemm_kernel(kernel: int):
    """f64 GEMM kernel (L.DGEMM_AUTO / _DMMA / _FFMA) for this thread only."""
    L.call("chelis_cuda_set_thread_modes", -1, -1, kernel)
    try:
        yield
    finally:
        L.call("chelis_cuda_set_thread_modes", -1, -1, -1)


@contextlib.contextmanager
def gemm_pairs(enable: bool):
    """3xTF32 main kernel on CTA pairs (256 x 256 tiles, the default) or on
    single CTAs (128 x 256 tiles)."""
    lib = L.load()
    old = lib.chelis_cuda_get_gemm_pairs()
    L.call("chelis_cuda_set_gemm_pairs", int(enable))
    try:
        yield
    finally:
        L.call("chelis_cuda_set_gemm_pairs", old)


@contextlib.contextmanager
def fused_jit(enable: bool):
    """FusedElem elementwise groups through per-chain compiled kernels (the
    default) or the ahead-of-time interpreter; the same bits either way."""
    lib = L.load()
    old = lib.chelis_cuda_get_fused_jit()
    L.call("chelis_cuda_set_fused_jit", int(enable))
    try:
        yield
    finally:
        L.call("chelis_cuda_set_fused_jit", old)


@contextlib.contextmanager
def rows_mode(mode: int):
    lib = L.load()
    old = lib.chelis_cuda_get_rows_mode()
    L.call("chelis_cuda_set_rows_mode", mode)
    try:
        yield
    finally:
        L.call("chelis_cuda_set_rows_mode", old)


def device_status() -> None:
    """Raise if a bounded device wait gave up since the last check."""
    L.call("chelis_cuda_device_status")


def launch_count() -> int:
    return int(L.load().chelis_cuda_launch_count())


# ---------------------------------------------------------------- matmul

def matmul(a: torch.Tensor, b: torch.Tensor, trans_a: bool = False, trans_b: bool = False,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """op(A).op(B) for f32 (3xTF32 tensor cores, or the exact tree mode) or f64
    (DMMA); rank-3 operands are a strided batch."""
    if a.dtype != b.dtype or a.dtype not in (torch.float32, torch.float64):
        raise ValueError("matmul takes two f32 or two f64 tensors")
    batched = a.dim() == 3
    if batched != (b.dim() == 3) or a.dim() not in (2, 3):
        raise ValueError("matmul takes rank-2 or rank-3 operands of equal rank")
    _prepare(a, b, out)
    ar, ac = a.shape[-2:]
    br, bc = b.shape[-2:]
    m, k = (ac, ar) if trans_a else (ar, ac)
    k2, n = (bc, br) if trans_b else (br, bc)
    if k != k2:
        raise ValueError(f"contraction extents differ: {k} vs {k2}")
    batch = a.shape[0] if batched else 1
    shape = (batch, m, n) if batched else (m, n)
    if out is None:
        out = torch.empty(shape, dtype=a.dtype, device=a.device)
    name = "chelis_cuda_sgemm" if a.dtype == torch.float32 else "chelis_cuda_dgemm"
    L.call(name, int(trans_a), int(trans_b), m, n, k, a.data_ptr(), ac, ar * ac,
           b.data_ptr(), bc, br * bc, out.data_ptr(), n, m * n, batch)
    return out


def matmul_host(a: torch.Tensor, b: torch.Tensor, trans_a: bool = False, trans_b: bool = False,
                out: torch.Tensor | None = None, device: int | None = None) -> torch.Tensor:
    """op(A).op(B) for host (CPU) tensors through chelis_cuda_[sd]gemm_host:
    uploads, GEMM panels and read-back overlap on the GPU's copy engines.
    Returns once the result is in `out` (pinned output memory is allocated
    when `out` is None and `a` is pinned)."""
    if a.device.type != "cpu" or b.device.type != "cpu":
        raise ValueError("matmul_host takes host tensors")
    if a.dtype != b.dtype or a.dtype not in (torch.float32, torch.float64):
        raise ValueError("matmul_host takes two f32 or two f64 tensors")
    if not (a.is_contiguous() and b.is_contiguous()):
        raise ValueError("matmul_host takes contiguous tensors")
    batched = a.dim() == 3
    if batched != (b.dim() == 3) or a.dim() not in (2, 3):
        raise ValueError("matmul_host takes rank-2 or rank-3 operands of equal rank")
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
    with torch.cuda.device(dev):
        _prepare()
        ar, ac = a.shape[-2:]
        br, bc = b.shape[-2:]
        m, k = (ac, ar) if trans_a else (ar, ac)
        k2, n = (bc, br) if trans_b else (br, bc)
        if k != k2:
            raise ValueError(f"contraction extents differ: {k} vs {k2}")
        batch = a.shape[0] if batched else 1
        shape = (batch, m, n) if batched else (m, n)
        if out is None:
            out = torch.empty(shape, dtype=a.dtype, pin_memory=a.is_pinned())
        elif out.device.type != "cpu" or not out.is_contiguous() or tuple(out.shape) != shape:
            raise ValueError("out must be a contiguous host tensor of the product's shape")
        name = "chelis_cuda_sgemm_host" if a.dtype == torch.float32 else "chelis_cuda_dgemm_host"
        L.call(name, int(trans_a), int(trans_b), m, n, k, a.data_ptr(), ac, ar * ac,
               b.data_ptr(), bc, br * bc, out.data_ptr(), n, m * n, batch)
        torch.cuda.current_stream(dev).synchronize()
    return out


def attention_causal(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                     with_lse: bool = False):
    """softmax(where(causal, (q.k^T)*scale, -inf)).v for f32 [..., seq, dh]
    heads (flattened to [bh, seq, dh]); head dims 32 and 64."""
    if not (q.dtype == k.dtype == v.dtype == torch.float32) or q.shape != k.shape or q.shape != v.shape:
        raise ValueError("attention_causal takes three f32 tensors of one shape")
    _prepare(q, k, v)
    seq, dh = q.shape[-2:]
    bh = q.numel() // (seq * dh) if q.numel() else 0
    o = torch.empty_like(q)
    lse = torch.empty(q.shape[:-1], dtype=torch.float32, device=q.device) if with_lse else None
    L.call("chelis_cuda_attention_causal_fwd", bh, seq, dh, float(scale), q.data_ptr(),
           k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr() if with_lse else None)
    return (o, lse) if with_lse else o


def attention_causal_bwd(q, k, v, o, lse, dout, scale: float):
    """(dq, dk, dv) of attention_causal given its output o and lse."""
    _prepare(q, k, v, o, lse, dout)
    seq, dh = q.shape[-2:]
    bh = q.numel() // (seq * dh) if q.numel() else 0
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    L.call("chelis_cuda_attention_causal_bwd", bh, seq, dh, float(scale), q.data_ptr(),
           k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(), dout.data_ptr(),
           dq.data_ptr(), dk.data_ptr(), dv.data_ptr())
    return dq, dk, dv


# ---------------------------------------------------------------- rows

def row_sum(x: torch.Tensor) -> torch.Tensor:
    _prepare(x)
    out = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    L.call("chelis_cuda_row_sum_f32", x.data_ptr(), x.shape[0], x.shape[1], out.data_ptr())
    return out


def col_sum(x: torch.Tensor) -> torch.Tensor:
    _prepare(x)
    out = torch.empty(x.shape[1], dtype=torch.float32, device=x.device)
    L.call("chelis_cuda_col_sum_f32", x.data_ptr(), x.shape[0], x.shape[1], out.data_ptr())
    return out


def row_max(x: torch.Tensor) -> torch.Tensor:
    _prepare(x)
    out = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    L.call("chelis_cuda_row_max_f32", x.data_ptr(), x.shape[0], x.shape[1], out.data_ptr())
    return out


def count(x: torch.Tensor) -> int:
    _prepare(x)
    out = torch.empty(1, dtype=torch.int64, device=x.device)
    L.call("chelis_cuda_count_bool", x.data_ptr(), x.numel(), out.data_ptr())
    return int(out.item())


def dropout(x: torch.Tensor, key: int, rate: float, index_base: int = 0) -> torch.Tensor:
    _prepare(x)
    y = torch.empty_like(x)
    L.call("chelis_cuda_dropout_f32", x.data_ptr(), y.data_ptr(), x.numel(), key, rate, index_base)
    return y


def dropout_mask(n: int, key: int, rate: float, index_base: int = 0,
                 device: torch.device | None = None) -> torch.Tensor:
    keep = torch.empty(n, dtype=torch.uint8, device=device or "cuda")
    _prepare(keep)
    L.call("chelis_cuda_dropout_mask", keep.data_ptr(), n, key, rate, index_base)
    return keep


def layer_norm(x, gamma, beta, eps: float) -> torch.Tensor:
    _prepare(x, gamma, beta)
    y = torch.empty_like(x)
    L.call("chelis_cuda_layer_norm_f32", x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), eps,
           y.data_ptr(), x.shape[0], x.shape[1])
    return y


def softmax_rows(x) -> torch.Tensor:
    _prepare(x)
    y = torch.empty_like(x)
    L.call("chelis_cuda_softmax_rows_f32", x.data_ptr(), y.data_ptr(), x.shape[0], x.shape[1])
    return y


def softmax_rows_bwd(y, g) -> torch.Tensor:
    _prepare(y, g)
    dx = torch.empty_like(y)
    L.call("chelis_cuda_softmax_rows_bwd_f32", y.data_ptr(), g.data_ptr(), dx.data_ptr(),
           y.shape[0], y.shape[1])
    return dx


def chain_fwd(x, gamma, beta, eps: float, key: int, rate: float, index_base: int = 0,
              want_stats: bool = False):
    _prepare(x, gamma, beta)
    rows, hidden = x.shape
    rowsum = torch.empty(rows, dtype=torch.float32, device=x.device)
    stats = torch.empty((rows, 4), dtype=torch.float32, device=x.device) if want_stats else None
    L.call("chelis_cuda_chain_fwd", x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), eps, key,
           rate, rows, hidden, index_base, rowsum.data_ptr(), _ptr(stats))
    return (rowsum, stats) if want_stats else rowsum


def chain_bwd(x, gamma, beta, eps: float, key: int, rate: float, index_base: int = 0,
              stats: torch.Tensor | None = None):
    _prepare(x, gamma, beta, stats)
    rows, hidden = x.shape
    dx = torch.empty_like(x)
    dg = torch.empty(hidden, dtype=torch.float32, device=x.device)
    db = torch.empty(hidden, dtype=torch.float32, device=x.device)
    L.call("chelis_cuda_chain_bwd", x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), eps, key,
           rate, rows, hidden, index_base, _ptr(stats), dx.data_ptr(), dg.data_ptr(),
           db.data_ptr())
    return dx, dg, db


def chain_fwd_save(x, gamma, beta, eps: float, key: int, rate: float, index_base: int = 0):
    """Forward that also returns the saved state (statistics + keep bits)."""
    _prepare(x, gamma, beta)
    rows, hidden = x.shape
    nbytes = int(L.load().chelis_cuda_chain_saved_bytes(rows, hidden))
    if nbytes < 0:
        raise ValueError("unsupported chain shape")
    saved = torch.empty(max(nbytes, 16) // 4, dtype=torch.float32, device=x.device)
    rowsum = torch.empty(rows, dtype=torch.float32, device=x.device)
    L.call("chelis_cuda_chain_fwd_save", x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), eps, key,
           rate, rows, hidden, index_base, rowsum.data_ptr(), saved.data_ptr())
    return rowsum, saved


def chain_bwd_saved(x, gamma, beta, eps: float, rate: float, saved: torch.Tensor):
    _prepare(x, gamma, beta, saved)
    rows, hidden = x.shape
    dx = torch.empty_like(x)
    dg = torch.empty(hidden, dtype=torch.float32, device=x.device)
    db = torch.empty(hidden, dtype=torch.float32, device=x.device)
    L.call("chelis_cuda_chain_bwd_saved", x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), eps,
           rate, rows, hidden, saved.data_ptr(), dx.data_ptr(), dg.data_ptr(), db.data_ptr())
    return dx, dg, db


def cumsum(x: torch.Tensor, reverse: bool = False) -> torch.Tensor:
    _prepare(x)
    y = torch.empty_like(x)
    name = "chelis_cuda_cumsum_f64" if x.dtype == torch.float64 else "chelis_cuda_cumsum_f32"
    L.call(name, x.data_ptr(), y.data_ptr(), x.shape[0], x.shape[1], int(reverse))
    return y


# ---------------------------------------------------------------- programs

def portfolio(r: torch.Tensor, w: torch.Tensor):
    _prepare(r, w)
    count_, t, a = r.shape
    sigma = torch.empty((count_, a, a), dtype=torch.float64, device=r.device)
    risk = torch.empty(count_, dtype=torch.float64, device=r.device)
    cum = torch.empty((count_, t), dtype=torch.float64, device=r.device)
    L.call("chelis_cuda_portfolio_f64", r.data_ptr(), w.data_ptr(), count_, t, a,
           sigma.data_ptr(), risk.data_ptr(), cum.data_ptr())
    return sigma, risk, cum


BLOCK_WEIGHTS = ("w_qkv", "w_o", "w_1", "w_2", "ln1_gamma", "ln1_beta", "ln2_gamma", "ln2_beta")


def block_step(x, weights: dict, heads: int, eps: float = 1e-5, dy=None, workspace=None,
               out: dict | None = None, reduce_grads: bool = False):
    """Transformer block forward (+ vector-Jacobian product when dy is given).
    Returns a dict with y and, with dy, dx and d<weight> for every weight.
    reduce_grads: one rank of a data-parallel step (chelis_cuda_block_step_dp):
    every weight gradient is summed across the ranks of the library's
    communicator while the reverse pass runs."""
    import ctypes
    _prepare(x, dy, *[weights[k] for k in BLOCK_WEIGHTS])
    batch, seq, d = x.shape
    dff = weights["w_1"].shape[1]
    o = out if out is not None else {}
    if "y" not in o:
        o["y"] = torch.empty_like(x)
    if dy is not None:
        if "dx" not in o:
            o["dx"] = torch.empty_like(x)
        for k in BLOCK_WEIGHTS:
            if "d" + k not in o:
                o["d" + k] = torch.empty_like(weights[k])
    p = L.BlockParams()
    p.batch, p.seq, p.d_model, p.heads, p.d_ff, p.eps = batch, seq, d, heads, dff, eps
    p.x = x.data_ptr()
    p.dy = dy.data_ptr() if dy is not None else None
    for k in BLOCK_WEIGHTS:
        setattr(p, k, weights[k].data_ptr())
    p.y = o["y"].data_ptr()
    if dy is not None:
        p.dx = o["dx"].data_ptr()
        for k in BLOCK_WEIGHTS:
            setattr(p, "d" + k if k.startswith("w") else "d" + k, o["d" + k].data_ptr())
    L.call("chelis_cuda_block_step_dp" if reduce_grads else "chelis_cuda_block_step",
           ctypes.byref(p), None if workspace is None else workspace.data_ptr())
    return o


def block_workspace(x, weights: dict, heads: int) -> torch.Tensor:
    import ctypes
    batch, seq, d = x.shape
    p = L.BlockParams()
    p.batch, p.seq, p.d_model, p.heads, p.d_ff = batch, seq, d, heads, weights["w_1"].shape[1]
    nbytes = int(L.load().chelis_cuda_block_workspace_bytes(ctypes.byref(p)))
    if nbytes < 0:
        raise ValueError("transformer block shape not admitted")
    return torch.empty(nbytes // 4 + 64, dtype=torch.float32, device=x.device)


def mlp_step(x, labels, w1, b1, w2, b2):
    _prepare(x, labels, w1, b1, w2, b2)
    batch, din = x.shape
    dh = w1.shape[1]
    dout = w2.shape[1]
    dev = x.device
    loss = torch.empty(1, dtype=torch.float32, device=dev)
    dw1 = torch.empty_like(w1)
    db1 = torch.empty_like(b1)
    dw2 = torch.empty_like(w2)
    db2 = torch.empty_like(b2)
    L.call("chelis_cuda_mlp_step", x.data_ptr(), labels.data_ptr(), w1.data_ptr(),
           b1.data_ptr(), w2.data_ptr(), b2.data_ptr(), batch, din, dh, dout, loss.data_ptr(),
           dw1.data_ptr(), db1.data_ptr(), dw2.data_ptr(), db2.data_ptr())
    return loss, dw1, db1, dw2, db2


def _fused_args(steps, inputs, shape):
    from . import fused as F
    if not steps:
        raise ValueError("a fused group has at least one step")
    dtypes = {t.dtype for t in inputs}
    if len(dtypes) > 1:
        raise ValueError("fused group inputs share one dtype")
    dtype = dtypes.pop() if dtypes else torch.float32
    if dtype not in (torch.float32, torch.float64):
        raise ValueError("fused groups compute in f32 or f64")
    for t in inputs:
        if not t.is_cuda:
            raise ValueError("chelis_b200 ops take CUDA tensors (device memory)")
    shape = tuple(torch.broadcast_shapes(*(t.shape for t in inputs))) if shape is None else tuple(shape)
    rank = len(shape)
    strides = []
    for t in inputs:
        strides.extend(t.expand(shape).stride() if rank else ())
    c_i64 = ctypes.c_int64
    arrays = dict(
        steps=F.encode(steps),
        ptrs=(ctypes.c_void_p * max(len(inputs), 1))(*[t.data_ptr() for t in inputs]),
        strides=(c_i64 * max(len(strides), 1))(*strides),
        shape=(c_i64 * max(rank, 1))(*shape),
    )
    dt = L.DTYPE_F32 if dtype == torch.float32 else L.DTYPE_F64
    return dt, dtype, shape, arrays


def fused_elementwise(steps, inputs, shape=None) -> torch.Tensor:
    """Evaluate a FusedElem chain (a list of chelis_b200.fused.FusedStep)
    over `inputs` broadcast to `shape` (default: their broadcast shape)."""
    dt, dtype, shape, a = _fused_args(steps, inputs, shape)
    device = inputs[0].device if inputs else torch.device("cuda", torch.cuda.current_device())
    out = torch.empty(shape, dtype=dtype, device=device)
    _prepare(out)
    L.call("chelis_cuda_fused_elementwise", dt, a["steps"], len(steps), a["ptrs"], a["strides"],
           len(inputs), a["shape"], len(shape), out.data_ptr())
    return out


def fused_reduce(steps, inputs, axis: int, kind: str = "sum", shape=None) -> torch.Tensor:
    """The chain reduced along `axis` ("sum" or "max", emit_fused_reduce):
    the result has the iteration shape without `axis`."""
    from . import fused as F
    dt, dtype, shape, a = _fused_args(steps, inputs, shape)
    if not shape:
        raise ValueError("fused_reduce needs rank >= 1")
    axis = axis % len(shape)
    device = inputs[0].device if inputs else torch.device("cuda", torch.cuda.current_device())
    out = torch.empty(shape[:axis] + shape[axis + 1:], dtype=dtype, device=device)
    _prepare(out)
    L.call("chelis_cuda_fused_reduce", dt, a["steps"], len(steps), a["ptrs"], a["strides"],
           len(inputs), a["shape"], len(shape), axis, F.REDUCE_KIND[kind], out.data_ptr())
    return out


def _dt(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return L.DTYPE_F32
    if t.dtype == torch.float64:
        return L.DTYPE_F64
    raise ValueError("f32 or f64 tensors")


def relu(x: torch.Tensor) -> torch.Tensor:
    _prepare(x)
    y = torch.empty_like(x)
    L.call("chelis_cuda_relu", _dt(x), x.data_ptr(), y.data_ptr(), x.numel())
    return y


def relu_adjoint(x: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
    _prepare(x, g)
    dx = torch.empty_like(g)
    L.call("chelis_cuda_relu_adjoint", _dt(x), x.data_ptr(), g.data_ptr(), dx.data_ptr(), x.numel())
    return dx


def gelu(x: torch.Tensor) -> torch.Tensor:
    _prepare(x)
    y = torch.empty_like(x)
    L.call("chelis_cuda_gelu_f32", x.data_ptr(), y.data_ptr(), x.numel())
    return y


def gelu_adjoint(x: torch.Tensor, g: torch.Tensor) -> torch.Tensor:
    _prepare(x, g)
    dx = torch.empty_like(g)
    L.call("chelis_cuda_gelu_adjoint_f32", x.data_ptr(), g.data_ptr(), dx.data_ptr(), x.numel())
    return dx


def layer_norm_bwd(x, gamma, eps: float, dy):
    _prepare(x, gamma, dy)
    rows, hidden = x.shape
    dx = torch.empty_like(x)
    dg = torch.empty(hidden, dtype=torch.float32, device=x.device)
    db = torch.empty(hidden, dtype=torch.float32, device=x.device)
    L.call("chelis_cuda_layer_norm_bwd_f32", x.data_ptr(), gamma.data_ptr(), eps, dy.data_ptr(),
           rows, hidden, dx.data_ptr(), dg.data_ptr(), db.data_ptr())
    return dx, dg, db


def cross_entropy(logits, labels, want_grad: bool = True):
    """Mean cross-entropy of row softmax at int64 labels; returns (loss, dlogits)."""
    _prepare(logits, labels)
    rows, classes = logits.shape
    loss = torch.empty((), dtype=torch.float32, device=logits.device)
    dz = torch.empty_like(logits) if want_grad else None
    L.call("chelis_cuda_cross_entropy_f32", logits.data_ptr(), labels.data_ptr(), rows, classes,
           loss.data_ptr(), _ptr(dz))
    return loss, dz
