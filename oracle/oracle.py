"""ctypes front end of the parity oracle (liborc.so).

TEST INFRASTRUCTURE ONLY: the CPU restatement of the Chelis C backend that the
CUDA backend is checked against.  Only tests/, __graft_entry__.smoke() and the
cpu_baseline leg of bench.py import this module; the product package
(chelis_b200) never does.

Every wrapper takes and returns numpy arrays; see chelis_oracle.h for the
reference file:line each kernel restates.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liborc.so")
_lib = None

_f32p = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")
_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64


def build() -> None:
    """Compile liborc.so (and the reference CORE-MATH shim when the reference
    tree is present) with oracle/Makefile."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = ctypes.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


def _declare(L: ctypes.CDLL) -> None:
    sig = {
        "orc_splitmix64": (_u64, [_u64]),
        "orc_word": (_u64, [_u64, _u64]),
        "orc_derive": (_u64, [_u64, _u64]),
        "orc_unit": (ctypes.c_double, [_u64, _u64]),
        "orc_tree_sum_f32": (ctypes.c_float, [_f32p, _i64, _i64]),
        "orc_tree_sum_f64": (ctypes.c_double, [_f64p, _i64, _i64]),
        "orc_row_sum_f32": (None, [_f32p, _i64, _i64, _f32p]),
        "orc_col_sum_f32": (None, [_f32p, _i64, _i64, _f32p]),
        "orc_row_max_f32": (None, [_f32p, _i64, _i64, _f32p]),
        "orc_count_bool": (_i64, [_u8p, _i64]),
        "orc_sgemm": (None, [_f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64]),
        "orc_dgemm": (None, [_f64p, _f64p, _f64p, _i64, _i64, _i64, _i64, _i64]),
        "orc_sgemm_strided": (None, [_f32p, _i64, _i64, _f32p, _i64, _i64, _f32p, _i64, _i64, _i64]),
        "orc_dgemm_strided": (None, [_f64p, _i64, _i64, _f64p, _i64, _i64, _f64p, _i64, _i64, _i64]),
        "orc_dropout_f32": (None, [_f32p, _f32p, _i64, _u64, ctypes.c_float, _i64]),
        "orc_dropout_mask": (None, [_u8p, _i64, _u64, ctypes.c_float, _i64]),
        "orc_layer_norm_f32": (None, [_f32p, _f32p, _f32p, ctypes.c_float, _f32p, _i64, _i64]),
        "orc_softmax_rows_f32": (None, [_f32p, _f32p, _i64, _i64]),
        "orc_softmax_rows_bwd_f32": (None, [_f32p, _f32p, _f32p, _i64, _i64]),
        "orc_chain_fwd": (None, [_f32p, _f32p, _f32p, ctypes.c_float, _u64, ctypes.c_float,
                                 _i64, _i64, _i64, _f32p]),
        "orc_chain_bwd": (None, [_f32p, _f32p, _f32p, ctypes.c_float, _u64, ctypes.c_float,
                                 _i64, _i64, _i64, _f32p, _f32p, _f32p]),
        "orc_cumsum_f64": (None, [_f64p, _f64p, _i64, _i64, ctypes.c_int]),
        "orc_cumsum_f32": (None, [_f32p, _f32p, _i64, _i64, ctypes.c_int]),
        "orc_portfolio": (None, [_f64p, _f64p, _i64, _i64, _i64, _f64p, _f64p, _f64p]),
        "orc_mlp_step": (None, [_f32p, _i64p, _f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64,
                                _f32p, _f32p, _f32p, _f32p, _f32p]),
        "orc_add_f32": (ctypes.c_float, [ctypes.c_float, ctypes.c_float]),
        "orc_mul_f32": (ctypes.c_float, [ctypes.c_float, ctypes.c_float]),
        "orc_div_f32": (ctypes.c_float, [ctypes.c_float, ctypes.c_float]),
        "orc_sqrt_f32": (ctypes.c_float, [ctypes.c_float]),
        "orc_expf": (ctypes.c_float, [ctypes.c_float]),
        "orc_logf": (ctypes.c_float, [ctypes.c_float]),
        "orc_crmath_check_f32": (ctypes.c_int64, [ctypes.c_int32, ctypes.c_uint32, ctypes.c_int64,
                                                  ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64)]),
        "orc_erfcf": (ctypes.c_float, [ctypes.c_float]),
        "orc_exp": (ctypes.c_double, [ctypes.c_double]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


def key_from_seed(seed: int) -> int:
    """[05-OP-69] key_from_seed: the i64 seed's two's-complement bits."""
    return seed & 0xFFFFFFFFFFFFFFFF


def splitmix64(v: int) -> int:
    return lib().orc_splitmix64(v)


def word(key: int, index: int) -> int:
    return lib().orc_word(key, index)


def derive(key: int, j: int) -> int:
    return lib().orc_derive(key, j)


def unit(key: int, index: int) -> float:
    return lib().orc_unit(key, index)


def tree_sum(x: np.ndarray) -> float:
    x = np.ascontiguousarray(x)
    if x.dtype == np.float32:
        return np.float32(lib().orc_tree_sum_f32(x, x.size, 1))
    return np.float64(lib().orc_tree_sum_f64(_c(x, np.float64), x.size, 1))


def row_sum(x: np.ndarray) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape[0], np.float32)
    lib().orc_row_sum_f32(x, x.shape[0], x.shape[1], out)
    return out


def col_sum(x: np.ndarray) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape[1], np.float32)
    lib().orc_col_sum_f32(x, x.shape[0], x.shape[1], out)
    return out


def row_max(x: np.ndarray) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.shape[0], np.float32)
    lib().orc_row_max_f32(x, x.shape[0], x.shape[1], out)
    return out


def count(x: np.ndarray) -> int:
    return int(lib().orc_count_bool(_c(x, np.uint8), x.size))


def gemm(a: np.ndarray, b: np.ndarray, rows: tuple[int, int] | None = None) -> np.ndarray:
    """Row-major C = A.B with the canonical tree over k.  `rows` limits the
    computed rows to [r0, r1) (a bounded sample); other rows stay zero."""
    m, k = a.shape
    k2, n = b.shape
    assert k == k2
    r0, r1 = rows if rows is not None else (0, m)
    if a.dtype == np.float64:
        c = np.zeros((m, n), np.float64)
        lib().orc_dgemm(_c(a, np.float64), _c(b, np.float64), c, m, n, k, r0, r1)
    else:
        c = np.zeros((m, n), np.float32)
        lib().orc_sgemm(_c(a, np.float32), _c(b, np.float32), c, m, n, k, r0, r1)
    return c


def gemm_t(a: np.ndarray, b: np.ndarray, trans_a: bool, trans_b: bool) -> np.ndarray:
    """op(A).op(B) with the tree over the contracted axis in increasing order."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    if trans_a:
        k, m = a.shape
        sa0, sa1 = 1, m
    else:
        m, k = a.shape
        sa0, sa1 = k, 1
    if trans_b:
        n, k2 = b.shape
        sb0, sb1 = 1, k2
    else:
        k2, n = b.shape
        sb0, sb1 = n, 1
    assert k == k2
    if a.dtype == np.float64:
        c = np.zeros((m, n), np.float64)
        lib().orc_dgemm_strided(a, sa0, sa1, b, sb0, sb1, c, m, n, k)
    else:
        c = np.zeros((m, n), np.float32)
        lib().orc_sgemm_strided(a, sa0, sa1, b, sb0, sb1, c, m, n, k)
    return c


def dropout(x: np.ndarray, key: int, rate: float, index_base: int = 0) -> np.ndarray:
    x = _c(x, np.float32)
    y = np.empty_like(x)
    lib().orc_dropout_f32(x.reshape(-1), y.reshape(-1), x.size, key, rate, index_base)
    return y


def dropout_mask(n: int, key: int, rate: float, index_base: int = 0) -> np.ndarray:
    keep = np.empty(n, np.uint8)
    lib().orc_dropout_mask(keep, n, key, rate, index_base)
    return keep


def layer_norm(x, gamma, beta, eps):
    x = _c(x, np.float32)
    y = np.empty_like(x)
    lib().orc_layer_norm_f32(x, _c(gamma, np.float32), _c(beta, np.float32), eps, y,
                             x.shape[0], x.shape[1])
    return y


def softmax_rows(x):
    x = _c(x, np.float32)
    y = np.empty_like(x)
    lib().orc_softmax_rows_f32(x, y, x.shape[0], x.shape[1])
    return y


def softmax_rows_bwd(y, g):
    y = _c(y, np.float32)
    dx = np.empty_like(y)
    lib().orc_softmax_rows_bwd_f32(y, _c(g, np.float32), dx, y.shape[0], y.shape[1])
    return dx


def chain_fwd(x, gamma, beta, eps, key, rate, index_base=0):
    x = _c(x, np.float32)
    out = np.empty(x.shape[0], np.float32)
    lib().orc_chain_fwd(x, _c(gamma, np.float32), _c(beta, np.float32), eps, key, rate,
                        x.shape[0], x.shape[1], index_base, out)
    return out


def chain_bwd(x, gamma, beta, eps, key, rate, index_base=0):
    x = _c(x, np.float32)
    dx = np.empty_like(x)
    dg = np.empty(x.shape[1], np.float32)
    db = np.empty(x.shape[1], np.float32)
    lib().orc_chain_bwd(x, _c(gamma, np.float32), _c(beta, np.float32), eps, key, rate,
                        x.shape[0], x.shape[1], index_base, dx, dg, db)
    return dx, dg, db


def cumsum(x, reverse=False):
    if x.dtype == np.float64:
        x = _c(x, np.float64)
        y = np.empty_like(x)
        lib().orc_cumsum_f64(x, y, x.shape[0], x.shape[1], int(reverse))
    else:
        x = _c(x, np.float32)
        y = np.empty_like(x)
        lib().orc_cumsum_f32(x, y, x.shape[0], x.shape[1], int(reverse))
    return y


def portfolio(r, w):
    r = _c(r, np.float64)
    w = _c(w, np.float64)
    count_, t, a = r.shape
    sigma = np.empty((count_, a, a), np.float64)
    risk = np.empty(count_, np.float64)
    cum = np.empty((count_, t), np.float64)
    lib().orc_portfolio(r, w, count_, t, a, sigma, risk, cum)
    return sigma, risk, cum


def mlp_step(x, labels, w1, b1, w2, b2):
    x = _c(x, np.float32)
    batch, din = x.shape
    dh = w1.shape[1]
    dout = w2.shape[1]
    loss = np.zeros(1, np.float32)
    dw1 = np.empty((din, dh), np.float32)
    db1 = np.empty(dh, np.float32)
    dw2 = np.empty((dh, dout), np.float32)
    db2 = np.empty(dout, np.float32)
    lib().orc_mlp_step(x, _c(labels, np.int64), _c(w1, np.float32), _c(b1, np.float32),
                       _c(w2, np.float32), _c(b2, np.float32), batch, din, dh, dout,
                       loss, dw1, db1, dw2, db2)
    return loss[0], dw1, db1, dw2, db2


def expf(x: float) -> float:
    return lib().orc_expf(x)


def logf(x: float) -> float:
    return lib().orc_logf(x)


def crmath_check_f32(op: int, start: int, got) -> tuple[int, int]:
    """Mismatches of `got` (float32 results at bit patterns start, start+1,
    ...) against CORE-MATH exp (op 0) / log (op 1), and the first one's offset."""
    got = np.ascontiguousarray(got, dtype=np.float32)
    first = ctypes.c_int64(-1)
    bad = lib().orc_crmath_check_f32(op, start, got.size, got.ctypes.data, ctypes.byref(first))
    return int(bad), int(first.value)


def _fused_call(name, triplets, inputs, shape, extra):
    inputs = [np.asarray(x) for x in inputs]
    dtypes = {x.dtype for x in inputs} or {np.dtype(np.float32)}
    assert len(dtypes) == 1, "fused inputs share one dtype"
    dt = dtypes.pop()
    assert dt in (np.float32, np.float64)
    shape = tuple(np.broadcast_shapes(*(x.shape for x in inputs))) if shape is None else tuple(shape)
    rank = len(shape)
    keep = [x if x.flags.c_contiguous else x.copy(order="C") for x in inputs]  # rank 0 stays rank 0
    strides = []
    for k in keep:  # element strides of each (contiguous) input over the shape
        strides.extend(s // k.itemsize for s in np.broadcast_to(k, shape).strides)
    steps = np.ascontiguousarray(np.asarray(triplets, dtype=np.int32).reshape(-1))
    ptrs = (ctypes.c_void_p * max(len(keep), 1))(*[k.ctypes.data for k in keep])
    st = np.ascontiguousarray(np.asarray(strides if strides else [0], dtype=np.int64))
    sh = np.ascontiguousarray(np.asarray(shape if shape else [1], dtype=np.int64))
    fn = getattr(lib(), name + ("_f32" if dt == np.float32 else "_f64"))
    fn.restype = None
    out_shape, args = extra(shape)
    out = np.empty(out_shape, dtype=dt)
    fn(steps.ctypes.data_as(ctypes.c_void_p), ctypes.c_int32(len(triplets)), ptrs,
       st.ctypes.data_as(ctypes.c_void_p), ctypes.c_int32(len(keep)),
       sh.ctypes.data_as(ctypes.c_void_p), ctypes.c_int32(rank), *args,
       out.ctypes.data_as(ctypes.c_void_p))
    return out


def fused_elementwise(triplets, inputs, shape=None) -> np.ndarray:
    """FusedElem chain of (op, a, b) triplets (op the FusedStepOp index; an
    operand >= 0 an input, < 0 the step -1 - operand) over the inputs
    broadcast to `shape`; C-lane step semantics with CORE-MATH."""
    return _fused_call("orc_fused_elementwise", triplets, inputs, shape, lambda s: (s, ()))


def fused_reduce(triplets, inputs, axis: int, kind: str = "sum", shape=None) -> np.ndarray:
    """The chain reduced along `axis`: "sum" (carry tree) or "max"
    (chelis_fmax_propnan fold from -inf)."""
    k = {"sum": 0, "max": 1}[kind]

    def extra(s):
        ax = axis % len(s)
        return s[:ax] + s[ax + 1:], (ctypes.c_int32(ax), ctypes.c_int32(k))
    return _fused_call("orc_fused_reduce", triplets, inputs, shape, extra)


def relu(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x)
    y = np.empty_like(x)
    fn = lib().orc_relu_f32 if x.dtype == np.float32 else lib().orc_relu_f64
    fn.restype = None
    fn(x.ctypes.data_as(ctypes.c_void_p), y.ctypes.data_as(ctypes.c_void_p), _i64(x.size))
    return y


def relu_adjoint(x: np.ndarray, g: np.ndarray) -> np.ndarray:
    x, g = np.ascontiguousarray(x), np.ascontiguousarray(g)
    dx = np.empty_like(g)
    fn = lib().orc_relu_adjoint_f32 if x.dtype == np.float32 else lib().orc_relu_adjoint_f64
    fn.restype = None
    fn(x.ctypes.data_as(ctypes.c_void_p), g.ctypes.data_as(ctypes.c_void_p),
       dx.ctypes.data_as(ctypes.c_void_p), _i64(x.size))
    return dx


def gelu(x: np.ndarray) -> np.ndarray:
    x = _c(x, np.float32)
    y = np.empty_like(x)
    fn = lib().orc_gelu_f32
    fn.restype = None
    fn(x.ctypes.data_as(ctypes.c_void_p), y.ctypes.data_as(ctypes.c_void_p), _i64(x.size))
    return y


def layer_norm_bwd(x, gamma, eps, dy):
    x, gamma, dy = _c(x, np.float32), _c(gamma, np.float32), _c(dy, np.float32)
    rows, hidden = x.shape
    dx = np.empty_like(x)
    dg = np.empty(hidden, np.float32)
    db = np.empty(hidden, np.float32)
    fn = lib().orc_layer_norm_bwd_f32
    fn.restype = None
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    fn(p(x), p(gamma), ctypes.c_float(eps), p(dy), _i64(rows), _i64(hidden), p(dx), p(dg), p(db))
    return dx, dg, db


def cross_entropy(z, labels):
    """(loss, dz) of the mean cross-entropy at int64 labels."""
    z = _c(z, np.float32)
    labels = np.ascontiguousarray(labels, dtype=np.int64)
    rows, classes = z.shape
    loss = np.zeros(1, np.float32)
    dz = np.empty_like(z)
    fn = lib().orc_cross_entropy_f32
    fn.restype = ctypes.c_int
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    if fn(p(z), p(labels), _i64(rows), _i64(classes), p(loss), p(dz)) != 0:
        raise ValueError("label out of range")
    return loss[0], dz


BLOCK_WEIGHTS = ("w_qkv", "w_o", "w_1", "w_2", "ln1_gamma", "ln1_beta", "ln2_gamma", "ln2_beta")


def gelu_adjoint(x: np.ndarray, g: np.ndarray) -> np.ndarray:
    x, g = _c(x, np.float32), _c(g, np.float32)
    dx = np.empty_like(x)
    fn = lib().orc_gelu_adjoint_f32
    fn.restype = None
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    fn(p(x), p(g), p(dx), _i64(x.size))
    return dx


def block_step(x, w: dict, heads: int, eps: float, dy=None):
    """Transformer block forward (+ VJP when dy is given), orc_block_step.
    Returns (y, grads) with grads keyed "dx" and "d<weight>" (None without dy)."""
    x = _c(x, np.float32)
    batch, seq, d = x.shape
    dff = w["w_1"].shape[1]
    ws = [_c(w[k], np.float32) for k in BLOCK_WEIGHTS]
    y = np.empty_like(x)
    grads = None
    p = lambda a: None if a is None else a.ctypes.data_as(ctypes.c_void_p)
    if dy is not None:
        dy = _c(dy, np.float32)
        grads = {"dx": np.empty_like(x)}
        grads.update({"d" + k: np.empty_like(a) for k, a in zip(BLOCK_WEIGHTS, ws)})
    outs = [None] * 9 if grads is None else [grads["dx"]] + [grads["d" + k] for k in BLOCK_WEIGHTS]
    fn = lib().orc_block_step
    fn.restype = ctypes.c_int
    rc = fn(p(x), p(dy), _i64(batch), _i64(seq), _i64(d), _i64(heads), _i64(dff),
            ctypes.c_float(eps), *[p(a) for a in ws], p(y), *[p(a) for a in outs])
    if rc:
        raise ValueError("orc_block_step: shape not admitted")
    return y, grads


def attention_causal(q, k, v, scale: float, dout=None):
    """Causal attention per head on [bh, S, Dh]: o, and (dq, dk, dv) with dout."""
    q, k, v = (_c(t, np.float32) for t in (q, k, v))
    bh, seq, dh = q.shape
    o = np.empty_like(q)
    g = [np.empty_like(q) for _ in range(3)] if dout is not None else [None] * 3
    p = lambda a: None if a is None else a.ctypes.data_as(ctypes.c_void_p)
    fn = lib().orc_attention_causal
    fn.restype = None
    fn(p(q), p(k), p(v), p(None if dout is None else _c(dout, np.float32)), _i64(bh), _i64(seq),
       _i64(dh), ctypes.c_float(scale), p(o), *[p(a) for a in g])
    return (o, tuple(g)) if dout is not None else o
