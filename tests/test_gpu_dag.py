"""The DAG executor on the GPU: the config-1 MLP program, built the way the
reference lowers it (tests/_dag_programs.py), run from its JSON and checked
against the oracle's MLP step (the C lane's algorithm) within f32 rel 1e-5;
single-op programs against numpy; the host-array entry; a caller arena."""
import ctypes

import numpy as np
import pytest
import torch

from chelis_b200 import lib as L
from chelis_b200 import workloads as W
import _dag_programs as D

pytestmark = pytest.mark.gpu


def program(g):
    h = ctypes.c_void_p()
    raw = g.json().encode()
    L.call("chelis_dag_from_json", raw, len(raw), ctypes.byref(h))
    return h


def run(h, tensors):
    lib = L.load()
    owners = []
    for t in tensors:
        t = t.contiguous()
        dt = {torch.float32: L.DTYPE_F32, torch.float64: L.DTYPE_F64, torch.int64: L.DTYPE_I64,
              torch.int32: L.DTYPE_I32, torch.bool: L.DTYPE_BOOL, torch.int8: 7, torch.int16: 8,
              torch.float16: L.DTYPE_F16, torch.bfloat16: L.DTYPE_BF16}[t.dtype]
        shape = (ctypes.c_int64 * max(t.dim(), 1))(*t.shape)
        o = lib.chelis_device_tensor_borrow_shape(dt, t.dim(), shape, t.data_ptr(),
                                                   t.numel() * t.element_size())
        assert o, L.last_error()
        owners.append(o)
    n_out = lib.chelis_dag_output_count(h)
    ins = (ctypes.c_void_p * len(owners))(*owners)
    outs = (ctypes.c_void_p * n_out)()
    L.call("chelis_dag_run_device", h, ins, len(owners), outs, n_out)
    L.call("chelis_cuda_device_status")
    res = []
    for i in range(n_out):
        v = lib.chelis_device_tensor_view(outs[i]).contents
        shape = [v.shape[d] for d in range(v.rank)]
        np_dt = {L.DTYPE_F32: np.float32, L.DTYPE_F64: np.float64, L.DTYPE_I64: np.int64,
                 L.DTYPE_I32: np.int32, L.DTYPE_BOOL: np.uint8, 9: np.uint64,  # 9: key
                 7: np.int8, 8: np.int16, L.DTYPE_F16: np.uint16, L.DTYPE_BF16: np.uint16}[v.dtype]
        host = np.empty(shape, dtype=np_dt)
        L.call("chelis_device_tensor_copy_to_host_bytes", host.ctypes.data, host.nbytes, outs[i])
        res.append(host)
        lib.chelis_device_tensor_release(outs[i])
    L.call("chelis_cuda_synchronize")
    for o in owners:
        lib.chelis_device_tensor_release(o)
    return res


def rel(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def test_mlp_program_matches_oracle(cuda, orc):
    x, labels, w1, b1, w2, b2 = W.mlp_inputs(seed=0)
    h = program(D.mlp_step_dag())
    try:
        T = [torch.from_numpy(v).cuda() for v in (x, w1, b1, w2, b2, labels)]
        loss, dw1, db1, dw2, db2 = run(h, T)
        ref = orc.mlp_step(x, labels, w1, b1, w2, b2)
        for got, want in zip((loss, dw1, db1, dw2, db2), ref):
            assert rel(got, want) <= 1e-5
        # twice in a row: the same bits (slots reused, nothing left over)
        again = run(h, T)
        for a, b in zip((loss, dw1, db1, dw2, db2), again):
            assert np.array_equal(a, b)
    finally:
        L.load().chelis_dag_release(h)


def test_mlp_program_in_a_caller_arena(cuda, orc):
    lib = L.load()
    x, labels, w1, b1, w2, b2 = W.mlp_inputs(seed=0)
    h = program(D.mlp_step_dag())
    try:
        T = [torch.from_numpy(v).cuda() for v in (x, w1, b1, w2, b2, labels)]
        want = run(h, T)
        arena = torch.empty(lib.chelis_dag_arena_bytes(h), dtype=torch.uint8, device="cuda")
        owners = []
        for t in T:
            dt = {torch.float32: L.DTYPE_F32, torch.int64: L.DTYPE_I64}[t.dtype]
            shape = (ctypes.c_int64 * t.dim())(*t.shape)
            owners.append(lib.chelis_device_tensor_borrow_shape(dt, t.dim(), shape, t.data_ptr(),
                                                                 t.numel() * t.element_size()))
        ins = (ctypes.c_void_p * 6)(*owners)
        outs = (ctypes.c_void_p * 5)()
        assert lib.chelis_dag_run_device_arena(h, ins, 6, outs, 5, arena.data_ptr(), 16) == 1
        L.call("chelis_dag_run_device_arena", h, ins, 6, outs, 5, arena.data_ptr(), arena.numel())
        for i in range(5):
            v = lib.chelis_device_tensor_view(outs[i]).contents
            host = np.empty([v.shape[d] for d in range(v.rank)], dtype=np.float32)
            L.call("chelis_device_tensor_copy_to_host_bytes", host.ctypes.data, host.nbytes, outs[i])
            assert np.array_equal(host, want[i])
            lib.chelis_device_tensor_release(outs[i])
        for o in owners:
            lib.chelis_device_tensor_release(o)
    finally:
        lib.chelis_dag_release(h)


def single(op_builder, inputs, want):
    g = D.Dag()
    ids = [g.load(f"x{i}", list(a.shape), {np.float32: "f32", np.float64: "f64", np.int64: "i64"}[a.dtype.type])
           for i, a in enumerate(inputs)]
    g.roots = [op_builder(g, *ids)]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(a).cuda() for a in inputs])
    finally:
        L.load().chelis_dag_release(h)
    return got


def test_movement_and_index_ops(cuda):
    rng = np.random.default_rng(5)
    x = rng.standard_normal((6, 9)).astype(np.float32)
    idx = rng.integers(0, 9, size=(4,)).astype(np.int64)
    # permute + stride + shrink views feeding an elementwise op
    got = single(lambda g, a: g.unary("Neg", g.stride(g.shrink(g.permute(a, [1, 0]), [(1, 8), (0, 6)]), [2, 3])),
                 [x], None)
    assert np.array_equal(got, -x.T[1:8, 0:6][::2, ::3])
    # gather along axis 1: out[r, j] = x[r, idx[j]]
    got = single(lambda g, a, i: g.add({"Gather": {"axis": 1, "batch_rank": 0}}, [a, i], [6, 4]), [x, idx], None)
    assert np.array_equal(got, x[:, idx])
    # scatter-add with repeated indices (increasing update order)
    upd = rng.standard_normal((6, 4)).astype(np.float32)
    got = single(lambda g, a, i, u: g.add({"ScatterAdd": {"axis": 1, "batch_rank": 0}}, [a, i, u], [6, 9]),
                 [x, idx, upd], None)
    want = x.copy()
    for r in range(6):
        for j in range(4):
            want[r, idx[j]] = np.float32(want[r, idx[j]] + upd[r, j])
    assert np.array_equal(got, want)
    # pad with a fill value
    got = single(lambda g, a: g.pad(a, [(1, 2), (0, 3)], fill=7.5), [x], None)
    want = np.full((9, 12), 7.5, np.float32)
    want[1:7, 0:9] = x
    assert np.array_equal(got, want)
    # a batched matmul with a transposed operand taken in place
    a = rng.standard_normal((3, 40, 24)).astype(np.float64)
    b = rng.standard_normal((3, 40, 16)).astype(np.float64)
    def bmm(g, p, q):
        pt = g.permute(p, [0, 2, 1])
        return g.add({"BlasMatmul": {"batch_dims": [{"Concrete": 3}], "m": {"Concrete": 24},
                                     "n": {"Concrete": 16}, "k": {"Concrete": 40}, "accumulator": "F64"}},
                     [pt, q], [3, 24, 16], "f64")
    got = single(bmm, [a, b], None)
    assert rel(got, np.einsum("bki,bkj->bij", a, b)) <= 1e-12


def test_out_of_range_gather_index_traps(cuda):
    x = np.ones((2, 3), np.float32)
    idx = np.array([0, 3], np.int64)
    g = D.Dag()
    a = g.load("x", [2, 3])
    i = g.load("i", [2], "i64")
    g.roots = [g.add({"Gather": {"axis": 1, "batch_rank": 0}}, [a, i], [2, 2])]
    h = program(g)
    try:
        with pytest.raises(L.ChelisCudaError, match="gather index 3 out of bounds at axis 1 of extent 3\nnumeric trap: domain in gather at i64"):
            run(h, [torch.from_numpy(x).cuda(), torch.from_numpy(idx).cuda()])
    finally:
        L.load().chelis_dag_release(h)


# crates/chelis-backend-c/tests/exec_compile.rs:761-900: the sparse mappings
# move stored bits.  Base cell i holds seed + i, update cell i holds
# seed + i + 32 (bool: ((i / 2 + i) % 2) ^ update); `map` names, per output
# cell, the update cell it holds, or -(base cell) - 1.
SPARSE_SEEDS = [("f32", 0x3F800000), ("f64", 0x3FF0000000000000), ("f16", 0x3C00), ("bf16", 0x3F80),
                ("i8", 10), ("i16", 100), ("i32", 100), ("i64", 9_007_199_254_740_993), ("bool", 0)]
SPARSE_CASES = [
    ({"Gather": {"axis": 1, "batch_rank": 0}}, [2, 3, 2], [2, 2, 2, 2], [2, 0, 1, 2],
     [4, 5, 0, 1, 2, 3, 4, 5, 10, 11, 6, 7, 8, 9, 10, 11]),
    ({"Scatter": {"axis": 1, "batch_rank": 0}}, [2, 3, 2], [2, 3, 2], [2, 0, 2, 0],
     [6, 7, -3, -4, 4, 5, 14, 15, -9, -10, 12, 13]),
    ({"ScatterElements": {"axis": 1}}, [2, 3], [2, 3], [2, 0, 1, 1], [1, -2, 0, -4, 3, -6]),
]
_STORAGE = {"f32": (np.uint32, torch.float32), "f64": (np.uint64, torch.float64), "f16": (np.uint16, torch.float16),
            "bf16": (np.uint16, torch.bfloat16), "i8": (np.uint8, torch.int8), "i16": (np.uint16, torch.int16),
            "i32": (np.uint32, torch.int32), "i64": (np.uint64, torch.int64), "bool": (np.uint8, torch.bool)}


def _bits_tensor(bits, shape, prec):
    np_t, torch_t = _STORAGE[prec]
    raw = np.asarray(bits, dtype=np.uint64).astype(np_t).reshape(shape)
    signed = {np.uint8: np.uint8, np.uint16: np.int16, np.uint32: np.int32, np.uint64: np.int64}[np_t]
    return torch.from_numpy(raw.view(signed).copy()).view(torch_t).cuda()


@pytest.mark.parametrize("index_prec", ["i32", "i64"])
@pytest.mark.parametrize("prec,seed", SPARSE_SEEDS)
def test_sparse_mappings_preserve_stored_bits(cuda, prec, seed, index_prec):
    def bits(i, update):
        if prec == "bool":
            return ((i // 2 + i) % 2) ^ update
        return seed + i + (32 if update else 0)
    for op, base_shape, out_shape, selected, mapping in SPARSE_CASES:
        gather = "Gather" in op
        elements = "ScatterElements" in op
        update_shape = [2, 2] if elements else [2, 2, 2, 2]
        g = D.Dag()
        base = g.load("base", base_shape, prec)
        idx = g.load("indices", [2, 2], index_prec)
        ins = [base, idx] + ([] if gather else [g.load("updates", update_shape, prec)])
        g.roots = [g.add(op, ins, out_shape, prec)]
        h = program(g)
        try:
            nb, nu = int(np.prod(base_shape)), int(np.prod(update_shape))
            args = [_bits_tensor([bits(i, 0) for i in range(nb)], base_shape, prec),
                    torch.tensor(selected, dtype=torch.int32 if index_prec == "i32" else torch.int64).view(2, 2).cuda()]
            if not gather:
                args.append(_bits_tensor([bits(i, 1) for i in range(nu)], update_shape, prec))
            (got,) = run(h, args)
        finally:
            L.load().chelis_dag_release(h)
        np_t = _STORAGE[prec][0]
        want = np.array([bits(-m - 1, 0) if m < 0 else bits(m, (not gather)) for m in mapping],
                        dtype=np.uint64).astype(np_t)
        assert list(got.shape) == out_shape, op
        assert np.array_equal(got.reshape(-1).view(np_t), want), (op, prec, index_prec)


def _scatter_replace(target, idx, upd, axis, batch_rank):
    """eval.rs scatter_replace: updates visited in row-major order, last write wins."""
    out = target.copy()
    qrank = idx.ndim - batch_rank
    for c in np.ndindex(*upd.shape):
        p, q, t = c[:axis], c[axis:axis + qrank], c[axis + qrank:]
        k = int(idx[p[:batch_rank] + q])
        out[p + (k,) + t] = upd[c]
    return out


def _scatter_elements(data, idx, upd, axis):
    """eval.rs:2276 scatter_elements, the same order rule."""
    out = data.copy()
    for c in np.ndindex(*upd.shape):
        d = list(c)
        d[axis] = int(idx[c])
        out[tuple(d)] = upd[c]
    return out


@pytest.mark.parametrize("axis,batch_rank", [(0, 0), (1, 0), (1, 1), (2, 1)])
def test_scatter_last_write_wins(cuda, axis, batch_rank):
    rng = np.random.default_rng(60 + axis + batch_rank)
    shape = [3, 5, 4]
    lead = shape[:batch_rank]
    qshape = [6, 2]                                   # many duplicates into an axis of 3..5
    idx = rng.integers(0, shape[axis], size=lead + qshape)
    upd_shape = shape[:axis] + qshape + shape[axis + 1:]
    target = rng.standard_normal(shape).astype(np.float64)
    upd = rng.standard_normal(upd_shape).astype(np.float64)
    g = D.Dag()
    a = g.load("t", shape, "f64")
    i = g.load("i", lead + qshape, "i64")
    u = g.load("u", upd_shape, "f64")
    g.roots = [g.add({"Scatter": {"axis": axis, "batch_rank": batch_rank}}, [a, i, u], shape, "f64")]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(x).cuda() for x in (target, idx, upd)])
    finally:
        L.load().chelis_dag_release(h)
    assert np.array_equal(got, _scatter_replace(target, idx, upd, axis, batch_rank))


@pytest.mark.parametrize("axis", [0, 1, 2])
@pytest.mark.parametrize("prec", ["f32", "i64", "i16"])
def test_scatter_elements_last_write_wins(cuda, axis, prec):
    rng = np.random.default_rng(70 + axis)
    shape = [4, 5, 6]
    ishape = [3, 4, 5]
    ishape[axis] = 9                                  # longer than the axis: duplicates
    dt = {"f32": np.float32, "i64": np.int64, "i16": np.int16}[prec]
    data = (rng.standard_normal(shape) * 100).astype(dt)
    upd = (rng.standard_normal(ishape) * 100).astype(dt)
    idx = rng.integers(0, shape[axis], size=ishape).astype(np.int32)
    g = D.Dag()
    a = g.load("d", shape, prec)
    i = g.load("i", ishape, "i32")
    u = g.load("u", ishape, prec)
    g.roots = [g.add({"ScatterElements": {"axis": axis}}, [a, i, u], shape, prec)]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(x).cuda() for x in (data, idx, upd)])
    finally:
        L.load().chelis_dag_release(h)
    assert np.array_equal(got, _scatter_elements(data, idx, upd, axis))


@pytest.mark.parametrize("op,message", [
    ({"Scatter": {"axis": 1, "batch_rank": 0}}, "scatter index 3 out of bounds at axis 1 of extent 3"),
    ({"ScatterElements": {"axis": 1}}, "scatter_elements index -1 out of bounds at axis 1 of extent 3"),
    ({"ScatterAdd": {"axis": 1, "batch_rank": 0}}, "scatter_add index 3 out of bounds at axis 1 of extent 3"),
])
def test_out_of_range_scatter_index_traps(cuda, op, message):
    elements = "ScatterElements" in op
    x = np.zeros((2, 3), np.float32)
    idx = np.array([[0, -1], [1, 2]] if elements else [0, 3], np.int64)
    ushape = [2, 2]
    g = D.Dag()
    a = g.load("x", [2, 3])
    i = g.load("i", list(idx.shape), "i64")
    u = g.load("u", ushape)
    g.roots = [g.add(op, [a, i, u], [2, 3])]
    h = program(g)
    try:
        with pytest.raises(L.ChelisCudaError, match=message):
            run(h, [torch.from_numpy(x).cuda(), torch.from_numpy(idx).cuda(),
                    torch.ones(ushape, device="cuda")])
        L.call("chelis_cuda_device_status")  # cleared by the report
    finally:
        L.load().chelis_dag_release(h)


def _pair_tree(leaves):
    """grad.rs / eval.rs:5470 OrderedAdjointSum: adjacent pairs level by level,
    an odd last element carried; one leaf unchanged; none gives +0."""
    xs = list(leaves)
    if not xs:
        return None
    if len(xs) == 1:
        return xs[0]
    while len(xs) > 1:
        xs = [xs[i] + xs[i + 1] if i + 1 < len(xs) else xs[i] for i in range(0, len(xs), 2)]
    return xs[0]


@pytest.mark.parametrize("prec,groups", [
    ("f32", [(2, 5), (1, None), (3, 7)]),          # (width, rows); rows None: a scalar
    ("f32", [(2, 3000), (1, None), (3, 3000)]),    # 15001 leaves: runs of 16 per thread
    ("f64", [(1, 1), (4, 257)]),
    ("f32", [(1, None)]),                          # one leaf: the adjoint unchanged
    ("f32", [(2, 0)]),                             # empty columns: +0
])
def test_ordered_adjoint_sum(cuda, prec, groups):
    dt = np.float32 if prec == "f32" else np.float64
    rng = np.random.default_rng(80 + len(groups))
    g = D.Dag()
    ins, arrays, leaves, widths = [], [], [], []
    for gi, (width, rows) in enumerate(groups):
        shape = [] if rows is None else [rows]
        cols = []
        for j in range(width):
            a = np.asarray(rng.standard_normal(shape) * 10.0 ** rng.integers(-3, 4, size=shape), dtype=dt)
            cols.append(a.reshape(-1))
            ins.append(g.load(f"c{gi}_{j}", shape, prec))
            arrays.append(a)
        widths.append(width)
        for r in range(1 if rows is None else rows):   # row first, then input order
            leaves.extend(c[r] for c in cols)
    g.roots = [g.add({"OrderedAdjointSum": {"groups": widths}}, ins, [], prec)]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(a).cuda() for a in arrays])
    finally:
        L.load().chelis_dag_release(h)
    want = _pair_tree(leaves)
    want = dt(0) if want is None else want
    assert got.shape == ()
    assert got.tobytes() == np.asarray(want, dtype=dt).tobytes()


def test_ordered_adjoint_sum_nan_and_zero_rules(cuda):
    payload = np.array([0x7FC01234], np.uint32).view(np.float32)[0]
    neg0 = np.float32(-0.0)
    cases = [([payload], 0x7FC01234),                 # one leaf: its payload kept
             ([np.float32(1), payload], 0x7FC00000),  # an addition: canonical NaN
             ([neg0, neg0, neg0], 0x80000000)]        # -0 + -0 stays -0
    for vals, bits in cases:
        g = D.Dag()
        ins = [g.load(f"v{i}", [], "f32") for i in range(len(vals))]
        g.roots = [g.add({"OrderedAdjointSum": {"groups": [1] * len(vals)}}, ins, [], "f32")]
        h = program(g)
        try:
            (got,) = run(h, [torch.from_numpy(np.array(v, np.float32)).cuda() for v in vals])
        finally:
            L.load().chelis_dag_release(h)
        assert int(got.view(np.uint32)) == bits


def test_shape_reads_the_extent(cuda):
    g = D.Dag()
    x = g.load("x", [3, 5, 7])
    g.roots = [g.add({"Shape": {"axis": a}}, [x], [], "i64") for a in range(3)]
    h = program(g)
    try:
        got = run(h, [torch.zeros(3, 5, 7, device="cuda")])
    finally:
        L.load().chelis_dag_release(h)
    assert [int(v) for v in got] == [3, 5, 7]


def test_host_array_entry(cuda, orc):
    """chelis_dag_run: host tensors in, runtime-owned host tensors out."""
    lib = L.load()
    g = D.Dag()
    a = g.load("a", [5, 7])
    b = g.load("b", [7], )
    g.roots = [g.binary("Mul", a, g.expand(b, 0, 5))]
    h = program(g)
    rng = np.random.default_rng(2)
    A = rng.standard_normal((5, 7)).astype(np.float32)
    B = rng.standard_normal(7).astype(np.float32)
    try:
        hs = []
        for arr in (A, B):
            shape = (ctypes.c_int64 * arr.ndim)(*arr.shape)
            hs.append(lib.chelis_tensor_entry_borrow(arr.ndim, shape, L.DTYPE_F32, arr.ctypes.data, arr.nbytes))
        ins = (ctypes.c_void_p * 2)(*hs)
        outs = (ctypes.c_void_p * 1)()
        L.call("chelis_dag_run", h, ins, 2, outs, 1)
        view = lib.chelis_tensor_read_view(outs[0])
        got = np.ctypeslib.as_array(ctypes.cast(view.data, ctypes.POINTER(ctypes.c_float)), shape=(5, 7)).copy()
        assert np.array_equal(got, A * B)
        lib.chelis_tensor_release(outs[0])
        for t in hs:
            lib.chelis_tensor_release(t)
    finally:
        lib.chelis_dag_release(h)


# ---- Compare / Logical / Where / MinReduce (the C lane's semantics,
# crates/chelis-backend-c/src/emit.rs comparison_operator, emit_reduce_extreme)

CMP = {"CmpLt": np.less, "Lt": np.less, "Eq": np.equal, "Neq": np.not_equal,
       "Gt": np.greater, "Gte": np.greater_equal, "Lte": np.less_equal}


def _edge_f32(shape, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(shape).astype(np.float32)
    flat = x.reshape(-1)
    special = np.array([np.nan, -0.0, 0.0, np.inf, -np.inf, 1.0, 1.0, -2.5], np.float32)
    flat[:special.size] = special
    return x


@pytest.mark.parametrize("kind", list(CMP))
def test_compare_f32_ieee(cuda, kind):
    """NaN makes every ordered comparison and eq false, neq true; -0 == +0."""
    a = _edge_f32((6, 37), 1)
    b = _edge_f32((6, 37), 2)
    b.reshape(-1)[:8] = np.array([np.nan, 0.0, -0.0, np.inf, np.inf, np.nan, 1.0, -2.5], np.float32)
    g = D.Dag()
    x, y = g.load("a", [6, 37]), g.load("b", [6, 37])
    g.roots = [g.compare(kind, x, y)]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    with np.errstate(invalid="ignore"):
        want = CMP[kind](a, b)
    assert np.array_equal(got, want.astype(np.uint8))


@pytest.mark.parametrize("prec,dt", [("i64", np.int64), ("i32", np.int32), ("f64", np.float64)])
def test_compare_other_precisions(cuda, prec, dt):
    rng = np.random.default_rng(4)
    a = rng.integers(-5, 5, (9, 11)).astype(dt)
    b = rng.integers(-5, 5, (9, 11)).astype(dt)
    if dt == np.int64:
        a[0, 0], b[0, 0] = np.iinfo(np.int64).min, np.iinfo(np.int64).max  # exact order at full width
    for kind in ("Lt", "Eq", "Gte"):
        g = D.Dag()
        x, y = g.load("a", [9, 11], prec), g.load("b", [9, 11], prec)
        g.roots = [g.compare(kind, x, y)]
        h = program(g)
        try:
            (got,) = run(h, [torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()])
        finally:
            L.load().chelis_dag_release(h)
        assert np.array_equal(got, CMP[kind](a, b).astype(np.uint8)), kind


def test_logical_and_bool_equality(cuda):
    rng = np.random.default_rng(5)
    a = rng.integers(0, 2, (4, 33)).astype(bool)
    b = rng.integers(0, 2, (4, 33)).astype(bool)
    g = D.Dag()
    x, y = g.load("a", [4, 33], "bool"), g.load("b", [4, 33], "bool")
    g.roots = [g.logical("And", x, y), g.logical("Or", x, y), g.logical("Not", x),
               g.compare("Eq", x, y), g.compare("Neq", x, y)]
    h = program(g)
    try:
        got = run(h, [torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    for r, w in zip(got, (a & b, a | b, ~a, a == b, a != b)):
        assert np.array_equal(r, w.astype(np.uint8))


def test_where_keeps_stored_bits(cuda):
    """Where selects stored bits: NaN payloads and signed zeros come through."""
    rng = np.random.default_rng(6)
    c = rng.integers(0, 2, (5, 40)).astype(bool)
    a = rng.standard_normal((5, 40)).astype(np.float32)
    b = rng.standard_normal((5, 40)).astype(np.float32)
    a.view(np.uint32)[0, :4] = [0x7fc12345, 0xffc00001, 0x80000000, 0x00000001]
    b.view(np.uint32)[0, :4] = [0x80000000, 0x7f800000, 0x7fa00000, 0x80000001]
    c[0, :4] = [True, True, False, False]
    ai = rng.integers(-9, 9, (5, 40)).astype(np.int64)
    bi = rng.integers(-9, 9, (5, 40)).astype(np.int64)
    g = D.Dag()
    cc = g.load("c", [5, 40], "bool")
    x, y = g.load("a", [5, 40]), g.load("b", [5, 40])
    xi, yi = g.load("ai", [5, 40], "i64"), g.load("bi", [5, 40], "i64")
    g.roots = [g.where(cc, x, y), g.where(cc, xi, yi)]
    h = program(g)
    try:
        got = run(h, [torch.from_numpy(t).cuda() for t in (c, a, b, ai, bi)])
    finally:
        L.load().chelis_dag_release(h)
    assert np.array_equal(got[0].view(np.uint32), np.where(c, a, b).view(np.uint32))
    assert np.array_equal(got[1], np.where(c, ai, bi))


def _min_scan(x, axis):
    """The C lane's in-order MinReduce: the first NaN, else the first of the
    smallest values; the selected element's stored bits."""
    x = np.moveaxis(x, axis, -1)
    out = np.empty(x.shape[:-1], x.dtype)
    for idx in np.ndindex(*x.shape[:-1]):
        row = x[idx]
        best = None
        for v in row:
            if best is None or (not np.isnan(best) and (np.isnan(v) or v < best)):
                best = v
        out[idx] = best
    return out


@pytest.mark.parametrize("axis", [0, 1])
def test_min_reduce_selection_rules(cuda, axis):
    x = np.random.default_rng(7).standard_normal((70, 45)).astype(np.float32)
    x.view(np.uint32)[3, 5] = 0x7fc0abcd   # first NaN of its row / column
    x.view(np.uint32)[3, 9] = 0xffc00002   # a later NaN
    x.view(np.uint32)[10, 6] = 0xffc00003
    x.view(np.uint32)[40, 6] = 0x7fc00004  # later NaN in column 6
    x[12, :] = 5.0
    x[12, 20], x[12, 30] = -0.0, 0.0       # tie of signed zeros: the first one
    x[:, 33] = 7.0
    x[50, 33], x[60, 33] = 0.0, -0.0
    g = D.Dag()
    a = g.load("x", [70, 45])
    g.roots = [g.min_reduce(a, axis)]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(x).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    assert np.array_equal(got.view(np.uint32), _min_scan(x, axis).view(np.uint32))


def test_min_reduce_i64_and_strided_view(cuda):
    """MinReduce of a permuted (strided) view and of integers."""
    x = np.random.default_rng(8).integers(-1000, 1000, (33, 17)).astype(np.int64)
    g = D.Dag()
    a = g.load("x", [33, 17], "i64")
    g.roots = [g.min_reduce(g.permute(a, [1, 0]), 1)]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(x).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    assert np.array_equal(got, x.min(axis=0))


def test_min_reduce_empty_axis_traps(cuda):
    g = D.Dag()
    a = g.load("x", [4, 0])
    g.roots = [g.min_reduce(a, 1)]
    h = program(g)
    try:
        with pytest.raises(L.ChelisCudaError, match="numeric trap: domain in min_reduce at f32"):
            run(h, [torch.empty((4, 0), device="cuda")])
    finally:
        L.load().chelis_dag_release(h)


def test_causal_masked_softmax_program(cuda):
    """where(cmplt(col, row) | eq, s, -inf) then Softmax: the causal-attention
    mask as the reference writes it (spec/05-risc-primitives.md:5146-5181),
    against numpy."""
    n = 64
    s = np.random.default_rng(9).standard_normal((n, n)).astype(np.float32)
    rows = np.repeat(np.arange(n, dtype=np.int64)[:, None], n, axis=1)
    cols = np.repeat(np.arange(n, dtype=np.int64)[None, :], n, axis=0)
    g = D.Dag()
    x = g.load("s", [n, n])
    r, c = g.load("rows", [n, n], "i64"), g.load("cols", [n, n], "i64")
    keep = g.logical("Or", g.compare("CmpLt", c, r), g.compare("Eq", c, r))
    ninf = g.expand(g.expand(g.const(float("-inf")), 0, n), 1, n)
    masked = g.where(keep, x, ninf)
    g.roots = [g.add({"Softmax": {"axis": 1}}, [masked], [n, n])]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(t).cuda() for t in (s, rows, cols)])
    finally:
        L.load().chelis_dag_release(h)
    m = np.where(cols <= rows, s.astype(np.float64), -np.inf)
    e = np.exp(m - m.max(axis=1, keepdims=True))
    want = e / e.sum(axis=1, keepdims=True)
    assert rel(got, want) <= 1e-6
    assert np.all(got[np.triu_indices(n, 1)] == 0.0)


def _arg_scan(x, axis, take_max):
    """emit_reduce_argcmp's in-order choice: first NaN, else the first extreme."""
    x = np.moveaxis(x, axis, -1)
    out = np.empty(x.shape[:-1], np.int64)
    for idx in np.ndindex(*x.shape[:-1]):
        best, bi = None, -1
        for i, v in enumerate(x[idx]):
            if bi < 0:
                best, bi = v, i
                continue
            better = (v > best) if take_max else (v < best)
            if not np.isnan(best) and (np.isnan(v) or better):
                best, bi = v, i
        out[idx] = bi
    return out


@pytest.mark.parametrize("op,axis", [("Argmax", 1), ("Argmin", 1), ("Argmax", 0), ("Argmin", 0)])
def test_argmax_argmin_selection_rules(cuda, op, axis):
    x = np.random.default_rng(10).standard_normal((50, 41)).astype(np.float32)
    x[4, :] = 2.0                       # ties: the first position
    x[7, 3], x[7, 30] = np.nan, np.nan  # the first NaN wins
    x[9, :] = 0.0
    x[9, 5] = -0.0                      # signed zeros tie
    x[:, 12] = 1.0
    x[20, 12] = np.nan
    g = D.Dag()
    a = g.load("x", [50, 41])
    g.roots = [g.arg_reduce(op, a, axis)]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(x).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    with np.errstate(invalid="ignore"):
        assert np.array_equal(got, _arg_scan(x, axis, op == "Argmax"))


def test_prod_reduce_in_axis_order(cuda):
    """ProdReduce multiplies from 1 in axis order, each product rounded to f32."""
    x = (1.0 + 0.3 * np.random.default_rng(11).standard_normal((13, 60))).astype(np.float32)
    g = D.Dag()
    a = g.load("x", [13, 60])
    g.roots = [g.prod_reduce(a, 1), g.prod_reduce(a, 0)]
    h = program(g)
    try:
        got = run(h, [torch.from_numpy(x).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    for r, ax in zip(got, (1, 0)):
        xm = np.moveaxis(x, ax, -1)
        want = np.empty(xm.shape[:-1], np.float32)
        for idx in np.ndindex(*xm.shape[:-1]):
            acc = np.float32(1.0)
            for v in xm[idx]:
                acc = np.float32(acc * v)
            want[idx] = acc
        assert np.array_equal(r.view(np.uint32), want.view(np.uint32))


def test_float_classify_and_extrema_adjoint(cuda):
    a = _edge_f32((3, 50), 12)
    b = _edge_f32((3, 50), 13)
    b.reshape(-1)[:8] = np.array([1.0, np.nan, -0.0, np.inf, 3.0, np.nan, 1.0, -9.0], np.float32)
    gr = np.random.default_rng(14).standard_normal((3, 50)).astype(np.float32)
    g = D.Dag()
    x, y, c = g.load("a", [3, 50]), g.load("b", [3, 50]), g.load("g", [3, 50])
    g.roots = [g.classify("Nan", x), g.classify("Finite", x), g.classify("Infinite", x),
               g.extrema_adjoint("Max", "Left", x, y, c), g.extrema_adjoint("Max", "Right", x, y, c),
               g.extrema_adjoint("Min", "Left", x, y, c), g.extrema_adjoint("Min", "Right", x, y, c)]
    h = program(g)
    try:
        got = run(h, [torch.from_numpy(t).cuda() for t in (a, b, gr)])
    finally:
        L.load().chelis_dag_release(h)
    assert np.array_equal(got[0], np.isnan(a).astype(np.uint8))
    assert np.array_equal(got[1], np.isfinite(a).astype(np.uint8))
    assert np.array_equal(got[2], np.isinf(a).astype(np.uint8))
    with np.errstate(invalid="ignore"):
        left_max = np.isnan(a) | (~np.isnan(b) & (a >= b))
        left_min = np.isnan(a) | (~np.isnan(b) & (a <= b))
    zero = np.zeros_like(gr)
    for r, sel in zip(got[3:], (left_max, ~left_max, left_min, ~left_min)):
        assert np.array_equal(r.view(np.uint32), np.where(sel, gr, zero).view(np.uint32))


# ---- keys and keyed dropout ([05-OP-37], [05-OP-69..72]; the C lane's
# emit_explicitly_keyed_dropout, emit_split_key, emit_fold_in, emit_split_keys)

def test_key_derivations_match_oracle(cuda, orc):
    seeds = np.array([0, 1, 42, -7, 2 ** 62, -(2 ** 63)], np.int64)
    data = np.array([3, -1, 0, 99, 5, 2 ** 40], np.int64)
    g = D.Dag()
    sd, dd = g.load("seed", [6], "i64"), g.load("n", [6], "i64")
    k = g.key_from_seed(sd)
    g.roots = [k, g.split_key(k, "Left"), g.split_key(k, "Right"), g.fold_in(k, dd), g.split_n(k, 3)]
    h = program(g)
    try:
        got = run(h, [torch.from_numpy(seeds).cuda(), torch.from_numpy(data).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    u = [int(v) & (2 ** 64 - 1) for v in seeds]
    assert [int(v) for v in got[0]] == u
    assert [int(v) for v in got[1]] == [orc.derive(x, 0) for x in u]
    assert [int(v) for v in got[2]] == [orc.derive(x, 1) for x in u]
    assert [int(v) for v in got[3]] == [orc.derive(orc.derive(x, 2), int(n) & (2 ** 64 - 1))
                                         for x, n in zip(u, data)]
    assert [[int(v) for v in row] for row in got[4]] == [[orc.derive(orc.derive(x, 2), j) for j in range(3)]
                                                         for x in u]


@pytest.mark.parametrize("replay", [False, True])
def test_keyed_dropout_rank0_key_matches_oracle(cuda, orc, replay):
    """One key for the whole draw: element e of the flat data uses word(key, e)."""
    x = np.random.default_rng(20).standard_normal((37, 129)).astype(np.float32)
    x.view(np.uint32)[0, :2] = [0x7fc00123, 0xffc00001]  # NaN payloads come out canonical
    g = D.Dag()
    xs = g.load("x", [37, 129])
    rate = g.const(0.3)
    k = g.key_from_seed(g.load("seed", [], "i64"))
    g.roots = [g.dropout(xs, rate, k, replay)]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(x).cuda(), torch.tensor(1234, dtype=torch.int64).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    want = orc.dropout(x, 1234, 0.3)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_keyed_dropout_per_row_keys_and_rates(cuda, orc):
    """A key per row (the key's shape leads the data's) and a rate per row:
    row b draws word(key[b], e) for its own elements e = 0, 1, ..."""
    x = np.random.default_rng(21).standard_normal((6, 5, 40)).astype(np.float32)
    seeds = np.arange(100, 106, dtype=np.int64)
    rates = np.array([0.0, 0.1, 0.5, 0.9, 0.25, 0.75], np.float32)
    g = D.Dag()
    xs = g.load("x", [6, 5, 40])
    r = g.load("rate", [6])
    k = g.split_key(g.key_from_seed(g.load("seed", [6], "i64")), "Right")
    g.roots = [g.dropout(xs, r, k)]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(t).cuda() for t in (x, rates, seeds)])
    finally:
        L.load().chelis_dag_release(h)
    for b in range(6):
        want = orc.dropout(x[b], orc.derive(int(seeds[b]), 1), float(rates[b]))
        assert np.array_equal(got[b].view(np.uint32), want.view(np.uint32)), b


def test_keyed_dropout_f64(cuda, orc):
    """At f64 the unit value is compared with the rate unrounded."""
    x = np.random.default_rng(22).standard_normal(300)
    g = D.Dag()
    xs = g.load("x", [300], "f64")
    rate = g.const(0.4, prec="f64")
    k = g.key_from_seed(g.load("seed", [], "i64"))
    g.roots = [g.dropout(xs, rate, k)]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(x).cuda(), torch.tensor(77, dtype=torch.int64).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    want = np.array([0.0 if orc.unit(77, e) < 0.4 else x[e] / (1.0 - 0.4) for e in range(300)])
    assert np.array_equal(got, want)


def test_keyed_dropout_rate_out_of_range_traps(cuda):
    g = D.Dag()
    xs = g.load("x", [8])
    rate = g.const(1.0)
    k = g.key_from_seed(g.load("seed", [], "i64"))
    g.roots = [g.dropout(xs, rate, k)]
    h = program(g)
    try:
        with pytest.raises(L.ChelisCudaError, match="numeric trap: domain in dropout at f32"):
            run(h, [torch.ones(8, device="cuda"), torch.tensor(1, dtype=torch.int64).cuda()])
    finally:
        L.load().chelis_dag_release(h)


# ---- exact integer arithmetic (chelis_runtime.h chelis_int_checked_*; [04-NUM-9])

def _trunc_div(a, b):
    q = abs(a) // abs(b)
    return q if (a < 0) == (b < 0) else -q


def _rem(a, b):
    r = abs(a) % abs(b)
    return r if a >= 0 else -r


INT_OPS = {"Add": lambda a, b: a + b, "Sub": lambda a, b: a - b, "Mul": lambda a, b: a * b,
           "TruncDiv": _trunc_div, "FloorDiv": lambda a, b: a // b, "Mod": lambda a, b: 0 if b == -1 else _rem(a, b),
           "MaxElem": max, "MinElem": min}


@pytest.mark.parametrize("prec,dt", [("i64", np.int64), ("i32", np.int32), ("i16", np.int16), ("i8", np.int8)])
def test_integer_arithmetic_exact(cuda, prec, dt):
    info = np.iinfo(dt)
    rng = np.random.default_rng(30)
    lim = 2 ** (info.bits // 2 - 2)  # products stay in range
    a = rng.integers(-lim, lim, 257).astype(dt)
    b = rng.integers(-lim, lim, 257).astype(dt)
    b[b == 0] = 3
    b[:4] = [-1, 1, -7, 7]
    a[:4] = [info.min + 1, -13, 13, -14]
    g = D.Dag()
    x, y = g.load("a", [257], prec), g.load("b", [257], prec)
    g.roots = [g.binary(op, x, y) for op in INT_OPS] + [g.unary("Neg", x), g.unary("Abs", x)]
    h = program(g)
    try:
        got = run(h, [torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    for (name, f), r in zip(INT_OPS.items(), got):
        if name == "Mul":
            want = [f(int(p), int(q)) for p, q in zip(a[4:], b[4:])]
            assert [int(v) for v in r[4:]] == want, name
            continue
        want = [f(int(p), int(q)) for p, q in zip(a, b)]
        assert [int(v) for v in r] == want, name
    assert [int(v) for v in got[-2]] == [-int(v) for v in a]
    assert [int(v) for v in got[-1]] == [abs(int(v)) for v in a]


@pytest.mark.parametrize("op,prec,av,bv,message", [
    ("Add", "i64", 2 ** 63 - 1, 1, "overflow in add at i64"),
    ("Sub", "i32", -(2 ** 31), 1, "overflow in sub at i32"),
    ("Mul", "i64", 2 ** 32, 2 ** 31, "overflow in mul at i64"),
    ("Mul", "i16", 300, 300, "overflow in mul at i16"),
    ("TruncDiv", "i64", 5, 0, "division by zero in trunc_div at i64"),
    ("FloorDiv", "i32", -(2 ** 31), -1, "overflow in floor_div at i32"),
    ("Mod", "i64", 5, 0, "division by zero in mod at i64"),
    ("Neg", "i8", -128, 0, "overflow in neg at i8"),
    ("Abs", "i64", -(2 ** 63), 0, "overflow in abs at i64"),
])
def test_integer_arithmetic_traps(cuda, op, prec, av, bv, message):
    dt = {"i64": np.int64, "i32": np.int32, "i16": np.int16, "i8": np.int8}[prec]
    a = np.array([1, av, 2], dt)
    b = np.array([1, bv, 1], dt)
    g = D.Dag()
    x, y = g.load("a", [3], prec), g.load("b", [3], prec)
    g.roots = [g.unary(op, x) if op in ("Neg", "Abs") else g.binary(op, x, y)]
    h = program(g)
    try:
        with pytest.raises(L.ChelisCudaError, match="numeric trap: " + message):
            run(h, [torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    L.call("chelis_cuda_device_status")  # read-and-clear: the next check is clean


def test_integer_mod_of_minimum_by_minus_one_is_zero(cuda):
    a = np.array([-(2 ** 63), 7, -7], np.int64)
    b = np.array([-1, -1, -1], np.int64)
    g = D.Dag()
    x, y = g.load("a", [3], "i64"), g.load("b", [3], "i64")
    g.roots = [g.binary("Mod", x, y)]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    assert list(got) == [0, 0, 0]


def test_float_mod_is_fmod(cuda):
    rng = np.random.default_rng(31)
    a = (rng.standard_normal(200) * 10).astype(np.float32)
    b = rng.standard_normal(200).astype(np.float32)
    b[0], a[1], b[2] = 0.0, np.inf, np.inf
    g = D.Dag()
    x, y = g.load("a", [200]), g.load("b", [200])
    g.roots = [g.binary("Mod", x, y)]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    with np.errstate(invalid="ignore"):
        want = np.fmod(a, b)
    want[np.isnan(want)] = np.float32(np.nan)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# ---- the checked cast (host_emit.rs checked_cast_*; the reference's default cast)

NP = {"f32": np.float32, "f64": np.float64, "i64": np.int64, "i32": np.int32, "i16": np.int16,
      "i8": np.int8, "bool": np.bool_}


@pytest.mark.parametrize("src,dst,values", [
    ("f32", "i32", [0.0, -0.0, 7.0, -2147483648.0, 2147483520.0, -3.0]),
    ("f64", "i64", [1e18, -9223372036854775808.0, 42.0]),
    ("f32", "i8", [127.0, -128.0, 5.0]),
    ("f32", "bool", [0.0, 1.0, -0.0]),
    ("i64", "i32", [2 ** 31 - 1, -(2 ** 31), 0]),
    ("i32", "i64", [-5, 2 ** 31 - 1, 9]),
    ("i64", "bool", [0, 1, 1]),
    ("bool", "i64", [True, False, True]),
    ("i64", "f32", [2 ** 53 + 1, -(2 ** 40) - 3, 16777217]),
    ("i16", "f64", [-32768, 12, 32767]),
])
def test_checked_cast_values(cuda, src, dst, values):
    x = np.array(values, NP[src])
    g = D.Dag()
    a = g.load("x", [len(values)], src)
    g.roots = [g.cast(a, dst)]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(x).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    if dst == "bool":
        assert list(got) == [1 if v == 1 else 0 for v in values]
    elif dst in ("f32", "f64"):
        want = np.array([NP[dst](int(v)) for v in values], NP[dst])
        assert np.array_equal(got, want)
    else:
        assert [int(v) for v in got] == [int(v) for v in values]


@pytest.mark.parametrize("src,dst,bad,message", [
    ("f32", "i32", 1.5, "domain in cast at i32"),
    ("f32", "i64", float("inf"), "domain in cast at i64"),
    ("f32", "i64", float("nan"), "domain in cast at i64"),
    ("f32", "i32", 3e9, "overflow in cast at i32"),
    ("f64", "i64", 9.3e18, "overflow in cast at i64"),
    ("i64", "i8", 300, "overflow in cast at i8"),
    ("i64", "bool", 2, "domain in cast at bool"),
    ("f32", "bool", 0.5, "domain in cast at bool"),
])
def test_checked_cast_traps(cuda, src, dst, bad, message):
    x = np.array([1, bad, 0], NP[src])
    g = D.Dag()
    a = g.load("x", [3], src)
    g.roots = [g.cast(a, dst)]
    h = program(g)
    try:
        with pytest.raises(L.ChelisCudaError, match="numeric trap: " + message):
            run(h, [torch.from_numpy(x).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    L.call("chelis_cuda_device_status")


# ---- named lossy casts (cast_trunc [05-OP-6], cast_saturate [05-OP-23], cast_wrap [05-OP-24])

def _wrap(v, bits):
    v &= (1 << bits) - 1
    return v - (1 << bits) if v >= 1 << (bits - 1) else v


@pytest.mark.parametrize("mode,src,dst,values,want", [
    ("Trunc", "f32", "i32", [2.9, -2.9, -0.0, 1e9, -2147483648.0], [2, -2, 0, 1000000000, -2147483648]),
    ("Trunc", "f64", "i8", [127.9, -128.99, 3.5], [127, -128, 3]),
    ("Saturate", "f32", "i8", [300.0, -1e30, 5.7, -5.7, float("inf"), float("-inf")], [127, -128, 5, -5, 127, -128]),
    ("Saturate", "f64", "i64", [1e19, -1e19, 123.9], [2 ** 63 - 1, -(2 ** 63), 123]),
    ("Saturate", "i64", "i16", [40000, -40000, 12], [32767, -32768, 12]),
    ("Wrap", "i64", "i8", [300, -129, 127, 2 ** 40 + 5], [_wrap(300, 8), _wrap(-129, 8), 127, 5]),
    ("Wrap", "i32", "i64", [-5, 7, 2 ** 31 - 1], [-5, 7, 2 ** 31 - 1]),
])
def test_named_cast_values(cuda, mode, src, dst, values, want):
    x = np.array(values, NP[src])
    g = D.Dag()
    a = g.load("x", [len(values)], src)
    g.roots = [g.named_cast(a, mode, dst)]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(x).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    assert [int(v) for v in got] == want


@pytest.mark.parametrize("mode,src,dst,bad,message", [
    ("Trunc", "f32", "i32", float("nan"), "domain in cast_trunc at i32"),
    ("Trunc", "f32", "i32", float("inf"), "domain in cast_trunc at i32"),
    ("Trunc", "f64", "i8", 128.5, "overflow in cast_trunc at i8"),
    ("Saturate", "f32", "i64", float("nan"), "domain in cast_saturate at i64"),
])
def test_named_cast_traps(cuda, mode, src, dst, bad, message):
    x = np.array([1, bad, 0], NP[src])
    g = D.Dag()
    a = g.load("x", [3], src)
    g.roots = [g.named_cast(a, mode, dst)]
    h = program(g)
    try:
        with pytest.raises(L.ChelisCudaError, match="numeric trap: " + message):
            run(h, [torch.from_numpy(x).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    L.call("chelis_cuda_device_status")


# ---- Bitwise ([05-OP-47]; chelis_runtime.h chelis_int_shl / chelis_int_shr)

def _shl(v, k, bits):
    return 0 if k >= bits else _wrap(v << k, bits)


def _shr(v, k, bits):
    return (-1 if v < 0 else 0) if k >= bits else v >> k


@pytest.mark.parametrize("prec,dt,bits", [("i64", np.int64, 64), ("i32", np.int32, 32), ("i8", np.int8, 8)])
def test_bitwise(cuda, prec, dt, bits):
    rng = np.random.default_rng(40)
    info = np.iinfo(dt)
    a = rng.integers(info.min, info.max, 300, endpoint=True, dtype=np.int64).astype(dt)
    b = rng.integers(info.min, info.max, 300, endpoint=True, dtype=np.int64).astype(dt)
    k = rng.integers(0, min(bits + 10, int(info.max)), 300).astype(dt)
    g = D.Dag()
    x, y, c = g.load("a", [300], prec), g.load("b", [300], prec), g.load("k", [300], prec)
    bw = lambda kind, p, q: g.add({"Bitwise": kind}, [p, q], [300], prec)
    g.roots = [bw("And", x, y), bw("Or", x, y), bw("Xor", x, y), bw("ShiftLeft", x, c), bw("ShiftRight", x, c)]
    h = program(g)
    try:
        got = run(h, [torch.from_numpy(t).cuda() for t in (a, b, k)])
    finally:
        L.load().chelis_dag_release(h)
    A, B, K = [int(v) for v in a], [int(v) for v in b], [int(v) for v in k]
    assert [int(v) for v in got[0]] == [p & q for p, q in zip(A, B)]
    assert [int(v) for v in got[1]] == [p | q for p, q in zip(A, B)]
    assert [int(v) for v in got[2]] == [p ^ q for p, q in zip(A, B)]
    assert [int(v) for v in got[3]] == [_shl(p, q, bits) for p, q in zip(A, K)]
    assert [int(v) for v in got[4]] == [_shr(p, q, bits) for p, q in zip(A, K)]


def test_negative_shift_count_is_reported(cuda):
    a = np.array([1, 2, 3], np.int64)
    k = np.array([0, -3, 1], np.int64)
    g = D.Dag()
    x, c = g.load("a", [3], "i64"), g.load("k", [3], "i64")
    g.roots = [g.add({"Bitwise": "ShiftLeft"}, [x, c], [3], "i64")]
    h = program(g)
    try:
        with pytest.raises(L.ChelisCudaError, match="shift amount must be non-negative, got -3"):
            run(h, [torch.from_numpy(a).cuda(), torch.from_numpy(k).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    L.call("chelis_cuda_device_status")


# ---- GuardedFail ([05-OP-68]; the C lane's emit_guarded_fail)

@pytest.mark.parametrize("trap_on_true", [True, False])
def test_guarded_fail(cuda, trap_on_true):
    """The result is the fallback; where the condition fires the program
    aborts with its own message (CHELIS_CUDA_ERR_FAIL)."""
    fb = np.arange(6, dtype=np.float32)
    quiet = np.full(4, not trap_on_true)
    loud = quiet.copy()
    loud[2] = trap_on_true
    g = D.Dag()
    c, x = g.load("c", [4], "bool"), g.load("x", [6])
    g.roots = [g.add({"GuardedFail": {"message": "withdrawal exceeds the balance", "trap_on_true": trap_on_true}},
                     [c, x], [6])]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(quiet).cuda(), torch.from_numpy(fb).cuda()])
        assert np.array_equal(got, fb)
        with pytest.raises(L.ChelisCudaError, match="withdrawal exceeds the balance") as e:
            run(h, [torch.from_numpy(loud).cuda(), torch.from_numpy(fb).cuda()])
        assert e.value.status == 7
    finally:
        L.load().chelis_dag_release(h)


# ---- UniformLike ([05-OP-8]; the C lane's emit_explicitly_keyed_uniform_like)

def _round_f32(x):
    """The float32 nearest to the exact rational x (ties to even)."""
    from fractions import Fraction
    f = np.float32(float(x))
    cands = [np.nextafter(f, np.float32(-np.inf)), f, np.nextafter(f, np.float32(np.inf))]
    best = min(cands, key=lambda c: (abs(Fraction(float(c)) - x), int(np.array(c).view(np.uint32)) & 1))
    return best


def test_uniform_like_f32_and_f64_match_the_sampler(cuda, orc):
    from fractions import Fraction
    g = D.Dag()
    t32, t64 = g.load("t32", [4, 50]), g.load("t64", [4, 50], "f64")
    k = g.key_from_seed(g.load("seed", [4], "i64"))
    lo32, hi32 = g.load("lo", [4]), g.load("hi", [4])
    g.roots = [g.uniform_like(t32, lo32, hi32, k),
               g.uniform_like(t64, g.const(-1.5, prec="f64"), g.const(2.25, prec="f64"), g.split_key(k, "Left"))]
    seeds = np.array([3, 9, -4, 100], np.int64)
    lows = np.array([0.0, -2.0, 5.0, 1e-3], np.float32)
    highs = np.array([1.0, 3.0, 5.0, 7.5], np.float32)
    h = program(g)
    try:
        got = run(h, [torch.zeros(4, 50).cuda(), torch.zeros(4, 50, dtype=torch.float64).cuda(),
                      torch.from_numpy(seeds).cuda(), torch.from_numpy(lows).cuda(), torch.from_numpy(highs).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    for b in range(4):
        key = int(seeds[b]) & (2 ** 64 - 1)
        span = np.float32(highs[b] - lows[b])
        for e in range(50):
            u = np.float32(orc.unit(key, e))
            want = _round_f32(Fraction(float(span)) * Fraction(float(u)) + Fraction(float(lows[b])))
            assert got[0][b, e].view(np.uint32) == np.float32(want).view(np.uint32), (b, e)
            k2 = orc.derive(key, 0)
            w64 = float(Fraction(3.75) * Fraction(orc.unit(k2, e)) + Fraction(-1.5))
            assert got[1][b, e] == w64, (b, e)


def test_uniform_like_bad_bounds_trap(cuda):
    g = D.Dag()
    t = g.load("t", [8])
    k = g.key_from_seed(g.load("seed", [], "i64"))
    g.roots = [g.uniform_like(t, g.const(2.0), g.const(1.0), k)]
    h = program(g)
    try:
        with pytest.raises(L.ChelisCudaError, match="numeric trap: domain in uniform_like at f32"):
            run(h, [torch.zeros(8).cuda(), torch.tensor(5, dtype=torch.int64).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    L.call("chelis_cuda_device_status")


@pytest.mark.parametrize("prec,shape,key_rank,out_rank", [
    ("f32", [4, 50], 1, 1),        # a key per row, a bound per row
    ("f32", [4, 3, 700], 2, 1),    # 12 key rows summed in groups of 3 (2100 leaves: runs of 16)
    ("f64", [6, 40], 1, 0),        # every row into one scalar
    ("f32", [33], 0, 0),           # one scalar key
])
@pytest.mark.parametrize("bound", ["Low", "High"])
def test_uniform_bound_adjoint(cuda, orc, prec, shape, key_rank, out_rank, bound):
    """dtype_semantics.rs:4429: leaf g_i * (1 - u_i) (Low) or g_i * u_i (High),
    u_i rounded to f32 for an f32 draw, each product rounded, then the
    adjacent-pair tree in row-major order at the draw's precision."""
    dt = np.float32 if prec == "f32" else np.float64
    rng = np.random.default_rng(90 + len(shape) + key_rank)
    gv = (rng.standard_normal(shape) * 3).astype(dt)
    kshape = shape[:key_rank]
    seeds = rng.integers(-2 ** 40, 2 ** 40, size=kshape).astype(np.int64)
    g = D.Dag()
    t = g.load("t", shape, prec)
    cot = g.load("g", shape, prec)
    k = g.key_from_seed(g.load("seed", kshape, "i64"))
    g.roots = [g.add({"UniformBoundAdjoint": {"bound": bound}}, [t, cot, k], shape[:out_rank], prec)]
    h = program(g)
    try:
        (got,) = run(h, [torch.zeros(shape, dtype=torch.float32 if prec == "f32" else torch.float64).cuda(),
                         torch.from_numpy(gv).cuda(), torch.from_numpy(seeds).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    rows = int(np.prod(kshape)) if kshape else 1
    row_len = gv.size // rows
    groups = int(np.prod(shape[:out_rank])) if out_rank else 1
    keys = [int(v) & (2 ** 64 - 1) for v in seeds.reshape(-1)] if kshape else [int(seeds) & (2 ** 64 - 1)]
    flat = gv.reshape(-1)
    per = gv.size // groups
    want = []
    for e in range(groups):
        leaves = []
        for i in range(e * per, (e + 1) * per):
            u = orc.unit(keys[i // row_len], i % row_len)
            if prec == "f32":
                u = np.float32(u)
                w = u if bound == "High" else np.float32(1.0) - u
            else:
                w = u if bound == "High" else 1.0 - u
            leaves.append(dt(flat[i] * dt(w)))
        want.append(_pair_tree(leaves))
    want = np.array(want, dtype=dt).reshape(shape[:out_rank])
    assert got.shape == want.shape
    assert got.tobytes() == want.tobytes()


# ---- Iota ([05-OP-54]; the C lane's emit_iota)

def _iota(g, start, end, n):
    return g.add("Iota", [start, end], [n], "i64")


@pytest.mark.parametrize("start,end,n", [(-3, 5, 8), (5, 2, 0), (0, 1, 1), (2 ** 62, 2 ** 62 + 4, 4)])
def test_iota_values(cuda, start, end, n):
    g = D.Dag()
    a, b = g.load("start", [], "i64"), g.load("end", [], "i64")
    g.roots = [_iota(g, a, b, n)]
    h = program(g)
    try:
        (got,) = run(h, [torch.tensor(start, dtype=torch.int64).cuda(), torch.tensor(end, dtype=torch.int64).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    assert [int(v) for v in got] == list(range(start, end))


@pytest.mark.parametrize("start,end,n,message", [
    (0, 4, 5, "domain in range at i64"),
    (-(2 ** 63), 2 ** 63 - 1, 3, "overflow in range at i64"),
])
def test_iota_traps(cuda, start, end, n, message):
    g = D.Dag()
    a, b = g.load("start", [], "i64"), g.load("end", [], "i64")
    g.roots = [_iota(g, a, b, n)]
    h = program(g)
    try:
        with pytest.raises(L.ChelisCudaError, match="numeric trap: " + message):
            run(h, [torch.tensor(start, dtype=torch.int64).cuda(), torch.tensor(end, dtype=torch.int64).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    L.call("chelis_cuda_device_status")


def test_iota_causal_mask_program(cuda):
    """The causal mask from iota: keep[i, j] = j <= i, then where(keep, s, -inf)
    and Softmax, against numpy."""
    n = 48
    s = np.random.default_rng(50).standard_normal((n, n)).astype(np.float32)
    g = D.Dag()
    x = g.load("s", [n, n])
    zero, size = g.load("zero", [], "i64"), g.load("n", [], "i64")
    ix = _iota(g, zero, size, n)
    rows, cols = g.expand(ix, 1, n), g.expand(ix, 0, n)
    keep = g.logical("Not", g.compare("Gt", cols, rows))
    ninf = g.expand(g.expand(g.const(float("-inf")), 0, n), 1, n)
    g.roots = [g.add({"Softmax": {"axis": 1}}, [g.where(keep, x, ninf)], [n, n])]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(s).cuda(), torch.tensor(0, dtype=torch.int64).cuda(),
                         torch.tensor(n, dtype=torch.int64).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    m = np.where(np.arange(n)[None, :] <= np.arange(n)[:, None], s.astype(np.float64), -np.inf)
    e = np.exp(m - m.max(axis=1, keepdims=True))
    assert rel(got, e / e.sum(axis=1, keepdims=True)) <= 1e-6


# ---- ReduceWindow / ReduceWindowGrad ([05-OP-39], spec/05-risc-primitives.md 2.3.1)

def _rw(g, op, x, kind, win, steps, out_dims=None, gr=None):
    body = {"reducer": kind, "window_shape": list(win), "strides": list(steps)}
    if op == "ReduceWindow":
        return g.add({"ReduceWindow": body}, [x], out_dims, g.prec(x))
    return g.add({"ReduceWindowGrad": body}, [x, gr], g.dims(x), g.prec(x))


def _windows(shape, win, steps):
    """For each output index (row-major), its window's leaf positions (row-major)."""
    r, nw = len(shape), len(win)
    lead = shape[:r - nw]
    outs = [(shape[r - nw + k] - win[k]) // steps[k] + 1 for k in range(nw)]
    res = []
    for oc in np.ndindex(*(list(lead) + outs)):
        leaves = []
        for lc in np.ndindex(*win):
            leaves.append(tuple(oc[:r - nw]) + tuple(oc[r - nw + k] * steps[k] + lc[k] for k in range(nw)))
        res.append(leaves)
    return list(lead) + outs, res


def _pick(vals, take_max):
    best, bi = None, -1
    for i, v in enumerate(vals):
        if bi < 0:
            best, bi = v, i
            continue
        if not np.isnan(best) and (np.isnan(v) or (v > best if take_max else v < best)):
            best, bi = v, i
    return best, bi


@pytest.mark.parametrize("kind", ["Sum", "Mean", "Max", "Min"])
def test_reduce_window_and_grad_match_the_c_lane(cuda, orc, kind):
    shape, win, steps = (2, 3, 9, 8), (3, 2), (2, 2)
    rng = np.random.default_rng(60)
    x = rng.standard_normal(shape).astype(np.float32)
    x[0, 0, :3, :2] = 1.5            # ties inside one window
    x[1, 2, 4, 4] = np.nan           # a NaN window
    out_dims, wins = _windows(shape, win, steps)
    gr = rng.standard_normal(out_dims).astype(np.float32)
    g = D.Dag()
    a, b = g.load("x", list(shape)), g.load("g", out_dims)
    g.roots = [_rw(g, "ReduceWindow", a, kind, win, steps, out_dims), _rw(g, "ReduceWindowGrad", a, kind, win, steps, gr=b)]
    h = program(g)
    try:
        fwd, din = run(h, [torch.from_numpy(x).cuda(), torch.from_numpy(gr).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    vol = win[0] * win[1]
    want = np.empty(len(wins), np.float32)
    contrib = {}
    for o, leaves in enumerate(wins):
        vals = np.array([x[p] for p in leaves], np.float32)
        gv = gr.reshape(-1)[o]
        if kind in ("Sum", "Mean"):
            t = np.float32(orc.tree_sum(vals))
            want[o] = t if kind == "Sum" else np.float32(t / np.float32(vol))
            c = gv if kind == "Sum" else np.float32(gv / np.float32(vol))
            for p in leaves:
                contrib.setdefault(p, []).append(c)
        else:
            best, bi = _pick(vals, kind == "Max")
            want[o] = best
            if np.isnan(best):
                contrib.setdefault(leaves[bi], []).append(gv)
            else:
                ties = int((vals == best).sum())
                for p, v in zip(leaves, vals):
                    if v == best:
                        contrib.setdefault(p, []).append(np.float32(gv / np.float32(ties)))
    want = want.reshape(out_dims)
    with np.errstate(invalid="ignore"):
        assert np.array_equal(fwd.view(np.uint32), want.view(np.uint32)) or \
            (kind in ("Sum", "Mean") and np.array_equal(np.isnan(fwd), np.isnan(want)) and
             np.array_equal(np.nan_to_num(fwd), np.nan_to_num(want)))
    dwant = np.zeros(shape, np.float32)
    for p, cs in contrib.items():
        dwant[p] = np.float32(orc.tree_sum(np.array(cs, np.float32)))
    assert np.array_equal(din.view(np.uint32), dwant.view(np.uint32)) or \
        (np.array_equal(np.isnan(din), np.isnan(dwant)) and np.array_equal(np.nan_to_num(din), np.nan_to_num(dwant)))


def test_reduce_window_integer_sum_and_overflow(cuda):
    x = np.arange(40, dtype=np.int32).reshape(5, 8)
    g = D.Dag()
    a = g.load("x", [5, 8], "i32")
    g.roots = [_rw(g, "ReduceWindow", a, "Sum", (2, 3), (1, 2), [4, 3]), _rw(g, "ReduceWindow", a, "Max", (5,), (3,), [5, 2])]
    h = program(g)
    try:
        sums, mx = run(h, [torch.from_numpy(x).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    want = np.array([[x[i:i + 2, j * 2:j * 2 + 3].sum() for j in range(3)] for i in range(4)])
    assert np.array_equal(sums, want)
    assert np.array_equal(mx, np.array([[x[i, j * 3:j * 3 + 5].max() for j in range(2)] for i in range(5)]))
    big = np.full((1, 4), 2 ** 30, np.int32)
    g = D.Dag()
    a = g.load("x", [1, 4], "i32")
    g.roots = [_rw(g, "ReduceWindow", a, "Sum", (4,), (1,), [1, 1])]
    h = program(g)
    try:
        with pytest.raises(L.ChelisCudaError, match="numeric trap: overflow in reduce_window_sum at i32"):
            run(h, [torch.from_numpy(big).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    L.call("chelis_cuda_device_status")


# ---- symbolic extents: names bound from the inputs' shapes per run

def _sym_mlp(n):
    """x[n, 64] @ w[64, 32] + b -> Relu; column sums and the activations.
    `n` is a name (symbolic program) or an int (static program)."""
    g = D.Dag()
    x = g.load("x", [n, 64])
    w = g.load("w", [64, 32])
    b = g.load("b", [32])
    h = g.unary("Relu", g.binary("Add", g.matmul(x, w), g.expand(b, 0, n)))
    g.roots = [g.sum(h, 0), h]
    return g


def test_symbolic_program_runs_at_each_binding(cuda):
    rng = np.random.default_rng(7)
    w = torch.from_numpy(rng.standard_normal((64, 32)).astype(np.float32)).cuda()
    b = torch.from_numpy(rng.standard_normal(32).astype(np.float32)).cuda()
    hs = program(_sym_mlp("n"))
    launches = []
    try:
        for n in (100, 37, 100, 1, 37):                    # repeats reuse the planned instance
            x = torch.from_numpy(rng.standard_normal((n, 64)).astype(np.float32)).cuda()
            got = run(hs, [x, w, b])
            hn = program(_sym_mlp(n))
            try:
                want = run(hn, [x, w, b])
            finally:
                L.load().chelis_dag_release(hn)
            assert len(got) == len(want) == 2
            for a, e in zip(got, want):
                assert a.shape == e.shape and a.tobytes() == e.tobytes(), n
            ref = np.maximum(x.cpu().double().numpy() @ w.cpu().double().numpy() + b.cpu().double().numpy(), 0)
            assert rel(got[0], ref.sum(0)) <= 1e-5
    finally:
        L.load().chelis_dag_release(hs)


def test_symbolic_dim_mismatch_is_reported(cuda):
    g = D.Dag()
    a, c = g.load("a", ["n", 4]), g.load("c", ["n", 4])
    g.roots = [g.binary("Add", a, c)]
    h = program(g)
    try:
        with pytest.raises(L.ChelisCudaError, match=r"symbolic dim `n` mismatch: c\[0\]=3 but n=5"):
            run(h, [torch.zeros(5, 4, device="cuda"), torch.zeros(3, 4, device="cuda")])
        (got,) = run(h, [torch.ones(3, 4, device="cuda"), torch.ones(3, 4, device="cuda")])
        assert got.shape == (3, 4) and (got == 2).all()
    finally:
        L.load().chelis_dag_release(h)


def test_symbolic_program_in_a_caller_arena(cuda):
    """chelis_dag_bind gives the plan for a binding; its arena runs the symbolic program."""
    lib = L.load()
    hs = program(_sym_mlp("n"))
    bound = ctypes.c_void_p()
    try:
        L.call("chelis_dag_bind", hs, (ctypes.c_int64 * 1)(50), 1, ctypes.byref(bound))
        need = lib.chelis_dag_arena_bytes(bound)
        assert need > 0
        arena = torch.empty(need, dtype=torch.uint8, device="cuda")
        rng = np.random.default_rng(8)
        ts = [torch.from_numpy(rng.standard_normal(s).astype(np.float32)).cuda() for s in ((50, 64), (64, 32), (32,))]
        owners = []
        for t in ts:
            shape = (ctypes.c_int64 * t.dim())(*t.shape)
            owners.append(lib.chelis_device_tensor_borrow_shape(L.DTYPE_F32, t.dim(), shape, t.data_ptr(),
                                                                t.numel() * 4))
        ins = (ctypes.c_void_p * 3)(*owners)
        outs = (ctypes.c_void_p * 2)()
        L.call("chelis_dag_run_device_arena", hs, ins, 3, outs, 2, arena.data_ptr(), need)
        L.call("chelis_cuda_synchronize")
        with pytest.raises(L.ChelisCudaError, match="arena of"):
            L.call("chelis_dag_run_device_arena", hs, ins, 3, outs, 2, arena.data_ptr(), need - 256)
        for o in list(outs):
            if o:
                lib.chelis_device_tensor_release(o)
        for o in owners:
            lib.chelis_device_tensor_release(o)
    finally:
        if bound.value:
            lib.chelis_dag_release(bound)
        lib.chelis_dag_release(hs)


# ---- shape contracts (ExtentWitness / CheckedExtent / CheckedUnitAxis;
# eval.rs:5149-5299): decided from the bound extents, reported when the node runs

def _witness(g, x, param, axis, reqs=(), claims=(), site="Caller"):
    body = {"site": site, "parameter": param, "axis": {"Lit": axis},
            "requirements": [{"dtype": "int64", "value": r} for r in reqs],
            "claims": [{"claim": c, "requirement_declares": d} for c, d, _ in claims]}
    return g.add({"ExtentWitness": body}, [x] + [e for _, _, e in claims], [], "i64")


def _contract_program():
    g = D.Dag()
    x, y = g.load("x", ["n", 4]), g.load("y", ["m", 4])
    wx = _witness(g, x, "x", 0)
    wy = _witness(g, y, "y", 0, claims=[("n", True, wx)])
    w4 = _witness(g, x, "x", 1, reqs=[4])
    g.roots = [wx, wy, w4, g.binary("Add", x, x)]
    return g


def test_extent_witnesses_pass_and_return_the_extent(cuda):
    h = program(_contract_program())
    try:
        got = run(h, [torch.ones(5, 4, device="cuda"), torch.ones(5, 4, device="cuda")])
    finally:
        L.load().chelis_dag_release(h)
    assert [int(v) for v in got[:3]] == [5, 5, 4]
    assert (got[3] == 2).all()


def test_extent_witness_claim_mismatch_is_reported(cuda):
    h = program(_contract_program())
    try:
        with pytest.raises(L.ChelisCudaError,
                           match=r"extent `n`: x axis 0 = 5, y axis 0 = 3\nnumeric trap: domain in load at i64"):
            run(h, [torch.ones(5, 4, device="cuda"), torch.ones(3, 4, device="cuda")])
    finally:
        L.load().chelis_dag_release(h)


@pytest.mark.parametrize("site,message", [
    ("Caller", r"extent `8`: claimed = 8, x axis 0 = 5\nnumeric trap: domain in load at i64"),
    ("LocalExpand", r"extent `8`: claimed = 8, node 0 axis 0 = 5\nnumeric trap: domain in expand at i64"),
])
def test_extent_witness_literal_requirement(cuda, site, message):
    g = D.Dag()
    x = g.load("x", ["n", 4])
    g.roots = [_witness(g, x, "x", 0, reqs=[8], site=site)]
    h = program(g)
    try:
        with pytest.raises(L.ChelisCudaError, match=message):
            run(h, [torch.ones(5, 4, device="cuda")])
        (got,) = run(h, [torch.ones(8, 4, device="cuda")])
        assert int(got) == 8
    finally:
        L.load().chelis_dag_release(h)


def test_checked_extent_and_unit_axis(cuda):
    g = D.Dag()
    x = g.load("x", ["n", 1])
    shape0 = g.add({"Shape": {"axis": 0}}, [x], [], "i64")
    six = g.add({"Const": {"value": {"dtype": "int64", "value": 6}}}, [], [], "i64")
    chk = g.add({"CheckedExtent": {"owner": "reshape", "claims": ["n"], "axis": {"Lit": 0}}}, [shape0, six], [], "i64")
    w1 = _witness(g, x, "x", 1, reqs=[1])
    unit = g.add({"CheckedUnitAxis": {"axis": {"Lit": 1}}}, [x, w1], ["n", 1])
    g.roots = [chk, g.binary("Mul", unit, unit)]
    h = program(g)
    try:
        with pytest.raises(L.ChelisCudaError,
                           match=r"extent `n`: claimed = 6, reshape axis 0 = 5\nnumeric trap: domain in reshape at i64"):
            run(h, [torch.ones(5, 1, device="cuda")])
        xs = torch.arange(6, dtype=torch.float32, device="cuda").view(6, 1)
        got = run(h, [xs])
        assert int(got[0]) == 6
        assert np.array_equal(got[1], (xs * xs).cpu().numpy())
    finally:
        L.load().chelis_dag_release(h)


@pytest.mark.parametrize("axes", [[2], [1], [0], [2, 0], [2, 1], [2, 1, 0]])
@pytest.mark.parametrize("permuted", [False, True])
def test_count_over_axes(cuda, axes, permuted):
    """Count (dag.rs: true elements over the listed axes, descending, i64)
    against numpy, on a dense mask and on a permuted view of one."""
    rng = np.random.default_rng(sum(axes) + 10 * permuted)
    base = rng.random((6, 5, 4)) < 0.4
    g = D.Dag()
    m = g.load("m", [6, 5, 4], "bool")
    if permuted:
        m = g.permute(m, [2, 1, 0])
        view = base.transpose(2, 1, 0)
    else:
        view = base
    dims = [d for i, d in enumerate(view.shape) if i not in axes]
    g.roots = [g.add({"Count": {"axes": axes}}, [m], dims, "i64")]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(base).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    want = np.count_nonzero(view, axis=tuple(axes))
    assert np.array_equal(got, want)


@pytest.mark.parametrize("prec", ["f32", "f64"])
@pytest.mark.parametrize("axis,reverse", [(0, False), (0, True), (1, False), (1, True)])
def test_cumsum_along_a_leading_axis(cuda, orc, prec, axis, reverse):
    """Cumsum over axis 0 / 1 of a rank-3 value equals the oracle's scan
    (orc_cumsum, the C lane's order) applied to that axis moved last."""
    dt = np.float32 if prec == "f32" else np.float64
    rng = np.random.default_rng(axis * 2 + reverse)
    x = (rng.standard_normal((33, 20, 7)) * 10.0 ** rng.integers(-3, 4, size=(33, 20, 7))).astype(dt)
    x[3, 4, 5] = np.nan
    g = D.Dag()
    a = g.load("x", list(x.shape), prec)
    g.roots = [g.add({"Cumsum": {"axis": axis, "direction": "Decreasing" if reverse else "Increasing"}},
                     [a], list(x.shape), prec)]
    h = program(g)
    try:
        (got,) = run(h, [torch.from_numpy(x).cuda()])
    finally:
        L.load().chelis_dag_release(h)
    moved = np.ascontiguousarray(np.moveaxis(x, axis, -1))
    length = moved.shape[-1]
    want = orc.cumsum(moved.reshape(-1, length), reverse=reverse).reshape(moved.shape)
    want = np.moveaxis(want, -1, axis)
    w = np.uint32 if prec == "f32" else np.uint64
    assert np.array_equal(got.view(w), want.view(w))
