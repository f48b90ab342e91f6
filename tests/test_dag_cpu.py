"""The DAG executor without a GPU: reading the reference's wire format,
checking, and the storage plan (slot reuse, arena bytes).  Nothing here
launches a kernel."""
import ctypes

import pytest

from chelis_b200 import lib as L
import _dag_programs as D


def load(text):
    lib = L.load()
    h = ctypes.c_void_p()
    raw = text.encode()
    st = lib.chelis_dag_from_json(raw, len(raw), ctypes.byref(h))
    return st, h


def test_reference_wire_snapshot_parses():
    # the exact JSON of crates/chelis-dag-core/tests/wire_behavior.rs:121-122
    text = ('{"nodes":[{"id":0,"op":{"Load":{"name":"grads.1"}},"inputs":[],"output_type":'
            '{"dims":[],"precision":"Int64"},"reusable_input":null,"span_id":"x","merged_spans":[],'
            '"shape_deps":[],"result_claim_deps":[],"owner":{"decl":0,"activation":null}},{"id":1,'
            '"op":{"Const":{"value":{"dtype":"int64","value":9007199254740993}}},"inputs":[],'
            '"output_type":{"dims":[],"precision":"Int64"},"reusable_input":null,"span_id":"c",'
            '"merged_spans":[],"shape_deps":[],"result_claim_deps":[],"owner":{"decl":0,'
            '"activation":null}}],"roots":[1,0],"declarations":[{"name":"fixture","value":false}]}')
    st, h = load(text)
    assert st == 0, L.last_error()
    lib = L.load()
    try:
        assert lib.chelis_dag_input_count(h) == 1
        assert lib.chelis_dag_input_label(h, 0) == b"grads.1"
        assert lib.chelis_dag_output_count(h) == 2
        assert [lib.chelis_dag_output_label(h, i) for i in range(2)] == [b"root0", b"root1"]
        assert lib.chelis_dag_arena_bytes(h) == 0  # the Const is written into its output
    finally:
        lib.chelis_dag_release(h)


def test_plan_reuses_slots_after_last_use():
    g = D.Dag()
    x = g.load("x", [1000])
    a = g.unary("Exp", x)      # slot 0
    b = g.unary("Log", a)      # slot 1 (a is read here)
    c = g.unary("Neg", b)      # slot 0 again (a's last reader has run)
    d = g.unary("Exp", c)      # the output: written into its owner
    g.roots = [d]
    st, h = load(g.json())
    assert st == 0, L.last_error()
    lib = L.load()
    try:
        assert lib.chelis_dag_slot_count(h) == 2
        assert lib.chelis_dag_arena_bytes(h) == 2 * 4096  # 4000 bytes rounded to 256
        assert lib.chelis_dag_live_peak_bytes(h) == 2 * 4096
        assert lib.chelis_dag_output_bytes(h) == 4000
    finally:
        lib.chelis_dag_release(h)


def test_views_and_inlined_reductions_take_no_slots():
    g = D.Dag()
    x = g.load("x", [64, 32])
    t = g.permute(x, [1, 0])                          # a view
    e = g.fused([("Mul", (0, 0))], [t], t)            # read only by the Sum: inlined
    s = g.sum(e, 1)
    g.roots = [s]
    st, h = load(g.json())
    assert st == 0, L.last_error()
    lib = L.load()
    try:
        assert lib.chelis_dag_slot_count(h) == 0
        assert lib.chelis_dag_arena_bytes(h) == 0
    finally:
        lib.chelis_dag_release(h)


def test_mlp_program_plans():
    st, h = load(D.mlp_step_dag().json())
    assert st == 0, L.last_error()
    lib = L.load()
    try:
        assert [lib.chelis_dag_input_label(h, i) for i in range(lib.chelis_dag_input_count(h))] == \
            [b"x", b"w1", b"b1", b"w2", b"b2", b"labels"]
        assert lib.chelis_dag_output_count(h) == 5
        arena, live = lib.chelis_dag_arena_bytes(h), lib.chelis_dag_live_peak_bytes(h)
        assert 0 < live <= arena
        # reuse: the arena is below the sum of every materialised value
        assert arena < 2_000_000
    finally:
        lib.chelis_dag_release(h)


@pytest.mark.parametrize("text,status,needle", [
    ('{"nodes": [', 1, "malformed JSON"),
    ('{"nodes": [], "roots": [3]}', 1, "root"),
    ('{"nodes":[{"id":0,"op":"KeySelect","inputs":[],"output_type":{"dims":[{"Lit":4}],'
     '"precision":"Key"},"owner":{"decl":0,"activation":null}}],"roots":[0]}', 4, "KeySelect"),
    ('{"nodes":[{"id":0,"op":{"Load":{"name":"x"}},"inputs":[],"output_type":{"dims":'
     '[{"Lit":4}],"precision":"F32"},"owner":{"decl":0,"activation":null}},{"id":1,"op":{"Shrink":'
     '{"bounds":[[{"Node":2},{"Lit":4}]]}},"inputs":[0],"output_type":{"dims":[{"Lit":4}],"precision":"F32"},'
     '"owner":{"decl":0,"activation":null}}],"roots":[1]}', 4, "a runtime bound"),
    ('{"nodes":[{"id":0,"op":"Neg","inputs":[0],"output_type":{"dims":[],"precision":"F32"},'
     '"owner":{"decl":0,"activation":null}}],"roots":[0]}', 1, "earlier"),
])
def test_rejections(text, status, needle):
    st, h = load(text)
    assert st == status
    assert needle in L.last_error()
    assert not h.value


def test_compare_logical_where_min_reduce_plan():
    """The mask pattern of causal attention parses, checks and plans: Compare,
    Logical, Where over an expanded scalar, MinReduce."""
    g = D.Dag()
    s = g.load("s", [8, 8])
    r, c = g.load("rows", [8, 8], "i64"), g.load("cols", [8, 8], "i64")
    keep = g.logical("Or", g.compare("CmpLt", c, r), g.compare("Eq", c, r))
    ninf = g.expand(g.expand(g.const(float("-inf")), 0, 8), 1, 8)
    g.roots = [g.min_reduce(g.where(keep, s, ninf), 0), g.logical("Not", keep)]
    st, h = load(g.json())
    assert st == 0, L.last_error()
    lib = L.load()
    try:
        assert lib.chelis_dag_input_count(h) == 3
        assert lib.chelis_dag_output_count(h) == 2
    finally:
        lib.chelis_dag_release(h)


@pytest.mark.parametrize("build,message", [
    (lambda g, a, b, t: g.add({"Compare": "Less"}, [a, b], [4], "bool"), "Compare kind"),
    (lambda g, a, b, t: g.compare("Lt", t, t), "ordered comparison of bool"),
    (lambda g, a, b, t: g.add({"Compare": "Eq"}, [a, b], [4], "f32"), "Compare result must be bool"),
    (lambda g, a, b, t: g.logical("And", a, b), "Logical operand must be bool"),
    (lambda g, a, b, t: g.add({"Logical": "Xor"}, [t, t], [4], "bool"), "Logical kind"),
    (lambda g, a, b, t: g.where(a, a, b), "Where condition must be bool"),
    (lambda g, a, b, t: g.min_reduce(t, 0), "MinReduce"),
])
def test_compare_logical_where_min_reduce_rejections(build, message):
    g = D.Dag()
    a, b = g.load("a", [4]), g.load("b", [4])
    t = g.load("t", [4], "bool")
    g.roots = [build(g, a, b, t)]
    st, h = load(g.json())
    assert st != 0
    assert message in L.last_error()


@pytest.mark.parametrize("build,message", [
    (lambda g, a: g.add({"Argmax": {"axis": 0}}, [a], [], "f32"), "reduction result dtype"),
    (lambda g, a: g.add({"FloatClassify": "Odd"}, [a], [4], "bool"), "FloatClassify kind"),
    (lambda g, a: g.add({"ExtremaAdjoint": {"kind": "Mid", "operand": "Left"}}, [a, a, a], [4], "f32"),
     "ExtremaAdjoint kind"),
])
def test_arg_classify_extrema_rejections(build, message):
    g = D.Dag()
    a = g.load("a", [4])
    g.roots = [build(g, a)]
    st, h = load(g.json())
    assert st != 0
    assert message in L.last_error()


@pytest.mark.parametrize("build,message", [
    (lambda g, x, sd: g.add({"Split": {"branch": "Middle"}}, [g.key_from_seed(sd)], [], "key"), "Split branch"),
    (lambda g, x, sd: g.key_from_seed(x), "KeyFromSeed seed must be i64"),
    (lambda g, x, sd: g.add({"SplitN": {"count": {"Node": 1}}}, [g.key_from_seed(sd)], [2], "key"),
     "SplitN with a runtime count"),
    (lambda g, x, sd: g.dropout(x, g.const(0.5), sd), "Dropout key must be a key"),
])
def test_key_and_dropout_rejections(build, message):
    g = D.Dag()
    x = g.load("x", [4])
    sd = g.load("seed", [], "i64")
    g.roots = [build(g, x, sd)]
    st, h = load(g.json())
    assert st != 0
    assert message in L.last_error()


def test_dropout_under_an_activation_is_rejected():
    g = D.Dag()
    x = g.load("x", [4])
    act = g.load("on", [], "bool")
    k = g.key_from_seed(g.load("seed", [], "i64"))
    d = g.dropout(x, g.const(0.5), k)
    g.nodes[d]["owner"]["activation"] = act
    g.roots = [d]
    st, h = load(g.json())
    assert st != 0
    assert "under an activation" in L.last_error()


@pytest.mark.parametrize("mode,src,message", [
    ("Trunc", "i64", "cast_trunc converts a float source"),
    ("Wrap", "f32", "cast_wrap converts an integer source"),
    ("Round", "f32", "NamedCast mode"),
])
def test_named_cast_rejections(mode, src, message):
    g = D.Dag()
    a = g.load("a", [4], src)
    g.roots = [g.named_cast(a, mode, "i32")]
    st, h = load(g.json())
    assert st != 0
    assert message in L.last_error()


@pytest.mark.parametrize("body,dims,message", [
    ({"reducer": "Max", "window_shape": [2], "strides": [2, 1]}, [3], "window_shape / strides"),
    ({"reducer": "Max", "window_shape": [0], "strides": [1]}, [3], "window_shape / strides"),
    ({"reducer": "Median", "window_shape": [2], "strides": [1]}, [5], "ReduceWindow reducer"),
    ({"reducer": "Sum", "window_shape": [7], "strides": [1]}, [1], "window larger than its axis"),
    ({"reducer": "Sum", "window_shape": [2], "strides": [2]}, [4], "ReduceWindow result shape"),
])
def test_reduce_window_rejections(body, dims, message):
    g = D.Dag()
    a = g.load("a", [6])
    g.roots = [g.add({"ReduceWindow": body}, [a], dims)]
    st, h = load(g.json())
    assert st != 0
    assert message in L.last_error()


@pytest.mark.parametrize("ishape,ushape,iprec,message", [
    ([2, 2], [2, 3], "i64", "ScatterElements shapes"),
    ([2], [2], "i64", "ScatterElements shapes"),
    ([3, 2], [3, 2], "i64", "index extent beyond the data"),
    ([2, 2], [2, 2], "f32", "index dtype must be a signed integer"),
])
def test_scatter_elements_rejections(ishape, ushape, iprec, message):
    g = D.Dag()
    a = g.load("a", [2, 3])
    i = g.load("i", ishape, iprec)
    u = g.load("u", ushape)
    g.roots = [g.add({"ScatterElements": {"axis": 1}}, [a, i, u], [2, 3])]
    st, h = load(g.json())
    assert st != 0
    assert message in L.last_error()


@pytest.mark.parametrize("body,dims,shapes,message", [
    ({"groups": [2]}, [], [[3], [4]], "ordered List cotangent columns have different lengths"),
    ({"groups": [2]}, [], [[], []], "rank-one columns or one scalar"),
    ({"groups": [1]}, [3], [[3]], "result must be a scalar"),
    ({"groups": [0, 1]}, [], [[3]], "group width"),
])
def test_ordered_adjoint_sum_rejections(body, dims, shapes, message):
    g = D.Dag()
    ins = [g.load(f"c{i}", s) for i, s in enumerate(shapes)]
    g.roots = [g.add({"OrderedAdjointSum": body}, ins, dims)]
    st, h = load(g.json())
    assert st != 0
    assert message in L.last_error()


def test_shape_rejections():
    g = D.Dag()
    x = g.load("x", [3])
    g.roots = [g.add({"Shape": {"axis": 1}}, [x], [], "i64")]
    st, h = load(g.json())
    assert st != 0
    assert "Shape axis beyond the input rank" in L.last_error()


@pytest.mark.parametrize("bound,kshape,dims,message", [
    ("Middle", [4], [4], "UniformBoundAdjoint bound"),
    ("Low", [5], [5], "UniformBoundAdjoint key shape"),
    ("Low", [4], [4, 6], "not a leading part of its keys' shape"),
])
def test_uniform_bound_adjoint_rejections(bound, kshape, dims, message):
    g = D.Dag()
    t, cot = g.load("t", [4, 6]), g.load("g", [4, 6])
    k = g.key_from_seed(g.load("seed", kshape, "i64"))
    g.roots = [g.add({"UniformBoundAdjoint": {"bound": bound}}, [t, cot, k], dims)]
    st, h = load(g.json())
    assert st != 0
    assert message in L.last_error()


def _symbolic_program():
    """x[n, 64] @ w[64, 32] -> Relu -> column sums, plus a bias expanded to n rows."""
    g = D.Dag()
    x = g.load("x", ["n", 64])
    w = g.load("w", [64, 32])
    b = g.load("b", [32])
    h = g.unary("Relu", g.binary("Add", g.matmul(x, w), g.expand(b, 0, "n")))
    g.roots = [g.sum(h, 0), h]
    return g


def test_symbolic_program_loads_and_binds():
    lib = L.load()
    st, h = load(_symbolic_program().json())
    assert st == 0, L.last_error()
    try:
        assert lib.chelis_dag_symbol_count(h) == 1
        assert lib.chelis_dag_symbol_name(h, 0) == b"n"
        assert lib.chelis_dag_input_count(h) == 3
        assert lib.chelis_dag_output_count(h) == 2
        assert lib.chelis_dag_arena_bytes(h) == -1          # unbound: no plan yet
        for n in (1, 300):
            bound = ctypes.c_void_p()
            vals = (ctypes.c_int64 * 1)(n)
            assert lib.chelis_dag_bind(h, vals, 1, ctypes.byref(bound)) == 0, L.last_error()
            try:
                assert lib.chelis_dag_symbol_count(bound) == 0
                assert lib.chelis_dag_output_bytes(bound) == 4 * 32 + 4 * n * 32
                # the same plan a static program of that size gets
                g = _symbolic_program()
                for node in g.nodes:
                    node["output_type"]["dims"] = [{"Lit": n} if "Named" in d else d
                                                   for d in node["output_type"]["dims"]]
                st2, h2 = load(g.json())
                assert st2 == 0, L.last_error()
                try:
                    for q in ("chelis_dag_arena_bytes", "chelis_dag_live_peak_bytes", "chelis_dag_slot_count"):
                        assert getattr(lib, q)(bound) == getattr(lib, q)(h2), q
                finally:
                    lib.chelis_dag_release(h2)
            finally:
                lib.chelis_dag_release(bound)
        bound = ctypes.c_void_p()
        assert lib.chelis_dag_bind(h, (ctypes.c_int64 * 2)(1, 2), 2, ctypes.byref(bound)) != 0
        assert "expected 1 symbol values" in L.last_error()
    finally:
        lib.chelis_dag_release(h)


def test_symbol_bound_by_no_input_is_reported_at_bind():
    g = D.Dag()
    x = g.load("x", [4])
    g.roots = [g.expand(x, 0, "m")]          # m names no input axis
    st, h = load(g.json())
    assert st == 0, L.last_error()
    lib = L.load()
    try:
        assert lib.chelis_dag_symbol_count(h) == 0
        assert lib.chelis_dag_arena_bytes(h) == -1
        bound = ctypes.c_void_p()
        assert lib.chelis_dag_bind(h, None, 0, ctypes.byref(bound)) == 1
        assert "missing symbolic dimension binding: `m`" in L.last_error()
        assert not bound.value
    finally:
        lib.chelis_dag_release(h)


def test_symbolic_program_still_rejects_unsupported_ops():
    g = D.Dag()
    x = g.load("x", ["n"])
    g.roots = [g.add("KeySelect", [x], ["n"])]
    st, h = load(g.json())
    assert st == 4
    assert "KeySelect" in L.last_error()


def test_broken_static_contract_loads_and_fails_only_when_run():
    g = D.Dag()
    x = g.load("x", [5, 4])
    w = g.add({"ExtentWitness": {"site": "Caller", "parameter": "x", "axis": {"Lit": 0},
                                 "requirements": [{"dtype": "int64", "value": 8}], "claims": []}}, [x], [], "i64")
    g.roots = [w]
    st, h = load(g.json())
    assert st == 0, L.last_error()
    L.load().chelis_dag_release(h)


def test_count_axes_must_descend():
    g = D.Dag()
    m = g.load("m", [3, 4], "bool")
    g.roots = [g.add({"Count": {"axes": [0, 1]}}, [m], [], "i64")]
    st, h = load(g.json())
    assert st != 0
    assert "descending order" in L.last_error()
