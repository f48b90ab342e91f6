"""DAGs in the reference's wire format, for the DAG executor's tests.

`Dag` writes the JSON serde produces for crates/chelis-dag-core's `Dag`
(src/dag.rs:2364-2400, 2913-2920; node layout as in
crates/chelis-dag-core/tests/wire_behavior.rs): nodes with id, op (a unit
variant as a string, a struct variant as {"Name": {...}}), inputs,
output_type {dims: [{"Lit": n}], precision}, reusable_input, span_id,
merged_spans, shape_deps, result_claim_deps, owner; then roots and
declarations.  Scalars are {"dtype": "f32", "bits": "3f800000"} /
{"dtype": "int64", "value": n} (crates/chelis-numeric-core/src/
dtype_semantics/wire_codec.rs:488-530).

`mlp_step_dag` builds config 1 (2-layer MLP, mean cross-entropy, gradients of
the four parameters) the way the reference produces it for a backend:
matmul specialised to BlasMatmul (crates/chelis-ir-core/src/specialize.rs:
150-226), bias broadcast as Expand, relu as Relu (tier2.rs:77-85),
cross-entropy as log(softmax) -> Gather -> diagonal -> neg
(spec/05-risc-primitives.md:5044-5063; diagonal = Shrink, Shrink, Reshape,
Stride: tier2_ordered.rs:154-206), mean as Sum / Const (tier2.rs:1180-1215);
reverse mode by the adjoint rules of grad.rs (Div :1943, Sum :2589, Neg,
Softmax :2248, Relu :2282, Permute :2834, Expand :2847, Shrink :3013, Stride
:3072, Gather :3433 with fill_like :1688, BlasMatmul :3527 with transposing
Permutes, fan-in by balanced_adjoint_sum :1713); the forward Softmax expanded
afterwards (tier2.rs:1097-1178 decompose_softmax); single-consumer
elementwise chains fused into FusedElem and a FusedElem read only by a Sum
left for the backend to inline (fuse.rs:144-203, 463-500).
"""
from __future__ import annotations

import json
import struct

PRIM = {"f32": "F32", "f64": "F64", "i64": "Int64", "i32": "Int32", "bool": "Bool", "key": "Key", "i8": "Int8",
        "i16": "Int16", "f16": "F16", "bf16": "Bf16"}


def f32_scalar(v: float) -> dict:
    return {"dtype": "f32", "bits": "%08x" % struct.unpack("<I", struct.pack("<f", v))[0]}


def f64_scalar(v: float) -> dict:
    return {"dtype": "f64", "bits": "%016x" % struct.unpack("<Q", struct.pack("<d", v))[0]}


def lit(n) -> dict:
    """An RtDim: a literal, or a symbolic name ({"Sym": name})."""
    return {"Lit": n} if isinstance(n, int) else {"Sym": n}


def dim_info(d) -> dict:
    """A DimInfo: Lit(n), or Named(name, None) for a symbolic extent."""
    return {"Lit": d} if isinstance(d, int) else {"Named": [d, None]}


def dim_expr(d) -> dict:
    """A DimExpr: Concrete(n) or Sym(name)."""
    return {"Concrete": d} if isinstance(d, int) else {"Sym": d}


class Dag:
    def __init__(self):
        self.nodes: list[dict] = []
        self.roots: list[int] = []

    def add(self, op, inputs, dims, prec="f32") -> int:
        i = len(self.nodes)
        self.nodes.append({
            "id": i, "op": op, "inputs": list(inputs),
            "output_type": {"dims": [dim_info(d) for d in dims], "precision": PRIM[prec]},
            "reusable_input": None, "span_id": None, "merged_spans": [], "shape_deps": [],
            "result_claim_deps": [], "owner": {"decl": 0, "activation": None}})
        return i

    def dims(self, i: int) -> list:
        return [d["Lit"] if "Lit" in d else d["Named"][0] for d in self.nodes[i]["output_type"]["dims"]]

    def prec(self, i: int) -> str:
        inv = {v: k for k, v in PRIM.items()}
        return inv[self.nodes[i]["output_type"]["precision"]]

    def json(self) -> str:
        return json.dumps({"nodes": self.nodes, "roots": self.roots,
                           "declarations": [{"name": "entry", "value": False}]},
                          separators=(",", ":"))

    # ---- helpers named after the RiscOps
    def load(self, name, dims, prec="f32"):
        return self.add({"Load": {"name": name}}, [], dims, prec)

    def const(self, value: float, dims=(), prec="f32"):
        sc = f32_scalar(value) if prec == "f32" else f64_scalar(value)
        return self.add({"Const": {"value": sc}}, [], list(dims), prec)

    def binary(self, op, a, b):
        return self.add(op, [a, b], self.dims(a), self.prec(a))

    def unary(self, op, a):
        return self.add(op, [a], self.dims(a), self.prec(a))

    def expand(self, x, axis, size, shape_src=None):
        dims = self.dims(x)
        dims.insert(axis, size)
        rt = lit(size) if shape_src is None else {"InputAxis": {"tensor": 1, "axis": {"Lit": axis}}}
        return self.add({"Expand": {"axis": axis, "size": rt}},
                        [x] if shape_src is None else [x, shape_src], dims, self.prec(x))

    def sum(self, x, axis):
        dims = self.dims(x)
        del dims[axis]
        p = self.prec(x)
        return self.add({"Sum": {"axis": axis, "accumulator": PRIM[p]}}, [x], dims, p)

    def max_reduce(self, x, axis):
        dims = self.dims(x)
        del dims[axis]
        return self.add({"MaxReduce": {"axis": axis}}, [x], dims, self.prec(x))

    def min_reduce(self, x, axis):
        dims = self.dims(x)
        del dims[axis]
        return self.add({"MinReduce": {"axis": axis}}, [x], dims, self.prec(x))

    def arg_reduce(self, op, x, axis):
        """Argmax / Argmin: i64 positions along axis."""
        dims = self.dims(x)
        del dims[axis]
        return self.add({op: {"axis": axis}}, [x], dims, "i64")

    def prod_reduce(self, x, axis):
        dims = self.dims(x)
        del dims[axis]
        return self.add({"ProdReduce": {"axis": axis}}, [x], dims, self.prec(x))

    def classify(self, kind, x):
        """FloatClassify: Nan, Finite or Infinite."""
        return self.add({"FloatClassify": kind}, [x], self.dims(x), "bool")

    def extrema_adjoint(self, kind, operand, a, b, g):
        return self.add({"ExtremaAdjoint": {"kind": kind, "operand": operand}}, [a, b, g],
                        self.dims(a), self.prec(a))

    def key_from_seed(self, seed):
        return self.add("KeyFromSeed", [seed], self.dims(seed), "key")

    def split_key(self, k, branch):
        """Split {branch: Left | Right}: derive(k, 0) or derive(k, 1)."""
        return self.add({"Split": {"branch": branch}}, [k], self.dims(k), "key")

    def fold_in(self, k, n):
        return self.add("FoldIn", [k, n], self.dims(k), "key")

    def split_n(self, k, count):
        return self.add({"SplitN": {"count": {"Concrete": count}}}, [k], self.dims(k) + [count], "key")

    def dropout(self, x, rate, key, replay=False):
        """Dropout / DropoutReplay: inputs [data, rate, key]."""
        return self.add("DropoutReplay" if replay else "Dropout", [x, rate, key], self.dims(x), self.prec(x))

    def cast(self, x, prec):
        return self.add({"Cast": {"new_precision": PRIM[prec]}}, [x], self.dims(x), prec)

    def named_cast(self, x, mode, prec):
        """NamedCast {mode: Trunc | Saturate | Wrap} to a signed integer."""
        return self.add({"NamedCast": {"mode": mode, "new_precision": PRIM[prec]}}, [x], self.dims(x), prec)

    def uniform_like(self, template, low, high, key):
        return self.add("UniformLike", [template, low, high, key], self.dims(template), self.prec(template))

    def compare(self, kind, a, b):
        """Compare(ComparisonKind): kind one of CmpLt, Lt, Eq, Neq, Gt, Gte, Lte."""
        return self.add({"Compare": kind}, [a, b], self.dims(a), "bool")

    def logical(self, kind, a, b=None):
        """Logical(LogicalKind): And, Or (two bool operands) or Not (one)."""
        return self.add({"Logical": kind}, [a] if b is None else [a, b], self.dims(a), "bool")

    def where(self, cond, a, b):
        return self.add("Where", [cond, a, b], self.dims(a), self.prec(a))

    def matmul(self, a, b):
        (m, k), (_, n) = self.dims(a), self.dims(b)
        return self.add({"BlasMatmul": {"batch_dims": [], "m": dim_expr(m), "n": dim_expr(n),
                                        "k": dim_expr(k), "accumulator": PRIM[self.prec(a)]}},
                        [a, b], [m, n], self.prec(a))

    def permute(self, x, axes):
        d = self.dims(x)
        return self.add({"Permute": {"axes": list(axes)}}, [x], [d[a] for a in axes], self.prec(x))

    def reshape(self, x, dims):
        return self.add({"Reshape": {"new_shape": [lit(d) for d in dims]}}, [x], dims, self.prec(x))

    def shrink(self, x, bounds):
        return self.add({"Shrink": {"bounds": [[lit(a), lit(b)] for a, b in bounds]}}, [x],
                        [b - a for a, b in bounds], self.prec(x))

    def stride(self, x, steps):
        d = self.dims(x)
        return self.add({"Stride": {"strides": [lit(s) for s in steps]}}, [x],
                        [(e + s - 1) // s for e, s in zip(d, steps)], self.prec(x))

    def pad(self, x, padding, fill=0.0):
        d = self.dims(x)
        p = self.prec(x)
        sc = f32_scalar(fill) if p == "f32" else f64_scalar(fill)
        return self.add({"Pad": {"padding": [[lit(a), lit(b)] for a, b in padding], "fill": sc}},
                        [x], [e + a + b for e, (a, b) in zip(d, padding)], p)

    def fused(self, ops, inputs, like):
        steps = []
        for op, operands in ops:
            ii = [{"External": o} if isinstance(o, int) else {"PreviousStep": int(o[1:])}
                  for o in operands]
            steps.append({"op": op, "input_indices": ii})
        return self.add({"FusedElem": {"ops": steps}}, inputs, self.dims(like), self.prec(like))


def mlp_step_dag(batch=128, n_in=784, hidden=256, classes=10) -> Dag:
    """Config 1 forward + reverse mode; roots: loss, dW1, db1, dW2, db2.
    Inputs (first-Load order): x, w1, b1, w2, b2, labels."""
    g = Dag()
    x = g.load("x", [batch, n_in])
    w1 = g.load("w1", [n_in, hidden])
    b1 = g.load("b1", [hidden])
    w2 = g.load("w2", [hidden, classes])
    b2 = g.load("b2", [classes])
    labels = g.load("labels", [batch], "i64")
    # forward
    h = g.matmul(x, w1)
    h1 = g.binary("Add", h, g.expand(b1, 0, batch))
    a1 = g.unary("Relu", h1)
    z = g.matmul(a1, w2)
    logits = g.binary("Add", z, g.expand(b2, 0, batch))
    # softmax(logits, 1), expanded after differentiation (decompose_softmax)
    mx = g.max_reduce(logits, 1)
    ex = g.fused([("Sub", (0, 1)), ("Exp", ("p0",))], [logits, g.expand(mx, 1, classes)], logits)
    se = g.sum(ex, 1)
    p = g.binary("Div", ex, g.expand(se, 1, classes))
    lp = g.unary("Log", p)
    sel = g.add({"Gather": {"axis": 1, "batch_rank": 0}}, [lp, labels], [batch, batch])
    t = g.shrink(sel, [(0, batch), (0, batch)])
    t = g.shrink(t, [(0, batch), (0, batch)])
    flat = g.reshape(t, [batch * batch])
    diag = g.stride(flat, [batch + 1])
    nll = g.fused([("Neg", (0,))], [diag], diag)
    total = g.sum(nll, 0)
    loss = g.binary("Div", total, g.const(float(batch)))
    # reverse mode from d loss = 1
    seed = g.const(1.0)
    g_total = g.binary("Div", seed, g.const(float(batch)))
    g_nll = g.expand(g_total, 0, batch, shape_src=nll)
    g_diag = g.unary("Neg", g_nll)
    # Stride adjoint: split, zero-pad the new axis to the step, merge, trim
    split = g.reshape(g_diag, [batch, 1])
    padded = g.pad(split, [(0, 0), (0, batch)])
    merged = g.reshape(padded, [batch * (batch + 1)])
    trimmed = g.shrink(merged, [(0, batch * batch)])
    g_t = g.reshape(trimmed, [batch, batch])
    g_t = g.pad(g_t, [(0, 0), (0, 0)])    # Shrink adjoints (full-extent bounds)
    g_sel = g.pad(g_t, [(0, 0), (0, 0)])
    zero = g.expand(g.expand(g.const(0.0), 0, batch), 1, classes)   # fill_like(lp, 0)
    g_lp = g.add({"ScatterAdd": {"axis": 1, "batch_rank": 0}}, [zero, labels, g_sel],
                 [batch, classes])
    g_p = g.binary("Div", g_lp, p)                                 # Log adjoint
    gy_sum = g.sum(g.fused([("Mul", (0, 1))], [g_p, p], p), 1)     # Softmax adjoint
    bcast = g.expand(gy_sum, 1, classes, shape_src=logits)
    g_logits = g.fused([("Sub", (0, 1)), ("Mul", (2, "p0"))], [g_p, bcast, p], p)
    g_b2 = g.sum(g_logits, 0)                                      # Expand adjoint
    g_a1 = g.matmul(g_logits, g.permute(w2, [1, 0]))               # BlasMatmul adjoints
    g_w2 = g.matmul(g.permute(a1, [1, 0]), g_logits)
    g_h1 = g.add("ReluAdjoint", [h1, g_a1], [batch, hidden])
    g_b1 = g.sum(g_h1, 0)
    g_w1 = g.matmul(g.permute(x, [1, 0]), g_h1)
    g.roots = [loss, g_w1, g_b1, g_w2, g_b2]
    return g
