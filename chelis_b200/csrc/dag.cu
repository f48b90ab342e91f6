// dag.cu -- executes a serialized Chelis DAG on the GPU.
//
// The reference turns a verified DAG into C++ source per program
// (crates/chelis-backend-hip/src/emit.rs: emit_dag :488, the host entry
// :660-800, the device entry :838-958) with a storage plan fixed at compile
// time (src/memory.rs:39-98, MemoryPlan::from_shared: input mirrors, owned
// slots reused after their last use, metadata views, terminal drops, store
// aliases; the peak-bytes figure of src/lib.rs:47-53).  Here the same DAG,
// as the JSON serde writes for crates/chelis-dag-core's `Dag`
// (dag.rs:2364-2400, 2913-2920), is read at run time, checked, planned once
// (placements, slot reuse, arena bytes) and executed node by node with this
// library's kernels:
//
//   Load                  input owner (a view; no copy)
//   Const / ConstTensor   filled slot
//   Add..MinElem, Neg..Round, FusedElem
//                         chelis_cuda_fused_elementwise (one kernel per
//                         node; Expand / Permute / Shrink / Stride views
//                         become per-input strides, stride 0 broadcasts)
//   Sum / MaxReduce       chelis_cuda_fused_reduce; a FusedElem whose one
//                         consumer is the reduction is inlined into it
//                         (fuse.rs:463-500 reduction_inlined_fused_elems)
//   BlasMatmul            chelis_cuda_sgemm / _dgemm; a transposing Permute
//                         view of a dense operand becomes trans_a / trans_b
//   Relu, ReluAdjoint, Softmax (last axis), Count, Cumsum (last axis)
//                         the dedicated kernels
//   Gather, ScatterAdd, Scatter, ScatterElements
//                         index kernels
//   Shape                 a constant (extents are concrete)
//   OrderedAdjointSum     the adjacent-pair tree over List cotangents
//   UniformBoundAdjoint   a bound's pathwise adjoint under the forward key
//   ExtentWitness, CheckedExtent, CheckedUnitAxis
//                         shape contracts, decided when the program is planned
//                         and reported when the node runs ([05-OP-52]; bad indices set the
//                         device error word: "numeric trap: domain in gather")
//   Reshape, Permute, Expand, Shrink, Stride, Store
//                         metadata views (a Reshape of a non-dense view is
//                         materialised first)
//   Pad, Cast, Copy, Realize
//                         materialising kernels;  Drop: nothing
//   Compare, Logical, Where
//                         element-wise kernels over strided operands (the C
//                         lane's C comparisons, bool logic, stored-bit select)
//   MinReduce, Argmax, Argmin
//                         warp per output, the C lane's in-order selection
//                         (first NaN, else the first extreme value)
//   ProdReduce            sequential product per output, in axis order
//   FloatClassify, ExtremaAdjoint
//                         element-wise kernels
//   KeyFromSeed, Split, FoldIn, SplitN (static count)
//                         u64 keys derived element-wise ([05-RNG-2] derive)
//   Dropout, DropoutReplay
//                         keyed draw per key row ([05-OP-37]), the C lane's
//                         word / unit and rate rule
//   UniformLike           keyed affine sampler per key row ([05-OP-8])
//   Iota                  start + i over the declared extent, length checked
//   ReduceWindow, ReduceWindowGrad
//                         thread per output (forward) / per input position
//                         (adjoint), canonical trees in window order
//   Add, Sub, Mul, TruncDiv, FloorDiv, Mod, MaxElem, MinElem, Neg, Abs on
//   integers (and float Mod)
//                         exact at the stored width; overflow / division by
//                         zero recorded as numeric traps on the device
//   GuardedFail           the fallback, and the node's message reported by
//                         chelis_cuda_device_status when the condition fires
//
// Extents may be symbolic (bound per run from the inputs' shapes).  Inputs are
// bound in first-Load order and outputs are the Store nodes then the roots
// (emit.rs:5881-5934).  Outputs come back as new device owners.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <limits>
#include <memory>
#include <mutex>
#include <string>
#include <type_traits>
#include <vector>

#include "chelis_dag.h"
#include "common.cuh"
#include "dag_json.cuh"

namespace chelis {
int dtype_width(chelis_dtype dt);

namespace dag {

constexpr int kMaxRank = 8;

enum class Op {
    Load, Const, ConstTensor, Elementwise, Fused, Relu, ReluAdjoint, Softmax, Sum, MaxReduce,
    Count, Matmul, Gather, ScatterAdd, Cumsum, Reshape, Permute, Expand, Shrink, Stride, Pad, Cast,
    Copy, Drop, Store, Compare, Logical, Where, MinReduce, Argmax, Argmin, ProdReduce,
    FloatClassify, ExtremaAdjoint, KeyFromSeed, SplitKey, FoldIn, SplitN, Dropout, Arith, NamedCast,
    GuardedFail, UniformLike, Iota, ReduceWindow, ReduceWindowGrad, Scatter, ScatterElements, Shape,
    OrderedAdjointSum, UniformBoundAdjoint, ExtentWitness, CheckedExtent
};

constexpr int kMaxAdjointInputs = 64;  // OrderedAdjointSum inputs taken in one launch

// Compare kinds (ComparisonKind order) and Logical kinds (LogicalKind order)
enum { CMP_CMPLT = 0, CMP_LT, CMP_EQ, CMP_NEQ, CMP_GT, CMP_GTE, CMP_LTE };
enum { LOG_AND = 0, LOG_OR, LOG_NOT };
// FloatClassify kinds (dtype_semantics.rs FloatClassify order); ExtremaAdjoint kind
// (Max = 0, Min = 1) and operand (Left = 0, Right = 1) in Node::kind / Node::axis
enum { FC_NAN = 0, FC_FINITE, FC_INFINITE };
// exact integer element-wise operations (and float Mod) in Node::kind
// ReduceWindowKind (dag.rs:587-592 order)
enum { RW_MAX = 0, RW_MIN, RW_SUM, RW_MEAN };
// NamedCast modes (NamedCastMode order)
enum { NC_TRUNC = 0, NC_SATURATE, NC_WRAP };
enum { IA_ADD = 0, IA_SUB, IA_MUL, IA_TRUNC_DIV, IA_FLOOR_DIV, IA_MOD, IA_MAX, IA_MIN, IA_NEG, IA_ABS,
       IA_AND, IA_OR, IA_XOR, IA_SHL, IA_SHR };

struct Node {
    Op op = Op::Drop;
    std::string opname;
    std::vector<int> in;
    chelis_dtype dtype = 0;
    std::vector<int64_t> shape;
    std::vector<chelis_fused_step> steps;  // Elementwise (one step) / Fused
    int axis = 0, batch_rank = 0;
    bool reverse = false;
    std::vector<int> axes;                             // Permute
    std::vector<std::pair<int64_t, int64_t>> bounds;   // Shrink (start, end) / Pad (before, after)
    std::vector<int64_t> step;                         // Stride
    uint64_t bits = 0;                                 // Const / Pad fill value
    std::vector<uint8_t> data;                         // ConstTensor payload
    std::string name;                                  // Load / Store
    int accumulator = -1;                              // Sum / BlasMatmul
    int kind = 0;                                      // Compare / Logical (CMP_* / LOG_*)
    int activation = -1;                               // owner.activation node, if any
    std::string message;                               // GuardedFail
    uint32_t fail_id = 0;                              // its registered message id
    std::vector<int64_t> window, wstride;             // ReduceWindow(Grad)
    std::vector<std::string> dim_names;                // per axis: the unbound name, or ""
    std::vector<std::pair<std::string, bool>> claims;  // ExtentWitness (claim, requirement_declares) /
                                                       // CheckedExtent labels
};

// Static layout of a node's value: elements at root storage + offset +
// sum(coord * stride).
struct Layout {
    int root = -1;  // node owning the storage (a Load, a slot node, or itself)
    int64_t offset = 0;
    std::vector<int64_t> strides;
};

enum class Place { Input, View, Slot, Output, Skip, Inlined };

struct Program {
    std::vector<Node> nodes;
    std::vector<Layout> layout;
    std::vector<Place> place;
    std::vector<int> slot;        // Slot: slot index; Output: output index
    std::vector<int64_t> slot_off;  // byte offset of each slot in the arena
    std::vector<int64_t> slot_cap;
    int64_t arena_bytes = 0;
    int64_t live_peak_bytes = 0;
    std::vector<std::string> input_labels;
    std::vector<int> input_of_load;  // node -> input slot (Loads), -1 otherwise
    std::vector<std::string> output_labels;
    std::vector<int> output_node;    // the node whose value is the output
    std::vector<int> direct_output;  // node -> output index when it writes into the owner
    std::vector<uint32_t> fail_ids;  // registered GuardedFail messages, released with the program
    ~Program() {
        for (uint32_t id : fail_ids) unregister_fail_message(id);
    }
    Program() = default;
    Program(const Program &) = delete;
    Program &operator=(const Program &) = delete;
};

int64_t count_of(const std::vector<int64_t> &shape) {
    int64_t c = 1;
    for (int64_t e : shape) c *= e;
    return c;
}

std::vector<int64_t> dense_strides(const std::vector<int64_t> &shape) {
    std::vector<int64_t> st(shape.size(), 1);
    int64_t run = 1;
    for (int d = static_cast<int>(shape.size()) - 1; d >= 0; --d) {
        st[d] = run;
        run *= shape[d];
    }
    return st;
}

bool is_dense(const std::vector<int64_t> &shape, const std::vector<int64_t> &strides) {
    int64_t run = 1;
    for (int d = static_cast<int>(shape.size()) - 1; d >= 0; --d) {
        if (shape[d] != 1 && strides[d] != run) return false;
        run *= shape[d];
    }
    return true;
}

// ---------------------------------------------------------------- parsing

int bad(const char *what, const std::string &detail = std::string()) {
    return set_error(CHELIS_CUDA_ERR_DOMAIN, "dag: %s%s%s", what, detail.empty() ? "" : ": ",
                     detail.c_str());
}
int unsupported(const std::string &what) {
    return set_error(CHELIS_CUDA_ERR_UNSUPPORTED, "dag: %s is not supported by the CUDA lane",
                     what.c_str());
}

// Prim (crates/chelis-numeric-core/src/prim.rs:14-37, serde variant names)
int prim_dtype(const std::string &p) {
    if (p == "F32") return CHELIS_DTYPE_F32;
    if (p == "F64") return CHELIS_DTYPE_F64;
    if (p == "Int32") return CHELIS_DTYPE_I32;
    if (p == "Bool") return CHELIS_DTYPE_BOOL;
    if (p == "Int64") return CHELIS_DTYPE_I64;
    if (p == "Bf16") return CHELIS_DTYPE_BF16;
    if (p == "F16") return CHELIS_DTYPE_F16;
    if (p == "Int8") return CHELIS_DTYPE_I8;
    if (p == "Int16") return CHELIS_DTYPE_I16;
    if (p == "Key") return CHELIS_DTYPE_KEY;
    return -1;
}
// scalar / tensor payload dtype names (wire_codec.rs: "f32", "int64", ...)
int wire_dtype(const std::string &p) {
    if (p == "f32") return CHELIS_DTYPE_F32;
    if (p == "f64") return CHELIS_DTYPE_F64;
    if (p == "int32") return CHELIS_DTYPE_I32;
    if (p == "bool") return CHELIS_DTYPE_BOOL;
    if (p == "int64") return CHELIS_DTYPE_I64;
    if (p == "bf16") return CHELIS_DTYPE_BF16;
    if (p == "f16") return CHELIS_DTYPE_F16;
    if (p == "int8") return CHELIS_DTYPE_I8;
    if (p == "int16") return CHELIS_DTYPE_I16;
    return -1;
}

bool as_index(const json::Value *v, int64_t *out) {
    if (!v || v->kind != json::Value::Int || v->i < 0) return false;
    *out = v->i;
    return true;
}

// the single key of an externally tagged enum value ({"Lit": 3})
const json::Value *variant(const json::Value &v, const char *name) {
    if (v.kind != json::Value::Obj || v.o.size() != 1 || v.o[0].first != name) return nullptr;
    return &v.o[0].second;
}

// Symbolic extents.  A program is parsed once with every unbound name read
// as 1 (placeholder mode: the ops are checked, the shapes are not), and again
// for each set of bindings its inputs' shapes give, which is checked and
// planned like a static program.
struct SymbolScope {
    const std::vector<std::pair<std::string, int64_t>> *bind = nullptr;
    bool placeholder = false;
    bool saw_symbol = false;
    int placeholders = 0;  // placeholder reads so far
};
thread_local SymbolScope t_sym;

// the extent a name stands for: a binding, the placeholder, or an error
int symbol_extent(const std::string &name, int64_t *out, bool *found) {
    *found = true;
    if (t_sym.bind) {
        for (const auto &b : *t_sym.bind)
            if (b.first == name) {
                *out = b.second;
                return CHELIS_CUDA_OK;
            }
        return bad("missing symbolic dimension binding", "`" + name + "`");
    }
    if (t_sym.placeholder) {
        t_sym.saw_symbol = true;
        ++t_sym.placeholders;
        *out = 1;
        return CHELIS_CUDA_OK;
    }
    *found = false;
    return CHELIS_CUDA_OK;
}

// An extent: DimInfo::Lit(n) / Named(_, Some(n)) / Named(name, None), the
// DimExpr forms Concrete(n), Sym(name), Mul(a, b), Div(a, b) (exact, as
// DimExpr::evaluate, dag.rs:293-317), RtDim::Lit(n) / Sym(name).  *found is
// false for any other form (a runtime bound the caller names).
int extent_expr(const json::Value &v, int64_t *out, bool *found) {
    *found = true;
    if (const json::Value *l = variant(v, "Lit")) return as_index(l, out) ? CHELIS_CUDA_OK : bad("extent literal");
    if (const json::Value *c = variant(v, "Concrete"))
        return as_index(c, out) ? CHELIS_CUDA_OK : bad("extent literal");
    if (const json::Value *nm = variant(v, "Named")) {
        if (nm->kind != json::Value::Arr || nm->a.size() != 2 || nm->a[0].kind != json::Value::Str)
            return bad("Named dimension");
        if (nm->a[1].kind != json::Value::Null)
            return as_index(&nm->a[1], out) ? CHELIS_CUDA_OK : bad("Named dimension size");
        return symbol_extent(nm->a[0].s, out, found);
    }
    if (const json::Value *sy = variant(v, "Sym")) {
        if (sy->kind != json::Value::Str) return bad("Sym dimension");
        return symbol_extent(sy->s, out, found);
    }
    const json::Value *mul = variant(v, "Mul"), *div = variant(v, "Div");
    if (mul || div) {
        const json::Value *ab = mul ? mul : div;
        if (ab->kind != json::Value::Arr || ab->a.size() != 2) return bad("dimension expression");
        int64_t a = 0, b = 0;
        bool fa = false, fb = false;
        const int before = t_sym.placeholders;
        CHELIS_TRY(extent_expr(ab->a[0], &a, &fa));
        CHELIS_TRY(extent_expr(ab->a[1], &b, &fb));
        if (!fa || !fb) {
            *found = false;
            return CHELIS_CUDA_OK;
        }
        if (mul) {
            if (a != 0 && b > std::numeric_limits<int64_t>::max() / a)
                return bad("symbolic dimension product overflowed usize");
            *out = a * b;
        } else {
            if (b == 0) return bad("symbolic dimension expression divided by zero");
            // (a placeholder operand is not its value: the check waits for the binding)
            if (a % b != 0 && t_sym.placeholders == before)
                return bad("symbolic dimension expression is not evenly divisible");
            *out = a / b;
        }
        return CHELIS_CUDA_OK;
    }
    *found = false;
    return CHELIS_CUDA_OK;
}

// an extent, or CHELIS_CUDA_ERR_UNSUPPORTED naming `what` for a runtime form
int extent(const json::Value &v, int64_t *out, const char *what) {
    bool found = false;
    CHELIS_TRY(extent_expr(v, out, &found));
    return found ? CHELIS_CUDA_OK : unsupported(what);
}

int hex_bits(const json::Value *v, size_t digits, uint64_t *out) {
    if (!v || v->kind != json::Value::Str || v->s.size() != digits) return bad("bad hex bits");
    uint64_t b = 0;
    for (char c : v->s) {
        int h = (c >= '0' && c <= '9') ? c - '0' : (c >= 'a' && c <= 'f') ? c - 'a' + 10 : -1;
        if (h < 0) return bad("bad hex bits");
        b = (b << 4) | static_cast<uint64_t>(h);
    }
    *out = b;
    return CHELIS_CUDA_OK;
}

// ScalarValue wire form (wire_codec.rs:488-530): {"dtype": .., "bits"|"value": ..}
int scalar(const json::Value *v, int *dtype, uint64_t *bits) {
    if (!v || v->kind != json::Value::Obj) return bad("scalar payload expected");
    const json::Value *d = v->get("dtype");
    if (!d || d->kind != json::Value::Str || (*dtype = wire_dtype(d->s)) < 0)
        return bad("scalar dtype");
    switch (*dtype) {
        case CHELIS_DTYPE_F64: return hex_bits(v->get("bits"), 16, bits);
        case CHELIS_DTYPE_F32: return hex_bits(v->get("bits"), 8, bits);
        case CHELIS_DTYPE_F16: case CHELIS_DTYPE_BF16: return hex_bits(v->get("bits"), 4, bits);
        case CHELIS_DTYPE_BOOL: {
            const json::Value *b = v->get("value");
            if (!b || b->kind != json::Value::Bool) return bad("bool scalar");
            *bits = b->b ? 1 : 0;
            return CHELIS_CUDA_OK;
        }
        default: {
            const json::Value *i = v->get("value");
            if (!i || i->kind != json::Value::Int) return bad("integer scalar");
            *bits = static_cast<uint64_t>(i->i);
            return CHELIS_CUDA_OK;
        }
    }
}

// TensorStorage wire form: {"dtype": .., "bits": [hex..]} / {"dtype": .., "values": [..]}
int tensor_payload(const json::Value *v, int *dtype, std::vector<uint8_t> *out) {
    if (!v || v->kind != json::Value::Obj) return bad("tensor payload expected");
    const json::Value *d = v->get("dtype");
    if (!d || d->kind != json::Value::Str || (*dtype = wire_dtype(d->s)) < 0)
        return bad("tensor payload dtype");
    const int w = dtype_width(static_cast<chelis_dtype>(*dtype));
    const bool floaty = *dtype == CHELIS_DTYPE_F32 || *dtype == CHELIS_DTYPE_F64 ||
                        *dtype == CHELIS_DTYPE_F16 || *dtype == CHELIS_DTYPE_BF16;
    const json::Value *arr = v->get(floaty ? "bits" : "values");
    if (!arr || arr->kind != json::Value::Arr) return bad("tensor payload values");
    out->resize(arr->a.size() * static_cast<size_t>(w));
    for (size_t i = 0; i < arr->a.size(); ++i) {
        uint64_t b = 0;
        if (floaty) {
            CHELIS_TRY(hex_bits(&arr->a[i], static_cast<size_t>(2 * w), &b));
        } else if (*dtype == CHELIS_DTYPE_BOOL) {
            if (arr->a[i].kind != json::Value::Bool) return bad("bool payload");
            b = arr->a[i].b;
        } else {
            if (arr->a[i].kind != json::Value::Int) return bad("integer payload");
            b = static_cast<uint64_t>(arr->a[i].i);
        }
        std::memcpy(out->data() + i * w, &b, static_cast<size_t>(w));  // little-endian low bytes
    }
    return CHELIS_CUDA_OK;
}

bool integer_dtype(int dt) {
    return dt == CHELIS_DTYPE_I8 || dt == CHELIS_DTYPE_I16 || dt == CHELIS_DTYPE_I32 || dt == CHELIS_DTYPE_I64;
}

// the RiscOps that run as exact integer arithmetic at the stored width
int arith_code(const std::string &n) {
    static const char *names[] = {"Add", "Sub", "Mul", "TruncDiv", "FloorDiv", "Mod", "MaxElem", "MinElem",
                                  "Neg", "Abs"};
    for (int i = 0; i < 10; ++i)
        if (n == names[i]) return i;
    return -1;
}

// FusedStepOp (dag.rs:494-526) / binary and unary RiscOps -> step code
int fused_code(const std::string &n) {
    static const char *names[] = {"Add", "Sub", "Mul", "Div", "Pow", "FloorDiv", "TruncDiv",
                                  "MaxElem", "MinElem", "Neg", "Recip", "Exp", "Log", "Sin",
                                  "Sqrt", "Cos", "Tan", "Atan", "Tanh", "Erf", "Erfc", "Abs",
                                  "Floor", "Ceil", "Round"};
    for (int i = 0; i < 25; ++i)
        if (n == names[i]) return i;
    return -1;
}

int fused_operand(const json::Value &v, int32_t *out) {
    int64_t i = 0;
    if (const json::Value *e = variant(v, "External")) {
        if (!as_index(e, &i)) return bad("fused operand");
        *out = static_cast<int32_t>(i);
        return CHELIS_CUDA_OK;
    }
    if (const json::Value *p = variant(v, "PreviousStep")) {
        if (!as_index(p, &i)) return bad("fused operand");
        *out = -1 - static_cast<int32_t>(i);
        return CHELIS_CUDA_OK;
    }
    return bad("fused operand");
}

int axis_list(const json::Value *v, std::vector<int> *out) {
    if (!v || v->kind != json::Value::Arr) return bad("axis list");
    for (const auto &e : v->a) {
        int64_t a = 0;
        if (!as_index(&e, &a)) return bad("axis list");
        out->push_back(static_cast<int>(a));
    }
    return CHELIS_CUDA_OK;
}

int bound_pairs(const json::Value *v, std::vector<std::pair<int64_t, int64_t>> *out,
                const std::vector<int64_t> &input_shape, bool shrink) {
    if (!v || v->kind != json::Value::Arr) return bad("bounds");
    for (size_t d = 0; d < v->a.size(); ++d) {
        const json::Value &p = v->a[d];
        if (p.kind != json::Value::Arr || p.a.size() != 2) return bad("bounds");
        int64_t lo = 0, hi = 0;
        CHELIS_TRY(extent(p.a[0], &lo, "a runtime bound"));
        if (shrink && p.a[1].kind == json::Value::Str && p.a[1].s == "ToEnd") {
            if (d >= input_shape.size()) return bad("bounds rank");
            hi = input_shape[d];
        } else {
            CHELIS_TRY(extent(p.a[1], &hi, "a runtime bound"));
        }
        out->emplace_back(lo, hi);
    }
    return CHELIS_CUDA_OK;
}

int parse_node(const json::Value &jn, size_t index, std::vector<Node> &nodes) {
    Node n;
    int64_t id = -1;
    if (!as_index(jn.get("id"), &id) || id != static_cast<int64_t>(index))
        return bad("node ids must be 0..n-1 in order");
    const json::Value *inputs = jn.get("inputs");
    if (!inputs || inputs->kind != json::Value::Arr) return bad("node inputs");
    for (const auto &e : inputs->a) {
        int64_t i = 0;
        if (!as_index(&e, &i) || i >= id) return bad("inputs must name earlier nodes");
        n.in.push_back(static_cast<int>(i));
    }
    const json::Value *ty = jn.get("output_type");
    const json::Value *dims = ty ? ty->get("dims") : nullptr;
    const json::Value *prec = ty ? ty->get("precision") : nullptr;
    if (!dims || dims->kind != json::Value::Arr || !prec || prec->kind != json::Value::Str)
        return bad("output_type");
    const int dt = prim_dtype(prec->s);
    if (dt < 0) return unsupported("precision " + prec->s);
    if (const json::Value *own = jn.get("owner")) {
        const json::Value *act = own->get("activation");
        int64_t a = 0;
        if (act && act->kind != json::Value::Null) {
            if (!as_index(act, &a) || a >= id) return bad("owner activation");
            n.activation = static_cast<int>(a);
        }
    }
    n.dtype = static_cast<chelis_dtype>(dt);
    for (const auto &d : dims->a) {
        int64_t e = 0;
        CHELIS_TRY(extent(d, &e, "a runtime extent"));
        n.shape.push_back(e);
        const json::Value *nm = variant(d, "Named");
        n.dim_names.push_back(nm && nm->kind == json::Value::Arr && nm->a.size() == 2 &&
                                      nm->a[1].kind == json::Value::Null
                                  ? nm->a[0].s
                                  : std::string());
    }
    if (n.shape.size() > static_cast<size_t>(kMaxRank)) return unsupported("rank above 8");

    const json::Value *op = jn.get("op");
    if (!op) return bad("node op");
    std::string name;
    const json::Value *body = nullptr;
    if (op->kind == json::Value::Str) {
        name = op->s;
    } else if (op->kind == json::Value::Obj && op->o.size() == 1) {
        name = op->o[0].first;
        body = &op->o[0].second;
    } else {
        return bad("node op");
    }
    n.opname = name;
    auto in_shape = [&](int k) -> const std::vector<int64_t> & { return nodes[n.in[k]].shape; };
    auto need_inputs = [&](size_t k) {
        return n.in.size() == k ? CHELIS_CUDA_OK : bad("wrong input count for", name);
    };
    auto field = [&](const char *f) -> const json::Value * { return body ? body->get(f) : nullptr; };
    int64_t v = 0;
    const int code = fused_code(name);
    if (name == "Load") {
        n.op = Op::Load;
        const json::Value *nm = field("name");
        if (!nm || nm->kind != json::Value::Str) return bad("Load name");
        n.name = nm->s;
        CHELIS_TRY(need_inputs(0));
    } else if (name == "Store") {
        n.op = Op::Store;
        const json::Value *nm = field("name");
        if (!nm || nm->kind != json::Value::Str) return bad("Store name");
        n.name = nm->s;
        CHELIS_TRY(need_inputs(1));
    } else if (name == "Const") {
        n.op = Op::Const;
        int sdt = 0;
        CHELIS_TRY(scalar(field("value"), &sdt, &n.bits));
        if (sdt != n.dtype) return bad("Const value dtype differs from the node's precision");
    } else if (name == "ConstTensor") {
        n.op = Op::ConstTensor;
        int sdt = 0;
        CHELIS_TRY(tensor_payload(field("data"), &sdt, &n.data));
        if (sdt != n.dtype ||
            static_cast<int64_t>(n.data.size()) != count_of(n.shape) * dtype_width(n.dtype))
            return bad("ConstTensor payload does not match the node's type");
    } else if (name == "Bitwise") {
        // [05-OP-47] BitwiseKind: And, Or, Xor, ShiftLeft, ShiftRight
        static const char *kinds[] = {"And", "Or", "Xor", "ShiftLeft", "ShiftRight"};
        n.op = Op::Arith;
        n.kind = -1;
        if (body && body->kind == json::Value::Str)
            for (int i = 0; i < 5; ++i)
                if (body->s == kinds[i]) n.kind = IA_AND + i;
        if (n.kind < 0) return bad("Bitwise kind");
        if (!integer_dtype(n.dtype)) return bad("Bitwise operands must be integers");
        CHELIS_TRY(need_inputs(2));
    } else if (arith_code(name) >= 0 && (integer_dtype(n.dtype) || name == "Mod")) {
        // integer arithmetic checked at the stored width ([04-NUM-9]); float Mod is C fmod ([05-OP-64])
        n.op = Op::Arith;
        n.kind = arith_code(name);
        CHELIS_TRY(need_inputs(n.kind == IA_NEG || n.kind == IA_ABS ? 1 : 2));
    } else if (code >= 0 && name != "TruncDiv") {
        n.op = Op::Elementwise;
        const bool binary = code <= CHELIS_FUSED_MIN_ELEM;
        CHELIS_TRY(need_inputs(binary ? 2 : 1));
        n.steps.push_back({code, 0, binary ? 1 : 0});
    } else if (name == "FusedElem") {
        n.op = Op::Fused;
        const json::Value *ops = field("ops");
        if (!ops || ops->kind != json::Value::Arr || ops->a.empty()) return bad("FusedElem ops");
        for (const auto &st : ops->a) {
            const json::Value *o = st.get("op");
            const json::Value *ii = st.get("input_indices");
            if (!o || o->kind != json::Value::Str || !ii || ii->kind != json::Value::Arr ||
                ii->a.empty())
                return bad("FusedElem step");
            chelis_fused_step s{fused_code(o->s), 0, 0};
            if (s.op < 0) return bad("FusedElem step op", o->s);
            CHELIS_TRY(fused_operand(ii->a[0], &s.a));
            s.b = s.a;
            if (ii->a.size() > 1) CHELIS_TRY(fused_operand(ii->a[1], &s.b));
            n.steps.push_back(s);
        }
    } else if (name == "Relu") {
        n.op = Op::Relu;
        CHELIS_TRY(need_inputs(1));
    } else if (name == "ReluAdjoint") {
        n.op = Op::ReluAdjoint;
        CHELIS_TRY(need_inputs(2));
    } else if (name == "Softmax") {
        n.op = Op::Softmax;
        CHELIS_TRY(need_inputs(1));
        if (!as_index(field("axis"), &v)) return bad("Softmax axis");
        n.axis = static_cast<int>(v);
    } else if (name == "Sum" || name == "MaxReduce") {
        n.op = name == "Sum" ? Op::Sum : Op::MaxReduce;
        CHELIS_TRY(need_inputs(1));
        if (!as_index(field("axis"), &v)) return bad("reduction axis");
        n.axis = static_cast<int>(v);
        if (n.op == Op::Sum) {
            const json::Value *acc = field("accumulator");
            if (!acc || acc->kind != json::Value::Str || prim_dtype(acc->s) < 0)
                return bad("Sum accumulator");
            n.accumulator = prim_dtype(acc->s);
        }
    } else if (name == "Compare") {
        // ComparisonKind (dag.rs:528-536), in declaration order
        static const char *kinds[] = {"CmpLt", "Lt", "Eq", "Neq", "Gt", "Gte", "Lte"};
        n.op = Op::Compare;
        n.kind = -1;
        if (body && body->kind == json::Value::Str)
            for (int i = 0; i < 7; ++i)
                if (body->s == kinds[i]) n.kind = i;
        if (n.kind < 0) return bad("Compare kind");
        CHELIS_TRY(need_inputs(2));
    } else if (name == "Logical") {
        // LogicalKind (dag.rs:555-559)
        static const char *kinds[] = {"And", "Or", "Not"};
        n.op = Op::Logical;
        n.kind = -1;
        if (body && body->kind == json::Value::Str)
            for (int i = 0; i < 3; ++i)
                if (body->s == kinds[i]) n.kind = i;
        if (n.kind < 0) return bad("Logical kind");
        CHELIS_TRY(need_inputs(n.kind == LOG_NOT ? 1 : 2));
    } else if (name == "Where") {
        n.op = Op::Where;
        CHELIS_TRY(need_inputs(3));
    } else if (name == "MinReduce" || name == "Argmax" || name == "Argmin" || name == "ProdReduce") {
        n.op = name == "MinReduce" ? Op::MinReduce
               : name == "Argmax" ? Op::Argmax
               : name == "Argmin" ? Op::Argmin
                                  : Op::ProdReduce;
        CHELIS_TRY(need_inputs(1));
        if (!as_index(field("axis"), &v)) return bad("reduction axis");
        n.axis = static_cast<int>(v);
    } else if (name == "FloatClassify") {
        static const char *kinds[] = {"Nan", "Finite", "Infinite"};
        n.op = Op::FloatClassify;
        n.kind = -1;
        if (body && body->kind == json::Value::Str)
            for (int i = 0; i < 3; ++i)
                if (body->s == kinds[i]) n.kind = i;
        if (n.kind < 0) return bad("FloatClassify kind");
        CHELIS_TRY(need_inputs(1));
    } else if (name == "ExtremaAdjoint") {
        n.op = Op::ExtremaAdjoint;
        const json::Value *k = field("kind"), *o = field("operand");
        if (!k || k->kind != json::Value::Str || (k->s != "Max" && k->s != "Min") || !o ||
            o->kind != json::Value::Str || (o->s != "Left" && o->s != "Right"))
            return bad("ExtremaAdjoint kind / operand");
        n.kind = k->s == "Max" ? 0 : 1;
        n.axis = o->s == "Left" ? 0 : 1;
        CHELIS_TRY(need_inputs(3));
    } else if (name == "KeyFromSeed" || name == "FoldIn") {
        // [05-OP-69] key_from_seed, [05-OP-72] fold_in
        n.op = name == "KeyFromSeed" ? Op::KeyFromSeed : Op::FoldIn;
        CHELIS_TRY(need_inputs(n.op == Op::KeyFromSeed ? 1 : 2));
    } else if (name == "Split") {
        // one half of [05-OP-70] split_key: derive(k, 0) (Left) or derive(k, 1) (Right)
        n.op = Op::SplitKey;
        const json::Value *b = field("branch");
        if (!b || b->kind != json::Value::Str || (b->s != "Left" && b->s != "Right"))
            return bad("Split branch");
        n.kind = b->s == "Left" ? 0 : 1;
        CHELIS_TRY(need_inputs(1));
    } else if (name == "SplitN") {
        // [05-OP-71] split_keys with a static count: row j = derive(derive(k, 2), j)
        n.op = Op::SplitN;
        const json::Value *c = field("count");
        const json::Value *cc = c ? variant(*c, "Concrete") : nullptr;
        if (!cc || !as_index(cc, &v)) return unsupported("SplitN with a runtime count");
        n.axis = static_cast<int>(v);
        CHELIS_TRY(need_inputs(1));
    } else if (name == "ReduceWindow" || name == "ReduceWindowGrad") {
        // [05-OP-39] windowed reductions over the trailing axes (spec 05 2.3.1)
        static const char *kinds[] = {"Max", "Min", "Sum", "Mean"};
        n.op = name == "ReduceWindow" ? Op::ReduceWindow : Op::ReduceWindowGrad;
        const json::Value *r = field("reducer"), *w = field("window_shape"), *st = field("strides");
        n.kind = -1;
        if (r && r->kind == json::Value::Str)
            for (int i = 0; i < 4; ++i)
                if (r->s == kinds[i]) n.kind = i;
        if (n.kind < 0) return bad("ReduceWindow reducer");
        if (!w || w->kind != json::Value::Arr || !st || st->kind != json::Value::Arr || w->a.empty() ||
            w->a.size() != st->a.size())
            return bad("ReduceWindow window_shape / strides ([05-RWIN-1])");
        for (size_t k = 0; k < w->a.size(); ++k) {
            int64_t a = 0, b = 0;
            if (!as_index(&w->a[k], &a) || !as_index(&st->a[k], &b) || a < 1 || b < 1)
                return bad("ReduceWindow window_shape / strides ([05-RWIN-1])");
            n.window.push_back(a);
            n.wstride.push_back(b);
        }
        CHELIS_TRY(need_inputs(n.op == Op::ReduceWindow ? 1 : 2));
    } else if (name == "Shape") {
        // a scalar read of one input extent; the input's values are never read
        n.op = Op::Shape;
        CHELIS_TRY(need_inputs(1));
        if (!as_index(field("axis"), &v)) return bad("Shape axis");
        n.axis = static_cast<int>(v);
    } else if (name == "ExtentWitness" || name == "CheckedExtent") {
        // shape contracts (dag.rs:1236-1275): an observed extent checked
        // against literal requirements and other witnesses, as a scalar i64
        n.op = name == "ExtentWitness" ? Op::ExtentWitness : Op::CheckedExtent;
        const json::Value *ax = field("axis");
        const json::Value *axl = ax ? variant(*ax, "Lit") : nullptr;
        if (!axl || !as_index(axl, &v)) return bad("shape contract axis", name);
        n.axis = static_cast<int>(v);
        const json::Value *cl = field("claims");
        if (!cl || cl->kind != json::Value::Arr) return bad("shape contract claims", name);
        if (n.op == Op::ExtentWitness) {
            static const char *sites[] = {"LiteralResultClaim", "Caller", "LocalExpand", "ResultClaim",
                                          "LocalAscriptionClaim"};
            const json::Value *st = field("site");
            n.kind = -1;
            for (int k = 0; k < 5 && st; ++k)
                if ((st->kind == json::Value::Str && st->s == sites[k]) ||
                    (st->kind == json::Value::Obj && st->o.size() == 1 && st->o[0].first == sites[k]))
                    n.kind = k;
            if (n.kind < 0) return bad("ExtentWitness site");
            const json::Value *pm = field("parameter");
            if (!pm || pm->kind != json::Value::Str) return bad("ExtentWitness parameter");
            n.name = pm->s;
            const json::Value *rq = field("requirements");
            if (!rq || rq->kind != json::Value::Arr) return bad("ExtentWitness requirements");
            for (const auto &r : rq->a) {
                int sdt = 0;
                uint64_t bits = 0;
                CHELIS_TRY(scalar(&r, &sdt, &bits));
                if (sdt != CHELIS_DTYPE_I64) return bad("extent witness requires i64");
                n.window.push_back(static_cast<int64_t>(bits));
            }
            for (const auto &c : cl->a) {
                const json::Value *cn = c.get("claim"), *rd = c.get("requirement_declares");
                if (!cn || cn->kind != json::Value::Str || !rd || rd->kind != json::Value::Bool)
                    return bad("ExtentWitness claim");
                n.claims.emplace_back(cn->s, rd->b);
            }
            if (n.in.size() != 1 + n.claims.size()) return bad("wrong input count for", name);
        } else {
            const json::Value *ow = field("owner");
            if (!ow || ow->kind != json::Value::Str || (ow->s != "reshape" && ow->s != "concat"))
                return bad("CheckedExtent owner");
            n.name = ow->s;
            for (const auto &c : cl->a) {
                if (c.kind != json::Value::Str) return bad("CheckedExtent claim");
                n.claims.emplace_back(c.s, false);
            }
            if (n.in.size() != 1 + n.claims.size()) return bad("wrong input count for", name);
        }
    } else if (name == "CheckedUnitAxis") {
        // the tensor with one axis refined to 1 after its witness: a view
        n.op = Op::Reshape;
        CHELIS_TRY(need_inputs(2));
        const json::Value *ax = field("axis");
        const json::Value *axl = ax ? variant(*ax, "Lit") : nullptr;
        if (!axl || !as_index(axl, &v)) return bad("CheckedUnitAxis axis");
        n.axis = static_cast<int>(v);
    } else if (name == "OrderedAdjointSum") {
        // spec/06 2.4: the adjacent-pair tree over queued List cotangent
        // contributions; `groups` gives each group's input count
        n.op = Op::OrderedAdjointSum;
        const json::Value *gr = field("groups");
        if (!gr || gr->kind != json::Value::Arr) return bad("OrderedAdjointSum groups");
        size_t total = 0;
        for (const auto &e : gr->a) {
            if (!as_index(&e, &v) || v < 1) return bad("OrderedAdjointSum group width");
            n.window.push_back(v);
            total += static_cast<size_t>(v);
        }
        CHELIS_TRY(need_inputs(total));
    } else if (name == "UniformBoundAdjoint") {
        // [05-OP-8] inputs [template, g, key]; the bound's pathwise adjoint
        n.op = Op::UniformBoundAdjoint;
        const json::Value *b = field("bound");
        n.kind = -1;
        if (b && b->kind == json::Value::Str) n.kind = b->s == "Low" ? 0 : b->s == "High" ? 1 : -1;
        if (n.kind < 0) return bad("UniformBoundAdjoint bound");
        CHELIS_TRY(need_inputs(3));
    } else if (name == "Iota") {
        // [05-OP-54] range(start, end) as a rank-one i64 tensor
        n.op = Op::Iota;
        CHELIS_TRY(need_inputs(2));
    } else if (name == "UniformLike") {
        // [05-OP-8] under an explicit key: inputs [template, low, high, key]
        n.op = Op::UniformLike;
        CHELIS_TRY(need_inputs(4));
    } else if (name == "Dropout" || name == "DropoutReplay") {
        // [05-OP-37] under an explicit key; the replay applies the same draw to the cotangent
        n.op = Op::Dropout;
        CHELIS_TRY(need_inputs(3));
    } else if (name == "Count") {
        n.op = Op::Count;
        CHELIS_TRY(need_inputs(1));
        CHELIS_TRY(axis_list(field("axes"), &n.axes));
    } else if (name == "BlasMatmul") {
        n.op = Op::Matmul;
        CHELIS_TRY(need_inputs(2));
        const json::Value *acc = field("accumulator");
        if (!acc || acc->kind != json::Value::Str || prim_dtype(acc->s) < 0)
            return bad("BlasMatmul accumulator");
        n.accumulator = prim_dtype(acc->s);
    } else if (name == "ScatterElements") {
        // element-wise replace-scatter (ONNX ScatterElements; spec 05 3.5.1)
        n.op = Op::ScatterElements;
        CHELIS_TRY(need_inputs(3));
        if (!as_index(field("axis"), &v)) return bad("ScatterElements axis");
        n.axis = static_cast<int>(v);
    } else if (name == "Gather" || name == "ScatterAdd" || name == "Scatter") {
        n.op = name == "Gather" ? Op::Gather : name == "ScatterAdd" ? Op::ScatterAdd : Op::Scatter;
        CHELIS_TRY(need_inputs(n.op == Op::Gather ? 2 : 3));
        int64_t br = 0;
        if (!as_index(field("axis"), &v) || !as_index(field("batch_rank"), &br))
            return bad("Gather / ScatterAdd fields");
        n.axis = static_cast<int>(v);
        n.batch_rank = static_cast<int>(br);
    } else if (name == "Cumsum") {
        n.op = Op::Cumsum;
        CHELIS_TRY(need_inputs(1));
        const json::Value *dir = field("direction");
        if (!as_index(field("axis"), &v) || !dir || dir->kind != json::Value::Str)
            return bad("Cumsum fields");
        n.axis = static_cast<int>(v);
        if (dir->s != "Increasing" && dir->s != "Decreasing") return bad("Cumsum direction");
        n.reverse = dir->s == "Decreasing";
    } else if (name == "Reshape") {
        n.op = Op::Reshape;
        if (n.in.empty()) return bad("Reshape input");
    } else if (name == "Permute") {
        n.op = Op::Permute;
        CHELIS_TRY(need_inputs(1));
        CHELIS_TRY(axis_list(field("axes"), &n.axes));
    } else if (name == "Expand") {
        n.op = Op::Expand;
        if (n.in.empty()) return bad("Expand input");
        if (!as_index(field("axis"), &v)) return bad("Expand axis");
        n.axis = static_cast<int>(v);
    } else if (name == "Shrink") {
        n.op = Op::Shrink;
        if (n.in.empty()) return bad("Shrink input");
        CHELIS_TRY(bound_pairs(field("bounds"), &n.bounds, in_shape(0), true));
    } else if (name == "Stride") {
        n.op = Op::Stride;
        if (n.in.empty()) return bad("Stride input");
        const json::Value *st = field("strides");
        if (!st || st->kind != json::Value::Arr) return bad("Stride strides");
        for (const auto &e : st->a) {
            int64_t s = 0;
            CHELIS_TRY(extent(e, &s, "a runtime stride"));
            if (s < 1) return bad("Stride step below 1");
            n.step.push_back(s);
        }
    } else if (name == "Pad") {
        n.op = Op::Pad;
        if (n.in.empty()) return bad("Pad input");
        CHELIS_TRY(bound_pairs(field("padding"), &n.bounds, in_shape(0), false));
        int fdt = 0;
        CHELIS_TRY(scalar(field("fill"), &fdt, &n.bits));
        if (fdt != n.dtype) return bad("Pad fill dtype");
    } else if (name == "GuardedFail") {
        // [05-OP-68]: abort with `message` where the condition fires
        // (true when trap_on_true, else false); the result is the fallback
        n.op = Op::GuardedFail;
        const json::Value *m = field("message"), *t = field("trap_on_true");
        if (!m || m->kind != json::Value::Str || !t || t->kind != json::Value::Bool)
            return bad("GuardedFail message / trap_on_true");
        n.message = m->s;
        n.kind = t->b ? 1 : 0;
        CHELIS_TRY(need_inputs(2));
    } else if (name == "NamedCast") {
        // cast_trunc [05-OP-6], cast_saturate [05-OP-23], cast_wrap [05-OP-24]
        static const char *modes[] = {"Trunc", "Saturate", "Wrap"};
        n.op = Op::NamedCast;
        const json::Value *m = field("mode");
        n.kind = -1;
        if (m && m->kind == json::Value::Str)
            for (int i = 0; i < 3; ++i)
                if (m->s == modes[i]) n.kind = i;
        if (n.kind < 0) return bad("NamedCast mode");
        CHELIS_TRY(need_inputs(1));
    } else if (name == "Cast") {
        n.op = Op::Cast;
        CHELIS_TRY(need_inputs(1));
    } else if (name == "Copy" || name == "Realize") {
        n.op = Op::Copy;
        CHELIS_TRY(need_inputs(1));
    } else if (name == "Drop") {
        n.op = Op::Drop;
    } else {
        return unsupported("RiscOp::" + name);
    }
    nodes.push_back(std::move(n));
    return CHELIS_CUDA_OK;
}

// ---------------------------------------------------------------- checking

bool floating_dtype(int dt) {
    return dt == CHELIS_DTYPE_F32 || dt == CHELIS_DTYPE_F64 || dt == CHELIS_DTYPE_BF16 ||
           dt == CHELIS_DTYPE_F16;
}

int check_same_shape(const Node &n, const Node &src, const char *what) {
    if (src.shape != n.shape) return bad(what, "operand shape differs from the node's");
    return CHELIS_CUDA_OK;
}

// Shapes and dtypes of each node against its operands; layouts of views.
// an i64 scalar whose value the plan knows: a Const, a Shape read or a
// decided shape contract
bool host_extent(const Node &n, int64_t *out) {
    if (n.dtype != CHELIS_DTYPE_I64 || !n.shape.empty()) return false;
    if (n.op != Op::Const && n.op != Op::Shape && n.op != Op::ExtentWitness && n.op != Op::CheckedExtent)
        return false;
    *out = static_cast<int64_t>(n.bits);
    return true;
}

int check_and_layout(Program &P) {
    std::vector<Node> &N = P.nodes;
    const int count = static_cast<int>(N.size());
    P.layout.assign(count, Layout());
    for (int i = 0; i < count; ++i) {
        Node &n = N[i];
        Layout &L = P.layout[i];
        auto src = [&](int k) -> const Node & { return N[n.in[k]]; };
        auto own = [&] {
            L.root = i;
            L.offset = 0;
            L.strides = dense_strides(n.shape);
        };
        const bool floating = n.dtype == CHELIS_DTYPE_F32 || n.dtype == CHELIS_DTYPE_F64;
        switch (n.op) {
            case Op::Load: case Op::Const: case Op::ConstTensor: case Op::Drop: own(); break;
            case Op::Elementwise: case Op::Fused:
                if (!floating) return unsupported(n.opname + " on a non-float precision");
                for (size_t k = 0; k < n.in.size(); ++k) {
                    if (src(k).dtype != n.dtype) return bad("elementwise operand dtype", n.opname);
                    CHELIS_TRY(check_same_shape(n, src(k), n.opname.c_str()));
                }
                for (const auto &s : n.steps)
                    if ((s.a >= 0 && s.a >= static_cast<int>(n.in.size())) ||
                        (s.b >= 0 && s.b >= static_cast<int>(n.in.size())))
                        return bad("FusedElem operand out of range");
                own();
                break;
            case Op::Relu: case Op::Softmax: case Op::Cumsum:
                if (!floating || src(0).dtype != n.dtype) return unsupported(n.opname + " precision");
                CHELIS_TRY(check_same_shape(n, src(0), n.opname.c_str()));
                if (n.op == Op::Softmax && (n.shape.empty() || n.axis != static_cast<int>(n.shape.size()) - 1))
                    return unsupported(n.opname + " along a non-last axis");
                if (n.op == Op::Cumsum && (n.shape.empty() || n.axis >= static_cast<int>(n.shape.size())))
                    return bad("Cumsum axis");
                if (n.op == Op::Softmax && n.dtype != CHELIS_DTYPE_F32)
                    return unsupported("Softmax at f64");
                own();
                break;
            case Op::ReluAdjoint:
                if (!floating || src(0).dtype != n.dtype || src(1).dtype != n.dtype)
                    return unsupported("ReluAdjoint precision");
                CHELIS_TRY(check_same_shape(n, src(0), "ReluAdjoint"));
                CHELIS_TRY(check_same_shape(n, src(1), "ReluAdjoint"));
                own();
                break;
            case Op::Sum: case Op::MaxReduce: {
                const auto &xs = src(0).shape;
                if (!floating || src(0).dtype != n.dtype) return unsupported(n.opname + " precision");
                if (n.op == Op::Sum && n.accumulator != n.dtype)
                    return unsupported("Sum with a wider accumulator");
                if (n.axis >= static_cast<int>(xs.size())) return bad("reduction axis out of range");
                std::vector<int64_t> want = xs;
                want.erase(want.begin() + n.axis);
                if (want != n.shape) return bad("reduction result shape");
                own();
                break;
            }
            case Op::Compare: {
                // [05-OP-36]: two operands of one dtype and shape, a bool result;
                // bool admits only eq / neq
                const int dt = src(0).dtype;
                if (src(1).dtype != dt) return bad("Compare operand dtypes differ");
                if (n.dtype != CHELIS_DTYPE_BOOL) return bad("Compare result must be bool");
                if (dt == CHELIS_DTYPE_BOOL && n.kind != CMP_EQ && n.kind != CMP_NEQ)
                    return bad("ordered comparison of bool");
                if (dt == CHELIS_DTYPE_KEY) return unsupported("Compare of keys");
                CHELIS_TRY(check_same_shape(n, src(0), "Compare"));
                CHELIS_TRY(check_same_shape(n, src(1), "Compare"));
                own();
                break;
            }
            case Op::Logical:
                // [05-OP-26..28]: bool operands only
                for (size_t k = 0; k < n.in.size(); ++k) {
                    if (src(static_cast<int>(k)).dtype != CHELIS_DTYPE_BOOL)
                        return bad("Logical operand must be bool");
                    CHELIS_TRY(check_same_shape(n, src(static_cast<int>(k)), "Logical"));
                }
                if (n.dtype != CHELIS_DTYPE_BOOL) return bad("Logical result must be bool");
                own();
                break;
            case Op::Where:
                // a bool condition selecting between two values of the result's dtype
                if (src(0).dtype != CHELIS_DTYPE_BOOL) return bad("Where condition must be bool");
                if (src(1).dtype != n.dtype || src(2).dtype != n.dtype) return bad("Where value dtype");
                if (n.dtype == CHELIS_DTYPE_KEY) return unsupported("Where of keys");
                for (int k = 0; k < 3; ++k) CHELIS_TRY(check_same_shape(n, src(k), "Where"));
                own();
                break;
            case Op::MinReduce: case Op::Argmax: case Op::Argmin: case Op::ProdReduce: {
                const auto &xs = src(0).shape;
                const int dt = src(0).dtype;
                const bool arg = n.op == Op::Argmax || n.op == Op::Argmin;
                if (arg ? n.dtype != CHELIS_DTYPE_I64 : dt != n.dtype)
                    return bad("reduction result dtype", n.opname);
                if (dt != CHELIS_DTYPE_F32 && dt != CHELIS_DTYPE_F64 && dt != CHELIS_DTYPE_I32 &&
                    dt != CHELIS_DTYPE_I64)
                    return unsupported(n.opname + " precision");
                if (n.axis >= static_cast<int>(xs.size())) return bad("reduction axis out of range");
                std::vector<int64_t> want = xs;
                want.erase(want.begin() + n.axis);
                if (want != n.shape) return bad("reduction result shape");
                own();
                break;
            }
            case Op::KeyFromSeed: case Op::SplitKey: case Op::FoldIn: case Op::SplitN: {
                if (n.activation >= 0) return unsupported(n.opname + " under an activation");
                const bool seed = n.op == Op::KeyFromSeed;
                if (src(0).dtype != (seed ? CHELIS_DTYPE_I64 : CHELIS_DTYPE_KEY))
                    return bad(seed ? "KeyFromSeed seed must be i64" : "key operand must be a key");
                if (n.dtype != CHELIS_DTYPE_KEY) return bad("key operation result must be a key");
                if (n.op == Op::FoldIn) {
                    if (src(1).dtype != CHELIS_DTYPE_I64) return bad("FoldIn data must be i64");
                    CHELIS_TRY(check_same_shape(n, src(1), "FoldIn"));
                }
                if (n.op == Op::SplitN) {
                    std::vector<int64_t> want = src(0).shape;
                    want.push_back(n.axis);
                    if (want != n.shape) return bad("SplitN result shape");
                } else {
                    CHELIS_TRY(check_same_shape(n, src(0), n.opname.c_str()));
                }
                own();
                break;
            }
            case Op::ReduceWindow: case Op::ReduceWindowGrad: {
                const Node &x = src(0);
                const size_t r = x.shape.size(), nw = n.window.size();
                if (nw > r) return bad("ReduceWindow window arity above the input rank ([05-RWIN-1])");
                if (x.dtype != n.dtype) return bad("window reductions preserve the operand dtype");
                const bool fl = n.dtype == CHELIS_DTYPE_F32 || n.dtype == CHELIS_DTYPE_F64;
                if (!fl && (n.op == Op::ReduceWindowGrad || n.kind == RW_MEAN || !integer_dtype(n.dtype)))
                    return unsupported(n.opname + " precision");
                std::vector<int64_t> outs = x.shape;
                for (size_t k = 0; k < nw; ++k) {
                    const int64_t d = x.shape[r - nw + k] - n.window[k];
                    if (d < 0) return bad("ReduceWindow window larger than its axis ([05-RWIN-1])");
                    outs[r - nw + k] = d / n.wstride[k] + 1;
                }
                if (n.op == Op::ReduceWindow) {
                    if (outs != n.shape) return bad("ReduceWindow result shape");
                } else {
                    if (src(1).dtype != n.dtype || src(1).shape != outs) return bad("ReduceWindowGrad cotangent");
                    CHELIS_TRY(check_same_shape(n, x, "ReduceWindowGrad"));
                }
                own();
                break;
            }
            case Op::Shape: {
                const Node &x = src(0);
                if (n.axis >= static_cast<int>(x.shape.size())) return bad("Shape axis beyond the input rank");
                if (n.dtype != CHELIS_DTYPE_I64 || !n.shape.empty()) return bad("Shape result must be an i64 scalar");
                // extents are concrete here: the read is a constant written into its output
                n.bits = static_cast<uint64_t>(x.shape[n.axis]);
                own();
                break;
            }
            case Op::ExtentWitness: case Op::CheckedExtent: {
                // every extent is concrete here, so the contract is decided now;
                // a broken one is reported when the node runs
                if (n.dtype != CHELIS_DTYPE_I64 || !n.shape.empty()) return bad("a shape contract result must be an i64 scalar", n.opname);
                char buf[512];
                n.message.clear();
                if (n.op == Op::ExtentWitness) {
                    if (n.kind == 0 || (n.kind == 4 && !n.window.empty())) {
                        if (n.window.empty()) return bad("ExtentWitness literal claim without a requirement");
                        n.bits = static_cast<uint64_t>(n.window[0]);  // the claimed extent itself
                        own();
                        break;
                    }
                    const Node &x = src(0);
                    if (n.axis >= static_cast<int>(x.shape.size())) return bad("extent witness axis out of bounds");
                    const int64_t observed = x.shape[n.axis];
                    const char *op = n.kind == 1 ? "load" : n.kind == 2 ? "expand" : "shape";
                    const std::string label = n.kind == 2 ? "node " + std::to_string(n.in[0]) : n.name;
                    for (int64_t req : n.window)
                        if (n.message.empty() && req != observed) {
                            snprintf(buf, sizeof buf,
                                     "extent `%lld`: claimed = %lld, %s axis %d = %lld\nnumeric trap: domain in %s at i64",
                                     static_cast<long long>(req), static_cast<long long>(req), label.c_str(), n.axis,
                                     static_cast<long long>(observed), op);
                            n.message = buf;
                        }
                    for (size_t k = 0; k < n.claims.size() && n.message.empty(); ++k) {
                        const Node &e = src(static_cast<int>(k + 1));
                        if (e.op != Op::ExtentWitness) return bad("extent claim requires a witness edge");
                        const int64_t required = static_cast<int64_t>(e.bits);
                        if (required == observed) continue;
                        char here[160], there[160];
                        snprintf(here, sizeof here, "%s axis %d = %lld", label.c_str(), n.axis,
                                 static_cast<long long>(observed));
                        snprintf(there, sizeof there, "%s axis %d = %lld", e.name.c_str(), e.axis,
                                 static_cast<long long>(required));
                        const bool declares = n.claims[k].second;
                        snprintf(buf, sizeof buf, "extent `%s`: %s, %s\nnumeric trap: domain in %s at i64",
                                 n.claims[k].first.c_str(), declares ? there : here, declares ? here : there, op);
                        n.message = buf;
                    }
                    n.bits = static_cast<uint64_t>(observed);
                } else {
                    int64_t actual = 0;
                    if (!host_extent(src(0), &actual)) return unsupported("CheckedExtent over a computed extent");
                    for (size_t k = 0; k < n.claims.size() && n.message.empty(); ++k) {
                        int64_t required = 0;
                        if (!host_extent(src(static_cast<int>(k + 1)), &required))
                            return unsupported("CheckedExtent over a computed extent");
                        if (required != actual) {
                            snprintf(buf, sizeof buf,
                                     "extent `%s`: claimed = %lld, %s axis %d = %lld\nnumeric trap: domain in %s at i64",
                                     n.claims[k].first.c_str(), static_cast<long long>(required), n.name.c_str(),
                                     n.axis, static_cast<long long>(actual), n.name.c_str());
                            n.message = buf;
                        }
                    }
                    n.bits = static_cast<uint64_t>(actual);
                }
                own();
                break;
            }
            case Op::OrderedAdjointSum: {
                if (n.dtype != CHELIS_DTYPE_F32 && n.dtype != CHELIS_DTYPE_F64)
                    return unsupported("OrderedAdjointSum precision");
                if (!n.shape.empty()) return bad("OrderedAdjointSum result must be a scalar");
                if (n.in.size() > static_cast<size_t>(kMaxAdjointInputs))
                    return unsupported("OrderedAdjointSum with more than 64 inputs");
                size_t k = 0;
                for (int64_t width : n.window) {
                    const Node &first = src(static_cast<int>(k));
                    for (int64_t j = 0; j < width; ++j, ++k) {
                        const Node &x = src(static_cast<int>(k));
                        if (x.dtype != n.dtype) return bad("OrderedAdjointSum contribution dtype");
                        if (x.shape.size() > 1 || (x.shape.empty() && width != 1))
                            return bad("OrderedAdjointSum contributions are rank-one columns or one scalar");
                        if (count_of(x.shape) != count_of(first.shape))
                            return bad("ordered List cotangent columns have different lengths");
                    }
                }
                own();
                break;
            }
            case Op::Iota:
                if (n.activation >= 0) return unsupported("Iota under an activation");
                for (int k = 0; k < 2; ++k)
                    if (src(k).dtype != CHELIS_DTYPE_I64 || !src(k).shape.empty())
                        return bad("Iota bounds must be i64 scalars");
                if (n.dtype != CHELIS_DTYPE_I64 || n.shape.size() != 1) return bad("Iota result must be i64[n]");
                own();
                break;
            case Op::UniformLike: {
                if (n.activation >= 0) return unsupported("UniformLike under an activation");
                if (n.dtype != CHELIS_DTYPE_F32 && n.dtype != CHELIS_DTYPE_F64)
                    return unsupported("UniformLike precision");
                for (int k = 0; k < 3; ++k)
                    if (src(k).dtype != n.dtype) return bad("UniformLike operand dtype");
                if (src(3).dtype != CHELIS_DTYPE_KEY) return bad("UniformLike key must be a key");
                CHELIS_TRY(check_same_shape(n, src(0), "UniformLike"));
                const auto &ks = src(3).shape;
                if (ks.size() > n.shape.size() || !std::equal(ks.begin(), ks.end(), n.shape.begin()))
                    return bad("UniformLike key shape");
                for (int k = 1; k < 3; ++k) {
                    const auto &bs = src(k).shape;
                    if (bs.size() > ks.size() || !std::equal(bs.begin(), bs.end(), ks.begin()))
                        return bad("UniformLike bound shape");
                }
                own();
                break;
            }
            case Op::UniformBoundAdjoint: {
                if (n.activation >= 0) return unsupported("UniformBoundAdjoint under an activation");
                if (n.dtype != CHELIS_DTYPE_F32 && n.dtype != CHELIS_DTYPE_F64)
                    return unsupported("UniformBoundAdjoint precision");
                const Node &t = src(0), &g = src(1), &k = src(2);
                if (t.dtype != n.dtype || g.dtype != n.dtype) return bad("UniformBoundAdjoint operand dtype");
                if (g.shape != t.shape) return bad("UniformBoundAdjoint cotangent shape");
                if (k.dtype != CHELIS_DTYPE_KEY) return bad("UniformBoundAdjoint key must be a key");
                if (k.shape.size() > t.shape.size() || !std::equal(k.shape.begin(), k.shape.end(), t.shape.begin()))
                    return bad("UniformBoundAdjoint key shape");
                if (n.shape.size() > k.shape.size() || !std::equal(n.shape.begin(), n.shape.end(), k.shape.begin()))
                    return bad("UniformBoundAdjoint result is not a leading part of its keys' shape");
                own();
                break;
            }
            case Op::Dropout: {
                if (n.activation >= 0) return unsupported("Dropout under an activation");
                if (n.dtype != CHELIS_DTYPE_F32 && n.dtype != CHELIS_DTYPE_F64)
                    return unsupported("Dropout precision");
                if (src(0).dtype != n.dtype || src(1).dtype != n.dtype) return bad("Dropout operand dtype");
                if (src(2).dtype != CHELIS_DTYPE_KEY) return bad("Dropout key must be a key");
                CHELIS_TRY(check_same_shape(n, src(0), "Dropout"));
                // the key is rank 0 or shaped like a leading part of the data;
                // the rate rank 0 or a leading part of the key's shape
                const auto &ks = src(2).shape, &rs = src(1).shape;
                if (ks.size() > n.shape.size() || !std::equal(ks.begin(), ks.end(), n.shape.begin()))
                    return bad("Dropout key shape");
                if (rs.size() > ks.size() || !std::equal(rs.begin(), rs.end(), ks.begin()))
                    return bad("Dropout rate shape");
                own();
                break;
            }
            case Op::GuardedFail:
                if (src(0).dtype != CHELIS_DTYPE_BOOL) return bad("GuardedFail condition must be bool");
                if (src(1).dtype != n.dtype) return bad("GuardedFail fallback dtype");
                CHELIS_TRY(check_same_shape(n, src(1), "GuardedFail"));
                own();
                break;
            case Op::NamedCast: {
                const int from = src(0).dtype;
                const bool ffrom = from == CHELIS_DTYPE_F32 || from == CHELIS_DTYPE_F64;
                if (!integer_dtype(n.dtype)) return bad("NamedCast targets a signed integer");
                if (n.kind == NC_TRUNC && !ffrom) return bad("cast_trunc converts a float source");
                if (n.kind == NC_WRAP && !integer_dtype(from)) return bad("cast_wrap converts an integer source");
                if (n.kind == NC_SATURATE && !ffrom && !integer_dtype(from))
                    return bad("cast_saturate converts a float or integer source");
                CHELIS_TRY(check_same_shape(n, src(0), "NamedCast"));
                own();
                break;
            }
            case Op::Arith:
                if (!integer_dtype(n.dtype) && n.dtype != CHELIS_DTYPE_F32 && n.dtype != CHELIS_DTYPE_F64)
                    return unsupported(n.opname + " precision");
                for (size_t k = 0; k < n.in.size(); ++k) {
                    if (src(static_cast<int>(k)).dtype != n.dtype) return bad("elementwise operand dtype", n.opname);
                    CHELIS_TRY(check_same_shape(n, src(static_cast<int>(k)), n.opname.c_str()));
                }
                own();
                break;
            case Op::FloatClassify:
                if (!floating_dtype(src(0).dtype)) return bad("FloatClassify operand must be a float");
                if (n.dtype != CHELIS_DTYPE_BOOL) return bad("FloatClassify result must be bool");
                CHELIS_TRY(check_same_shape(n, src(0), "FloatClassify"));
                own();
                break;
            case Op::ExtremaAdjoint:
                if (!floating) return unsupported("ExtremaAdjoint precision");
                for (int k = 0; k < 3; ++k) {
                    if (src(k).dtype != n.dtype) return bad("ExtremaAdjoint operand dtype");
                    CHELIS_TRY(check_same_shape(n, src(k), "ExtremaAdjoint"));
                }
                own();
                break;
            case Op::Count: {
                if (src(0).dtype != CHELIS_DTYPE_BOOL || n.dtype != CHELIS_DTYPE_I64)
                    return unsupported("Count other than bool -> i64");
                // axes: distinct positions of the input, listed in descending order (dag.rs Count)
                const int r = static_cast<int>(src(0).shape.size());
                std::vector<int64_t> kept;
                for (size_t k = 0; k < n.axes.size(); ++k)
                    if (n.axes[k] < 0 || n.axes[k] >= r || (k > 0 && n.axes[k] >= n.axes[k - 1]))
                        return bad("Count axes must be distinct input axes in descending order");
                for (int d = 0; d < r; ++d)
                    if (std::find(n.axes.begin(), n.axes.end(), d) == n.axes.end()) kept.push_back(src(0).shape[d]);
                if (kept != n.shape) return bad("Count result shape");
                own();
                break;
            }
            case Op::Matmul: {
                const auto &a = src(0).shape, &b = src(1).shape;
                if (!floating || src(0).dtype != n.dtype || src(1).dtype != n.dtype ||
                    n.accumulator != n.dtype)
                    return unsupported("BlasMatmul precision");
                const size_t r = n.shape.size();
                if (r < 2 || a.size() != r || b.size() != r || a[r - 1] != b[r - 2] ||
                    a[r - 2] != n.shape[r - 2] || b[r - 1] != n.shape[r - 1])
                    return bad("BlasMatmul operand shapes");
                for (size_t d = 0; d + 2 < r; ++d)
                    if (a[d] != n.shape[d] || b[d] != n.shape[d]) return bad("BlasMatmul batch axes");
                own();
                break;
            }
            case Op::Gather: case Op::ScatterAdd: case Op::Scatter: {
                const Node &vals = src(0);
                const Node &idx = src(1);
                const int it = idx.dtype;
                if (it != CHELIS_DTYPE_I64 && it != CHELIS_DTYPE_I32 && it != CHELIS_DTYPE_I16 &&
                    it != CHELIS_DTYPE_I8)
                    return bad("index dtype must be a signed integer ([05-SPARSE-1])");
                if (vals.dtype != n.dtype) return bad("gather / scatter value dtype");
                const int vr = static_cast<int>(vals.shape.size());
                const int ir = static_cast<int>(idx.shape.size());
                if (n.axis >= vr || n.batch_rank > n.axis || n.batch_rank > ir)
                    return bad("gather / scatter axis or batch rank");
                for (int d = 0; d < n.batch_rank; ++d)
                    if (idx.shape[d] != vals.shape[d]) return bad("gather / scatter batch axes");
                std::vector<int64_t> sel(vals.shape.begin(), vals.shape.begin() + n.axis);
                sel.insert(sel.end(), idx.shape.begin() + n.batch_rank, idx.shape.end());
                sel.insert(sel.end(), vals.shape.begin() + n.axis + 1, vals.shape.end());
                if (sel.size() > static_cast<size_t>(kMaxRank)) return unsupported("gather rank");
                if (n.op == Op::Gather) {
                    if (sel != n.shape) return bad("Gather result shape");
                } else {
                    if (n.shape != vals.shape || src(2).shape != sel || src(2).dtype != n.dtype)
                        return bad("ScatterAdd shapes");
                }
                own();
                break;
            }
            case Op::ScatterElements: {
                const Node &data = src(0), &idx = src(1), &upd = src(2);
                const int it = idx.dtype;
                if (it != CHELIS_DTYPE_I64 && it != CHELIS_DTYPE_I32 && it != CHELIS_DTYPE_I16 &&
                    it != CHELIS_DTYPE_I8)
                    return bad("index dtype must be a signed integer ([05-SPARSE-1])");
                if (data.dtype != n.dtype || upd.dtype != n.dtype) return bad("ScatterElements value dtype");
                const size_t r = data.shape.size();
                if (n.axis >= static_cast<int>(r) || idx.shape.size() != r || upd.shape != idx.shape ||
                    n.shape != data.shape)
                    return bad("ScatterElements shapes");
                for (size_t d = 0; d < r; ++d)
                    if (static_cast<int>(d) != n.axis && idx.shape[d] > data.shape[d])
                        return bad("ScatterElements index extent beyond the data");
                own();
                break;
            }
            case Op::Reshape: {
                const Node &s = src(0);
                if (n.opname == "CheckedUnitAxis") {
                    std::vector<int64_t> want = s.shape;
                    if (n.axis >= static_cast<int>(want.size())) return bad("CheckedUnitAxis axis");
                    if (want[n.axis] != 1) return bad("CheckedUnitAxis over an axis whose extent is not 1");
                    if (n.shape != want) return bad("CheckedUnitAxis result shape");
                }
                if (s.dtype != n.dtype || count_of(s.shape) != count_of(n.shape))
                    return bad("Reshape changes the element count");
                const Layout &SL = P.layout[n.in[0]];
                if (is_dense(s.shape, SL.strides)) {
                    L.root = SL.root;
                    L.offset = SL.offset;
                    L.strides = dense_strides(n.shape);
                } else {
                    own();  // materialised
                }
                break;
            }
            case Op::Permute: {
                const Node &s = src(0);
                const size_t r = s.shape.size();
                if (n.axes.size() != r || n.shape.size() != r || s.dtype != n.dtype)
                    return bad("Permute axes");
                std::vector<bool> seen(r, false);
                const Layout &SL = P.layout[n.in[0]];
                L.root = SL.root;
                L.offset = SL.offset;
                L.strides.assign(r, 0);
                for (size_t d = 0; d < r; ++d) {
                    const int a = n.axes[d];
                    if (a < 0 || a >= static_cast<int>(r) || seen[a] || s.shape[a] != n.shape[d])
                        return bad("Permute axes");
                    seen[a] = true;
                    L.strides[d] = SL.strides[a];
                }
                break;
            }
            case Op::Expand: {
                const Node &s = src(0);
                const Layout &SL = P.layout[n.in[0]];
                const size_t r = n.shape.size();
                if (s.dtype != n.dtype || n.axis >= static_cast<int>(r)) return bad("Expand axis");
                L.root = SL.root;
                L.offset = SL.offset;
                if (s.shape.size() + 1 == r) {  // rank-increasing: insert a broadcast axis
                    std::vector<int64_t> back = n.shape;
                    back.erase(back.begin() + n.axis);
                    if (back != s.shape) return bad("Expand shape");
                    L.strides = SL.strides;
                    L.strides.insert(L.strides.begin() + n.axis, 0);
                } else if (s.shape.size() == r) {  // same rank: a size-1 axis broadcast
                    for (size_t d = 0; d < r; ++d)
                        if (static_cast<int>(d) != n.axis ? s.shape[d] != n.shape[d]
                                                          : s.shape[d] != 1)
                            return bad("Expand shape");
                    L.strides = SL.strides;
                    L.strides[n.axis] = 0;
                } else {
                    return bad("Expand rank");
                }
                break;
            }
            case Op::Shrink: {
                const Node &s = src(0);
                const Layout &SL = P.layout[n.in[0]];
                if (n.bounds.size() != s.shape.size() || n.shape.size() != s.shape.size() ||
                    s.dtype != n.dtype)
                    return bad("Shrink bounds");
                L.root = SL.root;
                L.offset = SL.offset;
                L.strides = SL.strides;
                for (size_t d = 0; d < n.bounds.size(); ++d) {
                    const auto b = n.bounds[d];
                    if (b.first < 0 || b.second < b.first || b.second > s.shape[d] ||
                        n.shape[d] != b.second - b.first)
                        return bad("Shrink bounds");
                    L.offset += b.first * SL.strides[d];
                }
                break;
            }
            case Op::Stride: {
                const Node &s = src(0);
                const Layout &SL = P.layout[n.in[0]];
                if (n.step.size() != s.shape.size() || n.shape.size() != s.shape.size() ||
                    s.dtype != n.dtype)
                    return bad("Stride steps");
                L.root = SL.root;
                L.offset = SL.offset;
                L.strides = SL.strides;
                for (size_t d = 0; d < n.step.size(); ++d) {
                    if (n.shape[d] != (s.shape[d] + n.step[d] - 1) / n.step[d])
                        return bad("Stride result shape");
                    L.strides[d] *= n.step[d];
                }
                break;
            }
            case Op::Pad: {
                const Node &s = src(0);
                if (n.bounds.size() != s.shape.size() || n.shape.size() != s.shape.size() ||
                    s.dtype != n.dtype)
                    return bad("Pad");
                for (size_t d = 0; d < n.bounds.size(); ++d)
                    if (n.shape[d] != s.shape[d] + n.bounds[d].first + n.bounds[d].second)
                        return bad("Pad result shape");
                own();
                break;
            }
            case Op::Cast: {
                const int from = src(0).dtype;
                const bool to_float = floating;
                const bool from_ok = from == CHELIS_DTYPE_F32 || from == CHELIS_DTYPE_F64 ||
                                     from == CHELIS_DTYPE_I32 || from == CHELIS_DTYPE_I64 ||
                                     from == CHELIS_DTYPE_I16 || from == CHELIS_DTYPE_I8 ||
                                     from == CHELIS_DTYPE_BOOL;
                const bool to_ok = to_float || integer_dtype(n.dtype) || n.dtype == CHELIS_DTYPE_BOOL;
                if (!to_ok || !from_ok) return unsupported("Cast between these precisions");
                CHELIS_TRY(check_same_shape(n, src(0), "Cast"));
                own();
                break;
            }
            case Op::Copy:
                if (src(0).dtype != n.dtype) return bad("Copy dtype");
                CHELIS_TRY(check_same_shape(n, src(0), "Copy"));
                own();
                break;
            case Op::Store: {
                const Node &s = src(0);
                if (s.dtype != n.dtype) return bad("Store dtype");
                CHELIS_TRY(check_same_shape(n, s, "Store"));
                L = P.layout[n.in[0]];
                break;
            }
        }
    }
    return CHELIS_CUDA_OK;
}

bool is_view(Op op) {
    return op == Op::Permute || op == Op::Expand || op == Op::Shrink || op == Op::Stride ||
           op == Op::Store;
}

// ---------------------------------------------------------------- planning

// Placement of every node, outputs (Store nodes, then the roots:
// emit.rs:5901-5934), reduction-inlined FusedElems, slot reuse after last
// use and the arena size (memory.rs:39-98).
// The entry's interface: inputs in the order of the first Load of each name;
// outputs the Stores in node order, then the roots not already outputs
// (labels "root<i>").
int io_plan(Program &P, const std::vector<int> &roots) {
    const std::vector<Node> &N = P.nodes;
    const int count = static_cast<int>(N.size());
    P.input_of_load.assign(count, -1);
    P.input_labels.clear();
    P.output_labels.clear();
    P.output_node.clear();
    for (int i = 0; i < count; ++i) {
        if (N[i].op != Op::Load) continue;
        int slot = -1;
        for (size_t k = 0; k < P.input_labels.size(); ++k)
            if (P.input_labels[k] == N[i].name) slot = static_cast<int>(k);
        if (slot < 0) {
            slot = static_cast<int>(P.input_labels.size());
            P.input_labels.push_back(N[i].name);
        }
        P.input_of_load[i] = slot;
    }
    for (int i = 0; i < count; ++i)
        if (N[i].op == Op::Store) {
            P.output_labels.push_back(N[i].name);
            P.output_node.push_back(i);
        }
    std::vector<int> rs = roots;
    if (rs.empty() && count > 0) rs.push_back(count - 1);
    for (size_t k = 0; k < rs.size(); ++k) {
        if (rs[k] < 0 || rs[k] >= count) return bad("root out of range");
        if (std::find(P.output_node.begin(), P.output_node.end(), rs[k]) != P.output_node.end())
            continue;
        P.output_labels.push_back("root" + std::to_string(k));
        P.output_node.push_back(rs[k]);
    }
    return CHELIS_CUDA_OK;
}

int plan(Program &P, const std::vector<int> &roots) {
    std::vector<Node> &N = P.nodes;
    const int count = static_cast<int>(N.size());
    P.place.assign(count, Place::Slot);
    P.slot.assign(count, -1);
    P.direct_output.assign(count, -1);
    CHELIS_TRY(io_plan(P, roots));
    for (int i = 0; i < count; ++i) {
        const Node &n = N[i];
        if (n.op == Op::Load) {
            P.place[i] = Place::Input;
        } else if (n.op == Op::Drop) {
            P.place[i] = Place::Skip;
        } else if (is_view(n.op) || (n.op == Op::Reshape && P.layout[i].root != i)) {
            P.place[i] = Place::View;
        }
    }
    // consumers
    std::vector<std::vector<int>> users(count);
    for (int i = 0; i < count; ++i)
        for (int j : N[i].in) users[j].push_back(i);
    std::vector<bool> is_output(count, false);
    for (int o : P.output_node) is_output[o] = true;
    // a FusedElem read only by a Sum / MaxReduce runs inside the reduction
    for (int i = 0; i < count; ++i) {
        const Node &n = N[i];
        if ((n.op == Op::Sum || n.op == Op::MaxReduce) && N[n.in[0]].op == Op::Fused) {
            const int f = n.in[0];
            if (users[f].size() == 1 && !is_output[f] && N[f].in.size() <= 7)
                P.place[f] = Place::Inlined;
        }
    }
    // outputs written straight into their owners: a slot node whose value is
    // the output unchanged (the node itself, or a Store of it)
    for (size_t k = 0; k < P.output_node.size(); ++k) {
        int o = P.output_node[k];
        while (N[o].op == Op::Store) o = N[o].in[0];
        if (P.place[o] == Place::Slot && P.direct_output[o] < 0) {
            P.place[o] = Place::Output;
            P.direct_output[o] = static_cast<int>(k);
        }
    }
    // last use of each storage root (through views; inlined nodes' inputs
    // are read by their reduction)
    std::vector<int> last(count, -1);
    auto root_of = [&](int j) { return P.layout[j].root; };
    for (int i = 0; i < count; ++i) {
        if (P.place[i] == Place::Inlined) continue;
        std::vector<int> reads = N[i].in;
        if ((N[i].op == Op::Sum || N[i].op == Op::MaxReduce) && P.place[N[i].in[0]] == Place::Inlined)
            reads = N[N[i].in[0]].in;
        for (int j : reads) last[root_of(j)] = std::max(last[root_of(j)], i);
    }
    for (int o : P.output_node) last[root_of(o)] = count;  // copied out at the end
    // slots: best fit among slots free before node i runs
    std::vector<int64_t> slot_free_at;  // last use of the slot's current owner
    int64_t live = 0;
    for (int i = 0; i < count; ++i) {
        if (P.place[i] != Place::Slot) continue;
        const int64_t bytes = ((std::max<int64_t>(count_of(N[i].shape), 1) *
                                dtype_width(N[i].dtype)) + 255) / 256 * 256;
        int best = -1;
        for (size_t s = 0; s < P.slot_cap.size(); ++s)
            if (slot_free_at[s] < i && P.slot_cap[s] >= bytes &&
                (best < 0 || P.slot_cap[s] < P.slot_cap[best]))
                best = static_cast<int>(s);
        if (best < 0) {
            best = static_cast<int>(P.slot_cap.size());
            P.slot_cap.push_back(bytes);
            slot_free_at.push_back(-1);
        }
        slot_free_at[best] = std::max(last[i], i);
        P.slot[i] = best;
        // bytes live while node i runs: slots whose owner is still needed
        live = 0;
        for (size_t s = 0; s < P.slot_cap.size(); ++s)
            if (slot_free_at[s] >= i) live += P.slot_cap[s];
        P.live_peak_bytes = std::max(P.live_peak_bytes, live);
    }
    P.slot_off.resize(P.slot_cap.size());
    int64_t off = 0;
    for (size_t s = 0; s < P.slot_cap.size(); ++s) {
        P.slot_off[s] = off;
        off += P.slot_cap[s];
    }
    P.arena_bytes = off;
    return CHELIS_CUDA_OK;
}

// ---------------------------------------------------------------- kernels

struct Strided {
    int32_t rank;
    int64_t shape[kMaxRank];
    int64_t stride[kMaxRank];
};

__device__ __forceinline__ int64_t offset_of(const Strided &s, int64_t linear) {
    int64_t off = 0;
    for (int d = s.rank - 1; d >= 0; --d) {
        const int64_t c = linear % s.shape[d];
        linear /= s.shape[d];
        off += c * s.stride[d];
    }
    return off;
}

template <typename T>
__global__ void copy_kernel(const T *__restrict__ src, Strided s, T *__restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        dst[i] = src[offset_of(s, i)];
}

template <typename T>
__global__ void fill_kernel(T *__restrict__ dst, T v, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        dst[i] = v;
}

// out (dense, `o` its shape) = src at coordinate - before, or the fill
template <typename T>
__global__ void pad_kernel(const T *__restrict__ src, Strided s, Strided o, Strided before, T fill,
                           T *__restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t rem = i, off = 0;
        bool in = true;
        for (int d = o.rank - 1; d >= 0; --d) {
            const int64_t c = rem % o.shape[d] - before.shape[d];
            rem /= o.shape[d];
            if (c < 0 || c >= s.shape[d]) in = false;
            off += c * s.stride[d];
        }
        dst[i] = in ? src[off] : fill;
    }
}

template <typename From, typename To>
__global__ void cast_kernel(const From *__restrict__ src, Strided s, To *__restrict__ dst, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        dst[i] = static_cast<To>(src[offset_of(s, i)]);
}

// The checked cast to an integer or bool target (the reference's default
// cast, host_emit.rs checked_cast_*): from a float, a non-finite or
// non-integral value traps Domain and an out-of-range one Overflow; from an
// integer or bool, an out-of-range value traps Overflow; to bool, only 0 and 1
// are admitted (others trap Domain) and 1 gives true.  A trapping element is
// written as 0 and recorded with report_trap.
template <typename From, typename To>
__global__ void cast_checked_kernel(const From *__restrict__ src, Strided s, To *__restrict__ dst, int64_t n,
                                    unsigned int to_dt) {
    constexpr bool to_bool = sizeof(To) == 1 && !std::is_signed<To>::value;
    constexpr int64_t lo = to_bool ? 0 : sizeof(To) == 8 ? INT64_MIN : sizeof(To) == 4 ? INT32_MIN
                                                          : sizeof(To) == 2 ? INT16_MIN : INT8_MIN;
    constexpr int64_t hi = to_bool ? 1 : sizeof(To) == 8 ? INT64_MAX : sizeof(To) == 4 ? INT32_MAX
                                                          : sizeof(To) == 2 ? INT16_MAX : INT8_MAX;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const From x = src[offset_of(s, i)];
        int64_t w = 0;
        bool domain = false, overflow = false;
        if constexpr (std::is_floating_point<From>::value) {
            const double v = static_cast<double>(x);
            if (!isfinite(v) || trunc(v) != v || (to_bool && v != 0.0 && v != 1.0)) {
                domain = true;
            } else if (to_bool) {
                w = v == 1.0 ? 1 : 0;
            } else if (sizeof(To) == 8 ? (v < -9223372036854775808.0 || v >= 9223372036854775808.0)
                                       : (v < static_cast<double>(lo) || v > static_cast<double>(hi))) {
                overflow = true;
            } else {
                w = static_cast<int64_t>(v);
            }
        } else {
            w = static_cast<int64_t>(x);
            if (to_bool) domain = w != 0 && w != 1;
            else overflow = w < lo || w > hi;
        }
        if (domain || overflow) {
            report_trap(domain ? TRAP_DOMAIN : TRAP_OVERFLOW, TRAP_OP_CAST, to_dt);
            w = 0;
        }
        dst[i] = static_cast<To>(w);
    }
}

// The named lossy casts to a signed integer (host_emit.rs named_cast_c_expr):
// cast_trunc (float source) truncates toward zero, trapping Domain on a
// non-finite value and Overflow out of range; cast_saturate truncates and
// clamps to the target range, trapping Domain on NaN only; cast_wrap
// (integer source) keeps the target width's low bits, sign-extended.
template <typename From, typename To>
__global__ void named_cast_kernel(const From *__restrict__ src, Strided s, int mode, To *__restrict__ dst,
                                  int64_t n, unsigned int to_dt) {
    constexpr int bits = 8 * sizeof(To);
    constexpr int64_t lo = bits == 64 ? INT64_MIN : -(int64_t(1) << (bits - 1));
    constexpr int64_t hi = bits == 64 ? INT64_MAX : (int64_t(1) << (bits - 1)) - 1;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const From x = src[offset_of(s, i)];
        int64_t w = 0;
        if constexpr (std::is_floating_point<From>::value) {
            const double v = static_cast<double>(x);
            if (mode == NC_TRUNC) {
                const double t = trunc(v);
                if (!isfinite(v)) report_trap(TRAP_DOMAIN, TRAP_OP_CAST_TRUNC, to_dt);
                else if (bits == 64 ? (t < -9223372036854775808.0 || t >= 9223372036854775808.0)
                                    : (t < static_cast<double>(lo) || t > static_cast<double>(hi)))
                    report_trap(TRAP_OVERFLOW, TRAP_OP_CAST_TRUNC, to_dt);
                else w = static_cast<int64_t>(t);
            } else {  // saturate
                if (isnan(v)) report_trap(TRAP_DOMAIN, TRAP_OP_CAST_SATURATE, to_dt);
                else if (v <= static_cast<double>(lo)) w = lo;
                else if (v >= static_cast<double>(hi)) w = hi;
                else w = static_cast<int64_t>(trunc(v));
            }
        } else {
            const int64_t v = static_cast<int64_t>(x);
            if (mode == NC_SATURATE) w = v < lo ? lo : (v > hi ? hi : v);
            else if (bits >= 8 * static_cast<int>(sizeof(From))) w = v;
            else {
                const uint64_t sign = uint64_t(1) << (bits - 1), mask = (sign << 1) - 1;
                w = static_cast<int64_t>(((static_cast<uint64_t>(v) & mask) ^ sign) - sign);
            }
        }
        dst[i] = static_cast<To>(w);
    }
}

// GuardedFail: any condition element equal to `fires` (1 or 0) records the
// guard's message id (the first guard to fire in stream order keeps it)
__global__ void guard_kernel(const uint8_t *__restrict__ c, Strided sc, int fires, uint32_t id, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        if ((c[offset_of(sc, i)] != 0) == (fires != 0)) {
            atomicCAS(&g_fail_id, 0u, id);
            atomicOr(&g_device_error, static_cast<unsigned int>(DEVERR_FAIL));
        }
}

template <typename I>
__device__ __forceinline__ int64_t load_index(const void *p, int64_t off) {
    return static_cast<int64_t>(static_cast<const I *>(p)[off]);
}
__device__ __forceinline__ int64_t read_index(const void *p, int64_t off, int width) {
    switch (width) {
        case 8: return load_index<int64_t>(p, off);
        case 4: return load_index<int32_t>(p, off);
        case 2: return load_index<int16_t>(p, off);
        default: return load_index<int8_t>(p, off);
    }
}

// Gather (spec [05-OP-52]): out[p, q, t] = values[p, idx[p_batch, q], t] for
// p over values' axes before `axis`, q over the index axes after the batch
// ones, t over values' axes after `axis`.  `v` / `x` are values' and
// indices' layouts, the output dense.  An index outside [0, values.shape[axis])
// writes 0 and records a domain trap with the index.
struct GatherGeom {
    Strided v, x;
    int32_t axis, batch_rank, qrank, trank;
    int64_t qshape[kMaxRank], tshape[kMaxRank];
    int32_t index_width;
};

template <typename T>
__device__ __forceinline__ T canonical_nan(T r) {
    if (r == r) return r;
    if constexpr (sizeof(T) == 4) return __int_as_float(0x7fc00000);
    else return __longlong_as_double(0x7ff8000000000000ll);
}

// Cumsum along a leading axis (spec 05 4310-4325, the C lane's scan): the
// first element of a line is its first prefix, each later one is added to
// the previous prefix in axis order (reversed for a decreasing scan); NaN
// results are stored canonical.  One thread per line; adjacent threads take
// adjacent lines, which are adjacent in memory for a dense input.
template <typename T>
__global__ void cumsum_axis_kernel(const T *__restrict__ x, Strided lines, int64_t xstep, Strided o, int64_t ostep,
                                   int64_t len, int reverse, T *__restrict__ out, int64_t lanes) {
    for (int64_t l = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; l < lanes;
         l += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t xb = offset_of(lines, l), ob = offset_of(o, l);
        T acc = T(0);
        for (int64_t t = 0; t < len; ++t) {
            const int64_t i = reverse ? len - 1 - t : t;
            const T v = x[xb + i * xstep];
            if (t == 0) acc = v;
            else if constexpr (sizeof(T) == 4) acc = __fadd_rn(acc, v);
            else acc = __dadd_rn(acc, v);
            out[ob + i * ostep] = canonical_nan(acc);
        }
    }
}

// Count over some axes: block b counts the true elements of output b's
// counted sub-space (`counted`, in input axis order) at `kept`'s offset; the
// count is exact in any order.
__global__ void count_axes_kernel(const uint8_t *__restrict__ x, Strided kept, Strided counted, int64_t outputs,
                                  int64_t volume, int64_t *__restrict__ out) {
    __shared__ unsigned long long part[4];
    for (int64_t o = blockIdx.x; o < outputs; o += gridDim.x) {
        const int64_t base = offset_of(kept, o);
        unsigned long long c = 0;
        for (int64_t e = threadIdx.x; e < volume; e += blockDim.x) c += x[base + offset_of(counted, e)] != 0;
        for (int off = 16; off > 0; off >>= 1) c += __shfl_xor_sync(0xffffffffu, c, off);
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = c;
        __syncthreads();
        if (threadIdx.x == 0) out[o] = static_cast<int64_t>(part[0] + part[1] + part[2] + part[3]);
        __syncthreads();
    }
}

template <typename T>
__global__ void gather_kernel(const T *__restrict__ values, const void *__restrict__ idx,
                              GatherGeom g, T *__restrict__ out, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t rem = i, voff = 0, xoff = 0;
        for (int d = g.trank - 1; d >= 0; --d) {  // trailing value axes
            const int64_t c = rem % g.tshape[d];
            rem /= g.tshape[d];
            voff += c * g.v.stride[g.axis + 1 + d];
        }
        for (int d = g.qrank - 1; d >= 0; --d) {  // index axes after the batch ones
            const int64_t c = rem % g.qshape[d];
            rem /= g.qshape[d];
            xoff += c * g.x.stride[g.batch_rank + d];
        }
        for (int d = g.axis - 1; d >= 0; --d) {  // leading value axes (batch ones pair with idx)
            const int64_t c = rem % g.v.shape[d];
            rem /= g.v.shape[d];
            voff += c * g.v.stride[d];
            if (d < g.batch_rank) xoff += c * g.x.stride[d];
        }
        const int64_t k = read_index(idx, xoff, g.index_width);
        if (k < 0 || k >= g.v.shape[g.axis]) {
            report_index_trap(TRAP_OP_GATHER, k, g.axis, g.v.shape[g.axis]);
            out[i] = T(0);
        } else {
            out[i] = values[voff + k * g.v.stride[g.axis]];
        }
    }
}

// ScatterAdd: out (a dense copy of the target) [p, idx[p_batch, q], t] +=
// updates[p, q, t].  One thread per (p, t) adds its updates in increasing q,
// which is the updates' increasing flat order for every target cell.
template <typename T>
__global__ void scatter_add_kernel(const T *__restrict__ upd, Strided u, const void *__restrict__ idx,
                                   GatherGeom g, T *__restrict__ out, int64_t lanes, int64_t nq, int replace) {
    const Strided o = g.v;  // the output's dense layout and shape
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < lanes;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t rem = i, ooff = 0, uoff = 0, xbase = 0;
        for (int d = g.trank - 1; d >= 0; --d) {
            const int64_t c = rem % g.tshape[d];
            rem /= g.tshape[d];
            ooff += c * o.stride[g.axis + 1 + d];
            uoff += c * u.stride[g.axis + g.qrank + d];
        }
        for (int d = g.axis - 1; d >= 0; --d) {
            const int64_t c = rem % o.shape[d];
            rem /= o.shape[d];
            ooff += c * o.stride[d];
            uoff += c * u.stride[d];
            if (d < g.batch_rank) xbase += c * g.x.stride[d];
        }
        for (int64_t q = 0; q < nq; ++q) {
            int64_t qr = q, xoff = xbase, qoff = 0;
            for (int d = g.qrank - 1; d >= 0; --d) {
                const int64_t c = qr % g.qshape[d];
                qr /= g.qshape[d];
                xoff += c * g.x.stride[g.batch_rank + d];
                qoff += c * u.stride[g.axis + d];
            }
            const int64_t k = read_index(idx, xoff, g.index_width);
            if (k < 0 || k >= o.shape[g.axis]) {
                report_index_trap(replace ? TRAP_OP_SCATTER : TRAP_OP_SCATTER_ADD, k, g.axis, o.shape[g.axis]);
                continue;
            }
            T *cell = out + ooff + k * o.stride[g.axis];
            if (replace) *cell = upd[uoff + qoff];  // Scatter: the last write in update order wins
            else *cell = *cell + upd[uoff + qoff];
        }
    }
}

// ScatterElements: update c (indices' shape) replaces data[c with its axis
// coordinate set to indices[c]].  One thread per line of updates along the
// axis, visited in order, so the last write in row-major update order wins.
template <typename T>
__global__ void scatter_elements_kernel(const T *__restrict__ upd, Strided su, const void *__restrict__ idx,
                                        Strided si, int index_width, Strided o, int axis, T *__restrict__ out,
                                        int64_t lanes, int64_t len) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < lanes;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t rem = i, uoff = 0, xoff = 0, ooff = 0;
        for (int d = su.rank - 1; d >= 0; --d) {
            if (d == axis) continue;
            const int64_t c = rem % su.shape[d];
            rem /= su.shape[d];
            uoff += c * su.stride[d];
            xoff += c * si.stride[d];
            ooff += c * o.stride[d];
        }
        for (int64_t j = 0; j < len; ++j) {
            const int64_t k = read_index(idx, xoff + j * si.stride[axis], index_width);
            if (k < 0 || k >= o.shape[axis]) {
                report_index_trap(TRAP_OP_SCATTER_ELEMENTS, k, axis, o.shape[axis]);
                continue;
            }
            out[ooff + k * o.stride[axis]] = upd[uoff + j * su.stride[axis]];
        }
    }
}

// A stored element as the value it compares by: 16-bit floats widen to f32
// (the C lane's comparison converts bf16 / f16 to f32 first).
template <typename T> struct CmpVal { using V = T; __device__ static V get(T x) { return x; } };
struct Bf16Bits { uint16_t b; };
struct F16Bits { uint16_t b; };
template <> struct CmpVal<Bf16Bits> {
    using V = float;
    __device__ static float get(Bf16Bits x) { return __uint_as_float(static_cast<uint32_t>(x.b) << 16); }
};
template <> struct CmpVal<F16Bits> {
    using V = float;
    __device__ static float get(F16Bits x) { return __half2float(__ushort_as_half(x.b)); }
};

// [05-OP-36] element-wise comparison into bool bytes: C's <, ==, !=, >, >=,
// <= on the operands' values (a NaN makes every ordered comparison and ==
// false and != true; signed zeros are equal; integers compare exactly).
template <typename T>
__global__ void compare_kernel(const T *__restrict__ a, Strided sa, const T *__restrict__ b, Strided sb,
                               int kind, uint8_t *__restrict__ out, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const auto x = CmpVal<T>::get(a[offset_of(sa, i)]);
        const auto y = CmpVal<T>::get(b[offset_of(sb, i)]);
        bool r;
        switch (kind) {
            case CMP_EQ: r = x == y; break;
            case CMP_NEQ: r = x != y; break;
            case CMP_GT: r = x > y; break;
            case CMP_GTE: r = x >= y; break;
            case CMP_LTE: r = x <= y; break;
            default: r = x < y; break;  // cmplt, lt
        }
        out[i] = r ? 1 : 0;
    }
}

// [05-OP-26..28] and / or / not on bool bytes (a stored bool is 0 or 1)
__global__ void logical_kernel(const uint8_t *__restrict__ a, Strided sa, const uint8_t *__restrict__ b,
                               Strided sb, int kind, uint8_t *__restrict__ out, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const bool x = a[offset_of(sa, i)] != 0;
        bool r;
        if (kind == LOG_NOT) r = !x;
        else {
            const bool y = b[offset_of(sb, i)] != 0;
            r = kind == LOG_AND ? (x && y) : (x || y);
        }
        out[i] = r ? 1 : 0;
    }
}

// where(c, a, b): the stored bits of a where c is true, of b elsewhere
template <typename T>
__global__ void where_kernel(const uint8_t *__restrict__ c, Strided sc, const T *__restrict__ a, Strided sa,
                             const T *__restrict__ b, Strided sb, T *__restrict__ out, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = c[offset_of(sc, i)] ? a[offset_of(sa, i)] : b[offset_of(sb, i)];
}

// MinReduce / MaxReduce-style selection along one axis, as the C lane's
// in-order scans pick (emit_reduce_extreme, emit_reduce_argcmp): the first
// NaN if any, else the first of the smallest (MAX: largest) values, signed
// zeros comparing equal.  The result is the chosen element's stored bits
// (MinReduce) or its position on the axis (Argmax / Argmin, i64).  One warp
// per output: each lane scans a strided subset and the lanes combine
// (value, position) pairs, which gives the scan's choice in any grouping.
// `o` maps an output index to the offset of its first element; `len` /
// `step` walk the reduced axis.
template <bool MAX, typename T>
__device__ __forceinline__ bool pick_better(T v, int64_t p, T bv, int64_t bp) {
    // does (v, p) win over the current choice (bv, bp)?  bp < 0: none yet
    if (bp < 0) return true;
    const bool vn = v != v, bn = bv != bv;  // NaN tests (false for integers)
    if (bn || vn) return vn && (!bn || p < bp);
    if (MAX) return v > bv || (!(bv > v) && p < bp);
    return v < bv || (!(bv < v) && p < bp);
}
template <bool MAX, bool INDEX, typename T, typename O>
__global__ void extreme_reduce_kernel(const T *__restrict__ x, Strided o, int64_t len, int64_t step,
                                      O *__restrict__ out, int64_t nout) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
    for (int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); w < nout;
         w += warps) {
        const T *base = x + offset_of(o, w);
        T best = T(0);
        int64_t bp = -1;
        for (int64_t k = lane; k < len; k += 32) {
            const T v = base[k * step];
            if (pick_better<MAX>(v, k, best, bp)) {
                best = v;
                bp = k;
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const T ov = __shfl_xor_sync(0xffffffffu, best, off);
            const int64_t op = __shfl_xor_sync(0xffffffffu, bp, off);
            if (op >= 0 && pick_better<MAX>(ov, op, best, bp)) {
                best = ov;
                bp = op;
            }
        }
        if (lane == 0) {
            if constexpr (INDEX) out[w] = static_cast<O>(bp);
            else out[w] = best;
        }
    }
}

// ProdReduce: the product in axis order from 1 (the C lane's `acc *= x`
// loop), one thread per output
template <typename T>
__global__ void prod_reduce_kernel(const T *__restrict__ x, Strided o, int64_t len, int64_t step,
                                   T *__restrict__ out, int64_t nout) {
    for (int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; w < nout;
         w += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const T *base = x + offset_of(o, w);
        T acc = T(1);
        for (int64_t k = 0; k < len; ++k) acc = acc * base[k * step];
        out[w] = acc;
    }
}
template <>
__global__ void prod_reduce_kernel<float>(const float *__restrict__ x, Strided o, int64_t len, int64_t step,
                                          float *__restrict__ out, int64_t nout) {
    for (int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; w < nout;
         w += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float *base = x + offset_of(o, w);
        float acc = 1.0f;
        for (int64_t k = 0; k < len; ++k) acc = __fmul_rn(acc, base[k * step]);
        out[w] = acc;
    }
}
template <>
__global__ void prod_reduce_kernel<double>(const double *__restrict__ x, Strided o, int64_t len, int64_t step,
                                           double *__restrict__ out, int64_t nout) {
    for (int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; w < nout;
         w += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const double *base = x + offset_of(o, w);
        double acc = 1.0;
        for (int64_t k = 0; k < len; ++k) acc = __dmul_rn(acc, base[k * step]);
        out[w] = acc;
    }
}

// FloatClassify ([05-OP-20..22]): is_nan / is_finite / is_infinite into bool bytes
template <typename T>
__global__ void classify_kernel(const T *__restrict__ x, Strided sx, int kind, uint8_t *__restrict__ out,
                                int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const auto v = CmpVal<T>::get(x[offset_of(sx, i)]);
        const bool r = kind == FC_NAN ? isnan(v) : kind == FC_FINITE ? isfinite(v) : isinf(v);
        out[i] = r ? 1 : 0;
    }
}

// ExtremaAdjoint ([05-OP-40]): the cotangent where `operand` was the
// selected side of max_elem / min_elem (left wins when it is NaN, or when
// right is not NaN and left >= right for max, <= for min), +0 elsewhere
template <typename T>
__global__ void extrema_adjoint_kernel(const T *__restrict__ a, Strided sa, const T *__restrict__ b, Strided sb,
                                       const T *__restrict__ g, Strided sg, int is_min, int right,
                                       T *__restrict__ out, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const T av = a[offset_of(sa, i)], bv = b[offset_of(sb, i)];
        const bool left = isnan(av) || (!isnan(bv) && (is_min ? av <= bv : av >= bv));
        out[i] = (right ? !left : left) ? g[offset_of(sg, i)] : T(0);
    }
}

// [05-RNG-2] derive(k, j) = splitmix64(k XOR rotl64(splitmix64(j), 29))
__device__ __forceinline__ uint64_t key_derive(uint64_t k, uint64_t j) {
    const uint64_t m = splitmix64(j);
    return splitmix64(k ^ ((m << 29) | (m >> 35)));
}

// Key operations, element-wise over the result: KEY_SEED key = the seed's
// bits ([05-OP-69]); KEY_SPLIT derive(k, branch) ([05-OP-70]); KEY_FOLD
// derive(derive(k, 2), n) ([05-OP-72]); KEY_SPLITN row j of `count` new keys
// derive(derive(k, 2), j) ([05-OP-71], the new axis last).
enum { KEY_SEED = 0, KEY_SPLIT, KEY_FOLD, KEY_SPLITN };
__global__ void key_kernel(const uint64_t *__restrict__ k, Strided sk, const int64_t *__restrict__ d,
                           Strided sd, int mode, int64_t arg, uint64_t *__restrict__ out, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        uint64_t r;
        switch (mode) {
            case KEY_SEED: r = static_cast<uint64_t>(d[offset_of(sd, i)]); break;
            case KEY_SPLIT: r = key_derive(k[offset_of(sk, i)], static_cast<uint64_t>(arg)); break;
            case KEY_FOLD:
                r = key_derive(key_derive(k[offset_of(sk, i)], 2), static_cast<uint64_t>(d[offset_of(sd, i)]));
                break;
            default: r = key_derive(key_derive(k[offset_of(sk, i / arg)], 2), static_cast<uint64_t>(i % arg)); break;
        }
        out[i] = r;
    }
}

// [05-OP-37] dropout under an explicit key, as the C lane draws it: the data
// splits into `rows` rows of `row_len` elements, one per key (a rank-0 key
// is one row); element e of row b is dropped when the unit value of
// word(key[b], e) -- the word's high 53 bits over 2^53, rounded to the draw's
// precision -- is below row b's rate, else it becomes x / (1 - rate) (NaN
// canonical).  A rate outside [0, 1) sets the device error word (the C
// lane's "numeric trap: domain in dropout").
template <typename T>
__global__ void keyed_dropout_kernel(const T *__restrict__ x, Strided sx, const T *__restrict__ rate,
                                     Strided sr, int64_t rate_size, const uint64_t *__restrict__ keys,
                                     Strided sk, int64_t rows, int64_t row_len, T *__restrict__ out,
                                     int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = i / row_len, e = i - b * row_len;
        const T r = rate[offset_of(sr, rate_size <= 1 ? 0 : b / (rows / rate_size))];
        if (!(r >= T(0) && r < T(1))) {
            report_device_error(sizeof(T) == 4 ? DEVERR_DROPOUT_F32 : DEVERR_DROPOUT_F64);
            out[i] = T(0);
            continue;
        }
        const uint64_t w = rng_word(keys[offset_of(sk, b)], static_cast<uint64_t>(e));
        const double u = static_cast<double>(w >> 11) * 0x1p-53;
        T y;
        if constexpr (sizeof(T) == 4) {
            y = __double2float_rn(u) < r ? 0.0f : canon(__fdiv_rn(x[offset_of(sx, i)], __fsub_rn(1.0f, r)));
        } else {
            const double q = __ddiv_rn(x[offset_of(sx, i)], __dsub_rn(1.0, r));
            y = u < r ? 0.0 : (isnan(q) ? __longlong_as_double(0x7ff8000000000000ll) : q);
        }
        out[i] = y;
    }
}

// Exact integer arithmetic at the stored width, as the C lane's checked
// helpers compute it (chelis_runtime.h chelis_int_checked_*): add, sub, mul
// and neg / abs of the minimum trap Overflow; trunc_div, floor_div and mod
// trap DivZero on a zero divisor, trunc_div and floor_div Overflow on MIN /
// -1, while mod by -1 is 0; floor_div rounds the quotient toward -inf and
// mod keeps the dividend's sign.  A trap is recorded on the device
// (report_trap) and the element is written as 0.  Float Mod is fmod.
template <typename T>
__device__ __forceinline__ T arith_int(T a, T b, int op, unsigned int dt) {
    constexpr T lo = sizeof(T) == 8 ? static_cast<T>(INT64_MIN) : sizeof(T) == 4 ? static_cast<T>(INT32_MIN)
                     : sizeof(T) == 2 ? static_cast<T>(INT16_MIN) : static_cast<T>(INT8_MIN);
    constexpr T hi = static_cast<T>(~lo);
    auto trap = [&](unsigned int kind, unsigned int top) -> T {
        report_trap(kind, top, dt);
        return T(0);
    };
    switch (op) {
        case IA_ADD: case IA_SUB: {
            if constexpr (sizeof(T) == 8) {
                const uint64_t ua = static_cast<uint64_t>(a), ub = static_cast<uint64_t>(b);
                const int64_t r = static_cast<int64_t>(op == IA_ADD ? ua + ub : ua - ub);
                const bool ovf = op == IA_ADD ? (((a ^ r) & (b ^ r)) < 0) : (((a ^ b) & (a ^ r)) < 0);
                return ovf ? trap(TRAP_OVERFLOW, op == IA_ADD ? TRAP_OP_ADD : TRAP_OP_SUB) : static_cast<T>(r);
            } else {
                const int64_t r = op == IA_ADD ? int64_t(a) + b : int64_t(a) - b;
                return (r < lo || r > hi) ? trap(TRAP_OVERFLOW, op == IA_ADD ? TRAP_OP_ADD : TRAP_OP_SUB)
                                          : static_cast<T>(r);
            }
        }
        case IA_MUL: {
            if constexpr (sizeof(T) == 8) {
                const int64_t p = static_cast<int64_t>(static_cast<uint64_t>(a) * static_cast<uint64_t>(b));
                const int64_t h = __mul64hi(static_cast<long long>(a), static_cast<long long>(b));
                return h != (p >> 63) ? trap(TRAP_OVERFLOW, TRAP_OP_MUL) : static_cast<T>(p);
            } else {
                const int64_t p = int64_t(a) * b;
                return (p < lo || p > hi) ? trap(TRAP_OVERFLOW, TRAP_OP_MUL) : static_cast<T>(p);
            }
        }
        case IA_TRUNC_DIV: case IA_FLOOR_DIV: {
            const unsigned int top = op == IA_TRUNC_DIV ? TRAP_OP_TRUNC_DIV : TRAP_OP_FLOOR_DIV;
            if (b == 0) return trap(TRAP_DIVZERO, top);
            if (a == lo && b == T(-1)) return trap(TRAP_OVERFLOW, top);
            T q = static_cast<T>(a / b);
            const T r = static_cast<T>(a % b);
            if (op == IA_FLOOR_DIV && r != 0 && ((r < 0) != (b < 0))) q = static_cast<T>(q - 1);
            return q;
        }
        case IA_MOD:
            if (b == T(-1)) return T(0);
            if (b == 0) return trap(TRAP_DIVZERO, TRAP_OP_MOD);
            return static_cast<T>(a % b);
        case IA_MAX: return a >= b ? a : b;
        case IA_MIN: return a <= b ? a : b;
        case IA_NEG: return a == lo ? trap(TRAP_OVERFLOW, TRAP_OP_NEG) : static_cast<T>(-a);
        case IA_ABS: return a == lo ? trap(TRAP_OVERFLOW, TRAP_OP_ABS) : static_cast<T>(a < 0 ? -a : a);
        case IA_AND: return static_cast<T>(a & b);
        case IA_OR: return static_cast<T>(a | b);
        case IA_XOR: return static_cast<T>(a ^ b);
        default: {
            // width-bounded two's-complement shifts (chelis_runtime.h
            // chelis_int_shl / _shr): a count of at least the width gives 0
            // (left) or the sign fill (right); a negative count is reported
            constexpr int bits = 8 * sizeof(T);
            const int64_t amount = static_cast<int64_t>(b);
            if (amount < 0) {
                atomicCAS(&g_shift_count, 0ull, static_cast<unsigned long long>(amount));
                atomicOr(&g_device_error, static_cast<unsigned int>(DEVERR_SHIFT));
                return T(0);
            }
            if (op == IA_SHL) {
                if (amount >= bits) return T(0);
                using U = typename std::make_unsigned<T>::type;
                return static_cast<T>(static_cast<U>(static_cast<U>(a) << amount));
            }
            if (amount >= bits) return a < 0 ? T(-1) : T(0);
            return static_cast<T>(a >> amount);  // arithmetic shift of a signed value
        }
    }
}
template <typename T>
__global__ void arith_kernel(const T *__restrict__ a, Strided sa, const T *__restrict__ b, Strided sb, int op,
                             unsigned int dt, T *__restrict__ out, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const T x = a[offset_of(sa, i)], y = b[offset_of(sb, i)];
        if constexpr (std::is_floating_point<T>::value) {
            const T r = fmod(x, y);  // Mod: exact ([05-OP-64]); NaN canonical
            if constexpr (sizeof(T) == 4) out[i] = r != r ? __int_as_float(0x7fc00000) : r;
            else out[i] = r != r ? __longlong_as_double(0x7ff8000000000000ll) : r;
        } else {
            out[i] = arith_int<T>(x, y, op, dt);
        }
    }
}

// [05-OP-8] uniform_like under an explicit key, as the C lane samples it:
// rows as for keyed dropout; element e of row b is fma(high - low, u, low)
// with u the unit value of word(key[b], e) and the span, u and the fma at the
// result's precision (f32: u rounded to f32, span in f32, fmaf).  A row whose
// bounds are non-finite, reversed or give a non-finite span traps Domain.
template <typename T>
__global__ void keyed_uniform_kernel(const T *__restrict__ lo, Strided sl, int64_t lo_size,
                                     const T *__restrict__ hi, Strided sh, int64_t hi_size,
                                     const uint64_t *__restrict__ keys, Strided sk, int64_t rows, int64_t row_len,
                                     T *__restrict__ out, int64_t n, unsigned int dt) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t b = i / row_len, e = i - b * row_len;
        const T l = lo[offset_of(sl, lo_size <= 1 ? 0 : b / (rows / lo_size))];
        const T h = hi[offset_of(sh, hi_size <= 1 ? 0 : b / (rows / hi_size))];
        const T span = h - l;
        if (!(isfinite(l) && isfinite(h) && l <= h && isfinite(span))) {
            report_trap(TRAP_DOMAIN, TRAP_OP_UNIFORM_LIKE, dt);
            out[i] = T(0);
            continue;
        }
        const uint64_t w = rng_word(keys[offset_of(sk, b)], static_cast<uint64_t>(e));
        const double u = static_cast<double>(w >> 11) * 0x1p-53;
        if constexpr (sizeof(T) == 4) out[i] = __fmaf_rn(span, __double2float_rn(u), l);
        else out[i] = __fma_rn(span, u, l);
    }
}

// [05-OP-54] range(start, end) into a declared extent `len`: the count is
// max(end - start, 0), an overflowing difference traps Overflow and a count
// other than the declared extent Domain (op "range"); element i is start + i.
__global__ void iota_kernel(const int64_t *__restrict__ start, const int64_t *__restrict__ end, int64_t len,
                            int64_t *__restrict__ out) {
    const int64_t s = *start, e = *end;
    bool ok = true;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        const int64_t d = static_cast<int64_t>(static_cast<uint64_t>(e) - static_cast<uint64_t>(s));
        if (e > s && d < 0) {
            report_trap(TRAP_OVERFLOW, TRAP_OP_RANGE, CHELIS_DTYPE_I64);
            ok = false;
        } else if ((e <= s ? 0 : d) != len) {
            report_trap(TRAP_DOMAIN, TRAP_OP_RANGE, CHELIS_DTYPE_I64);
            ok = false;
        }
    }
    (void)ok;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < len;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = static_cast<int64_t>(static_cast<uint64_t>(s) + static_cast<uint64_t>(i));
}

// Window geometry: the input (rank axes, strides in elements), the output
// extents, and the trailing `nw` windowed axes' window and stride.
struct WinGeom {
    int32_t rank, nw;
    int64_t in_shape[kMaxRank], in_stride[kMaxRank], out_shape[kMaxRank];
    int64_t win[kMaxRank], step[kMaxRank];
    int64_t volume;
};

// The canonical adjacent-pair tree over a sequence of leaves (the C lane's
// carry tree: completed 2^d-leaf subtrees in level[d], the partial ones
// combined from the lowest level up at the end).
template <typename T>
struct LeafTree {
    T level[24];
    uint32_t count = 0;
    template <typename Add>
    __device__ void push(T v, Add add) {
        int d = 0;
        for (uint32_t c = count; c & 1u; c >>= 1, ++d) v = add(level[d], v);
        level[d] = v;
        ++count;
    }
    template <typename Add>
    __device__ T total(Add add) const {
        T tot = T(0);
        bool found = false;
        for (int d = 0; d < 24; ++d)
            if ((count >> d) & 1u) {
                tot = found ? add(level[d], tot) : level[d];
                found = true;
            }
        return tot;
    }
};

template <typename T>
__device__ __forceinline__ T win_add(T a, T b, unsigned int dt) {
    if constexpr (std::is_floating_point<T>::value) {
        return a + b;
    } else {
        // checked at the stored width; an overflow traps in reduce_window_sum
        bool ovf;
        T r;
        if constexpr (sizeof(T) == 8) {
            const int64_t q = static_cast<int64_t>(static_cast<uint64_t>(a) + static_cast<uint64_t>(b));
            ovf = ((a ^ q) & (b ^ q)) < 0;
            r = static_cast<T>(q);
        } else {
            const int64_t q = int64_t(a) + b;
            ovf = q < int64_t(std::numeric_limits<T>::min()) || q > int64_t(std::numeric_limits<T>::max());
            r = static_cast<T>(q);
        }
        if (ovf) {
            report_trap(TRAP_OVERFLOW, TRAP_OP_REDUCE_WINDOW_SUM, dt);
            return T(0);
        }
        return r;
    }
}

// offset of window leaf `leaf` (row-major over the window) of output `o`
__device__ __forceinline__ int64_t win_base(const WinGeom &g, int64_t o) {
    int64_t off = 0;
    const int lead = g.rank - g.nw;
    for (int d = g.rank - 1; d >= 0; --d) {
        const int64_t c = o % g.out_shape[d];
        o /= g.out_shape[d];
        off += (d >= lead ? c * g.step[d - lead] : c) * g.in_stride[d];
    }
    return off;
}
__device__ __forceinline__ int64_t win_leaf(const WinGeom &g, int64_t leaf) {
    int64_t off = 0;
    const int lead = g.rank - g.nw;
    for (int j = g.nw - 1; j >= 0; --j) {
        off += (leaf % g.win[j]) * g.in_stride[lead + j];
        leaf /= g.win[j];
    }
    return off;
}

// [05-OP-39] forward: max / min pick in row-major window order (first NaN,
// else the first extreme); sum / mean combine the leaves by the canonical
// tree at the operand width (integers checked: overflow in
// reduce_window_sum), mean dividing the root by the window volume.
template <typename T>
__global__ void window_reduce_kernel(const T *__restrict__ x, WinGeom g, int kind, T *__restrict__ out,
                                     int64_t nout, unsigned int dt) {
    for (int64_t o = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; o < nout;
         o += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const T *base = x + win_base(g, o);
        if (kind == RW_MAX || kind == RW_MIN) {
            T best = T(0);
            int64_t bp = -1;
            for (int64_t l = 0; l < g.volume; ++l) {
                const T v = base[win_leaf(g, l)];
                const bool better = kind == RW_MAX ? pick_better<true>(v, l, best, bp) : pick_better<false>(v, l, best, bp);
                if (better) {
                    best = v;
                    bp = l;
                }
            }
            out[o] = best;
        } else {
            LeafTree<T> t;
            auto add = [&](T a, T b) { return win_add<T>(a, b, dt); };
            for (int64_t l = 0; l < g.volume; ++l) t.push(base[win_leaf(g, l)], add);
            T r = t.total(add);
            if constexpr (std::is_floating_point<T>::value) {
                if (kind == RW_MEAN) r = r / static_cast<T>(g.volume);
                out[o] = r != r ? (sizeof(T) == 4 ? T(__int_as_float(0x7fc00000)) : T(__longlong_as_double(0x7ff8000000000000ll))) : r;
            } else {
                out[o] = r;
            }
        }
    }
}

// OrderedAdjointSum: the leaves are each group's columns interleaved row
// first, then input order, groups in order; the result is their
// adjacent-pair tree (level by level, an odd last element carried up).  One
// block: thread t folds the aligned run of `chunk` leaves (a power of two)
// starting at t * chunk, which is a complete subtree of that tree (the last
// run is the tree of what remains), then the block pairs the runs' sums level
// by level in shared memory.  One leaf is the adjoint unchanged; a NaN made by
// the additions is written canonical; no leaves give +0.
constexpr int kAdjointThreads = 1024;
struct AdjointLeaves {
    const void *ptr[kMaxAdjointInputs];
    int64_t stride[kMaxAdjointInputs];
    int32_t first[kMaxAdjointInputs];   // a group's first input
    int32_t width[kMaxAdjointInputs];   // its input count
    int64_t leaf0[kMaxAdjointInputs + 1];  // its first leaf
    int32_t ngroups;
};

template <typename T>
__device__ __forceinline__ T adjoint_leaf(const AdjointLeaves &a, int64_t l) {
    int g = 0;
    while (g + 1 < a.ngroups && l >= a.leaf0[g + 1]) ++g;
    const int64_t r = (l - a.leaf0[g]) / a.width[g];
    const int in = a.first[g] + static_cast<int>((l - a.leaf0[g]) % a.width[g]);
    return static_cast<const T *>(a.ptr[in])[r * a.stride[in]];
}

// The adjacent-pair tree of leaf(0 .. n) folded by one block of NT threads:
// thread t folds the aligned run of `chunk` leaves (a power of two with
// ceil(n / chunk) <= NT) starting at t * chunk, a complete subtree of the
// tree (the last run is the tree of what remains), then the block pairs the
// runs' sums level by level in `part`.  Every thread returns the total; no
// leaves give +0.  The leaf function is expected to round its own products
// (no contraction into the additions).
template <typename T, int NT, typename Leaf>
__device__ T block_pair_tree(int64_t n, int64_t chunk, Leaf leaf, T *part) {
    const int64_t runs = (n + chunk - 1) / chunk;
    auto add = [](T x, T y) { return x + y; };
    for (int64_t t = threadIdx.x; t < runs; t += NT) {
        LeafTree<T> tree;
        const int64_t lo = t * chunk, hi = lo + chunk < n ? lo + chunk : n;
        for (int64_t l = lo; l < hi; ++l) tree.push(leaf(l), add);
        part[t] = tree.total(add);
    }
    __syncthreads();
    for (int64_t m = runs; m > 1; m = (m + 1) / 2) {
        T v = T(0);
        const int64_t j = threadIdx.x;
        if (j < (m + 1) / 2) v = 2 * j + 1 < m ? part[2 * j] + part[2 * j + 1] : part[2 * j];
        __syncthreads();
        if (j < (m + 1) / 2) part[j] = v;
        __syncthreads();
    }
    const T r = runs > 0 ? part[0] : T(0);
    __syncthreads();  // `part` may be reused by the caller
    return r;
}

template <typename T>
__global__ void __launch_bounds__(kAdjointThreads) ordered_adjoint_sum_kernel(AdjointLeaves a, int64_t n, int64_t chunk,
                                                                              T *__restrict__ out) {
    __shared__ T part[kAdjointThreads];
    const T r = block_pair_tree<T, kAdjointThreads>(n, chunk, [&](int64_t l) { return adjoint_leaf<T>(a, l); }, part);
    if (threadIdx.x == 0) *out = n > 1 ? canonical_nan(r) : r;
}

// [05-OP-8] the pathwise adjoint of a UniformLike bound: element i of the
// cotangent g contributes g_i * (1 - u_i) to `low` and g_i * u_i to `high`,
// u_i the forward draw's unit (rounded to f32 for an f32 draw), each product
// and the sum at the draw's precision.  Result element e (one block) sums by
// one adjacent-pair tree the rows of g whose keys fall in its leading-part
// group, in row-major order.
constexpr int kBoundThreads = 256;
template <typename T>
__global__ void __launch_bounds__(kBoundThreads) uniform_bound_adjoint_kernel(
    const T *__restrict__ g, Strided sg, const uint64_t *__restrict__ keys, Strided sk, int64_t row_len,
    int64_t rows_per_group, int64_t chunk, int high, T *__restrict__ out) {
    __shared__ T part[kBoundThreads];
    const int64_t e = blockIdx.x, n = rows_per_group * row_len, base = e * n;
    auto leaf = [&](int64_t l) -> T {
        const int64_t i = base + l, b = i / row_len, k = i - b * row_len;
        const uint64_t w = rng_word(keys[offset_of(sk, b)], static_cast<uint64_t>(k));
        const double u = static_cast<double>(w >> 11) * 0x1p-53;
        const T x = g[offset_of(sg, i)];
        if constexpr (sizeof(T) == 4) {
            const float uf = __double2float_rn(u);
            return __fmul_rn(x, high ? uf : __fsub_rn(1.0f, uf));
        } else {
            return __dmul_rn(x, high ? u : __dsub_rn(1.0, u));
        }
    };
    const T r = block_pair_tree<T, kBoundThreads>(n, chunk, leaf, part);
    if (threadIdx.x == 0) out[e] = canonical_nan(r);
}

// ReduceWindowGrad: input position p folds, by the canonical tree in window
// order, the contributions of the windows covering it: g (sum), g / volume
// (mean); for max / min only where p is the window's first NaN (full g) or,
// with no NaN, one of its k values equal to the extreme (g / k).
template <typename T>
__global__ void window_grad_kernel(const T *__restrict__ x, const T *__restrict__ gr, WinGeom g, int kind,
                                   T *__restrict__ out, int64_t nin) {
    const int lead = g.rank - g.nw;
    for (int64_t p = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; p < nin;
         p += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        int64_t c[kMaxRank], lo[kMaxRank], hi[kMaxRank], cur[kMaxRank];
        int64_t q = p, xoff = 0;
        for (int d = g.rank - 1; d >= 0; --d) {
            c[d] = q % g.in_shape[d];
            q /= g.in_shape[d];
            xoff += c[d] * g.in_stride[d];
        }
        bool any = true;
        for (int j = 0; j < g.nw; ++j) {
            const int64_t i = c[lead + j], w = g.win[j], s = g.step[j];
            const int64_t a = i - w + 1;
            lo[j] = a <= 0 ? 0 : (a + s - 1) / s;
            hi[j] = i / s;
            if (hi[j] > g.out_shape[lead + j] - 1) hi[j] = g.out_shape[lead + j] - 1;
            if (lo[j] > hi[j]) any = false;
            cur[j] = lo[j];
        }
        LeafTree<T> t;
        auto add = [](T a, T b) { return a + b; };
        const T xp = x[xoff];
        while (any) {
            // output index of window `cur` (leading coordinates those of p)
            int64_t o = 0;
            for (int d = 0; d < g.rank; ++d) o = o * g.out_shape[d] + (d < lead ? c[d] : cur[d - lead]);
            T contribution = gr[o];
            bool push = true;
            if (kind == RW_MEAN) {
                contribution = contribution / static_cast<T>(g.volume);
            } else if (kind == RW_MAX || kind == RW_MIN) {
                const T *base = x + win_base(g, o);
                T best = T(0);
                int64_t bp = -1;
                for (int64_t l = 0; l < g.volume; ++l) {
                    const T v = base[win_leaf(g, l)];
                    const bool better = kind == RW_MAX ? pick_better<true>(v, l, best, bp) : pick_better<false>(v, l, best, bp);
                    if (better) {
                        best = v;
                        bp = l;
                    }
                }
                if (best != best) {
                    push = base + win_leaf(g, bp) == x + xoff;
                } else if (!(xp == best)) {
                    push = false;
                } else {
                    int64_t ties = 0;
                    for (int64_t l = 0; l < g.volume; ++l) ties += base[win_leaf(g, l)] == best ? 1 : 0;
                    contribution = contribution / static_cast<T>(ties);
                }
            }
            if (push) t.push(contribution, add);
            // next covering window, row-major
            int j = g.nw - 1;
            while (j >= 0 && cur[j] == hi[j]) {
                cur[j] = lo[j];
                --j;
            }
            if (j < 0) break;
            ++cur[j];
        }
        const T r = t.total(add);
        out[p] = r != r ? (sizeof(T) == 4 ? T(__int_as_float(0x7fc00000)) : T(__longlong_as_double(0x7ff8000000000000ll))) : r;
    }
}

unsigned grid_for(int64_t n) {
    int64_t b = (n + 255) / 256;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
    if (b > cap) b = cap;
    return static_cast<unsigned>(b < 1 ? 1 : b);
}

// ---------------------------------------------------------------- running

struct Value {
    char *ptr = nullptr;  // element (0, ..., 0)
    chelis_dtype dtype = 0;
    std::vector<int64_t> shape, strides;
};

Strided strided(const Value &v) {
    Strided s{};
    s.rank = static_cast<int32_t>(v.shape.size());
    for (int d = 0; d < s.rank; ++d) {
        s.shape[d] = v.shape[d];
        s.stride[d] = v.strides[d];
    }
    if (s.rank == 0) {
        s.rank = 1;
        s.shape[0] = 1;
        s.stride[0] = 1;
    }
    return s;
}

template <typename From>
void launch_named_cast(const Value &x, char *out, int64_t cnt, chelis_dtype to, int mode, cudaStream_t s) {
    const Strided sx = strided(x);
    const From *src = reinterpret_cast<const From *>(x.ptr);
    const unsigned int g = grid_for(cnt), d = static_cast<unsigned int>(to);
    switch (to) {
        case CHELIS_DTYPE_I64: named_cast_kernel<From, int64_t><<<g, 256, 0, s>>>(src, sx, mode, reinterpret_cast<int64_t *>(out), cnt, d); break;
        case CHELIS_DTYPE_I32: named_cast_kernel<From, int32_t><<<g, 256, 0, s>>>(src, sx, mode, reinterpret_cast<int32_t *>(out), cnt, d); break;
        case CHELIS_DTYPE_I16: named_cast_kernel<From, int16_t><<<g, 256, 0, s>>>(src, sx, mode, reinterpret_cast<int16_t *>(out), cnt, d); break;
        default: named_cast_kernel<From, int8_t><<<g, 256, 0, s>>>(src, sx, mode, reinterpret_cast<int8_t *>(out), cnt, d); break;
    }
}

// Cast of x (source type From) to the node's dtype: floats by C conversion,
// integers and bool by the checked cast (cast_checked_kernel).
template <typename From>
void launch_cast(const Value &x, char *out, int64_t cnt, chelis_dtype to, cudaStream_t s) {
    const Strided sx = strided(x);
    const From *src = reinterpret_cast<const From *>(x.ptr);
    const unsigned int g = grid_for(cnt), d = static_cast<unsigned int>(to);
    switch (to) {
        case CHELIS_DTYPE_F64: cast_kernel<From, double><<<g, 256, 0, s>>>(src, sx, reinterpret_cast<double *>(out), cnt); break;
        case CHELIS_DTYPE_F32: cast_kernel<From, float><<<g, 256, 0, s>>>(src, sx, reinterpret_cast<float *>(out), cnt); break;
        case CHELIS_DTYPE_I64: cast_checked_kernel<From, int64_t><<<g, 256, 0, s>>>(src, sx, reinterpret_cast<int64_t *>(out), cnt, d); break;
        case CHELIS_DTYPE_I32: cast_checked_kernel<From, int32_t><<<g, 256, 0, s>>>(src, sx, reinterpret_cast<int32_t *>(out), cnt, d); break;
        case CHELIS_DTYPE_I16: cast_checked_kernel<From, int16_t><<<g, 256, 0, s>>>(src, sx, reinterpret_cast<int16_t *>(out), cnt, d); break;
        case CHELIS_DTYPE_I8: cast_checked_kernel<From, int8_t><<<g, 256, 0, s>>>(src, sx, reinterpret_cast<int8_t *>(out), cnt, d); break;
        default: cast_checked_kernel<From, uint8_t><<<g, 256, 0, s>>>(src, sx, reinterpret_cast<uint8_t *>(out), cnt, d); break;
    }
}

template <typename T>
int launch_copy(const Value &src, void *dst, int64_t n, cudaStream_t s) {
    if (n == 0) return CHELIS_CUDA_OK;
    copy_kernel<T><<<grid_for(n), 256, 0, s>>>(reinterpret_cast<const T *>(src.ptr), strided(src),
                                               static_cast<T *>(dst), n);
    g_launches++;
    CHELIS_LAUNCH_CHECK("dag::copy_kernel");
    return CHELIS_CUDA_OK;
}

int materialize(const Value &src, void *dst, cudaStream_t s) {
    const int64_t n = count_of(src.shape);
    switch (dtype_width(src.dtype)) {
        case 8: return launch_copy<uint64_t>(src, dst, n, s);
        case 4: return launch_copy<uint32_t>(src, dst, n, s);
        case 2: return launch_copy<uint16_t>(src, dst, n, s);
        default: return launch_copy<uint8_t>(src, dst, n, s);
    }
}

struct Run {
    const Program &P;
    std::vector<Value> val;
    char *arena = nullptr;
    std::vector<char *> out_ptr;  // device memory of each output owner
    std::vector<void *> temps;    // materialised operands, freed at the end
    cudaStream_t s;
    explicit Run(const Program &p) : P(p), val(p.nodes.size()) {}
    ~Run() {
        for (void *t : temps) scratch_free(t, s);
    }

    // a dense copy of `v` when it is not dense already
    int dense(Value &v) {
        if (is_dense(v.shape, v.strides)) return CHELIS_CUDA_OK;
        void *t = nullptr;
        const int64_t bytes = std::max<int64_t>(count_of(v.shape), 1) * dtype_width(v.dtype);
        CHELIS_TRY(scratch_alloc(&t, static_cast<size_t>(bytes), s));
        temps.push_back(t);
        CHELIS_TRY(materialize(v, t, s));
        v.ptr = static_cast<char *>(t);
        v.strides = dense_strides(v.shape);
        return CHELIS_CUDA_OK;
    }

    char *storage(int i) {
        if (P.place[i] == Place::Output) return out_ptr[P.direct_output[i]];
        return arena + P.slot_off[P.slot[i]];
    }

    int node(int i, const std::vector<const chelis_gpu_tensor *> &inputs);
};

int elementwise(const Node &n, const std::vector<const Value *> &ins,
                const std::vector<chelis_fused_step> &steps, void *out, int reduce_axis, int kind) {
    std::vector<int64_t> shape = reduce_axis >= 0 ? ins[0]->shape : n.shape;
    int rank = static_cast<int>(shape.size());
    std::vector<const void *> ptrs;
    std::vector<int64_t> strides;
    if (rank == 0) {  // a scalar group runs as shape [1]
        shape = {1};
        rank = 1;
    }
    if (rank > 6) return unsupported("an elementwise group of rank above 6");
    for (const Value *v : ins) {
        ptrs.push_back(v->ptr);
        if (v->shape.empty()) strides.push_back(1);
        else strides.insert(strides.end(), v->strides.begin(), v->strides.end());
    }
    if (reduce_axis >= 0)
        return chelis_cuda_fused_reduce(n.dtype, steps.data(), static_cast<int32_t>(steps.size()),
                                        ptrs.data(), strides.data(),
                                        static_cast<int32_t>(ptrs.size()), shape.data(), rank,
                                        reduce_axis, kind, out);
    return chelis_cuda_fused_elementwise(n.dtype, steps.data(), static_cast<int32_t>(steps.size()),
                                         ptrs.data(), strides.data(),
                                         static_cast<int32_t>(ptrs.size()), shape.data(), rank, out);
}

int Run::node(int i, const std::vector<const chelis_gpu_tensor *> &inputs) {
    const Node &n = P.nodes[i];
    Value &v = val[i];
    v.dtype = n.dtype;
    v.shape = n.shape;
    const Place pl = P.place[i];
    if (pl == Place::Inlined || pl == Place::Skip) return CHELIS_CUDA_OK;
    if (pl == Place::Input) {
        const chelis_gpu_tensor *t = inputs[P.input_of_load[i]];
        v.ptr = static_cast<char *>(t->data);
        v.strides.assign(t->strides, t->strides + t->rank);
        return CHELIS_CUDA_OK;
    }
    if (pl == Place::View) {
        // derived from the operand's run-time value (the plan's static
        // layouts agree, inputs having been made dense)
        const Value &src = val[n.in[0]];
        v.strides.assign(n.shape.size(), 0);
        v.ptr = src.ptr;
        const int w = dtype_width(n.dtype);
        switch (n.op) {
            case Op::Store: v.ptr = src.ptr; v.strides = src.strides; break;
            case Op::Reshape: v.strides = dense_strides(n.shape); break;
            case Op::Permute:
                for (size_t d = 0; d < n.axes.size(); ++d) v.strides[d] = src.strides[n.axes[d]];
                break;
            case Op::Expand:
                if (src.shape.size() + 1 == n.shape.size()) {
                    v.strides = src.strides;
                    v.strides.insert(v.strides.begin() + n.axis, 0);
                } else {
                    v.strides = src.strides;
                    v.strides[n.axis] = 0;
                }
                break;
            case Op::Shrink:
                v.strides = src.strides;
                for (size_t d = 0; d < n.bounds.size(); ++d)
                    v.ptr += n.bounds[d].first * src.strides[d] * w;
                break;
            case Op::Stride:
                v.strides = src.strides;
                for (size_t d = 0; d < n.step.size(); ++d) v.strides[d] *= n.step[d];
                break;
            default: return bad("view of an unexpected op");
        }
        return CHELIS_CUDA_OK;
    }
    // a node with its own storage
    char *out = storage(i);
    v.ptr = out;
    v.strides = dense_strides(n.shape);
    const int64_t cnt = count_of(n.shape);
    const int w = dtype_width(n.dtype);
    auto in = [&](int k) -> Value & { return val[n.in[k]]; };
    switch (n.op) {
        case Op::ExtentWitness: case Op::CheckedExtent:
            if (!n.message.empty()) return set_error(CHELIS_CUDA_ERR_DOMAIN, "%s", n.message.c_str());
            // fall through: the extent is a constant
        case Op::Const: case Op::Shape: {
            if (cnt == 0) return CHELIS_CUDA_OK;
            switch (w) {
                case 8: fill_kernel<uint64_t><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<uint64_t *>(out), n.bits, cnt); break;
                case 4: fill_kernel<uint32_t><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<uint32_t *>(out), static_cast<uint32_t>(n.bits), cnt); break;
                case 2: fill_kernel<uint16_t><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<uint16_t *>(out), static_cast<uint16_t>(n.bits), cnt); break;
                default: fill_kernel<uint8_t><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<uint8_t *>(out), static_cast<uint8_t>(n.bits), cnt); break;
            }
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::fill_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::ConstTensor:
            if (n.data.empty()) return CHELIS_CUDA_OK;
            return check_cuda(cudaMemcpyAsync(out, n.data.data(), n.data.size(), cudaMemcpyHostToDevice, s),
                              "ConstTensor upload");
        case Op::Copy: case Op::Reshape:
            return materialize(in(0), out, s);
        case Op::Elementwise: case Op::Fused: {
            std::vector<const Value *> ins;
            for (size_t k = 0; k < n.in.size(); ++k) ins.push_back(&in(static_cast<int>(k)));
            return elementwise(n, ins, n.steps, out, -1, 0);
        }
        case Op::Sum: case Op::MaxReduce: {
            const int kind = n.op == Op::Sum ? CHELIS_FUSED_REDUCE_SUM : CHELIS_FUSED_REDUCE_MAX;
            const int f = n.in[0];
            std::vector<const Value *> ins;
            std::vector<chelis_fused_step> steps;
            Value one;  // the multiplicative identity, broadcast: x * 1 is x exactly
            if (P.place[f] == Place::Inlined) {
                for (int j : P.nodes[f].in) ins.push_back(&val[j]);
                steps = P.nodes[f].steps;
            } else {
                ins.push_back(&in(0));
                void *t = nullptr;
                CHELIS_TRY(scratch_alloc(&t, 8, s));
                temps.push_back(t);
                if (n.dtype == CHELIS_DTYPE_F32)
                    fill_kernel<uint32_t><<<1, 32, 0, s>>>(static_cast<uint32_t *>(t), 0x3f800000u, 1);
                else
                    fill_kernel<uint64_t><<<1, 32, 0, s>>>(static_cast<uint64_t *>(t), 0x3ff0000000000000ull, 1);
                g_launches++;
                CHELIS_LAUNCH_CHECK("dag::fill_kernel");
                one.ptr = static_cast<char *>(t);
                one.dtype = n.dtype;
                one.shape = in(0).shape;
                one.strides.assign(one.shape.size(), 0);
                ins.push_back(&one);
                steps.push_back({CHELIS_FUSED_MUL, 0, 1});
            }
            return elementwise(n, ins, steps, out, n.axis, kind);
        }
        case Op::Relu: {
            Value x = in(0);
            CHELIS_TRY(dense(x));
            return chelis_cuda_relu(n.dtype, x.ptr, out, cnt);
        }
        case Op::ReluAdjoint: {
            Value x = in(0), g = in(1);
            CHELIS_TRY(dense(x));
            CHELIS_TRY(dense(g));
            return chelis_cuda_relu_adjoint(n.dtype, x.ptr, g.ptr, out, cnt);
        }
        case Op::Softmax: {
            Value x = in(0);
            CHELIS_TRY(dense(x));
            const int64_t cols = n.shape.back();
            return chelis_cuda_softmax_rows_f32(reinterpret_cast<const float *>(x.ptr),
                                                reinterpret_cast<float *>(out),
                                                cols ? cnt / cols : 0, cols);
        }
        case Op::Cumsum: {
            if (n.axis != static_cast<int>(n.shape.size()) - 1) {
                // a leading axis: one thread per line, the scan in axis order
                const Value &x = in(0);
                const int64_t len = n.shape[n.axis];
                const int64_t lanes = len ? cnt / len : 0;
                if (lanes == 0) return CHELIS_CUDA_OK;
                Strided lines{}, o{};
                const std::vector<int64_t> ds = dense_strides(n.shape);
                for (int d = 0; d < static_cast<int>(n.shape.size()); ++d) {
                    if (d == n.axis) continue;
                    lines.shape[lines.rank] = o.shape[o.rank] = n.shape[d];
                    lines.stride[lines.rank++] = x.strides[d];
                    o.stride[o.rank++] = ds[d];
                }
                if (n.dtype == CHELIS_DTYPE_F64)
                    cumsum_axis_kernel<double><<<grid_for(lanes), 256, 0, s>>>(
                        reinterpret_cast<const double *>(x.ptr), lines, x.strides[n.axis], o, ds[n.axis], len,
                        n.reverse, reinterpret_cast<double *>(out), lanes);
                else
                    cumsum_axis_kernel<float><<<grid_for(lanes), 256, 0, s>>>(
                        reinterpret_cast<const float *>(x.ptr), lines, x.strides[n.axis], o, ds[n.axis], len,
                        n.reverse, reinterpret_cast<float *>(out), lanes);
                g_launches++;
                CHELIS_LAUNCH_CHECK("dag::cumsum_axis_kernel");
                return CHELIS_CUDA_OK;
            }
            Value x = in(0);
            CHELIS_TRY(dense(x));
            const int64_t len = n.shape.back();
            const int64_t lanes = len ? cnt / len : 0;
            return n.dtype == CHELIS_DTYPE_F64
                       ? chelis_cuda_cumsum_f64(reinterpret_cast<const double *>(x.ptr),
                                                reinterpret_cast<double *>(out), lanes, len, n.reverse)
                       : chelis_cuda_cumsum_f32(reinterpret_cast<const float *>(x.ptr),
                                                reinterpret_cast<float *>(out), lanes, len, n.reverse);
        }
        case Op::Count: {
            const Value &x = in(0);
            if (n.shape.empty()) {
                Value d = x;
                CHELIS_TRY(dense(d));
                return chelis_cuda_count_bool(reinterpret_cast<const uint8_t *>(d.ptr), count_of(d.shape),
                                              reinterpret_cast<int64_t *>(out));
            }
            if (cnt == 0) return CHELIS_CUDA_OK;
            Strided kept{}, counted{};
            for (int d = 0; d < static_cast<int>(x.shape.size()); ++d) {
                Strided &t = std::find(n.axes.begin(), n.axes.end(), d) == n.axes.end() ? kept : counted;
                t.shape[t.rank] = x.shape[d];
                t.stride[t.rank] = x.strides[d];
                ++t.rank;
            }
            const int64_t volume = count_of(in(0).shape) / cnt;
            const unsigned grid = static_cast<unsigned>(cnt < 65535 ? cnt : 65535);
            count_axes_kernel<<<grid, 128, 0, s>>>(reinterpret_cast<const uint8_t *>(x.ptr), kept, counted, cnt,
                                                   volume, reinterpret_cast<int64_t *>(out));
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::count_axes_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::Matmul: {
            const int r = static_cast<int>(n.shape.size());
            const int64_t m = n.shape[r - 2], nn = n.shape[r - 1], k = in(0).shape[r - 1];
            int64_t batch = 1;
            for (int d = 0; d + 2 < r; ++d) batch *= n.shape[d];
            // an operand is used in place when its matrix is dense or a
            // dense transpose and its batch axes collapse to one stride
            auto operand = [&](Value &x, int *trans, int64_t *ld, int64_t *bstride) -> int {
                for (int pass = 0; pass < 2; ++pass) {
                    const int64_t s1 = x.strides[r - 1], s0 = x.strides[r - 2];
                    const int64_t rows = x.shape[r - 2], cols = x.shape[r - 1];
                    bool ok = true;
                    if (s1 == 1 && (s0 >= cols || rows == 1)) {
                        *trans = 0;
                        *ld = rows == 1 ? cols : s0;
                    } else if (s0 == 1 && (s1 >= rows || cols == 1)) {
                        *trans = 1;
                        *ld = cols == 1 ? rows : s1;
                    } else {
                        ok = false;
                    }
                    // batch axes: one uniform stride over the flattened batch
                    int64_t bs = 0;
                    bool first = true;
                    for (int d = r - 3; d >= 0 && ok; --d) {
                        if (x.shape[d] == 1) continue;
                        if (first) {
                            bs = x.strides[d];
                            first = false;
                        } else {
                            int64_t inner = 1;
                            for (int e = d + 1; e <= r - 3; ++e) inner *= x.shape[e];
                            if (x.strides[d] != bs * inner) ok = false;
                        }
                    }
                    *bstride = bs;
                    if (ok && *ld >= 1) return CHELIS_CUDA_OK;
                    if (pass == 0) CHELIS_TRY(dense(x));
                }
                return bad("BlasMatmul operand layout");
            };
            Value a = in(0), b = in(1);
            int ta = 0, tb = 0;
            int64_t lda = 0, ldb = 0, sa = 0, sb = 0;
            CHELIS_TRY(operand(a, &ta, &lda, &sa));
            CHELIS_TRY(operand(b, &tb, &ldb, &sb));
            if (n.dtype == CHELIS_DTYPE_F32)
                return chelis_cuda_sgemm(ta, tb, m, nn, k, reinterpret_cast<const float *>(a.ptr), lda,
                                         sa, reinterpret_cast<const float *>(b.ptr), ldb, sb,
                                         reinterpret_cast<float *>(out), nn, m * nn, batch);
            return chelis_cuda_dgemm(ta, tb, m, nn, k, reinterpret_cast<const double *>(a.ptr), lda, sa,
                                     reinterpret_cast<const double *>(b.ptr), ldb, sb,
                                     reinterpret_cast<double *>(out), nn, m * nn, batch);
        }
        case Op::Gather: case Op::ScatterAdd: case Op::Scatter: {
            const Value &vals = in(0);
            const Value &idx = in(1);
            GatherGeom g{};
            g.axis = n.axis;
            g.batch_rank = n.batch_rank;
            g.index_width = dtype_width(idx.dtype);
            g.x = strided(idx);
            g.qrank = static_cast<int32_t>(idx.shape.size()) - n.batch_rank;
            for (int d = 0; d < g.qrank; ++d) g.qshape[d] = idx.shape[n.batch_rank + d];
            g.trank = static_cast<int32_t>(vals.shape.size()) - n.axis - 1;
            for (int d = 0; d < g.trank; ++d) g.tshape[d] = vals.shape[n.axis + 1 + d];
            if (n.op == Op::Gather) {
                g.v = strided(vals);
                if (cnt == 0) return CHELIS_CUDA_OK;
                if (n.dtype == CHELIS_DTYPE_F64 || w == 8)
                    gather_kernel<uint64_t><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const uint64_t *>(vals.ptr), idx.ptr, g, reinterpret_cast<uint64_t *>(out), cnt);
                else if (w == 4)
                    gather_kernel<uint32_t><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const uint32_t *>(vals.ptr), idx.ptr, g, reinterpret_cast<uint32_t *>(out), cnt);
                else if (w == 2)
                    gather_kernel<uint16_t><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const uint16_t *>(vals.ptr), idx.ptr, g, reinterpret_cast<uint16_t *>(out), cnt);
                else
                    gather_kernel<uint8_t><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const uint8_t *>(vals.ptr), idx.ptr, g, reinterpret_cast<uint8_t *>(out), cnt);
                g_launches++;
                CHELIS_LAUNCH_CHECK("dag::gather_kernel");
                return CHELIS_CUDA_OK;
            }
            // ScatterAdd / Scatter: out = dense copy of the target, then the updates
            if (n.op == Op::ScatterAdd && n.dtype != CHELIS_DTYPE_F32 && n.dtype != CHELIS_DTYPE_F64)
                return unsupported("ScatterAdd on a non-float precision");
            CHELIS_TRY(materialize(vals, out, s));
            Value dense_out;
            dense_out.shape = n.shape;
            dense_out.strides = dense_strides(n.shape);
            g.v = strided(dense_out);
            const Value &upd = in(2);
            int64_t nq = 1;
            for (int d = 0; d < g.qrank; ++d) nq *= g.qshape[d];
            const int64_t lanes = nq ? count_of(upd.shape) / nq : 0;
            if (lanes == 0 || nq == 0) return CHELIS_CUDA_OK;
            if (n.op == Op::Scatter) {
                // replacement copies stored bits: any element width
#define CHELIS_DAG_SCATTER(T)                                                                              \
    scatter_add_kernel<T><<<grid_for(lanes), 256, 0, s>>>(reinterpret_cast<const T *>(upd.ptr), strided(upd), \
                                                          idx.ptr, g, reinterpret_cast<T *>(out), lanes, nq, 1)
                switch (dtype_width(n.dtype)) {
                    case 8: CHELIS_DAG_SCATTER(uint64_t); break;
                    case 4: CHELIS_DAG_SCATTER(uint32_t); break;
                    case 2: CHELIS_DAG_SCATTER(uint16_t); break;
                    default: CHELIS_DAG_SCATTER(uint8_t); break;
                }
#undef CHELIS_DAG_SCATTER
            } else if (n.dtype == CHELIS_DTYPE_F64) {
                scatter_add_kernel<double><<<grid_for(lanes), 256, 0, s>>>(reinterpret_cast<const double *>(upd.ptr), strided(upd), idx.ptr, g, reinterpret_cast<double *>(out), lanes, nq, 0);
            } else {
                scatter_add_kernel<float><<<grid_for(lanes), 256, 0, s>>>(reinterpret_cast<const float *>(upd.ptr), strided(upd), idx.ptr, g, reinterpret_cast<float *>(out), lanes, nq, 0);
            }
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::scatter_add_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::ScatterElements: {
            const Value &data = in(0), &idx = in(1), &upd = in(2);
            CHELIS_TRY(materialize(data, out, s));
            const int64_t len = upd.shape[n.axis];
            const int64_t nu = count_of(upd.shape);
            const int64_t lanes = len ? nu / len : 0;
            if (lanes == 0 || len == 0) return CHELIS_CUDA_OK;
            Value dense_out;
            dense_out.shape = n.shape;
            dense_out.strides = dense_strides(n.shape);
            const Strided so = strided(dense_out), su = strided(upd), si = strided(idx);
            const int iw = dtype_width(idx.dtype);
#define CHELIS_DAG_SCATTER_EL(T)                                                                           \
    scatter_elements_kernel<T><<<grid_for(lanes), 256, 0, s>>>(reinterpret_cast<const T *>(upd.ptr), su, idx.ptr, \
                                                               si, iw, so, n.axis, reinterpret_cast<T *>(out),    \
                                                               lanes, len)
            switch (dtype_width(n.dtype)) {
                case 8: CHELIS_DAG_SCATTER_EL(uint64_t); break;
                case 4: CHELIS_DAG_SCATTER_EL(uint32_t); break;
                case 2: CHELIS_DAG_SCATTER_EL(uint16_t); break;
                default: CHELIS_DAG_SCATTER_EL(uint8_t); break;
            }
#undef CHELIS_DAG_SCATTER_EL
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::scatter_elements_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::Pad: {
            const Value &x = in(0);
            if (cnt == 0) return CHELIS_CUDA_OK;
            Strided o{}, before{};
            Value dense_out;
            dense_out.shape = n.shape;
            dense_out.strides = dense_strides(n.shape);
            o = strided(dense_out);
            Strided sx = strided(x);
            before.rank = o.rank;
            for (size_t d = 0; d < n.bounds.size(); ++d) before.shape[d] = n.bounds[d].first;
            if (x.shape.empty()) sx.shape[0] = 1;
            if (w == 8)
                pad_kernel<uint64_t><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const uint64_t *>(x.ptr), sx, o, before, n.bits, reinterpret_cast<uint64_t *>(out), cnt);
            else if (w == 4)
                pad_kernel<uint32_t><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const uint32_t *>(x.ptr), sx, o, before, static_cast<uint32_t>(n.bits), reinterpret_cast<uint32_t *>(out), cnt);
            else if (w == 2)
                pad_kernel<uint16_t><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const uint16_t *>(x.ptr), sx, o, before, static_cast<uint16_t>(n.bits), reinterpret_cast<uint16_t *>(out), cnt);
            else
                pad_kernel<uint8_t><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const uint8_t *>(x.ptr), sx, o, before, static_cast<uint8_t>(n.bits), reinterpret_cast<uint8_t *>(out), cnt);
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::pad_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::Cast: {
            const Value &x = in(0);
            if (cnt == 0) return CHELIS_CUDA_OK;
            switch (x.dtype) {
                case CHELIS_DTYPE_F32: launch_cast<float>(x, out, cnt, n.dtype, s); break;
                case CHELIS_DTYPE_F64: launch_cast<double>(x, out, cnt, n.dtype, s); break;
                case CHELIS_DTYPE_I8: launch_cast<int8_t>(x, out, cnt, n.dtype, s); break;
                case CHELIS_DTYPE_I16: launch_cast<int16_t>(x, out, cnt, n.dtype, s); break;
                case CHELIS_DTYPE_I32: launch_cast<int32_t>(x, out, cnt, n.dtype, s); break;
                case CHELIS_DTYPE_I64: launch_cast<int64_t>(x, out, cnt, n.dtype, s); break;
                default: launch_cast<uint8_t>(x, out, cnt, n.dtype, s); break;  // bool: 0 / 1
            }
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::cast_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::GuardedFail: {
            const Value &c = in(0);
            const int64_t nc = count_of(c.shape);
            if (nc > 0) {
                guard_kernel<<<grid_for(nc), 256, 0, s>>>(reinterpret_cast<const uint8_t *>(c.ptr), strided(c),
                                                          n.kind, n.fail_id, nc);
                g_launches++;
                CHELIS_LAUNCH_CHECK("dag::guard_kernel");
            }
            return materialize(in(1), out, s);
        }
        case Op::NamedCast: {
            const Value &x = in(0);
            if (cnt == 0) return CHELIS_CUDA_OK;
            switch (x.dtype) {
                case CHELIS_DTYPE_F32: launch_named_cast<float>(x, out, cnt, n.dtype, n.kind, s); break;
                case CHELIS_DTYPE_F64: launch_named_cast<double>(x, out, cnt, n.dtype, n.kind, s); break;
                case CHELIS_DTYPE_I8: launch_named_cast<int8_t>(x, out, cnt, n.dtype, n.kind, s); break;
                case CHELIS_DTYPE_I16: launch_named_cast<int16_t>(x, out, cnt, n.dtype, n.kind, s); break;
                case CHELIS_DTYPE_I32: launch_named_cast<int32_t>(x, out, cnt, n.dtype, n.kind, s); break;
                default: launch_named_cast<int64_t>(x, out, cnt, n.dtype, n.kind, s); break;
            }
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::named_cast_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::Compare: {
            const Value &a = in(0), &b = in(1);
            if (cnt == 0) return CHELIS_CUDA_OK;
            const Strided sa = strided(a), sb = strided(b);
            uint8_t *o = reinterpret_cast<uint8_t *>(out);
#define CHELIS_DAG_CMP(T)                                                                                \
    compare_kernel<T><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const T *>(a.ptr), sa,             \
                                                    reinterpret_cast<const T *>(b.ptr), sb, n.kind, o, cnt)
            switch (a.dtype) {
                case CHELIS_DTYPE_F32: CHELIS_DAG_CMP(float); break;
                case CHELIS_DTYPE_F64: CHELIS_DAG_CMP(double); break;
                case CHELIS_DTYPE_I32: CHELIS_DAG_CMP(int32_t); break;
                case CHELIS_DTYPE_I64: CHELIS_DAG_CMP(int64_t); break;
                case CHELIS_DTYPE_I16: CHELIS_DAG_CMP(int16_t); break;
                case CHELIS_DTYPE_I8: CHELIS_DAG_CMP(int8_t); break;
                case CHELIS_DTYPE_BF16: CHELIS_DAG_CMP(Bf16Bits); break;
                case CHELIS_DTYPE_F16: CHELIS_DAG_CMP(F16Bits); break;
                default: CHELIS_DAG_CMP(uint8_t); break;  // bool: eq / neq of the stored 0 / 1
            }
#undef CHELIS_DAG_CMP
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::compare_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::Logical: {
            const Value &a = in(0);
            const Value &b = n.kind == LOG_NOT ? in(0) : in(1);
            if (cnt == 0) return CHELIS_CUDA_OK;
            logical_kernel<<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const uint8_t *>(a.ptr), strided(a),
                                                         reinterpret_cast<const uint8_t *>(b.ptr), strided(b),
                                                         n.kind, reinterpret_cast<uint8_t *>(out), cnt);
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::logical_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::Where: {
            const Value &c = in(0), &a = in(1), &b = in(2);
            if (cnt == 0) return CHELIS_CUDA_OK;
            const Strided sc = strided(c), sa = strided(a), sb = strided(b);
            const uint8_t *cp = reinterpret_cast<const uint8_t *>(c.ptr);
#define CHELIS_DAG_WHERE(T)                                                                               \
    where_kernel<T><<<grid_for(cnt), 256, 0, s>>>(cp, sc, reinterpret_cast<const T *>(a.ptr), sa,          \
                                                  reinterpret_cast<const T *>(b.ptr), sb,                \
                                                  reinterpret_cast<T *>(out), cnt)
            switch (dtype_width(n.dtype)) {
                case 8: CHELIS_DAG_WHERE(uint64_t); break;
                case 4: CHELIS_DAG_WHERE(uint32_t); break;
                case 2: CHELIS_DAG_WHERE(uint16_t); break;
                default: CHELIS_DAG_WHERE(uint8_t); break;
            }
#undef CHELIS_DAG_WHERE
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::where_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::MinReduce: case Op::Argmax: case Op::Argmin: case Op::ProdReduce: {
            const Value &x = in(0);
            const int64_t len = x.shape[n.axis];
            if (len == 0 && n.op != Op::ProdReduce) {
                static const char *const names[] = {"f32", "f64", "i32", "bool", "i64"};
                const char *what = n.op == Op::MinReduce ? "min_reduce"
                                   : n.op == Op::Argmax  ? "argmax_reduce"
                                                         : "argmin_reduce";
                return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in %s at %s", what,
                                 n.op == Op::MinReduce ? names[n.dtype] : "i64");
            }
            if (cnt == 0) return CHELIS_CUDA_OK;
            // outputs walk the input's other axes; the reduced axis is `step` apart
            Strided o{};
            o.rank = 0;
            for (size_t d = 0; d < x.shape.size(); ++d) {
                if (static_cast<int>(d) == n.axis) continue;
                o.shape[o.rank] = x.shape[d];
                o.stride[o.rank] = x.strides[d];
                ++o.rank;
            }
            const int64_t step = x.strides[n.axis];
            int64_t blocks = (cnt + 7) / 8;
            const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
            if (blocks > cap) blocks = cap;
            const unsigned gb = static_cast<unsigned>(blocks);
            int64_t *idx = reinterpret_cast<int64_t *>(out);
#define CHELIS_DAG_EXTREME(T)                                                                              \
    do {                                                                                                   \
        const T *xp = reinterpret_cast<const T *>(x.ptr);                                                  \
        if (n.op == Op::MinReduce)                                                                         \
            extreme_reduce_kernel<false, false, T, T><<<gb, 256, 0, s>>>(xp, o, len, step, reinterpret_cast<T *>(out), cnt); \
        else if (n.op == Op::Argmax)                                                                       \
            extreme_reduce_kernel<true, true, T, int64_t><<<gb, 256, 0, s>>>(xp, o, len, step, idx, cnt);  \
        else if (n.op == Op::Argmin)                                                                       \
            extreme_reduce_kernel<false, true, T, int64_t><<<gb, 256, 0, s>>>(xp, o, len, step, idx, cnt); \
        else                                                                                               \
            prod_reduce_kernel<T><<<grid_for(cnt), 256, 0, s>>>(xp, o, len, step, reinterpret_cast<T *>(out), cnt); \
    } while (0)
            switch (x.dtype) {
                case CHELIS_DTYPE_F32: CHELIS_DAG_EXTREME(float); break;
                case CHELIS_DTYPE_F64: CHELIS_DAG_EXTREME(double); break;
                case CHELIS_DTYPE_I32: CHELIS_DAG_EXTREME(int32_t); break;
                default: CHELIS_DAG_EXTREME(int64_t); break;
            }
#undef CHELIS_DAG_EXTREME
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::extreme_reduce_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::FloatClassify: {
            const Value &x = in(0);
            if (cnt == 0) return CHELIS_CUDA_OK;
            const Strided sx = strided(x);
            uint8_t *o = reinterpret_cast<uint8_t *>(out);
            switch (x.dtype) {
                case CHELIS_DTYPE_F32: classify_kernel<float><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const float *>(x.ptr), sx, n.kind, o, cnt); break;
                case CHELIS_DTYPE_F64: classify_kernel<double><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const double *>(x.ptr), sx, n.kind, o, cnt); break;
                case CHELIS_DTYPE_BF16: classify_kernel<Bf16Bits><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const Bf16Bits *>(x.ptr), sx, n.kind, o, cnt); break;
                default: classify_kernel<F16Bits><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const F16Bits *>(x.ptr), sx, n.kind, o, cnt); break;
            }
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::classify_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::ExtremaAdjoint: {
            const Value &a = in(0), &b = in(1), &g = in(2);
            if (cnt == 0) return CHELIS_CUDA_OK;
            if (n.dtype == CHELIS_DTYPE_F64)
                extrema_adjoint_kernel<double><<<grid_for(cnt), 256, 0, s>>>(
                    reinterpret_cast<const double *>(a.ptr), strided(a), reinterpret_cast<const double *>(b.ptr),
                    strided(b), reinterpret_cast<const double *>(g.ptr), strided(g), n.kind, n.axis,
                    reinterpret_cast<double *>(out), cnt);
            else
                extrema_adjoint_kernel<float><<<grid_for(cnt), 256, 0, s>>>(
                    reinterpret_cast<const float *>(a.ptr), strided(a), reinterpret_cast<const float *>(b.ptr),
                    strided(b), reinterpret_cast<const float *>(g.ptr), strided(g), n.kind, n.axis,
                    reinterpret_cast<float *>(out), cnt);
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::extrema_adjoint_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::KeyFromSeed: case Op::SplitKey: case Op::FoldIn: case Op::SplitN: {
            if (cnt == 0) return CHELIS_CUDA_OK;
            const Value &a = in(0);
            const bool seed = n.op == Op::KeyFromSeed;
            const Value &d = n.op == Op::FoldIn ? in(1) : a;
            const int mode = seed ? KEY_SEED : n.op == Op::SplitKey ? KEY_SPLIT : n.op == Op::FoldIn ? KEY_FOLD : KEY_SPLITN;
            const int64_t arg = n.op == Op::SplitKey ? n.kind : n.axis;
            key_kernel<<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const uint64_t *>(a.ptr), strided(a),
                                                     reinterpret_cast<const int64_t *>(d.ptr), strided(d), mode,
                                                     arg, reinterpret_cast<uint64_t *>(out), cnt);
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::key_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::ReduceWindow: case Op::ReduceWindowGrad: {
            const Value &x = in(0);
            WinGeom g{};
            g.rank = static_cast<int32_t>(x.shape.size());
            g.nw = static_cast<int32_t>(n.window.size());
            g.volume = 1;
            const int lead = g.rank - g.nw;
            for (int d = 0; d < g.rank; ++d) {
                g.in_shape[d] = x.shape[d];
                g.in_stride[d] = x.strides[d];
                g.out_shape[d] = d < lead ? x.shape[d] : (x.shape[d] - n.window[d - lead]) / n.wstride[d - lead] + 1;
            }
            for (int j = 0; j < g.nw; ++j) {
                g.win[j] = n.window[j];
                g.step[j] = n.wstride[j];
                g.volume *= n.window[j];
            }
            if (cnt == 0) return CHELIS_CUDA_OK;
            const unsigned int dt = static_cast<unsigned int>(n.dtype);
            if (n.op == Op::ReduceWindowGrad) {
                Value gv = in(1);
                CHELIS_TRY(dense(gv));
                if (n.dtype == CHELIS_DTYPE_F64)
                    window_grad_kernel<double><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const double *>(x.ptr),
                        reinterpret_cast<const double *>(gv.ptr), g, n.kind, reinterpret_cast<double *>(out), cnt);
                else
                    window_grad_kernel<float><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const float *>(x.ptr),
                        reinterpret_cast<const float *>(gv.ptr), g, n.kind, reinterpret_cast<float *>(out), cnt);
            } else {
#define CHELIS_DAG_WIN(T)                                                                                 \
    window_reduce_kernel<T><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const T *>(x.ptr), g, n.kind,   \
                                                          reinterpret_cast<T *>(out), cnt, dt)
                switch (n.dtype) {
                    case CHELIS_DTYPE_F64: CHELIS_DAG_WIN(double); break;
                    case CHELIS_DTYPE_I64: CHELIS_DAG_WIN(int64_t); break;
                    case CHELIS_DTYPE_I32: CHELIS_DAG_WIN(int32_t); break;
                    case CHELIS_DTYPE_I16: CHELIS_DAG_WIN(int16_t); break;
                    case CHELIS_DTYPE_I8: CHELIS_DAG_WIN(int8_t); break;
                    default: CHELIS_DAG_WIN(float); break;
                }
#undef CHELIS_DAG_WIN
            }
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::window_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::OrderedAdjointSum: {
            AdjointLeaves a{};
            int64_t leaves = 0;
            int k = 0;
            for (size_t g = 0; g < n.window.size(); ++g) {
                const int width = static_cast<int>(n.window[g]);
                a.first[g] = k;
                a.width[g] = width;
                a.leaf0[g] = leaves;
                for (int j = 0; j < width; ++j, ++k) {
                    const Value &x = in(k);
                    a.ptr[k] = x.ptr;
                    a.stride[k] = x.shape.empty() ? 0 : x.strides[0];
                }
                leaves += count_of(in(a.first[g]).shape) * width;
            }
            a.ngroups = static_cast<int32_t>(n.window.size());
            a.leaf0[a.ngroups] = leaves;
            int64_t chunk = 1;
            while ((leaves + chunk - 1) / chunk > kAdjointThreads) chunk *= 2;
            if (n.dtype == CHELIS_DTYPE_F64)
                ordered_adjoint_sum_kernel<double><<<1, kAdjointThreads, 0, s>>>(a, leaves, chunk,
                                                                                 reinterpret_cast<double *>(out));
            else
                ordered_adjoint_sum_kernel<float><<<1, kAdjointThreads, 0, s>>>(a, leaves, chunk,
                                                                                reinterpret_cast<float *>(out));
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::ordered_adjoint_sum_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::UniformBoundAdjoint: {
            const Value &g = in(1), &k = in(2);
            const int64_t rows = count_of(k.shape), total = count_of(g.shape), groups = cnt;
            const int64_t row_len = rows > 0 ? total / rows : 0;
            const int64_t rows_per_group = groups > 0 ? rows / groups : 0;
            if (groups == 0) return CHELIS_CUDA_OK;
            const int64_t leaves = rows_per_group * row_len;
            int64_t chunk = 1;
            while ((leaves + chunk - 1) / chunk > kBoundThreads) chunk *= 2;
            if (groups > INT32_MAX) return unsupported("UniformBoundAdjoint with more than 2^31 result elements");
            const unsigned int grid = static_cast<unsigned int>(groups);
            if (n.dtype == CHELIS_DTYPE_F64)
                uniform_bound_adjoint_kernel<double><<<grid, kBoundThreads, 0, s>>>(
                    reinterpret_cast<const double *>(g.ptr), strided(g), reinterpret_cast<const uint64_t *>(k.ptr),
                    strided(k), row_len, rows_per_group, chunk, n.kind, reinterpret_cast<double *>(out));
            else
                uniform_bound_adjoint_kernel<float><<<grid, kBoundThreads, 0, s>>>(
                    reinterpret_cast<const float *>(g.ptr), strided(g), reinterpret_cast<const uint64_t *>(k.ptr),
                    strided(k), row_len, rows_per_group, chunk, n.kind, reinterpret_cast<float *>(out));
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::uniform_bound_adjoint_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::Iota: {
            iota_kernel<<<grid_for(cnt > 0 ? cnt : 1), 256, 0, s>>>(reinterpret_cast<const int64_t *>(in(0).ptr),
                                                                    reinterpret_cast<const int64_t *>(in(1).ptr), cnt,
                                                                    reinterpret_cast<int64_t *>(out));
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::iota_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::UniformLike: {
            if (cnt == 0) return CHELIS_CUDA_OK;
            const Value &l = in(1), &h = in(2), &k = in(3);
            const int64_t rows = count_of(k.shape);
            const int64_t row_len = rows > 0 ? cnt / rows : 0;
            const unsigned int dt = static_cast<unsigned int>(n.dtype);
            if (n.dtype == CHELIS_DTYPE_F64)
                keyed_uniform_kernel<double><<<grid_for(cnt), 256, 0, s>>>(
                    reinterpret_cast<const double *>(l.ptr), strided(l), count_of(l.shape),
                    reinterpret_cast<const double *>(h.ptr), strided(h), count_of(h.shape),
                    reinterpret_cast<const uint64_t *>(k.ptr), strided(k), rows, row_len,
                    reinterpret_cast<double *>(out), cnt, dt);
            else
                keyed_uniform_kernel<float><<<grid_for(cnt), 256, 0, s>>>(
                    reinterpret_cast<const float *>(l.ptr), strided(l), count_of(l.shape),
                    reinterpret_cast<const float *>(h.ptr), strided(h), count_of(h.shape),
                    reinterpret_cast<const uint64_t *>(k.ptr), strided(k), rows, row_len,
                    reinterpret_cast<float *>(out), cnt, dt);
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::keyed_uniform_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::Dropout: {
            if (cnt == 0) return CHELIS_CUDA_OK;
            const Value &x = in(0), &r = in(1), &k = in(2);
            const int64_t rows = count_of(k.shape);
            const int64_t row_len = rows > 0 ? cnt / rows : 0;
            const int64_t rsize = count_of(r.shape);
            if (n.dtype == CHELIS_DTYPE_F64)
                keyed_dropout_kernel<double><<<grid_for(cnt), 256, 0, s>>>(
                    reinterpret_cast<const double *>(x.ptr), strided(x), reinterpret_cast<const double *>(r.ptr),
                    strided(r), rsize, reinterpret_cast<const uint64_t *>(k.ptr), strided(k), rows, row_len,
                    reinterpret_cast<double *>(out), cnt);
            else
                keyed_dropout_kernel<float><<<grid_for(cnt), 256, 0, s>>>(
                    reinterpret_cast<const float *>(x.ptr), strided(x), reinterpret_cast<const float *>(r.ptr),
                    strided(r), rsize, reinterpret_cast<const uint64_t *>(k.ptr), strided(k), rows, row_len,
                    reinterpret_cast<float *>(out), cnt);
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::keyed_dropout_kernel");
            return CHELIS_CUDA_OK;
        }
        case Op::Arith: {
            if (cnt == 0) return CHELIS_CUDA_OK;
            const Value &a = in(0);
            const Value &b = n.kind == IA_NEG || n.kind == IA_ABS ? in(0) : in(1);
            const Strided sa = strided(a), sb = strided(b);
            const unsigned int dt = static_cast<unsigned int>(n.dtype);
#define CHELIS_DAG_ARITH(T)                                                                               \
    arith_kernel<T><<<grid_for(cnt), 256, 0, s>>>(reinterpret_cast<const T *>(a.ptr), sa,                 \
                                                  reinterpret_cast<const T *>(b.ptr), sb, n.kind, dt,     \
                                                  reinterpret_cast<T *>(out), cnt)
            switch (n.dtype) {
                case CHELIS_DTYPE_I8: CHELIS_DAG_ARITH(int8_t); break;
                case CHELIS_DTYPE_I16: CHELIS_DAG_ARITH(int16_t); break;
                case CHELIS_DTYPE_I32: CHELIS_DAG_ARITH(int32_t); break;
                case CHELIS_DTYPE_I64: CHELIS_DAG_ARITH(int64_t); break;
                case CHELIS_DTYPE_F64: CHELIS_DAG_ARITH(double); break;
                default: CHELIS_DAG_ARITH(float); break;
            }
#undef CHELIS_DAG_ARITH
            g_launches++;
            CHELIS_LAUNCH_CHECK("dag::arith_kernel");
            return CHELIS_CUDA_OK;
        }
        default: return bad("unexpected node kind", n.opname);
    }
}

}  // namespace dag
}  // namespace chelis

using namespace chelis;

struct chelis_dag_program {
    dag::Program prog;  // the planned program; for a symbolic one, its interface only
    // symbolic extents: the nodes are re-parsed and planned for each binding
    bool symbolic = false;
    json::Value nodes;
    std::vector<int> roots;
    std::vector<std::string> symbols;  // in the order their first Load axis appears
    struct Source {
        int input, axis, symbol;
    };
    std::vector<Source> sources;       // every Load axis a name is bound from
    std::mutex mu;
    std::vector<std::pair<std::vector<int64_t>, std::shared_ptr<chelis_dag_program>>> cache;  // newest last
};

namespace chelis {
namespace dag {

constexpr size_t kMaxBindings = 8;  // planned instances kept per symbolic program

// Parse, check and plan `nodes` with every name bound (`bind` null: a static
// program).
int build(const json::Value &nodes, const std::vector<int> &roots,
          const std::vector<std::pair<std::string, int64_t>> *bind, Program &P) {
    t_sym = SymbolScope{};
    t_sym.bind = bind;
    int st = CHELIS_CUDA_OK;
    for (size_t i = 0; i < nodes.a.size() && st == CHELIS_CUDA_OK; ++i) st = parse_node(nodes.a[i], i, P.nodes);
    t_sym = SymbolScope{};
    CHELIS_TRY(st);
    CHELIS_TRY(check_and_layout(P));
    CHELIS_TRY(plan(P, roots));
    for (auto &n : P.nodes)
        if (n.op == Op::GuardedFail) {
            n.fail_id = register_fail_message(n.message.c_str());
            P.fail_ids.push_back(n.fail_id);
        }
    return CHELIS_CUDA_OK;
}

std::vector<std::pair<std::string, int64_t>> bindings(const chelis_dag_program &p, const std::vector<int64_t> &v) {
    std::vector<std::pair<std::string, int64_t>> b;
    for (size_t k = 0; k < p.symbols.size(); ++k) b.emplace_back(p.symbols[k], v[k]);
    return b;
}

// The symbols' values read from the inputs' shapes; every Load axis that
// names a symbol must agree (the generated entries' check, emit.rs:1141-1170).
int bind_values(const chelis_dag_program &p, const chelis_gpu_tensor *const *views, std::vector<int64_t> *values) {
    values->assign(p.symbols.size(), -1);
    std::vector<int> first(p.symbols.size(), -1);
    for (size_t k = 0; k < p.sources.size(); ++k) {
        const auto &src = p.sources[k];
        const chelis_gpu_tensor *t = views[src.input];
        if (!t || src.axis >= t->rank) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in load at i64");
        const int64_t e = t->shape[src.axis];
        int64_t &v = (*values)[src.symbol];
        if (v < 0) {
            v = e;
            first[src.symbol] = static_cast<int>(k);
        } else if (v != e) {
            const std::string &name = p.symbols[src.symbol];
            return set_error(CHELIS_CUDA_ERR_DOMAIN, "dag: symbolic dim `%s` mismatch: %s[%d]=%lld but %s=%lld",
                             name.c_str(), p.prog.input_labels[src.input].c_str(), src.axis,
                             static_cast<long long>(e), name.c_str(), static_cast<long long>(v));
        }
    }
    return CHELIS_CUDA_OK;
}

// The planned instance for these values: from the cache, or built and cached.
int instance(chelis_dag_program &p, const std::vector<int64_t> &values, std::shared_ptr<chelis_dag_program> *out) {
    std::lock_guard<std::mutex> lock(p.mu);
    for (size_t k = 0; k < p.cache.size(); ++k)
        if (p.cache[k].first == values) {
            auto hit = p.cache[k];
            p.cache.erase(p.cache.begin() + static_cast<std::ptrdiff_t>(k));
            p.cache.push_back(hit);
            *out = hit.second;
            return CHELIS_CUDA_OK;
        }
    auto inst = std::make_shared<chelis_dag_program>();
    const auto b = bindings(p, values);
    CHELIS_TRY(build(p.nodes, p.roots, &b, inst->prog));
    if (p.cache.size() >= kMaxBindings) p.cache.erase(p.cache.begin());
    p.cache.emplace_back(values, inst);
    *out = inst;
    return CHELIS_CUDA_OK;
}

}  // namespace dag
}  // namespace chelis

extern "C" {

int chelis_dag_from_json(const char *text, int64_t len, chelis_dag_program **out) {
    if (!out) return dag::bad("null output handle");
    *out = nullptr;
    if (!text || len < 0) return dag::bad("null or negative-length text");
    json::Value doc;
    json::Reader rd(text, static_cast<size_t>(len));
    if (!rd.parse(&doc)) return dag::bad("malformed JSON", rd.error());
    const json::Value *nodes = doc.get("nodes");
    const json::Value *roots = doc.get("roots");
    if (!nodes || nodes->kind != json::Value::Arr || !roots || roots->kind != json::Value::Arr)
        return dag::bad("a Dag object has \"nodes\" and \"roots\" arrays");
    std::vector<int> rs;
    for (const auto &r : roots->a) {
        int64_t v = 0;
        if (!dag::as_index(&r, &v) || v >= static_cast<int64_t>(nodes->a.size()))
            return dag::bad("root out of range");
        rs.push_back(static_cast<int>(v));
    }
    auto p = std::make_unique<chelis_dag_program>();
    // one parse with unbound names read as placeholders: every op is checked
    // here; a program with no unbound name is planned from it at once
    dag::t_sym = dag::SymbolScope{};
    dag::t_sym.placeholder = true;
    int st = CHELIS_CUDA_OK;
    for (size_t i = 0; i < nodes->a.size() && st == CHELIS_CUDA_OK; ++i)
        st = dag::parse_node(nodes->a[i], i, p->prog.nodes);
    const bool symbolic = dag::t_sym.saw_symbol;
    dag::t_sym = dag::SymbolScope{};
    CHELIS_TRY(st);
    if (!symbolic) {
        CHELIS_TRY(dag::check_and_layout(p->prog));
        CHELIS_TRY(dag::plan(p->prog, rs));
        for (auto &n : p->prog.nodes)
            if (n.op == dag::Op::GuardedFail) {
                n.fail_id = register_fail_message(n.message.c_str());
                p->prog.fail_ids.push_back(n.fail_id);
            }
        *out = p.release();
        return CHELIS_CUDA_OK;
    }
    p->symbolic = true;
    CHELIS_TRY(dag::io_plan(p->prog, rs));
    for (size_t i = 0; i < p->prog.nodes.size(); ++i) {
        const dag::Node &n = p->prog.nodes[i];
        if (n.op != dag::Op::Load) continue;
        for (size_t a = 0; a < n.dim_names.size(); ++a) {
            if (n.dim_names[a].empty()) continue;
            int sym = -1;
            for (size_t k = 0; k < p->symbols.size(); ++k)
                if (p->symbols[k] == n.dim_names[a]) sym = static_cast<int>(k);
            if (sym < 0) {
                sym = static_cast<int>(p->symbols.size());
                p->symbols.push_back(n.dim_names[a]);
            }
            p->sources.push_back({p->prog.input_of_load[i], static_cast<int>(a), sym});
        }
    }
    p->nodes = *nodes;
    p->roots = rs;
    *out = p.release();
    return CHELIS_CUDA_OK;
}

int32_t chelis_dag_symbol_count(const chelis_dag_program *p) {
    return p ? static_cast<int32_t>(p->symbols.size()) : -1;
}
const char *chelis_dag_symbol_name(const chelis_dag_program *p, int32_t i) {
    if (!p || i < 0 || i >= static_cast<int32_t>(p->symbols.size())) return nullptr;
    return p->symbols[i].c_str();
}

int chelis_dag_bind(chelis_dag_program *p, const int64_t *values, int32_t n, chelis_dag_program **out) {
    if (!p || !out) return dag::bad("null program or output handle");
    *out = nullptr;
    if (!p->symbolic) return dag::bad("the program has no symbolic extent to bind");
    if (n != static_cast<int32_t>(p->symbols.size()) || (n && !values))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "dag: expected %d symbol values, got %d",
                         static_cast<int>(p->symbols.size()), static_cast<int>(n));
    std::vector<int64_t> v(values, values + (n ? n : 0));
    for (int64_t e : v)
        if (e < 0) return dag::bad("a symbol value below 0");
    auto q = std::make_unique<chelis_dag_program>();
    const auto b = dag::bindings(*p, v);
    CHELIS_TRY(dag::build(p->nodes, p->roots, &b, q->prog));
    *out = q.release();
    return CHELIS_CUDA_OK;
}

void chelis_dag_release(chelis_dag_program *p) { delete p; }

int32_t chelis_dag_input_count(const chelis_dag_program *p) {
    return p ? static_cast<int32_t>(p->prog.input_labels.size()) : -1;
}
const char *chelis_dag_input_label(const chelis_dag_program *p, int32_t i) {
    if (!p || i < 0 || i >= static_cast<int32_t>(p->prog.input_labels.size())) return nullptr;
    return p->prog.input_labels[i].c_str();
}
int32_t chelis_dag_output_count(const chelis_dag_program *p) {
    return p ? static_cast<int32_t>(p->prog.output_labels.size()) : -1;
}
const char *chelis_dag_output_label(const chelis_dag_program *p, int32_t i) {
    if (!p || i < 0 || i >= static_cast<int32_t>(p->prog.output_labels.size())) return nullptr;
    return p->prog.output_labels[i].c_str();
}
int64_t chelis_dag_arena_bytes(const chelis_dag_program *p) { return p && !p->symbolic ? p->prog.arena_bytes : -1; }
int64_t chelis_dag_live_peak_bytes(const chelis_dag_program *p) {
    return p && !p->symbolic ? p->prog.live_peak_bytes : -1;
}
int32_t chelis_dag_slot_count(const chelis_dag_program *p) {
    return p && !p->symbolic ? static_cast<int32_t>(p->prog.slot_cap.size()) : -1;
}
int64_t chelis_dag_output_bytes(const chelis_dag_program *p) {
    if (!p || p->symbolic) return -1;
    int64_t b = 0;
    for (int o : p->prog.output_node)
        b += dag::count_of(p->prog.nodes[o].shape) * dtype_width(p->prog.nodes[o].dtype);
    return b;
}

int chelis_dag_run_device_arena(chelis_dag_program *p, const chelis_device_tensor_owner *const *inputs,
                                chelis_device_rank n_in, chelis_device_tensor_owner **outputs,
                                chelis_device_rank n_out, void *arena, int64_t arena_bytes) {
    if (!p) return dag::bad("null program");
    const dag::Program &P = p->prog;
    if (n_in != static_cast<int>(P.input_labels.size()) ||
        n_out != static_cast<int>(P.output_labels.size()))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "dag: expected %d inputs and %d outputs, got %d and %d",
                         static_cast<int>(P.input_labels.size()),
                         static_cast<int>(P.output_labels.size()), n_in, n_out);
    if ((n_in && !inputs) || (n_out && !outputs)) return dag::bad("null argument array");
    if (p->symbolic) {
        // bind the names from the inputs' shapes, then run that planned instance
        std::vector<const chelis_gpu_tensor *> tv(n_in, nullptr);
        for (int k = 0; k < n_in; ++k) tv[k] = chelis_device_tensor_view(inputs[k]);
        std::vector<int64_t> values;
        CHELIS_TRY(dag::bind_values(*p, tv.data(), &values));
        std::shared_ptr<chelis_dag_program> inst;
        CHELIS_TRY(dag::instance(*p, values, &inst));
        return chelis_dag_run_device_arena(inst.get(), inputs, n_in, outputs, n_out, arena, arena_bytes);
    }
    if (arena && arena_bytes < P.arena_bytes)
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "dag: arena of %lld bytes, the plan needs %lld",
                         static_cast<long long>(arena_bytes), static_cast<long long>(P.arena_bytes));
    for (int k = 0; k < n_out; ++k) outputs[k] = nullptr;
    // inputs: the dtype and shape each Load declares
    std::vector<const chelis_gpu_tensor *> views(n_in, nullptr);
    for (int k = 0; k < n_in; ++k) {
        views[k] = chelis_device_tensor_view(inputs[k]);
        if (!views[k]) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in load at i64");
    }
    for (size_t i = 0; i < P.nodes.size(); ++i) {
        if (P.input_of_load[i] < 0) continue;
        const chelis_gpu_tensor *t = views[P.input_of_load[i]];
        const dag::Node &n = P.nodes[i];
        bool ok = t->dtype == n.dtype && t->rank == static_cast<int32_t>(n.shape.size());
        for (int d = 0; ok && d < t->rank; ++d) ok = t->shape[d] == n.shape[d];
        if (!ok) return set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in load at i64");
    }
    dag::Run run(P);
    run.s = current_stream();
    void *owned_arena = nullptr;
    if (!arena && P.arena_bytes) {
        CHELIS_TRY(scratch_alloc(&owned_arena, static_cast<size_t>(P.arena_bytes), run.s));
        arena = owned_arena;
    }
    run.arena = static_cast<char *>(arena);
    int st = CHELIS_CUDA_OK;
    // output owners (outputs written in place allocate before the run)
    run.out_ptr.assign(n_out, nullptr);
    for (int k = 0; k < n_out && st == CHELIS_CUDA_OK; ++k) {
        const dag::Node &n = P.nodes[P.output_node[k]];
        outputs[k] = chelis_device_tensor_alloc_shape(n.dtype, static_cast<int32_t>(n.shape.size()),
                                                      n.shape.data());
        if (!outputs[k]) st = CHELIS_CUDA_ERR_CUDA;
        else run.out_ptr[k] = static_cast<char *>(chelis_device_tensor_view(outputs[k])->data);
    }
    // inputs that are not dense are copied once, so every layout is known
    std::vector<chelis_gpu_tensor> dense_in(n_in);
    std::vector<std::vector<int64_t>> dense_strides(n_in);
    for (int k = 0; k < n_in && st == CHELIS_CUDA_OK; ++k) {
        const chelis_gpu_tensor *t = views[k];
        std::vector<int64_t> shape(t->shape, t->shape + t->rank), strides(t->strides, t->strides + t->rank);
        dense_in[k] = *t;
        if (dag::is_dense(shape, strides)) continue;
        dag::Value v;
        v.ptr = static_cast<char *>(t->data);
        v.dtype = t->dtype;
        v.shape = shape;
        v.strides = strides;
        st = run.dense(v);
        dense_strides[k] = v.strides;
        dense_in[k].data = v.ptr;
        dense_in[k].strides = dense_strides[k].data();
        views[k] = &dense_in[k];
    }
    for (size_t i = 0; i < P.nodes.size() && st == CHELIS_CUDA_OK; ++i)
        st = run.node(static_cast<int>(i), views);
    // outputs not written in place: dense copies of their values
    for (int k = 0; k < n_out && st == CHELIS_CUDA_OK; ++k) {
        int o = P.output_node[k];
        while (P.nodes[o].op == dag::Op::Store) o = P.nodes[o].in[0];
        if (P.direct_output[o] == k) continue;
        st = dag::materialize(run.val[P.output_node[k]], run.out_ptr[k], run.s);
    }
    if (owned_arena) scratch_free(owned_arena, run.s);
    if (st != CHELIS_CUDA_OK) {
        for (int k = 0; k < n_out; ++k) {
            chelis_device_tensor_release(outputs[k]);
            outputs[k] = nullptr;
        }
        return st;
    }
    return CHELIS_CUDA_OK;
}

int chelis_dag_run_device(chelis_dag_program *p, const chelis_device_tensor_owner *const *inputs,
                          chelis_device_rank n_in, chelis_device_tensor_owner **outputs,
                          chelis_device_rank n_out) {
    return chelis_dag_run_device_arena(p, inputs, n_in, outputs, n_out, nullptr, 0);
}

int chelis_dag_run(chelis_dag_program *p, chelis_tensor **inputs, int n_in, chelis_tensor **outputs,
                   int n_out) {
    if (!p) return dag::bad("null program");
    const dag::Program &P = p->prog;
    if (n_in != static_cast<int>(P.input_labels.size()) ||
        n_out != static_cast<int>(P.output_labels.size()))
        return set_error(CHELIS_CUDA_ERR_DOMAIN, "dag: expected %d inputs and %d outputs, got %d and %d",
                         static_cast<int>(P.input_labels.size()),
                         static_cast<int>(P.output_labels.size()), n_in, n_out);
    if ((n_in && !inputs) || (n_out && !outputs)) return dag::bad("null argument array");
    for (int k = 0; k < n_out; ++k) outputs[k] = nullptr;
    std::vector<chelis_device_tensor_owner *> din(n_in, nullptr), dout(n_out, nullptr);
    int st = CHELIS_CUDA_OK;
    for (int k = 0; k < n_in && st == CHELIS_CUDA_OK; ++k) {
        if (!inputs[k]) {
            st = set_error(CHELIS_CUDA_ERR_DOMAIN, "numeric trap: domain in load at i64");
            break;
        }
        const chelis_read_view v = chelis_tensor_read_view(inputs[k]);
        const int32_t rank = chelis_tensor_rank(inputs[k]);
        std::vector<int64_t> shape(rank);
        for (int32_t d = 0; d < rank; ++d) shape[d] = chelis_tensor_shape(inputs[k], d);
        din[k] = chelis_device_tensor_alloc_shape(v.dtype, rank, shape.data());
        if (!din[k]) {
            st = CHELIS_CUDA_ERR_CUDA;
            break;
        }
        if (v.count)
            st = chelis_device_tensor_copy_from_host_bytes(din[k], v.data, v.count * dtype_width(v.dtype));
    }
    if (st == CHELIS_CUDA_OK) st = chelis_dag_run_device(p, din.data(), n_in, dout.data(), n_out);
    for (int k = 0; k < n_out && st == CHELIS_CUDA_OK; ++k) {
        const chelis_gpu_tensor *d = chelis_device_tensor_view(dout[k]);
        outputs[k] = chelis_alloc(d->rank, d->shape, d->dtype);
        chelis_tensor_write *guard = chelis_tensor_begin_write(outputs[k]);
        st = chelis_device_tensor_copy_to_host_status(guard, dout[k]);
        chelis_tensor_end_write(guard);
    }
    if (st == CHELIS_CUDA_OK) st = chelis_cuda_device_status();
    for (auto *o : din) chelis_device_tensor_release(o);
    for (auto *o : dout) chelis_device_tensor_release(o);
    if (st != CHELIS_CUDA_OK)
        for (int k = 0; k < n_out; ++k)
            if (outputs[k]) {
                chelis_tensor_release(outputs[k]);
                outputs[k] = nullptr;
            }
    return st;
}

}  // extern "C"
