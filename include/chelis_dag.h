/*
 * chelis_dag.h -- run a serialized Chelis DAG on the GPU.
 *
 * The reference's GPU lane compiles each verified DAG into C++ with a
 * storage plan fixed at build time (crates/chelis-backend-hip/src/lib.rs:104
 * codegen_hip, src/emit.rs:488 emit_dag, src/memory.rs:39-98 MemoryPlan,
 * peak bytes src/lib.rs:47-53).  This interface takes the same DAG as the
 * JSON serde writes for crates/chelis-dag-core's `Dag`
 * (src/dag.rs:2364-2400, 2913-2920: {"nodes": [...], "roots": [...],
 * "declarations": [...]}), plans it once and runs it on the current device
 * and the calling thread's stream.
 *
 * Inputs are bound in the order of the first Load of each name and outputs
 * are the Store nodes in node order, then the roots (labels "root<i>"), as
 * the generated entries order them (emit.rs:5881-5934).
 *
 * Extents: literal, Named with a size, or symbolic -- DimInfo::Named(name,
 * None), DimExpr Sym / Mul / Div and RtDim::Sym.  A program with symbolic
 * extents binds each name from the input axes its Loads declare with it
 * (every such axis must agree: "symbolic dim `n` mismatch: x[0]=5 but n=4",
 * the generated entries' check, emit.rs:1141-1170) and is checked and
 * planned once per set of values (the latest eight are kept).  Runtime
 * bounds read from a node (RtDim::Node, InputAxis) are
 * CHELIS_CUDA_ERR_UNSUPPORTED.
 *
 * Supported RiscOps: Load, Store, Const, ConstTensor; the elementwise
 * arithmetic (Add, Sub, Mul, Div, Pow, FloorDiv, TruncDiv, Mod, MaxElem,
 * MinElem, Neg, Recip, Exp, Log, Sin, Sqrt, Cos, Tan, Atan, Tanh, Erf, Erfc,
 * Abs, Floor, Ceil, Round on f32 / f64; the integer forms at i8-i64 with the
 * C lane's traps), Bitwise, Compare, Logical, Where, FloatClassify,
 * ExtremaAdjoint, FusedElem, Relu, ReluAdjoint, Softmax (last axis, f32),
 * Sum, MaxReduce, MinReduce, ProdReduce, Argmax, Argmin, Count (any axes),
 * Cumsum (any axis), ReduceWindow, ReduceWindowGrad, BlasMatmul (batched,
 * transposed views taken in place), Gather, ScatterAdd, Scatter,
 * ScatterElements, Reshape, Permute, Expand, Shrink, Stride, Pad, Cast,
 * NamedCast, Copy, Realize, Drop, Shape, Iota, GuardedFail, the keyed RNG
 * (KeyFromSeed, Split, FoldIn, SplitN, Dropout, DropoutReplay, UniformLike,
 * UniformBoundAdjoint), OrderedAdjointSum and the shape contracts
 * (ExtentWitness, CheckedExtent, CheckedUnitAxis).  Any other op, or a node
 * under a runtime activation, is CHELIS_CUDA_ERR_UNSUPPORTED at load time
 * (the HIP lane's Unsupported result, lib.rs:104).
 */
#ifndef CHELIS_DAG_H
#define CHELIS_DAG_H

#include <stdint.h>

#include "chelis_cuda.h"
#include "chelis_host_runtime.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct chelis_dag_program chelis_dag_program;

/* Parse, check and plan a DAG (`len` bytes of JSON).  Errors:
 * CHELIS_CUDA_ERR_DOMAIN for a malformed or inconsistent graph,
 * CHELIS_CUDA_ERR_UNSUPPORTED for an op or extent this lane does not run. */
int chelis_dag_from_json(const char *json, int64_t len, chelis_dag_program **out);
void chelis_dag_release(chelis_dag_program *program);

int32_t chelis_dag_input_count(const chelis_dag_program *program);
const char *chelis_dag_input_label(const chelis_dag_program *program, int32_t i);
int32_t chelis_dag_output_count(const chelis_dag_program *program);
const char *chelis_dag_output_label(const chelis_dag_program *program, int32_t i);

/* Symbolic extents: the names to bind (0 for a static program), and a
 * static program with the names bound to `values` (in symbol order), for the
 * plan queries below or a caller-sized arena; release it with
 * chelis_dag_release.  The plan queries return -1 for an unbound program. */
int32_t chelis_dag_symbol_count(const chelis_dag_program *program);
const char *chelis_dag_symbol_name(const chelis_dag_program *program, int32_t i);
int chelis_dag_bind(chelis_dag_program *program, const int64_t *values, int32_t n,
                    chelis_dag_program **out);
/* The storage plan (memory.rs:39-98): every value that needs storage of its
 * own (not an input, a view, an output, a dropped or an inlined node) gets a
 * slot; a slot is reused by a later value once every reader of its previous
 * value has run (best fit by size).  arena_bytes is the device memory of all
 * slots (each rounded to 256 bytes): the scratch a run needs besides its
 * outputs (output_bytes).  live_peak_bytes is the most slot memory live at
 * one time (the reference's max_live_bytes). */
int64_t chelis_dag_arena_bytes(const chelis_dag_program *program);
int64_t chelis_dag_live_peak_bytes(const chelis_dag_program *program);
int32_t chelis_dag_slot_count(const chelis_dag_program *program);
int64_t chelis_dag_output_bytes(const chelis_dag_program *program);

/* Generated-entry device ABI (emit.rs:838-958): borrowed input owners (of the
 * dtypes and shapes the Loads declare; non-dense inputs are copied once),
 * outputs as new owners the caller releases.  The slots come from the
 * library's stream-ordered pool; _arena runs them in the caller's device
 * buffer of at least chelis_dag_arena_bytes() bytes instead. */
int chelis_dag_run_device(chelis_dag_program *program,
                          const chelis_device_tensor_owner *const *inputs, chelis_device_rank n_in,
                          chelis_device_tensor_owner **outputs, chelis_device_rank n_out);
int chelis_dag_run_device_arena(chelis_dag_program *program,
                                const chelis_device_tensor_owner *const *inputs,
                                chelis_device_rank n_in, chelis_device_tensor_owner **outputs,
                                chelis_device_rank n_out, void *arena, int64_t arena_bytes);
/* Generated-entry host-array ABI (emit.rs:660-800): host inputs, new
 * runtime-owned host outputs; returns with the work complete and the device
 * error word checked (an out-of-range Gather / Scatter index is the
 * reference's "gather index 3 out of bounds at axis 1 of extent 3" then
 * "numeric trap: domain in gather at i64"). */
int chelis_dag_run(chelis_dag_program *program, chelis_tensor **inputs, int n_in,
                   chelis_tensor **outputs, int n_out);

#ifdef __cplusplus
}
#endif
#endif /* CHELIS_DAG_H */
