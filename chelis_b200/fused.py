"""FusedElem groups on the CUDA backend: the host-side form of a chain.

Mirrors chelis-dag-core's fusion vocabulary (crates/chelis-dag-core/src/
dag.rs): a group is a list of ``FusedStep``s (dag.rs:483-490), each a
``FusedStepOp`` (dag.rs:494-526; same names and order as ``OPS`` here) over
``FusedInput`` operands (dag.rs:673-678): ``External(i)`` is the group's
i-th input, ``PreviousStep(j)`` the value of step j.  The group's value is
its last step.  ``encode`` turns a chain into the C ABI's
``chelis_fused_step`` triplets (op, a, b) with a >= 0 an input and a < 0 the
step -1 - a.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Sequence, Union

# FusedStepOp, dag.rs:494-526, in declaration order (the C ABI's numbering)
OPS = ("add", "sub", "mul", "div", "pow", "floor_div", "trunc_div", "max_elem", "min_elem",
       "neg", "recip", "exp", "log", "sin", "sqrt", "cos", "tan", "atan", "tanh", "erf", "erfc",
       "abs", "floor", "ceil", "round")
OP_CODE = {name: i for i, name in enumerate(OPS)}
BINARY = frozenset(OPS[:OP_CODE["min_elem"] + 1])
# steps whose value the C lane takes from a correctly rounded CORE-MATH call
TRANSCENDENTAL = frozenset(("pow", "exp", "log", "sin", "cos", "tan", "atan", "tanh", "erf",
                            "erfc"))
REDUCE_KIND = {"sum": 0, "max": 1}
MAX_STEPS, MAX_INPUTS, MAX_RANK = 32, 8, 6


@dataclass(frozen=True)
class External:
    index: int


@dataclass(frozen=True)
class PreviousStep:
    index: int


FusedInput = Union[External, PreviousStep]


@dataclass(frozen=True)
class FusedStep:
    op: str
    inputs: tuple

    def __init__(self, op: str, *inputs: FusedInput):
        if op not in OP_CODE:
            raise ValueError(f"unknown fused step op {op!r}")
        want = 2 if op in BINARY else 1
        if len(inputs) != want:
            raise ValueError(f"fused step {op} takes {want} operand(s), got {len(inputs)}")
        object.__setattr__(self, "op", op)
        object.__setattr__(self, "inputs", tuple(inputs))


class StepArray(ctypes.Structure):
    _fields_ = [("op", ctypes.c_int32), ("a", ctypes.c_int32), ("b", ctypes.c_int32)]


def _operand(x: FusedInput) -> int:
    if isinstance(x, External):
        return x.index
    if isinstance(x, PreviousStep):
        return -1 - x.index
    raise TypeError(f"fused operand must be External or PreviousStep, not {type(x).__name__}")


def triplets(steps: Sequence[FusedStep]) -> list[tuple[int, int, int]]:
    """(op, a, b) per step; a unary step repeats its operand as b."""
    out = []
    for s in steps:
        a = _operand(s.inputs[0])
        b = _operand(s.inputs[1]) if len(s.inputs) > 1 else a
        out.append((OP_CODE[s.op], a, b))
    return out


def encode(steps: Sequence[FusedStep]):
    """The chain as a ctypes array of chelis_fused_step."""
    t = triplets(steps)
    arr = (StepArray * max(len(t), 1))()
    for i, (op, a, b) in enumerate(t):
        arr[i].op, arr[i].a, arr[i].b = op, a, b
    return arr


def parse(text: str) -> list[FusedStep]:
    """A chain from a compact text form, one step per ';'-separated item:
    ``op operand [operand]`` with operands ``x<i>`` (External) or ``v<j>``
    (PreviousStep), e.g. ``"mul x0 x1; add v0 x2; tanh v1"``."""
    steps = []
    for item in text.split(";"):
        words = item.split()
        if not words:
            continue
        ops = []
        for w in words[1:]:
            if w[0] == "x":
                ops.append(External(int(w[1:])))
            elif w[0] == "v":
                ops.append(PreviousStep(int(w[1:])))
            else:
                raise ValueError(f"fused operand {w!r}: want x<i> or v<j>")
        steps.append(FusedStep(words[0], *ops))
    return steps
