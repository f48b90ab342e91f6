"""Regenerate the golden fixtures under tests/golden/ from the reference tree.

Usage: python tests/golden/make_golden.py <reference-root> (or set
CHELIS_REFERENCE to the reference checkout).  The outputs are committed;
tests never read the reference tree at run time.

* crmath_f32.txt -- the f32 exp / log / erfc rows of the reference's CORE-MATH
  canary fixture (crates/chelis-crmath/tests/fixtures/canary.txt): function,
  input bits, expected bits.  They pin the oracle's transcendentals.
* ieee_f32.txt -- the f32 add / mul / div / sqrt rows of
  crates/chelis-crmath/tests/fixtures/profile_obligations.txt: primitive,
  expected bits, operand bits.  They pin the oracle's finalized arithmetic
  (round to nearest even, subnormals kept, canonical NaN).
* fused_steps.txt -- one row per single-step FusedElem chain: step op, width
  (f32 / f64), expected bits, operand bits.  The add / sub / mul / div / sqrt
  / pow rows of profile_obligations.txt, every canary.txt row (exp, log, sin,
  cos, tan, atan, tanh, erf, erfc) and the pow_worst_cases.txt sample; they
  pin the fused oracle's steps and bound the CUDA steps.
"""
import os
import sys

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("CHELIS_REFERENCE", "")
if not REF or not os.path.isdir(REF):
    sys.exit("usage: make_golden.py <reference-root> (or CHELIS_REFERENCE=<reference-root>)")
FIX = os.path.join(REF, "crates/chelis-crmath/tests/fixtures")
OUT = os.path.dirname(os.path.abspath(__file__))


def rows(path, keep):
    with open(path) as f:
        for line in f:
            line = line.split("#", 1)[0].strip()
            if not line:
                continue
            parts = line.split()
            if keep(parts):
                yield parts


def main():
    canary = list(rows(os.path.join(FIX, "canary.txt"),
                       lambda p: p[1] == "f32" and p[0] in ("exp", "log", "erfc")))
    with open(os.path.join(OUT, "crmath_f32.txt"), "w") as f:
        f.write("# function input-bits expected-bits (from the reference CORE-MATH canary fixture)\n")
        for p in canary:
            f.write(f"{p[0]} {p[2]} {p[3]}\n")
    ieee = list(rows(os.path.join(FIX, "profile_obligations.txt"),
                     lambda p: p[1] == "f32" and p[0] in ("add", "mul", "div", "sqrt")))
    with open(os.path.join(OUT, "ieee_f32.txt"), "w") as f:
        f.write("# primitive expected-bits operand-bits... (from the reference profile obligations)\n")
        for p in ieee:
            f.write(" ".join([p[0]] + p[2:]) + "\n")
    steps = [[p[0], p[1], p[2], *p[3:]] for p in rows(
        os.path.join(FIX, "profile_obligations.txt"),
        lambda p: p[0] in ("add", "sub", "mul", "div", "sqrt", "pow"))]
    steps += [[p[0], p[1], p[3], p[2]] for p in rows(os.path.join(FIX, "canary.txt"), lambda p: True)]
    steps += [[p[0], p[1], p[4], p[2], p[3]]
              for p in rows(os.path.join(FIX, "pow_worst_cases.txt"), lambda p: True)]
    with open(os.path.join(OUT, "fused_steps.txt"), "w") as f:
        f.write("# op width expected-bits operand-bits... (reference CORE-MATH / profile fixtures)\n")
        for p in steps:
            f.write(" ".join(p) + "\n")
    print(len(canary), len(ieee), len(steps))


if __name__ == "__main__":
    main()
