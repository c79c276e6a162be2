"""Build recipe for the oracle (test infrastructure only).

Compiles oracle/feml_oracle.c into oracle/_build/liboracle.so with f32
contraction disabled, so `acc += a * b` rounds the product and the sum
separately, as the reference's Rust code does (feml-cpu/src/ops/mul_mat.rs:46-48).

The reference itself is a Rust workspace and there is no cargo/rustc in this
image, so there is no oracle/_ref build: the restatement is the oracle.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "feml_oracle.c")
OUT_DIR = os.path.join(HERE, "_build")
OUT = os.path.join(OUT_DIR, "liboracle.so")

CFLAGS = ["-O2", "-ffp-contract=off", "-fno-fast-math", "-fno-tree-vectorize",
          "-fPIC", "-shared", "-pthread", "-std=c11", "-Wall"]


def build(force: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    if (not force and os.path.exists(OUT)
            and os.path.getmtime(OUT) >= os.path.getmtime(SRC)):
        return OUT
    tmp = OUT + f".tmp{os.getpid()}"
    subprocess.check_call(["gcc", *CFLAGS, SRC, "-o", tmp, "-lm"])
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
