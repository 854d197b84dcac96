"""Build recipe for the CPU oracle (test infrastructure only).

Compiles ``pf_oracle.c`` into ``oracle/libpf_oracle.so`` with gcc.  The flags
keep fp32 arithmetic exactly as written (no FMA contraction, no fast-math) so
the oracle's float results are reproducible operation by operation.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "pf_oracle.c")
OUT = os.path.join(HERE, "libpf_oracle.so")


def build(force: bool = False) -> str:
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= os.path.getmtime(SRC):
        return OUT
    cmd = [
        "gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
        "-fno-fast-math", "-Wall", "-Wextra", "-o", OUT, SRC, "-lm",
    ]
    subprocess.check_call(cmd)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
