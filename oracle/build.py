"""Build recipe for the CPU oracle (test infrastructure only).

Compiles ``oracle/kvq_oracle.c`` into ``oracle/libkvq_oracle.so`` with gcc,
OpenMP and no floating-point contraction (the quantize rule and the rounding
points of the restated op graph are IEEE f32 operations and must stay so).
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "kvq_oracle.c")
OUT = os.path.join(HERE, "libkvq_oracle.so")


def build(force: bool = False) -> str:
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= os.path.getmtime(SRC):
        return OUT
    cmd = ["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-fno-fast-math", "-fPIC",
           "-shared", "-std=c11", "-Wall", "-o", OUT, SRC, "-lm"]
    subprocess.check_call(cmd)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
