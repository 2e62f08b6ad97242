"""Build the oracle's C restatement (TEST INFRASTRUCTURE ONLY) into oracle/_liboracle.so.

    python oracle/build.py

gcc with OpenMP, no CUDA.  The product package never loads this library; the tests and
the bench's CPU-baseline leg do, as the parity checker.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRCS = [os.path.join(HERE, "cham_rank2.c")]
LIB = os.path.join(HERE, "_liboracle.so")


def build():
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(s) for s in SRCS + [__file__]):
        return LIB
    cmd = ["gcc", "-O3", "-march=x86-64-v2", "-fopenmp", "-shared", "-fPIC", "-o", LIB, *SRCS, "-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build())
    sys.exit(0)
