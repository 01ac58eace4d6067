"""Builds the CPU oracle (test infrastructure only) into oracle/build/libbi_oracle.so.

    python oracle/build.py [--force]

The reference itself cannot be built or run here: its kernels are Metal Shading
Language strings launched through MLX (mlx_batch_invariant/_gemm.py:29-157,
_attention.py:32-158), and neither MLX nor Metal exists on Linux.  So there is no
oracle/_ref/ build; bi_oracle.c restates the reference's algorithm instead.
"""

import argparse
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "bi_oracle.c")
OUT_DIR = os.path.join(HERE, "build")
LIB = os.path.join(OUT_DIR, "libbi_oracle.so")
# -ffp-contract=off: every a*b+c the restatement does not spell as fmaf stays two
# rounded operations, as the epilogue requires.
CFLAGS = ["-O3", "-ffp-contract=off", "-fno-fast-math", "-mavx2", "-mfma", "-mf16c",
          "-fopenmp", "-fPIC", "-shared", "-std=gnu11"]


def build(force=False):
    os.makedirs(OUT_DIR, exist_ok=True)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        cmd = ["gcc"] + CFLAGS + [SRC, "-o", LIB, "-lm"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("oracle build failed:\n%s\n%s" % (" ".join(cmd), r.stderr))
    return LIB


if __name__ == "__main__":
    p = argparse.ArgumentParser()
    p.add_argument("--force", action="store_true")
    print(build(p.parse_args().force))
