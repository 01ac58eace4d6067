"""Builds libbi.so (the C-ABI kernel library) in-tree for sm_100a with nvcc.

    python mlx-batch-invariant_b200/build.py [--force] [-j N]

Objects go to mlx-batch-invariant_b200/_build/, the library to
mlx-batch-invariant_b200/mlx_batch_invariant_b200/libbi.so, where the Python
package loads it.  A source is recompiled only when it, or a header, is newer
than its object.
"""

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "mlx_batch_invariant_b200", "libbi.so")
INCLUDE = os.path.join(ROOT, "include")

SOURCES = ["capi.cu", "gemm_tcgen05.cu", "gemm_tf32x3.cu", "gemm_simt.cu", "sdpa.cu",
           "harness.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I" + INCLUDE, "-I" + CSRC]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: libbi.so cannot be built")


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(INCLUDE, "bi.h"))
    return hs


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, extra):
    obj = os.path.join(BUILD, os.path.basename(src).replace(".cu", ".o"))
    cmd = [nvcc()] + ARCH + FLAGS + extra + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed on %s:\n%s\n%s" % (src, " ".join(cmd), r.stderr))
    return obj, r.stderr


def build(force=False, jobs=None, verbose=False, extra=()):
    os.makedirs(BUILD, exist_ok=True)
    headers = _headers()
    srcs = [os.path.join(CSRC, s) for s in SOURCES]
    objs = [os.path.join(BUILD, s.replace(".cu", ".o")) for s in SOURCES]
    todo = [s for s, o in zip(srcs, objs) if force or _stale(o, [s] + headers)]
    if todo:
        with concurrent.futures.ThreadPoolExecutor(max_workers=jobs or len(todo)) as ex:
            for obj, err in ex.map(lambda s: _compile(s, list(extra)), todo):
                if verbose and err.strip():
                    print(err, file=sys.stderr)
    if force or todo or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart_static", "-ldl",
                                                               "-lrt", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n%s\n%s" % (" ".join(cmd), r.stderr))
    return LIB


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--force", action="store_true")
    p.add_argument("-j", "--jobs", type=int, default=None)
    p.add_argument("-v", "--verbose", action="store_true")
    p.add_argument("--ptxas-info", action="store_true", help="print registers / spills")
    a = p.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.ptxas_info else []
    print(build(force=a.force or a.ptxas_info, jobs=a.jobs, verbose=a.verbose or a.ptxas_info,
                extra=extra))


if __name__ == "__main__":
    main()
