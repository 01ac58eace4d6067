"""Generates tests/golden/golden.npz: small seeded inputs and the CPU oracle's outputs
for the GEMM and attention restatements.

    python tests/golden/make_golden.py

The reference (mlx-batch-invariant 0.2.0) runs only under MLX on Apple GPUs and
ships no golden vectors, so these fixtures cannot be reference outputs.  They pin the
oracle (tests/test_oracle.py checks that it still reproduces them bit for bit and
that every stored output meets the reference tests' float64 tolerances) and, through
it, the GPU kernels.  16-bit arrays are stored as uint16 bit patterns.
"""

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import ml_dtypes  # noqa: E402

from oracle import oracle as orc  # noqa: E402

DT = {"float32": np.float32, "float16": np.float16, "bfloat16": ml_dtypes.bfloat16}


def store(a):
    a = np.ascontiguousarray(a)
    if a.dtype.itemsize == 2:
        return a.view(np.uint16)
    return a


def main():
    rng = np.random.default_rng(20240601)
    out = {}
    gemm_cases = [(5, 40, 24), (3, 37, 19), (9, 128, 64)]
    for name, dt in DT.items():
        for ci, (M, K, N) in enumerate(gemm_cases):
            for nk in (0, 1):
                for has_bias in (0, 1):
                    a = rng.standard_normal((M, K)).astype(np.float32).astype(dt)
                    b = (rng.standard_normal((N, K) if nk else (K, N)) / np.sqrt(K)).astype(
                        np.float32).astype(dt)
                    bias = (rng.standard_normal(N) * 0.1).astype(np.float32).astype(dt) \
                        if has_bias else None
                    y = orc.gemm(a, b, bias, b_is_nk=bool(nk))
                    key = "gemm_%s_%d_nk%d_b%d" % (name, ci, nk, has_bias)
                    out[key + "_a"] = store(a)
                    out[key + "_b"] = store(b)
                    if bias is not None:
                        out[key + "_bias"] = store(bias)
                    out[key + "_y"] = store(y)
    for name in ("float32", "bfloat16", "float16"):
        dt = DT[name]
        for mi, mode in enumerate(("none", "causal", "additive", "sinks")):
            B, H, Hkv, qL, N, D = 2, 4, 2, 3, 45, 32
            q = rng.standard_normal((B, H, qL, D)).astype(np.float32).astype(dt)
            k = rng.standard_normal((B, Hkv, N, D)).astype(np.float32).astype(dt)
            v = rng.standard_normal((B, Hkv, N, D)).astype(np.float32).astype(dt)
            kw = {}
            sinks = None
            if mode == "causal":
                kw = dict(mask_mode=1, causal_offset=N - qL)
            elif mode == "additive":
                m = rng.standard_normal((1, 1, qL, N)).astype(np.float32).astype(dt)
                m[..., 5] = -np.inf
                kw = dict(mask=m, mask_mode=2)
                out["sdpa_%s_%s_mask" % (name, mode)] = store(m)
            elif mode == "sinks":
                sinks = rng.standard_normal(H).astype(np.float32).astype(dt)
                kw = dict(sinks=sinks)
                out["sdpa_%s_%s_sinks" % (name, mode)] = store(sinks)
            y = orc.sdpa(q, k, v, **kw)
            key = "sdpa_%s_%s" % (name, mode)
            out[key + "_q"] = store(q)
            out[key + "_k"] = store(k)
            out[key + "_v"] = store(v)
            out[key + "_y"] = store(y)
    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print("wrote %s (%d arrays)" % (path, len(out)))


if __name__ == "__main__":
    main()
