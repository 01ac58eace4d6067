"""Shared test setup: import paths, the `gpu` marker and tensor helpers."""

import os
import sys

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "mlx-batch-invariant_b200")
for p in (ROOT, PKG_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU and libbi.so")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def to_np(t):
    """torch tensor (any supported dtype, any device) -> NumPy array of that dtype."""
    import ml_dtypes
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16).view(ml_dtypes.bfloat16)
    return t.numpy()


def bits(t):
    """Bit patterns of a tensor as a flat NumPy unsigned array."""
    t = t.detach().contiguous().reshape(-1)
    if t.element_size() == 4:
        return t.view(torch.int32).cpu().numpy().view(np.uint32)
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def randn(shape, dtype, seed, device="cpu", std=1.0):
    """Seeded N(0, std^2) tensor, generated in fp32 on the CPU then cast."""
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g, dtype=torch.float32) * std).to(dtype).to(device)


def batch_with(ref, pool, B, idx):
    """Batch of size B holding `ref` at row `idx` and pool rows elsewhere
    (tests/test_invariance.py:28-33 of the reference)."""
    if B == 1:
        return ref
    parts = ([pool[:idx]] if idx > 0 else []) + [ref] + ([pool[idx + 1:B]] if idx + 1 < B else [])
    return torch.cat(parts)


# ---------------------------------------------------------------- attention parity bar
# Elementwise: the oracle (bi_oracle.c) keeps the fold's fp32 result w before the final
# rounding to the output type (same inputs, same lane split); each GPU output element
# must satisfy
#     |gpu - w| <= 0.5 ulp_T(w) + tau * A_j   (float16 / bfloat16)
#     |gpu - w| <= 2 ulp_f32(w) + tau * A_j   (float32)
# with A_j = sum_i p_i |v_ij| / sum_i p_i (float64 weights on |v|), the size of the terms
# output j sums, and tau = 2^-20 on every route.  The CUDA-core route runs the oracle's
# fold and order (only CUDA's expf and the C library's differ); the GQA route (16-bit,
# D = 64 / 128, H / Hkv a multiple of 4) departs in two places -- score = scale * (q . k)
# from a tensor-core dot product instead of pre-scaled q, and the visible keys of a
# stage folded 4 at a time -- and runs P.V in fp32 with the weights exact; over decode,
# prefill, mask and sink shapes its worst element measured 0.999 of this bar.
_MANT = {torch.float16: 10, torch.bfloat16: 7, torch.float32: 23}
_MIN_NORMAL = {torch.float16: 2.0 ** -14, torch.bfloat16: 2.0 ** -126, torch.float32: 2.0 ** -126}


def ulp_of(x, dtype):
    """Spacing of `dtype` values at |x| (float64 array)."""
    mag = np.maximum(np.abs(x), _MIN_NORMAL[dtype])
    return 2.0 ** (np.floor(np.log2(mag)) - _MANT[dtype])


def attn_worst(got, q, k, v, mask_mode=0, mask=None, causal_offset=0, sinks=None):
    """Largest |gpu - w| / bar over the elements of `got` (see the bar above); <= 1 passes.
    q (B,H,qL,D), k/v (B,Hkv,N,D) torch tensors; mask the additive mask (4-D, in q's
    dtype, -inf = masked) for mask_mode 2, or mask_mode 1 with causal_offset."""
    from oracle import oracle as orc
    dtype = q.dtype
    B, H, qL, D = q.shape
    Hkv, N = k.shape[1], k.shape[2]
    f32 = lambda t: np.ascontiguousarray(to_np(t).astype(np.float32))
    q32, k32, v32 = f32(q), f32(k), f32(v)
    s32 = f32(sinks) if sinks is not None else None
    m32 = f32(mask) if mask_mode == 2 else None
    w = orc.sdpa(to_np(q), to_np(k), to_np(v), mask=to_np(mask) if mask_mode == 2 else None,
                 mask_mode=mask_mode, causal_offset=causal_offset,
                 sinks=to_np(sinks) if sinks is not None else None, out_dtype=np.float32)
    m64 = m32
    if mask_mode == 1:
        i = np.arange(N)[None, :]
        s = np.arange(qL)[:, None]
        m64 = np.where(i <= causal_offset + s, 0.0, -np.inf)[None, None]
    absv = orc.attention_f64(q32, k32, np.abs(v32), mask=m64, sinks=s32)
    g = to_np(got).astype(np.float64)
    w = w.astype(np.float64)
    tau = 2.0 ** -20
    if dtype == torch.float32:
        bar = 2 * ulp_of(w, dtype) + tau * absv
    else:
        bar = 0.5 * ulp_of(w, dtype) * (1 + 1e-7) + tau * absv
    return float((np.abs(g - w) / bar).max())
