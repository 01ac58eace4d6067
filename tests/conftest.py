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
