"""CPU tests of the host side: libbi.so loads and exports every entry point of
include/bi.h, argument validation and status codes (no compute call), the Python
API's validation errors, and batch_invariant_mode's routing, strict semantics,
restoration and nesting (mlx_batch_invariant/__init__.py:46-147 and
tests/test_invariance.py:643-708 of the reference), exercised with CPU tensors,
which the library never computes on."""

import ctypes
import os
import re

import pytest
import torch
import torch.nn.functional as F

import mlx_batch_invariant_b200 as bi
from mlx_batch_invariant_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "bi.h")


def _declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(bi_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    names = _declared()
    assert {"bi_gemm", "bi_sdpa", "bi_gemm_route", "bi_status_string"} <= set(names)
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for n in names:
        assert hasattr(lib, n), n


def test_status_strings_and_version():
    L = _lib.lib()
    assert L.bi_status_string(0) == b"ok"
    assert L.bi_status_string(-3).startswith(b"misaligned")
    assert L.bi_status_string(-99) == b"unknown status"
    assert L.bi_version() >= 100


def test_route_depends_on_k_n_dtype_layout_never_m():
    # the ABI has no M argument at all; spot-check the table
    assert bi.tile_for(torch.bfloat16, 4096, 4096, True) == dict(route="tcgen05", BM=128, BN=256,
                                                                  BK=64)
    assert bi.tile_for(torch.float16, 8192, 57344, False)["route"] == "tcgen05"
    assert bi.tile_for(torch.float32, 4096, 4096, True) == dict(route="simt", BM=128, BN=128, BK=8)
    assert bi.tile_for(torch.bfloat16, 4095, 4096, True)["route"] == "simt"  # K % 8
    assert bi.tile_for(torch.bfloat16, 4096, 4095, False)["route"] == "simt"  # (K,N) row stride
    assert bi.tile_for(torch.bfloat16, 4096, 4095, True)["route"] == "tcgen05"
    assert bi.TILE == dict(BM=128, BN=256, BK=64, UMMA_M=256, UMMA_N=256, UMMA_K=16,
                           CTA_GROUP=2)


def test_gemm_argument_errors_are_status_codes():
    L = _lib.lib()
    s = L.bi_gemm(None, 8, None, 8, None, None, 8, 4, 4, 8, 1, 1.0, 1.0, 7, None)
    assert s == -1 and b"dtype" in L.bi_last_error()
    assert L.bi_gemm(None, 8, None, 8, None, None, 8, -1, 4, 8, 1, 1.0, 1.0, 2, None) == -1
    assert L.bi_gemm(None, 8, None, 8, None, None, 8, 0, 4, 8, 1, 1.0, 1.0, 2, None) == 0  # empty
    assert L.bi_gemm(None, 4, None, 8, None, None, 8, 4, 4, 8, 1, 1.0, 1.0, 2, None) == -1  # lda<K


def test_sdpa_argument_errors_are_status_codes():
    L = _lib.lib()
    z3, z2 = _lib.i64_3([0, 0, 0]), _lib.i64_2([0, 0])
    args = lambda H, Hkv, D, V, mode: (None, z3, None, z2, None, z2, None, z3, mode, 0, None, 1.0,
                                       1, H, Hkv, 1, 16, D, V, 2, None, z3, None)
    assert L.bi_sdpa(*args(8, 3, 64, 64, 0)) == -1  # H % Hkv
    assert L.bi_sdpa(*args(8, 4, 48, 48, 0)) == -1  # D % 32
    assert L.bi_sdpa(*args(8, 4, 672, 512, 0)) == -2  # head dims above 640 not built
    assert L.bi_sdpa(*args(8, 4, 64, 128, 0)) == -1  # D != V is built: fails on null q
    assert L.bi_sdpa(*args(8, 4, 64, 64, 3)) == -1  # mask mode
    assert L.bi_sdpa(*args(8, 4, 64, 64, 2)) == -1  # mode 2 without a mask


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device status")
def test_valid_call_without_a_gpu_reports_no_device():
    L = _lib.lib()
    buf = (ctypes.c_uint16 * 64)()
    p = ctypes.addressof(buf)
    assert L.bi_gemm(p, 8, p, 8, None, p, 8, 2, 2, 8, 1, 1.0, 1.0, 2, None) == -6


def test_gemm_validation_errors():
    a = torch.zeros(4, 8)
    with pytest.raises(ValueError, match="share a dtype"):
        bi.matmul(a, torch.zeros(8, 3, dtype=torch.float16))
    with pytest.raises(ValueError, match="ndim"):
        bi.matmul(torch.zeros(8), torch.zeros(8, 3))
    with pytest.raises(ValueError, match="inner dimensions"):
        bi.matmul(a, torch.zeros(7, 3))
    with pytest.raises(ValueError, match="bias must have shape"):
        bi.linear(a, torch.zeros(3, 8), torch.zeros(4))
    with pytest.raises(ValueError, match="unsupported dtype"):
        bi.matmul(a.double(), torch.zeros(8, 3, dtype=torch.float64))
    with pytest.raises(ValueError, match="CUDA tensors"):
        bi.linear(a, torch.zeros(3, 8))


def test_sdpa_validation_errors():
    q, k, v = torch.zeros(1, 8, 2, 64), torch.zeros(1, 4, 10, 64), torch.zeros(1, 4, 10, 64)
    with pytest.raises(ValueError, match="4-dimensional"):
        bi.scaled_dot_product_attention(q[0], k, v)
    with pytest.raises(ValueError, match="share a dtype"):
        bi.scaled_dot_product_attention(q.half(), k, v)
    with pytest.raises(ValueError, match="inconsistent"):
        bi.scaled_dot_product_attention(q, k[:, :, :5], v)
    with pytest.raises(ValueError, match="multiple of kv head"):
        bi.scaled_dot_product_attention(q, k[:, :3], v[:, :3])
    with pytest.raises(ValueError, match="multiples of 32"):
        bi.scaled_dot_product_attention(q[..., :48], k[..., :48], v[..., :48])
    with pytest.raises(ValueError, match="'causal'"):
        bi.scaled_dot_product_attention(q, k, v, mask="top-left")
    with pytest.raises(ValueError, match="broadcastable"):
        bi.scaled_dot_product_attention(q, k, v, mask=torch.zeros(1, 1, 3, 10))
    with pytest.raises(ValueError, match="sinks must have shape"):
        bi.scaled_dot_product_attention(q, k, v, sinks=torch.zeros(4))
    with pytest.raises(NotImplementedError):  # head dims above 640 are not built
        bi.scaled_dot_product_attention(q, k, torch.zeros(1, 4, 10, 672))
    with pytest.raises(ValueError, match="CUDA tensors"):  # D != V is built (CUDA only)
        bi.scaled_dot_product_attention(q, k, torch.zeros(1, 4, 10, 128))
    with pytest.raises(ValueError, match="CUDA tensors"):
        bi.scaled_dot_product_attention(q, k, v)


def test_quantized_path_is_not_built():
    assert bi.QUANT_BITS == ()
    with pytest.raises(NotImplementedError):
        bi.quantized_linear(None, None, None, None, 64, 4)


# ------------------------------------------------------------------ the mode
# CPU tensors are never computed on by the library, so under strict mode every
# routed call on them must raise, and with strict=False must equal stock exactly.

def _stock():
    return (torch.matmul, torch.Tensor.__matmul__, torch.addmm, F.linear,
            torch.nn.Linear.forward, F.scaled_dot_product_attention)


def test_mode_patches_and_restores():
    before = _stock()
    assert not bi.is_enabled()
    with bi.batch_invariant_mode():
        assert bi.is_enabled()
        assert torch.matmul is not before[0]
        assert F.linear is not before[3]
    assert _stock() == before
    assert not bi.is_enabled()


def test_strict_mode_raises_for_unsupported_calls():
    a, b = torch.randn(4, 8), torch.randn(8, 3)
    lin = torch.nn.Linear(8, 3)
    q = torch.randn(1, 4, 1, 48)
    with bi.batch_invariant_mode(strict=True):
        for fn in (lambda: torch.matmul(a, b), lambda: a @ b, lambda: lin(a),
                   lambda: F.linear(a, b.t()), lambda: torch.addmm(torch.zeros(3), a, b),
                   lambda: F.scaled_dot_product_attention(q, q, q, scale=0.1)):
            with pytest.raises(NotImplementedError, match="not batch-invariant"):
                fn()


def test_linear_on_1d_input_raises_under_strict():
    """The reference silently used stock for x.ndim < 2 even when strict; here it raises."""
    with bi.batch_invariant_mode(strict=True):
        with pytest.raises(NotImplementedError):
            F.linear(torch.randn(8), torch.randn(3, 8))


def test_non_strict_falls_back_to_stock_exactly():
    torch.manual_seed(0)
    a, b = torch.randn(4, 8), torch.randn(8, 3)
    lin = torch.nn.Linear(8, 3)
    q = torch.randn(1, 4, 1, 48)
    ref = (torch.matmul(a, b), a @ b, lin(a), torch.addmm(torch.ones(3), a, b, beta=0.5, alpha=2),
           F.scaled_dot_product_attention(q, q, q, scale=0.1))
    with bi.batch_invariant_mode(strict=False):
        got = (torch.matmul(a, b), a @ b, lin(a),
               torch.addmm(torch.ones(3), a, b, beta=0.5, alpha=2),
               F.scaled_dot_product_attention(q, q, q, scale=0.1))
    for r, g in zip(ref, got):
        assert torch.equal(r, g)


def test_originals_are_restored_even_on_exception():
    before = _stock()
    with pytest.raises(RuntimeError, match="boom"):
        with bi.batch_invariant_mode():
            assert bi.is_enabled()
            raise RuntimeError("boom")
    assert _stock() == before
    assert not bi.is_enabled()


def test_nesting_restores_only_at_the_outermost_exit():
    stock = torch.matmul
    with bi.batch_invariant_mode():
        patched = torch.matmul
        assert patched is not stock
        with bi.batch_invariant_mode(strict=False):
            assert torch.matmul is patched  # no second set of shims
        assert torch.matmul is patched, "inner exit unpatched too early"
        assert bi.is_enabled()
    assert torch.matmul is stock


def _gather_call(L, cols, world=2, rank=0, stages_null=False, ldo=None, dtype=None):
    vp = ctypes.c_void_p
    n_total = cols[-1]
    stages = None if stages_null else (vp * world)(*([16] * world))
    flags = (vp * world)(*([256] * world))
    c = (ctypes.c_int64 * len(cols))(*cols)
    return L.bi_gemm_allgather(16, 8, 16, 8, None, 16, n_total if ldo is None else ldo,
                               stages, c, 4, 8, 1, 1.0, 1.0,
                               _lib.BI_BF16 if dtype is None else dtype, flags, rank, world,
                               0, None)


def test_fused_allgather_validates_its_partition_before_touching_a_device():
    """bi_gemm_allgather checks the column partition, staging areas and rank set on the
    host and returns a status (no device needed to reach these errors)."""
    L = _lib.lib()
    assert _gather_call(L, [0, 16, 32]) in (0, -6)  # valid; BI_ERR_NO_DEVICE here
    assert _gather_call(L, [8, 16, 32]) == -1                 # cols[0] != 0
    assert _gather_call(L, [0, 24, 16]) == -1                 # decreasing
    assert _gather_call(L, [0, 12, 32]) == -3                 # not a multiple of 8
    assert b"multiples of 8" in L.bi_last_error()
    assert _gather_call(L, [0, 16, 32], stages_null=True) == -1
    assert _gather_call(L, [0, 16, 32], rank=2) == -1          # rank outside the world
    assert _gather_call(L, [0] * 10, world=9) == -1            # above BI_MAX_PEERS
    assert _gather_call(L, [0, 16, 32], ldo=24) == -3          # ldo < cols[world]
    assert _gather_call(L, [0, 16, 32], dtype=_lib.BI_F32) == -2  # tensor-core dtypes only


def test_static_allgather_rejects_two_ranks_on_one_device():
    """bi_gemm_allgather_static keeps one flag block per device, so a device named twice
    is refused before any CUDA call (no GPU needed)."""
    L = _lib.lib()
    devices = (ctypes.c_int * 2)(0, 0)
    stages = (ctypes.c_void_p * 2)()
    cols = (ctypes.c_int64 * 3)(0, 8, 16)
    st = L.bi_gemm_allgather_static(None, 8, None, 8, None, None, 16, stages, cols, 1, 8, 1,
                                    1.0, 1.0, _lib.BI_BF16, devices, 0, 2, 1, None)
    assert st == -1
    assert b"both on device 0" in L.bi_last_error()


def test_static_allgather_rejects_a_rank_outside_the_world():
    L = _lib.lib()
    devices = (ctypes.c_int * 2)(0, 1)
    stages = (ctypes.c_void_p * 2)()
    cols = (ctypes.c_int64 * 3)(0, 8, 16)
    st = L.bi_gemm_allgather_static(None, 8, None, 8, None, None, 16, stages, cols, 1, 8, 1,
                                    1.0, 1.0, _lib.BI_BF16, devices, 2, 2, 1, None)
    assert st == -1 and b"rank" in L.bi_last_error()


def test_mlx_bi_console_entry_point_is_declared_and_callable():
    """The reference installs `mlx-bi` (pyproject.toml [project.scripts]); so does this
    build, pointing at the same verify / decoder front end."""
    import importlib
    import tomllib
    path = os.path.join(ROOT, "mlx-batch-invariant_b200", "pyproject.toml")
    with open(path, "rb") as f:
        meta = tomllib.load(f)
    target = meta["project"]["scripts"]["mlx-bi"]
    mod, func = target.split(":")
    main = getattr(importlib.import_module(mod), func)
    assert main([]) == 2  # usage on no sub-command, as `mlx-bi` alone
    assert "libbi.so" in meta["tool"]["setuptools"]["package-data"]["mlx_batch_invariant_b200"]


def test_custom_ops_are_registered_with_shape_only_fakes():
    """mlx_bi::gemm and mlx_bi::sdpa (the opaque ops torch.compile sees) give the output
    shape and dtype on fake tensors, without touching a GPU."""
    from torch._subclasses.fake_tensor import FakeTensorMode
    with FakeTensorMode():
        a = torch.empty(3, 5, 64, dtype=torch.bfloat16, device="cuda")
        w = torch.empty(96, 64, dtype=torch.bfloat16, device="cuda")
        y = torch.ops.mlx_bi.gemm(a, w, None, True, 1.0, 1.0)
        assert y.shape == (3, 5, 96) and y.dtype == torch.bfloat16
        wk = torch.empty(64, 40, dtype=torch.bfloat16, device="cuda")
        assert torch.ops.mlx_bi.gemm(a, wk, None, False, 1.0, 1.0).shape == (3, 5, 40)
        q = torch.empty(2, 8, 3, 64, dtype=torch.float16, device="cuda")
        k = torch.empty(2, 2, 10, 64, dtype=torch.float16, device="cuda")
        o = torch.ops.mlx_bi.sdpa(q, k, k, 0.125, 1, 7, None, [0, 0, 0], None)
        assert o.shape == (2, 8, 3, 64) and o.dtype == torch.float16
