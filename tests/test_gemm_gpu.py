"""GPU parity and invariance tests of the batch-invariant GEMM (libbi.so bi_gemm).

Parity bar: float32 (CUDA-core route) and float16 / bfloat16 shapes on the CUDA-core
route are bit-exact against the host oracle (same K order).  float16 / bfloat16 on
the tensor-core route accumulate the same K products in fp32 in another order (K=16
hardware steps), so they must be within 1 ulp of the oracle's emulation after
rounding plus the fp32 reordering allowance 2^-21 * sum_k |a[m,k] * b[k,n]| -- the
allowance only matters where the sum nearly cancels and an output-type ulp is finer
than fp32 accumulation noise.  Invariance bar: 0 differing bits.
"""

import numpy as np
import pytest
import torch

from conftest import batch_with, bits, randn, to_np
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.float16, torch.bfloat16]
UNIT = {torch.float16: 2.0 ** -10, torch.bfloat16: 2.0 ** -7}


@pytest.fixture(scope="module")
def bi():
    import mlx_batch_invariant_b200 as bi
    return bi


def _ulp_ok(got, want, dtype, absterm=None):
    """Tolerance stated in the module docstring; absterm = |a| @ |b| (float64)."""
    if dtype == torch.float32:
        return np.array_equal(bits(got), bits(torch.from_numpy(to_np(want).copy())))
    g = to_np(got).astype(np.float64)
    w = to_np(want).astype(np.float64)
    u = UNIT[dtype]
    mag = np.maximum(np.abs(w), 2.0 ** -24)
    ulp = 2.0 ** np.floor(np.log2(mag)) * u
    tol = ulp + (2.0 ** -21 * absterm if absterm is not None else 0.0)
    bad = np.abs(g - w) > tol * (1 + 1e-9)
    return not bad.any()


def _absterm(x, w, b_is_nk):
    a = np.abs(to_np(x).astype(np.float64))
    b = np.abs(to_np(w).astype(np.float64))
    return a @ (b.T if b_is_nk else b)


def _case(bi, dtype, M, K, N, b_is_nk, with_bias, alpha=1.0, beta=1.0, seed=0):
    x = randn((M, K), dtype, seed, "cuda")
    w = randn((N, K) if b_is_nk else (K, N), dtype, seed + 1, "cuda", std=K ** -0.5)
    bias = randn((N,), dtype, seed + 2, "cuda", std=0.1) if with_bias else None
    if b_is_nk:
        y = bi.linear(x, w, bias) if (alpha, beta) == (1.0, 1.0) else \
            bi._gemm._gemm(x, w, bias, True, alpha, beta)
    elif with_bias:
        y = bi.addmm(bias, x, w, alpha, beta)
    else:
        y = bi.matmul(x, w)
    want = orc.gemm(to_np(x), to_np(w), to_np(bias) if with_bias else None, b_is_nk=b_is_nk,
                    alpha=alpha, beta=beta)
    absterm = abs(alpha) * _absterm(x, w, b_is_nk)
    return y, torch.from_numpy(want.view(np.uint16) if dtype == torch.bfloat16 else want), absterm


SHAPES = [(1, 64, 8), (3, 72, 100), (7, 128, 256), (130, 264, 300), (129, 1000, 520),
          (256, 4096, 512), (17, 1024, 512), (64, 8, 16)]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("b_is_nk", [True, False])
@pytest.mark.parametrize("with_bias", [False, True])
def test_parity_against_oracle(bi, dtype, b_is_nk, with_bias):
    for (M, K, N) in SHAPES:
        y, want, absterm = _case(bi, dtype, M, K, N, b_is_nk, with_bias, seed=M + K)
        if dtype == torch.bfloat16:
            want = want.view(torch.bfloat16)
        assert _ulp_ok(y, want, dtype, absterm), "%s M=%d K=%d N=%d nk=%d bias=%d" % (
            dtype, M, K, N, b_is_nk, with_bias)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_alpha_beta_epilogue(bi, dtype):
    y, want, absterm = _case(bi, dtype, 33, 256, 264, False, True, alpha=0.5, beta=-2.0, seed=9)
    if dtype == torch.bfloat16:
        want = want.view(torch.bfloat16)
    assert _ulp_ok(y, want, dtype, absterm)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_unaligned_k_takes_cuda_core_route_bit_exact(bi, dtype):
    """K % 8 != 0 cannot feed TMA; the CUDA-core route is the oracle's exact order."""
    assert bi.tile_for(dtype, 1001, 64, True)["route"] == "simt"
    for b_is_nk in (True, False):
        y, want, _ = _case(bi, dtype, 9, 1001, 70, b_is_nk, True, seed=3)
        assert np.array_equal(bits(y), want.numpy().reshape(-1).view(
            np.uint16 if dtype != torch.float32 else np.uint32))


@pytest.mark.parametrize("dtype", DTYPES)
def test_batch_invariance_c1(bi, dtype):
    """Config 1: x (M,4096), w (4096,4096) (N,K), bias; row 0 fixed, other rows from
    fresh seeds; row 0's bits identical for every M (linear, matmul, addmm)."""
    K = N = 4096
    w_nk = randn((N, K), dtype, 1, "cuda", std=K ** -0.5)
    w_kn = w_nk.t().contiguous()
    bias = randn((N,), dtype, 4, "cuda", std=0.1)
    row0 = randn((1, K), dtype, 0, "cuda")
    ref = {}
    for M in (1, 2, 3, 4, 7, 8, 15, 16, 32, 64, 128):
        x = row0 if M == 1 else torch.cat([row0, randn((M - 1, K), dtype, 1000 + M, "cuda")])
        outs = {"linear": bi.linear(x, w_nk, bias), "matmul": bi.matmul(x, w_kn),
                "addmm": bi.addmm(bias, x, w_kn)}
        for name, y in outs.items():
            assert bool((y != 0).any()), "degenerate output"
            b0 = bits(y[0])
            if M == 1:
                ref[name] = b0
            else:
                nd = int((b0 != ref[name]).sum())
                assert nd == 0, "%s %s M=%d: %d/%d bits differ" % (name, dtype, M, nd, b0.size)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("K,N", [(512, 1024), (11008, 4096), (1024, 4096)])
def test_batch_invariance_placement(bi, dtype, K, N):
    """tests/test_invariance.py:36-69: the reference row at idx 0 and B//2."""
    W = randn((K, N), dtype, 1, "cuda", std=K ** -0.5)
    c = randn((N,), dtype, 4, "cuda")
    ref = randn((1, K), dtype, 3, "cuda")
    pool = randn((128, K), dtype, 2, "cuda")
    base = {}
    for B in (1, 2, 3, 5, 8, 16, 31, 32, 33, 64, 128):
        for idx in sorted({0, B // 2}):
            x = batch_with(ref, pool, B, idx)
            for name, f in (("matmul", lambda t: bi.matmul(t, W)),
                            ("addmm", lambda t: bi.addmm(c, t, W))):
                got = bits(f(x)[idx])
                if B == 1:
                    base[name] = got
                else:
                    assert int((got != base[name]).sum()) == 0, (name, dtype, K, N, B, idx)


def test_leading_dims_collapse_invariantly(bi):
    """tests/test_invariance.py:93-103."""
    for dtype in DTYPES:
        W = randn((1024, 512), dtype, 1, "cuda")
        x = randn((24, 1024), dtype, 5, "cuda")
        flat = bi.matmul(x, W)
        shaped = bi.matmul(x.reshape(4, 6, 1024), W).reshape(24, 512)
        assert np.array_equal(bits(flat), bits(shaped))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_column_shards_match_full_output(bi, dtype):
    """GPU-count invariance, emulated on one GPU: a column shard of the weight at any
    offset gives the same bits as the same columns of the full product."""
    K, N = 2048, 1536
    x = randn((77, K), dtype, 1, "cuda")
    w = randn((N, K), dtype, 2, "cuda", std=K ** -0.5)
    bias = randn((N,), dtype, 3, "cuda", std=0.1)
    full = bi.linear(x, w, bias)
    for n0, n1 in ((0, 256), (256, 768), (8, 520), (1000, 1536), (1528, 1536), (120, 128)):
        part = bi.linear(x, w[n0:n1], bias[n0:n1])
        assert np.array_equal(bits(part), bits(full[:, n0:n1])), (n0, n1)


def test_accuracy_against_float64(bi):
    """tests/test_invariance.py:114-146, with the fp32 bound tightened to 5e-6."""
    cases = [(17, 1024, 512), (128, 2048, 256), (1, 4096, 512), (8, 11008, 4096),
             (128, 11008, 4096)]
    for dtype, bound in ((torch.float32, 5e-6), (torch.float16, 5e-3), (torch.bfloat16, 4e-2)):
        for M, K, N in cases:
            a = randn((M, K), dtype, 11, "cuda")
            b = randn((K, N), dtype, 12, "cuda")
            exact = to_np(a).astype(np.float64) @ to_np(b).astype(np.float64)
            err = orc.rel_error(to_np(bi.matmul(a, b)).astype(np.float64), exact)
            assert err < bound, "%s M=%d K=%d N=%d rel err %g" % (dtype, M, K, N, err)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_addmm_epilogue_is_single_rounded(bi, dtype):
    """tests/test_invariance.py:148-158: bias added to the fp32 accumulator, rounded once."""
    a, b = randn((8, 512), dtype, 11, "cuda"), randn((512, 128), dtype, 12, "cuda")
    c = randn((128,), dtype, 4, "cuda")
    fused = to_np(bi.addmm(c, a, b)).astype(np.float64)
    acc32 = to_np(bi.matmul(a.float(), b.float())).astype(np.float64)
    want = torch.tensor(acc32 + to_np(c).astype(np.float64), dtype=torch.float32).to(dtype)
    want = to_np(want).astype(np.float64)
    assert np.abs(fused - want).max() / max(np.abs(want).max(), 1e-9) < 1e-2


def test_every_output_element_is_written(bi):
    """Poisoned output buffer: no NaN may survive (catches unwritten tiles)."""
    for dtype in DTYPES:
        for (M, K, N) in ((1, 64, 8), (129, 264, 300), (300, 512, 1000)):
            x = randn((M, K), dtype, 1, "cuda")
            w = randn((N, K), dtype, 2, "cuda", std=K ** -0.5)
            out = torch.full((M, N), float("nan"), dtype=dtype, device="cuda")
            bi._gemm._gemm(x, w, None, True, out=out)
            assert not torch.isnan(out).any(), (dtype, M, K, N)


def test_cuda_graph_capture_is_bitwise_identical(bi):
    for dtype in DTYPES:
        x = randn((64, 1024), dtype, 1, "cuda")
        w = randn((768, 1024), dtype, 2, "cuda", std=1 / 32)
        bias = randn((768,), dtype, 3, "cuda")
        eager = bi.linear(x, w, bias)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            bi.linear(x, w, bias)  # warm-up outside capture (attributes, tensor maps)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            y = bi.linear(x, w, bias)
        g.replay()
        torch.cuda.synchronize()
        assert np.array_equal(bits(y), bits(eager)), dtype


def test_large_shape_row_invariance_persistent_schedule(bi):
    """Enough tiles that every CTA loops several times (persistent schedule, both
    TMEM accumulator buffers): rows still match the single-row result."""
    dtype = torch.bfloat16
    K, N = 4096, 8192
    w = randn((N, K), dtype, 2, "cuda", std=K ** -0.5)
    x = randn((2048, K), dtype, 3, "cuda")
    full = bi.linear(x, w)
    for r in (0, 1, 127, 128, 1000, 2047):
        one = bi.linear(x[r:r + 1], w)
        assert np.array_equal(bits(one), bits(full[r:r + 1])), r
    assert bi._lib.device_error() == 0


def test_stock_matmul_is_batch_variant_control():
    """Negative control (tests/test_invariance.py:161-180): stock torch.matmul on this
    GPU must be batch-variant somewhere, or this suite proves nothing."""
    found = []
    for dtype in DTYPES:
        for K, N in ((2048, 1024), (4096, 4096), (11008, 4096)):
            W = randn((K, N), dtype, 1, "cuda")
            ref, pool = randn((1, K), dtype, 3, "cuda"), randn((128, K), dtype, 2, "cuda")
            base = bits((ref @ W)[0])
            for B in (2, 33, 128):
                y = batch_with(ref, pool, B, 0) @ W
                if int((bits(y[0]) != base).sum()) > 0:
                    found.append((dtype, K, N, B))
    assert found, "stock torch.matmul looks batch-invariant everywhere"
