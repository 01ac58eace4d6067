"""GPU tests of the float32 tensor-core GEMM route (bi_gemm_tf32x3, selected with
bi.set_float32_gemm("tf32x3")): three tf32 products per K step with fp32 accumulation.

Accuracy bar (the reference's float32 bar of tests/test_invariance.py:114-127,
tightened to 5e-6 as for the CUDA-core route): max |gpu - float64| / max |float64|
<= 5e-6.  Invariance bar: 0 differing bits over batch size, row placement and column
shards.  The route is not bit-equal to the "exact" CUDA-core route (different
arithmetic), so the two are compared only within the accuracy bar."""

import numpy as np
import pytest
import torch

from conftest import batch_with, bits, randn, to_np
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def bi():
    import mlx_batch_invariant_b200 as bi
    with bi.float32_gemm("tf32x3"):
        yield bi


def _exact(a, b, b_is_nk, bias=None):
    a64 = to_np(a).astype(np.float64)
    b64 = to_np(b).astype(np.float64)
    y = a64 @ (b64.T if b_is_nk else b64)
    if bias is not None:
        y = y + to_np(bias).astype(np.float64)
    return y


@pytest.mark.parametrize("b_is_nk", [True, False])
def test_accuracy_against_float64(bi, b_is_nk):
    assert bi.get_float32_gemm() == "tf32x3"
    cases = [(17, 1024, 512), (128, 2048, 256), (1, 4096, 512), (8, 11008, 4096),
             (128, 11008, 4096), (300, 1004, 1000), (4096, 4096, 4096)]
    for M, K, N in cases:
        if not b_is_nk and N % 4:
            continue
        assert bi.tile_for(torch.float32, K, N, b_is_nk)["route"] == "tf32x3"
        a = randn((M, K), torch.float32, 11, "cuda")
        b = randn((N, K) if b_is_nk else (K, N), torch.float32, 12, "cuda")
        bias = randn((N,), torch.float32, 13, "cuda")
        y = bi.linear(a, b, bias) if b_is_nk else bi.addmm(bias, a, b)
        err = orc.rel_error(to_np(y).astype(np.float64), _exact(a, b, b_is_nk, bias))
        assert err < 5e-6, "M=%d K=%d N=%d nk=%d rel err %.3e" % (M, K, N, b_is_nk, err)
    assert bi._lib.device_error() == 0


@pytest.mark.parametrize("b_is_nk", [True, False])
def test_error_does_not_grow_with_k(bi, b_is_nk):
    """The tensor core's fp32 accumulation drifts by a fraction of an ulp per MMA, so one
    accumulator over all of K let the error grow linearly with K (2.2e-4 at K = 28672).
    Uniform [0, 1) data, where every product has the same sign, shows it most.  K is summed in
    256-deep chunks added in fp32 round to nearest: the error stays flat in K (measured
    ~6e-6 on uniform data at every K from 256 to 28672), inside the reference's float32
    bar of 2e-5 (tests/test_invariance.py:114-127)."""
    g = torch.Generator(device="cuda").manual_seed(21)
    errs = []
    for K in (256, 4096, 28672):
        a = torch.rand((17, K), generator=g, device="cuda")
        b = torch.rand((512, K) if b_is_nk else (K, 512), generator=g, device="cuda")
        y = bi.linear(a, b) if b_is_nk else bi.matmul(a, b)
        errs.append(orc.rel_error(to_np(y).astype(np.float64), _exact(a, b, b_is_nk)))
    assert max(errs) < 1e-5, errs
    assert errs[-1] < 2.0 * errs[0] + 1e-6, errs  # flat in K, not linear
    assert bi._lib.device_error() == 0


def test_config1_rows_are_batch_invariant(bi):
    """Config 1 in float32 on the tensor-core route: row 0's bits for every M."""
    K = N = 4096
    w = randn((N, K), torch.float32, 1, "cuda", std=K ** -0.5)
    bias = randn((N,), torch.float32, 4, "cuda", std=0.1)
    row0 = randn((1, K), torch.float32, 0, "cuda")
    ref = None
    for M in (1, 2, 3, 4, 7, 8, 15, 16, 32, 64, 128, 300, 1100):
        x = row0 if M == 1 else torch.cat([row0, randn((M - 1, K), torch.float32, 1000 + M,
                                                       "cuda")])
        b0 = bits(bi.linear(x, w, bias)[0])
        if ref is None:
            ref = b0
        else:
            assert np.array_equal(b0, ref), M


@pytest.mark.parametrize("b_is_nk", [True, False])
def test_placement_and_column_shards(bi, b_is_nk):
    K, N = 2048, 1536
    w = randn((N, K) if b_is_nk else (K, N), torch.float32, 2, "cuda", std=K ** -0.5)
    ref = randn((1, K), torch.float32, 3, "cuda")
    pool = randn((300, K), torch.float32, 5, "cuda")
    f = (lambda t, ww: bi.linear(t, ww)) if b_is_nk else (lambda t, ww: bi.matmul(t, ww))
    base = bits(f(ref, w)[0])
    for B in (2, 33, 300):
        for idx in (0, B // 2, B - 1):
            assert np.array_equal(bits(f(batch_with(ref, pool, B, idx), w)[idx]), base), (B, idx)
    x = randn((77, K), torch.float32, 6, "cuda")
    full = f(x, w)
    for n0, n1 in ((0, 256), (256, 768), (8, 520), (1000, 1536), (1528, 1536)):
        ws = w[n0:n1] if b_is_nk else w[:, n0:n1].contiguous()
        assert np.array_equal(bits(f(x, ws)), bits(full[:, n0:n1])), (n0, n1)


def test_every_output_element_is_written_and_close_to_the_exact_route(bi):
    for (M, K, N) in ((1, 64, 8), (129, 264, 300), (300, 512, 1000), (513, 1004, 260)):
        x = randn((M, K), torch.float32, 1, "cuda")
        w = randn((N, K), torch.float32, 2, "cuda", std=K ** -0.5)
        out = torch.full((M, N), float("nan"), device="cuda")
        bi._gemm._gemm(x, w, None, True, out=out)
        assert not torch.isnan(out).any(), (M, K, N)
        with bi.float32_gemm("exact"):
            exact_route = bi.linear(x, w)
        scale = exact_route.abs().max().item()
        assert (out - exact_route).abs().max().item() <= 1e-5 * scale, (M, K, N)


def test_unaligned_k_keeps_the_exact_route(bi):
    """K % 4 != 0 cannot feed TMA: the route falls back to the CUDA-core kernel (a
    function of K, never of M), bit-exact against the oracle."""
    assert bi.tile_for(torch.float32, 1001, 64, True)["route"] == "simt"
    x = randn((9, 1001), torch.float32, 3, "cuda")
    w = randn((70, 1001), torch.float32, 4, "cuda")
    want = orc.gemm(to_np(x), to_np(w), b_is_nk=True)
    assert np.array_equal(bits(bi.linear(x, w)), want.reshape(-1).view(np.uint32))


def test_cuda_graph_capture_is_bitwise_identical(bi):
    x = randn((64, 1024), torch.float32, 1, "cuda")
    w = randn((768, 1024), torch.float32, 2, "cuda", std=1 / 32)
    eager = bi.linear(x, w)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        bi.linear(x, w)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y = bi.linear(x, w)
    g.replay()
    torch.cuda.synchronize()
    assert np.array_equal(bits(y), bits(eager))
