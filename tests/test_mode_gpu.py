"""batch_invariant_mode on CUDA tensors: the patched torch entry points route to the
invariant kernels (same bits as calling bi.* directly), models stay invariant across
batch size, strict / non-strict behaviour on an unsupported head dim
(tests/test_invariance.py:595-708 of the reference), CUDA-graph capture of a model
under the mode, and the regression guard on the stock torch ops a model uses
unwrapped (tests/test_invariance.py:183-212)."""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import batch_with, bits, randn

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def bi():
    import mlx_batch_invariant_b200 as bi
    return bi


def test_patched_entry_points_route_to_the_kernels(bi):
    dt = torch.bfloat16
    x = randn((4, 6, 512), dt, 1, "cuda")
    w = randn((512, 384), dt, 2, "cuda", std=1 / 16)
    wl = randn((384, 512), dt, 3, "cuda", std=1 / 16)
    c = randn((384,), dt, 4, "cuda")
    q = randn((2, 8, 5, 64), dt, 5, "cuda")
    k = randn((2, 2, 40, 64), dt, 6, "cuda")
    v = randn((2, 2, 40, 64), dt, 7, "cuda")
    lin = torch.nn.Linear(512, 384, dtype=dt, device="cuda")
    want = {
        "matmul": bi.matmul(x, w), "op": bi.matmul(x, w),
        "addmm": bi.addmm(c, x.reshape(-1, 512), w, alpha=0.5, beta=2.0),
        "linear": bi.linear(x, wl), "module": bi.linear(x, lin.weight, lin.bias),
    }
    with bi.batch_invariant_mode(strict=True):
        got = {
            "matmul": torch.matmul(x, w), "op": x @ w,
            "addmm": torch.addmm(c, x.reshape(-1, 512), w, beta=2.0, alpha=0.5),
            "linear": F.linear(x, wl), "module": lin(x),
        }
        sd_gqa = F.scaled_dot_product_attention(q, k, v, enable_gqa=True)
        qq = randn((2, 8, 40, 64), dt, 8, "cuda")
        sd_causal = F.scaled_dot_product_attention(qq, k.repeat_interleave(4, 1),
                                                   v.repeat_interleave(4, 1), is_causal=True)
    for name in want:
        assert np.array_equal(bits(got[name]), bits(want[name])), name
    assert np.array_equal(bits(sd_gqa), bits(bi.scaled_dot_product_attention(q, k, v)))
    # Lq == Lk: torch's top-left causal rule and the reference's bottom-right coincide
    assert np.array_equal(bits(sd_causal), bits(bi.scaled_dot_product_attention(
        qq, k.repeat_interleave(4, 1), v.repeat_interleave(4, 1), mask="causal")))


def test_model_under_the_mode_is_batch_invariant(bi):
    """tests/test_invariance.py:619-640 (without mx.compile): a small MLP run under
    the mode gives row idx the same bits for every batch size."""
    torch.manual_seed(54)
    net = torch.nn.Sequential(torch.nn.Linear(256, 512), torch.nn.GELU(),
                              torch.nn.Linear(512, 128)).to("cuda", torch.float16)
    ref = randn((1, 256), torch.float16, 55, "cuda")
    pool = randn((16, 256), torch.float16, 56, "cuda")
    base = None
    with bi.batch_invariant_mode(strict=True):
        for B in (1, 2, 3, 8, 16):
            idx = B // 2
            got = bits(net(batch_with(ref, pool, B, idx))[idx])
            if base is None:
                base = got
            else:
                assert np.array_equal(got, base), B


def test_stock_model_is_batch_variant_control():
    """The same MLP without the mode: stock cuBLAS must make some row variant."""
    torch.manual_seed(57)
    net = torch.nn.Sequential(torch.nn.Linear(4096, 4096), torch.nn.GELU(),
                              torch.nn.Linear(4096, 4096)).to("cuda", torch.float32)
    ref = randn((1, 4096), torch.float32, 58, "cuda")
    pool = randn((128, 4096), torch.float32, 59, "cuda")
    base = bits(net(ref)[0])
    assert any(not np.array_equal(bits(net(batch_with(ref, pool, B, 0))[0]), base)
               for B in (2, 33, 128))


def test_unsupported_attention_raises_under_strict_and_falls_back_otherwise(bi):
    """tests/test_invariance.py:646-664: head dim 48 is not a multiple of 32."""
    q = randn((1, 4, 1, 48), torch.float16, 61, "cuda")
    k = randn((1, 4, 128, 48), torch.float16, 62, "cuda")
    v = randn((1, 4, 128, 48), torch.float16, 63, "cuda")
    with bi.batch_invariant_mode(strict=True):
        with pytest.raises(NotImplementedError):
            F.scaled_dot_product_attention(q, k, v, scale=0.1)
    ref = F.scaled_dot_product_attention(q, k, v, scale=0.1)
    with bi.batch_invariant_mode(strict=False):
        y = F.scaled_dot_product_attention(q, k, v, scale=0.1)
    assert y.shape == (1, 4, 1, 48)
    assert np.array_equal(bits(y), bits(ref))


def test_broadcast_kv_head_without_enable_gqa_raises_under_strict(bi):
    """Stock SDPA broadcasts a single KV head when enable_gqa is False; that call is not
    the invariant kernel, so strict mode must refuse it rather than pass it through."""
    q = randn((1, 8, 2, 64), torch.bfloat16, 64, "cuda")
    k = randn((1, 1, 128, 64), torch.bfloat16, 65, "cuda")
    v = randn((1, 1, 128, 64), torch.bfloat16, 66, "cuda")
    with bi.batch_invariant_mode(strict=True):
        with pytest.raises(NotImplementedError):
            F.scaled_dot_product_attention(q, k, v)
        # the same heads with enable_gqa take the kernel
        y = F.scaled_dot_product_attention(q, k, v, enable_gqa=True)
    assert np.array_equal(bits(y), bits(bi.scaled_dot_product_attention(q, k, v)))
    try:
        ref = F.scaled_dot_product_attention(q, k, v)
    except RuntimeError:  # a stock backend that refuses the broadcast: same under the mode
        with bi.batch_invariant_mode(strict=False):
            with pytest.raises(RuntimeError):
                F.scaled_dot_product_attention(q, k, v)
        return
    with bi.batch_invariant_mode(strict=False):
        y = F.scaled_dot_product_attention(q, k, v)
    assert np.array_equal(bits(y), bits(ref))


def test_graph_capture_of_a_model_under_the_mode(bi):
    torch.manual_seed(3)
    net = torch.nn.Sequential(torch.nn.Linear(1024, 2048), torch.nn.SiLU(),
                              torch.nn.Linear(2048, 1024)).to("cuda", torch.bfloat16)
    x = randn((32, 1024), torch.bfloat16, 4, "cuda")
    with bi.batch_invariant_mode(strict=True):
        eager = net(x)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            net(x)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            y = net(x)
    g.replay()
    torch.cuda.synchronize()
    assert np.array_equal(bits(y), bits(eager))


BATCHES = [1, 2, 3, 5, 8, 16, 31, 32, 33, 64, 128]


def _row_invariant(fn, ref, pool):
    base = None
    for B in BATCHES:
        idx = B // 2
        got = bits(fn(batch_with(ref, pool, B, idx))[idx])
        if base is None:
            base = got
        elif not np.array_equal(got, base):
            return False
    return True


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_stock_fused_norms_softmax_and_silu_are_batch_invariant(dtype):
    """Regression guard for the stock ops a model uses unwrapped (the reference's
    tests/test_invariance.py:199-212 for MLX).  On B200, torch's fused rms_norm,
    layer_norm and softmax kernels and silu keep a row's bits whatever the batch."""
    for D in (1024, 4096, 8192):
        w, b = randn((D,), dtype, 1, "cuda"), randn((D,), dtype, 4, "cuda")
        ref, pool = randn((1, D), dtype, 3, "cuda"), randn((128, D), dtype, 2, "cuda")
        for name, fn in (("rms_norm", lambda x: F.rms_norm(x, (D,), w, 1e-5)),
                         ("layer_norm", lambda x: F.layer_norm(x, (D,), w, b, 1e-5)),
                         ("softmax", lambda x: torch.softmax(x, -1)),
                         ("silu", F.silu)):
            assert _row_invariant(fn, ref, pool), (name, dtype, D)


def test_stock_row_sum_is_batch_variant_on_b200():
    """Unlike MLX (the reference asserts sum and mean invariant), torch's float32
    last-dim sum changes a row's bits with the batch size on B200: code that needs
    invariance must not build norms from torch.sum / torch.mean."""
    found = []
    for D in (1024, 4096, 8192):
        ref = randn((1, D), torch.float32, 3, "cuda")
        pool = randn((128, D), torch.float32, 2, "cuda")
        if not _row_invariant(lambda x: x.sum(-1, keepdim=True), ref, pool):
            found.append(D)
    assert found, "torch's row sum now looks batch-invariant on this device"
