"""torch.compile around the invariant kernels (tests/test_invariance.py:595-640 of the
reference, which pins the same under mx.compile): the compiler may fuse and reorder
the graph around bi.* calls but must not reach inside them, so the bits of a row stay
independent of the batch and the query length.  The kernels are registered as the
opaque torch.library ops mlx_bi::gemm and mlx_bi::sdpa."""

import numpy as np
import pytest
import torch

from conftest import batch_with, bits, randn

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def bi():
    import mlx_batch_invariant_b200 as bi
    return bi


@pytest.fixture(autouse=True)
def _fresh_dynamo():
    torch._dynamo.reset()
    yield
    torch._dynamo.reset()


def test_attention_is_invariant_under_compile(bi):
    H, Hkv, N, D = 16, 8, 2048, 128
    QLS = [1, 2, 4, 8, 9, 16]
    for dtype in (torch.float32, torch.float16, torch.bfloat16):
        k = randn((1, Hkv, N, D), dtype, 51, "cuda")
        v = randn((1, Hkv, N, D), dtype, 52, "cuda")
        qf = randn((1, H, max(QLS), D), dtype, 53, "cuda")
        fn = torch.compile(lambda q: bi.scaled_dot_product_attention(q, k, v))
        base = None
        for qL in QLS:
            q = qf[:, :, max(QLS) - qL:, :].contiguous()
            y = fn(q)
            got = bits(y[:, :, -1, :])
            if base is None:
                base = got
                # the compiled call runs the same kernel as the eager one
                eager = bi.scaled_dot_product_attention(q, k, v)
                assert np.array_equal(got, bits(eager[:, :, -1, :]))
            else:
                assert int((got != base).sum()) == 0, "compiled sdpa %s qL=%d" % (dtype, qL)


def test_mode_holds_for_function_compiled_inside(bi):
    """A module first traced inside the context captures the invariant kernels (as
    opaque ops) and stays invariant for every later call inside it."""
    torch.manual_seed(54)
    net = torch.nn.Sequential(torch.nn.Linear(256, 512), torch.nn.GELU(),
                              torch.nn.Linear(512, 128)).to("cuda", torch.float16)
    ref = randn((1, 256), torch.float16, 55, "cuda")
    pool = randn((16, 256), torch.float16, 56, "cuda")
    # inference, as in the reference: the kernels are forward-only (no autograd formula)
    with torch.no_grad(), bi.batch_invariant_mode(strict=True):
        fn = torch.compile(net)
        base = None
        for B in (1, 2, 3, 8, 16):
            idx = B // 2
            y = fn(batch_with(ref, pool, B, idx))
            got = bits(y[idx])
            if base is None:
                base = got
            else:
                assert int((got != base).sum()) == 0, "compiled-inside mode B=%d" % B


def test_compiled_graph_holds_the_opaque_ops(bi):
    """The traced graph calls mlx_bi::gemm / mlx_bi::sdpa (no graph break, no stock
    matmul), and running it gives the eager bits."""
    seen = []

    def backend(gm, example_inputs):
        seen.extend(str(n.target) for n in gm.graph.nodes if n.op == "call_function")
        return gm.forward

    x = randn((7, 256), torch.bfloat16, 1, "cuda")
    w = randn((384, 256), torch.bfloat16, 2, "cuda", std=1 / 16)
    b = randn((384,), torch.bfloat16, 3, "cuda")
    q = randn((2, 8, 5, 64), torch.bfloat16, 4, "cuda")
    k = randn((2, 2, 300, 64), torch.bfloat16, 5, "cuda")

    def f(x, q):
        return bi.linear(x, w, b), bi.scaled_dot_product_attention(q, k, k, mask="causal")

    cf = torch.compile(f, backend=backend, fullgraph=True)
    y1, a1 = cf(x, q)
    assert any("mlx_bi.gemm" in s for s in seen), seen
    assert any("mlx_bi.sdpa" in s for s in seen), seen
    y0, a0 = f(x, q)
    assert np.array_equal(bits(y1), bits(y0))
    assert np.array_equal(bits(a1), bits(a0))
