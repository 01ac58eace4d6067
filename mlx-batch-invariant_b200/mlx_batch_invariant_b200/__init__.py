"""Batch-invariant kernels for NVIDIA B200 on PyTorch tensors.

Every function here returns bitwise identical results for a given row of input
regardless of what else was in the batch, how many query tokens were submitted
together, or how many GPUs shared the work.

    import mlx_batch_invariant_b200 as bi

    with bi.batch_invariant_mode():
        logits = model(tokens)

The API is that of mlx-batch-invariant 0.2.0 (mlx_batch_invariant/__init__.py),
with PyTorch CUDA tensors in place of MLX arrays.  The arithmetic is in libbi.so,
hand-written sm_100a CUDA behind a C ABI (include/bi.h).
"""

import contextlib
import math

import torch
import torch.nn.functional as F

from . import _ops  # noqa: F401  (registers mlx_bi::gemm and mlx_bi::sdpa)
from ._attention import _mask_args, _sdpa, scaled_dot_product_attention
from ._attention import head_dims_built
from ._gemm import QUANT_BITS, SIMT_TILE, TILE, addmm, linear, matmul, quantized_linear, tile_for
from ._gemm import float32_gemm, get_float32_gemm, set_float32_gemm

__all__ = [
    "quantized_linear",
    "QUANT_BITS",
    "matmul",
    "addmm",
    "linear",
    "scaled_dot_product_attention",
    "batch_invariant_mode",
    "is_enabled",
    "TILE",
    "SIMT_TILE",
    "tile_for",
    "set_float32_gemm",
    "get_float32_gemm",
    "float32_gemm",
    "__version__",
]

__version__ = "0.1.0"

_depth = 0
_SUPPORTED = (torch.float32, torch.float16, torch.bfloat16)


def is_enabled():
    """True inside a :func:`batch_invariant_mode` block."""
    return _depth > 0


def _unsupported(what, strict, fallback, *args, **kwargs):
    """mlx_batch_invariant/__init__.py:_unsupported (:46-53)."""
    if strict:
        raise NotImplementedError(
            "%s is not batch-invariant in this build. Pass strict=False to "
            "batch_invariant_mode() to fall back to stock PyTorch for this call, "
            "accepting that its result is not invariant." % what
        )
    return fallback(*args, **kwargs)


def _kernel_ok(*ts):
    """All tensors CUDA, one supported dtype."""
    dt = None
    for t in ts:
        if t is None:
            continue
        if not isinstance(t, torch.Tensor) or not t.is_cuda or t.dtype not in _SUPPORTED:
            return False
        if dt is None:
            dt = t.dtype
        elif t.dtype != dt:
            return False
    return True


def _desc(*ts):
    return ", ".join("%s %s %s" % (tuple(t.shape), t.dtype, t.device.type)
                     if isinstance(t, torch.Tensor) else repr(t) for t in ts)


@contextlib.contextmanager
def batch_invariant_mode(strict=True):
    """Route torch.matmul, ``@``, torch.addmm, F.linear / nn.Linear and
    F.scaled_dot_product_attention through invariant kernels.

    Calls this library cannot make invariant raise ``NotImplementedError``.  With
    ``strict=False`` they fall back to stock PyTorch instead, which means the result
    is no longer guaranteed bitwise reproducible -- use it to find out what a model
    needs, not to ship.  Nesting re-uses the outer block's patches; the originals are
    restored when the outermost block exits, even on an exception
    (mlx_batch_invariant/__init__.py:56-147).
    """
    global _depth

    if _depth:  # already patched; nesting must not stack another set of shims
        _depth += 1
        try:
            yield
        finally:
            _depth -= 1
        return

    saved = {
        "matmul": torch.matmul,
        "matmul_op": torch.Tensor.__matmul__,
        "addmm": torch.addmm,
        "linear": F.linear,
        "linear_forward": torch.nn.Linear.forward,
        "sdpa": F.scaled_dot_product_attention,
    }

    def bi_matmul(a, b, *, out=None):
        if (out is not None or not isinstance(a, torch.Tensor) or not isinstance(b, torch.Tensor)
                or a.ndim < 2 or b.ndim != 2 or not _kernel_ok(a, b)):
            kw = {} if out is None else {"out": out}
            return _unsupported("matmul with %s @ %s" % (_desc(a), _desc(b)),
                                strict, saved["matmul"], a, b, **kw)
        return matmul(a, b)

    def bi_addmm(input, mat1, mat2, *, beta=1, alpha=1, out=None):
        ok = (out is None and isinstance(input, torch.Tensor) and input.ndim == 1
              and mat1.ndim == 2 and mat2.ndim == 2 and input.shape[0] == mat2.shape[-1]
              and _kernel_ok(input, mat1, mat2))
        if not ok:
            kw = {} if out is None else {"out": out}
            return _unsupported("addmm with %s, %s @ %s" % (_desc(input), _desc(mat1), _desc(mat2)),
                                strict, saved["addmm"], input, mat1, mat2, beta=beta,
                                alpha=alpha, **kw)
        return addmm(input, mat1, mat2, alpha=alpha, beta=beta)

    def bi_linear(input, weight, bias=None):
        # The reference silently used stock MLX for x.ndim < 2 even when strict
        # (__init__.py:127-128); here strict means strict.
        if input.ndim < 2 or weight.ndim != 2 or not _kernel_ok(input, weight, bias):
            return _unsupported("linear with %s, weight %s" % (_desc(input), _desc(weight)),
                                strict, saved["linear"], input, weight, bias)
        return linear(input, weight, bias)

    def bi_linear_forward(self, input):
        return bi_linear(input, self.weight, self.bias)

    def bi_sdpa(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None,
                enable_gqa=False):
        def stock():
            return _unsupported(
                "scaled_dot_product_attention with q %s, v %s, dropout_p=%s, is_causal=%s"
                % (_desc(query), _desc(value), dropout_p, is_causal),
                strict, saved["sdpa"], query, key, value, attn_mask=attn_mask,
                dropout_p=dropout_p, is_causal=is_causal, scale=scale, enable_gqa=enable_gqa)

        if (query.ndim != 4 or key.ndim != 4 or value.ndim != 4 or dropout_p
                or not _kernel_ok(query, key, value)):
            return stock()
        B, H, qL, D = query.shape
        Hkv, N, V = key.shape[1], key.shape[2], value.shape[-1]
        if (D % 32 or V % 32 or not head_dims_built(D, V, query.dtype) or Hkv == 0
                or H % Hkv):
            return stock()
        if H != Hkv and not enable_gqa:
            # stock torch broadcasts a single KV head here; that call is not invariant
            return stock()
        if attn_mask is not None and is_causal:
            return stock()
        if attn_mask is not None and not (isinstance(attn_mask, torch.Tensor)
                                          and attn_mask.is_cuda and attn_mask.ndim <= 4):
            return stock()
        sc = 1.0 / math.sqrt(D) if scale is None else float(scale)
        if is_causal:
            # torch's is_causal is top-left aligned: query s sees keys i <= s.
            return _sdpa(query, key, value, sc, 1, 0, None, [0, 0, 0], None)
        m, ms, mode = _mask_args(attn_mask, B, H, qL, N, query.dtype)
        return _sdpa(query, key, value, sc, mode, 0, m, ms, None)

    torch.matmul = bi_matmul
    torch.Tensor.__matmul__ = lambda a, b: bi_matmul(a, b)
    torch.addmm = bi_addmm
    F.linear = bi_linear
    torch.nn.Linear.forward = bi_linear_forward
    F.scaled_dot_product_attention = bi_sdpa
    _depth = 1
    try:
        yield
    finally:
        _depth = 0
        torch.matmul = saved["matmul"]
        torch.Tensor.__matmul__ = saved["matmul_op"]
        torch.addmm = saved["addmm"]
        F.linear = saved["linear"]
        torch.nn.Linear.forward = saved["linear_forward"]
        F.scaled_dot_product_attention = saved["sdpa"]
