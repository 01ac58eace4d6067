"""Batch-invariant GEMM: matmul, addmm, linear.

Mirrors mlx_batch_invariant/_gemm.py (reference v0.2.0): the same signatures,
argument meaning and ValueError messages, on PyTorch CUDA tensors.  The arithmetic
runs in libbi.so (bi_gemm): one CTA owns the whole K reduction of its output tile,
the tile and the K order depend only on (K, N, dtype, layout) -- never on M -- and the
bias is added to the fp32 accumulator before the single rounding, so a row's bits do
not depend on the other rows computed with it.
"""

import contextlib

import torch

from . import _lib

# How float32 GEMMs run: "exact" -- the CUDA-core route, the reference's fp32 K order
# bit for bit -- or "tf32x3" -- the tensor-core route, three tf32 products per K step
# (within the reference's float32 accuracy bar, not bit-equal to "exact").  Either is
# batch-invariant; pick one per process or model run, not per call.
_FLOAT32_GEMM = "exact"
_FLOAT32_GEMMS = ("exact", "tf32x3")


def set_float32_gemm(mode):
    """Selects the float32 GEMM route: "exact" (default) or "tf32x3"."""
    global _FLOAT32_GEMM
    if mode not in _FLOAT32_GEMMS:
        raise ValueError("float32 GEMM route must be one of %s, got %r" % (_FLOAT32_GEMMS, mode))
    _FLOAT32_GEMM = mode


def get_float32_gemm():
    return _FLOAT32_GEMM


@contextlib.contextmanager
def float32_gemm(mode):
    """Runs the block with the float32 GEMM route `mode`, restoring the previous one."""
    prev = _FLOAT32_GEMM
    set_float32_gemm(mode)
    try:
        yield
    finally:
        set_float32_gemm(prev)


def _tf32x3_takes(dtype, K, N, b_is_nk):
    return (dtype == torch.float32 and _FLOAT32_GEMM == "tf32x3" and K > 0 and K % 4 == 0
            and (b_is_nk or N % 4 == 0))

# The tensor-core tile used for float16 / bfloat16, fixed for every shape and every M
# (cf. the reference's TILE, _gemm.py:27): BM rows per CTA, a pair of CTAs
# (CTA_GROUP = 2) on a 256 x BN tile, 64-deep K blocks, and the 2-SM tcgen05
# instruction UMMA_M x UMMA_N x UMMA_K.
TILE = dict(BM=128, BN=256, BK=64, UMMA_M=256, UMMA_N=256, UMMA_K=16, CTA_GROUP=2)
# The CUDA-core tile (float32, and float16/bfloat16 when K % 8 != 0).
SIMT_TILE = dict(BM=128, BN=128, BK=8)


def tile_for(dtype, K, N, b_is_nk=True):
    """The route and tile bi_gemm takes for (dtype, K, N, layout) under the current
    float32 setting; independent of M."""
    if _tf32x3_takes(dtype, K, N, b_is_nk):
        return dict(route="tf32x3", BM=128, BN=256, BK=32)
    r, bm, bn, bk = _lib.route(dtype, K, N, b_is_nk)
    return dict(route="tcgen05" if r == _lib.ROUTE_TCGEN05 else "simt", BM=bm, BN=bn, BK=bk)


def _aligned(t):
    """`t` made row-contiguous with a 16-byte aligned base (copied only if needed)."""
    if not t.is_contiguous():
        t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


def _check_cuda(*ts):
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("batch-invariant kernels take CUDA tensors, got a %s tensor"
                             % t.device.type)
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("tensors are on different devices: %s and %s" % (dev, t.device))
    return dev


def _gemm(a, b, bias, transpose_b, alpha=1.0, beta=1.0, out=None):
    """Validation follows mlx_batch_invariant/_gemm.py:_gemm (:185-222).  Under
    torch.compile the call is the opaque op mlx_bi::gemm (same implementation)."""
    if out is None and torch.compiler.is_compiling():
        _validate(a, b, bias, transpose_b)
        if bias is not None and bias.dtype != a.dtype:
            bias = bias.to(a.dtype)
        return torch.ops.mlx_bi.gemm(a, b, bias, bool(transpose_b), float(alpha), float(beta))
    return _gemm_eager(a, b, bias, transpose_b, alpha, beta, out)


def _validate(a, b, bias, transpose_b):
    """The reference's argument checks (_gemm.py:187-207); returns (lead, M, K, N)."""
    if a.dtype != b.dtype:
        raise ValueError("a and b must share a dtype, got %s and %s" % (a.dtype, b.dtype))
    if a.ndim < 2 or b.ndim != 2:
        raise ValueError("expected a.ndim >= 2 and b.ndim == 2")
    _lib.dtype_code(a.dtype)
    lead, K = tuple(a.shape[:-1]), a.shape[-1]
    M = 1
    for d in lead:
        M *= d
    kb, N = (b.shape[1], b.shape[0]) if transpose_b else (b.shape[0], b.shape[1])
    if kb != K:
        raise ValueError("inner dimensions do not match: %d vs %d" % (K, kb))
    if bias is not None and tuple(bias.shape) != (N,):
        raise ValueError("bias must have shape (%d,), got %s" % (N, tuple(bias.shape)))
    _check_cuda(a, b, bias)
    return lead, M, K, N


def _gemm_eager(a, b, bias, transpose_b, alpha=1.0, beta=1.0, out=None):
    """The libbi.so call behind matmul / addmm / linear (and the mlx_bi::gemm op)."""
    lead, M, K, N = _validate(a, b, bias, transpose_b)
    code = _lib.dtype_code(a.dtype)
    if bias is not None and bias.dtype != a.dtype:
        bias = bias.to(a.dtype)
    dev = a.device

    a2 = _aligned(a.reshape(M, K))
    b2 = _aligned(b)
    bias2 = bias.contiguous() if bias is not None else None
    if out is None:
        out = torch.empty((M, N), dtype=a.dtype, device=dev)
    elif tuple(out.shape) != (M, N) or out.dtype != a.dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous (%d, %d) %s tensor" % (M, N, a.dtype))
    if M and N:
        with torch.cuda.device(dev):
            if _tf32x3_takes(a.dtype, K, N, transpose_b):
                st = _lib.lib().bi_gemm_tf32x3(
                    a2.data_ptr(), K, b2.data_ptr(), b2.shape[1],
                    bias2.data_ptr() if bias2 is not None else None,
                    out.data_ptr(), N, M, N, K, 1 if transpose_b else 0, float(alpha),
                    float(beta), _lib.stream_handle(dev))
                _lib.check(st, "bi_gemm_tf32x3")
            else:
                st = _lib.lib().bi_gemm(
                    a2.data_ptr(), K, b2.data_ptr(), b2.shape[1],
                    bias2.data_ptr() if bias2 is not None else None,
                    out.data_ptr(), N, M, N, K, 1 if transpose_b else 0, float(alpha),
                    float(beta), code, _lib.stream_handle(dev))
                _lib.check(st, "bi_gemm")
    return out.reshape(*lead, N)


def matmul(a, b):
    """a @ b with b laid out (K, N). Bitwise independent of a's leading dimensions."""
    return _gemm(a, b, None, transpose_b=False)


def addmm(c, a, b, alpha=1.0, beta=1.0):
    """alpha * (a @ b) + beta * c, with b laid out (K, N) and c of shape (N,)."""
    return _gemm(a, b, c, transpose_b=False, alpha=alpha, beta=beta)


def linear(x, w, bias=None):
    """x @ w.T (+ bias) with w laid out (N, K), the nn.Linear convention.

    Takes the weight in its stored layout so no transposed copy is made.
    """
    return _gemm(x, w, bias, transpose_b=True)


# The reference's affine-quantized path (_gemm.py:163-173, 243-285) works on MLX's
# packed uint32 format, which has no PyTorch counterpart; it is not part of this
# build, so no bit width is supported.
QUANT_BITS = ()


def quantized_linear(x, w, scales, qbias, group_size, bits):
    """Not built: MLX's affine-quantized weights have no PyTorch equivalent."""
    raise NotImplementedError(
        "quantized_linear is not part of the B200 build (MLX affine-quantized weights "
        "have no PyTorch counterpart)")
