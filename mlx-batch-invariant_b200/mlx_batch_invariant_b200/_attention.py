"""Batch-invariant scaled dot-product attention.

Mirrors mlx_batch_invariant/_attention.py (reference v0.2.0): same signature, mask
forms, sinks and errors, on PyTorch CUDA tensors.  libbi.so's bi_sdpa runs one CTA
per query row and (group of) head(s) over all keys in 32 fixed strides with an fp32
online softmax; no split-KV, no second pass, no route switch on query length, GQA
factor or context length, so a token's output bits are the same in decode and in
any chunked prefill.
"""

import math

import torch

from . import _lib

BN = 32  # partial softmax states per row -- also the stride of the key walk
BD = 32  # head dims must be multiples of this (reference _attention.py:29-30)
MAX_HEAD_DIM = 640  # largest head dim this build has a kernel for (16-bit types)
MAX_HEAD_DIM_F32 = 384  # float32: D, V <= 384 and D + V <= 768


def head_dims_built(D, V, dtype):
    """Whether libbi.so has a kernel for head dims (D, V) (multiples of 32) in dtype."""
    if dtype == torch.float32:
        return D <= MAX_HEAD_DIM_F32 and V <= MAX_HEAD_DIM_F32 and D + V <= 2 * MAX_HEAD_DIM_F32
    return D <= MAX_HEAD_DIM and V <= MAX_HEAD_DIM


def _mask_args(mask, B, H, qL, N, dtype):
    """Returns (tensor or None, [b_stride, h_stride, q_stride], mode).

    Follows mlx_batch_invariant/_attention.py:_mask_args (:173-202): a bool mask
    becomes 0 / -inf in q's dtype, every mask is cast to q's dtype, left-padded to 4-D
    and must broadcast over (B, H, qL, N); broadcast dims get stride 0.
    """
    if mask is None:
        return None, [0, 0, 0], 0
    if isinstance(mask, str):
        if mask != "causal":
            raise ValueError("string mask must be 'causal', got %r" % (mask,))
        return None, [0, 0, 0], 1

    m = mask
    if m.dtype == torch.bool:
        zero = torch.zeros((), dtype=dtype, device=m.device)
        ninf = torch.full((), -math.inf, dtype=dtype, device=m.device)
        m = torch.where(m, zero, ninf)
    m = m.to(dtype)
    while m.ndim < 4:
        m = m.unsqueeze(0)
    if m.ndim != 4:
        raise ValueError("mask must have at most 4 dimensions, got %d" % mask.ndim)
    Bm, Hm, Lm, Nm = m.shape
    if Nm != N or Lm not in (1, qL) or Hm not in (1, H) or Bm not in (1, B):
        raise ValueError(
            "mask shape %s is not broadcastable to (%d, %d, %d, %d)"
            % (tuple(m.shape), B, H, qL, N))
    m = m.contiguous()
    strides = [0 if Bm == 1 else Hm * Lm * N, 0 if Hm == 1 else Lm * N, 0 if Lm == 1 else N]
    return m, strides, 2


def _aligned_heads(t, row_contiguous):
    """`t` with a contiguous last dim (and row-contiguous (L, D) blocks when asked),
    16-byte aligned base and strides; copied only when needed."""
    es = t.element_size()
    vec = 16 // es
    ok = t.stride(-1) == 1 and t.data_ptr() % 16 == 0
    # (a zero stride over an extent above 1 -- an expanded tensor -- is copied too:
    # the tensor-core route reads k and v through TMA, which needs real strides)
    ok = ok and all(s % vec == 0 and (s > 0 or n == 1)
                    for s, n in zip(t.stride()[:-1], t.shape[:-1]))
    if row_contiguous:
        ok = ok and (t.shape[2] <= 1 or t.stride(2) == t.shape[3])
    if not ok:
        t = t.contiguous()
        if t.data_ptr() % 16:
            t = t.clone()
    return t


def _sdpa(q, k, v, scale, mask_mode, causal_offset, m, mstrides, sinks):
    """bi_sdpa on validated arguments; under torch.compile the opaque op mlx_bi::sdpa
    (same implementation)."""
    if torch.compiler.is_compiling():
        return torch.ops.mlx_bi.sdpa(q, k, v, float(scale), int(mask_mode), int(causal_offset),
                                     m, [int(x) for x in mstrides], sinks)
    return _sdpa_eager(q, k, v, scale, mask_mode, causal_offset, m, mstrides, sinks)


def _sdpa_eager(q, k, v, scale, mask_mode, causal_offset, m, mstrides, sinks):
    B, H, qL, D = q.shape
    _, Hkv, N, V = v.shape
    dev = q.device
    out = torch.empty((B, H, qL, V), dtype=q.dtype, device=dev)
    if B == 0 or H == 0 or qL == 0:
        return out
    q2 = _aligned_heads(q, False)
    k2 = _aligned_heads(k, True)
    v2 = _aligned_heads(v, True)
    with torch.cuda.device(dev):
        st = _lib.lib().bi_sdpa(
            q2.data_ptr(), _lib.i64_3(q2.stride()[:3]),
            k2.data_ptr(), _lib.i64_2(k2.stride()[:2]),
            v2.data_ptr(), _lib.i64_2(v2.stride()[:2]),
            m.data_ptr() if m is not None else None, _lib.i64_3(mstrides), mask_mode,
            int(causal_offset), sinks.data_ptr() if sinks is not None else None, float(scale),
            B, H, Hkv, qL, N, D, V, _lib.dtype_code(q.dtype),
            out.data_ptr(), _lib.i64_3(out.stride()[:3]), _lib.stream_handle(dev))
    _lib.check(st, "bi_sdpa")
    return out


def scaled_dot_product_attention(q, k, v, *, scale=None, mask=None, sinks=None):
    """Bitwise-invariant SDPA. ``q`` is (B, H, L, D), ``k``/``v`` are (B, Hkv, N, ...).

    ``mask`` may be ``None``, ``"causal"`` (bottom-right aligned: query s of qL sees
    keys i <= N - qL + s), or an additive/boolean tensor broadcastable over the
    batch, head and query dimensions.  ``sinks`` is an optional per-query-head logit
    of shape ``(H,)``.  Validation follows mlx_batch_invariant/_attention.py:205-250.
    """
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("q, k and v must be 4-dimensional (B, H, L, D)")
    if not (q.dtype == k.dtype == v.dtype):
        raise ValueError("q, k and v must share a dtype")

    B, H, qL, D = q.shape
    Bk, Hkv, N, Dk = k.shape
    Bv, Hv, Nv, V = v.shape
    if (Bk, Hv, Nv, Dk) != (B, Hkv, N, D) or Bv != B:
        raise ValueError("inconsistent q/k/v shapes: %s %s %s"
                         % (tuple(q.shape), tuple(k.shape), tuple(v.shape)))
    if Hkv == 0 or H % Hkv:
        raise ValueError("head count %d is not a multiple of kv head count %d" % (H, Hkv))
    if D % BD or V % BD:
        raise ValueError("head dimensions must be multiples of %d, got D=%d V=%d" % (BD, D, V))
    if not head_dims_built(D, V, q.dtype):
        raise NotImplementedError(
            "attention with D=%d, V=%d in %s is not built (D, V <= %d for 16-bit types; "
            "D, V <= %d and D + V <= %d for float32)"
            % (D, V, q.dtype, MAX_HEAD_DIM, MAX_HEAD_DIM_F32, 2 * MAX_HEAD_DIM_F32))
    _lib.dtype_code(q.dtype)

    scale = 1.0 / math.sqrt(D) if scale is None else float(scale)
    m, mstrides, mode = _mask_args(mask, B, H, qL, N, q.dtype)
    if sinks is not None:
        if tuple(sinks.shape) != (H,):
            raise ValueError("sinks must have shape (%d,), got %s" % (H, tuple(sinks.shape)))
        sinks = sinks.to(q.dtype).contiguous()
    _check = [t for t in (q, k, v, m, sinks) if t is not None]
    for t in _check:
        if not t.is_cuda:
            raise ValueError("batch-invariant kernels take CUDA tensors, got a %s tensor"
                             % t.device.type)
    causal_offset = N - qL if mode == 1 else 0
    return _sdpa(q, k, v, scale, mode, causal_offset, m, mstrides, sinks)
