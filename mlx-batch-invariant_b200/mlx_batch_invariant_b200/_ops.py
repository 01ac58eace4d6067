"""torch.library registrations of the invariant operators, so torch.compile sees each
as one opaque op (the reference's kernels are likewise opaque to mx.compile).

Eager calls go straight to libbi.so; under torch.compile the public functions call
these ops, whose real implementation is that same eager path -- the bits are the
same either way.  The fake implementations give the output's shape and dtype only.
"""

from typing import List, Optional

import torch

_NS = "mlx_bi"


@torch.library.custom_op(_NS + "::gemm", mutates_args=())
def gemm(a: torch.Tensor, b: torch.Tensor, bias: Optional[torch.Tensor], transpose_b: bool,
         alpha: float, beta: float) -> torch.Tensor:
    """bi_gemm: alpha * (a @ B) + beta * bias with B = b.T if transpose_b else b."""
    from ._gemm import _gemm_eager
    return _gemm_eager(a, b, bias, transpose_b, alpha, beta)


@gemm.register_fake
def _gemm_fake(a, b, bias, transpose_b, alpha, beta):
    n = b.shape[0] if transpose_b else b.shape[1]
    return a.new_empty((*a.shape[:-1], n))


@torch.library.custom_op(_NS + "::sdpa", mutates_args=())
def sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, mask_mode: int,
         causal_offset: int, mask: Optional[torch.Tensor], mask_strides: List[int],
         sinks: Optional[torch.Tensor]) -> torch.Tensor:
    """bi_sdpa on validated arguments (see _attention._sdpa)."""
    from ._attention import _sdpa_eager
    return _sdpa_eager(q, k, v, scale, mask_mode, causal_offset, mask, mask_strides, sinks)


@sdpa.register_fake
def _sdpa_fake(q, k, v, scale, mask_mode, causal_offset, mask, mask_strides, sinks):
    return q.new_empty((q.shape[0], q.shape[1], q.shape[2], v.shape[3]))
