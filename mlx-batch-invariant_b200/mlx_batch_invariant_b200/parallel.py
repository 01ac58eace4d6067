"""Multi-GPU execution of the invariant operators: one process per GPU over
torch.distributed (NCCL on GPUs, gloo in the CPU tests).

The reference is single-device; these are the B200 build's sharding plans, chosen so
that sharding never adds a reduction and therefore never changes a bit:

* GEMM, column-parallel over N: rank r owns rows [s_r, e_r) of the (N, K) weight and
  the matching bias slice, computes its (M, e_r - s_r) block with the same kernel,
  tile and K order as a single GPU would use for those columns, and an all-gather
  (pure data movement) assembles (M, N).  K-split or row-parallel plans are not
  offered: their cross-GPU sum would change the bits.
* Attention, head-parallel: rank r owns query heads [r*H/g, (r+1)*H/g) and the KV
  heads they read, [r*Hkv/g, (r+1)*Hkv/g) (Hkv % g == 0); each row is folded by one
  CTA exactly as on one GPU, and an all-gather over heads assembles the output.
"""

import torch
import torch.distributed as dist

from ._attention import scaled_dot_product_attention
from ._gemm import linear

# Shard widths are rounded up to this many columns so every shard's row stride and
# output offset stay 16-byte aligned for 16-bit types.
SHARD_ALIGN = 8


def shard_bounds(n, world, align=SHARD_ALIGN):
    """[(start, stop)] column ranges of an N-wide output over `world` ranks: equal
    widths rounded up to `align`, the last shard ragged (possibly empty)."""
    if world <= 0:
        raise ValueError("world size must be positive")
    per = -(-n // world)
    per = -(-per // align) * align
    return [(min(r * per, n), min((r + 1) * per, n)) for r in range(world)]


def shard_weight(w, bias, rank, world, align=SHARD_ALIGN):
    """This rank's rows of an (N, K) weight and its bias slice (views, no copy)."""
    s, e = shard_bounds(w.shape[0], world, align)[rank]
    return w[s:e], (bias[s:e] if bias is not None else None)


def _group_info(group):
    return dist.get_world_size(group), dist.get_rank(group)


def gather_columns(y_local, n_total, group=None):
    """All-gather of every rank's (M, shard) output block into the full (M, n_total)
    output (shard_bounds layout).  Pure data movement: no arithmetic on the values."""
    world, rank = _group_info(group)
    bounds = shard_bounds(n_total, world)
    per = bounds[0][1] - bounds[0][0]
    M = y_local.shape[0]
    if world == 1:
        return y_local
    y = y_local
    if y.shape[1] != per:
        pad = torch.zeros((M, per), dtype=y.dtype, device=y.device)
        pad[:, :y.shape[1]] = y
        y = pad
    # rank blocks concatenated along dim 0 (the layout every backend accepts)
    gathered = torch.empty((world * M, per), dtype=y.dtype, device=y.device)
    dist.all_gather_into_tensor(gathered, y.contiguous(), group=group)
    out = gathered.view(world, M, per).permute(1, 0, 2).reshape(M, world * per)
    if world * per != n_total:
        out = out[:, :n_total]
    return out.contiguous()


def gather_columns_on(stream, y_local, n_total, group=None, ready=None):
    """gather_columns issued on `stream` (after `ready`, an event of the stream that
    produced y_local), so the exchange of one output overlaps the next GEMM on the
    producing stream.  The result is valid on `stream`; the caller orders its
    consumers after it (e.g. producer_stream.wait_stream(stream))."""
    with torch.cuda.stream(stream):
        if ready is not None:
            stream.wait_event(ready)
        y_local.record_stream(stream)
        return gather_columns(y_local, n_total, group)


def column_parallel_linear(x, w_shard, bias_shard, n_total, group=None, local_op=linear):
    """y = x @ w.T + bias over all ranks, w sharded by rows (shard_weight); every rank
    returns the full (..., n_total) output, bitwise equal to a single-GPU linear."""
    world, rank = _group_info(group)
    s, e = shard_bounds(n_total, world)[rank]
    if w_shard.shape[0] != e - s:
        raise ValueError("rank %d holds %d weight rows, the plan gives it %d"
                         % (rank, w_shard.shape[0], e - s))
    lead = tuple(x.shape[:-1])
    x2 = x.reshape(-1, x.shape[-1])
    if e > s:
        y = local_op(x2, w_shard, bias_shard)
    else:
        y = torch.empty((x2.shape[0], 0), dtype=x.dtype, device=x.device)
    return gather_columns(y, n_total, group).reshape(*lead, n_total)


def gather_heads(y_local, group=None):
    """All-gather of every rank's (B, H/g, qL, V) attention output into (B, H, qL, V)."""
    world, _ = _group_info(group)
    if world == 1:
        return y_local
    B, hl, qL, V = y_local.shape
    gathered = torch.empty((world * B, hl, qL, V), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(gathered, y_local.contiguous(), group=group)
    return gathered.view(world, B, hl, qL, V).permute(1, 0, 2, 3, 4).reshape(
        B, world * hl, qL, V).contiguous()


def head_shard(H, Hkv, rank, world):
    """(q-head range, kv-head range) owned by `rank`."""
    if H % world or Hkv % world:
        raise ValueError("head-parallel attention needs H %% g == 0 and Hkv %% g == 0 "
                         "(H=%d, Hkv=%d, g=%d)" % (H, Hkv, world))
    hq, hk = H // world, Hkv // world
    return (rank * hq, (rank + 1) * hq), (rank * hk, (rank + 1) * hk)


def head_parallel_sdpa(q, k, v, *, scale=None, mask=None, sinks=None, group=None,
                       local_op=scaled_dot_product_attention):
    """Attention with q/k/v replicated on every rank; each rank computes its heads and
    an all-gather assembles (B, H, qL, V), bitwise equal to a single-GPU call."""
    world, rank = _group_info(group)
    B, H, qL, D = q.shape
    Hkv = k.shape[1]
    (h0, h1), (k0, k1) = head_shard(H, Hkv, rank, world)
    m = mask
    if isinstance(mask, torch.Tensor):
        mm = mask
        while mm.ndim < 4:
            mm = mm.unsqueeze(0)
        m = mm[:, h0:h1] if mm.shape[1] == H else mm
    y = local_op(q[:, h0:h1], k[:, k0:k1], v[:, k0:k1], scale=scale, mask=m,
                 sinks=sinks[h0:h1] if sinks is not None else None)
    return gather_heads(y, group)
