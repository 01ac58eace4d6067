"""Multi-GPU execution of the invariant operators: one process per GPU over
torch.distributed (NCCL on GPUs, gloo in the CPU tests).

The reference is single-device; these are the B200 build's sharding plans, chosen so
that sharding never adds a reduction and therefore never changes a bit:

* GEMM, column-parallel over N: rank r owns rows [s_r, e_r) of the (N, K) weight and
  the matching bias slice, computes its (M, e_r - s_r) block with the same kernel,
  tile and K order as a single GPU would use for those columns, and an all-gather
  (pure data movement) assembles (M, N).  K-split or row-parallel plans are not
  offered: their cross-GPU sum would change the bits.
* The all-gather can be fused into the GEMM (FusedColumnParallel): each rank's
  epilogue stores its finished tiles into its own output and, over NVLink peer
  mappings, into every other rank's staging area as one dense block, so the exchange
  overlaps the math tile by tile; each rank then moves the received blocks into its
  output with one local copy kernel.
* Attention, head-parallel: rank r owns query heads [r*H/g, (r+1)*H/g) and the KV
  heads they read, [r*Hkv/g, (r+1)*Hkv/g) (Hkv % g == 0); each row is folded by one
  CTA exactly as on one GPU, and an all-gather over heads assembles the output.
"""

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from ._attention import scaled_dot_product_attention
from ._gemm import _aligned, linear

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


class FusedColumnParallel:
    """Column-parallel ``linear`` over the ranks of `group` with the all-gather fused
    into the GEMM epilogue (libbi.so bi_gemm_allgather).

    Rank r holds rows shard_bounds(n_total, world)[r] of the (n_total, K) weight; every
    rank gets the full (..., n_total) output, bitwise equal to a single-GPU
    ``linear``.  Each rank owns a peer-mapped staging area of `max_rows` x `n_total`
    elements into which the other ranks store their shards as dense blocks; ``linear``
    returns a new tensor (or fills `out`).  All ranks must call ``linear`` and
    ``close`` in the same order.  The flag block counts the calls on the device (epoch
    0), so ``linear`` may be captured in a CUDA graph and replayed.  float16 / bfloat16 only (the tensor-core route), and
    n_total a multiple of 8 (every shard's block rows stay 16-byte aligned).
    """

    def __init__(self, n_total, max_rows, dtype, group=None):
        if dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("the fused all-gather takes float16 or bfloat16")
        if n_total % SHARD_ALIGN:
            raise ValueError("the fused all-gather needs n_total %% %d == 0 (got %d)"
                             % (SHARD_ALIGN, n_total))
        self.group = group
        self.world, self.rank = _group_info(group)
        if self.world > _lib.MAX_PEERS:
            raise ValueError("at most %d ranks" % _lib.MAX_PEERS)
        self.n_total, self.max_rows, self.dtype = n_total, max_rows, dtype
        bounds = shard_bounds(n_total, self.world)
        self.col0, self.col1 = bounds[self.rank]
        self._cols = (ctypes.c_int64 * (self.world + 1))(*([b[0] for b in bounds] + [n_total]))
        es = torch.empty((), dtype=dtype).element_size()
        self._stage_bytes = -(-max_rows * n_total * es // 256) * 256
        L = _lib.lib()
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        _lib.check(L.bi_peer_alloc(self._stage_bytes + _lib.PEER_FLAG_BYTES, ctypes.byref(ptr),
                                   handle), "bi_peer_alloc")
        self._local = ptr.value
        self._ptrs, self._opened = [], []
        try:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group)
            for r, h in enumerate(handles):
                if r == self.rank:
                    self._ptrs.append(self._local)
                    continue
                q = ctypes.c_void_p()
                _lib.check(L.bi_peer_open(h, ctypes.byref(q)), "bi_peer_open")
                self._ptrs.append(q.value)
                self._opened.append(q.value)
        except BaseException:
            # release what this rank holds; its peers fail on their next exchange
            for q in self._opened:
                L.bi_peer_close(q)
            L.bi_peer_free(self._local)
            self._local, self._opened = None, []
            raise
        self._stages = (ctypes.c_void_p * self.world)(*self._ptrs)
        self._flags = (ctypes.c_void_p * self.world)(*[p + self._stage_bytes for p in self._ptrs])
        self._side = None      # stream of the deferred unpacks (linear(..., wait=False))
        self._pending = None   # event: the last deferred unpack has run

    @property
    def shard_rows(self):
        return self.col1 - self.col0

    def linear(self, x, w_shard, bias_shard=None, out=None, wait=True):
        """y = x @ w.T (+ bias) on all ranks; w_shard is this rank's (shard, K) rows.
        `out`, if given, is a contiguous (..., n_total) tensor on x's device.

        wait=False leaves the copy of the peers' blocks into `out` to a side stream,
        where it overlaps whatever the current stream runs next (the next call's GEMM):
        on return this rank's own columns are ready in stream order, the others only
        after ``finish()`` -- call it before anything on the current stream reads them.
        """
        if x.dtype != self.dtype or w_shard.dtype != self.dtype:
            raise ValueError("x and w must be %s" % self.dtype)
        if w_shard.shape[0] != self.shard_rows:
            raise ValueError("rank %d holds %d weight rows, the plan gives it %d"
                             % (self.rank, w_shard.shape[0], self.shard_rows))
        lead, K = tuple(x.shape[:-1]), x.shape[-1]
        M = 1
        for d in lead:
            M *= d
        if M > self.max_rows:
            raise ValueError("%d rows exceed the staging area's %d" % (M, self.max_rows))
        if w_shard.shape[0] and w_shard.shape[1] != K:
            raise ValueError("inner dimensions do not match: %d vs %d" % (K, w_shard.shape[1]))
        if out is None:
            out = torch.empty(*lead, self.n_total, dtype=self.dtype, device=x.device)
        elif (out.shape != (*lead, self.n_total) or out.dtype != self.dtype
              or out.device != x.device or not out.is_contiguous()):
            raise ValueError("out must be a contiguous %s tensor of shape %s on %s"
                             % (self.dtype, (*lead, self.n_total), x.device))
        x2 = _aligned(x.reshape(M, K))
        w2 = _aligned(w_shard) if w_shard.shape[0] else w_shard
        b2 = bias_shard.to(self.dtype).contiguous() if bias_shard is not None else None
        dev = x.device
        cur = torch.cuda.current_stream(dev)
        if self._pending is not None:
            # the previous deferred unpack reads the staging area this call's entry
            # barrier hands back to the peers
            cur.wait_event(self._pending)
            self._pending = None
        L = _lib.lib()
        args = (x2.data_ptr(), K, w2.data_ptr() if w2.numel() else None, K,
                b2.data_ptr() if b2 is not None else None, out.data_ptr(), self.n_total,
                self._stages, self._cols, M, K, 1, 1.0, 1.0, _lib.dtype_code(self.dtype),
                self._flags, self.rank, self.world, 0)
        with torch.cuda.device(dev):
            if wait:
                _lib.check(L.bi_gemm_allgather(*args, cur.cuda_stream), "bi_gemm_allgather")
                return out
            _lib.check(L.bi_gemm_allgather_deferred(*args, cur.cuda_stream),
                       "bi_gemm_allgather_deferred")
            if self._side is None:
                self._side = torch.cuda.Stream(device=dev)
            done = torch.cuda.Event()
            done.record(cur)
            self._side.wait_event(done)
            _lib.check(L.bi_gather_unpack(out.data_ptr(), self.n_total, self._stages, self._cols,
                                          M, self.rank, self.world, _lib.dtype_code(self.dtype),
                                          self._side.cuda_stream), "bi_gather_unpack")
            out.record_stream(self._side)
            self._pending = torch.cuda.Event()
            self._pending.record(self._side)
        return out

    def finish(self):
        """Orders the current stream after the last deferred unpack (linear(...,
        wait=False)): from here on its output holds every rank's columns."""
        if self._pending is not None:
            torch.cuda.current_stream().wait_event(self._pending)

    def close(self):
        """Unmaps the peers' buffers and frees this one (collective)."""
        if self._local is None:
            return
        self.finish()
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        L = _lib.lib()
        for q in self._opened:
            L.bi_peer_close(q)
        self._opened = []
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        L.bi_peer_free(self._local)
        self._local = None
