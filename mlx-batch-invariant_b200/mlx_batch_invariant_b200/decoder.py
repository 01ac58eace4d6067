"""Llama-shaped decoder: the end-to-end invariance harness.

The reference's harness (bench/bench.py:108-246: build_model, e2e, determinism) runs a
random-init Llama-style decoder under batch_invariant_mode and checks that the logits
of a prompt in batch slot 0 do not change when other prompts share the batch.  This is
the same check on PyTorch CUDA tensors, with the shape of BASELINE config 4: 32 layers,
d_model 4096, 32 query / 8 KV heads of 128, SwiGLU 14336, RMSNorm eps 1e-5, RoPE theta
500000, vocab 128256, bf16 weights ~ N(0, 0.02); one prefill, then greedy decode steps
against a static KV cache.

On g GPUs (one process each, torch.distributed) every layer is column-parallel, so no
value is ever summed across GPUs and the logits are also bitwise those of one GPU:

* q/k/v: one fused weight per rank holding the rows of its query heads
  [r*H/g, (r+1)*H/g) and KV heads [r*Hkv/g, (r+1)*Hkv/g); attention runs on the
  rank's own heads against its own shard of the KV cache;
* the attention output is all-gathered (pure data movement) before o_proj;
* o_proj, down_proj and the LM head are column-parallel GEMMs whose output is
  all-gathered -- fused into the GEMM epilogue (parallel.FusedColumnParallel) or,
  with exchange="nccl", by a separate NCCL all-gather;
* gate/up: rank r holds rows shard_bounds(inter, g)[r] of both, applies SwiGLU to its
  slice and all-gathers the activation before down_proj.

RMSNorm, the embedding lookup and the residual adds are stock PyTorch ops run on
replicated rows; RoPE with the KV-cache write, and SwiGLU, are two fused libbi.so
kernels (bi_rope_kv, bi_swiglu) on CUDA and the equivalent torch expressions on CPU.
Each computes every output element on its own, so all are batch-invariant on B200
(tests/test_mode_gpu.py and tests/test_decoder_gpu.py guard that).
"""

import dataclasses
import math
import time

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import _lib, parallel
from ._attention import scaled_dot_product_attention


@dataclasses.dataclass(frozen=True)
class DecoderConfig:
    layers: int = 32
    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    inter: int = 14336
    vocab: int = 128256
    eps: float = 1e-5
    rope_theta: float = 500000.0
    init_std: float = 0.02


LLAMA_8B = DecoderConfig()


def _weight(seed, rows, cols, std, device, dtype):
    """A seeded (rows, cols) ~ N(0, std) weight, the same bits on every device."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    w = torch.randn((rows, cols), generator=g, device=device, dtype=torch.float32)
    return (w * std).to(dtype)


def _rope(t, cos, sin):
    """Rotate-half RoPE in fp32 (each output element from its own inputs), rounded
    back to t's dtype.  t (B, heads, L, hd); cos/sin (L, hd/2) fp32."""
    h = t.shape[-1] // 2
    x = t.float()
    x1, x2 = x[..., :h], x[..., h:]
    return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1).to(t.dtype)


class Decoder:
    """Random-init Llama-style decoder with a static KV cache, sharded column-parallel
    over the ranks of `group` (or unsharded with single=True / no process group).

    prefill(ids) and decode(tok) return the logits of each row's last position,
    (B, vocab), on every rank.  Run them inside batch_invariant_mode() for the
    invariant path; outside it the local GEMMs and attention are stock PyTorch (the
    control, and the CPU runs of the sharding plan).
    """

    def __init__(self, cfg=LLAMA_8B, max_batch=8, max_len=640, dtype=torch.bfloat16,
                 device=None, seed=0, group=None, single=False, exchange="fused"):
        if exchange not in ("fused", "nccl"):
            raise ValueError("exchange must be 'fused' or 'nccl'")
        self.cfg, self.dtype = cfg, dtype
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        distributed = dist.is_available() and dist.is_initialized() and not single
        self.group = group
        self.world = dist.get_world_size(group) if distributed else 1
        self.rank = dist.get_rank(group) if distributed else 0
        self.exchange = exchange
        H, Hkv, hd, d, inter = cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.hidden, cfg.inter
        g, r = self.world, self.rank
        (h0, h1), (k0, k1) = parallel.head_shard(H, Hkv, r, g)
        self.hq, self.hk = h1 - h0, k1 - k0
        d0, d1 = parallel.shard_bounds(d, g)[r]
        i0, i1 = parallel.shard_bounds(inter, g)[r]
        v0, v1 = parallel.shard_bounds(cfg.vocab, g)[r]
        self.inter_local = i1 - i0
        dev, std = self.device, cfg.init_std

        def w(seed_off, rows, cols, lo, hi):
            full = _weight(seed * 1_000_003 + seed_off, rows, cols, std, dev, dtype)
            part = full[lo:hi].contiguous()
            del full
            return part

        self.layers = []
        for layer in range(cfg.layers):
            base = 16 * (layer + 1)
            wq = w(base + 1, H * hd, d, h0 * hd, h1 * hd)
            wk = w(base + 2, Hkv * hd, d, k0 * hd, k1 * hd)
            wv = w(base + 3, Hkv * hd, d, k0 * hd, k1 * hd)
            wg = w(base + 5, inter, d, i0, i1)
            wu = w(base + 6, inter, d, i0, i1)
            self.layers.append(dict(
                wqkv=torch.cat((wq, wk, wv)).contiguous(),
                wo=w(base + 4, d, H * hd, d0, d1),
                wgu=torch.cat((wg, wu)).contiguous(),
                wd=w(base + 7, d, inter, d0, d1),
                n1=torch.ones(d, dtype=dtype, device=dev),
                n2=torch.ones(d, dtype=dtype, device=dev)))
            del wq, wk, wv, wg, wu
        self.embed = w(1, cfg.vocab, d, 0, cfg.vocab)
        self.norm = torch.ones(d, dtype=dtype, device=dev)
        self.head = w(2, cfg.vocab, d, v0, v1)

        self.max_batch, self.max_len = max_batch, max_len
        shape = (max_batch, self.hk, max_len, hd)
        self.cache_k = [torch.zeros(shape, dtype=dtype, device=dev) for _ in self.layers]
        self.cache_v = [torch.zeros(shape, dtype=dtype, device=dev) for _ in self.layers]
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, hd, 2, device=dev,
                                                     dtype=torch.float32) / hd))
        ang = torch.arange(max_len, device=dev, dtype=torch.float32)[:, None] * inv[None, :]
        self.cos, self.sin = torch.cos(ang), torch.sin(ang)
        self._key_pos = torch.arange(max_len, device=dev)
        self.pos = 0
        self._fused = {}
        if self.world > 1 and exchange == "fused":
            rows = max_batch * max_len
            self._fused[d] = parallel.FusedColumnParallel(d, rows, dtype, group)
            self._fused["head"] = parallel.FusedColumnParallel(cfg.vocab, max_batch, dtype,
                                                               group)

    # ------------------------------------------------------------------ plumbing
    def close(self):
        """Releases the peer-mapped exchange buffers (collective when sharded)."""
        for f in self._fused.values():
            f.close()
        self._fused = {}

    def num_params(self):
        c = self.cfg
        per_layer = (c.heads + 2 * c.kv_heads) * c.head_dim * c.hidden \
            + c.heads * c.head_dim * c.hidden + 3 * c.hidden * c.inter + 2 * c.hidden
        return c.layers * per_layer + 2 * c.vocab * c.hidden + c.hidden

    def _gather(self, t, n_total):
        """(..., n_local) on every rank -> (..., n_total): the all-gather of a
        column-parallel activation (shard_bounds layout)."""
        if self.world == 1:
            return t
        lead = t.shape[:-1]
        y = parallel.gather_columns(t.reshape(-1, t.shape[-1]), n_total, self.group)
        return y.reshape(*lead, n_total)

    def _column(self, x, w_shard, n_total, key):
        """x @ w.T over the ranks (w sharded by rows), full output on every rank."""
        if self.world > 1 and self.exchange == "fused":
            return self._fused[key].linear(x, w_shard)
        return self._gather(F.linear(x, w_shard), n_total)

    def _rope_kv(self, qkv, B, L, li, pos):
        """libbi.so bi_rope_kv: rotated q (B, hq, L, hd), and the rotated k / the v of the
        L new rows written into layer li's cache at position (pos or self.pos) + l."""
        hd = self.cfg.head_dim
        q = torch.empty((B, self.hq, L, hd), dtype=self.dtype, device=self.device)
        qkv = qkv.contiguous()
        ck, cv = self.cache_k[li], self.cache_v[li]
        st = _lib.lib().bi_rope_kv(
            qkv.data_ptr(), B, L, self.hq, self.hk, hd, self.cos.data_ptr(), self.sin.data_ptr(),
            self.pos if pos is None else 0, pos.data_ptr() if pos is not None else None,
            self.max_len, q.data_ptr(), ck.data_ptr(), cv.data_ptr(), _lib.i64_3(ck.stride()[:3]),
            _lib.dtype_code(self.dtype), _lib.stream_handle(self.device))
        _lib.check(st, "bi_rope_kv")
        return q

    def _swiglu(self, gu):
        """libbi.so bi_swiglu: silu(gate) * up of a [gate | up] projection."""
        lead, width = gu.shape[:-1], gu.shape[-1]
        g2 = gu.reshape(-1, width).contiguous()
        out = torch.empty((g2.shape[0], width // 2), dtype=self.dtype, device=self.device)
        _lib.check(_lib.lib().bi_swiglu(g2.data_ptr(), out.data_ptr(), g2.shape[0], width // 2,
                                        _lib.dtype_code(self.dtype),
                                        _lib.stream_handle(self.device)), "bi_swiglu")
        return out.reshape(*lead, width // 2)

    def _attention(self, q, k, v, L, mask=None):
        from . import is_enabled
        if is_enabled():
            # bottom-right causal rule, right for chunked prefill too
            m = mask if mask is not None else ("causal" if L > 1 else None)
            return scaled_dot_product_attention(q, k, v, scale=1.0 / math.sqrt(q.shape[-1]),
                                                mask=m)
        if mask is not None:
            return F.scaled_dot_product_attention(q, k, v, attn_mask=mask, enable_gqa=True)
        if L > 1 and k.shape[2] != L:
            raise NotImplementedError("the stock path prefills from position 0 only")
        return F.scaled_dot_product_attention(q, k, v, is_causal=L > 1, enable_gqa=True)

    # ------------------------------------------------------------------ forward
    def _forward(self, ids, pos=None):
        """Logits of each row's last position.  pos None: the host position self.pos
        (prefill or an eager decode step).  pos a (1,) device tensor: one decode step
        whose position is read on the device -- RoPE rows by index_select, the cache
        write by index_copy_, and attention over the whole cache with the keys after
        the position masked out (a masked key is skipped, so the logits are those of
        the eager step) -- the form a CUDA graph can replay at every position."""
        cfg = self.cfg
        B, L = ids.shape
        static = pos is not None
        if B > self.max_batch or (static and L != 1) or (
                not static and self.pos + L > self.max_len):
            raise ValueError("batch %d / length %d do not fit the cache (%d, %d)"
                             % (B, self.pos + L, self.max_batch, self.max_len))
        d, hd, hq, hk = cfg.hidden, cfg.head_dim, self.hq, self.hk
        if static:
            cos, sin = self.cos.index_select(0, pos), self.sin.index_select(0, pos)
            mask = torch.where(self._key_pos <= pos, 0.0, float("-inf")).to(self.dtype)
            mask = mask.view(1, 1, 1, self.max_len)
        else:
            p0, mask = self.pos, None
            cos, sin = self.cos[p0:p0 + L], self.sin[p0:p0 + L]
        native = self.device.type == "cuda"  # fused kernels; CPU runs keep the torch ops
        x = F.embedding(ids, self.embed)
        for li, p in enumerate(self.layers):
            y = F.rms_norm(x, (d,), p["n1"], cfg.eps)
            qkv = F.linear(y, p["wqkv"])
            ck, cv = self.cache_k[li][:B], self.cache_v[li][:B]
            if native:
                q = self._rope_kv(qkv, B, L, li, pos)
            else:
                q, k, v = qkv.split((hq * hd, hk * hd, hk * hd), dim=-1)
                q = _rope(q.reshape(B, L, hq, hd).transpose(1, 2), cos, sin)
                k = _rope(k.reshape(B, L, hk, hd).transpose(1, 2), cos, sin)
                v = v.reshape(B, L, hk, hd).transpose(1, 2)
                if static:
                    ck.index_copy_(2, pos, k)
                    cv.index_copy_(2, pos, v)
                else:
                    ck[:, :, p0:p0 + L] = k
                    cv[:, :, p0:p0 + L] = v
            if static:
                a = self._attention(q, ck, cv, 1, mask)
            else:
                a = self._attention(q, ck[:, :, :p0 + L], cv[:, :, :p0 + L], L)
            a = self._gather(a.transpose(1, 2).reshape(B, L, hq * hd), cfg.heads * hd)
            x = x + self._column(a, p["wo"], d, d)
            y = F.rms_norm(x, (d,), p["n2"], cfg.eps)
            gu = F.linear(y, p["wgu"])
            if native:
                act = self._swiglu(gu)
            else:
                gate, up = gu.split((self.inter_local, self.inter_local), dim=-1)
                act = F.silu(gate) * up
            act = self._gather(act, cfg.inter)
            x = x + self._column(act, p["wd"], d, d)
        if not static:
            self.pos += L
        h = F.rms_norm(x[:, -1], (d,), self.norm, cfg.eps)
        return self._column(h, self.head, cfg.vocab, "head")

    def prefill(self, ids):
        """Resets the cache and runs the prompt ids (B, L); logits (B, vocab)."""
        self.pos = 0
        return self._forward(ids)

    def decode(self, tok):
        """One eager step for tok (B,) or (B, 1); logits (B, vocab)."""
        return self._forward(tok.reshape(-1, 1))

    def _greedy_step(self, tok, pos):
        """The static decode step: logits for tok (B, 1) at device position pos, then
        tok <- argmax and pos <- pos + 1, all on the device."""
        logits = self._forward(tok, pos)
        tok.copy_(logits.argmax(dim=-1, keepdim=True))
        pos.add_(1)
        return logits


class DecodeGraph:
    """One greedy decode step at a fixed batch, captured once in a CUDA graph and
    replayed for every position (the token and position live in device buffers that
    the step itself advances).  Capture inside batch_invariant_mode to record the
    invariant kernels; replays need no mode.  Sharded models capture their NCCL and
    fused all-gathers too (the fused exchange counts its epochs on the device)."""

    def __init__(self, model, batch):
        self.model, self.batch = model, batch
        dev = model.device
        self.tok = torch.zeros((batch, 1), dtype=torch.long, device=dev)
        # the warm-up writes the last cache slot, which every later step at that
        # position rewrites before reading it
        self.pos = torch.full((1,), model.max_len - 1, dtype=torch.long, device=dev)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            model._greedy_step(self.tok, self.pos)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.pos.fill_(model.max_len - 1)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits = model._greedy_step(self.tok, self.pos)

    def start(self, tok, pos):
        """Continue from host position `pos` with tokens tok (B,) (device tensors)."""
        pos = int(pos)
        if not 0 <= pos < self.model.max_len:
            raise ValueError("decode position %d is outside the cache [0, %d)"
                             % (pos, self.model.max_len))
        self.tok.copy_(tok.reshape(self.batch, 1))
        self.pos.fill_(pos)
        self._next = pos  # host copy of the position the next replay writes

    def step(self):
        """One decode step; returns the graph's logits buffer (overwritten by the next).
        Refuses to run past the end of the static cache (the replay's position lives on
        the device, where nothing else would stop it)."""
        nxt = getattr(self, "_next", None)
        if nxt is None:
            raise RuntimeError("DecodeGraph.start() must come before step()")
        if nxt >= self.model.max_len:
            raise ValueError("decode position %d is past the cache length %d"
                             % (nxt, self.model.max_len))
        self.graph.replay()
        self._next = nxt + 1
        return self.logits


def generate(model, ids, steps, graph=None):
    """Greedy: prefill, then `steps` decode steps (replays of `graph`, a DecodeGraph of
    this batch, if given).  Returns (list of (B, vocab) logits, prefill seconds, decode
    seconds), timed on the device."""
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    ev[0].record()
    logits = [model.prefill(ids)]
    ev[1].record()
    if graph is not None:
        graph.start(logits[0].argmax(dim=-1), model.pos)
        for _ in range(steps):
            logits.append(graph.step().clone())
    else:
        for _ in range(steps):
            logits.append(model.decode(logits[-1].argmax(dim=-1)))
    ev[2].record()
    torch.cuda.synchronize()
    return logits, ev[0].elapsed_time(ev[1]) / 1e3, ev[1].elapsed_time(ev[2]) / 1e3


def prompts(cfg, batch, length, device, seed=7):
    """The shared prompt in slot 0 and seeded random prompts in the other slots."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    shared = torch.randint(0, cfg.vocab, (1, length), generator=g, device=device)
    others = torch.randint(0, cfg.vocab, (max(batch - 1, 0), length), generator=g,
                           device=device)
    return torch.cat((shared, others))[:batch]


def slot0_bits(logits):
    """The slot-0 rows of a generate() run, as raw bit patterns (steps, vocab)."""
    rows = torch.stack([t[0] for t in logits])
    return rows.view(torch.int32 if rows.element_size() == 4 else torch.int16)


def differing(a, b):
    """Per step: how many slot-0 logits differ between two slot0_bits tensors."""
    return (a != b).sum(dim=-1).tolist()


def timed_run(model, batch, prompt, steps, device, warm=True, graph=None):
    """tokens/s of prefill and decode at `batch` (after one untimed run)."""
    ids = prompts(model.cfg, batch, prompt, device)
    if warm:
        generate(model, ids, min(steps, 4), graph)
    if model.world > 1:
        dist.barrier(group=model.group)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    logits, tp, td = generate(model, ids, steps, graph)
    wall = time.perf_counter() - t0
    if model.world > 1:
        t = torch.tensor([tp, td], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=model.group)
        tp, td = t.tolist()
    return {"batch": batch, "prefill_tokens_per_s": batch * prompt / tp,
            "decode_tokens_per_s": batch * steps / td if steps else None,
            "prefill_s": tp, "decode_s": td, "wall_s": wall}, logits
