"""World-size-2 gloo tests (CPU) of the multi-GPU plans in parallel.py: the
column-parallel GEMM with its all-gather, and head-parallel attention, must give
every rank the bits a single process computes; a rank that dies before a collective
makes the others fail within the process-group timeout instead of hanging.

The per-rank compute here is the CPU oracle (libbi.so needs a GPU); the sharding,
padding and gather logic under test is the product's."""

import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _setup_paths():
    for p in (ROOT, os.path.join(ROOT, "mlx-batch-invariant_b200"), HERE):
        if p not in sys.path:
            sys.path.insert(0, p)


def _np(t):
    from conftest import to_np
    return to_np(t)


def _from_np(a, dtype):
    if dtype == torch.bfloat16:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a))


def _oracle_linear(x, w, b):
    from oracle import oracle as orc
    y = orc.gemm(_np(x), _np(w), _np(b) if b is not None else None, b_is_nk=True)
    return _from_np(y, x.dtype)


def _oracle_sdpa(q, k, v, scale=None, mask=None, sinks=None):
    from oracle import oracle as orc
    kw = {}
    if isinstance(mask, str):
        kw = dict(mask_mode=1, causal_offset=k.shape[2] - q.shape[2])
    elif mask is not None:
        m = mask.to(q.dtype)
        kw = dict(mask=_np(m), mask_mode=2)
    y = orc.sdpa(_np(q.contiguous()), _np(k.contiguous()), _np(v.contiguous()), scale=scale,
                 sinks=_np(sinks) if sinks is not None else None, **kw)
    return _from_np(y, q.dtype)


GEMM_CASES = [(5, 64, 24, torch.float32), (3, 40, 1000, torch.bfloat16), (4, 16, 13, torch.float16),
              (2, 32, 1, torch.float32)]


def _inputs_gemm(M, K, N, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g).to(dtype)
    w = (torch.randn(N, K, generator=g) / 8).to(dtype)
    b = (torch.randn(N, generator=g) / 10).to(dtype)
    return x, w, b


def _inputs_attn(seed, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(2, 8, 3, 32, generator=g).to(dtype)
    k = torch.randn(2, 4, 50, 32, generator=g).to(dtype)
    v = torch.randn(2, 4, 50, 32, generator=g).to(dtype)
    m = torch.randn(1, 8, 3, 50, generator=g).to(dtype)
    s = torch.randn(8, generator=g).to(dtype)
    return q, k, v, m, s


def _worker(rank, world, port, queue):
    _setup_paths()
    import torch.distributed as dist
    from mlx_batch_invariant_b200 import parallel
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    out = {}
    for i, (M, K, N, dtype) in enumerate(GEMM_CASES):
        x, w, b = _inputs_gemm(M, K, N, dtype, 10 + i)
        ws, bs = parallel.shard_weight(w, b, rank, world)
        y = parallel.column_parallel_linear(x, ws, bs, N, local_op=_oracle_linear)
        out["gemm%d" % i] = _np(y).view(np.uint8).copy()
    q, k, v, m, s = _inputs_attn(5)
    for label, kw in (("none", {}), ("causal", {"mask": "causal"}), ("additive", {"mask": m}),
                      ("sinks", {"sinks": s})):
        y = parallel.head_parallel_sdpa(q, k, v, local_op=_oracle_sdpa, **kw)
        out["sdpa_" + label] = _np(y).view(np.uint8).copy()
    queue.put((rank, out))
    dist.barrier()
    dist.destroy_process_group()


def _dying_worker(rank, world, port, queue):
    _setup_paths()
    import torch.distributed as dist
    from mlx_batch_invariant_b200 import parallel
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    x, w, b = _inputs_gemm(4, 16, 32, torch.float32, 1)
    ws, bs = parallel.shard_weight(w, b, rank, world)
    if rank == 1:
        _put_and_exit(queue, (rank, "exiting"))  # dies between steps, before the collective
    try:
        parallel.column_parallel_linear(x, ws, bs, 32, local_op=_oracle_linear)
        msg = "no error"
    except Exception as e:  # noqa: BLE001 - any error is the point
        msg = "raised %s" % type(e).__name__
    _put_and_exit(queue, (rank, msg))


def _put_and_exit(queue, item):
    queue.put(item)
    queue.close()
    queue.join_thread()  # flush before the hard exit
    os._exit(0)


def _spawn(fn, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            r, val = queue.get(timeout=timeout)
            results[r] = val
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return results


def test_shard_bounds_cover_n_with_aligned_starts():
    _setup_paths()
    from mlx_batch_invariant_b200 import parallel
    for n in (1, 7, 8, 13, 1000, 1024, 4096, 57344, 128256, 16032):
        for g in (1, 2, 4, 8):
            b = parallel.shard_bounds(n, g)
            assert b[0][0] == 0 and b[-1][1] == n
            assert all(e0 == s1 for (_, e0), (s1, _) in zip(b, b[1:]))
            assert all(s % 8 == 0 for s, e in b if e > s)
    with pytest.raises(ValueError):
        parallel.head_shard(32, 8, 0, 3)


def test_column_and_head_parallel_match_single_process_bits():
    _setup_paths()
    results = _spawn(_worker)
    assert set(results) == {0, 1}
    from mlx_batch_invariant_b200 import parallel  # noqa: F401
    for i, (M, K, N, dtype) in enumerate(GEMM_CASES):
        x, w, b = _inputs_gemm(M, K, N, dtype, 10 + i)
        want = _np(_oracle_linear(x, w, b)).view(np.uint8)
        for r in (0, 1):
            assert np.array_equal(results[r]["gemm%d" % i], want.reshape(-1).reshape(
                results[r]["gemm%d" % i].shape)), (i, r)
    q, k, v, m, s = _inputs_attn(5)
    for label, kw in (("none", {}), ("causal", {"mask": "causal"}), ("additive", {"mask": m}),
                      ("sinks", {"sinks": s})):
        want = _np(_oracle_sdpa(q, k, v, **kw)).view(np.uint8)
        for r in (0, 1):
            assert np.array_equal(results[r]["sdpa_" + label], want), (label, r)


def test_a_rank_that_dies_makes_the_other_fail_not_hang():
    _setup_paths()
    results = _spawn(_dying_worker, timeout=90)
    assert results[1] == "exiting"
    assert results[0].startswith("raised"), results[0]


TINY_DECODER = dict(layers=2, hidden=64, heads=4, kv_heads=2, head_dim=16, inter=96, vocab=128)


def _greedy(model, ids, steps):
    out = [model.prefill(ids)]
    for _ in range(steps):
        out.append(model.decode(out[-1].argmax(dim=-1)))
    return torch.stack(out)


def _decoder_worker(rank, world, port, queue):
    _setup_paths()
    import torch.distributed as dist
    from mlx_batch_invariant_b200 import decoder as dec
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    cfg = dec.DecoderConfig(**TINY_DECODER)
    model = dec.Decoder(cfg, max_batch=2, max_len=12, dtype=torch.float32, device="cpu",
                        exchange="nccl")
    shards = {"wqkv": model.layers[1]["wqkv"].clone(), "wd": model.layers[1]["wd"].clone()}
    logits = _greedy(model, dec.prompts(cfg, 2, 6, "cpu"), 4)
    queue.put((rank, {"logits": logits.numpy(), **{k: v.numpy() for k, v in shards.items()}}))
    dist.barrier()
    dist.destroy_process_group()


def test_decoder_sharding_plan_matches_one_process():
    """The decoder's column-parallel plan on 2 gloo ranks (stock float32 ops on CPU):
    each rank holds the right rows of every weight and ends with the logits and greedy
    tokens of the unsharded model.  (Bitwise equality across GPU counts is the GPU
    test's job; CPU BLAS gives no per-element guarantee across shard widths.)"""
    _setup_paths()
    from mlx_batch_invariant_b200 import decoder as dec
    results = _spawn(_decoder_worker)
    cfg = dec.DecoderConfig(**TINY_DECODER)
    single = dec.Decoder(cfg, max_batch=2, max_len=12, dtype=torch.float32, device="cpu",
                         single=True)
    want = _greedy(single, dec.prompts(cfg, 2, 6, "cpu"), 4).numpy()
    hd, H, Hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
    wqkv = single.layers[1]["wqkv"].numpy()
    q, k, v = np.split(wqkv, [H * hd, (H + Hkv) * hd])
    for r in (0, 1):
        got = results[r]
        np.testing.assert_allclose(got["logits"], want, rtol=1e-4, atol=1e-5)
        assert np.array_equal(got["logits"].argmax(-1), want.argmax(-1))
        hq, hk = H // 2 * hd, Hkv // 2 * hd
        np.testing.assert_array_equal(got["wqkv"], np.concatenate(
            (q[r * hq:(r + 1) * hq], k[r * hk:(r + 1) * hk], v[r * hk:(r + 1) * hk])))
        half = cfg.hidden // 2
        np.testing.assert_array_equal(got["wd"], single.layers[1]["wd"].numpy()[r * half:(r + 1) * half])


def test_decoder_static_step_matches_eager_decode_on_cpu():
    """The graph-capturable step (device position, index_copy_ cache write, masked
    full-cache attention, on-device argmax and position advance) follows the eager
    decode on one process (stock float32 ops on CPU: close, same greedy tokens)."""
    _setup_paths()
    from mlx_batch_invariant_b200 import decoder as dec
    cfg = dec.DecoderConfig(**TINY_DECODER)
    model = dec.Decoder(cfg, max_batch=2, max_len=12, dtype=torch.float32, device="cpu",
                        single=True)
    ids = dec.prompts(cfg, 2, 6, "cpu")
    eager = _greedy(model, ids, 4)
    first = model.prefill(ids)
    tok = first.argmax(dim=-1, keepdim=True)
    pos = torch.tensor([model.pos])
    steps = [first]
    for _ in range(4):
        steps.append(model._greedy_step(tok, pos))
    static = torch.stack(steps)
    assert pos.item() == 10 and model.pos == 6
    np.testing.assert_allclose(static.numpy(), eager.numpy(), rtol=1e-5, atol=1e-6)
    assert np.array_equal(static.argmax(-1).numpy(), eager.argmax(-1).numpy())


def test_decode_graph_refuses_to_step_past_the_cache():
    """The host guard of DecodeGraph.step (no CUDA needed to reach it)."""
    _setup_paths()
    from mlx_batch_invariant_b200 import decoder as dec

    class _Fake:  # a DecodeGraph without a captured graph
        pass
    g = _Fake()
    g.model = type("M", (), {"max_len": 5})()
    g.graph = type("G", (), {"replay": staticmethod(lambda: None)})()
    g.logits = "logits"
    step = dec.DecodeGraph.step.__get__(g)
    with pytest.raises(RuntimeError):
        step()
    g._next = 4
    assert step() == "logits" and g._next == 5
    with pytest.raises(ValueError):
        step()
