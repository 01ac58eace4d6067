"""`python -m mlx_batch_invariant_b200 verify` -- prove on this machine that the
kernels are batch-invariant (the B200 counterpart of mlx_batch_invariant/_cli.py).
`... decoder` runs the same check end to end on a Llama-shaped model (decoder.py).

Same sweep as the reference (_cli.py:78-152): for each dtype, bi.linear over batch
sizes with a fixed row 0, and attention over query-chunk lengths with a fixed last
query, each compared as bit patterns against the first case; then the negative
control, which must show stock torch.matmul batch-variant or the run fails.  Under
torchrun (WORLD_SIZE > 1) it also checks the GPU-count axis: the column-parallel GEMM
and head-parallel attention must give every rank the single-GPU bits.
"""

import argparse
import dataclasses
import os
import platform
import sys

import torch

from . import __version__, scaled_dot_product_attention
from ._gemm import linear

_DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def _bits(t):
    t = t.detach().contiguous().reshape(-1)
    return t.view(torch.int32) if t.element_size() == 4 else t.view(torch.int16)


def _randn(shape, dtype, gen, dev):
    return torch.randn(*shape, generator=gen, device="cpu").to(dtype).to(dev)


def _gemm_case(dtype, K, N, batches, fn, gen, dev):
    """Rows of a fixed input must not change when other rows are added (_cli.py:21-35)."""
    x = _randn((max(batches), K), dtype, gen, dev)
    w = _randn((N, K), dtype, gen, dev)
    ref, bad = None, []
    for B in batches:
        y = fn(x[:B].contiguous(), w)
        b = _bits(y[0])
        if ref is None:
            ref = b
        elif not torch.equal(b, ref):
            bad.append(B)
    return bad


def _attn_case(dtype, H, Hkv, N, D, qLs, fn, gen, dev):
    """One query token must not change when other query tokens ride along (_cli.py:38-53)."""
    k = _randn((1, Hkv, N, D), dtype, gen, dev)
    v = _randn((1, Hkv, N, D), dtype, gen, dev)
    q = _randn((1, H, max(qLs), D), dtype, gen, dev)
    ref, bad = None, []
    for qL in qLs:
        y = fn(q[:, :, max(qLs) - qL:, :].contiguous(), k, v)
        b = _bits(y[:, :, -1, :])
        if ref is None:
            ref = b
        elif not torch.equal(b, ref):
            bad.append(qL)
    return bad


def _distributed_checks(dtypes, gen_seed, dev):
    """Column-parallel GEMM and head-parallel attention vs the single-GPU bits."""
    import torch.distributed as dist

    from . import parallel
    world, rank = dist.get_world_size(), dist.get_rank()
    fails = 0
    for dtype in dtypes:
        name = str(dtype).rsplit(".", 1)[-1]
        gen = torch.Generator().manual_seed(gen_seed)
        for K, N in ((4096, 4096), (4096, 1000)):
            x = _randn((33, K), dtype, gen, dev)
            w = _randn((N, K), dtype, gen, dev)
            b = _randn((N,), dtype, gen, dev)
            full = linear(x, w, b)
            ws, bs = parallel.shard_weight(w, b, rank, world)
            y = parallel.column_parallel_linear(x, ws, bs, N)
            ok = torch.equal(_bits(y), _bits(full))
            fails += not ok
            if rank == 0:
                print("  %-9s linear   K=%-6d N=%-6d g=%d %s"
                      % (name, K, N, world, "ok" if ok else "VARIANT across GPU count"))
            if dtype != torch.float32:
                fused = parallel.FusedColumnParallel(N, 64, dtype)
                try:
                    ok = True
                    for rows in (33, 1, 64):  # several calls reuse the exchange buffer
                        xr = x[:rows] if rows <= 33 else torch.cat([x, x[:31]])
                        y = fused.linear(xr, ws, bs)
                        ok = ok and torch.equal(_bits(y), _bits(linear(xr, w, b)))
                    # the unpack deferred to a side stream, two calls in flight
                    xs2 = [x, torch.cat([x, x[:31]])]
                    ys2 = [fused.linear(xr, ws, bs, wait=False) for xr in xs2]
                    fused.finish()
                    for xr, y in zip(xs2, ys2):
                        ok = ok and torch.equal(_bits(y), _bits(linear(xr, w, b)))
                finally:
                    fused.close()
                fails += not ok
                if rank == 0:
                    print("  %-9s linear   K=%-6d N=%-6d g=%d fused all-gather %s"
                          % (name, K, N, world, "ok" if ok else "VARIANT across GPU count"))
        H, Hkv = 32, 8
        if Hkv % world == 0:
            q = _randn((2, H, 3, 128), dtype, gen, dev)
            k = _randn((2, Hkv, 1000, 128), dtype, gen, dev)
            v = _randn((2, Hkv, 1000, 128), dtype, gen, dev)
            full = scaled_dot_product_attention(q, k, v, mask="causal")
            y = parallel.head_parallel_sdpa(q, k, v, mask="causal")
            ok = torch.equal(_bits(y), _bits(full))
            fails += not ok
            if rank == 0:
                print("  %-9s sdpa     H=%d/%-2d g=%d %s"
                      % (name, H, Hkv, world, "ok" if ok else "VARIANT across GPU count"))
    t = torch.tensor([fails], device=dev)
    dist.all_reduce(t)
    return int(t.item())


def verify(argv=None):
    p = argparse.ArgumentParser(prog="python -m mlx_batch_invariant_b200 verify")
    p.add_argument("--dtype", action="append", choices=sorted(_DTYPES),
                   help="repeatable; default is all three")
    p.add_argument("--quick", action="store_true", help="one shape per op")
    p.add_argument("--seed", type=int, default=0)
    args = p.parse_args(argv)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not torch.cuda.is_available():
        print("verify needs a CUDA device (the kernels run on sm_100)", file=sys.stderr)
        return 2
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    gen = torch.Generator().manual_seed(args.seed)
    dtypes = [_DTYPES[d] for d in (args.dtype or sorted(_DTYPES))]
    batches = [1, 2, 8, 32] if args.quick else [1, 2, 3, 5, 8, 16, 31, 32, 33, 64, 128]
    qLs = [1, 2, 8, 9] if args.quick else [1, 2, 3, 4, 7, 8, 9, 16, 17]
    gemms = [(4096, 4096)] if args.quick else [(512, 1024), (4096, 4096), (11008, 4096)]
    attns = [(8, 8, 1024, 128)] if args.quick else [
        (32, 8, 512, 128), (16, 8, 4096, 128), (8, 8, 4096, 128), (32, 8, 8192, 128)]

    say = print if rank == 0 else (lambda *a, **k: None)
    say("mlx-batch-invariant-b200 %s | torch %s | %s"
        % (__version__, torch.__version__, platform.machine()))
    prop = torch.cuda.get_device_properties(dev)
    say("device: %s (sm_%d%d, %d SMs)%s\n" % (prop.name, prop.major, prop.minor,
                                               prop.multi_processor_count,
                                               ", %d GPUs" % world if world > 1 else ""))

    fails = 0
    for dtype in dtypes:
        name = str(dtype).rsplit(".", 1)[-1]
        for K, N in gemms:
            bad = _gemm_case(dtype, K, N, batches, lambda x, w: linear(x, w), gen, dev)
            fails += bool(bad)
            say("  %-9s linear   K=%-6d N=%-6d %s"
                % (name, K, N, "ok" if not bad else "VARIANT at batch %s" % bad))
        for H, Hkv, N, D in attns:
            bad = _attn_case(dtype, H, Hkv, N, D, qLs,
                             lambda q, k, v: scaled_dot_product_attention(q, k, v), gen, dev)
            fails += bool(bad)
            say("  %-9s sdpa     H=%d/%-2d N=%-6d %s"
                % (name, H, Hkv, N, "ok" if not bad else "VARIANT at qL %s" % bad))

    if world > 1:
        say("\nGPU-count axis (torch.distributed, NCCL):")
        fails += _distributed_checks(dtypes, args.seed + 1, dev)

    # A suite that cannot fail proves nothing: confirm stock torch is still variant.
    stock = _gemm_case(torch.float32, 4096, 4096, batches, lambda x, w: x @ w.T, gen, dev)
    say("\ncontrol: stock torch.matmul float32 K=4096 N=4096 -> %s"
        % ("VARIANT at batch %s (expected)" % stock if stock
           else "invariant -- stock torch may have been fixed; this library is no longer "
                "proving anything"))
    if not stock:
        fails += 1
    import torch.nn.functional as F
    sbad = _attn_case(torch.bfloat16, 32, 32, 2048, 128, qLs,
                      lambda q, k, v: F.scaled_dot_product_attention(q, k, v), gen, dev)
    # Like the reference's quantized control, report but do not fail: which SDPA
    # backend torch picks depends on the device and build.
    say("control: stock F.scaled_dot_product_attention bfloat16 -> %s"
        % ("VARIANT at qL %s (expected)" % sbad if sbad
           else "query-length invariant on this device for this shape"))

    say("\n%s" % ("FAILED (%d cases)" % fails if fails else "all invariant"))
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 1 if fails else 0


SMALL_DECODER = dict(layers=2, hidden=1024, heads=16, kv_heads=8, head_dim=64, inter=2048,
                     vocab=4096)


def decoder(argv=None):
    """The end-to-end check of the reference's bench/bench.py:211-246 (determinism) and
    :161-208 (e2e) on the Llama-shaped decoder: the slot-0 logits of every prefill and
    decode step at batch 1 and at --batch must be bitwise equal under the mode (and,
    with --single-check under torchrun, equal to the unsharded model's); prints
    tokens/s of both phases.  Stock torch is run as the control on one GPU."""
    import json

    from . import batch_invariant_mode
    from . import decoder as dec

    p = argparse.ArgumentParser(prog="python -m mlx_batch_invariant_b200 decoder")
    p.add_argument("--layers", type=int, default=None, help="override the layer count")
    p.add_argument("--small", action="store_true", help="a 2-layer d=1024 model")
    p.add_argument("--batch", type=int, default=8)
    p.add_argument("--prompt", type=int, default=512)
    p.add_argument("--gen", type=int, default=128)
    p.add_argument("--exchange", choices=("fused", "nccl"), default="fused")
    p.add_argument("--no-stock", action="store_true", help="skip the stock-torch control")
    p.add_argument("--eager", action="store_true",
                   help="decode step by step from Python instead of replaying a CUDA graph")
    p.add_argument("--single-check", action="store_true",
                   help="under torchrun: also run the unsharded model on every rank")
    p.add_argument("--json", help="write the results here (rank 0)")
    args = p.parse_args(argv)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if not torch.cuda.is_available():
        print("decoder needs a CUDA device (the kernels run on sm_100)", file=sys.stderr)
        return 2
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    fields = dict(SMALL_DECODER) if args.small else {}
    if args.layers is not None:
        fields["layers"] = args.layers
    cfg = dec.DecoderConfig(**fields)
    say = print if rank == 0 else (lambda *a, **k: None)
    max_len = args.prompt + args.gen
    model = dec.Decoder(cfg, max_batch=args.batch, max_len=max_len, device=dev,
                        exchange=args.exchange)
    say("decoder: %d layers, d=%d, %d/%d heads x %d, ffn %d, vocab %d, %.2fB params, bf16, "
        "%d GPU%s (%s exchange)" % (cfg.layers, cfg.hidden, cfg.heads, cfg.kv_heads,
                                    cfg.head_dim, cfg.inter, cfg.vocab,
                                    model.num_params() / 1e9, world, "s" if world > 1 else "",
                                    args.exchange if world > 1 else "no"))
    say("prompt %d tokens, then %d greedy decode steps (%s); shared prompt in batch slot 0\n"
        % (args.prompt, args.gen, "eager" if args.eager else "CUDA graph replays"))

    def run(B, warm=True):
        graph = dec.DecodeGraph(model, B) if args.gen and not args.eager else None
        stats, logits = dec.timed_run(model, B, args.prompt, args.gen, dev, warm=warm,
                                      graph=graph)
        del graph  # a graph holding NCCL calls must go before the process group
        return stats, dec.slot0_bits(logits)

    results = {"config": dataclasses.asdict(cfg), "gpus": world, "prompt": args.prompt,
               "gen": args.gen, "exchange": args.exchange if world > 1 else None,
               "decode": "eager" if args.eager else "cuda graph"}
    fails = 0
    with batch_invariant_mode(strict=True):
        runs = {}
        for B in sorted({1, args.batch}):
            runs[B] = run(B)
    base = runs[1][1]
    diff = dec.differing(runs[args.batch][1], base)
    bad = sum(1 for d in diff if d)
    fails += bad > 0
    say("| path | batch | steps with slot-0 logits differing from batch 1 | logits differing |")
    say("|---|---:|---:|---:|")
    say("| batch invariant | %d | %d / %d | %d / %d |" % (args.batch, bad, len(diff), sum(diff),
                                                        len(diff) * cfg.vocab))
    results["invariant"] = {"batch": args.batch, "steps_differing": bad, "steps": len(diff),
                            "logits_differing": sum(diff)}
    if world == 1 and not args.no_stock:
        stock = {}
        for B in sorted({1, args.batch}):
            stock[B] = run(B, warm=False)[1]
        sd = dec.differing(stock[args.batch], stock[1])
        say("| stock torch (control) | %d | %d / %d | %d / %d |"
            % (args.batch, sum(1 for d in sd if d), len(sd), sum(sd), len(sd) * cfg.vocab))
        results["stock"] = {"steps_differing": sum(1 for d in sd if d),
                            "logits_differing": sum(sd)}
    if world > 1 and args.single_check:
        single = dec.Decoder(cfg, max_batch=1, max_len=max_len, device=dev, single=True)
        with batch_invariant_mode(strict=True):
            _, logits = dec.timed_run(single, 1, args.prompt, args.gen, dev, warm=False)
        sc = dec.differing(dec.slot0_bits(logits), base)
        ok = torch.tensor([int(any(sc))], device=dev)
        dist.all_reduce(ok)
        fails += int(ok.item()) > 0
        say("| %d GPUs vs 1 GPU | 1 | %d ranks differ |" % (world, int(ok.item())))
        results["vs_single_gpu_ranks_differing"] = int(ok.item())
        del single

    say("\n| phase | batch | tokens/s | seconds |")
    say("|---|---:|---:|---:|")
    for B in sorted(runs):
        st = runs[B][0]
        say("| prefill %d tok | %d | %.1f | %.4f |" % (args.prompt, B, st["prefill_tokens_per_s"],
                                                    st["prefill_s"]))
        if args.gen:
            say("| decode %d steps | %d | %.1f | %.4f |" % (args.gen, B, st["decode_tokens_per_s"],
                                                         st["decode_s"]))
    results["runs"] = [runs[B][0] for B in sorted(runs)]
    say("\n%s" % ("FAILED" if fails else "logits bitwise equal"))
    if args.json and rank == 0:
        with open(args.json, "w") as f:
            json.dump(results, f, indent=1)
    model.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 1 if fails else 0


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    if argv and argv[0] == "verify":
        return verify(argv[1:])
    if argv and argv[0] == "decoder":
        return decoder(argv[1:])
    print("usage: mlx-bi verify [--quick] [--dtype float32|float16|bfloat16] [--seed N]\n"
          "       mlx-bi decoder [--small] [--batch B] [--prompt L] [--gen S] "
          "[--exchange fused|nccl] [--single-check]\n"
          "(or python -m mlx_batch_invariant_b200 ...)", file=sys.stderr)
    return 2


if __name__ == "__main__":
    sys.exit(main())
