"""Throughput of the batch-invariant kernels on B200 (the driver's bench contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (N > 1)

A step is one pass of the hot path over config 5 of the build (BASELINE.json
configs[4]): the invariant GEMM y = bi.linear(x, w) on the four 70B-style (K, N)
shapes (8192,10240), (8192,8192), (8192,57344), (28672,8192) at M = 4096, bf16,
x ~ N(0,1), w ~ N(0,0.02) (synthetic, random init), column-parallel over N on N GPUs
with the all-gather fused into the GEMM epilogue (parallel.FusedColumnParallel; the
NCCL all-gather variant is reported beside it as nccl_allgather_tflops).  `value` is whole-job TFLOP/s (2*M*N*K per
shape, all ranks' columns) over the max-over-ranks device time of exactly K steps.
The weights (1.7 GB) exceed L2 (126 MB), so no flush is needed between steps.

Also reported:
  e2e       the same metric through the public API with host buffers: each step
            copies x from pinned host memory, runs bi.linear (+ all-gather) and
            copies every output back to pinned host memory.
  roofline  the dominant kernel (the N = 57344 GEMM), timed with CUDA events on its
            stream inside the timed region, against MEASURED_PEAKS.json.
  sdpa      decode attention (config 2's largest case: B=64, H=32, Hkv=8, L=8192,
            D=128, bf16, causal), GB/s of algorithmic bytes vs measured HBM copy
            bandwidth; head-parallel at N > 1.
  cpu_baseline  the CPU oracle (oracle/, the reference's algorithm restated in C;
            the reference itself is Metal-only) on a bounded sample, rank 0, N = 1.

--impl reference times that CPU implementation alone on the same metric (rank 0).
--profile gemm|gemm-decode|gemm-tf32x3|sdpa runs 3 warm-up launches and 1 launch of one
kernel (the bench's dominant GEMM, config 5's M = 1 GEMM on (28672, 8192), the fp32
tensor-core GEMM at M = 4096, K = N = 8192, or the bench's decode attention) and prints
nothing (the target of the committed ncu captures).
--sweep prints config 5's table: bi.linear vs cuBLAS at M in 1..16384 on every shape;
under torchrun (--gpus N > 1) the column-parallel form on N GPUs -- the fused GEMM +
NVLink all-gather against cuBLAS on the shard + NCCL all-gather -- timed as the max
over ranks.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "mlx-batch-invariant_b200"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

SHAPES = [(8192, 10240), (8192, 8192), (8192, 57344), (28672, 8192)]  # (K, N)
M = 4096
DOMINANT = 2  # index of the (8192, 57344) GEMM in SHAPES
SDPA_CFG = dict(B=64, H=32, Hkv=8, L=8192, D=128)
FLOPS_PER_STEP = sum(2 * M * K * N for K, N in SHAPES)
# NVLink 5 peer-copy bandwidth measured on these B200 nodes (GB/s per direction per GPU;
# 900 nominal): the link term of the fused all-gather's roofline.
LINK_GBS = 770.0


# ---------------------------------------------------------------- helpers

def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def _traffic():
    """Per-launch DRAM bytes of the dominant kernels from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f)
    return {}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self._thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS,
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self._thread = threading.Thread(target=self._read, daemon=True)
        self._thread.start()
        time.sleep(0.3)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.2)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._thread:
            self._thread.join(timeout=2)
        sm, mx, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        loaded = [s for s, p in zip(sm, power) if p > 0.5 * max(power)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def _dist_init(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit("bench.py --gpus %d but WORLD_SIZE=%d" % (args.gpus, world))
    if world > 1:
        import datetime
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        backend = "gloo" if args.impl == "reference" else "nccl"
        if backend == "nccl":
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def _max_over_ranks(x, world):
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier_sync(world):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


# ---------------------------------------------------------------- CPU baseline

CPU_ROWS = 64  # rows of the dominant GEMM in one CPU row block


def _cpu_operands():
    import numpy as np
    import ml_dtypes
    K, N = SHAPES[DOMINANT]
    rng = np.random.default_rng(0)
    x = rng.standard_normal((CPU_ROWS, K), dtype=np.float32).astype(ml_dtypes.bfloat16)
    w = (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(ml_dtypes.bfloat16)
    return x, w


def _oracle_blocks(x, w, blocks, threads):
    """`blocks` row blocks of the dominant GEMM through the CPU oracle; seconds taken."""
    from oracle import oracle as orc
    t0 = time.perf_counter()
    for _ in range(blocks):
        orc.gemm(x, w, b_is_nk=True, threads=threads)
    return time.perf_counter() - t0


def _blocks_for(x, w, threads, seconds):
    """Row blocks that take about `seconds` (one untimed block measures the rate)."""
    one = _oracle_blocks(x, w, 1, threads)
    return max(1, int(round(seconds / max(one, 1e-6))))


def cpu_baseline(budget_s=12.0):
    """The CPU oracle (oracle/bi_oracle.c, all host threads) on a bounded sample of the
    workload -- row blocks of the dominant (8192, 57344) GEMM, about budget_s of work --
    plus, beside it, the same sample's rate from NumPy float32 (OpenBLAS, the bf16
    operands upcast) and from the oracle on one core."""
    import numpy as np
    K, N = SHAPES[DOMINANT]
    x, w = _cpu_operands()
    threads = os.cpu_count() or 1  # all host threads (torchrun sets OMP_NUM_THREADS=1)
    blocks = _blocks_for(x, w, threads, budget_s)
    dt = _oracle_blocks(x, w, blocks, threads)
    flops_block = 2.0 * CPU_ROWS * K * N
    out = {"value": blocks * flops_block / dt / 1e12, "unit": "TFLOP/s", "cores": threads,
           "kind": "port",
           "sample": "%d row blocks of %d rows of the (K=%d, N=%d) bf16 bi.linear GEMM, "
                     "%.1f s, oracle/bi_oracle.c (fp32 fmaf in 8-deep K slices, OpenMP)"
                     % (blocks, CPU_ROWS, K, N, dt)}
    # a quarter block (16 rows) on one core: a few seconds
    t1 = _oracle_blocks(x[:16], w, 1, 1)
    # NumPy float32 x @ w.T on OpenBLAS (all threads), operands upcast once, untimed
    xf, wt = x.astype(np.float32), np.ascontiguousarray(w.astype(np.float32).T)
    _ = xf @ wt
    reps, t0 = 0, time.perf_counter()
    while True:
        _ = xf @ wt
        reps += 1
        if time.perf_counter() - t0 > 2.0:
            break
    tn = time.perf_counter() - t0
    out["also"] = [
        {"kind": "port-1-core", "value": flops_block / 4 / t1 / 1e12, "unit": "TFLOP/s",
         "cores": 1, "sample": "16 rows of the same GEMM, %.1f s" % t1},
        {"kind": "numpy-fp32-openblas", "value": reps * flops_block / tn / 1e12,
         "unit": "TFLOP/s", "cores": threads,
         "sample": "%d x (64 x %d) @ (%d x %d) float32 (bf16 operands upcast), %.1f s; not "
                   "the invariant algorithm (BLAS order), a throughput reference only"
                   % (reps, K, K, N, tn)},
    ]
    return out


# ---------------------------------------------------------------- reference arm

def run_reference(args):
    """Times the reference's algorithm on the host: the CPU oracle on all host threads.
    A step is a fixed number of 64-row blocks of the dominant GEMM (chosen once, so a
    step takes a few seconds); ms_per_step is the measured time of those steps."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    K, N = SHAPES[DOMINANT]
    x, w = _cpu_operands()
    threads = os.cpu_count() or 1
    per_step_s = max(1.0, min(10.0, 60.0 / max(1, args.steps + args.warmup)))
    blocks = _blocks_for(x, w, threads, per_step_s)
    for _ in range(args.warmup):
        _oracle_blocks(x, w, blocks, threads)
    times = [_oracle_blocks(x, w, blocks, threads) for _ in range(args.steps)]
    total = sum(times)
    flops_step = blocks * 2.0 * CPU_ROWS * K * N
    value = flops_step * len(times) / total / 1e12
    sample = ("%d steps of %d row blocks (%d rows each) of the (K=%d, N=%d) bf16 GEMM, "
              "oracle/bi_oracle.c on %d threads" % (len(times), blocks, CPU_ROWS, K, N, threads))
    line = {
        "metric": "invariant GEMM TFLOP/s (bf16, config 5 shapes, M=4096)",
        "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total / len(times) * 1e3,
        "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": "config 5: bi.linear at M=4096 on (K,N) in %s, bf16" % SHAPES,
                   "step": "%d blocks of %d rows of the (8192, 57344) GEMM (a bounded CPU "
                           "sample of the workload; the rate is the metric)"
                           % (blocks, CPU_ROWS)},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "reference_note": "the reference (mlx-batch-invariant 0.2.0) runs only under "
                          "MLX/Metal; its algorithm restated in C (oracle/) is timed",
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- our arm

def run_ours(args):
    import mlx_batch_invariant_b200 as bi
    from mlx_batch_invariant_b200 import parallel

    world, rank, local = _dist_init(args)
    dev = torch.device("cuda", local)
    # x replicated (same seed on every rank), weights: this rank's rows only.
    gx = torch.Generator(device=dev)
    gx.manual_seed(7)
    xs = {}
    for K, _ in SHAPES:
        if K not in xs:
            xs[K] = torch.randn((M, K), generator=gx, device=dev, dtype=torch.float32).to(
                torch.bfloat16)
    ws = []
    for i, (K, N) in enumerate(SHAPES):
        s, e = parallel.shard_bounds(N, world)[rank]
        gw = torch.Generator(device=dev)
        gw.manual_seed(100 + i)
        # rows [s, e) of a seeded (N, K) weight, generated shard by shard
        w = (torch.randn((e - s, K), generator=gw, device=dev, dtype=torch.float32) * 0.02).to(
            torch.bfloat16)
        ws.append(w)
    # one GEMM per shape; at N > 1 each fused call also launches its entry barrier and
    # the unpack of the blocks the peers stored
    launches_per_step = len(SHAPES) * (3 if world > 1 else 1)

    comm = torch.cuda.Stream() if world > 1 else None
    main = torch.cuda.current_stream()
    # At N > 1 the product path is the fused column-parallel GEMM: every rank's
    # epilogue writes its columns into its own output and, over NVLink, into every
    # peer's staging area.
    fused = [parallel.FusedColumnParallel(N, M, torch.bfloat16) for _, N in SHAPES] \
        if world > 1 else None
    ys = [torch.empty((M, N), dtype=torch.bfloat16, device=dev) for _, N in SHAPES] \
        if world > 1 else None

    def step(dom_events=None):
        # dom_events: one (start, end) event pair per shape, recorded around its call
        outs = []
        for i, (K, N) in enumerate(SHAPES):
            if dom_events is not None:
                dom_events[i][0].record()
            if world > 1:
                # the copy of the peers' blocks runs on a side stream, under the next GEMM
                y = fused[i].linear(xs[K], ws[i], out=ys[i], wait=False)
            else:
                y = bi.linear(xs[K], ws[i])
            if dom_events is not None:
                dom_events[i][1].record()
            outs.append(y)
        if world > 1:
            for f in fused:
                f.finish()
        return outs

    def nccl_step():
        # Baseline exchange: GEMM i on the main stream, NCCL all-gather of its columns
        # on `comm` while GEMM i+1 runs.
        for i, (K, N) in enumerate(SHAPES):
            y = bi.linear(xs[K], ws[i])
            ready = torch.cuda.Event()
            ready.record()
            parallel.gather_columns_on(comm, y, N, ready=ready)
        main.wait_stream(comm)

    for _ in range(args.warmup):
        step()
    _barrier_sync(world)

    clocks = ClockSampler(local)
    clocks.start()
    dom = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            for _ in SHAPES] for _ in range(args.steps)]
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier_sync(world)
    e0.record()
    for k in range(args.steps):
        step(dom[k])
    e1.record()
    _barrier_sync(world)
    clk = clocks.stop()
    ms = e0.elapsed_time(e1)
    ms = _max_over_ranks(ms, world)
    value = FLOPS_PER_STEP * args.steps / (ms / 1e3) / 1e12

    bits_check = _check_against_one_gpu(bi, parallel, xs, ys, world, dev) \
        if world > 1 else None

    nccl_value = None
    if world > 1:
        for _ in range(2):
            nccl_step()
        _barrier_sync(world)
        n0, n1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n0.record()
        for _ in range(args.steps):
            nccl_step()
        n1.record()
        _barrier_sync(world)
        nccl_ms = _max_over_ranks(n0.elapsed_time(n1), world)
        nccl_value = FLOPS_PER_STEP * args.steps / (nccl_ms / 1e3) / 1e12

    # dominant kernel alone (its own events on its stream), same as in the step
    K, N = SHAPES[DOMINANT]
    dom_ms = statistics.mean(ev[DOMINANT][0].elapsed_time(ev[DOMINANT][1]) for ev in dom)
    # every call's mean device time, max over ranks (at N > 1 a call spans its entry
    # barrier, the GEMM with its peer stores and the exit barrier)
    per_call_us = [_max_over_ranks(statistics.mean(ev[i][0].elapsed_time(ev[i][1])
                                                   for ev in dom) * 1e3, world)
                   for i in range(len(SHAPES))]
    n_local = ws[DOMINANT].shape[0]
    dom_flops = 2.0 * M * K * n_local
    peaks, peak_src = _peaks()
    long_region = ms * args.steps > 0 and ms > 1000.0
    peak = peaks["bf16_tflops_sustained"] if long_region else peaks["bf16_tflops"]
    achieved = dom_flops / (dom_ms / 1e3) / 1e12
    traffic = _traffic().get("gemm_tcgen05_bf16_m4096_k8192_n57344")
    if traffic is not None and n_local != N:
        traffic = traffic * n_local / N
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": traffic,
                "kernel": "gemm_tc_kernel<bf16, (N,K)> M=%d K=%d N=%d" % (M, K, n_local),
                "peak_source": "%s (%s)" % (peak_src,
                                            "sustained" if long_region else "burst")}
    if world > 1:
        # The fused call (entry barrier, GEMM whose epilogue stores this rank's shard
        # into every peer, local unpack of the peers' blocks) is bound by the slower of
        # the tensor work and the bytes this GPU must send over NVLink.
        link_bytes = (world - 1) * M * n_local * 2
        t_tensor = dom_flops / (peak * 1e12)
        t_link = link_bytes / (LINK_GBS * 1e9)
        target = max(t_tensor, t_link)
        roofline["fused_allgather"] = {
            "bound": "nvlink" if t_link > t_tensor else "tensor",
            "nvlink_bytes_out": link_bytes, "link_gbs": LINK_GBS,
            "link_peak_source": "measured peer copy, GB/s per direction per GPU",
            "target_us": target * 1e6, "achieved_us": dom_ms * 1e3,
            "frac": target / (dom_ms / 1e3),
            "scope": "entry barrier + GEMM with peer stores and exit barrier (the local "
                     "unpack of the received blocks runs on a side stream under the next "
                     "GEMM)"}

    # stock cuBLAS at the same shapes (the cost-of-invariance context)
    for _ in range(2):
        for i, (Kk, _) in enumerate(SHAPES):
            torch.nn.functional.linear(xs[Kk], ws[i])
    torch.cuda.synchronize()
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record()
    for _ in range(max(3, args.steps // 2)):
        for i, (Kk, _) in enumerate(SHAPES):
            torch.nn.functional.linear(xs[Kk], ws[i])
    c1.record()
    torch.cuda.synchronize()
    local_flops = sum(2 * M * Kk * w.shape[0] for (Kk, _), w in zip(SHAPES, ws))
    cublas_tflops = local_flops * max(3, args.steps // 2) / (c0.elapsed_time(c1) / 1e3) / 1e12

    # ---- e2e: public API with host buffers
    # The job's inputs start in pinned host memory and its results end there.  One GPU:
    # the whole x in and every output back.  N GPUs: each rank copies in its 1/N of x's
    # rows, NCCL all-gathers x over NVLink, and copies back only its own column block
    # of each output (the union over ranks is the whole result).  Copies run on their
    # own streams and overlap the GEMMs: step it copies its inputs into device buffer
    # it % 2 while the GEMMs of step it - 1 run, and each output block starts back to
    # the host as soon as its GEMM is done.  Every byte is copied every step inside the
    # timed region.
    bounds_m = parallel.shard_bounds(M, world, align=1)
    r0, r1 = bounds_m[rank]
    hx = {K: torch.empty((r1 - r0, K), dtype=torch.bfloat16, pin_memory=True).copy_(
        xs[K][r0:r1].cpu()) for K in xs}
    col = [parallel.shard_bounds(N, world)[rank] for _, N in SHAPES]
    hy = [torch.empty((M, c1 - c0), dtype=torch.bfloat16, pin_memory=True) for c0, c1 in col]
    h2d_rank = sum(t.numel() * t.element_size() for t in hx.values())
    d2h_rank = sum(t.numel() * t.element_size() for t in hy)
    h2d = h2d_rank * world if world > 1 else h2d_rank
    d2h = sum(M * N * 2 for _, N in SHAPES)

    copy_in, copy_out = torch.cuda.Stream(), torch.cuda.Stream()
    xgather = torch.cuda.Stream() if world > 1 else None
    dx_bufs = [{K: torch.empty_like(xs[K]) for K in xs} for _ in range(2)]
    dy_bufs = [[torch.empty((M, N), dtype=torch.bfloat16, device=dev) for _, N in SHAPES]
               for _ in range(2)] if world > 1 else None
    freed = [torch.cuda.Event() for _ in range(2)]  # last GEMM reading dx_bufs[b] done
    drained = [[torch.cuda.Event() for _ in SHAPES] for _ in range(2)]  # D2H of output b, i
    for b in range(2):
        freed[b].record(main)
        for e in drained[b]:
            e.record(main)

    def e2e_step(it):
        b = it & 1
        dx = dx_bufs[b]
        ready = {}
        with torch.cuda.stream(copy_in):
            copy_in.wait_event(freed[b])
            for K in hx:
                dx[K][r0:r1].copy_(hx[K], non_blocking=True)
                ready[K] = torch.cuda.Event()
                ready[K].record(copy_in)
        if world > 1:
            with torch.cuda.stream(xgather):
                for K in hx:
                    xgather.wait_event(ready[K])
                    dist.all_gather_into_tensor(dx[K], dx[K][r0:r1])
                    ready[K] = torch.cuda.Event()
                    ready[K].record(xgather)
        for i, (K, N) in enumerate(SHAPES):
            main.wait_event(ready[K])
            if world > 1:
                main.wait_event(drained[b][i])
                y = fused[i].linear(dx[K], ws[i], out=dy_bufs[b][i], wait=False)
                c0, c1 = col[i]
                y_own = y[:, c0:c1]
            else:
                y = bi.linear(dx[K], ws[i])
                y_own = y
            done = torch.cuda.Event()
            done.record(main)
            with torch.cuda.stream(copy_out):
                copy_out.wait_event(done)
                hy[i].copy_(y_own, non_blocking=True)
                y.record_stream(copy_out)
                drained[b][i].record(copy_out)
        freed[b].record(main)
        if world > 1:
            for f in fused:
                f.finish()

    e2e_steps = max(3, min(args.steps, 10))
    for it in range(2):
        e2e_step(it)
    main.wait_stream(copy_out)
    _barrier_sync(world)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(main)
    copy_in.wait_stream(main)
    for it in range(e2e_steps):
        e2e_step(it)
    main.wait_stream(copy_out)
    main.wait_stream(copy_in)
    if xgather is not None:
        main.wait_stream(xgather)
    f1.record(main)
    _barrier_sync(world)
    e2e_ms = _max_over_ranks(f0.elapsed_time(f1), world)
    e2e_value = FLOPS_PER_STEP * e2e_steps / (e2e_ms / 1e3) / 1e12

    # ---- decode attention (head-parallel at N > 1)
    sd = _bench_sdpa(bi, parallel, world, rank, dev, peaks, args)

    line = {
        "metric": "invariant GEMM TFLOP/s (bf16, config 5 shapes, M=4096)",
        "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random init, seeded)",
        "config": {"workload": "config 5: bi.linear at M=4096 on (K,N) in "
                               "(8192,10240),(8192,8192),(8192,57344),(28672,8192), bf16",
                   "M": M, "shapes_KN": SHAPES,
                   "parallelism": ("column-parallel N over %d GPUs, all-gather fused into the "
                                   "GEMM epilogue (NVLink peer stores of dense shard blocks; "
                                   "the local unpack on a side stream under the next GEMM)"
                                   % world) if world > 1
                   else "single GPU",
                   "l2": "inputs larger than L2 (1.7 GB of weights), no flush"},
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "copies": ("pinned host buffers; H2D and D2H on their own streams, "
                           "overlapping the GEMMs (device inputs double-buffered)")
                if world == 1 else
                ("pinned host buffers on every rank: each copies in its 1/%d of x's rows "
                 "(NCCL all-gather of x over NVLink) and copies back its own column block "
                 "of every output; copies on their own streams overlapping the fused "
                 "GEMMs; bytes are the whole job's (per rank: %d in, %d out)"
                 % (world, h2d_rank, d2h_rank)),
                "d2h_bytes_per_step": d2h, "steps": e2e_steps},
        "gpu_launches": launches_per_step * args.steps,
        "roofline": roofline,
        "per_call_us": per_call_us,
        "stock_cublas_tflops": cublas_tflops,
        "nccl_allgather_tflops": nccl_value,
        "fused_vs_single_gpu": bits_check,
        "sdpa": sd,
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        for f in fused:
            f.close()
        dist.barrier()
        dist.destroy_process_group()
    return 0


def _check_against_one_gpu(bi, parallel, xs, ys, world, dev):
    """Bits of the last timed step's gathered outputs against one GPU's result.

    For every shape and every rank's column block, 64 rows spread over all 16 pair tiles
    of M must equal bi.linear of those rows alone with that block's weight (regenerated
    here from its seed), computed on this GPU without any exchange: the fused
    all-gather moves data only, and a row's bits depend neither on M nor on the column
    block.  Returns the count of differing elements summed over ranks."""
    rows = sorted({int(r) for r in torch.linspace(0, M - 1, 48).round().tolist()}
                  | {0, 127, 128, 255, 256, 2047, 2048, M - 256, M - 129, M - 1})
    ri = torch.tensor(rows, device=dev)
    diff, checked = 0, 0
    for i, (K, N) in enumerate(SHAPES):
        xr = xs[K][ri]
        for s, e in parallel.shard_bounds(N, world):
            gw = torch.Generator(device=dev)
            gw.manual_seed(100 + i)
            w = (torch.randn((e - s, K), generator=gw, device=dev, dtype=torch.float32)
                 * 0.02).to(torch.bfloat16)
            ref = bi.linear(xr, w)
            got = ys[i][ri, s:e]
            diff += int((ref.view(torch.int16) != got.view(torch.int16)).sum())
            checked += ref.numel()
            del w
    t = torch.tensor([diff, checked], device=dev, dtype=torch.int64)
    dist.all_reduce(t)
    return {"rows": len(rows), "elements_checked": int(t[1]), "elements_differing": int(t[0]),
            "against": "bi.linear of the sampled rows with each rank's block, one GPU, "
                       "no exchange"}


def _bench_sdpa(bi, parallel, world, rank, dev, peaks, args):
    c = SDPA_CFG
    B, H, Hkv, L, D = c["B"], c["H"], c["Hkv"], c["L"], c["D"]
    gq = torch.Generator(device=dev)
    gq.manual_seed(11)
    (h0, h1), (k0, k1) = parallel.head_shard(H, Hkv, rank, world)
    hl, kl = h1 - h0, k1 - k0
    q = torch.randn((B, hl, 1, D), generator=gq, device=dev).to(torch.bfloat16)
    k = torch.randn((B, kl, L, D), generator=gq, device=dev).to(torch.bfloat16)
    v = torch.randn((B, kl, L, D), generator=gq, device=dev).to(torch.bfloat16)
    es = 2
    local_bytes = es * (B * hl * D + 2 * B * kl * L * D + B * hl * D)
    total_bytes = es * (B * H * D + 2 * B * Hkv * L * D + B * H * D)

    def call():
        y = bi.scaled_dot_product_attention(q, k, v, mask="causal")
        return parallel.gather_heads(y) if world > 1 else y

    for _ in range(3):
        call()
    _barrier_sync(world)
    n = max(5, args.steps)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(n)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for a, b in ev:
        a.record()
        y = bi.scaled_dot_product_attention(q, k, v, mask="causal")
        b.record()
        if world > 1:
            parallel.gather_heads(y)
    t1.record()
    _barrier_sync(world)
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
    achieved = local_bytes / (kern_ms / 1e3) / 1e9
    tot_ms = _max_over_ranks(t0.elapsed_time(t1) / n, world)
    # stock SDPA (torch's flash / cuDNN backends) at the same local shape
    import torch.nn.functional as F
    kk = k.repeat_interleave(hl // kl, dim=1)
    vv = v.repeat_interleave(hl // kl, dim=1)
    for _ in range(3):
        F.scaled_dot_product_attention(q, kk, vv)
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(n):
        F.scaled_dot_product_attention(q, kk, vv)
    s1.record()
    torch.cuda.synchronize()
    stock_gbs = local_bytes / (s0.elapsed_time(s1) / n / 1e3) / 1e9
    traffic = _traffic().get("sdpa_bf16_decode_b64_h32_kv8_l8192_d128")
    return {"value": total_bytes / (tot_ms / 1e3) / 1e9, "unit": "GB/s",
            "config": "decode B=%d H=%d Hkv=%d L=%d D=%d bf16 causal, heads over %d GPU%s"
                      % (B, H, Hkv, L, D, world, "s" if world > 1 else ""),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                         "traffic": traffic if world == 1 else None,
                         "kernel": "sdpa_gqa_kernel<bf16, D=128> (GQA route: q.k on the "
                                   "tensor cores, fold and P.V in fp32; heads per CTA and "
                                   "ring depth from the grid)"},
            "stock_sdpa_gbs": stock_gbs}


def run_profile(args):
    """3 warm-up launches + 1 launch of one kernel at the bench shape, for ncu."""
    import mlx_batch_invariant_b200 as bi
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    if args.profile in ("gemm", "gemm-decode"):
        # the bench's dominant GEMM, or config 5's decode case M = 1 on (28672, 8192)
        (K, N), rows = (SHAPES[DOMINANT], M) if args.profile == "gemm" else (SHAPES[3], 1)
        x = torch.randn((rows, K), generator=g, device=dev).to(torch.bfloat16)
        w = (torch.randn((N, K), generator=g, device=dev) * 0.02).to(torch.bfloat16)
        for _ in range(4):
            bi.linear(x, w)
    elif args.profile == "gemm-tf32x3":
        # float32 on the tensor cores (opt-in route): M = 4096, K = N = 8192
        x = torch.randn((M, 8192), generator=g, device=dev)
        w = torch.randn((8192, 8192), generator=g, device=dev) * 8192 ** -0.5
        with bi.float32_gemm("tf32x3"):
            for _ in range(4):
                bi.linear(x, w)
    else:
        c = SDPA_CFG
        q = torch.randn((c["B"], c["H"], 1, c["D"]), generator=g, device=dev).to(torch.bfloat16)
        k = torch.randn((c["B"], c["Hkv"], c["L"], c["D"]), generator=g, device=dev).to(
            torch.bfloat16)
        v = torch.randn_like(k)
        for _ in range(4):
            bi.scaled_dot_product_attention(q, k, v, mask="causal")
    torch.cuda.synchronize()
    return 0


SWEEP_M = (1, 8, 64, 512, 4096, 16384)


def run_sweep_parallel(args):
    """Config 5's sweep on N GPUs, column-parallel: every rank holds N/world rows of
    each (N, K) weight and ends with the full (M, N) output.  Ours: FusedColumnParallel
    (GEMM with the all-gather fused into the epilogue, the unpack included); stock:
    cuBLAS on the shard, then an NCCL all-gather of the column blocks into (M, N)
    (parallel.gather_columns).  Device time per call (CUDA events), max over ranks;
    one markdown table from rank 0."""
    from mlx_batch_invariant_b200 import parallel
    world, rank, local = _dist_init(args)
    dev = torch.device("cuda", local)
    peaks, src = _peaks()
    peak = peaks["bf16_tflops"]
    g = torch.Generator(device=dev)
    g.manual_seed(11 + rank)

    def timed(fn, reps):
        for _ in range(3):
            fn()
        _barrier_sync(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        _barrier_sync(world)
        return _max_over_ranks(e0.elapsed_time(e1) / reps / 1e3, world)

    if rank == 0:
        print("| K | N | M | GPUs | fused µs | TFLOP/s (all GPUs) | of %d× tensor peak | "
              "cuBLAS + NCCL µs | fused / stock |" % world)
        print("|---|---|---|---|---|---|---|---|---|")
    for K, N in SHAPES:
        s0, s1 = parallel.shard_bounds(N, world)[rank]
        w = (torch.randn((s1 - s0, K), generator=g, device=dev) * 0.02).to(torch.bfloat16)
        fused = parallel.FusedColumnParallel(N, max(SWEEP_M), torch.bfloat16)
        for Mr in SWEEP_M:
            x = torch.randn((Mr, K), generator=g, device=dev).to(torch.bfloat16)
            y = torch.empty((Mr, N), dtype=torch.bfloat16, device=dev)
            reps = 20 if Mr < 4096 else 5
            t_f = timed(lambda: fused.linear(x, w, out=y), reps)
            t_s = timed(lambda: parallel.gather_columns(torch.nn.functional.linear(x, w), N), reps)
            flops = 2.0 * Mr * N * K
            if rank == 0:
                print("| %d | %d | %d | %d | %.1f | %.1f | %.1f %% | %.1f | %.2f |"
                      % (K, N, Mr, world, t_f * 1e6, flops / t_f / 1e12,
                         100 * flops / t_f / 1e12 / (world * peak), t_s * 1e6, t_s / t_f),
                      flush=True)
            del x, y
        fused.close()
        del w
    if rank == 0:
        print("\npeaks: %s (bf16 %.0f TFLOP/s burst per GPU); fused / stock > 1 means the "
              "fused path is faster" % (src, peak))
    dist.barrier()
    dist.destroy_process_group()
    return 0


def run_sweep(args):
    """Config 5's sweep on one GPU: bi.linear and stock F.linear (cuBLAS) at every
    (K, N) of SHAPES and M in SWEEP_M, bf16; one markdown table on stdout.  Every
    weight exceeds L2 (>= 134 MB), so a GEMM re-reads it from HBM each launch."""
    import mlx_batch_invariant_b200 as bi
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    peaks, src = _peaks()
    peak, hbm = peaks["bf16_tflops"], peaks["hbm_gbs"]
    g = torch.Generator(device=dev)
    g.manual_seed(11)

    def timed(fn, reps):
        for _ in range(3):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps / 1e3

    print("| K | N | M | bi.linear µs | TFLOP/s | of tensor peak | HBM GB/s | cuBLAS µs | bi / cuBLAS |")
    print("|---|---|---|---|---|---|---|---|---|")
    for K, N in SHAPES:
        w = (torch.randn((N, K), generator=g, device=dev) * 0.02).to(torch.bfloat16)
        for Mr in SWEEP_M:
            x = torch.randn((Mr, K), generator=g, device=dev).to(torch.bfloat16)
            reps = 20 if Mr < 4096 else 5
            t_bi = timed(lambda: bi.linear(x, w), reps)
            t_cb = timed(lambda: torch.nn.functional.linear(x, w), reps)
            flops = 2.0 * Mr * N * K
            moved = 2.0 * (Mr * K + N * K + Mr * N)
            print("| %d | %d | %d | %.1f | %.1f | %.1f %% | %.0f | %.1f | %.2f |"
                  % (K, N, Mr, t_bi * 1e6, flops / t_bi / 1e12, 100 * flops / t_bi / 1e12 / peak,
                     moved / t_bi / 1e9, t_cb * 1e6, t_cb / t_bi), flush=True)
            del x
        del w
    print("\npeaks: %s (bf16 %.0f TFLOP/s burst, HBM %.0f GB/s); bi / cuBLAS > 1 means "
          "bi.linear is faster" % (src, peak, hbm))
    return 0


def main(argv=None):
    p = argparse.ArgumentParser(description="batch-invariant kernel throughput")
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--profile", choices=["gemm", "gemm-decode", "gemm-tf32x3", "sdpa"],
                   default=None)
    p.add_argument("--sweep", action="store_true",
                   help="config 5's M sweep (a markdown table, no JSON line); "
                        "column-parallel under torchrun with --gpus N > 1")
    args = p.parse_args(argv)
    if args.profile:
        return run_profile(args)
    if args.sweep:
        return run_sweep_parallel(args) if args.gpus > 1 else run_sweep(args)
    if args.warmup < 3:
        raise SystemExit("--warmup must be at least 3")
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
