"""bi_gemm_allgather_static: the fused column-parallel GEMM for callers that may not
allocate device memory (a server whose allocator owns all of HBM, a host that only
passes buffers it owns).  Its scratch (the CTA counter and the call count) lives in a
static device array inside libbi.so instead of memory from bi_peer_alloc; the flags
ranks post to one another sit at the head of the exchange areas the caller passes.

Called through the C ABI on one GPU (world = 1), twice in a row, and checked against
the existing entry point bi_gemm_allgather on the same inputs.  Both run the same
kernel, so the bar is the one the tests use for identical arithmetic: equal bits.
With two GPUs, two ranks driven by one process do real peer stores into each other's
staging area and static flag block, checked against one GPU's bits.  The argument
guards (one rank per device, the rank's device current) are checked too.
This file is collected last so that a failure here leaves every other test run.
"""

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_static_scratch_allgather_matches_the_allocating_entry_point():
    from mlx_batch_invariant_b200 import _lib
    L = _lib.lib()
    dev = torch.cuda.current_device()
    stream = torch.cuda.current_stream().cuda_stream
    M, K, N = 300, 1024, 768
    g = torch.Generator().manual_seed(2024)

    # the existing entry point needs a flag block from bi_peer_alloc
    flag_ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    _lib.check(L.bi_peer_alloc(_lib.PEER_FLAG_BYTES, ctypes.byref(flag_ptr), handle),
               "bi_peer_alloc")
    flags = (ctypes.c_void_p * 1)(flag_ptr.value)
    devices = (ctypes.c_int * 1)(dev)
    cols = (ctypes.c_int64 * 2)(0, N)
    # one rank: no peer stores into the staging area, which must still be given; the
    # static entry's exchange area is a zeroed flag block followed by that area
    stage = torch.empty(M * N, dtype=torch.bfloat16, device="cuda")
    stages = (ctypes.c_void_p * 1)(stage.data_ptr())
    xarea = torch.zeros(_lib.PEER_FLAG_BYTES // 2 + M * N, dtype=torch.bfloat16, device="cuda")
    xareas = (ctypes.c_void_p * 1)(xarea.data_ptr())
    try:
        for call in (1, 2):  # two calls in a row: the static block is reused
            x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
            w = (torch.randn(N, K, generator=g) / 32).to(torch.bfloat16).cuda()
            b = (torch.randn(N, generator=g) / 10).to(torch.bfloat16).cuda()
            want = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
            got = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
            _lib.check(L.bi_gemm_allgather(
                x.data_ptr(), K, w.data_ptr(), K, b.data_ptr(), want.data_ptr(), N, stages, cols,
                M, K, 1, 1.0, 1.0, _lib.BI_BF16, flags, 0, 1, call, stream), "bi_gemm_allgather")
            _lib.check(L.bi_gemm_allgather_static(
                x.data_ptr(), K, w.data_ptr(), K, b.data_ptr(), got.data_ptr(), N, xareas, cols,
                M, K, 1, 1.0, 1.0, _lib.BI_BF16, devices, 0, 1, call, stream),
                "bi_gemm_allgather_static")
            torch.cuda.synchronize()
            assert not torch.isnan(got).any(), "call %d left outputs unwritten" % call
            assert np.array_equal(got.view(torch.int16).cpu().numpy(),
                                  want.view(torch.int16).cpu().numpy()), "call %d" % call
        assert _lib.device_error() == 0
    finally:
        torch.cuda.synchronize()
        L.bi_peer_free(flag_ptr)


def test_static_scratch_rejects_more_ranks_than_it_holds():
    from mlx_batch_invariant_b200 import _lib
    L = _lib.lib()
    devices = (ctypes.c_int * 9)(*range(9))
    stages = (ctypes.c_void_p * 9)()
    cols = (ctypes.c_int64 * 10)(*range(0, 80, 8))
    st = L.bi_gemm_allgather_static(None, 8, None, 8, None, None, 72, stages, cols, 1, 8, 1,
                                    1.0, 1.0, _lib.BI_BF16, devices, 0, 9, 1, None)
    assert st == -1
    assert b"at most 8 ranks" in L.bi_last_error()



def test_static_scratch_rejects_a_rank_whose_device_is_not_current():
    """devices[rank] must be the current device: the local GEMM counts its CTAs in the
    block of the device it runs on."""
    from mlx_batch_invariant_b200 import _lib
    L = _lib.lib()
    other = torch.cuda.current_device() + 1
    devices = (ctypes.c_int * 1)(other)
    area = torch.zeros(256, dtype=torch.bfloat16, device="cuda")
    stages = (ctypes.c_void_p * 1)(area.data_ptr())
    cols = (ctypes.c_int64 * 2)(0, 8)
    st = L.bi_gemm_allgather_static(None, 8, None, 8, None, None, 8, stages, cols, 1, 8, 1,
                                    1.0, 1.0, _lib.BI_BF16, devices, 0, 1, 1, None)
    assert st == -1
    assert b"is current" in L.bi_last_error()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_static_scratch_two_devices_in_one_process_match_one_gpu():
    """Two ranks driven by one process on devices 0 and 1: real peer stores into the
    other device's staging area and flags.  The gathered output of both ranks, on two
    calls in a row, equals bi_gemm of the full weight on one GPU, and equals the
    allocating entry point's (flag blocks from bi_peer_alloc)."""
    from mlx_batch_invariant_b200 import _lib
    L = _lib.lib()
    M, K, N = 300, 1024, 1536
    cols = (ctypes.c_int64 * 3)(0, 768, N)
    devices = (ctypes.c_int * 2)(0, 1)
    g = torch.Generator().manual_seed(77)
    stages = [torch.empty(M * N, dtype=torch.bfloat16, device="cuda:%d" % r) for r in range(2)]
    stage_ptrs = (ctypes.c_void_p * 2)(*[t.data_ptr() for t in stages])
    # the static entry's exchange areas: a zeroed flag block, then the staging area
    xareas = [torch.zeros(_lib.PEER_FLAG_BYTES // 2 + M * N, dtype=torch.bfloat16,
                          device="cuda:%d" % r) for r in range(2)]
    xarea_ptrs = (ctypes.c_void_p * 2)(*[t.data_ptr() for t in xareas])
    flag_ptrs = []
    for r in range(2):
        with torch.cuda.device(r):
            p = ctypes.c_void_p()
            _lib.check(L.bi_peer_alloc(_lib.PEER_FLAG_BYTES, ctypes.byref(p),
                                       ctypes.create_string_buffer(64)), "bi_peer_alloc")
            flag_ptrs.append(p.value)
    flags = (ctypes.c_void_p * 2)(*flag_ptrs)
    try:
        for call in (1, 2):
            x = torch.randn(M, K, generator=g).to(torch.bfloat16)
            w = (torch.randn(N, K, generator=g) / 32).to(torch.bfloat16)
            b = (torch.randn(N, generator=g) / 10).to(torch.bfloat16)
            want = bits(_one_gpu(x, w, b))
            for entry in ("static", "allocating"):
                outs = []
                for r in range(2):
                    with torch.cuda.device(r):
                        dev = "cuda:%d" % r
                        xs = x.to(dev)
                        ws = w[cols[r]:cols[r + 1]].contiguous().to(dev)
                        bs = b[cols[r]:cols[r + 1]].contiguous().to(dev)
                        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=dev)
                        stream = torch.cuda.current_stream(r).cuda_stream
                        if entry == "static":
                            st = L.bi_gemm_allgather_static(
                                xs.data_ptr(), K, ws.data_ptr(), K, bs.data_ptr(), out.data_ptr(),
                                N, xarea_ptrs, cols, M, K, 1, 1.0, 1.0, _lib.BI_BF16, devices, r,
                                2, call, stream)
                        else:
                            st = L.bi_gemm_allgather(
                                xs.data_ptr(), K, ws.data_ptr(), K, bs.data_ptr(), out.data_ptr(),
                                N, stage_ptrs, cols, M, K, 1, 1.0, 1.0, _lib.BI_BF16, flags, r, 2,
                                call, stream)
                        _lib.check(st, entry)
                        outs.append((xs, ws, bs, out))
                for r in range(2):
                    torch.cuda.synchronize(r)
                for r in range(2):
                    assert np.array_equal(bits(outs[r][3]), want), (entry, call, r)
                for r in range(2):
                    with torch.cuda.device(r):
                        assert _lib.device_error() == 0
    finally:
        for r in range(2):
            torch.cuda.synchronize(r)
            with torch.cuda.device(r):
                L.bi_peer_free(ctypes.c_void_p(flag_ptrs[r]))


def _one_gpu(x, w, b):
    import mlx_batch_invariant_b200 as bi
    with torch.cuda.device(0):
        return bi.linear(x.cuda(0), w.cuda(0), b.cuda(0))


def bits(t):
    return t.detach().contiguous().view(torch.int16).cpu().numpy()
