"""bi_gemm_allgather_static: the fused column-parallel GEMM for callers that may not
allocate device memory (a server whose allocator owns all of HBM, a host that only
passes buffers it owns), whose epoch-flag block lives in a static device array inside
libbi.so instead of memory from bi_peer_alloc.

Called through the C ABI on one GPU (world = 1), twice in a row, and checked against
the existing entry point bi_gemm_allgather on the same inputs.  Both run the same
kernel, so the bar is the one the tests use for identical arithmetic: equal bits.
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
    # one rank: no peer stores into the staging area, which must still be given
    stage = torch.empty(M * N, dtype=torch.bfloat16, device="cuda")
    stages = (ctypes.c_void_p * 1)(stage.data_ptr())
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
                x.data_ptr(), K, w.data_ptr(), K, b.data_ptr(), got.data_ptr(), N, stages, cols,
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
    devices = (ctypes.c_int * 9)(*([torch.cuda.current_device()] * 9))
    stages = (ctypes.c_void_p * 9)()
    cols = (ctypes.c_int64 * 10)(*range(0, 80, 8))
    st = L.bi_gemm_allgather_static(None, 8, None, 8, None, None, 72, stages, cols, 1, 8, 1,
                                    1.0, 1.0, _lib.BI_BF16, devices, 0, 9, 1, None)
    assert st == -1
    assert b"at most 8 ranks" in L.bi_last_error()
