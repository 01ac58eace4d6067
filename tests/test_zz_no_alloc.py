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


def _bind(L):
    vp, i64 = ctypes.c_void_p, ctypes.c_int64
    L.bi_gemm_allgather_static.restype = ctypes.c_int
    L.bi_gemm_allgather_static.argtypes = [
        vp, i64, vp, i64, vp, ctypes.POINTER(vp), i64, i64, i64, i64, i64, ctypes.c_int,
        ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
        ctypes.c_int, ctypes.c_int, ctypes.c_uint32, vp]


def test_static_scratch_allgather_matches_the_allocating_entry_point():
    from mlx_batch_invariant_b200 import _lib
    L = _lib.lib()
    _bind(L)
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
    try:
        for call in (1, 2):  # two calls in a row: the static block is reused
            x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
            w = (torch.randn(N, K, generator=g) / 32).to(torch.bfloat16).cuda()
            b = (torch.randn(N, generator=g) / 10).to(torch.bfloat16).cuda()
            want = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
            got = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
            outs_want = (ctypes.c_void_p * 1)(want.data_ptr())
            outs_got = (ctypes.c_void_p * 1)(got.data_ptr())
            _lib.check(L.bi_gemm_allgather(
                x.data_ptr(), K, w.data_ptr(), K, b.data_ptr(), outs_want, N, 0, M, N, K, 1,
                1.0, 1.0, _lib.BI_BF16, flags, 0, 1, call, stream), "bi_gemm_allgather")
            _lib.check(L.bi_gemm_allgather_static(
                x.data_ptr(), K, w.data_ptr(), K, b.data_ptr(), outs_got, N, 0, M, N, K, 1,
                1.0, 1.0, _lib.BI_BF16, devices, 0, 1, call, stream), "bi_gemm_allgather_static")
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
    _bind(L)
    devices = (ctypes.c_int * 9)(*([torch.cuda.current_device()] * 9))
    outs = (ctypes.c_void_p * 9)()
    st = L.bi_gemm_allgather_static(None, 8, None, 8, None, outs, 8, 0, 1, 8, 8, 1, 1.0, 1.0,
                                    _lib.BI_BF16, devices, 0, 9, 1, None)
    assert st == -1
    assert b"at most 8 ranks" in L.bi_last_error()
