"""Failure detection on the GPU, without a fault: a bounded device-side wait that
nothing ends.

One process, one GPU, two flag blocks from bi_peer_alloc.  bi_peer_barrier runs as
rank 0 of a world of 2 whose rank 1 never posts, so rank 0's wait for it gives up
after its cycle budget (about 2 s), records the entry-barrier timeout in the device
error word (site 6, reason 1) and returns instead of hanging.  The context stays
usable: the error word reads back, clears, and a GEMM launched afterwards is right.
(Ranks that die are tested on the host, as gloo processes: test_parallel_gloo.py.)
"""

import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

SITE_PEER_ENTRY, REASON_TIMEOUT = 6, 1


def test_a_wait_nothing_ends_times_out_and_is_reported():
    import mlx_batch_invariant_b200 as bi
    from mlx_batch_invariant_b200 import _lib
    L = _lib.lib()
    assert _lib.device_error() == 0  # start clean
    blocks = []
    for _ in range(2):
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        _lib.check(L.bi_peer_alloc(_lib.PEER_FLAG_BYTES, ctypes.byref(ptr), handle),
                   "bi_peer_alloc")
        blocks.append(ptr.value)
    flags = (ctypes.c_void_p * 2)(*blocks)
    try:
        t0 = time.time()
        _lib.check(L.bi_peer_barrier(flags, 0, 2, 1, _lib.stream_handle(torch.device("cuda"))),
                   "bi_peer_barrier")
        code = _lib.device_error()  # synchronises: returns once the wait has given up
        elapsed = time.time() - t0
        assert code == (SITE_PEER_ENTRY << 8) | REASON_TIMEOUT, hex(code)
        assert 0.5 < elapsed < 60, elapsed
        assert _lib.device_error() == 0  # read with clear: the word is reset

        # the context still works
        g = torch.Generator().manual_seed(5)
        x = torch.randn(64, 512, generator=g).to(torch.bfloat16).cuda()
        w = (torch.randn(256, 512, generator=g) / 16).to(torch.bfloat16).cuda()
        y = bi.linear(x, w).float()
        ref = x.double() @ w.double().T
        assert (y.double() - ref).abs().max().item() < 0.02 * ref.abs().max().item()
        assert _lib.device_error() == 0
    finally:
        torch.cuda.synchronize()
        for p in blocks:
            L.bi_peer_free(p)
