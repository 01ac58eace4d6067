"""GPU parity and invariance tests of the batch-invariant attention (libbi.so bi_sdpa).

Parity bar against the host oracle (the reference's per-key fold), elementwise
(conftest.attn_worst): every output element within half an output ulp of the oracle's
unrounded fp32 result (2 fp32 ulps for float32) plus tau * sum_i p_i |v_ij| / sum_i p_i,
tau = 2^-20 on both routes: the CUDA-core one runs the oracle's fold, lane split and
order (C-library expf in place of CUDA's); the GQA one (16-bit, D = 64 / 128, GQA groups
of 4k heads) takes score = scale * (q . k) from a tensor-core dot product and folds a
partial's keys 4 at a time, with P.V in exact fp32.
Accuracy against float64 follows the reference (tests/test_invariance.py:408-432):
float32 < 2e-6, bfloat16 < 3e-2.  Invariance bar: 0 differing bits.
"""

import math

import numpy as np
import pytest
import torch

from conftest import attn_worst, batch_with, bits, randn, to_np
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.float16, torch.bfloat16]
TOL = {torch.float32: 2e-6, torch.float16: 2.0 ** -10, torch.bfloat16: 2.0 ** -7}


@pytest.fixture(scope="module")
def bi():
    import mlx_batch_invariant_b200 as bi
    return bi


def _np_mask(mask, dtype):
    """Additive mask in q's dtype as the kernel sees it (bool -> 0 / -inf)."""
    if mask.dtype == torch.bool:
        mask = torch.where(mask, torch.zeros((), dtype=dtype, device=mask.device),
                           torch.full((), -math.inf, dtype=dtype, device=mask.device))
    m = mask.to(dtype)
    while m.ndim < 4:
        m = m.unsqueeze(0)
    return to_np(m)


def _oracle(q, k, v, mask=None, sinks=None):
    B, H, qL, D = q.shape
    N = k.shape[2]
    if isinstance(mask, str):
        return orc.sdpa(to_np(q), to_np(k), to_np(v), mask_mode=1, causal_offset=N - qL,
                        sinks=to_np(sinks) if sinks is not None else None)
    if mask is not None:
        return orc.sdpa(to_np(q), to_np(k), to_np(v), mask=_np_mask(mask, q.dtype), mask_mode=2,
                        sinks=to_np(sinks) if sinks is not None else None)
    return orc.sdpa(to_np(q), to_np(k), to_np(v),
                    sinks=to_np(sinks) if sinks is not None else None)


def _close(got, want, dtype):
    g = to_np(got).astype(np.float64)
    w = np.asarray(want).astype(np.float64)
    scale = max(np.abs(w).max(), 1e-30)
    return np.abs(g - w).max() / scale <= TOL[dtype] * (1.0 if dtype == torch.float32 else 1.01)


CASES = [(8, 8, 1, 512, 128), (32, 8, 4, 1024, 128), (4, 2, 3, 777, 64), (8, 4, 8, 333, 64),
         (4, 4, 2, 100, 32), (2, 1, 5, 257, 96), (4, 2, 1, 130, 256), (2, 2, 3, 64, 160)]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("maskkind", ["none", "causal", "additive", "bool"])
def test_parity_against_oracle(bi, dtype, maskkind):
    for (H, Hkv, qL, N, D) in CASES:
        q = randn((2, H, qL, D), dtype, 41, "cuda")
        k = randn((2, Hkv, N, D), dtype, 42, "cuda")
        v = randn((2, Hkv, N, D), dtype, 43, "cuda")
        mask = None
        if maskkind == "causal":
            mask = "causal"
        elif maskkind == "additive":
            mask = randn((1, 1, qL, N), dtype, 44, "cuda")
        elif maskkind == "bool":
            g = torch.Generator().manual_seed(45)
            mask = (torch.rand(2, 1, qL, N, generator=g) > 0.1).cuda()
        y = bi.scaled_dot_product_attention(q, k, v, mask=mask)
        if mask == "causal":
            worst = attn_worst(y, q, k, v, mask_mode=1, causal_offset=N - qL)
        elif mask is not None:
            worst = attn_worst(y, q, k, v, mask_mode=2, mask=torch.from_numpy(
                np.asarray(_np_mask(mask, dtype), dtype=np.float32)).to(dtype))
        else:
            worst = attn_worst(y, q, k, v)
        assert worst <= 1.0, (dtype, maskkind, H, Hkv, qL, N, D, worst)


@pytest.mark.parametrize("dtype", DTYPES)
def test_sinks_parity_and_effect(bi, dtype):
    H, Hkv, qL, N, D = 8, 4, 3, 300, 64
    q = randn((1, H, qL, D), dtype, 45, "cuda")
    k = randn((1, Hkv, N, D), dtype, 46, "cuda")
    v = randn((1, Hkv, N, D), dtype, 47, "cuda")
    sinks = randn((H,), dtype, 48, "cuda")
    y = bi.scaled_dot_product_attention(q, k, v, sinks=sinks)
    assert attn_worst(y, q, k, v, sinks=sinks) <= 1.0


def test_accuracy_against_float64(bi):
    """tests/test_invariance.py:408-432."""
    for dtype, tol in ((torch.float32, 2e-6), (torch.bfloat16, 3e-2)):
        H, Hkv, qL, N, D = 8, 4, 4, 2048, 128
        q = randn((1, H, qL, D), dtype, 51, "cuda")
        k = randn((1, Hkv, N, D), dtype, 52, "cuda")
        v = randn((1, Hkv, N, D), dtype, 53, "cuda")
        want = orc.attention_f64(to_np(q).astype(np.float64), to_np(k).astype(np.float64),
                                 to_np(v).astype(np.float64))
        err = orc.rel_error(to_np(bi.scaled_dot_product_attention(q, k, v)), want)
        assert err < tol, "%s rel err %.3e" % (dtype, err)


QLS = [1, 2, 3, 4, 7, 8, 9, 16, 17]


@pytest.mark.parametrize("dtype", DTYPES)
def test_query_length_invariance(bi, dtype):
    """tests/test_invariance.py:246-276 (last row bits over qL)."""
    for H, Hkv, N, D in ((32, 8, 512, 128), (16, 8, 4096, 128), (8, 8, 4096, 128),
                         (32, 8, 8192, 128), (4, 4, 333, 64)):
        k = randn((1, Hkv, N, D), dtype, 11, "cuda")
        v = randn((1, Hkv, N, D), dtype, 12, "cuda")
        qf = randn((1, H, max(QLS), D), dtype, 13, "cuda")
        base = None
        for qL in QLS:
            y = bi.scaled_dot_product_attention(qf[:, :, max(QLS) - qL:, :].contiguous(), k, v)
            got = bits(y[:, :, -1, :])
            if base is None:
                base = got
                assert bool((y != 0).any())
            else:
                assert int((got != base).sum()) == 0, (dtype, H, Hkv, N, qL)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_decode_batch_and_kv_length_invariance_c2(bi, dtype):
    """Config 2: q (B,32,1,128), k/v (B,8,L,128), causal; the shared row in slot 0 has
    the same bits for every B, and L=4097 (one appended key masked out) equals L=4096."""
    H, Hkv, D = 32, 8, 128
    for L in (511, 1024, 4096):
        q1 = randn((1, H, 1, D), dtype, 3, "cuda")
        k1 = randn((1, Hkv, L, D), dtype, 4, "cuda")
        v1 = randn((1, Hkv, L, D), dtype, 5, "cuda")
        base = None
        for B in (1, 2, 4, 8, 16, 64):
            if B == 1:
                q, k, v = q1, k1, v1
            else:
                q = torch.cat([q1, randn((B - 1, H, 1, D), dtype, 100 + B, "cuda")])
                k = torch.cat([k1, randn((B - 1, Hkv, L, D), dtype, 200 + B, "cuda")])
                v = torch.cat([v1, randn((B - 1, Hkv, L, D), dtype, 300 + B, "cuda")])
            got = bits(bi.scaled_dot_product_attention(q, k, v, mask="causal")[0])
            if base is None:
                base = got
            else:
                assert int((got != base).sum()) == 0, (dtype, L, B)
        if L == 4096:
            # one more key, fully masked: an explicit boolean mask keeps keys < 4096
            k2 = torch.cat([k1, randn((1, Hkv, 1, D), dtype, 7, "cuda")], dim=2)
            v2 = torch.cat([v1, randn((1, Hkv, 1, D), dtype, 8, "cuda")], dim=2)
            keep = torch.ones(1, 1, 1, L + 1, dtype=torch.bool, device="cuda")
            keep[..., L] = False
            ext = bi.scaled_dot_product_attention(q1, k2, v2, mask=keep)
            plain = bi.scaled_dot_product_attention(q1, k1, v1, mask="causal")
            assert np.array_equal(bits(ext), bits(plain)), dtype
            # and keys 4096..8191 masked out of an 8192 context change nothing either
            k3 = torch.cat([k1, randn((1, Hkv, L, D), dtype, 9, "cuda")], dim=2)
            v3 = torch.cat([v1, randn((1, Hkv, L, D), dtype, 10, "cuda")], dim=2)
            keep3 = torch.zeros(1, 1, 1, 2 * L, dtype=torch.bool, device="cuda")
            keep3[..., :L] = True
            ext3 = bi.scaled_dot_product_attention(q1, k3, v3, mask=keep3)
            assert np.array_equal(bits(ext3), bits(plain)), dtype


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("D", [64, 128])
def test_gqa_launch_plans_keep_the_bits(bi, dtype, D):
    """The GQA kernel takes 1, 2 or 4 query heads per CTA and a 1- or 3-stage ring from
    the grid size (B * H * qL against the SM count); none of it may change a row.  With
    H = 32, Hkv = 8 the batches below run GH = 1 (B <= 4), GH = 2 (B = 8) and GH = 4
    (B >= 16, one or two CTAs per SM): slot 0's bits must not move."""
    H, Hkv, L = 32, 8, 1500
    q1 = randn((1, H, 1, D), dtype, 31, "cuda")
    k1 = randn((1, Hkv, L, D), dtype, 32, "cuda")
    v1 = randn((1, Hkv, L, D), dtype, 33, "cuda")
    sinks = randn((H,), dtype, 34, "cuda")
    base = None
    for B in (1, 3, 8, 16, 40, 64):
        q = torch.cat([q1, randn((B - 1, H, 1, D), dtype, 400 + B, "cuda")]) if B > 1 else q1
        k = torch.cat([k1, randn((B - 1, Hkv, L, D), dtype, 500 + B, "cuda")]) if B > 1 else k1
        v = torch.cat([v1, randn((B - 1, Hkv, L, D), dtype, 600 + B, "cuda")]) if B > 1 else v1
        got = bits(bi.scaled_dot_product_attention(q, k, v, mask="causal", sinks=sinks)[0])
        if base is None:
            base = got
        else:
            assert int((got != base).sum()) == 0, (dtype, D, B)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("Hkv", [32, 16, 8])
@pytest.mark.parametrize("D", [64, 128])
def test_chunked_prefill_invariance_c3(bi, dtype, Hkv, D):
    """Config 3: chunks of Lq in {1,2,4,8,9,16,64,512} against KV 2048, H=32; every
    absolute query position gives the same bits whatever chunk it was in, for causal,
    additive and boolean masks (mask rows sliced by absolute position)."""
    H, N, LMAX = 32, 2048, 512
    k = randn((1, Hkv, N, D), dtype, 61, "cuda")
    v = randn((1, Hkv, N, D), dtype, 62, "cuda")
    qf = randn((1, H, LMAX, D), dtype, 63, "cuda")
    add = randn((1, 1, LMAX, N), dtype, 64, "cuda")
    g = torch.Generator().manual_seed(65)
    keep = (torch.rand(1, 1, LMAX, N, generator=g) > 0.1).cuda()
    full = {}
    for label in ("causal", "additive", "bool"):
        for Lq in (512, 1, 2, 4, 8, 9, 16, 64):
            q = qf[:, :, LMAX - Lq:, :].contiguous()
            mk = {"causal": "causal", "additive": add[:, :, LMAX - Lq:, :],
                  "bool": keep[:, :, LMAX - Lq:, :]}[label]
            y = bi.scaled_dot_product_attention(q, k, v, mask=mk)
            if Lq == 512:
                full[label] = y
                continue
            a = bits(y)
            b = bits(full[label][:, :, LMAX - Lq:, :])
            assert int((a != b).sum()) == 0, (label, dtype, Hkv, D, Lq)


def test_batch_invariance(bi):
    """tests/test_invariance.py:278-299."""
    H, Hkv, N, D = 16, 8, 2048, 128
    for dtype in DTYPES:
        k1, v1 = randn((1, Hkv, N, D), dtype, 21, "cuda"), randn((1, Hkv, N, D), dtype, 22, "cuda")
        q1 = randn((1, H, 1, D), dtype, 23, "cuda")
        kp, vp = randn((16, Hkv, N, D), dtype, 24, "cuda"), randn((16, Hkv, N, D), dtype, 25, "cuda")
        qp = randn((16, H, 1, D), dtype, 26, "cuda")
        base = None
        for B in (1, 2, 3, 8, 16):
            idx = B // 2
            y = bi.scaled_dot_product_attention(batch_with(q1, qp, B, idx),
                                                batch_with(k1, kp, B, idx),
                                                batch_with(v1, vp, B, idx))
            got = bits(y[idx])
            if base is None:
                base = got
            else:
                assert int((got != base).sum()) == 0, (dtype, B)


def test_sinks_are_query_length_invariant_and_matter(bi):
    """tests/test_invariance.py:323-364."""
    H, Hkv, N, D = 32, 8, 1024, 128
    for dtype in DTYPES:
        k, v = randn((1, Hkv, N, D), dtype, 71, "cuda"), randn((1, Hkv, N, D), dtype, 72, "cuda")
        qf = randn((1, H, 17, D), dtype, 73, "cuda")
        sinks = randn((H,), dtype, 74, "cuda")
        base = None
        for qL in (1, 2, 3, 7, 8, 9, 16, 17):
            y = bi.scaled_dot_product_attention(qf[:, :, 17 - qL:, :].contiguous(), k, v,
                                                sinks=sinks)
            got = bits(y[:, :, -1, :])
            if base is None:
                base = got
            else:
                assert int((got != base).sum()) == 0, (dtype, qL)
    q = randn((1, 8, 1, 64), torch.float32, 75, "cuda")
    k = randn((1, 8, 256, 64), torch.float32, 76, "cuda")
    v = randn((1, 8, 256, 64), torch.float32, 77, "cuda")
    s = torch.full((8,), 10.0, device="cuda")
    assert int((bits(bi.scaled_dot_product_attention(q, k, v)) !=
                bits(bi.scaled_dot_product_attention(q, k, v, sinks=s))).sum()) > 0
    with pytest.raises(ValueError):
        bi.scaled_dot_product_attention(q, k, v, sinks=torch.zeros(4, device="cuda"))


def test_fully_masked_rows_are_zero(bi):
    q = randn((1, 4, 6, 64), torch.bfloat16, 1, "cuda")
    k = randn((1, 2, 4, 64), torch.bfloat16, 2, "cuda")
    v = randn((1, 2, 4, 64), torch.bfloat16, 3, "cuda")
    # bottom-right causal with qL > N: the first qL - N rows see no key
    y = bi.scaled_dot_product_attention(q, k, v, mask="causal")
    assert torch.count_nonzero(y[:, :, :2, :]) == 0
    assert torch.count_nonzero(y[:, :, 2:, :]) > 0
    none = torch.zeros(1, 1, 6, 4, dtype=torch.bool, device="cuda")
    assert torch.count_nonzero(bi.scaled_dot_product_attention(q, k, v, mask=none)) == 0


def test_head_shards_match_full_output(bi):
    """Head-parallel invariance emulated on one GPU: heads [r*H/g, (r+1)*H/g) with their
    kv heads give the same bits as the full call's slice."""
    dtype = torch.bfloat16
    H, Hkv, qL, N, D = 32, 8, 5, 1000, 128
    q = randn((2, H, qL, D), dtype, 1, "cuda")
    k = randn((2, Hkv, N, D), dtype, 2, "cuda")
    v = randn((2, Hkv, N, D), dtype, 3, "cuda")
    full = bi.scaled_dot_product_attention(q, k, v, mask="causal")
    for g in (2, 4, 8):
        for r in range(g):
            hs, ks = H // g, Hkv // g
            part = bi.scaled_dot_product_attention(q[:, r * hs:(r + 1) * hs], k[:, r * ks:(r + 1) * ks],
                                                   v[:, r * ks:(r + 1) * ks], mask="causal")
            assert np.array_equal(bits(part), bits(full[:, r * hs:(r + 1) * hs])), (g, r)


def test_strided_views_match_contiguous(bi):
    """(B, L, H, D) tensors transposed to (B, H, L, D) views give the same bits."""
    dtype = torch.float16
    q = randn((2, 7, 8, 64), dtype, 1, "cuda").transpose(1, 2)
    k = randn((2, 300, 4, 64), dtype, 2, "cuda").transpose(1, 2)
    v = randn((2, 300, 4, 64), dtype, 3, "cuda").transpose(1, 2)
    a = bi.scaled_dot_product_attention(q, k, v, mask="causal")
    b = bi.scaled_dot_product_attention(q.contiguous(), k.contiguous(), v.contiguous(),
                                        mask="causal")
    assert np.array_equal(bits(a), bits(b))


def test_cuda_graph_capture_is_bitwise_identical(bi):
    dtype = torch.bfloat16
    q = randn((4, 32, 1, 128), dtype, 1, "cuda")
    k = randn((4, 8, 2048, 128), dtype, 2, "cuda")
    v = randn((4, 8, 2048, 128), dtype, 3, "cuda")
    eager = bi.scaled_dot_product_attention(q, k, v, mask="causal")
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        bi.scaled_dot_product_attention(q, k, v, mask="causal")
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y = bi.scaled_dot_product_attention(q, k, v, mask="causal")
    g.replay()
    torch.cuda.synchronize()
    assert np.array_equal(bits(y), bits(eager))
    assert bi._lib.device_error() == 0


def test_stock_sdpa_is_query_variant_control():
    """Negative control (tests/test_invariance.py:435-455) on torch's SDPA backends:
    somewhere the last row changes with the query-chunk length."""
    import torch.nn.functional as F
    found = []
    for dtype in (torch.float16, torch.bfloat16):
        for H, Hkv, N, D in ((32, 8, 512, 128), (32, 32, 2048, 128), (16, 16, 4096, 64)):
            k = randn((1, H, N, D), dtype, 61, "cuda")
            v = randn((1, H, N, D), dtype, 62, "cuda")
            qf = randn((1, H, 64, D), dtype, 63, "cuda")
            outs = []
            for qL in (1, 8, 9, 16, 64):
                y = F.scaled_dot_product_attention(qf[:, :, 64 - qL:].contiguous(), k, v)
                outs.append(bits(y[:, :, -1, :]))
            if any(int((o != outs[0]).sum()) for o in outs[1:]):
                found.append((dtype, H, N, D))
    assert found, "stock torch SDPA looks query-length invariant everywhere"


# (H, Hkv, qL, N, D, V): head dims the generic kernel takes -- D != V (a DeepSeek-style
# 192 / 128, MLA's absorbed 576 / 512) or above 256.
GENERIC = [(8, 2, 3, 300, 192, 128), (4, 4, 2, 130, 64, 128), (8, 8, 1, 257, 128, 64),
           (4, 2, 5, 200, 320, 320), (4, 1, 2, 150, 96, 288), (2, 1, 3, 100, 576, 512),
           (2, 2, 2, 64, 512, 512), (4, 2, 2, 90, 640, 640)]


def _generic_built(dtype, D, V):
    if dtype == torch.float32:
        return D <= 384 and V <= 384 and D + V <= 768
    return D <= 640 and V <= 640


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("maskkind", ["none", "causal", "additive", "bool", "sinks"])
def test_generic_head_dims_parity_against_oracle(bi, dtype, maskkind):
    """D != V and head dims above 256 (the reference takes any multiples of 32,
    _attention.py:216-223): elementwise against the oracle's fold with the generic
    kernel's lane split (16 lanes, 2-element vectors)."""
    ran = 0
    for (H, Hkv, qL, N, D, V) in GENERIC:
        if not _generic_built(dtype, D, V):
            continue
        q = randn((2, H, qL, D), dtype, 71, "cuda")
        k = randn((2, Hkv, N, D), dtype, 72, "cuda")
        v = randn((2, Hkv, N, V), dtype, 73, "cuda")
        sinks = randn((H,), dtype, 74, "cuda") if maskkind == "sinks" else None
        if maskkind == "causal":
            y = bi.scaled_dot_product_attention(q, k, v, mask="causal")
            worst = attn_worst(y, q, k, v, mask_mode=1, causal_offset=N - qL)
        elif maskkind in ("additive", "bool"):
            if maskkind == "additive":
                mask = randn((1, 1, qL, N), dtype, 75, "cuda")
            else:
                g = torch.Generator().manual_seed(76)
                mask = (torch.rand(2, 1, qL, N, generator=g) > 0.1).cuda()
            y = bi.scaled_dot_product_attention(q, k, v, mask=mask)
            worst = attn_worst(y, q, k, v, mask_mode=2, mask=torch.from_numpy(
                np.asarray(_np_mask(mask, dtype), dtype=np.float32)).to(dtype))
        else:
            y = bi.scaled_dot_product_attention(q, k, v, sinks=sinks)
            worst = attn_worst(y, q, k, v, sinks=sinks)
        assert y.shape == (2, H, qL, V)
        assert worst <= 1.0, (dtype, maskkind, H, Hkv, qL, N, D, V, worst)
        ran += 1
    assert ran >= 5
    assert bi._lib.device_error() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_generic_head_dims_are_query_length_and_batch_invariant(bi, dtype):
    """The generic kernel keeps the fold's contract: a query's bits do not depend on
    the other queries of the call or on the batch around it; a masked extra key is a
    no-op."""
    shapes = [(8, 2, 1000, 192, 128)] + ([(4, 1, 700, 576, 512)] if dtype != torch.float32
                                          else [(4, 1, 700, 320, 320)])
    for H, Hkv, N, D, V in shapes:
        k = randn((1, Hkv, N, D), dtype, 81, "cuda")
        v = randn((1, Hkv, N, V), dtype, 82, "cuda")
        qf = randn((1, H, 17, D), dtype, 83, "cuda")
        base = None
        for qL in (1, 2, 7, 9, 17):
            y = bi.scaled_dot_product_attention(qf[:, :, 17 - qL:].contiguous(), k, v,
                                                mask="causal")
            got = bits(y[:, :, -1])
            if base is None:
                base = got
            else:
                assert np.array_equal(got, base), (D, V, qL)
        # batch: the same row in slot 0 of a batch of 3
        kb = torch.cat([k, randn((2, Hkv, N, D), dtype, 84, "cuda")])
        vb = torch.cat([v, randn((2, Hkv, N, V), dtype, 85, "cuda")])
        qb = torch.cat([qf[:, :, -1:], randn((2, H, 1, D), dtype, 86, "cuda")])
        yb = bi.scaled_dot_product_attention(qb, kb, vb, mask="causal")
        assert np.array_equal(bits(yb[:1, :, -1]), base), (D, V, "batch")
        # one more key, masked off: same bits
        k1 = torch.cat([k, randn((1, Hkv, 1, D), dtype, 87, "cuda")], dim=2)
        v1 = torch.cat([v, randn((1, Hkv, 1, V), dtype, 88, "cuda")], dim=2)
        keep = torch.ones(1, 1, 1, N + 1, dtype=torch.bool, device="cuda")
        keep[..., N] = False
        y1 = bi.scaled_dot_product_attention(qf[:, :, -1:].contiguous(), k1, v1, mask=keep)
        assert np.array_equal(bits(y1[:, :, -1]), base), (D, V, "masked extra key")


def test_head_dims_beyond_the_built_range_raise(bi):
    q = randn((1, 2, 1, 672), torch.bfloat16, 1, "cuda")
    with pytest.raises(NotImplementedError):
        bi.scaled_dot_product_attention(q, q, q)
    q32 = randn((1, 2, 1, 416), torch.float32, 1, "cuda")
    with pytest.raises(NotImplementedError):
        bi.scaled_dot_product_attention(q32, q32, q32)
