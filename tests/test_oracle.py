"""CPU tests of the oracle (bi_oracle.c): pinned against the golden fixtures and the
reference test suite's own assertions (tolerances against float64, single-rounding
addmm, mask and sink semantics), plus the bit / ULP helpers' self-test."""

import os

import ml_dtypes
import numpy as np
import pytest

from oracle import oracle as orc

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.npz")
DT = {"float32": np.float32, "float16": np.float16, "bfloat16": ml_dtypes.bfloat16}


def _load(arr, dt):
    return arr.view(dt) if arr.dtype == np.uint16 else arr


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(GOLDEN))


def test_oracle_reproduces_golden_gemm_fixtures(golden):
    n = 0
    for key in golden:
        if not (key.startswith("gemm_") and key.endswith("_y")):
            continue
        base = key[:-2]
        name = base.split("_")[1]
        dt = DT[name]
        nk = "_nk1_" in base
        a = _load(golden[base + "_a"], dt)
        b = _load(golden[base + "_b"], dt)
        bias = _load(golden[base + "_bias"], dt) if base + "_bias" in golden else None
        y = orc.gemm(a, b, bias, b_is_nk=nk)
        want = golden[key]
        got = y.view(np.uint16) if y.dtype.itemsize == 2 else y
        assert np.array_equal(got.view(want.dtype), want), base
        # and the fixture meets the reference's accuracy bounds against float64
        bb = b.astype(np.float64)
        ref = a.astype(np.float64) @ (bb.T if nk else bb)
        if bias is not None:
            ref = ref + bias.astype(np.float64)
        bound = {"float32": 5e-6, "float16": 5e-3, "bfloat16": 4e-2}[name]
        assert orc.rel_error(y.astype(np.float64), ref) < bound, base
        n += 1
    assert n == 36


def test_oracle_reproduces_golden_sdpa_fixtures(golden):
    n = 0
    for key in golden:
        if not (key.startswith("sdpa_") and key.endswith("_y")):
            continue
        base = key[:-2]
        _, name, mode = base.split("_")
        dt = DT[name]
        q, k, v = (_load(golden[base + s], dt) for s in ("_q", "_k", "_v"))
        N, qL = k.shape[2], q.shape[2]
        kw, mask64, sinks = {}, None, None
        if mode == "causal":
            kw = dict(mask_mode=1, causal_offset=N - qL)
            vis = np.arange(N)[None, :] <= (N - qL + np.arange(qL))[:, None]
            mask64 = np.where(vis, 0.0, -np.inf)[None, None]
        elif mode == "additive":
            m = _load(golden[base + "_mask"], dt)
            kw = dict(mask=m, mask_mode=2)
            mask64 = m.astype(np.float64)
        elif mode == "sinks":
            sinks = _load(golden[base + "_sinks"], dt)
            kw = dict(sinks=sinks)
        y = orc.sdpa(q, k, v, **kw)
        want = golden[key]
        got = y.view(np.uint16) if y.dtype.itemsize == 2 else y
        assert np.array_equal(got.view(want.dtype), want), base
        ref = orc.attention_f64(q.astype(np.float64), k.astype(np.float64), v.astype(np.float64),
                                mask=mask64,
                                sinks=None if sinks is None else sinks.astype(np.float64))
        bound = {"float32": 2e-6, "float16": 5e-3, "bfloat16": 3e-2}[name]
        assert orc.rel_error(y.astype(np.float64), ref) < bound, base
        n += 1
    assert n == 12


@pytest.mark.parametrize("M,K,N", [(17, 1024, 512), (128, 2048, 256), (1, 4096, 512),
                                   (8, 11008, 4096)])
def test_oracle_gemm_accuracy_float32(M, K, N):
    """tests/test_invariance.py:114-129 with the bound tightened to 5e-6."""
    rng = np.random.default_rng(M * 7 + K)
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.standard_normal((K, N)).astype(np.float32)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    assert orc.rel_error(orc.gemm(a, b), exact) < 5e-6


@pytest.mark.parametrize("dt,bound", [(np.float16, 5e-3), (ml_dtypes.bfloat16, 4e-2)])
def test_oracle_gemm_accuracy_low_precision(dt, bound):
    rng = np.random.default_rng(3)
    a = rng.standard_normal((8, 2048)).astype(np.float32).astype(dt)
    b = rng.standard_normal((2048, 256)).astype(np.float32).astype(dt)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    assert orc.rel_error(orc.gemm(a, b).astype(np.float64), exact) < bound


def test_oracle_gemm_rows_are_independent_of_the_batch():
    rng = np.random.default_rng(5)
    for dt in (np.float32, np.float16, ml_dtypes.bfloat16):
        w = rng.standard_normal((300, 96)).astype(np.float32).astype(dt)
        x = rng.standard_normal((33, 96)).astype(np.float32).astype(dt)
        full = orc.gemm(x, w, b_is_nk=True)
        for r in (0, 16, 32):
            one = orc.gemm(x[r:r + 1], w, b_is_nk=True)
            assert np.array_equal(one.view(np.uint8), full[r:r + 1].view(np.uint8))


def test_oracle_gemm_layouts_agree():
    """(N, K) and (K, N) layouts of the same weight give the same bits."""
    rng = np.random.default_rng(6)
    x = rng.standard_normal((7, 130)).astype(np.float32)
    w = rng.standard_normal((50, 130)).astype(np.float32)
    assert np.array_equal(orc.gemm(x, w, b_is_nk=True), orc.gemm(x, np.ascontiguousarray(w.T)))


def test_oracle_addmm_is_single_rounded():
    """tests/test_invariance.py:148-158: alpha*acc + beta*bias in fp32, then one
    rounding -- so the bf16 result equals round(fp32 result)."""
    rng = np.random.default_rng(7)
    for dt in (np.float16, ml_dtypes.bfloat16):
        a = rng.standard_normal((8, 512)).astype(np.float32).astype(dt)
        b = rng.standard_normal((512, 128)).astype(np.float32).astype(dt)
        c = rng.standard_normal(128).astype(np.float32).astype(dt)
        fused = orc.gemm(a, b, c)
        acc32 = orc.gemm(a.astype(np.float32), b.astype(np.float32), c.astype(np.float32))
        assert np.array_equal(fused.view(np.uint16), acc32.astype(dt).view(np.uint16))


def test_oracle_k_zero_gives_the_bias():
    a = np.zeros((3, 0), np.float32)
    b = np.zeros((0, 5), np.float32)
    c = np.arange(5, dtype=np.float32)
    assert np.array_equal(orc.gemm(a, b, c, alpha=2.0, beta=0.5), np.tile(c * 0.5, (3, 1)))


def _rand_attn(rng, B, H, Hkv, qL, N, D, dt):
    q = rng.standard_normal((B, H, qL, D)).astype(np.float32).astype(dt)
    k = rng.standard_normal((B, Hkv, N, D)).astype(np.float32).astype(dt)
    v = rng.standard_normal((B, Hkv, N, D)).astype(np.float32).astype(dt)
    return q, k, v


@pytest.mark.parametrize("dt,tol", [(np.float32, 2e-6), (ml_dtypes.bfloat16, 3e-2)])
def test_oracle_sdpa_accuracy_against_float64(dt, tol):
    """tests/test_invariance.py:408-432."""
    rng = np.random.default_rng(51)
    q, k, v = _rand_attn(rng, 1, 8, 4, 4, 2048, 128, dt)
    want = orc.attention_f64(q.astype(np.float64), k.astype(np.float64), v.astype(np.float64))
    assert orc.rel_error(orc.sdpa(q, k, v).astype(np.float64), want) < tol


def test_oracle_sdpa_causal_is_bottom_right_aligned():
    rng = np.random.default_rng(52)
    q, k, v = _rand_attn(rng, 1, 4, 2, 5, 200, 64, np.float32)
    got = orc.sdpa(q, k, v, mask_mode=1, causal_offset=200 - 5)
    vis = np.arange(200)[None, :] <= (195 + np.arange(5))[:, None]
    want = orc.attention_f64(q, k, v, mask=np.where(vis, 0.0, -np.inf)[None, None])
    assert orc.rel_error(got, want) < 2e-6
    # the same visibility as an explicit additive mask gives the same bits
    m = np.where(vis, 0.0, -np.inf).astype(np.float32)[None, None]
    assert np.array_equal(got, orc.sdpa(q, k, v, mask=m, mask_mode=2))


def test_oracle_sdpa_masked_extra_key_is_a_no_op():
    rng = np.random.default_rng(53)
    q, k, v = _rand_attn(rng, 2, 8, 2, 1, 4096, 128, ml_dtypes.bfloat16)
    k2 = np.concatenate([k, k[:, :, :1] * 3], axis=2)
    v2 = np.concatenate([v, v[:, :, :1] * 3], axis=2)
    m = np.zeros((1, 1, 1, 4097), np.float32)
    m[..., 4096] = -np.inf
    a = orc.sdpa(q, k, v, mask_mode=1, causal_offset=4096 - 1)
    b = orc.sdpa(q, k2, v2, mask=m.astype(ml_dtypes.bfloat16), mask_mode=2)
    assert np.array_equal(a.view(np.uint16), b.view(np.uint16))


def test_oracle_sdpa_fully_masked_rows_are_zero_and_sinks_count():
    rng = np.random.default_rng(54)
    q, k, v = _rand_attn(rng, 1, 4, 4, 3, 2, 32, np.float32)
    y = orc.sdpa(q, k, v, mask_mode=1, causal_offset=2 - 3)  # row 0 sees no key
    assert np.count_nonzero(y[:, :, 0]) == 0 and np.count_nonzero(y[:, :, 1:]) > 0
    sinks = np.full(4, 10.0, np.float32)
    q, k, v = _rand_attn(rng, 1, 4, 4, 1, 64, 32, np.float32)
    plain = orc.sdpa(q, k, v)
    sunk = orc.sdpa(q, k, v, sinks=sinks)
    assert not np.array_equal(plain, sunk)
    want = orc.attention_f64(q, k, v, sinks=sinks.astype(np.float64))
    assert orc.rel_error(sunk, want) < 2e-6


def test_oracle_sdpa_query_length_invariance():
    rng = np.random.default_rng(55)
    q, k, v = _rand_attn(rng, 1, 8, 2, 17, 333, 64, ml_dtypes.bfloat16)
    base = None
    for qL in (1, 2, 8, 9, 17):
        y = orc.sdpa(np.ascontiguousarray(q[:, :, 17 - qL:]), k, v, mask_mode=1,
                     causal_offset=333 - qL)
        last = y[:, :, -1].view(np.uint16)
        if base is None:
            base = last
        assert np.array_equal(last, base), qL


def test_lane_split_is_a_function_of_d_and_dtype():
    assert orc.lanes_for(128, ml_dtypes.bfloat16) == 8
    assert orc.lanes_for(128, np.float32) == 16
    assert orc.lanes_for(64, np.float16) == 4
    assert orc.lanes_for(96, ml_dtypes.bfloat16) == 4
    assert orc.lanes_for(256, np.float32) == 16
    assert orc.lanes_for(160, np.float32) == 16
    for D in range(32, 257, 32):
        for dt in (np.float32, np.float16):
            assert (D // orc.lanes_for(D, dt)) % 2 == 0


def test_bit_and_ulp_helpers_selftest():
    """probe/probe.py:390-408: a 1-ulp perturbation reads as one element at 1 ulp, and
    +0 / -0 are 0 ulp apart."""
    for dt in (np.float32, np.float16, ml_dtypes.bfloat16):
        a = np.array([1.0], dtype=dt)
        pa, n = orc.bits(a)
        pb = pa + 1
        assert int((pa != pb).sum()) == 1
        assert int(orc.ulp_distance(pa, pb, n)[0]) == 1
    pz, n = orc.bits(np.array([0.0, -0.0], dtype=np.float32))
    assert int(orc.ulp_distance(pz[:1], pz[1:], n)[0]) == 0
    pm, n = orc.bits(np.array([np.float32(1e-45), -np.float32(1e-45)], dtype=np.float32))
    assert int(orc.ulp_distance(pm[:1], pm[1:], n)[0]) == 2


@pytest.mark.parametrize("dt", ["bfloat16", "float16", "float32"])
def test_elementwise_attention_bar_accepts_the_rounded_fold(dt):
    """The GPU tests' elementwise attention bar (conftest.attn_worst) against the oracle's
    own output rounded to the input type: rounding alone uses at most half an output ulp,
    so it must pass with room only for the stated tau term."""
    import torch
    from conftest import attn_worst, to_np
    dtype = getattr(torch, dt)
    g = torch.Generator().manual_seed(1)
    q = torch.randn(1, 8, 3, 128, generator=g).to(dtype)
    k = torch.randn(1, 2, 300, 128, generator=g).to(dtype)
    v = torch.randn(1, 2, 300, 128, generator=g).to(dtype)
    o = orc.sdpa(to_np(q), to_np(k), to_np(v), mask_mode=1, causal_offset=297)
    if dtype == torch.bfloat16:
        ot = torch.from_numpy(o.view(np.uint16).astype(np.int32)).to(torch.int16).view(dtype)
    else:
        ot = torch.from_numpy(o)
    assert attn_worst(ot, q, k, v, mask_mode=1, causal_offset=297) <= 1.0
    # one output ulp off somewhere breaks it
    bad = ot.clone().float()
    bad.view(-1)[5] = bad.view(-1)[5] * (1 + 2.0 ** -6)
    assert attn_worst(bad.to(dtype), q, k, v, mask_mode=1, causal_offset=297) > 1.0


@pytest.mark.parametrize("D,V", [(192, 128), (64, 128), (576, 512)])
def test_oracle_sdpa_with_v_wider_or_narrower_than_d(D, V):
    """Head dims the reference takes (any multiples of 32, D != V allowed): the oracle's
    fold against float64, within the reference's float32 bar."""
    rng = np.random.default_rng(D + V)
    q = rng.standard_normal((1, 4, 3, D), dtype=np.float32)
    k = rng.standard_normal((1, 2, 200, D), dtype=np.float32)
    v = rng.standard_normal((1, 2, 200, V), dtype=np.float32)
    got = orc.sdpa(q, k, v, mask_mode=1, causal_offset=197)
    i = np.arange(200)[None, :]
    s = np.arange(3)[:, None]
    m = np.where(i <= 197 + s, 0.0, -np.inf)[None, None]
    want = orc.attention_f64(q, k, v, mask=m)
    assert got.shape == (1, 4, 3, V)
    assert orc.rel_error(got, want) < 2e-6
