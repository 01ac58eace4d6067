"""Parity against the host oracle at the sizes of the workloads the library is measured
on (2, 3 and 5), elementwise, on sampled rows.

The kernels run at full size on the GPU; the oracle (the reference's algorithm restated
in C) recomputes a sample of the output rows -- rows in several pair tiles of the
GEMM (M = 4096 covers 16 of them), every head of several batch entries of decode
attention, and query rows across a 512-row chunked prefill.

GEMM bar (every sampled element): within 1 ulp of the output type of the oracle's
rounded value plus the fp32 reordering allowance 2^-21 * sum_k |a[m,k] b[k,n]| (the
tensor cores add the same products in K=16 hardware steps).  float32 takes the
CUDA-core route, which runs the oracle's K order: bit-exact.

Attention bar (every sampled element): conftest.attn_worst -- within half an output
ulp of the oracle's unrounded fp32 result plus tau * sum_i p_i |v_ij| / sum_i p_i, with
tau = 2^-20 on both routes (the GQA route departs from the reference's per-key fold in
two places -- score = scale * (q . k) from a tensor-core dot product, keys folded 4 at
a time -- and runs P.V in exact fp32).
"""

import math

import numpy as np
import pytest
import torch

from conftest import attn_worst, to_np, ulp_of
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

BF16 = torch.bfloat16


@pytest.fixture(scope="module")
def bi():
    import mlx_batch_invariant_b200 as bi
    return bi


# ---------------------------------------------------------------- GEMM

def _gemm_ok(got, want, dtype, absterm):
    g = to_np(got).astype(np.float64)
    w = np.asarray(want).astype(np.float64)
    if dtype == torch.float32:
        return np.array_equal(g, w), 0.0
    tol = ulp_of(w, dtype) + 2.0 ** -21 * absterm
    worst = float((np.abs(g - w) / tol).max())
    return worst <= 1.0 + 1e-9, worst


def _rows_in_pair_tiles(M, n=64):
    """Rows of every 256-row pair tile: its first, last and a middle row, plus spread."""
    rows = set()
    for t0 in range(0, M, 256):
        rows.update((t0, min(t0 + 127, M - 1), min(t0 + 128, M - 1), min(t0 + 255, M - 1)))
    rows = sorted(rows)
    if len(rows) > n:
        idx = np.linspace(0, len(rows) - 1, n).round().astype(int)
        rows = [rows[i] for i in idx]
    return rows


def _cols_across_tiles(N, g):
    """All columns of the first and last 256-wide tiles, plus 512 random ones."""
    cols = set(range(0, min(256, N))) | set(range(max(0, N - 256), N))
    cols |= set(torch.randint(0, N, (512,), generator=g).tolist())
    return sorted(cols)


CONFIG5 = [(8192, 10240), (8192, 8192), (8192, 57344), (28672, 8192)]


@pytest.mark.parametrize("K,N", CONFIG5)
def test_config5_linear_sampled_rows_match_oracle(bi, K, N):
    """Config 5: y = bi.linear(x, w) at M = 4096, bf16, x ~ N(0,1), w ~ N(0, 0.02),
    64 rows spread over all 16 pair tiles of M and ~1000 columns across N."""
    M = 4096
    gd = torch.Generator(device="cuda").manual_seed(K + N)
    x = torch.randn(M, K, generator=gd, device="cuda").to(BF16)
    w = (torch.randn(N, K, generator=gd, device="cuda") * 0.02).to(BF16)
    y = bi.linear(x, w)
    gh = torch.Generator().manual_seed(N)
    rows = _rows_in_pair_tiles(M)
    cols = _cols_across_tiles(N, gh)
    ri = torch.tensor(rows, device="cuda")
    ci = torch.tensor(cols, device="cuda")
    xs, ws = to_np(x[ri]), to_np(w[ci])
    want = orc.gemm(xs, ws, b_is_nk=True)
    got = y[ri][:, ci]
    absterm = np.abs(xs.astype(np.float64)) @ np.abs(ws.astype(np.float64)).T
    ok, worst = _gemm_ok(got, want, BF16, absterm)
    assert ok, "K=%d N=%d worst |gpu-oracle|/bar = %.3f" % (K, N, worst)
    # the reference's own accuracy bar vs float64 (tests/test_invariance.py:129-132)
    exact = xs.astype(np.float64) @ ws.astype(np.float64).T
    assert orc.rel_error(to_np(got), exact) < 4e-2


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("op", ["linear", "matmul", "addmm"])
def test_config1_full_output_matches_oracle(bi, dtype, op):
    """Config 1 at its largest batch: M = 128, K = N = 4096, x ~ N(0,1),
    w ~ N(0,1)/64, bias ~ N(0, 0.1); every output element compared."""
    M, K, N = 128, 4096, 4096
    gd = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(M, K, generator=gd, device="cuda").to(dtype)
    w = (torch.randn(N, K, generator=gd, device="cuda") / 64).to(dtype)
    bias = (torch.randn(N, generator=gd, device="cuda") * 0.1).to(dtype)
    if op == "linear":
        y = bi.linear(x, w, bias)
        b, b_is_nk, c = w, True, bias
    elif op == "matmul":
        b = w.t().contiguous()
        y = bi.matmul(x, b)
        b_is_nk, c = False, None
    else:
        b = w.t().contiguous()
        y = bi.addmm(bias, x, b)
        b_is_nk, c = False, bias
    want = orc.gemm(to_np(x), to_np(b), to_np(c) if c is not None else None, b_is_nk=b_is_nk)
    a64 = np.abs(to_np(x).astype(np.float64))
    b64 = np.abs(to_np(b).astype(np.float64))
    absterm = a64 @ (b64.T if b_is_nk else b64)
    ok, worst = _gemm_ok(y, want, dtype, absterm)
    assert ok, "%s %s worst %.3f" % (dtype, op, worst)


# ---------------------------------------------------------------- attention

def _attn_check(got, q, k, v, mask4, dtype, H, Hkv, D):
    """Worst |gpu - w| / bar (conftest.attn_worst) for rows q of a call; mask4 the
    additive mask of those rows (-inf = masked) or None."""
    return attn_worst(got, q, k, v, mask_mode=2 if mask4 is not None else 0, mask=mask4)


def _causal_as_mask(S_rows, N, qL, dtype, device):
    """Bottom-right causal visibility of query rows S_rows of a qL-row call against N
    keys, as an additive mask (a masked key is skipped either way)."""
    i = torch.arange(N, device=device)[None, :]
    s = torch.tensor(S_rows, device=device)[:, None]
    vis = i <= (N - qL) + s
    m = torch.where(vis, torch.zeros((), device=device), torch.full((), -math.inf, device=device))
    return m.to(dtype)[None, None]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("L", [4095, 8192])
def test_config2_decode_sampled_batches_match_oracle(bi, dtype, L):
    """Config 2: q (64, 32, 1, 128), k/v (64, 8, L, 128) ~ N(0,1), causal; every head of
    batch entries 0, 17 and 63 compared."""
    B, H, Hkv, D = 64, 32, 8, 128
    gd = torch.Generator(device="cuda").manual_seed(L)
    q = torch.randn(B, H, 1, D, generator=gd, device="cuda").to(dtype)
    k = torch.randn(B, Hkv, L, D, generator=gd, device="cuda").to(dtype)
    v = torch.randn(B, Hkv, L, D, generator=gd, device="cuda").to(dtype)
    y = bi.scaled_dot_product_attention(q, k, v, mask="causal")
    bs = torch.tensor([0, 17, 63], device="cuda")
    # with one query row the bottom-right causal rule shows every key
    worst = _attn_check(y[bs], q[bs], k[bs], v[bs], None, dtype, H, Hkv, D)
    assert worst <= 1.0, "L=%d %s worst |gpu-oracle|/bar = %.3f" % (L, dtype, worst)


CONFIG3_ROWS = [0, 1, 9, 31, 32, 100, 255, 256, 400, 511]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("Hkv", [32, 16, 8])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("maskkind", ["causal", "additive", "bool"])
def test_config3_prefill_sampled_rows_match_oracle(bi, dtype, Hkv, D, maskkind):
    """Config 3 at its largest chunk: q (1, 32, 512, D) against k/v (1, Hkv, 2048, D);
    causal, additive N(0,1) and boolean (10% False) masks; 10 query rows spread over the
    chunk, every head, compared."""
    H, qL, N = 32, 512, 2048
    seed = 1000 * Hkv + D + {"causal": 1, "additive": 2, "bool": 3}[maskkind]
    gd = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(1, H, qL, D, generator=gd, device="cuda").to(dtype)
    k = torch.randn(1, Hkv, N, D, generator=gd, device="cuda").to(dtype)
    v = torch.randn(1, Hkv, N, D, generator=gd, device="cuda").to(dtype)
    rows = torch.tensor(CONFIG3_ROWS, device="cuda")
    if maskkind == "causal":
        y = bi.scaled_dot_product_attention(q, k, v, mask="causal")
        m4 = _causal_as_mask(CONFIG3_ROWS, N, qL, dtype, "cuda")
    elif maskkind == "additive":
        mask = torch.randn(1, 1, qL, N, generator=gd, device="cuda").to(dtype)
        y = bi.scaled_dot_product_attention(q, k, v, mask=mask)
        m4 = mask[:, :, rows]
    else:
        keep = torch.rand(1, 1, qL, N, generator=gd, device="cuda") > 0.1
        y = bi.scaled_dot_product_attention(q, k, v, mask=keep)
        m4 = torch.where(keep[:, :, rows], torch.zeros((), device="cuda"),
                         torch.full((), -math.inf, device="cuda")).to(dtype)
    worst = _attn_check(y[:, :, rows], q[:, :, rows], k, v, m4, dtype, H, Hkv, D)
    assert worst <= 1.0, "%s Hkv=%d D=%d %s worst |gpu-oracle|/bar = %.3f" % (
        dtype, Hkv, D, maskkind, worst)
