"""The Llama-shaped decoder harness on one GPU (the reference's bench/bench.py:211-246
determinism check, extended over decode steps): under batch_invariant_mode the
slot-0 logits of the prefill and of every greedy decode step are bitwise equal at
batch 1, 3 and 8.  A 2-layer d=1024 model with the config's head layout keeps the
test to seconds; the full 8B run is `python -m mlx_batch_invariant_b200 decoder`."""

import pytest
import torch

pytestmark = pytest.mark.gpu

SMALL = dict(layers=2, hidden=1024, heads=16, kv_heads=8, head_dim=64, inter=2048, vocab=4096)


@pytest.fixture(scope="module")
def model():
    from mlx_batch_invariant_b200 import decoder as dec
    m = dec.Decoder(dec.DecoderConfig(**SMALL), max_batch=8, max_len=48, device="cuda")
    yield m
    m.close()


def _slot0(model, batch, prompt=37, steps=6):
    from mlx_batch_invariant_b200 import decoder as dec
    ids = dec.prompts(model.cfg, batch, prompt, "cuda")
    logits, _, _ = dec.generate(model, ids, steps)
    return dec.slot0_bits(logits)


def test_decoder_logits_are_bitwise_equal_across_batch(model):
    import mlx_batch_invariant_b200 as bi
    from mlx_batch_invariant_b200 import decoder as dec
    with bi.batch_invariant_mode(strict=True):
        base = _slot0(model, 1)
        for B in (3, 8):
            assert dec.differing(_slot0(model, B), base) == [0] * base.shape[0], B


def test_decoder_runs_the_invariant_kernels(model):
    """The prefill's logits differ from stock torch's somewhere (the mode really
    routed the GEMMs and attention), yet stay close to them."""
    import mlx_batch_invariant_b200 as bi
    from mlx_batch_invariant_b200 import decoder as dec
    ids = dec.prompts(model.cfg, 2, 37, "cuda")
    with bi.batch_invariant_mode(strict=True):
        ours = model.prefill(ids).float()
    stock = model.prefill(ids).float()
    assert not torch.equal(ours, stock)
    assert (ours - stock).abs().max().item() < 0.05 * stock.abs().max().item()


def test_stock_rms_norm_is_row_invariant_at_prefill_sizes():
    """F.rms_norm runs unwrapped in the decoder on (B, L, d) activations: a row's bits
    must not depend on how many rows (up to a batch-8 x 512-token prefill) share it."""
    d = 4096
    g = torch.Generator(device="cuda").manual_seed(3)
    w = torch.randn(d, generator=g, device="cuda").to(torch.bfloat16)
    pool = torch.randn(4096, d, generator=g, device="cuda").to(torch.bfloat16)
    row = pool[:1].clone()
    want = torch.nn.functional.rms_norm(row, (d,), w, 1e-5).view(torch.int16)
    for rows, shape in ((512, (1, 512, d)), (4096, (8, 512, d)), (3, (3, 1, d))):
        x = pool[:rows].clone().reshape(shape)
        y = torch.nn.functional.rms_norm(x, (d,), w, 1e-5).reshape(rows, d)
        assert torch.equal(y[:1].view(torch.int16), want), rows


def test_graph_decode_matches_eager_decode_bitwise(model):
    """DecodeGraph replays (device position, full-cache attention with the later keys
    masked out) give the eager decode's bits, and stay batch-invariant."""
    import mlx_batch_invariant_b200 as bi
    from mlx_batch_invariant_b200 import decoder as dec
    with bi.batch_invariant_mode(strict=True):
        eager = _slot0(model, 3)
        graph = dec.DecodeGraph(model, 3)
        ids = dec.prompts(model.cfg, 3, 37, "cuda")
        logits, _, _ = dec.generate(model, ids, 6, graph)
        assert dec.differing(dec.slot0_bits(logits), eager) == [0] * eager.shape[0]
        g1 = dec.DecodeGraph(model, 1)
        logits1, _, _ = dec.generate(model, ids[:1], 6, g1)
        assert dec.differing(dec.slot0_bits(logits1), eager) == [0] * eager.shape[0]


def test_fused_rope_and_cache_write_match_the_torch_expression_bitwise():
    """bi_rope_kv against the decoder's torch RoPE (fp32 ops, then bf16) and plain cache
    writes, with the position given on the host and as a device tensor."""
    from mlx_batch_invariant_b200 import _lib
    from mlx_batch_invariant_b200.decoder import _rope
    B, L, hq, hk, hd, P, p0 = 3, 5, 4, 2, 64, 32, 7
    g = torch.Generator(device="cuda").manual_seed(9)
    qkv = torch.randn(B, L, (hq + 2 * hk) * hd, generator=g, device="cuda").to(torch.bfloat16)
    inv = 1.0 / (500000.0 ** (torch.arange(0, hd, 2, device="cuda", dtype=torch.float32) / hd))
    ang = torch.arange(P, device="cuda", dtype=torch.float32)[:, None] * inv[None, :]
    cos, sin = torch.cos(ang), torch.sin(ang)
    q, k, v = qkv.split((hq * hd, hk * hd, hk * hd), dim=-1)
    want_q = _rope(q.reshape(B, L, hq, hd).transpose(1, 2), cos[p0:p0 + L], sin[p0:p0 + L])
    want_k = _rope(k.reshape(B, L, hk, hd).transpose(1, 2), cos[p0:p0 + L], sin[p0:p0 + L])
    want_v = v.reshape(B, L, hk, hd).transpose(1, 2)
    for pos in (None, torch.tensor([p0], device="cuda")):
        q_out = torch.empty(B, hq, L, hd, dtype=torch.bfloat16, device="cuda")
        kc = torch.zeros(B, hk, P, hd, dtype=torch.bfloat16, device="cuda")
        vc = torch.zeros_like(kc)
        _lib.check(_lib.lib().bi_rope_kv(
            qkv.data_ptr(), B, L, hq, hk, hd, cos.data_ptr(), sin.data_ptr(),
            p0 if pos is None else 0, pos.data_ptr() if pos is not None else None, P,
            q_out.data_ptr(), kc.data_ptr(), vc.data_ptr(), _lib.i64_3(kc.stride()[:3]),
            _lib.BI_BF16, torch.cuda.current_stream().cuda_stream), "bi_rope_kv")
        torch.cuda.synchronize()
        assert torch.equal(q_out.view(torch.int16), want_q.contiguous().view(torch.int16))
        assert torch.equal(kc[:, :, p0:p0 + L].view(torch.int16), want_k.contiguous().view(torch.int16))
        assert torch.equal(vc[:, :, p0:p0 + L], want_v)
        assert not kc[:, :, :p0].any() and not kc[:, :, p0 + L:].any()
    assert _lib.device_error() == 0


def test_rope_position_past_the_cache_is_refused_not_written():
    """A position at the cache length: the host form is refused before launch; a device
    position (which the host cannot see) writes nothing and sets the device error word
    (site 1, reason 2, tagged bit 17)."""
    from mlx_batch_invariant_b200 import _lib
    B, L, hq, hk, hd, P = 2, 1, 4, 2, 64, 16
    qkv = torch.ones(B, L, (hq + 2 * hk) * hd, dtype=torch.bfloat16, device="cuda")
    cos = torch.ones(P, hd // 2, device="cuda")
    sin = torch.zeros(P, hd // 2, device="cuda")
    q_out = torch.zeros(B, hq, L, hd, dtype=torch.bfloat16, device="cuda")
    # a guard region after the caches: an unchecked write at position P would land there
    kc_all = torch.zeros(B, hk, P + 4, hd, dtype=torch.bfloat16, device="cuda")
    vc_all = torch.zeros_like(kc_all)
    kc, vc = kc_all[:, :, :P], vc_all[:, :, :P]
    assert _lib.device_error() == 0
    with pytest.raises(_lib.LibraryError):
        _lib.check(_lib.lib().bi_rope_kv(
            qkv.data_ptr(), B, L, hq, hk, hd, cos.data_ptr(), sin.data_ptr(), P, None, P,
            q_out.data_ptr(), kc.data_ptr(), vc.data_ptr(), _lib.i64_3(kc.stride()[:3]),
            _lib.BI_BF16, torch.cuda.current_stream().cuda_stream), "bi_rope_kv")
    pos = torch.tensor([P], device="cuda")
    _lib.check(_lib.lib().bi_rope_kv(
        qkv.data_ptr(), B, L, hq, hk, hd, cos.data_ptr(), sin.data_ptr(), 0, pos.data_ptr(), P,
        q_out.data_ptr(), kc.data_ptr(), vc.data_ptr(), _lib.i64_3(kc.stride()[:3]),
        _lib.BI_BF16, torch.cuda.current_stream().cuda_stream), "bi_rope_kv")
    torch.cuda.synchronize()
    assert _lib.device_error() == (1 << 17) | (1 << 8) | 2
    assert _lib.device_error() == 0  # read-and-clear
    assert not kc_all.any() and not vc_all.any() and not q_out.any()


def test_fused_swiglu_is_within_one_ulp_of_torch():
    from mlx_batch_invariant_b200 import _lib
    M, I = 37, 1024
    g = torch.Generator(device="cuda").manual_seed(10)
    gu = (torch.randn(M, 2 * I, generator=g, device="cuda") * 3).to(torch.bfloat16)
    out = torch.empty(M, I, dtype=torch.bfloat16, device="cuda")
    _lib.check(_lib.lib().bi_swiglu(gu.data_ptr(), out.data_ptr(), M, I, _lib.BI_BF16,
                                    torch.cuda.current_stream().cuda_stream), "bi_swiglu")
    want = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]
    torch.cuda.synchronize()
    a = out.float()
    w = want.float()
    ulp = torch.clamp(w.abs(), min=2.0 ** -126) * 2.0 ** -7
    assert ((a - w).abs() <= ulp).all()


def _eager_slot0(model, batch, prompt=21, steps=4):
    from mlx_batch_invariant_b200 import decoder as dec
    ids = dec.prompts(model.cfg, batch, prompt, "cuda")
    logits, _, _ = dec.generate(model, ids, steps)
    return dec.slot0_bits(logits)


def test_stock_decoder_is_batch_variant_somewhere_control():
    """Negative control for the decoder (the role of the reference's stock-MLX row in
    bench/bench.py:211-246): stock torch (cuBLAS + SDPA) on this model must give the
    shared slot-0 prompt different logits at some batch size or dtype -- and the
    invariant path, on that same model and batch, none."""
    import mlx_batch_invariant_b200 as bi
    from mlx_batch_invariant_b200 import decoder as dec
    found = []
    for dtype in (torch.bfloat16, torch.float32):
        m = dec.Decoder(dec.DecoderConfig(**SMALL), max_batch=64, max_len=32, dtype=dtype,
                        device="cuda")
        try:
            base = _eager_slot0(m, 1)
            variant = [B for B in (8, 33, 64) if any(dec.differing(_eager_slot0(m, B), base))]
            if variant:
                found.append((dtype, variant))
                with bi.batch_invariant_mode(strict=True):
                    ibase = _eager_slot0(m, 1)
                    for B in variant:
                        assert not any(dec.differing(_eager_slot0(m, B), ibase)), (dtype, B)
        finally:
            m.close()
    assert found, "stock torch gave every batch the same slot-0 logits in bf16 and fp32"


def test_invariant_logits_are_as_close_to_an_fp32_forward_as_stock():
    """The invariant bf16 model against a float32 forward of the same weights (stock
    torch, no TF32), on the prefill and three decode steps fed the fp32 model's greedy
    tokens: its normwise error max|ours - fp32| / max|fp32| stays within twice stock
    bf16's and under 5e-2 (the reference's bar for its quantized path,
    tests/test_invariance.py:585-592, and its bf16 GEMM bar)."""
    import mlx_batch_invariant_b200 as bi
    from mlx_batch_invariant_b200 import decoder as dec
    assert not torch.backends.cuda.matmul.allow_tf32
    cfg = dec.DecoderConfig(**SMALL)
    m16 = dec.Decoder(cfg, max_batch=2, max_len=40, device="cuda")
    m32 = dec.Decoder(cfg, max_batch=2, max_len=40, dtype=torch.float32, device="cuda")
    try:
        for l16, l32 in zip(m16.layers, m32.layers):
            for key in l16:
                l32[key].copy_(l16[key].float())
        for name in ("embed", "norm", "head"):
            getattr(m32, name).copy_(getattr(m16, name).float())
        ids = dec.prompts(cfg, 2, 37, "cuda")

        def run(model, mode):
            with (bi.batch_invariant_mode(strict=True) if mode else _null()):
                out = [model.prefill(ids).double()]
                for t in toks:
                    out.append(model.decode(t).double())
            return torch.stack(out)

        toks = []
        ref = [m32.prefill(ids).double()]
        for _ in range(3):
            toks.append(ref[-1].argmax(dim=-1))
            ref.append(m32.decode(toks[-1]).double())
        ref = torch.stack(ref)
        ours = run(m16, True)
        stock = run(m16, False)
        scale = ref.abs().max()
        e_ours = ((ours - ref).abs().max() / scale).item()
        e_stock = ((stock - ref).abs().max() / scale).item()
        assert e_ours <= 2 * e_stock + 1e-6 and e_ours < 5e-2, (e_ours, e_stock)
    finally:
        m16.close()
        m32.close()


class _null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False
