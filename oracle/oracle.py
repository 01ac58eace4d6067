"""NumPy-facing wrapper of the CPU oracle (bi_oracle.c) plus bit / ULP helpers.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline legs as the checker.  The library itself never imports it.

Parity unpinned at the bit level (the reference runs only under MLX/Metal, which
do not exist here, and ships no golden vectors); see bi_oracle.c's header for what
pins it instead.
"""

import ctypes
import os

import numpy as np

try:
    import ml_dtypes
    BF16 = np.dtype(ml_dtypes.bfloat16)
except ImportError:  # pragma: no cover
    BF16 = None

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "build", "libbi_oracle.so")

CODES = {np.dtype(np.float32): 0, np.dtype(np.float16): 1}
if BF16 is not None:
    CODES[BF16] = 2
UINT = {np.dtype(np.float32): np.uint32, np.dtype(np.float16): np.uint16}
if BF16 is not None:
    UINT[BF16] = np.uint16

_lib = None
_i64p = ctypes.POINTER(ctypes.c_int64)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            import importlib.util
            spec = importlib.util.spec_from_file_location("_oracle_build",
                                                          os.path.join(HERE, "build.py"))
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)
            mod.build()
        L = ctypes.CDLL(LIB_PATH)
        vp, i64 = ctypes.c_void_p, ctypes.c_int64
        L.oracle_gemm.restype = None
        L.oracle_gemm.argtypes = [vp, i64, vp, i64, vp, vp, i64, i64, i64, i64, ctypes.c_int,
                                  ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_int]
        L.oracle_sdpa.restype = None
        L.oracle_sdpa.argtypes = [vp, _i64p, vp, _i64p, vp, _i64p, vp, _i64p, ctypes.c_int, i64,
                                  vp, ctypes.c_float, i64, i64, i64, i64, i64, i64, ctypes.c_int,
                                  vp, _i64p, ctypes.c_int, ctypes.c_int]
        L.oracle_sdpa_ex.restype = None
        L.oracle_sdpa_ex.argtypes = [vp, _i64p, vp, _i64p, vp, _i64p, vp, _i64p, ctypes.c_int,
                                     i64, vp, ctypes.c_float, i64, i64, i64, i64, i64, i64, i64,
                                     ctypes.c_int, vp, _i64p, ctypes.c_int, ctypes.c_int,
                                     ctypes.c_int, ctypes.c_int]
        L.oracle_round.restype = ctypes.c_float
        L.oracle_round.argtypes = [ctypes.c_float, ctypes.c_int]
        _lib = L
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def _i64s(vals):
    arr = (ctypes.c_int64 * len(vals))(*[int(v) for v in vals])
    return arr


def gemm(a, b, bias=None, b_is_nk=False, alpha=1.0, beta=1.0, threads=0):
    """Sequential-K fp32 host emulation of bi_gemm.  a (M, K); b (N, K) if b_is_nk
    else (K, N); bias (N,) or None.  Arrays share one of float32/float16/bfloat16."""
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    dt = a.dtype
    assert b.dtype == dt and dt in CODES
    M, K = a.shape
    N = b.shape[0] if b_is_nk else b.shape[1]
    out = np.empty((M, N), dtype=dt)
    if bias is not None:
        bias = np.ascontiguousarray(bias.astype(dt))
    lib().oracle_gemm(_ptr(a), K, _ptr(b), b.shape[1], _ptr(bias), _ptr(out), N, M, N, K,
                      1 if b_is_nk else 0, alpha, beta, CODES[dt], threads)
    return out


def generic_route(D, V):
    """Whether bi_sdpa takes its kernel for other head dims (D != V or D > 256): 16
    lanes per key row and 2-element vectors, whatever the dtype."""
    return D != V or D > 256


def lanes_for(D, dtype):
    """Threads a key row is split over in bi_sdpa (a function of D and dtype only),
    for D == V <= 256."""
    es = np.dtype(dtype).itemsize
    lp = max(1, min(16, (D * es) // 32))
    p2 = 1
    while p2 * 2 <= lp:
        p2 *= 2
    while p2 > 1 and D % p2:
        p2 //= 2
    return p2


def sdpa(q, k, v, mask=None, mask_mode=0, causal_offset=0, sinks=None, scale=None, lanes=None,
         threads=0, out_dtype=None):
    """Host restatement of bi_sdpa.  q (B,H,qL,D), k/v (B,Hkv,N,D); mask is the
    additive mask (already in q's dtype, 4-D, broadcast dims of size 1) for mode 2.
    out_dtype=np.float32 returns the fold's fp32 result before the final rounding."""
    q = np.ascontiguousarray(q)
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    dt = q.dtype
    B, H, qL, D = q.shape
    _, Hkv, N, V = v.shape
    if scale is None:
        scale = 1.0 / np.sqrt(D)
    per = 0
    if generic_route(D, V):
        lanes, per = 16, 2
    elif lanes is None:
        lanes = lanes_for(D, dt)
    odt = np.dtype(out_dtype) if out_dtype is not None else dt
    out = np.empty((B, H, qL, V), dtype=odt)
    ms = [0, 0, 0]
    if mask_mode == 2:
        mask = np.ascontiguousarray(mask.astype(dt))
        Bm, Hm, Lm, Nm = mask.shape
        ms = [0 if Bm == 1 else Hm * Lm * Nm, 0 if Hm == 1 else Lm * Nm, 0 if Lm == 1 else Nm]
    else:
        mask = None
    if sinks is not None:
        sinks = np.ascontiguousarray(sinks.astype(dt))
    qs = [H * qL * D, qL * D, D]
    ks = [Hkv * N * D, N * D]
    vs = [Hkv * N * V, N * V]
    os_ = [H * qL * V, qL * V, V]
    lib().oracle_sdpa_ex(_ptr(q), _i64s(qs), _ptr(k), _i64s(ks), _ptr(v), _i64s(vs),
                         _ptr(mask), _i64s(ms), mask_mode, causal_offset, _ptr(sinks),
                         float(scale), B, H, Hkv, qL, N, D, V, CODES[dt], _ptr(out), _i64s(os_),
                         CODES[odt], lanes, per, threads)
    return out


# ------------------------------------------------------------ bits and ULPs
# Restates probe/probe.py:33-45 (bit_pattern, ulp_distance) on NumPy arrays.

def bits(a):
    """Flat array -> (unsigned bit patterns, bit width)."""
    a = np.ascontiguousarray(a)
    u = UINT[a.dtype]
    return a.reshape(-1).view(u), 8 * a.dtype.itemsize


def ulp_distance(x, y, n):
    """IEEE-754 ULP distance between two arrays of n-bit patterns."""
    top = 1 << (n - 1)
    xi, yi = x.astype(np.int64), y.astype(np.int64)
    xo = np.where(xi >= top, top - xi, xi)
    yo = np.where(yi >= top, top - yi, yi)
    return np.abs(xo - yo)


def rel_error(got, exact):
    """max |got - exact| / max |exact| (tests/test_invariance.py:122-123)."""
    got = np.asarray(got, dtype=np.float64)
    exact = np.asarray(exact, dtype=np.float64)
    scale = np.abs(exact).max()
    return float(np.abs(got - exact).max() / scale) if scale > 0 else float(np.abs(got).max())


def attention_f64(q, k, v, mask=None, scale=None, sinks=None):
    """float64 softmax attention (tests/test_invariance.py:408-424): q (B,H,qL,D),
    k/v (B,Hkv,N,D), additive mask broadcastable to (B,H,qL,N) with -inf for masked."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    B, H, qL, D = q.shape
    Hkv = k.shape[1]
    k = np.repeat(k, H // Hkv, axis=1)
    v = np.repeat(v, H // Hkv, axis=1)
    sc = (1.0 / np.sqrt(D)) if scale is None else scale
    s = np.einsum("bhqd,bhkd->bhqk", q, k) * sc
    if mask is not None:
        s = s + np.asarray(mask, dtype=np.float64)
    if sinks is not None:
        sk = np.asarray(sinks, dtype=np.float64).reshape(1, H, 1, 1) * np.ones((B, H, qL, 1))
        s = np.concatenate([s, sk], axis=-1)
    mx = s.max(axis=-1, keepdims=True)
    mx = np.where(np.isfinite(mx), mx, 0.0)
    p = np.exp(s - mx)
    den = p.sum(axis=-1, keepdims=True)
    if sinks is not None:
        p = p[..., :-1]
    with np.errstate(invalid="ignore", divide="ignore"):
        out = np.einsum("bhqk,bhkd->bhqd", p, v) / den
    return np.where(den > 0, out, 0.0)
