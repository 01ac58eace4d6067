"""ctypes binding of libbi.so, the C-ABI kernel library (include/bi.h).

The library is built in-tree by ``mlx-batch-invariant_b200/build.py``.  There is no
fallback: if it is missing or the device is not an sm_100 GPU, every operator raises.
"""

import ctypes
import os
import threading

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libbi.so")

BI_F32, BI_F16, BI_BF16 = 0, 1, 2
DTYPE_CODE = {torch.float32: BI_F32, torch.float16: BI_F16, torch.bfloat16: BI_BF16}

ROUTE_TCGEN05, ROUTE_SIMT = 0, 1
MAX_PEERS = 8          # BI_MAX_PEERS
PEER_FLAG_BYTES = 256  # BI_PEER_FLAG_BYTES

_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
_i64_3 = _i64 * 3
_i64_2 = _i64 * 2

_lock = threading.Lock()
_lib = None


class LibraryError(RuntimeError):
    """A libbi.so call returned a non-zero status."""

    def __init__(self, status, where, detail):
        self.status = status
        super().__init__("libbi %s failed: %s (%d)%s"
                         % (where, _status_string(status), status,
                            (": " + detail) if detail else ""))


def _bind(lib):
    lib.bi_gemm.restype = ctypes.c_int
    lib.bi_gemm.argtypes = [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.c_int,
                            ctypes.c_float, ctypes.c_float, ctypes.c_int, _vp]
    lib.bi_gemm_tf32x3.restype = ctypes.c_int
    lib.bi_gemm_tf32x3.argtypes = [_vp, _i64, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _i64,
                                   ctypes.c_int, ctypes.c_float, ctypes.c_float, _vp]
    lib.bi_gemm_route.restype = ctypes.c_int
    lib.bi_gemm_route.argtypes = [ctypes.c_int, _i64, _i64, ctypes.c_int,
                                  ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                                  ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]
    lib.bi_sdpa.restype = ctypes.c_int
    lib.bi_sdpa.argtypes = [_vp, _i64_3, _vp, _i64_2, _vp, _i64_2, _vp, _i64_3, ctypes.c_int,
                            _i64, _vp, ctypes.c_float, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                            ctypes.c_int, _vp, _i64_3, _vp]
    lib.bi_status_string.restype = ctypes.c_char_p
    lib.bi_status_string.argtypes = [ctypes.c_int]
    lib.bi_last_error.restype = ctypes.c_char_p
    lib.bi_last_error.argtypes = []
    lib.bi_device_error.restype = ctypes.c_int
    lib.bi_device_error.argtypes = [ctypes.c_int]
    lib.bi_version.restype = ctypes.c_int
    lib.bi_version.argtypes = []
    lib.bi_peer_alloc.restype = ctypes.c_int
    lib.bi_peer_alloc.argtypes = [_i64, ctypes.POINTER(ctypes.c_void_p), ctypes.c_char_p]
    lib.bi_peer_open.restype = ctypes.c_int
    lib.bi_peer_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]
    lib.bi_peer_close.restype = ctypes.c_int
    lib.bi_peer_close.argtypes = [_vp]
    lib.bi_peer_free.restype = ctypes.c_int
    lib.bi_peer_free.argtypes = [_vp]
    lib.bi_peer_barrier.restype = ctypes.c_int
    lib.bi_peer_barrier.argtypes = [ctypes.POINTER(_vp), ctypes.c_int, ctypes.c_int,
                                    ctypes.c_uint32, _vp]
    # (a, lda, b, ldb, bias, out, ldo, stages, cols, M, K, b_is_nk, alpha, beta, dtype,
    #  flags | devices, rank, world, epoch, stream)
    gather = [_vp, _i64, _vp, _i64, _vp, _vp, _i64, ctypes.POINTER(_vp), ctypes.POINTER(_i64),
              _i64, _i64, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_int]
    tail = [ctypes.c_int, ctypes.c_int, ctypes.c_uint32, _vp]
    lib.bi_gemm_allgather.restype = ctypes.c_int
    lib.bi_gemm_allgather.argtypes = gather + [ctypes.POINTER(_vp)] + tail
    lib.bi_gemm_allgather_deferred.restype = ctypes.c_int
    lib.bi_gemm_allgather_deferred.argtypes = gather + [ctypes.POINTER(_vp)] + tail
    lib.bi_gather_unpack.restype = ctypes.c_int
    lib.bi_gather_unpack.argtypes = [_vp, _i64, ctypes.POINTER(_vp), ctypes.POINTER(_i64), _i64,
                                     ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp]
    lib.bi_gemm_allgather_static.restype = ctypes.c_int
    lib.bi_gemm_allgather_static.argtypes = gather + [ctypes.POINTER(ctypes.c_int)] + tail
    lib.bi_rope_kv.restype = ctypes.c_int
    lib.bi_rope_kv.argtypes = [_vp, _i64, _i64, _i64, _i64, _i64, _vp, _vp, _i64, _vp, _i64,
                               _vp, _vp, _vp, _i64_3, ctypes.c_int, _vp]
    lib.bi_swiglu.restype = ctypes.c_int
    lib.bi_swiglu.argtypes = [_vp, _vp, _i64, _i64, ctypes.c_int, _vp]


def lib():
    """The loaded libbi.so; raises if it has not been built."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        "libbi.so is not built (%s); run python mlx-batch-invariant_b200/build.py"
                        % LIB_PATH)
                handle = ctypes.CDLL(LIB_PATH)
                _bind(handle)
                _lib = handle
    return _lib


def _status_string(status):
    try:
        return lib().bi_status_string(status).decode()
    except Exception:  # pragma: no cover - only while loading failed
        return "status"


def check(status, where):
    if status != 0:
        detail = lib().bi_last_error().decode()
        raise LibraryError(status, where, detail)


def dtype_code(dtype):
    try:
        return DTYPE_CODE[dtype]
    except KeyError:
        raise ValueError("unsupported dtype %s (float32, float16 and bfloat16 are built)" % dtype)


def route(dtype, K, N, b_is_nk):
    """(route, BM, BN, BK) the GEMM uses for this (dtype, K, N, layout) -- never M."""
    r, bm, bn, bk = (ctypes.c_int() for _ in range(4))
    check(lib().bi_gemm_route(dtype_code(dtype), K, N, int(bool(b_is_nk)), ctypes.byref(r),
                              ctypes.byref(bm), ctypes.byref(bn), ctypes.byref(bk)),
          "bi_gemm_route")
    return r.value, bm.value, bn.value, bk.value


def device_error(clear=True):
    """The device error word (non-zero if a kernel's bounded wait gave up)."""
    return lib().bi_device_error(1 if clear else 0)


def stream_handle(device):
    return torch.cuda.current_stream(device).cuda_stream


def i64_3(vals):
    return _i64_3(*[int(v) for v in vals])


def i64_2(vals):
    return _i64_2(*[int(v) for v in vals])
