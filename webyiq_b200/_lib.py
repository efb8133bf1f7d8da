"""ctypes binding of the C ABI (include/w4a8.h).  Loading fails loudly when the
CUDA library has not been built: there is no fallback path."""

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libwebyiq_w4a8.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "w4a8.h")

OK, EINVAL, ECUDA, ENCCL, ETIMEOUT, ENOTSUP = range(6)
STATUS_NAMES = {0: "OK", 1: "EINVAL", 2: "ECUDA", 3: "ENCCL", 4: "ETIMEOUT", 5: "ENOTSUP"}
ACT_GROUP32, ACT_TOKEN = 0, 1
STORE, ADD, SWIGLU = 0, 1, 2
GEMV_MAX_M = 16


class W4A8Error(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


class Weight(ctypes.Structure):
    """struct w4a8_weight"""

    _fields_ = [("q", ctypes.c_void_p), ("s", ctypes.c_void_p), ("n", ctypes.c_int32), ("k", ctypes.c_int32),
                ("group", ctypes.c_int32), ("has_min", ctypes.c_int32)]


_P = ctypes.c_void_p
_I = ctypes.c_int32
_SIGS = {
    "w4a8_weight_view": (ctypes.c_int, [_P, _P, _I, _I, _I, _I, ctypes.POINTER(Weight)]),
    "w4a8_quant": (ctypes.c_int, [_P, _P, ctypes.c_float, _I, _I, _I, _P, _P, _P]),
    "w4a8_gemv": (ctypes.c_int, [ctypes.POINTER(Weight), _P, _P, _I, _I, _I, _P, _P]),
    "w4a8_gemm": (ctypes.c_int, [ctypes.POINTER(Weight), _P, _P, _I, _I, _I, _P, _P]),
    "w4a8_gemv_x": (ctypes.c_int, [ctypes.POINTER(Weight), _P, _I, _I, _P, _P]),
    "w4a8_gemv_xn": (ctypes.c_int, [ctypes.POINTER(Weight), _P, _P, ctypes.c_float, _I, _I, _P, _P]),
    "w4a8_matmul": (ctypes.c_int, [ctypes.POINTER(Weight), _P, _P, _I, _I, _I, _P, _P]),
    "w4a8_argmax": (ctypes.c_int, [_P, _I, _I, _P, _P, _P]),
    "w4a8_lmhead_argmax": (ctypes.c_int, [ctypes.POINTER(Weight), _I, _P, _P, _I, _I, _P, _P, _P, _P, _P,
                                          ctypes.c_size_t, _P]),
    "w4a8_lmhead_workspace_bytes": (ctypes.c_size_t, [_I, _I]),
    "w4a8_lmhead_argmax_noalloc": (ctypes.c_int, [ctypes.POINTER(Weight), _I, _P, _P, _I, _I, _P, _P, _P, _P, _P]),
    "w4a8_group_dots": (ctypes.c_int, [ctypes.POINTER(Weight), _P, _I, _P, _P]),
    "w4a8_lmhead_argmax_allreduce": (ctypes.c_int, [ctypes.POINTER(Weight), _I, _P, _P, _I, _I, _P, _P, _P, _P, _P,
                                                    ctypes.c_size_t, _P, _P]),
    "w4a8_xchg_create": (ctypes.c_int, [_I, _I, _P, ctypes.POINTER(ctypes.c_void_p)]),
    "w4a8_xchg_open": (ctypes.c_int, [_P, _P]),
    "w4a8_xchg_destroy": (ctypes.c_int, [_P]),
    "w4a8_lmhead_argmax_xchg": (ctypes.c_int, [ctypes.POINTER(Weight), _I, _P, _P, _I, _I, _P, _P, _P, _P, _P,
                                               ctypes.c_size_t, _P, _P]),
    "w4a8_gather_rows": (ctypes.c_int, [ctypes.POINTER(Weight), _P, _I, _P, _P, _P]),
    "w4a8_spec_accept": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P]),
    "w4a8_attn_decode": (ctypes.c_int, [_P, _P, _P, _I, _I, _I, _I, _P, _I, _I, _P, _P]),
    "w4a8_attn_combine": (ctypes.c_int, [_P, _I, _I, _I, _I, _P, _I, _P, _P, _P, _P, _P]),
    "w4a8_deltanet": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, ctypes.c_float, _I, _P]),
    "w4a8_nccl_get_unique_id": (ctypes.c_int, [_P]),
    "w4a8_nccl_comm_init": (ctypes.c_int, [_I, _P, _I, ctypes.POINTER(ctypes.c_void_p)]),
    "w4a8_nccl_comm_destroy": (ctypes.c_int, [_P]),
    "w4a8_set_pdl": (None, [ctypes.c_int]),
    "w4a8_set_gemv_kernel": (None, [ctypes.c_int]),
    "w4a8_set_gemm_kernel": (None, [ctypes.c_int]),
    "w4a8_gemm_group_dots": (ctypes.c_int, [ctypes.POINTER(Weight), _P, _I, _P, _P]),
    "w4a8_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint32), _P]),
    "w4a8_selftest_wait_timeout": (ctypes.c_int, [_P]),
    "w4a8_last_error": (ctypes.c_char_p, []),
    "w4a8_version": (ctypes.c_char_p, []),
}

_lib = None


def header_symbols():
    """Names of the functions include/w4a8.h declares with W4A8_API."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"W4A8_API\s+[\w\s\*]+?\b(w4a8_\w+)\s*\(", text)))


def load(path=None):
    """Load the CUDA library (once).  Raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or os.environ.get("WEBYIQ_W4A8_LIB") or LIB_PATH
    if not os.path.exists(path):
        raise RuntimeError(f"webyiq_b200 CUDA library not built ({path}); run `python -m webyiq_b200.build`")
    L = ctypes.CDLL(path)
    for name, (res, args) in _SIGS.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def check(status):
    if status != OK:
        raise W4A8Error(status, load().w4a8_last_error().decode())
