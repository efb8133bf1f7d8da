"""TEST INFRASTRUCTURE ONLY: ctypes binding of the C oracle (liboracle_w4a8.so)."""

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle_w4a8.so")
_lib = None


def build():
    """make -C oracle (gcc): the checker is rebuilt when its source is newer."""
    src = os.path.join(HERE, "w4a8_oracle.c")
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        P = ctypes.c_void_p
        i = ctypes.c_int
        L.orc_set_threads.argtypes = [i]
        L.orc_unpack.argtypes = [P, i, i, P]
        L.orc_quant.argtypes = [P, P, ctypes.c_float, i, i, i, P, P]
        L.orc_group_dots.argtypes = [P, i, i, i, i, P, i, P]
        L.orc_gemv.argtypes = [P, P, i, i, i, i, P, P, i, i, i, P]
        L.orc_argmax.argtypes = [P, i, i, P, P]
        L.orc_set_threads(os.cpu_count() or 1)
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return None if a is None else np.ascontiguousarray(a, dtype=dtype)


def set_threads(n):
    lib().orc_set_threads(int(n))


def quant(x, norm_w=None, eps=1e-6, act=0):
    """-> (xq int8 [m, k], xs f32 [m, k/32, 2] (act 0) or [m] (act 1))."""
    x = _c(x, np.float32)
    m, k = x.shape
    nw = _c(norm_w, np.float32)
    xq = np.empty((m, k), np.int8)
    xs = np.empty((m, k // 32, 2) if act == 0 else (m,), np.float32)
    lib().orc_quant(_p(x), _p(nw), ctypes.c_float(eps), m, k, act, _p(xq), _p(xs))
    return xq, xs


def group_dots(q, k, group, has_min, xq):
    q = _c(q, np.uint32)
    xq = _c(xq, np.int8)
    n, m = q.shape[0], xq.shape[0]
    dots = np.empty((m, n, k // group), np.int32)
    lib().orc_group_dots(_p(q), n, k, group, int(has_min), _p(xq), m, _p(dots))
    return dots


def gemv(q, s, k, group, has_min, xq, xs, act, mode=0, y=None):
    """y [m, n_out]; for mode 1 pass the y to add into."""
    q = _c(q, np.uint32)
    s = _c(s, np.uint32 if has_min else np.uint16)
    xq = _c(xq, np.int8)
    xs = _c(xs, np.float32)
    n, m = q.shape[0], xq.shape[0]
    n_out = n // 2 if mode == 2 else n
    out = np.zeros((m, n_out), np.float32) if y is None else np.array(y, dtype=np.float32, copy=True)
    lib().orc_gemv(_p(q), _p(s), n, k, group, int(has_min), _p(xq), _p(xs), act, m, mode, _p(out))
    return out


def argmax(logits, ids=None):
    logits = _c(logits, np.float32)
    m, v = logits.shape
    ids = _c(ids, np.uint32)
    out = np.empty(m, np.uint32)
    lib().orc_argmax(_p(logits), m, v, _p(ids), _p(out))
    return out
