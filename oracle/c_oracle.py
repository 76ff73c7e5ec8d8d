"""TEST INFRASTRUCTURE ONLY: ctypes wrapper of the fp64 C oracle (lncc_oracle.c).

Mirrors the reference semantics cited in lncc_oracle.c (reference fused_lncc/csrc/lncc3d.cu:25-110,
166-235, fused_lncc/__init__.py:50-74).
"""
import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liblncc_oracle.so")
_lock = threading.Lock()
_lib = None


def build(force=False):
    """Compile liblncc_oracle.so with the committed Makefile (gcc, OpenMP)."""
    src = os.path.join(_HERE, "lncc_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE, "-B" if force else "all"], check=True)
    return LIB_PATH


def load():
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                build()
                lib = ctypes.CDLL(LIB_PATH)
                i64, vp = ctypes.c_int64, ctypes.c_void_p
                lib.oracle_lncc.restype = ctypes.c_int
                lib.oracle_lncc.argtypes = [vp, vp, i64, i64, i64, i64, ctypes.c_int, ctypes.c_double,
                                            i64, i64, vp, vp, ctypes.c_double, vp, vp, vp, vp,
                                            ctypes.c_int]
                lib.oracle_lncc_win.restype = ctypes.c_int
                lib.oracle_lncc_win.argtypes = [vp, vp, i64, i64, i64, i64, ctypes.c_int, ctypes.c_int,
                                                ctypes.c_int, ctypes.c_double, i64, i64, vp, vp,
                                                ctypes.c_double, vp, vp, vp, vp, ctypes.c_int]
                lib.oracle_box3d.restype = ctypes.c_int
                lib.oracle_box3d.argtypes = [vp, vp, i64, i64, i64, i64, ctypes.c_int]
                lib.oracle_num_threads.restype = ctypes.c_int
                lib.oracle_num_threads.argtypes = []
                _lib = lib
    return _lib


def _f32(a):
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    return a


def lncc(pred, target, kernel_size=7, smooth_dr=1e-5, *, grad=True, z_range=None, grad_scale=None,
         maps=False, direct=True):
    """Oracle loss for (..., D, H, W) arrays (flattened into B volumes).

    Returns dict(loss, cc_sum, count, grad (or None), and with maps=True ncc, A, B, C).
    grad is grad_scale * d(sum cc)/dpred (default -1/M: the gradient of 1 - mean(cc)).
    kernel_size: an odd int (the reference's cubic window) or a (kd, kh, kw) tuple of odd sides.
    """
    if isinstance(kernel_size, (tuple, list)):
        kd, kh, kw = (int(v) for v in kernel_size)
    else:
        kd = kh = kw = int(kernel_size)
    p = _f32(pred)
    t = _f32(target)
    assert p.shape == t.shape and p.ndim >= 3
    *lead, D, H, W = p.shape
    B = int(np.prod(lead)) if lead else 1
    z0, z1 = (0, D) if z_range is None else (int(z_range[0]), int(z_range[1]))
    count = B * (z1 - z0) * H * W
    if grad_scale is None:
        grad_scale = -1.0 / max(count, 1)
    g = np.empty((*lead, z1 - z0, H, W), np.float32) if grad else None
    mp = {}
    if maps:
        for name in ("ncc", "A", "B", "C"):
            mp[name] = np.empty(p.shape, np.float32)
    s = ctypes.c_double(0.0)
    ptr = lambda a: a.ctypes.data_as(ctypes.c_void_p) if a is not None else None
    rc = load().oracle_lncc_win(ptr(p), ptr(t), B, D, H, W, kd, kh, kw, float(smooth_dr), z0, z1,
                            ctypes.cast(ctypes.byref(s), ctypes.c_void_p), ptr(g), float(grad_scale),
                            ptr(mp.get("ncc")), ptr(mp.get("A")), ptr(mp.get("B")), ptr(mp.get("C")),
                            1 if direct else 0)
    if rc != 0:
        raise ValueError(f"oracle_lncc rejected its arguments (rc={rc})")
    out = dict(loss=1.0 - s.value / max(count, 1), cc_sum=s.value, count=count, grad=g)
    out.update(mp)
    return out


def box3d(x, kernel_size):
    """Zero-padded k^3 box sum of fp32 (..., D, H, W) (reference box3d_sep_forward)."""
    a = _f32(x)
    *lead, D, H, W = a.shape
    B = int(np.prod(lead)) if lead else 1
    y = np.empty_like(a)
    rc = load().oracle_box3d(a.ctypes.data_as(ctypes.c_void_p), y.ctypes.data_as(ctypes.c_void_p),
                             B, D, H, W, int(kernel_size))
    if rc != 0:
        raise ValueError("oracle_box3d rejected its arguments")
    return y


def num_threads():
    return int(load().oracle_num_threads())
