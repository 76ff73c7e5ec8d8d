"""ctypes binding of liblncc_sm100.so (declared in include/lncc.h).

This is the extension loader. The reference imports a prebuilt pybind module or JIT-builds one
(reference fused_lncc/__init__.py:10-19). Here the library is a plain C ABI, so any FFI can bind
it. If it is missing and nvcc is present it is compiled in-tree once. If that fails, the import
error propagates. There is no CPU or PyTorch fallback.
"""
import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liblncc_sm100.so")

LNCC_OK = 0
LNCC_ERR_WORKSPACE = 6
LNCC_F32 = 0
LNCC_BF16 = 1
LNCC_F16 = 2

_c_i64 = ctypes.c_int64
_vp = ctypes.c_void_p

# name -> (restype, argtypes); must list every function of include/lncc.h
SIGNATURES = {
    "lncc_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "lncc_version": (ctypes.c_int, []),
    "lncc_workspace_bytes": (ctypes.c_size_t, [_c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int, ctypes.c_int,
                                               _c_i64, _c_i64]),
    "lncc_fused_forward": (ctypes.c_int, [
        _vp, _vp, ctypes.c_int,                      # pred, target, dtype
        _c_i64, _c_i64, _c_i64, _c_i64,              # B, D, H, W
        ctypes.c_int, ctypes.c_float,                # kernel_size, smooth_dr
        _c_i64, _c_i64,                              # z_begin, z_end
        _vp, ctypes.c_float, _vp,                    # grad, grad_scale, grad_scale_dev
        _vp, _vp, ctypes.c_double,                   # cc_sum_out, loss_out, loss_count
        _vp, ctypes.c_size_t, _vp,                   # workspace, bytes, stream
    ]),
    "lncc_scale_grad": (ctypes.c_int, [_vp, ctypes.c_int, _c_i64, _vp, _vp]),
    "lncc_check_abort": (ctypes.c_int, [_vp, _vp]),
    "lncc_peer_exchange_bytes": (ctypes.c_size_t, [ctypes.c_int]),
    "lncc_peer_loss": (ctypes.c_int, [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_uint64, ctypes.c_double,
                                      _vp, _vp, _vp, _vp]),
    "lncc_checked_build": (ctypes.c_int, []),
    "lncc_wait_timeout_selftest": (ctypes.c_int, [_vp, ctypes.c_size_t, ctypes.c_uint, _vp]),
    "lncc_select_kernel": (ctypes.c_int, [ctypes.c_int]),
    "lncc_set_companion": (ctypes.c_int, [ctypes.c_int]),
    "lncc_launch_count": (ctypes.c_int, [_c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int, ctypes.c_int, _c_i64,
                                         _c_i64, ctypes.c_int]),
    "lncc_fused_forward_noalloc": (ctypes.c_int, [
        _vp, _vp, ctypes.c_int,                      # pred, target, dtype
        _c_i64, _c_i64, _c_i64, _c_i64,              # B, D, H, W
        ctypes.c_int, ctypes.c_float,                # kernel_size, smooth_dr
        _c_i64, _c_i64,                              # z_begin, z_end
        _vp, ctypes.c_float, _vp,                    # grad, grad_scale, grad_scale_dev
        _vp, _vp, ctypes.c_double,                   # cc_sum_out, loss_out, loss_count
        _vp,                                         # stream
    ]),
    "lncc_loss_map_scratch_bytes": (ctypes.c_size_t, [_c_i64, _c_i64, _c_i64, _c_i64]),
    "lncc_loss_map_forward": (ctypes.c_int, [
        _vp, _vp, ctypes.c_int,                      # pred, target, dtype
        _c_i64, _c_i64, _c_i64, _c_i64,              # B, D, H, W
        ctypes.c_int, ctypes.c_float,                # kernel_size, smooth_dr
        _vp, _vp,                                    # loss_map, stream
    ]),
    "lncc_loss_map_backward": (ctypes.c_int, [
        _vp, _vp, _vp, ctypes.c_int,                 # grad_map, pred, target, dtype
        _c_i64, _c_i64, _c_i64, _c_i64,              # B, D, H, W
        ctypes.c_int, ctypes.c_float,                # kernel_size, smooth_dr
        _vp, _vp, ctypes.c_size_t, _vp,              # grad, scratch, scratch_bytes, stream
    ]),
    "lncc_maps_forward": (ctypes.c_int, [
        _vp, _vp, ctypes.c_int,                      # pred, target, dtype
        _c_i64, _c_i64, _c_i64, _c_i64,              # B, D, H, W
        ctypes.c_int, ctypes.c_float,                # kernel_size, smooth_dr
        _vp, _vp, _vp, _vp, _vp,                     # ncc, A, Bc, Cc, stream
    ]),
    "lncc_maps_backward": (ctypes.c_int, [
        _vp, _vp, _vp, _vp, _vp, ctypes.c_int,       # A, Bc, Cc, pred, target, dtype
        _c_i64, _c_i64, _c_i64, _c_i64,              # B, D, H, W
        ctypes.c_int, ctypes.c_float, _vp, _vp,      # kernel_size, scale, grad, stream
    ]),
    "lncc_box3d": (ctypes.c_int, [_vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int, _vp]),
    "lncc_aniso_scratch_bytes": (ctypes.c_size_t, [_c_i64, _c_i64, _c_i64, _c_i64, ctypes.c_int]),
    "lncc_aniso_forward": (ctypes.c_int, [
        _vp, _vp, ctypes.c_int,                      # pred, target, dtype
        _c_i64, _c_i64, _c_i64, _c_i64,              # B, D, H, W
        ctypes.c_int, ctypes.c_int, ctypes.c_int,    # kd, kh, kw
        ctypes.c_float,                              # smooth_dr
        _vp, ctypes.c_float, _vp,                    # grad, grad_scale, grad_scale_dev
        _vp, _vp, ctypes.c_double,                   # cc_sum_out, loss_out, loss_count
        _vp, ctypes.c_size_t, _vp,                   # scratch, bytes, stream
    ]),
    "lncc_aniso_loss_map_forward": (ctypes.c_int, [
        _vp, _vp, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_i64,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, _vp, _vp,
    ]),
    "lncc_aniso_loss_map_backward": (ctypes.c_int, [
        _vp, _vp, _vp, ctypes.c_int, _c_i64, _c_i64, _c_i64, _c_i64,
        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, _vp, _vp, ctypes.c_size_t, _vp,
    ]),
}

_lock = threading.Lock()
_lib = None


def _build_if_missing():
    if os.path.exists(LIB_PATH):
        return
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "_lncc_build", os.path.join(os.path.dirname(_HERE), "build.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.build_library()


def load():
    """Load (building once if absent) and return the ctypes library handle."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            _build_if_missing()
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def strerror(status):
    return load().lncc_strerror(int(status)).decode()


def check(status, what):
    if status != LNCC_OK:
        raise RuntimeError(f"{what}: {strerror(status)} (status {status})")


KERNEL_AUTO, KERNEL_SWEEP, KERNEL_WS = 0, 1, 3


def select_kernel(which):
    """Process-wide kernel choice: 0 auto (warp-specialised cluster kernel where it applies, else the
    general sweep kernel), 1 general sweep kernel, 3 warp-specialised cluster kernel where supported.
    2 (an earlier cluster kernel, since retired) is rejected."""
    check(load().lncc_select_kernel(int(which)), "lncc_select_kernel")


def set_companion(enable):
    """Process-wide switch of the warp-specialised kernel's companion launch (clusters of 2 CTAs on
    the SMs that clusters of 8 leave idle, for the last volumes of a call); returns the previous
    setting."""
    return bool(load().lncc_set_companion(1 if enable else 0))
