"""CPU: the C-ABI library builds for sm_100a, loads, and exports every function include/*.h
declares; argument validation answers before any GPU work."""
import ctypes
import glob
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = []
    for h in sorted(glob.glob(os.path.join(ROOT, "include", "*.h"))):
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        src = re.sub(r"//[^\n]*", "", src)
        for m in re.finditer(r"\b(lncc_[a-z0-9_]+)\s*\(", src):
            names.append(m.group(1))
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    from fused_lncc import _lib
    return _lib.load()


def test_header_declares_entry_points():
    names = declared_functions()
    assert "lncc_fused_forward" in names and "lncc_scale_grad" in names and "lncc_strerror" in names


def test_library_exports_every_declared_symbol(lib):
    from fused_lncc import _lib
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\bT (lncc_\w+)", out))
    for name in declared_functions():
        assert name in exported, name
        assert name in _lib.SIGNATURES, f"ctypes binding misses {name}"
        getattr(lib, name)


def test_library_is_sm100a_only():
    from fused_lncc import _lib
    out = subprocess.run(["cuobjdump", "--list-elf", _lib.LIB_PATH], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("cuobjdump unavailable")
    arches = set(re.findall(r"sm_(\d+a?)", out.stdout))
    assert arches == {"100a"}, arches


def test_strerror_and_version(lib):
    from fused_lncc import _lib
    assert lib.lncc_version() >= 100
    for code in range(0, 9):
        s = _lib.strerror(code)
        assert isinstance(s, str) and s
    assert "unknown" in _lib.strerror(12345)


def test_workspace_bytes(lib):
    assert lib.lncc_workspace_bytes(2, 16, 16, 16, 7, 0, 0, 16) >= 8
    assert lib.lncc_workspace_bytes(2, 16, 16, 16, 4, 0, 0, 16) == 0     # bad k
    assert lib.lncc_workspace_bytes(2, 16, 16, 16, 7, 0, 5, 5) == 0      # empty range
    assert lib.lncc_workspace_bytes(0, 16, 16, 16, 7, 0, 0, 16) == 0     # no volumes


def _call(lib, **kw):
    a = dict(pred=8, target=8, dtype=0, B=1, D=8, H=8, W=8, k=7, dr=1e-5, z0=0, z1=8, grad=None,
             gscale=1.0, gdev=None, csum=None, loss=None, count=1.0, ws=8, wsb=1024, stream=None)
    a.update(kw)
    return lib.lncc_fused_forward(a["pred"], a["target"], a["dtype"], a["B"], a["D"], a["H"], a["W"],
                                  a["k"], a["dr"], a["z0"], a["z1"], a["grad"], a["gscale"], a["gdev"],
                                  a["csum"], a["loss"], a["count"], a["ws"], a["wsb"], a["stream"])


@pytest.mark.parametrize("kw,status", [
    (dict(k=4), 2), (dict(k=11), 2), (dict(k=1), 2),            # lncc3d.cu:123
    (dict(dtype=3), 3), (dict(dtype=-1), 3),                    # lncc3d.cu:158 (2 = fp16 is accepted)
    (dict(pred=None), 1), (dict(B=0), 1), (dict(z0=3, z1=3), 1), (dict(z1=9), 1),
    (dict(pred=2), 1),                                          # misaligned fp32 pointer
])
def test_forward_rejects_bad_arguments_without_gpu(lib, kw, status):
    assert _call(lib, **kw) == status


def test_scale_grad_rejects_bad_arguments(lib):
    assert lib.lncc_scale_grad(None, 0, 10, 8, None) == 1
    assert lib.lncc_scale_grad(8, 7, 10, 8, None) == 3
    assert lib.lncc_scale_grad(8, 0, 0, 8, None) == 0


def test_companion_switch_and_launch_count_validation(lib):
    # the switch is host state: it returns the previous setting
    prev = lib.lncc_set_companion(0)
    try:
        assert lib.lncc_set_companion(1) == 0
        assert lib.lncc_set_companion(0) == 1
    finally:
        lib.lncc_set_companion(prev)
    # lncc_launch_count validates its arguments before asking the device anything; errors come back
    # negated so that they cannot be mistaken for a launch count
    assert lib.lncc_launch_count(1, 8, 8, 8, 4, 0, 0, 8, 1) == -2   # LNCC_ERR_KERNEL_SIZE
    assert lib.lncc_launch_count(1, 8, 8, 8, 7, 5, 0, 8, 1) == -3   # LNCC_ERR_DTYPE
    assert lib.lncc_launch_count(1, 8, 8, 8, 7, 0, 4, 4, 1) == -1   # LNCC_ERR_BAD_ARG (empty plane range)
