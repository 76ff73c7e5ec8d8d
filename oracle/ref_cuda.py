"""TEST INFRASTRUCTURE ONLY: the reference's own CUDA extension, built from its sources, as a GPU oracle.

The reference ships one CUDA file, `fused_lncc/csrc/lncc3d.cu`, bound with pybind11 as the module
`fused_lncc_cuda` (lncc3d.cu:346-350). On a GPU it would JIT-compile that file with
`torch.utils.cpp_extension.load(..., extra_cuda_cflags=["-O3"])` for the running GPU's arch
(reference fused_lncc/__init__.py:10-19). `build()` does the same, with the B200 arch pinned
(TORCH_CUDA_ARCH_LIST=10.0, since the build machine has no GPU to detect), compiling the source where it
lies in the reference checkout and writing only into `oracle/_ref/`. Nothing is copied into this repository.

`loss_and_grad()` repeats the reference's autograd glue around the extension
(fused_lncc/__init__.py:50-74): forward gives the ncc map and the three adjoint maps, the loss is
`1 - ncc.mean()`, and the backward kernel is called with scale 1 and then multiplied by `-1/M`.

Used by the GPU parity tests at full sizes (where the CPU oracle would take minutes) and by their
speed comparison. The product never imports this module.
"""
import importlib.machinery
import importlib.util
import os

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
NAME = "fused_lncc_cuda"
# the reference checkout on the build machine (default: a directory "reference" beside this
# repository); the GPU machines only get the built module
REF_ROOT = os.environ.get("LNCC_REFERENCE_ROOT",
                          os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))
REF_SRC = os.path.join(REF_ROOT, "fused_lncc", "csrc", "lncc3d.cu")


def built_path():
    """Path of the built extension module, or None."""
    if not os.path.isdir(OUT_DIR):
        return None
    for f in sorted(os.listdir(OUT_DIR)):
        if f.startswith(NAME) and f.endswith(".so"):
            return os.path.join(OUT_DIR, f)
    return None


def build(force=False, verbose=False):
    """Compile the reference extension into oracle/_ref/. Returns the module path, or None when the
    reference sources are not on this machine."""
    if not os.path.isfile(REF_SRC):
        return built_path()
    so = built_path()
    if so and not force and os.path.getmtime(so) >= os.path.getmtime(REF_SRC):
        return so
    os.makedirs(OUT_DIR, exist_ok=True)
    old = os.environ.get("TORCH_CUDA_ARCH_LIST")
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0"
    try:
        from torch.utils.cpp_extension import load
        load(name=NAME, sources=[REF_SRC], extra_cuda_cflags=["-O3"], build_directory=OUT_DIR,
             verbose=verbose)
    finally:
        if old is None:
            os.environ.pop("TORCH_CUDA_ARCH_LIST", None)
        else:
            os.environ["TORCH_CUDA_ARCH_LIST"] = old
    return built_path()


_MOD = None


def load():
    """Import the built extension (torch must be importable). Returns the module or None."""
    global _MOD
    if _MOD is not None:
        return _MOD
    so = built_path()
    if so is None:
        return None
    import torch  # noqa: F401  (the extension links against torch's libraries)
    loader = importlib.machinery.ExtensionFileLoader(NAME, so)
    spec = importlib.util.spec_from_loader(NAME, loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    _MOD = mod
    return mod


def forward_maps(pred, target, kernel_size=7, smooth_dr=1e-5):
    """(ncc, A, Bc, Cc) fp32 maps of shape (N*C, D, H, W) from the reference forward kernel."""
    ext = load()
    if ext is None:
        raise RuntimeError("reference extension not built (oracle/_ref)")
    N, C = pred.shape[:2]
    S = pred.shape[2:]
    pf = pred.reshape(N * C, *S).contiguous()
    tf = target.reshape(N * C, *S).contiguous()
    return [t.contiguous() for t in ext.lncc_forward(pf, tf, kernel_size, smooth_dr)]


def loss_and_grad(pred, target, kernel_size=7, smooth_dr=1e-5):
    """Loss (0-dim fp32) and dL/dpred (pred's shape and dtype), computed as the reference's
    _FusedLNCC does for grad_out = 1 (fused_lncc/__init__.py:50-74)."""
    ext = load()
    if ext is None:
        raise RuntimeError("reference extension not built (oracle/_ref)")
    N, C = pred.shape[:2]
    S = pred.shape[2:]
    pf = pred.reshape(N * C, *S).contiguous()
    tf = target.reshape(N * C, *S).contiguous()
    ncc, A, Bc, Cc = [t.contiguous() for t in ext.lncc_forward(pf, tf, kernel_size, smooth_dr)]
    loss = 1.0 - ncc.mean()
    M = ncc.numel()
    g = ext.lncc_backward(A, Bc, Cc, pf, tf, kernel_size, 1.0).contiguous() * (-1.0 / M)
    return loss, g.reshape(pred.shape).to(pred.dtype)


def box3d(x, kernel_size):
    """The reference's separable zero-padded box sum of an fp32 (B, D, H, W) tensor
    (lncc3d.cu:287-344)."""
    ext = load()
    if ext is None:
        raise RuntimeError("reference extension not built (oracle/_ref)")
    return ext.box3d_sep_forward(x.contiguous(), kernel_size)
