"""Generate the golden vectors in tests/golden/ from the REFERENCE's own PyTorch oracle.

Run in a container where the reference checkout is mounted (it is read, never modified):
    python tests/golden/make_golden.py --reference /path/to/fused-lncc

It imports the reference's baselines/torch_lncc.py (`lncc_dense`, `lncc_separable`), evaluates it in
float64 on CPU (and in fp32 for config 1), and writes:
  golden.npz     small seeded inputs with the reference loss and full dL/dpred
  golden.json    config-1 (1,1,64,64,64) k=7 loss values + gradient fingerprints, input SHA-256s
The GPU box has no reference checkout; the tests read only these committed files.
"""
import argparse
import hashlib
import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "fused-lncc_b200"))
from fused_lncc import synth  # noqa: E402  (input constructions only; no CUDA needed)

# (name, shape, k, generator)  - small enough for exact float64 storage
RAND_CASES = [
    ("randn_k3", (1, 2, 9, 10, 11), 3),
    ("randn_k5", (1, 2, 9, 10, 11), 5),
    ("randn_k7", (1, 2, 9, 10, 11), 7),
    ("randn_k9", (1, 2, 9, 10, 11), 9),
    ("edge_2cube_k7", (1, 1, 2, 2, 2), 7),
    ("edge_7x9x11_k7", (1, 3, 7, 9, 11), 7),
    ("edge_line_k7", (1, 1, 16, 1, 1), 7),
    ("edge_5x3x4_k3", (2, 1, 5, 3, 4), 3),
    ("edge_13x17x19_k5", (1, 2, 13, 17, 19), 5),
    ("uniform_k5", (1, 1, 12, 12, 12), 5),
]


def load_reference(ref_root):
    path = os.path.join(ref_root, "baselines", "torch_lncc.py")
    spec = importlib.util.spec_from_file_location("ref_torch_lncc", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def ref_loss_grad(ref, p, t, k, fn="lncc_dense"):
    pp = p.clone().requires_grad_(True)
    loss = getattr(ref, fn)(pp, t, k, 1e-5)
    loss.backward()
    return float(loss.item()), pp.grad.detach()


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    ap = argparse.ArgumentParser()
    # default: a checkout named "reference" beside this repository
    sibling = os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(HERE))), "reference")
    ap.add_argument("--reference", default=os.environ.get("LNCC_REFERENCE_ROOT", sibling))
    args = ap.parse_args()
    ref = load_reference(args.reference)
    torch.set_num_threads(os.cpu_count() or 1)

    arrays = {}
    meta = {"generator": "tests/golden/make_golden.py", "reference_oracle": "baselines/torch_lncc.py",
            "smooth_dr": 1e-5, "cases": {}}
    for i, (name, shape, k) in enumerate(RAND_CASES):
        g = torch.Generator().manual_seed(1000 + i)
        if name.startswith("uniform"):
            p = torch.rand(shape, generator=g)
            t = torch.rand(shape, generator=g)
        else:
            p = torch.randn(shape, generator=g)
            t = torch.randn(shape, generator=g)
        loss64, grad64 = ref_loss_grad(ref, p.double(), t.double(), k)
        loss32, _ = ref_loss_grad(ref, p, t, k)
        arrays[f"{name}/pred"] = p.numpy()
        arrays[f"{name}/target"] = t.numpy()
        arrays[f"{name}/grad"] = grad64.numpy()
        meta["cases"][name] = {"shape": list(shape), "k": k, "loss_f64": loss64, "loss_f32": loss32,
                               "sha256_pred": sha(p.numpy()), "sha256_target": sha(t.numpy())}

    # config 1 of the benchmark: (1,1,64,64,64) fp32 k=7, blurred-noise construction (seeds 0/1)
    pred, target = synth.blurred_pair((1, 1, 64, 64, 64), device="cpu")
    l64, g64 = ref_loss_grad(ref, pred.double(), target.double(), 7)
    l32, g32 = ref_loss_grad(ref, pred, target, 7)
    ls32, _ = ref_loss_grad(ref, pred, target, 7, fn="lncc_separable")
    rng = np.random.default_rng(7)
    idx = rng.choice(g64.numel(), size=512, replace=False)
    flat = g64.flatten().numpy()
    meta["config1"] = {
        "shape": [1, 1, 64, 64, 64], "k": 7,
        "loss_f64": l64, "loss_f32_dense": l32, "loss_f32_separable": ls32,
        "grad_l2": float(np.linalg.norm(flat)), "grad_sum": float(flat.sum()),
        "grad_abs_sum": float(np.abs(flat).sum()),
        "sha256_pred": sha(pred.numpy()), "sha256_target": sha(target.numpy()),
    }
    arrays["config1/sample_idx"] = idx.astype(np.int64)
    arrays["config1/sample_grad"] = flat[idx]

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **arrays)
    meta["sha256_npz"] = hashlib.sha256(open(os.path.join(HERE, "golden.npz"), "rb").read()).hexdigest()
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    print(json.dumps(meta["config1"], indent=1))


if __name__ == "__main__":
    main()
