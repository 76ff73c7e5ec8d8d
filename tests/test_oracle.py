"""CPU: the oracles are pinned against golden vectors made by the reference's own PyTorch oracle
(tests/golden/make_golden.py imports reference baselines/torch_lncc.py)."""
import json
import os

import numpy as np
import pytest
import torch

from oracle import c_oracle, torch_port

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLD, "golden.npz")), json.load(open(os.path.join(GOLD, "golden.json")))


def test_golden_files_intact(golden):
    import hashlib
    _, meta = golden
    h = hashlib.sha256(open(os.path.join(GOLD, "golden.npz"), "rb").read()).hexdigest()
    assert h == meta["sha256_npz"]


@pytest.mark.parametrize("direct", [True, False])
def test_c_oracle_matches_reference_golden(golden, direct):
    arr, meta = golden
    for name, c in meta["cases"].items():
        o = c_oracle.lncc(arr[name + "/pred"], arr[name + "/target"], c["k"], direct=direct)
        ref = arr[name + "/grad"]
        assert abs(o["loss"] - c["loss_f64"]) < 1e-12, name
        assert np.linalg.norm(o["grad"] - ref) / np.linalg.norm(ref) < 1e-6, name


def test_torch_port_matches_reference_golden(golden):
    arr, meta = golden
    for name, c in meta["cases"].items():
        p = torch.from_numpy(arr[name + "/pred"]).double()
        t = torch.from_numpy(arr[name + "/target"]).double()
        loss, g = torch_port.loss_and_grad(p, t, c["k"])
        ref = arr[name + "/grad"]
        assert abs(loss - c["loss_f64"]) < 1e-12, name
        assert np.linalg.norm(g.numpy() - ref) / np.linalg.norm(ref) < 1e-10, name
        l32, _ = torch_port.loss_and_grad(p.float(), t.float(), c["k"])
        assert abs(l32 - c["loss_f32"]) < 1e-6, name


def test_config1_construction_and_oracle(golden):
    from fused_lncc import synth
    arr, meta = golden
    c1 = meta["config1"]
    pred, target = synth.blurred_pair((1, 1, 64, 64, 64), device="cpu")
    assert synth.sha256_of(pred) == c1["sha256_pred"]
    assert synth.sha256_of(target) == c1["sha256_target"]
    o = c_oracle.lncc(pred.numpy(), target.numpy(), 7)
    assert abs(o["loss"] - c1["loss_f64"]) < 1e-10
    flat = o["grad"].ravel()
    np.testing.assert_allclose(flat[arr["config1/sample_idx"]], arr["config1/sample_grad"], rtol=1e-5,
                               atol=1e-12)
    assert abs(np.linalg.norm(flat) / c1["grad_l2"] - 1) < 1e-6


def test_oracle_plane_range_is_a_slice():
    rng = np.random.default_rng(3)
    p = rng.standard_normal((2, 11, 6, 7)).astype(np.float32)
    t = rng.standard_normal((2, 11, 6, 7)).astype(np.float32)
    full = c_oracle.lncc(p, t, 5, grad_scale=1.0)
    part = c_oracle.lncc(p, t, 5, z_range=(3, 8), grad_scale=1.0)
    np.testing.assert_array_equal(part["grad"], full["grad"][:, 3:8])


def test_oracle_semantics_degenerate_and_nan():
    z = np.zeros((1, 8, 8, 8), np.float32)
    o = c_oracle.lncc(z, z, 7)
    assert np.isfinite(o["loss"]) and 0.0 <= o["loss"] <= 1.0
    assert np.isfinite(o["grad"]).all()
    c = np.full((1, 8, 8, 8), 1e4, np.float32)
    o = c_oracle.lncc(c, c, 7)
    assert np.isfinite(o["loss"]) and 0.0 <= o["loss"] <= 1.0
    p = np.random.default_rng(0).standard_normal((1, 8, 8, 8)).astype(np.float32)
    p[0, 4, 4, 4] = np.nan
    o = c_oracle.lncc(p, np.ones_like(p), 3)
    assert not np.isfinite(o["loss"])


def test_oracle_box3d_matches_conv():
    x = np.random.default_rng(1).standard_normal((2, 5, 6, 7)).astype(np.float32)
    y = c_oracle.box3d(x, 3)
    ref = torch_port.box_dense(torch.from_numpy(x).double()[None], 3)[0].numpy()
    np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-5)


def test_oracle_rejects_bad_args():
    x = np.zeros((1, 4, 4, 4), np.float32)
    with pytest.raises(ValueError):
        c_oracle.lncc(x, x, 4)
    with pytest.raises(ValueError):
        c_oracle.lncc(x, x, 3, z_range=(2, 2))


@pytest.mark.parametrize("win", [(3, 5, 7), (1, 7, 3), (9, 1, 5)])
def test_oracle_window_matches_conv_port(win):
    """The oracle's non-cubic window path (no reference counterpart) against the PyTorch port's grouped
    conv3d with a kd x kh x kw kernel, in fp64 through autograd; the data keep every variance positive,
    where the port (no variance clamp, as the reference's baseline) and the oracle agree."""
    g = torch.Generator().manual_seed(sum(win))
    p = torch.rand(1, 2, 9, 11, 13, generator=g, dtype=torch.float64)
    t = 0.5 * p + 0.5 * torch.rand(1, 2, 9, 11, 13, generator=g, dtype=torch.float64)
    o = c_oracle.lncc(p.float().numpy(), t.float().numpy(), win)
    # the oracle reads fp32 inputs: compare it with the port on the same fp32-rounded values
    pf = p.float().double().requires_grad_(True)
    lf = torch_port.lncc_dense(pf, t.float().double(), win)
    lf.backward()
    assert abs(o["loss"] - lf.item()) < 1e-10
    ref = pf.grad.numpy()
    assert np.linalg.norm(o["grad"] - ref) / np.linalg.norm(ref) < 1e-6
    # a cubic tuple is the cubic window
    oc = c_oracle.lncc(p.float().numpy(), t.float().numpy(), (5, 5, 5))
    ok = c_oracle.lncc(p.float().numpy(), t.float().numpy(), 5)
    assert abs(oc["loss"] - ok["loss"]) < 1e-12 and np.allclose(oc["grad"], ok["grad"], rtol=1e-6, atol=1e-12)
