"""Gradient of the filter with respect to the features (``PLOO.feature_grad``,
C ABI ``plattice_feature_grad``, ``PermutoLatticeFeatureFunction``).

The reference has no feature gradient (its Function returns None for the
features, plattice.py:19), so the checker is the oracle's analytic gradient
(oracle.feature_grad, double-precision lattice sweeps), itself pinned to
finite differences of the oracle's forward in tests/test_oracle.py.
Tolerance: |gpu - oracle| <= 2e-3 |oracle| + 1e-4 max|oracle| (the GPU sums
in float, in another order, and the slice term is a difference of nearly
equal products).
"""
import os

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from plattice_pytorch_b200 import _lib
    _lib.lib()
    return torch.device("cuda:0")


def _within(gpu, ref):
    err = np.abs(gpu - ref)
    bound = 2e-3 * np.abs(ref) + 1e-4 * max(float(np.abs(ref).max()), 1e-12)
    return float(np.max(err - bound)) <= 0.0


def _dense(pd, vd, h=24, w=20, seed=0, spread=0.6):
    rng = np.random.default_rng(seed)
    f = (rng.normal(size=(h, w, pd)) * spread).astype(np.float32)
    v = rng.uniform(0.1, 1.0, size=(h, w, vd)).astype(np.float32)
    g = rng.normal(size=(h, w, vd)).astype(np.float32)
    return f, v, g


CASES = [(2, 3), (3, 1), (5, 3), (5, 8), (8, 2), (12, 4), (16, 1)]


@pytest.mark.parametrize("pd,vd", CASES)
def test_feature_grad_equals_the_oracle(pd, vd, dev):
    from plattice_pytorch_b200 import PLOO
    f, v, g = _dense(pd, vd, seed=pd * 10 + vd)
    ft, vt, gt = (torch.from_numpy(a).to(dev) for a in (f, v, g))
    wo, out, lat = PLOO.lattice_forward(ft, vt)
    gf = PLOO.feature_grad(lat, ft, vt, gt, wo, out).cpu().numpy()
    ref = oracle.feature_grad(f, v, g)
    assert np.mean(np.abs(ref) > 1e-4) > 0.3   # the lattice is dense enough for non-zero slopes
    assert _within(gf, ref)
    assert PLOO.lattice_info(lat)["status"] == 0


def test_feature_grad_on_an_image(dev):
    """The reference-style bilateral features of a natural-looking image."""
    from plattice_pytorch_b200 import PLOO
    d = np.load(os.path.join(GOLDEN, "ref_blobs64_pd5_vd3.npz"))
    f, v, g = d["features"], d["values"], d["grad"]
    ft, vt, gt = (torch.from_numpy(a).to(dev) for a in (f, v, g))
    wo, out, lat = PLOO.lattice_forward(ft, vt)
    gf = PLOO.feature_grad(lat, ft, vt, gt, wo, out).cpu().numpy()
    assert _within(gf, oracle.feature_grad(f, v, g))


def test_autograd_gives_both_gradients(dev):
    from plattice_pytorch_b200 import PLOO, PermutoLatticeFeatureFunction, PermutoLatticeFunction
    f, v, g = _dense(5, 3, seed=4)
    ft = torch.from_numpy(f).to(dev).requires_grad_(True)
    vt = torch.from_numpy(v).to(dev).requires_grad_(True)
    gt = torch.from_numpy(g).to(dev)
    out = PermutoLatticeFeatureFunction.apply(ft, vt)
    gfe, gva = torch.autograd.grad(out, (ft, vt), (gt,))
    v2 = torch.from_numpy(v).to(dev).requires_grad_(True)
    out2 = PermutoLatticeFunction.apply(ft.detach(), v2)
    (gva2,) = torch.autograd.grad(out2, (v2,), (gt,))
    torch.cuda.synchronize()
    assert torch.allclose(out, out2, rtol=1e-5, atol=5e-6)
    assert torch.allclose(gva, gva2, rtol=1e-5, atol=5e-6)
    assert _within(gfe.cpu().numpy(), oracle.feature_grad(f, v, g))


def test_feature_grad_checks_its_lattice(dev):
    from plattice_pytorch_b200 import PLOO
    f, v, g = _dense(5, 3, seed=1)
    ft, vt, gt = (torch.from_numpy(a).to(dev) for a in (f, v, g))
    wo, out, lat = PLOO.lattice_forward(ft, vt)
    with pytest.raises(RuntimeError, match="not built from these features"):
        PLOO.feature_grad(lat, ft.clone(), vt, gt, wo, out)
