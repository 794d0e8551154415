"""The C++ build of PermutoLatticeFunction (csrc/plattice_torch.cpp), which
``PermutoLatticeFunction.apply`` runs when it is built.

Checkers: the golden vectors the reference CUDA build produced (forward output
and value gradient within 1e-5 relative + 5e-6 absolute), and the Python
Function over the same library; a second backward on the same graph (the
kept lattice, re-zeroed) gives the same gradient; the reference's input
messages on CUDA tensors.
"""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, allclose_report

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 5e-6


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from plattice_pytorch_b200 import plattice
    assert plattice._cpp_function() is not None, "the C++ Function extension must be built"
    return torch.device("cuda:0")


def _close(a, b):
    return allclose_report(a.detach().cpu().numpy(), np.asarray(b), RTOL, ATOL) <= 1.0


@pytest.mark.parametrize("name", ["ref_blobs64_pd5_vd3.npz", "ref_randn24x20_pd16_vd1.npz",
                                  "ref_ragged13x29_pd5_vd3.npz", "ref_ragged1x1_pd5_vd3.npz"])
def test_cpp_function_matches_golden_and_python_function(name, dev):
    from plattice_pytorch_b200 import plattice
    d = np.load(os.path.join(GOLDEN, name))
    f = torch.from_numpy(d["features"]).to(dev)
    g = torch.from_numpy(d["grad"]).to(dev)
    v = torch.from_numpy(d["values"]).to(dev).requires_grad_(True)
    out = plattice.PermutoLatticeFunction.apply(f, v)
    assert out.grad_fn is not None and "PermutoLattice" in out.grad_fn.name()
    (gv,) = torch.autograd.grad(out, (v,), (g,), retain_graph=True)
    assert _close(out, d["out"]) and _close(gv, d["grad_out"])
    (gv2,) = torch.autograd.grad(out, (v,), (g,))   # second backward: the kept lattice, rows re-zeroed
    assert _close(gv2, d["grad_out"])
    # the Python Function over the same library
    vp = v.detach().clone().requires_grad_(True)
    outp = torch.autograd.Function.apply.__func__(plattice.PermutoLatticeFunction, f, vp)
    (gvp,) = torch.autograd.grad(outp, (vp,), (g,))
    assert _close(out, outp.detach().cpu().numpy()) and _close(gv, gvp.detach().cpu().numpy())


def test_module_and_messages_on_the_device(dev):
    from plattice_pytorch_b200 import PermutoLattice, plattice
    f = torch.rand(8, 8, 5, device=dev)
    v = torch.rand(8, 9, 3, device=dev)
    with pytest.raises(RuntimeError, match="features and values must have matching H, W"):
        plattice.PermutoLatticeFunction.apply(f, v)
    with pytest.raises(RuntimeError, match="value dimension vd must be in"):
        plattice.PermutoLatticeFunction.apply(f, torch.rand(8, 8, 9, device=dev))
    with pytest.raises(RuntimeError, match="features must be contiguous"):
        plattice.PermutoLatticeFunction.apply(f.transpose(0, 1), torch.rand(8, 8, 3, device=dev))
    vv = torch.rand(8, 8, 3, device=dev, requires_grad=True)
    out = PermutoLattice()(f, vv)
    out.sum().backward()
    assert vv.grad is not None and torch.isfinite(vv.grad).all()
    assert f.grad is None
