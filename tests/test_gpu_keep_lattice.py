"""PLOO.set_keep_lattice(False): the forward keeps nothing for the backward and
the backward rebuilds the lattice from the saved features, as the reference
does (plattice.py:11-19, permutohedral.cu:615-635).

Checkers: the golden vectors the reference CUDA build produced (forward output
and value gradient within 1e-5 relative + 5e-6 absolute), through the C++
Function, the Python Function and PLOO.forward / PLOO.backward; and the device
memory a forward leaves allocated besides its outputs, measured with PyTorch's
allocator counters: nothing with the switch off, the lattice buffer with it on.
"""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, allclose_report

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 5e-6
GOLDENS = ["ref_blobs64_pd5_vd3.npz", "ref_randn24x20_pd16_vd1.npz", "ref_ragged13x29_pd5_vd3.npz"]


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from plattice_pytorch_b200 import _lib
    _lib.lib()
    return torch.device("cuda:0")


@pytest.fixture
def no_keep():
    from plattice_pytorch_b200 import PLOO
    prev = PLOO.get_keep_lattice()
    PLOO.set_keep_lattice(False)
    yield
    PLOO.set_keep_lattice(prev)


def _close(a, b):
    return allclose_report(a.detach().cpu().numpy(), np.asarray(b), RTOL, ATOL) <= 1.0


def _python_apply(f, v):
    from plattice_pytorch_b200 import plattice
    return torch.autograd.Function.apply.__func__(plattice.PermutoLatticeFunction, f, v)


@pytest.mark.parametrize("name", GOLDENS)
def test_rebuilding_backward_matches_golden(name, dev, no_keep):
    from plattice_pytorch_b200 import PLOO, plattice
    d = np.load(os.path.join(GOLDEN, name))
    f = torch.from_numpy(d["features"]).to(dev)
    g = torch.from_numpy(d["grad"]).to(dev)
    for apply in (plattice.PermutoLatticeFunction.apply, _python_apply):
        v = torch.from_numpy(d["values"]).to(dev).requires_grad_(True)
        out = apply(f, v)
        (gv,) = torch.autograd.grad(out, (v,), (g,), retain_graph=True)
        assert _close(out, d["out"]) and _close(gv, d["grad_out"])
        (gv2,) = torch.autograd.grad(out, (v,), (g,))   # a second backward rebuilds again
        assert _close(gv2, d["grad_out"])
    weight, out = PLOO.forward(f, torch.from_numpy(d["values"]).to(dev))
    assert PLOO._last is None
    gv = PLOO.backward(f, g, weight)
    assert _close(out, d["out"]) and _close(gv, d["grad_out"])


def test_switch_checks_its_argument():
    from plattice_pytorch_b200 import PLOO
    with pytest.raises(RuntimeError):
        PLOO.set_keep_lattice(0)


@pytest.mark.parametrize("keep", [True, False])
def test_retained_bytes_after_forward(keep, dev):
    from plattice_pytorch_b200 import PLOO, _lib, plattice
    from plattice_pytorch_b200.workloads import make_workload
    w = make_workload("crf512_pd5_vd3")
    f = torch.from_numpy(w["features"]).to(dev)
    h, wd, pd = f.shape
    vd = w["values"].shape[2]
    lb, _ = _lib.workspace_sizes(h, wd, pd, vd)
    prev = PLOO.get_keep_lattice()
    PLOO.set_keep_lattice(keep)
    try:
        for apply in (plattice.PermutoLatticeFunction.apply, _python_apply):
            v = torch.from_numpy(w["values"]).to(dev).requires_grad_(True)
            g = torch.from_numpy(w["grad"]).to(dev)
            torch.cuda.synchronize()
            base = torch.cuda.memory_allocated(dev)
            out = apply(f, v)
            torch.cuda.synchronize()
            outputs = h * wd * (vd + 1) * 4   # out and the saved weight
            retained = torch.cuda.memory_allocated(dev) - base - outputs
            if keep:
                assert lb <= retained <= lb + 2 * (1 << 20)
            else:
                assert retained <= 64 * 1024
            (gv,) = torch.autograd.grad(out, (v,), (g,))
            assert np.isfinite(gv.cpu().numpy()).all()
            del out, gv
    finally:
        PLOO.set_keep_lattice(prev)
