"""The blur's streaming passes (the large-lattice path) and the reduced-precision
lattice values (``PLOO.set_lattice_precision("bf16")``, C ABI
``plattice_set_lattice_precision(16)``).

* Streaming passes in float, forced on for small cases
  (``plattice_debug_set_blur_streaming``): the golden vectors of the reference
  at the parity bar (1e-5 relative + 5e-6 absolute), forward, backward, the
  kept-lattice filter and the feature gradient.
* bfloat16 rows: a tolerance contract of their own, since every pass rounds
  the rows it writes to 8 significant bits: forward output and value
  gradient within 2e-2 of the largest magnitude of the float result (the
  float path is itself pinned to the reference), the normaliser within 2e-2
  relative; lattices that stay in registers are unaffected.
"""
import contextlib
import os

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN, allclose_report

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 5e-6
BF16_TOL = 2e-2


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from plattice_pytorch_b200 import _lib
    _lib.lib()
    return torch.device("cuda:0")


@contextlib.contextmanager
def _mode(streaming=False, precision="fp32"):
    from plattice_pytorch_b200 import PLOO, _lib
    L = _lib.lib()
    try:
        L.plattice_debug_set_blur_streaming(1 if streaming else 0)
        PLOO.set_lattice_precision(precision)
        yield
    finally:
        L.plattice_debug_set_blur_streaming(0)
        PLOO.set_lattice_precision("fp32")


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _fwd_bwd(f, v, g, dev):
    from plattice_pytorch_b200 import PLOO
    ft, vt, gt = _t(f, dev), _t(v, dev), _t(g, dev)
    wo, out, lat = PLOO.lattice_forward(ft, vt)
    grad = PLOO.lattice_backward(ft, gt, wo, lat)
    assert PLOO.lattice_info(lat)["status"] == 0
    return wo.cpu().numpy(), out.cpu().numpy(), grad.cpu().numpy()


# row widths 1, 2, 4, 8 and 12 floats, pd 1 to 16, a ragged shape, a collapsed lattice
STREAM_CASES = ["ref_randn12x10_pd1_vd1.npz", "ref_randn24x20_pd1_vd2.npz", "ref_randn24x20_pd5_vd6.npz",
                "ref_randn24x20_pd7_vd8.npz", "ref_randn24x20_pd16_vd1.npz", "ref_randn24x20_pd15_vd8.npz",
                "ref_ragged13x29_pd5_vd3.npz", "ref_collapse64_pd2_vd8.npz", "ref_blobs64_pd5_vd3.npz"]


@pytest.mark.parametrize("fn", STREAM_CASES)
def test_streaming_passes_match_the_reference(fn, dev):
    d = np.load(os.path.join(GOLDEN, fn))
    with _mode(streaming=True):
        wo, out, grad = _fwd_bwd(d["features"], d["values"], d["grad"], dev)
    assert allclose_report(out, d["out"], RTOL, ATOL) <= 1.0
    assert allclose_report(wo, d["weight"], RTOL, ATOL) <= 1.0
    assert allclose_report(grad, d["grad_out"], RTOL, ATOL) <= 1.0


def test_streaming_passes_in_the_kept_lattice_filter_and_feature_gradient(dev):
    from plattice_pytorch_b200 import PLOO
    d = np.load(os.path.join(GOLDEN, "ref_blobs64_pd5_vd3.npz"))
    ft, vt, gt = _t(d["features"], dev), _t(d["values"], dev), _t(d["grad"], dev)
    wo, out, lat = PLOO.lattice_forward(ft, vt)
    gf_res = PLOO.feature_grad(lat, ft, vt, gt, wo, out).cpu().numpy()
    with _mode(streaming=True):
        w2, o2 = PLOO.lattice_filter(lat, vt)
        gv = PLOO.lattice_filter_backward(lat, gt, w2)
        gf = PLOO.feature_grad(lat, ft, vt, gt, wo, out).cpu().numpy()
    assert allclose_report(o2.cpu().numpy(), d["out"], RTOL, ATOL) <= 1.0
    assert allclose_report(gv.cpu().numpy(), d["grad_out"], RTOL, ATOL) <= 1.0
    ref = oracle.feature_grad(d["features"], d["values"], d["grad"])
    bound = 2e-3 * np.abs(ref) + 1e-4 * float(np.abs(ref).max())
    assert np.all(np.abs(gf - ref) <= bound)
    assert np.all(np.abs(gf - gf_res) <= bound)


def _within_bf16(x, ref):
    return float(np.abs(x - ref).max()) <= BF16_TOL * max(float(np.abs(ref).max()), 1e-30)


@pytest.mark.parametrize("fn", ["ref_randn24x20_pd7_vd8.npz", "ref_randn24x20_pd15_vd8.npz",
                                "ref_randn24x20_pd5_vd6.npz", "ref_randn12x10_pd1_vd1.npz",
                                "ref_blobs64_pd5_vd3.npz"])
def test_bf16_rows_within_their_contract(fn, dev):
    d = np.load(os.path.join(GOLDEN, fn))
    with _mode(streaming=True, precision="bf16"):
        wo, out, grad = _fwd_bwd(d["features"], d["values"], d["grad"], dev)
    assert _within_bf16(out, d["out"])
    assert _within_bf16(grad, d["grad_out"])
    assert np.all(np.abs(wo - d["weight"]) <= BF16_TOL * np.abs(d["weight"]))


def test_bf16_rows_are_used_and_resident_lattices_unaffected(dev):
    d = np.load(os.path.join(GOLDEN, "ref_randn24x20_pd7_vd8.npz"))
    with _mode(streaming=True, precision="bf16"):
        _, out_h, _ = _fwd_bwd(d["features"], d["values"], d["grad"], dev)
    with _mode(streaming=True):
        _, out_f, _ = _fwd_bwd(d["features"], d["values"], d["grad"], dev)
    assert float(np.abs(out_h - out_f).max()) > 0.0          # the rounding is there
    with _mode(precision="bf16"):                               # small lattice: rows stay in registers
        wo, out, grad = _fwd_bwd(d["features"], d["values"], d["grad"], dev)
    assert allclose_report(out, d["out"], RTOL, ATOL) <= 1.0
    assert allclose_report(grad, d["grad_out"], RTOL, ATOL) <= 1.0


def test_bf16_rows_on_a_large_lattice(dev):
    """512^2 pd16 vd8 (4.46 M vertices, the streaming path by size): bf16 rows
    against the float path of the same inputs."""
    from plattice_pytorch_b200 import workloads
    w = workloads.make_workload("gauss512_pd16_vd8", seed=0)
    f, v, g = w["features"], w["values"], w["grad"]
    wo_f, out_f, grad_f = _fwd_bwd(f, v, g, dev)
    with _mode(precision="bf16"):
        wo_h, out_h, grad_h = _fwd_bwd(f, v, g, dev)
    assert _within_bf16(out_h, out_f)
    assert _within_bf16(grad_h, grad_f)
    assert np.all(np.abs(wo_h - wo_f) <= BF16_TOL * np.abs(wo_f))
    assert float(np.abs(out_h - out_f).max()) > 0.0
