"""Parity of the sm_100a filter (through the C ABI) with the reference.

Three checkers, all test infrastructure:
  * golden vectors produced by the reference CUDA build (tests/golden/ref_*.npz);
  * the reference CUDA build itself, run here on the full-size workloads
    (oracle/_ref, skipped when it was not built);
  * the CPU oracle (oracle/plattice_oracle.c).
Bar: the sorted vertex key set and the vertex count are identical; forward
output, normaliser and value gradient within 1e-5 relative + 5e-6 absolute
(atomic summation order differs).
"""
import os

import numpy as np
import pytest
import torch

import oracle
from oracle import ref as oref
from conftest import GOLDEN, allclose_report, golden_files

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 5e-6


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from plattice_pytorch_b200 import _lib
    _lib.lib()   # the CUDA library must load: no fallback
    return torch.device("cuda:0")


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _run_ours(f, v, g, dev):
    from plattice_pytorch_b200 import PLOO
    ft, vt, gt = _t(f, dev), _t(v, dev), _t(g, dev)
    wo, out, lat = PLOO.lattice_forward(ft, vt, keep_scratch=True)
    info = PLOO.lattice_info(lat)
    assert info["status"] == 0, info
    keys = PLOO.vertex_keys(lat).cpu().numpy()
    grad = PLOO.lattice_backward(ft, gt, wo, lat)
    info = PLOO.lattice_info(lat)
    assert info["status"] == 0, info
    return {"weight": wo.cpu().numpy(), "out": out.cpu().numpy(), "grad_out": grad.cpu().numpy(),
            "vertex_keys": oref.sort_keys(keys), "m": info["m"], "ft": ft, "gt": gt, "wo": wo}


@pytest.mark.parametrize("fn", golden_files())
def test_golden(fn, dev):
    d = np.load(os.path.join(GOLDEN, fn))
    r = _run_ours(d["features"], d["values"], d["grad"], dev)
    assert r["m"] == int(d["m"])
    assert np.array_equal(r["vertex_keys"], d["vertex_keys"])
    assert allclose_report(r["out"], d["out"], RTOL, ATOL) <= 1.0
    assert allclose_report(r["weight"], d["weight"], RTOL, ATOL) <= 1.0
    assert allclose_report(r["grad_out"], d["grad_out"], RTOL, ATOL) <= 1.0


@pytest.mark.parametrize("fn", ["ref_blobs64_pd5_vd3.npz", "ref_randn24x20_pd16_vd1.npz",
                                "ref_collapse64_pd2_vd8.npz"])
def test_golden_backward_rebuild(fn, dev):
    """Standalone backward without a lattice from forward rebuilds it
    (the reference's only mode, permutohedral.cu:615-635)."""
    from plattice_pytorch_b200 import PLOO
    d = np.load(os.path.join(GOLDEN, fn))
    ft, gt, wt = _t(d["features"], dev), _t(d["grad"], dev), _t(d["weight"], dev)
    grad = PLOO.lattice_backward(ft, gt, wt, None)
    assert allclose_report(grad.cpu().numpy(), d["grad_out"], RTOL, ATOL) <= 1.0


FULL = ["blobs256_pd5_vd3", "voronoi1024_pd5_vd3", "voronoi1024_pd5_vd4", "gauss512_pd16_vd8",
        "collapse512_pd2_vd8", "crf512_pd5_vd3"]


@pytest.mark.parametrize("name", FULL)
def test_full_size_vs_reference_cuda(name, dev):
    """Full-size workloads against the reference CUDA build run on the same inputs."""
    if not oref.available():
        pytest.skip("reference build (oracle/_ref) not present")
    from plattice_pytorch_b200.workloads import make_workload
    w = make_workload(name)
    ours = _run_ours(w["features"], w["values"], w["grad"], dev)
    R = oref.RefLattice()
    ft, vt = ours["ft"], _t(w["values"], dev)
    wo_r, out_r, ws = R.forward(ft, vt)
    h, wdt, pd = ft.shape
    lat_r = R.lattice(ws, h * wdt, pd)
    del ws
    grad_r = R.backward(ft, ours["gt"], wo_r)
    assert ours["m"] == lat_r["m"]
    assert np.array_equal(ours["vertex_keys"], lat_r["vertex_keys"])
    assert allclose_report(ours["out"], out_r.cpu().numpy(), RTOL, ATOL) <= 1.0
    assert allclose_report(ours["weight"], wo_r.cpu().numpy(), RTOL, ATOL) <= 1.0
    # both backward passes from the reference's normaliser, so that the
    # gradient comparison isolates the backward
    from plattice_pytorch_b200 import PLOO
    grad_o = PLOO.lattice_backward(ft, ours["gt"], wo_r, None)
    assert allclose_report(grad_o.cpu().numpy(), grad_r.cpu().numpy(), RTOL, ATOL) <= 1.0


@pytest.mark.parametrize("name", ["blobs256_pd5_vd3", "crf512_pd5_vd3"])
def test_full_size_vs_oracle(name, dev):
    from plattice_pytorch_b200.workloads import make_workload
    w = make_workload(name)
    ours = _run_ours(w["features"], w["values"], w["grad"], dev)
    vk, _ = oracle.vertex_keys(w["features"])
    assert ours["m"] == vk.shape[0]
    assert np.array_equal(ours["vertex_keys"], oref.sort_keys(vk))
    wo, out, m = oracle.forward(w["features"], w["values"])
    assert allclose_report(ours["out"], out, RTOL, ATOL) <= 1.0
    assert allclose_report(ours["weight"], wo, RTOL, ATOL) <= 1.0
    g = oracle.backward(w["features"], w["grad"], ours["weight"])
    assert allclose_report(ours["grad_out"], g, RTOL, ATOL) <= 1.0


def test_headline_properties(dev):
    """Size-independent checks at 1024^2: adjointness of backward and forward
    (<g, F v> = <B g, v> with the normaliser fixed), normalisation of a
    constant image (a constant stays constant), finiteness."""
    from plattice_pytorch_b200 import PLOO
    from plattice_pytorch_b200.workloads import make_workload
    w = make_workload("voronoi1024_pd5_vd3")
    ft, vt, gt = _t(w["features"], dev), _t(w["values"], dev), _t(w["grad"], dev)
    wo, out, lat = PLOO.lattice_forward(ft, vt)
    gv = PLOO.lattice_backward(ft, gt, wo, lat)
    lhs = torch.sum(gt.double() * out.double()).item()
    rhs = torch.sum(gv.double() * vt.double()).item()
    assert abs(lhs - rhs) <= 1e-5 * max(1.0, abs(lhs))
    assert torch.isfinite(out).all() and torch.isfinite(gv).all()
    const = torch.full_like(vt, 0.375)
    _, oc, _ = PLOO.lattice_forward(ft, const)
    assert torch.allclose(oc, const, rtol=1e-5, atol=5e-6)


def test_autograd_module_matches_ploo(dev):
    from plattice_pytorch_b200 import PLOO, PermutoLattice
    d = np.load(os.path.join(GOLDEN, "ref_blobs64_pd5_vd3.npz"))
    ft = _t(d["features"], dev)
    vt = _t(d["values"], dev).requires_grad_(True)
    gt = _t(d["grad"], dev)
    out = PermutoLattice()(ft, vt)
    out.backward(gt)
    assert allclose_report(out.detach().cpu().numpy(), d["out"]) <= 1.0
    assert allclose_report(vt.grad.cpu().numpy(), d["grad_out"]) <= 1.0
    assert ft.grad is None
    w2, o2 = PLOO.forward(ft, vt.detach())
    g2 = PLOO.backward(ft, gt, w2)
    assert allclose_report(g2.cpu().numpy(), d["grad_out"]) <= 1.0


def test_repeated_backward_on_one_lattice(dev):
    from plattice_pytorch_b200 import PLOO
    d = np.load(os.path.join(GOLDEN, "ref_quant40_pd5_vd3.npz"))
    ft, vt, gt = _t(d["features"], dev), _t(d["values"], dev), _t(d["grad"], dev)
    wo, out, lat = PLOO.lattice_forward(ft, vt)
    g1 = PLOO.lattice_backward(ft, gt, wo, lat)
    g2 = PLOO.lattice_backward(ft, gt, wo, lat)
    assert lat.used
    for g in (g1, g2):
        assert allclose_report(g.cpu().numpy(), d["grad_out"]) <= 1.0


def test_modified_features_force_rebuild(dev):
    from plattice_pytorch_b200 import PLOO
    d = np.load(os.path.join(GOLDEN, "ref_randn16_pd5_vd3.npz"))
    ft, vt = _t(d["features"], dev), _t(d["values"], dev)
    wo, out, lat = PLOO.lattice_forward(ft, vt)
    ft.mul_(1.0)   # bumps the version counter
    assert not lat.matches(ft, vt.shape[2])
    g = PLOO.lattice_backward(ft, _t(d["grad"], dev), _t(d["weight"], dev), lat)
    assert allclose_report(g.cpu().numpy(), d["grad_out"]) <= 1.0


def test_reference_style_calls(dev):
    """The reference test's own calls (tests/test_plattice.py:93-116): shapes,
    finiteness and runtime pd/vd dispatch through PLOO.forward/backward."""
    from plattice_pytorch_b200 import PLOO
    torch.manual_seed(7)
    f = torch.randn(16, 16, 5, device=dev)
    v = torch.randn(16, 16, 3, device=dev)
    weight, out = PLOO.forward(f.contiguous(), v.contiguous())
    assert tuple(weight.shape) == (16, 16, 1) and tuple(out.shape) == (16, 16, 3)
    assert torch.isfinite(out).all()
    g = PLOO.backward(f.contiguous(), torch.ones_like(out), weight)
    assert tuple(g.shape) == (16, 16, 3) and torch.isfinite(g).all()
    torch.manual_seed(11)
    for pd, vd in [(1, 1), (2, 4), (5, 3), (8, 2), (16, 8), (12, 7)]:
        f = torch.randn(12, 10, pd, device=dev)
        v = torch.randn(12, 10, vd, device=dev)
        weight, out = PLOO.forward(f.contiguous(), v.contiguous())
        assert tuple(weight.shape) == (12, 10, 1) and tuple(out.shape) == (12, 10, vd)
        g = PLOO.backward(f.contiguous(), torch.ones_like(out), weight)
        assert tuple(g.shape) == (12, 10, vd)
        wo, o, _ = oracle.forward(f.cpu().numpy(), v.cpu().numpy())
        assert allclose_report(out.cpu().numpy(), o) <= 1.0


def test_bilateral_image_sanity(dev):
    """The reference test's PSNR check (tests/test_plattice.py:118-134) on this filter."""
    import math
    from plattice_pytorch_b200 import PLOO
    d = np.load(os.path.join(GOLDEN, "bilateral_crop.npz"))
    _, out = PLOO.forward(_t(d["features"], dev), _t(d["crop"], dev))
    lat = out.cpu().numpy()

    def psnr(a, b):
        mse = float(np.mean((a.astype(np.float64) - b) ** 2))
        return math.inf if mse < 1e-12 else 10.0 * math.log10(1.0 / mse)

    assert np.isfinite(lat).all()
    assert lat.min() >= -1e-3 and lat.max() <= 1 + 1e-3
    assert psnr(lat, d["brute"]) > float(d["psnr_floor"])
    assert psnr(lat, d["brute"]) > psnr(d["crop"], d["brute"])
    assert np.abs(lat - d["brute"]).max() < 5e-3


def test_small_image_vs_brute_force_gaussian(dev):
    """The lattice approximates the dense Gaussian; on the 64x64 blob image the
    new filter's error against it is that of the reference (same lattice)."""
    from plattice_pytorch_b200 import PLOO
    d = np.load(os.path.join(GOLDEN, "ref_blobs64_pd5_vd3.npz"))
    _, out = PLOO.forward(_t(d["features"], dev), _t(d["values"], dev))
    bf = oracle.brute_gaussian(d["features"], d["values"], threads=8).reshape(d["values"].shape)
    err_ours = np.abs(out.cpu().numpy() - bf).max()
    err_ref = np.abs(d["out"] - bf).max()
    assert err_ours <= err_ref + 1e-5


def test_nondefault_stream(dev):
    from plattice_pytorch_b200 import PLOO
    d = np.load(os.path.join(GOLDEN, "ref_blobs64_pd5_vd3.npz"))
    s = torch.cuda.Stream()
    ft, vt = _t(d["features"], dev), _t(d["values"], dev)
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        w, out = PLOO.forward(ft, vt)
    s.synchronize()
    assert allclose_report(out.cpu().numpy(), d["out"]) <= 1.0


def test_empty_image(dev):
    from plattice_pytorch_b200 import PLOO
    f = torch.zeros(0, 5, 5, device=dev)
    v = torch.zeros(0, 5, 3, device=dev)
    w, out = PLOO.forward(f, v)
    assert tuple(out.shape) == (0, 5, 3) and tuple(w.shape) == (0, 5, 1)
    g = PLOO.backward(f, torch.zeros_like(out), w)
    assert tuple(g.shape) == (0, 5, 3)


def test_undersized_table_reports_error(dev):
    """A hash table forced below the vertex count ends its probes at the limit
    and reports PLATTICE_DEV_TABLE_FULL through the status word (bounded
    loops, no hang).  Without PLATTICE_CHECK the failure raises at the first
    call after the failed call's kernels have finished (here the next call,
    after a synchronising read); with it, the failed call itself raises.  The
    next call with the automatic size is correct."""
    from plattice_pytorch_b200 import PLOO, _lib
    d = np.load(os.path.join(GOLDEN, "ref_blobs64_pd5_vd3.npz"))
    ft, vt = _t(d["features"], dev), _t(d["values"], dev)
    L = _lib.lib()
    check = PLOO._CHECK
    PLOO.check_device_status()   # nothing pending from earlier tests
    try:
        L.plattice_debug_set_table_cap_log2(6)   # 64 cells for 1225 vertices
        PLOO._CHECK = False
        _, _, lat = PLOO.lattice_forward(ft, vt)
        info = PLOO.lattice_info(lat)            # synchronises
        with pytest.raises(_lib.PlatticeError) as ei:
            PLOO.lattice_forward(ft, vt)         # refused: reports the earlier failure
        assert ei.value.status == _lib.ERR_DEVICE
        assert "plattice_forward" in str(ei.value) and "0x2" in str(ei.value)
        # the same through a backward that rebuilds, reported by a call of another kind
        gt = _t(d["grad"], dev)
        PLOO.lattice_backward(ft, gt, _t(d["weight"], dev), None)
        torch.cuda.synchronize()
        with pytest.raises(_lib.PlatticeError) as ei:
            PLOO.check_device_status()
        assert ei.value.status == _lib.ERR_DEVICE and "plattice_backward" in str(ei.value)
        # with per-call checking on, the failing call itself raises
        PLOO._CHECK = True
        with pytest.raises(_lib.PlatticeError) as ei:
            PLOO.lattice_forward(ft, vt)
        assert ei.value.status == _lib.ERR_DEVICE
        with pytest.raises(_lib.PlatticeError):   # ... and the ring still holds it once
            PLOO.check_device_status()
    finally:
        L.plattice_debug_set_table_cap_log2(0)
        PLOO._CHECK = check
    assert info["status"] & _lib.DEV_TABLE_FULL
    PLOO.check_device_status()   # reported once: nothing left
    _, out, lat = PLOO.lattice_forward(ft, vt)
    assert PLOO.lattice_info(lat)["status"] == 0
    assert allclose_report(out.cpu().numpy(), d["out"]) <= 1.0
    torch.cuda.synchronize()
    PLOO.check_device_status()
