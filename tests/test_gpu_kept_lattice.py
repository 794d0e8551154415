"""The kept lattice: filtering further values on a lattice built once.

``PLOO.lattice_filter`` / ``lattice_filter_backward`` (C ABI
``plattice_filter`` / ``plattice_filter_backward``) run splat, blur and slice
on the lattice that an earlier forward built for the same features.  The
reference has no such call -- it rebuilds the lattice every time
(permutohedral.cu:549-570, 615-635) -- so the checkers are the regular entry
points on the same features and the CPU oracle:
  * a filter of new values equals ``PLOO.forward(features, new values)``
    (out and weight), also for a vd other than the build's;
  * it equals the oracle's forward on those values;
  * a mean-field style loop of filters on one lattice equals fresh forwards;
  * the backward equals ``PLOO.backward`` and autograd through
    ``LatticeFilterFunction`` equals autograd through ``PermutoLatticeFunction``.
Tolerance: 1e-5 relative + 5e-6 absolute (float reductions in another order).
"""
import os

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN, allclose_report

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-5, 5e-6
CASES = ["ref_blobs64_pd5_vd3.npz", "ref_randn24x20_pd2_vd3.npz", "ref_randn24x20_pd7_vd8.npz",
         "ref_randn24x20_pd16_vd1.npz", "ref_ragged13x29_pd5_vd3.npz"]


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from plattice_pytorch_b200 import _lib
    _lib.lib()
    return torch.device("cuda:0")


def _close(a, b):
    return allclose_report(a.detach().cpu().numpy(), b.detach().cpu().numpy(), RTOL, ATOL) <= 1.0


def _load(name, dev):
    d = np.load(os.path.join(GOLDEN, name))
    return d, torch.from_numpy(d["features"]).to(dev), torch.from_numpy(d["values"]).to(dev)


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("vd2", [None, 4])
def test_filter_equals_a_fresh_forward(name, vd2, dev):
    from plattice_pytorch_b200 import PLOO
    d, f, v = _load(name, dev)
    _, _, lat = PLOO.lattice_forward(f, v)
    h, w, _ = f.shape
    g = torch.Generator().manual_seed(7)
    v2 = torch.rand((h, w, vd2 or v.shape[2]), generator=g).to(dev)
    wk, ok = PLOO.lattice_filter(lat, v2)
    wr, orr = PLOO.forward(f, v2)
    torch.cuda.synchronize()
    assert _close(ok, orr) and _close(wk, wr)
    assert PLOO.lattice_info(lat)["status"] == 0


@pytest.mark.parametrize("name", ["ref_blobs64_pd5_vd3.npz", "ref_randn24x20_pd12_vd5.npz"])
def test_filter_equals_the_oracle(name, dev):
    from plattice_pytorch_b200 import PLOO
    d, f, v = _load(name, dev)
    _, _, lat = PLOO.lattice_forward(f, v)
    v2 = torch.from_numpy(np.ascontiguousarray(d["grad"])).to(dev)   # another value tensor of the same shape
    wk, ok = PLOO.lattice_filter(lat, v2)
    w_o, out_o, m = oracle.forward(d["features"], d["grad"])
    assert m == PLOO.lattice_info(lat)["m"]
    assert allclose_report(ok.cpu().numpy(), out_o, RTOL, ATOL) <= 1.0
    assert allclose_report(wk.cpu().numpy(), w_o, RTOL, ATOL) <= 1.0


def test_mean_field_loop_on_one_lattice(dev):
    """Five rounds of softmax -> filter, as a dense-CRF inference does, on one
    kept lattice, against five fresh forwards."""
    from plattice_pytorch_b200 import PLOO
    from plattice_pytorch_b200.workloads import make_workload
    wl = make_workload("crf512_pd5_vd3", seed=3)
    f = torch.from_numpy(wl["features"]).to(dev)
    unary = torch.from_numpy(wl["values"]).to(dev).log()
    q = torch.softmax(unary, dim=2).contiguous()
    _, _, lat = PLOO.lattice_forward(f, q)
    qk, qr = q, q
    for _ in range(5):
        _, mk = PLOO.lattice_filter(lat, qk)
        _, mr = PLOO.forward(f, qr)
        assert _close(mk, mr)
        qk = torch.softmax(unary - mk, dim=2).contiguous()
        qr = torch.softmax(unary - mr, dim=2).contiguous()
    torch.cuda.synchronize()
    assert PLOO.lattice_info(lat)["status"] == 0


@pytest.mark.parametrize("name", ["ref_blobs64_pd5_vd3.npz", "ref_randn24x20_pd9_vd2.npz"])
def test_filter_backward_equals_the_regular_backward(name, dev):
    from plattice_pytorch_b200 import PLOO
    d, f, v = _load(name, dev)
    _, _, lat = PLOO.lattice_forward(f, v)
    h, w, _ = f.shape
    g = torch.Generator().manual_seed(11)
    for vd2 in (int(v.shape[2]), 6):
        v2 = torch.rand((h, w, vd2), generator=g).to(dev)
        gr = torch.randn((h, w, vd2), generator=g).to(dev)
        wk, _ = PLOO.lattice_filter(lat, v2)
        gk = PLOO.lattice_filter_backward(lat, gr, wk)
        wr, _ = PLOO.forward(f, v2)
        gref = PLOO.backward(f, gr, wr)
        torch.cuda.synchronize()
        assert _close(gk, gref)


def test_autograd_through_the_kept_lattice(dev):
    from plattice_pytorch_b200 import PLOO, LatticeFilterFunction, PermutoLatticeFunction
    d, f, v = _load("ref_blobs64_pd5_vd3.npz", dev)
    _, _, lat = PLOO.lattice_forward(f, v)
    g = torch.from_numpy(d["grad"]).to(dev)
    v2 = (v * 0.5 + 0.25).detach()
    a = v2.clone().requires_grad_(True)
    b = v2.clone().requires_grad_(True)
    oa = LatticeFilterFunction.apply(a, lat)
    ob = PermutoLatticeFunction.apply(f, b)
    (ga,) = torch.autograd.grad(oa, (a,), (g,))
    (gb,) = torch.autograd.grad(ob, (b,), (g,))
    assert _close(oa, ob) and _close(ga, gb)


def test_filter_checks_shapes(dev):
    from plattice_pytorch_b200 import PLOO
    d, f, v = _load("ref_blobs64_pd5_vd3.npz", dev)
    _, _, lat = PLOO.lattice_forward(f, v)
    with pytest.raises(RuntimeError, match="must match the lattice"):
        PLOO.lattice_filter(lat, torch.zeros((8, 8, 3), device=dev))
    with pytest.raises(RuntimeError, match="value dimension"):
        PLOO.lattice_filter(lat, torch.zeros((64, 64, 9), device=dev))


@pytest.mark.parametrize("streaming", [False, True])
def test_every_call_kind_in_turn_on_one_lattice(streaming, dev):
    """The cooperative kernels of a call (the blur; the zero-then-splat of a
    call on a used lattice) share the lattice's grid-barrier counters, which
    every call must leave at zero for the next: forward, backward (fresh and
    used lattice), filter, filter backward and feature gradient in turn on one
    kept lattice, twice over, each against the same call on a freshly built
    lattice; the status word stays clear.  Both blur paths (rows in registers,
    and the streaming passes)."""
    from plattice_pytorch_b200 import PLOO, _lib
    from plattice_pytorch_b200.workloads import make_workload
    L = _lib.lib()
    wl = make_workload("crf512_pd5_vd3", seed=5)
    f = torch.from_numpy(wl["features"]).to(dev)
    v = torch.from_numpy(wl["values"]).to(dev)
    g = torch.from_numpy(wl["grad"]).to(dev)
    v2 = torch.roll(v, 7, dims=1).contiguous()
    g2 = torch.roll(g, 11, dims=0).contiguous()
    try:
        L.plattice_debug_set_blur_streaming(1 if streaming else 0)
        w, out, lat = PLOO.lattice_forward(f, v)
        wf, outf, _ = PLOO.lattice_forward(f, v)
        assert _close(out, outf) and _close(w, wf)
        for _ in range(2):
            assert _close(PLOO.lattice_backward(f, g, w, lat), PLOO.lattice_backward(f, g, w))
            assert _close(PLOO.lattice_backward(f, g2, w, lat), PLOO.lattice_backward(f, g2, w))
            w2, m2 = PLOO.lattice_filter(lat, v2)
            w2f, m2f = PLOO.forward(f, v2)
            assert _close(m2, m2f) and _close(w2, w2f)
            assert _close(PLOO.lattice_filter_backward(lat, g2, w2), PLOO.lattice_backward(f, g2, w2f))
            _, _, latf = PLOO.lattice_forward(f, v)
            a = PLOO.feature_grad(lat, f, v, g, w, out).cpu().numpy()
            b = PLOO.feature_grad(latf, f, v, g, wf, outf).cpu().numpy()
            # the feature gradient's own tolerance (differences of nearby rows)
            assert np.all(np.abs(a - b) <= 2e-3 * np.abs(b) + 1e-4 * max(float(np.abs(b).max()), 1e-12))
        torch.cuda.synchronize()
        assert PLOO.lattice_info(lat)["status"] == 0
    finally:
        L.plattice_debug_set_blur_streaming(0)


def test_a_failed_call_marks_its_lattice_broken(dev):
    """A device failure of the build (a hash table forced below the vertex
    count) is reported by the next call, a backward on that lattice, which
    marks the lattice broken: the backward after it rebuilds (the golden value
    gradient), and the calls that need a kept lattice refuse it."""
    from plattice_pytorch_b200 import PLOO, _lib
    d = np.load(os.path.join(GOLDEN, "ref_blobs64_pd5_vd3.npz"))
    ft, vt, gt, wt = (torch.from_numpy(d[k]).to(dev) for k in ("features", "values", "grad", "weight"))
    L = _lib.lib()
    check = PLOO._CHECK
    PLOO.check_device_status()   # nothing pending from earlier tests
    try:
        PLOO._CHECK = False
        L.plattice_debug_set_table_cap_log2(6)   # 64 cells for 1225 vertices
        _, _, lat = PLOO.lattice_forward(ft, vt)
        PLOO.lattice_info(lat)                   # synchronises: the build's failure is recorded
        L.plattice_debug_set_table_cap_log2(0)
        with pytest.raises(_lib.PlatticeError) as ei:
            PLOO.lattice_backward(ft, gt, wt, lat)
        assert ei.value.status == _lib.ERR_DEVICE
        assert lat.broken
        gv = PLOO.lattice_backward(ft, gt, wt, lat)   # rebuilds
        assert _close(gv, torch.from_numpy(d["grad_out"]))
        with pytest.raises(RuntimeError, match="unusable"):
            PLOO.lattice_filter(lat, vt)
    finally:
        L.plattice_debug_set_table_cap_log2(0)
        PLOO._CHECK = check
